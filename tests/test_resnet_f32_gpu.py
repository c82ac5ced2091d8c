"""fp32 ResNet-50 conv stack on the bf16x3 tensor-core path (activations kept
as split bf16 hi/lo planes between layers).

At the workload's own batch (32 images, U(-1, 1) input, He-normal weights),
sampled images are run through the reference's own Conv2DOp and
MaxPool2DOp (compiled from its sources into oracle/_ref) as a chain, and
every one of the 53 layers and the pool is checked against it:
max |err| <= 1e-3 * max |ref| per layer (the fp32 bar of a single
convolution, held after all 53).  A second test checks a small batch against
a PyTorch fp32 chain where the reference library is not built."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

REL_TOL = 1e-3
SAMPLED = (0, 17, 31)


def _gpu_stack(batch, seed):
    import torch
    from computeengine_b200.resnet import ResNet50F32, make_f32_params, resnet50_layers
    layers = resnet50_layers()
    params = make_f32_params(layers, seed=seed)
    rng = np.random.default_rng(seed)
    x = rng.uniform(-1, 1, (batch, 3, 224, 224)).astype(np.float32)
    net = ResNet50F32(batch, params)
    net.run(torch.from_numpy(x).cuda())
    torch.cuda.synchronize()
    assert net.L.take_device_error() == 0
    return layers, params, x, net


def test_f32_stack_batch32_every_layer_matches_reference_conv(refconv):
    layers, params, x, net = _gpu_stack(32, seed=5)
    idx = list(SAMPLED)
    acts = {"input": np.ascontiguousarray(x[idx])}
    for l in layers:
        w, b = params[l.name]
        rc, y = refconv.conv2d(acts[l.src], w, b, strides=(l.stride, l.stride),
                               pads=(l.pad,) * 4, nthreads=len(idx))
        assert rc == 0, (l.name, rc)
        np.maximum(y, 0.0, out=y)  # the Relu node after each conv
        acts[l.name] = y
        if l.name == "stem":
            rc, p = refconv.pool2d(y, kernel=(3, 3), strides=(2, 2), pads=(1, 1, 1, 1), kind="max")
            assert rc == 0
            acts["pool"] = p
    for name in ["stem", "pool"] + [l.name for l in layers[1:]]:
        got = net.to_nchw_f32(name)[idx].cpu().numpy()
        want = acts[name]
        assert got.shape == want.shape, name
        err = float(np.abs(got - want).max())
        assert err <= REL_TOL * float(np.abs(want).max()), (name, err, float(np.abs(want).max()))


def test_f32_stack_matches_torch_fp32():
    import torch
    import torch.nn.functional as F
    layers, params, x, net = _gpu_stack(2, seed=3)
    acts = {"input": torch.from_numpy(x)}
    with torch.no_grad():
        for l in layers:
            w, b = params[l.name]
            y = F.conv2d(acts[l.src], torch.from_numpy(w), torch.from_numpy(b), stride=l.stride,
                         padding=l.pad)
            acts[l.name] = torch.relu(y)
            if l.name == "stem":
                acts["pool"] = F.max_pool2d(acts["stem"], 3, 2, 1)
    for name in ("stem", "pool", layers[-1].name):
        got = net.to_nchw_f32(name).cpu()
        want = acts[name]
        assert got.shape == want.shape, name
        err = float((got - want).abs().max())
        assert err <= REL_TOL * float(want.abs().max()), (name, err, float(want.abs().max()))
