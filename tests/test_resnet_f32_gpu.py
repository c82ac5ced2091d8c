"""fp32 ResNet-50 conv stack on the bf16x3 tensor-core path (activations kept
as split bf16 hi/lo planes between layers) against a plain PyTorch fp32
chain of the same convolutions, biases, ReLUs and the stem's 3x3/2 max pool.
Tolerance: max |err| <= 1e-3 * max |ref| on the stem, the pool and the last
layer (the fp32 bar for a single convolution, after all 53 layers)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

REL_TOL = 1e-3


def test_f32_stack_matches_torch_fp32():
    import torch
    import torch.nn.functional as F

    from computeengine_b200.resnet import ResNet50F32, make_f32_params, resnet50_layers
    batch = 2
    layers = resnet50_layers()
    params = make_f32_params(layers, seed=3)
    rng = np.random.default_rng(3)
    x = rng.uniform(-1, 1, (batch, 3, 224, 224)).astype(np.float32)
    net = ResNet50F32(batch, params)
    net.run(torch.from_numpy(x).cuda())
    torch.cuda.synchronize()
    assert net.L.take_device_error() == 0

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
