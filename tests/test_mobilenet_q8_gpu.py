"""MobileNetV2-style int8 block sweep (expand 1x1 -> depthwise 3x3 ->
project 1x1) on the B200 against the int8 oracle, layer by layer (each layer
fed with the GPU's own input for it) and end to end.  Bit-exact.  At batch 2,
every image; at the workload's batch of 64, sampled images."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _gpu_nchw(t, c, signed):
    a = t[..., :c].permute(0, 3, 1, 2).contiguous().cpu().numpy()
    return a.view(np.int8) if signed else a


def _oracle_layer(oracle, l, p, src):
    qmin, qmax = (-128, 127) if l.y_signed else (0, l.qmax)
    return oracle.conv2d_q8(src, p.w, p.bias, p.mult, l.zp_x, 0, qmin, qmax, y_signed=l.y_signed,
                            strides=(l.stride, l.stride), pads=(l.k // 2,) * 4,
                            group=l.cin if l.kind == "dw" else 1, depthwise=l.kind == "dw",
                            nthreads=4)


def test_mobilenet_sweep_every_layer(oracle):
    import torch
    from computeengine_b200.mobilenet import MobileNetV2Q8, make_input, make_params, mobilenetv2_layers
    layers = mobilenetv2_layers()
    params = make_params(layers)
    x = make_input(2, seed=3)
    net = MobileNetV2Q8(2, params)
    net.run(torch.from_numpy(x).cuda())
    torch.cuda.synchronize()
    gpu = {l.name: _gpu_nchw(net.acts[l.name], l.cout, l.y_signed) for l in layers}
    chain = {}
    for l in layers:
        src_gpu = x if l.src == "input" else gpu[l.src]
        want = _oracle_layer(oracle, l, params[l.name], src_gpu)
        np.testing.assert_array_equal(gpu[l.name], want, err_msg=l.name)
        src_chain = x if l.src == "input" else chain[l.src]
        chain[l.name] = _oracle_layer(oracle, l, params[l.name], src_chain)
    last = layers[-1].name
    np.testing.assert_array_equal(gpu[last], chain[last])
    # the sweep must not degenerate to constant outputs
    assert len(np.unique(gpu[last])) > 16


def test_mobilenet_sweep_batch64_sampled_images(oracle):
    import torch
    from computeengine_b200.mobilenet import MobileNetV2Q8, make_input, make_params, mobilenetv2_layers
    layers = mobilenetv2_layers()
    params = make_params(layers)
    x = make_input(64, seed=0)
    net = MobileNetV2Q8(64, params)
    net.run(torch.from_numpy(x).cuda())
    torch.cuda.synchronize()
    assert net.L.take_device_error() == 0
    idx = [0, 29, 63]
    gpu = {l.name: _gpu_nchw(net.acts[l.name], l.cout, l.y_signed)[idx] for l in layers}
    chain = {}
    for l in layers:
        src_gpu = x[idx] if l.src == "input" else gpu[l.src]
        np.testing.assert_array_equal(gpu[l.name], _oracle_layer(oracle, l, params[l.name], src_gpu),
                                      err_msg=l.name)
        src_chain = x[idx] if l.src == "input" else chain[l.src]
        chain[l.name] = _oracle_layer(oracle, l, params[l.name], src_chain)
    np.testing.assert_array_equal(gpu[layers[-1].name], chain[layers[-1].name])
