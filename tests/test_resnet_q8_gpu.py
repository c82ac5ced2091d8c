"""The 53-layer int8 ResNet-50 conv stack on the B200 against the int8 oracle,
layer by layer and end to end, bit-exact.  The stem runs through the
space-to-depth re-layout, so its check also proves that re-layout exact."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _nchw(t):
    return t.permute(0, 3, 1, 2).contiguous().cpu().numpy()


def test_stack_small_batch_every_layer(oracle):
    import torch
    from computeengine_b200.resnet import ResNet50Q8, make_input_u8, make_q8_params, resnet50_layers
    from oracle.oracle import resnet_q8_chain

    layers = resnet50_layers()
    params = make_q8_params(layers, seed=0)
    x = make_input_u8(3, seed=0)
    net = ResNet50Q8(3, params)
    net.run(torch.from_numpy(x).cuda())
    torch.cuda.synchronize()
    gpu = {name: _nchw(t) for name, t in net.acts.items()}
    # each layer on its own, fed with the GPU's own input for that layer
    want = resnet_q8_chain(oracle, layers, params, x, nthreads=3, inputs=gpu)
    for l in layers:
        np.testing.assert_array_equal(gpu[l.name], want[l.name], err_msg=l.name)
    np.testing.assert_array_equal(gpu["pool"], want["pool"])
    # and the whole chain from the input
    chain = resnet_q8_chain(oracle, layers, params, x, nthreads=3)
    np.testing.assert_array_equal(gpu[layers[-1].name], chain[layers[-1].name])


def test_stack_full_batch_sampled_images(oracle):
    """Batch 256 (the per-GPU benchmark batch) through the captured CUDA graph;
    images are independent, so sampled images check every tile position."""
    import torch
    from computeengine_b200 import _lib as L
    from computeengine_b200.resnet import ResNet50Q8, make_input_u8, make_q8_params, resnet50_layers
    from oracle.oracle import resnet_q8_chain

    layers = resnet50_layers()
    params = make_q8_params(layers, seed=0)
    x = make_input_u8(256, seed=7)
    net = ResNet50Q8(256, params)
    xd = torch.from_numpy(x).cuda()
    net.capture(xd)
    net.replay()
    net.replay()
    torch.cuda.synchronize()
    assert L.take_device_error() == 0
    out = net.output
    for img in (0, 131, 255):
        chain = resnet_q8_chain(oracle, layers, params, x[img:img + 1], nthreads=1)
        got = out[img:img + 1].permute(0, 3, 1, 2).cpu().numpy()
        np.testing.assert_array_equal(got, chain[layers[-1].name], err_msg=f"image {img}")
