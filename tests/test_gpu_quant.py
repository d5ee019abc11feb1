"""GPU parity of the activation amax / quantize kernels against the oracle (bit-exact)."""
import numpy as np
import pytest

from oracle import w8a8 as ow
from tests._util import bits_to_f32, nchw_to_nhwc, seeded_act, slab16_to_nchw

pytestmark = pytest.mark.gpu


def _torch():
    import torch

    return torch


@pytest.mark.parametrize("shape", [(2, 32, 10, 12), (3, 48, 7, 9), (1, 20, 5, 5), (1, 64, 80, 80), (4, 16, 1, 1)])
def test_amax_nchw_bitexact(shape):
    torch = _torch()
    from aexrt_b200 import ops

    rng = np.random.default_rng(sum(shape))
    x = seeded_act(rng, shape)
    x[0, 0, 0, 0] = -7.5  # a negative extreme must count by magnitude
    amax = ops.act_amax(torch.from_numpy(x).cuda(), ops.LAYOUT_NCHW_F16)
    torch.cuda.synchronize()
    at, ag = ow.act_amax(x)
    assert np.array_equal(bits_to_f32(amax.cpu().numpy()), ag)


@pytest.mark.parametrize("ldc,coff,c", [(64, 0, 64), (96, 32, 48), (48, 16, 32)])
def test_amax_nhwc_slice_bitexact(ldc, coff, c):
    torch = _torch()
    from aexrt_b200 import ops

    rng = np.random.default_rng(ldc + coff)
    full = seeded_act(rng, (3, ldc, 9, 11))
    amax = ops.act_amax(torch.from_numpy(nchw_to_nhwc(full)).cuda(), ops.LAYOUT_NHWC_F16, c=c, coff=coff)
    torch.cuda.synchronize()
    _, ag = ow.act_amax(full[:, coff:coff + c])
    assert np.array_equal(bits_to_f32(amax.cpu().numpy()), ag)


@pytest.mark.parametrize("mode", [0, 1])
@pytest.mark.parametrize("shape,stride", [((2, 32, 10, 12), 1), ((2, 32, 9, 11), 2), ((1, 64, 80, 80), 1)])
def test_quantize_nchw_bitexact(shape, stride, mode):
    torch = _torch()
    from aexrt_b200 import ops

    rng = np.random.default_rng(7 + mode)
    x = seeded_act(rng, shape)
    x[-1] = 0  # an all-zero image quantizes to zeros
    xt = torch.from_numpy(x).cuda()
    amax = ops.act_amax(xt, ops.LAYOUT_NCHW_F16)
    q, rec = ops.act_quantize(xt, amax, mode, ops.LAYOUT_NCHW_F16, consumer_stride=stride)
    torch.cuda.synchronize()
    n, c, h, w = shape
    qn = q.cpu().numpy()
    at, ag = ow.act_amax(x)
    expect = ow.quantize_act(x, at, ag, mode)
    assert np.array_equal(slab16_to_nchw(qn, c, h, w, stride), expect)
    # padding rows / columns of a stride-2 consumer's buffer are zero
    assert (qn[:, :, h:, :] == 0).all() and (qn[:, :, :, w:] == 0).all()
    r = rec.cpu().numpy()
    assert np.array_equal(r[:, 0], at) and np.array_equal(r[:, 1:], ag)


def test_quantize_nhwc_slice_matches_nchw():
    torch = _torch()
    from aexrt_b200 import ops

    rng = np.random.default_rng(11)
    full = seeded_act(rng, (2, 80, 6, 7))
    xs = full[:, 16:64]
    amax = ops.act_amax(torch.from_numpy(nchw_to_nhwc(full)).cuda(), ops.LAYOUT_NHWC_F16, c=48, coff=16)
    q, rec = ops.act_quantize(torch.from_numpy(nchw_to_nhwc(full)).cuda(), amax, 0, ops.LAYOUT_NHWC_F16, c=48, coff=16)
    torch.cuda.synchronize()
    at, ag = ow.act_amax(xs)
    assert np.array_equal(slab16_to_nchw(q.cpu().numpy(), 48, 6, 7), ow.quantize_act(xs, at, ag, 0))


def test_quantize_baseline_standalone_64x64x80x80():
    """BASELINE config 2's standalone amax + quantize tensor, full size, both modes."""
    torch = _torch()
    from aexrt_b200 import ops

    rng = np.random.default_rng(0)
    x = seeded_act(rng, (64, 64, 80, 80))
    xt = torch.from_numpy(x).cuda()
    amax = ops.act_amax(xt, ops.LAYOUT_NCHW_F16)
    at, ag = ow.act_amax(x)
    assert np.array_equal(bits_to_f32(amax.cpu().numpy()), ag)
    for mode in (0, 1):
        q, _ = ops.act_quantize(xt, amax, mode, ops.LAYOUT_NCHW_F16)
        expect = ow.quantize_act(x, at, ag, mode)
        assert np.array_equal(slab16_to_nchw(q.cpu().numpy(), 64, 80, 80), expect)
