"""GPU parity of the activation amax / quantize kernels against the oracle (bit-exact)."""
import numpy as np
import pytest

from oracle import w8a8 as ow
from tests._util import bits_to_f32, nchw_to_nhwc, seeded_act, slab16_to_nchw, unsplit_columns

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


def _concat_case(rng, n, h, w, specs):
    """NHWC fp16 source buffers for one concatenated consumer input.

    specs: (buffer channels, slice offset, slice channels, upsample) per source.  Returns the
    device buffers, the C source descriptors (amax slots filled by act_amax) and the logical
    NCHW concatenation the quantizer must see."""
    torch = _torch()
    from aexrt_b200 import ops
    from aexrt_b200._native import AexrtB200ActSource

    srcs = (AexrtB200ActSource * len(specs))()
    keep, parts = [], []
    for i, (ldc, coff, ch, up) in enumerate(specs):
        sh, sw = (h + up - 1) // up, (w + up - 1) // up
        full = seeded_act(rng, (n, ldc, sh, sw))
        buf = torch.from_numpy(nchw_to_nhwc(full)).cuda()
        amax = ops.act_amax(buf, ops.LAYOUT_NHWC_F16, c=ch, coff=coff)
        keep += [buf, amax]
        part = full[:, coff:coff + ch]
        if up == 2:
            part = part.repeat(2, axis=2).repeat(2, axis=3)
        parts.append(part[:, :, :h, :w])
        s = srcs[i]
        s.ptr, s.layout, s.ldc, s.coff, s.channels, s.upsample = buf.data_ptr(), ops.LAYOUT_NHWC_F16, ldc, coff, ch, up
        s.src_h, s.src_w = sh, sw
        s.amax_groups, s.amax_stride, s.amax_goff = amax.data_ptr(), amax.shape[1], 0
    return srcs, keep, np.concatenate(parts, axis=1)


@pytest.mark.parametrize("stride", [1, 2])
@pytest.mark.parametrize("mode", [0, 1])
@pytest.mark.parametrize("specs,h,w", [
    # aligned slices: the coalesced row kernel (upsampled source, odd chunk count in the last one)
    ([(64, 16, 32, 2), (48, 0, 48, 1), (24, 0, 24, 1)], 10, 14),
    ([(128, 0, 128, 1), (64, 0, 64, 1)], 9, 11),
    ([(16, 0, 16, 1)], 7, 5),
    ([(256, 0, 192, 1)], 6, 6),
    ([(1152, 0, 1040, 1)], 3, 4),  # more than 1024 channels: the per-slab generic kernel
])
def test_quantize_concat_sources_bitexact(specs, h, w, mode, stride):
    """Concatenated / upsampled NHWC sources quantized in one pass equal the oracle on the concatenation."""
    torch = _torch()
    from aexrt_b200 import _native, ops
    from aexrt_b200._native import check

    rng = np.random.default_rng(h * 100 + w + len(specs))
    n = 3
    srcs, keep, cat = _concat_case(rng, n, h, w, specs)
    c = cat.shape[1]
    shape = ops.packed_act_shape(n, c, h, w, stride)
    q = torch.full(shape, 99, dtype=torch.int8, device="cuda")
    rec = torch.empty((n, 1 + shape[1]), dtype=torch.float32, device="cuda")
    lib = _native.load()
    if mode == 1 and c % 16:
        # pg16 scales are per 16-channel group: a ragged last group is refused, as in the reference
        assert lib.aexrt_b200_act_quantize_concat(srcs, len(specs), n, h, w, mode, stride, q.data_ptr(),
                                                  rec.data_ptr(), None) == 0
        return
    check(lib.aexrt_b200_act_quantize_concat(srcs, len(specs), n, h, w, mode, stride, q.data_ptr(), rec.data_ptr(),
                                             None), "quantize concat")
    torch.cuda.synchronize()
    at, ag = ow.act_amax(cat)
    qn = q.cpu().numpy()
    assert np.array_equal(slab16_to_nchw(qn, c, h, w, stride), ow.quantize_act(cat, at, ag, mode))
    # channel padding of the last slab and the stride-2 padding rows / columns are zero
    full = slab16_to_nchw(qn, shape[1] * 16, shape[2], shape[3], stride)
    assert (full[:, c:] == 0).all() and (full[:, :, h:] == 0).all() and (full[:, :, :, w:] == 0).all()
    r = rec.cpu().numpy()
    assert np.array_equal(r[:, 0], at) and np.array_equal(r[:, 1:], ag)


@pytest.mark.parametrize("stride", [1, 2])
@pytest.mark.parametrize("specs,h,w", [
    ([(64, 16, 32, 2), (48, 0, 48, 1), (24, 0, 24, 1)], 10, 14),
    ([(64, 0, 64, 1)], 9, 11),
    ([(24, 8, 16, 1), (16, 0, 8, 1)], 9, 7),
])
def test_pack_f16_concat_sources_exact(specs, h, w, stride):
    """The fp16 repack of concatenated sources is a pure copy into the slab8 layout."""
    torch = _torch()
    from aexrt_b200 import _native
    from aexrt_b200._native import check

    rng = np.random.default_rng(h * 10 + w)
    n = 2
    srcs, keep, cat = _concat_case(rng, n, h, w, specs)
    c = cat.shape[1]
    hp, wp = (h + (h & 1), w + (w & 1)) if stride == 2 else (h, w)
    out = torch.full((n, (c + 7) // 8, hp, wp, 8), 5.0, dtype=torch.float16, device="cuda")
    check(_native.load().aexrt_b200_pack_f16_concat(srcs, len(specs), n, h, w, stride, out.data_ptr(), None),
          "pack concat")
    torch.cuda.synchronize()
    o = out.cpu().numpy()
    if stride == 2:
        o = unsplit_columns(o)
    got = o.transpose(0, 1, 4, 2, 3).reshape(n, -1, hp, wp)
    assert np.array_equal(got[:, :c, :h, :w], cat)
    assert (got[:, c:] == 0).all() and (got[:, :, h:] == 0).all() and (got[:, :, :, w:] == 0).all()


@pytest.mark.parametrize("mode", [0, 1])
@pytest.mark.parametrize("shape", [
    (64, 64, 80, 80),    # one 4-CTA cluster per image, strips of 200 KB in shared memory
    (3, 16, 13, 17),     # one strip per image, odd plane
    (2, 128, 20, 20),    # eight strips: the largest cluster
    (2, 48, 7, 9),
    (2, 24, 10, 12),     # channels not a multiple of 16: the two-kernel path
    (1, 256, 10, 10),    # sixteen strips: the two-kernel path
    (1, 32, 96, 96),     # strip larger than shared memory: the two-kernel path
])
def test_single_pass_amax_quantize_equals_two_kernels(shape, mode):
    """aexrt_b200_act_amax_quantize_f16 equals act_amax + act_quantize bit for bit (codes, scale
    record, amax slots), and the oracle's codes."""
    torch = _torch()
    from aexrt_b200 import ops

    rng = np.random.default_rng(sum(shape) + mode)
    x = seeded_act(rng, shape) * np.float16(3)
    if shape[0] > 1:
        x[1] = 0  # an all-zero image: amax 0, codes 0
    xt = torch.from_numpy(x).cuda()
    amax_ref = ops.act_amax(xt, ops.LAYOUT_NCHW_F16)
    if mode == 1 and shape[1] % 16:
        # pg16 needs whole 16-channel groups: both entry points refuse, before any launch
        from aexrt_b200._native import AexrtError

        with pytest.raises(AexrtError, match="pg16"):
            ops.act_quantize(xt, amax_ref, mode, ops.LAYOUT_NCHW_F16)
        with pytest.raises(AexrtError, match="pg16"):
            ops.act_amax_quantize(xt, mode)
        return
    q_ref, rec_ref = ops.act_quantize(xt, amax_ref, mode, ops.LAYOUT_NCHW_F16)
    amax = torch.full_like(amax_ref, -1)
    q = torch.full_like(q_ref, 55)
    rec = torch.full_like(rec_ref, -2.0)
    for _ in range(2):  # twice: nothing from the first call leaks into the second
        ops.act_amax_quantize(xt, mode, amax_out=amax, q_out=q, rec_out=rec)
        torch.cuda.synchronize()
        assert ops.act_status() == 0
        assert torch.equal(q, q_ref)
        assert torch.equal(rec, rec_ref)
        assert torch.equal(amax, amax_ref)
    n, c, h, w = shape
    at, ag = ow.act_amax(x)
    assert np.array_equal(slab16_to_nchw(q.cpu().numpy(), c, h, w), ow.quantize_act(x, at, ag, mode))


def test_single_pass_wait_timeout_reports_and_writes_nothing():
    """Failure detection without a fault: with the copy wait limited to 0 cycles the cluster kernel
    gives up, sets its status bit and writes nothing of an image whose slices did not all land (every
    CTA still waits, with the full limit, for its own copies before it exits); the context stays
    usable and the next normal call is exact."""
    torch = _torch()
    from aexrt_b200 import _native, ops

    rng = np.random.default_rng(77)
    x = seeded_act(rng, (64, 64, 80, 80))
    xt = torch.from_numpy(x).cuda()
    amax_ref = ops.act_amax(xt, ops.LAYOUT_NCHW_F16)
    q_ref, rec_ref = ops.act_quantize(xt, amax_ref, 0, ops.LAYOUT_NCHW_F16)
    torch.cuda.synchronize()
    assert ops.act_status() == 0
    amax = torch.full_like(amax_ref, -1)
    q = torch.full_like(q_ref, 55)
    rec = torch.full_like(rec_ref, -2.0)
    lib = _native.load()
    assert lib.aexrt_b200_act_amax_quantize_f16_wait_limit(xt.data_ptr(), 64, 64, 80, 80, 0, amax.data_ptr(), 4, 0,
                                                           q.data_ptr(), rec.data_ptr(), 0, None) == 1
    torch.cuda.synchronize()
    assert ops.act_status() & 1  # the timeout bit
    written = 0
    for i in range(64):
        # all of an image's outputs, or none of them
        if torch.equal(q[i], q_ref[i]):
            assert torch.equal(rec[i], rec_ref[i]) and torch.equal(amax[i], amax_ref[i])
            written += 1
        else:
            assert (q[i] == 55).all() and (rec[i] == -2.0).all() and (amax[i] == -1).all(), i
    assert written < 64
    ops.act_amax_quantize(xt, 0, amax_out=amax, q_out=q, rec_out=rec)
    torch.cuda.synchronize()
    assert ops.act_status() == 0
    assert torch.equal(q, q_ref) and torch.equal(rec, rec_ref) and torch.equal(amax, amax_ref)
