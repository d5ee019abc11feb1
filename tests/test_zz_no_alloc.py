"""The allocation-free amax + quantize entry point.

Callers that cannot allocate device memory (a real-time loop that allocates
nothing after start-up, a plugin whose memory belongs to its host's
allocator, an embedded caller with no allocator of its own) call
aexrt_b200_act_quantize_f16_noalloc, which keeps the amax scratch in a fixed
array inside the library.  Its results must equal those of the two ordinary
entry points (aexrt_b200_act_amax_f16 + aexrt_b200_act_quantize_f16, caller
scratch) bit for bit, on consecutive calls: the second call must not see the
first call's maxima left in the shared array.

This file is collected last on purpose (see the file name).
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _act(rng, shape, scale):
    z = rng.standard_normal(shape).astype(np.float32)
    return (scale * z / (1 + np.exp(-z))).astype(np.float16)


def _noalloc(lib, x, layout, c, h, w, ldc, mode, stride, q, rec):
    n = x.shape[0]
    return lib.aexrt_b200_act_quantize_f16_noalloc(x.data_ptr(), n, c, h, w, layout, ldc, 0, mode, stride,
                                                   q.data_ptr(), rec.data_ptr(), None)


def test_noalloc_matches_caller_scratch_on_consecutive_calls():
    import torch

    from aexrt_b200 import _native, ops

    lib = _native.load()
    rng = np.random.default_rng(99)
    cases = [
        # (layout, shape as stored, channels, h, w, mode, consumer stride, value scale)
        (ops.LAYOUT_NCHW_F16, (3, 48, 10, 12), 48, 10, 12, 0, 1, 4.0),
        (ops.LAYOUT_NHWC_F16, (2, 9, 11, 32), 32, 9, 11, 1, 2, 0.25),  # smaller values: stale maxima would show
        (ops.LAYOUT_NCHW_F16, (3, 48, 10, 12), 48, 10, 12, 0, 1, 0.5),
        # 20 x 8 = 160 (image, group) strips >= the SM count: the NCHW amax stores one block's maximum
        # per strip instead of clearing and max-ing; after a call with larger values, a stale slot
        # would show
        (ops.LAYOUT_NCHW_F16, (20, 128, 6, 5), 128, 6, 5, 0, 1, 8.0),
        (ops.LAYOUT_NCHW_F16, (20, 128, 6, 5), 128, 6, 5, 1, 1, 0.125),
    ]
    for layout, shape, c, h, w, mode, stride, scale in cases:
        x = torch.from_numpy(_act(rng, shape, scale)).cuda()
        n = shape[0]
        # the ordinary path, with caller-owned amax scratch
        amax = ops.act_amax(x, layout)
        q_ref, rec_ref = ops.act_quantize(x, amax, mode, layout, consumer_stride=stride)
        # the allocation-free path into fresh outputs
        q = torch.full_like(q_ref, 77)
        rec = torch.full_like(rec_ref, -1.0)
        assert _noalloc(lib, x, layout, c, h, w, shape[-1] if layout == ops.LAYOUT_NHWC_F16 else c, mode, stride, q,
                        rec) == 1, _native.last_error()
        torch.cuda.synchronize()
        assert torch.equal(q, q_ref)
        assert torch.equal(rec, rec_ref)


def test_noalloc_rejects_more_slots_than_the_fixed_array():
    from aexrt_b200 import _native

    lib = _native.load()
    # 2048 images x 64 groups > 65536 slots: refused before any launch (no pointer is touched)
    dummy = ctypes.c_void_p(16)
    assert lib.aexrt_b200_act_quantize_f16_noalloc(dummy, 2048, 1024, 4, 4, 1, 1024, 0, 0, 1, dummy, dummy,
                                                   None) == 0
    assert "exceed" in _native.last_error()


def test_noalloc_rejects_more_images_than_a_launch_takes():
    from aexrt_b200 import _native

    lib = _native.load()
    # 65536 images of 16 channels fit the 65536 slots but not a grid dimension: refused with a message
    dummy = ctypes.c_void_p(16)
    assert lib.aexrt_b200_act_quantize_f16_noalloc(dummy, 65536, 16, 1, 1, 1, 16, 0, 0, 1, dummy, dummy,
                                                   None) == 0
    assert "65535" in _native.last_error()
