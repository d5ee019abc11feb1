"""CPU oracle for the W8A8 convolution path (TEST INFRASTRUCTURE ONLY).

This module restates, on the CPU, the arithmetic of the reference's W8A8 path so
that the CUDA kernels of ``aexrt_b200`` can be checked against it.  Only
``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl
reference`` legs of ``bench.py`` may import it; the product never does.

Reference being restated (paths relative to the reference project root):

* weight quantizer ``_add_packed_conv_int8``      src/aexrt/engine.py:2418-2465
  (C++ twin ``ensure_conv_int8_weight``           native/aexrt_d3d12_runtime.cpp:21716-21742)
* activation amax ``aexrt_int8_quant_amax``      native/aexrt_d3d12_runtime.cpp:3212-3275
* activation pack ``aexrt_int8_quant_pack[_pg]`` native/aexrt_d3d12_runtime.cpp:3277-3361
* per-tensor prequant conv (kernels 51/52/53)    native/aexrt_d3d12_runtime.cpp:4614-4762
* pg16 prequant conv / LTS group ordering        native/aexrt_d3d12_runtime.cpp:4770-4923, 3440-3468, 3594-3618
* int8 guard ``can_use_conv_int8``               native/aexrt_d3d12_runtime.cpp:9398-9422

Parity pins:
* the weight quantizer is pinned bit-for-bit against the reference compiler's own
  layout-8 output (``tests/golden/make_golden.py`` imports the reference in the
  build container and stores its bytes in ``tests/golden/weights_layout8.npz``);
* the pg16 dequant order is pinned by the reference's known-answer test
  ``mobile/hal/vk_hal.c:187-252`` (LCG seed 12345, K=256, OC=8), restated in
  ``pg16_known_answer``;
* activation amax / pack and the int32 accumulation have no golden vectors in
  the reference (its only int8 test is a GPU-gated legacy kernel); they are pinned
  to the HLSL source lines above and to fixtures generated from this restatement.

Batch semantics: the reference computes the activation amax over the whole
tensor viewed as ``[C][N*H*W]`` (correct only at batch 1).  This oracle, like the
CUDA path, keeps one amax per image (per sample ``n``), which is the reference's
batch-1 behaviour applied image by image.
"""
from __future__ import annotations

import ctypes
import os
from typing import Optional, Tuple

import numpy as np

F32 = np.float32
SCALE_PER_TENSOR = 0
SCALE_PG16 = 1

# ----------------------------------------------------------------------------
# a1: weight quantizer (engine.py:2418-2465)
# ----------------------------------------------------------------------------


def quantize_conv_weight_int8(weight: np.ndarray, fp16_engine: bool = False) -> Tuple[np.ndarray, np.ndarray]:
    """Symmetric per-output-channel int8 weight quantization (layout 8).

    Follows src/aexrt/engine.py:2447-2457: ``scale = amax/127`` (1.0 when the
    channel is all zero), ``p = w * fl32(1/scale)``, ``q = sign(p)*floor(|p|+0.5)``
    clipped to [-127, 127].  FP16 engines round the fp32 weights through fp16
    first (engine.py:2443-2444).  Returns ``(q[OC, IC*KH*KW] int8, scale[OC] f32)``.
    """
    w = np.ascontiguousarray(weight, dtype="<f4")
    oc = w.shape[0]
    src = w.reshape(oc, -1)
    if fp16_engine:
        src = src.astype("<f2").astype(F32)
    amax = np.abs(src).max(axis=1) if oc else np.zeros(0, dtype=F32)
    scale = np.where(amax > 0.0, amax / F32(127.0), F32(1.0)).astype(F32)
    inv = (F32(1.0) / scale).astype(F32)
    prod = (src * inv[:, None]).astype(F32)
    q = np.sign(prod) * np.floor(np.abs(prod) + F32(0.5))
    q = np.clip(q, F32(-127.0), F32(127.0)).astype(np.int8)
    return q, scale


def layout8_payload(q: np.ndarray, scale: np.ndarray) -> bytes:
    """Layout-8 bytes: ``[OC*IC*KK int8 in [oc][ic][kk] order][OC fp32 scale]`` (engine.py:2458)."""
    return np.ascontiguousarray(q, dtype=np.int8).tobytes(order="C") + np.asarray(scale, dtype="<f4").tobytes(order="C")


# ----------------------------------------------------------------------------
# a3 / a4: activation amax and pack (aexrt_d3d12_runtime.cpp:3212-3361)
# ----------------------------------------------------------------------------


def act_amax(x: np.ndarray) -> Tuple[np.ndarray, np.ndarray]:
    """Per-image amax of |x| for an NCHW tensor.

    Returns ``(amax_tensor[N] f32, amax_group[N, C/16] f32)``: slot 0 and slots
    ``1+g`` of the reference's amax buffer (runtime.cpp:3241-3258), one set per
    image.  Values are compared as fp32 (fp16 inputs widen exactly).
    """
    xf = np.abs(np.asarray(x).astype(F32))
    n, c = xf.shape[:2]
    g = (c + 15) // 16
    if c % 16:  # a trailing partial group (in_channels % 4 == 0 is all the guard asks)
        pad = np.zeros((n, g * 16 - c) + xf.shape[2:], F32)
        xf = np.concatenate([xf, pad], axis=1)
    per_group = xf.reshape(n, g, -1).max(axis=2) if xf.size else np.zeros((n, g), F32)
    per_tensor = per_group.max(axis=1) if c else np.zeros(n, F32)
    return per_tensor.astype(F32), per_group.astype(F32)


def act_scale(amax: np.ndarray) -> np.ndarray:
    """Quantizer multiplier ``s = fl32(127 / amax)`` (runtime.cpp:3337), 0 where amax <= 0."""
    a = np.asarray(amax, dtype=F32)
    with np.errstate(divide="ignore"):
        s = np.where(a > 0, F32(127.0) / np.where(a > 0, a, F32(1.0)), F32(0.0))
    return s.astype(F32)


def dequant_scale(amax: np.ndarray) -> np.ndarray:
    """Conv-side activation scale ``fl32(amax / 127)`` (runtime.cpp:4650, 4805)."""
    return (np.asarray(amax, dtype=F32) / F32(127.0)).astype(F32)


def quantize_act(x: np.ndarray, amax_t: np.ndarray, amax_g: np.ndarray, mode: int) -> np.ndarray:
    """int8 codes of an NCHW activation (runtime.cpp:3333-3344).

    ``q = round_half_even(fl32(x) * s)`` with NO clamp: the code is the low byte
    of the int (``uint(q) & 0xFF``).  An image/group whose amax is <= 0 gets all
    zero codes.  ``mode`` selects the per-tensor (slot 0) or pg16 (slot 1+g) amax.
    """
    xf = np.asarray(x).astype(F32)
    n, c = xf.shape[:2]
    if mode == SCALE_PER_TENSOR:
        s = act_scale(amax_t).reshape(n, 1, 1)
        xs = xf.reshape(n, c, -1)
    else:
        s = act_scale(amax_g).reshape(n, c // 16, 1, 1)
        xs = xf.reshape(n, c // 16, 16, -1)
    prod = (xs * s).astype(F32)
    q = np.rint(prod).astype(np.int64)
    q = (q & 0xFF).astype(np.uint8).view(np.int8)
    return q.reshape(xf.shape)


# ----------------------------------------------------------------------------
# a9: the int8 guard (runtime.cpp:9398-9422)
# ----------------------------------------------------------------------------


def conv_out_hw(h: int, w: int, k: int, s: int, p: int) -> Tuple[int, int]:
    return (h + 2 * p - k) // s + 1, (w + 2 * p - k) // s + 1


def can_use_conv_int8(ic: int, oc: int, h: int, w: int, oh: int, ow: int, k: int, s: int, p: int, groups: int = 1) -> bool:
    """Shape guard of kernels 51/52/53 (runtime.cpp:9398-9422)."""
    if groups != 1 or ic % 4 or oc % 4:
        return False
    if k == 1:
        return s == 1 and p == 0 and oc % 8 == 0 and h == oh and w == ow
    if k == 3:
        if p != 1:
            return False
        if s == 2:
            return h >= oh * 2 - 1 and w >= ow * 2 - 1
        return s == 1 and h == oh and w == ow
    return False


# ----------------------------------------------------------------------------
# a6 / a7: int32 accumulation and epilogue (runtime.cpp:4614-4923)
# ----------------------------------------------------------------------------


_CLIB = None


def _clib():
    """The C restatement of the accumulation loops (oracle/w8a8_ref.c), or None."""
    global _CLIB
    if _CLIB is None:
        path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "liboracle_w8a8.so")
        if os.path.exists(path):
            lib = ctypes.CDLL(path)
            lib.oracle_conv_acc_i32.restype = None
            lib.oracle_conv_acc_i32.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p] + [ctypes.c_int] * 10
            lib.oracle_conv_f32.restype = None
            lib.oracle_conv_f32.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p] + [ctypes.c_int] * 10
            _CLIB = lib
        else:
            _CLIB = False
    return _CLIB or None


def _im2col(xq: np.ndarray, k: int, s: int, p: int, oh: int, ow: int, group_major: bool) -> np.ndarray:
    """im2col of NCHW -> [N, OH*OW, K] with K ordered (ic, kh, kw)."""
    n, c, h, w = xq.shape
    xp = np.zeros((n, c, h + 2 * p, w + 2 * p), dtype=xq.dtype)
    xp[:, :, p:p + h, p:p + w] = xq
    cols = np.empty((n, c, k, k, oh, ow), dtype=xq.dtype)
    for kh in range(k):
        for kw in range(k):
            cols[:, :, kh, kw] = xp[:, :, kh:kh + s * (oh - 1) + 1:s, kw:kw + s * (ow - 1) + 1:s]
    return cols.reshape(n, c * k * k, oh * ow).transpose(0, 2, 1)


def conv_acc_i32(xq: np.ndarray, wq: np.ndarray, k: int, s: int, p: int, group_ch: Optional[int] = None) -> np.ndarray:
    """Exact integer convolution of int8 codes.

    ``xq`` is NCHW int8, ``wq`` is ``[OC, IC*K*K]`` int8 in (ic, kh, kw) order.
    Returns int32 ``[N, OC, OH, OW]`` when ``group_ch`` is None, otherwise the
    per-16-channel-group partial sums ``[N, G, OC, OH, OW]`` that the pg16
    kernels convert to float one group at a time (runtime.cpp:3594-3618).
    """
    n, c, h, w = xq.shape
    oc = wq.shape[0]
    oh, ow = conv_out_hw(h, w, k, s, p)
    lib = _clib()
    if group_ch is None and lib is not None:
        xc = np.ascontiguousarray(xq, dtype=np.int8)
        wc = np.ascontiguousarray(wq, dtype=np.int8)
        out = np.empty((n, oc, oh, ow), dtype=np.int32)
        lib.oracle_conv_acc_i32(xc.ctypes.data, wc.ctypes.data, out.ctypes.data, n, c, h, w, oc, oh, ow, k, s, p)
        return out
    cols = _im2col(xq.astype(np.int32), k, s, p, oh, ow, False)  # [N, P, C*K*K]
    wt = wq.astype(np.int32)  # [OC, C*K*K]
    if group_ch is None:
        acc = cols @ wt.T  # [N, P, OC]
        return np.ascontiguousarray(acc.transpose(0, 2, 1).reshape(n, oc, oh, ow)).astype(np.int32)
    g = c // group_ch
    kk = k * k
    cols_g = cols.reshape(n, oh * ow, g, group_ch * kk)
    wt_g = wt.reshape(oc, g, group_ch * kk)
    acc = np.einsum("npgk,ogk->ngop", cols_g, wt_g, optimize=True)
    return acc.reshape(n, g, oc, oh, ow).astype(np.int32)


def silu_f32(y: np.ndarray) -> np.ndarray:
    """``y / (1 + exp(-y))`` in fp32 (runtime.cpp:4670)."""
    y = np.asarray(y, dtype=F32)
    with np.errstate(over="ignore"):
        return (y / (F32(1.0) + np.exp(-y).astype(F32))).astype(F32)


def epilogue_per_tensor(acc: np.ndarray, amax_t: np.ndarray, w_scale: np.ndarray, bias: np.ndarray) -> np.ndarray:
    """``fl32(fl32(float(acc) * in_scale) * w_scale[oc]) + bias[oc]`` (runtime.cpp:4753-4754)."""
    n, oc = acc.shape[:2]
    in_scale = dequant_scale(amax_t).reshape(n, 1, 1, 1)
    y = (acc.astype(F32) * in_scale).astype(F32)
    y = (y * np.asarray(w_scale, F32).reshape(1, oc, 1, 1)).astype(F32)
    return (y + np.asarray(bias, F32).reshape(1, oc, 1, 1)).astype(F32)


def pg16_sum(acc_g: np.ndarray, gscale: np.ndarray) -> np.ndarray:
    """``sum_g fl32(fl32(S_g) * gscale[n, g])`` accumulated in fp32 in ascending g.

    ``acc_g`` is ``[N, G, OC, ...]`` int32, ``gscale`` ``[N, G]`` fp32.  This is
    the float part of the pg16 kernels (runtime.cpp:3466-3468, 3616-3618) and of
    the reference's known-answer check (mobile/hal/vk_hal.c:238-245).  The
    shader source's ``fp += float(sub) * gs`` leaves contraction to its
    compiler; the CUDA kernels fuse each step into one FMA, so their fp32 sums
    may differ from these two-rounding sums in the last bit, which the fp16
    output tolerance absorbs.
    """
    n, g, oc = acc_g.shape[:3]
    gs = np.asarray(gscale, dtype=F32).reshape(n, g)
    extra = (1,) * (acc_g.ndim - 3)
    fp = np.zeros((n, oc) + acc_g.shape[3:], dtype=F32)
    for gi in range(g):
        fp = (fp + (acc_g[:, gi].astype(F32) * gs[:, gi].reshape((n, 1) + extra)).astype(F32)).astype(F32)
    return fp


def epilogue_pg16(acc_g: np.ndarray, amax_g: np.ndarray, w_scale: np.ndarray, bias: np.ndarray) -> np.ndarray:
    """``fp = sum_g fl32(S_g) * fl32(amax_g/127)`` in ascending g, then ``fp*w_scale + bias``.

    The per-group integer sub-sums and the ascending float accumulation follow
    the LTS kernels (runtime.cpp:3450-3468 and 3594-3618).
    """
    n, g, oc = acc_g.shape[:3]
    fp = pg16_sum(acc_g, dequant_scale(amax_g))
    y = (fp * np.asarray(w_scale, F32).reshape(1, oc, 1, 1)).astype(F32)
    return (y + np.asarray(bias, F32).reshape(1, oc, 1, 1)).astype(F32)


def conv_w8a8(
    x: np.ndarray,
    weight: np.ndarray,
    bias: np.ndarray,
    k: int,
    s: int,
    p: int,
    mode: int = SCALE_PER_TENSOR,
    silu: bool = True,
    residual: Optional[np.ndarray] = None,
    fp16_engine: bool = False,
    wq: Optional[np.ndarray] = None,
    w_scale: Optional[np.ndarray] = None,
) -> dict:
    """One W8A8 conv layer (CS2 step 4 int8 branch, runtime.cpp:23935-24318).

    ``x`` is NCHW fp16 (or fp32), ``weight`` ``[OC, IC, K, K]`` fp32.  Returns a
    dict with every intermediate the CUDA path is checked against: ``amax_t``,
    ``amax_g``, ``xq`` (int8 codes), ``acc`` (int32; per-tensor mode) or
    ``acc_g`` (int32 per group; pg16), ``y32`` (fp32 epilogue) and ``y`` (fp16).
    The residual (C2f tail) is added after SiLU in fp32, as the reference's
    BINARY Add does on the unfused sequence.
    """
    if wq is None:
        wq, w_scale = quantize_conv_weight_int8(weight, fp16_engine)
    amax_t, amax_g = act_amax(x)
    xq = quantize_act(x, amax_t, amax_g, mode)
    out = {"amax_t": amax_t, "amax_g": amax_g, "xq": xq, "wq": wq, "w_scale": w_scale}
    if mode == SCALE_PER_TENSOR:
        acc = conv_acc_i32(xq, wq, k, s, p)
        out["acc"] = acc
        y = epilogue_per_tensor(acc, amax_t, w_scale, bias)
    else:
        acc_g = conv_acc_i32(xq, wq, k, s, p, group_ch=16)
        out["acc_g"] = acc_g
        out["acc"] = acc_g.sum(axis=1, dtype=np.int64).astype(np.int32)
        y = epilogue_pg16(acc_g, amax_g, w_scale, bias)
    if silu:
        y = silu_f32(y)
    if residual is not None:
        y = (y + np.asarray(residual).astype(F32)).astype(F32)
    out["y32"] = y
    out["y"] = y.astype(np.float16)
    return out


# ----------------------------------------------------------------------------
# Known-answer test of the reference (mobile/hal/vk_hal.c:187-252)
# ----------------------------------------------------------------------------


def pg16_known_answer() -> Tuple[np.ndarray, np.ndarray, np.ndarray, np.ndarray, np.ndarray]:
    """Inputs and CPU expectation of the reference's pg16 quantized-GEMM check.

    LCG ``st = st*1664525 + 1013904223`` from seed 12345; ``a[k] = ((st>>20)%200)-100``
    for K=256, then ``w[o*K+k] = ((st>>20)%60)-30`` for OC=8; group scales
    ``0.01 + 0.005*g``; weight scales ``0.02 + 0.001*o``; expected
    ``out[o] = (sum_g float(sum_{k in g} a*w) * as[g]) * ws[o]`` (vk_hal.c:189-195, 238-247).
    Returns ``(a, w, a_scale, w_scale, expect)``.
    """
    K, OC = 256, 8
    st = 12345
    a = np.empty(K, np.int8)
    w = np.empty(K * OC, np.int8)
    for i in range(K):
        st = (st * 1664525 + 1013904223) & 0xFFFFFFFF
        a[i] = ((st >> 20) % 200) - 100
    for i in range(K * OC):
        st = (st * 1664525 + 1013904223) & 0xFFFFFFFF
        w[i] = ((st >> 20) % 60) - 30
    groups = K // 16
    a_scale = np.array([F32(0.01) + F32(0.005) * F32(g) for g in range(groups)], F32)
    w_scale = np.array([F32(0.02) + F32(0.001) * F32(o) for o in range(OC)], F32)
    expect = np.empty(OC, F32)
    for o in range(OC):
        acc = F32(0.0)
        for g in range(groups):
            gsum = int(np.dot(a[g * 16:(g + 1) * 16].astype(np.int64), w[o * K + g * 16:o * K + (g + 1) * 16].astype(np.int64)))
            acc = F32(acc + F32(F32(gsum) * a_scale[g]))
        expect[o] = F32(acc * w_scale[o])
    return a, w.reshape(OC, K), a_scale, w_scale, expect


# ----------------------------------------------------------------------------
# fp16 reference ops used by the model-level oracle (not W8A8)
# ----------------------------------------------------------------------------


def conv_f32(x: np.ndarray, weight: np.ndarray, bias: Optional[np.ndarray], k: int, s: int, p: int) -> np.ndarray:
    """Plain fp32 conv (NCHW) used for the fp16 stem/head of the model oracle."""
    n, c, h, w = x.shape
    oc = weight.shape[0]
    oh, ow = conv_out_hw(h, w, k, s, p)
    lib = _clib()
    xf = np.ascontiguousarray(x, dtype=F32)
    wf = np.ascontiguousarray(weight, dtype=F32).reshape(oc, -1)
    if lib is not None:
        out = np.empty((n, oc, oh, ow), dtype=F32)
        lib.oracle_conv_f32(xf.ctypes.data, wf.ctypes.data, out.ctypes.data, n, c, h, w, oc, oh, ow, k, s, p)
    else:
        cols = _im2col(xf, k, s, p, oh, ow, False)
        out = np.ascontiguousarray((cols @ wf.T).transpose(0, 2, 1).reshape(n, oc, oh, ow)).astype(F32)
    if bias is not None:
        out = (out + np.asarray(bias, F32).reshape(1, oc, 1, 1)).astype(F32)
    return out
