"""Tensor-level wrappers of the C ABI (torch is used only for device memory and streams).

The functions mirror the steps of the reference's int8 conv branch
(``record_replay_conv``, native/aexrt_d3d12_runtime.cpp:23935-24318):

* :func:`quantize_conv_weight_int8` — layout-8 weight quantizer (engine.py:2418-2465)
* :func:`act_amax`                   — aexrt_int8_quant_zero + _amax (runtime.cpp:3159-3275)
* :func:`act_quantize`               — aexrt_int8_quant_pack[_pg] (runtime.cpp:3277-3361)
* :class:`ConvPlan` / :meth:`ConvPlan.run` — prequant conv kernels 51/52/53 (runtime.cpp:4614-4923)
* :func:`conv_w8a8_layer`            — the whole branch: amax -> quantize -> conv
* :func:`yolo_nms_topk`              — decode-filter + NMS + top-k (runtime.cpp:27104-27219)

Every device call goes through ``libaexrt_b200.so``; there is no CPU or
PyTorch fallback for any of them.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Optional, Tuple

import numpy as np

from . import _native
from ._native import AexrtB200ConvPlanInfo, AexrtConv2DDesc, check

KIND_CONV = 1
KIND_CONV_SILU = 2
PLAN_FLAG_INT8_PERGROUP = 1 << 4
PLAN_FLAG_QUANT_ON_LOAD = 1 << 8
LAYOUT_NHWC_F16 = 0
LAYOUT_NCHW_F16 = 1
LAYOUT_NCHW_F32 = 2
SCALE_PER_TENSOR = 0
SCALE_PG16 = 1
NMS_MARK = 0
NMS_GREEDY = 1
NMS_CTAS_SHIFT = 8  # AEXRT_B200_NMS_CTAS_SHIFT: mode bits 8-11 = CTAs per image


def _torch():
    import torch

    return torch


def _stream(stream=None) -> int:
    torch = _torch()
    if stream is None:
        return torch.cuda.current_stream().cuda_stream
    return int(getattr(stream, "cuda_stream", stream))


def _ptr(t) -> Optional[int]:
    return None if t is None else t.data_ptr()


def quantize_conv_weight_int8(weight: np.ndarray, fp16_engine: bool = False) -> Tuple[np.ndarray, np.ndarray]:
    """Layout-8 weight quantization on the host (bit-identical to engine.py:2447-2457)."""
    w = np.ascontiguousarray(weight, dtype=np.float32)
    oc = w.shape[0]
    kk = int(np.prod(w.shape[2:])) if w.ndim > 2 else 1
    ic = w.shape[1] if w.ndim > 1 else 1
    codes = np.empty((oc, ic * kk), dtype=np.int8)
    scale = np.empty(oc, dtype=np.float32)
    check(_native.load().aexrt_b200_quantize_conv_weight_int8(
        w.ctypes.data, oc, ic, kk, int(bool(fp16_engine)), codes.ctypes.data, scale.ctypes.data), "quantize weights")
    return codes, scale


def conv_desc(n, ic, h, w, oc, k, s, p) -> AexrtConv2DDesc:
    oh = (h + 2 * p - k) // s + 1
    ow = (w + 2 * p - k) // s + 1
    return AexrtConv2DDesc(n, ic, h, w, oc, oh, ow, k, k, s, s, p, p, 1, 1, 1)


def kernel_id_for(k: int, s: int) -> int:
    """The reference's int8 kernel ids: 51 = 1x1, 52 = 3x3 s1, 53 = 3x3 s2 (runtime.cpp:8881-8940)."""
    if k == 1 and s == 1:
        return 51
    if k == 3 and s == 1:
        return 52
    if k == 3 and s == 2:
        return 53
    raise ValueError(f"no int8 kernel for k={k} s={s}")


def amax_groups_tensor(n: int, groups: int, device="cuda"):
    torch = _torch()
    return torch.zeros((n, groups), dtype=torch.int32, device=device)


def act_amax(x, layout: int = LAYOUT_NCHW_F16, c: Optional[int] = None, ldc: Optional[int] = None, coff: int = 0,
             out=None, groups_total: Optional[int] = None, group_offset: int = 0, zero_first: bool = True, stream=None):
    """Per-image amax of |x| per 16-channel group, as uint32 float bits in an int32 tensor [N, G]."""
    if layout == LAYOUT_NHWC_F16:
        n, h, w, cc = x.shape
        c = c or (cc - coff)
        ldc = ldc or cc
    else:
        n, c, h, w = x.shape
        ldc = c
    g = (c + 15) // 16
    groups_total = groups_total or g
    if out is None:
        out = amax_groups_tensor(n, groups_total, x.device)
    check(_native.load().aexrt_b200_act_amax_f16(
        x.data_ptr(), n, c, h, w, layout, ldc, coff, out.data_ptr(), groups_total, group_offset, int(zero_first),
        _stream(stream)), "act_amax")
    return out


def packed_act_shape(n: int, c: int, h: int, w: int, stride: int = 1):
    hp = h + (h & 1 if stride == 2 else 0)
    wp = w + (w & 1 if stride == 2 else 0)
    return (n, (c + 15) // 16, hp, wp, 16)


def act_quantize(x, amax_groups, mode: int = SCALE_PER_TENSOR, layout: int = LAYOUT_NCHW_F16, consumer_stride: int = 1,
                 c: Optional[int] = None, ldc: Optional[int] = None, coff: int = 0, group_offset: int = 0,
                 q_out=None, rec_out=None, stream=None):
    """int8 codes in the slab16 layout + per-image scale record [N, 1 + slabs] (fp32 amax values)."""
    torch = _torch()
    if layout == LAYOUT_NHWC_F16:
        n, h, w, cc = x.shape
        c = c or (cc - coff)
        ldc = ldc or cc
    else:
        n, c, h, w = x.shape
        ldc = c
    shape = packed_act_shape(n, c, h, w, consumer_stride)
    if q_out is None:
        q_out = torch.empty(shape, dtype=torch.int8, device=x.device)
    if rec_out is None:
        rec_out = torch.empty((n, 1 + shape[1]), dtype=torch.float32, device=x.device)
    check(_native.load().aexrt_b200_act_quantize_f16(
        x.data_ptr(), n, c, h, w, layout, ldc, coff, amax_groups.data_ptr(), amax_groups.shape[1], group_offset, mode,
        consumer_stride, q_out.data_ptr(), rec_out.data_ptr(), _stream(stream)), "act_quantize")
    return q_out, rec_out


def act_amax_quantize(x, mode: int = SCALE_PER_TENSOR, amax_out=None, q_out=None, rec_out=None, stream=None):
    """Standalone amax + quantize of an fp16 NCHW tensor for a stride-1 consumer in one call:
    returns (codes slab16, scale record, amax slots [n, ceil(c/16)])."""
    torch = _torch()
    n, c, h, w = x.shape
    groups = (c + 15) // 16
    if amax_out is None:
        amax_out = torch.empty((n, groups), dtype=torch.int32, device=x.device)
    if q_out is None:
        q_out = torch.empty(packed_act_shape(n, c, h, w, 1), dtype=torch.int8, device=x.device)
    if rec_out is None:
        rec_out = torch.empty((n, 1 + groups), dtype=torch.float32, device=x.device)
    check(_native.load().aexrt_b200_act_amax_quantize_f16(x.data_ptr(), n, c, h, w, mode, amax_out.data_ptr(),
                                                          amax_out.shape[1], 0, q_out.data_ptr(), rec_out.data_ptr(),
                                                          _stream(stream)), "act_amax_quantize")
    return q_out, rec_out, amax_out


def act_status() -> int:
    """Reads and clears the activation kernels' status word of the current device."""
    v = ctypes.c_uint32(0)
    check(_native.load().aexrt_b200_act_status(ctypes.byref(v)), "act_status")
    return v.value


def pack_f16(x, layout: int = LAYOUT_NHWC_F16, consumer_stride: int = 1, c: Optional[int] = None,
             ldc: Optional[int] = None, coff: int = 0, out=None, stream=None):
    """fp16 slab8 repack [N, ceil(C/8), Hp, Wp, 8] for the fp16 convs."""
    torch = _torch()
    if layout == LAYOUT_NHWC_F16:
        n, h, w, cc = x.shape
        c = c or (cc - coff)
        ldc = ldc or cc
    else:
        n, c, h, w = x.shape
        ldc = c
    hp = h + (h & 1 if consumer_stride == 2 else 0)
    wp = w + (w & 1 if consumer_stride == 2 else 0)
    if out is None:
        out = torch.empty((n, (c + 7) // 8, hp, wp, 8), dtype=torch.float16, device=x.device)
    check(_native.load().aexrt_b200_pack_f16(x.data_ptr(), n, c, h, w, layout, ldc, coff, consumer_stride,
                                             out.data_ptr(), _stream(stream)), "pack_f16")
    return out


@dataclass
class PlanInfo:
    kernel_id: int
    flags: int
    kind: int
    is_f16: bool
    tile_w: int
    tile_h: int
    block_n: int
    k_slots: int
    stages: int
    smem_bytes: int
    grid_m: int
    grid_n: int
    in_hp: int
    in_wp: int
    grid: int = 0
    variant: int = 0
    pitch: int = 0
    image_input: int = 0
    quant_on_load: int = 0
    staged_out: int = 0

    @staticmethod
    def from_c(i: AexrtB200ConvPlanInfo) -> "PlanInfo":
        return PlanInfo(i.kernel_id, i.flags, i.kind, bool(i.is_f16), i.tile_w, i.tile_h, i.block_n, i.k_slots,
                        i.stages, i.smem_bytes, i.grid_m, i.grid_n, i.in_hp, i.in_wp, i.grid, i.variant, i.pitch,
                        i.image_input, i.quant_on_load, i.staged_out)


class ConvPlan:
    """A device-resident conv plan: one reference kernel-plan command (kind, kernel, flags).

    ``ConvPlan.int8(...)`` takes layout-8 codes/scales (the reference's packed
    weights) and builds kernel 51/52/53 per ``can_use_conv_int8``;
    ``ConvPlan.fp16(...)`` builds the fp16 conv used for the stem and head.
    """

    def __init__(self, handle: int, desc: AexrtConv2DDesc, is_f16: bool):
        self._h = handle
        self.desc = desc
        self.is_f16 = is_f16
        self.info = self._info()

    @classmethod
    def int8(cls, n, ic, h, w, oc, k, s, codes, w_scale, bias, silu=True, pg16=False, block_n=0,
             quant_on_load=False):
        p = k // 2
        desc = conv_desc(n, ic, h, w, oc, k, s, p)
        codes = np.ascontiguousarray(codes, dtype=np.int8)
        w_scale = np.ascontiguousarray(w_scale, dtype=np.float32)
        bias = np.ascontiguousarray(bias, dtype=np.float32)
        flags = (PLAN_FLAG_INT8_PERGROUP if pg16 else 0) | (PLAN_FLAG_QUANT_ON_LOAD if quant_on_load else 0)
        h_ = _native.load().aexrt_b200_conv_plan_create(
            ctypes.byref(desc), KIND_CONV_SILU if silu else KIND_CONV, kernel_id_for(k, s), flags, codes.ctypes.data,
            w_scale.ctypes.data, bias.ctypes.data, block_n)
        if not h_:
            raise _native.AexrtError("conv_plan_create failed: " + _native.last_error())
        return cls(h_, desc, False)

    @classmethod
    def fp16(cls, n, ic, h, w, oc, k, s, weight, bias, silu=True, block_n=0):
        p = k // 2
        desc = conv_desc(n, ic, h, w, oc, k, s, p)
        weight = np.ascontiguousarray(weight, dtype=np.float32)
        bias = np.ascontiguousarray(bias, dtype=np.float32)
        h_ = _native.load().aexrt_b200_conv_plan_create_f16(
            ctypes.byref(desc), KIND_CONV_SILU if silu else KIND_CONV, weight.ctypes.data, bias.ctypes.data, block_n)
        if not h_:
            raise _native.AexrtError("conv_plan_create_f16 failed: " + _native.last_error())
        return cls(h_, desc, True)

    def _info(self) -> PlanInfo:
        i = AexrtB200ConvPlanInfo()
        check(_native.load().aexrt_b200_conv_plan_info(self._h, ctypes.byref(i)), "conv_plan_info")
        return PlanInfo.from_c(i)

    @property
    def out_shape(self):
        d = self.desc
        return (d.batch, d.out_h, d.out_w, d.out_channels)

    def run(self, x, rec=None, out=None, out_coff: int = 0, residual=None, res_coff: int = 0, amax_out=None,
            amax_goff: int = 0, acc_dump=None, stream=None):
        """Launches the conv; ``out`` is an fp16 NHWC tensor whose last dim is the channel stride."""
        torch = _torch()
        if out is None:
            out = torch.empty(self.out_shape, dtype=torch.float16, device=x.device)
        out_ldc = out.shape[-1]
        res_ldc = residual.shape[-1] if residual is not None else 0
        amax_stride = amax_out.shape[-1] if amax_out is not None else 0
        lib = _native.load()
        if self.is_f16:
            check(lib.aexrt_b200_conv_f16(self._h, x.data_ptr(), _ptr(residual), res_ldc, res_coff, out.data_ptr(),
                                          out_ldc, out_coff, _ptr(amax_out), amax_stride, amax_goff, _stream(stream)),
                  "conv_f16")
        else:
            check(lib.aexrt_b200_conv_w8a8(self._h, x.data_ptr(), rec.data_ptr(), _ptr(residual), res_ldc, res_coff,
                                           out.data_ptr(), out_ldc, out_coff, _ptr(amax_out), amax_stride, amax_goff,
                                           _ptr(acc_dump), _stream(stream)), "conv_w8a8")
        return out

    def run_sources(self, srcs, out=None, out_coff: int = 0, residual=None, res_coff: int = 0, amax_out=None,
                    amax_goff: int = 0, acc_dump=None, stream=None, device=None):
        """Quantize-on-load plans: the conv reads the fp16 NHWC sources (a ctypes array of
        AexrtB200ActSource with their amax slots) and quantizes them in shared memory."""
        torch = _torch()
        if out is None:
            out = torch.empty(self.out_shape, dtype=torch.float16, device=device or "cuda")
        res_ldc = residual.shape[-1] if residual is not None else 0
        amax_stride = amax_out.shape[-1] if amax_out is not None else 0
        check(_native.load().aexrt_b200_conv_w8a8_sources(self._h, srcs, len(srcs), _ptr(residual), res_ldc, res_coff,
                                                          out.data_ptr(), out.shape[-1], out_coff, _ptr(amax_out),
                                                          amax_stride, amax_goff, _ptr(acc_dump), _stream(stream)),
              "conv_w8a8_sources")
        return out

    def run_nhwc(self, x, x_coff: int = 0, out=None, out_coff: int = 0, residual=None, res_coff: int = 0,
                 amax_out=None, amax_goff: int = 0, stream=None):
        """fp16 stride-1 halo plans: the conv reads channels x_coff .. x_coff + in_channels of the fp16
        NHWC tensor ``x`` directly (no slab8 copy)."""
        torch = _torch()
        if out is None:
            out = torch.empty(self.out_shape, dtype=torch.float16, device=x.device)
        amax_stride = amax_out.shape[-1] if amax_out is not None else 0
        res_ldc = residual.shape[-1] if residual is not None else 0
        check(_native.load().aexrt_b200_conv_f16_nhwc(self._h, x.data_ptr(), x.shape[-1], x_coff, _ptr(residual),
                                                      res_ldc, res_coff, out.data_ptr(), out.shape[-1], out_coff,
                                                      _ptr(amax_out), amax_stride, amax_goff, _stream(stream)),
              "conv_f16_nhwc")
        return out

    def run_image(self, images, out=None, out_coff: int = 0, amax_out=None, amax_goff: int = 0, stream=None):
        """The image stem: fp16 or fp32 NCHW ``images`` straight into the fp16 NHWC ``out``
        (plans with info.image_input)."""
        torch = _torch()
        if out is None:
            out = torch.empty(self.out_shape, dtype=torch.float16, device=images.device)
        amax_stride = amax_out.shape[-1] if amax_out is not None else 0
        layout = LAYOUT_NCHW_F16 if images.dtype == torch.float16 else LAYOUT_NCHW_F32
        check(_native.load().aexrt_b200_conv_f16_image(self._h, images.data_ptr(), layout, out.data_ptr(),
                                                       out.shape[-1], out_coff, _ptr(amax_out), amax_stride,
                                                       amax_goff, _stream(stream)), "conv_f16_image")
        return out

    def status(self) -> int:
        v = ctypes.c_uint32(0)
        check(_native.load().aexrt_b200_conv_status(self._h, ctypes.byref(v)), "conv_status")
        return v.value

    def close(self):
        if self._h:
            _native.load().aexrt_b200_conv_plan_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def conv_w8a8_layer(plan: ConvPlan, x_nhwc, mode: int = SCALE_PER_TENSOR, residual=None, out=None, amax_out=None,
                    stream=None):
    """The reference's int8 conv branch on an fp16 NHWC input: amax -> quantize -> conv."""
    d = plan.desc
    amax = act_amax(x_nhwc, LAYOUT_NHWC_F16, stream=stream)
    q, rec = act_quantize(x_nhwc, amax, mode, LAYOUT_NHWC_F16, consumer_stride=d.stride_h, stream=stream)
    return plan.run(q, rec, out=out, residual=residual, amax_out=amax_out, stream=stream)


def yolo_nms_topk(output0, nc: int, conf: float = 0.25, iou: float = 0.45, max_candidates: int = 512,
                  max_detections: int = 100, mode: int = NMS_MARK, has_objectness: bool = False,
                  channels_last: bool = False, dets=None, counts=None, stream=None, ctas_per_image: int = 0):
    """Detections of a batch of fp32 output0 tensors ([n, 4 + nc, anchors], or [n, anchors, 4 + nc]
    when `channels_last`): returns (dets [n, max_detections, 6] fp32 rows x1, y1, x2, y2, score,
    class; counts [n] int32).  Rows at and beyond counts[i] are zero.

    Defaults are the reference model's (runtime.cpp:551-561): 512 candidates, 100 detections,
    conf 0.25, IoU 0.45, the GPU path's NMS rule; ``mode=NMS_GREEDY`` gives yolo_postprocess's.
    ``ctas_per_image`` (0 automatic, else 1, 2, 4 or 8): the thread-block cluster that shares one
    image's pair tests; the detections do not depend on it."""
    torch = _torch()
    n = output0.shape[0]
    channels = output0.shape[2] if channels_last else output0.shape[1]
    anchors = output0.shape[1] if channels_last else output0.shape[2]
    if dets is None:
        dets = torch.zeros((n, max_detections, 6), dtype=torch.float32, device=output0.device)
    if counts is None:
        counts = torch.zeros((n,), dtype=torch.int32, device=output0.device)
    check(_native.load().aexrt_b200_yolo_nms_topk(
        output0.data_ptr(), n, channels, anchors, nc, int(has_objectness), 2 if channels_last else 1, conf, iou,
        max_candidates, max_detections, mode | (ctas_per_image << NMS_CTAS_SHIFT), dets.data_ptr(), counts.data_ptr(),
        _stream(stream)), "yolo_nms_topk")
    return dets, counts
