"""ctypes binding of ``libaexrt_b200.so`` (the C ABI in include/aexrt_b200.h).

This plays the role of the reference's ``src/aexrt/cpp_runtime.py`` (which binds
``aexrt_native_cpp.dll`` with ctypes, cpp_runtime.py:543-662): it loads the
in-tree library, declares every entry point's signature and turns a 0 status
into a Python exception carrying ``aexrt_b200_get_last_error()``.  There is no
fallback: if the library is missing, importing the backend fails loudly.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, c_char_p, c_float, c_int, c_uint32, c_uint64, c_void_p

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libaexrt_b200.so")
HEADER_PATH = os.path.join(os.path.dirname(HERE), "include", "aexrt_b200.h")
LAUNCH_PROGRAMMATIC = 1  # AEXRT_B200_LAUNCH_PROGRAMMATIC


class AexrtConv2DDesc(ctypes.Structure):
    """Same field order as the reference's AexrtConv2DDesc (native/aexrt.h:98-115)."""

    _fields_ = [(name, c_uint32) for name in (
        "batch", "in_channels", "in_h", "in_w", "out_channels", "out_h", "out_w", "kernel_h", "kernel_w",
        "stride_h", "stride_w", "pad_top", "pad_left", "dilation_h", "dilation_w", "groups",
    )]


class AexrtB200ConvPlanInfo(ctypes.Structure):
    _fields_ = [(name, c_uint32) for name in (
        "struct_size", "kernel_id", "flags", "kind", "is_f16", "tile_w", "tile_h", "block_n", "k_slots", "stages",
        "smem_bytes", "grid_m", "grid_n", "in_hp", "in_wp", "grid", "variant", "pitch", "image_input",
        "quant_on_load", "staged_out",
    )]


class AexrtB200ActSource(ctypes.Structure):
    _fields_ = [("ptr", c_void_p), ("layout", c_uint32), ("ldc", c_uint32), ("coff", c_uint32), ("channels", c_uint32),
                ("upsample", c_uint32), ("src_h", c_uint32), ("src_w", c_uint32), ("amax_groups", c_void_p),
                ("amax_stride", c_uint32), ("amax_goff", c_uint32)]


class AexrtB200DecodeLevel(ctypes.Structure):
    _fields_ = [("box", c_void_p), ("box_ldc", c_uint32), ("box_coff", c_uint32), ("cls", c_void_p),
                ("cls_ldc", c_uint32), ("cls_coff", c_uint32), ("h", c_uint32), ("w", c_uint32), ("stride", c_float)]


class AexrtYoloDetection(ctypes.Structure):
    """Same layout as the reference's AexrtYoloDetection (native/aexrt.h:25-32, cpp_runtime.py:43-51)."""

    _fields_ = [(name, c_float) for name in ("x1", "y1", "x2", "y2", "score", "class_id")]


class AexrtError(RuntimeError):
    """A C-ABI call returned failure; the message is the library's last error."""


_SIGNATURES = {
    "aexrt_b200_abi_version": (c_uint32, []),
    "aexrt_b200_set_launch_flags": (c_int, [c_uint32]),
    "aexrt_b200_get_launch_flags": (c_uint32, []),
    "aexrt_b200_get_last_error": (c_char_p, []),
    "aexrt_b200_device_count": (c_int, []),
    "aexrt_b200_quantize_conv_weight_int8": (c_int, [c_void_p, c_uint32, c_uint32, c_uint32, c_uint32, c_void_p, c_void_p]),
    "aexrt_b200_act_amax_f16": (c_int, [c_void_p] + [c_uint32] * 7 + [c_void_p, c_uint32, c_uint32, c_uint32, c_void_p]),
    "aexrt_b200_packed_act_bytes": (c_uint64, [c_uint32] * 5),
    "aexrt_b200_act_quantize_f16": (c_int, [c_void_p] + [c_uint32] * 7 + [c_void_p, c_uint32, c_uint32, c_uint32, c_uint32,
                                                                         c_void_p, c_void_p, c_void_p]),
    "aexrt_b200_conv_plan_create": (c_void_p, [POINTER(AexrtConv2DDesc), c_uint32, c_uint32, c_uint32, c_void_p, c_void_p,
                                               c_void_p, c_uint32]),
    "aexrt_b200_conv_plan_create_f16": (c_void_p, [POINTER(AexrtConv2DDesc), c_uint32, c_void_p, c_void_p, c_uint32]),
    "aexrt_b200_conv_plan_info": (c_int, [c_void_p, POINTER(AexrtB200ConvPlanInfo)]),
    "aexrt_b200_conv_plan_destroy": (None, [c_void_p]),
    "aexrt_b200_conv_w8a8": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_uint32, c_uint32, c_void_p, c_uint32, c_uint32,
                                     c_void_p, c_uint32, c_uint32, c_void_p, c_void_p]),
    "aexrt_b200_conv_w8a8_sources": (c_int, [c_void_p, POINTER(AexrtB200ActSource), c_uint32, c_void_p, c_uint32,
                                             c_uint32, c_void_p, c_uint32, c_uint32, c_void_p, c_uint32, c_uint32,
                                             c_void_p, c_void_p]),
    "aexrt_b200_conv_f16": (c_int, [c_void_p, c_void_p, c_void_p, c_uint32, c_uint32, c_void_p, c_uint32, c_uint32, c_void_p,
                                    c_uint32, c_uint32, c_void_p]),
    "aexrt_b200_conv_f16_image": (c_int, [c_void_p, c_void_p, c_uint32, c_void_p, c_uint32, c_uint32, c_void_p, c_uint32,
                                          c_uint32, c_void_p]),
    "aexrt_b200_conv_f16_nhwc": (c_int, [c_void_p, c_void_p, c_uint32, c_uint32, c_void_p, c_uint32, c_uint32,
                                         c_void_p, c_uint32, c_uint32, c_void_p, c_uint32, c_uint32, c_void_p]),
    "aexrt_b200_conv_status": (c_int, [c_void_p, POINTER(c_uint32)]),
    "aexrt_b200_packed_f16_bytes": (c_uint64, [c_uint32] * 5),
    "aexrt_b200_pack_f16": (c_int, [c_void_p] + [c_uint32] * 8 + [c_void_p, c_void_p]),
    "aexrt_b200_act_quantize_concat": (c_int, [POINTER(AexrtB200ActSource), c_uint32, c_uint32, c_uint32, c_uint32,
                                               c_uint32, c_uint32, c_void_p, c_void_p, c_void_p]),
    "aexrt_b200_pack_f16_concat": (c_int, [POINTER(AexrtB200ActSource), c_uint32, c_uint32, c_uint32, c_uint32,
                                           c_uint32, c_void_p, c_void_p]),
    "aexrt_b200_sppf_pool": (c_int, [c_void_p] + [c_uint32] * 6 + [c_void_p, c_uint32, c_uint32, c_void_p, c_uint32,
                                                                   c_uint32, c_void_p]),
    "aexrt_b200_yolo_decode": (c_int, [POINTER(AexrtB200DecodeLevel), c_uint32, c_uint32, c_uint32, c_uint32, c_void_p,
                                       c_void_p]),
    "aexrt_b200_dwconv3x3_f16": (c_int, [c_void_p] + [c_uint32] * 9 + [c_void_p, c_void_p, c_uint32, c_uint32,
                                                                        c_void_p, c_uint32, c_uint32, c_void_p]),
    "aexrt_b200_psa_attention_f16": (c_int, [c_void_p] + [c_uint32] * 8 + [c_float, c_void_p, c_uint32, c_uint32,
                                                                            c_void_p, c_uint32, c_uint32, c_void_p,
                                                                            c_uint32, c_uint32, c_void_p]),
    "aexrt_b200_yolo_nms_topk": (c_int, [c_void_p] + [c_uint32] * 6 + [c_float, c_float] + [c_uint32] * 3
                                 + [c_void_p, c_void_p, c_void_p]),
    "aexrt_b200_act_amax_quantize_f16": (c_int, [c_void_p] + [c_uint32] * 5 + [c_void_p, c_uint32, c_uint32, c_void_p,
                                                                             c_void_p, c_void_p]),
    "aexrt_b200_act_amax_quantize_f16_wait_limit": (c_int, [c_void_p] + [c_uint32] * 5 + [c_void_p, c_uint32, c_uint32,
                                                                                        c_void_p, c_void_p, c_uint64,
                                                                                        c_void_p]),
    "aexrt_b200_act_status": (c_int, [POINTER(c_uint32)]),
    "aexrt_b200_zero": (c_int, [c_void_p, c_uint64, c_void_p]),
    "aexrt_b200_act_quantize_f16_noalloc": (c_int, [c_void_p] + [c_uint32] * 9 + [c_void_p, c_void_p, c_void_p]),
}

_LIB = None


def load() -> ctypes.CDLL:
    """Loads the library once and declares all signatures."""
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"{LIB_PATH} is missing: build it with `python -m aexrt_b200.build` (the W8A8 path has no fallback)")
        lib = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in _SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _LIB = lib
    return _LIB


def last_error() -> str:
    msg = load().aexrt_b200_get_last_error()
    return msg.decode() if msg else ""


def check(status: int, what: str) -> None:
    if not status:
        raise AexrtError(f"{what} failed: {last_error()}")


def header_functions() -> list:
    """Names of the functions declared in include/*.h (for the ABI test): the kernel-level ABI
    (aexrt_b200.h) and the reference runtime ABI (aexrt_yolo.h)."""
    import glob
    import re

    names = set()
    for path in glob.glob(os.path.join(os.path.dirname(HEADER_PATH), "*.h")):
        text = re.sub(r"/\*.*?\*/", "", open(path, encoding="utf-8").read(), flags=re.S)
        names.update(re.findall(r"\b(aexrt_[a-z0-9_]+)\s*\(", text))
    return sorted(names)
