"""The reference's native YOLO model interface on ``libaexrt_b200.so``.

The reference drives its engines through ``NativeCppYoloModel``
(src/aexrt/cpp_runtime.py:229-441), a ctypes binding of the ``aexrt_yolo_*`` C
ABI of its D3D12 runtime (native/aexrt.h:271-486).  The same C ABI is exported
by this library (include/aexrt_yolo.h), so the reference's binding loads it
unchanged; this module is this backend's own binding of it, with the same
class name, methods, properties, argument meaning and error behaviour
(``RuntimeError`` carrying ``aexrt_yolo_get_last_error``), plus the batch
extensions of this backend (``images`` per run, ``run_batch``, device
pointers for callers that stream themselves).
"""
from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, Structure, byref, c_char_p, c_double, c_float, c_int, c_uint32, c_uint64, c_void_p
from dataclasses import dataclass
from typing import Dict, List, Optional, Tuple

import numpy as np

from . import _native
from ._native import AexrtConv2DDesc, AexrtYoloDetection


@dataclass(frozen=True)
class Detection:
    """One detection, as the reference's ``aexrt.yolo.Detection`` (src/aexrt/yolo.py:15-19)."""

    class_id: int
    score: float
    xyxy: Tuple[float, float, float, float]


class AexrtD3D12Capabilities(Structure):
    """native/aexrt.h:34-41."""

    _fields_ = [("struct_size", c_uint32), ("highest_shader_model", c_uint32), ("native_fp16_supported", c_uint32),
                ("wave_mma_tier", c_uint32), ("dxc_available", c_uint32), ("reserved", c_uint32 * 3)]


class AexrtYoloRunTiming(Structure):
    """native/aexrt.h:43-51."""

    _fields_ = [("struct_size", c_uint32), ("valid", c_uint32), ("memcpy_ms", c_double), ("submit_ms", c_double),
                ("fence_ms", c_double), ("readback_ms", c_double), ("reserved", c_uint64 * 4)]


class AexrtConvPlanInfo(Structure):
    """native/aexrt.h:435-445."""

    _fields_ = [("struct_size", c_uint32), ("command_index", c_uint32), ("kind_is_silu", c_uint32),
                ("desc", AexrtConv2DDesc), ("current_algorithm", c_uint32), ("candidate_count", c_uint32),
                ("candidates", c_uint32 * 32), ("in_fusion_group", c_uint32), ("planned_algorithm", c_uint32)]


_U32_GETTERS = (
    "class_count", "anchor_count", "channel_count", "output_layout", "has_objectness", "package_mode",
    "graph_node_count", "graph_value_count", "constant_count", "prepared_command_count",
    "supported_prepared_command_count", "unsupported_prepared_command_count", "prepared_skipped_command_count",
    "late_concat_conv1x1_fusion_count", "concat_residual_conv1x1_fusion_count", "paired_conv3x3_fusion_count",
    "c2f_bottleneck_superblock_count", "c2f_tail_residual_fusion_count", "head_fusion_enabled",
    "head_final_conv_fusion_enabled", "tileflow_conv1x1_count", "tileflow_3x3_spatial_count",
    "tileflow_3x3_pack4_count", "tileflow_3x3_pack8_count", "tileflow_3x3_implicit_gemm_count",
    "tileflow_3x3_implicit_gemm_40x40_count", "tileflow_3x3_implicit_gemm_20x20_count",
    "tileflow_3x3_implicit_gemm_10x10_count", "tileflow_3x3_exact_40x40_64x64_count",
    "tileflow_3x3_exact_20x20_64x64_count", "tileflow_3x3_exact_10x10_128x128_count",
    "tileflow_3x3_exact_20x20_128x64_count", "tileflow_3x3_exact_10x10_256x64_count",
    "tileflow_native_fp16_count", "dxil_cache_hit_count", "shader_cache_hit_count", "pso_cache_hit_count",
    "conv_plan_count", "profile_event_count",
)

# name -> (restype, argtypes): the reference binding's declarations (cpp_runtime.py:543-662)
# and this backend's extensions
SIGNATURES: Dict[str, tuple] = {
    "aexrt_d3d12_probe": (c_int, []),
    "aexrt_d3d12_create_device": (c_void_p, [c_uint32]),
    "aexrt_cuda_create_device": (c_void_p, [c_uint32]),
    "aexrt_d3d12_get_capabilities": (c_int, [c_void_p, POINTER(AexrtD3D12Capabilities)]),
    "aexrt_d3d12_destroy_device": (None, [c_void_p]),
    "aexrt_yolo_compile_from_package": (c_void_p, [c_void_p, c_char_p]),
    "aexrt_yolo_compile_from_onnx": (c_void_p, [c_void_p, c_char_p]),
    "aexrt_yolo_load_engine": (c_void_p, [c_void_p, c_char_p]),
    "aexrt_yolo_input_element_count": (c_uint64, [c_void_p]),
    "aexrt_yolo_is_executable": (c_int, [c_void_p]),
    "aexrt_yolo_run": (c_int, [c_void_p, c_void_p, POINTER(c_float), c_uint64, POINTER(AexrtYoloDetection), c_uint32,
                               POINTER(c_uint32)]),
    "aexrt_yolo_flush_pipeline": (c_int, [c_void_p, POINTER(AexrtYoloDetection), c_uint32, POINTER(c_uint32)]),
    "aexrt_yolo_get_last_error": (c_char_p, [c_void_p]),
    "aexrt_yolo_get_last_run_timing": (c_int, [c_void_p, POINTER(AexrtYoloRunTiming)]),
    "aexrt_yolo_profile_event_label": (c_char_p, [c_void_p, c_uint32]),
    "aexrt_yolo_profile_event_ms": (c_double, [c_void_p, c_uint32]),
    "aexrt_yolo_conv_plan_info": (c_int, [c_void_p, c_uint32, POINTER(AexrtConvPlanInfo)]),
    "aexrt_yolo_override_conv_algorithm": (c_int, [c_void_p, c_uint32, c_uint32]),
    "aexrt_yolo_input_ptr": (c_void_p, [c_void_p, POINTER(c_uint64)]),
    "aexrt_yolo_debug_output": (c_int, [c_void_p, POINTER(c_float), c_uint64]),
    "aexrt_yolo_debug_value": (c_int, [c_void_p, c_uint32, POINTER(c_float), c_uint64]),
    "aexrt_yolo_debug_page": (c_int, [c_void_p, c_uint32, POINTER(c_float), c_uint64]),
    "aexrt_yolo_pipeline_cache_size": (c_uint64, [c_void_p]),
    "aexrt_yolo_export_pipeline_cache": (c_int, [c_void_p, c_void_p, c_uint64]),
    "aexrt_yolo_destroy": (None, [c_void_p]),
    "aexrt_b200_engine_validate": (c_int, [c_void_p, c_uint64]),
    "aexrt_b200_yolo_load_engine_batch": (c_void_p, [c_void_p, c_char_p, c_uint32]),
    "aexrt_b200_yolo_batch": (c_uint32, [c_void_p]),
    "aexrt_b200_yolo_run_batch": (c_int, [c_void_p, c_void_p, c_uint32, POINTER(AexrtYoloDetection), c_uint32,
                                          POINTER(c_uint32)]),
    "aexrt_b200_yolo_set_input_dtype": (c_int, [c_void_p, c_uint32]),
    "aexrt_b200_yolo_device_input": (c_void_p, [c_void_p]),
    "aexrt_b200_yolo_device_output0": (c_void_p, [c_void_p]),
    "aexrt_b200_yolo_device_detections": (c_void_p, [c_void_p, POINTER(c_uint64)]),
    "aexrt_b200_yolo_enqueue": (c_int, [c_void_p, c_void_p]),
    "aexrt_b200_yolo_launch_count": (c_uint32, [c_void_p]),
    "aexrt_b200_yolo_arena_bytes": (c_uint64, [c_void_p]),
    "aexrt_b200_yolo_override_conv_variant": (c_int, [c_void_p, c_uint32, c_uint32]),
    "aexrt_b200_yolo_set_profiling": (c_int, [c_void_p, c_uint32]),
    "aexrt_b200_yolo_set_arena_reuse": (c_int, [c_void_p, c_uint32]),
    "aexrt_b200_yolo_set_quant_on_load": (c_int, [c_void_p, c_uint32]),
    "aexrt_b200_yolo_status": (c_int, [c_void_p, POINTER(c_uint32)]),
    "aexrt_b200_arena_plan": (c_int, [c_uint32, POINTER(c_uint64), POINTER(c_uint32), POINTER(c_uint32), c_uint64,
                                      POINTER(c_uint64), POINTER(c_uint64)]),
}
for _name in _U32_GETTERS:
    SIGNATURES["aexrt_yolo_" + _name] = (c_uint32, [c_void_p])

_LIB = None


def load_library() -> ctypes.CDLL:
    """``libaexrt_b200.so`` with the runtime ABI declared (the role of the reference's
    ``_load_native_cpp``)."""
    global _LIB
    if _LIB is None:
        lib = _native.load()
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _LIB = lib
    return _LIB


def validate_engine(data: bytes) -> None:
    """Runs the C++ loader's checks on an engine image (no GPU needed); raises ValueError."""
    lib = load_library()
    buf = ctypes.create_string_buffer(bytes(data), len(data))
    if not lib.aexrt_b200_engine_validate(buf, len(data)):
        raise ValueError(_native.last_error())


def arena_plan(sizes, first, last, alignment: int = 256):
    """Lifetime-based arena placement (aexrt_b200_arena_plan): returns (offsets, total bytes)."""
    lib = load_library()
    n = len(sizes)
    b = (c_uint64 * n)(*[int(s) for s in sizes])
    f = (c_uint32 * n)(*[int(s) for s in first])
    l_ = (c_uint32 * n)(*[int(s) for s in last])
    off = (c_uint64 * max(n, 1))()
    total = c_uint64(0)
    _native.check(lib.aexrt_b200_arena_plan(n, b, f, l_, alignment, off, byref(total)), "arena_plan")
    return [int(off[i]) for i in range(n)], int(total.value)


class NativeCppYoloModel:
    """An ``.aexrt`` engine on a CUDA device (the reference's class of the same name).

    ``images`` (this backend's extension) sets how many images one run takes; the default is the
    engine's own graph batch (1 for ``aexrtc build``)."""

    def __init__(self, package_path, adapter_index: int = 0, images: Optional[int] = None) -> None:
        self.package_path = str(package_path)
        self.lib = load_library()
        self.model = None
        self.device = self.lib.aexrt_d3d12_create_device(adapter_index)
        if not self.device:
            raise RuntimeError(f"failed to create the CUDA device {adapter_index}: {_native.last_error()}")
        path = os.fsencode(self.package_path)
        if self.package_path.lower().endswith(".onnx"):
            self.model = self.lib.aexrt_yolo_compile_from_onnx(self.device, path)
        elif not self.package_path.lower().endswith(".aexrt"):
            self.model = self.lib.aexrt_yolo_compile_from_package(self.device, path)
        elif images is None:
            self.model = self.lib.aexrt_yolo_load_engine(self.device, path)
        else:
            self.model = self.lib.aexrt_b200_yolo_load_engine_batch(self.device, path, int(images))
        if not self.model:
            reason = _native.last_error()
            self.close()
            raise RuntimeError(f"failed to load the AEXRT YOLO model {self.package_path}: {reason}")
        self.closed = False

    def __getattr__(self, name):
        # the reference's uint32 counters and flags (class_count, tileflow_*_count, ...)
        if name in _U32_GETTERS and name not in ("conv_plan_count", "profile_event_count"):
            v = int(getattr(self.lib, "aexrt_yolo_" + name)(self.model))
            return bool(v) if name in ("has_objectness", "head_fusion_enabled", "head_final_conv_fusion_enabled") else v
        raise AttributeError(name)

    # ------------------------------------------------------------------ properties
    @property
    def input_element_count(self) -> int:
        return int(self.lib.aexrt_yolo_input_element_count(self.model))

    @property
    def executable(self) -> bool:
        return bool(self.lib.aexrt_yolo_is_executable(self.model))

    @property
    def images(self) -> int:
        return int(self.lib.aexrt_b200_yolo_batch(self.model))

    @property
    def capabilities(self) -> dict:
        raw = AexrtD3D12Capabilities()
        if not self.lib.aexrt_d3d12_get_capabilities(self.device, byref(raw)):
            raise RuntimeError("failed to query the device capabilities")
        return {"highest_shader_model": int(raw.highest_shader_model),
                "native_fp16_supported": bool(raw.native_fp16_supported),
                "wave_mma_tier": int(raw.wave_mma_tier), "dxc_available": bool(raw.dxc_available)}

    @property
    def launch_count(self) -> int:
        return int(self.lib.aexrt_b200_yolo_launch_count(self.model))

    @property
    def arena_bytes(self) -> int:
        return int(self.lib.aexrt_b200_yolo_arena_bytes(self.model))

    # ------------------------------------------------------------------ runs
    def _error(self, what: str) -> RuntimeError:
        raw = self.lib.aexrt_yolo_get_last_error(self.model)
        reason = raw.decode("utf-8", errors="replace") if raw else ""
        return RuntimeError(f"AEXRT YOLO {what} failed" + (f": {reason}" if reason else ""))

    @staticmethod
    def _detections(rows, n: int) -> List[Detection]:
        return [Detection(int(rows[i].class_id), float(rows[i].score),
                          (float(rows[i].x1), float(rows[i].y1), float(rows[i].x2), float(rows[i].y2)))
                for i in range(n)]

    def run(self, image, max_detections: int = 100) -> List[Detection]:
        """One image (fp32 NCHW, input_element_count elements) -> its detections, ranked by score."""
        if not self.executable:
            raise RuntimeError("the AEXRT YOLO model is not executable")
        arr = np.ascontiguousarray(image, dtype=np.float32).reshape(-1)
        if arr.size != self.input_element_count:
            raise ValueError(f"expected {self.input_element_count} input elements, got {arr.size}")
        rows = (AexrtYoloDetection * max(1, int(max_detections)))()
        count = c_uint32(0)
        ok = self.lib.aexrt_yolo_run(self.device, self.model, arr.ctypes.data_as(POINTER(c_float)), arr.size, rows,
                                     int(max_detections), byref(count))
        if not ok:
            raise self._error("run")
        return self._detections(rows, int(count.value))

    def run_batch(self, images, max_detections: int = 100):
        """A whole batch ([images, C, H, W], fp32 or fp16) -> (rows [images, max_detections, 6] fp32,
        counts [images] uint32)."""
        x = np.ascontiguousarray(images)
        dtype = 1 if x.dtype == np.float16 else 0
        if dtype == 0:
            x = np.ascontiguousarray(x, dtype=np.float32)
        n = self.images
        if x.size != self.input_element_count:
            raise ValueError(f"expected {self.input_element_count} input elements, got {x.size}")
        rows = np.zeros((n, max_detections, 6), np.float32)
        counts = np.zeros(n, np.uint32)
        ok = self.lib.aexrt_b200_yolo_run_batch(self.model, x.ctypes.data, dtype,
                                                rows.ctypes.data_as(POINTER(AexrtYoloDetection)), max_detections,
                                                counts.ctypes.data_as(POINTER(c_uint32)))
        if not ok:
            raise self._error("batch run")
        return rows, counts

    def flush_pipeline(self, max_detections: int = 100) -> List[Detection]:
        rows = (AexrtYoloDetection * max(1, int(max_detections)))()
        count = c_uint32(0)
        if not self.lib.aexrt_yolo_flush_pipeline(self.model, rows, int(max_detections), byref(count)):
            raise self._error("pipeline flush")
        return self._detections(rows, int(count.value))

    def debug_value(self, value_id: int, elements: int) -> np.ndarray:
        out = np.empty(int(elements), np.float32)
        if not self.lib.aexrt_yolo_debug_value(self.model, int(value_id), out.ctypes.data_as(POINTER(c_float)),
                                               out.size):
            raise self._error("debug_value")
        return out

    def output0(self) -> np.ndarray:
        """output0 of the last run: [images, channels, anchors] fp32."""
        n = self.images
        out = np.empty(n * self.channel_count * self.anchor_count, np.float32)
        if not self.lib.aexrt_yolo_debug_output(self.model, out.ctypes.data_as(POINTER(c_float)), out.size):
            raise self._error("debug_output")
        return out.reshape(n, self.channel_count, self.anchor_count)

    def profile_events(self) -> List[Tuple[str, float]]:
        out = []
        for i in range(int(self.lib.aexrt_yolo_profile_event_count(self.model))):
            raw = self.lib.aexrt_yolo_profile_event_label(self.model, i)
            out.append((raw.decode("utf-8", errors="replace") if raw else "",
                        float(self.lib.aexrt_yolo_profile_event_ms(self.model, i))))
        return out

    def set_profiling(self, enabled: bool) -> None:
        _native.check(self.lib.aexrt_b200_yolo_set_profiling(self.model, int(bool(enabled))), "set_profiling")

    def set_quant_on_load(self, enabled: bool) -> None:
        _native.check(self.lib.aexrt_b200_yolo_set_quant_on_load(self.model, int(bool(enabled))),
                      "set_quant_on_load")

    def set_arena_reuse(self, enabled: bool) -> None:
        _native.check(self.lib.aexrt_b200_yolo_set_arena_reuse(self.model, int(bool(enabled))), "set_arena_reuse")

    @property
    def last_run_timing(self) -> Optional[dict]:
        t = AexrtYoloRunTiming()
        t.struct_size = ctypes.sizeof(t)
        if not self.lib.aexrt_yolo_get_last_run_timing(self.model, byref(t)) or not t.valid:
            return None
        return {"memcpy_ms": t.memcpy_ms, "submit_ms": t.submit_ms, "fence_ms": t.fence_ms,
                "readback_ms": t.readback_ms}

    def conv_plans(self) -> List[dict]:
        """aexrt_yolo_conv_plan_info of every conv command (the autotuner's view)."""
        out = []
        for i in range(int(self.lib.aexrt_yolo_conv_plan_count(self.model))):
            info = AexrtConvPlanInfo()
            info.struct_size = ctypes.sizeof(info)
            if not self.lib.aexrt_yolo_conv_plan_info(self.model, i, byref(info)):
                raise self._error("conv_plan_info")
            d = info.desc
            out.append({"command_index": info.command_index, "silu": bool(info.kind_is_silu),
                        "desc": tuple(getattr(d, f) for f, _ in AexrtConv2DDesc._fields_),
                        "current_algorithm": info.current_algorithm,
                        "candidates": [info.candidates[k] for k in range(info.candidate_count)],
                        "in_fusion_group": bool(info.in_fusion_group),
                        "planned_algorithm": info.planned_algorithm})
        return out

    def override_conv_algorithm(self, command_index: int, algorithm_id: int) -> None:
        if not self.lib.aexrt_yolo_override_conv_algorithm(self.model, int(command_index), int(algorithm_id)):
            raise self._error("override_conv_algorithm")

    def override_conv_variant(self, command_index: int, block_n_bits: int) -> None:
        if not self.lib.aexrt_b200_yolo_override_conv_variant(self.model, int(command_index), int(block_n_bits)):
            raise self._error("override_conv_variant")

    def status(self) -> int:
        v = c_uint32(0)
        if not self.lib.aexrt_b200_yolo_status(self.model, byref(v)):
            raise self._error("status")
        return int(v.value)

    # ------------------------------------------------------------------ device-resident use
    def set_input_dtype(self, fp16: bool) -> None:
        if not self.lib.aexrt_b200_yolo_set_input_dtype(self.model, 1 if fp16 else 0):
            raise self._error("set_input_dtype")

    def device_input(self) -> int:
        return int(self.lib.aexrt_b200_yolo_device_input(self.model))

    def device_detections(self) -> Tuple[int, int]:
        n = c_uint64(0)
        p = self.lib.aexrt_b200_yolo_device_detections(self.model, byref(n))
        return int(p), int(n.value)

    def enqueue(self, stream: int = 0) -> None:
        """One forward (graph replay) on a CUDA stream handle (0: the model's own stream)."""
        if not self.lib.aexrt_b200_yolo_enqueue(self.model, c_void_p(stream) if stream else None):
            raise self._error("enqueue")

    def close(self) -> None:
        if getattr(self, "model", None):
            self.lib.aexrt_yolo_destroy(self.model)
            self.model = None
        if getattr(self, "device", None):
            self.lib.aexrt_d3d12_destroy_device(self.device)
            self.device = None
        self.closed = True

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
