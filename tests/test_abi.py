"""CPU tests of the C ABI boundary: the library loads, exports every declared
symbol, and its host-side logic (weight quantizer, validation) behaves like the
reference.  No kernel is launched here."""
import ctypes
import subprocess

import numpy as np
import pytest

from aexrt_b200 import _native, ops
from oracle import w8a8 as ow


def test_library_exports_every_header_symbol():
    lib = _native.load()
    names = _native.header_functions()
    assert len(names) >= 15
    for name in names:
        assert hasattr(lib, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", _native.LIB_PATH], capture_output=True, text=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if line.split()[-1].startswith("aexrt_")}
    assert exported == set(names)
    # both headers: the kernel-level ABI and the reference runtime ABI
    assert "aexrt_b200_conv_w8a8" in names and "aexrt_yolo_run" in names and "aexrt_d3d12_create_device" in names
    assert lib.aexrt_b200_abi_version() == 1


def test_conv_desc_layout_matches_reference():
    # native/aexrt.h:98-115: sixteen uint32 fields in this order
    assert ctypes.sizeof(_native.AexrtConv2DDesc) == 64
    assert [f[0] for f in _native.AexrtConv2DDesc._fields_][:4] == ["batch", "in_channels", "in_h", "in_w"]


def test_plan_info_struct_matches_header():
    # 21 uint32 fields (struct_size .. staged_out); the Python view carries every one but struct_size
    assert ctypes.sizeof(_native.AexrtB200ConvPlanInfo) == 21 * 4
    i = _native.AexrtB200ConvPlanInfo()
    for k, (name, _) in enumerate(_native.AexrtB200ConvPlanInfo._fields_):
        setattr(i, name, k + 1)
    info = ops.PlanInfo.from_c(i)
    assert info.kernel_id == 2 and info.in_wp == 15 and info.grid == 16 and info.image_input == 19
    assert info.quant_on_load == 20 and info.staged_out == 21


def test_c_weight_quantizer_matches_reference_payloads(golden_dir):
    d = np.load(f"{golden_dir}/weights_layout8.npz")
    for i in range(int(d["count"])):
        q, s = ops.quantize_conv_weight_int8(d[f"w{i}"], int(d[f"prec{i}"]) == 2)
        assert ow.layout8_payload(q, s) == d[f"payload{i}"].tobytes(), f"case {i}"


def test_c_weight_quantizer_random_matches_oracle():
    rng = np.random.default_rng(5)
    for shape in [(64, 32, 3, 3), (17, 8, 1, 1), (8, 4, 3, 3)]:
        w = (rng.standard_normal(shape) * rng.uniform(1e-3, 10)).astype(np.float32)
        for fp16 in (False, True):
            q, s = ops.quantize_conv_weight_int8(w, fp16)
            q2, s2 = ow.quantize_conv_weight_int8(w, fp16)
            assert np.array_equal(q, q2) and np.array_equal(s, s2)


@pytest.mark.parametrize("args,msg", [
    (dict(ic=64, k=3, s=1, pg16=False, kid=54), "unknown int8 kernel"),
    (dict(ic=20, k=3, s=1, pg16=True, kid=52), "pg16"),
    (dict(ic=6, k=3, s=1, pg16=False, kid=52), "in_channels % 4"),
    (dict(ic=64, k=1, s=1, pg16=False, kid=52), "kernels 52/53"),
    (dict(ic=64, k=3, s=1, pg16=False, kid=53), "kernel 53"),
])
def test_plan_create_rejects_like_the_reference_guard(args, msg):
    """can_use_conv_int8 (runtime.cpp:9398-9422): invalid plans fail closed, with a message, before any launch."""
    lib = _native.load()
    k, s = args["k"], args["s"]
    desc = ops.conv_desc(1, args["ic"], 16, 16, 32, k, s, k // 2)
    codes = np.zeros((32, args["ic"] * k * k), np.int8)
    scale = np.ones(32, np.float32)
    bias = np.zeros(32, np.float32)
    h = lib.aexrt_b200_conv_plan_create(ctypes.byref(desc), 2, args["kid"], 16 if args["pg16"] else 0,
                                        codes.ctypes.data, scale.ctypes.data, bias.ctypes.data, 0)
    assert not h
    assert msg in _native.last_error()


def test_entry_points_fail_closed_on_null():
    lib = _native.load()
    assert lib.aexrt_b200_act_amax_f16(None, 1, 16, 4, 4, 1, 16, 0, None, 1, 0, 1, None) == 0
    assert "null" in _native.last_error()
    assert lib.aexrt_b200_conv_w8a8(None, None, None, None, 0, 0, None, 0, 0, None, 0, 0, None, None) == 0
    assert lib.aexrt_b200_packed_act_bytes(2, 20, 7, 9, 2) == 2 * 2 * 8 * 10 * 16


def test_unaligned_nhwc_slices_are_refused_before_any_launch():
    """16-byte loads need 16-byte aligned slices: the entry points refuse others up front (no kernel runs)."""
    from aexrt_b200._native import AexrtB200ActSource

    lib = _native.load()
    dummy = ctypes.c_void_p(4096)
    srcs = (AexrtB200ActSource * 1)()
    s = srcs[0]
    s.ptr, s.layout, s.ldc, s.coff, s.channels, s.upsample, s.src_h, s.src_w = 4096, 0, 40, 4, 32, 1, 4, 4
    s.amax_groups, s.amax_stride, s.amax_goff = 4096, 4, 0
    assert lib.aexrt_b200_act_quantize_concat(srcs, 1, 1, 4, 4, 0, 1, dummy, dummy, None) == 0
    assert "aligned" in _native.last_error()
    assert lib.aexrt_b200_pack_f16_concat(srcs, 1, 1, 4, 4, 1, dummy, None) == 0
    assert "aligned" in _native.last_error()
    # a misaligned base pointer
    assert lib.aexrt_b200_act_quantize_f16(ctypes.c_void_p(4104), 1, 32, 4, 4, 0, 32, 0, dummy, 2, 0, 0, 1, dummy,
                                           dummy, None) == 0
    assert "aligned" in _native.last_error()
    assert lib.aexrt_b200_pack_f16(ctypes.c_void_p(4104), 1, 32, 4, 4, 0, 32, 0, 1, dummy, None) == 0
    assert "aligned" in _native.last_error()


@pytest.mark.parametrize("kw,msg", [
    (dict(channels=9), "do not match nc"),
    (dict(max_candidates=0), "max_candidates"),
    (dict(max_candidates=1025), "max_candidates"),
    (dict(max_detections=0), "max_detections"),
    (dict(mode=2), "bad mode"),
    (dict(layout=3), "bad layout"),
])
def test_nms_arguments_fail_closed(kw, msg):
    """Invalid post-process arguments are refused before any launch (no GPU needed)."""
    lib = _native.load()
    a = dict(channels=8, anchors=100, nc=4, has_obj=0, layout=1, max_candidates=512, max_detections=100, mode=0)
    a.update(kw)
    fake = ctypes.c_void_p(256)  # never dereferenced: validation fails first
    ok = lib.aexrt_b200_yolo_nms_topk(fake, 1, a["channels"], a["anchors"], a["nc"], a["has_obj"], a["layout"], 0.25,
                                      0.45, a["max_candidates"], a["max_detections"], a["mode"], fake, fake, None)
    assert ok == 0
    assert msg in _native.last_error()


def test_detection_struct_matches_reference():
    # native/aexrt.h:25-32: six floats
    assert ctypes.sizeof(_native.AexrtYoloDetection) == 24
    assert [f[0] for f in _native.AexrtYoloDetection._fields_] == ["x1", "y1", "x2", "y2", "score", "class_id"]


def test_conv_f16_nhwc_refuses_null_plan():
    lib = _native.load()
    assert lib.aexrt_b200_conv_f16_nhwc(None, ctypes.c_void_p(256), 64, 0, None, 0, 0, ctypes.c_void_p(256), 64, 0,
                                        None, 0, 0, None) == 0
    assert "null plan" in _native.last_error()
