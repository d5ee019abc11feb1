"""GPU tests of the reference runtime ABI (include/aexrt_yolo.h) on an engine the reference
compiler wrote: tests/golden/yolov8n_w8a8.aexrt, BASELINE config 3's YOLOv8n-320 (nc=4) compiled by
build_aexrt_engine with an algo map of 51/52/53 (tests/golden/make_golden.py).

* the engine runner (C++: parse, lower, arena, CUDA graph) gives the same detections and output0,
  bit for bit, as the yolo.py program of the same model run by CompiledYolo, whose layers are
  checked against the oracle in test_gpu_model.py; and output0 is within the reference's score gate
  of the oracle run of that model;
* an intermediate value read back through aexrt_yolo_debug_value, fed to the oracle conv, gives the
  next value within max-abs 1e-2 (teacher forcing through the ABI);
* batch extension: every image of a batch-4 model equals the same image run alone;
* the autotuner surface: conv plan info, algorithm override (int8 -> fp16 -> back) and profiling;
* fail-closed calls: wrong input size, unknown override.
"""
import json
import os
import sys

import numpy as np
import pytest

from oracle import w8a8 as ow
from oracle import yolo_model as om

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))
ENGINE = os.path.join(HERE, "golden", "yolov8n_w8a8.aexrt")


def _torch():
    import torch

    return torch


@pytest.fixture(scope="module")
def table():
    return json.load(open(os.path.join(HERE, "golden", "yolov8n_w8a8.json")))


@pytest.fixture(scope="module")
def program(table):
    """The yolo.py program the engine was compiled from, with the engine's int8 / fp16 split."""
    sys.path.insert(0, os.path.join(HERE, "golden"))
    try:
        import make_golden
    finally:
        sys.path.pop(0)
    from aexrt_b200 import yolo

    prog = make_golden.engine_program()
    plan = {int(r[0]): r for r in table["kernel_plan"]}
    int8 = {name for cmd, name in table["conv_commands"].items() if plan[int(cmd)][2] in (51, 52, 53)}
    assert len(int8) >= 20
    yolo.apply_algo_map(prog, int8=int8)
    return prog


def _images(n, seed):
    rng = np.random.default_rng(seed)
    return rng.uniform(0, 1, (n, 3, 320, 320)).astype(np.float16).astype(np.float32)


def _model(images=None):
    from aexrt_b200 import cpp_runtime

    return cpp_runtime.NativeCppYoloModel(ENGINE, 0, images=images)


def test_engine_runner_equals_the_program_and_the_oracle(program):
    from aexrt_b200 import engine

    torch = _torch()
    m = _model()
    assert m.executable and m.images == 1 and m.head_fusion_enabled
    assert (m.class_count, m.anchor_count, m.channel_count) == (4, 2100, 8)
    assert m.input_element_count == 3 * 320 * 320
    assert m.c2f_tail_residual_fusion_count == 6  # the six bottleneck Adds became conv residuals
    eng = engine.CompiledYolo(program, 1, nms=engine.NmsConfig())
    for seed in (1, 2):
        img = _images(1, seed)
        dets = m.run(img[0])
        out0 = m.output0()
        eng.forward(torch.from_numpy(img).cuda())
        counts, rows = (t.cpu().numpy() for t in eng.detections())
        want = eng.output.cpu().numpy()
        assert np.array_equal(out0, want), float(np.abs(out0 - want).max())
        assert len(dets) == counts[0]
        got = np.array([list(d.xyxy) + [d.score, d.class_id] for d in dets], np.float32).reshape(-1, 6)
        assert np.array_equal(got, rows[0, :counts[0]])
        ref = om.run_program(program, img)["output0"]
        assert np.abs(out0[:, 4:] - ref[:, 4:]).max() <= 0.02
        assert np.percentile(np.abs(out0[:, :4] - ref[:, :4]), 99) <= 4.0
    t = m.last_run_timing
    assert t is not None and t["fence_ms"] >= 0
    assert m.status() == 0
    m.close()


def test_engine_values_teacher_forced(program, table):
    """Values read back through aexrt_yolo_debug_value: every int8 conv's output against the oracle
    conv of its own read-back input (slots kept apart so every value stays readable)."""
    from aexrt_b200 import aexrt_engine as ae

    e = ae.load_engine(ENGINE)
    m = _model()
    m.set_arena_reuse(False)
    img = _images(1, 5)
    m.run(img[0])
    by_name = {c.name: c for c in program.commands if hasattr(c, "weight")}
    checked = 0
    for cmd_s, name in table["conv_commands"].items():
        cmd = e.commands[int(cmd_s)]
        if cmd.planned_kernel not in (51, 52, 53) or name not in by_name:
            continue
        c = by_name[name]
        xin = m.debug_value(cmd.inputs[0], int(np.prod(e.shape(cmd.inputs[0])))).reshape(e.shape(cmd.inputs[0]))
        yout = m.debug_value(cmd.output, int(np.prod(e.shape(cmd.output)))).reshape(e.shape(cmd.output))
        r = ow.conv_w8a8(xin.astype(np.float16), c.weight, c.bias, c.k, c.s, c.k // 2, silu=c.silu,
                         mode=ow.SCALE_PG16 if c.pg16 else ow.SCALE_PER_TENSOR)
        if c.residual is None:
            assert np.abs(yout - r["y32"]).max() <= 1e-2, name
            checked += 1
    assert checked >= 15
    m.close()


def test_batch_model_equals_single_images():
    m4 = _model(images=4)
    m1 = _model()
    imgs = _images(4, 9)
    rows, counts = m4.run_batch(imgs)
    for i in range(4):
        dets = m1.run(imgs[i])
        assert counts[i] == len(dets)
        got = np.array([list(d.xyxy) + [d.score, d.class_id] for d in dets], np.float32).reshape(-1, 6)
        assert np.array_equal(rows[i, :counts[i]], got), i
    # fp16 input of the same images: the stem rounds fp32 input to fp16, so the results are equal
    rows16, counts16 = m4.run_batch(imgs.astype(np.float16))
    assert np.array_equal(counts16, counts) and np.array_equal(rows16, rows)
    m4.close()
    m1.close()


def test_conv_plans_override_and_profile():
    m = _model()
    plans = m.conv_plans()
    assert len(plans) == 62  # the CONV / CONV_SILU commands before the head (the DFL conv is in it)
    int8 = [p for p in plans if p["planned_algorithm"] in (51, 52, 53)]
    assert int8 and all(p["current_algorithm"] == p["planned_algorithm"] for p in int8)
    img = _images(1, 3)[0]
    m.run(img)
    base = m.output0().copy()
    # an int8 conv without a fused residual, switched to the fp16 conv and back
    p = next(p for p in int8 if not p["in_fusion_group"])
    fp16 = [a for a in p["candidates"] if a not in (51, 52, 53)][0]
    m.override_conv_algorithm(p["command_index"], fp16)
    m.run(img)
    changed = m.output0()
    assert [q for q in m.conv_plans() if q["command_index"] == p["command_index"]][0]["current_algorithm"] == fp16
    assert np.abs(changed[:, 4:] - base[:, 4:]).max() <= 0.02
    m.override_conv_algorithm(p["command_index"], p["planned_algorithm"])
    m.run(img)
    assert np.array_equal(m.output0(), base)
    with pytest.raises(RuntimeError, match="not a candidate"):
        m.override_conv_algorithm(p["command_index"], 7)
    # the int8 convs quantizing their fp16 inputs on load instead of a separate quantize launch:
    # identical results
    m.set_quant_on_load(True)
    m.run(img)
    assert np.array_equal(m.output0(), base)
    m.set_quant_on_load(False)
    # variants of the tile choice give identical results
    m.override_conv_variant(p["command_index"], 2 << 20)
    m.run(img)
    assert np.array_equal(m.output0(), base)
    m.set_profiling(True)
    m.run(img)
    ev = m.profile_events()
    assert len(ev) >= 60 and all(lab.startswith(("cmd#", "post:")) and ms >= 0 for lab, ms in ev)
    assert np.array_equal(m.output0(), base)
    with pytest.raises(ValueError, match="input elements"):
        m.run(np.zeros(10, np.float32))
    m.close()


def test_engine_zero_copy_input_and_fail_closed():
    import ctypes

    from aexrt_b200 import cpp_runtime
    from aexrt_b200._native import AexrtYoloDetection

    m = _model()
    lib = cpp_runtime.load_library()
    n = ctypes.c_uint64(0)
    ptr = lib.aexrt_yolo_input_ptr(m.model, ctypes.byref(n))
    assert ptr and n.value == m.input_element_count
    img = _images(1, 4)[0].reshape(-1)
    host = np.ctypeslib.as_array(ctypes.cast(ptr, ctypes.POINTER(ctypes.c_float)), shape=(n.value,))
    host[:] = img
    rows = (AexrtYoloDetection * 100)()
    count = ctypes.c_uint32(0)
    assert lib.aexrt_yolo_run(m.device, m.model, ctypes.cast(ptr, ctypes.POINTER(ctypes.c_float)), n.value, rows, 100,
                              ctypes.byref(count)) == 1
    assert m.last_run_timing["memcpy_ms"] == 0.0
    want = m.run(img)
    assert count.value == len(want)
    # wrong element count: status 0 and a message, no launch
    assert lib.aexrt_yolo_run(m.device, m.model, ctypes.cast(ptr, ctypes.POINTER(ctypes.c_float)), 5, rows, 100,
                              ctypes.byref(count)) == 0
    assert b"input elements" in lib.aexrt_yolo_get_last_error(m.model)
    assert lib.aexrt_yolo_flush_pipeline(m.model, rows, 100, ctypes.byref(count)) == 1 and count.value == 0
    m.close()


def test_session_backend_runs_the_engine():
    """The reference InferenceSession's backend protocol (info / prepare / run) on the engine."""
    from aexrt_b200.session_backend import B200Backend

    be = B200Backend(0, images=2)
    be.prepare(ENGINE)
    imgs = _images(2, 11)
    out = be.run({"images": imgs})["output0"]
    m = _model(images=2)
    rows, counts = m.run_batch(imgs)
    assert np.array_equal(out, m.output0())
    assert np.array_equal(be.last_detections[1], counts) and np.array_equal(be.last_detections[0], rows)
    assert be.info().device == "cuda:0"
    be.close()
    m.close()
