"""GPU test of the autotuner (aexrt_b200.autotune, the reference's conv_autotune procedure over the
runtime ABI) on the reference-compiled YOLOv8n-320 engine: it tunes a few conv shapes under the
fail-closed gate, the final gate passes, the emitted algo map only names candidate algorithms of
conv commands, and loading the map and the tile sidecar into a fresh model reproduces the tuned
model's output0 bit for bit."""
import json
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
ENGINE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "yolov8n_w8a8.aexrt")


def test_autotune_gate_map_and_replay(tmp_path):
    from aexrt_b200 import autotune, cpp_runtime

    logs = []
    t = autotune.Tuner(ENGINE, images=1, runs=3, warmup=1, log=logs.append)
    assert t.tune(shape_limit=4)
    paths = {k: str(tmp_path / f"{k}.json") for k in ("map", "variants")}
    t.write(str(tmp_path / "report.md"), paths["map"], paths["variants"])
    tuned_out = t.tuned_out.copy()
    plans = {p["command_index"]: p for p in t.model.conv_plans()}
    t.close()
    amap = json.load(open(paths["map"]))
    for cmd, alg in amap.items():
        assert int(cmd) in plans and alg in plans[int(cmd)]["candidates"]
    assert "final numeric gate: PASS" in open(tmp_path / "report.md").read()
    m = cpp_runtime.NativeCppYoloModel(ENGINE, 0, images=1)
    autotune.apply(m, paths["map"], paths["variants"])
    m.run_batch(t.input)
    assert np.array_equal(m.output0(), tuned_out)
    assert m.status() == 0
    m.close()


def test_program_tile_tuning_replays_bit_identically():
    """The tile stage for the streaming engine's programs (autotune.tune_program): every choice it
    returns is a tile the int8 kernels accept, and a model compiled with the tuned tiles gives the
    default model's output0 and detections bit for bit."""
    import torch

    from aexrt_b200 import autotune, engine, yolo

    program = yolo.build_yolov8n(nc=4, imgsz=96, seed=3)
    logs = []
    tiles = autotune.tune_program(program, 2, runs=2, log=logs.append)
    int8 = {c.name for c in program.commands if getattr(c, "precision", None) == "int8"}
    convs = {c.name for c in program.commands if hasattr(c, "precision")}
    assert set(tiles) <= convs
    logged = {line.split(":")[0] for line in logs if not line.startswith(" ")}  # one summary line per conv
    assert int8 <= logged <= convs  # every int8 conv, plus the fp16 head convs that read NHWC
    imgs = torch.from_numpy(np.random.default_rng(5).uniform(0, 1, (2, 3, 96, 96)).astype(np.float16)).cuda()
    outs = []
    for bn in (None, tiles):
        eng = engine.CompiledYolo(program, 2, block_n=bn, nms=engine.NmsConfig())
        eng.forward(imgs)
        torch.cuda.synchronize()
        assert eng.status() == 0
        outs.append((eng.output.cpu().numpy(), eng.det_buf.cpu().numpy()))
    assert np.array_equal(outs[0][0], outs[1][0])
    assert np.array_equal(outs[0][1], outs[1][1])


def test_tile_map_quantize_on_load_bit():
    """A tile map can mark single int8 convs to quantize their fp16 sources themselves
    (engine.TILE_QUANT_ON_LOAD); those convs then run as quantize-on-load steps and the model's
    output0 and detections equal the default model's bit for bit."""
    import torch

    from aexrt_b200 import engine, yolo

    program = yolo.build_yolov8n(nc=4, imgsz=96, seed=4)
    names = [c.name for c in program.commands if getattr(c, "precision", None) == "int8" and engine.ql_eligible(c)]
    assert names
    tiles = {names[0]: engine.TILE_QUANT_ON_LOAD, names[-1]: engine.TILE_QUANT_ON_LOAD | 32}
    imgs = torch.from_numpy(np.random.default_rng(6).uniform(0, 1, (2, 3, 96, 96)).astype(np.float16)).cuda()
    outs = []
    for bn in (None, tiles):
        eng = engine.CompiledYolo(program, 2, block_n=bn, nms=engine.NmsConfig())
        if bn:
            ql = {st[1].name for st in eng.steps if st[0] == "conv_ql"}
            assert ql <= set(tiles) and ql, ql
        eng.forward(imgs)
        torch.cuda.synchronize()
        assert eng.status() == 0
        outs.append((eng.output.cpu().numpy(), eng.det_buf.cpu().numpy()))
    assert np.array_equal(outs[0][0], outs[1][0])
    assert np.array_equal(outs[0][1], outs[1][1])
