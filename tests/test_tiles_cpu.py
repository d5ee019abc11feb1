"""The committed tile maps (aexrt_b200/tuned/) against the programs they were tuned for, and the
quantize-on-load eligibility rule the maps' top bit relies on (CPU only)."""
import json
import os

import pytest

from aexrt_b200 import autotune, engine, yolo

TUNED = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "aexrt_b200", "tuned")
MAPS = sorted(f for f in os.listdir(TUNED) if f.endswith(".json"))


def _program(workload):
    builder, imgsz, nc = autotune.PROGRAMS[workload]
    return getattr(yolo, builder)(nc=nc, imgsz=imgsz, seed=0)


@pytest.mark.parametrize("name", MAPS)
def test_tuned_map_names_convs_and_known_bits(name):
    workload, batch = name[:-5].rsplit("_b", 1)
    assert workload in autotune.PROGRAMS and int(batch) > 0
    convs = {c.name: c for c in _program(workload).commands if isinstance(c, yolo.ConvCmd)}
    tiles = json.load(open(os.path.join(TUNED, name)))
    assert tiles
    for conv, bits in tiles.items():
        assert conv in convs, conv
        c = convs[conv]
        assert bits & 0xFFFF in (0, 16, 32, 64, 128, 256)                    # output-channel tile
        assert (bits >> 16) & 0xF in (0, 2)                                   # auto or halo kernel
        assert (bits >> 20) & 0xF in (0, 1, 2)                                # tile order
        assert (bits >> 24) & 0xF in (0, 1, 2, 4)                             # stacked M blocks cap
        if bits & engine.TILE_QUANT_ON_LOAD:
            assert c.precision == "int8" and engine.ql_eligible(c)
        if c.precision != "int8":
            assert not bits & engine.TILE_QUANT_ON_LOAD


def test_quantize_on_load_eligibility():
    p = _program("yolov8n-320")
    convs = [c for c in p.commands if isinstance(c, yolo.ConvCmd)]
    eligible = [c for c in convs if engine.ql_eligible(c)]
    assert eligible
    for c in eligible:
        assert c.silu and len(c.inputs) <= 4
        assert all(pt.value != "images" and pt.coff % 16 == 0 and pt.channels >= 16 for pt in c.inputs)
    # the stem reads the images and is never eligible; linear convs are not either
    assert not any(engine.ql_eligible(c) for c in convs if any(pt.value == "images" for pt in c.inputs))
    assert not any(engine.ql_eligible(c) for c in convs if not c.silu)
