"""A YOLOv8n-320 ONNX graph, imported without the `onnx` package, runs on the W8A8 kernels (B200):
int8 codes of every W8A8 conv bit-exact against the oracle on the device's own inputs, and class
scores within the reference's 0.02 gate end to end."""
import numpy as np
import pytest

from oracle import yolo_model as om
from tests._util import nhwc_to_nchw, slab16_to_nchw

pytestmark = pytest.mark.gpu


def test_imported_onnx_model_matches_the_oracle(tmp_path):
    import torch

    from aexrt_b200 import engine, onnx_yolo, yolo

    src = yolo.build_yolov8(0.25, 0.33, 4, 320, 0, fused_head=False)
    path = str(tmp_path / "yolov8n.onnx")
    onnx_yolo.export_onnx(src, path)
    prog = onnx_yolo.import_onnx(path)
    imgs = np.random.default_rng(5).uniform(0, 1, (2, 3, 320, 320)).astype(np.float16).astype(np.float32)
    eng = engine.CompiledYolo(prog, 2, nms=engine.NmsConfig())
    eng.capture()
    out = eng.forward(torch.from_numpy(imgs).cuda()).cpu().numpy()
    assert eng.status() == 0
    ref = om.run_program(prog, imgs)["output0"]
    assert np.abs(out[:, 4:] - ref[:, 4:]).max() <= 0.02
    assert np.percentile(np.abs(out[:, :4] - ref[:, :4]), 99) <= 4.0
    vals = {k: nhwc_to_nchw(t.cpu().numpy()) for k, t in eng.values.items()}
    vals["images"] = imgs
    n_int8 = 0
    for st in eng.steps:
        if st[0] == "conv" and st[1].precision == "int8":
            c = st[1]
            x = om._gather(vals, c.inputs)
            r = om.conv_cmd(c, x, None)
            assert np.array_equal(slab16_to_nchw(st[4][0].cpu().numpy(), c.ic, x.shape[2], x.shape[3], c.s), r["xq"])
            n_int8 += 1
    assert n_int8 >= 40
