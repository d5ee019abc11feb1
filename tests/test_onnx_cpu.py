"""ONNX ingest without the `onnx` package (CPU).

* the protobuf subset reads hand-encoded bytes of the published onnx.proto field numbers;
* a program exported as an ONNX graph (the export form, DFL decode included) evaluates, through a
  plain numpy evaluator of the ONNX operators, to the oracle's output0;
* importing that graph gives back the same command stream (W8A8 / fp16 split included), whose
  oracle output0 equals the original's bit for bit;
* operators off the YOLO path fail with the node's name.
"""
import struct

import numpy as np
import pytest

from aexrt_b200 import onnx_proto as op
from aexrt_b200 import onnx_yolo, yolo
from oracle import yolo_model as om
from tests import _onnx_eval


def _images(n, size, seed=0):
    return np.random.default_rng(seed).uniform(0, 1, (n, 3, size, size)).astype(np.float16).astype(np.float32)


def test_protobuf_subset_reads_the_published_wire_format():
    # TensorProto: dims = [2] (field 1), data_type = FLOAT (field 2), float_data packed (field 4),
    # name = "w" (field 8)
    raw = bytes([0x08, 0x02, 0x10, 0x01, 0x22, 0x08]) + struct.pack("<2f", 1.5, -2.0) + bytes([0x42, 0x01]) + b"w"
    t = op.TensorProto()
    t.ParseFromString(raw)
    assert t.name == "w" and np.array_equal(op.to_array(t), np.array([1.5, -2.0], np.float32))
    # NodeProto: input (1), output (2), op_type (4), attribute (5) {name (1), ints (8) unpacked, type (20) = INTS}
    attr = bytes([0x0A, 0x07]) + b"strides" + bytes([0x40, 0x02, 0x40, 0x02, 0xA0, 0x01, 0x07])
    raw = (bytes([0x0A, 0x01]) + b"x" + bytes([0x12, 0x01]) + b"y" + bytes([0x22, 0x04]) + b"Conv"
           + bytes([0x2A, len(attr)]) + attr)
    n = op.NodeProto()
    n.ParseFromString(raw)
    assert (list(n.input), list(n.output), n.op_type, op.attrs(n)) == (["x"], ["y"], "Conv", {"strides": [2, 2]})
    for a in (np.arange(6, dtype=np.int64).reshape(2, 3), np.array([0.5, -1.25], np.float16), np.float32(3.0)):
        assert np.array_equal(op.to_array(op.from_array(a, "t")), a)


def _program(fp16=False, size=64):
    p = yolo.build_yolov8(0.25, 0.33, 4, size, 0, fused_head=False)
    if fp16:
        yolo.apply_algo_map(p, int8=set())
    return p


def test_exported_graph_evaluates_to_the_oracle_output():
    p = _program(fp16=True)
    m = onnx_yolo.export_onnx(p, batch=2)
    imgs = _images(2, 64, seed=1)
    got = _onnx_eval.run(m, {"images": imgs})["output0"]
    ref = om.run_program(p, imgs)["output0"]
    assert got.shape == ref.shape == (2, 8, p.anchors)
    # the oracle stores every activation in fp16, the evaluator keeps fp32
    assert np.abs(got[:, 4:] - ref[:, 4:]).max() < 2e-3
    assert np.abs(got[:, :4] - ref[:, :4]).max() < 0.25


@pytest.mark.parametrize("builder", ["v8n", "v8s", "v11-head"])
def test_import_gives_back_the_program(tmp_path, builder):
    if builder == "v8n":
        p = _program()
    elif builder == "v8s":
        p = yolo.build_yolov8(0.5, 0.33, 80, 64, 1, fused_head=False)
    else:  # the YOLOv11 Detect head (depthwise convs in the class branch) on the YOLOv8n backbone
        p = yolo.build_yolov8(0.25, 0.33, 80, 64, 2, v11_head=True)
    path = str(tmp_path / "model.onnx")
    onnx_yolo.export_onnx(p, path)
    q = onnx_yolo.import_onnx(path)
    assert (q.imgsz, q.nc, q.reg_max, q.anchors) == (p.imgsz, p.nc, p.reg_max, p.anchors)
    kinds = [(type(c).__name__, getattr(c, "precision", None), getattr(c, "k", None), getattr(c, "s", None),
              getattr(c, "silu", None), getattr(c, "residual", None) is not None) for c in p.commands]
    assert kinds == [(type(c).__name__, getattr(c, "precision", None), getattr(c, "k", None), getattr(c, "s", None),
                      getattr(c, "silu", None), getattr(c, "residual", None) is not None) for c in q.commands]
    imgs = _images(2, 64, seed=2)
    assert np.array_equal(om.run_program(p, imgs)["output0"], om.run_program(q, imgs)["output0"])


def test_import_refuses_operators_off_the_path():
    p = _program()
    m = onnx_yolo.export_onnx(p)
    bad = op.make_node("MatMul", [m.graph.node[0].output[0], m.graph.node[0].output[0]], ["mm"], name="attn_mm")
    m.graph.node.insert(1, bad)
    with pytest.raises(onnx_yolo.OnnxImportError, match="attn_mm"):
        onnx_yolo.import_onnx(m)


def test_import_refuses_a_graph_without_the_head():
    p = _program()
    m = onnx_yolo.export_onnx(p)
    del m.graph.node[40:]
    with pytest.raises(onnx_yolo.OnnxImportError):
        onnx_yolo.import_onnx(m)
