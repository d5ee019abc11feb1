"""CPU tests of the reader for reference-compiled engines (aexrt_b200.aexrt_engine).

The committed engine tests/golden/tiny_w8a8.aexrt was written by the reference's own compiler
(build_aexrt_engine with algo overrides 51/52/53 and one INT8_PERGROUP command, fp16 precision);
its kernel-plan records and the graph's fp32 constants are in tests/golden/tiny_w8a8.npz."""
import struct
import zlib

import numpy as np
import pytest

from aexrt_b200 import aexrt_engine as ae
from oracle import w8a8 as ow


@pytest.fixture(scope="module")
def raw(golden_dir):
    return open(f"{golden_dir}/tiny_w8a8.aexrt", "rb").read()


def test_reads_the_reference_engine(raw, golden_dir):
    e = ae.load_engine(raw)
    gold = np.load(f"{golden_dir}/tiny_w8a8.npz")["kernel_plan"]
    assert [(i, c.kind, c.planned_kernel, c.precision, c.packed_value, c.flags) for i, c in enumerate(e.commands)] \
        == [tuple(int(v) for v in r) for r in gold]
    m = e.manifest
    assert (m["precision"], m["input_value"], m["output_value"]) == (2, 0, 10)
    assert (m["channels"], m["anchors"], m["classes"], m["max_candidates"], m["max_detections"]) == (8, 64, 4, 512, 100)
    assert m["conf_threshold"] == np.float32(0.25) and m["iou_threshold"] == np.float32(0.45)
    assert e.shape(0) == (1, 16, 16, 16) and e.shape(10) == (1, 1, 8, 64)
    assert sorted(e.sections) == list(range(1, 12))
    # conv descriptors: the AexrtConv2DDesc field order
    assert ae.conv_desc(e.commands[1]) == (1, 32, 16, 16, 32, 8, 8, 3, 3, 2, 2, 1, 1, 1, 1, 1)


def test_layout8_weights_are_the_reference_quantizer_output(raw, golden_dir):
    """The packed codes and scales equal the quantizer restatement on the fp16-rounded weights."""
    e = ae.load_engine(raw)
    gold = np.load(f"{golden_dir}/tiny_w8a8.npz")
    for cmd, name in zip(e.commands[:3], ("l0", "l1", "l2")):
        codes, scale = ae.int8_weights(e, cmd)
        q, s = ow.quantize_conv_weight_int8(gold[name + ".w"], fp16_engine=True)
        assert np.array_equal(codes, q) and np.array_equal(scale, s), name
        # fp16 engine: bias constants stored as fp16
        assert e.constant_dtype[cmd.inputs[2]] == 2
        assert np.array_equal(e.constants[cmd.inputs[2]], gold[name + ".b"].astype(np.float16).astype(np.float32))


def _patch(raw, off, new):
    b = bytearray(raw)
    b[off:off + len(new)] = new
    return bytes(b)


def _fix_crc(raw, sid):
    """Recomputes the CRC32 of section `sid` after a deliberate edit."""
    b = bytearray(raw)
    count = struct.unpack_from("<I", b, 16)[0]
    for i in range(count):
        t, f, off, size, crc, r = struct.unpack_from("<IIQQII", b, 64 + 32 * i)
        if t == sid:
            struct.pack_into("<IIQQII", b, 64 + 32 * i, t, f, off, size, zlib.crc32(b[off:off + size]), r)
    return bytes(b)


def _section(raw, sid):
    count = struct.unpack_from("<I", raw, 16)[0]
    for i in range(count):
        t, f, off, size, crc, r = struct.unpack_from("<IIQQII", raw, 64 + 32 * i)
        if t == sid:
            return off, size
    raise KeyError(sid)


def test_fails_closed_on_malformed_engines(raw):
    with pytest.raises(ae.EngineError, match="magic"):
        ae.load_engine(_patch(raw, 0, b"NOTANENG"))
    with pytest.raises(ae.EngineError, match="file size"):
        ae.load_engine(raw[:-8])
    off, size = _section(raw, 6)
    with pytest.raises(ae.EngineError, match="CRC32"):
        ae.load_engine(_patch(raw, off + size - 1, bytes([raw[off + size - 1] ^ 0xFF])))
    # a kernel-plan record that disagrees with its command (planned kernel 52 -> 53), CRC fixed up
    off, _ = _section(raw, 5)
    bad = _fix_crc(_patch(raw, off + 8 + 8, struct.pack("<I", 53)), 5)
    with pytest.raises(ae.EngineError, match="disagrees"):
        ae.load_engine(bad)
    # reserved header bytes and TOC fields must be zero; section ids are 1..12; section 11 needs 10
    with pytest.raises(ae.EngineError, match="reserved header"):
        ae.load_engine(_patch(raw, 50, b"\x01"))
    with pytest.raises(ae.EngineError, match="reserved table"):
        ae.load_engine(_patch(raw, 64 + 28, struct.pack("<I", 7)))
    with pytest.raises(ae.EngineError, match="unknown section id"):
        ae.load_engine(_patch(raw, 64, struct.pack("<I", 40)))
    count = struct.unpack_from("<I", raw, 16)[0]
    for i in range(count):
        if struct.unpack_from("<I", raw, 64 + 32 * i)[0] == 10:
            with pytest.raises(ae.EngineError, match="requires section 10"):
                ae.load_engine(_patch(raw, 64 + 32 * i, struct.pack("<I", 12)))
    # manifest fields out of the reference loader's ranges (output value id past the value table)
    off, _ = _section(raw, 1)
    bad = _fix_crc(_patch(raw, off + 64, struct.pack("<I", 10 ** 6)), 1)
    with pytest.raises(ae.EngineError, match="manifest fields"):
        ae.load_engine(bad)
    # the same change applied to command and plan alike loads, but the runner-side check refuses
    # a layout-8 payload of the wrong size
    e = ae.load_engine(raw)
    e.packed[e.commands[0].inputs[1]]["data"] = e.packed[e.commands[0].inputs[1]]["data"][:-4]
    with pytest.raises(ae.EngineError, match="layout-8 payload"):
        ae.int8_weights(e, e.commands[0])
