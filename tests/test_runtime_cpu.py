"""CPU tests of the reference runtime ABI served by libaexrt_b200.so (include/aexrt_yolo.h).

* the C++ engine loader accepts the engines the reference compiler wrote and fails closed on
  malformed ones, as the Python reader does;
* the arena planner never lets two buffers whose lifetimes overlap share bytes;
* the reference's own ctypes binding (NativeCppYoloModel._configure, imported from the reference
  source tree when it is present) binds every symbol it needs from this library, with the
  declarations this backend's binding uses;
* without a GPU, device creation fails with a message instead of crashing.
"""
import ctypes
import os
import struct
import sys
import zlib

import numpy as np
import pytest

from aexrt_b200 import _native, cpp_runtime

REFERENCE_SRC = "/root/reference/src"


@pytest.fixture(scope="module")
def v8n_engine(golden_dir):
    return open(f"{golden_dir}/yolov8n_w8a8.aexrt", "rb").read()


def _sections(raw):
    count = struct.unpack_from("<I", raw, 16)[0]
    out = {}
    for i in range(count):
        t, f, off, size, crc, r = struct.unpack_from("<IIQQII", raw, 64 + 32 * i)
        out[t] = (i, off, size)
    return out


def _edit(raw, sid, rel, new):
    """Replaces bytes inside section `sid` and fixes its CRC (a deliberate, well-formed corruption)."""
    i, off, size = _sections(raw)[sid]
    b = bytearray(raw)
    b[off + rel:off + rel + len(new)] = new
    t, f, o, s, crc, r = struct.unpack_from("<IIQQII", b, 64 + 32 * i)
    struct.pack_into("<IIQQII", b, 64 + 32 * i, t, f, o, s, zlib.crc32(b[off:off + size]) & 0xFFFFFFFF, r)
    return bytes(b)


def test_cxx_loader_accepts_the_reference_engines(golden_dir, v8n_engine):
    cpp_runtime.validate_engine(v8n_engine)
    cpp_runtime.validate_engine(open(f"{golden_dir}/tiny_w8a8.aexrt", "rb").read())


def test_cxx_loader_fails_closed(v8n_engine):
    raw = v8n_engine
    cases = [
        (b"NOTANENG" + raw[8:], "magic"),
        (raw[:-8], "file size"),
        (raw[:50] + b"\x01" + raw[51:], "reserved header"),
    ]
    secs = _sections(raw)
    # a payload byte flipped without fixing the CRC
    _, off, size = secs[6]
    cases.append((raw[:off + 7] + bytes([raw[off + 7] ^ 0xFF]) + raw[off + 8:], "CRC32"))
    # kernel plan record 1 planned kernel changed (CRC fixed): disagrees with its command
    cases.append((_edit(raw, 5, 8 + 24 + 8, struct.pack("<I", 999)), "disagrees"))
    # manifest output value past the value table
    cases.append((_edit(raw, 1, 64, struct.pack("<I", 10 ** 6)), "manifest fields"))
    # memory plan V2: the first value record's offset moved off the alignment
    npages = struct.unpack_from("<I", raw, secs[7][1] + 8)[0]
    cases.append((_edit(raw, 7, 32 + 24 * npages + 24, struct.pack("<Q", 8)), "memory record"))
    # physical dispatch plan: the first table entry repeated (a logical command owned twice)
    i10, off10, size10 = secs[10]
    nrec = struct.unpack_from("<I", raw, off10 + 4)[0]
    table = 32 + nrec * 48
    second = struct.unpack_from("<I", raw, off10 + table)[0]
    cases.append((_edit(raw, 10, table + 4, struct.pack("<I", second)), "physical dispatch"))
    # arena barrier plan: a record size other than 40
    cases.append((_edit(raw, 11, 20, struct.pack("<I", 44)), "arena barrier"))
    for bad, msg in cases:
        with pytest.raises(ValueError, match=msg):
            cpp_runtime.validate_engine(bad)


def test_python_and_cxx_readers_agree(v8n_engine):
    from aexrt_b200 import aexrt_engine as ae

    e = ae.load_engine(v8n_engine)
    assert e.manifest["command_count"] == 127 and e.manifest["anchors"] == 2100
    cpp_runtime.validate_engine(v8n_engine)


def test_arena_plan_separates_overlapping_lifetimes():
    rng = np.random.default_rng(0)
    for trial in range(20):
        n = int(rng.integers(1, 60))
        sizes = rng.integers(0, 5000, n)
        first = rng.integers(0, 40, n)
        last = first + rng.integers(0, 10, n)
        offs, total = cpp_runtime.arena_plan(sizes, first, last, 256)
        assert all(o % 256 == 0 for o in offs)
        for i in range(n):
            assert offs[i] + sizes[i] <= total
            for j in range(i + 1, n):
                if sizes[i] and sizes[j] and not (last[i] < first[j] or last[j] < first[i]):
                    assert offs[i] + sizes[i] <= offs[j] or offs[j] + sizes[j] <= offs[i], (trial, i, j)
    # disjoint lifetimes share the bytes: two 1 MB buffers, one after the other, need 1 MB
    offs, total = cpp_runtime.arena_plan([1 << 20, 1 << 20], [0, 2], [1, 3])
    assert total == 1 << 20 and offs == [0, 0]
    with pytest.raises(_native.AexrtError, match="first launch after last"):
        cpp_runtime.arena_plan([16], [3], [2])


def test_no_gpu_device_creation_fails_with_a_message():
    torch = pytest.importorskip("torch")
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    lib = cpp_runtime.load_library()
    assert lib.aexrt_d3d12_probe() == 0
    assert not lib.aexrt_d3d12_create_device(0)
    assert "not present" in _native.last_error()
    assert not lib.aexrt_yolo_load_engine(None, b"x.aexrt")
    with pytest.raises(RuntimeError, match="device"):
        cpp_runtime.NativeCppYoloModel("tests/golden/yolov8n_w8a8.aexrt")


class _Recorder:
    """Stands in for a CDLL: records the restype / argtypes a binding declares per function."""

    def __init__(self):
        object.__setattr__(self, "fns", {})

    def __getattr__(self, name):
        fns = object.__getattribute__(self, "fns")
        if name not in fns:
            fns[name] = type("Fn", (), {"argtypes": None, "restype": None})()
        return fns[name]


def _type_name(t):
    if t is None:
        return None
    if hasattr(t, "_type_") and isinstance(t._type_, type) and issubclass(t._type_, ctypes.Structure):
        return ("ptr", [f[0] for f in t._type_._fields_])
    if hasattr(t, "_type_") and hasattr(t, "contents"):
        return ("ptr", _type_name(t._type_))
    return getattr(t, "__name__", str(t))


@pytest.mark.skipif(not os.path.isdir(REFERENCE_SRC), reason="the reference source tree is not present")
def test_reference_binding_loads_this_library():
    """The reference's NativeCppYoloModel._configure (src/aexrt/cpp_runtime.py:543-662) against this
    library: every symbol it binds exists, and its declarations equal this backend's binding."""
    sys.path.insert(0, REFERENCE_SRC)
    try:
        from aexrt import cpp_runtime as ref
    finally:
        sys.path.remove(REFERENCE_SRC)
    obj = ref.NativeCppYoloModel.__new__(ref.NativeCppYoloModel)
    obj.lib = ctypes.CDLL(_native.LIB_PATH)
    obj._configure()  # raises AttributeError on a missing symbol
    rec = ref.NativeCppYoloModel.__new__(ref.NativeCppYoloModel)
    rec.lib = _Recorder()
    rec._configure()
    declared = rec.lib.fns
    assert len(declared) >= 50
    for name, fn in declared.items():
        assert name in cpp_runtime.SIGNATURES, name
        res, args = cpp_runtime.SIGNATURES[name]
        if fn.restype is not None or res is not None:
            assert _type_name(fn.restype) == _type_name(res), name
        if fn.argtypes is not None:
            assert [_type_name(a) for a in fn.argtypes] == [_type_name(a) for a in args], name
    # the structs the binding passes by pointer are layout-identical
    assert ctypes.sizeof(ref._YoloRunTiming) == ctypes.sizeof(cpp_runtime.AexrtYoloRunTiming)
    assert ctypes.sizeof(ref._D3D12Capabilities) == ctypes.sizeof(cpp_runtime.AexrtD3D12Capabilities)
    assert ctypes.sizeof(ref._YoloDetection) == ctypes.sizeof(_native.AexrtYoloDetection)


@pytest.mark.skipif(not os.path.isdir(REFERENCE_SRC), reason="the reference source tree is not present")
def test_session_backend_compiles_with_the_reference_compiler():
    """B200Backend.compile: a reference Graph through the reference's build_aexrt_engine (with a W8A8
    algo map), validated by this library's loader."""
    sys.path.insert(0, REFERENCE_SRC)
    try:
        import aexrt

        from aexrt_b200.session_backend import B200Backend

        rng = np.random.default_rng(3)
        g = aexrt.Graph("b200_backend")
        g.input("images", aexrt.TensorSpec((1, 16, 16, 16), "float32"))
        g.const("w", rng.normal(0, 0.05, (32, 16, 3, 3)).astype(np.float32))
        g.const("b", rng.normal(0, 0.1, (32,)).astype(np.float32))
        g.conv2d("c", "images", "w", "b", strides=(1, 1), pads=(1, 1, 1, 1))
        g.sigmoid("s", "c")
        g.mul("y", "c", "s")
        g.reshape("out", "y", [1, 32, 256])
        g.output("out")
        data = B200Backend.compile(g, algo_overrides={0: 52}, precision="fp16")
        cpp_runtime.validate_engine(data)
        assert B200Backend().info().name == "b200"
    finally:
        sys.path.remove(REFERENCE_SRC)
