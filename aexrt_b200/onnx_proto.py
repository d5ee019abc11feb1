"""The ONNX model format read and written without the `onnx` package.

The reference's importer (src/aexrt/onnx_importer.py:89) calls `onnx.load`; that package is not
installed on this machine, but `protobuf` is.  ONNX files are protobuf messages of the published
onnx.proto schema (proto2), so this module declares the subset of that schema an inference graph
uses -- ModelProto, GraphProto, NodeProto, AttributeProto, TensorProto, ValueInfoProto and the
type / shape messages -- with their published field numbers, and builds the message classes from
it at import time.  Fields outside the subset are kept as unknown fields by the parser, so a file
with them still loads.

    model = onnx_proto.load(path)          # ModelProto
    arr = onnx_proto.to_array(tensor)      # TensorProto -> numpy
    t = onnx_proto.from_array(arr, name)   # numpy -> TensorProto
    onnx_proto.save(model, path)
"""
from __future__ import annotations

import numpy as np
from google.protobuf import descriptor_pb2, descriptor_pool, message_factory

_F = descriptor_pb2.FieldDescriptorProto

# TensorProto.DataType values (onnx.proto)
FLOAT, UINT8, INT8, UINT16, INT16, INT32, INT64, STRING, BOOL, FLOAT16, DOUBLE, UINT32, UINT64 = (
    1, 2, 3, 4, 5, 6, 7, 8, 9, 10, 11, 12, 13)
_NP = {FLOAT: np.float32, UINT8: np.uint8, INT8: np.int8, UINT16: np.uint16, INT16: np.int16, INT32: np.int32,
       INT64: np.int64, BOOL: np.bool_, FLOAT16: np.float16, DOUBLE: np.float64, UINT32: np.uint32,
       UINT64: np.uint64}
_FROM_NP = {np.dtype(v): k for k, v in _NP.items()}

# AttributeProto.AttributeType values
ATTR_FLOAT, ATTR_INT, ATTR_STRING, ATTR_TENSOR, ATTR_GRAPH, ATTR_FLOATS, ATTR_INTS, ATTR_STRINGS, ATTR_TENSORS = (
    1, 2, 3, 4, 5, 6, 7, 8, 9)

# (message, [(field, number, label, type, type_name)]); labels: 1 optional, 3 repeated
_OPT, _REP = _F.LABEL_OPTIONAL, _F.LABEL_REPEATED
_SCHEMA = [
    ("StringStringEntryProto", [("key", 1, _OPT, _F.TYPE_STRING, None), ("value", 2, _OPT, _F.TYPE_STRING, None)]),
    ("TensorShapeProto.Dimension", [("dim_value", 1, _OPT, _F.TYPE_INT64, None),
                                    ("dim_param", 2, _OPT, _F.TYPE_STRING, None),
                                    ("denotation", 3, _OPT, _F.TYPE_STRING, None)]),
    ("TensorShapeProto", [("dim", 1, _REP, _F.TYPE_MESSAGE, ".onnx.TensorShapeProto.Dimension")]),
    ("TypeProto.Tensor", [("elem_type", 1, _OPT, _F.TYPE_INT32, None),
                          ("shape", 2, _OPT, _F.TYPE_MESSAGE, ".onnx.TensorShapeProto")]),
    ("TypeProto", [("tensor_type", 1, _OPT, _F.TYPE_MESSAGE, ".onnx.TypeProto.Tensor"),
                   ("denotation", 6, _OPT, _F.TYPE_STRING, None)]),
    ("ValueInfoProto", [("name", 1, _OPT, _F.TYPE_STRING, None), ("type", 2, _OPT, _F.TYPE_MESSAGE, ".onnx.TypeProto"),
                        ("doc_string", 3, _OPT, _F.TYPE_STRING, None)]),
    ("TensorProto", [("dims", 1, _REP, _F.TYPE_INT64, None), ("data_type", 2, _OPT, _F.TYPE_INT32, None),
                     ("float_data", 4, _REP, _F.TYPE_FLOAT, None), ("int32_data", 5, _REP, _F.TYPE_INT32, None),
                     ("string_data", 6, _REP, _F.TYPE_BYTES, None), ("int64_data", 7, _REP, _F.TYPE_INT64, None),
                     ("name", 8, _OPT, _F.TYPE_STRING, None), ("raw_data", 9, _OPT, _F.TYPE_BYTES, None),
                     ("double_data", 10, _REP, _F.TYPE_DOUBLE, None), ("uint64_data", 11, _REP, _F.TYPE_UINT64, None),
                     ("doc_string", 12, _OPT, _F.TYPE_STRING, None)]),
    ("AttributeProto", [("name", 1, _OPT, _F.TYPE_STRING, None), ("f", 2, _OPT, _F.TYPE_FLOAT, None),
                        ("i", 3, _OPT, _F.TYPE_INT64, None), ("s", 4, _OPT, _F.TYPE_BYTES, None),
                        ("t", 5, _OPT, _F.TYPE_MESSAGE, ".onnx.TensorProto"),
                        ("g", 6, _OPT, _F.TYPE_MESSAGE, ".onnx.GraphProto"),
                        ("floats", 7, _REP, _F.TYPE_FLOAT, None), ("ints", 8, _REP, _F.TYPE_INT64, None),
                        ("strings", 9, _REP, _F.TYPE_BYTES, None),
                        ("tensors", 10, _REP, _F.TYPE_MESSAGE, ".onnx.TensorProto"),
                        ("doc_string", 13, _OPT, _F.TYPE_STRING, None), ("type", 20, _OPT, _F.TYPE_INT32, None),
                        ("ref_attr_name", 21, _OPT, _F.TYPE_STRING, None)]),
    ("NodeProto", [("input", 1, _REP, _F.TYPE_STRING, None), ("output", 2, _REP, _F.TYPE_STRING, None),
                   ("name", 3, _OPT, _F.TYPE_STRING, None), ("op_type", 4, _OPT, _F.TYPE_STRING, None),
                   ("attribute", 5, _REP, _F.TYPE_MESSAGE, ".onnx.AttributeProto"),
                   ("doc_string", 6, _OPT, _F.TYPE_STRING, None), ("domain", 7, _OPT, _F.TYPE_STRING, None)]),
    ("GraphProto", [("node", 1, _REP, _F.TYPE_MESSAGE, ".onnx.NodeProto"), ("name", 2, _OPT, _F.TYPE_STRING, None),
                    ("initializer", 5, _REP, _F.TYPE_MESSAGE, ".onnx.TensorProto"),
                    ("doc_string", 10, _OPT, _F.TYPE_STRING, None),
                    ("input", 11, _REP, _F.TYPE_MESSAGE, ".onnx.ValueInfoProto"),
                    ("output", 12, _REP, _F.TYPE_MESSAGE, ".onnx.ValueInfoProto"),
                    ("value_info", 13, _REP, _F.TYPE_MESSAGE, ".onnx.ValueInfoProto")]),
    ("OperatorSetIdProto", [("domain", 1, _OPT, _F.TYPE_STRING, None), ("version", 2, _OPT, _F.TYPE_INT64, None)]),
    ("ModelProto", [("ir_version", 1, _OPT, _F.TYPE_INT64, None), ("producer_name", 2, _OPT, _F.TYPE_STRING, None),
                    ("producer_version", 3, _OPT, _F.TYPE_STRING, None), ("domain", 4, _OPT, _F.TYPE_STRING, None),
                    ("model_version", 5, _OPT, _F.TYPE_INT64, None), ("doc_string", 6, _OPT, _F.TYPE_STRING, None),
                    ("graph", 7, _OPT, _F.TYPE_MESSAGE, ".onnx.GraphProto"),
                    ("opset_import", 8, _REP, _F.TYPE_MESSAGE, ".onnx.OperatorSetIdProto"),
                    ("metadata_props", 14, _REP, _F.TYPE_MESSAGE, ".onnx.StringStringEntryProto")]),
]


def _build():
    fdp = descriptor_pb2.FileDescriptorProto()
    fdp.name = "aexrt_b200_onnx_subset.proto"
    fdp.package = "onnx"
    fdp.syntax = "proto2"
    top = {}
    # top-level messages first, then the nested ones into their parents
    for full, fields in sorted(_SCHEMA, key=lambda e: "." in e[0]):
        parts = full.split(".")
        if len(parts) == 1:
            msg = fdp.message_type.add()
            msg.name = parts[0]
            top[parts[0]] = msg
        else:
            msg = top[parts[0]].nested_type.add()
            msg.name = parts[1]
        for name, number, label, ftype, type_name in fields:
            f = msg.field.add()
            f.name, f.number, f.label, f.type = name, number, label, ftype
            if type_name:
                f.type_name = type_name
    pool = descriptor_pool.DescriptorPool()
    pool.Add(fdp)
    return {name: message_factory.GetMessageClass(pool.FindMessageTypeByName("onnx." + name))
            for name, _ in _SCHEMA if "." not in name}


_CLASSES = _build()
ModelProto = _CLASSES["ModelProto"]
GraphProto = _CLASSES["GraphProto"]
NodeProto = _CLASSES["NodeProto"]
TensorProto = _CLASSES["TensorProto"]
AttributeProto = _CLASSES["AttributeProto"]
ValueInfoProto = _CLASSES["ValueInfoProto"]


def load(path: str):
    """Parses an .onnx file into a ModelProto (weights stored inline in the file)."""
    m = ModelProto()
    with open(path, "rb") as f:
        m.ParseFromString(f.read())
    return m


def save(model, path: str) -> None:
    with open(path, "wb") as f:
        f.write(model.SerializeToString())


def to_array(t) -> np.ndarray:
    """TensorProto -> numpy array (raw_data or the typed repeated fields, little-endian)."""
    if t.data_type not in _NP:
        raise ValueError(f"tensor {t.name}: unsupported data type {t.data_type}")
    dt = np.dtype(_NP[t.data_type])
    shape = tuple(int(d) for d in t.dims)
    if t.raw_data:
        a = np.frombuffer(t.raw_data, dtype=dt.newbyteorder("<")).astype(dt)
    elif t.data_type in (FLOAT,):
        a = np.asarray(t.float_data, dtype=dt)
    elif t.data_type in (INT64,):
        a = np.asarray(t.int64_data, dtype=dt)
    elif t.data_type in (DOUBLE,):
        a = np.asarray(t.double_data, dtype=dt)
    elif t.data_type in (UINT32, UINT64):
        a = np.asarray(t.uint64_data, dtype=dt)
    elif t.data_type == FLOAT16:
        # int32_data carries the fp16 bit patterns
        a = np.asarray(t.int32_data, dtype=np.uint16).view(np.float16)
    else:
        a = np.asarray(t.int32_data, dtype=np.int64).astype(dt)
    return a.reshape(shape) if shape else a.reshape(())


def from_array(a: np.ndarray, name: str = ""):
    a = np.asarray(a)
    if a.dtype not in _FROM_NP:
        raise ValueError(f"unsupported dtype {a.dtype}")
    t = TensorProto()
    t.name = name
    t.data_type = _FROM_NP[a.dtype]
    t.dims.extend(int(d) for d in a.shape)
    t.raw_data = np.ascontiguousarray(a).astype(a.dtype.newbyteorder("<")).tobytes()
    return t


def attrs(node) -> dict:
    """A node's attributes as Python values (ints, floats, strings, tensors and their lists)."""
    out = {}
    for a in node.attribute:
        if a.type == ATTR_INT:
            out[a.name] = int(a.i)
        elif a.type == ATTR_FLOAT:
            out[a.name] = float(a.f)
        elif a.type == ATTR_STRING:
            out[a.name] = a.s.decode()
        elif a.type == ATTR_TENSOR:
            out[a.name] = to_array(a.t)
        elif a.type == ATTR_INTS:
            out[a.name] = [int(v) for v in a.ints]
        elif a.type == ATTR_FLOATS:
            out[a.name] = [float(v) for v in a.floats]
        elif a.type == ATTR_STRINGS:
            out[a.name] = [v.decode() for v in a.strings]
        else:
            out[a.name] = None
    return out


def make_attr(name: str, value):
    a = AttributeProto()
    a.name = name
    if isinstance(value, bool) or isinstance(value, (int, np.integer)):
        a.type, a.i = ATTR_INT, int(value)
    elif isinstance(value, (float, np.floating)):
        a.type, a.f = ATTR_FLOAT, float(value)
    elif isinstance(value, str):
        a.type, a.s = ATTR_STRING, value.encode()
    elif isinstance(value, np.ndarray):
        a.type = ATTR_TENSOR
        a.t.CopyFrom(from_array(value))
    elif isinstance(value, (list, tuple)) and all(isinstance(v, (int, np.integer)) for v in value):
        a.type = ATTR_INTS
        a.ints.extend(int(v) for v in value)
    elif isinstance(value, (list, tuple)):
        a.type = ATTR_FLOATS
        a.floats.extend(float(v) for v in value)
    else:
        raise ValueError(f"attribute {name}: unsupported value {value!r}")
    return a


def make_node(op_type: str, inputs, outputs, name: str = "", **attributes):
    n = NodeProto()
    n.op_type = op_type
    n.name = name
    n.input.extend(inputs)
    n.output.extend(outputs)
    for k, v in attributes.items():
        n.attribute.append(make_attr(k, v))
    return n


def make_value_info(name: str, elem_type: int, shape):
    v = ValueInfoProto()
    v.name = name
    v.type.tensor_type.elem_type = elem_type
    for d in shape:
        dim = v.type.tensor_type.shape.dim.add()
        if isinstance(d, str):
            dim.dim_param = d
        else:
            dim.dim_value = int(d)
    return v


def value_info_shape(v):
    """Shape of a ValueInfoProto: ints, -1 where the dimension is symbolic."""
    return tuple(int(d.dim_value) if d.HasField("dim_value") else -1 for d in v.type.tensor_type.shape.dim)
