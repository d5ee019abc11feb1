"""ONNX ingest (and export) of YOLO graphs for the W8A8 backend, without the `onnx` package.

The reference compiles ONNX models with `load_onnx` (src/aexrt/onnx_importer.py:89), which maps
the graph to its IR before the YOLO lowering (src/aexrt/yolo.py:464-537) fuses it into CONV /
CONV_SILU / CONCAT / RESIZE / MAXPOOL / BINARY commands.  `import_onnx` does both steps for the
graphs an ultralytics YOLOv8 / YOLOv11-head export contains, straight into this backend's command
stream (`yolo.YoloProgram`):

* Conv (groups 1, k 1 or 3, pad k/2, stride 1 or 2) -> ConvCmd; Conv with groups = channels
  (k 3) -> DwConvCmd; a following Sigmoid + Mul of the same tensor (SiLU) -> the command's SiLU;
* Add of a SiLU conv's only use and another tensor -> that conv's residual operand;
* Split / Slice on channels -> channel slices; Concat on channels -> multi-part inputs;
  Resize (nearest, x2) -> the upsample flag of the parts that read it;
* MaxPool(5, 1, 2) x 3 concatenated with its input (SPPF) -> SppfCmd;
* the detect head: per level a channel Concat of box (4 * reg_max) and class logits, reshaped to
  [N, C, H*W] and concatenated over the levels; everything after that Concat is the DFL / box
  decode, which becomes a DecodeCmd, as the reference replaces it by its fused decode
  (native/aexrt_d3d12_runtime.cpp:26956-27100).

Precision follows the reference's W8A8 rules: the image stem (3 input channels, refused by
`can_use_conv_int8`, runtime.cpp:9404) and the head convs (the single-consumer conv chains that
end in a head level) stay fp16; every other conv is W8A8.  Anything else fails with a message
naming the node.

`export_onnx` writes a program as such a graph (the export form, decode included), so that a
program can be handed to other ONNX tools and the importer can be checked against it.
"""
from __future__ import annotations

from collections import defaultdict
from dataclasses import dataclass
from typing import Dict, List, Optional, Tuple

import numpy as np

from . import onnx_proto as op
from .yolo import ConvCmd, DecodeCmd, DwConvCmd, Part, SppfCmd, ValueSpec, YoloProgram


class OnnxImportError(ValueError):
    pass


# ---------------------------------------------------------------------------------------- export
class _Exporter:
    def __init__(self, program: YoloProgram, batch: int):
        self.p = program
        self.n = batch
        self.nodes: List = []
        self.inits: List = []
        self.uid = 0
        # buffer value -> [(coff, ch, tensor)] written so far
        self.segments: Dict[str, List[Tuple[int, int, str]]] = defaultdict(list)
        self.split_cache: Dict[Tuple[str, int, int], str] = {}

    def name(self, base: str) -> str:
        self.uid += 1
        return f"{base}_{self.uid}"

    def const(self, base: str, arr) -> str:
        nm = self.name(base)
        self.inits.append(op.from_array(np.asarray(arr), nm))
        return nm

    def node(self, op_type: str, inputs, n_out: int = 1, **attrs) -> List[str]:
        outs = [self.name(op_type.lower()) for _ in range(n_out)]
        self.nodes.append(op.make_node(op_type, inputs, outs, name=self.name(op_type), **attrs))
        return outs

    def read(self, pt: Part) -> str:
        """A tensor holding channels [coff, coff + ch) of a buffer value (through its upsample)."""
        if pt.value == "images":
            t = "images"
        else:
            pieces = []
            lo, hi = pt.coff, pt.coff + pt.channels
            for c0, ch, tn in sorted(self.segments[pt.value]):
                a, b = max(lo, c0), min(hi, c0 + ch)
                if a >= b:
                    continue
                if a == c0 and b == c0 + ch:
                    pieces.append(tn)
                else:
                    key = (tn, a - c0, b - c0)
                    if key not in self.split_cache:
                        # channels [a, b) of tn: Split into (before, wanted, after)
                        sizes = [s for s in (a - c0, b - a, c0 + ch - b) if s > 0]
                        outs = self.node("Split", [tn, self.const("split", np.array(sizes, np.int64))],
                                         n_out=len(sizes), axis=1)
                        self.split_cache[key] = outs[1] if a > c0 else outs[0]
                    pieces.append(self.split_cache[key])
            covered = sum(min(hi, c0 + ch) - max(lo, c0) for c0, ch, _ in self.segments[pt.value]
                          if max(lo, c0) < min(hi, c0 + ch))
            if covered != pt.channels:
                raise OnnxImportError(f"export: {pt.value}[{lo}:{hi}] is read before it is written")
            t = pieces[0] if len(pieces) == 1 else self.node("Concat", pieces, axis=1)[0]
        if pt.upsample != 1:
            t = self.node("Resize", [t, "", self.const("scales", np.array([1, 1, pt.upsample, pt.upsample],
                                                                           np.float32))],
                          mode="nearest", coordinate_transformation_mode="asymmetric", nearest_mode="floor")[0]
        return t

    def inputs(self, parts: List[Part]) -> str:
        ts = [self.read(pt) for pt in parts]
        return ts[0] if len(ts) == 1 else self.node("Concat", ts, axis=1)[0]

    def silu(self, t: str) -> str:
        s = self.node("Sigmoid", [t])[0]
        return self.node("Mul", [t, s])[0]

    def write(self, value: str, coff: int, ch: int, t: str) -> None:
        self.segments[value].append((coff, ch, t))

    def conv(self, c: ConvCmd) -> None:
        x = self.inputs(c.inputs)
        w = self.const(c.name + ".w", c.weight.astype(np.float32))
        b = self.const(c.name + ".b", c.bias.astype(np.float32))
        p = c.k // 2
        y = self.node("Conv", [x, w, b], kernel_shape=[c.k, c.k], strides=[c.s, c.s], pads=[p, p, p, p],
                      group=1, dilations=[1, 1])[0]
        if c.silu:
            y = self.silu(y)
        if c.residual is not None:
            y = self.node("Add", [y, self.read(Part(c.residual[0], c.residual[1], c.oc))])[0]
        self.write(c.out[0], c.out[1], c.oc, y)

    def dwconv(self, c: DwConvCmd) -> None:
        g = c.group or c.c
        if g != c.c:
            raise OnnxImportError(f"export: {c.name} gathers per-head channels (an attention block)")
        x = self.read(Part(c.x.value, c.x.coff + c.group_off, c.c))
        w = self.const(c.name + ".w", c.weight.astype(np.float32))
        b = self.const(c.name + ".b", c.bias.astype(np.float32))
        y = self.node("Conv", [x, w, b], kernel_shape=[3, 3], strides=[c.s, c.s], pads=[1, 1, 1, 1], group=c.c,
                      dilations=[1, 1])[0]
        if c.silu:
            y = self.silu(y)
        self.write(c.out[0], c.out[1], c.c, y)

    def sppf(self, c: SppfCmd) -> None:
        t = self.read(c.x)
        for i in range(3):
            t = self.node("MaxPool", [t], kernel_shape=[5, 5], strides=[1, 1], pads=[2, 2, 2, 2])[0]
            self.write(c.out[0], c.out[1] + i * c.x.channels, c.x.channels, t)

    def decode(self, c: DecodeCmd) -> str:
        """The export form of the anchor-free head: per level cat(box, cls) -> [N, C, H*W], levels
        concatenated, then DFL (softmax expectation over reg_max bins, as a 1x1 conv with weights
        0..reg_max-1), distances -> box around the anchor centre, times the stride, class sigmoid."""
        n, rm, nc = self.n, c.reg_max, c.nc
        flat, anchors, strides = [], [], []
        for bp, cp, stride in c.levels:
            h, w = self.p.values[bp.value].h, self.p.values[bp.value].w
            lv = self.node("Concat", [self.read(bp), self.read(cp)], axis=1)[0]
            flat.append(self.node("Reshape", [lv, self.const("shape", np.array([n, 4 * rm + nc, -1], np.int64))])[0])
            gy, gx = np.meshgrid(np.arange(h, dtype=np.float32) + 0.5, np.arange(w, dtype=np.float32) + 0.5,
                                 indexing="ij")
            anchors.append(np.stack([gx.reshape(-1), gy.reshape(-1)]))
            strides.append(np.full((1, h * w), stride, np.float32))
        x = self.node("Concat", flat, axis=2)[0]
        a_total = sum(a.shape[1] for a in anchors)
        box, cls = self.node("Split", [x, self.const("split", np.array([4 * rm, nc], np.int64))], n_out=2, axis=1)
        t = self.node("Reshape", [box, self.const("shape", np.array([n, 4, rm, a_total], np.int64))])[0]
        t = self.node("Transpose", [t], perm=[0, 2, 1, 3])[0]
        t = self.node("Softmax", [t], axis=1)[0]
        dfl = self.const("dfl.w", np.arange(rm, dtype=np.float32).reshape(1, rm, 1, 1))
        t = self.node("Conv", [t, dfl], kernel_shape=[1, 1])[0]
        dist = self.node("Reshape", [t, self.const("shape", np.array([n, 4, a_total], np.int64))])[0]
        lt, rb = self.node("Split", [dist, self.const("split", np.array([2, 2], np.int64))], n_out=2, axis=1)
        anc = self.const("anchors", np.concatenate(anchors, axis=1)[None])
        x1y1 = self.node("Sub", [anc, lt])[0]
        x2y2 = self.node("Add", [anc, rb])[0]
        c_xy = self.node("Div", [self.node("Add", [x1y1, x2y2])[0], self.const("two", np.array(2.0, np.float32))])[0]
        wh = self.node("Sub", [x2y2, x1y1])[0]
        dbox = self.node("Mul", [self.node("Concat", [c_xy, wh], axis=1)[0],
                                 self.const("strides", np.concatenate(strides, axis=1)[None])])[0]
        return self.node("Concat", [dbox, self.node("Sigmoid", [cls])[0]], axis=1)[0]


def export_onnx(program: YoloProgram, path: Optional[str] = None, batch: int = 1, opset: int = 17):
    """The program as an ONNX ModelProto (and file, when `path` is given): input `images`
    [batch, 3, imgsz, imgsz] fp32, output `output0` [batch, 4 + nc, anchors]."""
    ex = _Exporter(program, batch)
    out = None
    for c in program.commands:
        if isinstance(c, ConvCmd):
            ex.conv(c)
        elif isinstance(c, DwConvCmd):
            ex.dwconv(c)
        elif isinstance(c, SppfCmd):
            ex.sppf(c)
        elif isinstance(c, DecodeCmd):
            out = ex.decode(c)
        else:
            raise OnnxImportError(f"export: command {type(c).__name__} {c.name} has no ONNX form here")
    if out is None:
        raise OnnxImportError("export: the program has no detect head")
    for nd in ex.nodes:  # name the graph output
        for i, o in enumerate(nd.output):
            if o == out:
                nd.output[i] = "output0"
    m = op.ModelProto()
    m.ir_version = 8
    m.producer_name = "aexrt_b200"
    oi = m.opset_import.add()
    oi.domain, oi.version = "", opset
    g = m.graph
    g.name = program.name
    g.node.extend(ex.nodes)
    g.initializer.extend(ex.inits)
    g.input.append(op.make_value_info("images", op.FLOAT, [batch, program.in_channels, program.imgsz, program.imgsz]))
    g.output.append(op.make_value_info("output0", op.FLOAT, [batch, 4 + program.nc, program.anchors]))
    if path:
        op.save(m, path)
    return m


# ---------------------------------------------------------------------------------------- import
@dataclass
class _Act:
    """An NCHW activation of the graph as channel ranges of the program's buffers."""

    parts: List[Part]
    h: int
    w: int

    @property
    def channels(self) -> int:
        return sum(p.channels for p in self.parts)

    def slice(self, lo: int, hi: int) -> "_Act":
        out, base = [], 0
        for p in self.parts:
            a, b = max(lo, base), min(hi, base + p.channels)
            if a < b:
                out.append(Part(p.value, p.coff + a - base, b - a, p.upsample))
            base += p.channels
        return _Act(out, self.h, self.w)


def _merge(parts: List[Part]) -> List[Part]:
    """Adjacent ranges of one buffer (same upsample) joined into one part."""
    out: List[Part] = []
    for p in parts:
        q = out[-1] if out else None
        if q is not None and q.value == p.value and q.upsample == p.upsample and q.coff + q.channels == p.coff:
            out[-1] = Part(q.value, q.coff, q.channels + p.channels, q.upsample)
        else:
            out.append(Part(p.value, p.coff, p.channels, p.upsample))
    return out


class _Importer:
    def __init__(self, model, name: Optional[str]):
        g = model.graph
        self.g = g
        self.consts: Dict[str, np.ndarray] = {t.name: op.to_array(t) for t in g.initializer}
        self.nodes = list(g.node)
        self.producer = {o: i for i, nd in enumerate(self.nodes) for o in nd.output}
        self.consumers: Dict[str, List[int]] = defaultdict(list)
        for i, nd in enumerate(self.nodes):
            for t in nd.input:
                self.consumers[t].append(i)
        for nd in self.nodes:  # Constant nodes become constants
            if nd.op_type == "Constant":
                self.consts[nd.output[0]] = op.attrs(nd)["value"]
        inputs = [v for v in g.input if v.name not in self.consts]
        if len(inputs) != 1:
            raise OnnxImportError(f"expected one image input, found {[v.name for v in inputs]}")
        shape = op.value_info_shape(inputs[0])
        if len(shape) != 4 or shape[1] != 3 or shape[2] != shape[3] or shape[2] <= 0:
            raise OnnxImportError(f"image input {inputs[0].name}: expected [N, 3, S, S], got {shape}")
        self.imgsz = shape[2]
        outs = list(g.output)
        if len(outs) != 1:
            raise OnnxImportError(f"expected one output (output0), found {len(outs)}")
        oshape = op.value_info_shape(outs[0])
        if len(oshape) != 3 or oshape[1] <= 4:
            raise OnnxImportError(f"output {outs[0].name}: expected [N, 4 + nc, anchors], got {oshape}")
        self.nc = oshape[1] - 4
        self.output = outs[0].name
        self.prog = YoloProgram(name=name or (g.name or "onnx_yolo"), in_channels=3, imgsz=self.imgsz, nc=self.nc,
                                reg_max=16)
        self.prog.values["images"] = ValueSpec(3, self.imgsz, self.imgsz)
        self.acts: Dict[str, _Act] = {inputs[0].name: _Act([Part("images", 0, 3)], self.imgsz, self.imgsz)}
        self.done = set()
        self.convs: Dict[str, ConvCmd] = {}  # tensor -> the conv (or depthwise conv) that produced it
        self.pools: Dict[str, Tuple[str, int]] = {}  # MaxPool output -> (SPPF source tensor, depth)
        self.levels: Dict[str, _Act] = {}  # a head level [N, C, H*W] reshape -> its channels
        self.head_sources: List[str] = []
        self.uid = 0

    def fail(self, nd, why: str):
        raise OnnxImportError(f"node {nd.name or nd.op_type} ({nd.op_type}): {why}")

    def value(self, base: str, ch: int, h: int, w: int) -> str:
        self.uid += 1
        name = f"{base}#{self.uid}"
        self.prog.values[name] = ValueSpec(ch, h, w)
        return name

    def act(self, nd, t: str) -> _Act:
        if t not in self.acts:
            self.fail(nd, f"input {t} is not an activation this importer tracks")
        return self.acts[t]

    def const(self, nd, t: str) -> np.ndarray:
        if t not in self.consts:
            self.fail(nd, f"input {t} must be a constant")
        return self.consts[t]

    def only_use(self, t: str):
        c = self.consumers.get(t, [])
        return c[0] if len(c) == 1 else None

    # ------------------------------------------------------------------ nodes
    def conv(self, i: int, nd) -> None:
        a = op.attrs(nd)
        x = self.act(nd, nd.input[0])
        w = self.const(nd, nd.input[1]).astype(np.float32)
        b = (self.const(nd, nd.input[2]).astype(np.float32) if len(nd.input) > 2 and nd.input[2]
             else np.zeros(w.shape[0], np.float32))
        oc, _, kh, kw = w.shape
        k = kh
        s = a.get("strides", [1, 1])
        pads = a.get("pads", [0, 0, 0, 0])
        group = a.get("group", 1)
        if kh != kw or s[0] != s[1] or s[0] not in (1, 2) or any(p != k // 2 for p in pads) or \
                any(d != 1 for d in a.get("dilations", [1, 1])) or a.get("auto_pad", "NOTSET") != "NOTSET":
            self.fail(nd, f"needs a square kernel, stride 1 or 2, pad kernel/2 and no dilation ({a})")
        s = s[0]
        oh, ow = (x.h + 2 * (k // 2) - k) // s + 1, (x.w + 2 * (k // 2) - k) // s + 1
        y = nd.output[0]
        silu = False
        cons = self.consumers.get(y, [])
        if len(cons) == 2:
            sg = next((c for c in cons if self.nodes[c].op_type == "Sigmoid"), None)
            if sg is not None:
                mul = next((c for c in cons if self.nodes[c].op_type == "Mul" and
                            set(self.nodes[c].input) == {y, self.nodes[sg].output[0]}), None)
                if mul is not None:
                    silu = True
                    self.done.update((sg, mul))
                    y = self.nodes[mul].output[0]
        name = nd.name or f"conv{i}"
        if group == 1:
            if k not in (1, 3):
                self.fail(nd, f"kernel {k}x{k}: the W8A8 and fp16 conv kernels take 1x1 and 3x3")
            v = self.value(name, oc, oh, ow)
            cmd = ConvCmd(name, _merge(x.parts), (v, 0), x.channels, oc, k, s, silu, w, b, precision="int8")
            add = self.only_use(y)
            if add is not None and self.nodes[add].op_type == "Add":
                other = [t for t in self.nodes[add].input if t != y]
                if len(other) == 1 and other[0] in self.acts:
                    r = self.acts[other[0]]
                    rp = _merge(r.parts)
                    if (len(rp) == 1 and rp[0].upsample == 1 and r.channels == oc and (r.h, r.w) == (oh, ow)
                            and (silu or cmd.precision == "int8")):
                        cmd.residual = (rp[0].value, rp[0].coff)
                        self.done.add(add)
                        y = self.nodes[add].output[0]
            self.prog.commands.append(cmd)
        elif group == x.channels == oc and k == 3:
            xp = _merge(x.parts)
            if len(xp) != 1 or xp[0].upsample != 1:
                self.fail(nd, "a depthwise conv needs its input in one buffer")
            v = self.value(name, oc, oh, ow)
            cmd = DwConvCmd(name, xp[0], (v, 0), oc, s, silu, w, b)
            self.prog.commands.append(cmd)
        else:
            self.fail(nd, f"groups {group} with {x.channels} input and {oc} output channels")
        self.convs[y] = cmd
        self.conv_node[cmd.name] = nd
        self.acts[y] = _Act([Part(v, 0, oc)], oh, ow)

    def split(self, nd) -> None:
        a = op.attrs(nd)
        x = self.act(nd, nd.input[0])
        axis = a.get("axis", 0)
        if axis not in (1, -3):
            self.fail(nd, "only channel splits")
        if len(nd.input) > 1 and nd.input[1]:
            sizes = [int(v) for v in self.const(nd, nd.input[1])]
        elif "split" in a:
            sizes = a["split"]
        else:
            sizes = [x.channels // len(nd.output)] * len(nd.output)
        if sum(sizes) != x.channels:
            self.fail(nd, f"split sizes {sizes} do not cover {x.channels} channels")
        base = 0
        for t, sz in zip(nd.output, sizes):
            self.acts[t] = x.slice(base, base + sz)
            base += sz

    def slice(self, nd) -> None:
        x = self.act(nd, nd.input[0])
        starts = [int(v) for v in self.const(nd, nd.input[1])]
        ends = [int(v) for v in self.const(nd, nd.input[2])]
        axes = [int(v) for v in self.const(nd, nd.input[3])] if len(nd.input) > 3 and nd.input[3] else [0]
        steps = [int(v) for v in self.const(nd, nd.input[4])] if len(nd.input) > 4 and nd.input[4] else [1]
        if axes not in ([1], [-3]) or steps != [1]:
            self.fail(nd, "only unit-step channel slices")
        lo = starts[0] + (x.channels if starts[0] < 0 else 0)
        hi = min(ends[0] + (x.channels if ends[0] < 0 else 0), x.channels)
        self.acts[nd.output[0]] = x.slice(lo, hi)

    def resize(self, nd) -> None:
        a = op.attrs(nd)
        x = self.act(nd, nd.input[0])
        if a.get("mode", "nearest") != "nearest":
            self.fail(nd, "only nearest resize")
        if len(nd.input) > 2 and nd.input[2] and nd.input[2] in self.consts and self.consts[nd.input[2]].size:
            sc = [float(v) for v in self.consts[nd.input[2]]]
        elif len(nd.input) > 3 and nd.input[3]:
            sz = [int(v) for v in self.const(nd, nd.input[3])]
            sc = [1.0, 1.0, sz[2] / x.h, sz[3] / x.w]
        else:
            self.fail(nd, "no scales or sizes")
        if sc != [1.0, 1.0, 2.0, 2.0] or any(p.upsample != 1 for p in x.parts):
            self.fail(nd, f"only one nearest 2x upsample per tensor (scales {sc})")
        self.acts[nd.output[0]] = _Act([Part(p.value, p.coff, p.channels, 2) for p in x.parts], 2 * x.h, 2 * x.w)

    def maxpool(self, nd) -> None:
        a = op.attrs(nd)
        if a.get("kernel_shape") != [5, 5] or a.get("strides", [1, 1]) != [1, 1] or a.get("pads") != [2, 2, 2, 2]:
            self.fail(nd, "only the SPPF pool (5x5, stride 1, pad 2)")
        src = nd.input[0]
        self.pools[nd.output[0]] = (self.pools[src][0], self.pools[src][1] + 1) if src in self.pools else (src, 1)

    def concat(self, i: int, nd) -> bool:
        """Channel concat (multi-part input, or the SPPF pattern); returns True at the head's level
        concat (axis 2), where the import stops."""
        a = op.attrs(nd)
        axis = a.get("axis", 0)
        if axis in (2, -1) and all(t in self.levels for t in nd.input):
            self.head(nd)
            return True
        if axis not in (1, -3):
            self.fail(nd, f"concat on axis {axis}")
        ins = list(nd.input)
        if len(ins) == 4 and ins[0] in self.acts and all(
                self.pools.get(t) == (ins[0], d) for d, t in zip((1, 2, 3), ins[1:])):
            # SPPF: x, pool(x), pool(pool(x)), pool(pool(pool(x))) -> one SPPF command writing the three
            # pooled slices of a new buffer
            x = self.acts[ins[0]]
            xp = _merge(x.parts)
            if len(xp) != 1 or xp[0].upsample != 1 or x.channels % 16:
                self.fail(nd, "SPPF input must be one buffer slice of 16k channels")
            v = self.value((nd.name or f"sppf{i}") + ".m", 3 * x.channels, x.h, x.w)
            self.prog.commands.append(SppfCmd(nd.name or f"sppf{i}", xp[0], (v, 0)))
            self.acts[nd.output[0]] = _Act(xp + [Part(v, 0, 3 * x.channels)], x.h, x.w)
            return False
        acts = [self.act(nd, t) for t in ins]
        if len({(x.h, x.w) for x in acts}) != 1:
            self.fail(nd, "concatenated maps differ in size")
        self.acts[nd.output[0]] = _Act(_merge([p for x in acts for p in x.parts]), acts[0].h, acts[0].w)
        return False

    def reshape(self, nd) -> None:
        x = self.act(nd, nd.input[0])
        shape = [int(v) for v in self.const(nd, nd.input[1])]
        if len(shape) != 3 or shape[1] != x.channels or shape[2] not in (-1, x.h * x.w):
            self.fail(nd, f"reshape {shape} of a [{x.channels}, {x.h}, {x.w}] map is not a head level")
        self.levels[nd.output[0]] = x

    def head(self, nd) -> None:
        nc = self.nc
        lv = [self.levels[t] for t in nd.input]
        extra = lv[0].channels - nc
        if extra <= 0 or extra % 4 or any(x.channels != lv[0].channels for x in lv):
            self.fail(nd, f"head levels of {[x.channels for x in lv]} channels do not fit nc={nc}")
        reg_max = extra // 4
        levels = []
        for x in lv:
            box, cls = x.slice(0, 4 * reg_max), x.slice(4 * reg_max, x.channels)
            if len(box.parts) != 1 or len(cls.parts) != 1 or box.parts[0].upsample != 1:
                self.fail(nd, "box and class logits of a level must each be one buffer slice")
            if self.imgsz % x.h:
                self.fail(nd, f"a {x.h}x{x.w} level does not divide the {self.imgsz} input")
            levels.append((box.parts[0], cls.parts[0], float(self.imgsz // x.h)))
            self.head_sources += [box.parts[0].value, cls.parts[0].value]
        self.prog.reg_max = reg_max
        self.prog.commands.append(DecodeCmd(nd.name or "decode", levels, nc, reg_max))
        if sum(x.h * x.w for x in lv) != self.prog.anchors:
            self.fail(nd, "head levels are not the stride 8 / 16 / 32 maps of the input")
        # what follows is the DFL + box decode (softmax over the bins, anchors, strides, class sigmoid):
        # the decode command computes it; the graph must end in output0 after it
        rest = {self.nodes[j].op_type for j in range(self.producer[nd.output[0]] + 1, len(self.nodes))}
        if "Softmax" not in rest or self.output not in self.producer or \
                self.producer[self.output] <= self.producer[nd.output[0]]:
            self.fail(nd, "the head concat is not followed by the DFL decode of output0")

    # ------------------------------------------------------------------ driver
    def run(self) -> YoloProgram:
        self.conv_node = {}
        handlers = {"Split": self.split, "Slice": self.slice, "Resize": self.resize, "MaxPool": self.maxpool,
                    "Reshape": self.reshape}
        for i, nd in enumerate(self.nodes):
            if i in self.done or nd.op_type == "Constant":
                continue
            if nd.op_type == "Conv":
                self.conv(i, nd)
            elif nd.op_type == "Concat":
                if self.concat(i, nd):
                    break
            elif nd.op_type == "Identity":
                self.acts[nd.output[0]] = self.act(nd, nd.input[0])
            elif nd.op_type in handlers:
                handlers[nd.op_type](nd)
            else:
                self.fail(nd, "operator not on the YOLO path this importer lowers")
        if not any(isinstance(c, DecodeCmd) for c in self.prog.commands):
            raise OnnxImportError("no detect head (per-level [N, C, H*W] reshapes concatenated on axis 2) found")
        self.precision()
        return self.prog

    def upstream(self, t: str) -> List[str]:
        """The tensors a head chain continues from: `t` itself when it has one use; the inputs of a
        channel Concat that is its only use; the source of channel slices that are the source's only
        uses.  Empty at a junction of several consumers (a neck output feeding both head branches)."""
        j = self.producer.get(t)
        if j is not None and self.nodes[j].op_type in ("Split", "Slice"):
            src = self.nodes[j].input[0]
            if all(self.nodes[c].op_type in ("Split", "Slice") for c in self.consumers[src]):
                return self.upstream(src) if src not in self.convs else [src]
            return []
        if len(self.consumers.get(t, [])) != 1:
            return []
        if j is not None and self.nodes[j].op_type == "Concat":
            return [u for s in self.nodes[j].input for u in self.upstream(s)]
        return [t]

    def precision(self) -> None:
        """fp16 for the image stem, the head chains and convs the int8 guard refuses; W8A8 otherwise."""
        by_value = {c.out[0]: c for c in self.prog.commands if isinstance(c, (ConvCmd, DwConvCmd))}
        todo = [by_value[v] for v in self.head_sources if v in by_value]
        seen = set()
        while todo:
            c = todo.pop()
            if id(c) in seen:
                continue
            seen.add(id(c))
            if isinstance(c, ConvCmd):
                c.precision = "fp16"
            for t in self.upstream(self.conv_node[c.name].input[0]):
                if t in self.convs:
                    todo.append(self.convs[t])
        for c in self.prog.commands:
            if not isinstance(c, ConvCmd):
                continue
            if any(p.value == "images" for p in c.inputs) or c.ic % 4 or c.oc % 4:
                c.precision = "fp16"  # can_use_conv_int8 refuses it (runtime.cpp:9404)
            if c.precision == "fp16" and c.residual is not None and not c.silu:
                raise OnnxImportError(f"{c.name}: an fp16 conv with a residual needs SiLU")


def import_onnx(path_or_model, name: Optional[str] = None) -> YoloProgram:
    """An ONNX YOLO model (file path or ModelProto) as this backend's command stream."""
    model = op.load(path_or_model) if isinstance(path_or_model, str) else path_or_model
    return _Importer(model, name).run()
