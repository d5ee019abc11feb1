"""YOLOv8-architecture command streams for the W8A8 backend.

The reference lowers an ONNX YOLO graph into a prepared command stream of
CONV / CONV_SILU / CONCAT / RESIZE / MAXPOOL / BINARY ... commands
(src/aexrt/yolo.py:464-537, kinds in src/aexrt/engine.py:103-118) and then
chooses a kernel per command (kernel plan, engine.py:1046-1222; W8A8 ids
51/52/53 via algo overrides, engine.py:1112-1215).  This module builds the same
kind of command stream directly from the architecture (no ONNX is available on
this machine), with random seeded weights, already in the fused form this
backend executes:

* CONCAT + conv            -> one conv whose input lists the concatenated parts
* RESIZE (nearest 2x)      -> an upsample flag on the consumer's input part
* C2f split / chunk        -> channel slices of one NHWC buffer
* C2f bottleneck Add       -> the residual operand of the second conv's epilogue
* SPPF MaxPool x3 + CONCAT -> one SPPF pool command writing three slices

Architecture and scaling follow the public YOLOv8 definition (width / depth
multipliers, C2f, SPPF k=5, anchor-free decoupled Detect head with DFL
reg_max=16).  Weights are random: N(0, 1/sqrt(fan_in)) and biases N(0, 0.1),
seeded, so activations stay O(1) through the network.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Tuple

import numpy as np


@dataclass
class Part:
    """One channel range of a command input: value[..., coff:coff+channels], read through an upsample."""

    value: str
    coff: int
    channels: int
    upsample: int = 1


@dataclass
class ConvCmd:
    name: str
    inputs: List[Part]
    out: Tuple[str, int]          # (value, channel offset)
    ic: int
    oc: int
    k: int
    s: int
    silu: bool
    weight: np.ndarray            # [oc, ic, k, k] fp32
    bias: np.ndarray              # [oc] fp32
    precision: str = "int8"       # "int8" (W8A8 kernel 51/52/53) or "fp16"
    residual: Optional[Tuple[str, int]] = None  # (value, channel offset), added after SiLU
    pg16: bool = False            # INT8_PERGROUP plan flag
    block_n: int = 0              # preferred output-channel tile of the plan (0: the plan's choice)

    @property
    def kind(self) -> str:
        return "CONV_SILU" if self.silu else "CONV"


@dataclass
class SppfCmd:
    name: str
    x: Part
    out: Tuple[str, int]  # three consecutive slices of x.channels each


@dataclass
class DwConvCmd:
    """Depthwise 3x3 conv (pad 1) in fp16: YOLOv11's DWConv and the C2PSA positional encoding.

    Output channel k reads input channel x.coff + (k // group) * group_stride + group_off + k % group
    (group = c: the plain slice x)."""

    name: str
    x: Part
    out: Tuple[str, int]
    c: int
    s: int
    silu: bool
    weight: np.ndarray            # [c, 1, 3, 3] fp32
    bias: np.ndarray              # [c] fp32
    group: int = 0
    group_stride: int = 0
    group_off: int = 0

    def in_channel(self, k: int) -> int:
        g = self.group or self.c
        return self.x.coff + (k // g) * (self.group_stride or g) + self.group_off + k % g


@dataclass
class PsaAttnCmd:
    """C2PSA attention core: per head softmax(q^T k * key_dim^-0.5) applied to v, plus pe."""

    name: str
    qkv: Part                     # heads * (2 * key_dim + head_dim) channels
    pe: Part                      # heads * head_dim channels
    out: Tuple[str, int]
    heads: int
    key_dim: int
    head_dim: int

    @property
    def scale(self) -> float:
        return float(self.key_dim) ** -0.5


@dataclass
class DecodeCmd:
    name: str
    levels: List[Tuple[Part, Part, float]]  # (box logits, class logits, stride)
    nc: int
    reg_max: int


@dataclass
class ValueSpec:
    channels: int
    h: int
    w: int


@dataclass
class YoloProgram:
    """Command stream + value table of one model at one input size."""

    name: str
    in_channels: int
    imgsz: int
    nc: int
    reg_max: int
    values: Dict[str, ValueSpec] = field(default_factory=dict)
    commands: list = field(default_factory=list)
    output: str = "output0"

    @property
    def anchors(self) -> int:
        return sum((self.imgsz // s) ** 2 for s in (8, 16, 32))

    def conv_macs_per_image(self, precision: Optional[str] = None) -> int:
        total = 0
        for c in self.commands:
            if isinstance(c, ConvCmd) and (precision is None or c.precision == precision):
                v = self.values[c.out[0]]
                total += v.h * v.w * c.oc * c.ic * c.k * c.k
        return total


def _make_divisible(x: float, d: int = 8) -> int:
    return int(math.ceil(x / d) * d)


class _Builder:
    def __init__(self, name: str, imgsz: int, nc: int, seed: int, reg_max: int = 16, gain: float = 1.0,
                 cls_gain: float = 1.0, cls_bias: float = 0.0):
        self.p = YoloProgram(name=name, in_channels=3, imgsz=imgsz, nc=nc, reg_max=reg_max)
        self.rng = np.random.default_rng(seed)
        self.gain = gain
        self.cls_gain = cls_gain
        self.cls_bias = cls_bias
        self.p.values["images"] = ValueSpec(3, imgsz, imgsz)

    def value(self, name: str, channels: int, h: int, w: int) -> str:
        self.p.values[name] = ValueSpec(channels, h, w)
        return name

    def _weights(self, oc: int, ic: int, k: int) -> Tuple[np.ndarray, np.ndarray]:
        w = self.rng.normal(0.0, self.gain / math.sqrt(ic * k * k), (oc, ic, k, k)).astype(np.float32)
        b = self.rng.normal(0.0, 0.1, (oc,)).astype(np.float32)
        return w, b

    def conv(self, name: str, inputs: List[Part], out: Tuple[str, int], oc: int, k: int, s: int, silu: bool = True,
             precision: str = "int8", residual=None) -> ConvCmd:
        ic = sum(pt.channels for pt in inputs)
        w, b = self._weights(oc, ic, k)
        cmd = ConvCmd(name, inputs, out, ic, oc, k, s, silu, w, b, precision, residual)
        self.p.commands.append(cmd)
        return cmd

    def spatial(self, value: str) -> Tuple[int, int]:
        v = self.p.values[value]
        return v.h, v.w

    # ---------------------------------------------------------------- blocks
    def conv_block(self, name: str, src: List[Part], oc: int, k: int, s: int, precision: str = "int8") -> str:
        h, w = self.spatial(src[0].value)
        h *= src[0].upsample
        w *= src[0].upsample
        oh, ow = (h + 2 * (k // 2) - k) // s + 1, (w + 2 * (k // 2) - k) // s + 1
        out = self.value(name, oc, oh, ow)
        self.conv(name, src, (out, 0), oc, k, s, precision=precision)
        return out

    def c2f(self, name: str, src: List[Part], c2: int, n: int, shortcut: bool) -> str:
        """C2f: cv1 -> split(c, c) -> n bottlenecks on the last chunk -> concat -> cv2."""
        h, w = self.spatial(src[0].value)
        h *= src[0].upsample
        w *= src[0].upsample
        c = c2 // 2
        y = self.value(name + ".y", (2 + n) * c, h, w)
        self.conv(name + ".cv1", src, (y, 0), 2 * c, 1, 1)
        for i in range(n):
            t = self.value(f"{name}.m{i}.t", c, h, w)
            self.conv(f"{name}.m{i}.cv1", [Part(y, (1 + i) * c, c)], (t, 0), c, 3, 1)
            self.conv(f"{name}.m{i}.cv2", [Part(t, 0, c)], (y, (2 + i) * c), c, 3, 1,
                      residual=(y, (1 + i) * c) if shortcut else None)
        out = self.value(name, c2, h, w)
        self.conv(name + ".cv2", [Part(y, 0, (2 + n) * c)], (out, 0), c2, 1, 1)
        return out

    def sppf(self, name: str, src: str, c2: int) -> str:
        v = self.p.values[src]
        c_ = v.channels // 2
        cat = self.value(name + ".cat", 4 * c_, v.h, v.w)
        self.conv(name + ".cv1", [Part(src, 0, v.channels)], (cat, 0), c_, 1, 1)
        self.p.commands.append(SppfCmd(name + ".m", Part(cat, 0, c_), (cat, c_)))
        out = self.value(name, c2, v.h, v.w)
        self.conv(name + ".cv2", [Part(cat, 0, 4 * c_)], (out, 0), c2, 1, 1)
        return out

    def detect(self, name: str, feats: List[str], strides: List[float], fused: bool = True):
        nc, reg_max = self.p.nc, self.p.reg_max
        chs = [self.p.values[f].channels for f in feats]
        c2 = max(16, chs[0] // 4, reg_max * 4)
        c3 = max(chs[0], min(nc, 100))
        if not fused:
            return self._detect_branches(name, feats, strides, c2, c3)
        levels = []
        for i, (f, st) in enumerate(zip(feats, strides)):
            v = self.p.values[f]
            h0 = self.value(f"{name}.{i}.h0", c2 + c3, v.h, v.w)
            h1 = self.value(f"{name}.{i}.h1", c2 + c3, v.h, v.w)
            # box logits then class logits; rows padded to a multiple of 8 channels (16-byte stores)
            o = self.value(f"{name}.{i}.out", _make_divisible(4 * reg_max + nc, 8), v.h, v.w)
            # cv2[i][0] and cv3[i][0] read the same input: one conv with c2 + c3 outputs
            self.conv(f"{name}.{i}.cv23_0", [Part(f, 0, chs[i])], (h0, 0), c2 + c3, 3, 1, precision="fp16")
            self.conv(f"{name}.{i}.cv2_1", [Part(h0, 0, c2)], (h1, 0), c2, 3, 1, precision="fp16")
            self.conv(f"{name}.{i}.cv3_1", [Part(h0, c2, c3)], (h1, c2), c3, 3, 1, precision="fp16")
            levels.append(self._head_logits(f"{name}.{i}", h1, o, c2, c3, st))
        self.p.commands.append(DecodeCmd(name + ".decode", levels, nc, reg_max))

    def _detect_branches(self, name: str, feats: List[str], strides: List[float], c2: int, c3: int):
        """The Detect head in its model form: per level a box branch (3x3, 3x3, 1x1 to 4 * reg_max) and
        a class branch (3x3, 3x3, 1x1 to nc), each conv its own command; the two 1x1s write the box and
        class logits side by side in the level's output buffer."""
        nc, reg_max = self.p.nc, self.p.reg_max
        levels = []
        for i, (f, st) in enumerate(zip(feats, strides)):
            v = self.p.values[f]
            ch = self.p.values[f].channels
            pre = f"{name}.{i}"
            o = self.value(pre + ".out", 4 * reg_max + nc, v.h, v.w)
            for br, cm, oc in (("cv2", c2, 4 * reg_max), ("cv3", c3, nc)):
                a = self.value(f"{pre}.{br}.0", cm, v.h, v.w)
                b = self.value(f"{pre}.{br}.1", cm, v.h, v.w)
                self.conv(f"{pre}.{br}_0", [Part(f, 0, ch)], (a, 0), cm, 3, 1, precision="fp16")
                self.conv(f"{pre}.{br}_1", [Part(a, 0, cm)], (b, 0), cm, 3, 1, precision="fp16")
                w, bias = self._weights(oc, cm, 1)
                if br == "cv3":
                    w, bias = w * np.float32(self.cls_gain), bias + np.float32(self.cls_bias)
                self.p.commands.append(ConvCmd(f"{pre}.{br}_2", [Part(b, 0, cm)], (o, 0 if br == "cv2" else 4 * reg_max),
                                               cm, oc, 1, 1, False, w, bias, "fp16"))
            levels.append((Part(o, 0, 4 * reg_max), Part(o, 4 * reg_max, nc), float(st)))
        self.p.commands.append(DecodeCmd(name + ".decode", levels, nc, reg_max))

    def _head_logits(self, name: str, h1: str, o: str, c2: int, c3: int, stride: float):
        """cv2[i][2] (box logits from h1[:c2]) and cv3[i][2] (class logits from h1[c2:]) as one 1x1
        conv over all of h1 with block-diagonal weights: one launch instead of two small,
        latency-bound ones; the zero blocks add exact zeros.  Returns the decode level."""
        nc, reg_max = self.p.nc, self.p.reg_max
        w2, b2 = self._weights(4 * reg_max, c2, 1)
        w3, b3 = self._weights(nc, c3, 1)
        oc = self.p.values[o].channels
        wf = np.zeros((oc, c2 + c3, 1, 1), np.float32)
        wf[:4 * reg_max, :c2] = w2
        wf[4 * reg_max:4 * reg_max + nc, c2:] = w3 * np.float32(self.cls_gain)
        bf = np.zeros(oc, np.float32)
        bf[:4 * reg_max], bf[4 * reg_max:4 * reg_max + nc] = b2, b3 + np.float32(self.cls_bias)
        bn = 16
        while bn < min(oc, 256):
            bn *= 2
        self.p.commands.append(ConvCmd(f"{name}.cv23_2", [Part(h1, 0, c2 + c3)], (o, 0), c2 + c3, oc, 1, 1,
                                       False, wf, bf, "fp16", block_n=bn))
        return (Part(o, 0, 4 * reg_max), Part(o, 4 * reg_max, nc), float(stride))

    # ---------------------------------------------------------------- YOLOv11 blocks
    def dwconv(self, name: str, x: Part, out: Tuple[str, int], c: int, s: int = 1, silu: bool = True,
               group: int = 0, group_stride: int = 0, group_off: int = 0) -> DwConvCmd:
        w = self.rng.normal(0.0, self.gain / 3.0, (c, 1, 3, 3)).astype(np.float32)
        b = self.rng.normal(0.0, 0.1, (c,)).astype(np.float32)
        cmd = DwConvCmd(name, x, out, c, s, silu, w, b, group, group_stride, group_off)
        self.p.commands.append(cmd)
        return cmd

    def bottleneck(self, name: str, x: Part, out: Tuple[str, int], c: int, e: float, shortcut: bool) -> None:
        """Bottleneck(c, c, shortcut, k=(3, 3), e): 3x3 c -> c*e, 3x3 c*e -> c, plus x when shortcut."""
        h, w = self.spatial(x.value)
        c_ = int(c * e)
        t = self.value(name + ".t", c_, h, w)
        self.conv(name + ".cv1", [x], (t, 0), c_, 3, 1)
        self.conv(name + ".cv2", [Part(t, 0, c_)], out, c, 3, 1, residual=(x.value, x.coff) if shortcut else None)

    def c3k(self, name: str, x: Part, out: Tuple[str, int], c2: int, n: int, shortcut: bool, e: float = 0.5) -> None:
        """C3k (C3 with k=3 bottlenecks of e=1): cv3(cat(m(cv1(x)), cv2(x))).  cv1 and cv2 read the
        same input: one 1x1 conv writes both (output channels are independent, so this is exact)."""
        h, w = self.spatial(x.value)
        c_ = int(c2 * e)
        z = self.value(name + ".z", 2 * c_, h, w)
        self.conv(name + ".cv12", [x], (z, 0), 2 * c_, 1, 1)
        cur = Part(z, 0, c_)
        for j in range(n):
            o = self.value(f"{name}.m{j}", c_, h, w)
            self.bottleneck(f"{name}.m{j}", cur, (o, 0), c_, 1.0, shortcut)
            cur = Part(o, 0, c_)
        self.conv(name + ".cv3", [cur, Part(z, c_, c_)], out, c2, 1, 1)

    def c3k2(self, name: str, src: List[Part], c2: int, n: int, c3k: bool, e: float = 0.5,
             shortcut: bool = True) -> str:
        """C3k2: the C2f layout (cv1 -> split -> n blocks on the last chunk -> concat -> cv2) with
        Bottleneck(c, c, e=0.5) blocks, or C3k(c, c, n=2) blocks when c3k."""
        h, w = self.spatial(src[0].value)
        h *= src[0].upsample
        w *= src[0].upsample
        c = int(c2 * e)
        y = self.value(name + ".y", (2 + n) * c, h, w)
        self.conv(name + ".cv1", src, (y, 0), 2 * c, 1, 1)
        for i in range(n):
            x = Part(y, (1 + i) * c, c)
            if c3k:
                self.c3k(f"{name}.m{i}", x, (y, (2 + i) * c), c, 2, shortcut)
            else:
                self.bottleneck(f"{name}.m{i}", x, (y, (2 + i) * c), c, 0.5, shortcut)
        out = self.value(name, c2, h, w)
        self.conv(name + ".cv2", [Part(y, 0, (2 + n) * c)], (out, 0), c2, 1, 1)
        return out

    def c2psa(self, name: str, src: str, c1: int, n: int, e: float = 0.5) -> str:
        """C2PSA: cv1 -> split (a, b) -> n PSABlocks on b -> cv2(cat(a, b)).  PSABlock:
        b += proj(attention(qkv(b)) + pe(v)); b += ffn(b), with qkv / proj / ffn on the W8A8 path
        and the attention core and the depthwise pe in fp16 (num_heads = c / 64, key_dim 32)."""
        h, w = self.spatial(src)
        c = int(c1 * e)
        heads, hd = c // 64, 64
        kd = hd // 2
        y = self.value(name + ".y", 2 * c, h, w)
        self.conv(name + ".cv1", [Part(src, 0, c1)], (y, 0), 2 * c, 1, 1)
        cur = Part(y, c, c)
        for i in range(n):
            pre = f"{name}.m{i}"
            qkv = self.value(pre + ".qkv", heads * (2 * kd + hd), h, w)
            self.conv(pre + ".attn.qkv", [cur], (qkv, 0), heads * (2 * kd + hd), 1, 1, silu=False)
            pe = self.value(pre + ".pe", c, h, w)
            self.dwconv(pre + ".attn.pe", Part(qkv, 0, heads * (2 * kd + hd)), (pe, 0), c, silu=False,
                        group=hd, group_stride=2 * kd + hd, group_off=2 * kd)
            xa = self.value(pre + ".xa", c, h, w)
            self.p.commands.append(PsaAttnCmd(pre + ".attn", Part(qkv, 0, heads * (2 * kd + hd)), Part(pe, 0, c),
                                              (xa, 0), heads, kd, hd))
            x1 = self.value(pre + ".x1", c, h, w)
            self.conv(pre + ".attn.proj", [Part(xa, 0, c)], (x1, 0), c, 1, 1, silu=False,
                      residual=(cur.value, cur.coff))
            f = self.value(pre + ".f", 2 * c, h, w)
            self.conv(pre + ".ffn0", [Part(x1, 0, c)], (f, 0), 2 * c, 1, 1)
            x2 = self.value(pre, c, h, w)
            self.conv(pre + ".ffn1", [Part(f, 0, 2 * c)], (x2, 0), c, 1, 1, silu=False, residual=(x1, 0))
            cur = Part(x2, 0, c)
        out = self.value(name, c1, h, w)
        self.conv(name + ".cv2", [Part(y, 0, c), cur], (out, 0), c1, 1, 1)
        return out

    def detect_v11(self, name: str, feats: List[str], strides: List[float]):
        """YOLOv11 Detect: box branch 3x3, 3x3, 1x1; class branch DWConv 3x3 + 1x1, DWConv 3x3 + 1x1,
        1x1 (all fp16), the final 1x1s fused as in the v8 head."""
        nc, reg_max = self.p.nc, self.p.reg_max
        chs = [self.p.values[f].channels for f in feats]
        c2 = max(16, chs[0] // 4, reg_max * 4)
        c3 = max(chs[0], min(nc, 100))
        levels = []
        for i, (f, st) in enumerate(zip(feats, strides)):
            v = self.p.values[f]
            pre = f"{name}.{i}"
            hb = self.value(pre + ".b0", c2, v.h, v.w)
            h1 = self.value(pre + ".h1", c2 + c3, v.h, v.w)
            o = self.value(pre + ".out", _make_divisible(4 * reg_max + nc, 8), v.h, v.w)
            self.conv(pre + ".cv2_0", [Part(f, 0, chs[i])], (hb, 0), c2, 3, 1, precision="fp16")
            self.conv(pre + ".cv2_1", [Part(hb, 0, c2)], (h1, 0), c2, 3, 1, precision="fp16")
            d0 = self.value(pre + ".d0", chs[i], v.h, v.w)
            self.dwconv(pre + ".cv3_0dw", Part(f, 0, chs[i]), (d0, 0), chs[i])
            e0 = self.value(pre + ".e0", c3, v.h, v.w)
            self.conv(pre + ".cv3_0pw", [Part(d0, 0, chs[i])], (e0, 0), c3, 1, 1, precision="fp16")
            d1 = self.value(pre + ".d1", c3, v.h, v.w)
            self.dwconv(pre + ".cv3_1dw", Part(e0, 0, c3), (d1, 0), c3)
            self.conv(pre + ".cv3_1pw", [Part(d1, 0, c3)], (h1, c2), c3, 1, 1, precision="fp16")
            levels.append(self._head_logits(pre, h1, o, c2, c3, st))
        self.p.commands.append(DecodeCmd(name + ".decode", levels, nc, reg_max))


def build_yolov8(width: float = 0.25, depth: float = 0.33, nc: int = 4, imgsz: int = 320, seed: int = 0,
                 max_channels: int = 1024, name: Optional[str] = None, gain: float = 1.0,
                 cls_gain: float = 1.0, cls_bias: float = 0.0, fused_head: bool = True,
                 v11_head: bool = False) -> YoloProgram:
    """YOLOv8 command stream (n: width 0.25 depth 0.33; s: width 0.5 depth 0.33).

    ``gain`` scales the random weights' standard deviation (1.0: N(0, 1/sqrt(fan_in)), under which
    activations shrink through the SiLU layers); ``cls_gain`` scales the class-logit weights and
    ``cls_bias`` is added to the class-logit biases, which spreads the class scores and moves them
    away from 0.5 so that only some anchors pass a confidence threshold.  ``fused_head=False`` keeps
    the Detect head's box and class branches as separate convs (the model's own form, as an ONNX
    export has it) instead of this backend's merged launches; ``v11_head=True`` puts the YOLOv11 Detect
    head (depthwise class branch) on the YOLOv8 backbone."""
    def ch(c):
        return _make_divisible(min(c, max_channels) * width, 8)

    def dep(n):
        return max(round(n * depth), 1) if n > 1 else n

    b = _Builder(name or f"yolov8_w{width}_d{depth}_{imgsz}", imgsz, nc, seed, gain=gain, cls_gain=cls_gain,
                 cls_bias=cls_bias)
    img = [Part("images", 0, 3)]
    x = b.conv_block("l0", img, ch(64), 3, 2, precision="fp16")  # stem: 3 input channels fail IC % 4
    x = b.conv_block("l1", [Part(x, 0, ch(64))], ch(128), 3, 2)
    x = b.c2f("l2", [Part(x, 0, ch(128))], ch(128), dep(3), True)
    x = b.conv_block("l3", [Part(x, 0, ch(128))], ch(256), 3, 2)
    p3 = b.c2f("l4", [Part(x, 0, ch(256))], ch(256), dep(6), True)
    x = b.conv_block("l5", [Part(p3, 0, ch(256))], ch(512), 3, 2)
    p4 = b.c2f("l6", [Part(x, 0, ch(512))], ch(512), dep(6), True)
    x = b.conv_block("l7", [Part(p4, 0, ch(512))], ch(1024), 3, 2)
    x = b.c2f("l8", [Part(x, 0, ch(1024))], ch(1024), dep(3), True)
    p5 = b.sppf("l9", x, ch(1024))
    # neck (PAN): upsample + concat feed the next C2f's cv1 directly
    h12 = b.c2f("l12", [Part(p5, 0, ch(1024), 2), Part(p4, 0, ch(512))], ch(512), dep(3), False)
    h15 = b.c2f("l15", [Part(h12, 0, ch(512), 2), Part(p3, 0, ch(256))], ch(256), dep(3), False)
    x = b.conv_block("l16", [Part(h15, 0, ch(256))], ch(256), 3, 2)
    h18 = b.c2f("l18", [Part(x, 0, ch(256)), Part(h12, 0, ch(512))], ch(512), dep(3), False)
    x = b.conv_block("l19", [Part(h18, 0, ch(512))], ch(512), 3, 2)
    h21 = b.c2f("l21", [Part(x, 0, ch(512)), Part(p5, 0, ch(1024))], ch(1024), dep(3), False)
    if v11_head:
        b.detect_v11("l22", [h15, h18, h21], [8.0, 16.0, 32.0])
    else:
        b.detect("l22", [h15, h18, h21], [8.0, 16.0, 32.0], fused=fused_head)
    return b.p


def build_yolov8n(nc: int = 4, imgsz: int = 320, seed: int = 0, gain: float = 1.0, cls_gain: float = 1.0,
                  cls_bias: float = 0.0) -> YoloProgram:
    """YOLOv8n (width 0.25, depth 0.33), nc=4, 320x320."""
    return build_yolov8(0.25, 0.33, nc, imgsz, seed, name=f"yolov8n_{imgsz}", gain=gain, cls_gain=cls_gain,
                        cls_bias=cls_bias)


def build_yolov8s(nc: int = 80, imgsz: int = 640, seed: int = 0) -> YoloProgram:
    """YOLOv8s (width 0.5, depth 0.33), nc=80, 640x640."""
    return build_yolov8(0.5, 0.33, nc, imgsz, seed, name=f"yolov8s_{imgsz}")


def build_yolov11(width: float = 0.5, depth: float = 0.5, nc: int = 80, imgsz: int = 320, seed: int = 0,
                  max_channels: int = 1024, name: Optional[str] = None, gain: float = 1.0) -> YoloProgram:
    """YOLOv11 command stream (the public yolo11 definition: C3k2 blocks, SPPF, C2PSA, DWConv
    class branch in the head; s: width 0.5 depth 0.5).  C3k2 uses C3k blocks in layers 6, 8 and
    22, as the definition asks for scale s."""
    def ch(c):
        return _make_divisible(min(c, max_channels) * width, 8)

    def dep(n):
        return max(round(n * depth), 1) if n > 1 else n

    b = _Builder(name or f"yolov11_w{width}_d{depth}_{imgsz}", imgsz, nc, seed, gain=gain)
    img = [Part("images", 0, 3)]
    x = b.conv_block("l0", img, ch(64), 3, 2, precision="fp16")
    x = b.conv_block("l1", [Part(x, 0, ch(64))], ch(128), 3, 2)
    x = b.c3k2("l2", [Part(x, 0, ch(128))], ch(256), dep(2), False, e=0.25)
    x = b.conv_block("l3", [Part(x, 0, ch(256))], ch(256), 3, 2)
    p3 = b.c3k2("l4", [Part(x, 0, ch(256))], ch(512), dep(2), False, e=0.25)
    x = b.conv_block("l5", [Part(p3, 0, ch(512))], ch(512), 3, 2)
    p4 = b.c3k2("l6", [Part(x, 0, ch(512))], ch(512), dep(2), True)
    x = b.conv_block("l7", [Part(p4, 0, ch(512))], ch(1024), 3, 2)
    x = b.c3k2("l8", [Part(x, 0, ch(1024))], ch(1024), dep(2), True)
    x = b.sppf("l9", x, ch(1024))
    p5 = b.c2psa("l10", x, ch(1024), dep(2))
    h13 = b.c3k2("l13", [Part(p5, 0, ch(1024), 2), Part(p4, 0, ch(512))], ch(512), dep(2), False)
    h16 = b.c3k2("l16", [Part(h13, 0, ch(512), 2), Part(p3, 0, ch(512))], ch(256), dep(2), False)
    x = b.conv_block("l17", [Part(h16, 0, ch(256))], ch(256), 3, 2)
    h19 = b.c3k2("l19", [Part(x, 0, ch(256)), Part(h13, 0, ch(512))], ch(512), dep(2), False)
    x = b.conv_block("l20", [Part(h19, 0, ch(512))], ch(512), 3, 2)
    h22 = b.c3k2("l22", [Part(x, 0, ch(512)), Part(p5, 0, ch(1024))], ch(1024), dep(2), True)
    b.detect_v11("l23", [h16, h19, h22], [8.0, 16.0, 32.0])
    return b.p


def build_yolov11s(nc: int = 80, imgsz: int = 320, seed: int = 0) -> YoloProgram:
    """YOLOv11s (width 0.5, depth 0.5), 320x320."""
    return build_yolov11(0.5, 0.5, nc, imgsz, seed, name=f"yolov11s_{imgsz}")


def apply_algo_map(program: YoloProgram, int8: Optional[set] = None, pergroup: Optional[set] = None) -> None:
    """The analogue of ``aexrtc --algo-map`` / ``int8_pergroup`` (engine.py:192-210):
    ``int8`` limits the W8A8 kernels to the named convs (others run fp16),
    ``pergroup`` sets the INT8_PERGROUP flag (pg16 activation scales)."""
    for c in program.commands:
        if not isinstance(c, ConvCmd) or c.precision != "int8":
            continue
        if int8 is not None and c.name not in int8:
            c.precision = "fp16"
        if pergroup is not None and c.name in pergroup:
            c.pg16 = True
