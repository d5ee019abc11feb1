"""CPU oracle of a whole YOLO command stream (TEST INFRASTRUCTURE ONLY).

Runs the command stream built by ``aexrt_b200.yolo`` with the W8A8 restatement
of ``oracle.w8a8`` for the int8 convs and plain fp32 math for the rest, storing
every value in fp16 as the device does.  Used by tests (per-layer parity with
each layer fed the device's own inputs, and whole-model tolerance checks) and
as the timed CPU baseline / ``--impl reference`` arm of ``bench.py``: the
reference's W8A8 path only runs through D3D12, so its arithmetic restated on
the CPU is the reference implementation timed on the host cores.

Ops restated here besides oracle.w8a8:
* SPPF pooling: three cascaded MaxPool2d(5, 1, 2) (reference kind MAXPOOL);
* nearest 2x upsample (RESIZE) and channel concat (CONCAT);
* detect decode: DFL softmax expectation over reg_max bins, distance -> box
  around the anchor centre, class sigmoid; the reference post-processes this
  output0 layout in src/aexrt/yolo.py:92-138;
* YOLOv11's fp16 ops: the depthwise 3x3 conv (a grouped CONV in the reference,
  refused by its int8 guard, native/aexrt_d3d12_runtime.cpp:9404) and the C2PSA
  attention core (MATMUL / SOFTMAX commands in the reference,
  runtime.cpp:17305-17307): softmax(q^T k * key_dim^-0.5) applied to v, plus the
  positional encoding, per head, as the public ultralytics Attention module
  defines it.
"""
from __future__ import annotations

from typing import Dict, Optional

import numpy as np

from . import w8a8 as ow

F32 = np.float32


def _gather(values: Dict[str, np.ndarray], parts) -> np.ndarray:
    xs = []
    for pt in parts:
        v = values[pt.value][:, pt.coff:pt.coff + pt.channels]
        if pt.upsample != 1:
            v = v.repeat(pt.upsample, axis=2).repeat(pt.upsample, axis=3)
        xs.append(v)
    return np.concatenate(xs, axis=1) if len(xs) > 1 else xs[0]


def conv_cmd(c, x: np.ndarray, residual: Optional[np.ndarray]) -> dict:
    """One conv command on NCHW input `x`; returns the oracle intermediates and fp16 output."""
    p = c.k // 2
    if c.precision == "int8":
        return ow.conv_w8a8(x.astype(np.float16), c.weight, c.bias, c.k, c.s, p,
                            mode=ow.SCALE_PG16 if c.pg16 else ow.SCALE_PER_TENSOR, silu=c.silu, residual=residual)
    xf = x.astype(np.float16).astype(F32)
    wf = c.weight.astype(np.float16).astype(F32)
    y = ow.conv_f32(xf, wf, c.bias, c.k, c.s, p)
    if c.silu:
        y = ow.silu_f32(y)
    if residual is not None:
        y = (y + residual.astype(F32)).astype(F32)
    return {"y32": y, "y": y.astype(np.float16)}


def dwconv3x3(c, x: np.ndarray) -> np.ndarray:
    """Depthwise 3x3 conv (pad 1, stride c.s) of NCHW `x` (already gathered per c.in_channel) with
    fp16-rounded operands, fp32 accumulation, optional SiLU; returns fp32."""
    xf = x.astype(np.float16).astype(F32)
    wf = c.weight.astype(np.float16).astype(F32).reshape(c.c, 3, 3)
    n, ch, h, w = xf.shape
    oh, owd = (h - 1) // c.s + 1, (w - 1) // c.s + 1
    pad = np.zeros((n, ch, h + 2, w + 2), F32)
    pad[:, :, 1:1 + h, 1:1 + w] = xf
    y = np.broadcast_to(c.bias.astype(F32).reshape(1, ch, 1, 1), (n, ch, oh, owd)).copy()
    for kh in range(3):
        for kw in range(3):
            tap = pad[:, :, kh:kh + (oh - 1) * c.s + 1:c.s, kw:kw + (owd - 1) * c.s + 1:c.s]
            y = (y + tap * wf[:, kh, kw].reshape(1, ch, 1, 1)).astype(F32)
    if c.silu:
        y = ow.silu_f32(y)
    return y


def psa_attention(c, qkv: np.ndarray, pe: np.ndarray) -> np.ndarray:
    """C2PSA attention core on NCHW fp16 tensors: per image and head, q, k, v are the head's
    consecutive (key_dim, key_dim, head_dim) qkv channels over the N = H*W pixels;
    out = v @ softmax(q^T k * scale)^T + pe, computed in fp32 (returns fp32)."""
    n, _, h, w = qkv.shape
    nh, kd, hd = c.heads, c.key_dim, c.head_dim
    t = qkv.astype(F32).reshape(n, nh, 2 * kd + hd, h * w)
    q, k, v = t[:, :, :kd], t[:, :, kd:2 * kd], t[:, :, 2 * kd:]
    s = np.einsum("bhdi,bhdj->bhij", q, k).astype(F32) * F32(c.scale)
    s = s - s.max(axis=-1, keepdims=True)
    e = np.exp(s).astype(F32)
    a = (e / e.sum(axis=-1, keepdims=True)).astype(F32)
    o = np.einsum("bhcj,bhij->bhci", v, a).astype(F32).reshape(n, nh * hd, h, w)
    return (o + pe.astype(F32)).astype(F32)


def sppf_pool(x: np.ndarray) -> np.ndarray:
    """Three cascaded 5x5 stride-1 max pools with -inf padding, concatenated [m1, m2, m3]."""
    def mp(a):
        n, c, h, w = a.shape
        pad = np.full((n, c, h + 4, w + 4), -np.inf, dtype=F32)
        pad[:, :, 2:2 + h, 2:2 + w] = a
        out = np.full_like(a, -np.inf, dtype=F32)
        for dy in range(5):
            for dx in range(5):
                out = np.maximum(out, pad[:, :, dy:dy + h, dx:dx + w])
        return out

    m1 = mp(x.astype(F32))
    m2 = mp(m1)
    m3 = mp(m2)
    return np.concatenate([m1, m2, m3], axis=1).astype(np.float16)


def decode(levels, values: Dict[str, np.ndarray], nc: int, reg_max: int) -> np.ndarray:
    """[N, 4+nc, anchors]: cx, cy, w, h in input pixels, then class sigmoid."""
    outs = []
    for bp, cp, stride in levels:
        box = values[bp.value][:, bp.coff:bp.coff + bp.channels].astype(F32)
        cls = values[cp.value][:, cp.coff:cp.coff + cp.channels].astype(F32)
        n, _, h, w = box.shape
        b = box.reshape(n, 4, reg_max, h * w)
        e = np.exp(b - b.max(axis=2, keepdims=True))
        dist = (e * np.arange(reg_max, dtype=F32).reshape(1, 1, reg_max, 1)).sum(axis=2) / e.sum(axis=2)
        gy, gx = np.meshgrid(np.arange(h, dtype=F32), np.arange(w, dtype=F32), indexing="ij")
        cx = (gx.reshape(-1) + 0.5)[None]
        cy = (gy.reshape(-1) + 0.5)[None]
        x1, y1 = cx - dist[:, 0], cy - dist[:, 1]
        x2, y2 = cx + dist[:, 2], cy + dist[:, 3]
        xywh = np.stack([(x1 + x2) / 2, (y1 + y2) / 2, x2 - x1, y2 - y1], axis=1) * stride
        prob = 1.0 / (1.0 + np.exp(-cls.reshape(n, nc, h * w)))
        outs.append(np.concatenate([xywh, prob], axis=1))
    return np.concatenate(outs, axis=2).astype(F32)


def run_program(program, images: np.ndarray, keep: bool = False) -> dict:
    """Whole-program oracle forward.  Returns {"output0": ..., "values": {...} if keep}."""
    values: Dict[str, np.ndarray] = {"images": images.astype(F32)}
    n = images.shape[0]
    for name, v in program.values.items():
        if name != "images":
            values[name] = np.zeros((n, v.channels, v.h, v.w), np.float16)
    out0 = None
    from aexrt_b200.yolo import ConvCmd, DecodeCmd, DwConvCmd, PsaAttnCmd, SppfCmd  # the program's command classes

    for c in program.commands:
        if isinstance(c, ConvCmd):
            x = _gather(values, c.inputs)
            res = None
            if c.residual is not None:
                res = values[c.residual[0]][:, c.residual[1]:c.residual[1] + c.oc]
            r = conv_cmd(c, x, res)
            values[c.out[0]][:, c.out[1]:c.out[1] + c.oc] = r["y"]
        elif isinstance(c, SppfCmd):
            x = values[c.x.value][:, c.x.coff:c.x.coff + c.x.channels]
            values[c.out[0]][:, c.out[1]:c.out[1] + 3 * c.x.channels] = sppf_pool(x)
        elif isinstance(c, DwConvCmd):
            src = values[c.x.value]
            idx = [c.in_channel(k) for k in range(c.c)]
            values[c.out[0]][:, c.out[1]:c.out[1] + c.c] = dwconv3x3(c, src[:, idx]).astype(np.float16)
        elif isinstance(c, PsaAttnCmd):
            qkv = values[c.qkv.value][:, c.qkv.coff:c.qkv.coff + c.qkv.channels]
            pe = values[c.pe.value][:, c.pe.coff:c.pe.coff + c.pe.channels]
            values[c.out[0]][:, c.out[1]:c.out[1] + c.heads * c.head_dim] = \
                psa_attention(c, qkv, pe).astype(np.float16)
        elif isinstance(c, DecodeCmd):
            out0 = decode(c.levels, values, c.nc, c.reg_max)
    res = {"output0": out0}
    if keep:
        res["values"] = values
    return res
