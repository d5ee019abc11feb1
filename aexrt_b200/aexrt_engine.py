"""Reader for engines compiled by the reference's own compiler (``aexrtc build`` /
``build_aexrt_engine``), and a runner for their W8A8 conv path on the B200 kernels.

Container format (docs/AEXRT_ENGINE.md:54-104, written by src/aexrt/engine.py:3952 and the
section encoders at :2583-2700; parsed by the reference runtime's ``parse_aexrt_engine``,
native/aexrt_d3d12_runtime.cpp:17560): a 64-byte header ``AEXRTENG``, a table of 32-byte
``<IIQQII>`` section entries, and section payloads each with its own CRC32.  :func:`load_engine`
checks what the reference's loader checks before it trusts an engine (magic, version, sizes,
section bounds, CRC32 of every section, the nine base sections present once, the kernel plan
repeating each command's kind, planned kernel and precision) and fails closed with a message
otherwise.

:class:`EngineRunner` lowers the command stream onto this backend:

* CONV / CONV_SILU with planned kernel 51 / 52 / 53 become W8A8 plans built from the engine's
  own layout-8 packed weights (int8 codes + per-output-channel scale, no re-quantization) and
  its bias constants, with the INT8_PERGROUP plan flag selecting pg16 scales;
* other CONV / CONV_SILU commands become fp16 plans from the raw weight constants;
* CONCAT along channels and nearest 2x RESIZE are read in place by the consumers (the
  quantizer and fp16 packer take channel slices and upsampled sources);
* ALIAS, VIEW and a single-input CONCAT are accepted only as a reshape of the graph output.

Any other command kind (BINARY, SLICE, MAXPOOL, MATMUL, ...) is refused: those belong to the
reference's generic fp16/fp32 path, not the W8A8 path this backend replaces.  Activations are
fp16 NHWC between commands; the graph input is rounded to fp16 on upload (the rule of this
backend's image stem), so fp16-representable inputs give the reference's integer codes exactly.
"""
from __future__ import annotations

import struct
import zlib
from dataclasses import dataclass
from typing import Dict, List, Optional, Tuple

import numpy as np

MAGIC = b"AEXRTENG"
HEADER_SIZE = 64
TOC_ENTRY = 32
BASE_SECTIONS = tuple(range(1, 10))
SECTION_NAMES = {1: "manifest", 2: "values", 3: "commands", 4: "raw constants", 5: "kernel plan",
                 6: "packed weights", 7: "memory plan", 8: "fusion plan", 9: "pipeline cache",
                 10: "physical dispatch plan", 11: "arena barrier plan", 12: "parallel plan"}
# command kinds and flags: src/aexrt/engine.py:85-118
KIND = {"CONV": 1, "CONV_SILU": 2, "CONCAT_CONV1X1": 3, "VIEW": 4, "ALIAS": 5, "SLICE": 6, "CONCAT": 7,
        "RESIZE": 8, "MAXPOOL": 9, "UNARY": 10, "BINARY": 11, "MATMUL": 12, "TRANSPOSE": 13, "SOFTMAX": 14}
KIND_NAME = {v: k for k, v in KIND.items()}
PLAN_FLAG_INT8_PERGROUP = 1 << 4
PACKED_LAYOUT_CONV_INT8 = 8
INT8_KERNELS = (51, 52, 53)
PRECISION_FP32, PRECISION_FP16 = 1, 2


class EngineError(ValueError):
    """The engine is malformed or uses something this backend does not run (fail closed)."""


@dataclass
class Command:
    kind: int
    output: int
    inputs: Tuple[int, ...]
    params: Tuple[int, ...]
    planned_kernel: int
    precision: int
    flags: int = 0            # from the kernel plan
    packed_value: int = 0xFFFFFFFF

    @property
    def name(self) -> str:
        return KIND_NAME.get(self.kind, str(self.kind))


@dataclass
class Engine:
    manifest: Dict[str, object]
    values: List[Dict[str, object]]
    commands: List[Command]
    constants: Dict[int, np.ndarray]                   # value id -> float32 array (fp16 payloads widened)
    constant_dtype: Dict[int, int]                      # value id -> 1 fp32 / 2 fp16
    packed: Dict[int, Dict[str, object]]                # value id -> layout, in/out channels, payload bytes
    sections: Dict[int, Tuple[int, int, int, int]]      # id -> (flags, offset, size, crc32)

    def shape(self, value_id: int) -> Tuple[int, int, int, int]:
        return tuple(self.values[value_id]["shape"])  # type: ignore[return-value]


def _u(fmt: str, buf: bytes, off: int, what: str):
    try:
        return struct.unpack_from(fmt, buf, off)
    except struct.error as e:
        raise EngineError(f"{what}: truncated ({e})") from None


def load_engine(src) -> Engine:
    """Parses and validates an ``.aexrt`` engine (path or bytes)."""
    data = bytes(src) if isinstance(src, (bytes, bytearray, memoryview)) else open(src, "rb").read()
    magic, version, hsize, count, flags, fsize, toc, toc_size, reserved = _u("<8sIIIIQQQ16s", data, 0, "header")
    if magic != MAGIC:
        raise EngineError("not an .aexrt engine (bad magic)")
    if version != 1 or hsize != HEADER_SIZE:
        raise EngineError(f"unsupported engine version {version} / header size {hsize}")
    if not flags & 1:
        raise EngineError("engine header flag bit 0 is not set")
    if fsize != len(data):
        raise EngineError(f"file size {len(data)} does not match the header's {fsize}")
    if toc != HEADER_SIZE or toc_size != count * TOC_ENTRY or toc + toc_size > len(data):
        raise EngineError("bad section table")
    if any(reserved):
        raise EngineError("reserved header bytes are not zero")
    if not len(BASE_SECTIONS) <= count <= max(SECTION_NAMES):
        raise EngineError(f"section count {count} outside {len(BASE_SECTIONS)}..{max(SECTION_NAMES)}")
    sections: Dict[int, Tuple[int, int, int, int]] = {}
    for i in range(count):
        sid, sflags, off, size, crc, rsv = _u("<IIQQII", data, toc + TOC_ENTRY * i, "section table")
        if sid not in SECTION_NAMES:
            raise EngineError(f"unknown section id {sid}")
        if rsv != 0:
            raise EngineError(f"section {sid}: reserved table field is not zero")
        if sid in sections:
            raise EngineError(f"duplicate section {sid}")
        if off < toc + toc_size or off + size > len(data):
            raise EngineError(f"section {sid} lies outside the file")
        if zlib.crc32(data[off:off + size]) & 0xFFFFFFFF != crc:
            raise EngineError(f"section {sid} ({SECTION_NAMES.get(sid, '?')}) fails its CRC32")
        sections[sid] = (sflags, off, size, crc)
    missing = [s for s in BASE_SECTIONS if s not in sections]
    if missing:
        raise EngineError(f"missing sections {missing}")
    if 11 in sections and 10 not in sections:
        raise EngineError("section 11 (arena barrier plan) requires section 10 (physical dispatch plan)")
    body = lambda sid: data[sections[sid][1]:sections[sid][1] + sections[sid][2]]  # noqa: E731

    m = body(1)
    if len(m) != 124:
        raise EngineError("manifest must be 124 bytes")
    u = _u("<17I", m, 0, "manifest")
    input_elements, arena_nbytes = _u("<QQ", m, 68, "manifest")
    conf, iou = _u("<ff", m, 84, "manifest")
    if u[0] != 1:
        raise EngineError(f"unsupported manifest version {u[0]}")
    # the manifest rules of the reference loader (parse_aexrt_engine, runtime.cpp:17613-17618)
    if (u[1] != 1 or u[2] not in (1, 2) or u[3] != 2 or u[4] not in (1, 2) or u[5] > 1 or 0 in (u[6], u[7], u[8])
            or u[12] == 0 or u[14] == 0 or u[15] >= u[12] or u[16] >= u[12] or input_elements == 0
            or arena_nbytes == 0):
        raise EngineError("manifest fields out of range (target, precision, mode, layout, counts or value ids)")
    manifest = dict(runtime_target=u[1], precision=u[2], mode=u[3], output_layout=u[4], objectness=u[5],
                    channels=u[6], anchors=u[7], classes=u[8], max_candidates=u[9], max_detections=u[10],
                    nodes=u[11], value_count=u[12], constant_count=u[13], command_count=u[14],
                    input_value=u[15], output_value=u[16], input_elements=input_elements,
                    arena_nbytes=arena_nbytes, conf_threshold=conf, iou_threshold=iou,
                    source_sha256=m[92:124].hex())

    v = body(2)
    nval, _ = _u("<II", v, 0, "values")
    values = []
    for i in range(nval):
        vid, vflags, elems, s0, s1, s2, s3, aoff, anb = _u("<IIQ4IQQ", v, 8 + 48 * i, "values")
        if vid != i:
            raise EngineError("value records are not dense and ordered by id")
        values.append(dict(id=vid, flags=vflags, elements=elems, shape=(s0, s1, s2, s3), arena_offset=aoff,
                           arena_nbytes=anb))
    if nval != manifest["value_count"]:
        raise EngineError("value count differs from the manifest")

    c = body(3)
    ncmd, _ = _u("<II", c, 0, "commands")
    commands = []
    p = 8
    for _i in range(ncmd):
        kind, out, nin, npar, pk, prec = _u("<6I", c, p, "commands")
        p += 24
        ins = _u(f"<{nin}I", c, p, "command inputs")
        p += 4 * nin
        pars = _u(f"<{npar}I", c, p, "command params")
        p += 4 * npar
        if kind not in KIND_NAME:
            raise EngineError(f"unknown command kind {kind}")
        if out >= nval or any(x >= nval for x in ins):
            raise EngineError("command references a value outside the value table")
        commands.append(Command(kind, out, tuple(ins), tuple(pars), pk, prec))
    if ncmd != manifest["command_count"]:
        raise EngineError("command count differs from the manifest")

    k = body(5)
    nplan, plan_version = _u("<II", k, 0, "kernel plan")
    if nplan != ncmd or plan_version != 1:
        raise EngineError("kernel plan does not cover the command stream")
    for i in range(nplan):
        idx, kind, pk, prec, packed_value, pflags = _u("<6I", k, 8 + 24 * i, "kernel plan")
        cmd = commands[i]
        if idx != i or kind != cmd.kind or pk != cmd.planned_kernel or prec != cmd.precision:
            raise EngineError(f"kernel plan record {i} disagrees with its command")
        if not pflags & 1:
            raise EngineError(f"kernel plan record {i} is not authoritative")
        cmd.flags, cmd.packed_value = pflags, packed_value

    r = body(4)
    nconst, _ = _u("<II", r, 0, "raw constants")
    constants, cdtype = {}, {}
    for i in range(nconst):
        vid, dt, elems, off, nbytes = _u("<IIQQQ", r, 8 + 32 * i, "raw constants")
        width = {PRECISION_FP32: 4, PRECISION_FP16: 2}.get(dt)
        if width is None or nbytes != elems * width or off + nbytes > len(r) or vid >= nval:
            raise EngineError(f"bad constant record for value {vid}")
        arr = np.frombuffer(r, dtype="<f4" if dt == PRECISION_FP32 else "<f2", count=elems, offset=off)
        constants[vid] = arr.astype(np.float32)
        cdtype[vid] = dt

    w = body(6)
    npk, _ = _u("<II", w, 0, "packed weights")
    packed = {}
    for i in range(npk):
        vid, layout, ic, oc, elems, off, nbytes = _u("<4IQQQ", w, 8 + 40 * i, "packed weights")
        if off + nbytes > len(w):
            raise EngineError(f"packed weights of value {vid} lie outside their section")
        packed[vid] = dict(layout=layout, in_channels=ic, out_channels=oc, elements=elems,
                           data=bytes(w[off:off + nbytes]))
    return Engine(manifest, values, commands, constants, cdtype, packed, sections)


def conv_desc(cmd: Command) -> Tuple[int, ...]:
    """The command's AexrtConv2DDesc fields (native/aexrt.h:98-115): its first 16 params."""
    if cmd.kind not in (KIND["CONV"], KIND["CONV_SILU"]) or len(cmd.params) < 16:
        raise EngineError(f"command {cmd.name} carries no conv descriptor")
    return tuple(cmd.params[:16])


def int8_weights(engine: Engine, cmd: Command) -> Tuple[np.ndarray, np.ndarray]:
    """(codes [oc][ic*kk] int8, scale [oc] fp32) of a W8A8 conv from its layout-8 packed payload
    (``[oc*ic*kk int8 in [oc][ic][kh][kw] order][oc fp32 scale]``, src/aexrt/engine.py:2458)."""
    _, ic, _, _, oc, _, _, kh, kw = conv_desc(cmd)[:9]
    rec = engine.packed.get(cmd.inputs[1])
    if rec is None or cmd.packed_value != cmd.inputs[1]:
        raise EngineError(f"int8 conv writing value {cmd.output} has no packed weights")
    kk = kh * kw
    if rec["layout"] != PACKED_LAYOUT_CONV_INT8 or rec["in_channels"] != ic or rec["out_channels"] != oc:
        raise EngineError(f"packed weights of value {cmd.inputs[1]} are not layout 8 for {oc}x{ic}x{kh}x{kw}")
    data = rec["data"]
    if len(data) != oc * ic * kk + 4 * oc:
        raise EngineError(f"layout-8 payload of value {cmd.inputs[1]} has {len(data)} bytes")
    codes = np.frombuffer(data, dtype=np.int8, count=oc * ic * kk).reshape(oc, ic * kk).copy()
    scale = np.frombuffer(data, dtype="<f4", count=oc, offset=oc * ic * kk).astype(np.float32)
    return codes, scale


@dataclass
class _Part:
    value: int      # a value with its own buffer
    coff: int
    channels: int
    upsample: int = 1


class EngineRunner:
    """Runs an engine's conv-path command stream on the current CUDA device (eager launches, or one
    CUDA graph after :meth:`capture`)."""

    def __init__(self, engine: Engine, device=None):
        import torch

        from . import _native, ops

        self.torch, self.ops, self.lib = torch, ops, _native.load()
        self.engine = engine
        self.device = torch.device("cuda", torch.cuda.current_device() if device is None else device)
        mf = engine.manifest
        self.input_id, self.output_id = int(mf["input_value"]), int(mf["output_value"])
        n, ci, hi, wi = engine.shape(self.input_id)
        self.batch = n
        self.parts: Dict[int, List[_Part]] = {self.input_id: [_Part(self.input_id, 0, ci)]}
        self.bufs: Dict[int, "torch.Tensor"] = {
            self.input_id: torch.zeros((n, ci, hi, wi), dtype=torch.float16, device=self.device)}  # NCHW
        self.steps: List[tuple] = []
        self.out_reshape: Optional[int] = None
        for i, cmd in enumerate(engine.commands):
            if cmd.kind in (KIND["CONV"], KIND["CONV_SILU"]):
                self._add_conv(cmd)
            elif cmd.kind == KIND["CONCAT"] and len(cmd.inputs) > 1:
                self._add_concat(cmd)
            elif cmd.kind == KIND["RESIZE"]:
                self._add_resize(cmd)
            elif cmd.kind in (KIND["ALIAS"], KIND["VIEW"], KIND["CONCAT"]) and cmd.output == self.output_id \
                    and len(cmd.inputs) == 1 and i == len(engine.commands) - 1:
                self.out_reshape = cmd.inputs[0]
            else:
                raise EngineError(f"command {i} ({cmd.name}) is outside the conv path this backend runs")
        # amax slots: one per (image, 16 channels) of every buffer an int8 conv reads
        int8_in = {p.value for st in self.steps if st[1].planned_kernel in INT8_KERNELS for p in st[3]}
        self.amax: Dict[int, "torch.Tensor"] = {}
        for vid in int8_in:
            groups = (self.bufs[vid].shape[1 if vid == self.input_id else -1] + 15) // 16
            self.amax[vid] = torch.zeros((n, groups), dtype=torch.int32, device=self.device)
        self.graph = None

    # ------------------------------------------------------------------ lowering
    def _parts(self, vid: int) -> List[_Part]:
        if vid not in self.parts:
            raise EngineError(f"value {vid} is read before any supported command produced it")
        return self.parts[vid]

    def _add_conv(self, cmd: Command):
        torch, ops = self.torch, self.ops
        e = self.engine
        n, ic, ih, iw, oc, oh, ow, kh, kw, sh, sw, pt, pl, dh, dw, groups = conv_desc(cmd)
        if kh != kw or sh != sw or dh != 1 or dw != 1 or groups != 1 or pt != kh // 2 or pl != kw // 2:
            raise EngineError(f"conv writing value {cmd.output}: only square kernels, pad k//2, no dilation or groups")
        silu = cmd.kind == KIND["CONV_SILU"]
        bias = e.constants.get(cmd.inputs[2])
        if bias is None or bias.size != oc:
            raise EngineError(f"conv writing value {cmd.output}: bias constant missing")
        parts = self._parts(cmd.inputs[0])
        if sum(p.channels for p in parts) != ic:
            raise EngineError(f"conv writing value {cmd.output}: input has the wrong channel count")
        if cmd.planned_kernel in INT8_KERNELS:
            if ops.kernel_id_for(kh, sh) != cmd.planned_kernel:
                raise EngineError(f"conv writing value {cmd.output}: planned kernel {cmd.planned_kernel} does not fit "
                                  f"a {kh}x{kw} stride-{sh} conv")
            codes, scale = int8_weights(e, cmd)
            plan = ops.ConvPlan.int8(n, ic, ih, iw, oc, kh, sh, codes, scale, bias, silu=silu,
                                     pg16=bool(cmd.flags & PLAN_FLAG_INT8_PERGROUP))
            shape = ops.packed_act_shape(n, ic, ih, iw, sh)
            scratch = (torch.empty(shape, dtype=torch.int8, device=self.device),
                       torch.empty((n, 1 + shape[1]), dtype=torch.float32, device=self.device))
        else:
            wt = e.constants.get(cmd.inputs[1])
            if wt is None or wt.size != oc * ic * kh * kw:
                raise EngineError(f"conv writing value {cmd.output}: weight constant missing")
            plan = ops.ConvPlan.fp16(n, ic, ih, iw, oc, kh, sh, wt.reshape(oc, ic, kh, kw), bias, silu=silu)
            hp, wp = ih + (ih & 1 if sh == 2 else 0), iw + (iw & 1 if sh == 2 else 0)
            scratch = (torch.empty((n, (ic + 7) // 8, hp, wp, 8), dtype=torch.float16, device=self.device),)
        self.bufs[cmd.output] = torch.zeros((n, oh, ow, oc), dtype=torch.float16, device=self.device)
        self.parts[cmd.output] = [_Part(cmd.output, 0, oc)]
        self.steps.append(("conv", cmd, plan, parts, scratch, (ih, iw)))

    def _add_concat(self, cmd: Command):
        numel, rank, axis = cmd.params[:3]
        if axis != 1 + (0 if rank == 4 else 4 - rank) or rank != 4:
            raise EngineError(f"CONCAT writing value {cmd.output}: only channel concat of NCHW tensors")
        parts: List[_Part] = []
        for vid in cmd.inputs:
            parts.extend(self._parts(vid))
        self.parts[cmd.output] = parts

    def _add_resize(self, cmd: Command):
        n, c, ih, iw, oh, ow = cmd.params[:6]
        src = self._parts(cmd.inputs[0])
        if oh != 2 * ih or ow != 2 * iw or any(p.upsample != 1 for p in src):
            raise EngineError(f"RESIZE writing value {cmd.output}: only nearest 2x")
        self.parts[cmd.output] = [_Part(p.value, p.coff, p.channels, 2) for p in src]

    # ------------------------------------------------------------------ run
    def _sources(self, parts: List[_Part], with_amax: bool):
        from ._native import AexrtB200ActSource

        srcs = (AexrtB200ActSource * len(parts))()
        for i, p in enumerate(parts):
            buf = self.bufs[p.value]
            s = srcs[i]
            s.ptr = buf.data_ptr()
            if p.value == self.input_id:
                s.layout, s.ldc, s.src_h, s.src_w = self.ops.LAYOUT_NCHW_F16, buf.shape[1], buf.shape[2], buf.shape[3]
            else:
                s.layout, s.ldc, s.src_h, s.src_w = self.ops.LAYOUT_NHWC_F16, buf.shape[-1], buf.shape[1], buf.shape[2]
            s.coff, s.channels, s.upsample = p.coff, p.channels, p.upsample
            if with_amax:
                am = self.amax[p.value]
                s.amax_groups, s.amax_stride, s.amax_goff = am.data_ptr(), am.shape[1], p.coff // 16
        return srcs

    def launch(self, stream: int) -> None:
        from ._native import check

        lib, ops, n = self.lib, self.ops, self.batch
        if self.input_id in self.amax:
            x = self.bufs[self.input_id]
            check(lib.aexrt_b200_act_amax_f16(x.data_ptr(), n, x.shape[1], x.shape[2], x.shape[3],
                                              ops.LAYOUT_NCHW_F16, x.shape[1], 0, self.amax[self.input_id].data_ptr(),
                                              self.amax[self.input_id].shape[1], 0, 1, stream), "input amax")
        for vid, am in self.amax.items():
            if vid != self.input_id:
                check(lib.aexrt_b200_zero(am.data_ptr(), am.numel() * 4, stream), "zero amax")
        for _, cmd, plan, parts, scratch, (ih, iw) in self.steps:
            out = self.bufs[cmd.output]
            amax_out = self.amax.get(cmd.output)
            s = plan.desc.stride_h
            if plan.info.kernel_id in INT8_KERNELS:
                q, rec = scratch
                srcs = self._sources(parts, True)
                pg16 = 1 if plan.info.flags & PLAN_FLAG_INT8_PERGROUP else 0
                check(lib.aexrt_b200_act_quantize_concat(srcs, len(srcs), n, ih, iw, pg16, s, q.data_ptr(),
                                                         rec.data_ptr(), stream), "quantize")
                plan.run(q, rec, out=out, amax_out=amax_out, stream=stream)
            else:
                (x8,) = scratch
                srcs = self._sources(parts, False)
                check(lib.aexrt_b200_pack_f16_concat(srcs, len(srcs), n, ih, iw, s, x8.data_ptr(), stream), "pack")
                plan.run(x8, out=out, amax_out=amax_out, stream=stream)

    def capture(self) -> None:
        torch = self.torch
        s = torch.cuda.Stream(device=self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(s):
            self.launch(s.cuda_stream)
        torch.cuda.synchronize(self.device)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=s):
            self.launch(s.cuda_stream)
        torch.cuda.synchronize(self.device)

    def run(self, x) -> np.ndarray:
        """One inference on `x` (the graph input, NCHW; rounded to fp16 on upload); returns the graph
        output as float32 in its NCHW shape (the reference's InferenceSession.run contract)."""
        torch = self.torch
        xt = torch.as_tensor(np.asarray(x, dtype=np.float32)).reshape(self.bufs[self.input_id].shape)
        self.bufs[self.input_id].copy_(xt.to(self.device).half())
        if self.graph is not None:
            self.graph.replay()
        else:
            self.launch(torch.cuda.current_stream(self.device).cuda_stream)
        src = self.out_reshape if self.out_reshape is not None else self.output_id
        parts = self._parts(src)
        host = [self.bufs[p.value].float().cpu().numpy() for p in parts]  # NHWC, read back after the run
        chans = []
        for p, h in zip(parts, host):
            y = h[..., p.coff:p.coff + p.channels].transpose(0, 3, 1, 2)
            if p.upsample != 1:
                y = y.repeat(p.upsample, axis=2).repeat(p.upsample, axis=3)
            chans.append(y)
        y = np.concatenate(chans, axis=1) if len(chans) > 1 else chans[0]
        shape = self.engine.shape(self.output_id)
        return np.ascontiguousarray(y).reshape(shape)

    def status(self) -> int:
        st = 0
        for step in self.steps:
            st |= step[2].status()
        return st
