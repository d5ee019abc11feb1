"""Compile a YOLO command stream into device plans and replay it as a CUDA graph.

This is the B200 counterpart of the reference runtime's prepared physical
replay (``ensure_prepared_yolo_replay`` / ``record_prepared_physical_stream``,
native/aexrt_d3d12_runtime.cpp:28758-29010, replayed per frame at :29732-29940):
the command list is lowered once into C-ABI launches on one stream, recorded
into one CUDA graph per batch size, and replayed per batch.

Memory plan: every value of the program is one fp16 NHWC buffer (the reference
keeps fp16 "activation islands" in arena pages, memory_v2.py:202); producers
write their channel slice of the consumer-facing buffer, so CONCAT and C2f
split/chunk cost nothing.  Every value also owns one amax slot per (image,
16-channel group) that its producers max into (epilogue amax), and that the
consumers' quantizers read.  All amax slots live in one arena cleared at the
start of each replay.

Kernel plan: int8 convs become W8A8 plans with the reference's kernel ids
(51 1x1, 52 3x3 s1, 53 3x3 s2) and INT8_PERGROUP flag; the rest (stem with 3
input channels, detect head) become fp16 plans.

Post-process: with an :class:`NmsConfig`, the replay ends with the GPU
confidence filter + NMS + top-k (the reference's record_yolo_decode_nms_topk,
runtime.cpp:27104-27219), and :meth:`CompiledYolo.detections` holds each
image's AexrtYoloDetection rows and count, the output of ``aexrt_yolo_run``.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, List, Optional

import numpy as np

from . import _native, ops
from ._native import AexrtB200ActSource, AexrtB200DecodeLevel, check
from .yolo import ConvCmd, DecodeCmd, DwConvCmd, Part, PsaAttnCmd, SppfCmd, YoloProgram


def _torch():
    import torch

    return torch


@dataclass
class NmsConfig:
    """Post-process settings; the defaults are the reference model's (runtime.cpp:551-561)."""

    conf: float = 0.25
    iou: float = 0.45
    max_candidates: int = 512
    max_detections: int = 100
    mode: int = ops.NMS_MARK  # the reference GPU path's rule; ops.NMS_GREEDY = yolo_postprocess's
    ctas_per_image: int = 0   # 0 automatic (8 for small batches), else 1, 2, 4 or 8


# A tuned tile map's bit for "this int8 conv quantizes its fp16 sources itself" (above the plan's
# tuning bits, which end at bit 30; stripped before the plan is created)
TILE_QUANT_ON_LOAD = 1 << 31


def ql_eligible(c: ConvCmd) -> bool:
    """Whether an int8 conv can quantize on load: every input part fits the rules of
    conv_w8a8_sources; SiLU convs only (the linear ones, with or without a residual, have no instance
    of every tile)."""
    return c.silu and all(
        pt.value != "images" and pt.coff % 16 == 0 and pt.channels >= 16
        and (pt.channels % 16 == 0 or i == len(c.inputs) - 1) and (pt.upsample == 1 or c.s == 1)
        for i, pt in enumerate(c.inputs)) and len(c.inputs) <= 4


class CompiledYolo:
    """One program compiled for one batch size on the current CUDA device."""

    def __init__(self, program: YoloProgram, batch: int, device=None, block_n: Optional[Dict[str, int]] = None,
                 image_dtype=None, nms: Optional[NmsConfig] = None, quant_on_load: bool = False,
                 plan_bits: int = 0, programmatic: Optional[bool] = None):
        torch = _torch()
        self.program = program
        self.batch = batch
        self.device = torch.device("cuda", torch.cuda.current_device() if device is None else device)
        self.lib = _native.load()
        n = batch
        p = program
        int8_inputs = set()
        for c in p.commands:
            if isinstance(c, ConvCmd) and c.precision == "int8":
                int8_inputs.update(pt.value for pt in c.inputs)
        self.needs_amax = int8_inputs
        # ---- values: fp16 NHWC buffers + amax slots
        self.values: Dict[str, "torch.Tensor"] = {}
        self.amax_off: Dict[str, int] = {}
        self.amax_groups: Dict[str, int] = {}
        off = 0
        for name, v in p.values.items():
            if name == "images":
                continue
            self.values[name] = torch.empty((n, v.h, v.w, v.channels), dtype=torch.float16, device=self.device)
            g = (v.channels + 15) // 16
            self.amax_off[name] = off
            self.amax_groups[name] = g
            off += n * g
        self.amax_arena = torch.zeros(max(off, 1), dtype=torch.int32, device=self.device)
        # fp16 images by default (the reference feeds fp16; the stem rounds fp32 inputs to fp16 anyway)
        self.image_dtype = torch.float16 if image_dtype is None else image_dtype
        self.images = torch.zeros((n, p.in_channels, p.imgsz, p.imgsz), dtype=self.image_dtype, device=self.device)
        self.output = torch.zeros((n, 4 + p.nc, p.anchors), dtype=torch.float32, device=self.device)
        self.nms = nms
        self.quant_on_load = quant_on_load
        # programmatic dependent launch (aexrt_b200_set_launch_flags): each kernel's launch and set-up
        # overlap the previous kernel; by default at batch 1 (measured: YOLOv8n-320 0.626 against
        # 0.690 ms per step at batch 1, 0.641 against 0.688 at batch 2, no gain at 4 and a loss at 8;
        # YOLOv11s-320 even at batch 1, slower from batch 2)
        self.programmatic = batch == 1 if programmatic is None else bool(programmatic)
        self.det_buf = self._new_det_buf()
        # ---- plans and per-command scratch
        self.steps: List[tuple] = []
        self.plans: Dict[str, ops.ConvPlan] = {}
        for c in p.commands:
            if isinstance(c, ConvCmd):
                # plan_bits: tuning bits above the tile (aexrt_b200_conv_plan_create) for every conv
                self._compile_conv(c, (block_n or {}).get(c.name, c.block_n) | plan_bits)
            elif isinstance(c, SppfCmd):
                self.steps.append(("sppf", c))
            elif isinstance(c, DwConvCmd):
                # fp16-rounded weights as [9][c] fp32 (kh-major taps), fp32 bias
                w9 = c.weight.astype(np.float16).astype(np.float32).reshape(c.c, 9).T.copy()
                self.steps.append(("dwconv", c, torch.from_numpy(w9).to(self.device),
                                   torch.from_numpy(c.bias.astype(np.float32)).to(self.device)))
            elif isinstance(c, PsaAttnCmd):
                self.steps.append(("attn", c))
            elif isinstance(c, DecodeCmd):
                self.steps.append(("decode", c))
                if nms is not None:
                    self.steps.append(("nms", c))
        self.graph = None
        self.launches_per_run = self._count_launches()

    # ------------------------------------------------------------------ compile
    def _new_det_buf(self):
        """One byte buffer per output slot: int32 counts [batch], then AexrtYoloDetection [batch][max_det]
        (a single device->host copy reads both)."""
        if self.nms is None:
            return None
        torch = _torch()
        n, md = self.batch, self.nms.max_detections
        return torch.zeros(n * 4 + n * md * 24, dtype=torch.uint8, device=self.device)

    def split_detections(self, buf):
        """(counts int32 [batch], detections fp32 [batch, max_det, 6]) views of a detection buffer
        (device or host)."""
        import torch

        n, md = self.batch, self.nms.max_detections
        return buf[:n * 4].view(torch.int32), buf[n * 4:].view(torch.float32).view(n, md, 6)

    def detections(self):
        """(counts, detections) of the last forward."""
        return self.split_detections(self.det_buf)

    def _amax_view(self, value: str):
        g = self.amax_groups[value]
        o = self.amax_off[value]
        return self.amax_arena[o:o + self.batch * g].view(self.batch, g)

    def _spatial(self, part: Part):
        if part.value == "images":
            return self.program.imgsz, self.program.imgsz
        v = self.program.values[part.value]
        return v.h, v.w

    def _compile_conv(self, c: ConvCmd, block_n: int):
        torch = _torch()
        n = self.batch
        sh, sw = self._spatial(c.inputs[0])
        h, w = sh * c.inputs[0].upsample, sw * c.inputs[0].upsample
        if c.precision == "int8":
            codes, scale = ops.quantize_conv_weight_int8(c.weight)
            # quantize on load: the conv reads the producers' fp16 slices and quantizes them itself,
            # for every eligible conv with the engine's quant_on_load, or for the convs a tuned tile map
            # marks with TILE_QUANT_ON_LOAD
            ql = (self.quant_on_load or bool(block_n & TILE_QUANT_ON_LOAD)) and ql_eligible(c)
            plan = ops.ConvPlan.int8(n, c.ic, h, w, c.oc, c.k, c.s, codes, scale, c.bias, silu=c.silu, pg16=c.pg16,
                                     block_n=block_n & ~TILE_QUANT_ON_LOAD, quant_on_load=ql)
            if ql and plan.info.quant_on_load:
                self.plans[c.name] = plan
                self.steps.append(("conv_ql", c, plan, self._sources(c.inputs, True), (h, w)))
                return
            shape = ops.packed_act_shape(n, c.ic, h, w, c.s)
            q = torch.empty(shape, dtype=torch.int8, device=self.device)
            rec = torch.empty((n, 1 + shape[1]), dtype=torch.float32, device=self.device)
            scratch = (q, rec)
        else:
            plan = ops.ConvPlan.fp16(n, c.ic, h, w, c.oc, c.k, c.s, c.weight, c.bias, silu=c.silu, block_n=block_n)
            if (len(c.inputs) == 1 and c.inputs[0].value == "images" and plan.info.image_input
                    and c.residual is None):
                # the stem reads the images directly: no packed copy
                self.plans[c.name] = plan
                self.steps.append(("stem", c, plan))
                return
            pt = c.inputs[0]
            if (len(c.inputs) == 1 and pt.value != "images" and pt.upsample == 1 and c.s == 1
                    and plan.info.variant == 2 and c.ic % 8 == 0 and pt.coff % 8 == 0
                    and self.values[pt.value].shape[-1] % 8 == 0):
                # the conv's TMA reads the NHWC activation itself: no slab8 copy
                self.plans[c.name] = plan
                self.steps.append(("conv_nhwc", c, plan))
                return
            hp = h + (h & 1 if c.s == 2 else 0)
            wp = w + (w & 1 if c.s == 2 else 0)
            x8 = torch.empty((n, (c.ic + 7) // 8, hp, wp, 8), dtype=torch.float16, device=self.device)
            scratch = (x8,)
        self.plans[c.name] = plan
        self.steps.append(("conv", c, plan, self._sources(c.inputs, c.precision == "int8"), scratch, (h, w)))

    def _sources(self, inputs, int8: bool):
        """AexrtB200ActSource array of a conv's input parts (with their amax slots for int8)."""
        torch = _torch()
        srcs = (AexrtB200ActSource * len(inputs))()
        for i, pt in enumerate(inputs):
            ph, pw = self._spatial(pt)
            s = srcs[i]
            if pt.value == "images":
                s.ptr = self.images.data_ptr()
                s.layout = ops.LAYOUT_NCHW_F16 if self.image_dtype == torch.float16 else ops.LAYOUT_NCHW_F32
                s.ldc = self.program.in_channels
                s.coff = 0
            else:
                buf = self.values[pt.value]
                s.ptr = buf.data_ptr()
                s.layout = ops.LAYOUT_NHWC_F16
                s.ldc = buf.shape[-1]
                s.coff = pt.coff
                if int8:
                    s.amax_groups = self._amax_view(pt.value).data_ptr()
                    s.amax_stride = self.amax_groups[pt.value]
                    s.amax_goff = pt.coff // 16
            s.channels = pt.channels
            s.upsample = pt.upsample
            s.src_h, s.src_w = ph, pw
        return srcs

    def _count_launches(self) -> int:
        k = 1  # amax arena clear
        for st in self.steps:
            k += 2 if st[0] == "conv" else 1
        return k

    # ------------------------------------------------------------------ run
    def launch(self, stream: int) -> None:
        """Issues every launch of one forward on `stream` (capturable)."""
        lib = self.lib
        prev = lib.aexrt_b200_get_launch_flags()
        check(lib.aexrt_b200_set_launch_flags(_native.LAUNCH_PROGRAMMATIC if self.programmatic else 0), "launch flags")
        try:
            self._launch(stream)
        finally:
            lib.aexrt_b200_set_launch_flags(prev)

    def _launch(self, stream: int) -> None:
        lib = self.lib
        n = self.batch
        check(lib.aexrt_b200_zero(self.amax_arena.data_ptr(), self.amax_arena.numel() * 4, stream), "zero amax")
        for st in self.steps:
            kind = st[0]
            if kind == "conv":
                _, c, plan, srcs, scratch, (h, w) = st
                out = self.values[c.out[0]]
                amax_out = self._amax_view(c.out[0]) if c.out[0] in self.needs_amax else None
                res = self.values[c.residual[0]] if c.residual is not None else None
                res_coff = c.residual[1] if c.residual is not None else 0
                if c.precision == "int8":
                    q, rec = scratch
                    check(lib.aexrt_b200_act_quantize_concat(srcs, len(srcs), n, h, w, int(c.pg16), c.s, q.data_ptr(),
                                                             rec.data_ptr(), stream), f"quantize {c.name}")
                    plan.run(q, rec, out=out, out_coff=c.out[1], residual=res, res_coff=res_coff, amax_out=amax_out,
                             amax_goff=c.out[1] // 16, stream=stream)
                else:
                    (x8,) = scratch
                    check(lib.aexrt_b200_pack_f16_concat(srcs, len(srcs), n, h, w, c.s, x8.data_ptr(), stream),
                          f"pack {c.name}")
                    plan.run(x8, out=out, out_coff=c.out[1], residual=res, res_coff=res_coff, amax_out=amax_out,
                             amax_goff=c.out[1] // 16, stream=stream)
            elif kind == "conv_ql":
                _, c, plan, srcs, _ = st
                out = self.values[c.out[0]]
                amax_out = self._amax_view(c.out[0]) if c.out[0] in self.needs_amax else None
                res = self.values[c.residual[0]] if c.residual is not None else None
                plan.run_sources(srcs, out=out, out_coff=c.out[1], residual=res,
                                 res_coff=c.residual[1] if c.residual is not None else 0, amax_out=amax_out,
                                 amax_goff=c.out[1] // 16, stream=stream)
            elif kind == "conv_nhwc":
                _, c, plan = st
                out = self.values[c.out[0]]
                amax_out = self._amax_view(c.out[0]) if c.out[0] in self.needs_amax else None
                res = self.values[c.residual[0]] if c.residual is not None else None
                plan.run_nhwc(self.values[c.inputs[0].value], x_coff=c.inputs[0].coff, out=out, out_coff=c.out[1],
                              residual=res, res_coff=c.residual[1] if c.residual is not None else 0,
                              amax_out=amax_out, amax_goff=c.out[1] // 16, stream=stream)
            elif kind == "stem":
                _, c, plan = st
                out = self.values[c.out[0]]
                amax_out = self._amax_view(c.out[0]) if c.out[0] in self.needs_amax else None
                plan.run_image(self.images, out=out, out_coff=c.out[1], amax_out=amax_out, amax_goff=c.out[1] // 16,
                               stream=stream)
            elif kind == "sppf":
                c = st[1]
                x = self.values[c.x.value]
                out = self.values[c.out[0]]
                v = self.program.values[c.x.value]
                am = self._amax_view(c.out[0])
                check(lib.aexrt_b200_sppf_pool(x.data_ptr(), n, v.h, v.w, c.x.channels, x.shape[-1], c.x.coff,
                                               out.data_ptr(), out.shape[-1], c.out[1], am.data_ptr(), am.shape[1],
                                               c.out[1] // 16, stream), "sppf")
            elif kind == "dwconv":
                _, c, w9, bias = st
                x = self.values[c.x.value]
                out = self.values[c.out[0]]
                v = self.program.values[c.x.value]
                g = c.group or c.c
                check(lib.aexrt_b200_dwconv3x3_f16(x.data_ptr(), n, v.h, v.w, c.c, x.shape[-1], c.x.coff, g,
                                                   c.group_stride or g, c.group_off, w9.data_ptr(), bias.data_ptr(),
                                                   c.s, int(c.silu), out.data_ptr(), out.shape[-1], c.out[1], stream),
                      f"dwconv {c.name}")
            elif kind == "attn":
                c = st[1]
                qkv, pe, out = self.values[c.qkv.value], self.values[c.pe.value], self.values[c.out[0]]
                v = self.program.values[c.qkv.value]
                am = self._amax_view(c.out[0]) if c.out[0] in self.needs_amax else None
                check(lib.aexrt_b200_psa_attention_f16(
                    qkv.data_ptr(), n, v.h, v.w, qkv.shape[-1], c.qkv.coff, c.heads, c.key_dim, c.head_dim, c.scale,
                    pe.data_ptr(), pe.shape[-1], c.pe.coff, out.data_ptr(), out.shape[-1], c.out[1],
                    am.data_ptr() if am is not None else None, am.shape[1] if am is not None else 0,
                    c.out[1] // 16, stream), f"attention {c.name}")
            elif kind == "decode":
                c = st[1]
                lv = (AexrtB200DecodeLevel * len(c.levels))()
                for i, (bp, cp, stride) in enumerate(c.levels):
                    bb, cb = self.values[bp.value], self.values[cp.value]
                    v = self.program.values[bp.value]
                    lv[i].box, lv[i].box_ldc, lv[i].box_coff = bb.data_ptr(), bb.shape[-1], bp.coff
                    lv[i].cls, lv[i].cls_ldc, lv[i].cls_coff = cb.data_ptr(), cb.shape[-1], cp.coff
                    lv[i].h, lv[i].w, lv[i].stride = v.h, v.w, stride
                check(lib.aexrt_b200_yolo_decode(lv, len(c.levels), n, c.nc, c.reg_max, self.output.data_ptr(), stream),
                      "decode")
            elif kind == "nms":
                c, cfg = st[1], self.nms
                counts, dets = self.split_detections(self.det_buf)
                check(lib.aexrt_b200_yolo_nms_topk(self.output.data_ptr(), n, 4 + c.nc, self.program.anchors, c.nc, 0,
                                                   1, cfg.conf, cfg.iou, cfg.max_candidates, cfg.max_detections,
                                                   cfg.mode | (cfg.ctas_per_image << ops.NMS_CTAS_SHIFT),
                                                   dets.data_ptr(), counts.data_ptr(), stream), "nms")

    def capture(self) -> None:
        """Records one forward into a CUDA graph (warm-up run first, as graph capture requires)."""
        torch = _torch()
        s = torch.cuda.Stream(device=self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(s):
            self.launch(s.cuda_stream)
        torch.cuda.current_stream(self.device).wait_stream(s)
        torch.cuda.synchronize(self.device)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=s):
            self.launch(s.cuda_stream)
        torch.cuda.synchronize(self.device)

    def forward(self, images=None):
        """One forward on device-resident `images` (copied into the input buffer if given)."""
        if images is not None:
            self.images.copy_(images, non_blocking=True)
        if self.graph is not None:
            self.graph.replay()
        else:
            torch = _torch()
            self.launch(torch.cuda.current_stream(self.device).cuda_stream)
        return self.output

    # ------------------------------------------------------------------ streaming
    def capture_slots(self, slots: int = 2) -> None:
        """Records one graph per input/output slot for :meth:`stream` (double-buffered I/O).

        The slots own their image and output buffers; the activations between the layers are
        shared, since the graphs replay one after another on the compute stream."""
        torch = _torch()
        n, p = self.batch, self.program
        self.slot_images, self.slot_output0, self.slot_outputs, self.slot_graphs = [], [], [], []
        images, output, graph, det_buf = self.images, self.output, self.graph, self.det_buf
        for _ in range(slots):
            self.images = torch.zeros((n, p.in_channels, p.imgsz, p.imgsz), dtype=self.image_dtype, device=self.device)
            self.output = torch.zeros((n, 4 + p.nc, p.anchors), dtype=torch.float32, device=self.device)
            self.det_buf = self._new_det_buf()
            self.graph = None
            self.capture()
            # every buffer a slot graph touches stays referenced as long as the graph: the next
            # capture empties the allocator cache, which would unmap a released one
            self.slot_images.append(self.images)
            self.slot_output0.append(self.output)
            # with NMS the slot's read-back is its detection buffer, else its output0
            self.slot_outputs.append(self.det_buf if self.nms is not None else self.output)
            self.slot_graphs.append(self.graph)
        self.images, self.output, self.graph, self.det_buf = images, output, graph, det_buf
        self.compute_stream = torch.cuda.Stream(device=self.device)
        self.upload_stream = torch.cuda.Stream(device=self.device)
        self.download_stream = torch.cuda.Stream(device=self.device)

    def stream(self, host_inputs, host_outputs) -> None:
        """Runs len(host_inputs) batches host -> device -> host with the copies of one batch
        overlapping the forward of the previous one (uploads, forwards and read-backs run on three
        streams; the caller's current stream waits for all of them, so synchronize it before
        reading host_outputs).

        host_inputs[k] (pinned, the engine's image dtype, [batch, 3, imgsz, imgsz]) is uploaded into slot k % slots,
        its forward replays that slot's graph, and its result is read back into
        host_outputs[k % len(host_outputs)]: with NMS a pinned uint8 buffer shaped like
        ``det_buf`` (split it with :meth:`split_detections`), else pinned fp32 output0
        [batch, 4 + nc, anchors]."""
        torch = _torch()
        slots = len(self.slot_graphs)
        cs, us, ds = self.compute_stream, self.upload_stream, self.download_stream
        if not hasattr(self, "_slot_events"):
            ev = lambda: [torch.cuda.Event() for _ in range(slots)]  # noqa: E731
            self._slot_events = (ev(), ev(), ev())  # uploaded, computed, downloaded
        uploaded, computed, downloaded = self._slot_events
        cur = torch.cuda.current_stream(self.device)
        for st in (us, cs, ds):
            st.wait_stream(cur)
        for k, host in enumerate(host_inputs):
            j = k % slots
            with torch.cuda.stream(us):
                if k >= slots:
                    us.wait_event(computed[j])  # the slot's previous forward has read its images
                self.slot_images[j].copy_(host, non_blocking=True)
                uploaded[j].record(us)
            with torch.cuda.stream(cs):
                cs.wait_event(uploaded[j])
                if k >= slots:
                    cs.wait_event(downloaded[j])  # the slot's previous detections have been read back
                self.slot_graphs[j].replay()
                computed[j].record(cs)
            with torch.cuda.stream(ds):
                ds.wait_event(computed[j])
                host_outputs[k % len(host_outputs)].copy_(self.slot_outputs[j], non_blocking=True)
                downloaded[j].record(ds)
        for st in (us, cs, ds):
            cur.wait_stream(st)

    def status(self) -> int:
        """OR of every plan's device status word (non-zero: a pipeline wait gave up)."""
        st = 0
        for p in self.plans.values():
            st |= p.status()
        return st


def main(argv=None) -> int:
    """Runs eager forwards of a synthetic YOLO model (profiling entry: one forward = one launch list)."""
    import argparse

    from . import yolo

    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--batch", type=int, default=256)
    ap.add_argument("--imgsz", type=int, default=320)
    ap.add_argument("--forwards", type=int, default=2)
    ap.add_argument("--no-nms", action="store_true", help="stop at output0 (no GPU filter + NMS + top-k)")
    ap.add_argument("--model", default="yolov8n", choices=["yolov8n", "yolov8s", "yolov11s"])
    ap.add_argument("--programmatic", default="auto", choices=["auto", "on", "off"])
    ap.add_argument("--tiles", default=None, help="a tuned {conv name: tile bits} map (python -m "
                    "aexrt_b200.autotune --program ... --tiles-out FILE)")
    a = ap.parse_args(argv)
    torch = _torch()
    if a.model == "yolov8n":
        program = yolo.build_yolov8n(nc=4, imgsz=a.imgsz, seed=0)
    else:
        program = getattr(yolo, f"build_{a.model}")(nc=80, imgsz=a.imgsz, seed=0)
    tiles = None
    if a.tiles:
        import json

        with open(a.tiles) as f:
            tiles = json.load(f)
    eng = CompiledYolo(program, a.batch, nms=None if a.no_nms else NmsConfig(), block_n=tiles,
                       programmatic=None if a.programmatic == "auto" else a.programmatic == "on")
    x = torch.from_numpy(np.random.default_rng(0).uniform(0, 1, (a.batch, 3, a.imgsz, a.imgsz)).astype(np.float16))
    x = x.to(eng.device)
    for i in range(a.forwards):
        # one NVTX range per forward, so a profiler can select exactly one (ncu --nvtx --nvtx-include "forward1/")
        torch.cuda.nvtx.range_push(f"forward{i}")
        eng.forward(x)
        torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize(eng.device)
    print(f"{a.forwards} forwards of batch {a.batch}: {eng.launches_per_run - 1} kernels each, status {eng.status()}")
    return 0 if eng.status() == 0 else 1


if __name__ == "__main__":
    raise SystemExit(main())
