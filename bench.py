"""Benchmark: W8A8 YOLOv8n-320 images/s on 1..8 B200s (data-parallel replicas).

    python bench.py [--gpus N --steps K --warmup W --batch B] [--impl reference]
    python -m torch.distributed.run --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1 \
        --master-port P bench.py --gpus N ...

One step = one forward of the YOLOv8n-320 W8A8 command stream (backbone and
neck on the tcgen05 int8 convs, fp16 detect head, DFL decode, confidence
filter + NMS + top-k) over a batch of B synthetic images per GPU, replayed as
one CUDA graph.  Images never exchange
data, so each rank runs its own replica on its own batch ("weak" scaling, no
collective on the data path; torch.distributed only brackets the timed region
and takes the max over ranks).  Rank 0 prints one JSON line.

--impl reference times the reference's W8A8 arithmetic on the host cores (the
reference path is D3D12/HLSL and cannot run here; its CPU restatement in
oracle/ is the reference implementation) on a bounded sample of the same
workload, on rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

METRIC = "W8A8 YOLOv8n-320 images/s"
WORKLOAD = "yolov8n-320 W8A8 forward (int8 backbone+neck, fp16 head, DFL decode, NMS + top-k)"
# whole-model workloads: builder, metric, description, imgsz, nc, per-GPU batch (None: global batch / ranks), scaling
MODELS = {
    "yolov8n-320": ("build_yolov8n", METRIC, WORKLOAD, 320, 4, None, "weak"),
    # global batch 512 split evenly over the GPUs
    "yolov8s-640": ("build_yolov8s", "W8A8 YOLOv8s-640 images/s",
                    "yolov8s-640 W8A8 forward (int8 backbone+neck, fp16 head, nc=80, DFL decode, NMS + top-k)",
                    640, 80, 512, "strong"),
    # YOLOv11s-320 (C3k2, SPPF, C2PSA; W8A8 except the head, the depthwise convs and the
    # attention core), batch sweep 1 / 8 / 64 on one GPU (--batch)
    "yolov11s-320": ("build_yolov11s", "W8A8 YOLOv11s-320 images/s",
                     "yolov11s-320 W8A8 forward (int8 C3k2/SPPF/C2PSA convs, fp16 head + depthwise + attention, "
                     "nc=80, DFL decode, NMS + top-k)", 320, 80, None, "weak"),
}
L2_BYTES = 126 * 1024 * 1024
# DRAM read + write bytes of the 44 W8A8 conv launches of one forward, per image, from one ncu
# capture at batch 256 (profiles/conv_family_dram_b256.md); valid for that batch only
CONV_DRAM_BYTES_PER_IMAGE_B256 = 1495.3e6 / 256


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--batch", type=int, default=None,
                    help="images per GPU per step (default: 256 for yolov8n-320, 512 / GPUs for yolov8s-640, "
                         "64 for the layer workloads)")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--conv-table", action="store_true",
                    help="model workloads: print every W8A8 conv launch of the roofline pass (time, GB/s, TOPS) "
                         "to stderr")
    ap.add_argument("--onnx", default=None,
                    help="model workloads: the program comes from this ONNX YOLO graph (imported without onnx)")
    ap.add_argument("--programmatic", default="auto", choices=["auto", "on", "off"],
                    help="model workloads: programmatic dependent launch (auto: the engine's choice by batch)")
    ap.add_argument("--quant-on-load", action="store_true",
                    help="model workloads: int8 convs quantize their fp16 sources on load (no separate quantize)")
    ap.add_argument("--cpu-sample", type=int, default=None,
                    help="images in the CPU baseline sample (default 160 for yolov8n-320, 8 for yolov8s-640: "
                         "about 12-25 s)")
    ap.add_argument("--workload", default="yolov8n-320",
                    help="yolov8n-320 (the metric), yolov8s-640 (BASELINE config 5), or a BASELINE layer: "
                         + ", ".join(LAYERS)
                    + ", or amax-quant, " + ", ".join(QUANTS) + ", " + ", ".join(HEAD_LAYERS))
    ap.add_argument("--mode", type=int, default=0, help="layer workloads: 0 per-tensor, 1 pg16 scales")
    ap.add_argument("--order", type=int, default=0,
                    help="layer workloads: halo tile order (0 auto, 1 strided, 2 contiguous)")
    ap.add_argument("--plan-bits", type=lambda s: int(s, 0), default=0,
                    help="extra plan tuning bits for every conv (block_n bits 16-31, e.g. 0x10000000 direct stores)")
    ap.add_argument("--amax-out", action="store_true",
                    help="layer workloads: the conv also maxes |y| per 16-channel group for the next layer")
    ap.add_argument("--chain", type=int, default=0,
                    help="layer workloads: time N back-to-back conv launches in one CUDA graph (programmatic "
                         "dependent launch, as inside a batch-1 model graph) and report the time per launch")
    ap.add_argument("--engine", default=None,
                    help="time an .aexrt engine compiled by the reference (e.g. tests/golden/yolov8n_w8a8.aexrt) "
                         "through the reference runtime ABI (libaexrt_b200.so aexrt_yolo_*), batch --batch (256)")
    ap.add_argument("--algo-map", default=None, help="--engine: a tuned {command: algorithm} map to apply")
    ap.add_argument("--tiles", default=None,
                    help="model workloads: a tuned {conv name: tile bits} map (python -m aexrt_b200.autotune "
                         "--program ... --tiles-out FILE) applied at compile time; default "
                         "aexrt_b200/tuned/<workload>_b<batch>.json when it exists, 'none' for the heuristics")
    ap.add_argument("--variants", default=None, help="--engine: a tuned {command: tile bits} sidecar to apply")
    return ap.parse_args()


# the C1 block and the layer sweep (name: ic, h, w, oc, k, s)
LAYERS = {
    "c1": (64, 80, 80, 128, 3, 1),
    "sweep-1x1": (128, 40, 40, 128, 1, 1),
    "sweep-3x3s1": (64, 80, 80, 64, 3, 1),
    "sweep-3x3s2": (32, 160, 160, 64, 3, 2),
    "sweep-3x3s2-small": (128, 20, 20, 256, 3, 2),
    # narrow high-resolution layers of YOLOv8n-320 (l1, l2.m0.cv1, l2.cv1)
    "n-l1": (16, 160, 160, 32, 3, 2),
    "n-l2m": (16, 80, 80, 16, 3, 1),
    "n-l2cv1": (32, 80, 80, 32, 1, 1),
}
# fp16 detect-head convs of YOLOv8n-320 (each level's first 3x3 conv): ic, h, w, oc
HEAD_LAYERS = {"head-p3": (64, 40, 40, 128), "head-p4": (128, 20, 20, 128), "head-p5": (256, 10, 10, 128)}
# between-layer quantize passes of YOLOv8n-320: (h, w, channels)
QUANTS = {"quant-nhwc": (40, 40, 192), "quant-nhwc-16": (160, 160, 16), "quant-nhwc-32": (80, 80, 32)}


def run_layer(args):
    """One BASELINE layer (or the standalone amax + quantize tensor) on one GPU: quantize + conv per step."""
    import torch

    from aexrt_b200 import ops

    torch.cuda.set_device(0)
    rng = np.random.default_rng(0)
    n = args.batch or 64
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device="cuda")
    hbm, bf16, src = measured_peaks()
    if args.workload == "amax-quant":
        x = torch.from_numpy((lambda z: z / (1 + np.exp(-z)))(rng.standard_normal((n, 64, 80, 80)).astype(np.float32))
                             .astype(np.float16)).cuda()
        q, rec, amax = ops.act_amax_quantize(x, args.mode)

        def step():
            # one call: a thread-block cluster per image reads the tensor once
            ops.act_amax_quantize(x, args.mode, amax_out=amax, q_out=q, rec_out=rec)

        byts, ops_ = 5.0 * x.numel(), 0.0
        desc = f"standalone amax + quantize of {n}x64x80x80 fp16 NCHW (BASELINE config 2)"
    elif args.workload in QUANTS:
        # the model's between-layer quantize: fp16 NHWC activations (amax already in the slots)
        qh, qw, qc = QUANTS[args.workload]
        x = torch.from_numpy((lambda z: z / (1 + np.exp(-z)))(rng.standard_normal((n, qh, qw, qc)).astype(np.float32))
                             .astype(np.float16)).cuda()
        amax = ops.act_amax(x, ops.LAYOUT_NHWC_F16)
        q, rec = ops.act_quantize(x, amax, args.mode, ops.LAYOUT_NHWC_F16)

        def step():
            ops.act_quantize(x, amax, args.mode, ops.LAYOUT_NHWC_F16, q_out=q, rec_out=rec)

        byts, ops_ = 3.0 * x.numel(), 0.0
        desc = f"quantize of {n}x{qh}x{qw}x{qc} fp16 NHWC into int8 slabs (the model's between-layer pass)"
    elif args.workload in HEAD_LAYERS:
        # the detect head's first 3x3 conv of a level (fp16, both branches' channels), reading the
        # fp16 NHWC activation directly
        ic, h, w, oc = HEAD_LAYERS[args.workload]
        k, s = 3, 1
        wt = rng.normal(0, 0.05, (oc, ic, k, k)).astype(np.float32)
        b = rng.normal(0, 0.1, oc).astype(np.float32)
        plan = ops.ConvPlan.fp16(n, ic, h, w, oc, k, s, wt, b, silu=True, block_n=(args.order << 20) | args.plan_bits)
        x = torch.from_numpy(rng.standard_normal((n, h, w, ic)).astype(np.float16)).cuda()
        out = torch.empty(plan.out_shape, dtype=torch.float16, device="cuda")

        def step():
            plan.run_nhwc(x, out=out)

        ops_ = 2.0 * n * h * w * oc * ic * k * k
        byts = 2.0 * n * ic * h * w + 2.0 * n * oc * h * w + 2.0 * oc * ic * k * k
        desc = f"fp16 head conv {ic}->{oc} k3 s1 @{h}x{w}, batch {n}, NHWC input"
    else:
        ic, h, w, oc, k, s = LAYERS[args.workload]
        wt = rng.normal(0, 0.05, (oc, ic, k, k)).astype(np.float32)
        b = rng.normal(0, 0.1, oc).astype(np.float32)
        codes, scale = ops.quantize_conv_weight_int8(wt)
        plan = ops.ConvPlan.int8(n, ic, h, w, oc, k, s, codes, scale, b, pg16=bool(args.mode),
                                 block_n=(args.order << 20) | args.plan_bits)
        x = torch.from_numpy((lambda z: z / (1 + np.exp(-z)))(rng.standard_normal((n, ic, h, w)).astype(np.float32))
                             .astype(np.float16)).cuda()
        amax = ops.act_amax(x, ops.LAYOUT_NCHW_F16)
        q, rec = ops.act_quantize(x, amax, args.mode, ops.LAYOUT_NCHW_F16, consumer_stride=s)
        out = torch.empty(plan.out_shape, dtype=torch.float16, device="cuda")
        amax_next = torch.zeros((n, (oc + 15) // 16), dtype=torch.int32, device="cuda") if args.amax_out else None

        def step():
            plan.run(q, rec, out=out, amax_out=amax_next)

        d = plan.desc
        ops_ = 2.0 * n * d.out_h * d.out_w * oc * ic * k * k
        byts = n * ic * h * w + 2.0 * n * oc * d.out_h * d.out_w + oc * ic * k * k
        desc = (f"conv {ic}->{oc} k{k} s{s} @{h}x{w}, batch {n}, {'pg16' if args.mode else 'per-tensor'}"
                f"{', amax out' if args.amax_out else ''}{f', order {args.order}' if args.order else ''}"
                " (BASELINE configs 1-2)")
    per = 1
    if args.chain > 0 and args.workload in LAYERS:
        # N launches of the conv in one graph, each a programmatic dependent of the one before (the
        # form a batch-1 model graph takes): the time per launch is the conv's cost inside a forward
        from aexrt_b200 import _native

        lib = _native.load()
        _native.check(lib.aexrt_b200_set_launch_flags(_native.LAUNCH_PROGRAMMATIC), "launch flags")
        step()
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s):
                for _ in range(args.chain):
                    step()
        torch.cuda.current_stream().wait_stream(s)
        lib.aexrt_b200_set_launch_flags(0)
        step = g.replay
        per = args.chain
    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize()
    ts = []
    for _ in range(args.steps):
        flush.zero_()  # inputs of some layers fit in L2: flush it between timed iterations
        # the stream waits ~0.5 ms while the host enqueues the events and the launch, so the event
        # pair brackets the kernel, not the host's launch latency
        torch.cuda._sleep(1_000_000)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        step()
        e1.record()
        torch.cuda.synchronize()
        ts.append(e0.elapsed_time(e1) / 1e3)
    t = statistics.median(ts) / per
    # tensor peak: dense int8 is twice bf16 on B200; the fp16 head convs run at the bf16/fp16 rate
    tensor_peak = bf16 if args.workload in HEAD_LAYERS else 2.0 * bf16
    line = {"metric": f"{args.workload} kernel time", "value": t * 1e3, "unit": "ms", "higher_is_better": False,
            "steps": args.steps, "warmup": args.warmup,
            "config": {"workload": desc + (f", {per} launches per graph (programmatic)" if per > 1 else ""),
                       "l2": "flushed between steps"},
            "achieved_gbs": byts / t / 1e9, "hbm_frac": byts / t / 1e9 / hbm}
    if ops_:
        line.update({"achieved_tops": ops_ / t / 1e12, "tensor_frac": ops_ / t / 1e12 / tensor_peak,
                     "plan": vars(plan.info)})
    print(json.dumps(line), flush=True)
    return 0


def shard_range(global_batch: int, world: int, rank: int):
    """Images [start, start + count) of a global batch that rank `rank` of `world` runs: contiguous
    shards, the first global_batch % world ranks one image larger, so the shards cover the batch
    exactly once."""
    base, extra = divmod(global_batch, world)
    count = base + (1 if rank < extra else 0)
    start = rank * base + min(rank, extra)
    return start, count


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def host_cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def cpu_reference(program, n_images: int, seed: int = 1, warm: bool = True):
    """Times the oracle (the reference's W8A8 arithmetic on the CPU, then its post-process) on n_images;
    the warm-up image (which loads the C helper) is outside the returned time."""
    from oracle import yolo_model as om
    from oracle import yolo_post as op

    rng = np.random.default_rng(seed)
    imgs = rng.uniform(0, 1, (n_images, 3, program.imgsz, program.imgsz)).astype(np.float16)
    if warm:
        om.run_program(program, imgs[:1])
    chunk = 4
    t0 = time.perf_counter()
    for i in range(0, n_images, chunk):
        out = om.run_program(program, imgs[i:i + chunk])["output0"]
        for y in out:
            op.postprocess(y, program.nc)
    dt = time.perf_counter() - t0
    return n_images / dt, dt


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 50 ms while running."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        # nvidia-smi numbers the GPUs physically: map this process's device through CUDA_VISIBLE_DEVICES
        vis = [v.strip() for v in os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",") if v.strip()]
        self.gpu = vis[gpu_index] if gpu_index < len(vis) else str(gpu_index)
        self.proc = None
        self.path = None

    def __enter__(self):
        import tempfile

        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
            # the sampler takes a moment to start (longer when every rank starts one): wait for its
            # first sample, so that the timed region is covered
            t0 = time.time()
            while time.time() - t0 < 5.0 and os.path.getsize(self.path) == 0 and self.proc.poll() is None:
                time.sleep(0.05)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        if not self.path or not os.path.exists(self.path):
            return None
        rows = []
        for line in open(self.path):
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append(parts)
            except Exception:
                pass
        os.unlink(self.path)
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if "Active" in r[5 + i] and "Not" not in r[5 + i]})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


def measured_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        d = json.load(open(path))
        return d.get("hbm_gbs", 6650.0), d.get("bf16_tflops", 1590.0), "measured"
    return 6650.0, 1590.0, "fallback"


def conv_roofline(eng, torch, stream):
    """Per-launch CUDA-event timing of the W8A8 conv kernels (eager pass, after the timed region).

    Algorithmic ops per launch = 2*N*OH*OW*OC*IC*KH*KW (benchmarks/roofline_report.py:94 convention);
    achieved = sum(ops) / sum(kernel time) over all W8A8 conv launches of one step."""
    from aexrt_b200._native import check

    lib = eng.lib
    n = eng.batch
    recs = []
    torch.cuda.synchronize()
    # hold the stream for ~0.1 s so that the host enqueues every launch below before the first one
    # runs: an event pair then brackets its kernel alone, not the host's launch latency
    torch.cuda._sleep(200_000_000)
    check(lib.aexrt_b200_zero(eng.amax_arena.data_ptr(), eng.amax_arena.numel() * 4, stream), "zero")
    for st in eng.steps:
        if st[0] not in ("conv", "conv_ql") or st[1].precision != "int8":
            continue
        c = st[1]
        out = eng.values[c.out[0]]
        res = eng.values[c.residual[0]] if c.residual else None
        amax_out = eng._amax_view(c.out[0]) if c.out[0] in eng.needs_amax else None
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        if st[0] == "conv_ql":
            # quantize on load: the conv reads the fp16 sources (2 bytes per input element)
            _, _, plan, srcs, (h, w) = st
            in_bytes = 2
            e0.record(torch.cuda.current_stream())
            plan.run_sources(srcs, out=out, out_coff=c.out[1], residual=res,
                             res_coff=c.residual[1] if c.residual else 0, amax_out=amax_out,
                             amax_goff=c.out[1] // 16, stream=stream)
        else:
            _, _, plan, srcs, scratch, (h, w) = st
            in_bytes = 1
            q, rec = scratch
            check(lib.aexrt_b200_act_quantize_concat(srcs, len(srcs), n, h, w, int(c.pg16), c.s, q.data_ptr(),
                                                     rec.data_ptr(), stream), "quantize")
            e0.record(torch.cuda.current_stream())
            plan.run(q, rec, out=out, out_coff=c.out[1], residual=res, res_coff=c.residual[1] if c.residual else 0,
                     amax_out=amax_out, amax_goff=c.out[1] // 16, stream=stream)
        e1.record(torch.cuda.current_stream())
        d = eng.program.values[c.out[0]]
        ops = 2.0 * n * d.h * d.w * c.oc * c.ic * c.k * c.k
        byts = n * (in_bytes * c.ic * h * w + 2 * c.oc * d.h * d.w) + c.oc * c.ic * c.k * c.k
        name = f"{c.name} {c.ic}->{c.oc} k{c.k} s{c.s} @{h}x{w}{' pg16' if c.pg16 else ''}"
        recs.append((e0, e1, ops, byts, name))
    torch.cuda.synchronize()
    t = sum(r[0].elapsed_time(r[1]) for r in recs) / 1e3
    ops = sum(r[2] for r in recs)
    byts = sum(r[3] for r in recs)
    table = [{"conv": r[4], "us": r[0].elapsed_time(r[1]) * 1e3, "gbs": r[3] / (r[0].elapsed_time(r[1]) / 1e3) / 1e9,
              "tops": r[2] / (r[0].elapsed_time(r[1]) / 1e3) / 1e12} for r in recs]
    return {"time_s": t, "ops": ops, "bytes": byts, "launches": len(recs), "table": table}


def run_reference(args):
    rank, world, local = dist_env()
    if rank != 0:
        return 0
    from aexrt_b200 import yolo

    builder, metric, workload, imgsz, nc, _, scaling = MODELS[args.workload]
    program = getattr(yolo, builder)(nc=nc, imgsz=imgsz, seed=0)
    cores = host_cores()
    os.environ.setdefault("OMP_NUM_THREADS", str(cores))
    per_step = 4
    for _ in range(args.warmup):
        cpu_reference(program, per_step, seed=2)
    dt = 0.0
    for k in range(args.steps):
        dt += cpu_reference(program, per_step, seed=3 + k, warm=False)[1]
    ips = args.steps * per_step / dt
    line = {
        "impl": "reference", "metric": metric, "value": ips, "unit": "images/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt / args.steps * 1e3, "higher_is_better": True,
        "scaling": scaling, "vs_baseline": None, "dtype": "int8", "data": "synthetic",
        "config": {"workload": workload + " on the host CPU", "global_batch": per_step, "imgsz": imgsz, "nc": nc,
                   "parallelism": "host cores",
                   "batch_note": ("a bounded sample of 4 images per step, where the GPU arm runs 256: every image has "
                                  "its own activation scales, so an image's work and result do not depend on the "
                                  "batch it runs in, and images/s compare directly")},
        "cpu_baseline": {"value": ips, "unit": "images/s", "cores": cores, "kind": "port",
                         "sample": f"{per_step} images per step x {args.steps} steps through the CPU restatement "
                                   "of the reference's W8A8 arithmetic (oracle/), C/OpenMP int32 convolutions"},
        "e2e": {"value": ips, "unit": "images/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def run_ours(args):
    import torch

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    from aexrt_b200 import engine, yolo

    builder, metric, workload, imgsz, nc, global_batch, scaling = MODELS[args.workload]
    program = getattr(yolo, builder)(nc=nc, imgsz=imgsz, seed=0)
    if args.onnx:
        from aexrt_b200 import onnx_yolo

        program = onnx_yolo.import_onnx(args.onnx)
        imgsz, nc = program.imgsz, program.nc
        workload = f"{args.onnx} (ONNX import): " + workload
    if args.batch is None and global_batch:
        # strong scaling: this rank's shard of the global batch (image k is drawn from seed 1000 + k)
        start, B = shard_range(global_batch, world, rank)
    else:
        B = args.batch or 256
        start = rank * B
    total = B
    if dist is not None:
        tb = torch.tensor([B], device="cuda")
        dist.all_reduce(tb)
        total = int(tb.item())  # images of one step over all ranks
    # the autotuner's tile plan for this workload and batch (aexrt_b200/tuned/), unless --tiles names
    # another map or "none"
    tiles_path = args.tiles
    if tiles_path is None:
        cand = os.path.join(ROOT, "aexrt_b200", "tuned", f"{args.workload}_b{B}.json")
        tiles_path = cand if os.path.exists(cand) and not args.onnx else None
    elif tiles_path == "none":
        tiles_path = None
    tiles = json.load(open(tiles_path)) if tiles_path else None
    eng = engine.CompiledYolo(program, B, nms=engine.NmsConfig(), quant_on_load=args.quant_on_load,
                              plan_bits=args.plan_bits, block_n=tiles,
                              programmatic=None if args.programmatic == "auto" else args.programmatic == "on")
    # fp16 images, as BASELINE's config feeds them (uniform[0,1]); image k of the job from seed 1000 + k
    host_in = torch.from_numpy(np.stack([np.random.default_rng(1000 + start + k).uniform(0, 1, (3, imgsz, imgsz))
                                         for k in range(B)]).astype(np.float16)).pin_memory()
    # the read-back is the detection buffer: per image a count and up to 100 AexrtYoloDetection rows
    host_out = torch.empty(tuple(eng.det_buf.shape), dtype=torch.uint8).pin_memory()
    eng.images.copy_(host_in)
    eng.capture()
    stream = torch.cuda.current_stream()

    def barrier():
        if dist is not None:
            dist.barrier()

    def timed(fn, steps):
        barrier()
        torch.cuda.synchronize()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            fn()
        e1.record(stream)
        torch.cuda.synchronize()
        barrier()
        t = e0.elapsed_time(e1) / 1e3
        if dist is not None:
            tt = torch.tensor([t], device="cuda")
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            t = float(tt.item())
        return t

    def step_device():
        eng.graph.replay()

    with ClockSampler(local) as clk:
        for _ in range(max(3, args.warmup) + 50):  # warm-up (also lets the clock sampler start)
            step_device()
        torch.cuda.synchronize()
        t_dev = timed(step_device, args.steps)
    clocks = clk.summary()
    e2e = None
    if not args.no_e2e:
        # end to end through the engine's streaming API: every step uploads its images from
        # pinned host memory and reads its detections back; the upload of step k+1 and the
        # read-back of step k-1 overlap the forward of step k (double-buffered slots)
        eng.capture_slots(2)
        host_ins = [host_in, host_in.clone().pin_memory()]
        host_outs = [host_out, host_out.clone().pin_memory()]
        eng.stream([host_ins[k % 2] for k in range(4)], host_outs)  # warm-up
        torch.cuda.synchronize()
        t_e2e = timed(lambda: eng.stream([host_ins[k % 2] for k in range(args.steps)], host_outs), 1)
        e2e = {"value": total * args.steps / t_e2e, "unit": "images/s",
               "h2d_bytes_per_step": int(host_in.numel() * host_in.element_size()),
               "d2h_bytes_per_step": int(host_out.numel() * host_out.element_size()),
               "pipeline": "double-buffered: upload k+1 and read-back k-1 overlap forward k"}
    latency = None
    if B <= 8:
        # small batches: synchronous latency of one batch through the same graph, the upload of its
        # images from pinned memory and the read-back of its detections inside each timed step
        # (one batch in flight, as an interactive caller runs it)
        dev_out = eng.det_buf

        def one_batch():
            eng.images.copy_(host_in, non_blocking=True)
            eng.graph.replay()
            host_out.copy_(dev_out, non_blocking=True)
            stream.synchronize()

        for _ in range(10):
            one_batch()
        ts = []
        for _ in range(max(20, args.steps)):
            t0 = time.perf_counter()
            one_batch()
            ts.append(time.perf_counter() - t0)
        ts.sort()
        latency = {"ms_per_batch_median": ts[len(ts) // 2] * 1e3, "ms_per_batch_p90": ts[int(len(ts) * 0.9)] * 1e3,
                   "batch": B, "device_ms_per_step": t_dev / args.steps * 1e3,
                   "how": "host wall clock around upload + graph replay + read-back + synchronize, one batch in flight"}
    status = eng.status()
    # roofline of the dominant kernel (W8A8 conv), measured per launch with CUDA events
    rf = conv_roofline(eng, torch, stream.cuda_stream)
    if args.conv_table and rank == 0:
        for r in sorted(rf["table"], key=lambda r: -r["us"]):
            print(f"{r['conv']:48s} {r['us']:8.1f} us {r['gbs']:7.0f} GB/s {r['tops']:6.0f} TOPS", file=sys.stderr)
    hbm, bf16, src = measured_peaks()
    int8_peak = 2.0 * bf16  # dense int8 tensor throughput is twice bf16 on B200
    achieved = rf["ops"] / rf["time_s"] / 1e12
    line = None
    if rank == 0:
        cpu = None
        if world == 1:
            os.environ["OMP_NUM_THREADS"] = str(host_cores())  # every host thread for the CPU baseline
            sample = args.cpu_sample or (160 if args.workload == "yolov8n-320" else 8)
            ips, dt = cpu_reference(program, sample)
            cpu = {"value": ips, "unit": "images/s", "cores": host_cores(), "kind": "port",
                   "sample": f"{sample} images through the CPU restatement of the reference's W8A8 "
                             f"arithmetic (oracle/, C/OpenMP int32 convolutions), {dt:.1f} s"}
        line = {
            "metric": metric, "value": total * args.steps / t_dev, "unit": "images/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": t_dev / args.steps * 1e3,
            "higher_is_better": True, "scaling": scaling, "vs_baseline": None, "dtype": "int8",
            "data": f"synthetic (uniform[0,1] fp16 images, seeded random-init {builder[6:]} weights)",
            "config": {"workload": workload, "global_batch": total, "per_gpu_batch": B, "imgsz": imgsz, "nc": nc,
                       "parallelism": f"dp{world} (independent replicas)",
                       "l2": f"inputs larger than L2 ({B * 3 * imgsz * imgsz * 2 / 1e6:.0f} MB of fp16 images "
                             "per step)",
                       **({"quant_on_load": True} if args.quant_on_load else {}),
                       "programmatic_launch": eng.programmatic,
                       **({"plan_bits": hex(args.plan_bits)} if args.plan_bits else {}),
                       "tiles": (f"autotuned: {os.path.relpath(tiles_path, ROOT)} ({len(tiles)} of the int8 convs "
                                 "off the default tile)" if tiles_path else "default heuristics")},
            "e2e": e2e,
            "gpu_launches": eng.launches_per_run * args.steps,
            "roofline": {"bound": "hbm", "achieved": rf["bytes"] / rf["time_s"] / 1e9, "peak": hbm, "unit": "GB/s",
                         "frac": rf["bytes"] / rf["time_s"] / 1e9 / hbm,
                         "traffic": (CONV_DRAM_BYTES_PER_IMAGE_B256 * B
                                     if B == 256 and args.workload == "yolov8n-320" else None),
                         "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum over the step's W8A8 "
                                           "conv launches at batch 256 (profiles/conv_family_dram_b256.md)",
                         "kernel": "conv_halo_kernel / conv_tc_kernel: all W8A8 conv launches of one step "
                                   "(algorithmic bytes: int8 input + fp16 output + weights per launch)",
                         "peak_source": f"{src} hbm_gbs from MEASURED_PEAKS.json",
                         "tensor_achieved_tops": achieved, "tensor_peak_tops": int8_peak,
                         "tensor_frac": achieved / int8_peak,
                         "tensor_peak_source": f"2 x {src} bf16 dense ({bf16} TFLOP/s), MEASURED_PEAKS.json",
                         "conv_ms_per_step": rf["time_s"] * 1e3, "conv_launches": rf["launches"]},
            "cpu_baseline": cpu,
            **({"latency": latency} if latency else {}),
            "clocks": clocks,
            "status": status,
        }
        print(json.dumps(line), flush=True)
    if dist is not None:
        eng.graph = None
        dist.barrier()
        dist.destroy_process_group()
    return 0


def run_engine(args):
    """An engine compiled by the reference, loaded and run through the C++ runtime (the
    NativeCppYoloModel interface): device-resident graph replays for `value`, and per step a
    synchronous aexrt_b200_yolo_run_batch (fp16 host images in the model's pinned staging buffer,
    detections read back) for `e2e`."""
    import ctypes

    import torch

    from aexrt_b200 import cpp_runtime

    torch.cuda.set_device(0)
    B = args.batch or 256
    m = cpp_runtime.NativeCppYoloModel(args.engine, 0, images=B)
    if args.algo_map or args.variants:
        from aexrt_b200 import autotune

        autotune.apply(m, args.algo_map, args.variants)
    m.set_input_dtype(True)
    imgsz = 320
    host = np.random.default_rng(1000).uniform(0, 1, (B, 3, imgsz, imgsz)).astype(np.float16)
    ptr = m.lib.aexrt_yolo_input_ptr(m.model, None)
    staging = np.ctypeslib.as_array(ctypes.cast(ptr, ctypes.POINTER(ctypes.c_uint16)), shape=(host.size,))
    staging[:] = host.reshape(-1).view(np.uint16)
    m.run_batch(host)  # uploads the images and warms up
    stream = torch.cuda.Stream()  # a stream of its own (handle 0 would select the model's stream)
    for _ in range(max(3, args.warmup)):
        m.enqueue(stream.cuda_stream)
    torch.cuda.synchronize()
    with ClockSampler(0) as clk:
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            m.enqueue(stream.cuda_stream)
        e1.record(stream)
        torch.cuda.synchronize()
        t_dev = e0.elapsed_time(e1) / 1e3
        # end to end: upload from pinned host memory, forward, detections back, per step
        rows = np.zeros((B, 100, 6), np.float32)
        counts = np.zeros(B, np.uint32)
        t0 = time.perf_counter()
        for _ in range(args.steps):
            ok = m.lib.aexrt_b200_yolo_run_batch(m.model, ptr, 1,
                                                 rows.ctypes.data_as(ctypes.POINTER(cpp_runtime.AexrtYoloDetection)),
                                                 100, counts.ctypes.data_as(ctypes.POINTER(ctypes.c_uint32)))
            assert ok, m.lib.aexrt_yolo_get_last_error(m.model)
        t_e2e = time.perf_counter() - t0
    _, det_bytes = m.device_detections()
    line = {"metric": METRIC + " (reference-compiled engine)", "value": B * args.steps / t_dev, "unit": "images/s",
            "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": t_dev / args.steps * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8",
            "data": "synthetic (uniform[0,1] fp16 images)",
            "config": {"workload": f"{os.path.basename(args.engine)} via the aexrt_yolo runtime ABI "
                                   "(reference-compiled W8A8 engine, its own int8/fp16 kernel plan)",
                       "algo_map": args.algo_map, "variants": args.variants,
                       "per_gpu_batch": B, "l2": "inputs larger than L2"},
            "e2e": {"value": B * args.steps / t_e2e, "unit": "images/s", "h2d_bytes_per_step": int(host.nbytes),
                    "d2h_bytes_per_step": int(det_bytes), "pipeline": "synchronous per step (one frame in flight)"},
            "gpu_launches": m.launch_count * args.steps, "arena_bytes": m.arena_bytes,
            "int8_convs": sum(1 for p in m.conv_plans() if p["current_algorithm"] in (51, 52, 53)),
            "status": m.status(), "clocks": clk.summary()}
    print(json.dumps(line), flush=True)
    m.close()
    return 0


def main():
    args = parse_args()
    if args.engine:
        return run_engine(args)
    if args.workload not in MODELS:
        return run_layer(args)
    if args.impl == "reference":
        # rank 0 alone runs the CPU reference: give it every host thread (torchrun exports
        # OMP_NUM_THREADS=1 to its workers), before the oracle's OpenMP runtime starts
        os.environ["OMP_NUM_THREADS"] = str(host_cores())
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
