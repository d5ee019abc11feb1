"""Per-device conv tuning of an ``.aexrt`` engine with a fail-closed numeric gate.

The reference tunes its engines with ``conv_autotune`` (examples/cpp/conv_autotune.cpp), a C++ tool
over the runtime ABI: per unique conv shape it tries every candidate algorithm the runtime lists
(``aexrt_yolo_conv_plan_info``, :198-215), accepts a candidate only if the detections of a run with
it match the baseline's (same count, |d score| <= 1e-3, |d corner| <= 0.05 px, :108-120), times the
accepted ones by the per-command GPU profile events (:88-104), keeps a winner only when it is more
than 5 % faster than the current algorithm (:336-345), applies all winners with incremental
rejection if the combination fails (:398-445), re-checks the tuned engine against the baseline
(final gate) and writes a report plus the ``{command: algorithm}`` map that ``aexrtc build
--algo-map`` compiles into the engine (:493-503).

This module runs the same procedure over the same ABI, served by ``libaexrt_b200.so``:

* the candidates are the W8A8 kernel of the shape (51 / 52 / 53, where the int8 guard passes) and
  the fp16 tensor-core conv, as the runtime lists them;
* a second, B200-only stage sweeps the tile choice of every conv that keeps an int8 or fp16 plan
  (output-channel tile, tile order, stacked M blocks: ``aexrt_b200_yolo_override_conv_variant``).
  For int8 plans those choices never change a result (integer accumulation); an fp16 plan moved
  between the halo and slot kernels sums K in another order.  Their gate is therefore stricter than
  the detections gate: output0 must equal the baseline's bit for bit, which rejects such fp16
  choices.  Winners go to a sidecar JSON (``--variants``) that
  :func:`apply` (or ``bench.py --engine ... --variants``) loads next to the algo map.

    python -m aexrt_b200.autotune ENGINE.aexrt [--images N] [--runs R] [--emit-map map.json]
        [--variants variants.json] [--report report.md] [--shape-limit K]
"""
from __future__ import annotations

import argparse
import json
import statistics
import time
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Tuple

import numpy as np

SCORE_TOL = 1e-3  # conv_autotune.cpp:108-120
BOX_TOL = 0.05
SIGNIFICANCE = 0.95  # a winner must take < 95 % of the current time (> 5 % faster)


def detections_match(a: Tuple[np.ndarray, np.ndarray], b: Tuple[np.ndarray, np.ndarray]) -> bool:
    """The reference's gate, per image: the same count, and rows in rank order within 1e-3 in score
    and 0.05 px in every corner."""
    (ra, ca), (rb, cb) = a, b
    if not np.array_equal(ca, cb):
        return False
    for i in range(len(ca)):
        x, y = ra[i, :ca[i]], rb[i, :cb[i]]
        if np.abs(x[:, 4] - y[:, 4]).max(initial=0) > SCORE_TOL or np.abs(x[:, :4] - y[:, :4]).max(initial=0) > BOX_TOL:
            return False
    return True


def shape_key(p: dict) -> tuple:
    d = p["desc"]  # AexrtConv2DDesc field order
    return (p["silu"], d[1], d[2], d[3], d[4], d[5], d[6], d[7], d[9], d[15], d[13])


def shape_str(key: tuple) -> str:
    silu, ic, ih, iw, oc, oh, ow, k, s, g, dil = key
    return f"{'silu' if silu else 'lin '} {ic}x{ih}x{iw} -> {oc}x{oh}x{ow} k{k}s{s} g{g} d{dil}"


@dataclass
class Row:
    key: tuple
    command: int
    current: int
    best: int
    current_ms: float = -1.0
    best_ms: float = -1.0
    blocked: List[int] = field(default_factory=list)
    variant: int = 0
    variant_ms: float = -1.0


class Tuner:
    def __init__(self, engine: str, images: int = 1, runs: int = 10, warmup: int = 3, seed: int = 0xC2A11,
                 log=print):
        from .cpp_runtime import NativeCppYoloModel

        self.engine, self.runs, self.warmup, self.log = engine, runs, warmup, log
        self.model = NativeCppYoloModel(engine, 0, images=images)
        self.model.set_profiling(True)
        rng = np.random.default_rng(seed)
        n = self.model.input_element_count // self.model.images
        side = int(round((n // 3) ** 0.5))
        self.input = rng.uniform(0, 1, (self.model.images, 3, side, side)).astype(np.float32)

    # ------------------------------------------------------------------ runs
    def run(self):
        """One run: (detections, counts, output0, host ms)."""
        t0 = time.perf_counter()
        rows, counts = self.model.run_batch(self.input)
        ms = (time.perf_counter() - t0) * 1e3
        return (rows, counts), self.model.output0(), ms

    def event_ms(self, command: int) -> float:
        """Median over `runs` runs of the command's own profile event (GPU time)."""
        prefix = f"cmd#{command} "
        samples = []
        for i in range(self.warmup + self.runs):
            self.run()
            if i < self.warmup:
                continue
            for label, ms in self.model.profile_events():
                if label.startswith(prefix):
                    samples.append(ms)
                    break
        return statistics.median(samples) if samples else -1.0

    # ------------------------------------------------------------------ stages
    def tune(self, shape_limit: int = 0, variants: bool = True):
        m = self.model
        for _ in range(self.warmup):
            self.run()
        self.base_dets, self.base_out, _ = self.run()
        self.base_ms = statistics.median(self.run()[2] for _ in range(self.runs))
        self.log(f"baseline e2e median {self.base_ms:.3f} ms, detections {int(self.base_dets[1].sum())}")
        plans = m.conv_plans()
        uniq: Dict[tuple, dict] = {}
        for p in plans:
            uniq.setdefault(shape_key(p), p)
        shapes = list(uniq.items())
        if shape_limit:
            shapes = shapes[:shape_limit]
        self.log(f"conv commands {len(plans)}, unique shapes {len(uniq)}, tuning {len(shapes)}")
        self.rows: List[Row] = []
        for key, p in shapes:
            row = Row(key, p["command_index"], p["current_algorithm"], p["current_algorithm"])
            if p["in_fusion_group"]:
                self.log(f"  {shape_str(key)}: [in fusion group] keep alg={row.current}")
                self.rows.append(row)
                continue
            row.current_ms = self.event_ms(row.command)
            results = []
            for alg in p["candidates"]:
                if alg == row.current:
                    continue
                m.override_conv_algorithm(row.command, alg)
                try:
                    dets, _, _ = self.run()
                    ok = detections_match(dets, self.base_dets)
                except RuntimeError:
                    ok = False
                if ok:
                    results.append((self.event_ms(row.command), alg))
                else:
                    row.blocked.append(alg)
                m.override_conv_algorithm(row.command, p["planned_algorithm"])
            best = min(results) if results else None
            if best and row.current_ms > 0 and best[0] < row.current_ms * SIGNIFICANCE:
                row.best, row.best_ms = best[1], best[0]
            else:
                row.best_ms = row.current_ms
            self.log(f"  {shape_str(key)}: alg {row.current} -> {row.best} ({row.current_ms:.4f} -> "
                     f"{row.best_ms:.4f} ms gpu), blocked {row.blocked}")
            self.rows.append(row)
        self.winners = self._winners(plans)
        self._apply_with_rejection()
        if variants:
            self._tune_variants()
        # final gate: the tuned engine against the baseline
        for _ in range(self.warmup):
            self.run()
        self.tuned_dets, self.tuned_out, _ = self.run()
        self.tuned_ms = statistics.median(self.run()[2] for _ in range(self.runs))
        self.final_gate = detections_match(self.tuned_dets, self.base_dets)
        self.log(f"tuned e2e median {self.tuned_ms:.3f} ms (baseline {self.base_ms:.3f}), final gate "
                 f"{'PASS' if self.final_gate else 'FAIL'}")
        return self.final_gate

    def _winners(self, plans) -> Dict[int, int]:
        best = {r.key: r.best for r in self.rows}
        out = {}
        for p in plans:
            b = best.get(shape_key(p))
            if b is not None and b != p["current_algorithm"] and not p["in_fusion_group"]:
                out[p["command_index"]] = b
        return out

    def _apply_with_rejection(self):
        """Applies every winner; while the combination fails to run or to pass the gate, drops the
        first remaining winner (conv_autotune.cpp:398-445)."""
        m = self.model
        planned = {p["command_index"]: p["planned_algorithm"] for p in m.conv_plans() if not p["in_fusion_group"]}
        live = dict(self.winners)
        while True:
            for cmd, alg in planned.items():
                m.override_conv_algorithm(cmd, live.get(cmd, alg))
            try:
                dets, _, _ = self.run()
                if detections_match(dets, self.base_dets):
                    break
            except RuntimeError as e:
                self.log(f"  combination failed: {e}")
            if not live:
                break
            cmd = next(iter(live))
            self.log(f"  rejecting winner cmd#{cmd} alg={live.pop(cmd)}")
        self.applied = live
        self.log(f"overrides applied: {len(live)}")

    def _variant_candidates(self, p: dict) -> List[int]:
        d = p["desc"]
        oc, k, s = d[4], d[7], d[9]
        bns = [b for b in (32, 64, 128, 256) if b <= max(32, 2 * oc)]
        cands = [bn for bn in bns] + [2 << 20, 1 << 20]
        if k == 3 and s == 1:
            cands.append(1 << 24)  # no stacked M blocks
        cands.append(1 << 29)  # staged epilogue: tiles written by TMA tensor stores (bit-identical)
        return cands

    def _tune_variants(self):
        """Tile choices per conv (results identical by construction: the gate is bit equality)."""
        m = self.model
        _, ref_out, _ = self.run()
        self.variants: Dict[int, int] = {}
        plans = {p["command_index"]: p for p in m.conv_plans()}
        seen = {}
        for row in self.rows:
            p = plans[row.command]
            base = self.event_ms(row.command)
            best = (base, 0)
            for bits in self._variant_candidates(p):
                try:
                    m.override_conv_variant(row.command, bits)
                    _, out, _ = self.run()
                except RuntimeError:
                    continue  # this tile does not fit the conv: the plan is refused
                if not np.array_equal(out, ref_out):
                    self.log(f"  cmd#{row.command} variant {bits:#x}: output differs, rejected")
                    continue
                t = self.event_ms(row.command)
                if t > 0 and t < best[0] * SIGNIFICANCE:
                    best = (t, bits)
            m.override_conv_variant(row.command, best[1])
            row.variant, row.variant_ms = best[1], best[0]
            if best[1]:
                seen[row.key] = best[1]
        # every command of a tuned shape takes the shape's winning tile
        for cmd, p in plans.items():
            bits = seen.get(shape_key(p))
            if bits:
                m.override_conv_variant(cmd, bits)
                self.variants[cmd] = bits
        _, out, _ = self.run()
        if not np.array_equal(out, ref_out):
            self.log("  variant combination changed output0: dropped")
            for cmd in self.variants:
                m.override_conv_variant(cmd, 0)
            self.variants = {}

    # ------------------------------------------------------------------ outputs
    def write(self, report: Optional[str] = None, algo_map: Optional[str] = None,
              variants: Optional[str] = None) -> None:
        if algo_map:
            with open(algo_map, "w") as f:
                json.dump({str(k): int(v) for k, v in sorted(self.winners.items())}, f, indent=4)
        if variants:
            with open(variants, "w") as f:
                json.dump({str(k): int(v) for k, v in sorted(getattr(self, "variants", {}).items())}, f, indent=4)
        if report:
            lines = ["# conv autotune report", "", f"- engine: {self.engine}",
                     f"- images per run: {self.model.images}",
                     f"- unique shapes tuned: {len(self.rows)}, overrides applied: {len(self.applied)}, "
                     f"tile variants: {len(getattr(self, 'variants', {}))}",
                     f"- baseline e2e median: {self.base_ms:.3f} ms; tuned: {self.tuned_ms:.3f} ms",
                     f"- final numeric gate: {'PASS' if self.final_gate else 'FAIL'}", "",
                     "| shape | current alg | best alg | current ms | best ms | blocked | tile bits | tile ms |",
                     "|---|---|---|---|---|---|---|---|"]
            for r in self.rows:
                lines.append(f"| {shape_str(r.key)} | {r.current} | {r.best} | {r.current_ms:.4f} | {r.best_ms:.4f} | "
                             f"{' '.join(map(str, r.blocked))} | {r.variant:#x} | {r.variant_ms:.4f} |")
            with open(report, "w") as f:
                f.write("\n".join(lines) + "\n")

    def close(self):
        self.model.close()


def apply(model, algo_map: Optional[str] = None, variants: Optional[str] = None) -> None:
    """Loads a tuned map (and the tile sidecar) into a NativeCppYoloModel."""
    if algo_map:
        for cmd, alg in json.load(open(algo_map)).items():
            model.override_conv_algorithm(int(cmd), int(alg))
    if variants:
        for cmd, bits in json.load(open(variants)).items():
            model.override_conv_variant(int(cmd), int(bits))


# built-in programs: builder, image size, classes (the bench's workloads)
PROGRAMS = {"yolov8n-320": ("build_yolov8n", 320, 4), "yolov8s-640": ("build_yolov8s", 640, 80),
            "yolov11s-320": ("build_yolov11s", 320, 80)}


def program_tile_candidates(c, bn_default: int) -> List[int]:
    """Tile choices of one int8 conv of a program: every output-channel tile the halo kernel has
    (16-256, at most twice the channels), then, around the best of those, strided and contiguous tile
    order, one or two stacked M blocks (3x3 stride 1) and the staged epilogue."""
    bns = [b for b in (16, 32, 64, 128, 256) if b <= max(32, 2 * c.oc) and (not c.pg16 or b in (64, 128))]
    return [b for b in bns if b != bn_default]


def tune_program(program, batch: int, runs: int = 10, log=print, seed: int = 0) -> Dict[str, int]:
    """Per-conv tile choice for a program compiled by :class:`aexrt_b200.engine.CompiledYolo` (the
    streaming engine the bench runs), on the current GPU.

    After one forward on seeded images every int8 conv's own inputs (codes and scale record) are in
    its scratch.  Each conv is then timed alone, ``runs`` back-to-back launches between one CUDA-event
    pair, with its default plan and with every candidate tile (:func:`program_tile_candidates`, then
    order / stacked-M / staged / two-issuer bits on the best tile).  A candidate must write the default
    plan's output bit for bit (integer accumulation makes every int8 tile exact, so the gate only
    rejects a broken plan) and is kept only when more than 5 % faster (the reference tuner's rule,
    ``conv_autotune.cpp:336-345``).  An int8 conv that can quantize its fp16 sources itself is then
    also timed that way against its best tile plus the separate quantize launch it replaces, and
    marked with ``engine.TILE_QUANT_ON_LOAD`` when that is more than 5 % faster (same codes, so the
    same output).  The fp16 convs that read their NHWC input directly (the detect head) are swept
    the same way, halo tiles only.  Returns ``{conv name: block_n bits}`` for
    ``CompiledYolo(block_n=...)``; convs whose default stays best are left out."""
    import torch

    from . import engine, ops
    from ._native import check

    eng = engine.CompiledYolo(program, batch)
    rng = np.random.default_rng(seed)
    imgs = torch.from_numpy(rng.uniform(0, 1, (batch, program.in_channels, program.imgsz, program.imgsz))
                            .astype(np.float16)).cuda()
    eng.forward(imgs)
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()

    def timed_fn(fn):
        fn()
        torch.cuda.synchronize()
        torch.cuda._sleep(20_000_000)  # the host enqueues every launch before the first one runs
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(runs):
            fn()
        e1.record(stream)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / runs

    def timed(plan, q, rec, c, out, res, amax_out):
        def once():
            if plan.is_f16:
                # fp16 head convs read the NHWC activation itself (q is that tensor)
                plan.run_nhwc(q, x_coff=c.inputs[0].coff, out=out, out_coff=c.out[1], residual=res,
                              res_coff=c.residual[1] if c.residual is not None else 0, amax_out=amax_out,
                              amax_goff=c.out[1] // 16, stream=stream.cuda_stream)
            else:
                plan.run(q, rec, out=out, out_coff=c.out[1], residual=res,
                         res_coff=c.residual[1] if c.residual is not None else 0, amax_out=amax_out,
                         amax_goff=c.out[1] // 16, stream=stream.cuda_stream)
        return timed_fn(once)

    chosen: Dict[str, int] = {}
    for st in eng.steps:
        if st[0] == "conv" and st[1].precision == "int8":
            _, c, plan0, _, (q, rec), (h, w) = st
        elif st[0] == "conv_nhwc":
            # fp16 stride-1 convs reading the NHWC activation: within the halo kernel every tile sums
            # K in the same order, so these are exact too (the gate still checks)
            _, c, plan0 = st
            q, rec = eng.values[c.inputs[0].value], None
            h, w = eng._spatial(c.inputs[0])
        else:
            continue
        out = eng.values[c.out[0]]
        res = eng.values[c.residual[0]] if c.residual is not None else None
        amax_out = eng._amax_view(c.out[0]) if c.out[0] in eng.needs_amax else None
        t0 = timed(plan0, q, rec, c, out, res, amax_out)
        ref = out[..., c.out[1]:c.out[1] + c.oc].clone()
        codes, scale = (None, None) if plan0.is_f16 else ops.quantize_conv_weight_int8(c.weight)

        def trial(bits):
            try:
                if plan0.is_f16:
                    plan = ops.ConvPlan.fp16(batch, c.ic, h, w, c.oc, c.k, c.s, c.weight, c.bias, silu=c.silu,
                                             block_n=bits)
                    if plan.info.variant != 2:
                        return None  # the slot kernel cannot read NHWC (and sums K in another order)
                else:
                    plan = ops.ConvPlan.int8(batch, c.ic, h, w, c.oc, c.k, c.s, codes, scale, c.bias,
                                             silu=c.silu, pg16=c.pg16, block_n=bits)
            except RuntimeError:
                return None  # this tile does not fit the conv: the plan is refused
            out[..., c.out[1]:c.out[1] + c.oc].fill_(0.0)
            t = timed(plan, q, rec, c, out, res, amax_out)
            if plan.status() != 0 or not torch.equal(out[..., c.out[1]:c.out[1] + c.oc], ref):
                log(f"  {c.name} bits {bits:#x}: output differs, rejected")
                return None
            return t

        bn0 = plan0.info.block_n
        best_t, best_bits = t0, 0
        for bn in program_tile_candidates(c, bn0):
            t = trial(bn)
            if t is not None and t < best_t:
                best_t, best_bits = t, bn
        base = best_bits or bn0
        extra = [base | (1 << 20), base | (2 << 20), base | (1 << 29), base | (1 << 30)]
        if c.k == 3 and c.s == 1 and base <= 64:
            extra += [base | (1 << 24), base | (2 << 24)]
        for bits in extra:
            t = trial(bits)
            if t is not None and t < best_t:
                best_t, best_bits = t, bits
        if not (best_bits and best_t < t0 * SIGNIFICANCE):
            best_t, best_bits = t0, 0
        note = ""
        if not plan0.is_f16 and engine.ql_eligible(c):
            # quantize on load: the conv quantizes its fp16 sources itself and the quantize launch
            # before it goes away, so it competes with that launch and the conv together
            srcs = st[3]
            lib = eng.lib

            def quantize():
                check(lib.aexrt_b200_act_quantize_concat(srcs, len(srcs), batch, h, w, int(c.pg16), c.s, q.data_ptr(),
                                                         rec.data_ptr(), stream.cuda_stream), "quantize")

            tq = timed_fn(quantize)
            ql_bits = best_bits | engine.TILE_QUANT_ON_LOAD
            try:
                plan = ops.ConvPlan.int8(batch, c.ic, h, w, c.oc, c.k, c.s, codes, scale, c.bias, silu=c.silu,
                                         pg16=c.pg16, block_n=best_bits, quant_on_load=True)
            except RuntimeError:
                plan = None
            if plan is not None and plan.info.quant_on_load:
                out[..., c.out[1]:c.out[1] + c.oc].fill_(0.0)
                t = timed_fn(lambda: plan.run_sources(
                    srcs, out=out, out_coff=c.out[1], residual=res,
                    res_coff=c.residual[1] if c.residual is not None else 0, amax_out=amax_out,
                    amax_goff=c.out[1] // 16, stream=stream.cuda_stream))
                if plan.status() != 0 or not torch.equal(out[..., c.out[1]:c.out[1] + c.oc], ref):
                    log(f"  {c.name} quantize on load: output differs, rejected")
                elif t < (best_t + tq) * SIGNIFICANCE:
                    note = f" (quantize on load: {(best_t + tq) * 1e3:.1f} -> {t * 1e3:.1f} us with the quantize)"
                    best_bits = ql_bits
        out[..., c.out[1]:c.out[1] + c.oc].copy_(ref)
        if best_bits:
            chosen[c.name] = best_bits
            log(f"{c.name}: {t0 * 1e3:.1f} -> {best_t * 1e3:.1f} us with bits {best_bits:#x}{note}")
        else:
            log(f"{c.name}: {t0 * 1e3:.1f} us, default kept")
    return chosen


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("engine", nargs="?", default=None)
    ap.add_argument("--program", default=None,
                    help="instead of an engine: tune the tiles of a built-in program (yolov8n-320, yolov8s-640, "
                         "yolov11s-320) compiled for --batch by the streaming engine; writes --tiles-out")
    ap.add_argument("--batch", type=int, default=256)
    ap.add_argument("--tiles-out", default=None, help="--program: JSON {conv name: block_n bits}")
    ap.add_argument("--images", type=int, default=1)
    ap.add_argument("--runs", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--shape-limit", type=int, default=0)
    ap.add_argument("--no-variants", action="store_true")
    ap.add_argument("--emit-map", default=None, help="JSON {command: algorithm} for aexrtc build --algo-map")
    ap.add_argument("--variants", default=None, help="JSON {command: tile bits} of this backend")
    ap.add_argument("--report", default=None)
    a = ap.parse_args(argv)
    if a.program:
        from . import yolo

        builder, imgsz, nc = PROGRAMS[a.program]
        tiles = tune_program(getattr(yolo, builder)(nc=nc, imgsz=imgsz, seed=0), a.batch, runs=a.runs)
        if a.tiles_out:
            with open(a.tiles_out, "w") as f:
                json.dump(tiles, f, indent=1, sort_keys=True)
        print(json.dumps(tiles))
        return 0
    if a.engine is None:
        ap.error("an engine file or --program is required")
    t = Tuner(a.engine, a.images, a.runs, a.warmup)
    ok = t.tune(a.shape_limit, variants=not a.no_variants)
    t.write(a.report, a.emit_map, a.variants)
    t.close()
    return 0 if ok else 3


if __name__ == "__main__":
    raise SystemExit(main())
