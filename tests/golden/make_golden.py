"""Generate the golden fixtures under tests/golden/ (run in the build container).

Two kinds of fixture are written:

1. ``weights_layout8.npz`` — layout-8 payloads produced by the REFERENCE'S OWN
   weight quantizer ``_add_packed_conv_int8`` (src/aexrt/engine.py:2418-2465),
   imported from the reference source tree, for seeded weights including edge
   cases (an all-zero output channel, exact half-way products, fp16 engines).
   These pin ``oracle.w8a8.quantize_conv_weight_int8`` and the product's
   weight packer bit-for-bit.
2. ``tiny_w8a8.aexrt`` + ``tiny_w8a8.npz`` — a small engine compiled by the
   reference's ``build_aexrt_engine`` with algo overrides 51/52/53 and one
   pg16 command, plus the graph's constants.  They pin the kernel-plan record
   semantics (kernel id, flags) and the packed-weight section format the
   product's engine reader consumes.
3. ``act_cases.npz`` — seeded activation / conv cases run through the CPU
   oracle (amax, int8 codes, int32 accumulators, fp32/fp16 outputs).  The
   reference has no W8A8 golden vectors of its own, so these are regression
   pins of the restatement, not of the reference.
4. ``yolo_post.npz`` — synthetic YOLO output0 tensors (clustered boxes, so NMS
   has work) and the detections that the REFERENCE'S OWN ``yolo_postprocess``
   (src/aexrt/yolo.py:92-138) returns for them.  They pin the greedy mode of
   the post-process oracle and kernel.

Usage (needs the reference source tree, which only the build container has)::

    python tests/golden/make_golden.py --reference-src <reference>/src
"""
from __future__ import annotations

import argparse
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))


def _silu(z):
    return z / (1.0 + np.exp(-z))


def weight_cases():
    rng = np.random.default_rng(1234)
    cases = []
    for i, (shape, prec) in enumerate([
        ((32, 16, 3, 3), 1), ((32, 16, 3, 3), 2), ((16, 32, 1, 1), 1), ((24, 16, 3, 3), 2),
        ((16, 48, 1, 1), 2), ((32, 32, 3, 3), 1),
    ]):
        w = rng.normal(0.0, 0.05, shape).astype(np.float32)
        if i == 0:
            w[3] = 0.0  # all-zero channel -> scale 1.0
            # exact half-way products: amax 1.27 -> scale 0.01, inv 100 -> 0.005*100 = 0.5
            w[5] = 0.0
            w[5, 0, 0, 0] = 1.27
            w[5, 1, 0, 0] = 0.005
            w[5, 2, 0, 0] = -0.015
        cases.append((w, prec))
    return cases


def make_weights(ref_engine):
    out = {}
    for i, (w, prec) in enumerate(weight_cases()):
        oc, ic, kh, kw = w.shape
        packed = {}
        values = [{"raw": w.astype("<f4").tobytes()}]
        ref_engine._add_packed_conv_int8(
            packed, values, weight_id=0, in_channels=ic, out_channels=oc,
            kernel_elems=kh * kw, precision=prec,
        )
        out[f"w{i}"] = w
        out[f"prec{i}"] = np.int32(prec)
        out[f"payload{i}"] = np.frombuffer(packed[0]["data"], dtype=np.uint8)
    out["count"] = np.int32(len(weight_cases()))
    np.savez_compressed(os.path.join(HERE, "weights_layout8.npz"), **out)


def make_tiny_engine(aexrt):
    """conv3x3 s1 16->32 (pg16) -> conv3x3 s2 32->32 -> conv1x1 32->16 -> rank-3 output."""
    rng = np.random.default_rng(7)
    g = aexrt.Graph("tiny_w8a8")
    g.input("images", aexrt.TensorSpec((1, 16, 16, 16), "float32"))
    consts = {}

    def conv(name, x, ic, oc, k, s):
        w = rng.normal(0, 0.05, (oc, ic, k, k)).astype(np.float32)
        b = rng.normal(0, 0.1, (oc,)).astype(np.float32)
        g.const(name + ".w", w)
        g.const(name + ".b", b)
        consts[name + ".w"] = w
        consts[name + ".b"] = b
        p = k // 2
        g.conv2d(name + ".c", x, name + ".w", name + ".b", strides=(s, s), pads=(p, p, p, p))
        g.sigmoid(name + ".s", name + ".c")
        g.mul(name + ".y", name + ".c", name + ".s")
        return name + ".y"

    y = conv("l0", "images", 16, 32, 3, 1)
    y = conv("l1", y, 32, 32, 3, 2)
    y = conv("l2", y, 32, 8, 1, 1)
    g.reshape("out", y, [1, 8, 64])
    g.output("out")
    eng = aexrt.build_aexrt_engine(
        g, algo_overrides={0: 52, 1: 53, 2: 51}, int8_pergroup=[0], precision="fp16",
    )
    with open(os.path.join(HERE, "tiny_w8a8.aexrt"), "wb") as f:
        f.write(eng)
    info = aexrt.inspect_aexrt_engine(eng)
    plan = np.array(info["kernel_plan"], dtype=np.uint32)
    np.savez_compressed(os.path.join(HERE, "tiny_w8a8.npz"), kernel_plan=plan, **consts)


def engine_program():
    """The YOLOv8n-320 program that yolov8n_w8a8.aexrt is compiled from: BASELINE config 3's model
    (nc=4) with its weights and biases rounded to fp16 (an fp16 engine stores them so, and the
    reference quantizer rounds fp16-engine weights through fp16 before the int8 step), and the one
    concat + 1x1 that the reference compiler keeps fused (l2.cv2, an 80x80 output) in fp16."""
    sys.path.insert(0, ROOT)
    from aexrt_b200 import yolo

    prog = yolo.build_yolov8n(nc=4, imgsz=320, seed=0)
    for c in prog.commands:
        if isinstance(c, yolo.ConvCmd):
            c.weight = c.weight.astype(np.float16).astype(np.float32)
            c.bias = c.bias.astype(np.float16).astype(np.float32)
    int8 = {c.name for c in prog.commands
            if isinstance(c, yolo.ConvCmd) and c.precision == "int8" and c.name != "l2.cv2"}
    yolo.apply_algo_map(prog, int8=int8)
    return prog


def program_graph(aexrt, prog):
    """The program as an ONNX-export-style graph (Conv + Sigmoid + Mul, Split, Add, Concat,
    Resize, MaxPool, and the Detect head's per-level Concat, Reshape and DFL decode), so that the
    reference compiler lowers it like an exported YOLOv8.  Returns (graph, {conv name: the conv's own
    output tensor, before any residual Add}).  The merged head convs of the program are split back
    into the model's separate box and class branches (the same weights)."""
    from aexrt_b200 import yolo

    g = aexrt.Graph(prog.name)
    n_img, size = 1, prog.imgsz
    g.input("images", aexrt.TensorSpec((n_img, 3, size, size), "float32"))
    segs = {}            # value -> list of (coff, channels, tensor)
    conv_out = {}
    counter = [0]

    def fresh(base):
        counter[0] += 1
        return f"{base}#{counter[0]}"

    def conv_node(name, x, w, b, k, s, silu):
        g.const(name + ".w", w)
        g.const(name + ".b", b)
        p = k // 2
        g.conv2d(name + ".c", x, name + ".w", name + ".b", strides=(s, s), pads=(p, p, p, p))
        y = name + ".c"
        if silu:
            g.sigmoid(name + ".s", name + ".c")
            g.mul(name + ".y", name + ".c", name + ".s")
            y = name + ".y"
        conv_out[name] = y
        return y

    def tensor(value, coff, ch):
        if value == "images":
            return "images"
        parts = sorted(segs[value])
        for (o, c, t) in parts:
            if (o, c) == (coff, ch):
                return t
        for (o, c, t) in parts:  # a chunk of one segment: Split it (C2f's chunk(2, 1))
            if o <= coff and coff + ch <= o + c and c % ch == 0 and (coff - o) % ch == 0:
                outs = [fresh(t + ".chunk") for _ in range(c // ch)]
                g.node("Split", outs, t, axis=1, split=[ch] * (c // ch))
                segs[value].remove((o, c, t))
                segs[value].extend((o + i * ch, ch, outs[i]) for i in range(c // ch))
                return outs[(coff - o) // ch]
        pieces = [t for (o, c, t) in parts if coff <= o and o + c <= coff + ch]
        assert sum(c for (o, c, t) in parts if coff <= o and o + c <= coff + ch) == ch, (value, coff, ch)
        out = fresh(value + ".cat")
        g.concat(out, *pieces, axis=1)
        return out

    def gather(inputs):
        xs = []
        for pt in inputs:
            t = tensor(pt.value, pt.coff, pt.channels)
            if pt.upsample != 1:
                up = fresh(t + ".up")
                g.node("Resize", up, t, mode="nearest", scales=[1.0, 1.0, float(pt.upsample), float(pt.upsample)])
                t = up
            xs.append(t)
        if len(xs) == 1:
            return xs[0]
        out = fresh("cat")
        g.concat(out, *xs, axis=1)
        return out

    levels = []
    for c in prog.commands:
        if isinstance(c, yolo.ConvCmd):
            if ".cv23_" in c.name or ".cv2_1" in c.name or ".cv3_1" in c.name:
                continue  # the head: below
            x = gather(c.inputs)
            y = conv_node(c.name, x, c.weight, c.bias, c.k, c.s, c.silu)
            if c.residual is not None:
                r = tensor(c.residual[0], c.residual[1], c.oc)
                g.add(c.name + ".add", r, y)  # Bottleneck: x + cv2(cv1(x))
                y = c.name + ".add"
            segs.setdefault(c.out[0], []).append((c.out[1], c.oc, y))
        elif isinstance(c, yolo.SppfCmd):
            x = tensor(c.x.value, c.x.coff, c.x.channels)
            m = x
            for i in range(3):
                nm = f"{c.name}.pool{i}"
                g.node("MaxPool", nm, m, kernel_shape=[5, 5], strides=[1, 1], pads=[2, 2, 2, 2])
                segs.setdefault(c.out[0], []).append((c.out[1] + i * c.x.channels, c.x.channels, nm))
                m = nm
        elif isinstance(c, yolo.DecodeCmd):
            levels = c.levels
    # Detect head per level: cv2 (box: 3x3, 3x3, 1x1 -> 64) and cv3 (class: 3x3, 3x3, 1x1 -> nc),
    # then Concat(box, class) along channels
    by_name = {c.name: c for c in prog.commands if isinstance(c, yolo.ConvCmd)}
    reg = 4 * prog.reg_max
    flat = []
    for i, (bp, cp, stride) in enumerate(levels):
        pre = bp.value.rsplit(".", 1)[0]                    # "l22.<i>"
        c0, c1b, c1c, c2 = (by_name[pre + sfx] for sfx in (".cv23_0", ".cv2_1", ".cv3_1", ".cv23_2"))
        feat = gather(c0.inputs)
        c2n = c1b.ic
        hb = conv_node(pre + ".cv2_0", feat, c0.weight[:c2n], c0.bias[:c2n], 3, 1, True)
        hc = conv_node(pre + ".cv3_0", feat, c0.weight[c2n:], c0.bias[c2n:], 3, 1, True)
        hb = conv_node(pre + ".cv2_1", hb, c1b.weight, c1b.bias, 3, 1, True)
        hc = conv_node(pre + ".cv3_1", hc, c1c.weight, c1c.bias, 3, 1, True)
        box = conv_node(pre + ".cv2_2", hb, c2.weight[:reg, :c2n], c2.bias[:reg], 1, 1, False)
        cls = conv_node(pre + ".cv3_2", hc, c2.weight[reg:reg + prog.nc, c2n:], c2.bias[reg:reg + prog.nc], 1, 1,
                        False)
        cat = f"{pre}.cat"
        g.concat(cat, box, cls, axis=1)
        v = prog.values[bp.value]
        g.reshape(f"{pre}.flat", cat, [n_img, reg + prog.nc, v.h * v.w])
        flat.append((f"{pre}.flat", v.h, v.w, stride))
    # DFL decode to output0 [1, 4 + nc, anchors] (the exported model's tail; an engine's YOLO head
    # fusion replaces everything from the level concat on)
    anchors = sum(h * w for _, h, w, _ in flat)
    g.concat("head", *[f for f, _, _, _ in flat], axis=2)
    g.node("Split", ["box", "cls"], "head", axis=1, split=[reg, prog.nc])
    g.reshape("box4", "box", [n_img, 4, prog.reg_max, anchors])
    g.transpose("boxt", "box4", [0, 2, 1, 3])
    g.softmax("boxp", "boxt", axis=1)
    g.const("dfl.w", np.arange(prog.reg_max, dtype=np.float32).reshape(1, prog.reg_max, 1, 1))
    g.conv2d("dist4", "boxp", "dfl.w")
    g.reshape("dist", "dist4", [n_img, 4, anchors])
    g.node("Slice", "lt", "dist", starts=[0], ends=[2], axes=[1])
    g.node("Slice", "rb", "dist", starts=[2], ends=[4], axes=[1])
    pts = np.concatenate([np.stack(np.meshgrid(np.arange(w) + 0.5, np.arange(h) + 0.5, indexing="xy"), 0).reshape(2, -1)
                          for _, h, w, _ in flat], axis=1).astype(np.float32)[None]
    strides = np.concatenate([np.full(h * w, st, np.float32) for _, h, w, st in flat])[None]
    g.const("anchor_points", pts)
    g.const("stride_tensor", strides)
    g.const("half", np.array([0.5], np.float32))
    g.sub("x1y1", "anchor_points", "lt")
    g.add("x2y2", "anchor_points", "rb")
    g.add("cxy2", "x1y1", "x2y2")
    g.mul("cxy", "cxy2", "half")
    g.sub("wh", "x2y2", "x1y1")
    g.concat("xywh", "cxy", "wh", axis=1)
    g.mul("dbox", "xywh", "stride_tensor")
    g.sigmoid("prob", "cls")
    g.concat("output0", "dbox", "prob", axis=1)
    g.output("output0")
    return g, conv_out


def make_yolov8n_engine(aexrt):
    """yolov8n_w8a8.aexrt: the engine_program() model compiled by the reference's build_aexrt_engine
    with an algo map of 51/52/53 on every int8-capable conv (the map `aexrtc build --algo-map` takes),
    fp16 precision, and the concat + conv un-fusion the reference applies for int8 builds
    (AEXRTC_UNFUSE_SMALL_CONCAT=2).  yolov8n_w8a8.json holds the command -> kernel map and the
    conv command -> program conv name table."""
    import json

    from aexrt import engine as ref_engine
    from aexrt import yolo as ref_yolo

    prog = engine_program()
    g, conv_out = program_graph(aexrt, prog)
    os.environ["AEXRTC_UNFUSE_SMALL_CONCAT"] = "2"
    pkg = ref_yolo.build_yolo_native_d3d12_graph_package(g, classes=prog.nc)
    replay = ref_engine._parse_replay_text(str(pkg["cxx_replay_text"]))
    names = {}
    for line in str(pkg["cxx_replay_text"]).splitlines():
        f = line.split("|")
        if f[0] in ("INPUT", "VALUE", "CONST"):
            names[int(f[1])] = f[2]
    tensor_conv = {t: n for n, t in conv_out.items()}
    int8_names = {c.name for c in prog.commands if getattr(c, "precision", "") == "int8"}
    algo, cmd_conv = {}, {}
    for i, cmd in enumerate(replay["commands"]):
        if cmd["kind"] not in ("CONV", "CONV_SILU"):
            continue
        conv = tensor_conv.get(names[int(cmd["output"])])
        if conv is None:
            continue
        cmd_conv[i] = conv
        if conv in int8_names:
            desc = cmd["params"][:16]
            algo[i] = 51 if desc[7] == 1 else (52 if desc[9] == 1 else 53)
    eng = aexrt.build_aexrt_engine(g, classes=prog.nc, precision="fp16", algo_overrides=algo)
    with open(os.path.join(HERE, "yolov8n_w8a8.aexrt"), "wb") as f:
        f.write(eng)
    info = aexrt.inspect_aexrt_engine(eng)
    with open(os.path.join(HERE, "yolov8n_w8a8.json"), "w") as f:
        json.dump({"algo_map": {str(k): v for k, v in sorted(algo.items())},
                   "conv_commands": {str(k): v for k, v in sorted(cmd_conv.items())},
                   "kernel_plan": [list(map(int, r)) for r in info["kernel_plan"]]}, f, indent=1)


def make_act_cases():
    sys.path.insert(0, ROOT)
    from oracle import w8a8 as ow

    rng = np.random.default_rng(2024)
    out = {}
    specs = [
        # name, N, IC, H, W, OC, K, S, mode, silu, residual
        ("c3s1_pt", 2, 32, 10, 12, 32, 3, 1, 0, True, False),
        ("c3s1_pg", 2, 32, 10, 12, 32, 3, 1, 1, True, False),
        ("c3s2_pt", 2, 16, 12, 14, 32, 3, 2, 0, True, False),
        ("c3s2_pg", 1, 48, 9, 11, 16, 3, 2, 1, True, False),
        ("c1_pt", 2, 48, 7, 9, 32, 1, 1, 0, True, False),
        ("c1_pg", 2, 32, 7, 9, 48, 1, 1, 1, False, False),
        ("c3s1_res", 2, 16, 8, 8, 16, 3, 1, 0, True, True),
    ]
    for name, n, ic, h, w, oc, k, s, mode, silu, res in specs:
        x = _silu(rng.standard_normal((n, ic, h, w)).astype(np.float32)).astype(np.float16)
        if name == "c3s1_pt":
            x[1] = 0  # an all-zero image: amax 0 -> zero codes
        wt = rng.normal(0, 0.05, (oc, ic, k, k)).astype(np.float32)
        b = rng.normal(0, 0.1, (oc,)).astype(np.float32)
        p = k // 2
        oh, ow_ = ow.conv_out_hw(h, w, k, s, p)
        r = rng.standard_normal((n, oc, oh, ow_)).astype(np.float16) if res else None
        o = ow.conv_w8a8(x, wt, b, k, s, p, mode=mode, silu=silu, residual=r)
        meta = np.array([n, ic, h, w, oc, k, s, p, mode, int(silu), int(res)], dtype=np.int32)
        out[name + ".meta"] = meta
        out[name + ".x"] = x
        out[name + ".w"] = wt
        out[name + ".b"] = b
        if r is not None:
            out[name + ".res"] = r
        for key in ("amax_t", "amax_g", "xq", "wq", "w_scale", "acc", "y"):
            out[name + "." + key] = o[key]
    out["names"] = np.array([s[0] for s in specs])
    np.savez_compressed(os.path.join(HERE, "act_cases.npz"), **out)


def synthetic_head_output(rng, nc: int, anchors: int, objects: int, imgsz: float = 320.0) -> np.ndarray:
    """One image's output0 [4 + nc][anchors] float32: anchors scattered around `objects` boxes
    (jittered copies of each, so neighbours overlap) plus background anchors with low class
    scores.  Scores are continuous, so ties (whose order the reference leaves to numpy's sort)
    do not occur."""
    sig = lambda z: 1.0 / (1.0 + np.exp(-z))  # noqa: E731
    ctr = rng.uniform(0, imgsz, (objects, 2))
    size = rng.uniform(8, 120, (objects, 2))
    cls = rng.integers(0, nc, objects)
    owner = rng.integers(-objects, objects, anchors)  # negative: background anchor
    y = np.empty((4 + nc, anchors), dtype=np.float32)
    fg = owner >= 0
    o = np.where(fg, owner, 0)
    y[0] = np.where(fg, ctr[o, 0] + rng.normal(0, 0.08, anchors) * size[o, 0], rng.uniform(0, imgsz, anchors))
    y[1] = np.where(fg, ctr[o, 1] + rng.normal(0, 0.08, anchors) * size[o, 1], rng.uniform(0, imgsz, anchors))
    y[2] = np.where(fg, size[o, 0] * np.exp(rng.normal(0, 0.15, anchors)), rng.uniform(4, 60, anchors))
    y[3] = np.where(fg, size[o, 1] * np.exp(rng.normal(0, 0.15, anchors)), rng.uniform(4, 60, anchors))
    logits = rng.normal(-4.0, 1.5, (nc, anchors))
    logits[cls[o[fg]], np.nonzero(fg)[0]] = rng.normal(1.0, 1.5, int(fg.sum()))
    y[4:] = sig(logits)
    return y


POST_CASES = [
    # name, nc, anchors, objects, conf, iou, seed
    ("nc4_a", 4, 1000, 12, 0.25, 0.45, 11),
    ("nc4_b", 4, 1000, 30, 0.25, 0.45, 12),
    ("nc4_iou07", 4, 1000, 20, 0.25, 0.7, 13),
    ("nc20_conf01", 20, 600, 16, 0.1, 0.45, 14),
    ("nc1", 1, 800, 25, 0.3, 0.5, 15),
]


def make_post_cases(ref_yolo):
    out = {}
    for name, nc, anchors, objects, conf, iou, seed in POST_CASES:
        y = synthetic_head_output(np.random.default_rng(seed), nc, anchors, objects)
        dets = ref_yolo.yolo_postprocess(y[None], conf, iou, layout="channels_first",
                                         objectness=False)
        rows = np.array([list(d.xyxy) + [d.score, d.class_id] for d in dets], dtype=np.float32).reshape(-1, 6)
        out[name + ".y"] = y
        out[name + ".meta"] = np.array([nc, conf, iou], dtype=np.float64)
        out[name + ".dets"] = rows
    out["names"] = np.array([c[0] for c in POST_CASES])
    np.savez_compressed(os.path.join(HERE, "yolo_post.npz"), **out)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference-src", default=None, help="path to the reference's src/ directory")
    ap.add_argument("--only", default=None, choices=["weights", "engine", "act", "post", "yolov8n"])
    args = ap.parse_args()
    want = lambda k: args.only in (None, k)  # noqa: E731
    if args.reference_src:
        sys.path.insert(0, args.reference_src)
        import aexrt
        from aexrt import engine as ref_engine
        from aexrt import yolo as ref_yolo

        if want("weights"):
            make_weights(ref_engine)
        if want("engine"):
            make_tiny_engine(aexrt)
        if want("post"):
            make_post_cases(ref_yolo)
        if want("yolov8n"):
            make_yolov8n_engine(aexrt)
    if want("act"):
        make_act_cases()


if __name__ == "__main__":
    main()
