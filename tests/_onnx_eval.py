"""A plain numpy evaluator of the ONNX operators a YOLO export uses (test infrastructure).

It runs an ONNX graph in fp32 by the operator definitions of the ONNX specification (Conv with
groups, Sigmoid, Mul, Add, Sub, Div, Split, Slice, Concat, Resize nearest, MaxPool, Reshape,
Transpose, Softmax, Identity), so that the graphs `aexrt_b200.onnx_yolo.export_onnx` writes can
be checked against the oracle independently of the importer.
"""
import numpy as np

from aexrt_b200 import onnx_proto as op


def _conv(x, w, b, a):
    s = a.get("strides", [1, 1])
    pads = a.get("pads", [0, 0, 0, 0])
    g = a.get("group", 1)
    n, c, h, wd = x.shape
    oc, icg, kh, kw = w.shape
    xp = np.zeros((n, c, h + pads[0] + pads[2], wd + pads[1] + pads[3]), np.float32)
    xp[:, :, pads[0]:pads[0] + h, pads[1]:pads[1] + wd] = x
    oh = (h + pads[0] + pads[2] - kh) // s[0] + 1
    ow = (wd + pads[1] + pads[3] - kw) // s[1] + 1
    out = np.zeros((n, oc, oh, ow), np.float32)
    ocg = oc // g
    for gi in range(g):
        xs = xp[:, gi * icg:(gi + 1) * icg]
        ws = w[gi * ocg:(gi + 1) * ocg]
        for i in range(kh):
            for j in range(kw):
                patch = xs[:, :, i:i + (oh - 1) * s[0] + 1:s[0], j:j + (ow - 1) * s[1] + 1:s[1]]
                out[:, gi * ocg:(gi + 1) * ocg] += np.einsum("nchw,oc->nohw", patch, ws[:, :, i, j], optimize=True)
    if b is not None:
        out += b.reshape(1, -1, 1, 1)
    return out


def _maxpool(x, a):
    k, s, p = a["kernel_shape"], a.get("strides", [1, 1]), a.get("pads", [0, 0, 0, 0])
    n, c, h, w = x.shape
    xp = np.full((n, c, h + p[0] + p[2], w + p[1] + p[3]), -np.inf, np.float32)
    xp[:, :, p[0]:p[0] + h, p[1]:p[1] + w] = x
    oh, ow = (h + p[0] + p[2] - k[0]) // s[0] + 1, (w + p[1] + p[3] - k[1]) // s[1] + 1
    out = np.full((n, c, oh, ow), -np.inf, np.float32)
    for i in range(k[0]):
        for j in range(k[1]):
            out = np.maximum(out, xp[:, :, i:i + (oh - 1) * s[0] + 1:s[0], j:j + (ow - 1) * s[1] + 1:s[1]])
    return out


def run(model, feeds):
    env = {t.name: op.to_array(t) for t in model.graph.initializer}
    env.update({k: np.asarray(v, np.float32) for k, v in feeds.items()})
    for nd in model.graph.node:
        a = op.attrs(nd)
        x = [env[t] if t else None for t in nd.input]
        t = nd.op_type
        if t == "Conv":
            y = [_conv(x[0], x[1], x[2] if len(x) > 2 else None, a)]
        elif t == "Sigmoid":
            y = [(1.0 / (1.0 + np.exp(-x[0]))).astype(np.float32)]
        elif t in ("Mul", "Add", "Sub", "Div"):
            f = {"Mul": np.multiply, "Add": np.add, "Sub": np.subtract, "Div": np.divide}[t]
            y = [f(x[0], x[1]).astype(np.float32)]
        elif t == "Split":
            sizes = list(x[1]) if len(x) > 1 and x[1] is not None else a["split"]
            y = np.split(x[0], np.cumsum(sizes)[:-1], axis=a.get("axis", 0))
        elif t == "Concat":
            y = [np.concatenate(x, axis=a["axis"])]
        elif t == "Resize":
            sc = [int(v) for v in x[2]]
            y = [x[0].repeat(sc[2], axis=2).repeat(sc[3], axis=3)]
        elif t == "MaxPool":
            y = [_maxpool(x[0], a)]
        elif t == "Reshape":
            y = [x[0].reshape([int(v) for v in x[1]])]
        elif t == "Transpose":
            y = [x[0].transpose(a["perm"])]
        elif t == "Softmax":
            e = np.exp(x[0] - x[0].max(axis=a.get("axis", -1), keepdims=True))
            y = [(e / e.sum(axis=a.get("axis", -1), keepdims=True)).astype(np.float32)]
        elif t == "Identity":
            y = [x[0]]
        else:
            raise NotImplementedError(t)
        for name, v in zip(nd.output, y):
            env[name] = v
    return {o.name: env[o.name] for o in model.graph.output}
