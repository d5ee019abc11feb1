"""GPU parity of the YOLOv11s graph against the CPU oracle.

* the two fp16 ops it adds: the depthwise 3x3 conv against a plain PyTorch fp32 grouped conv of
  the fp16-rounded operands, and the C2PSA attention core against the oracle's restatement;
* per layer, fed the device's own inputs: int8 codes bit-exact and fp16 outputs within max-abs
  1e-2 for every conv (C3k2, C3k, SPPF, the C2PSA qkv / proj / ffn convs on the W8A8 path), the
  depthwise convs and the attention within 1e-2;
* end to end from the same images: class scores within 0.02, boxes within a few pixels, and the
  detections of the GPU post-process equal the oracle's post-process of the device's own output0.
"""
import numpy as np
import pytest

from oracle import yolo_model as om
from tests._util import nchw_to_nhwc, nhwc_to_nchw, slab16_to_nchw

pytestmark = pytest.mark.gpu


def _torch():
    import torch

    return torch


@pytest.mark.parametrize("n,c,h,w,s,silu,grp,gstride,goff,ldc,coff", [
    (2, 64, 20, 20, 1, True, 0, 0, 0, 64, 0),
    (2, 128, 13, 11, 2, True, 0, 0, 0, 160, 32),     # stride 2, odd map, a slice of a wider buffer
    (2, 256, 10, 10, 1, False, 64, 128, 64, 512, 0),  # the C2PSA pe: per-head v channels of the qkv tensor
])
def test_dwconv_vs_torch(n, c, h, w, s, silu, grp, gstride, goff, ldc, coff):
    torch = _torch()
    from aexrt_b200 import _native

    lib = _native.load()
    rng = np.random.default_rng(c + h + s)
    buf = rng.uniform(-2, 2, (n, h, w, ldc)).astype(np.float16)
    wt = rng.normal(0, 1 / 3, (c, 1, 3, 3)).astype(np.float32)
    b = rng.normal(0, 0.1, (c,)).astype(np.float32)
    g = grp or c
    idx = [coff + (k // g) * (gstride or g) + goff + k % g for k in range(c)]
    xt = torch.from_numpy(buf).cuda()
    w9 = torch.from_numpy(wt.astype(np.float16).astype(np.float32).reshape(c, 9).T.copy()).cuda()
    bt = torch.from_numpy(b).cuda()
    oh, ow = (h - 1) // s + 1, (w - 1) // s + 1
    out = torch.zeros((n, oh, ow, c + 8), dtype=torch.float16, device="cuda")
    _native.check(lib.aexrt_b200_dwconv3x3_f16(xt.data_ptr(), n, h, w, c, ldc, coff, grp, gstride, goff, w9.data_ptr(),
                                               bt.data_ptr(), s, int(silu), out.data_ptr(), c + 8, 8, None), "dwconv")
    torch.cuda.synchronize()
    xr = torch.from_numpy(nhwc_to_nchw(buf[..., idx]).astype(np.float32))
    wr = torch.from_numpy(wt.astype(np.float16).astype(np.float32))
    ref = torch.nn.functional.conv2d(xr, wr, torch.from_numpy(b), stride=s, padding=1, groups=c)
    if silu:
        ref = ref * torch.sigmoid(ref)
    got = torch.from_numpy(nhwc_to_nchw(out.cpu().numpy()[..., 8:8 + c]).astype(np.float32))
    assert (got - ref).abs().max().item() <= 1e-2
    assert not out[..., :8].any().item()  # channels outside the slice untouched


@pytest.mark.parametrize("n,heads,kd,h,w", [(2, 4, 32, 10, 10), (1, 2, 32, 20, 20), (3, 1, 16, 7, 9)])
def test_psa_attention_vs_oracle(n, heads, kd, h, w):
    torch = _torch()
    from aexrt_b200 import _native, ops, yolo

    lib = _native.load()
    rng = np.random.default_rng(heads * 10 + h)
    hd = 64
    per = 2 * kd + hd
    qkv = rng.normal(0, 1.0, (n, heads * per, h, w)).astype(np.float16)
    pe = rng.normal(0, 0.5, (n, heads * hd, h, w)).astype(np.float16)
    cmd = yolo.PsaAttnCmd("attn", yolo.Part("qkv", 0, heads * per), yolo.Part("pe", 0, heads * hd), ("out", 0),
                          heads, kd, hd)
    ref = om.psa_attention(cmd, qkv, pe)
    qt = torch.from_numpy(nchw_to_nhwc(qkv)).cuda()
    pt = torch.from_numpy(nchw_to_nhwc(pe)).cuda()
    out = torch.zeros((n, h, w, heads * hd), dtype=torch.float16, device="cuda")
    am = torch.zeros((n, heads * hd // 16), dtype=torch.int32, device="cuda")
    _native.check(lib.aexrt_b200_psa_attention_f16(qt.data_ptr(), n, h, w, heads * per, 0, heads, kd, hd, cmd.scale,
                                                   pt.data_ptr(), heads * hd, 0, out.data_ptr(), heads * hd, 0,
                                                   am.data_ptr(), am.shape[1], 0, None), "attention")
    torch.cuda.synchronize()
    got = nhwc_to_nchw(out.cpu().numpy())
    assert np.abs(got.astype(np.float32) - ref).max() <= 1e-2
    # epilogue amax: exactly the per-16-channel max |y| of the stored fp16 output
    want = np.abs(got.astype(np.float32)).reshape(n, heads * hd // 16, 16, h * w).max(axis=(2, 3))
    assert np.array_equal(am.cpu().numpy().view(np.float32), want.astype(np.float32))
    assert ops  # the package imported


@pytest.fixture(scope="module")
def v11s():
    from aexrt_b200 import yolo

    return yolo.build_yolov11s(nc=80, imgsz=320, seed=0)


def _images(n, seed=0, size=320):
    rng = np.random.default_rng(seed)
    return rng.uniform(0, 1, (n, 3, size, size)).astype(np.float16).astype(np.float32)


def test_yolov11s_per_layer_teacher_forced(v11s):
    torch = _torch()
    from aexrt_b200 import engine, yolo

    eng = engine.CompiledYolo(v11s, 2)
    imgs = _images(2)
    eng.forward(torch.from_numpy(imgs).cuda())
    torch.cuda.synchronize()
    assert eng.status() == 0
    vals = {k: nhwc_to_nchw(t.cpu().numpy()) for k, t in eng.values.items()}
    vals["images"] = imgs
    seen = set()
    for st in eng.steps:
        if st[0] in ("conv", "stem", "conv_nhwc"):
            c = st[1]
            x = om._gather(vals, c.inputs)
            res = vals[c.residual[0]][:, c.residual[1]:c.residual[1] + c.oc] if c.residual else None
            r = om.conv_cmd(c, x, res)
            got = vals[c.out[0]][:, c.out[1]:c.out[1] + c.oc].astype(np.float32)
            if c.precision == "int8":
                q = st[4][0].cpu().numpy()
                assert np.array_equal(slab16_to_nchw(q, c.ic, x.shape[2], x.shape[3], c.s), r["xq"]), c.name
            assert np.abs(got - r["y32"]).max() <= 1e-2, (c.name, float(np.abs(got - r["y32"]).max()))
            seen.add("conv")
        elif st[0] == "dwconv":
            c = st[1]
            src = vals[c.x.value][:, [c.in_channel(k) for k in range(c.c)]]
            got = vals[c.out[0]][:, c.out[1]:c.out[1] + c.c].astype(np.float32)
            assert np.abs(got - om.dwconv3x3(c, src)).max() <= 1e-2, c.name
            seen.add("dwconv")
        elif st[0] == "attn":
            c = st[1]
            qkv = vals[c.qkv.value][:, c.qkv.coff:c.qkv.coff + c.qkv.channels]
            pe = vals[c.pe.value][:, c.pe.coff:c.pe.coff + c.pe.channels]
            got = vals[c.out[0]][:, c.out[1]:c.out[1] + c.heads * c.head_dim].astype(np.float32)
            assert np.abs(got - om.psa_attention(c, qkv, pe)).max() <= 1e-2, c.name
            seen.add("attn")
        elif st[0] == "sppf":
            c = st[1]
            x = vals[c.x.value][:, c.x.coff:c.x.coff + c.x.channels]
            assert np.array_equal(vals[c.out[0]][:, c.out[1]:c.out[1] + 3 * c.x.channels], om.sppf_pool(x)), c.name
    assert seen == {"conv", "dwconv", "attn"}
    assert sum(isinstance(c, yolo.ConvCmd) and c.precision == "int8" for c in v11s.commands) >= 50


def test_yolov11s_end_to_end_against_oracle(v11s):
    from aexrt_b200 import engine
    from oracle import yolo_post as op

    torch = _torch()
    eng = engine.CompiledYolo(v11s, 2, nms=engine.NmsConfig())
    eng.capture()
    imgs = _images(2, seed=11)
    out = eng.forward(torch.from_numpy(imgs).cuda()).cpu().numpy()
    ref = om.run_program(v11s, imgs)["output0"]
    assert np.abs(out[:, 4:] - ref[:, 4:]).max() <= 0.02
    assert np.percentile(np.abs(out[:, :4] - ref[:, :4]), 99) <= 4.0
    counts, dets = (t.cpu().numpy() for t in eng.detections())
    for i in range(2):
        want, cnt = op.postprocess(out[i], 80)
        assert counts[i] == cnt and np.array_equal(dets[i, :cnt], want)
    assert eng.status() == 0


def test_yolov11s_batch_independence(v11s):
    """Graph replay at batch 3 equals each image run alone at batch 1 (per-image scales)."""
    from aexrt_b200 import engine

    torch = _torch()
    imgs = _images(3, seed=12)
    e3 = engine.CompiledYolo(v11s, 3)
    e3.capture()
    o3 = e3.forward(torch.from_numpy(imgs).cuda()).cpu().numpy()
    e1 = engine.CompiledYolo(v11s, 1)
    for i in range(3):
        o1 = e1.forward(torch.from_numpy(imgs[i:i + 1]).cuda()).cpu().numpy()
        assert np.array_equal(o1[0], o3[i])
