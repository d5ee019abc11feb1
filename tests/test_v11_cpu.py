"""YOLOv11s on the CPU: the program's structure follows the public yolo11
definition at scale s, and the oracle's C2PSA attention and depthwise conv restatements agree
with PyTorch's own fp32 operators (the checker of the checker; no GPU)."""
import numpy as np
import torch

from aexrt_b200 import yolo
from oracle import yolo_model as om


def test_yolov11s_structure():
    p = yolo.build_yolov11s(nc=80, imgsz=320)
    convs = {c.name: c for c in p.commands if isinstance(c, yolo.ConvCmd)}
    # stage widths at scale s (width 0.5, max 1024 channels): 32/64/128/256/512
    assert [convs[k].oc for k in ("l0", "l1", "l3", "l5", "l7")] == [32, 64, 128, 256, 512]
    # C3k2 with e=0.25 in layers 2 and 4, C3k blocks (two bottlenecks each) in 6, 8, 22
    assert convs["l2.cv1"].oc == 64 and convs["l2.m0.cv1"].oc == 16 and convs["l2.cv2"].ic == 96
    for layer in ("l6", "l8", "l22"):
        assert f"{layer}.m0.m1.cv2" in convs and convs[f"{layer}.m0.cv3"].ic == 2 * convs[f"{layer}.m0.cv12"].oc // 2 * 2 // 2 * 2 // 2 * 2 // 2 * 2 // 2 * 2 // 2 * 2 // 2 * 2 // 2 * 2 // 2 * 2 // 2 * 2 // 2
    # C2PSA: 4 heads of 64 channels over the 10x10 map, key_dim 32
    attn = [c for c in p.commands if isinstance(c, yolo.PsaAttnCmd)]
    assert len(attn) == 1 and (attn[0].heads, attn[0].key_dim, attn[0].head_dim) == (4, 32, 64)
    assert p.values[attn[0].qkv.value].h == 10 and convs["l10.m0.attn.qkv"].oc == 512
    # head: DWConv class branch, fp16; everything else before it W8A8 except the stem
    dws = [c for c in p.commands if isinstance(c, yolo.DwConvCmd)]
    assert len(dws) == 7  # 2 per level + the positional encoding
    assert all(c.precision == "fp16" for c in convs.values() if c.name.startswith("l23") or c.name == "l0")
    assert all(c.precision == "int8" for c in convs.values() if not c.name.startswith("l23") and c.name != "l0")


def test_oracle_attention_matches_torch():
    rng = np.random.default_rng(0)
    n, heads, kd, hd, h, w = 2, 4, 32, 64, 10, 10
    qkv = rng.normal(0, 1, (n, heads * (2 * kd + hd), h, w)).astype(np.float16)
    pe = rng.normal(0, 0.5, (n, heads * hd, h, w)).astype(np.float16)
    cmd = yolo.PsaAttnCmd("a", yolo.Part("q", 0, 0), yolo.Part("p", 0, 0), ("o", 0), heads, kd, hd)
    got = om.psa_attention(cmd, qkv, pe)
    t = torch.from_numpy(qkv.astype(np.float32)).view(n, heads, 2 * kd + hd, h * w)
    q, k, v = t.split([kd, kd, hd], dim=2)
    a = ((q.transpose(-2, -1) @ k) * kd ** -0.5).softmax(dim=-1)
    ref = (v @ a.transpose(-2, -1)).view(n, heads * hd, h, w) + torch.from_numpy(pe.astype(np.float32))
    assert np.abs(got - ref.numpy()).max() < 1e-4


def test_oracle_dwconv_matches_torch():
    rng = np.random.default_rng(1)
    for s in (1, 2):
        c = yolo.DwConvCmd("d", yolo.Part("x", 0, 48), ("o", 0), 48, s, True,
                           rng.normal(0, 0.3, (48, 1, 3, 3)).astype(np.float32),
                           rng.normal(0, 0.1, (48,)).astype(np.float32))
        x = rng.uniform(-1, 1, (2, 48, 9, 11)).astype(np.float16)
        got = om.dwconv3x3(c, x)
        ref = torch.nn.functional.conv2d(torch.from_numpy(x.astype(np.float32)),
                                         torch.from_numpy(c.weight.astype(np.float16).astype(np.float32)),
                                         torch.from_numpy(c.bias), stride=s, padding=1, groups=48)
        ref = ref * torch.sigmoid(ref)
        assert np.abs(got - ref.numpy()).max() < 1e-4
