"""GPU parity of the tcgen05 W8A8 conv against the oracle.

Bars (BASELINE parity gates): int8 codes and int32 accumulators bit-exact;
fp16 layer outputs within max-abs 1e-2 of the oracle's fp32 epilogue rounded to
fp16; the next-layer amax equals the amax of the stored fp16 output exactly.
"""
import numpy as np
import pytest

from oracle import w8a8 as ow
from tests._util import bits_to_f32, nchw_to_nhwc, nhwc_to_nchw, seeded_act, slab16_to_nchw

pytestmark = pytest.mark.gpu
TOL = 1e-2  # max-abs on fp16 layer outputs (BASELINE / README.md:62-63 gate family)


def _torch():
    import torch

    return torch


def run_gpu_layer(x, weight, bias, k, s, mode, silu=True, residual=None, block_n=0, wq=None, w_scale=None,
                  out_ldc=None, out_coff=0, variant=0):
    """quantize (NCHW fp16 input) + conv through the C ABI; returns numpy results."""
    torch = _torch()
    from aexrt_b200 import ops

    n, ic, h, w = x.shape
    oc = weight.shape[0]
    if wq is None:
        wq, w_scale = ops.quantize_conv_weight_int8(weight)
    plan = ops.ConvPlan.int8(n, ic, h, w, oc, k, s, wq, w_scale, bias, silu=silu, pg16=(mode == 1),
                             block_n=block_n | (variant << 16))
    xt = torch.from_numpy(x).cuda()
    amax = ops.act_amax(xt, ops.LAYOUT_NCHW_F16)
    q, rec = ops.act_quantize(xt, amax, mode, ops.LAYOUT_NCHW_F16, consumer_stride=s)
    oh, ow_ = plan.desc.out_h, plan.desc.out_w
    ldc = out_ldc or oc
    out = torch.zeros((n, oh, ow_, ldc), dtype=torch.float16, device="cuda")
    groups = (ic + 15) // 16
    dump_shape = (groups, n * oh * ow_, oc) if mode == 1 else (n * oh * ow_, oc)
    dump = torch.zeros(dump_shape, dtype=torch.int32, device="cuda")
    amax_out = torch.zeros((n, ldc // 16), dtype=torch.int32, device="cuda")
    res_t = torch.from_numpy(nchw_to_nhwc(residual)).cuda() if residual is not None else None
    plan.run(q, rec, out=out, out_coff=out_coff, residual=res_t, amax_out=amax_out, amax_goff=out_coff // 16,
             acc_dump=dump)
    torch.cuda.synchronize()
    assert plan.status() == 0
    y = nhwc_to_nchw(out.cpu().numpy()[..., out_coff:out_coff + oc])
    d = dump.cpu().numpy()
    if mode == 1:
        acc_g = d.reshape(groups, n, oh, ow_, oc).transpose(1, 0, 4, 2, 3)
        acc = acc_g.sum(axis=1).astype(np.int32)
    else:
        acc_g = None
        acc = d.reshape(n, oh, ow_, oc).transpose(0, 3, 1, 2)
    return dict(y=y, acc=acc, acc_g=acc_g, xq=slab16_to_nchw(q.cpu().numpy(), ic, h, w, s), plan=plan,
                amax_out=bits_to_f32(amax_out.cpu().numpy()), out_full=out.cpu().numpy())


def check_against_oracle(x, weight, bias, k, s, mode, silu=True, residual=None, block_n=0, variant=0):
    g = run_gpu_layer(x, weight, bias, k, s, mode, silu=silu, residual=residual, block_n=block_n, variant=variant)
    o = ow.conv_w8a8(x, weight, bias, k, s, k // 2, mode=mode, silu=silu, residual=residual)
    assert np.array_equal(g["xq"], o["xq"]), "int8 codes differ"
    assert np.array_equal(g["acc"], o["acc"]), "int32 accumulators differ"
    if mode == 1:
        assert np.array_equal(g["acc_g"], o["acc_g"]), "pg16 group sub-sums differ"
    err = np.abs(g["y"].astype(np.float32) - o["y32"]).max()
    assert err <= TOL, f"fp16 output max-abs error {err}"
    # epilogue amax of the stored fp16 output (the next layer's quantizer input)
    _, ag = ow.act_amax(g["y"])
    assert np.array_equal(g["amax_out"][:, :ag.shape[1]], ag)
    return g, o, err


def test_golden_act_cases(golden_dir):
    d = np.load(f"{golden_dir}/act_cases.npz")
    for name in d["names"]:
        name = str(name)
        n, ic, h, w, oc, k, s, p, mode, silu, res = (int(v) for v in d[name + ".meta"])
        g = run_gpu_layer(d[name + ".x"], d[name + ".w"], d[name + ".b"], k, s, mode, silu=bool(silu),
                          residual=d[name + ".res"] if res else None)
        assert np.array_equal(g["xq"], d[name + ".xq"]), name
        assert np.array_equal(g["acc"], d[name + ".acc"]), name
        err = np.abs(g["y"].astype(np.float32) - d[name + ".y"].astype(np.float32)).max()
        assert err <= TOL, (name, err)


@pytest.mark.parametrize("mode", [0, 1])
@pytest.mark.parametrize("n,ic,h,w,oc,k,s", [
    (1, 64, 80, 80, 128, 3, 1),    # BASELINE config 1 (C1 block)
    (1, 128, 40, 40, 128, 1, 1),   # config 2 sweep, batch 1
    (1, 64, 80, 80, 64, 3, 1),
    (1, 32, 160, 160, 64, 3, 2),
    (1, 128, 20, 20, 256, 3, 2),
    (2, 16, 13, 11, 32, 3, 1),     # ragged: H*W not a multiple of the tile, 16 input channels
    (2, 48, 9, 7, 16, 1, 1),
    (3, 32, 11, 9, 48, 3, 2),      # odd input dims for stride 2
])
def test_conv_parity(n, ic, h, w, oc, k, s, mode):
    rng = np.random.default_rng(n * 1000 + ic + oc + k + s + mode)
    x = seeded_act(rng, (n, ic, h, w))
    weight = rng.normal(0, 0.05, (oc, ic, k, k)).astype(np.float32)
    bias = rng.normal(0, 0.1, (oc,)).astype(np.float32)
    check_against_oracle(x, weight, bias, k, s, mode)


@pytest.mark.parametrize("block_n", [16, 32, 64, 128, 256])
def test_block_n_variants_bitexact(block_n):
    """Every output-channel tile gives the same accumulators (the autotuner's candidates)."""
    rng = np.random.default_rng(3)
    x = seeded_act(rng, (2, 32, 12, 10))
    weight = rng.normal(0, 0.05, (256, 32, 3, 3)).astype(np.float32)
    bias = rng.normal(0, 0.1, (256,)).astype(np.float32)
    check_against_oracle(x, weight, bias, 3, 1, 0, block_n=block_n)
    if block_n <= 128:
        check_against_oracle(x, weight, bias, 3, 1, 1, block_n=block_n)


def test_residual_and_no_silu():
    rng = np.random.default_rng(4)
    x = seeded_act(rng, (2, 32, 10, 10))
    weight = rng.normal(0, 0.05, (32, 32, 3, 3)).astype(np.float32)
    bias = rng.normal(0, 0.1, (32,)).astype(np.float32)
    res = rng.standard_normal((2, 32, 10, 10)).astype(np.float16)
    check_against_oracle(x, weight, bias, 3, 1, 0, residual=res)
    w1 = rng.normal(0, 0.05, (32, 32, 1, 1)).astype(np.float32)
    check_against_oracle(x, w1, bias, 1, 1, 1, silu=False)


def test_output_slice_of_concat_buffer():
    """The epilogue writes into a channel slice of a wider NHWC buffer (concat by placement)."""
    rng = np.random.default_rng(6)
    x = seeded_act(rng, (2, 32, 8, 8))
    weight = rng.normal(0, 0.05, (32, 32, 3, 3)).astype(np.float32)
    bias = rng.normal(0, 0.1, (32,)).astype(np.float32)
    g = run_gpu_layer(x, weight, bias, 3, 1, 0, out_ldc=96, out_coff=48)
    o = ow.conv_w8a8(x, weight, bias, 3, 1, 1)
    assert np.abs(g["y"].astype(np.float32) - o["y32"]).max() <= TOL
    full = g["out_full"]
    assert (full[..., :48] == 0).all() and (full[..., 80:] == 0).all()
    assert (g["amax_out"][:, :3] == 0).all() and (g["amax_out"][:, 5:] == 0).all()


def test_baseline_pg16_output_channel_variant():
    """BASELINE.json's wording: weights quantized per 16-output-channel group; the
    epilogue takes any per-oc scale vector, so this is the group scale broadcast."""
    rng = np.random.default_rng(8)
    x = seeded_act(rng, (1, 64, 20, 20))
    weight = rng.normal(0, 0.05, (128, 64, 3, 3)).astype(np.float32)
    bias = rng.normal(0, 0.1, (128,)).astype(np.float32)
    grp = np.abs(weight).reshape(8, -1).max(axis=1)
    scale = np.repeat((grp / np.float32(127)).astype(np.float32), 16)
    inv = (np.float32(1) / scale).astype(np.float32)
    prod = (weight.reshape(128, -1) * inv[:, None]).astype(np.float32)
    wq = np.clip(np.sign(prod) * np.floor(np.abs(prod) + np.float32(0.5)), -127, 127).astype(np.int8)
    g = run_gpu_layer(x, weight, bias, 3, 1, 0, wq=wq, w_scale=scale)
    o = ow.conv_w8a8(x, weight, bias, 3, 1, 1, wq=wq, w_scale=scale)
    assert np.array_equal(g["acc"], o["acc"])
    assert np.abs(g["y"].astype(np.float32) - o["y32"]).max() <= TOL


@pytest.mark.parametrize("mode", [0, 1])
@pytest.mark.parametrize("n,ic,h,w,oc,k,s", [
    (64, 128, 40, 40, 128, 1, 1),
    (64, 64, 80, 80, 64, 3, 1),
    (64, 32, 160, 160, 64, 3, 2),
    (64, 128, 20, 20, 256, 3, 2),
])
def test_conv_parity_batch64(n, ic, h, w, oc, k, s, mode):
    """BASELINE config 2 at batch 64, per-tensor and pg16 (the INT8_PERGROUP scheme): per-image
    scales, exact codes, accumulators and (pg16) per-group sub-sums."""
    rng = np.random.default_rng(64 + ic + oc)
    x = seeded_act(rng, (n, ic, h, w))
    weight = rng.normal(0, 0.05, (oc, ic, k, k)).astype(np.float32)
    bias = rng.normal(0, 0.1, (oc,)).astype(np.float32)
    check_against_oracle(x, weight, bias, k, s, mode)


@pytest.mark.parametrize("n,ic,h,w,oc,k,s,silu", [
    (2, 3, 32, 32, 16, 3, 2, True),   # the model's stem (3 input channels padded to 8)
    (2, 64, 10, 10, 64, 3, 1, True),
    (2, 64, 10, 10, 64, 1, 1, False),
    (1, 64, 20, 20, 4, 1, 1, False),  # class logits: 4 outputs
])
def test_fp16_conv_vs_torch(n, ic, h, w, oc, k, s, silu):
    """fp16 conv (stem / detect head) against a plain PyTorch fp32 conv of the fp16-rounded operands."""
    torch = _torch()
    from aexrt_b200 import ops

    rng = np.random.default_rng(ic + oc)
    x = rng.uniform(0, 1, (n, ic, h, w)).astype(np.float32)
    weight = rng.normal(0, 1 / np.sqrt(ic * k * k), (oc, ic, k, k)).astype(np.float32)
    bias = rng.normal(0, 0.1, (oc,)).astype(np.float32)
    plan = ops.ConvPlan.fp16(n, ic, h, w, oc, k, s, weight, bias, silu=silu)
    xt = torch.from_numpy(x).cuda()
    packed = ops.pack_f16(xt, ops.LAYOUT_NCHW_F32, consumer_stride=s)
    out = plan.run(packed)
    torch.cuda.synchronize()
    assert plan.status() == 0
    xr = torch.from_numpy(x.astype(np.float16).astype(np.float32))
    wr = torch.from_numpy(weight.astype(np.float16).astype(np.float32))
    ref = torch.nn.functional.conv2d(xr, wr, torch.from_numpy(bias), stride=s, padding=k // 2)
    if silu:
        ref = ref * torch.sigmoid(ref)
    got = torch.from_numpy(nhwc_to_nchw(out.cpu().numpy()).astype(np.float32))
    err = (got - ref).abs().max().item()
    assert err <= 1e-2 * max(1.0, ref.abs().max().item() / 8), err


# variant bits: 1 slot streaming, 2 halo (auto order), 0x12 halo strided, 0x22 halo contiguous runs
@pytest.mark.parametrize("variant", [1, 2, 0x12, 0x22])
@pytest.mark.parametrize("n,ic,h,w,oc,k,s", [
    (2, 64, 20, 20, 64, 3, 1),
    (2, 48, 17, 13, 32, 3, 1),   # odd slab count (3 slabs): zero-padded slab pair
    (2, 16, 10, 10, 16, 3, 1),   # one slab
    (2, 32, 20, 18, 64, 3, 2),
    (1, 32, 9, 11, 48, 3, 2),
    (2, 96, 10, 10, 32, 1, 1),
    (1, 64, 80, 80, 128, 3, 1),
])
def test_kernel_variants_bitexact(n, ic, h, w, oc, k, s, variant):
    """Slot-streaming and halo kernels (both halo tile orders): identical int32 accumulators and
    epilogue amax, all equal to the oracle."""
    rng = np.random.default_rng(ic * 7 + oc + s)
    x = seeded_act(rng, (n, ic, h, w))
    weight = rng.normal(0, 0.05, (oc, ic, k, k)).astype(np.float32)
    bias = rng.normal(0, 0.1, (oc,)).astype(np.float32)
    g, _, _ = check_against_oracle(x, weight, bias, k, s, 0, variant=variant)
    assert g["plan"].info  # plan built with the requested variant


@pytest.mark.parametrize("n,ic,h,w,oc,k,s,silu", [
    (2, 64, 20, 20, 128, 3, 1, True),
    (2, 16, 32, 32, 16, 3, 2, True),
    (2, 64, 10, 10, 64, 1, 1, False),
])
def test_fp16_halo_vs_slot_streaming(n, ic, h, w, oc, k, s, silu):
    """The fp16 conv variants agree with each other and with a torch fp32 reference."""
    torch = _torch()
    from aexrt_b200 import ops

    rng = np.random.default_rng(ic + 3 * oc)
    x = rng.uniform(0, 1, (n, ic, h, w)).astype(np.float32)
    weight = rng.normal(0, 1 / np.sqrt(ic * k * k), (oc, ic, k, k)).astype(np.float32)
    bias = rng.normal(0, 0.1, (oc,)).astype(np.float32)
    outs = []
    for variant in (1, 2):
        plan = ops.ConvPlan.fp16(n, ic, h, w, oc, k, s, weight, bias, silu=silu, block_n=variant << 16)
        packed = ops.pack_f16(torch.from_numpy(x).cuda(), ops.LAYOUT_NCHW_F32, consumer_stride=s)
        outs.append(plan.run(packed).float().cpu())
        torch.cuda.synchronize()
        assert plan.status() == 0
    xr = torch.from_numpy(x.astype(np.float16).astype(np.float32))
    wr = torch.from_numpy(weight.astype(np.float16).astype(np.float32))
    ref = torch.nn.functional.conv2d(xr, wr, torch.from_numpy(bias), stride=s, padding=k // 2)
    if silu:
        ref = ref * torch.sigmoid(ref)
    ref = ref.permute(0, 2, 3, 1)
    for o in outs:
        assert (o - ref).abs().max().item() <= 1e-2 * max(1.0, ref.abs().max().item() / 8)


@pytest.mark.parametrize("dtype", ["float32", "float16"])
@pytest.mark.parametrize("n,h,w,oc,s,silu", [
    (2, 64, 64, 16, 2, True),    # the YOLOv8n stem shape, small
    (3, 33, 47, 32, 2, True),    # odd sizes: clipped windows on the right/bottom
    (2, 20, 20, 64, 1, False),
    (1, 17, 16, 48, 2, True),
    (2, 21, 19, 16, 1, True),    # two-pixel form: odd output width (last pair has one pixel)
    (1, 18, 17, 32, 2, False),   # two-pixel form, stride 2, odd output width
    (2, 40, 36, 32, 1, True),
])
def test_stem_image_input(n, h, w, oc, s, silu, dtype):
    """The direct stem (fp32 or fp16 NCHW images in) against torch fp32 and the packed fp16 path; amax_out exact."""
    torch = _torch()
    from aexrt_b200 import ops

    rng = np.random.default_rng(oc + h)
    x = rng.uniform(0, 1, (n, 3, h, w)).astype(dtype)
    weight = rng.normal(0, 1 / np.sqrt(27), (oc, 3, 3, 3)).astype(np.float32)
    bias = rng.normal(0, 0.1, (oc,)).astype(np.float32)
    plan = ops.ConvPlan.fp16(n, 3, h, w, oc, 3, s, weight, bias, silu=silu)
    assert plan.info.image_input == 1
    xt = torch.from_numpy(x).cuda()
    # write into a channel slice of a wider buffer, with amax slots behind the slice
    oh, ow = plan.out_shape[1], plan.out_shape[2]
    buf = torch.full((n, oh, ow, oc + 32), 7.0, dtype=torch.float16, device="cuda")
    amax = torch.zeros((n, (oc + 32) // 16), dtype=torch.int32, device="cuda")
    plan.run_image(xt, out=buf, out_coff=16, amax_out=amax, amax_goff=1)
    layout = ops.LAYOUT_NCHW_F16 if dtype == "float16" else ops.LAYOUT_NCHW_F32
    packed_out = plan.run(ops.pack_f16(xt, layout, consumer_stride=s))
    torch.cuda.synchronize()
    got = buf[..., 16:16 + oc].float().cpu()
    assert torch.all(buf[..., :16] == 7.0) and torch.all(buf[..., 16 + oc:] == 7.0)
    xr = torch.from_numpy(x.astype(np.float16).astype(np.float32))
    wr = torch.from_numpy(weight.astype(np.float16).astype(np.float32))
    ref = torch.nn.functional.conv2d(xr, wr, torch.from_numpy(bias), stride=s, padding=1)
    if silu:
        ref = ref * torch.sigmoid(ref)
    ref = ref.permute(0, 2, 3, 1)
    tol = 1e-2 * max(1.0, ref.abs().max().item() / 8)
    assert (got - ref).abs().max().item() <= tol
    assert (got - packed_out.float().cpu()).abs().max().item() <= tol
    # amax slots: exact max |y| of the fp16 outputs per (image, 16-channel group)
    g = got.abs().reshape(n, -1, oc // 16, 16).amax(dim=(1, 3))
    want = g.numpy().astype(np.float32).view(np.int32)
    am = amax.cpu().numpy()
    assert np.array_equal(am[:, 1:1 + oc // 16], want)
    assert not am[:, 0].any() and not am[:, 1 + oc // 16:].any()


@pytest.mark.parametrize("n,ic,h,w,oc,k,s,block_n", [
    (256, 128, 20, 20, 128, 3, 2, 0),   # few ring stages (large resident weights), 1-2 tiles per CTA
    (256, 512, 10, 10, 256, 1, 1, 0),   # a whole tile's slab pairs fill the ring
    (64, 64, 10, 10, 256, 3, 1, 64),    # 4 weight tiles, fewer M tiles than CTAs: weight reloads mid-run
    (64, 16, 40, 40, 16, 3, 1, 0),      # narrow: deep ring, two MMA issuers
])
def test_halo_pipeline_corner_cases_match_slot_kernel(n, ic, h, w, oc, k, s, block_n):
    """Halo-tile pipeline corner cases (ring depth vs tile stages, weight reloads, issuer split):
    int32 accumulators equal the slot-streaming kernel's, and no pipeline wait gives up."""
    torch = _torch()
    from aexrt_b200 import ops

    rng = np.random.default_rng(n + ic + oc)
    x = seeded_act(rng, (n, ic, h, w))
    weight = rng.normal(0, 0.05, (oc, ic, k, k)).astype(np.float32)
    bias = rng.normal(0, 0.1, (oc,)).astype(np.float32)
    wq, w_scale = ops.quantize_conv_weight_int8(weight)
    xt = torch.from_numpy(x).cuda()
    amax = ops.act_amax(xt, ops.LAYOUT_NCHW_F16)
    q, rec = ops.act_quantize(xt, amax, 0, ops.LAYOUT_NCHW_F16, consumer_stride=s)
    accs = []
    for variant in (1, 2):
        plan = ops.ConvPlan.int8(n, ic, h, w, oc, k, s, wq, w_scale, bias, block_n=block_n | (variant << 16))
        assert plan.info.variant == variant
        d = plan.desc
        dump = torch.zeros((n * d.out_h * d.out_w, oc), dtype=torch.int32, device="cuda")
        am = torch.zeros((n, (oc + 15) // 16), dtype=torch.int32, device="cuda")
        out = plan.run(q, rec, amax_out=am, acc_dump=dump)
        torch.cuda.synchronize()
        assert plan.status() == 0
        accs.append((dump.cpu(), out.cpu(), am.cpu()))
    assert torch.equal(accs[0][0], accs[1][0])
    assert torch.equal(accs[0][1], accs[1][1])
    assert torch.equal(accs[0][2], accs[1][2])


@pytest.mark.parametrize("variant", [1, 2, 0x12, 0x22])
@pytest.mark.parametrize("n,ic,h,w,oc,k,s", [
    (2, 64, 20, 20, 128, 3, 1),
    (2, 48, 17, 13, 64, 3, 1),    # 3 slabs: the odd slab of the last pair has no MMAs
    (2, 32, 20, 18, 64, 3, 2),    # stride 2: tap pairs across parity boxes
    (2, 96, 10, 10, 128, 1, 1),   # 1x1: one tap per slab, zero second half of K
    (1, 64, 80, 80, 128, 3, 1),   # BASELINE config 1 (C1), batch 1
])
def test_pg16_kernel_variants_bitexact(n, ic, h, w, oc, k, s, variant):
    """pg16 on the slot-streaming kernel and on the halo kernel (tap-paired K steps, one
    accumulation unit per slab): identical per-group int32 sub-sums, all equal to the oracle."""
    rng = np.random.default_rng(ic * 5 + oc + s + k)
    x = seeded_act(rng, (n, ic, h, w))
    weight = rng.normal(0, 0.05, (oc, ic, k, k)).astype(np.float32)
    bias = rng.normal(0, 0.1, (oc,)).astype(np.float32)
    g, _, _ = check_against_oracle(x, weight, bias, k, s, 1, variant=variant)
    assert g["plan"].info.variant == (1 if variant == 1 else 2)


def test_pg16_halo_residual_and_linear():
    """pg16 halo epilogue without SiLU and with the C2f residual."""
    rng = np.random.default_rng(7)
    x = seeded_act(rng, (2, 64, 12, 12))
    weight = rng.normal(0, 0.05, (64, 64, 3, 3)).astype(np.float32)
    bias = rng.normal(0, 0.1, (64,)).astype(np.float32)
    res = seeded_act(rng, (2, 64, 12, 12))
    check_against_oracle(x, weight, bias, 3, 1, 1, silu=True, residual=res, variant=2)
    check_against_oracle(x, weight, bias, 3, 1, 1, silu=False, variant=2)


@pytest.mark.parametrize("n,ic,h,w,oc,k,s", [
    (16, 16, 80, 80, 16, 3, 1),    # narrow 3x3: 4 M blocks per super-tile
    (16, 16, 81, 77, 32, 3, 2),    # stride 2, ragged map: partial super-tiles at the bottom
    (16, 32, 80, 80, 32, 1, 1),    # 1x1
    (16, 64, 40, 40, 64, 3, 1),    # 2 M blocks
])
def test_super_tiles_match_single_blocks(n, ic, h, w, oc, k, s):
    """Halo super-tiles (several M blocks per pipeline step) give the same accumulators, outputs and
    epilogue amax as one block per tile (block_n bits 24-27 = 1), and both match the oracle."""
    rng = np.random.default_rng(ic * 3 + oc + h + s)
    x = seeded_act(rng, (n, ic, h, w))
    weight = rng.normal(0, 0.05, (oc, ic, k, k)).astype(np.float32)
    bias = rng.normal(0, 0.1, (oc,)).astype(np.float32)
    g_auto, _, _ = check_against_oracle(x, weight, bias, k, s, 0, variant=2)
    g_one, _, _ = check_against_oracle(x, weight, bias, k, s, 0, variant=2 | (1 << 8))
    assert np.array_equal(g_auto["acc"], g_one["acc"])
    assert np.array_equal(g_auto["out_full"], g_one["out_full"])
    assert np.array_equal(g_auto["amax_out"], g_one["amax_out"])
    assert g_auto["plan"].info.tile_h == g_one["plan"].info.tile_h


@pytest.mark.parametrize("n,ic,h,w,oc,k,ldc,coff,silu,block_n", [
    (2, 64, 20, 20, 64, 3, 64, 0, True, 0),      # detect-head 3x3 shape
    (2, 64, 40, 40, 64, 1, 64, 0, False, 0),     # detect-head 1x1 (box logits)
    (3, 24, 13, 17, 16, 3, 72, 40, True, 0),     # odd slab count, channel slice of a wider buffer
    (2, 32, 9, 30, 128, 3, 48, 8, True, 64),     # two weight tiles, ragged tiles
    (1, 16, 80, 80, 16, 3, 16, 0, True, 16),     # narrow: stacked M blocks
])
def test_fp16_nhwc_input_matches_packed(n, ic, h, w, oc, k, ldc, coff, silu, block_n):
    """aexrt_b200_conv_f16_nhwc (TMA boxes straight from the NHWC activation) equals pack_f16 +
    conv_f16 bit for bit, including the epilogue amax."""
    torch = _torch()
    from aexrt_b200 import ops

    rng = np.random.default_rng(ic * 7 + oc + ldc)
    buf = rng.uniform(-1, 1, (n, h, w, ldc)).astype(np.float16)
    weight = rng.normal(0, 1 / np.sqrt(ic * k * k), (oc, ic, k, k)).astype(np.float32)
    bias = rng.normal(0, 0.1, (oc,)).astype(np.float32)
    plan = ops.ConvPlan.fp16(n, ic, h, w, oc, k, 1, weight, bias, silu=silu, block_n=block_n)
    assert plan.info.variant == 2
    xt = torch.from_numpy(buf).cuda()
    groups = (oc + 15) // 16
    am0 = torch.zeros((n, groups), dtype=torch.int32, device="cuda")
    am1 = torch.zeros((n, groups), dtype=torch.int32, device="cuda")
    packed = ops.pack_f16(xt, ops.LAYOUT_NHWC_F16, c=ic, ldc=ldc, coff=coff)
    ref = plan.run(packed, amax_out=am0)
    got = plan.run_nhwc(xt, x_coff=coff, amax_out=am1)
    torch.cuda.synchronize()
    assert plan.status() == 0
    assert torch.equal(ref, got)
    assert torch.equal(am0, am1)


def _ql_sources(parts):
    """AexrtB200ActSource array of fp16 NHWC torch tensors [(tensor, coff, channels, upsample), ...] with
    their amax slots (computed here, as a producer's epilogue would leave them)."""
    from aexrt_b200 import ops
    from aexrt_b200._native import AexrtB200ActSource

    srcs = (AexrtB200ActSource * len(parts))()
    keep = []
    for i, (t, coff, ch, up) in enumerate(parts):
        am = ops.act_amax(t, ops.LAYOUT_NHWC_F16)  # every group of the buffer
        keep.append(am)
        s = srcs[i]
        s.ptr, s.layout, s.ldc, s.coff, s.channels, s.upsample = t.data_ptr(), ops.LAYOUT_NHWC_F16, t.shape[-1], coff, ch, up
        s.src_h, s.src_w = t.shape[1], t.shape[2]
        s.amax_groups, s.amax_stride, s.amax_goff = am.data_ptr(), am.shape[1], coff // 16
    return srcs, keep


@pytest.mark.parametrize("mode", [0, 1])
@pytest.mark.parametrize("n,ic,h,w,oc,k,s,split", [
    (2, 32, 12, 10, 64, 3, 1, None),
    (2, 16, 13, 11, 32, 3, 1, None),       # narrow: stacked M blocks
    (3, 32, 11, 9, 48, 3, 2, None),        # stride 2, odd input
    (2, 48, 9, 7, 32, 1, 1, None),
    (8, 64, 80, 80, 128, 3, 1, None),      # C1 at batch 8
    (2, 48, 16, 16, 64, 1, 1, (32, 2)),    # concat: 32 channels upsampled 2x, then 16 at full size
    (2, 48, 16, 16, 32, 3, 1, (32, 2)),
    (2, 40, 10, 12, 32, 3, 1, (16, 1)),    # last part of 24 channels: a partial slab
    (64, 64, 80, 80, 64, 3, 1, None),      # BASELINE config 2 layers at batch 64
    (64, 32, 160, 160, 64, 3, 2, None),
    (64, 128, 20, 20, 256, 3, 2, None),
    (64, 128, 40, 40, 128, 1, 1, None),
])
def test_quantize_on_load_equals_quantize_then_conv(n, ic, h, w, oc, k, s, split, mode):
    """aexrt_b200_conv_w8a8_sources (the conv quantizes its fp16 NHWC sources in shared memory) equals
    aexrt_b200_act_quantize_concat + aexrt_b200_conv_w8a8 bit for bit: fp16 outputs, int32
    accumulators (pg16: every group's sub-sum) and the next-layer amax."""
    torch = _torch()
    from aexrt_b200 import _native, ops

    if mode == 1 and ic % 16:
        pytest.skip("pg16 needs 16-channel groups")
    rng = np.random.default_rng(n * 7 + ic + oc + k + s + mode)
    weight = rng.normal(0, 0.05, (oc, ic, k, k)).astype(np.float32)
    bias = rng.normal(0, 0.1, (oc,)).astype(np.float32)
    wq, ws = ops.quantize_conv_weight_int8(weight)
    if split is None:
        x = torch.from_numpy(nchw_to_nhwc(seeded_act(rng, (n, ic, h, w)) * np.float16(2))).cuda()
        parts = [(x, 0, ic, 1)]
    else:
        c0, up = split
        a = torch.from_numpy(nchw_to_nhwc(seeded_act(rng, (n, c0, h // up, w // up)))).cuda()
        b = torch.from_numpy(nchw_to_nhwc(seeded_act(rng, (n, 48, h, w)) * np.float16(3))).cuda()
        parts = [(a, 0, c0, up), (b, 16, ic - c0, 1)]
    res = torch.from_numpy(nchw_to_nhwc(rng.standard_normal((n, oc, (h - 1) // s + 1 if k == 3 else h,
                                                             (w - 1) // s + 1 if k == 3 else w)).astype(np.float16))).cuda()
    results = []
    for ql in (False, True):
        plan = ops.ConvPlan.int8(n, ic, h, w, oc, k, s, wq, ws, bias, silu=True, pg16=bool(mode), quant_on_load=ql)
        srcs, keep = _ql_sources(parts)
        out = torch.zeros(plan.out_shape, dtype=torch.float16, device="cuda")
        amax_out = torch.zeros((n, (oc + 15) // 16), dtype=torch.int32, device="cuda")
        d = plan.desc
        groups = (ic + 15) // 16
        dump = torch.zeros((groups, n * d.out_h * d.out_w, oc) if mode else (n * d.out_h * d.out_w, oc),
                           dtype=torch.int32, device="cuda")
        if ql:
            if not plan.info.quant_on_load:
                # the planner keeps quantize-then-conv where the raw ring does not fit: narrow pg16
                # convs stream slots (pg16 halo tiles are 64 or 128 channels wide), and wide convs
                # whose resident weights leave no room for the ring next to 4 stages; such a plan
                # refuses sources
                assert ic >= 128 or (plan.info.variant != 2 and mode == 1 and oc < 64)
                with pytest.raises(_native.AexrtError):
                    plan.run_sources(srcs, out=out, residual=res, amax_out=amax_out, acc_dump=dump)
                return
            plan.run_sources(srcs, out=out, residual=res, amax_out=amax_out, acc_dump=dump)
        else:
            q = torch.empty(ops.packed_act_shape(n, ic, h, w, s), dtype=torch.int8, device="cuda")
            rec = torch.empty((n, 1 + groups), dtype=torch.float32, device="cuda")
            _native.check(_native.load().aexrt_b200_act_quantize_concat(srcs, len(srcs), n, h, w, mode, s, q.data_ptr(),
                                                                        rec.data_ptr(), None), "quantize")
            plan.run(q, rec, out=out, residual=res, amax_out=amax_out, acc_dump=dump)
        torch.cuda.synchronize()
        assert plan.status() == 0
        results.append((out.cpu(), dump.cpu(), amax_out.cpu()))
    for a, b in zip(results[0], results[1]):
        assert torch.equal(a, b)


STAGED, DIRECT = 0x20000000, 0x10000000  # plan bits: staged TMA-store epilogue / direct stores


@pytest.mark.parametrize("mode", [0, 1])
@pytest.mark.parametrize("n,ic,h,w,oc,k,s,block_n,res,ldc,coff", [
    (2, 64, 20, 20, 128, 3, 1, 0, False, None, 0),
    (2, 96, 10, 10, 32, 1, 1, 0, True, None, 0),      # 1x1 with the C2f residual
    (2, 48, 17, 13, 48, 3, 1, 64, False, 80, 16),     # odd channel count: partial column blocks, slice
    (2, 32, 20, 18, 64, 3, 2, 0, False, None, 0),     # stride 2
    (1, 128, 10, 10, 256, 1, 1, 256, False, None, 0),  # BN 256: 128-byte rows (128B swizzle)
    (2, 16, 80, 80, 16, 3, 1, 0, True, None, 0),      # narrow 3x3: stacked M blocks, tile groups
    (1, 64, 40, 40, 32, 3, 1, 32, False, 96, 64),     # BN 32 written into a concat buffer
])
def test_staged_epilogue_equals_direct_stores(n, ic, h, w, oc, k, s, block_n, res, ldc, coff, mode):
    """The staged epilogue (swizzled shared-memory boxes, one TMA tensor store per tile and column
    block) writes exactly the bytes and amax of the direct-store epilogue, both equal to the oracle."""
    if mode == 1 and (ic % 16 or block_n not in (0, 64, 128) or oc < 64):
        pytest.skip("pg16 halo plans need 16k input channels and 64 / 128-wide output tiles")
    rng = np.random.default_rng(ic * 3 + oc + k + s)
    x = seeded_act(rng, (n, ic, h, w))
    weight = rng.normal(0, 0.05, (oc, ic, k, k)).astype(np.float32)
    bias = rng.normal(0, 0.1, (oc,)).astype(np.float32)
    oh, ow_ = (h + 2 * (k // 2) - k) // s + 1, (w + 2 * (k // 2) - k) // s + 1
    residual = seeded_act(rng, (n, oc, oh, ow_)) if res else None
    runs = {}
    for bits in (STAGED, DIRECT):
        runs[bits] = run_gpu_layer(x, weight, bias, k, s, mode, residual=residual, block_n=block_n | bits,
                                   out_ldc=ldc, out_coff=coff)
    st, di = runs[STAGED], runs[DIRECT]
    assert st["plan"].info.staged_out > 0 and di["plan"].info.staged_out == 0
    assert np.array_equal(st["out_full"], di["out_full"])
    assert np.array_equal(st["amax_out"], di["amax_out"])
    o = ow.conv_w8a8(x, weight, bias, k, s, k // 2, mode=mode, residual=residual)
    assert np.array_equal(st["acc"], o["acc"])
    assert np.abs(st["y"].astype(np.float32) - o["y32"]).max() <= TOL


@pytest.mark.parametrize("n,ic,h,w,oc,k,silu,block_n", [
    (2, 64, 20, 20, 64, 3, True, 0),
    (2, 192, 40, 40, 144, 1, False, 128),   # the fused head logits conv (a partial second tile)
    (1, 16, 80, 80, 16, 3, True, 16),
])
def test_fp16_staged_epilogue_equals_direct_stores(n, ic, h, w, oc, k, silu, block_n):
    torch = _torch()
    from aexrt_b200 import ops

    rng = np.random.default_rng(ic + oc + k)
    xt = torch.from_numpy(rng.uniform(-1, 1, (n, h, w, ic)).astype(np.float16)).cuda()
    weight = rng.normal(0, 1 / np.sqrt(ic * k * k), (oc, ic, k, k)).astype(np.float32)
    bias = rng.normal(0, 0.1, (oc,)).astype(np.float32)
    outs = []
    for bits in (STAGED, DIRECT):
        plan = ops.ConvPlan.fp16(n, ic, h, w, oc, k, 1, weight, bias, silu=silu, block_n=block_n | bits)
        am = torch.zeros((n, (oc + 15) // 16), dtype=torch.int32, device="cuda")
        out = plan.run_nhwc(xt, amax_out=am)
        torch.cuda.synchronize()
        assert plan.status() == 0
        outs.append((plan.info.staged_out, out, am))
    assert outs[0][0] > 0 and outs[1][0] == 0
    assert torch.equal(outs[0][1], outs[1][1]) and torch.equal(outs[0][2], outs[1][2])


@pytest.mark.parametrize("n,ic,h,w,oc,k,s,f16", [
    (4, 256, 10, 10, 128, 3, 1, False),   # 16 slab pairs a tile: one issuer by default
    (2, 512, 10, 10, 64, 1, 1, False),
    (4, 256, 10, 10, 128, 3, 1, True),    # the fp16 detect head's P5 shape (NHWC input)
])
def test_two_issuers_equal_one(n, ic, h, w, oc, k, s, f16):
    """Per-tensor plans whose tiles have more stages than half the stage ring holds run two MMA
    issuers (each walks its half ring through its own tiles); int8 results equal the oracle's, and
    plan bit 30 (which asks for two issuers explicitly) changes nothing."""
    torch = _torch()
    from aexrt_b200 import ops

    rng = np.random.default_rng(77 + ic + oc)
    x = seeded_act(rng, (n, ic, h, w))
    wt = rng.normal(0, 0.05, (oc, ic, k, k)).astype(np.float32)
    b = rng.normal(0, 0.1, oc).astype(np.float32)
    if not f16:
        g, _, _ = check_against_oracle(x, wt, b, k, s, 0)
        g2, _, _ = check_against_oracle(x, wt, b, k, s, 0, block_n=1 << 30)
        assert np.array_equal(g["acc"], g2["acc"]) and np.array_equal(g["y"], g2["y"])
        return
    xt = torch.from_numpy(nchw_to_nhwc(x)).cuda()
    outs = []
    for bits in (0, 1 << 30):
        plan = ops.ConvPlan.fp16(n, ic, h, w, oc, k, s, wt, b, silu=True, block_n=bits)
        out = torch.zeros((n, h, w, oc), dtype=torch.float16, device="cuda")
        plan.run_nhwc(xt, out=out)
        torch.cuda.synchronize()
        assert plan.status() == 0
        outs.append(out)
    assert torch.equal(outs[0], outs[1])
