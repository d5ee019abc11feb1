"""CPU tests of the oracle itself: pinned against the reference's own outputs
and known-answer test, and against its committed regression fixtures."""
import numpy as np
import pytest

from oracle import w8a8 as ow


def test_weight_quantizer_matches_reference_compiler(golden_dir):
    """Layout-8 bytes equal those of the reference's _add_packed_conv_int8 (engine.py:2418-2465)."""
    d = np.load(f"{golden_dir}/weights_layout8.npz")
    for i in range(int(d["count"])):
        q, s = ow.quantize_conv_weight_int8(d[f"w{i}"], int(d[f"prec{i}"]) == 2)
        assert ow.layout8_payload(q, s) == d[f"payload{i}"].tobytes(), f"case {i}"


def test_weight_quantizer_edge_cases():
    w = np.zeros((3, 1, 1, 4), np.float32)
    w[1] = [[[1.27, 0.005, -0.015, -1.27]]]  # scale 0.01 -> 0.5, -1.5 are exact half-way products
    w[2] = [[[1e-30, -2e-30, 0.0, 3e-30]]]
    q, s = ow.quantize_conv_weight_int8(w)
    assert s[0] == np.float32(1.0) and (q[0] == 0).all()  # all-zero channel
    assert list(q[1]) == [127, 1, -2, -127]  # half away from zero, not half even
    assert abs(int(q[2][3])) == 127


def test_pg16_known_answer_of_reference():
    """mobile/hal/vk_hal.c:187-252: LCG inputs, K=256, OC=8, pg16 dequant in ascending groups."""
    a, w, a_scale, w_scale, expect = ow.pg16_known_answer()
    acc_g = ow.conv_acc_i32(a.reshape(1, 256, 1, 1), w, 1, 1, 0, group_ch=16)
    fp = ow.pg16_sum(acc_g, a_scale.reshape(1, 16)).reshape(8)
    got = (fp * w_scale).astype(np.float32)
    assert np.array_equal(got, expect)
    assert np.all(np.abs(got - expect) <= 1e-3 * (1 + np.abs(expect)))  # the reference's own gate


def test_act_quantize_rounding_and_wrap():
    # amax 127 -> s = 1: codes are round-half-even of x
    x = np.array([0.5, 1.5, 2.5, -0.5, -1.5, -2.5, 127.0, -127.0] + [0.0] * 8, np.float32).reshape(1, 16, 1, 1)
    at, ag = ow.act_amax(x)
    q = ow.quantize_act(x, at, ag, ow.SCALE_PER_TENSOR).reshape(-1)
    assert list(q[:8]) == [0, 2, 2, 0, -2, -2, 127, -127]
    # no clamp: a code beyond 127 wraps through the low byte (runtime.cpp:3339-3344)
    q2 = ow.quantize_act(np.full((1, 16, 1, 1), 128.0, np.float32), np.array([127.0], np.float32), ag,
                         ow.SCALE_PER_TENSOR)
    assert (q2 == -128).all()
    # amax 0 -> zero codes
    z = np.zeros((2, 16, 3, 3), np.float16)
    at, ag = ow.act_amax(z)
    assert (ow.quantize_act(z, at, ag, ow.SCALE_PG16) == 0).all()


def test_act_amax_partial_group():
    rng = np.random.default_rng(0)
    x = rng.standard_normal((2, 20, 3, 5)).astype(np.float16)
    at, ag = ow.act_amax(x)
    assert ag.shape == (2, 2)
    np.testing.assert_array_equal(ag[:, 1], np.abs(x[:, 16:].astype(np.float32)).reshape(2, -1).max(1))
    np.testing.assert_array_equal(at, np.abs(x.astype(np.float32)).reshape(2, -1).max(1))


@pytest.mark.parametrize("k,s,p", [(1, 1, 0), (3, 1, 1), (3, 2, 1)])
def test_conv_acc_c_matches_numpy(k, s, p):
    rng = np.random.default_rng(k * 10 + s)
    x = rng.integers(-128, 128, (2, 32, 9, 7)).astype(np.int8)
    w = rng.integers(-127, 128, (16, 32 * k * k)).astype(np.int8)
    a = ow.conv_acc_i32(x, w, k, s, p)
    lib = ow._CLIB
    try:
        ow._CLIB = False
        b = ow.conv_acc_i32(x, w, k, s, p)
    finally:
        ow._CLIB = lib
    g = ow.conv_acc_i32(x, w, k, s, p, group_ch=16)
    assert np.array_equal(a, b)
    assert np.array_equal(a, g.sum(axis=1))


def test_int8_guard_table():
    g = ow.can_use_conv_int8
    assert g(64, 128, 80, 80, 80, 80, 3, 1, 1)
    assert g(64, 128, 80, 80, 40, 40, 3, 2, 1)
    assert g(64, 128, 81, 81, 41, 41, 3, 2, 1)
    assert g(128, 128, 40, 40, 40, 40, 1, 1, 0)
    assert not g(128, 124, 40, 40, 40, 40, 1, 1, 0)  # 1x1 needs oc % 8
    assert not g(3, 16, 320, 320, 160, 160, 3, 2, 1)  # ic % 4 (the stem stays fp16)
    assert not g(64, 64, 80, 80, 80, 80, 3, 1, 1, groups=2)
    assert not g(64, 64, 80, 80, 80, 80, 3, 1, 0)


def test_act_cases_regression(golden_dir):
    """The committed oracle fixtures are reproduced exactly (incl. fp16 outputs)."""
    d = np.load(f"{golden_dir}/act_cases.npz")
    for name in d["names"]:
        name = str(name)
        n, ic, h, w, oc, k, s, p, mode, silu, res = (int(v) for v in d[name + ".meta"])
        o = ow.conv_w8a8(d[name + ".x"], d[name + ".w"], d[name + ".b"], k, s, p, mode=mode, silu=bool(silu),
                         residual=d[name + ".res"] if res else None)
        for key in ("amax_t", "amax_g", "xq", "wq", "w_scale", "acc", "y"):
            assert np.array_equal(o[key], d[name + "." + key]), (name, key)


def test_tiny_engine_kernel_plan(golden_dir):
    """The reference compiler's plan for the tiny engine: kernels 52 (pg16), 53, 51."""
    d = np.load(f"{golden_dir}/tiny_w8a8.npz")
    plan = d["kernel_plan"]
    convs = [r for r in plan if int(r[1]) in (1, 2)]
    assert [int(r[2]) for r in convs] == [52, 53, 51]
    assert [bool(int(r[5]) & 16) for r in convs] == [True, False, False]


# ---------------------------------------------------------------- YOLO post-process
def _post_cases(golden_dir):
    d = np.load(f"{golden_dir}/yolo_post.npz")
    for name in d["names"]:
        nc, conf, iou = d[name + ".meta"]
        yield str(name), d[name + ".y"], int(nc), float(conf), float(iou), d[name + ".dets"]


def test_post_greedy_matches_reference_yolo_postprocess(golden_dir):
    """Greedy mode reproduces the reference's own yolo_postprocess (src/aexrt/yolo.py:92-138) bit for bit."""
    from oracle import yolo_post as op

    for name, y, nc, conf, iou, ref in _post_cases(golden_dir):
        dets, count = op.postprocess(y, nc, conf, iou, max_candidates=1 << 20, max_detections=1 << 20,
                                     mode=op.MODE_GREEDY)
        assert count == ref.shape[0], name
        assert np.array_equal(dets, ref), name


def test_post_mark_rule_matches_shader_loops(golden_dir):
    """The vectorised mark rule equals the mark shader's loop (runtime.cpp:15664-15684) written out."""
    from oracle import yolo_post as op

    for name, y, nc, conf, iou, _ in _post_cases(golden_dir):
        cand = op.decode_filter(y, nc, conf, 300)
        assert np.array_equal(op.nms_keep(cand, iou, op.MODE_MARK), op.nms_mark_loops(cand, iou)), name
    # ties: equal scores rank by candidate index, as the shader's `score_j == score_i && j < i`
    cand = np.array([[0, 0, 10, 10, 0.5, 0], [1, 1, 11, 11, 0.5, 0], [2, 2, 12, 12, 0.5, 0],
                     [50, 50, 60, 60, 0.5, 0], [0, 0, 10, 10, 0.9, 1]], np.float32)
    keep = op.nms_keep(cand, 0.45, op.MODE_MARK)
    assert list(keep) == [True, False, False, True, True]
    assert np.array_equal(keep, op.nms_mark_loops(cand, 0.45))
    # mark drops box 2 (suppressed by box 1, itself suppressed); greedy keeps it
    cand = np.array([[0, 0, 10, 10, 0.9, 0], [4, 0, 14, 10, 0.8, 0], [8, 0, 18, 10, 0.7, 0]], np.float32)
    assert list(op.nms_keep(cand, 0.3, op.MODE_MARK)) == [True, False, False]
    assert list(op.nms_keep(cand, 0.3, op.MODE_GREEDY)) == [True, False, True]


def test_post_candidate_cap_and_topk():
    from oracle import yolo_post as op

    rng = np.random.default_rng(3)
    y = rng.uniform(0, 1, (6, 400)).astype(np.float32)
    y[:2] *= 320
    y[2:4] = y[2:4] * 20 + 2
    cand = op.decode_filter(y, 2, 0.0, 100)
    assert cand.shape[0] == 100  # the first 100 anchors in anchor order
    assert np.array_equal(cand[:, 4], np.maximum(y[4], y[5])[:100])
    dets, count = op.postprocess(y, 2, 0.0, 0.45, 100, 7)
    assert count == 7 and dets.shape == (7, 6)
    assert np.all(np.diff(dets[:, 4]) <= 0)
    dets, count = op.postprocess(y, 2, 2.0, 0.45, 100, 7)
    assert count == 0 and dets.shape == (0, 6)
