"""GPU parity of the YOLO post-process kernel (aexrt_b200_yolo_nms_topk) against the oracle.

The bar is bit-exact: the same candidates, kept set, order and float32 rows.  Greedy mode is
also checked directly against the detections that the reference's own yolo_postprocess
returned for the committed fixtures."""
import numpy as np
import pytest

from oracle import yolo_post as op

pytestmark = pytest.mark.gpu


def _run(y, nc, conf, iou, mc, md, mode, has_obj=False, channels_last=False, ctas=0):
    import torch

    from aexrt_b200 import ops

    t = torch.from_numpy(np.ascontiguousarray(y, dtype=np.float32)).cuda()
    dets, counts = ops.yolo_nms_topk(t, nc, conf, iou, mc, md, mode, has_objectness=has_obj,
                                     channels_last=channels_last, ctas_per_image=ctas)
    torch.cuda.synchronize()
    return dets.cpu().numpy(), counts.cpu().numpy()


def _check(y, nc, conf, iou, mc, md, mode, has_obj=False, channels_last=False, ctas=0):
    dets, counts = _run(y, nc, conf, iou, mc, md, mode, has_obj, channels_last, ctas)
    for i in range(y.shape[0]):
        ref, cnt = op.postprocess(y[i], nc, conf, iou, mc, md, mode, has_obj, channels_last)
        assert counts[i] == cnt, (i, counts[i], cnt)
        assert np.array_equal(dets[i, :cnt], ref), i
    return counts


def _clustered(rng, n, nc, anchors, objects, channels_last=False, has_obj=False):
    from tests.golden.make_golden import synthetic_head_output

    ys = [synthetic_head_output(rng, nc, anchors, objects) for _ in range(n)]
    y = np.stack(ys)
    if has_obj:
        obj = rng.uniform(0.3, 1.0, (n, 1, anchors)).astype(np.float32)
        y = np.concatenate([y[:, :4], obj, y[:, 4:]], axis=1)
    if channels_last:
        y = np.ascontiguousarray(y.transpose(0, 2, 1))
    return y


def test_greedy_matches_reference_yolo_postprocess(golden_dir):
    d = np.load(f"{golden_dir}/yolo_post.npz")
    for name in d["names"]:
        nc, conf, iou = d[name + ".meta"]
        y = d[name + ".y"][None]
        dets, counts = _run(y, int(nc), float(conf), float(iou), 1024, 1024, op.MODE_GREEDY)
        ref = d[name + ".dets"]
        assert counts[0] == ref.shape[0], name
        assert np.array_equal(dets[0, :counts[0]], ref), name


@pytest.mark.parametrize("mode", [op.MODE_MARK, op.MODE_GREEDY])
def test_batch_matches_oracle(mode):
    rng = np.random.default_rng(40 + mode)
    y = _clustered(rng, 5, 4, 2100, 25)  # YOLOv8n-320: 2100 anchors
    counts = _check(y, 4, 0.25, 0.45, 512, 100, mode)
    assert counts.max() > 0


@pytest.mark.parametrize("ctas", [1, 2, 4, 8])
@pytest.mark.parametrize("mode", [op.MODE_MARK, op.MODE_GREEDY])
def test_cluster_sizes_give_the_same_detections(mode, ctas):
    # one image's pair tests shared by a cluster of 1-8 CTAs; the full candidate cap (the greedy
    # matrix at its largest) and a small one that leaves most CTAs without rows
    rng = np.random.default_rng(70 + mode)
    y = _clustered(rng, 3, 4, 8400, 120)
    _check(y, 4, 0.05, 0.45, 1024, 300, mode, ctas=ctas)
    _check(y[:1], 4, 0.25, 0.45, 40, 10, mode, ctas=ctas)


def test_automatic_cluster_size_across_batches():
    # automatic CTAs per image: 8 (batch 1-37), 4, 2, then 1 from batch 149 on
    rng = np.random.default_rng(77)
    base = _clustered(rng, 4, 4, 2100, 25)
    for n in (1, 40, 100, 160):
        y = base[np.arange(n) % 4]
        _check(y, 4, 0.25, 0.45, 512, 100, op.MODE_MARK)


def test_bad_cluster_size_is_refused():
    import torch

    from aexrt_b200 import ops

    t = torch.zeros((1, 8, 64), dtype=torch.float32, device="cuda")
    with pytest.raises(RuntimeError, match="mode"):
        ops.yolo_nms_topk(t, 4, ctas_per_image=3)


@pytest.mark.parametrize("mc,md", [(512, 100), (300, 1000), (1024, 1024), (1, 1), (37, 5)])
def test_candidate_cap_and_detection_limit(mc, md):
    """More passing anchors than max_candidates: the first ones in anchor order are kept."""
    rng = np.random.default_rng(mc + md)
    y = _clustered(rng, 2, 3, 2100, 60)
    for mode in (op.MODE_MARK, op.MODE_GREEDY):
        _check(y, 3, 0.05, 0.5, mc, md, mode)


def test_objectness_and_channels_last():
    rng = np.random.default_rng(9)
    for has_obj in (False, True):
        for cl in (False, True):
            y = _clustered(rng, 2, 6, 1500, 20, channels_last=cl, has_obj=has_obj)
            for mode in (op.MODE_MARK, op.MODE_GREEDY):
                _check(y, 6, 0.2, 0.45, 512, 100, mode, has_obj, cl)


def test_score_ties_rank_by_anchor_order():
    """fp16-rounded scores tie often; both rules rank ties by candidate (anchor) index."""
    rng = np.random.default_rng(11)
    y = _clustered(rng, 3, 4, 2100, 30).astype(np.float16).astype(np.float32)
    y[:, 4:] = np.round(y[:, 4:] * 16) / 16
    for mode in (op.MODE_MARK, op.MODE_GREEDY):
        _check(y, 4, 0.25, 0.45, 512, 100, mode)


def test_no_candidates_and_eighty_classes():
    rng = np.random.default_rng(12)
    y = _clustered(rng, 2, 80, 8400, 40)  # YOLOv8s-640 head: 8400 anchors, 80 classes
    counts = _check(y, 80, 2.0, 0.45, 512, 100, op.MODE_MARK)  # nothing reaches conf 2
    assert (counts == 0).all()
    _check(y, 80, 0.25, 0.45, 512, 100, op.MODE_MARK)
    _check(y, 80, 0.25, 0.6, 1024, 300, op.MODE_GREEDY)


def test_iou_exactly_at_and_next_to_the_threshold():
    """Thresholds equal to a pair's float32 IoU (not suppressed: the rule is IoU > threshold) and one
    float step either side of it: the kernel's decision, which divides only near the threshold,
    equals the float32 division's."""
    rng = np.random.default_rng(77)
    pairs = 24
    y = np.zeros((1, 5, 2 * pairs), np.float32)
    y[0, 4] = np.linspace(0.9, 0.3, 2 * pairs, dtype=np.float32)  # one class, distinct scores
    for pidx in range(pairs):
        w, h = rng.uniform(5, 50, 2).astype(np.float32)
        dx, dy = rng.uniform(0, 0.4, 2).astype(np.float32) * np.array([w, h], np.float32)
        for member, (ox, oy) in enumerate(((0, 0), (dx, dy))):
            k = 2 * pidx + member
            y[0, 0:4, k] = [np.float32(200 * pidx) + ox, oy, w, h]
    cand = op.decode_filter(y[0], 1, 0.25, 512)
    ious = [float(op.iou_matrix(cand[[2 * q, 2 * q + 1], :4])[0, 1]) for q in range(pairs)]
    for q in (0, 5, 11):
        t = np.float32(ious[q])
        for thr in (t, np.nextafter(t, np.float32(0)), np.nextafter(t, np.float32(1))):
            for mode in (op.MODE_MARK, op.MODE_GREEDY):
                _check(y, 1, 0.25, float(thr), 512, 100, mode)
