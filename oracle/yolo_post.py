"""CPU oracle of the YOLO post-process: confidence filter, NMS, top-k (TEST INFRASTRUCTURE ONLY).

Restates, per image, the two post-processes of the reference:

* the GPU path that ``aexrt_yolo_run`` records (native/aexrt_d3d12_runtime.cpp:27104-27219):
  - decode-filter shader (``:15300-15355``): per anchor, best class = first maximum of
    objectness * class score, kept when best >= conf_threshold, box cx/cy/w/h -> x1y1x2y2;
    candidates appended up to ``max_candidates``;
  - NMS "mark" shader (``:15637-15691``): candidate i is kept unless some candidate j of the
    same class ranks above it (higher score, or equal score and j < i) with IoU > threshold,
    whether or not j itself is kept;
  - top-k shader (``:15693-15733``): kept candidates ranked by (score desc, index asc); the
    first ``max_detections`` are written, count = min(kept, max_detections);
* the Python path ``yolo_postprocess`` (src/aexrt/yolo.py:92-138, ``_nms`` :996-1007,
  ``_iou`` :1010-1018): the same filter, then greedy per-class NMS (a box is dropped only by a
  KEPT higher-scoring box) with no candidate cap, sorted by score.

The reference appends GPU candidates with an atomic counter, so their order (and which ones
survive the cap) is whatever order the atomics ran in.  This restatement fixes it to ascending
anchor index, one of the orders the reference can produce, and the CUDA kernel does the same.
All box and IoU arithmetic is float32, one IEEE operation at a time, in the shader's order.

Modes: ``MODE_MARK`` (0) = the GPU shaders; ``MODE_GREEDY`` (1) = yolo_postprocess's greedy NMS
(with the same candidate cap and top-k as the GPU path).
"""
from __future__ import annotations

from typing import Tuple

import numpy as np

F32 = np.float32
MODE_MARK = 0
MODE_GREEDY = 1


def decode_filter(y: np.ndarray, nc: int, conf: float, max_candidates: int, has_objectness: bool = False,
                  channels_last: bool = False) -> np.ndarray:
    """Candidates of one image: rows (x1, y1, x2, y2, score, class) float32, anchor order, capped.

    `y` is one image's output0: [channels][anchors], or [anchors][channels] when channels_last
    (the shader's ``layout == 2``)."""
    y = np.asarray(y, dtype=F32)
    if channels_last:
        y = y.T
    off = 5 if has_objectness else 4
    scores = y[off:off + nc].T.copy()
    if has_objectness:
        scores = scores * y[4][:, None]
    cls = np.argmax(scores, axis=1)  # first maximum, like the shader's strict `s > best`
    best = scores[np.arange(scores.shape[0]), cls]
    keep = np.nonzero(~(best < F32(conf)))[0][:max_candidates]
    cx, cy, w, h = (y[i][keep] for i in range(4))
    half = F32(0.5)
    out = np.empty((keep.size, 6), dtype=F32)
    out[:, 0] = cx - w * half
    out[:, 1] = cy - h * half
    out[:, 2] = cx + w * half
    out[:, 3] = cy + h * half
    out[:, 4] = best[keep]
    out[:, 5] = cls[keep].astype(F32)
    return out


def iou_matrix(b: np.ndarray) -> np.ndarray:
    """IoU of every pair of x1y1x2y2 boxes, float32, in the mark shader's operation order (:15646-15658)."""
    x1 = np.maximum(b[:, None, 0], b[None, :, 0])
    y1 = np.maximum(b[:, None, 1], b[None, :, 1])
    x2 = np.minimum(b[:, None, 2], b[None, :, 2])
    y2 = np.minimum(b[:, None, 3], b[None, :, 3])
    zero = F32(0)
    inter = np.maximum(zero, x2 - x1) * np.maximum(zero, y2 - y1)
    area = np.maximum(zero, b[:, 2] - b[:, 0]) * np.maximum(zero, b[:, 3] - b[:, 1])
    return inter / np.maximum((area[:, None] + area[None, :]) - inter, F32(1e-7))


def rank_order(cand: np.ndarray) -> np.ndarray:
    """Candidate indices by (score desc, index asc): the ordering both NMS shaders use."""
    return np.lexsort((np.arange(cand.shape[0]), -cand[:, 4].astype(np.float64)))


def nms_keep(cand: np.ndarray, iou: float, mode: int) -> np.ndarray:
    """Keep flags per candidate (candidate order)."""
    m = cand.shape[0]
    if m == 0:
        return np.zeros(0, dtype=bool)
    order = rank_order(cand)
    b = cand[order]
    same = b[:, None, 5] == b[None, :, 5]
    sup = same & (iou_matrix(b[:, :4]) > F32(iou))
    sup &= np.triu(np.ones((m, m), dtype=bool), 1)  # row r suppresses only lower-ranked columns
    kept_sorted = np.ones(m, dtype=bool)
    if mode == MODE_MARK:
        kept_sorted = ~sup.any(axis=0)
    else:
        for r in range(m):
            if kept_sorted[r]:
                kept_sorted &= ~sup[r]
    keep = np.zeros(m, dtype=bool)
    keep[order] = kept_sorted
    return keep


def postprocess(y: np.ndarray, nc: int, conf: float = 0.25, iou: float = 0.45, max_candidates: int = 512,
                max_detections: int = 100, mode: int = MODE_MARK, has_objectness: bool = False,
                channels_last: bool = False) -> Tuple[np.ndarray, int]:
    """Detections of one image: ([count][6] float32 rows x1, y1, x2, y2, score, class; count)."""
    cand = decode_filter(y, nc, conf, max_candidates, has_objectness, channels_last)
    keep = nms_keep(cand, iou, mode)
    order = rank_order(cand)
    ranked = [i for i in order if keep[i]][:max_detections]
    return cand[ranked].reshape(-1, 6), len(ranked)


def nms_mark_loops(cand: np.ndarray, iou: float) -> np.ndarray:
    """The mark shader's per-candidate loop, written out literally (small cases only): cross-check
    of :func:`nms_keep` in MODE_MARK."""
    m = cand.shape[0]
    keep = np.ones(m, dtype=bool)
    for i in range(m):
        for j in range(m):
            if j == i or cand[j, 5] != cand[i, 5]:
                continue
            higher = cand[j, 4] > cand[i, 4] or (cand[j, 4] == cand[i, 4] and j < i)
            if higher and iou_matrix(cand[[i, j], :4])[0, 1] > F32(iou):
                keep[i] = False
                break
    return keep
