"""Times the reference's own fp32 CPU path on the YOLOv8n-320 graph (TEST INFRASTRUCTURE).

The reference has no CPU W8A8 path; its fp32 graph runs on the host through
`InferenceSession(graph, backend="torch", device="cpu")` (src/aexrt/session.py:10-94,
src/aexrt/backends/torch_backend.py).  This script builds the same YOLOv8n-320 program the bench
runs as the reference's own `aexrt.Graph` (the ONNX-export form, `tests/golden/make_golden.py`
`program_graph`), compiles it into that session and times `run` over single images on every host
thread.  It needs the reference's source tree (the build container only):

    python oracle/time_reference_torch.py --reference-src <reference>/src [--images 20]
"""
import argparse
import importlib.util
import json
import os
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference-src", required=True)
    ap.add_argument("--images", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    a = ap.parse_args()
    sys.path.insert(0, a.reference_src)
    sys.path.insert(0, ROOT)
    import torch

    import aexrt
    from aexrt.session import InferenceSession

    from aexrt_b200 import yolo

    spec = importlib.util.spec_from_file_location("make_golden", os.path.join(ROOT, "tests", "golden", "make_golden.py"))
    mg = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mg)
    cores = len(os.sched_getaffinity(0))
    torch.set_num_threads(cores)
    prog = yolo.build_yolov8n(nc=4, imgsz=320, seed=0)
    graph, _ = mg.program_graph(aexrt, prog)
    sess = InferenceSession(graph, backend="torch", device="cpu")
    rng = np.random.default_rng(0)
    imgs = rng.uniform(0, 1, (a.warmup + a.images, 1, 3, 320, 320)).astype(np.float32)
    for i in range(a.warmup):
        sess.run({"images": imgs[i]})
    t0 = time.perf_counter()
    for i in range(a.images):
        sess.run({"images": imgs[a.warmup + i]})
    dt = time.perf_counter() - t0
    print(json.dumps({"what": "reference InferenceSession(backend='torch', device='cpu'), fp32, YOLOv8n-320 nc=4, batch 1",
                      "images_per_s": a.images / dt, "ms_per_image": dt / a.images * 1e3, "threads": cores,
                      "images": a.images}))
    return 0


if __name__ == "__main__":
    sys.exit(main())
