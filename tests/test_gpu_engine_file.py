"""GPU run of an engine compiled by the reference's own compiler (tests/golden/tiny_w8a8.aexrt:
3x3 s1 pg16 -> 3x3 s2 -> 1x1, all CONV_SILU on kernels 52/53/51, fp16 precision) through
aexrt_b200.aexrt_engine.EngineRunner, checked layer by layer against the oracle fed the device's
own inputs: int8 codes bit-exact, fp16 outputs within 1e-2."""
import numpy as np
import pytest

from aexrt_b200 import aexrt_engine as ae
from oracle import w8a8 as ow
from tests._util import slab16_to_nchw

pytestmark = pytest.mark.gpu


def test_reference_engine_runs_layer_by_layer_against_oracle(golden_dir):
    import torch

    e = ae.load_engine(f"{golden_dir}/tiny_w8a8.aexrt")
    runner = ae.EngineRunner(e)
    rng = np.random.default_rng(17)
    # fp16-representable input (the runner rounds the graph input to fp16 on upload)
    x = rng.uniform(-2, 2, e.shape(0)).astype(np.float16).astype(np.float32)
    y = runner.run(x)
    torch.cuda.synchronize()
    assert runner.status() == 0
    assert y.shape == e.shape(10)
    cur = x.astype(np.float16)
    for _, cmd, plan, parts, scratch, _hw in runner.steps:
        n, ic, ih, iw, oc, oh, ow_, k, _, s = ae.conv_desc(cmd)[:10]
        codes, scale = ae.int8_weights(e, cmd)
        mode = 1 if cmd.flags & ae.PLAN_FLAG_INT8_PERGROUP else 0
        o = ow.conv_w8a8(cur, None, e.constants[cmd.inputs[2]], k, s, k // 2, mode=mode, wq=codes, w_scale=scale)
        q = scratch[0].cpu().numpy()
        assert np.array_equal(slab16_to_nchw(q, ic, ih, iw, s), o["xq"]), cmd.output
        got = runner.bufs[cmd.output].float().cpu().numpy().transpose(0, 3, 1, 2)
        assert np.abs(got - o["y32"]).max() <= 1e-2, cmd.output
        cur = runner.bufs[cmd.output].cpu().numpy().transpose(0, 3, 1, 2)  # the device's own fp16 output
    # the graph output is the last conv's output reshaped to [1, 8, 64] (NCHW order)
    assert np.array_equal(y.reshape(-1), cur.astype(np.float32).reshape(-1))
    # a CUDA-graph replay gives the same output
    runner.capture()
    assert np.array_equal(runner.run(x), y)
