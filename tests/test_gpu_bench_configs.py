"""Parity at the sizes the benchmark runs, in both tensor-core modes.

* Config 3, det: one session at B=64 x 3x960x960 (the bench's per-GPU batch:
  its tile counts, persistent schedule, 32-bit row maps and arena reuse), with
  images spread over the batch compared against the oracle; and every fused
  node at 960x960 with teacher forcing.
* Config 4, rec: B=256 x 3x48x320 through the CTC argmax exit and through the
  full-probability path, against the oracle; and every fused node at B=256.

Metric max|d|/max|ref| (tests/kernels.rs:51-77 of the reference).  Per node:
1e-3 (TF32), 1e-5 (3xTF32).  End to end: 1e-5 in 3xTF32; in TF32 the
random-init networks amplify the per-node rounding ~10-60x, so the end-to-end
TF32 bound is E2E_TF32 (the per-node bound is the one TF32 meets).
"""
import numpy as np
import pytest

import oracle as orc
import qppocr_b200 as q
from qppocr_b200 import nets
from test_gpu_layers import per_node
from test_gpu_session import E2E, TOL, check_ctc, load, rel

pytestmark = pytest.mark.gpu

DET_B = 64
DET_SAMPLE = (0, 21, 42, 63)   # images compared with the oracle (~0.15 s each on the host)
REC_B = 256


@pytest.mark.parametrize("math", ["tf32", "3xtf32"])
def test_det_config3_b64_960(cuda_ctx, math):
    g, w = load(nets.build_det)
    x = nets.det_input(DET_B, 960, 960)
    s = cuda_ctx.create_session(g, w, role="det", math=math)
    got = s.run({"x": x})[0]
    s.close()
    assert got.shape == (DET_B, 1, 960, 960)
    assert np.isfinite(got).all()
    ref = orc.run_graph(g, w, {"x": np.ascontiguousarray(x[list(DET_SAMPLE)])})[0]
    for j, i in enumerate(DET_SAMPLE):
        assert rel(got[i], ref[j]) < E2E[math], (i, rel(got[i], ref[j]))


@pytest.mark.parametrize("math", ["tf32", "3xtf32"])
def test_det_per_node_960(cuda_ctx, math):
    fused, errs = per_node(cuda_ctx, nets.build_det, nets.det_input(1, 960, 960, seed=9), math, "det")
    worst = max(errs.items(), key=lambda kv: kv[1][1])
    assert len(errs) >= 40
    assert worst[1][1] < TOL[math], worst


@pytest.mark.parametrize("math", ["tf32", "3xtf32"])
def test_rec_config4_b256(cuda_ctx, math):
    g, w = load(nets.build_rec)
    x = nets.rec_input(REC_B)
    probs = orc.run_graph(g, w, {"x": x})[0]
    s = cuda_ctx.create_session(g, w, role="rec", math=math)
    pairs = s.run({"x": x})[0]
    s.close()
    assert pairs.shape == (REC_B, 40, 2)
    check_ctc(pairs, probs, TOL[math], E2E[math])
    s2 = cuda_ctx.create_session(g, w, role="rec", math=math, argmax_exit=False)
    p2 = s2.run({"x": x})[0]
    s2.close()
    assert p2.shape == probs.shape == (REC_B, 40, nets.REC_CLASSES)
    assert rel(p2, probs) < E2E[math]


@pytest.mark.parametrize("math", ["tf32", "3xtf32"])
def test_rec_per_node_b256(cuda_ctx, math):
    fused, errs = per_node(cuda_ctx, nets.build_rec, nets.rec_input(REC_B, seed=8), math, "rec")
    worst = max(errs.items(), key=lambda kv: kv[1][1])
    assert worst[1][1] < TOL[math], worst
