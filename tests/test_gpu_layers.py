"""Per-node parity with teacher forcing (dump-compare stepping, as the
reference's QPPOCR_GPU_DUMP_CMP does, vulkan/session.rs:542-600).

Every fused node's output is exposed as a graph output; the oracle evaluates
each reference node on the GPU's own inputs to that node, so each kernel's
error is measured alone rather than after amplification by the layers before
it.  Tolerance per node: max|d|/max|ref| < 1e-3 (TF32), < 1e-5 (3xTF32)."""
import copy

import numpy as np
import pytest

import oracle as orc
import qppocr_b200 as q
from qppocr_b200 import nets

pytestmark = pytest.mark.gpu

TOL = {"tf32": 1e-3, "3xtf32": 1e-5}


def rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return np.abs(a - b).max() / max(np.abs(b).max(), 1e-6)


def per_node(ctx, builder, x, math, role, **kw):
    g, w = builder(**kw)
    g = q.optimize(g, w)
    s0 = ctx.create_session(g, w, role=role, math=math, argmax_exit=False)
    fused = s0.fused_nodes()
    s0.close()
    outs = list(dict.fromkeys([o for _, _, o in fused] + list(g.outputs)))
    g2 = copy.deepcopy(g)
    g2.outputs = outs
    s = ctx.create_session(g2, w, role=role, math=math, argmax_exit=False)
    assert [f[0] for f in s.fused_nodes()] == [f[0] for f in fused]  # same fusion
    gpu = dict(zip(outs, s.run({"x": x})))
    s.close()
    vals = {"x": x}
    errs = {}

    def get(name):
        if name in gpu:
            return gpu[name]
        if name in vals:
            return vals[name]
        return w[name]

    for n in g.nodes:
        y = orc.eval_node(n, get)
        vals[n.outputs[0]] = y
        if n.outputs[0] in gpu:
            errs[n.outputs[0]] = (n.op_type, rel(gpu[n.outputs[0]], y))
    return fused, errs


@pytest.mark.parametrize("math", ["tf32", "3xtf32"])
def test_det_per_node(cuda_ctx, math):
    fused, errs = per_node(cuda_ctx, nets.build_det, nets.det_input(2, 128, 160), math, "det")
    ops = [f[0] for f in fused]
    assert "QpcConvTPair" in ops and ops.count("Conv") >= 40
    worst = max(errs.items(), key=lambda kv: kv[1][1])
    assert worst[1][1] < TOL[math], worst


@pytest.mark.parametrize("math", ["tf32", "3xtf32"])
def test_rec_per_node(cuda_ctx, math):
    fused, errs = per_node(cuda_ctx, nets.build_rec, nets.rec_input(4), math, "rec")
    ops = [f[0] for f in fused]
    assert ops.count("QpcLayerNorm") == 5 and ops.count("QpcLinear") >= 9
    # the fused attention (scale, QK^T, softmax, PV) is bit-exact on its own input
    att = [o for op, _, o in fused if op == "QpcAttention"]
    assert len(att) == 2
    assert all(errs[o][1] == 0.0 for o in att), [errs[o] for o in att]
    worst = max(errs.items(), key=lambda kv: kv[1][1])
    assert worst[1][1] < TOL[math], worst


@pytest.mark.parametrize("math", ["tf32", "3xtf32"])
def test_cls_per_node(cuda_ctx, math):
    fused, errs = per_node(cuda_ctx, nets.build_cls, nets.cls_input(8), math, "cls")
    worst = max(errs.items(), key=lambda kv: kv[1][1])
    assert worst[1][1] < TOL[math], worst


@pytest.mark.parametrize("rows,c", [(77, 120), (8, 120), (1, 12), (300, 36), (45, 30), (19, 400)])
def test_layernorm_bit_exact(cuda_ctx, rows, c):
    """The fused LayerNorm (sequential f64 sums per row in index order,
    shape.rs:510-566) equals the oracle's decomposed chain bit for bit, for
    ragged row counts and both kernel paths: rows of <= 352 channels with
    C % 4 == 0 take the shared-memory kernel (8 rows per warp), the others
    one thread per row.  The output is a graph output, so it is stored
    unrounded; a linear consumer would get it tf32-rounded."""
    b = nets.Builder(5, "ln")
    y = b.layernorm("x", c)
    g, w = b.graph(["x"], [y], [[1, 0, c]])
    g = q.optimize(g, w)
    rng = np.random.Generator(np.random.PCG64(rows * 1000 + c))
    x = (rng.standard_normal((1, rows, c)) * 3 + 0.5).astype(np.float32)
    ref = orc.run_graph(g, w, {"x": x})[0]
    s = cuda_ctx.create_session(g, w, role="other", math="tf32")
    assert [f[0] for f in s.fused_nodes()] == ["QpcLayerNorm"]
    got = s.run({"x": x})[0]
    assert got.shape == ref.shape == (1, rows, c)
    assert np.array_equal(got, ref), rel(got, ref)


def test_layernorm_edge_rows(cuda_ctx):
    """Rows whose f64 sums are sensitive to order or sign: constant (all
    deviations zero), zeros of both signs, a 1e-30 .. 1e3 range, small
    perturbations of 1 (tiny squared deviations), near-underflow terms, and
    ordinary ones; the fused LayerNorm must equal the oracle's sequential
    f64 sums bit for bit."""
    c, rows = 120, 37
    b = nets.Builder(6, "lnx")
    y = b.layernorm("x", c)
    g, w = b.graph(["x"], [y], [[1, 0, c]])
    g = q.optimize(g, w)
    rng = np.random.Generator(np.random.PCG64(99))
    x = (rng.standard_normal((1, rows, c)) * 2).astype(np.float32)
    x[0, 0] = 0.75
    x[0, 1] = 0.0
    x[0, 1, ::3] = -0.0
    x[0, 2] = rng.standard_normal(c) * 1e3
    x[0, 2, ::7] = 1e-30
    x[0, 3] = 1.0 + rng.standard_normal(c) * 1e-6
    x[0, 4, ::5] = 3e-38
    x = x.astype(np.float32)
    ref = orc.run_graph(g, w, {"x": x})[0]
    s = cuda_ctx.create_session(g, w, role="other", math="tf32")
    got = s.run({"x": x})[0]
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32)) or np.array_equal(got, ref), rel(got, ref)


@pytest.mark.parametrize("width", [200, 56])
def test_rec_attention_runtime_sizes(cuda_ctx, width):
    """The fused attention at token counts other than the compile-time 40
    (width / 8: T = 25, a partial group of 4 query rows, and T = 7, a row
    shorter than the softmax's 8 accumulators) stays bit-exact on its own
    input."""
    fused, errs = per_node(cuda_ctx, nets.build_rec, nets.rec_input(2, w=width), "tf32", "rec")
    att = [o for op, _, o in fused if op == "QpcAttention"]
    assert len(att) == 2
    assert all(errs[o][1] == 0.0 for o in att), [errs[o] for o in att]
