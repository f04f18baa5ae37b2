"""The fused depthwise-separable kernel (dwpw.cu) against the unfused path.

In TF32 a depthwise conv whose only consumer is a pointwise conv runs as one
tcgen05 kernel (depthwise into shared memory, tf32-rounded, straight into the
pointwise MMA).  Its depthwise half keeps the reference's per-element chain
(conv.rs:45-71) and the MMA sees exactly the A operand the unfused GEMM sees,
so the fused network must equal the unfused one bit for bit.  The unfused
reference run exposes every fused node's output as a graph output, which
keeps each depthwise output in memory (no fusion) without changing any
kernel.  The det backbone covers every fused geometry: 16-channel input
(block 2), stride 2 (block 3a), 3x3 at 64 and 128 channels, and 5x5 at 256
channels; image sizes that are multiples of 32 (as the det input always
is) but not of the tile give partial tiles on both edges.
"""
import copy

import numpy as np
import pytest

import oracle as orc
import qppocr_b200 as q
from qppocr_b200 import nets

pytestmark = pytest.mark.gpu


def rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return np.abs(a - b).max() / max(np.abs(b).max(), 1e-6)


def _fused_and_unfused(ctx, builder, x, role):
    g, w = builder()
    g = q.optimize(g, w)
    s = ctx.create_session(g, w, role=role, math="tf32")
    fused_kernels = {k for k, *_ in s.profile({"x": x}, iters=1)}
    got = s.run({"x": x})[0]
    nodes = s.fused_nodes()
    s.close()
    g2 = copy.deepcopy(g)
    g2.outputs = list(dict.fromkeys([o for _, _, o in nodes] + list(g.outputs)))
    s2 = ctx.create_session(g2, w, role=role, math="tf32")
    unfused_kernels = {k for k, *_ in s2.profile({"x": x}, iters=1)}
    ref = s2.run({"x": x})[g2.outputs.index(g.outputs[0])]
    s2.close()
    return g, w, got, ref, fused_kernels, unfused_kernels


@pytest.mark.parametrize("shape", [(2, 3, 160, 224), (1, 3, 288, 352)])
def test_det_fused_equals_unfused(cuda_ctx, shape):
    x = nets.det_input(shape[0], shape[2], shape[3], seed=11)
    g, w, got, ref, fk, uk = _fused_and_unfused(cuda_ctx, nets.build_det, x, "det")
    assert "dwpw" in fk and "dwpw" not in uk
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32)), rel(got, ref)
    # and both against the oracle, at the end-to-end TF32 bound
    assert rel(got, orc.run_graph(g, w, {"x": x})[0]) < 1e-2


def test_block_config1_fused_per_launch(cuda_ctx):
    """Config 1 runs as the fused kernel plus the layout copies around it."""
    g, w = nets.build_block()
    g = q.optimize(g, w)
    x = nets.block_input(0)
    s = cuda_ctx.create_session(g, w, math="tf32")
    kernels = [k for k, *_ in s.profile({"x": x}, iters=1)]
    got = s.run({"x": x})[0]
    s.close()
    assert kernels.count("dwpw") == 1 and "dwconv" not in kernels and "gemm_tc" not in kernels, kernels
    assert rel(got, orc.run_graph(g, w, {"x": x})[0]) < 1e-3
