"""k x k stride-1 convolutions on the tensor-core implicit GEMM (and narrow 1x1
convs on the row-packed GEMM), one Conv node
per graph, against the oracle's conv (qppocr-kernels conv.rs im2col + panel
GEMM), metric max|d|/max|ref| (reference tests/kernels.rs:51-77).

The cases cover the implicit-GEMM tilings: in TF32, kernels at most 3 wide
with at most 32 output channels take the kx-folded band (the kw taps stacked
in N), output rows >= 64 wide with at most 64 output channels and a filter
that fits in shared memory the row-band tiling (4 output rows per tile,
resident filter); other
rows >= 64 wide take the halo-row tiling (one 128-pixel row per tile, kernel
taps as shifted views of one staged halo row); narrower rows the 2-D
pixel-tile tiling.  Edges cover
left/right/top/bottom padding, rows that end mid-tile, channel counts that
are not a multiple of the 32-channel block, 5x5 kernels, output channel
counts above the halo limit, and a fused ReLU + residual epilogue."""
import numpy as np
import pytest

import oracle as orc
import qppocr_b200 as q
from qppocr_b200 import nets

pytestmark = pytest.mark.gpu

TOL = {"tf32": 1e-3, "3xtf32": 1e-5}

# (batch, cin, cout, k, h, w, act, residual)
CASES = [
    (2, 96, 24, 3, 40, 240, None, False),    # kx-folded band (tf32) / halo, DBFPN-like, 2 x-tiles
    (1, 48, 16, 3, 7, 200, "relu", False),   # kx-folded, M = 16, ragged channel block, 7 rows
    (1, 24, 24, 3, 20, 64, None, True),      # kx-folded with a residual
    (1, 64, 64, 3, 17, 128, "relu", True),   # halo (filter too big for band), relu + residual
    (1, 32, 32, 3, 13, 150, "relu", True),   # band, 13 rows = 3 full bands + 1, relu + residual
    (1, 20, 40, 3, 9, 200, None, False),     # band N=40 (64-col tile), ragged channel block (20 of 32)
    (1, 32, 100, 5, 12, 70, "relu", False),  # 5x5: wider than the halo buffer, tile path
    (1, 24, 32, (1, 3), 8, 100, None, False), # halo, one kernel row
    (1, 24, 32, (3, 1), 8, 100, None, False), # halo, one tap per kernel row
    (1, 48, 136, 3, 10, 96, None, False),    # above the halo N limit: tile path
    (2, 96, 24, 3, 30, 30, None, False),     # tile path, narrow rows
    # 1x1 with 8 / 16 input channels: P = 32 / C pixels packed per GEMM row
    (1, 16, 32, 1, 20, 30, "relu", False),   # P = 2
    (1, 16, 16, 1, 10, 12, "relu", True),    # P = 2 with a residual
    (2, 8, 24, 1, 10, 12, None, False),      # P = 4
    (2, 8, 24, 1, 9, 11, None, False),       # 198 pixels, not a multiple of 4: unpacked
]


def build_conv(cin, cout, k, act, residual, seed=11):
    b = nets.Builder(seed, "cv")
    y = b.conv("x", cin, cout, k, bias=True, bn=True, act=act)
    if residual:
        y = b.node("Add", [y, "x"])
    return b.graph(["x"], [y], [[1, cin, 0, 0]])


@pytest.mark.parametrize("math", ["tf32", "3xtf32"])
@pytest.mark.parametrize("case", CASES, ids=[f"{c[1]}x{c[2]}k{c[3]}_{c[4]}x{c[5]}".replace(" ", "") for c in CASES])
def test_conv_kxk(cuda_ctx, case, math):
    n, cin, cout, k, h, w, act, residual = case
    g, wts = build_conv(cin, cout, k, act, residual)
    g = q.optimize(g, wts)
    x = np.random.Generator(np.random.PCG64(7)).uniform(-1, 1, (n, cin, h, w)).astype(np.float32)
    ref = orc.run_graph(g, wts, {"x": x})[0]
    s = cuda_ctx.create_session(g, wts, role="other", math=math)
    got = s.run({"x": x})[0]
    assert got.shape == ref.shape == (n, cout, h, w)
    err = np.abs(got.astype(np.float64) - ref).max() / max(np.abs(ref).max(), 1e-6)
    assert err < TOL[math], err


UP_CASES = [(1, 32, 24, 1, 20, 30, 2), (1, 32, 24, 3, 16, 96, 2), (2, 16, 16, 1, 24, 24, 4)]


@pytest.mark.parametrize("math", ["tf32", "3xtf32"])
@pytest.mark.parametrize("case", UP_CASES, ids=[f"k{c[3]}_{c[4]}x{c[5]}_up{c[6]}" for c in UP_CASES])
def test_conv_upsampled_residual(cuda_ctx, case, math):
    """Conv + Add(Resize_nearest(z)): the resize is absorbed into the conv's
    epilogue (residual rows read through the nearest-source remap), so the
    upsampled map is never written; results match the unfused oracle."""
    n, cin, cout, k, h, w, up = case
    b = nets.Builder(13, "up")
    y = b.conv("x", cin, cout, k, bias=True, bn=False, act="relu")
    r = b.resize2("z", float(up))
    y = b.node("Add", [y, r])
    g, wts = b.graph(["x", "z"], [y], [[1, cin, 0, 0], [1, cout, 0, 0]])
    g = q.optimize(g, wts)
    rng = np.random.Generator(np.random.PCG64(9))
    x = rng.uniform(-1, 1, (n, cin, h, w)).astype(np.float32)
    z = rng.uniform(-1, 1, (n, cout, h // up, w // up)).astype(np.float32)
    ref = orc.run_graph(g, wts, {"x": x, "z": z})[0]
    s = cuda_ctx.create_session(g, wts, role="other", math=math)
    assert [f[0] for f in s.fused_nodes()] == ["Conv"]
    got = s.run({"x": x, "z": z})[0]
    err = np.abs(got.astype(np.float64) - ref).max() / max(np.abs(ref).max(), 1e-6)
    assert err < TOL[math], err


@pytest.mark.parametrize("hw", [(10, 14), (5, 6), (16, 16)])  # tiles crossing images; images < 128 px; aligned
@pytest.mark.parametrize("math", ["tf32", "3xtf32"])
def test_se_gate_fused_into_pointwise(cuda_ctx, math, hw):
    """SE block (GAP -> 1x1 -> relu -> 1x1 -> HardSigmoid -> Mul) feeding a
    1x1 conv: the gate multiply runs inside the conv's GEMM as A is rounded,
    so the plan has no separate elementwise Mul; results match the oracle."""
    b = nets.Builder(17, "se")
    y = b.se("x", 64)
    y = b.conv(y, 64, 96, 1, bias=True, bn=False, act="hswish")
    g, wts = b.graph(["x"], [y], [[1, 64, 0, 0]])
    g = q.optimize(g, wts)
    x = np.random.Generator(np.random.PCG64(5)).uniform(-1, 1, (3, 64) + hw).astype(np.float32)
    ref = orc.run_graph(g, wts, {"x": x})[0]
    s = cuda_ctx.create_session(g, wts, role="other", math=math)
    got = s.run({"x": x})[0]
    err = np.abs(got.astype(np.float64) - ref).max() / max(np.abs(ref).max(), 1e-6)
    assert err < TOL[math], err
    kinds = [p[0] for p in s.profile({"x": x}, iters=1)]
    assert "binary" not in kinds and "gemm_tc" in kinds, kinds


# (batch, cin, mid, h, w, bn, act1, act2)
PAIR_CASES = [
    (2, 24, 24, 12, 40, True, "Relu", "Sigmoid"),   # DB head tail, rows span images
    (1, 8, 7, 5, 9, False, None, None),            # no BN, no activations, mid < 32, 45 pixels
    (3, 36, 32, 3, 50, True, "Sigmoid", None),     # K = 36: two k-blocks, 32 mid channels
]


@pytest.mark.parametrize("math", ["tf32", "3xtf32"])
@pytest.mark.parametrize("case", PAIR_CASES)
def test_convt_pair_fused(cuda_ctx, math, case):
    """ConvT(C -> M) [+ BN] [+ act] -> ConvT(M -> 1) [-> act]: one tensor-core
    GEMM of the first layer whose epilogue applies the second, so the plan has
    no convt2x2 step; the 4x-upsampled output matches the oracle's two
    ConvTranspose layers (conv.rs:730-838)."""
    n, c, m, h, w, use_bn, act1, act2 = case
    b = nets.Builder(23, "ctp")
    w1 = b.const(b.normal((c, m, 2, 2), np.sqrt(2.0 / (c * 4))), "ct_w")
    y = b.node("ConvTranspose", ["x", w1], {"kernel_shape": [2, 2], "strides": [2, 2]})
    if use_bn:
        y = b.bn(y, m)
    if act1:
        y = b.node(act1, [y])
    w2 = b.const(b.normal((m, 1, 2, 2), np.sqrt(2.0 / (m * 4))), "ct_w")
    y = b.node("ConvTranspose", [y, w2], {"kernel_shape": [2, 2], "strides": [2, 2]})
    if act2:
        y = b.node(act2, [y])
    g, wts = b.graph(["x"], [y], [[1, c, 0, 0]])
    g = q.optimize(g, wts)
    x = np.random.Generator(np.random.PCG64(11)).uniform(-1, 1, (n, c, h, w)).astype(np.float32)
    ref = orc.run_graph(g, wts, {"x": x})[0]
    s = cuda_ctx.create_session(g, wts, role="other", math=math)
    got = s.run({"x": x})[0]
    assert got.shape == (n, 1, 4 * h, 4 * w)
    err = np.abs(got.astype(np.float64) - ref).max() / max(np.abs(ref).max(), 1e-6)
    assert err < TOL[math], err
    kinds = [p[0] for p in s.profile({"x": x}, iters=1)]
    assert "convt_pair" in kinds and "convt2x2" not in kinds, kinds
