"""Operator-level parity on the B200 through the C ABI (device pointers)
against the CPU oracle.  Tolerances: the reference's max|d|/max|ref| metric;
bit-exact for the depthwise kernel (same fma chain), 1e-3 for TF32 tensor-core
GEMMs, 1e-5 for the 3xTF32 mode."""
import numpy as np
import pytest

import oracle as orc
import qppocr_b200 as q

pytestmark = pytest.mark.gpu

TOL_TF32 = 1e-3
TOL_3XTF32 = 1e-5


def rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return np.abs(a - b).max() / max(np.abs(b).max(), 1e-6)


def dev(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("n,h,w,c,k,s,act,res", [
    (1, 160, 160, 64, 3, (1, 1), "hswish", False),
    (2, 33, 31, 16, 3, (2, 2), "hswish", True),
    (1, 40, 40, 24, 5, (1, 1), "relu", False),
    (1, 41, 37, 32, 5, (2, 2), None, True),
    (3, 12, 80, 64, 3, (2, 1), "hswish", False),
    (1, 9, 9, 8, 7, (1, 1), "sigmoid", False),
    (1, 1, 1, 4, 3, (1, 1), None, False),
    (1, 10, 10, 6, 3, (1, 1), "swish", True),   # C % 4 != 0 -> generic kernel
    # TMA-tiled kernel (C % 16 == 0): several channel chunks, partial tiles,
    # 16- and 32-channel chunks, both strides, both kernel sizes
    (2, 70, 45, 96, 5, (1, 1), "hswish", True),
    (1, 64, 100, 48, 3, (1, 1), "relu", False),
    (2, 37, 29, 32, 3, (2, 2), "hswish", False),
    (1, 23, 50, 64, 5, (2, 2), None, True),
    (3, 8, 33, 16, 5, (1, 1), "sigmoid", False),
    (1, 3, 2, 32, 3, (1, 1), "hswish", True),
    (1, 30, 30, 64, 5, (1, 1), "hswish", True),    # 5x5, narrow map: 10 x 16 tiles
    (1, 50, 70, 16, 3, (1, 1), "relu", False),     # 16 channels: 32 x 16 tiles
])
def test_dwconv_bit_exact(cuda_ctx, n, h, w, c, k, s, act, res):
    import torch
    rng = np.random.Generator(np.random.PCG64(7))
    x = rng.uniform(-1, 1, (n, h, w, c)).astype(np.float32)
    wt = (rng.standard_normal((c, 1, k, k)) * 0.3).astype(np.float32)
    b = rng.standard_normal(c).astype(np.float32) * 0.1
    p = (k - 1) // 2
    oh = (h + 2 * p - k) // s[0] + 1
    ow = (w + 2 * p - k) // s[1] + 1
    r = rng.uniform(-1, 1, (n, oh, ow, c)).astype(np.float32) if res else None
    tap = np.ascontiguousarray(wt.reshape(c, k * k).T)
    y = q.op_dwconv_nhwc(dev(x), dev(tap), k, k, s, (p, p, p, p), bias=dev(b), act=act,
                         residual=dev(r) if res else None)
    torch.cuda.synchronize()
    got = y.cpu().numpy()
    # reference: NCHW depthwise (conv.rs:45-71) then act then residual
    ref = orc.conv2d(np.transpose(x, (0, 3, 1, 2)), wt, b, s, (p, p, p, p), c)
    if act == "hswish":
        ref = orc.binary("Mul", ref, orc.hardsigmoid(ref, np.float32(1 / 6), 0.5))
    elif act == "relu":
        ref = orc.relu(ref)
    elif act == "sigmoid":
        ref = orc.sigmoid(ref)
    elif act == "swish":
        ref = orc.binary("Mul", ref, orc.sigmoid(ref))
    ref = np.transpose(ref, (0, 2, 3, 1))
    if res:
        ref = orc.binary("Add", ref, r)
    assert got.shape == ref.shape
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32)), rel(got, ref)
    assert q.kernel_error(0) == 0


@pytest.mark.parametrize("m,k,n", [(6400, 16, 32), (6400, 64, 128), (25600, 128, 256),
                                   (6400, 256, 512), (6400, 512, 512), (1000, 120, 360),
                                   (77, 36, 24), (300, 480, 120), (129, 120, 18709),
                                   # 24-wide k-blocks (K % 24 == 0, K % 32 != 0), ragged rows
                                   (3000, 24, 96), (1001, 48, 64), (517, 240, 120), (260, 72, 300)])
@pytest.mark.parametrize("math", ["tf32", "3xtf32"])
def test_gemm_parity(cuda_ctx, m, k, n, math):
    import torch
    from qppocr_b200 import nets
    x, w, b = nets.gemm_case(m, k, n)
    r = np.random.Generator(np.random.PCG64(2)).uniform(-1, 1, (m, n)).astype(np.float32)
    wn = np.ascontiguousarray(w.T)   # [N, K]
    hi, lo = q.op_split_tf32(dev(wn))   # RN tf32 weight preparation (both modes)
    wd = hi
    if math == "tf32":
        lo = None
    y = q.op_gemm(dev(x), wd, bias=dev(b), act="hswish", residual=dev(r), math=math, w_lo=lo)
    torch.cuda.synchronize()
    got = y.cpu().numpy()
    ref = orc.conv1x1_nhwc(x, w, b)
    ref = orc.binary("Add", orc.binary("Mul", ref, orc.hardsigmoid(ref, np.float32(1 / 6), 0.5)), r)
    tol = TOL_TF32 if math == "tf32" else TOL_3XTF32
    e = rel(got, ref)
    assert e < tol, e
    assert q.kernel_error(0) == 0


def test_gemm_rejects_unaligned_k(cuda_ctx):
    import torch
    x = torch.zeros((8, 6), device="cuda")
    w = torch.zeros((4, 6), device="cuda")
    with pytest.raises(q.GraphError):
        q.op_gemm(x, w)


@pytest.mark.parametrize("rows,n", [(10240, 18709), (77, 1000), (300, 37)])
@pytest.mark.parametrize("math", ["tf32", "3xtf32"])
def test_ctc_head_parity(cuda_ctx, rows, n, math):
    """Fused head vs oracle: logits = x W + b -> softmax (activation.rs:321-403)
    -> first strict argmax (rec.rs:34-79).  Indices identical except rows whose
    top-2 probabilities differ by less than the tolerance; values within it."""
    import torch
    rng = np.random.Generator(np.random.PCG64(11))
    k = 120
    x = rng.uniform(-1, 1, (rows, k)).astype(np.float32)
    w = (rng.standard_normal((k, n)) * np.sqrt(1.0 / k)).astype(np.float32)
    b = (rng.standard_normal(n) * 0.02).astype(np.float32)
    hi, lo = q.op_split_tf32(dev(np.ascontiguousarray(w.T)))
    pairs = q.op_ctc_head(dev(x), hi, bias=dev(b), math=math, w_lo=lo if math == "3xtf32" else None)
    torch.cuda.synchronize()
    got = pairs.cpu().numpy()
    probs = orc.softmax_last(orc.binary("Add", orc.sgemm(x, w), b))
    ref = orc.argmax_pairs(probs)
    tol = TOL_TF32 if math == "tf32" else TOL_3XTF32
    gi, ri = got[:, 1].view(np.uint32), ref[:, 1].view(np.uint32)
    top2 = np.sort(probs, axis=1)[:, -2:]
    gap = top2[:, 1] - top2[:, 0]
    assert not ((gi != ri) & (gap >= tol * probs.max())).any()
    assert rel(got[:, 0], ref[:, 0]) < 10 * tol
    assert q.kernel_error(0) == 0


@pytest.mark.parametrize("n", [240, 120])
@pytest.mark.parametrize("math", ["tf32", "3xtf32"])
def test_gemm_column_split_is_bit_identical(cuda_ctx, math, n):
    """A GEMM whose grid would leave SMs idle runs narrower column tiles
    (60 row blocks here: N = 240 as 128-column tiles instead of 256, N = 120
    as 64 instead of 128, against 160 row blocks for the same rows inside a
    larger M).  The tile width changes no output element's arithmetic: the
    shared rows must match bit for bit."""
    import torch
    rng = np.random.Generator(np.random.PCG64(17))
    k, small, large = 120, 128 * 60, 128 * 160
    x = rng.uniform(-1, 1, (large, k)).astype(np.float32)
    w = (rng.standard_normal((n, k)) * np.sqrt(2.0 / k)).astype(np.float32)
    b = (rng.standard_normal(n) * 0.1).astype(np.float32)
    hi, lo = q.op_split_tf32(dev(w))
    lo = lo if math == "3xtf32" else None
    y_large = q.op_gemm(dev(x), hi, bias=dev(b), act="hswish", math=math, w_lo=lo)
    y_small = q.op_gemm(dev(x[:small]), hi, bias=dev(b), act="hswish", math=math, w_lo=lo)
    torch.cuda.synchronize()
    assert np.array_equal(y_small.cpu().numpy(), y_large.cpu().numpy()[:small])
    assert q.kernel_error(0) == 0
