"""The allocation-free CTC head entry point against the allocating one.

qpc_op_ctc_head_noalloc serves callers that cannot let a library allocate
GPU memory (an engine that owns all device memory in its own pool, or a
serving loop that must not call the CUDA allocator once running).  It must
give the same (value, index) pairs as qpc_op_ctc_head, call after call, even
though every call reuses the same fixed scratch array.  This file is collected
last so a failure here cannot stop the rest of a -x run.
"""
import ctypes

import numpy as np
import pytest

import qppocr_b200 as q

pytestmark = pytest.mark.gpu

TOL = 1e-5  # same kernels on both paths; the suite's fp32-mode tolerance


def _dev(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _case(seed, rows, n, k=120):
    rng = np.random.Generator(np.random.PCG64(seed))
    x = rng.uniform(-1, 1, (rows, k)).astype(np.float32)
    w = (rng.standard_normal((n, k)) * np.sqrt(1.0 / k)).astype(np.float32)
    b = (rng.standard_normal(n) * 0.02).astype(np.float32)
    return x, w, b


def test_noalloc_matches_allocating_entry_point_twice():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test run without a visible CUDA device")
    L = q.lib()
    for call, (seed, rows, n, math) in enumerate([(21, 4096, 18709, "3xtf32"), (22, 777, 5003, "tf32")]):
        x, w, b = _case(seed, rows, n)
        hi, lo = q.op_split_tf32(_dev(w))
        xd, bd = _dev(x), _dev(b)
        ref = q.op_ctc_head(xd, hi, bias=bd, math=math, w_lo=lo)
        got = torch.full((rows, 2), float("nan"), device="cuda")
        rc = L.qpc_op_ctc_head_noalloc(xd.data_ptr(), rows, x.shape[1], hi.data_ptr(), lo.data_ptr(), n,
                                       bd.data_ptr(), q.MATH[math], got.data_ptr(), None)
        assert rc == q.QPC_OK, L.qpc_last_error()
        torch.cuda.synchronize()
        g, r = got.cpu().numpy(), ref.cpu().numpy()
        assert np.array_equal(g[:, 1].view(np.uint32), r[:, 1].view(np.uint32)), f"call {call}: indices"
        err = np.abs(g[:, 0].astype(np.float64) - r[:, 0]).max() / np.abs(r[:, 0]).max()
        assert err < TOL, f"call {call}: values {err:.2e}"


def test_noalloc_rejects_oversize():
    import torch
    L = q.lib()
    x = torch.zeros((8, 8), device="cuda")
    rows_too_many = (1 << 21) // 1 + 1   # with n <= 128 one column tile per row
    rc = L.qpc_op_ctc_head_noalloc(x.data_ptr(), rows_too_many, 8, x.data_ptr(), None, 8, None, 0,
                                   x.data_ptr(), None)
    assert rc == q.QPC_ERR_INVALID
    assert b"exceeds" in L.qpc_last_error()
