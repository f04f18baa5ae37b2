"""The allocation-free CTC head entry point against the allocating one.

qpc_op_ctc_head_noalloc serves callers that cannot let a library allocate
GPU memory (an engine that owns all device memory in its own pool, or a
serving loop that must not call the CUDA allocator once running).  It must
give the same (value, index) pairs as qpc_op_ctc_head, call after call, even
though every call reuses the same fixed scratch array, and a pipeline wait
that runs out inside it must reach the caller through qpc_kernel_error like
any other kernel fault.  This file is collected last so a failure here cannot
stop the rest of a -x run.
"""
import ctypes

import numpy as np
import pytest

import qppocr_b200 as q

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


def _noalloc(L, xd, rows, k, hi, lo, n, bd, math, out):
    return L.qpc_op_ctc_head_noalloc(xd.data_ptr(), rows, k, hi.data_ptr(), lo.data_ptr(), n, bd.data_ptr(),
                                     q.MATH[math], out.data_ptr(), None)


@pytest.mark.gpu
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
        rc = _noalloc(L, xd, rows, x.shape[1], hi, lo, n, bd, math, got)
        assert rc == q.QPC_OK, L.qpc_last_error()
        torch.cuda.synchronize()
        assert q.kernel_error(0) == 0
        g, r = got.cpu().numpy(), ref.cpu().numpy()
        assert np.array_equal(g[:, 1].view(np.uint32), r[:, 1].view(np.uint32)), f"call {call}: indices"
        err = np.abs(g[:, 0].astype(np.float64) - r[:, 0]).max() / np.abs(r[:, 0]).max()
        assert err < TOL, f"call {call}: values {err:.2e}"


@pytest.mark.gpu
def test_noalloc_timed_out_wait_is_reported_then_cleared():
    """A wait that runs out in the entry point's kernels (made to happen by
    the self-test kernel on the entry point's own fault word, with a 2 ms
    limit) is kept until qpc_kernel_error reads it; the next call still
    matches the allocating entry point."""
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test run without a visible CUDA device")
    L = q.lib()
    assert q.kernel_error(0) == 0
    q.selftest_wait_timeout(0, "noalloc", 2000)
    assert q.kernel_error(0) == 1      # KERR_MBAR_TIMEOUT, kept across the call's return
    assert q.kernel_error(0) == 0      # read clears it
    x, w, b = _case(23, 300, 1000)
    hi, lo = q.op_split_tf32(_dev(w))
    xd, bd = _dev(x), _dev(b)
    ref = q.op_ctc_head(xd, hi, bias=bd, math="tf32", w_lo=lo)
    got = torch.full((300, 2), float("nan"), device="cuda")
    assert _noalloc(L, xd, 300, 120, hi, lo, 1000, bd, "tf32", got) == q.QPC_OK, L.qpc_last_error()
    torch.cuda.synchronize()
    assert q.kernel_error(0) == 0
    assert np.array_equal(got.cpu().numpy()[:, 1].view(np.uint32), ref.cpu().numpy()[:, 1].view(np.uint32))


def test_noalloc_rejects_oversize_before_touching_the_device():
    """The size check runs before any CUDA call, so this needs no GPU: the
    pointers are non-null dummies that nothing dereferences."""
    L = q.lib()
    dummy = ctypes.c_void_p(0x1000)
    rows_too_many = (1 << 21) + 1   # n <= 32: one column tile per row
    rc = L.qpc_op_ctc_head_noalloc(dummy, rows_too_many, 8, dummy, None, 8, None, 0, dummy, None)
    assert rc == q.QPC_ERR_INVALID
    msg = L.qpc_last_error()
    assert b"exceeds" in msg and b"column tiles" in msg
    # 2^21 rows of one column tile is exactly the limit; 2^20 rows of 3 tiles
    # (n = 600: TF32 heads use 256-column tiles) is over
    rc = L.qpc_op_ctc_head_noalloc(dummy, 1 << 20, 8, dummy, None, 600, None, 0, dummy, None)
    assert rc == q.QPC_ERR_INVALID
