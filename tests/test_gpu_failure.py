"""Failure paths made on the host or by a bounded wait, never by a GPU fault
(the reference's failure handling: no silent fallback and bounded device
waits, crates/qppocr-core/src/device.rs:88-94,
crates/qppocr-gpu/src/vulkan/session.rs:306-312).

* A wait that nothing completes runs out after a 2 ms limit, raises the
  timeout flag in the device's fault word and returns; the context stays
  usable and the next session run is correct.
* A forced device allocation failure makes the run that uploads weights and
  builds the plan (or the CTC head's scratch allocation) fail with
  QPC_ERR_OOM and leaves nothing behind.
* Sessions on two devices in one process (when two are visible) each set
  their kernels' shared-memory limits on their own device.
"""
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


def _block():
    g, w = nets.build_block()
    return q.optimize(g, w), w


def test_bounded_wait_runs_out_and_context_survives(cuda_ctx):
    assert q.kernel_error(0) == 0
    q.selftest_wait_timeout(0, "device", 2000)
    assert q.kernel_error(0) == 1   # KERR_MBAR_TIMEOUT
    assert q.kernel_error(0) == 0   # cleared by the read
    g, w = _block()
    x = nets.block_input(0, (1, 64, 32, 32))
    s = cuda_ctx.create_session(g, w, math="3xtf32")
    got = s.run({"x": x})[0]
    assert rel(got, orc.run_graph(g, w, {"x": x})[0]) < 1e-5
    s.close()


def test_forced_allocation_failure_in_first_run(cuda_ctx):
    """Weights go to the device, and the plan's arena is allocated, when a
    shape is first run: a failed allocation there fails that run only, at the
    first allocation or deep inside the upload, and the next run is correct."""
    g, w = _block()
    s = cuda_ctx.create_session(g, w, math="3xtf32")
    x = nets.block_input(0, (1, 64, 32, 32))
    for nth in (1, 3):
        q.inject_alloc_failure(nth)
        with pytest.raises(q.OutOfMemoryError, match="injected"):
            s.run({"x": x})
    q.inject_alloc_failure(0)
    assert rel(s.run({"x": x})[0], orc.run_graph(g, w, {"x": x})[0]) < 1e-5
    s.close()


def test_forced_allocation_failure_in_ctc_head():
    import torch
    rng = np.random.Generator(np.random.PCG64(5))
    x = torch.from_numpy(rng.uniform(-1, 1, (64, 120)).astype(np.float32)).cuda()
    w = torch.from_numpy(rng.standard_normal((500, 120)).astype(np.float32)).cuda()
    hi, _ = q.op_split_tf32(w)
    q.inject_alloc_failure(1)
    with pytest.raises(q.OutOfMemoryError):
        q.op_ctc_head(x, hi)
    q.inject_alloc_failure(0)
    q.op_ctc_head(x, hi)
    torch.cuda.synchronize()


def test_sessions_on_two_devices_in_one_process():
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("one GPU visible: the per-device shared-memory opt-in is exercised on one device only")
    g, w = nets.build_det()
    g = q.optimize(g, w)
    x = nets.det_input(1, 128, 128)
    outs = []
    for d in (0, 1):
        s = q.CudaContext.open(d).create_session(g, w, role="det", math="3xtf32")
        outs.append(s.run({"x": x})[0])
        s.close()
    assert np.array_equal(outs[0], outs[1])
