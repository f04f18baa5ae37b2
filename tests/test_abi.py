"""C-ABI surface checks that need no GPU: the library loads, exports every
function include/qppocr_cuda.h declares, and fails loudly (no CPU fallback)
when no device is present."""
import ctypes
import os
import re

import pytest

import qppocr_b200 as q

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    names = set()
    for fn in os.listdir(os.path.join(ROOT, "include")):
        if fn.endswith(".h"):
            src = open(os.path.join(ROOT, "include", fn)).read()
            src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
            names |= set(re.findall(r"\b(qpc_\w+)\s*\(", src))
    return sorted(names)


def test_library_exports_every_declared_symbol():
    lib = q.lib()
    decl = declared_symbols()
    assert len(decl) >= 20
    missing = [n for n in decl if not hasattr(lib, n)]
    assert not missing, missing
    assert set(q.EXPORTED) <= set(decl)


def test_invalid_arguments_are_rejected():
    lib = q.lib()
    assert lib.qpc_device_count(None) == q.QPC_ERR_INVALID
    t = ctypes.c_void_p()
    assert lib.qpc_run_async(None, None, 0, ctypes.byref(t)) == q.QPC_ERR_INVALID
    assert lib.qpc_complete(None, 0) == q.QPC_ERR_INVALID
    assert lib.qpc_session_caps(None, None) == q.QPC_ERR_INVALID


def test_no_device_means_error_not_fallback():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is visible")
    assert q.device_count() == 0
    with pytest.raises(q.DeviceError):
        q.CudaContext.open(0)
    from qppocr_b200 import nets
    g, w = nets.build_block()
    g = q.optimize(g, w)
    ctx = q.CudaContext(0, "none", 0, (10, 0))
    with pytest.raises(q.DeviceError):
        ctx.create_session(g, w)
