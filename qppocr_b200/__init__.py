"""qppocr_b200 — B200-native (sm_100a) device backend for qppocr.

Python mirror of the reference's device seam over the C ABI of
libqppocr_cuda.so (include/qppocr_cuda.h):

  CudaContext.open(index)        crates/qppocr-gpu/src/cuda.rs:121-200 (CudaContext::open)
  CudaContext.create_session()   crates/qppocr-core/src/device.rs:88-101 (DeviceContext::create_session)
  CudaSession.run(inputs)        device.rs:130 (DeviceSession::run)
  CudaSession.run_deferred()     device.rs:164-176 (-> DeferredRun)
  DeferredRun.complete()         device.rs:105-108
  caps: prefers_host_parallelism / bucket_grain / batch_grain / rec_chunk /
        rec_argmax_pairs         device.rs:134-163

Errors mirror Error::Graph / Error::Device (crates/qppocr-core/src/error.rs):
GraphError for unsupported ops or shapes, DeviceError for CUDA failures.  There
is no CPU fallback: if the CUDA library cannot be loaded, every entry point
raises.
"""
from __future__ import annotations

import ctypes
import os
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np

from .graph import Graph, Node, optimize  # noqa: F401

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libqppocr_cuda.so")

QPC_OK, QPC_ERR_INVALID, QPC_ERR_GRAPH, QPC_ERR_DEVICE, QPC_ERR_TIMEOUT, QPC_ERR_OOM = range(6)
QPC_U8 = 4  # qpc_dtype of u8 outputs (the det mask)
ROLE = {"other": 0, "det": 1, "rec": 2, "cls": 3}
MATH = {"tf32": 0, "3xtf32": 1}
ACT = {None: 0, "none": 0, "relu": 1, "hswish": 2, "sigmoid": 3, "gelu": 4, "hsigmoid": 5, "swish": 6}


class QppocrError(RuntimeError):
    pass


class GraphError(QppocrError):
    """Error::Graph — unsupported op / shape, missing tensor."""


class DeviceError(QppocrError):
    """Error::Device — no device, CUDA failure, kernel fault or timeout."""


class TimeoutError_(DeviceError):
    pass


class OutOfMemoryError(DeviceError):
    """A device or pinned-host allocation failed (QPC_ERR_OOM)."""


# ------------------------------------------------------------------ C structs
class QpcAttr(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char_p), ("kind", ctypes.c_int), ("f", ctypes.c_float),
                ("i", ctypes.c_int64), ("s", ctypes.c_char_p),
                ("floats", ctypes.POINTER(ctypes.c_float)), ("ints", ctypes.POINTER(ctypes.c_int64)),
                ("n", ctypes.c_int)]


class QpcNode(ctypes.Structure):
    _fields_ = [("op_type", ctypes.c_char_p), ("name", ctypes.c_char_p),
                ("inputs", ctypes.POINTER(ctypes.c_char_p)), ("n_inputs", ctypes.c_int),
                ("outputs", ctypes.POINTER(ctypes.c_char_p)), ("n_outputs", ctypes.c_int),
                ("attrs", ctypes.POINTER(QpcAttr)), ("n_attrs", ctypes.c_int)]


class QpcGraph(ctypes.Structure):
    _fields_ = [("nodes", ctypes.POINTER(QpcNode)), ("n_nodes", ctypes.c_int),
                ("inputs", ctypes.POINTER(ctypes.c_char_p)), ("n_inputs", ctypes.c_int),
                ("outputs", ctypes.POINTER(ctypes.c_char_p)), ("n_outputs", ctypes.c_int)]


class QpcTensor(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char_p), ("shape", ctypes.POINTER(ctypes.c_int64)),
                ("rank", ctypes.c_int), ("dtype", ctypes.c_int), ("data", ctypes.c_void_p)]


class QpcOptions(ctypes.Structure):
    _fields_ = [("math", ctypes.c_int), ("argmax_exit", ctypes.c_int),
                ("plan_budget_bytes", ctypes.c_int64), ("use_cuda_graph", ctypes.c_int),
                ("det_mask_exit", ctypes.c_int), ("mask_thresh", ctypes.c_float), ("mask_dilate", ctypes.c_int)]


class QpcCaps(ctypes.Structure):
    _fields_ = [("prefers_host_parallelism", ctypes.c_int), ("bucket_grain", ctypes.c_int),
                ("batch_grain", ctypes.c_int), ("rec_chunk", ctypes.c_int),
                ("argmax_pairs", ctypes.c_int)]


# Every symbol include/qppocr_cuda.h declares (checked by the CPU test suite).
EXPORTED = (
    "qpc_last_error", "qpc_device_count", "qpc_device_info", "qpc_session_create",
    "qpc_session_caps", "qpc_run_async", "qpc_complete", "qpc_ticket_output_count",
    "qpc_ticket_output", "qpc_ticket_output_copy", "qpc_ticket_output_info", "qpc_ticket_release", "qpc_run", "qpc_ticket_device_ms",
    "qpc_host_alloc", "qpc_host_free",
    "qpc_session_destroy", "qpc_session_profile", "qpc_session_profile_step",
    "qpc_session_replay", "qpc_session_node_count", "qpc_session_node", "qpc_op_dwconv_nhwc", "qpc_op_gemm", "qpc_op_ctc_head", "qpc_op_ctc_head_noalloc",
    "qpc_op_split_tf32", "qpc_op_resize_bilinear_rgb_u8", "qpc_op_det_preprocess", "qpc_op_db_mask",
    "qpc_op_rec_pack",
    "qpc_kernel_error", "qpc_selftest_wait_timeout", "qpc_inject_alloc_failure",
    "qpc_op_box_score", "qpc_crop_size", "qpc_op_crop_text_boxes", "qpc_op_line_pack",
)

_lib = None


def lib():
    """Load libqppocr_cuda.so (raises DeviceError if it is missing)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise DeviceError(f"{LIB_PATH} not built (run __graft_entry__.build())")
    L = ctypes.CDLL(LIB_PATH)
    L.qpc_last_error.restype = ctypes.c_char_p
    P = ctypes.c_void_p
    L.qpc_session_create.argtypes = [ctypes.c_int, ctypes.POINTER(QpcGraph), ctypes.POINTER(QpcTensor),
                                     ctypes.c_int, ctypes.c_int, ctypes.POINTER(QpcOptions),
                                     ctypes.POINTER(P)]
    L.qpc_session_caps.argtypes = [P, ctypes.POINTER(QpcCaps)]
    L.qpc_run_async.argtypes = [P, ctypes.POINTER(QpcTensor), ctypes.c_int, ctypes.POINTER(P)]
    L.qpc_run.argtypes = [P, ctypes.POINTER(QpcTensor), ctypes.c_int, ctypes.POINTER(P)]
    L.qpc_complete.argtypes = [P, ctypes.c_int]
    L.qpc_ticket_output_count.argtypes = [P, ctypes.POINTER(ctypes.c_int)]
    L.qpc_ticket_output.argtypes = [P, ctypes.c_int, ctypes.POINTER(ctypes.POINTER(ctypes.c_float)),
                                    ctypes.POINTER(ctypes.POINTER(ctypes.c_int64)),
                                    ctypes.POINTER(ctypes.c_int)]
    L.qpc_ticket_output_copy.argtypes = [P, ctypes.c_int, ctypes.c_void_p, ctypes.c_int64]
    L.qpc_ticket_output_info.argtypes = [P, ctypes.c_int, ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_int),
                                         ctypes.POINTER(ctypes.c_void_p)]
    L.qpc_host_alloc.argtypes = [ctypes.c_int64, ctypes.POINTER(P)]
    L.qpc_host_free.argtypes = [P]
    L.qpc_ticket_release.argtypes = [P]
    L.qpc_ticket_device_ms.argtypes = [P, ctypes.POINTER(ctypes.c_float)]
    L.qpc_session_destroy.argtypes = [P]
    L.qpc_session_profile.argtypes = [P, ctypes.POINTER(QpcTensor), ctypes.c_int, ctypes.c_int,
                                      ctypes.POINTER(ctypes.c_int)]
    L.qpc_session_profile_step.argtypes = [P, ctypes.c_int, ctypes.POINTER(ctypes.c_char_p),
                                           ctypes.POINTER(ctypes.c_char_p),
                                           ctypes.POINTER(ctypes.c_double),
                                           ctypes.POINTER(ctypes.c_double),
                                           ctypes.POINTER(ctypes.c_float)]
    L.qpc_session_replay.argtypes = [P, ctypes.POINTER(QpcTensor), ctypes.c_int, ctypes.c_int,
                                     ctypes.POINTER(ctypes.c_float)]
    L.qpc_session_node_count.argtypes = [P, ctypes.POINTER(ctypes.c_int)]
    L.qpc_session_node.argtypes = [P, ctypes.c_int, ctypes.POINTER(ctypes.c_char_p),
                                   ctypes.POINTER(ctypes.c_char_p), ctypes.POINTER(ctypes.c_char_p)]
    L.qpc_op_dwconv_nhwc.argtypes = [P, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, P,
                                     ctypes.c_int, ctypes.c_int, P, P, P, ctypes.c_int, P, P, P, P]
    L.qpc_op_gemm.argtypes = [P, ctypes.c_int64, ctypes.c_int, P, P, ctypes.c_int, P, ctypes.c_int, P,
                              P, P, ctypes.c_int, P]
    L.qpc_op_split_tf32.argtypes = [P, ctypes.c_int64, P, P, P]
    I = ctypes.c_int
    L.qpc_op_resize_bilinear_rgb_u8.argtypes = [P, I, I, I, P, I, I, P]
    L.qpc_op_det_preprocess.argtypes = [P, I, I, I, P, I, I, P]
    L.qpc_op_db_mask.argtypes = [P, P, P, I, I, I, ctypes.c_float, I, P]
    L.qpc_op_rec_pack.argtypes = [P, P, P, P, P, P, I, I, I, P, P]
    L.qpc_op_ctc_head.argtypes = [P, ctypes.c_int64, ctypes.c_int, P, P, ctypes.c_int, P, ctypes.c_int,
                                  P, P]
    L.qpc_op_ctc_head_noalloc.argtypes = [P, ctypes.c_int64, ctypes.c_int, P, P, ctypes.c_int, P,
                                          ctypes.c_int, P, P]
    L.qpc_kernel_error.argtypes = [ctypes.c_int, ctypes.POINTER(ctypes.c_uint)]
    L.qpc_selftest_wait_timeout.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int]
    L.qpc_inject_alloc_failure.argtypes = [ctypes.c_int]
    L.qpc_op_box_score.argtypes = [P, I, I, P, P, I, P, P]
    L.qpc_crop_size.argtypes = [P, I, P, P, P]
    L.qpc_op_crop_text_boxes.argtypes = [P, I, I, I, P, P, P, P, P, I, I, P, P]
    L.qpc_op_line_pack.argtypes = [P, P, P, P, P, P, P, P, P, I, I, I, P, P]
    _lib = L
    return L


def _check(rc: int):
    if rc == QPC_OK:
        return
    msg = lib().qpc_last_error().decode(errors="replace")
    if rc == QPC_ERR_GRAPH:
        raise GraphError(msg)
    if rc == QPC_ERR_TIMEOUT:
        raise TimeoutError_(msg)
    if rc == QPC_ERR_OOM:
        raise OutOfMemoryError(msg)
    if rc == QPC_ERR_DEVICE:
        raise DeviceError(msg)
    raise QppocrError(f"status {rc}: {msg}")


def device_count() -> int:
    n = ctypes.c_int(0)
    _check(lib().qpc_device_count(ctypes.byref(n)))
    return n.value


# ------------------------------------------------------------------ marshalling
class _Keep:
    """Holds ctypes buffers alive for the duration of a call."""

    def __init__(self):
        self.objs = []

    def add(self, o):
        self.objs.append(o)
        return o


def _cstrs(keep: _Keep, names: Sequence[str]):
    arr = (ctypes.c_char_p * max(len(names), 1))(*[n.encode() for n in names])
    return keep.add(arr)


def _attr(keep: _Keep, name: str, v) -> QpcAttr:
    a = QpcAttr()
    a.name = keep.add(name.encode())
    if isinstance(v, bool) or isinstance(v, (int, np.integer)):
        a.kind, a.i = 2, int(v)
    elif isinstance(v, (float, np.floating)):
        a.kind, a.f = 1, float(v)
    elif isinstance(v, str):
        a.kind, a.s = 3, keep.add(v.encode())
    elif isinstance(v, (list, tuple, np.ndarray)):
        vals = list(v)
        if all(isinstance(x, (int, np.integer)) for x in vals):
            arr = keep.add((ctypes.c_int64 * max(len(vals), 1))(*[int(x) for x in vals]))
            a.kind, a.ints, a.n = 5, arr, len(vals)
        else:
            arr = keep.add((ctypes.c_float * max(len(vals), 1))(*[float(x) for x in vals]))
            a.kind, a.floats, a.n = 4, arr, len(vals)
    else:
        raise TypeError(f"attribute {name}: {type(v)}")
    return a


def _tensor(keep: _Keep, name: str, arr) -> QpcTensor:
    if hasattr(arr, "is_cuda") and arr.is_cuda:
        # tensor already on the device: f32 (QPC_F32_DEVICE) or a u8 n x h x w x
        # 3 image batch (QPC_U8_IMAGE_DEVICE), copied on the GPU
        import torch
        assert arr.dtype in (torch.float32, torch.uint8) and arr.is_contiguous(), "contiguous device tensor expected"
        keep.add(arr)
        shp = keep.add((ctypes.c_int64 * max(arr.dim(), 1))(*arr.shape))
        t = QpcTensor()
        t.name = keep.add(name.encode())
        t.shape = shp
        t.rank = arr.dim()
        t.dtype = 3 if arr.dtype == torch.float32 else 5
        t.data = arr.data_ptr()
        return t
    if arr.dtype == np.int64 or arr.dtype == np.int32:
        arr = keep.add(np.ascontiguousarray(arr, np.int64))
        dt = 1
    elif arr.dtype == np.uint8:
        # n x h x w x 3 images for an [n, 3, h, w] f32 input, normalised on
        # the device (engine.rs:963-982); run inputs only
        arr = keep.add(np.ascontiguousarray(arr))
        dt = 2
    else:
        arr = keep.add(np.ascontiguousarray(arr, np.float32))
        dt = 0
    shp = keep.add((ctypes.c_int64 * max(arr.ndim, 1))(*arr.shape))
    t = QpcTensor()
    t.name = keep.add(name.encode())
    t.shape = shp
    t.rank = arr.ndim
    t.dtype = dt
    t.data = arr.ctypes.data
    return t


def _tensors(keep: _Keep, items: Dict[str, np.ndarray]):
    arr = (QpcTensor * max(len(items), 1))()
    for k, (n, a) in enumerate(items.items()):
        arr[k] = _tensor(keep, n, a)
    return keep.add(arr), len(items)


def _graph(keep: _Keep, g: Graph) -> QpcGraph:
    nodes = (QpcNode * max(len(g.nodes), 1))()
    for k, n in enumerate(g.nodes):
        qn = QpcNode()
        qn.op_type = keep.add(n.op_type.encode())
        qn.name = keep.add(n.name.encode())
        qn.inputs = _cstrs(keep, n.inputs)
        qn.n_inputs = len(n.inputs)
        qn.outputs = _cstrs(keep, n.outputs)
        qn.n_outputs = len(n.outputs)
        attrs = (QpcAttr * max(len(n.attrs), 1))()
        for j, (an, av) in enumerate(n.attrs.items()):
            attrs[j] = _attr(keep, an, av)
        qn.attrs = keep.add(attrs)
        qn.n_attrs = len(n.attrs)
        nodes[k] = qn
    qg = QpcGraph()
    qg.nodes = keep.add(nodes)
    qg.n_nodes = len(g.nodes)
    qg.inputs = _cstrs(keep, g.inputs)
    qg.n_inputs = len(g.inputs)
    qg.outputs = _cstrs(keep, g.outputs)
    qg.n_outputs = len(g.outputs)
    return qg


# ------------------------------------------------------------------ pinned host memory
class _PinnedBlock:
    """Owner of one qpc_host_alloc block (freed with the last array on it)."""

    def __init__(self, nbytes: int):
        p = ctypes.c_void_p()
        _check(lib().qpc_host_alloc(nbytes, ctypes.byref(p)))
        self.ptr = p.value

    def __del__(self):
        try:
            if self.ptr:
                lib().qpc_host_free(ctypes.c_void_p(self.ptr))
                self.ptr = None
        except Exception:
            pass


def host_empty(shape, dtype=np.float32) -> np.ndarray:
    """An uninitialised array in pinned host memory.  Passed as a run input,
    it is copied to the device by DMA straight from this memory (no staging
    copy); keep it unchanged until the run completes."""
    dt = np.dtype(dtype)
    shape = tuple(int(d) for d in shape)
    nbytes = int(np.prod(shape, dtype=np.int64)) * dt.itemsize
    blk = _PinnedBlock(max(nbytes, 1))
    buf = (ctypes.c_char * max(nbytes, 1)).from_address(blk.ptr)
    buf._owner = blk  # the ctypes buffer keeps the block alive, the array keeps the buffer
    return np.frombuffer(buf, dtype=dt, count=int(np.prod(shape, dtype=np.int64))).reshape(shape)


def _pinned_view(data, shape, cnt: int, owner, dtype=np.float32) -> np.ndarray:
    """Read-only array over a run's pinned output buffer; holds `owner` (the
    DeferredRun, whose ticket keeps the buffer) alive."""
    dt = np.dtype(dtype)
    buf = (ctypes.c_char * max(cnt * dt.itemsize, 1)).from_address(ctypes.addressof(data.contents))
    buf._owner = owner
    a = np.frombuffer(buf, dtype=dt, count=cnt).reshape(shape)
    a.flags.writeable = False
    return a


class DeviceOutput:
    """An output a run keeps in device memory (the det mask exit's
    probability map): shape, dtype and device address, valid while the
    DeferredRun that produced it is alive.  `torch()` is a zero-copy view."""

    def __init__(self, ptr: int, shape, dtype, owner, device: int):
        self.ptr = ptr
        self.shape = tuple(shape)
        self.dtype = np.dtype(dtype)
        self.device = device
        self._owner = owner

    @property
    def __cuda_array_interface__(self):
        return {"shape": self.shape, "typestr": self.dtype.str, "data": (self.ptr, False), "version": 3,
                "strides": None}

    def torch(self):
        import torch
        return torch.as_tensor(self, device=f"cuda:{self.device}")


# ------------------------------------------------------------------ device seam
class DeferredRun:
    """A submitted run (DeferredRun, device.rs:105-108)."""

    def __init__(self, session: "CudaSession", ticket: ctypes.c_void_p, keep=None):
        self._s = session
        self._t = ticket
        self._keep = keep  # device inputs are read by the run's own copy: hold them until it completes

    def complete(self, timeout_ms: int = -1, copy: bool = True) -> List[np.ndarray]:
        """Wait for the run and return its outputs.  copy=True: fresh arrays
        (the ticket is released).  copy=False: read-only views of the run's
        pinned output buffers, no host copy; the ticket (and its plan
        instance) stays held until every view has been dropped."""
        L = lib()
        _check(L.qpc_complete(self._t, timeout_ms))
        n = ctypes.c_int(0)
        _check(L.qpc_ticket_output_count(self._t, ctypes.byref(n)))
        outs = []
        for k in range(n.value):
            data = ctypes.POINTER(ctypes.c_float)()
            shp = ctypes.POINTER(ctypes.c_int64)()
            rank = ctypes.c_int(0)
            _check(L.qpc_ticket_output(self._t, k, ctypes.byref(data), ctypes.byref(shp), ctypes.byref(rank)))
            shape = tuple(shp[i] for i in range(rank.value))
            cnt = int(np.prod(shape)) if shape else 1
            dt, dev_only, dptr = ctypes.c_int(0), ctypes.c_int(0), ctypes.c_void_p()
            _check(L.qpc_ticket_output_info(self._t, k, ctypes.byref(dt), ctypes.byref(dev_only), ctypes.byref(dptr)))
            np_dt = np.uint8 if dt.value == QPC_U8 else np.float32
            if dev_only.value:
                out = DeviceOutput(dptr.value, shape, np.float32, self, self._s.device)
                self._device_outputs = True
            elif copy:
                out = np.empty(shape, np_dt)
                _check(L.qpc_ticket_output_copy(self._t, k, out.ctypes.data, cnt))
            else:
                out = _pinned_view(data, shape, cnt, self, np_dt)
            outs.append(out)
        ms = ctypes.c_float(0)
        _check(L.qpc_ticket_device_ms(self._t, ctypes.byref(ms)))
        self.device_ms = ms.value
        if copy and not getattr(self, "_device_outputs", False):
            self.release()  # (a run with device outputs is released when dropped)
        return outs

    def release(self):
        if self._t:
            lib().qpc_ticket_release(self._t)
            self._t = None
        self._keep = None

    def __del__(self):
        try:
            self.release()
        except Exception:
            pass


class CudaSession:
    """One model on one device (DeviceSession, device.rs:125-176)."""

    def __init__(self, handle: ctypes.c_void_p, input_names: List[str]):
        self._h = handle
        self.input_names = input_names
        self.device = 0

    def _inputs(self, keep, inputs):
        if isinstance(inputs, dict):
            items = inputs
        else:
            items = {n: a for n, a in inputs}
        return _tensors(keep, items)

    def run(self, inputs) -> List[np.ndarray]:
        return self.run_deferred(inputs).complete()

    def run_deferred(self, inputs) -> DeferredRun:
        keep = _Keep()
        arr, n = self._inputs(keep, inputs)
        t = ctypes.c_void_p()
        _check(lib().qpc_run_async(self._h, arr, n, ctypes.byref(t)))
        return DeferredRun(self, t, keep)

    def caps(self) -> Dict[str, int]:
        c = QpcCaps()
        _check(lib().qpc_session_caps(self._h, ctypes.byref(c)))
        return {k: getattr(c, k) for k, _ in QpcCaps._fields_}

    def prefers_host_parallelism(self) -> bool:
        return bool(self.caps()["prefers_host_parallelism"])

    def bucket_grain(self) -> int:
        return self.caps()["bucket_grain"]

    def batch_grain(self) -> int:
        return self.caps()["batch_grain"]

    def rec_chunk(self) -> int:
        return self.caps()["rec_chunk"]

    def rec_argmax_pairs(self) -> bool:
        return bool(self.caps()["argmax_pairs"])

    def profile(self, inputs, iters: int = 3):
        """Per-step device times: list of (kernel, node, bytes, flops, ms)."""
        keep = _Keep()
        arr, n = self._inputs(keep, inputs)
        ns = ctypes.c_int(0)
        _check(lib().qpc_session_profile(self._h, arr, n, iters, ctypes.byref(ns)))
        out = []
        for k in range(ns.value):
            kern, node = ctypes.c_char_p(), ctypes.c_char_p()
            by, fl = ctypes.c_double(), ctypes.c_double()
            ms = ctypes.c_float()
            _check(lib().qpc_session_profile_step(self._h, k, ctypes.byref(kern), ctypes.byref(node),
                                                  ctypes.byref(by), ctypes.byref(fl), ctypes.byref(ms)))
            out.append((kern.value.decode(), node.value.decode(), by.value, fl.value, ms.value))
        return out

    def fused_nodes(self):
        """(op, name, output) of every node after load-time fusion."""
        n = ctypes.c_int(0)
        _check(lib().qpc_session_node_count(self._h, ctypes.byref(n)))
        out = []
        for k in range(n.value):
            op, nm, o = ctypes.c_char_p(), ctypes.c_char_p(), ctypes.c_char_p()
            _check(lib().qpc_session_node(self._h, k, ctypes.byref(op), ctypes.byref(nm), ctypes.byref(o)))
            out.append((op.value.decode(), nm.value.decode(), o.value.decode()))
        return out

    def replay(self, inputs, iters: int) -> float:
        """Device ms per replay of the captured graph, inputs staged once."""
        keep = _Keep()
        arr, n = self._inputs(keep, inputs)
        ms = ctypes.c_float(0)
        _check(lib().qpc_session_replay(self._h, arr, n, iters, ctypes.byref(ms)))
        return ms.value

    def close(self):
        if self._h:
            lib().qpc_session_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class CudaContext:
    """One CUDA device (CudaContext, crates/qppocr-gpu/src/cuda.rs:112-230)."""

    def __init__(self, index: int, name: str, driver: int, cc: Tuple[int, int]):
        self.index = index
        self.name = name
        self.driver = driver
        self.cc = cc

    @classmethod
    def open(cls, index: Optional[int] = None) -> "CudaContext":
        idx = 0 if index is None else int(index)
        name = ctypes.create_string_buffer(256)
        drv, ma, mi = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
        _check(lib().qpc_device_info(idx, name, 256, ctypes.byref(drv), ctypes.byref(ma), ctypes.byref(mi)))
        return cls(idx, name.value.decode(), drv.value, (ma.value, mi.value))

    def info(self) -> Dict[str, str]:
        v = self.driver
        return {"kind": "cuda", "name": self.name, "api": f"cuda {v // 1000}.{v % 1000 // 10}"}

    def create_session(self, graph: Graph, initializers: Dict[str, np.ndarray], role: str = "other",
                       math: str = "tf32", argmax_exit: Optional[bool] = None,
                       use_cuda_graph: bool = True, plan_budget_bytes: int = 0, det_mask_exit: bool = False,
                       mask_thresh: float = 0.3, mask_dilate: bool = True) -> CudaSession:
        keep = _Keep()
        qg = _graph(keep, graph)
        wt, nw = _tensors(keep, initializers)
        opts = QpcOptions()
        opts.math = MATH[math]
        opts.argmax_exit = -1 if argmax_exit is None else int(bool(argmax_exit))
        opts.plan_budget_bytes = plan_budget_bytes
        opts.use_cuda_graph = 1 if use_cuda_graph else 0
        opts.det_mask_exit = 1 if det_mask_exit else 0
        opts.mask_thresh = mask_thresh
        opts.mask_dilate = 1 if mask_dilate else 0
        h = ctypes.c_void_p()
        _check(lib().qpc_session_create(self.index, ctypes.byref(qg), wt, nw, ROLE[role], ctypes.byref(opts),
                                        ctypes.byref(h)))
        sess = CudaSession(h, list(graph.inputs))
        sess.device = self.index  # the GPU the session's buffers and streams live on
        return sess


# ------------------------------------------------------------------ operator entry points
def _dptr(t) -> int:
    """Device pointer of a torch CUDA tensor (None -> 0)."""
    if t is None:
        return None
    assert t.is_cuda and t.is_contiguous(), "device tensor expected"
    return t.data_ptr()


def op_dwconv_nhwc(x, w_tap_major, kh, kw, strides, pads, bias=None, act=None, act_p=None,
                   residual=None, out=None, stream=None):
    """Depthwise conv on torch CUDA tensors (NHWC)."""
    import torch
    n, h, w, c = x.shape
    oh = (h + pads[0] + pads[2] - kh) // strides[0] + 1
    ow = (w + pads[1] + pads[3] - kw) // strides[1] + 1
    y = out if out is not None else torch.empty((n, oh, ow, c), dtype=torch.float32, device=x.device)
    st = (ctypes.c_int * 2)(*strides)
    pd = (ctypes.c_int * 4)(*pads)
    ap = (ctypes.c_float * 5)(*act_p) if act_p is not None else None
    _check(lib().qpc_op_dwconv_nhwc(_dptr(x), n, h, w, c, _dptr(w_tap_major), kh, kw,
                                    ctypes.cast(st, ctypes.c_void_p), ctypes.cast(pd, ctypes.c_void_p),
                                    _dptr(bias), ACT[act],
                                    ctypes.cast(ap, ctypes.c_void_p) if ap is not None else None,
                                    _dptr(residual), _dptr(y), stream))
    return y


def op_gemm(x, w, n=None, bias=None, act=None, act_p=None, residual=None, math="tf32", w_lo=None,
            out=None, stream=None):
    """y[M,N] = act(x[M,K] w[N,K]^T + bias) + residual on torch CUDA tensors."""
    import torch
    m, k = x.shape
    nn = w.shape[0]
    y = out if out is not None else torch.empty((m, nn), dtype=torch.float32, device=x.device)
    ap = (ctypes.c_float * 5)(*act_p) if act_p is not None else None
    _check(lib().qpc_op_gemm(_dptr(x), m, k, _dptr(w), _dptr(w_lo), nn, _dptr(bias), ACT[act],
                             ctypes.cast(ap, ctypes.c_void_p) if ap is not None else None,
                             _dptr(residual), _dptr(y), MATH[math], stream))
    return y


def op_ctc_head(x, w, bias=None, math="tf32", w_lo=None, out=None, stream=None):
    """(value, index-bits) pairs [rows, 2] of softmax(x w^T + bias) per row."""
    import torch
    rows, k = x.shape
    n = w.shape[0]
    y = out if out is not None else torch.empty((rows, 2), dtype=torch.float32, device=x.device)
    _check(lib().qpc_op_ctc_head(_dptr(x), rows, k, _dptr(w), _dptr(w_lo), n, _dptr(bias), MATH[math],
                                 _dptr(y), stream))
    return y


def op_split_tf32(v, stream=None):
    import torch
    hi = torch.empty_like(v)
    lo = torch.empty_like(v)
    _check(lib().qpc_op_split_tf32(_dptr(v), v.numel(), _dptr(hi), _dptr(lo), stream))
    return hi, lo


def op_resize_bilinear_rgb_u8(src, dh: int, dw: int, stream=None):
    """[n, sh, sw, 3] uint8 device tensor -> [n, dh, dw, 3] (resize.rs:158-210)."""
    import torch
    n, sh, sw, _ = src.shape
    dst = torch.empty((n, dh, dw, 3), dtype=torch.uint8, device=src.device)
    _check(lib().qpc_op_resize_bilinear_rgb_u8(_dptr(src), n, sh, sw, _dptr(dst), dh, dw, stream))
    return dst


def op_det_preprocess(src, dh: int, dw: int, stream=None):
    """[n, sh, sw, 3] uint8 device images -> det input [n, 3, dh, dw] f32
    (engine.rs:930-982)."""
    import torch
    n, sh, sw, _ = src.shape
    dst = torch.empty((n, 3, dh, dw), dtype=torch.float32, device=src.device)
    _check(lib().qpc_op_det_preprocess(_dptr(src), n, sh, sw, _dptr(dst), dh, dw, stream))
    return dst


def op_db_mask(pred=None, thresh: float = 0.3, dilate: bool = True, mask_in=None, stream=None):
    """DB mask (geometry.rs:286-296): [n, h, w] probabilities (or an existing
    uint8 mask to dilate) -> [n, h, w] uint8."""
    import torch
    src = pred if pred is not None else mask_in
    n, h, w = src.shape
    out = torch.empty((n, h, w), dtype=torch.uint8, device=src.device)
    _check(lib().qpc_op_db_mask(_dptr(pred) if pred is not None else None,
                                _dptr(mask_in) if mask_in is not None else None, _dptr(out), n, h, w,
                                ctypes.c_float(thresh), 1 if dilate else 0, stream))
    return out


def op_rec_pack(crops, off, h, w, rw, pad, img_h: int, img_w: int, stream=None):
    """Device rec line pack (crop.rs:153-185): crops = concatenated uint8 HWC
    crops, off (int64) / h / w / rw / pad (int32) per line, all device tensors
    -> [n, 3, img_h, img_w] f32."""
    import torch
    n = int(h.numel())
    out = torch.empty((n, 3, img_h, img_w), dtype=torch.float32, device=crops.device)
    # on the tensors' own GPU and its current torch stream, whatever the caller's current device
    with torch.cuda.device(crops.device):
        st = stream if stream is not None else torch.cuda.current_stream(crops.device).cuda_stream
        _check(lib().qpc_op_rec_pack(_dptr(crops), _dptr(off), _dptr(h), _dptr(w), _dptr(rw), _dptr(pad), n, img_h,
                                     img_w, _dptr(out), st))
    return out


def kernel_error(device: int = 0) -> int:
    f = ctypes.c_uint(0)
    _check(lib().qpc_kernel_error(device, ctypes.byref(f)))
    return f.value


def selftest_wait_timeout(device: int = 0, path: str = "device", limit_us: int = 2000) -> None:
    """Run the bounded-wait self-test kernel: a wait on an mbarrier nothing
    arrives on runs out after limit_us and reports into the device's fault
    word (path "device") or the allocation-free CTC head's (path "noalloc");
    read the flag with kernel_error(device)."""
    _check(lib().qpc_selftest_wait_timeout(device, {"device": 0, "noalloc": 1}[path], limit_us))


def inject_alloc_failure(nth: int = 1) -> None:
    """Make the nth device allocation of the library from now on fail as if
    the device were out of memory (0 cancels)."""
    _check(lib().qpc_inject_alloc_failure(nth))


def _stream_of(t, stream):
    import torch
    return stream if stream is not None else torch.cuda.current_stream(t.device).cuda_stream


def op_box_score(pred, boxes, img, stream=None):
    """box_score_fast (geometry.rs:221-269) on the device: pred [n, h, w] f32,
    boxes [k, 4, 2] f32 corners, img [k] int32 image index (device tensors)
    -> scores [k] f32."""
    import torch
    n, h, w = pred.shape
    k = int(img.numel())
    out = torch.empty(k, dtype=torch.float32, device=pred.device)
    with torch.cuda.device(pred.device):
        _check(lib().qpc_op_box_score(_dptr(pred), h, w, _dptr(boxes.contiguous()), _dptr(img), k, _dptr(out),
                                      _stream_of(pred, stream)))
    return out


def crop_size(pts):
    """Host helper: (cw, ch, rotated) int32 arrays of crop_text_box's output
    for boxes pts [k, 4, 2] (crop.rs:9-15)."""
    pts = np.ascontiguousarray(pts, np.float32).reshape(-1, 8)
    k = pts.shape[0]
    cw, ch, rot = (np.empty(k, np.int32) for _ in range(3))
    _check(lib().qpc_crop_size(pts.ctypes.data, k, cw.ctypes.data, ch.ctypes.data, rot.ctypes.data))
    return cw, ch, rot


def op_crop_text_boxes(images, pts, img, stream=None):
    """crop_text_box (crop.rs:8-127) for every box on the device.  images:
    [n, h, w, 3] uint8 device tensor; pts [k, 4, 2] f32 and img [k] int32 host
    arrays.  Returns (crops: one uint8 device buffer, off int64 [k], cw, ch,
    rotated int32 [k]); crop k is (cw x ch x 3 if rotated else ch x cw x 3)
    bytes at off[k]."""
    import torch
    n, h, w, _ = images.shape
    pts = np.ascontiguousarray(pts, np.float32).reshape(-1, 8)
    k = pts.shape[0]
    cw, ch, rot = crop_size(pts)
    sizes = cw.astype(np.int64) * ch * 3
    off = np.zeros(k, np.int64)
    if k:
        off[1:] = np.cumsum(sizes)[:-1]
    total = int(sizes.sum()) if k else 0
    dev = images.device
    out = torch.empty(max(total, 16), dtype=torch.uint8, device=dev)
    if k:
        tp = torch.from_numpy(pts).to(dev)
        ti = torch.from_numpy(np.ascontiguousarray(img, np.int32)).to(dev)
        tcw, tch = torch.from_numpy(cw).to(dev), torch.from_numpy(ch).to(dev)
        toff = torch.from_numpy(off).to(dev)
        with torch.cuda.device(dev):
            _check(lib().qpc_op_crop_text_boxes(_dptr(images), n, h, w, _dptr(tp), _dptr(ti), _dptr(tcw), _dptr(tch),
                                                _dptr(toff), k, int((cw.astype(np.int64) * ch).max()), _dptr(out),
                                                _stream_of(images, stream)))
    return out, off, cw, ch, rot


def op_line_pack(crops, off, stride, x0, h, w, rw, pad, img_h, img_w, flip=None, stream=None):
    """Line pack (crop.rs:153-185, cls_view windows crop.rs:193-218) on the
    device.  crops: uint8 device buffer; the per-line arrays are host numpy
    arrays (copied to the device here).  Returns [n, 3, img_h, img_w] f32."""
    import torch
    n = len(h)
    dev = crops.device
    out = torch.empty((n, 3, img_h, img_w), dtype=torch.float32, device=dev)
    if n == 0:
        return out
    i32 = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.int32)).to(dev)
    toff = torch.from_numpy(np.ascontiguousarray(off, np.int64)).to(dev)
    arrs = [i32(a) for a in (stride, x0, h, w, rw, pad)]
    tflip = i32(flip) if flip is not None else None
    with torch.cuda.device(dev):
        _check(lib().qpc_op_line_pack(_dptr(crops), _dptr(toff), *[_dptr(a) for a in arrs],
                                      _dptr(tflip) if tflip is not None else None, n, img_h, img_w, _dptr(out),
                                      _stream_of(crops, stream)))
    return out
