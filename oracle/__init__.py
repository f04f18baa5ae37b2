"""TEST INFRASTRUCTURE ONLY — CPU oracle for the qppocr hot path.

ctypes bindings to liboracle.so (oracle.cpp: a C++ restatement of the
reference's qppocr-kernels scalar semantics) and `run_graph`, a restatement of
the reference's CPU graph executor (crates/qppocr-core/src/executor.rs:213-1839)
for the operator set of the synthetic networks.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference
legs may import this package.  The product (libqppocr_cuda.so and the
qppocr_b200 package) never does.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from typing import Dict, List

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None

F32P = ctypes.POINTER(ctypes.c_float)
I64P = ctypes.POINTER(ctypes.c_int64)
I32P = ctypes.POINTER(ctypes.c_int32)


def build() -> str:
    """Compile liboracle.so in place (make -C oracle)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        _lib = ctypes.CDLL(_LIB_PATH)
    return _lib


def _f(a: np.ndarray):
    assert a.dtype == np.float32 and a.flags["C_CONTIGUOUS"], (a.dtype, a.flags)
    return a.ctypes.data_as(F32P)


def _i64(v):
    a = np.ascontiguousarray(np.asarray(v, np.int64))
    return a, a.ctypes.data_as(I64P)


def _i32(v):
    a = np.ascontiguousarray(np.asarray(v, np.int32))
    return a, a.ctypes.data_as(I32P)


def _c(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def threads() -> int:
    return int(lib().orc_threads())


# ------------------------------------------------------------------ primitives
def xorshift_fill(state: int, n: int):
    """tests/kernels.rs:30-48 RNG; returns (values, new_state)."""
    out = np.empty(n, np.float32)
    st = ctypes.c_uint64(state)
    lib().orc_xorshift_fill(ctypes.byref(st), _f(out), ctypes.c_int64(n))
    return out, st.value


def exp1(x):
    x = _c(x)
    y = np.empty_like(x)
    lib().orc_exp1(_f(x), _f(y), ctypes.c_int64(x.size))
    return y


def erf1(x):
    x = _c(x)
    y = np.empty_like(x)
    lib().orc_erf1(_f(x), _f(y), ctypes.c_int64(x.size))
    return y


def hardsigmoid(x, alpha=0.2, beta=0.5):
    x = _c(x)
    y = np.empty_like(x)
    lib().orc_hardsigmoid(_f(x), _f(y), ctypes.c_int64(x.size), ctypes.c_float(alpha), ctypes.c_float(beta))
    return y


def sigmoid(x):
    x = _c(x)
    y = np.empty_like(x)
    lib().orc_sigmoid(_f(x), _f(y), ctypes.c_int64(x.size))
    return y


def relu(x):
    y = _c(x).copy()
    lib().orc_relu(_f(y), ctypes.c_int64(y.size))
    return y


def sqrt(x):
    y = _c(x).copy()
    lib().orc_sqrt(_f(y), ctypes.c_int64(y.size))
    return y


def clip(x, lo, hi):
    y = _c(x).copy()
    lib().orc_clip(_f(y), ctypes.c_int64(y.size), ctypes.c_float(lo), ctypes.c_float(hi))
    return y


def gelu(x, c1=1.4142135, c2=1.0, c3=0.5):
    y = _c(x).copy()
    lib().orc_gelu(_f(y), ctypes.c_int64(y.size), ctypes.c_float(c1), ctypes.c_float(c2), ctypes.c_float(c3))
    return y


def softmax_last(x):
    y = _c(x).copy()
    inner = y.shape[-1]
    lib().orc_softmax_last_dim(_f(y), ctypes.c_int64(y.size // inner), ctypes.c_int64(inner))
    return y


def _act_c(act_c):
    if act_c is None:
        return None, None
    a = np.asarray(act_c, np.float32)
    return a, a.ctypes.data_as(F32P)


def sgemm(a, b, bias=None, act=0, act_c=None, residual=None):
    """gemm.rs sgemm / sgemm_res: C[M,N] = A[M,K] B[K,N] (+bias per row)."""
    a, b = _c(a), _c(b)
    m, k = a.shape
    n = b.shape[1]
    c = np.empty((m, n), np.float32)
    bias = None if bias is None else _c(bias)
    residual = None if residual is None else _c(residual)
    ac, acp = _act_c(act_c)
    lib().orc_sgemm(_f(a), _f(b), _f(c), ctypes.c_int64(m), ctypes.c_int64(n), ctypes.c_int64(k),
                    _f(bias) if bias is not None else None, ctypes.c_int(act), acp,
                    _f(residual) if residual is not None else None)
    return c


def conv2d(x, w, bias=None, strides=(1, 1), pads=(0, 0, 0, 0), group=1, act=0, act_c=None,
           residual=None):
    """conv.rs conv2d_res (NCHW). pads = (ph, pw, peh, pew)."""
    x, w = _c(x), _c(w)
    n, c, h, wd = x.shape
    m, cg, kh, kw = w.shape
    ph, pw, peh, pew = pads
    oh = (h + ph + peh - kh) // strides[0] + 1
    ow = (wd + pw + pew - kw) // strides[1] + 1
    y = np.empty((n, m, oh, ow), np.float32)
    xs, xsp = _i64(x.shape)
    ws, wsp = _i64(w.shape)
    prm, prmp = _i32([strides[0], strides[1], ph, pw, peh, pew, group])
    bias = None if bias is None else _c(bias)
    residual = None if residual is None else _c(residual)
    ac, acp = _act_c(act_c)
    rc = lib().orc_conv2d(_f(x), xsp, _f(w), wsp, _f(bias) if bias is not None else None, prmp,
                          ctypes.c_int(act), acp, _f(residual) if residual is not None else None, _f(y))
    if rc != 0:
        raise ValueError("orc_conv2d: unsupported configuration")
    return y


def convtranspose2d(x, w):
    x, w = _c(x), _c(w)
    n, c, h, wd = x.shape
    y = np.empty((n, w.shape[1], 2 * h, 2 * wd), np.float32)
    xs, xsp = _i64(x.shape)
    ws, wsp = _i64(w.shape)
    if lib().orc_convtranspose2d(_f(x), xsp, _f(w), wsp, _f(y)) != 0:
        raise ValueError("orc_convtranspose2d: only 2x2 s2")
    return y


def depthwise_nhwc(x, wt, kh, kw, strides=(1, 1), pads=(0, 0, 0, 0), bias=None, act=0, act_c=None,
                   residual=None):
    x, wt = _c(x), _c(wt)
    n, h, wd, c = x.shape
    ph, pw, peh, pew = pads
    oh = (h + ph + peh - kh) // strides[0] + 1
    ow = (wd + pw + pew - kw) // strides[1] + 1
    y = np.empty((n, oh, ow, c), np.float32)
    prm, prmp = _i32([strides[0], strides[1], ph, pw, peh, pew])
    bias = None if bias is None else _c(bias)
    residual = None if residual is None else _c(residual)
    ac, acp = _act_c(act_c)
    lib().orc_depthwise_nhwc(_f(x), ctypes.c_int64(n), ctypes.c_int64(h), ctypes.c_int64(wd), ctypes.c_int64(c),
                             _f(wt), ctypes.c_int64(kh), ctypes.c_int64(kw), prmp,
                             _f(bias) if bias is not None else None, ctypes.c_int(act), acp,
                             _f(residual) if residual is not None else None, _f(y))
    return y


def conv1x1_nhwc(x, wt, bias=None, act=0, act_c=None, residual=None):
    """conv.rs:856-901: Y[R,M] = X[R,K] Wt[K,M] then bias, act, residual."""
    x, wt = _c(x), _c(wt)
    r, k = x.shape
    m = wt.shape[1]
    y = np.empty((r, m), np.float32)
    bias = None if bias is None else _c(bias)
    residual = None if residual is None else _c(residual)
    ac, acp = _act_c(act_c)
    lib().orc_conv1x1_nhwc(_f(x), _f(wt), ctypes.c_int64(r), ctypes.c_int64(k), ctypes.c_int64(m),
                           _f(bias) if bias is not None else None, ctypes.c_int(act), acp,
                           _f(residual) if residual is not None else None, _f(y))
    return y


def batchnorm(x, scale, bias, mean, var, eps=1e-5):
    x = _c(x)
    n, c = x.shape[0], x.shape[1]
    plane = x.size // (n * c)
    y = np.empty_like(x)
    lib().orc_batchnorm(_f(x), ctypes.c_int64(n), ctypes.c_int64(c), ctypes.c_int64(plane),
                        _f(_c(scale)), _f(_c(bias)), _f(_c(mean)), _f(_c(var)), ctypes.c_float(eps), _f(y))
    return y


def reduce_mean(x, outer, mid, inner):
    x = _c(x)
    y = np.empty(outer * inner, np.float32)
    lib().orc_reduce_mean(_f(x), ctypes.c_int64(outer), ctypes.c_int64(mid), ctypes.c_int64(inner), _f(y))
    return y


def global_avg_pool(x):
    x = _c(x)
    n, c = x.shape[:2]
    y = np.empty((n, c, 1, 1), np.float32)
    lib().orc_global_avg_pool(_f(x), ctypes.c_int64(n * c), ctypes.c_int64(x.size // (n * c)), _f(y))
    return y


def pool2d(x, kh, kw, sh, sw, ph, pw, peh, pew, is_max):
    x = _c(x)
    n, c, h, wd = x.shape
    oh = (h + ph + peh - kh) // sh + 1
    ow = (wd + pw + pew - kw) // sw + 1
    y = np.empty((n, c, oh, ow), np.float32)
    L = ctypes.c_int64
    lib().orc_pool2d(_f(x), L(n), L(c), L(h), L(wd), L(kh), L(kw), L(sh), L(sw), L(ph), L(pw), L(peh),
                     L(pew), ctypes.c_int(1 if is_max else 0), _f(y))
    return y


def resize_nearest(x, oh, ow):
    x = _c(x)
    n, c, h, wd = x.shape
    y = np.empty((n, c, oh, ow), np.float32)
    lib().orc_resize_nearest(_f(x), ctypes.c_int64(n * c), ctypes.c_int64(h), ctypes.c_int64(wd),
                             ctypes.c_int64(oh), ctypes.c_int64(ow), _f(y))
    return y


def mul_add_scale(f, g, r):
    f, g, r = _c(f), _c(g), _c(r)
    c = f.shape[1]
    hw = f.size // (f.shape[0] * c)
    y = np.empty_like(f)
    lib().orc_mul_add_scale(_f(f), _f(g), _f(r), _f(y), ctypes.c_int64(f.size // hw), ctypes.c_int64(c),
                            ctypes.c_int64(hw))
    return y


_BINOPS = {"Add": 0, "Sub": 1, "Mul": 2, "Div": 3, "Pow": 4}


def binary(op, a, b):
    a, b = _c(a), _c(b)
    oshape = np.broadcast_shapes(a.shape, b.shape)
    r = max(len(oshape), 1)
    ash = [1] * (r - a.ndim) + list(a.shape)
    bsh = [1] * (r - b.ndim) + list(b.shape)
    if not oshape:
        ash, bsh = [1], [1]
    y = np.empty(oshape if oshape else (), np.float32)
    asv, asp = _i64(ash)
    bsv, bsp = _i64(bsh)
    lib().orc_binary(_f(a), asp, _f(b), bsp, ctypes.c_int(r), ctypes.c_int(_BINOPS[op]),
                     y.ctypes.data_as(F32P))
    return y


def matmul(a, b):
    """shape.rs:568-698 batched matmul with right-aligned batch broadcast."""
    a, b = _c(a), _c(b)
    m, k = a.shape[-2:]
    n = b.shape[-1]
    ba, bb = a.shape[:-2], b.shape[:-2]
    bs = np.broadcast_shapes(ba, bb)
    nb = int(np.prod(bs)) if bs else 1
    abatch = int(np.prod(ba)) if ba else 1
    bbatch = int(np.prod(bb)) if bb else 1
    if not ((abatch in (1, nb)) and (bbatch in (1, nb))):
        a = np.ascontiguousarray(np.broadcast_to(a, tuple(bs) + (m, k)))
        b = np.ascontiguousarray(np.broadcast_to(b, tuple(bs) + (k, n)))
        abatch = bbatch = nb
    y = np.empty(tuple(bs) + (m, n), np.float32)
    large = 1 if m * n * k >= 1 << 17 else 0
    L = ctypes.c_int64
    lib().orc_matmul(_f(a), L(abatch), _f(b), L(bbatch), L(nb), L(m), L(k), L(n), ctypes.c_int(large),
                     y.ctypes.data_as(F32P))
    return y


def argmax_pairs(p):
    """rec.rs ctc_decode argmax (first strict max, ties -> lowest index)."""
    p = _c(p)
    cols = p.shape[-1]
    rows = p.size // cols
    out = np.empty(p.shape[:-1] + (2,), np.float32)
    lib().orc_argmax_pairs(_f(p), ctypes.c_int64(rows), ctypes.c_int64(cols), out.ctypes.data_as(F32P))
    return out


# ------------------------------------------------------ det / rec pre and post
U8P = ctypes.POINTER(ctypes.c_uint8)


def _u8(a):
    return a.ctypes.data_as(U8P)


def resize_bilinear_rgb_u8(src, dh, dw):
    """resize.rs:158-210 on [n, sh, sw, 3] uint8 -> [n, dh, dw, 3] uint8."""
    src = np.ascontiguousarray(src, np.uint8)
    n, sh, sw, _ = src.shape
    out = np.empty((n, dh, dw, 3), np.uint8)
    lib().orc_resize_bilinear_rgb_u8(_u8(src), ctypes.c_int64(n), ctypes.c_int64(sh), ctypes.c_int64(sw),
                                     _u8(out), ctypes.c_int64(dh), ctypes.c_int64(dw))
    return out


def det_normalize(img):
    """engine.rs:963-982 on [n, h, w, 3] uint8 -> [n, 3, h, w] float32."""
    img = np.ascontiguousarray(img, np.uint8)
    n, h, w, _ = img.shape
    out = np.empty((n, 3, h, w), np.float32)
    lib().orc_det_normalize(_u8(img), ctypes.c_int64(n), ctypes.c_int64(h), ctypes.c_int64(w), _f(out))
    return out


def rec_pack_line(crop, rw, img_h, img_w, pad=False):
    """crop.rs:153-185 pack_crop of one h x w x 3 uint8 crop into a zeroed
    [3, img_h, img_w] float32 slot."""
    crop = np.ascontiguousarray(crop, np.uint8)
    h, w, _ = crop.shape
    out = np.empty((3, img_h, img_w), np.float32)
    lib().orc_rec_pack_line(_u8(crop), ctypes.c_int64(h), ctypes.c_int64(w), ctypes.c_int64(rw),
                            ctypes.c_int(1 if pad else 0), ctypes.c_int64(img_h), ctypes.c_int64(img_w), _f(out))
    return out


def dilate2x2(mask):
    """resize.rs:213-245 on [n, h, w] uint8."""
    mask = np.ascontiguousarray(mask, np.uint8)
    n, h, w = mask.shape
    out = np.empty_like(mask)
    lib().orc_dilate2x2(_u8(mask), ctypes.c_int64(n), ctypes.c_int64(h), ctypes.c_int64(w), _u8(out))
    return out


def db_mask(pred, thresh, dilate=True):
    """geometry.rs:286-296: (pred > thresh), then the 2x2 dilation; [n, h, w]."""
    pred = _c(pred)
    n, h, w = pred.shape
    out = np.empty((n, h, w), np.uint8)
    lib().orc_db_mask(_f(pred), ctypes.c_int64(n), ctypes.c_int64(h), ctypes.c_int64(w),
                      ctypes.c_float(thresh), ctypes.c_int(1 if dilate else 0), _u8(out))
    return out


def box_scores(pred, boxes, img=None):
    """geometry.rs:221-269 box_score_fast for each box: pred [n, h, w] f32,
    boxes [k, 4, 2] (x, y) corners in pred coordinates, img [k] image index."""
    pred = _c(pred)
    n, h, w = pred.shape
    boxes = np.ascontiguousarray(boxes, np.float32).reshape(-1, 8)
    k = boxes.shape[0]
    img = np.zeros(k, np.int32) if img is None else np.ascontiguousarray(img, np.int32)
    out = np.empty(k, np.float32)
    lib().orc_box_scores(_f(pred), ctypes.c_int64(h), ctypes.c_int64(w), _f(boxes),
                         img.ctypes.data_as(ctypes.POINTER(ctypes.c_int)), ctypes.c_int64(k), _f(out))
    return out


def crop_size(pts):
    """crop.rs:8-20: (cw, ch, rotated) of crop_text_box for corners pts [4, 2]."""
    pts = np.ascontiguousarray(pts, np.float32).reshape(8)
    cw, ch, rot = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
    lib().orc_crop_size(_f(pts), ctypes.byref(cw), ctypes.byref(ch), ctypes.byref(rot))
    return cw.value, ch.value, bool(rot.value)


def crop_text_box(src, pts):
    """crop.rs:8-127 on one h x w x 3 uint8 image: the perspective crop of the
    quadrilateral pts [4, 2] (ch x cw x 3, or cw x ch x 3 when rotated)."""
    src = np.ascontiguousarray(src, np.uint8)
    h, w, _ = src.shape
    cw, ch, rot = crop_size(pts)
    out = np.empty((cw, ch, 3) if rot else (ch, cw, 3), np.uint8)
    pts = np.ascontiguousarray(pts, np.float32).reshape(8)
    lib().orc_crop_text_box(_u8(src), ctypes.c_int(h), ctypes.c_int(w), _f(pts), _u8(out))
    return out


def cls_pack_line(crop, cls_h, cls_w):
    """crop.rs:193-218 cls_view then pack_crop (resize) into a zeroed
    [3, cls_h, cls_w] float32 slot."""
    crop = np.ascontiguousarray(crop, np.uint8)
    h, w, _ = crop.shape
    out = np.empty((3, cls_h, cls_w), np.float32)
    lib().orc_cls_pack_line(_u8(crop), ctypes.c_int64(h), ctypes.c_int64(w), ctypes.c_int64(cls_h),
                            ctypes.c_int64(cls_w), _f(out))
    return out


def ctc_decode(probs, charset=None):
    """rec.rs:34-79 greedy CTC over one line's [T, C] probabilities: per step
    the first strict maximum; emit when best != 0 and best != previous; conf =
    f64 mean of the emitted steps' values.  Returns (indices, conf); with a
    charset, indices past it are not emitted as text (but count for conf)."""
    probs = np.asarray(probs, np.float32)
    out, conf_sum, conf_n, prev = [], 0.0, 0, -1
    for t in range(probs.shape[0]):
        row = probs[t]
        best, bv = 0, row[0]
        for c in range(1, row.shape[0]):
            if row[c] > bv:
                best, bv = c, row[c]
        if best != 0 and best != prev:
            if charset is None or best < len(charset):
                out.append(best)
            conf_sum += float(bv)
            conf_n += 1
        prev = best
    conf = np.float32(conf_sum / conf_n) if conf_n else np.float32(0.0)
    return out, conf


# ------------------------------------------------------------------ executor
def _resolve_pads(node, h, w, kh, kw, sh, sw):
    ap = node.attrs.get("auto_pad", "NOTSET")
    if ap in ("SAME_UPPER", "SAME_LOWER"):
        res = []
        for size, k, s in ((h, kh, sh), (w, kw, sw)):
            out = (size + s - 1) // s
            tot = max(0, (out - 1) * s + k - size)
            b = tot // 2 if ap == "SAME_UPPER" else tot - tot // 2
            res.append((b, tot - b))
        return res[0][0], res[1][0], res[0][1], res[1][1]
    p = node.attrs.get("pads", [0, 0, 0, 0])
    return int(p[0]), int(p[1]), int(p[2]), int(p[3])


def run_graph(graph, weights: Dict[str, np.ndarray], inputs: Dict[str, np.ndarray]) -> List[np.ndarray]:
    """Execute an optimized graph on the CPU oracle (executor.rs op arms)."""
    vals: Dict[str, np.ndarray] = dict(inputs)

    def get(name):
        if name in vals:
            return vals[name]
        return weights[name]

    for n in graph.nodes:
        vals[n.outputs[0]] = eval_node(n, get)
    return [vals[o] for o in graph.outputs]


def eval_node(n, get) -> np.ndarray:
    """One node of the reference executor; `get(name)` supplies its inputs."""
    op = n.op_type
    a = n.attrs
    if op == "Conv":
        x, w = get(n.inputs[0]), get(n.inputs[1])
        bias = get(n.inputs[2]) if len(n.inputs) > 2 and n.inputs[2] else None
        res = get(n.inputs[3]) if len(n.inputs) > 3 and n.inputs[3] else None
        st = a.get("strides", [1, 1])
        kh, kw = w.shape[2], w.shape[3]
        pads = _resolve_pads(n, x.shape[2], x.shape[3], kh, kw, st[0], st[1])
        act = int(a.get("act", 0))
        act_c = [a.get("act_c1", 1.4142135), a.get("act_c2", 1.0), a.get("act_c3", 0.5)]
        y = conv2d(x, w, bias, st, pads, int(a.get("group", 1)), act, act_c, res)
    elif op == "ConvTranspose":
        y = convtranspose2d(get(n.inputs[0]), get(n.inputs[1]))
    elif op == "BatchNormalization":
        y = batchnorm(get(n.inputs[0]), *(get(n.inputs[k]) for k in range(1, 5)), eps=a.get("epsilon", 1e-5))
    elif op == "Relu":
        y = relu(get(n.inputs[0]))
    elif op == "Sigmoid":
        y = sigmoid(get(n.inputs[0]))
    elif op == "HardSigmoid":
        y = hardsigmoid(get(n.inputs[0]), a.get("alpha", 0.2), a.get("beta", 0.5))
    elif op == "Sqrt":
        y = sqrt(get(n.inputs[0]))
    elif op in _BINOPS:
        y = binary(op, get(n.inputs[0]), get(n.inputs[1]))
    elif op == "MulAddScale":
        f, g, r = (get(i) for i in n.inputs)
        if f.ndim == 4 and g.size == f.shape[1] and r.shape == f.shape and f.size:
            y = mul_add_scale(f, g, r)
        else:
            y = binary("Add", binary("Mul", f, g), r)
    elif op == "Softmax":
        x = get(n.inputs[0])
        axis = int(a.get("axis", -1))
        if axis not in (-1, x.ndim - 1):
            raise NotImplementedError("softmax axis")
        y = softmax_last(x)
    elif op == "GlobalAveragePool":
        y = global_avg_pool(get(n.inputs[0]))
    elif op in ("AveragePool", "MaxPool"):
        x = get(n.inputs[0])
        ks = a["kernel_shape"]
        st = a.get("strides", [1, 1])
        ph, pw, peh, pew = _resolve_pads(n, x.shape[2], x.shape[3], ks[0], ks[1], st[0], st[1])
        y = pool2d(x, ks[0], ks[1], st[0], st[1], ph, pw, peh, pew, op == "MaxPool")
    elif op == "Resize":
        x = get(n.inputs[0])
        if len(n.inputs) >= 4 and n.inputs[3]:
            sz = get(n.inputs[3]).astype(np.int64)
            oh, ow = int(sz[-2]), int(sz[-1])
        else:
            sc = get(n.inputs[2]).astype(np.float32)
            oh = int(np.float32(x.shape[2]) * sc[-2])
            ow = int(np.float32(x.shape[3]) * sc[-1])
        y = resize_nearest(x, oh, ow)
    elif op == "Concat":
        y = np.concatenate([get(i) for i in n.inputs], axis=int(a.get("axis", 0)))
    elif op == "Slice":
        x = get(n.inputs[0])
        starts = get(n.inputs[1]).astype(np.int64)
        ends = get(n.inputs[2]).astype(np.int64)
        axes = get(n.inputs[3]).astype(np.int64) if len(n.inputs) > 3 and n.inputs[3] else range(len(starts))
        sl = [slice(None)] * x.ndim
        for s0, e0, ax in zip(starts, ends, axes):
            sl[int(ax)] = slice(int(s0), int(e0))
        y = np.ascontiguousarray(x[tuple(sl)])
    elif op == "Transpose":
        y = np.ascontiguousarray(np.transpose(get(n.inputs[0]), a.get("perm")))
    elif op == "Reshape":
        x = get(n.inputs[0])
        shp = [int(v) for v in get(n.inputs[1])]
        shp = [x.shape[i] if d == 0 else d for i, d in enumerate(shp)]
        y = x.reshape(shp)
    elif op == "Squeeze":
        x = get(n.inputs[0])
        axes = a.get("axes") or [int(v) for v in get(n.inputs[1])]
        y = np.squeeze(x, axis=tuple(int(v) for v in axes))
    elif op == "Unsqueeze":
        x = get(n.inputs[0])
        axes = a.get("axes") or [int(v) for v in get(n.inputs[1])]
        y = np.expand_dims(x, tuple(int(v) for v in axes))
    elif op == "ReduceMean":
        x = get(n.inputs[0])
        axes = [int(v) % x.ndim for v in a.get("axes", range(x.ndim))]
        lo, hi = min(axes), max(axes)
        outer = int(np.prod(x.shape[:lo]))
        mid = int(np.prod(x.shape[lo:hi + 1]))
        inner = int(np.prod(x.shape[hi + 1:]))
        y = reduce_mean(x, outer, mid, inner)
        shp = [d if i not in axes else 1 for i, d in enumerate(x.shape)]
        if not int(a.get("keepdims", 1)):
            shp = [d for i, d in enumerate(x.shape) if i not in axes]
        y = y.reshape(shp)
    elif op == "MatMul":
        y = matmul(get(n.inputs[0]), get(n.inputs[1]))
    elif op in ("Identity", "Dropout"):
        y = get(n.inputs[0])
    else:
        raise NotImplementedError(f"oracle executor: op {op}")
    return np.ascontiguousarray(y, dtype=np.float32)
