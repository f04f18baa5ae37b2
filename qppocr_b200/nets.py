"""Synthetic random-init PP-OCR networks for the benchmark configurations.

The reference's real models (PP-OCR ONNX files) and its image corpus are not
published with it, so every configuration the benchmark names is a
random-init network of the stated architecture, built here as a graph in the
reference's own operator vocabulary (what its ONNX loader produces: Conv with
BN, HardSigmoid+Mul hardswish, Sigmoid+Mul swish, Resize, Concat,
ConvTranspose, decomposed LayerNorm, MatMul, Reshape/Transpose/Slice/Squeeze,
Softmax).  `build_*` return (Graph, initializers) BEFORE the loader passes;
`qppocr_b200.graph.optimize` applies them.

Initialisation (all seeded numpy PCG64):
  conv / linear weights  N(0, sqrt(2 / fan_in))
  BN gamma U[0.5, 1.5], beta and mean N(0, 0.1), var U[0.5, 1.5]
  LayerNorm gamma 1 + N(0, 0.1), beta N(0, 0.1)

Architecture choices where the configuration text is open:
  det  backbone: the PP-LCNet x1.0 13-block table (strides 2 at blocks
       2, 4, 6, 12; SE on the last 2), which is what "strides 2 at blocks
       2,4,6,12 ... SE on the last 2" describes; DBFPN neck (1x1 -> 96,
       nearest-upsample adds, 3x3 -> 24 per level, concat at 1/4); DB head.
  rec  conv stages stated below (downsample 48x320 -> 1x40, 480 ch); neck
       1x1 -> 120 + swish; 2 pre-LN transformer blocks (8 heads x 15);
       final LayerNorm; linear head 120 -> 18709 + Softmax.
  cls  PP-LCNet x0.25 (make_divisible(ch * 0.25, 8)), SE on the last 2
       blocks, GAP -> 1x1 conv 128 -> 1280 + hardswish -> linear -> 2.
"""
from __future__ import annotations

from typing import Dict, List, Optional, Tuple

import numpy as np

from .graph import Graph, Node

F32 = np.float32
HS_ALPHA = float(F32(1.0 / 6.0))
REC_CLASSES = 18709

# ImageNet normalisation used by the det / cls / rec host pre-processing
# (engine.rs:963-982 normalises on the host before the graph).
IMAGENET_MEAN = np.array([0.485, 0.456, 0.406], F32)
IMAGENET_STD = np.array([0.229, 0.224, 0.225], F32)


class Builder:
    def __init__(self, seed: int, prefix: str):
        self.rng = np.random.Generator(np.random.PCG64(seed))
        self.nodes: List[Node] = []
        self.w: Dict[str, np.ndarray] = {}
        self.k = 0
        self.prefix = prefix

    def uid(self, p: str) -> str:
        self.k += 1
        return f"{self.prefix}.{p}{self.k}"

    def const(self, arr, p="c") -> str:
        n = self.uid(p)
        self.w[n] = np.asarray(arr)
        return n

    def i64(self, vals, p="shape") -> str:
        return self.const(np.asarray(vals, np.int64), p)

    def node(self, op: str, inputs: List[str], attrs: Optional[dict] = None) -> str:
        out = self.uid(op.lower() + "_o")
        self.nodes.append(Node(op, self.uid(op), list(inputs), [out], dict(attrs or {})))
        return out

    # ---- layers
    def normal(self, shape, std):
        return (self.rng.standard_normal(shape) * std).astype(F32)

    def conv(self, x, cin, cout, k, stride=1, group=1, bias=False, bn=True, act=None, pad=None):
        kh, kw = (k, k) if isinstance(k, int) else k
        sh, sw = (stride, stride) if isinstance(stride, int) else stride
        fan_in = (cin // group) * kh * kw
        w = self.const(self.normal((cout, cin // group, kh, kw), np.sqrt(2.0 / fan_in)), "w")
        ph, pw = ((kh - 1) // 2, (kw - 1) // 2) if pad is None else pad
        ins = [x, w]
        if bias:
            ins.append(self.const(self.normal((cout,), 0.1), "b"))
        y = self.node("Conv", ins, {"kernel_shape": [kh, kw], "strides": [sh, sw],
                                    "pads": [ph, pw, ph, pw], "group": group,
                                    "dilations": [1, 1]})
        if bn:
            y = self.bn(y, cout)
        return self.act(y, act)

    def bn(self, x, c):
        g = self.const(self.rng.uniform(0.5, 1.5, c).astype(F32), "bn_g")
        b = self.const(self.normal((c,), 0.1), "bn_b")
        m = self.const(self.normal((c,), 0.1), "bn_m")
        v = self.const(self.rng.uniform(0.5, 1.5, c).astype(F32), "bn_v")
        return self.node("BatchNormalization", [x, g, b, m, v], {"epsilon": 1e-5})

    def act(self, x, act):
        if act is None:
            return x
        if act == "hswish":
            h = self.node("HardSigmoid", [x], {"alpha": HS_ALPHA, "beta": 0.5})
            return self.node("Mul", [x, h])
        if act == "swish":
            s = self.node("Sigmoid", [x])
            return self.node("Mul", [x, s])
        if act == "relu":
            return self.node("Relu", [x])
        raise ValueError(act)

    def se(self, x, c):
        p = self.node("GlobalAveragePool", [x])
        h = self.conv(p, c, c // 4, 1, bias=True, bn=False, act="relu")
        g = self.conv(h, c // 4, c, 1, bias=True, bn=False, act=None)
        g = self.node("HardSigmoid", [g], {"alpha": HS_ALPHA, "beta": 0.5})
        return self.node("Mul", [x, g])

    def dwsep(self, x, k, cin, cout, stride, se=False):
        y = self.conv(x, cin, cin, k, stride=stride, group=cin, act="hswish")
        if se:
            y = self.se(y, cin)
        return self.conv(y, cin, cout, 1, act="hswish")

    def resize2(self, x, scale):
        roi = ""
        sc = self.const(np.array([1, 1, scale, scale], F32), "scales")
        return self.node("Resize", [x, roi, sc], {"mode": "nearest",
                                                 "coordinate_transformation_mode": "asymmetric",
                                                 "nearest_mode": "floor"})

    def linear(self, x, k, n, bias=True, std=None):
        w = self.const(self.normal((k, n), np.sqrt(2.0 / k) if std is None else std), "lw")
        y = self.node("MatMul", [x, w])
        if bias:
            y = self.node("Add", [y, self.const(self.normal((n,), 0.02), "lb")])
        return y

    def layernorm(self, x, c, eps=1e-6):
        m = self.node("ReduceMean", [x], {"axes": [-1], "keepdims": 1})
        d = self.node("Sub", [x, m])
        p = self.node("Pow", [d, self.const(np.array(2.0, F32), "two")])
        v = self.node("ReduceMean", [p], {"axes": [-1], "keepdims": 1})
        ve = self.node("Add", [v, self.const(np.array(eps, F32), "eps")])
        s = self.node("Sqrt", [ve])
        nrm = self.node("Div", [d, s])
        g = self.const((1.0 + self.normal((c,), 0.1)).astype(F32), "ln_g")
        b = self.const(self.normal((c,), 0.1), "ln_b")
        y = self.node("Mul", [nrm, g])
        return self.node("Add", [y, b])

    def graph(self, inputs, outputs, input_dims) -> Tuple[Graph, Dict[str, np.ndarray]]:
        return Graph(self.nodes, inputs, outputs, input_dims), self.w


# ------------------------------------------------------------------ config 1
def build_block(seed: int = 0, c_in: int = 64, c_out: int = 128):
    """Config 1: dw 3x3 s1 p1 + BN + hardswish, then pw 1x1 c_in -> c_out + bias + hardswish."""
    b = Builder(seed, "blk")
    x = "x"
    y = b.conv(x, c_in, c_in, 3, group=c_in, act="hswish")
    y = b.conv(y, c_in, c_out, 1, bias=True, bn=False, act="hswish")
    return b.graph(["x"], [y], [[1, c_in, 0, 0]])


def block_input(seed: int = 0, shape=(1, 64, 160, 160)) -> np.ndarray:
    rng = np.random.Generator(np.random.PCG64(seed))
    return rng.uniform(-1.0, 1.0, shape).astype(F32)


# ------------------------------------------------------------------ config 2
GEMM_SWEEP_M = (6400, 25600, 102400, 409600)
GEMM_SWEEP_KN = ((16, 32), (64, 128), (128, 256), (256, 512), (512, 512))


def gemm_case(m: int, k: int, n: int, seed: int = 1):
    """Config 2: X [M,K] U[-1,1], W [K,N] N(0, sqrt(2/K)), bias, hardswish."""
    rng = np.random.Generator(np.random.PCG64(seed))
    x = rng.uniform(-1.0, 1.0, (m, k)).astype(F32)
    w = (rng.standard_normal((k, n)) * np.sqrt(2.0 / k)).astype(F32)
    bias = (rng.standard_normal(n) * 0.1).astype(F32)
    return x, w, bias


def build_gemm(k: int, n: int, seed: int = 1):
    """Config 2 as a graph: MatMul -> Add(bias) -> HardSigmoid -> Mul."""
    _, w, bias = gemm_case(1, k, n, seed)
    b = Builder(seed, "gemm")
    wn = b.const(w, "w")
    y = b.node("MatMul", ["x", wn])
    y = b.node("Add", [y, b.const(bias, "b")])
    y = b.act(y, "hswish")
    return b.graph(["x"], [y], [[0, k]])


# ------------------------------------------------------------------ config 3
# PP-LCNet x1.0 block table: (kernel, in, out, stride, se)
LCNET_BLOCKS = {
    "blocks2": [(3, 16, 32, 1, False)],
    "blocks3": [(3, 32, 64, 2, False), (3, 64, 64, 1, False)],
    "blocks4": [(3, 64, 128, 2, False), (3, 128, 128, 1, False)],
    "blocks5": [(3, 128, 256, 2, False)] + [(5, 256, 256, 1, False)] * 5,
    "blocks6": [(5, 256, 512, 2, True), (5, 512, 512, 1, True)],
}


def build_det(seed: int = 3, fpn_ch: int = 96, scale: float = 1.0):
    """Config 3: DB text detector (PP-LCNet backbone, DBFPN, DB head)."""

    def ch(c):
        return max(8, int(c * scale + 4) // 8 * 8) if scale != 1.0 else c

    b = Builder(seed, "det")
    x = b.conv("x", 3, ch(16), 3, stride=2, act="hswish")
    feats = []
    for stage in ("blocks2", "blocks3", "blocks4", "blocks5", "blocks6"):
        for (k, cin, cout, s, se) in LCNET_BLOCKS[stage]:
            x = b.dwsep(x, k, ch(cin), ch(cout), s, se)
        if stage != "blocks2":
            feats.append((x, ch(LCNET_BLOCKS[stage][-1][2])))
    (c2, n2), (c3, n3), (c4, n4), (c5, n5) = feats
    # DBFPN: lateral 1x1 convs (no bias), top-down nearest-upsample adds
    in5 = b.conv(c5, n5, fpn_ch, 1, bn=False)
    up5 = b.resize2(in5, 2.0)
    in4 = b.conv(c4, n4, fpn_ch, 1, bn=False)
    out4 = b.node("Add", [in4, up5])
    up4 = b.resize2(out4, 2.0)
    in3 = b.conv(c3, n3, fpn_ch, 1, bn=False)
    out3 = b.node("Add", [in3, up4])
    up3 = b.resize2(out3, 2.0)
    in2 = b.conv(c2, n2, fpn_ch, 1, bn=False)
    out2 = b.node("Add", [in2, up3])
    q = fpn_ch // 4
    p5 = b.conv(in5, fpn_ch, q, 3, bn=False)
    p4 = b.conv(out4, fpn_ch, q, 3, bn=False)
    p3 = b.conv(out3, fpn_ch, q, 3, bn=False)
    p2 = b.conv(out2, fpn_ch, q, 3, bn=False)
    p5 = b.resize2(p5, 8.0)
    p4 = b.resize2(p4, 4.0)
    p3 = b.resize2(p3, 2.0)
    fuse = b.node("Concat", [p5, p4, p3, p2], {"axis": 1})
    # DB head (binarize branch)
    h = b.conv(fuse, fpn_ch, q, 3, bn=True, act="relu")
    wt1 = b.const(b.normal((q, q, 2, 2), np.sqrt(2.0 / (q * 4))), "ct_w")
    h = b.node("ConvTranspose", [h, wt1], {"kernel_shape": [2, 2], "strides": [2, 2]})
    h = b.bn(h, q)
    h = b.node("Relu", [h])
    wt2 = b.const(b.normal((q, 1, 2, 2), np.sqrt(2.0 / (q * 4))), "ct_w")
    h = b.node("ConvTranspose", [h, wt2], {"kernel_shape": [2, 2], "strides": [2, 2]})
    y = b.node("Sigmoid", [h])
    return b.graph(["x"], [y], [[0, 3, 0, 0]])


def det_input(batch: int, h: int = 960, w: int = 960, seed: int = 3) -> np.ndarray:
    """ImageNet-normalised U[0,1] pixels, NCHW float32."""
    rng = np.random.Generator(np.random.PCG64(seed + 1000))
    px = rng.uniform(0.0, 1.0, (batch, 3, h, w)).astype(F32)
    return ((px - IMAGENET_MEAN[None, :, None, None]) / IMAGENET_STD[None, :, None, None]).astype(F32)


# ------------------------------------------------------------------ config 4
# (kernel, in, out, (stride_h, stride_w))
REC_BLOCKS = [
    (3, 16, 32, (1, 1)),
    (3, 32, 64, (2, 2)),
    (3, 64, 64, (1, 1)),
    (3, 64, 128, (2, 1)),
    (3, 128, 128, (1, 1)),
    (3, 128, 256, (2, 2)),
    (5, 256, 256, (1, 1)),
    (5, 256, 480, (1, 1)),
]


def build_rec(seed: int = 4, dim: int = 120, heads: int = 8, depth: int = 2,
              classes: int = REC_CLASSES, mlp_ratio: int = 2):
    """Config 4: SVTR-style CTC recogniser."""
    b = Builder(seed, "rec")
    x = b.conv("x", 3, 16, 3, stride=2, act="hswish")               # 24 x 160
    for (k, cin, cout, s) in REC_BLOCKS:
        y = b.conv(x, cin, cin, k, stride=s, group=cin, act="hswish")
        x = b.conv(y, cin, cout, 1, act="hswish")                     # -> 3 x 40
    x = b.node("AveragePool", [x], {"kernel_shape": [3, 1], "strides": [3, 1],
                                    "pads": [0, 0, 0, 0]})            # 1 x 40
    x = b.conv(x, 480, dim, 1, act="swish")                           # [B,120,1,T]
    x = b.node("Reshape", [x, b.i64([0, 0, -1])])                     # [B,120,T]
    x = b.node("Transpose", [x], {"perm": [0, 2, 1]})                 # [B,T,120]
    hd = dim // heads
    scale = np.array(hd ** -0.5, F32)
    for _ in range(depth):
        h = b.layernorm(x, dim)
        qkv = b.linear(h, dim, 3 * dim)
        qkv = b.node("Reshape", [qkv, b.i64([0, 0, 3, heads, hd])])   # [B,T,3,H,hd]
        qkv = b.node("Transpose", [qkv], {"perm": [2, 0, 3, 1, 4]})  # [3,B,H,T,hd]
        parts = []
        for j in range(3):
            s = b.node("Slice", [qkv, b.i64([j], "st"), b.i64([j + 1], "en"), b.i64([0], "ax")])
            parts.append(b.node("Squeeze", [s, b.i64([0], "ax")]))
        q, k, v = parts
        q = b.node("Mul", [q, b.const(scale, "scale")])
        kt = b.node("Transpose", [k], {"perm": [0, 1, 3, 2]})
        att = b.node("MatMul", [q, kt])                               # [B,H,T,T]
        att = b.node("Softmax", [att], {"axis": -1})
        o = b.node("MatMul", [att, v])                                # [B,H,T,hd]
        o = b.node("Transpose", [o], {"perm": [0, 2, 1, 3]})          # [B,T,H,hd]
        o = b.node("Reshape", [o, b.i64([0, 0, dim])])
        o = b.linear(o, dim, dim)
        x = b.node("Add", [x, o])
        h = b.layernorm(x, dim)
        f = b.linear(h, dim, dim * mlp_ratio)
        f = b.act(f, "swish")
        f = b.linear(f, dim * mlp_ratio, dim)
        x = b.node("Add", [x, f])
    x = b.layernorm(x, dim)
    logits = b.linear(x, dim, classes, std=np.sqrt(1.0 / dim))
    y = b.node("Softmax", [logits], {"axis": -1})
    return b.graph(["x"], [y], [[0, 3, 48, 0]])


def rec_input(batch: int, h: int = 48, w: int = 320, seed: int = 4) -> np.ndarray:
    """Normalised U[0,1] pixels ((p - 0.5) / 0.5, the rec pre-processing)."""
    rng = np.random.Generator(np.random.PCG64(seed + 1000))
    px = rng.uniform(0.0, 1.0, (batch, 3, h, w)).astype(F32)
    return ((px - F32(0.5)) / F32(0.5)).astype(F32)


# ------------------------------------------------------------------ config 5 (cls)
LCNET_X025 = {
    "blocks2": [(3, 8, 8, 1, False)],
    "blocks3": [(3, 8, 16, 2, False), (3, 16, 16, 1, False)],
    "blocks4": [(3, 16, 32, 2, False), (3, 32, 32, 1, False)],
    "blocks5": [(3, 32, 64, 2, False)] + [(5, 64, 64, 1, False)] * 5,
    "blocks6": [(5, 64, 128, 2, True), (5, 128, 128, 1, True)],
}


def build_cls(seed: int = 5, classes: int = 2):
    """Config 5 classifier: PP-LCNet x0.25 on 3x80x160 crops, 2 classes."""
    b = Builder(seed, "cls")
    x = b.conv("x", 3, 8, 3, stride=2, act="hswish")
    for stage in ("blocks2", "blocks3", "blocks4", "blocks5", "blocks6"):
        for (k, cin, cout, s, se) in LCNET_X025[stage]:
            x = b.dwsep(x, k, cin, cout, s, se)
    x = b.node("GlobalAveragePool", [x])                               # [B,128,1,1]
    x = b.conv(x, 128, 1280, 1, bias=True, bn=False, act="hswish")
    x = b.node("Reshape", [x, b.i64([0, -1])])                         # [B,1280]
    x = b.linear(x, 1280, classes, std=np.sqrt(1.0 / 1280))
    y = b.node("Softmax", [x], {"axis": -1})
    return b.graph(["x"], [y], [[0, 3, 80, 160]])


def cls_input(batch: int, seed: int = 5) -> np.ndarray:
    rng = np.random.Generator(np.random.PCG64(seed + 1000))
    px = rng.uniform(0.0, 1.0, (batch, 3, 80, 160)).astype(F32)
    return ((px - F32(0.5)) / F32(0.5)).astype(F32)
