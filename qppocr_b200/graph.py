"""In-memory model graph and the reference's load-time graph passes.

`Graph` / `Node` mirror the reference's ONNX model structs
(crates/qppocr-core/src/onnx/model.rs:13-127): nodes in topological order,
attributes keyed by name, graph inputs / outputs by name, and the weights held
separately (the loader moves `Graph.initializers` out before
`DeviceContext::create_session`, crates/qppocr-core/src/executor.rs:160-199).

`optimize()` applies the reference loader's structural passes in its order
(crates/qppocr-core/src/onnx/parse.rs:731-747) to a graph built from scratch,
so the CUDA session and the CPU oracle both receive exactly the graph the
reference would hand its device backends:

* fold_conv_batchnorm  optimize.rs:512-653
* fuse_conv_activation optimize.rs:337-427 (Relu only; the synthetic nets
  carry no GELU subgraphs, so fuse_gelu / FusedGelu never appear)
* fuse_conv_residual   optimize.rs:662-770
* fuse_mul_add         optimize.rs:437-497

All arithmetic is float32 with one rounding per operation, as in Rust.
"""
from __future__ import annotations

import copy
from dataclasses import dataclass, field
from typing import Dict, List, Optional

import numpy as np


@dataclass
class Node:
    op_type: str
    name: str
    inputs: List[str]
    outputs: List[str]
    attrs: Dict[str, object] = field(default_factory=dict)

    def attr(self, key, default=None):
        return self.attrs.get(key, default)


@dataclass
class Graph:
    nodes: List[Node]
    inputs: List[str]
    outputs: List[str]
    input_dims: List[List[int]] = field(default_factory=list)

    def is_graph_output(self, name: str) -> bool:
        return name in self.outputs


def _consumer_counts(g: Graph) -> Dict[str, int]:
    c: Dict[str, int] = {}
    for n in g.nodes:
        for i in n.inputs:
            if i:
                c[i] = c.get(i, 0) + 1
    return c


def _first_consumer(g: Graph) -> Dict[str, int]:
    c: Dict[str, int] = {}
    for k, n in enumerate(g.nodes):
        for i in n.inputs:
            if i and i not in c:
                c[i] = k
    return c


def fold_conv_batchnorm(g: Graph, w: Dict[str, np.ndarray]) -> int:
    """Conv -> BatchNormalization folding (optimize.rs:512-653).

    a = scale / sqrt(var + eps); W' = W * a per output channel;
    b' = (b - mean) * a + beta, or (-mean) * a + beta without a conv bias.
    """
    consumers = _consumer_counts(g)
    first = _first_consumer(g)
    fold = []
    for i, cn in enumerate(g.nodes):
        if cn.op_type != "Conv" or len(cn.inputs) < 2 or len(cn.outputs) != 1:
            continue
        out = cn.outputs[0]
        if g.is_graph_output(out) or consumers.get(out, 0) != 1:
            continue
        bu = first.get(out)
        if bu is None:
            continue
        bn = g.nodes[bu]
        if bn.op_type != "BatchNormalization" or len(bn.inputs) != 5 or bn.inputs[0] != out:
            continue
        wt = w.get(cn.inputs[1])
        if wt is None or wt.dtype != np.float32:
            continue
        m = wt.shape[0]
        if not all(bn.inputs[k] in w and w[bn.inputs[k]].size == m for k in range(1, 5)):
            continue
        fold.append((i, bu, m))
    drop = set()
    f32 = np.float32
    for ci, bi, m in fold:
        bn = g.nodes[bi]
        eps = f32(bn.attr("epsilon", 1e-5))
        scale, beta, mean, var = (w[bn.inputs[k]].astype(f32) for k in range(1, 5))
        a = (scale / np.sqrt(var + eps)).astype(f32)
        wn = g.nodes[ci].inputs[1]
        wt = w[wn]
        w[wn] = (wt.reshape(m, -1) * a[:, None]).astype(f32).reshape(wt.shape)
        cn = g.nodes[ci]
        if len(cn.inputs) >= 3 and cn.inputs[2]:
            b = w[cn.inputs[2]].astype(f32)
            nb = ((b - mean) * a + beta).astype(f32)
            w[cn.inputs[2]] = nb
        else:
            nb = ((-mean) * a + beta).astype(f32)
            name = bn.outputs[0] + ".bnb"
            w[name] = nb
            cn.inputs = cn.inputs[:2] + [name]
        cn.outputs[0] = bn.outputs[0]
        drop.add(bi)
    g.nodes = [n for k, n in enumerate(g.nodes) if k not in drop]
    return len(fold)


def fuse_conv_activation(g: Graph) -> int:
    """Conv (group == 1) -> Relu becomes Conv act=2 (optimize.rs:337-427)."""
    consumers = _consumer_counts(g)
    first = _first_consumer(g)
    fuse = []
    for i, cn in enumerate(g.nodes):
        if cn.op_type != "Conv" or len(cn.outputs) != 1:
            continue
        co = cn.outputs[0]
        if g.is_graph_output(co) or consumers.get(co, 0) != 1:
            continue
        cu = first.get(co)
        if cu is None:
            continue
        an = g.nodes[cu]
        if an.op_type not in ("FusedGelu", "Relu") or len(an.inputs) != 1 or an.inputs[0] != co:
            continue
        if int(cn.attr("group", 1)) != 1:
            continue
        fuse.append((i, cu))
    drop = set()
    for ci, ai in fuse:
        an = g.nodes[ai]
        cn = g.nodes[ci]
        cn.attrs["act"] = 1 if an.op_type == "FusedGelu" else 2
        cn.outputs[0] = an.outputs[0]
        drop.add(ai)
    g.nodes = [n for k, n in enumerate(g.nodes) if k not in drop]
    return len(fuse)


def fuse_conv_residual(g: Graph, w: Dict[str, np.ndarray]) -> int:
    """Conv -> Add(conv_out, R) folds R into Conv inputs[3] (optimize.rs:662-770)."""
    consumers = _consumer_counts(g)
    first = _first_consumer(g)
    producer = {}
    for k, n in enumerate(g.nodes):
        for o in n.outputs:
            producer[o] = k
    fuse = []
    for i, cn in enumerate(g.nodes):
        if cn.op_type != "Conv" or len(cn.inputs) < 2 or len(cn.outputs) != 1:
            continue
        co = cn.outputs[0]
        if g.is_graph_output(co) or consumers.get(co, 0) != 1:
            continue
        au = first.get(co)
        if au is None:
            continue
        an = g.nodes[au]
        if an.op_type != "Add" or len(an.inputs) != 2 or len(an.outputs) != 1:
            continue
        if an.inputs[0] == co:
            r = an.inputs[1]
        elif an.inputs[1] == co:
            r = an.inputs[0]
        else:
            continue
        if not r or r in w or r in g.inputs:
            continue
        rp = producer.get(r)
        if rp is None or rp >= i:
            continue
        fuse.append((i, au))
    drop = set()
    for ci, ai in fuse:
        an = g.nodes[ai]
        cn = g.nodes[ci]
        co = cn.outputs[0]
        r = an.inputs[1] if an.inputs[0] == co else an.inputs[0]
        if len(cn.inputs) == 2:
            m = w[cn.inputs[1]].shape[0]
            zname = an.outputs[0] + ".zb"
            w[zname] = np.zeros(m, np.float32)
            cn.inputs.append(zname)
        cn.inputs.append(r)
        cn.outputs[0] = an.outputs[0]
        drop.add(ai)
    g.nodes = [n for k, n in enumerate(g.nodes) if k not in drop]
    return len(fuse)


def fuse_mul_add(g: Graph) -> int:
    """Add(Mul(f, g), r) -> MulAddScale(f, g, r) (optimize.rs:437-497)."""
    consumers = _consumer_counts(g)
    producer = {}
    for k, n in enumerate(g.nodes):
        for o in n.outputs:
            producer[o] = k
    fuse = []
    for i, an in enumerate(g.nodes):
        if an.op_type != "Add" or len(an.inputs) != 2 or len(an.outputs) != 1:
            continue
        for side in range(2):
            mo = an.inputs[side]
            if not mo or consumers.get(mo, 0) != 1:
                continue
            mi = producer.get(mo)
            if mi is None:
                continue
            mn = g.nodes[mi]
            if mn.op_type != "Mul" or len(mn.inputs) != 2 or len(mn.outputs) != 1:
                continue
            fuse.append((i, mi, side == 0))
            break
    drop = set()
    for ai, mi, mul_first in fuse:
        mn = copy.deepcopy(g.nodes[mi])
        an = g.nodes[ai]
        residual = an.inputs[1 if mul_first else 0]
        an.op_type = "MulAddScale"
        an.inputs = [mn.inputs[0], mn.inputs[1], residual]
        an.attrs = {}
        an.name = "fused:" + an.name
        drop.add(mi)
    g.nodes = [n for k, n in enumerate(g.nodes) if k not in drop]
    return len(fuse)


def optimize(g: Graph, w: Dict[str, np.ndarray]) -> Graph:
    """The reference loader's pass order (parse.rs:731-747) on a copy of `g`.

    `w` (the initializers) is modified in place, as the reference folds into
    its initializer table.
    """
    g = copy.deepcopy(g)
    fold_conv_batchnorm(g, w)
    fuse_conv_activation(g)
    fuse_conv_residual(g, w)
    fuse_mul_add(g)
    return g
