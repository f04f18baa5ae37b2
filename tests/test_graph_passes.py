"""Host-side graph logic on CPU: the reference loader passes applied to the
synthetic networks, checked numerically on the oracle."""
import numpy as np
import pytest

import oracle as orc
from qppocr_b200 import graph as G
from qppocr_b200 import nets


def rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return np.abs(a - b).max() / max(np.abs(b).max(), 1e-6)


def test_block_passes():
    g, w = nets.build_block()
    w0 = {k: v.copy() for k, v in w.items()}
    go = G.optimize(g, w)
    ops = [n.op_type for n in go.nodes]
    assert "BatchNormalization" not in ops
    assert ops.count("Conv") == 2
    x = nets.block_input(0, (1, 64, 24, 24))
    y0 = orc.run_graph(g, w0, {"x": x})[0]
    y1 = orc.run_graph(go, w, {"x": x})[0]
    assert y0.shape == (1, 128, 24, 24)
    assert rel(y1, y0) < 1e-5  # BN folding is exact in math, ~ulp in fp32


def test_det_passes_small():
    g, w = nets.build_det()
    w0 = {k: v.copy() for k, v in w.items()}
    go = G.optimize(g, w)
    ops = [n.op_type for n in go.nodes]
    # BN after every backbone conv folded; only the head's ConvT BN remains
    assert ops.count("BatchNormalization") == 1
    # FPN top-down adds became conv residuals (optimize.rs:662-770)
    assert sum(1 for n in go.nodes if n.op_type == "Conv" and len(n.inputs) == 4) == 3
    # head 3x3 conv + ReLU fused (act = 2)
    assert any(n.attrs.get("act") == 2 for n in go.nodes if n.op_type == "Conv")
    x = nets.det_input(1, 64, 64)
    y0 = orc.run_graph(g, w0, {"x": x})[0]
    y1 = orc.run_graph(go, w, {"x": x})[0]
    assert y1.shape == (1, 1, 64, 64)
    assert rel(y1, y0) < 1e-4


def test_rec_passes_small():
    g, w = nets.build_rec()
    w0 = {k: v.copy() for k, v in w.items()}
    go = G.optimize(g, w)
    ops = [n.op_type for n in go.nodes]
    assert "MulAddScale" in ops  # LayerNorm affine tail collapsed
    x = nets.rec_input(2)
    y0 = orc.run_graph(g, w0, {"x": x})[0]
    y1 = orc.run_graph(go, w, {"x": x})[0]
    assert y1.shape == (2, 40, nets.REC_CLASSES)
    assert rel(y1, y0) < 1e-4
    pr = orc.argmax_pairs(y1)
    assert pr.shape == (2, 40, 2)


def test_cls_passes_small():
    g, w = nets.build_cls()
    go = G.optimize(g, w)
    y = orc.run_graph(go, w, {"x": nets.cls_input(3)})[0]
    assert y.shape == (3, 2)
    assert np.allclose(y.sum(-1), 1.0, atol=1e-5)
