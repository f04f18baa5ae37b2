"""The device line pack (crop.rs:153-185) bit-exact against the oracle, and
the whole recognition stage (grouping, device packing, pipelined runs with
device-tensor inputs, CTC decode) against the oracle run batch by batch."""
import numpy as np
import pytest

import oracle as orc
import qppocr_b200 as q
from qppocr_b200 import nets
from qppocr_b200 import rec_pipeline as rp

pytestmark = pytest.mark.gpu


def crops(n, seed=0, hmin=16, hmax=64, wmin=8, wmax=420):
    rng = np.random.Generator(np.random.PCG64(seed))
    out = []
    for _ in range(n):
        h = int(rng.integers(hmin, hmax + 1))
        w = int(rng.integers(wmin, wmax + 1))
        out.append(rng.integers(0, 256, (h, w, 3), dtype=np.uint8))
    return out


def test_rec_pack_bit_exact(cuda_ctx):
    import torch
    cs = crops(12, seed=1)
    cs.append(np.full((48, 20, 3), 200, np.uint8))           # already at img_h
    cs.append(np.arange(40 * 30 * 3, dtype=np.uint8).reshape(40, 30, 3))  # pad-only below
    img_h, img_w = 48, 256
    pads = [0] * (len(cs) - 1) + [1]
    rws = [min(c.shape[1], img_w) if p else rp.resized_width(c.shape[0], c.shape[1], img_h, img_w)
           for c, p in zip(cs, pads)]
    offs = np.concatenate([[0], np.cumsum([c.size for c in cs])[:-1]]).astype(np.int64)
    blob = torch.from_numpy(np.concatenate([c.reshape(-1) for c in cs])).cuda()
    dv = lambda a: torch.from_numpy(np.asarray(a)).cuda()
    got = q.op_rec_pack(blob, dv(offs), dv(np.array([c.shape[0] for c in cs], np.int32)),
                        dv(np.array([c.shape[1] for c in cs], np.int32)), dv(np.array(rws, np.int32)),
                        dv(np.array(pads, np.int32)), img_h, img_w).cpu().numpy()
    for k, (c, rw, p) in enumerate(zip(cs, rws, pads)):
        ref = orc.rec_pack_line(c, rw, img_h, img_w, bool(p))
        assert np.array_equal(got[k].view(np.uint32), ref.view(np.uint32)), k


def test_rec_stage_matches_oracle(cuda_ctx):
    g, w = nets.build_rec()
    g = q.optimize(g, w)
    s = cuda_ctx.create_session(g, w, role="rec", math="3xtf32")
    stage = rp.RecStage(s, per_batch=8)
    cs = crops(30, seed=3)
    got = stage.run(cs)
    assert stage.batches >= 3
    shapes = [(c.shape[0], c.shape[1]) for c in cs]
    n_diff = 0
    for ids, img_w in stage.plan(shapes):
        batch = np.stack([orc.rec_pack_line(cs[i], rp.resized_width(*shapes[i], 48, img_w), 48, img_w)
                          for i in ids])
        probs = orc.run_graph(g, w, {"x": batch})[0]
        for k, i in enumerate(ids):
            ref_idx, ref_conf = orc.ctc_decode(probs[k])
            got_idx, got_conf = got[i]
            if got_idx != ref_idx:
                # only where the oracle's top-2 probabilities nearly tie
                top2 = np.sort(probs[k], axis=1)[:, -2:]
                assert np.min(top2[:, 1] - top2[:, 0]) < 1e-5, (i, got_idx, ref_idx)
                n_diff += 1
            else:
                assert abs(float(got_conf) - float(ref_conf)) <= 1e-5 * max(1.0, abs(float(ref_conf)))
    assert n_diff <= 1
