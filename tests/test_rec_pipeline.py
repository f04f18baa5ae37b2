"""Host logic of the recognition stage (engine.rs:1160-1500, crop.rs:129-185,
rec.rs:34-120) on hand-worked cases and against the oracle's CTC decoder."""
import numpy as np
import pytest

import oracle as orc
from qppocr_b200 import rec_pipeline as rp


def test_group_lines_relative_span():
    # raw widths at img_h 48: 48, 96, 120, 192, 480 (grain 64)
    ratios = [np.float32(r) for r in (1.0, 2.0, 2.5, 4.0, 10.0)]
    assert rp.group_lines(ratios, 48, 64, 256) == [(0, 2), (2, 3), (3, 4), (4, 5)]
    # per_batch caps a group
    assert rp.group_lines([np.float32(1.0)] * 5, 48, 64, 2) == [(0, 2), (2, 4), (4, 5)]
    # grain <= 1: fixed chunks
    assert rp.group_lines(ratios, 48, 1, 2) == [(0, 2), (2, 4), (4, 5)]


def test_batch_width_and_resized_width():
    assert rp.batch_width([np.float32(1.0), np.float32(2.0)], 48, 16, 64) == 128  # 96 -> 128
    assert rp.batch_width([np.float32(0.2)], 48, 16, 64) == 64                    # min width 16 -> 64
    assert rp.batch_width([np.float32(2.0)], 48, 16, 1) == 96                     # no rounding
    assert rp.resized_width(32, 100, 48, 512) == 150                               # ceil(48 * 3.125)
    assert rp.resized_width(32, 100, 48, 128) == 128                               # clamped to the batch
    assert rp.resized_width(1000, 1, 48, 128) == 1                                 # at least 1


def test_batch_ratio_and_pads():
    assert rp.batch_ratio(32, 96, 48) == np.float32(3.0)
    assert not rp.crop_pads(40, 48, 0.0)          # default pad_min_h = 0: never pad-only
    assert rp.crop_pads(40, 48, 0.8)
    assert rp.batch_ratio(40, 96, 48, 0.8) == np.float32(2.0)  # w / img_h when pad-only


def test_ctc_decode_pairs_matches_oracle():
    rng = np.random.Generator(np.random.PCG64(2))
    for _ in range(20):
        t, c = 40, 30
        logits = rng.standard_normal((t, c)).astype(np.float32) * 3
        logits[rng.uniform(size=t) < 0.4, 0] += 6  # plenty of blanks
        p = np.exp(logits - logits.max(1, keepdims=True)).astype(np.float32)
        p /= p.sum(1, keepdims=True)
        pairs = orc.argmax_pairs(p)
        got_i, got_c = rp.ctc_decode_pairs(pairs)
        ref_i, ref_c = orc.ctc_decode(p)
        assert got_i == ref_i and got_c == ref_c
        assert rp.ctc_decode_probs(p) == (ref_i, ref_c)
    # charset: indices past it are skipped in the text but count for conf
    pairs = np.array([[0.9, 0], [0.8, 2], [0.7, 5], [0.6, 1]], np.float32)
    pairs[:, 1] = pairs[:, 1].astype(np.uint32).view(np.float32)
    text, conf = rp.ctc_decode_pairs(pairs, charset=["_", "a", "b"])
    assert text == "ba" and conf == np.float32((0.8 + 0.7 + 0.6) / 3)


class _FakeRecSession:
    """Capability queries only (DeviceSession caps, device.rs:134-163)."""

    def __init__(self, device):
        self.device = device

    def bucket_grain(self):
        return 64

    def rec_chunk(self):
        return 256

    def rec_argmax_pairs(self):
        return True


def test_rec_stage_uses_the_sessions_gpu():
    """The stage's device tensors (crops, packed batches) live on the GPU of
    the session they feed, so a rank driving GPU 1 never hands it GPU-0
    memory; an explicit device still wins."""
    from qppocr_b200.rec_pipeline import RecStage

    assert RecStage(_FakeRecSession(1)).device == 1
    assert RecStage(_FakeRecSession(3), device=2).device == 2


def test_batch_decode_matches_per_line():
    """The array form of the pairs decode gives the per-line loop's indices,
    text and f64-mean confidence exactly (rec.rs:82-120), blanks, repeats,
    out-of-charset indices and all-blank lines included."""
    from qppocr_b200.rec_pipeline import ctc_decode_pairs, ctc_decode_pairs_batch

    rng = np.random.Generator(np.random.PCG64(12))
    b, t = 37, 40
    pairs = np.empty((b, t, 2), np.float32)
    pairs[:, :, 0] = rng.uniform(1e-6, 1.0, (b, t)).astype(np.float32)
    idx = rng.integers(0, 6, (b, t)).astype(np.uint32)
    idx[3] = 0  # an all-blank line
    pairs[:, :, 1] = idx.view(np.float32)
    charset = ["_", "a", "b", "c", "d"]  # index 5 is outside the charset
    for cs in (None, charset):
        got = ctc_decode_pairs_batch(pairs, cs)
        for k in range(b):
            ref = ctc_decode_pairs(pairs[k], cs)
            assert got[k][0] == ref[0] and got[k][1] == ref[1] and type(got[k][1]) == type(ref[1])


def _plan_scalar(shapes, img_h, pad_min_h, min_width, grain, per_batch):
    """The plan line by line with the scalar restatements (batch_ratio,
    sorted, group_lines, batch_width)."""
    ratios = [rp.batch_ratio(h, w, img_h, pad_min_h) for h, w in shapes]
    order = sorted(range(len(shapes)), key=lambda i: ratios[i])
    groups = rp.group_lines([ratios[i] for i in order], img_h, grain, per_batch)
    return [(order[b:e], rp.batch_width([ratios[i] for i in order[b:e]], img_h, min_width, grain)) for b, e in groups]


@pytest.mark.parametrize("pad_min_h", [0.0, 0.8])
@pytest.mark.parametrize("grain,per_batch", [(1, 6), (16, 8), (64, 256), (32, 1)])
def test_vectorised_plan_and_line_table_match_the_scalar_rules(pad_min_h, grain, per_batch):
    """RecStage's array-form plan and per-line table equal the line-by-line
    restatements exactly: same order, groups, batch widths, resized widths and
    pad flags (ties in ratio included)."""
    rng = np.random.Generator(np.random.PCG64(int(pad_min_h * 10) + grain * 7 + per_batch))
    for n in (0, 1, 7, 300, 1024):
        hs = rng.integers(1, 80, n)
        ws = rng.integers(1, 900, n)
        if n > 20:
            hs[:10], ws[:10] = 32, 96  # equal ratios: the stable order decides
        shapes = [(int(h), int(w)) for h, w in zip(hs, ws)]
        got = rp.plan_lines(shapes, 48, pad_min_h, 16, grain, per_batch)
        ref = _plan_scalar(shapes, 48, pad_min_h, 16, grain, per_batch)
        assert got == ref
        offs = np.cumsum([0] + [h * w * 3 for h, w in shapes])[:-1]
        tab = rp.line_table(shapes, got, offs, 48, pad_min_h)
        col = 0
        for ids, img_w in got:
            for i in ids:
                h, w = shapes[i]
                p = rp.crop_pads(h, 48, pad_min_h)
                rw = min(w, img_w) if p else rp.resized_width(h, w, 48, img_w)
                assert tuple(tab[:, col]) == (offs[i], h, w, rw, int(p)), (i, tab[:, col])
                col += 1
        assert tab.shape == (5, n)
    # zero-height crops keep ratio 1 in the plan
    shapes = [(0, 50), (10, 40), (0, 5), (20, 20)]
    assert rp.plan_lines(shapes, 48, 0.0, 16, 16, 8) == _plan_scalar(shapes, 48, 0.0, 16, 16, 8)
