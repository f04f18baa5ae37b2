"""Recognition stage around a rec session: the reference engine's line
grouping, batch packing, pipelined submission and CTC decoding, with the
packing on the device.

  * lines sorted by width ratio, stably (engine.rs:1162-1163), ratio = w / h
    (crop.rs:136-145 batch_ratio);
  * consecutive lines grouped while their raw widths (img_h * ratio,
    truncated) stay within one width grain of the group's first line, at most
    `per_batch` lines (engine.rs:1238-1286, the default relative-span rule;
    the grain and per_batch default to the session's bucket_grain and
    rec_chunk, device.rs:139-163);
  * batch width = img_h * max(rec_min_width / img_h, max ratio), truncated,
    rounded up to the grain (engine.rs:1416-1423);
  * each line resized to ceil(img_h * w / h) x img_h (at most the batch width)
    and normalised (v / 255 - 0.5) / 0.5 into a zeroed batch
    (crop.rs:153-185, engine.rs:1425-1440) - on the device, by
    qpc_op_rec_pack;
  * batch k + 1 packed and submitted while batch k runs (run_deferred,
    engine.rs:1409-1450), the packed batch handed over as a device tensor;
  * greedy CTC decoding of the (value, index) pairs of the argmax exit
    (rec.rs:82-120) or of full probabilities (rec.rs:34-79).
"""
from typing import List, Optional, Sequence, Tuple

import numpy as np

from . import op_rec_pack

F32 = np.float32


def crop_pads(h: int, img_h: int, pad_min_h: float) -> bool:
    """crop.rs:129-131: a crop close to img_h is centred, not resized."""
    return pad_min_h > 0.0 and 0 < h <= img_h and h >= pad_min_h * img_h


def batch_ratio(h: int, w: int, img_h: int, pad_min_h: float = 0.0) -> np.float32:
    """crop.rs:136-145 (f32)."""
    if h <= 0:
        return F32(1.0)
    if crop_pads(h, img_h, pad_min_h):
        return F32(w) / F32(img_h)
    return F32(w) / F32(h)


def raw_width(img_h: int, ratio) -> int:
    """engine.rs:1228: (img_h as f32 * r) as i32."""
    return int(F32(img_h) * F32(ratio))


def group_lines(ratios_sorted: Sequence, img_h: int, grain: int, per_batch: int) -> List[Tuple[int, int]]:
    """engine.rs:1238-1286 (relative span when grain > 1, else fixed chunks):
    [begin, end) ranges over the ratio-sorted lines."""
    n = len(ratios_sorted)
    out = []
    beg = 0
    while beg < n:
        end = beg + 1
        if grain > 1:
            w0 = raw_width(img_h, ratios_sorted[beg])
            while end < n and end - beg < per_batch and raw_width(img_h, ratios_sorted[end]) - w0 <= grain:
                end += 1
        else:
            end = min(beg + per_batch, n)
        out.append((beg, end))
        beg = end
    return out


def batch_width(ratios: Sequence, img_h: int, min_width: int, grain: int) -> int:
    """engine.rs:1416-1423."""
    m = F32(min_width) / F32(img_h)
    for r in ratios:
        m = max(m, F32(r))
    w = int(F32(img_h) * m)
    if grain > 1:
        w = (w + grain - 1) // grain * grain
    return w


def resized_width(h: int, w: int, img_h: int, img_w: int) -> int:
    """crop.rs:171-173: ceil(img_h * (w / h)), clamped to [1, img_w]."""
    ratio = F32(w) / F32(h)
    rw = int(np.ceil(F32(img_h) * ratio))
    return max(min(rw, img_w), 1)


def ctc_decode_pairs(pairs, charset: Optional[Sequence[str]] = None):
    """rec.rs:82-120: pairs [T, 2] = (value, index as f32 bits).  A step emits
    when its index is not 0 (blank) and differs from the previous step's;
    conf = f64 mean of the emitted steps' values.  Returns (indices or text,
    conf)."""
    pairs = np.asarray(pairs, np.float32).reshape(-1, 2)
    idx = pairs[:, 1].copy().view(np.uint32).astype(np.int64)
    vals = pairs[:, 0]
    out, conf_sum, conf_n, prev = [], 0.0, 0, -1
    for t in range(pairs.shape[0]):
        b = int(idx[t])
        if b != 0 and b != prev:
            if charset is None or b < len(charset):
                out.append(b)
            conf_sum += float(vals[t])
            conf_n += 1
        prev = b
    conf = np.float32(conf_sum / conf_n) if conf_n else np.float32(0.0)
    if charset is not None:
        return "".join(charset[i] for i in out), conf
    return out, conf


def ctc_decode_pairs_batch(pairs, charset: Optional[Sequence[str]] = None):
    """ctc_decode_pairs over a batch [B, T, 2] with array operations.  The
    confidence sum runs left to right in f64 (cumsum), as the per-line loop
    does, so the results are identical."""
    pairs = np.asarray(pairs, np.float32)
    b, t = pairs.shape[0], pairs.shape[1]
    idx = np.ascontiguousarray(pairs[:, :, 1]).view(np.uint32).astype(np.int64)
    vals = pairs[:, :, 0].astype(np.float64)
    prev = np.empty_like(idx)
    prev[:, 0] = -1
    prev[:, 1:] = idx[:, :-1]
    emit = (idx != 0) & (idx != prev)
    cnt = emit.sum(axis=1)
    sums = np.cumsum(np.where(emit, vals, 0.0), axis=1)[:, -1] if t else np.zeros(b)
    keep = emit if charset is None else emit & (idx < len(charset))
    with np.errstate(divide="ignore", invalid="ignore"):
        conf = np.where(cnt > 0, sums / np.maximum(cnt, 1), 0.0).astype(np.float32)
    flat = idx[keep].tolist()  # row-major: line k's kept indices are consecutive
    lens = keep.sum(axis=1).tolist()
    out, pos = [], 0
    for k in range(b):
        ids = flat[pos:pos + lens[k]]
        pos += lens[k]
        out.append(("".join(map(charset.__getitem__, ids)) if charset is not None else ids, conf[k]))
    return out


def ctc_decode_probs(probs, charset: Optional[Sequence[str]] = None):
    """rec.rs:34-79 on one line's [T, C] probabilities (first strict max)."""
    probs = np.asarray(probs, np.float32)
    best = np.argmax(probs, axis=1)  # numpy: first maximum, as the reference's strict '>'
    pairs = np.empty((probs.shape[0], 2), np.float32)
    pairs[:, 0] = probs[np.arange(probs.shape[0]), best]
    pairs[:, 1] = best.astype(np.uint32).view(np.float32)
    return ctc_decode_pairs(pairs, charset)


def plan_lines(shapes: Sequence[Tuple[int, int]], img_h: int, pad_min_h: float, min_width: int, grain: int,
               per_batch: int):
    """The engine's line plan (batch_ratio, a stable sort, group_lines,
    batch_width) with array operations: the same float32 arithmetic per line,
    the same stable order; the raw widths are non-decreasing along the sorted
    ratios, so each group's end is one binary search.  Returns [(ids, img_w)]."""
    hw = np.asarray(shapes, np.int64).reshape(-1, 2)
    h, w = hw[:, 0], hw[:, 1]
    pads = (pad_min_h > 0.0) & (h > 0) & (h <= img_h) & (h >= pad_min_h * img_h)
    with np.errstate(divide="ignore", invalid="ignore"):
        ratio = np.where(pads, w.astype(F32) / F32(img_h), w.astype(F32) / h.astype(F32)).astype(F32)
    ratio[h <= 0] = F32(1.0)
    order = np.argsort(ratio, kind="stable")
    rs = ratio[order]
    raw = (F32(img_h) * rs).astype(np.int64)
    m0 = F32(min_width) / F32(img_h)
    out, beg, n = [], 0, len(rs)
    while beg < n:
        if grain > 1:
            lim = int(np.searchsorted(raw, raw[beg] + grain, side="right"))
            end = max(beg + 1, min(beg + per_batch, lim))
        else:
            end = max(beg + 1, min(beg + per_batch, n))
        wb = int(F32(img_h) * max(m0, rs[beg:end].max()))
        if grain > 1:
            wb = (wb + grain - 1) // grain * grain
        out.append((order[beg:end].tolist(), wb))
        beg = end
    return out


def line_table(shapes: Sequence[Tuple[int, int]], batches, offs, img_h: int, pad_min_h: float) -> np.ndarray:
    """[5, lines] int64 in batch order: crop offset, h, w, resized width
    (ceil(img_h * w / h) clamped to [1, img_w], or min(w, img_w) for a padded
    crop, as resized_width / crop_pads), pad flag."""
    ids = np.asarray([i for b, _ in batches for i in b], np.int64)
    img_w = np.asarray([wb for b, wb in batches for _ in b], np.int64)
    hw = np.asarray(shapes, np.int64).reshape(-1, 2)[ids] if len(ids) else np.zeros((0, 2), np.int64)
    h, w = hw[:, 0], hw[:, 1]
    if (h <= 0).any():
        raise ValueError("crop of height 0")
    pads = (pad_min_h > 0.0) & (h <= img_h) & (h >= pad_min_h * img_h)
    rw = np.ceil(F32(img_h) * (w.astype(F32) / h.astype(F32))).astype(np.int64)
    rw = np.where(pads, np.minimum(w, img_w), np.maximum(np.minimum(rw, img_w), 1))
    return np.stack([np.asarray(offs, np.int64)[ids], h, w, rw, pads.astype(np.int64)])


class RecStage:
    """Lines (uint8 h x w x 3 crops) -> (text or indices, confidence), through
    a rec session created by CudaContext.create_session(role="rec")."""

    def __init__(self, session, img_h: int = 48, min_width: int = 16, pad_min_h: float = 0.0,
                 grain: Optional[int] = None, per_batch: Optional[int] = None, charset=None,
                 device: Optional[int] = None):
        self.s = session
        self.img_h = img_h
        self.min_width = min_width
        self.pad_min_h = pad_min_h
        self.grain = session.bucket_grain() if grain is None else grain
        self.per_batch = session.rec_chunk() if per_batch is None else per_batch
        self.charset = charset
        self.pairs = session.rec_argmax_pairs()
        # device tensors (crops, packed batches) live on the session's own GPU
        self.device = getattr(session, "device", 0) if device is None else device
        self.batches = 0

    def plan(self, shapes: Sequence[Tuple[int, int]]):
        """Order, batches and per-line widths for crops of these (h, w)."""
        return plan_lines(shapes, self.img_h, self.pad_min_h, self.min_width, self.grain, self.per_batch)

    def run(self, crops: Sequence[np.ndarray]):
        import torch

        shapes = [(int(c.shape[0]), int(c.shape[1])) for c in crops]
        batches = self.plan(shapes)
        dev = torch.device("cuda", self.device)
        # all crops uploaded once, back to back: concatenated straight into
        # pinned memory (one copy), then one DMA
        sizes = [c.size for c in crops]
        offs = np.zeros(len(crops), np.int64)
        if len(crops) > 1:
            offs[1:] = np.cumsum(sizes)[:-1]
        total = int(sum(sizes))
        pinned = torch.empty(max(total, 1), dtype=torch.uint8, pin_memory=True)
        if total:
            np.concatenate([np.ascontiguousarray(c, np.uint8).reshape(-1) for c in crops], out=pinned.numpy()[:total])
        blob = pinned.to(dev, non_blocking=True)
        # every batch's line table (offset, h, w, resized width, pad flag), in
        # batch order, also uploaded once; each batch takes its columns
        n_lines = sum(len(ids) for ids, _ in batches)
        table = torch.empty((5, max(n_lines, 1)), dtype=torch.int64, pin_memory=True)
        if n_lines:
            table.numpy()[:, :n_lines] = line_table(shapes, batches, offs, self.img_h, self.pad_min_h)
        spans, col = [], 0
        for ids, _ in batches:
            spans.append((col, col + len(ids)))
            col += len(ids)
        dtab = table.to(dev, non_blocking=True)
        d32 = dtab[1:].to(torch.int32)  # h, w, resized width, pad flag: one conversion for all lines
        results: List = [None] * len(crops)

        def submit(ids, img_w, span):
            a, b = span  # this batch's columns: contiguous slices of each table row
            x = op_rec_pack(blob, dtab[0, a:b], d32[0, a:b], d32[1, a:b], d32[2, a:b], d32[3, a:b], self.img_h,
                            img_w)
            torch.cuda.current_stream(dev).synchronize()  # packed before the session's stream copies it
            self.batches += 1
            return self.s.run_deferred({"x": x})

        pending = None
        for (ids, img_w), span in zip(batches, spans):
            d = submit(ids, img_w, span)
            if pending is not None:
                self._finish(*pending, results)
            pending = (d, ids)
        if pending is not None:
            self._finish(*pending, results)
        return results

    def _finish(self, d, ids, results):
        out = d.complete()[0]
        if self.pairs:
            for i, r in zip(ids, ctc_decode_pairs_batch(out[:len(ids)], self.charset)):
                results[i] = r
        else:
            for k, i in enumerate(ids):
                results[i] = ctc_decode_probs(out[k], self.charset)
