"""Full det -> cls -> rec pipeline over a batch of images on one GPU, in the
stage order of the reference engine's run_once
(crates/qppocr-core/src/pipeline/engine.rs:836-1740), with every image-sized
step on the device:

  1. det: the uint8 images (already in device memory) through the det session
     with the DB mask exit: the u8 mask comes back to the host, where the
     connected components that find text boxes run (geometry.rs:170-216); the
     probability map stays on the device.
  2. boxes: the caller supplies them (config 5: axis-aligned boxes at seeded
     random positions, in place of the host's connected-component boxes).
     They are scored on the device against the kept map, as the DB post does
     before filtering (box_score_fast, geometry.rs:221-269).
  3. crops: crop_text_box (crop.rs:8-127) of every box, on the device.
  4. cls: batches of up to cls_batch lines (engine.rs:1297-1327), each line the
     cls_view window (crop.rs:193-218) packed to cls_h x cls_w (pack_crop),
     through the cls session; a line flips when p1 > p0 and p1 >= cls_thresh
     (engine.rs:1380-1407).  The batch dimension enters no reduction, so the
     batch size changes no result (engine.rs:1309-1312).
  5. rec: batches of up to rec_batch lines packed at rec_h x rec_w (flipped
     lines rotated 180 degrees as they are packed), submitted while the
     previous batch runs (run_deferred, engine.rs:1409-1450), through the rec
     session's argmax exit, decoded on the host (rec.rs:82-120).
"""
import time
from typing import Dict, Iterable, Iterator, Optional

import numpy as np

from . import DeviceOutput, op_box_score, op_crop_text_boxes, op_line_pack
from .rec_pipeline import ctc_decode_pairs_batch

F32 = np.float32


def cls_windows(h: np.ndarray, w: np.ndarray, cls_h: int, cls_w: int):
    """crop.rs:193-218 cls_view: (x0, view width) per crop; crops wider than
    h * cls_w / cls_h (integer) keep that many centred columns."""
    h = np.asarray(h, np.int64)
    w = np.asarray(w, np.int64)
    max_w = h * cls_w // cls_h
    cut = (h > 0) & (w > max_w)
    vw = np.where(cut, np.maximum(1, max_w), w)
    x0 = np.where(cut, (w - vw) // 2, 0)
    return x0.astype(np.int32), vw.astype(np.int32)


def packed_width(h: np.ndarray, w: np.ndarray, img_h: int, img_w: int) -> np.ndarray:
    """crop.rs:171-173 per line: ceil(img_h * (w / h)) in f32, within [1, img_w]."""
    ratio = np.asarray(w, F32) / np.asarray(h, F32)
    return np.clip(np.ceil(F32(img_h) * ratio), 1, img_w).astype(np.int32)


def synthetic_boxes(n_images: int, per_image: int, h: int, w: int, seed: int = 50) -> np.ndarray:
    """Config 5's boxes: per image `per_image` axis-aligned text boxes at
    seeded random positions, 16-48 px high and 2-12 heights wide, inside the
    image; [n_images, per_image, 4, 2] (x, y) corners TL, TR, BR, BL."""
    rng = np.random.Generator(np.random.PCG64(seed))
    bh = rng.integers(16, 49, (n_images, per_image)).astype(np.float32)
    bw = np.minimum(bh * rng.uniform(2, 12, (n_images, per_image)), w - 2).astype(np.float32)
    x0 = (rng.random((n_images, per_image)) * (w - 1 - bw)).astype(np.float32)
    y0 = (rng.random((n_images, per_image)) * (h - 1 - bh)).astype(np.float32)
    x0, y0 = np.floor(x0), np.floor(y0)
    pts = np.stack([np.stack([x0, y0], -1), np.stack([x0 + bw, y0], -1), np.stack([x0 + bw, y0 + bh], -1),
                    np.stack([x0, y0 + bh], -1)], axis=2)
    return np.floor(pts).astype(np.float32)


class OcrPipeline:
    """det -> box scores -> crops -> cls -> rec on one GPU.  det: a det
    session created with det_mask_exit=True; cls / rec: sessions of the cls
    and rec roles (rec with its argmax exit)."""

    def __init__(self, det, cls, rec, device: Optional[int] = None, cls_h: int = 80, cls_w: int = 160,
                 rec_h: int = 48, rec_w: int = 320, cls_batch: int = 32, cls_thresh: float = 0.9,
                 rec_batch: Optional[int] = None):
        self.det, self.cls, self.rec = det, cls, rec
        self.device = getattr(det, "device", 0) if device is None else device
        self.cls_h, self.cls_w, self.rec_h, self.rec_w = cls_h, cls_w, rec_h, rec_w
        self.cls_batch = max(1, cls_batch)
        self.cls_thresh = F32(cls_thresh)
        self.rec_batch = rec.rec_chunk() if rec_batch is None else rec_batch
        assert rec.rec_argmax_pairs(), "the rec session needs its argmax exit"

    def run(self, images, boxes: np.ndarray, keep: bool = False) -> Dict:
        """images: [n, h, w, 3] uint8 torch tensor on this pipeline's GPU;
        boxes: [n, k, 4, 2] f32 corners in image coordinates.  Returns the
        mask, box scores, cls probabilities and flips, and per line the
        decoded (indices, confidence); keep=True adds the device
        intermediates (crops, packed cls and rec batches) for checking.
        `timings` holds the wall-clock ms of each stage, as the reference
        bench reports det / crop / cls / rec (crates/qppocr-cli/src/main.rs:
        860-880): det (to the mask on the host), boxes + crops, cls, rec
        (packing, runs and CTC decode)."""
        import torch

        t0 = time.perf_counter()
        torch.cuda.current_stream(torch.device("cuda", self.device)).synchronize()  # images in place
        # 1. det with the mask exit; the probability map stays on the device
        mask, pred = self.det.run({"x": images})
        return self._after_det(images, boxes, mask, pred, keep, t0)

    def run_many(self, batches: Iterable, keep: bool = False) -> Iterator[Dict]:
        """run() over an iterable of (images, boxes) or (images, boxes,
        ready) batches, yielding one result per batch, with det one batch
        ahead: as soon as a batch's det finishes, the next batch's det is
        submitted (run_deferred, a second plan instance) and runs on the GPU
        while this batch's boxes, crops, cls and rec are done - the overlap
        the reference engine gets from keeping two batches in flight
        (engine.rs:1409-1450).  `ready`, when given, is a torch.cuda.Event
        recorded after the batch's images were copied to the device (on any
        stream); without it the current stream is synchronised.  Results are
        those of run() batch by batch; `timings["det_ms"]` is then the wait for
        that batch's det after the previous batch was done."""
        import torch

        dev = torch.device("cuda", self.device)

        def submit(b):
            if len(b) > 2 and b[2] is not None:
                b[2].synchronize()
            else:
                torch.cuda.current_stream(dev).synchronize()
            return self.det.run_deferred({"x": b[0]})

        it = iter(batches)
        cur = next(it, None)
        if cur is None:
            return
        pend = submit(cur)
        nxt = next(it, None)  # the caller may start its upload now
        while cur is not None:
            t0 = time.perf_counter()
            mask, pred = pend.complete()
            pend = submit(nxt) if nxt is not None else None
            after = next(it, None) if nxt is not None else None
            res = self._after_det(cur[0], cur[1], mask, pred, keep, t0)
            mask = pred = None
            yield res
            cur, nxt = nxt, after

    def _after_det(self, images, boxes, mask, pred, keep, t0) -> Dict:
        """Steps 2-5 of run() for one batch whose det outputs are at hand."""
        import torch

        dev = torch.device("cuda", self.device)
        n, h, w, _ = images.shape
        k = boxes.shape[1]
        assert isinstance(pred, DeviceOutput)
        out: Dict = {"mask": mask}
        t_det = time.perf_counter()
        # 2. boxes scored on the kept map
        pts = np.ascontiguousarray(boxes, np.float32).reshape(n * k, 4, 2)
        img = np.repeat(np.arange(n, dtype=np.int32), k)
        pmap = pred.torch()
        scale = np.array([pmap.shape[3] / w, pmap.shape[2] / h], np.float32)
        sc = op_box_score(pmap[:, 0], torch.from_numpy(pts * scale).to(dev), torch.from_numpy(img).to(dev))
        # 3. crops from the original images
        crops, off, cw, ch, rot = op_crop_text_boxes(images, pts, img)
        ch_, cw_ = np.where(rot, cw, ch), np.where(rot, ch, cw)  # rows, columns of each crop
        lines = n * k
        # 4. cls over cls_batch-line batches
        x0, vw = cls_windows(ch_, cw_, self.cls_h, self.cls_w)
        crw = packed_width(ch_, vw, self.cls_h, self.cls_w)
        probs = np.empty((lines, 2), np.float32)
        cls_in = []
        torch.cuda.current_stream(dev).synchronize()  # crops complete before the sessions read them
        t_crop = time.perf_counter()
        for b in range(0, lines, self.cls_batch):
            e = min(b + self.cls_batch, lines)
            xb = op_line_pack(crops, off[b:e], cw_[b:e], x0[b:e], ch_[b:e], vw[b:e], crw[b:e],
                              np.zeros(e - b, np.int32), self.cls_h, self.cls_w)
            torch.cuda.current_stream(dev).synchronize()
            probs[b:e] = self.cls.run({"x": xb})[0].reshape(e - b, 2)
            if keep:
                cls_in.append(xb.cpu().numpy())
        flips = ((probs[:, 1] > probs[:, 0]) & (probs[:, 1] >= self.cls_thresh)).astype(np.int32)
        t_cls = time.perf_counter()
        # 5. rec, one batch packed and submitted while the previous one runs
        rrw = packed_width(ch_, cw_, self.rec_h, self.rec_w)
        zeros = np.zeros(lines, np.int32)
        results = [None] * lines
        rec_in, rec_pairs = [], []
        pending = None
        for b in range(0, lines, self.rec_batch):
            e = min(b + self.rec_batch, lines)
            xb = op_line_pack(crops, off[b:e], cw_[b:e], zeros[b:e], ch_[b:e], cw_[b:e], rrw[b:e], zeros[b:e],
                              self.rec_h, self.rec_w, flip=flips[b:e])
            torch.cuda.current_stream(dev).synchronize()
            if keep:
                rec_in.append(xb.cpu().numpy())
            d = self.rec.run_deferred({"x": xb})
            if pending is not None:
                rec_pairs.append(self._finish(*pending, results))
            pending = (d, b, e)
        if pending is not None:
            rec_pairs.append(self._finish(*pending, results))
        t_rec = time.perf_counter()
        out["scores"] = sc.cpu().numpy()
        if keep:
            out["pred"] = pmap.cpu().numpy()
        del pmap, pred
        out.update(probs=probs, flips=flips.astype(bool), results=results, lines=lines,
                   seconds=time.perf_counter() - t0,
                   timings={"det_ms": 1e3 * (t_det - t0), "crop_ms": 1e3 * (t_crop - t_det),
                            "cls_ms": 1e3 * (t_cls - t_crop), "rec_ms": 1e3 * (t_rec - t_cls)})
        if keep:
            out.update(crops=crops.cpu().numpy(), off=off, crop_h=ch_, crop_w=cw_, cls_in=np.concatenate(cls_in),
                       rec_in=np.concatenate(rec_in), rec_pairs=np.concatenate(rec_pairs))
        return out

    @staticmethod
    def _finish(d, b, e, results):
        pairs = d.complete()[0][:e - b]
        for i, r in enumerate(ctc_decode_pairs_batch(pairs)):
            results[b + i] = r
        return pairs
