"""Config 5's det -> cls -> rec pipeline (qppocr_b200/pipeline.py) on 8
images end to end against the oracle pipeline, in 3xTF32.

Bit-exact: the mask against db_mask of the device's own probability map, the
box scores against box_score_fast on that map, every crop, every packed cls
and rec line.  Networks: the probability map, cls probabilities and rec
pairs within the fp32-mode tolerances; cls flips identical except lines whose
p1 lies within the tolerance of the threshold or of p0."""
import numpy as np
import pytest

import oracle as orc
import qppocr_b200 as q
from qppocr_b200 import nets
from qppocr_b200.pipeline import OcrPipeline, synthetic_boxes
from test_gpu_session import check_ctc, rel

pytestmark = pytest.mark.gpu

H = W = 320   # image size (config 5 uses 960; the checks do not depend on it)
N, K = 8, 16


def test_pipeline_matches_oracle(cuda_ctx):
    import torch
    gd, wd = nets.build_det()
    gd = q.optimize(gd, wd)
    gc, wc = nets.build_cls()
    gc = q.optimize(gc, wc)
    gr, wr = nets.build_rec()
    gr = q.optimize(gr, wr)
    det = cuda_ctx.create_session(gd, wd, role="det", math="3xtf32", det_mask_exit=True)
    cls = cuda_ctx.create_session(gc, wc, role="cls", math="3xtf32")
    rec = cuda_ctx.create_session(gr, wr, role="rec", math="3xtf32")
    rng = np.random.Generator(np.random.PCG64(60))
    imgs = rng.integers(0, 256, (N, H, W, 3), dtype=np.uint8)
    boxes = synthetic_boxes(N, K, H, W)
    # a few tall boxes, which crop_text_box rotates
    boxes[:, 0] = np.array([[10, 10], [40, 10], [40, 120], [10, 120]], np.float32)
    pipe = OcrPipeline(det, cls, rec, cls_batch=48, rec_batch=64)
    out = pipe.run(torch.from_numpy(imgs).cuda(), boxes, keep=True)
    pts = boxes.reshape(-1, 4, 2)
    img = np.repeat(np.arange(N), K).astype(np.int32)
    # det and its post
    pred = out["pred"]
    ref_pred = orc.run_graph(gd, wd, {"x": orc.det_normalize(imgs)})[0]
    assert rel(pred, ref_pred) < 1e-4
    assert np.array_equal(out["mask"], orc.db_mask(pred[:, 0], 0.3, dilate=True))
    assert np.array_equal(out["scores"].view(np.uint32), orc.box_scores(pred[:, 0], pts, img).view(np.uint32))
    # crops
    crops = []
    for j in range(N * K):
        c = orc.crop_text_box(imgs[img[j]], pts[j])
        got = out["crops"][out["off"][j]:out["off"][j] + c.size].reshape(c.shape)
        assert np.array_equal(got, c), j
        crops.append(c)
    assert crops[0].shape[1] > crops[0].shape[0]  # the tall box came out rotated
    # cls
    cls_in = np.stack([orc.cls_pack_line(c, 80, 160) for c in crops])
    assert np.array_equal(out["cls_in"].view(np.uint32), cls_in.view(np.uint32))
    ref_probs = orc.run_graph(gc, wc, {"x": cls_in})[0]
    assert rel(out["probs"], ref_probs) < 1e-5
    ref_flips = (ref_probs[:, 1] > ref_probs[:, 0]) & (ref_probs[:, 1] >= np.float32(0.9))
    near = (np.abs(ref_probs[:, 1] - 0.9) < 1e-5) | (np.abs(ref_probs[:, 1] - ref_probs[:, 0]) < 1e-5)
    assert not ((out["flips"] != ref_flips) & ~near).any()
    # rec, with the device's flips
    from qppocr_b200.pipeline import packed_width
    hs = np.array([c.shape[0] for c in crops])
    ws = np.array([c.shape[1] for c in crops])
    rw = packed_width(hs, ws, 48, 320)
    rec_in = np.stack([orc.rec_pack_line(np.ascontiguousarray(c[::-1, ::-1]) if f else c, int(r), 48, 320)
                       for c, f, r in zip(crops, out["flips"], rw)])
    assert np.array_equal(out["rec_in"].view(np.uint32), rec_in.view(np.uint32))
    probs = orc.run_graph(gr, wr, {"x": rec_in})[0]
    check_ctc(out["rec_pairs"], probs, 1e-5, 1e-5)
    assert len(out["results"]) == N * K and all(r is not None for r in out["results"])
    for s in (det, cls, rec):
        s.close()


def test_run_many_equals_run(cuda_ctx):
    """run_many (det one batch ahead, two det plan instances in flight) gives
    run()'s results batch by batch, bit for bit, including batches of
    different sizes and uploads signalled by events from a side stream."""
    import torch
    gd, wd = nets.build_det()
    gd = q.optimize(gd, wd)
    gc, wc = nets.build_cls()
    gc = q.optimize(gc, wc)
    gr, wr = nets.build_rec()
    gr = q.optimize(gr, wr)
    det = cuda_ctx.create_session(gd, wd, role="det", math="tf32", det_mask_exit=True)
    cls = cuda_ctx.create_session(gc, wc, role="cls", math="tf32")
    rec = cuda_ctx.create_session(gr, wr, role="rec", math="tf32")
    pipe = OcrPipeline(det, cls, rec, cls_batch=64, rec_batch=64)
    rng = np.random.Generator(np.random.PCG64(61))
    sizes = [4, 4, 3, 4]
    host = [rng.integers(0, 256, (n, H, W, 3), dtype=np.uint8) for n in sizes]
    boxes = [synthetic_boxes(n, K, H, W, seed=90 + i) for i, n in enumerate(sizes)]
    ref = [pipe.run(torch.from_numpy(h).cuda(), b) for h, b in zip(host, boxes)]
    up = torch.cuda.Stream()

    def batches():
        for h, b in zip(host, boxes):
            with torch.cuda.stream(up):
                t = torch.from_numpy(h).pin_memory().cuda(non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(up)
            yield t, b, ev

    got = list(pipe.run_many(batches()))
    assert len(got) == len(ref)
    for g, r in zip(got, ref):
        assert np.array_equal(g["mask"], r["mask"])
        assert np.array_equal(g["scores"].view(np.uint32), r["scores"].view(np.uint32))
        assert np.array_equal(g["probs"].view(np.uint32), r["probs"].view(np.uint32))
        assert np.array_equal(g["flips"], r["flips"])
        assert [list(x[0]) for x in g["results"]] == [list(x[0]) for x in r["results"]]
        assert np.array_equal(np.array([x[1] for x in g["results"]], np.float32).view(np.uint32),
                              np.array([x[1] for x in r["results"]], np.float32).view(np.uint32))
    for s_ in (det, cls, rec):
        s_.close()
