"""Device text-box post-processing and line preparation against the oracle's
restatements of the reference host code, bit for bit:
box_score_fast (geometry.rs:221-269), crop_text_box (crop.rs:8-127), and the
line pack (crop.rs:153-185) with cls_view windows (crop.rs:193-218) and the
180-degree flip of lines the classifier flags (engine.rs:1402-1407)."""
import numpy as np
import pytest

import oracle as orc
import qppocr_b200 as q

pytestmark = pytest.mark.gpu


def _quads(rng, n, h, w, tall=False):
    out = []
    for k in range(n):
        cx, cy = rng.uniform(-10, w + 10), rng.uniform(-10, h + 10)
        bw, bh = rng.uniform(2, 120), rng.uniform(2, 40)
        if tall and k % 3 == 0:
            bw, bh = bh, bw * 2
        a = 0.0 if k % 4 == 0 else rng.uniform(-0.5, 0.5)
        c, s = np.cos(a), np.sin(a)
        corners = np.array([[-bw, -bh], [bw, -bh], [bw, bh], [-bw, bh]]) / 2
        out.append(corners @ np.array([[c, s], [-s, c]]) + [cx, cy])
    # exact axis-aligned boxes on integer and half-integer corners
    out.append(np.array([[10, 20], [90, 20], [90, 60], [10, 60]], np.float64))
    out.append(np.array([[10.5, 20.5], [30.5, 20.5], [30.5, 22.5], [10.5, 22.5]], np.float64))
    return np.array(out, np.float32)


def test_box_score_bit_exact(cuda_ctx):
    import torch
    rng = np.random.Generator(np.random.PCG64(31))
    pred = rng.random((3, 240, 320), dtype=np.float32)
    boxes = _quads(rng, 150, 240, 320)
    img = rng.integers(0, 3, len(boxes)).astype(np.int32)
    got = q.op_box_score(torch.from_numpy(pred).cuda(), torch.from_numpy(boxes).cuda(),
                         torch.from_numpy(img).cuda())
    torch.cuda.synchronize()
    ref = orc.box_scores(pred, boxes, img)
    assert np.array_equal(got.cpu().numpy().view(np.uint32), ref.view(np.uint32))


def test_crop_text_boxes_bit_exact(cuda_ctx):
    import torch
    rng = np.random.Generator(np.random.PCG64(32))
    imgs = rng.integers(0, 256, (2, 240, 320, 3), dtype=np.uint8)
    pts = _quads(rng, 60, 240, 320, tall=True)
    img = rng.integers(0, 2, len(pts)).astype(np.int32)
    crops, off, cw, ch, rot = q.op_crop_text_boxes(torch.from_numpy(imgs).cuda(), pts, img)
    torch.cuda.synchronize()
    buf = crops.cpu().numpy()
    assert rot.any()
    for k in range(len(pts)):
        ref = orc.crop_text_box(imgs[img[k]], pts[k])
        got = buf[off[k]:off[k] + ref.size].reshape(ref.shape)
        assert np.array_equal(got, ref), k


@pytest.mark.parametrize("cls_h,cls_w", [(48, 192), (80, 160)])
def test_cls_pack_with_window_bit_exact(cuda_ctx, cls_h, cls_w):
    import torch
    rng = np.random.Generator(np.random.PCG64(33))
    crops = [rng.integers(0, 256, (int(rng.integers(8, 70)), int(rng.integers(4, 900)), 3), dtype=np.uint8)
             for _ in range(40)]
    flat = np.concatenate([c.ravel() for c in crops])
    off = np.cumsum([0] + [c.size for c in crops[:-1]]).astype(np.int64)
    hs = np.array([c.shape[0] for c in crops], np.int32)
    ws = np.array([c.shape[1] for c in crops], np.int32)
    # cls_view (crop.rs:193-218): centred window of h * cls_w / cls_h columns
    max_w = hs.astype(np.int64) * cls_w // cls_h
    vw = np.where(ws > max_w, np.maximum(1, max_w), ws).astype(np.int32)
    x0 = np.where(ws > max_w, (ws - vw) // 2, 0).astype(np.int32)
    ratio = vw.astype(np.float32) / hs.astype(np.float32)
    rw = np.clip(np.ceil(np.float32(cls_h) * ratio), 1, cls_w).astype(np.int32)
    assert (vw < ws).any()
    got = q.op_line_pack(torch.from_numpy(flat).cuda(), off, ws, x0, hs, vw, rw, np.zeros(len(crops), np.int32),
                         cls_h, cls_w)
    torch.cuda.synchronize()
    got = got.cpu().numpy()
    for k, c in enumerate(crops):
        ref = orc.cls_pack_line(c, cls_h, cls_w)
        assert np.array_equal(got[k].view(np.uint32), ref.view(np.uint32)), k


def test_rec_pack_flipped_lines_bit_exact(cuda_ctx):
    import torch
    rng = np.random.Generator(np.random.PCG64(34))
    crops = [rng.integers(0, 256, (int(rng.integers(20, 60)), int(rng.integers(10, 400)), 3), dtype=np.uint8)
             for _ in range(24)]
    flat = np.concatenate([c.ravel() for c in crops])
    off = np.cumsum([0] + [c.size for c in crops[:-1]]).astype(np.int64)
    hs = np.array([c.shape[0] for c in crops], np.int32)
    ws = np.array([c.shape[1] for c in crops], np.int32)
    rw = np.clip(np.ceil(np.float32(48) * (ws.astype(np.float32) / hs.astype(np.float32))), 1, 320).astype(np.int32)
    pad = (np.arange(len(crops)) % 5 == 0).astype(np.int32) * (hs <= 48)
    flip = (np.arange(len(crops)) % 2).astype(np.int32)
    got = q.op_line_pack(torch.from_numpy(flat).cuda(), off, ws, np.zeros(len(crops), np.int32), hs, ws, rw,
                         pad.astype(np.int32), 48, 320, flip=flip)
    torch.cuda.synchronize()
    got = got.cpu().numpy()
    for k, c in enumerate(crops):
        src = np.ascontiguousarray(c[::-1, ::-1]) if flip[k] else c
        ref = orc.rec_pack_line(src, int(rw[k]), 48, 320, pad=bool(pad[k]))
        assert np.array_equal(got[k].view(np.uint32), ref.view(np.uint32)), k
