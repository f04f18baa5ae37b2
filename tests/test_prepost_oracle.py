"""CPU checks of the oracle's restatements of the det / rec host code: the
2x2 dilation against the reference test's scalar triple loop
(crates/qppocr-kernels/tests/rsz_par.rs:51-66), the det normalisation against
its f32 formula (engine.rs:963-982), the bilinear resize's identity case, and
greedy CTC decoding (rec.rs:34-79) on hand-made rows."""
import numpy as np

import oracle as orc


def scalar_dilate(m):
    h, w = m.shape
    d = np.zeros_like(m)
    for y in range(h):
        for x in range(w):
            v = 0
            for dy in (-1, 0):
                for dx in (-1, 0):
                    ny, nx = y + dy, x + dx
                    if 0 <= ny < h and 0 <= nx < w:
                        v = max(v, int(m[ny, nx]))
            d[y, x] = v
    return d


def test_dilate_matches_scalar_loop():
    for h, w in ((37, 129), (1, 1), (5, 30), (30, 5)):
        i = np.arange(h * w, dtype=np.uint64)
        m = ((((i * np.uint64(2654435761)) >> np.uint64(24)) & np.uint64(0xFF)) % np.uint64(3)).astype(np.uint8)
        m = m.reshape(h, w)
        assert np.array_equal(orc.dilate2x2(m[None])[0], scalar_dilate(m))


def test_det_normalize_formula():
    img = np.arange(256, dtype=np.uint8).reshape(1, 16, 16, 1).repeat(3, axis=3)
    got = orc.det_normalize(img)
    scale, mean, istd = np.float32(1.0) / np.float32(255.0), np.float32(0.5), np.float32(1.0) / np.float32(0.5)
    v = img.astype(np.float32) * scale
    ref = ((v - mean) * istd).transpose(0, 3, 1, 2)
    assert np.array_equal(got.view(np.uint32), ref.astype(np.float32).view(np.uint32))


def test_resize_identity_is_copy():
    i = np.arange(2 * 20 * 30 * 3, dtype=np.int64)
    src = ((i * 7919) % 256).astype(np.uint8).reshape(2, 20, 30, 3)
    assert np.array_equal(orc.resize_bilinear_rgb_u8(src, 20, 30), src)


def test_ctc_decode_greedy():
    # blank = 0; repeats collapse; a blank separates repeats; conf = mean of emitted
    rows = [[0.9, 0.1, 0.0], [0.1, 0.8, 0.1], [0.1, 0.7, 0.2], [0.6, 0.3, 0.1], [0.2, 0.6, 0.2], [0.1, 0.2, 0.7]]
    idx, conf = orc.ctc_decode(np.array(rows, np.float32))
    assert idx == [1, 1, 2]
    assert conf == np.float32((0.8 + 0.6 + 0.7) / 3)
    # ties keep the lowest index
    idx, _ = orc.ctc_decode(np.array([[0.2, 0.4, 0.4]], np.float32))
    assert idx == [1]


def test_crop_size_host_helper_matches_oracle():
    """qpc_crop_size (host code in the library) against the oracle's
    restatement of crop.rs:9-15, including tall boxes that rotate."""
    import qppocr_b200 as q
    rng = np.random.Generator(np.random.PCG64(12))
    pts = []
    for _ in range(200):
        cx, cy = rng.uniform(0, 500, 2)
        w, h = rng.uniform(1, 300), rng.uniform(1, 300)
        a = rng.uniform(-0.6, 0.6)
        c, s = np.cos(a), np.sin(a)
        corners = np.array([[-w, -h], [w, -h], [w, h], [-w, h]]) / 2
        pts.append(corners @ np.array([[c, s], [-s, c]]) + [cx, cy])
    pts = np.array(pts, np.float32)
    cw, ch, rot = q.crop_size(pts)
    for k in range(len(pts)):
        assert (cw[k], ch[k], bool(rot[k])) == orc.crop_size(pts[k])
    assert rot.any() and not rot.all()
