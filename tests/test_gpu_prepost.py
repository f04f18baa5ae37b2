"""Det / rec pre- and post-processing kernels against the oracle, bit-exact
(byte and f32 arithmetic of the reference's host code).  Inputs and sizes
follow the reference's own bit-exactness tests
(crates/qppocr-kernels/tests/rsz_par.rs:3-78)."""
import numpy as np
import pytest

import oracle as orc
import qppocr_b200 as q

pytestmark = pytest.mark.gpu


def dev(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def rsz_src(sw=848, sh=816, n=1, salt=0):
    i = np.arange(n * sw * sh * 3, dtype=np.int64)
    return ((i * 7919 + salt) % 256).astype(np.uint8).reshape(n, sh, sw, 3)


@pytest.mark.parametrize("dw,dh", [(832, 832), (400, 48), (960, 1216), (17, 33), (848, 816)])
def test_resize_bilinear_rgb_u8(cuda_ctx, dw, dh):
    src = rsz_src(n=2, salt=11)
    ref = orc.resize_bilinear_rgb_u8(src, dh, dw)
    got = q.op_resize_bilinear_rgb_u8(dev(src), dh, dw).cpu().numpy()
    assert np.array_equal(got, ref)


@pytest.mark.parametrize("sh,sw,dh,dw", [(96, 128, 96, 128), (300, 500, 224, 416), (61, 37, 64, 32)])
def test_det_preprocess(cuda_ctx, sh, sw, dh, dw):
    src = rsz_src(sw=sw, sh=sh, n=3, salt=5)
    img = src if (sh, sw) == (dh, dw) else orc.resize_bilinear_rgb_u8(src, dh, dw)
    ref = orc.det_normalize(img)
    got = q.op_det_preprocess(dev(src), dh, dw).cpu().numpy()
    assert got.shape == (3, 3, dh, dw)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


def ref_mask(h, w, n=1):
    # tests/rsz_par.rs:67-69: ((i * 2654435761) >> 24) as u8 % 3 (u64 arithmetic)
    i = np.arange(n * h * w, dtype=np.uint64)
    v = ((i * np.uint64(2654435761)) >> np.uint64(24)) & np.uint64(0xFF)
    return (v % np.uint64(3)).astype(np.uint8).reshape(n, h, w)


@pytest.mark.parametrize("h,w", [(832, 832), (37, 129), (1, 1), (5, 300), (300, 5)])
def test_dilate2x2(cuda_ctx, h, w):
    m = ref_mask(h, w, n=2)
    ref = orc.dilate2x2(m)
    got = q.op_db_mask(mask_in=dev(m), dilate=True).cpu().numpy()
    assert np.array_equal(got, ref)


@pytest.mark.parametrize("h,w,dilate", [(960, 960, True), (37, 129, True), (5, 300, False), (1, 1, True)])
def test_db_mask(cuda_ctx, h, w, dilate):
    rng = np.random.Generator(np.random.PCG64(3))
    pred = rng.uniform(0, 1, (2, h, w)).astype(np.float32)
    pred[0, 0, :min(w, 4)] = 0.3  # == thresh: not above it
    ref = orc.db_mask(pred, 0.3, dilate)
    got = q.op_db_mask(dev(pred), 0.3, dilate).cpu().numpy()
    assert np.array_equal(got, ref)


def test_session_u8_image_input(cuda_ctx):
    """A det session fed u8 HWC images (QPC_U8_IMAGE) normalises them on the
    device like the reference engine; outputs equal the f32 run on the
    oracle-normalised input, bit for bit (same plan after the first step)."""
    from qppocr_b200 import nets
    g, w = nets.build_det()
    g = q.optimize(g, w)
    s = cuda_ctx.create_session(g, w, role="det", math="3xtf32")
    img = rsz_src(sw=128, sh=96, n=2, salt=7)
    x = orc.det_normalize(img)
    ref = s.run({"x": x})[0]
    got = s.run({"x": img})[0]
    assert got.shape == ref.shape == (2, 1, 96, 128)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))
    d = s.run_deferred({"x": img})
    assert np.array_equal(d.complete()[0].view(np.uint32), ref.view(np.uint32))


def test_pinned_inputs_and_output_views(cuda_ctx):
    """Inputs in library-pinned host memory (qpc_host_alloc) go to the device by
    DMA straight from the caller's buffer; complete(copy=False) returns
    read-only views of the run's pinned outputs.  Both give the bytes of the
    staged / copied path; the plan instance held by the views is reused once
    they are dropped."""
    from qppocr_b200 import nets
    g, w = nets.build_det()
    g = q.optimize(g, w)
    s = cuda_ctx.create_session(g, w, role="det", math="3xtf32")
    img = rsz_src(sw=128, sh=96, n=2, salt=9)
    ref = s.run({"x": img})[0]
    pin = q.host_empty(img.shape, np.uint8)
    pin[...] = img
    a = s.run_deferred({"x": pin})
    b = s.run_deferred({"x": pin})
    va = a.complete(copy=False)[0]
    vb = b.complete(copy=False)[0]
    assert not va.flags.writeable
    assert np.array_equal(va.view(np.uint32), ref.view(np.uint32))
    assert np.array_equal(vb.view(np.uint32), ref.view(np.uint32))
    del va, vb, a, b
    x = orc.det_normalize(img)
    xf = q.host_empty(x.shape, np.float32)
    xf[...] = x
    for _ in range(3):
        got = s.run({"x": xf})[0]
        assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))
