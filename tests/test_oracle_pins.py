"""Pins the CPU oracle to the reference's own known answers.

* activation.rs:472-513 — erf known values (|err| < 5e-7), exp relative error
  < 1e-5 over [-80, 80] step 0.07, +/-88 saturation, erf odd symmetry bit for bit.
* tests/kernels.rs:51-1467 — every conv case of the reference's table and the
  other op tests, against naive f64 references, with the reference's check
  max|d| / max|ref| < 1e-5, inputs from the reference's xorshift64* RNG
  (kernels.rs:30-48, seed 0x243F6A8885A308D3).
"""
import numpy as np
import pytest

import oracle as orc

SEED = 0x243F6A8885A308D3


class Rng:
    def __init__(self):
        self.state = SEED

    def fill(self, shape):
        n = int(np.prod(shape))
        v, self.state = orc.xorshift_fill(self.state, n)
        return v.reshape(shape)


def check(name, got, ref, tol=1e-5):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    assert got.shape == ref.shape, (name, got.shape, ref.shape)
    d = np.abs(got - ref).max() if got.size else 0.0
    scale = max(np.abs(ref).max() if ref.size else 0.0, 1e-6)
    assert d / scale < tol, f"{name}: max diff {d:.3e} (rel {d / scale:.1e})"


def test_xorshift_range_and_determinism():
    a, s1 = orc.xorshift_fill(SEED, 1000)
    b, s2 = orc.xorshift_fill(SEED, 1000)
    assert s1 == s2 and np.array_equal(a, b)
    assert a.min() >= -1.0 and a.max() < 1.0
    # xorshift64* reference computation in Python for the first values
    s = SEED
    for k in range(16):
        s ^= s >> 12
        s ^= (s << 25) & 0xFFFFFFFFFFFFFFFF
        s ^= s >> 27
        v = (s * 0x2545F4914F6CDD1D) & 0xFFFFFFFFFFFFFFFF
        expect = np.float32(((v >> 40) - (1 << 23)) / float(1 << 23))
        assert a[k] == expect


def test_erf_known_values():
    known = [(0.0, 0.0), (0.1, 0.1124629160182849), (0.25, 0.2763263901682369),
             (0.5, 0.5204998778130465), (1.0, 0.8427007929497149), (1.5, 0.9661051464753108),
             (2.0, 0.9953222650189527), (3.0, 0.9999779095030014), (4.0, 0.9999999845827421),
             (6.0, 0.9999999999984626)]
    x = np.array([k for k, _ in known], np.float32)
    got = orc.erf1(x)
    for g, (xv, r) in zip(got, known):
        assert abs(float(g) - r) < 5e-7, (xv, g, r)


def test_exp_polynomial_accuracy_and_saturation():
    x = np.float32(-80.0) + np.arange(0, 2286, dtype=np.float32) * np.float32(0.07)
    x = x[x <= 80.0]
    # the reference steps x += 0.07 in f32; reproduce that accumulation
    xs = [np.float32(-80.0)]
    while True:
        nx = np.float32(xs[-1] + np.float32(0.07))
        if nx > 80.0:
            break
        xs.append(nx)
    x = np.array(xs, np.float32)
    got = orc.exp1(x).astype(np.float64)
    ref = np.exp(x.astype(np.float64))
    rel = np.abs(got - ref) / np.maximum(ref, 1e-30)
    assert rel.max() < 1e-5
    sat = orc.exp1(np.array([100.0, 88.0, -100.0, -88.0], np.float32))
    assert sat[0] == sat[1] and sat[2] == sat[3]


def test_erf_odd_bitwise():
    v = np.array([0.5, -1.25, 3.75, -5.5, 0.0], np.float32)
    a = orc.erf1(-v).view(np.uint32)
    b = (-orc.erf1(v)).view(np.uint32)
    assert np.array_equal(a, b)


def ref_conv(x, w, bias, sh, sw, ph, pw, group):
    """Naive NCHW conv in f64 (kernels.rs:94-143)."""
    x = x.astype(np.float64)
    w = w.astype(np.float64)
    n, c, h, wd = x.shape
    m, cg, kh, kw = w.shape
    oh = (h + 2 * ph - kh) // sh + 1
    ow = (wd + 2 * pw - kw) // sw + 1
    xp = np.zeros((n, c, h + 2 * ph + kh, wd + 2 * pw + kw))
    xp[:, :, ph:ph + h, pw:pw + wd] = x
    mg = m // group
    y = np.zeros((n, m, oh, ow))
    for mm in range(m):
        g = mm // mg
        for ch in range(cg):
            ci = g * cg + ch
            for ky in range(kh):
                for kx in range(kw):
                    patch = xp[:, ci, ky:ky + sh * oh:sh, kx:kx + sw * ow:sw][:, :oh, :ow]
                    y[:, mm] += w[mm, ch, ky, kx] * patch
        if bias is not None:
            y[:, mm] += bias[mm]
    return y


# The reference's conv case table (tests/kernels.rs:163-592):
# (name, n, c, m, h, w, kh, kw, sh, sw, ph, pw, group, bias)
CONV_CASES = [
    ("1x1 conv (gemm path)", 1, 16, 24, 32, 32, 1, 1, 1, 1, 0, 0, 1, True),
    ("3x3 s1 p1", 1, 3, 16, 64, 64, 3, 3, 1, 1, 1, 1, 1, True),
    ("3x3 s2 p1", 1, 3, 16, 65, 65, 3, 3, 2, 2, 1, 1, 1, True),
    ("5x5 s1 p2", 1, 8, 16, 33, 33, 5, 5, 1, 1, 2, 2, 1, False),
    ("5x5 s2 p2", 1, 8, 16, 64, 64, 5, 5, 2, 2, 2, 2, 1, True),
    ("depthwise 3x3 s1 p1", 1, 16, 16, 64, 64, 3, 3, 1, 1, 1, 1, 16, True),
    ("depthwise 3x3 s1 p1 on 1x1", 1, 4, 4, 1, 1, 3, 3, 1, 1, 1, 1, 4, False),
    ("depthwise 3x3 s2 p1", 1, 32, 32, 65, 65, 3, 3, 2, 2, 1, 1, 32, True),
    ("depthwise 5x5 s1 p2", 1, 24, 24, 40, 40, 5, 5, 1, 1, 2, 2, 24, True),
    ("depthwise 5x5 s2 p2", 1, 24, 24, 40, 40, 5, 5, 2, 2, 2, 2, 24, False),
    ("depthwise 3x3 s[1,2] p1", 1, 32, 32, 40, 40, 3, 3, 1, 2, 1, 1, 32, True),
    ("depthwise 3x3 s[2,1] p1", 1, 32, 32, 40, 40, 3, 3, 2, 1, 1, 1, 32, True),
    ("depthwise 5x5 s[1,2] p2", 1, 24, 24, 40, 40, 5, 5, 1, 2, 2, 2, 24, True),
    ("3x3 s[1,2] p1", 1, 8, 16, 40, 40, 3, 3, 1, 2, 1, 1, 1, True),
    ("3x3 s[2,1] p1", 1, 8, 16, 40, 40, 3, 3, 2, 1, 1, 1, 1, True),
    ("depthwise 7x7 s1 p3", 1, 32, 32, 40, 40, 7, 7, 1, 1, 3, 3, 32, True),
    ("depthwise 7x7 s2 p3", 1, 32, 32, 40, 40, 7, 7, 2, 2, 3, 3, 32, True),
    ("grouped g=4", 1, 16, 24, 32, 32, 3, 3, 1, 1, 1, 1, 4, True),
    ("grouped g=2 5x5 s2", 1, 6, 12, 33, 33, 5, 5, 2, 2, 2, 2, 2, True),
    ("batch=2 3x3", 2, 8, 16, 24, 24, 3, 3, 1, 1, 1, 1, 1, True),
    ("M=17 N=713 (tail rows)", 1, 8, 17, 30, 24, 1, 1, 1, 1, 0, 0, 1, True),
    ("M=3 3x3 (all tail)", 1, 4, 3, 16, 16, 3, 3, 1, 1, 1, 1, 1, True),
]


def test_conv2d_reference_cases():
    rng = Rng()
    for (name, n, c, m, h, w, kh, kw, sh, sw, ph, pw, g, has_b) in CONV_CASES:
        x = rng.fill((n, c, h, w))
        wt = rng.fill((m, c // g, kh, kw))
        b = rng.fill((m,))
        bias = b if has_b else None
        got = orc.conv2d(x, wt, bias, (sh, sw), (ph, pw, ph, pw), g)
        check(name, got, ref_conv(x, wt, bias, sh, sw, ph, pw, g))


def test_conv2d_activation_and_residual_order():
    # act (relu) then + residual, executor.rs:459-475 / gemm.rs:478-507
    rng = Rng()
    x = rng.fill((1, 8, 20, 20))
    w = rng.fill((12, 8, 1, 1))
    b = rng.fill((12,))
    r = rng.fill((1, 12, 20, 20))
    got = orc.conv2d(x, w, b, act=2, residual=r)
    ref = np.maximum(ref_conv(x, w, b, 1, 1, 0, 0, 1), 0) + r
    check("1x1 relu+res", got, ref)
    w3 = rng.fill((12, 8, 3, 3))
    got = orc.conv2d(x, w3, b, pads=(1, 1, 1, 1), act=2, residual=r)
    check("3x3 relu+res", got, np.maximum(ref_conv(x, w3, b, 1, 1, 1, 1, 1), 0) + r)


def test_depthwise_nhwc_matches_nchw_path():
    rng = Rng()
    x = rng.fill((2, 9, 11, 16))
    w = rng.fill((16, 1, 3, 3))
    b = rng.fill((16,))
    nchw = orc.conv2d(np.transpose(x, (0, 3, 1, 2)), w, b, (1, 1), (1, 1, 1, 1), 16)
    wt = np.ascontiguousarray(w.reshape(16, 9).T)
    nhwc = orc.depthwise_nhwc(x, wt, 3, 3, (1, 1), (1, 1, 1, 1), b)
    check("dw nhwc", np.transpose(nhwc, (0, 3, 1, 2)), nchw, 1e-6)


def test_sgemm_vs_f64():
    rng = Rng()
    for (m, n, k) in [(1, 1, 1), (4, 32, 7), (17, 713, 8), (5, 33, 64), (64, 48, 100)]:
        a = rng.fill((m, k))
        b = rng.fill((k, n))
        bias = rng.fill((m,))
        check(f"sgemm {m}x{n}x{k}", orc.sgemm(a, b, bias), a.astype(np.float64) @ b + bias[:, None].astype(np.float64))


def test_conv1x1_nhwc_vs_f64():
    rng = Rng()
    x = rng.fill((300, 24))
    wt = rng.fill((24, 40))
    b = rng.fill((40,))
    check("conv1x1_nhwc", orc.conv1x1_nhwc(x, wt, b), x.astype(np.float64) @ wt + b)


def test_softmax_vs_f64():
    rng = Rng()
    for shape in [(7, 3), (5, 8), (4, 40), (3, 18709)]:
        x = rng.fill(shape) * 10
        e = np.exp(x.astype(np.float64) - x.max(-1, keepdims=True))
        check(f"softmax {shape}", orc.softmax_last(x), e / e.sum(-1, keepdims=True))


def test_convtranspose_vs_naive():
    rng = Rng()
    x = rng.fill((2, 6, 5, 7))
    w = rng.fill((6, 4, 2, 2))
    ref = np.zeros((2, 4, 10, 14))
    for ky in range(2):
        for kx in range(2):
            ref[:, :, ky::2, kx::2] = np.einsum("nchw,cm->nmhw", x.astype(np.float64), w[:, :, ky, kx])
    check("convT", orc.convtranspose2d(x, w), ref)


def test_pools_reduce_bn_resize_matmul():
    rng = Rng()
    x = rng.fill((2, 5, 9, 8))
    check("gap", orc.global_avg_pool(x), x.astype(np.float64).mean((2, 3), keepdims=True))
    check("avgpool 3x1", orc.pool2d(x, 3, 1, 3, 1, 0, 0, 0, 0, False),
          x[:, :, :9].astype(np.float64).reshape(2, 5, 3, 3, 8).mean(3))
    mx = orc.pool2d(x, 2, 2, 2, 2, 0, 0, 0, 0, True)
    check("maxpool", mx, x.reshape(2, 5, 4, 2, 4, 2)[:, :, :, :, :, :].max((3, 5)) if False else
          x[:, :, :8, :8].reshape(2, 5, 4, 2, 4, 2).max((3, 5)))
    check("reduce_mean", orc.reduce_mean(x, 10, 72, 1), x.astype(np.float64).reshape(10, 72).mean(1))
    sc, bi, me, va = rng.fill((5,)) + 1.5, rng.fill((5,)), rng.fill((5,)), rng.fill((5,)) + 1.5
    a = sc.astype(np.float64) / np.sqrt(va.astype(np.float64) + 1e-5)
    check("batchnorm", orc.batchnorm(x, sc, bi, me, va),
          (x - me[None, :, None, None]) * a[None, :, None, None] + bi[None, :, None, None])
    up = orc.resize_nearest(x, 18, 16)
    assert np.array_equal(up, x.repeat(2, 2).repeat(2, 3))
    q = rng.fill((3, 4, 7, 5))
    k = rng.fill((3, 4, 5, 6))
    check("matmul", orc.matmul(q, k), q.astype(np.float64) @ k)


def test_argmax_first_strict_max():
    p = np.array([[0.1, 0.5, 0.5, 0.2], [0.9, 0.0, 0.9, 0.9]], np.float32)
    pr = orc.argmax_pairs(p)
    assert pr[0, 0] == np.float32(0.5) and pr[0, 1].view(np.uint32) == 1
    assert pr[1, 1].view(np.uint32) == 0
