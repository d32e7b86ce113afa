"""Host tests of the shared deterministic math (csrc/detmath.h) through the C oracle build."""
import numpy as np

import graph_ref


def test_exp_accuracy():
    lib = graph_ref.oracle_postproc()
    xs = np.concatenate([np.linspace(-87, 88, 20001, dtype=np.float32),
                         np.random.default_rng(0).uniform(-20, 20, 20000).astype(np.float32),
                         np.float32([0.0, -0.0, 1e-30, -1e-30, 0.5, -0.5])])
    got = np.array([lib.oref_exp(float(x)) for x in xs], np.float32)
    want = np.exp(xs.astype(np.float64))
    ulp = np.spacing(want.astype(np.float32)).astype(np.float64)
    err = np.abs(got.astype(np.float64) - want) / ulp
    assert err.max() <= 2.0, err.max()
    assert lib.oref_exp(-100.0) == 0.0
    assert np.isinf(lib.oref_exp(100.0))


def test_sigmoid_monotone_and_bounds():
    lib = graph_ref.oracle_postproc()
    xs = np.linspace(-30, 30, 4001, dtype=np.float32)
    s = np.array([lib.oref_sigmoid(float(x)) for x in xs])
    assert np.all(np.diff(s) >= 0) and s.min() >= 0 and s.max() <= 1
    ref = 1 / (1 + np.exp(-xs.astype(np.float64)))
    assert np.abs(s - ref).max() < 1e-6


def test_f2h_matches_numpy_rne():
    lib = graph_ref.oracle_postproc()
    rng = np.random.default_rng(1)
    xs = np.concatenate([rng.standard_normal(20000).astype(np.float32) * 10 ** rng.uniform(-8, 5, 20000).astype(np.float32),
                         np.float32([0, -0.0, 65504, 65519.9, 65520, 1e-8, 6e-8, 2.98e-8, 5.96e-8, np.inf, -np.inf])])
    got = np.array([lib.oref_f2h(float(x)) for x in xs], np.uint16)
    want = xs.astype(np.float16).view(np.uint16)
    assert np.array_equal(got, want)


def test_sincos_log_accuracy():
    """dm_sincos on the decode's angle range and beyond, dm_log over the normal range: within
    2 ulp (sin / cos: 2 ulp of 1 near zeros) of float64 libm."""
    lib = graph_ref.oracle_postproc()
    xs = np.linspace(-3.3, 3.3, 20001, dtype=np.float32)
    s = np.array([lib.oref_sin(float(x)) for x in xs], np.float64)
    c = np.array([lib.oref_cos(float(x)) for x in xs], np.float64)
    tol = 2 * np.spacing(np.float32(1.0))
    assert np.abs(s - np.sin(xs.astype(np.float64))).max() <= tol
    assert np.abs(c - np.cos(xs.astype(np.float64))).max() <= tol
    ys = np.exp(np.random.default_rng(2).uniform(-80, 80, 20000)).astype(np.float32)
    ys = np.concatenate([ys, np.float32([1.0, 0.5, 2.0, 1e-30, 3e38])])
    lg = np.array([lib.oref_log(float(y)) for y in ys], np.float64)
    want = np.log(ys.astype(np.float64))
    ulp = np.maximum(np.spacing(np.abs(want).astype(np.float32)).astype(np.float64), 1e-9)
    assert (np.abs(lg - want) / ulp).max() <= 2.0
    assert lib.oref_log(1.0) == 0.0


def test_probiou_properties():
    """probiou: 1 - O(sqrt(eps)) for identical boxes, symmetric, ~0 for far-apart boxes,
    unchanged by a pi rotation of either box."""
    import ctypes as C
    lib = graph_ref.oracle_postproc()

    def piou(a, b):
        a, b = np.float32(a), np.float32(b)
        return lib.oref_probiou(a.ctypes.data_as(C.c_void_p), b.ctypes.data_as(C.c_void_p))

    a = [100, 100, 40, 20, 0.3]
    assert piou(a, a) > 0.999
    b = [110, 95, 30, 25, -0.4]
    assert abs(piou(a, b) - piou(b, a)) < 1e-6
    assert piou(a, [900, 900, 40, 20, 0.3]) < 1e-3
    assert abs(piou(a, b) - piou([100, 100, 40, 20, 0.3 + np.pi], b)) < 1e-4


def _probiou64(a, b, eps=1e-7):
    """float64 restatement of ultralytics batch_probiou (Gaussian boxes: a = w^2/12,
    b = h^2/12 rotated by theta; Bhattacharyya distance clamped to [eps, 100])."""
    def cov(w, h, t):
        aa, bb = w * w / 12.0, h * h / 12.0
        c, s = np.cos(t), np.sin(t)
        return aa * c * c + bb * s * s, aa * s * s + bb * c * c, (aa - bb) * c * s
    a1, b1, c1 = cov(*a[2:5])
    a2, b2, c2 = cov(*b[2:5])
    x1, y1, x2, y2 = a[0], a[1], b[0], b[1]
    den = (a1 + a2) * (b1 + b2) - (c1 + c2) ** 2 + eps
    t1 = ((a1 + a2) * (y1 - y2) ** 2 + (b1 + b2) * (x1 - x2) ** 2) / den * 0.25
    t2 = ((c1 + c2) * (x2 - x1) * (y1 - y2)) / den * 0.5
    t3 = np.log(((a1 + a2) * (b1 + b2) - (c1 + c2) ** 2)
                / (4 * np.sqrt(max(a1 * b1 - c1 * c1, 0) * max(a2 * b2 - c2 * c2, 0)) + eps) + eps) * 0.5
    bd = min(max(t1 + t2 + t3, eps), 100.0)
    return 1 - np.sqrt(1 - np.exp(-bd) + eps)


def test_probiou_matches_float64_formula():
    """dm_probiou (explicitly rounded fp32) against the float64 formula on random pairs of
    overlapping boxes: absolute difference < 1e-4 (measured worst 8e-6)."""
    import ctypes as C
    lib = graph_ref.oracle_postproc()
    rng = np.random.default_rng(3)
    worst = 0.0
    for _ in range(3000):
        a = np.array([rng.uniform(0, 640), rng.uniform(0, 640), rng.uniform(4, 200),
                      rng.uniform(4, 200), rng.uniform(-0.785, 2.356)])
        b = a + np.array([rng.normal(0, 20), rng.normal(0, 20), rng.normal(0, 10),
                          rng.normal(0, 10), rng.normal(0, 0.3)])
        b[2:4] = np.abs(b[2:4]) + 1
        fa, fb = np.float32(a), np.float32(b)
        got = lib.oref_probiou(fa.ctypes.data_as(C.c_void_p), fb.ctypes.data_as(C.c_void_p))
        worst = max(worst, abs(got - _probiou64(fa.astype(np.float64), fb.astype(np.float64))))
    assert worst < 1e-4, worst


def test_div255_is_the_division():
    """dm_div255 (product + one Markstein correction, used by the letterbox kernel) equals
    v / 255 on [0, 256]: every 5th binary32 pattern of the range, and every pattern among the subnormals,
    near 1 and in [254, 256].  (An exhaustive pass over all 1.13e9 values of the range also
    found no mismatch.)"""
    lib = graph_ref.oracle_postproc()
    bits = lambda f: int(np.float32(f).view(np.uint32))
    assert lib.oref_div255_check(0, bits(256.0), 5) == 0
    for lo, hi in ((0.0, 2e-39), (0.999, 1.001), (254.0, 256.0)):
        assert lib.oref_div255_check(bits(lo), bits(hi), 1) == 0


def test_quot_gt_matches_division():
    """dm_quot_gt(a, b, t) (the division-free IoU threshold test of NMS) equals
    RN(a / b) > t: random quotients near and far from random thresholds and next to the
    midpoint between t and its successor, where the rounding decides."""
    lib = graph_ref.oracle_postproc()
    rng = np.random.default_rng(7)
    n = 400000
    t = rng.uniform(0, 1, n).astype(np.float32)
    t[:1000] = np.float32(0.7)
    t[1000:2000] = np.float32(0.45)
    t[2000:2100] = 0.0
    b = (rng.uniform(1, 1e5, n)).astype(np.float32)
    near = (t.astype(np.float64) * b * (1 + rng.uniform(-1e-6, 1e-6, n))).astype(np.float32)
    far = (b * rng.uniform(0, 1, n)).astype(np.float32)
    tp = (t.view(np.uint32) + 1).view(np.float32)
    mid = ((t.astype(np.float64) + tp) / 2 * b).astype(np.float32)   # near the midpoint
    for a in (near, far, mid, np.nextafter(mid, np.float32(np.inf)), np.nextafter(mid, np.float32(0))):
        a = np.ascontiguousarray(a, np.float32)
        got = np.zeros(n, np.int32)
        lib.oref_quot_gt(a.ctypes.data, b.ctypes.data, t.ctypes.data, n, got.ctypes.data)
        want = (a / b) > t
        assert np.array_equal(got.astype(bool), want)
    # an exact tie a / b == m cannot occur: m = t + ulp(t)/2 has a 25-bit odd significand,
    # so m * b needs more than the 24 bits a float a holds
