"""CPU: the logit interval of the fused decode (decode.cu, dec_interval) holds
the reference's sequential chain.

The reference's logit is acc = RN(acc + RN(x_j * w_j)), j = 0..D-1 in order,
then RN(acc * s) for an int8 router and RN(logit + bias) with a router bias
(engines/olmoe.c:74-85, engines/qwen.c:116-121; the bias is this library's).
The decode kernel streams the experts' weights as soon as intervals on those
logits decide the top-k set, so an interval that misses the chain's value
could select the wrong experts.  This test restates the interval's arithmetic
(double sums of the same rounded products and of the absolute prefix sums,
then the bound u * sum|S_j| * (1 + 2Du) + (D + 64) 2^-52 sum|p| terms, with
every bound step rounded outwards) and checks it against the chain on inputs
chosen to stress it: cancellation, prefix sums that climb and fall back,
magnitudes from 1e-20 to 1e20, subnormal products, a negative row scale.
"""
import numpy as np
import pytest

F32 = np.float32
INF = np.inf


def _up(x):
    return np.nextafter(x, INF)


def _down(x):
    return np.nextafter(x, -INF)


def _f32_rd(x):
    """Largest float32 <= x (x float64 array)."""
    f = x.astype(F32)
    over = f.astype(np.float64) > x
    f[over] = np.nextafter(f[over], F32(-INF))
    return f


def _f32_ru(x):
    f = x.astype(F32)
    under = f.astype(np.float64) < x
    f[under] = np.nextafter(f[under], F32(INF))
    return f


def chain(x, w):
    """The reference's fp32 chain for every row pair: x, w [n][D] float32."""
    acc = np.zeros(x.shape[0], dtype=F32)
    for j in range(x.shape[1]):
        acc = (acc + (x[:, j] * w[:, j]).astype(F32)).astype(F32)
    return acc


def interval(x, w, scale=None, bias=None):
    """The interval the decode kernel publishes, restated: [lo, hi] float32."""
    n, D = x.shape
    p = (x * w).astype(F32)                      # the chain's rounded products
    pd = p.astype(np.float64)
    c = np.zeros(n)                               # double sum (any order is covered by em)
    B = np.zeros(n)                               # sum_j |S_j| of the double prefix sums, rounded up
    P = np.zeros(n, dtype=F32)                    # sum_j |p_j| in float32, rounded up
    for j in range(D):
        c = c + pd[:, j]
        B = _up(B + np.abs(c))
        P = np.nextafter((P + np.abs(p[:, j])).astype(F32), F32(INF))
    u = 2.0 ** -24
    Pd = P.astype(np.float64)
    em = _up(_up((D + 64.0) * 2.0 ** -52) * Pd)
    Bp = _up(B + _up(D * em))
    beta = _up(_up(u * Bp) * _up(1.0 + _up(2.0 * D * u)))
    beta = _up(_up(beta + em) + _up(D * 2.0 ** -150))
    lo = _f32_rd(_down(c - beta))
    hi = _f32_ru(_up(c + beta))
    if scale is not None:
        s = scale.astype(np.float64)
        a, b = lo.astype(np.float64) * s, hi.astype(np.float64) * s   # exact in double
        lo, hi = _f32_rd(np.minimum(a, b)), _f32_ru(np.maximum(a, b))
    if bias is not None:
        bb = bias.astype(np.float64)
        lo = _f32_rd(_down(lo.astype(np.float64) + bb))
        hi = _f32_ru(_up(hi.astype(np.float64) + bb))
    return lo, hi


def logit(x, w, scale=None, bias=None):
    v = chain(x, w)
    if scale is not None:
        v = (v * scale).astype(F32)
    if bias is not None:
        v = (v + bias).astype(F32)
    return v


def _check(x, w, scale=None, bias=None):
    v = logit(x, w, scale, bias)
    lo, hi = interval(x, w, scale, bias)
    bad = ~((lo <= v) & (v <= hi))
    assert not bad.any(), (np.nonzero(bad)[0][:5], v[bad][:5], lo[bad][:5], hi[bad][:5])
    return v, lo, hi


D = 2048


def test_random_router_rows_are_inside_and_tight():
    rng = np.random.default_rng(1)
    x = rng.standard_normal((64, D)).astype(F32)
    w = (rng.standard_normal((64, D)) * 0.02).astype(F32)
    v, lo, hi = _check(x, w)
    # the interval is narrow next to the logits' spread (~0.9): a set is
    # undecided only when two logits lie within about this of each other
    assert float(np.max(hi - lo)) < 5e-4


@pytest.mark.parametrize("kind", ["alternating", "climb_and_fall", "wide_magnitudes", "subnormal"])
def test_adversarial_rows_are_inside(kind):
    rng = np.random.default_rng(hash(kind) % 2**32)
    n = 48
    if kind == "alternating":
        # products +a, -a, ... with small noise: prefix sums swing every step
        a = rng.uniform(1.0, 1e4, (n, 1))
        sgn = np.where(np.arange(D) % 2 == 0, 1.0, -1.0)[None, :]
        x = (a * sgn * (1 + 1e-3 * rng.standard_normal((n, D)))).astype(F32)
        w = np.ones((n, D), dtype=F32)
    elif kind == "climb_and_fall":
        # the prefix sums climb for half the row and come back: the chain's
        # rounding errors accumulate on large partial sums of a small result
        x = np.concatenate([rng.uniform(0.5, 1.5, (n, D // 2)), -rng.uniform(0.5, 1.5, (n, D // 2))], axis=1)
        x = (x * 1e3).astype(F32)
        w = (1 + 1e-2 * rng.standard_normal((n, D))).astype(F32)
    elif kind == "wide_magnitudes":
        x = (np.exp(rng.uniform(np.log(1e-20), np.log(1e20), (n, D))) *
             rng.choice([-1.0, 1.0], (n, D))).astype(F32)
        w = rng.standard_normal((n, D)).astype(F32)
    else:
        # products around 1e-42: subnormal partial sums
        x = (rng.standard_normal((n, D)) * 1e-21).astype(F32)
        w = (rng.standard_normal((n, D)) * 1e-21).astype(F32)
    _check(x, w)


def test_int8_rows_with_scale_of_either_sign_and_bias():
    rng = np.random.default_rng(7)
    n = 64
    x = rng.standard_normal((n, D)).astype(F32)
    w = rng.integers(-127, 128, (n, D)).astype(F32)
    scale = (rng.uniform(1e-4, 1e-3, n) * rng.choice([-1.0, 1.0], n)).astype(F32)
    bias = rng.standard_normal(n).astype(F32)
    _check(x, w, scale, bias)
