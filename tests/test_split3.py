"""The fp32 path's tensor-core attention splits every fp32 operand into three
bf16 parts (hi = rn(x), mid = rn(x - hi), lo = rn(x - hi - mid)) and sums
six part products.  These CPU checks pin the arithmetic that relies on: both
differences are exact in fp32, the parts reproduce x to fp32 precision, and
the six kept products of order <= 2 leave an error below 2^-22 of |a*b|.
bf16 round-to-nearest-even is restated on the float32 bit patterns."""
import numpy as np


def bf16_rn(x: np.ndarray) -> np.ndarray:
    """float32 -> nearest bf16 (ties to even), returned as float32."""
    b = x.astype(np.float32).view(np.uint32).astype(np.uint64)
    b = (b + 0x7FFF + ((b >> 16) & 1)) & 0xFFFF0000
    return b.astype(np.uint32).view(np.float32)


def split3(x: np.ndarray):
    x = x.astype(np.float32)
    hi = bf16_rn(x)
    r = (x - hi).astype(np.float32)
    mid = bf16_rn(r)
    lo = bf16_rn((r - mid).astype(np.float32))
    return hi, r, mid, lo


def _samples(n=200_000, seed=7):
    g = np.random.default_rng(seed)
    x = g.standard_normal(n) * np.exp2(g.integers(-20, 20, n))
    return x.astype(np.float32)


def test_differences_are_exact():
    x = _samples()
    hi, r, mid, _ = split3(x)
    # fp32 results equal the exact (float64) differences
    assert np.array_equal(r.astype(np.float64), x.astype(np.float64) - hi.astype(np.float64))
    r2 = (r - mid).astype(np.float32)
    assert np.array_equal(r2.astype(np.float64), r.astype(np.float64) - mid.astype(np.float64))


def test_parts_reproduce_fp32():
    x = _samples()
    hi, _, mid, lo = split3(x)
    s = hi.astype(np.float64) + mid.astype(np.float64) + lo.astype(np.float64)
    err = np.abs(s - x.astype(np.float64)) / np.abs(x.astype(np.float64))
    assert err.max() <= 2.0 ** -24, err.max()


def test_six_products_match_the_fp32_product():
    x, y = _samples(seed=1), _samples(seed=2)
    xp, yp = split3(x), split3(y)
    px = [xp[0], xp[2], xp[3]]
    py = [yp[0], yp[2], yp[3]]
    terms = [(1, 1), (2, 0), (0, 2), (1, 0), (0, 1), (0, 0)]
    acc = np.zeros(x.shape, np.float64)
    for a, b in terms:
        acc += px[a].astype(np.float64) * py[b].astype(np.float64)
    exact = x.astype(np.float64) * y.astype(np.float64)
    rel = np.abs(acc - exact) / np.abs(exact)
    assert rel.max() <= 2.0 ** -22, rel.max()
