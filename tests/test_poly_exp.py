"""The FMA-pipe 2^x of the attention softmax (ex2_poly2 in k_awa_tc.cu,
off by default) evaluates a cubic on f in [-1/2, 1/2].  Its coefficients
come from a relative least-squares fit of 2^f on 64 Chebyshev nodes; this
test redoes the fit and checks the constants in the kernel source and the
stated error bound (7.7e-5, below bf16's 2^-9 rounding of P)."""
import os
import re

import numpy as np

SRC = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "seedvr2-2b-ncnn_b200", "csrc",
                   "k_awa_tc.cu")


def kernel_coefficients():
    src = open(SRC).read()
    body = src[src.index("void ex2_poly2("):]
    body = body[:body.index("\n}\n")]
    vals = [float(v) for v in re.findall(r"f2pack\(([0-9.]+)f, \1f\)", body) if v not in ("12582912.",)]
    # c3, c2 (first ffma2), c1, c0
    return vals


def test_cubic_is_the_chebyshev_least_squares_fit():
    c3, c2, c1, c0 = kernel_coefficients()
    n = 64
    k = np.arange(n)
    x = 0.5 * np.cos((2 * k + 1) * np.pi / (2 * n))
    A = np.stack([x ** i for i in range(4)], 1) / np.exp2(x)[:, None]
    fit, *_ = np.linalg.lstsq(A, np.ones(n), rcond=None)
    np.testing.assert_allclose([c0, c1, c2, c3], fit, rtol=1e-6)
    f = np.linspace(-0.5, 0.5, 100001)
    p = c0 + f * (c1 + f * (c2 + f * c3))
    assert np.abs(p / np.exp2(f) - 1).max() < 7.8e-5
