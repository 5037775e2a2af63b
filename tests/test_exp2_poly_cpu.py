"""The degree-3 polynomial the attention kernel uses for 2^f on the FMA pipe
(exp2_poly2 in ipu-stack_b200/csrc/sm100.cuh): a near-minimax relative-error
fit of 2^f on [-0.5, 0.5] by Lawson's iteratively reweighted least squares.
Re-derives the fit here and checks the kernel's coefficients against it and
against the error bound the kernel relies on (below half an f16 ulp, 2^-11)."""
import re
import os

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def kernel_coefficients():
    src = open(os.path.join(ROOT, "ipu-stack_b200", "csrc", "sm100.cuh")).read()
    body = src[src.index("uint64_t exp2_poly2("):]
    body = body[:body.index("\n}\n")]
    vals = [float(v) for v in re.findall(r"f2_pack\((0\.\d+)f, \1f\)", body)]
    c3, c2, c1, c0 = vals  # Horner order in the kernel: ((c3 f + c2) f + c1) f + c0
    return np.array([c0, c1, c2, c3])


def test_coefficients_are_the_lawson_minimax_fit():
    f = np.linspace(-0.5, 0.5, 4001)
    # rows scaled by 1/2^f: the residual A c - 1 is the relative error
    A = np.stack([f ** i for i in range(4)], axis=1) / np.exp2(f)[:, None]
    w = np.full_like(f, 1.0 / len(f))
    for _ in range(300):  # Lawson: reweight by |error| until the fit equioscillates
        sw = np.sqrt(w)
        fit, *_ = np.linalg.lstsq(A * sw[:, None], sw, rcond=None)
        w = w * np.abs(A @ fit - 1.0)
        w /= w.sum()
    assert np.allclose(kernel_coefficients(), fit, atol=5e-6)


def test_relative_error_below_half_an_f16_ulp():
    c = kernel_coefficients()
    f = np.linspace(-0.5, 0.5, 200001)
    p = ((c[3] * f + c[2]) * f + c[1]) * f + c[0]
    rel = np.abs(p / np.exp2(f) - 1.0).max()
    assert rel <= 7.6e-5 < 2.0 ** -11
