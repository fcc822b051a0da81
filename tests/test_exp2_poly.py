"""Provenance of the FMA-pipe exp2 polynomial of the tensor-core epilogues.

2^x = 2^j * 2^f with j = round(x), f = x - j in [-1/2, 1/2] (Cody-Waite style
range reduction; j goes into the exponent field).  2^f is approximated by a
polynomial p(f) with p(0) = 1 chosen to minimise the maximum RELATIVE error on
[-1/2, 1/2] (Remez exchange on the weighted error (p(f) - 2^f) / 2^f).  This
test refits the degree-4 polynomial, compares it with the coefficients
compiled into flashdiffusion_b200/csrc/fd_tc_common.cuh (exp2_poly2), and
re-measures the error of those fp32 coefficients in fp32 Horner arithmetic
(the device evaluation order).  CPU only; the device implementation is held
to the same bound in tests/test_gpu_exp2.py.
"""
import os
import re

import numpy as np

HDR = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                   "flashdiffusion_b200", "csrc", "fd_tc_common.cuh")
BOUND = 3.7e-6   # fp32 Horner relative error of the fitted degree-4 coefficients


def remez_rel(deg, iters=40):
    n = deg + 1                                     # reference points (c0 fixed to 1)
    x = 0.5 * np.cos(np.pi * np.arange(n)[::-1] / (n - 1))
    g = np.linspace(-0.5, 0.5, 200001)
    for _ in range(iters):
        t = 2.0 ** x
        A = np.column_stack([x ** k for k in range(1, deg + 1)] + [((-1.0) ** np.arange(n)) * t])
        sol = np.linalg.solve(A, t - 1.0)
        c = np.concatenate([[1.0], sol[:deg]])
        err = (np.polyval(c[::-1], g) - 2.0 ** g) / 2.0 ** g
        d = np.diff(err)
        ext = np.concatenate([[0], np.nonzero(d[:-1] * d[1:] <= 0)[0] + 1, [len(g) - 1]])
        pts = np.sort(ext[np.argsort(-np.abs(err[ext]))[:n]])
        x = g[pts]
    return c


def fp32_horner_error(c):
    c32 = np.asarray(c, dtype=np.float32)
    g = np.linspace(-0.5, 0.5, 400001).astype(np.float32)
    p = np.full_like(g, c32[-1])
    for ck in c32[-2::-1]:
        p = (p * g + ck).astype(np.float32)
    ref = 2.0 ** g.astype(np.float64)
    return float(np.max(np.abs(p.astype(np.float64) - ref) / ref))


def compiled_coefficients():
    src = open(HDR).read()
    body = src[src.index("uint64_t exp2_poly2"):]
    body = body[:body.index("unpack2")]
    vals = [float(v) for v in re.findall(r"pack2\(([0-9.eE+-]+)f,", body)]
    coef = [v for v in vals if v != 12582912.0]     # drop the range-reduction shift
    assert len(coef) == 5, coef
    c4, c3, c2, c1, c0 = coef                        # Horner order in the source
    return np.array([c0, c1, c2, c3, c4])


def test_compiled_coefficients_are_the_remez_fit():
    fit = remez_rel(4).astype(np.float32)
    comp = compiled_coefficients().astype(np.float32)
    assert np.allclose(fit, comp, rtol=2e-6, atol=0), (fit, comp)


def test_compiled_coefficients_error_bound():
    assert fp32_horner_error(compiled_coefficients()) < BOUND
