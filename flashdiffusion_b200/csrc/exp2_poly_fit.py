"""Derive the polynomial used for the FMA-pipe share of exp2 in fd_tc.cu.

2^x = 2^j * 2^f with j = round(x), f = x - j in [-1/2, 1/2] (Cody-Waite style
range reduction; j goes into the exponent field).  2^f is approximated by a
polynomial p(f) with p(0) = 1 chosen to minimise the maximum RELATIVE error
on [-1/2, 1/2] (Remez exchange on the weighted error (p(f) - 2^f) / 2^f).
Coefficients are then rounded to fp32 and the error re-measured in fp32
Horner arithmetic.  Run: python flashdiffusion_b200/csrc/exp2_poly_fit.py
"""
import numpy as np


def remez_rel(deg, iters=60):
    # unknowns: c1..c_deg (c0 fixed to 1) and the levelled error E
    n = deg + 1                      # reference points
    x = 0.5 * np.cos(np.pi * np.arange(n)[::-1] / (n - 1))
    for _ in range(iters):
        A = np.zeros((n, deg + 1))
        b = np.zeros(n)
        for i, xi in enumerate(x):
            t = 2.0 ** xi
            A[i, :deg] = [xi ** k for k in range(1, deg + 1)]
            A[i, deg] = ((-1) ** i) * t
            b[i] = t - 1.0
        sol = np.linalg.solve(A, b)
        c = np.concatenate([[1.0], sol[:deg]])
        g = np.linspace(-0.5, 0.5, 200001)
        err = (np.polyval(c[::-1], g) - 2.0 ** g) / 2.0 ** g
        # new reference points: extrema of err on each sign-alternating segment
        idx = [0]
        for k in range(1, len(g) - 1):
            if (err[k] - err[k - 1]) * (err[k + 1] - err[k]) <= 0:
                idx.append(k)
        idx.append(len(g) - 1)
        cand = sorted(idx, key=lambda k: -abs(err[k]))
        pts = sorted(cand[:n])
        x = g[pts]
    return c, np.abs(err).max()


def fp32_error(c):
    c32 = np.array(c, dtype=np.float32)
    g = np.linspace(-0.5, 0.5, 400001).astype(np.float32)
    p = np.full_like(g, c32[-1])
    for ck in c32[-2::-1]:
        p = (p * g + ck).astype(np.float32)
    return float(np.max(np.abs(p.astype(np.float64) - 2.0 ** g.astype(np.float64)) / 2.0 ** g.astype(np.float64)))


if __name__ == "__main__":
    for deg in (3, 4, 5):
        c, e = remez_rel(deg)
        print(f"degree {deg}: max rel err {e:.3e} (exact coefs), {fp32_error(c):.3e} (fp32 Horner)")
        print("   coefficients c0..c%d:" % deg, ", ".join(f"{np.float32(v)!r}" for v in c))
