"""CPU oracle for the FlashDiffusion Gaussian-kernel operator — TEST INFRASTRUCTURE ONLY.

This module is the checker, never the product.  Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference arm may
import it.  The shipped path (``flashdiffusion_b200``) never calls into it and
fails loudly when its CUDA library is missing.

It restates, in plain NumPy, the reference algorithm of sparsetrace/FlashDiffusion
(paths below are relative to that project; ``FD/`` = ``src/flashdiffusion/``):

* ``dist2_tile``        — ``FD/kernel.py:125-134``  (fp32 GEMM law of cosines, clamp >= 0, fp64 cast)
* ``prepass_rowsum``    — ``FD/kernel.py:141-182``  (row sums sum_j exp(-beta d2_ij) w_j, fp64)
* ``flash_diffusion``   — ``FD/kernel.py:189-257``  (rscale_q * K (rscale_k * h * V), fp64 accumulate)
* ``dmap_fit``          — ``FD/dmap.py:78-117``     (D, w = D^-alpha, D_alpha = (K w) w, rscale)
* ``dmap_matvec``       — ``FD/dmap.py:119-136``
* ``doob_ph`` / ``doob_matvec`` — ``FD/dmap.py:221-261``
* ``amap_normalise``    — ``FD/utils.py:92-102``    (the reference's only Q != K normaliser)
* ``nystrom_extend``    — ``FD/utils.py:59-123``
* ``dense_kernel`` / ``dense_dmap_operator`` — ``tests/test_kernel.py:17-30``
* ``lanczos_eigsh``     — ``FD/eigensolver.py:33-85`` (ARPACK IRLM via SciPy, descending sort)
* ``transform_coords``  — ``FD/dmap.py:184-189``
* ``median_bandwidth``  — ``FD/utils.py:16-28``   (seeded subsample, median of positive d^2)
* ``knn_bandwidth``     — ``FD/utils.py:31-52``   (distance to the k-th neighbour, self at index 0)
* ``apply_pplus`` / ``carre_du_champ`` / ``metric_tensor`` — ``FD/cdc.py:45-168``

Parity is pinned: ``tests/test_oracle.py`` checks every function here against
golden vectors produced by running the reference itself
(``tests/golden/make_golden.py``).
"""

from __future__ import annotations

import numpy as np

__all__ = [
    "dist2_tile", "prepass_rowsum", "flash_diffusion", "dmap_fit", "dmap_matvec",
    "doob_ph", "doob_matvec", "amap_normalise", "nystrom_extend", "dense_kernel",
    "dense_dmap_operator", "lanczos_eigsh", "transform_coords", "sym_doob_operator",
    "median_bandwidth", "knn_bandwidth", "sq_dists", "apply_pplus", "carre_du_champ", "metric_tensor",
]


def dist2_tile(qi32, kj32, sq_q, sq_k):
    """Squared distances of one (Q-tile, K-tile) pair (``FD/kernel.py:125-134``).

    The cross term is an fp32 GEMM; the three-term sum is formed in fp32 and
    clamped at zero before being widened to fp64.
    """
    cross = qi32 @ kj32.T                       # fp32 GEMM
    d2 = sq_q[:, None] + sq_k[None, :] - np.float32(2.0) * cross
    d2 = np.maximum(d2, np.float32(0.0))
    return d2.astype(np.float64)


def _tiled_apply(Q, K, beta, U, tile):
    """sum_j exp(-beta d2_ij) U_j over tiles of ``tile`` rows/cols, fp64 result."""
    q32 = np.asarray(Q, dtype=np.float32)
    k32 = np.asarray(K, dtype=np.float32)
    sq_q = (q32 * q32).sum(axis=1)
    sq_k = (k32 * k32).sum(axis=1)
    nq, nk = q32.shape[0], k32.shape[0]
    out = np.zeros((nq, U.shape[1]), dtype=np.float64)
    for a in range(0, nq, tile):
        b = min(a + tile, nq)
        for c in range(0, nk, tile):
            e = min(c + tile, nk)
            kt = np.exp(-beta * dist2_tile(q32[a:b], k32[c:e], sq_q[a:b], sq_k[c:e]))
            out[a:b] += kt @ U[c:e]
    return out


def prepass_rowsum(Q, K, beta, weights_k=None, tile=512):
    """out_i = sum_j exp(-beta ||q_i-k_j||^2) w_j  (``FD/kernel.py:141-182``); (N_q,) fp64."""
    nk = np.asarray(K).shape[0]
    w = np.ones(nk) if weights_k is None else np.asarray(weights_k, dtype=np.float64)
    return _tiled_apply(Q, K, beta, w.reshape(-1, 1), tile)[:, 0]


def flash_diffusion(Q, K, V, beta, rscale_q=None, rscale_k=None, h=None, tile=512):
    """rscale_q_i sum_j exp(-beta d2_ij) rscale_k_j h_j V_j  (``FD/kernel.py:189-257``).

    The right-hand side is pre-scaled in fp64 (``:227-232``), the kernel tile
    is evaluated in fp64 from fp32 distances and the row scale is applied
    after the sum (``:254-255``).
    """
    U = np.asarray(V, dtype=np.float64)
    if U.ndim == 1:
        U = U[:, None]
    if rscale_k is not None:
        U = np.asarray(rscale_k, dtype=np.float64)[:, None] * U
    if h is not None:
        U = np.asarray(h, dtype=np.float64)[:, None] * U
    out = _tiled_apply(Q, K, beta, U, tile)
    if rscale_q is not None:
        out = out * np.asarray(rscale_q, dtype=np.float64)[:, None]
    return out


def dmap_fit(X, beta, alpha, tile=512):
    """Coifman-Lafon normalisation (``FD/dmap.py:108-115``).

    Returns (D, D_alpha, rscale) with w = D^-alpha, D_alpha = (K w) * w and
    rscale = D_alpha^-1/2 * w.
    """
    D = prepass_rowsum(X, X, beta, None, tile)
    w = D ** (-alpha)
    D_alpha = prepass_rowsum(X, X, beta, w, tile) * w
    rscale = D_alpha ** (-0.5) * w
    return D, D_alpha, rscale


def dmap_matvec(X, beta, rscale, v, tile=512):
    """M v = rscale * K (rscale * v)  (``FD/dmap.py:128-136``)."""
    return flash_diffusion(X, X, np.asarray(v).reshape(-1, 1), beta, rscale, rscale, None, tile)[:, 0]


def doob_ph(X, beta, rscale, h, tile=512):
    """Ph = M h, the Doob row normaliser (``FD/dmap.py:238-247``)."""
    return dmap_matvec(X, beta, rscale, h, tile)


def doob_matvec(X, beta, rscale, h, Ph, v, tile=512):
    """M_h v = M (h * v) / Ph  (``FD/dmap.py:249-261``)."""
    return dmap_matvec(X, beta, rscale, np.asarray(h) * np.asarray(v), tile) / Ph


def amap_normalise(Q, K, beta, alpha, D_k, tile=512):
    """Query-side normalisation for Q != K (``FD/utils.py:92-102``).

    w_k = D_k^-alpha; D_q = K(Q,K) w_k; w_q = D_q^-alpha;
    D_alpha_q = D_q * w_q; rscale_q = D_alpha_q^-1/2 * w_q.
    Returns rscale_q; the key-side scale is the training set's own rscale.
    """
    w_k = np.asarray(D_k, dtype=np.float64) ** (-alpha)
    D_q = prepass_rowsum(Q, K, beta, w_k, tile)
    w_q = D_q ** (-alpha)
    D_alpha_q = D_q * w_q
    return D_alpha_q ** (-0.5) * w_q


def nystrom_extend(X_new, X_train, beta, alpha, D_train, rscale_train, eigvals, eigvecs, t=1, tile=512):
    """Out-of-sample coordinates (``FD/utils.py:59-123``)."""
    rq = amap_normalise(X_new, X_train, beta, alpha, D_train, tile)
    phi = eigvecs / rscale_train[:, None]
    phi = phi / np.linalg.norm(phi, axis=0, keepdims=True)
    coords = flash_diffusion(X_new, X_train, phi[:, 1:], beta, rq, rscale_train, None, tile)
    return coords * (eigvals[1:] ** (t - 1))[None, :]


def dense_kernel(X, beta):
    """Materialised fp64 Gaussian kernel (``tests/test_kernel.py:17-20``)."""
    X = np.asarray(X, dtype=np.float64)
    sq = np.einsum("ij,ij->i", X, X)
    return np.exp(-beta * np.maximum(sq[:, None] + sq[None, :] - 2.0 * X @ X.T, 0.0))


def dense_dmap_operator(X, beta, alpha):
    """Dense M = dh K_alpha dh and rscale = dh w (``tests/test_kernel.py:23-30``)."""
    Kx = dense_kernel(X, beta)
    w = Kx.sum(1) ** (-alpha)
    Ka = Kx * w[:, None] * w[None, :]
    dh = Ka.sum(1) ** (-0.5)
    return dh[:, None] * Ka * dh[None, :], dh * w


def sym_doob_operator(M, h, Ph):
    """Symmetric similar form S M S of M_h = diag(1/Ph) M diag(h), S = sqrt(h/Ph).

    Both operators share eigenvalues; the symmetric form is what a
    symmetric Lanczos can solve exactly (the reference feeds the
    non-symmetric operator to ``eigsh``, ``tests/test_kernel.py:87-88``).
    """
    s = np.sqrt(np.asarray(h) / np.asarray(Ph))
    return s[:, None] * M * s[None, :]


def lanczos_eigsh(matvec, N, k=8, tol=0.0, maxiter=None, ncv=None, v0=None):
    """Top-k by ARPACK IRLM, ``which='LM'``, descending (``FD/eigensolver.py:33-85``)."""
    from scipy.sparse.linalg import LinearOperator, eigsh

    if ncv is None:
        ncv = min(max(2 * k + 1, 20), N)
    op = LinearOperator((N, N), matvec=lambda x: matvec(np.asarray(x, np.float64).ravel()),
                        dtype=np.float64)
    vals, vecs = eigsh(op, k=k, which="LM", tol=tol, maxiter=maxiter, ncv=ncv, v0=v0)
    order = np.argsort(vals)[::-1]
    return vals[order], vecs[:, order]


def transform_coords(vals, vecs, rscale, t=1):
    """psi = vecs / rscale, column-normalised; coords = psi[:,1:] lambda^t (``FD/dmap.py:184-189``)."""
    psi = vecs / rscale[:, None]
    psi = psi / np.linalg.norm(psi, axis=0, keepdims=True)
    return psi[:, 1:] * (vals[1:] ** t)[None, :]


def sq_dists(A, B):
    """Squared distances by the law of cosines in the inputs' dtype, clamped at 0
    (the form ``FD/utils.py:23-24,46-47`` use)."""
    A = np.asarray(A)
    B = np.asarray(B)
    return np.maximum((A * A).sum(1)[:, None] + (B * B).sum(1)[None, :] - 2 * A @ B.T, 0)


def median_bandwidth(X, subsample=2000):
    """beta = 1 / (2 median of the positive pairwise d^2) over a seeded subsample
    (``default_rng(0)``, without replacement, only when N > subsample) — ``FD/utils.py:16-28``."""
    X = np.asarray(X)
    if X.shape[0] > subsample:
        X = X[np.random.default_rng(0).choice(X.shape[0], subsample, replace=False)]
    d2 = sq_dists(X, X)
    med = np.median(d2[d2 > 0])
    return 1.0 / (2.0 * med) if med > 0 else 1.0


def knn_bandwidth(X, k=7):
    """sigma_i = sqrt(k-th smallest d^2 of row i, index 0 being the point itself),
    floored at 1e-10 — ``FD/utils.py:31-52``."""
    d2 = np.sort(sq_dists(X, X), axis=1)
    return np.maximum(np.sqrt(d2[:, k]), 1e-10)


def apply_pplus(X, beta, alpha, D, D_alpha, F, tile=512):
    """P+ F = diag(w / D_alpha) K diag(w) F with w = D^-alpha (``FD/cdc.py:107-130``)."""
    w = np.asarray(D, np.float64) ** (-alpha)
    F = np.asarray(F, np.float64)
    out = flash_diffusion(X, X, F.reshape(F.shape[0], -1), beta, w / np.asarray(D_alpha, np.float64), w, None, tile)
    return out if F.ndim == 2 else out[:, 0]


def carre_du_champ(X, beta, alpha, D, D_alpha, phi_k, phi_l, lambda_k, lambda_l, tile=512):
    """Gamma(phi_k, phi_l) = (P+(phi_k phi_l) - lambda_k phi_k phi_l - lambda_l phi_l phi_k) / 2,
    the reference's formula as written (``FD/cdc.py:96-104``)."""
    pkl = np.asarray(phi_k) * np.asarray(phi_l)
    return 0.5 * (apply_pplus(X, beta, alpha, D, D_alpha, pkl, tile) - lambda_k * pkl - lambda_l * pkl)


def metric_tensor(X, beta, alpha, D, D_alpha, vals, phi, pairs=None, tile=512):
    """G[i,k,l] = Gamma(phi_k, phi_l)(i) over the pairs (default: all k <= l), symmetric;
    M = sum_i G_i G_i^T (``FD/cdc.py:133-168``)."""
    k = len(vals)
    G = np.zeros((phi.shape[0], k, k))
    for a, b in (pairs if pairs is not None else [(i, j) for i in range(k) for j in range(i, k)]):
        g = carre_du_champ(X, beta, alpha, D, D_alpha, phi[:, a], phi[:, b], vals[a], vals[b], tile)
        G[:, a, b] = g
        G[:, b, a] = g
    return G, np.einsum("ikm,ilm->kl", G, G)
