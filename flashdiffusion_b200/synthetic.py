"""Seeded synthetic point clouds for the five benchmark configurations.

No public dataset is involved: each generator follows the recipe of one
benchmark configuration (Swiss roll, Gaussian mixture, 6-D manifold with a
drifted query set, a Langevin trajectory in a double well, a 10-D tanh
manifold).  Every generator takes an explicit seed and returns float32
points plus the bandwidth ``beta`` from the median rule
beta = 1 / median(pairwise squared distance) over a seeded 1024-point
subsample (off-diagonal pairs).
"""

from __future__ import annotations

import ctypes
import math
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))


def median_beta(X, subsample=1024, seed=0):
    """beta = 1 / median(||x_i - x_j||^2) over i<j of a seeded subsample."""
    X = np.asarray(X, dtype=np.float64)
    n = X.shape[0]
    if n > subsample:
        idx = np.random.default_rng(seed).choice(n, subsample, replace=False)
        X = X[idx]
    sq = (X * X).sum(1)
    d2 = np.maximum(sq[:, None] + sq[None, :] - 2.0 * X @ X.T, 0.0)
    iu = np.triu_indices(X.shape[0], k=1)
    med = float(np.median(d2[iu]))
    return 1.0 / med if med > 0 else 1.0


def swiss_roll(n=4096, seed=0, noise=0.05):
    """Config 1: t~U(1.5pi,4.5pi), h~U(0,21); (t cos t, h, t sin t) + N(0, noise^2)."""
    rng = np.random.default_rng(seed)
    t = rng.uniform(1.5 * np.pi, 4.5 * np.pi, n)
    h = rng.uniform(0.0, 21.0, n)
    X = np.stack([t * np.cos(t), h, t * np.sin(t)], axis=1)
    X += rng.normal(0.0, noise, X.shape)
    return X.astype(np.float32), median_beta(X, seed=seed), t


def gaussian_mixture(n=200_000, d=64, n_comp=10, seed=0):
    """Config 2: equal-weight isotropic mixture, means ~N(0,16 I), sigma_c ~U(0.5,1.5)."""
    rng = np.random.default_rng(seed)
    means = rng.normal(0.0, 4.0, (n_comp, d))
    sig = rng.uniform(0.5, 1.5, n_comp)
    lab = rng.integers(0, n_comp, n)
    X = means[lab] + sig[lab, None] * rng.standard_normal((n, d))
    X = X.astype(np.float32)
    return X, median_beta(X, seed=seed)


def amap_manifold(n=500_000, d=64, seed=0, drift=0.05):
    """Config 3: K on a 6-D manifold (sin/cos features, orthogonal 24->d lift, N(0,.01^2));
    Q = K + drift * K A^T with A seeded and scaled to spectral norm 1."""
    rng = np.random.default_rng(seed)
    u = rng.uniform(-1.0, 1.0, (n, 6))
    feats = np.concatenate([np.sin(np.pi * u), np.cos(np.pi * u),
                            np.sin(2 * np.pi * u), np.cos(2 * np.pi * u)], axis=1)   # (n, 24)
    E, _ = np.linalg.qr(rng.standard_normal((d, 24)))                                 # (d, 24) orthonormal columns
    K = feats @ E.T + rng.normal(0.0, 0.01, (n, d))
    A = rng.standard_normal((d, d))
    A /= np.linalg.norm(A, 2)
    Q = K + drift * (K @ A.T)
    K = K.astype(np.float32)
    Q = Q.astype(np.float32)
    return Q, K, median_beta(K, seed=seed)


def _langevin_c(noise, x0, y0, dt, kT, keep):
    lib_path = os.path.join(_HERE, "libfd_synth.so")
    if not os.path.exists(lib_path):
        return None
    lib = ctypes.CDLL(lib_path)
    lib.fd_synth_langevin.restype = ctypes.c_int
    nsteps = noise.shape[0]
    nout = nsteps // keep
    out = np.empty((nout, 2), dtype=np.float64)
    noise = np.ascontiguousarray(noise, dtype=np.float64)
    rc = lib.fd_synth_langevin(
        noise.ctypes.data_as(ctypes.c_void_p), ctypes.c_long(nsteps),
        ctypes.c_double(x0), ctypes.c_double(y0), ctypes.c_double(dt), ctypes.c_double(kT),
        ctypes.c_long(keep), out.ctypes.data_as(ctypes.c_void_p))
    if rc != 0:
        raise RuntimeError(f"fd_synth_langevin failed: {rc}")
    return out


def langevin_trajectory(n_frames=500_000, d=66, seed=0, dt=1e-3, kT=0.5, keep=10):
    """Config 4: overdamped Langevin in U(x,y) = (x^2-1)^2 + y^2 by Euler-Maruyama,
    every ``keep``-th step kept, lifted by a seeded Gaussian 2->d map + N(0,.01^2).
    Returns (X float32, beta, h = exp(-0.5 x^2) of the latent x, latent)."""
    rng = np.random.default_rng(seed)
    nsteps = n_frames * keep
    noise = rng.standard_normal((nsteps, 2))
    x0, y0 = -1.0, 0.0
    lat = _langevin_c(noise, x0, y0, dt, kT, keep)
    if lat is None:                      # small cases without the helper library
        lat = np.empty((n_frames, 2))
        x, y = x0, y0
        amp = math.sqrt(2.0 * kT * dt)
        for s in range(nsteps):
            gx = 4.0 * x * (x * x - 1.0)
            gy = 2.0 * y
            x = x - gx * dt + amp * noise[s, 0]
            y = y - gy * dt + amp * noise[s, 1]
            if (s + 1) % keep == 0:
                lat[(s + 1) // keep - 1] = (x, y)
    W = rng.standard_normal((2, d))
    X = lat @ W + rng.normal(0.0, 0.01, (n_frames, d))
    h = np.exp(-0.5 * lat[:, 0] ** 2)
    X = X.astype(np.float32)
    return X, median_beta(X, seed=seed), h, lat


def tanh_manifold(n=2_000_000, d=128, seed=0, latent=10, hidden=256, noise=0.02, chunk=1 << 18):
    """Config 5: z~N(0,I_10) -> tanh(z W1) (W1 10x256, N(0,1/10)) -> linear 256->d
    (N(0,1/256)) + N(0, noise^2).  Generated in chunks to bound host memory."""
    rng = np.random.default_rng(seed)
    W1 = rng.normal(0.0, 1.0 / math.sqrt(latent), (latent, hidden))
    W2 = rng.normal(0.0, 1.0 / math.sqrt(hidden), (hidden, d))
    X = np.empty((n, d), dtype=np.float32)
    for a in range(0, n, chunk):
        b = min(a + chunk, n)
        z = rng.standard_normal((b - a, latent))
        X[a:b] = (np.tanh(z @ W1) @ W2 + rng.normal(0.0, noise, (b - a, d))).astype(np.float32)
    return X, median_beta(X, seed=seed)
