"""On-device eigensolvers for the FlashDiffusion operator.

Drop-in names from ``FD/eigensolver.py`` of the reference:

* ``lanczos_eigsh(matvec, N, k, tol, maxiter, ncv)`` (``:33-85``) — the reference
  wraps SciPy ARPACK (implicitly restarted Lanczos, ``which='LM'``,
  ncv = min(max(2k+1, 20), N), fp64 reorthogonalisation on the host).  Here the
  same problem is solved by a thick-restart Lanczos (Wu & Simon, SIAM J. Matrix
  Anal. Appl. 22 (2000) — mathematically equivalent to implicit restarting)
  whose Krylov basis, full fp64 reorthogonalisation (classical Gram-Schmidt
  applied twice) and restarts all stay in GPU memory; only the small projected
  matrix goes to the host.
* ``lobpcg_eigsh(matvec, N, k, tol, maxiter, seed)`` (``:88-131``) — block
  LOBPCG (Knyazev 2001) with the block on the device, X0 = QR of a seeded
  N(0,1) block as in the reference.

``matvec`` may be a NumPy callable (as in the reference: one host round trip
per product) or an object with ``matvec_device(v: cuda fp64) -> cuda fp64``
(no host traffic).  Eigenvalues are returned in descending order, fp64.

Precision ramp (``ramp_eigsh``): the docstrings of the reference describe a
bf16 -> fp32 -> fp64 ramp that its code does not implement.  Here it is:
Lanczos on the bf16-tile operator until its Ritz residuals reach the bf16
floor, then restarted from those Ritz vectors on the fp32-tile operator, with
the final Rayleigh-Ritz in fp64.
"""

from __future__ import annotations

import time
from dataclasses import dataclass, field
from typing import Callable, Optional, Tuple

import numpy as np
import torch


@dataclass
class SolveInfo:
    n_matvec: int = 0
    n_restart: int = 0
    residuals: Optional[np.ndarray] = None
    seconds: float = 0.0
    converged: bool = False
    stages: list = field(default_factory=list)


def _device_op(matvec, device):
    if hasattr(matvec, "matvec_device"):
        return lambda v: matvec.matvec_device(v)

    def host(v):
        out = matvec(v.detach().cpu().numpy())
        return torch.from_numpy(np.asarray(out, dtype=np.float64).ravel()).to(device)

    return host


def _default_device():
    if not torch.cuda.is_available():
        raise RuntimeError("flashdiffusion_b200 eigensolvers run on a CUDA B200 device; none is visible")
    return torch.device("cuda", torch.cuda.current_device())


def _orth_against(Vb: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """Classical Gram-Schmidt twice: w <- (I - Vb^T Vb) w; returns the projection coefficients."""
    h = Vb @ w
    w -= Vb.T @ h
    h2 = Vb @ w
    w -= Vb.T @ h2
    return h + h2


def _native_rows_limit():
    try:
        from . import native
        native.load()
        return native.LANCZOS_MAX_ROWS
    except (ImportError, OSError):
        return 0


def _lanczos_cycle(op, V, T, kk, m, N, it, device, info):
    """Steps kk..m-1 of one restart cycle with host reads of the coefficients
    (bases wider than the library's row limit, and breakdowns).  Returns the
    last beta."""
    beta = 0.0
    for j in range(kk, m):
        w = op(V[j]).to(torch.float64).reshape(-1).clone()
        info.n_matvec += 1
        h = _orth_against(V[: j + 1], w)
        hc = h.cpu().numpy()
        T[: j + 1, j] = hc
        T[j, : j + 1] = hc
        beta = float(torch.linalg.vector_norm(w))
        if beta < 1e-300 or not np.isfinite(beta):
            # invariant subspace: continue from a fresh orthogonal direction
            g = torch.Generator(device="cpu").manual_seed(1000 + j + it)
            w = torch.randn(N, generator=g, dtype=torch.float64).to(device)
            _orth_against(V[: j + 1], w)
            V[j + 1] = w / torch.linalg.vector_norm(w)
            beta = 0.0
        else:
            V[j + 1] = w / beta
    return beta


def trlan(op: Callable[[torch.Tensor], torch.Tensor], N: int, k: int, tol: float, maxiter: int, ncv: int,
          v0: Optional[torch.Tensor], device, info: SolveInfo, stall_restarts: int = 3):
    """Thick-restart Lanczos for the k eigenvalues of largest magnitude.

    Returns (theta (k,) fp64 host, Y (N,k) fp64 device, residual norms (k,)).
    Convergence: ||A y - theta y|| <= tol * |theta| for all k pairs, or no 10 %
    improvement of the largest relative residual for ``stall_restarts``
    consecutive restarts (the matvec's own rounding floor).
    """
    m = max(min(ncv, N), k + 1)
    V = torch.zeros((m + 1, N), dtype=torch.float64, device=device)
    T = np.zeros((m, m))
    if v0 is None:
        g = torch.Generator(device="cpu").manual_seed(0)
        v0 = torch.randn(N, generator=g, dtype=torch.float64).to(device)
    v = v0.to(device=device, dtype=torch.float64).clone()
    V[0] = v / torch.linalg.vector_norm(v)
    kk = 0
    best = np.inf
    stall = 0
    theta = Y = res = None
    # the library's reorthogonalisation (three passes over V per step; the
    # projected-matrix coefficients stay on the device and are read once per
    # restart) whenever the basis fits its row limit
    fast = device.type == "cuda" and m + 1 <= _native_rows_limit()
    if fast:
        from . import native
        Tdev = torch.zeros((m, m + 2), dtype=torch.float64, device=device)
        ws = native.lanczos_workspace(N, m + 1, device)
    for it in range(maxiter):
        if fast:
            for j in range(kk, m):
                w = op(V[j]).to(torch.float64).reshape(-1).contiguous()
                info.n_matvec += 1
                native.lanczos_reorth(V, j + 1, w, V[j + 1], Tdev[j], ws)
            Tc = Tdev.cpu().numpy()
            betas = np.array([Tc[j, j + 1] for j in range(kk, m)])
            if np.all(np.isfinite(Tc[kk:m])) and np.all(betas > 1e-300):
                for j in range(kk, m):
                    T[: j + 1, j] = Tc[j, : j + 1]
                    T[j, : j + 1] = Tc[j, : j + 1]
                beta = float(betas[-1])
            else:
                # a breakdown (invariant subspace) in this cycle: redo it on the
                # host-synchronised path, which continues from a fresh direction
                beta = _lanczos_cycle(op, V, T, kk, m, N, it, device, info)
        else:
            beta = _lanczos_cycle(op, V, T, kk, m, N, it, device, info)
        Ts = 0.5 * (T + T.T)
        evals, evecs = np.linalg.eigh(Ts)
        order = np.argsort(-np.abs(evals))
        theta = evals[order[:k]]
        res = np.abs(beta * evecs[m - 1, order[:k]])
        rel = res / np.maximum(np.abs(theta), 1e-300)
        worst = float(rel.max())
        info.n_restart = it + 1
        if worst <= tol:
            info.converged = True
            break
        if worst < 0.9 * best:
            best, stall = worst, 0
        else:
            stall += 1
            if stall >= stall_restarts:
                break
        if it == maxiter - 1:
            break
        p = min(k + (m - k) // 2, m - 1)
        Yp = torch.from_numpy(np.ascontiguousarray(evecs[:, order[:p]])).to(device)
        V[:p] = Yp.T @ V[:m]
        V[p] = V[m]
        T = np.zeros((m, m))
        T[np.arange(p), np.arange(p)] = evals[order[:p]]
        kk = p
    Yk = torch.from_numpy(np.ascontiguousarray(evecs[:, order[:k]])).to(device)
    vecs = (Yk.T @ V[:m]).T.contiguous()
    info.residuals = res
    return theta, vecs, res


def lanczos_eigsh(matvec, N: int, k: int = 8, tol: float = 0.0, maxiter: Optional[int] = None,
                  ncv: Optional[int] = None, v0=None, return_info: bool = False):
    """Top-k eigenpairs (largest magnitude) of a symmetric operator, descending.

    Same signature and defaults as the reference (``FD/eigensolver.py:33-85``);
    ``tol=0`` means "as tight as the operator's rounding allows".
    Returns (eigenvalues (k,) fp64 NumPy, eigenvectors (N,k) fp64 NumPy).
    """
    device = _default_device()
    if ncv is None:
        ncv = min(max(2 * k + 1, 20), N)
    maxiter = 10 * N if maxiter is None else maxiter
    info = SolveInfo()
    t0 = time.perf_counter()
    v0d = None if v0 is None else torch.as_tensor(np.asarray(v0, dtype=np.float64)).to(device)
    theta, vecs, _ = trlan(_device_op(matvec, device), N, k, tol if tol > 0 else 1e-12, maxiter, ncv, v0d,
                           device, info)
    info.seconds = time.perf_counter() - t0
    idx = np.argsort(theta)[::-1]
    vals = theta[idx]
    out = (vals, vecs[:, torch.as_tensor(idx.copy(), device=device)].cpu().numpy())
    return (*out, info) if return_info else out


def ramp_eigsh(op_lo, op_hi_factory, N: int, k: int, tol: float = 0.0, ncv: Optional[int] = None,
               maxiter: int = 1000, lo_tol: float = 1e-3, v0=None) -> Tuple[np.ndarray, torch.Tensor, SolveInfo]:
    """bf16 -> fp32 -> fp64 precision ramp.

    Stage 1 runs Lanczos on ``op_lo`` (bf16 tiles) until the Ritz residuals
    reach ``lo_tol`` or the bf16 rounding floor; stage 2 builds the fp32-tile
    operator (``op_hi_factory()``) and restarts Lanczos from the sum of the
    stage-1 Ritz vectors; the Ritz values of the final fp64 projected matrix
    are returned.  Returns (vals desc (k,), vecs (N,k) device, info).
    """
    device = _default_device()
    if ncv is None:
        ncv = min(max(2 * k + 1, 20), N)
    info = SolveInfo()
    t0 = time.perf_counter()
    i1 = SolveInfo()
    v0d = None if v0 is None else torch.as_tensor(np.asarray(v0, dtype=np.float64)).to(device)
    _, y1, _ = trlan(_device_op(op_lo, device), N, k, lo_tol, maxiter, ncv, v0d, device, i1, stall_restarts=2)
    torch.cuda.synchronize(device)
    t1 = time.perf_counter()
    info.stages.append({"precision": "16-bit", "n_matvec": i1.n_matvec, "seconds": t1 - t0})
    op_hi = op_hi_factory()
    torch.cuda.synchronize(device)
    t2 = time.perf_counter()
    i2 = SolveInfo()
    start = y1.sum(dim=1)
    theta, vecs, res = trlan(_device_op(op_hi, device), N, k, tol if tol > 0 else 1e-9, maxiter, ncv, start,
                             device, i2, stall_restarts=4)
    torch.cuda.synchronize(device)
    t3 = time.perf_counter()
    info.stages.append({"precision": getattr(getattr(op_hi, "op", None), "precision", "fp32"),
                        "n_matvec": i2.n_matvec, "seconds": t3 - t2,
                        "setup_seconds": t2 - t1, "max_rel_residual": float(np.max(res / np.abs(theta)))})
    info.n_matvec = i1.n_matvec + i2.n_matvec
    info.residuals = res
    info.converged = i2.converged
    info.seconds = t3 - t0
    idx = np.argsort(theta)[::-1]
    return theta[idx], vecs[:, torch.as_tensor(idx.copy(), device=device)], info


def lobpcg_eigsh(matvec, N: int, k: int = 8, tol: float = 1e-8, maxiter: int = 300, seed: int = 42,
                 return_info: bool = False, block_matvec=None):
    """Top-k eigenpairs by LOBPCG (``FD/eigensolver.py:88-131``), block kept on the device.

    ``block_matvec`` (device (N,r) fp64 -> (N,r) fp64) applies the operator to
    a whole block in one call (one tile pass with r right-hand sides); by
    default a ``matvec_device`` object is applied to the block directly and a
    NumPy callable column by column.  Convergence: every column residual norm
    <= tol * |lambda|.  Returns (vals (k,) desc, vecs (N,k)) as NumPy.
    """
    device = _default_device()
    if block_matvec is None:
        if hasattr(matvec, "matvec_device"):
            def block_matvec(B):
                return matvec.matvec_device(B)
        else:
            op = _device_op(matvec, device)

            def block_matvec(B):
                return torch.stack([op(B[:, i].contiguous()) for i in range(B.shape[1])], dim=1)
    info = SolveInfo()
    t0 = time.perf_counter()
    vals, vecs = lobpcg_core(block_matvec, N, k, tol, maxiter, seed, device, info)
    info.seconds = time.perf_counter() - t0
    out = (vals, vecs.cpu().numpy())
    return (*out, info) if return_info else out


def lobpcg_core(block_matvec, N: int, k: int, tol: float, maxiter: int, seed: int, device, info: SolveInfo,
                guard: int = 0, X0: Optional[torch.Tensor] = None):
    """LOBPCG iteration (largest eigenvalues) with Rayleigh-Ritz on span[X, R, P].

    X0 = QR(N(0,1) block) seeded like the reference.  The trial basis is
    orthonormalised by QR (twice); A is applied to the R and P parts only,
    A X being carried over.  ``guard`` extra columns ride along (faster
    convergence of clustered spectra); convergence is judged on the top k.
    ``X0`` (N, k + guard) warm-starts the block (e.g. the vectors of a
    lower-precision stage).  Returns (vals desc host (k,), vecs device (N, k + guard)).
    """
    kk = k
    k = k + guard
    if X0 is not None:
        X = torch.linalg.qr(X0.to(device=device, dtype=torch.float64))[0]
    else:
        rng = np.random.default_rng(seed)
        X = torch.from_numpy(np.linalg.qr(rng.standard_normal((N, k)))[0]).to(device)
    AX = block_matvec(X).to(torch.float64)
    info.n_matvec += k
    P = None
    for it in range(maxiter):
        G = X.T @ AX
        G = 0.5 * (G + G.T)
        R = AX - X @ G
        rn = torch.linalg.vector_norm(R, dim=0)
        lam = torch.diagonal(G)
        top = torch.argsort(lam, descending=True)[:kk]
        info.residuals = (rn[top] / lam[top].abs().clamp_min(1e-300)).cpu().numpy()
        if float(info.residuals.max()) <= tol:
            info.converged = True
            break
        S = torch.cat([X, R] + ([P] if P is not None else []), dim=1)
        Q, _ = torch.linalg.qr(S)
        Q, _ = torch.linalg.qr(Q)
        AQ = block_matvec(Q[:, k:].contiguous()).to(torch.float64)
        info.n_matvec += Q.shape[1] - k
        AQ_full = torch.cat([AX @ (X.T @ Q[:, :k]), AQ], dim=1)
        H = Q.T @ AQ_full
        w, Z = torch.linalg.eigh(0.5 * (H + H.T))
        Zk = Z[:, torch.argsort(w, descending=True)[:k]]
        Xn = Q @ Zk
        AXn = AQ_full @ Zk
        P = Xn - X @ (X.T @ Xn)
        X, AX = Xn, AXn
        info.n_restart = it + 1
    G = X.T @ AX
    w, Z = torch.linalg.eigh(0.5 * (G + G.T))
    order = torch.argsort(w, descending=True)
    return w[order[:kk]].cpu().numpy(), X @ Z[:, order]
