"""Coifman-Lafon diffusion maps on the B200 operator.

Drop-in for ``FD/dmap.py`` of the reference:

* ``DiffusionMap(beta, alpha, n_components, tile)`` with ``fit`` (``:78-117``),
  ``matvec`` (``:119-136``), ``transform(X_new, t, tol, maxiter)``
  (``:142-190``) and ``doob_transform(h)`` (``:196-208``).  Fitted fields
  ``X_, D_, D_alpha_, rscale_, eigenvalues_, eigenvectors_, embedding_`` are
  NumPy float64 mirrors exactly as in the reference.
* ``DoobTransformedMap(base, h)`` (``:221-261``): ``Ph_ = M h`` and
  ``matvec(v) = M (h v) / Ph`` — here on the GPU with the division fused into
  the tile epilogue (the reference always runs it in NumPy).

Extra keyword ``precision`` ("ramp" default, "f16", "bf16", "fp32"): "ramp"
fits and starts the eigensolver on 16-bit tensor-core tiles, then finishes on fp32 tiles
with an fp64 Rayleigh-Ritz (the precision ramp the reference's docstrings
describe, ``FD/eigensolver.py:15-23``); after ``transform`` the fitted mirrors
hold the fp32 normalisation.
"""

from __future__ import annotations

import time
from typing import Optional

import numpy as np
import torch

from . import native
from .kernel import GaussianOperator, to_device
from .kernel_cuda_sm100 import CUDAStateSM100, normalise
from .eigensolver import lanczos_eigsh, ramp_eigsh, trlan, SolveInfo


class DiffusionMap:
    """Coifman-Lafon diffusion maps (see module docstring)."""

    def __init__(self, beta: float = 1.0, alpha: float = 0.5, n_components: int = 8, tile: int = 512,
                 precision: str = "ramp", verbose: bool = False):
        if precision not in ("ramp", "f16", "bf16", "fp32", "f16x3"):
            raise ValueError(f"precision must be 'ramp', 'f16', 'bf16', 'fp32' or 'f16x3' (got {precision!r})")
        self.beta = beta
        self.alpha = alpha
        self.n_components = n_components
        self.tile = tile
        self.precision = precision
        self.verbose = verbose
        self.X_: Optional[np.ndarray] = None
        self.rscale_: Optional[np.ndarray] = None
        self.D_: Optional[np.ndarray] = None
        self.D_alpha_: Optional[np.ndarray] = None
        self._cuda_state: Optional[CUDAStateSM100] = None
        self._hi_state: Optional[CUDAStateSM100] = None
        self.eigenvalues_: Optional[np.ndarray] = None
        self.eigenvectors_: Optional[np.ndarray] = None
        self.embedding_: Optional[np.ndarray] = None
        self.solve_info_ = None
        self.timings_ = {}

    # ------------------------------------------------------------------
    def _state(self, precision: str) -> CUDAStateSM100:
        op = GaussianOperator(self._Xd, None, self.beta, precision)
        t0 = time.perf_counter()
        D, Da, rs = normalise(op, self.alpha)
        torch.cuda.synchronize()
        st = CUDAStateSM100(op, rs, D, Da, self.beta, self.alpha, X=self._Xd)
        st.timings["precompute_s"] = time.perf_counter() - t0
        return st

    def _mirror(self, st: CUDAStateSM100):
        self.D_ = st.D.double().cpu().numpy()
        self.D_alpha_ = st.D_alpha.double().cpu().numpy()
        self.rscale_ = st.rscale.double().cpu().numpy()

    def fit(self, X) -> "DiffusionMap":
        """Two prepass reductions on the GPU: D, w = D^-alpha, D_alpha, rscale."""
        self.X_ = np.asarray(X, dtype=np.float64) if not isinstance(X, torch.Tensor) else None
        self._Xd = to_device(X, torch.float32)
        first = "f16" if self.precision == "ramp" else self.precision
        self._cuda_state = self._state(first)
        self._hi_state = self._cuda_state if self.precision in ("fp32", "f16x3") else None
        self.timings_["fit_s"] = self._cuda_state.timings["precompute_s"]
        self._mirror(self._cuda_state)
        if self.verbose:
            print(f"[DiffusionMap.fit] N={self._Xd.shape[0]} beta={self.beta} alpha={self.alpha} "
                  f"({first} tiles) {self.timings_['fit_s']:.3f}s")
        return self

    def _best_state(self) -> CUDAStateSM100:
        return self._hi_state if self._hi_state is not None else self._cuda_state

    def matvec(self, v: np.ndarray) -> np.ndarray:
        """M v = rscale * K (rscale * v) for a host vector (``FD/dmap.py:119-136``)."""
        self._check_fitted()
        st = self._best_state()
        vd = torch.from_numpy(np.ascontiguousarray(v, dtype=np.float64)).to(st.op.device)
        return st.matvec_device(vd).cpu().numpy()

    def matvec_device(self, v: torch.Tensor) -> torch.Tensor:
        self._check_fitted()
        return self._best_state().matvec_device(v)

    # ------------------------------------------------------------------
    def transform(self, X_new=None, t: int = 1, tol: float = 0.0, maxiter: Optional[int] = None):
        """Diffusion coordinates (N, n_components-1); Nystrom extension when X_new is given."""
        self._check_fitted()
        if X_new is not None:
            return self.nystrom(X_new, t=t)
        N = self._Xd.shape[0]
        k = self.n_components
        t0 = time.perf_counter()
        if self.precision == "ramp":
            def hi():
                # fp32-class tensor-core tiles (split operands) when d <= 136, else fp32 SIMT tiles
                self._hi_state = self._state("f16x3")
                return self._hi_state
            vals, vecs, info = ramp_eigsh(self._cuda_state, hi, N, k, tol=tol,
                                          maxiter=maxiter if maxiter else 1000)
            self._mirror(self._hi_state)
            vecs = vecs.cpu().numpy()
        else:
            vals, vecs, info = lanczos_eigsh(self._cuda_state, N, k=k, tol=tol, maxiter=maxiter,
                                             return_info=True)
        self.timings_["transform_s"] = time.perf_counter() - t0
        self.solve_info_ = info
        self.eigenvalues_ = vals
        self.eigenvectors_ = vecs
        psi = vecs / self.rscale_[:, None]
        psi /= np.linalg.norm(psi, axis=0, keepdims=True)
        coords = psi[:, 1:] * (vals[1:] ** t)[None, :]
        self.embedding_ = coords
        if self.verbose:
            print(f"[DiffusionMap.transform] k={k} matvecs={info.n_matvec} {self.timings_['transform_s']:.3f}s")
        return coords

    def nystrom(self, X_new, t: int = 1) -> np.ndarray:
        """Out-of-sample coordinates (``FD/utils.py:59-123``) with the AMAP (Q != K) operator.

        D_new = K(X_new, X) w_train; w_new = D_new^-alpha;
        rscale_new = (D_new w_new)^-1/2 w_new; coords = rscale_new K(X_new, X) rscale phi  * lambda^(t-1).
        """
        if self.eigenvalues_ is None:
            raise RuntimeError("Call transform() on training data first.")
        st = self._best_state()
        op = GaussianOperator(to_device(X_new, torch.float32), st.X, self.beta, st.op.precision, shift=st.op.shift)
        w_train = native.dmap_weights(st.D, self.alpha)
        D_new = op.apply(w_train, out_dtype=torch.float32)[:, 0].contiguous()
        w_new = native.dmap_weights(D_new, self.alpha)
        _, rs_new = native.dmap_rscale(D_new, w_new)
        phi = self.eigenvectors_ / self.rscale_[:, None]
        phi = phi / np.linalg.norm(phi, axis=0, keepdims=True)
        V = torch.from_numpy(np.ascontiguousarray(phi[:, 1:])).to(op.device)
        coords = op.apply(V, col_scale=st.rscale, row_scale=rs_new, out_dtype=torch.float64).cpu().numpy()
        lam = self.eigenvalues_[1:]
        return coords * (lam ** (t - 1))[None, :]

    def doob_transform(self, h: np.ndarray) -> "DoobTransformedMap":
        self._check_fitted()
        return DoobTransformedMap(self, h)

    def _check_fitted(self):
        if self._cuda_state is None:
            raise RuntimeError("Call fit(X) before transform() or matvec().")


class DoobTransformedMap:
    """Doob h-transform M_h v = M (h v) / (M h) of a fitted DiffusionMap (``FD/dmap.py:221-261``)."""

    def __init__(self, base: DiffusionMap, h):
        self.base = base
        self.h = np.asarray(h, dtype=np.float64)
        st = base._best_state()
        self._h = torch.from_numpy(self.h.astype(np.float32)).to(st.op.device)
        Ph = st.op.apply(self._h, col_scale=st.rscale, row_scale=st.rscale, out_dtype=torch.float32)[:, 0]
        self._Ph = Ph.contiguous()
        self.Ph_ = self._Ph.double().cpu().numpy()

    def matvec_device(self, v: torch.Tensor) -> torch.Tensor:
        st = self.base._best_state()
        squeeze = v.dim() == 1
        out = st.op.apply(v[:, None] if squeeze else v, col_scale=st.rscale, col_h=self._h, row_scale=st.rscale,
                          row_div=self._Ph, out_dtype=torch.float64)
        return out[:, 0] if squeeze else out

    def matvec(self, v: np.ndarray) -> np.ndarray:
        """Apply the Doob-transformed operator to a host vector."""
        vd = torch.from_numpy(np.ascontiguousarray(v, dtype=np.float64)).to(self._h.device)
        return self.matvec_device(vd).cpu().numpy()

    def symmetric(self) -> "_SymDoob":
        """S M S with S = sqrt(h / Ph): symmetric, same spectrum as M_h."""
        return _SymDoob(self)

    def eigsh(self, k: int = 8, tol: float = 0.0, maxiter: Optional[int] = None):
        """Top-k eigenpairs of M_h through its symmetric similar form.

        Eigenvectors of M_h are returned: y = x / sqrt(h Ph) for x of S M S.
        (The reference hands the non-symmetric M_h to a symmetric solver,
        ``tests/test_kernel.py:87-88``.)
        """
        sym = self.symmetric()
        vals, x = lanczos_eigsh(sym, len(self.h), k=k, tol=tol, maxiter=maxiter)
        y = x / np.sqrt(self.h * self.Ph_)[:, None]
        return vals, y / np.linalg.norm(y, axis=0, keepdims=True)


class _SymDoob:
    def __init__(self, doob: DoobTransformedMap):
        st = doob.base._best_state()
        self.st = st
        s = torch.sqrt(doob._h.double() / doob._Ph.double())
        self.scale = (st.rscale.double() * s).float().contiguous()

    def matvec_device(self, v: torch.Tensor) -> torch.Tensor:
        squeeze = v.dim() == 1
        out = self.st.op.apply(v[:, None] if squeeze else v, col_scale=self.scale, row_scale=self.scale,
                               out_dtype=torch.float64)
        return out[:, 0] if squeeze else out
