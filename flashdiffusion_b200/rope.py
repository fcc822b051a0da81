"""RoPE-DMAP encoder on Hankel windows (reference ``FD/ROPE.py``), on the GPU.

The reference builds the dense K x K Gram, distance and kernel matrices of the
rotated window vectors and hands the dense symmetric operator to ARPACK.  Here
the rotation is a per-row preprocessing kernel (``fd_rope_windows``: Hankel
windows read in place from the series, centred, pairs rotated in fp64) and
everything after it is the existing never-materialised operator:

  fit     : rotated windows Y -> DiffusionMap(beta, alpha).fit(Y) (two prepasses:
            q = K 1, d = (K q^-alpha) q^-alpha) -> device Lanczos on
            d^-1/2 K_alpha d^-1/2 = diag(rscale) K diag(rscale) -> psi = d^-1/2 phi
  encode  : rotated query windows -> two Q != K prepasses (row sums, then with
            the training weights q_T^-alpha) -> one block pass with
            V = psi / lambda (the Nystrom formula of ``FD/ROPE.py:489-526``)

``G_`` and ``Kmat_`` (dense K x K in the reference) are never formed and are
None here; every other learned attribute keeps its name and meaning.  The
+1e-18 guards of the reference are kept where they change a result (row sums
of far query windows).
"""

from __future__ import annotations

import numpy as np
import torch

from . import native
from .dmap import DiffusionMap
from .kernel import GaussianOperator

__all__ = ["ROPE", "make_hankel_windows", "make_window_positions"]

_WINDOW_POSITION = {"start": 0, "center": 1, "end": 2}


def make_hankel_windows(F_tX, L: int, step: int = 1) -> np.ndarray:
    """(K, L, D) Hankel windows W[T, c] = F[T + c step], K = N - (L-1) step (``FD/ROPE.py:31-57``)."""
    F = np.asarray(F_tX, dtype=float)
    if F.ndim == 1:
        F = F[:, None]
    L, step = int(L), int(step)
    if L <= 0:
        raise ValueError("L must be positive.")
    if step <= 0:
        raise ValueError("step must be positive.")
    K = F.shape[0] - (L - 1) * step
    if K <= 0:
        raise ValueError(f"Need N={F.shape[0]} >= (L-1)*step+1 = {(L - 1) * step + 1}")
    idx = np.arange(K)[:, None] + step * np.arange(L)[None, :]
    return F[idx]


def make_window_positions(sample_positions, L: int, step: int = 1, mode: str = "sample",
                          window_position: str = "end") -> np.ndarray:
    """(K, L) sample positions, or (K,) one per window (``FD/ROPE.py:60-106``)."""
    pos = np.asarray(sample_positions, dtype=float)
    if pos.ndim != 1:
        raise ValueError("sample_positions must be one-dimensional.")
    K = len(pos) - (L - 1) * step
    if K <= 0:
        raise ValueError("Not enough positions for windows.")
    P = pos[np.arange(K)[:, None] + step * np.arange(L)[None, :]]
    if mode == "sample":
        return P
    if mode != "window":
        raise ValueError("mode must be 'sample' or 'window'.")
    if window_position not in _WINDOW_POSITION:
        raise ValueError("window_position must be 'start', 'center', or 'end'.")
    return P[:, (0, L // 2, L - 1)[_WINDOW_POSITION[window_position]]]


class ROPE:
    """RoPE-DMAP encoder (``FD/ROPE.py:109-590``); fits on construction like the reference.

    Extra keyword ``precision`` selects the operator tiles ("ramp": 16-bit then
    fp32-class Lanczos stage, the default; "f16", "fp32", "f16x3").
    """

    def __init__(self, F_tX, L: int, rank: int = 20, beta: float | None = None, alpha: float = 1.0,
                 center: bool = True, scale: bool = False, drop_first: bool = True, step: int = 1,
                 sample_positions=None, rope_mode: str = "sample", window_position: str = "end",
                 pos_scale: float = 1.0, base: float = 10000.0, freqs=None, n_freqs: int | None = None,
                 beta_sample_pairs: int = 20000, seed: int = 0, precision: str = "ramp"):
        R = np.asarray(F_tX, dtype=float)
        if R.ndim == 1:
            R = R[:, None]
        self.center, self.scale = bool(center), bool(scale)
        self.mu_ = R.mean(axis=0, keepdims=True) if self.center else np.zeros((1, R.shape[1]))
        sd = R.std(axis=0, keepdims=True) if self.scale else np.ones((1, R.shape[1]))
        self.sigma_ = np.where(sd == 0, 1.0, sd)
        self.R_raw_ = R
        self.R_ = (R - self.mu_) / self.sigma_
        self.N_, self.D_ = R.shape
        self.L, self.step = int(L), int(step)
        self.K_ = self.N_ - (self.L - 1) * self.step
        if self.K_ <= 0:
            raise ValueError(f"N={self.N_} too small for L={self.L}, step={self.step}")
        self.rank_req_ = int(rank)
        self.beta_in_ = beta
        self.alpha_ = float(alpha)
        self.drop_first_ = bool(drop_first)
        if rope_mode not in ("sample", "window"):
            raise ValueError("rope_mode must be 'sample' or 'window'.")
        if window_position not in _WINDOW_POSITION:
            raise ValueError("window_position must be 'start', 'center', or 'end'.")
        self.rope_mode_ = rope_mode
        self.window_position_ = window_position
        self.pos_scale_ = float(pos_scale)
        self.base_ = float(base)
        self.freqs_in_ = None if freqs is None else np.asarray(freqs, dtype=float)
        self.n_freqs_ = None if n_freqs is None else int(n_freqs)
        if sample_positions is None:
            sample_positions = np.arange(self.N_, dtype=float)
        self.sample_positions_ = np.asarray(sample_positions, dtype=float)
        if self.sample_positions_.shape != (self.N_,):
            raise ValueError(f"sample_positions must have shape ({self.N_},).")
        self.beta_sample_pairs_ = int(beta_sample_pairs)
        self.rng_ = np.random.default_rng(int(seed))
        self.precision = precision
        self.G_ = None          # dense Gram: never formed
        self.Kmat_ = None       # dense kernel: never formed
        self.W_TcX_ = None
        self.Pos_ = None
        self.beta_ = self.lam_ = self.phi_ = self.psi_ = self.freqs_ = None
        self.K_T_ = self.d_T_ = self.inv_sqrt_d_ = self.r2_T_ = None
        self.dm_ = None
        self.fit()

    # ---- RoPE internals ---------------------------------------------------------
    def _freqs(self, dim: int) -> np.ndarray:
        """Frequency of each adjacent pair (``FD/ROPE.py:231-259``)."""
        n_pairs = dim // 2
        if n_pairs == 0:
            return np.zeros((0,))
        if self.freqs_in_ is not None:
            f = self.freqs_in_[:n_pairs]
            return np.concatenate([f, np.zeros(n_pairs - f.size)]) if f.size < n_pairs else f
        m = np.arange(n_pairs, dtype=float)
        f = self.base_ ** (-2.0 * m / max(2, 2 * n_pairs))
        if self.n_freqs_ is not None:
            f = f * (np.arange(n_pairs) < max(0, min(self.n_freqs_, n_pairs)))
        return f

    def _rotate(self, F, sT, sC, pos, pT, pC, K) -> torch.Tensor:
        """fd_rope_windows on device copies of F (raw, uncentred) and the positions."""
        dev = native.require_device()
        L, D = self.L, self.D_
        freqs = self._freqs(D if self.rope_mode_ == "sample" else L * D)
        self.freqs_ = freqs
        if self.pos_scale_ == 0.0:
            freqs = np.zeros(0)
        Fd = torch.as_tensor(np.ascontiguousarray(F, dtype=np.float64), device=dev)
        Pd = torch.as_tensor(np.ascontiguousarray(pos, dtype=np.float64), device=dev)
        fd_ = torch.as_tensor(np.ascontiguousarray(freqs, dtype=np.float64), device=dev)
        mu = torch.as_tensor(self.mu_.ravel(), dtype=torch.float64, device=dev)
        sg = torch.as_tensor(self.sigma_.ravel(), dtype=torch.float64, device=dev)
        Y = torch.empty((K, L * D), dtype=torch.float32, device=dev)
        c_w = (0, L // 2, L - 1)[_WINDOW_POSITION[self.window_position_]]
        native.check(native.load().fd_rope_windows(
            native._ptr(Fd), sT, sC, native._ptr(Pd), pT, pC, K, D, L, 1 if self.rope_mode_ == "window" else 0,
            c_w, self.pos_scale_, native._ptr(fd_) if freqs.size else None, int(freqs.size), native._ptr(mu),
            native._ptr(sg), native._ptr(Y), native._stream(dev)))
        return Y

    def _choose_beta(self, Y: torch.Tensor) -> float:
        """Median rule on seeded off-diagonal pairs, beta = 1/(median + 1e-12) (``FD/ROPE.py:347-369``)."""
        if self.beta_in_ is not None:
            return float(self.beta_in_)
        K = self.K_
        M = min(self.beta_sample_pairs_, K * (K - 1) // 2)
        if M <= 0:
            return 1.0
        ii = self.rng_.integers(0, K, size=M)
        jj = self.rng_.integers(0, K, size=M)
        keep = ii != jj
        ii, jj = ii[keep], jj[keep]
        if ii.size == 0:
            return 1.0
        a = torch.as_tensor(ii, device=Y.device)
        b = torch.as_tensor(jj, device=Y.device)
        d2 = ((Y[a].double() - Y[b].double()) ** 2).sum(1).cpu().numpy()
        return 1.0 / (np.median(d2) + 1e-12)

    # ---- training -----------------------------------------------------------------
    def fit(self) -> "ROPE":
        D, L, step = self.D_, self.L, self.step
        self.Pos_ = make_window_positions(self.sample_positions_, L, step, self.rope_mode_, self.window_position_)
        # windows read in place from the raw series (the kernel centres them)
        if self.rope_mode_ == "sample":
            Y = self._rotate(self.R_raw_, D, step * D, self.sample_positions_, 1, step, self.K_)
        else:
            c_w = (0, L // 2, L - 1)[_WINDOW_POSITION[self.window_position_]]
            Y = self._rotate(self.R_raw_, D, step * D, self.sample_positions_[c_w * step:], 1, 0, self.K_)
        self._Y = Y
        self.r2_T_ = (Y.double() ** 2).sum(1).cpu().numpy()
        self.beta_ = self._choose_beta(Y)
        k = min(self.rank_req_ + (1 if self.drop_first_ else 0), self.K_ - 1)
        dm = DiffusionMap(beta=self.beta_, alpha=self.alpha_, n_components=max(k, 1), precision=self.precision)
        dm.fit(Y)
        self.dm_ = dm
        if k <= 0:
            self.lam_ = np.zeros((0,))
            self.phi_ = np.zeros((self.K_, 0))
            self.psi_ = np.zeros((self.K_, 0))
        else:
            dm.transform()
            w, V = dm.eigenvalues_, dm.eigenvectors_
            if self.drop_first_ and w.size > 0:
                w, V = w[1:], V[:, 1:]
            self.lam_, self.phi_ = w, V
        # q(T) and d(T) of the fitted (most precise) state
        self.K_T_ = dm.D_ + 1e-18
        self.d_T_ = dm.D_alpha_ + 1e-18
        self.inv_sqrt_d_ = 1.0 / np.sqrt(self.d_T_)
        if k > 0:
            self.psi_ = self.inv_sqrt_d_[:, None] * self.phi_
        return self

    @property
    def Y_(self) -> np.ndarray:
        """Rotated training window vectors (K, L*D)."""
        return self._Y.double().cpu().numpy()

    # ---- encoding / Nystrom ---------------------------------------------------------
    def _prepare_query_windows(self, W_BLX, positions=None):
        """Validate query windows and build their positions (``FD/ROPE.py:446-487``)."""
        W = np.asarray(W_BLX, dtype=float)
        if W.ndim == 2:
            W = W[None, :, :]
        if W.ndim != 3:
            raise ValueError("Expected query windows with shape (B,L,D) or (L,D).")
        if W.shape[1:] != (self.L, self.D_):
            raise ValueError(f"Expected window shape (*,{self.L},{self.D_}), got {W.shape}")
        B = W.shape[0]
        if self.rope_mode_ == "sample":
            if positions is None:
                Pos = np.tile(np.arange(self.L, dtype=float), (B, 1))
            else:
                Pos = np.asarray(positions, dtype=float)
                if Pos.ndim == 1 and Pos.shape[0] == self.L:
                    Pos = np.tile(Pos[None, :], (B, 1))
                if Pos.shape != (B, self.L):
                    raise ValueError(f"For sample mode, positions must have shape ({B},{self.L}) or ({self.L},).")
            return W, Pos
        if positions is None:
            Pos = np.zeros((B,))
        else:
            Pos = np.asarray(positions, dtype=float)
            if Pos.ndim == 0:
                Pos = np.full((B,), float(Pos))
            if Pos.shape != (B,):
                raise ValueError(f"For window mode, positions must have shape ({B},) or scalar.")
        return W, Pos

    def encode_windows(self, W_BLX, positions=None) -> np.ndarray:
        """Nystrom coordinates (B, r) of query windows (``FD/ROPE.py:489-526``)."""
        if self.psi_ is None or self.lam_ is None or self.psi_.shape[1] == 0:
            B = 1 if np.asarray(W_BLX).ndim == 2 else np.asarray(W_BLX).shape[0]
            return np.zeros((B, 0))
        W, Pos = self._prepare_query_windows(W_BLX, positions)
        B, L, D = W.shape
        if self.rope_mode_ == "sample":
            Yq = self._rotate(W, L * D, D, Pos, L, 1, B)
        else:
            Yq = self._rotate(W, L * D, D, Pos, 1, 0, B)
        return self._nystrom(Yq)

    def _nystrom(self, Yq: torch.Tensor) -> np.ndarray:
        st = self.dm_._best_state()
        op = GaussianOperator(Yq, st.X, self.beta_, st.op.precision, shift=st.op.shift)
        dev = op.device
        a = self.alpha_
        wT = torch.as_tensor(self.K_T_ ** (-a), dtype=torch.float32, device=dev)
        Kq = op.apply(out_dtype=torch.float64)[:, 0] + 1e-18                 # row sums of k(q, T)
        wq = Kq ** (-a)
        dq = wq * op.apply(wT, out_dtype=torch.float64)[:, 0] + 1e-18        # sum_T k_alpha(q, T)
        lam_safe = np.maximum(self.lam_, 1e-12)
        V = torch.as_tensor(self.psi_ / lam_safe[None, :], dtype=torch.float64, device=dev)
        out = op.apply(V.contiguous(), col_scale=wT, row_scale=(wq / dq).float().contiguous(),
                       out_dtype=torch.float64)
        return out.cpu().numpy()

    def encode_window(self, W_cX, positions=None) -> np.ndarray:
        return self.encode_windows(np.asarray(W_cX)[None, :, :], positions=positions)[0]

    def encode_series(self, F_aX, sample_positions=None) -> np.ndarray:
        """Encode every Hankel window of a new series (``FD/ROPE.py:537-580``); windows read in place."""
        F = np.asarray(F_aX, dtype=float)
        if F.ndim == 1:
            F = F[:, None]
        N, D = F.shape
        if D != self.D_:
            raise ValueError(f"Expected D={self.D_}, got D={D}.")
        if sample_positions is None:
            sample_positions = np.arange(N, dtype=float)
        sample_positions = np.asarray(sample_positions, dtype=float)
        if sample_positions.shape != (N,):
            raise ValueError(f"sample_positions must have shape ({N},).")
        K = N - (self.L - 1) * self.step
        if K <= 0:
            raise ValueError(f"Need N={N} >= (L-1)*step+1 = {(self.L - 1) * self.step + 1}")
        if self.psi_ is None or self.psi_.shape[1] == 0:
            return np.zeros((K, 0))
        if self.rope_mode_ == "sample":
            Yq = self._rotate(F, D, self.step * D, sample_positions, 1, self.step, K)
        else:
            c_w = (0, self.L // 2, self.L - 1)[_WINDOW_POSITION[self.window_position_]]
            Yq = self._rotate(F, D, self.step * D, sample_positions[c_w * self.step:], 1, 0, K)
        return self._nystrom(Yq)

    @property
    def embedding_(self) -> np.ndarray:
        return self.psi_

    def fit_transform(self) -> np.ndarray:
        return self.psi_
