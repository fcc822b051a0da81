"""Bandwidth selection and the Nystrom extension (reference ``FD/utils.py``), on the GPU.

``median_bandwidth`` and ``knn_bandwidth`` keep the reference's names, arguments
and return values; the O(m^2) / O(N^2) distance work runs in libfd_sm100.so
(``fd_pairwise_sqdist``, ``fd_knn_sqdist``: fp32 coordinate differences on the
CUDA cores, the k smallest per row kept in registers, so no N x N matrix is
formed or sorted; ``fd_knn_sqdist_tc``: every pair screened on the tensor cores,
the candidates refined with the same exact arithmetic).  The seeded subsample of the median rule is drawn on the host
exactly as the reference draws it.
"""

from __future__ import annotations

import numpy as np
import torch

from . import native
from .kernel import to_device

__all__ = ["median_bandwidth", "knn_bandwidth", "knn_sqdist", "nystrom_extend", "to_f32", "to_f64"]


def median_bandwidth(X, subsample: int = 2000) -> float:
    """beta = 1 / (2 median(||x_i - x_j||^2 > 0)) over a seeded subsample (``FD/utils.py:16-28``)."""
    dev = native.require_device()
    Xh = X.detach().cpu().numpy() if isinstance(X, torch.Tensor) else np.asarray(X)
    N = Xh.shape[0]
    if N > subsample:
        Xh = Xh[np.random.default_rng(0).choice(N, subsample, replace=False)]
    Xd = to_device(np.ascontiguousarray(Xh), torch.float32, dev).contiguous()
    m, d = Xd.shape
    d2 = torch.empty((m, m), dtype=torch.float32, device=dev)
    native.check(native.load().fd_pairwise_sqdist(native._ptr(Xd), m, d, native._ptr(d2), native._stream(dev)))
    pos = d2[d2 > 0]
    if pos.numel() == 0:
        return 1.0
    s = torch.sort(pos.double()).values
    n = s.numel()
    med = float(s[n // 2]) if n % 2 else 0.5 * float(s[n // 2 - 1] + s[n // 2])
    return 1.0 / (2.0 * med) if med > 0 else 1.0


def knn_sqdist(Q, K=None, k: int = 8, method: str = "auto") -> torch.Tensor:
    """(N_q, k) device fp32: the k smallest squared distances of each query row to the keys, ascending.

    ``method``: "tc" screens every pair on the tensor cores and refines the
    candidates exactly (``fd_knn_sqdist_tc``: d <= 66, k <= 24), "simt" runs
    the CUDA-core kernel (``fd_knn_sqdist``: any d <= 1024, k <= 64), "auto"
    takes "tc" where it applies.  Both return the same exactly computed
    squared distances (fp32 coordinate differences)."""
    dev = native.require_device()
    Qd = to_device(Q, torch.float32, dev).contiguous()
    Kd = Qd if K is None else to_device(K, torch.float32, dev).contiguous()
    nq, d = Qd.shape
    nk = Kd.shape[0]
    out = torch.empty((nq, k), dtype=torch.float32, device=dev)
    lib = native.load()
    if method not in ("auto", "tc", "simt"):
        raise ValueError(f"method must be auto, tc or simt (got {method!r})")
    if method == "tc" or (method == "auto" and d <= 66 and k <= 24 and 1 <= k <= nk and nq > 0):
        nb = int(lib.fd_knn_tc_workspace_bytes(nq, nk, d, k))
        ws = torch.empty(nb + 256, dtype=torch.uint8, device=dev)
        base = ws.data_ptr()
        aligned = (base + 255) & ~255
        native.check(lib.fd_knn_sqdist_tc(native._ptr(Qd), nq, native._ptr(Kd), nk, d, k, native._ptr(out),
                                          native.ctypes.c_void_p(aligned), nb, native._stream(dev)))
        return out
    native.check(lib.fd_knn_sqdist(native._ptr(Qd), nq, native._ptr(Kd), nk, d, k,
                                   native._ptr(out), native._stream(dev)))
    return out


def knn_bandwidth(X, k: int = 7) -> np.ndarray:
    """Self-tuning per-point bandwidth sigma_i = ||x_i - x_(i,k)|| (``FD/utils.py:31-52``).

    Index 0 is the point itself (distance 0), as in the reference's sorted rows.
    Returns sigma (N,) fp64, floored at 1e-10.
    """
    d2 = knn_sqdist(X, None, k + 1)[:, k]
    return np.maximum(np.sqrt(d2.double().cpu().numpy()), 1e-10)


def nystrom_extend(dm, X_new, t: int = 1) -> np.ndarray:
    """Out-of-sample coordinates of a fitted, transformed DiffusionMap (``FD/utils.py:59-123``)."""
    return dm.nystrom(X_new, t=t)


def to_f32(X) -> np.ndarray:
    """dtype helper of the reference (``FD/utils.py:130-131``)."""
    return np.asarray(X, dtype=np.float32)


def to_f64(X) -> np.ndarray:
    """dtype helper of the reference (``FD/utils.py:133-134``)."""
    return np.asarray(X, dtype=np.float64)
