"""Carre du Champ operator and diffusion metric tensor (reference ``FD/cdc.py``) on the GPU.

Gamma(phi_k, phi_l)(i) = (P+(phi_k phi_l)(i) - lambda_k phi_k(i) phi_l(i) - lambda_l phi_l(i) phi_k(i)) / 2
with P+ = diag(w / D_alpha) K diag(w), w = D^-alpha — the reference's formula as
written (``FD/cdc.py:96-104``; it has no ``+ phi_k phi_l`` term, and it is kept).

``metric_tensor`` batches the products of all requested pairs into ONE block
right-hand side, so the k(k+1)/2 applications of P+ are a single tile pass with
r = number of pairs (the block tensor-core kernel, 32 columns per launch),
instead of one pass per pair; G and M = sum_i G_i G_i^T stay on the device until
returned.  The operator is the map's most precise fitted state (fp32-class after
the precision ramp).
"""

from __future__ import annotations

from typing import Optional

import numpy as np
import torch

from . import native

__all__ = ["carre_du_champ", "metric_tensor", "apply_pplus"]


def _state(dm):
    dm._check_fitted()
    return dm._best_state()


def apply_pplus(dm, F) -> torch.Tensor:
    """P+ F for a host or device (N,) / (N, r) array; returns device fp64 of F's shape (``FD/cdc.py:107-130``)."""
    st = _state(dm)
    Fd = torch.as_tensor(np.asarray(F) if not isinstance(F, torch.Tensor) else F).to(st.op.device, torch.float64)
    squeeze = Fd.dim() == 1
    w = native.dmap_weights(st.D, dm.alpha)
    left = (w.double() / st.D_alpha.double()).float().contiguous()
    out = st.op.apply(Fd[:, None] if squeeze else Fd.contiguous(), col_scale=w, row_scale=left,
                      out_dtype=torch.float64)
    return out[:, 0] if squeeze else out


def carre_du_champ(dm, phi_k, phi_l, lambda_k: float, lambda_l: float) -> np.ndarray:
    """Gamma(phi_k, phi_l) for all points (``FD/cdc.py:45-104``); phi in the P+ basis (vecs / rscale)."""
    dev = _state(dm).op.device
    pk = torch.as_tensor(np.asarray(phi_k), dtype=torch.float64, device=dev)
    pl = torch.as_tensor(np.asarray(phi_l), dtype=torch.float64, device=dev)
    pkl = pk * pl
    return (0.5 * (apply_pplus(dm, pkl) - lambda_k * pkl - lambda_l * pkl)).cpu().numpy()


def metric_tensor(dm, eigenvalues, eigenvectors, pairs: Optional[list] = None):
    """G (N, k, k) with G[i,k,l] = Gamma(phi_k, phi_l)(i), and M = sum_i G_i G_i^T (``FD/cdc.py:133-168``)."""
    dev = _state(dm).op.device
    lam = np.asarray(eigenvalues, dtype=np.float64)
    k = lam.shape[0]
    phi = torch.as_tensor(np.asarray(eigenvectors), dtype=torch.float64, device=dev)
    N = phi.shape[0]
    if pairs is None:
        pairs = [(i, j) for i in range(k) for j in range(i, k)]
    a = torch.tensor([p[0] for p in pairs], device=dev)
    b = torch.tensor([p[1] for p in pairs], device=dev)
    prods = phi[:, a] * phi[:, b]                                # (N, pairs): one block right-hand side
    lam_d = torch.as_tensor(lam, device=dev)
    gam = 0.5 * (apply_pplus(dm, prods) - (lam_d[a] + lam_d[b])[None, :] * prods)
    G = torch.zeros((N, k, k), dtype=torch.float64, device=dev)
    G[:, a, b] = gam
    G[:, b, a] = gam
    M = torch.einsum("ikm,ilm->kl", G, G)
    return G.cpu().numpy(), M.cpu().numpy()


def _apply_Pplus(dm, f) -> np.ndarray:
    """The reference's private name for P+ f (``FD/cdc.py:103-130``), host in and out."""
    return apply_pplus(dm, f).cpu().numpy()
