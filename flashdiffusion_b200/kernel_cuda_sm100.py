"""B200 backend behind the reference's backend contract.

Same names and contract as ``FD/kernel_cuda_sm100.py`` of the reference
(``CUDAStateSM100`` ``:52-64``, ``precompute_sm100`` ``:67-103``,
``matvec_sm100`` ``:106-119``): ``precompute_sm100(X, beta, alpha)`` runs the
two Coifman-Lafon prepasses on the GPU and returns a state whose ``.D``,
``.D_alpha`` and ``.rscale`` are CUDA tensors; ``matvec_sm100(state, v)``
applies M = diag(rscale) K diag(rscale) to a NumPy vector and returns float64.

The kernels are this package's sm_100a tcgen05 tiles (fp16 operands like the
reference's X_fp16, fp32 accumulation) instead of the reference's WMMA
kernel; ``precision="fp32"`` selects the fp32 tiles.
"""

from __future__ import annotations

import time

import numpy as np
import torch

from . import native
from .kernel import GaussianOperator, to_device


class CUDAStateSM100:
    """Device-resident normalised DMAP operator."""

    def __init__(self, op: GaussianOperator, rscale, D, D_alpha, beta, alpha, X=None):
        self.op = op
        self.X = X            # device copy of the points (for re-packing at another precision)
        self.rscale = rscale
        self.D = D
        self.D_alpha = D_alpha
        self.beta = beta
        self.alpha = alpha
        self.N = op.nq
        self.d = op.d
        self.timings = {}

    def matvec_device(self, v: torch.Tensor, out_dtype=torch.float64) -> torch.Tensor:
        """M v for a device vector (N,) or block (N, r); no host round trip."""
        squeeze = v.dim() == 1
        out = self.op.apply(v[:, None] if squeeze else v, col_scale=self.rscale, row_scale=self.rscale,
                            out_dtype=out_dtype)
        return out[:, 0] if squeeze else out


def normalise(op: GaussianOperator, alpha: float):
    """Two prepasses (``FD/kernel_cuda_sm100.py:89-98``): D, w = D^-alpha, D_alpha, rscale."""
    D = op.apply(out_dtype=torch.float32)[:, 0].contiguous()
    w = native.dmap_weights(D, alpha)
    Kw = op.apply(w, out_dtype=torch.float32)[:, 0].contiguous()
    D_alpha, rscale = native.dmap_rscale(Kw, w)
    return D, D_alpha, rscale


def precompute_sm100(X, beta: float, alpha: float = 0.5, precision: str = "f16") -> CUDAStateSM100:
    """Two-pass Coifman-Lafon precomputation on the GPU."""
    Xd = to_device(X)
    op = GaussianOperator(Xd, None, beta, precision)
    t0 = time.perf_counter()
    D, D_alpha, rscale = normalise(op, alpha)
    torch.cuda.synchronize()
    st = CUDAStateSM100(op, rscale, D, D_alpha, beta, alpha, X=Xd)
    st.timings["precompute_s"] = time.perf_counter() - t0
    return st


def matvec_sm100(state: CUDAStateSM100, v: np.ndarray) -> np.ndarray:
    """M v for a host vector; float64 out (the reference copies v H2D and out D2H each call)."""
    vd = torch.from_numpy(np.ascontiguousarray(v, dtype=np.float64)).to(state.op.device, non_blocking=False)
    return state.matvec_device(vd).cpu().numpy()
