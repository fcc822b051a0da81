"""The FlashDiffusion primitive on B200 (sm_100a).

Public names and argument meanings follow the reference module
``FD/kernel.py`` of sparsetrace/FlashDiffusion (``FD/`` = ``src/flashdiffusion/``):

* ``FlashDiffusion(Q, K, V, beta, rscale_q, rscale_k, h, tile, coord_dtype, accum_dtype)``
  (``FD/kernel.py:189-257``)::

      out_i = rscale_q_i * sum_j exp(-beta ||q_i - k_j||^2) * rscale_k_j * h_j * V_j

* ``prepass_rowsum(Q, K, beta, weights_k, tile)`` (``FD/kernel.py:141-182``)
* ``_get_cuda_backend()`` / ``_SM_BACKEND`` (``FD/kernel.py:48-118``)

What differs: every call runs on the GPU through libfd_sm100 (tcgen05 bf16
tiles, or fp32 SIMT tiles), never on the host, and the kernel matrix is never
materialised.  The reference's ``tile`` argument (host tile size) is accepted
for compatibility; device tile shapes are fixed by the kernels.
``coord_dtype`` selects the tile precision: ``np.float32`` (the reference
default) runs fp32 tiles (relative error ~1e-6, the reference's own class),
``np.float16`` runs the tcgen05 tensor-core tiles with fp16 operands (relative
L2 error <= 2e-3; bf16 operands are used automatically when a point lies too
far from the data mean for the fp16 range), bfloat16 forces bf16 operands.
``precision="f16"|"bf16"|"fp32"`` overrides it.  NumPy inputs give NumPy
outputs of ``accum_dtype``; CUDA tensor inputs give CUDA tensors.
"""

from __future__ import annotations

from typing import Optional

import warnings

import numpy as np
import torch

from . import native

# SM -> kernel family.  This build ships the B200 family only.
_SM_BACKEND = {100: "sm100", 103: "sm100"}

TILE_NAMES = {"f16": native.TILE_F16, "bf16": native.TILE_BF16, "fp32": native.TILE_F32,
              "f16x3": native.TILE_F16X3}


def _cuda_sm() -> Optional[int]:
    if not torch.cuda.is_available():
        return None
    major, minor = torch.cuda.get_device_capability()
    return major * 10 + minor


def _get_cuda_backend():
    """Return ``(precompute_fn, matvec_fn)`` for the current device.

    Mirrors ``FD/kernel.py:68-118`` but never returns None: without a
    B200-class device or without the native library this raises, because the
    framework has no host fallback.
    """
    sm = _cuda_sm()
    if sm is None:
        raise RuntimeError("flashdiffusion_b200: no CUDA device visible (B200 / sm_100a required)")
    if _SM_BACKEND.get(sm) != "sm100":
        raise RuntimeError(f"flashdiffusion_b200: SM {sm} is not supported (B200 / sm_100a required)")
    from .kernel_cuda_sm100 import matvec_sm100, precompute_sm100
    native.load()
    return precompute_sm100, matvec_sm100


def tile_of(precision=None, coord_dtype=np.float32) -> int:
    """Tile code for a precision name or a reference ``coord_dtype``."""
    if precision is not None:
        if precision not in TILE_NAMES:
            raise ValueError(f"precision must be one of {sorted(TILE_NAMES)} (got {precision!r})")
        return TILE_NAMES[precision]
    if coord_dtype is torch.bfloat16:
        return native.TILE_BF16
    cd = np.dtype(coord_dtype) if not isinstance(coord_dtype, torch.dtype) else coord_dtype
    if cd in (np.dtype(np.float16), torch.float16):
        return native.TILE_F16
    # fp32 coordinates (the reference default): the fp32-class tensor-core
    # tiles, which meet the fp32 tiles' 1e-5 bound at the tensor-core rate; the
    # operator falls back to the fp32 SIMT tiles where they do not apply
    # (d > 136, or split values outside the fp16 range)
    return native.TILE_F16X3


PREC_OF_TILE = {v: k for k, v in TILE_NAMES.items()}


def to_device(x, dtype=None, device=None) -> Optional[torch.Tensor]:
    """NumPy / torch input -> contiguous CUDA tensor (None passes through)."""
    if x is None:
        return None
    dev = native.require_device(device)
    if isinstance(x, torch.Tensor):
        t = x.to(device=dev)
    else:
        t = torch.from_numpy(np.ascontiguousarray(x)).to(device=dev)
    if dtype is not None:
        t = t.to(dtype)
    return t.contiguous()


class GaussianOperator:
    """K(Q, K) = exp(-beta ||q_i - k_j||^2) resident in HBM as packed tile operands.

    This is the device-resident state the solvers reuse every iteration (the
    reference keeps the equivalent in ``CUDAStateSM100``,
    ``FD/kernel_cuda_sm100.py:52-64``).  Q and K are shifted by a common
    vector (the mean of K) before rounding; the kernel is translation
    invariant so the operator is unchanged.
    """

    def __init__(self, Q, K=None, beta: float = 1.0, precision: str = "f16", device=None, shift=None):
        self.device = native.require_device(device)
        Qd = to_device(Q, device=self.device)
        Kd = Qd if K is None else to_device(K, device=self.device)
        if Qd.dim() != 2 or Kd.dim() != 2 or Qd.shape[1] != Kd.shape[1]:
            raise ValueError(f"Q {tuple(Qd.shape)} and K {tuple(Kd.shape)} must be 2-D with the same d")
        if not beta > 0:
            raise ValueError(f"beta must be positive (got {beta})")
        self.beta = float(beta)
        self.precision = precision
        self.tile = TILE_NAMES[precision]
        self.nq, self.d = Qd.shape
        self.nk = Kd.shape[0]
        self.shift = native.mean_rows(Kd) if shift is None else shift
        if self.tile == native.TILE_F16X3 and self.d > 136:
            self.tile, self.precision = native.TILE_F32, "fp32"     # split operand rows would not fit
        if self.tile in (native.TILE_F16, native.TILE_F16X3):
            # fp16 operands unless some packed value would leave the fp16 range
            native.check_status(self.device)
            self.qop = native.pack(Qd, self.beta, native.SIDE_QUERY, self.tile, self.shift)
            self.kop = native.pack(Kd, self.beta, native.SIDE_KEY, self.tile, self.shift)
            try:
                native.check_status(self.device)
            except native.FDError as e:
                if e.code != native.FD_ERR_RANGE:
                    raise
                if self.tile == native.TILE_F16X3:
                    self.tile, self.precision = native.TILE_F32, "fp32"
                else:
                    # bf16 operands round 8x more coarsely: their matvec error
                    # budget is 1e-2, not the 2e-3 of the fp16 tiles
                    warnings.warn("flashdiffusion_b200: packed fp16 tile values would overflow for these points "
                                  "and beta; falling back to bf16 tiles, whose matvec relative error bound is "
                                  "1e-2 instead of 2e-3 (pass precision='f16x3' or 'fp32' for tighter results)",
                                  RuntimeWarning, stacklevel=2)
                    self.tile, self.precision = native.TILE_BF16, "bf16"
        if self.tile not in (native.TILE_F16, native.TILE_F16X3):
            self.qop = native.pack(Qd, self.beta, native.SIDE_QUERY, self.tile, self.shift)
            self.kop = native.pack(Kd, self.beta, native.SIDE_KEY, self.tile, self.shift)
        self.symmetric = K is None

    def apply(self, V=None, col_scale=None, col_h=None, row_scale=None, row_div=None,
              out_dtype=torch.float32, out=None) -> torch.Tensor:
        """diag(row_scale/row_div) K diag(col_scale*col_h) V  ->  (nq, r) device tensor."""
        return native.apply(self.qop, self.nq, self.kop, self.nk, self.d, self.tile, V,
                            col_scale=col_scale, col_h=col_h, row_scale=row_scale, row_div=row_div,
                            out_dtype=out_dtype, out=out)

    def with_precision(self, precision: str, Q=None, K=None) -> "GaussianOperator":
        """Same operator at another tile precision (needs the points again)."""
        return GaussianOperator(Q, K, self.beta, precision, self.device, self.shift)


def _f32(x, device):
    return None if x is None else to_device(x, torch.float32, device)


def prepass_rowsum(Q, K, beta: float, weights_k=None, tile: int = 512, precision=None,
                   coord_dtype=np.float32):
    """out_i = sum_j exp(-beta ||q_i - k_j||^2) * weights_k_j  (``FD/kernel.py:141-182``).

    Returns (N_q,) float64 (NumPy for NumPy inputs, CUDA tensor otherwise).
    """
    numpy_io = not isinstance(Q, torch.Tensor)
    op = GaussianOperator(Q, None if K is Q else K, beta, PREC_OF_TILE[tile_of(precision, coord_dtype)])
    w = _f32(weights_k, op.device)
    out = op.apply(w, out_dtype=torch.float64)[:, 0]
    return out.cpu().numpy() if numpy_io else out


def FlashDiffusion(Q, K, V, beta: float, rscale_q=None, rscale_k=None, h=None, tile: int = 512,
                   coord_dtype=np.float32, accum_dtype=np.float64, alpha: Optional[float] = None,
                   precision: Optional[str] = None, row_div=None):
    """The FlashDiffusion primitive (``FD/kernel.py:189-257``) on the GPU.

    out_i = rscale_q_i * sum_j exp(-beta ||q_i-k_j||^2) * rscale_k_j * h_j * V_j  [/ row_div_i]

    ``alpha`` (documented in the reference README but not implemented there):
    when given and both rscales are None, the Coifman-Lafon scales are computed
    first — DMAP normalisation of K (``FD/dmap.py:108-115``) and, for Q != K,
    the query normalisation of ``FD/utils.py:92-102``.  ``row_div`` divides
    each output row (the Doob normaliser, ``FD/dmap.py:249-261``).
    """
    numpy_io = not isinstance(Q, torch.Tensor)
    prec = PREC_OF_TILE[tile_of(precision, coord_dtype)]
    same = K is Q
    op = GaussianOperator(Q, None if same else K, beta, prec)
    dev = op.device
    Vd = to_device(V, device=dev)
    if Vd.dtype not in (torch.float32, torch.float64):
        Vd = Vd.double()
    squeeze = Vd.dim() == 1
    if squeeze:
        Vd = Vd[:, None]
    if Vd.shape[0] != op.nk:
        raise ValueError(f"V has {Vd.shape[0]} rows, K has {op.nk}")
    rq, rk = _f32(rscale_q, dev), _f32(rscale_k, dev)
    if alpha is not None and rq is None and rk is None:
        kop = op if same else GaussianOperator(K, None, beta, prec, dev, op.shift)
        D = kop.apply(out_dtype=torch.float32)[:, 0].contiguous()
        w = native.dmap_weights(D, alpha)
        Kw = kop.apply(w, out_dtype=torch.float32)[:, 0].contiguous()
        _, rk = native.dmap_rscale(Kw, w)
        if same:
            rq = rk
        else:
            Dq = op.apply(w, out_dtype=torch.float32)[:, 0].contiguous()   # D_q = K(Q,K) w_k
            wq = native.dmap_weights(Dq, alpha)
            _, rq = native.dmap_rscale(Dq, wq)       # D_alpha_q = D_q w_q; rscale_q = D_alpha_q^-1/2 w_q
    out = op.apply(Vd, col_scale=rk, col_h=_f32(h, dev), row_scale=rq, row_div=_f32(row_div, dev),
                   out_dtype=torch.float64 if np.dtype(accum_dtype) == np.float64 else torch.float32)
    if numpy_io:
        return out.cpu().numpy().astype(accum_dtype, copy=False)
    return out
