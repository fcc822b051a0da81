"""Drop-in for the reference's compiled module ``flash_diffusion_sm100``.

The reference builds a pybind11 module of that name from
``FD/csrc/flash_diffusion_sm100.cu`` (bindings ``:456-588``) with three
functions on CUDA tensors.  This module keeps the names, argument order,
shapes and RuntimeError-on-bad-input behaviour, and routes them to
libfd_sm100's C ABI (``fd_compute_sq_norms``, ``fd_prepass``, ``fd_matvec``).

Differences, by design: X may be float16, bfloat16 or float32 (the reference
accepts float16 only); the kernels evaluate distances from their own rounded
fp16 tile operands (norms folded into the operand), so ``sq_X`` is checked for
shape but not read.
"""

from __future__ import annotations

import torch

from . import native


def _check_x(X, name="X_fp16"):
    if not isinstance(X, torch.Tensor) or not X.is_cuda:
        raise RuntimeError(f"{name} must be CUDA")
    if X.dtype not in (torch.float16, torch.bfloat16, torch.float32):
        raise RuntimeError(f"{name} must be float16/half (bfloat16 and float32 are also accepted)")
    if X.dim() != 2:
        raise RuntimeError(f"{name} must be 2D")
    if not X.is_contiguous():
        raise RuntimeError(f"{name} must be contiguous")


def _check_vec(x, n, name):
    if not isinstance(x, torch.Tensor) or not x.is_cuda:
        raise RuntimeError(f"{name} must be CUDA")
    if x.dtype != torch.float32:
        raise RuntimeError(f"{name} must be float32")
    if x.dim() != 1:
        raise RuntimeError(f"{name} must be 1D")
    if not x.is_contiguous():
        raise RuntimeError(f"{name} must be contiguous")
    if x.shape[0] != n:
        raise RuntimeError(f"{name} length must equal N")


def _ws(n, d):
    lib = native.load()
    nbytes = int(lib.fd_workspace_bytes(n, n, d, 1, native.TILE_F16))
    return native.workspace.get(nbytes, torch.device("cuda", torch.cuda.current_device()))


def compute_sq_norms(X_fp16: torch.Tensor) -> torch.Tensor:
    _check_x(X_fp16)
    n, d = X_fp16.shape
    sq = torch.empty(n, dtype=torch.float32, device=X_fp16.device)
    native.check(native.load().fd_compute_sq_norms(native._ptr(X_fp16), native._TORCH_DTYPE[X_fp16.dtype], n, d,
                                                   native._ptr(sq), native._stream(X_fp16.device)))
    return sq


def prepass(X_fp16: torch.Tensor, w: torch.Tensor, sq_X: torch.Tensor, beta: float) -> torch.Tensor:
    _check_x(X_fp16)
    n, d = X_fp16.shape
    _check_vec(w, n, "w")
    _check_vec(sq_X, n, "sq_X")
    D = torch.empty(n, dtype=torch.float32, device=X_fp16.device)
    ws = _ws(n, d)
    native.check(native.load().fd_prepass(native._ptr(X_fp16), native._TORCH_DTYPE[X_fp16.dtype], n, d,
                                          native._ptr(w), float(beta), native.TILE_F16, native._ptr(D),
                                          native._ptr(ws), ws.numel(), native._stream(X_fp16.device)))
    return D


def matvec(X_fp16: torch.Tensor, v: torch.Tensor, rscale: torch.Tensor, sq_X: torch.Tensor,
           beta: float) -> torch.Tensor:
    _check_x(X_fp16)
    n, d = X_fp16.shape
    _check_vec(v, n, "v")
    _check_vec(rscale, n, "rscale")
    _check_vec(sq_X, n, "sq_X")
    out = torch.empty(n, dtype=torch.float32, device=X_fp16.device)
    ws = _ws(n, d)
    native.check(native.load().fd_matvec(native._ptr(X_fp16), native._TORCH_DTYPE[X_fp16.dtype], n, d,
                                         native._ptr(v), native._ptr(rscale), float(beta), native.TILE_F16,
                                         native._ptr(out), native._ptr(ws), ws.numel(),
                                         native._stream(X_fp16.device)))
    return out
