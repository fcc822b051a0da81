"""ctypes binding of libfd_sm100.so (C ABI in include/fd_sm100.h) on torch tensors.

torch is used only as plumbing: device memory, the current CUDA stream and
the caching allocator for workspaces.  Every O(N^2) operation runs in the
library's own sm_100a kernels.  There is no CPU fallback: if the library or a
B200-class device is missing, calls raise.
"""

from __future__ import annotations

import ctypes
import os
import threading

import torch

PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG, "libfd_sm100.so")

FD_OK, FD_ERR_ARG, FD_ERR_CUDA, FD_ERR_UNSUPPORTED, FD_ERR_TIMEOUT, FD_ERR_WORKSPACE, FD_ERR_RANGE = range(7)
DTYPE_F32, DTYPE_F16, DTYPE_BF16, DTYPE_F64 = range(4)
TILE_BF16, TILE_F32, TILE_F16, TILE_F16X3 = 0, 1, 2, 3
SIDE_QUERY, SIDE_KEY = 0, 1

_TORCH_DTYPE = {torch.float32: DTYPE_F32, torch.float16: DTYPE_F16, torch.bfloat16: DTYPE_BF16,
                torch.float64: DTYPE_F64}

# every symbol declared in include/fd_sm100.h: (restype, argtypes)
_P, _I, _L, _F, _S = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float, ctypes.c_size_t
SIGNATURES = {
    "fd_last_error": (ctypes.c_char_p, []),
    "fd_version": (_I, []),
    "fd_device_supported": (_I, [_I]),
    "fd_check_status": (_I, [_P]),
    "fd_compute_sq_norms": (_I, [_P, _I, _L, _I, _P, _P]),
    "fd_prepass": (_I, [_P, _I, _L, _I, _P, _F, _I, _P, _P, _S, _P]),
    "fd_matvec": (_I, [_P, _I, _L, _I, _P, _P, _F, _I, _P, _P, _S, _P]),
    "fd_workspace_bytes": (_S, [_L, _L, _I, _I, _I]),
    "fd_flash_diffusion": (_I, [_P, _P, _I, _L, _L, _I, _P, _I, _F, _P, _P, _P, _P, _I, _P, _P, _S, _P]),
    "fd_operand_bytes": (_S, [_L, _I, _I]),
    "fd_mean_rows": (_I, [_P, _I, _L, _I, _P, _P]),
    "fd_pack_operand": (_I, [_P, _I, _L, _I, _P, _F, _I, _I, _P, _P]),
    "fd_apply_workspace_bytes": (_S, [_L, _L, _I, _I]),
    "fd_apply": (_I, [_P, _L, _P, _L, _I, _I, _P, _I, _I, _P, _P, _P, _P, _P, _I, _P, _S, _P]),
    "fd_apply_noalloc": (_I, [_P, _L, _P, _L, _I, _I, _P, _I, _I, _P, _P, _P, _P, _P, _I, _P]),
    "fd_dmap_weights": (_I, [_P, _L, _F, _P, _P]),
    "fd_dmap_rscale": (_I, [_P, _P, _L, _P, _P, _P]),
    "fd_set_block_options": (_I, [_I, _I]),
    "fd_selftest_wait_timeout": (_I, [_L, _P]),
    "fd_set_exp2_fma_cols": (_I, [_I]),
    "fd_lanczos_workspace_bytes": (_S, [_L, _I]),
    "fd_comm_id_bytes": (_S, []),
    "fd_comm_get_id": (_I, [_P]),
    "fd_comm_init": (_I, [_P, _P, _I, _I]),
    "fd_comm_allgather": (_I, [_P, _P, _P, _S, _P]),
    "fd_comm_check": (_I, [_P]),
    "fd_comm_abort": (_I, [_P]),
    "fd_comm_destroy": (_I, [_P]),
    "fd_lanczos_reorth": (_I, [_P, _L, _I, _L, _P, _P, _P, _P, _S, _P]),
    "fd_selftest_exp2_poly": (_I, [_P, _L, _P, _P]),
    "fd_knn_sqdist": (_I, [_P, _L, _P, _L, _I, _I, _P, _P]),
    "fd_pairwise_sqdist": (_I, [_P, _L, _I, _P, _P]),
    "fd_knn_tc_workspace_bytes": (_S, [_L, _L, _I, _I]),
    "fd_knn_sqdist_tc": (_I, [_P, _L, _P, _L, _I, _I, _P, _P, _S, _P]),
    "fd_rope_windows": (_I, [_P, _L, _L, _P, _L, _L, _L, _I, _I, _I, _I, ctypes.c_double, _P, _I, _P, _P, _P,
                             _P]),
}

_lib = None
_lock = threading.Lock()


class FDError(RuntimeError):
    """Error returned by libfd_sm100 (status code in ``.code``)."""

    def __init__(self, code, msg):
        super().__init__(f"libfd_sm100 error {code}: {msg}")
        self.code = code


def load(path: str | None = None) -> ctypes.CDLL:
    """Load (once) and return the native library; raises ImportError if absent."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        p = path or LIB_PATH
        if not os.path.exists(p):
            raise ImportError(f"{p} not built: run `python -m flashdiffusion_b200.build` (needs nvcc)")
        lib = ctypes.CDLL(p)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


def check(rc: int) -> None:
    if rc != FD_OK:
        raise FDError(rc, load().fd_last_error().decode())


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(device=None):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def require_device(device=None) -> torch.device:
    """The CUDA device to run on; raises unless it is a B200-class (sm_100) GPU."""
    if not torch.cuda.is_available():
        raise RuntimeError("flashdiffusion_b200 needs a CUDA B200 (sm_100a) device; none is visible")
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    if dev.type != "cuda":
        raise RuntimeError(f"flashdiffusion_b200 runs on CUDA devices only (got {dev})")
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    if not load().fd_device_supported(idx):
        cap = torch.cuda.get_device_capability(idx)
        raise RuntimeError(f"device {idx} has compute capability {cap}; libfd_sm100 needs 10.x (B200)")
    return torch.device("cuda", idx)


class _Workspace:
    """Per-device grow-only scratch buffer handed to the library."""

    def __init__(self):
        self.buf = {}

    def get(self, nbytes: int, device) -> torch.Tensor:
        key = (device.index, torch.cuda.current_stream(device).cuda_stream)
        b = self.buf.get(key)
        if b is None or b.numel() < nbytes:
            b = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=device)
            self.buf[key] = b
        return b


workspace = _Workspace()


def _as_input(X: torch.Tensor) -> torch.Tensor:
    if X.dtype not in _TORCH_DTYPE:
        X = X.float()
    return X.contiguous()


def mean_rows(X: torch.Tensor) -> torch.Tensor:
    X = _as_input(X)
    n, d = X.shape
    shift = torch.empty(d, dtype=torch.float32, device=X.device)
    check(load().fd_mean_rows(_ptr(X), _TORCH_DTYPE[X.dtype], n, d, _ptr(shift), _stream(X.device)))
    return shift


def operand_bytes(n: int, d: int, tile: int) -> int:
    return int(load().fd_operand_bytes(n, d, tile))


def pack(X: torch.Tensor, beta: float, side: int, tile: int, shift: torch.Tensor | None) -> torch.Tensor:
    """Pack points into a tile operand (device uint8 buffer)."""
    X = _as_input(X)
    n, d = X.shape
    op = torch.empty(max(operand_bytes(n, d, tile), 256), dtype=torch.uint8, device=X.device)
    check(load().fd_pack_operand(_ptr(X), _TORCH_DTYPE[X.dtype], n, d, _ptr(shift), float(beta), side, tile,
                                 _ptr(op), _stream(X.device)))
    return op


def apply(qop, nq, kop, nk, d, tile, V=None, r=1, col_scale=None, col_h=None, row_scale=None,
          row_div=None, out_dtype=torch.float32, out=None) -> torch.Tensor:
    """out = diag(row_scale/row_div) K diag(col_scale*col_h) V on resident operands."""
    dev = qop.device
    if V is not None:
        if V.dtype not in (torch.float32, torch.float64):
            V = V.float()
        V = V.contiguous()
        r = 1 if V.dim() == 1 else V.shape[1]
    for t in (col_scale, col_h, row_scale, row_div):
        if t is not None and (t.dtype != torch.float32 or not t.is_contiguous()):
            raise TypeError("scale vectors must be contiguous float32 device tensors")
    if out is None:
        out = torch.empty((nq, r), dtype=out_dtype, device=dev)
    lib = load()
    nbytes = int(lib.fd_apply_workspace_bytes(nq, nk, r, tile))
    ws = workspace.get(nbytes, dev)
    check(lib.fd_apply(_ptr(qop), nq, _ptr(kop), nk, d, tile, _ptr(V),
                       DTYPE_F64 if (V is not None and V.dtype == torch.float64) else DTYPE_F32, r,
                       _ptr(col_scale), _ptr(col_h), _ptr(row_scale), _ptr(row_div), _ptr(out),
                       DTYPE_F64 if out.dtype == torch.float64 else DTYPE_F32, _ptr(ws), ws.numel(),
                       _stream(dev)))
    return out


def dmap_weights(D: torch.Tensor, alpha: float) -> torch.Tensor:
    w = torch.empty_like(D)
    check(load().fd_dmap_weights(_ptr(D), D.numel(), float(alpha), _ptr(w), _stream(D.device)))
    return w


def dmap_rscale(Kw: torch.Tensor, w: torch.Tensor):
    Da = torch.empty_like(Kw)
    rs = torch.empty_like(Kw)
    check(load().fd_dmap_rscale(_ptr(Kw), _ptr(w), Kw.numel(), _ptr(Da), _ptr(rs), _stream(Kw.device)))
    return Da, rs


def set_block_options(group_tiles: int = 0, products: int = 0) -> None:
    """Block-path options for later launches (0 = default); see include/fd_sm100.h."""
    check(load().fd_set_block_options(int(group_tiles), int(products)))


def set_exp2_fma_cols(cols: int = -1) -> None:
    """Columns per 16 of the 16-bit r = 1 epilogue on the FMA-pipe exp2 (-1 = default)."""
    check(load().fd_set_exp2_fma_cols(int(cols)))


def exp2_poly(x: torch.Tensor) -> torch.Tensor:
    """The epilogues' FMA-pipe 2^x on a float32 device tensor (self-test entry point)."""
    x = x.contiguous()
    y = torch.empty_like(x)
    check(load().fd_selftest_exp2_poly(_ptr(x), x.numel(), _ptr(y), _stream(x.device)))
    return y


LANCZOS_MAX_ROWS = 96


def lanczos_workspace(n: int, rows: int, device) -> torch.Tensor:
    """Workspace for ``lanczos_reorth`` with up to ``rows`` basis rows."""
    nb = int(load().fd_lanczos_workspace_bytes(int(n), int(rows)))
    return torch.empty(nb + 256, dtype=torch.uint8, device=device)


def lanczos_reorth(V: torch.Tensor, rows: int, w: torch.Tensor, out: torch.Tensor, coef: torch.Tensor,
                   ws: torch.Tensor) -> None:
    """CGS2 of w (overwritten) against V[:rows]: coef[:rows] = projections,
    coef[rows] = beta, out = w2 / beta.  fp64 device tensors; no host sync."""
    for t in (V, w, out, coef):
        if t.dtype != torch.float64 or not t.is_cuda:
            raise TypeError("lanczos_reorth: fp64 CUDA tensors expected")
    if V.stride(1) != 1 or not (w.is_contiguous() and out.is_contiguous() and coef.is_contiguous()):
        raise ValueError("lanczos_reorth: contiguous rows expected")
    base = ws.data_ptr()
    aligned = (base + 255) & ~255
    check(load().fd_lanczos_reorth(_ptr(V), V.stride(0), int(rows), V.shape[1], _ptr(w), _ptr(out), _ptr(coef),
                                   ctypes.c_void_p(aligned), ws.numel() - (aligned - base), _stream(V.device)))


class Comm:
    """The library's NCCL communicator (fd_comm_*), for hosts without torch.distributed.

    ``Comm.new_id()`` on one rank; pass the bytes to every rank; ``Comm(id, nranks, rank)``."""

    @staticmethod
    def new_id() -> bytes:
        lib = load()
        buf = ctypes.create_string_buffer(int(lib.fd_comm_id_bytes()))
        check(lib.fd_comm_get_id(buf))
        return buf.raw

    def __init__(self, uid: bytes, nranks: int, rank: int):
        self.handle = ctypes.c_void_p()
        check(load().fd_comm_init(ctypes.byref(self.handle), ctypes.create_string_buffer(uid, len(uid)),
                                  int(nranks), int(rank)))
        self.nranks, self.rank = nranks, rank

    def allgather_(self, buf: torch.Tensor) -> torch.Tensor:
        """In-place all-gather: chunk ``rank`` of the contiguous ``buf`` (split in nranks) to every rank."""
        chunk = buf.numel() * buf.element_size() // self.nranks
        send = ctypes.c_void_p(buf.data_ptr() + self.rank * chunk)
        check(load().fd_comm_allgather(self.handle, send, _ptr(buf), chunk, _stream(buf.device)))
        return buf

    def check(self) -> None:
        check(load().fd_comm_check(self.handle))

    def abort(self) -> None:
        check(load().fd_comm_abort(self.handle))
        self.handle = ctypes.c_void_p()

    def close(self) -> None:
        check(load().fd_comm_destroy(self.handle))
        self.handle = ctypes.c_void_p()


def check_status(device=None) -> None:
    """Raise FDError if a bounded device-side wait gave up since the last check."""
    check(load().fd_check_status(_stream(device)))
