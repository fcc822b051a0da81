"""Row-sharded operator over several GPUs of one node (one process per GPU).

Sharding (the reference has no distributed code; this is new): output rows
are independent given all of K and the full right-hand side, so rank r owns a
contiguous block of 256-row tiles of Q and holds all of K.  A matvec is one
local tile pass over the rank's rows followed by ONE collective, an NCCL
all-gather of the output shards (NVLink / NVSwitch), so every rank ends with
the full vector and can run the (replicated, deterministic) fp64 Krylov
update locally.  The prepass needs the same gather twice (D, then K w).
"""

from __future__ import annotations

from typing import Callable, Optional

import torch
import torch.distributed as dist

ROW_TILE = 256


def shard_rows(n: int, world: int, rank: int, tile: int = ROW_TILE):
    """[begin, end) rows of rank ``rank``: contiguous tiles, sizes differ by at most one tile."""
    n_t = (n + tile - 1) // tile
    t0 = rank * n_t // world
    t1 = (rank + 1) * n_t // world
    return min(t0 * tile, n), min(t1 * tile, n)


def all_shards(n: int, world: int, tile: int = ROW_TILE):
    return [shard_rows(n, world, r, tile) for r in range(world)]


class RowGather:
    """All-gather of uneven contiguous row shards into the full (n, r) array.

    NCCL gathers equal-sized chunks, so each rank's chunk is its shard padded
    to the largest shard.  The padded buffer is allocated once per (r, dtype)
    and reused; the tile kernel writes this rank's rows straight into its chunk
    (``slot``), the all-gather runs in place, and the result is a view of the
    buffer when every shard has the same size, else one gather-copy of the
    valid rows.
    """

    def __init__(self, n: int, world: int, group=None):
        self.n = n
        self.world = world
        self.group = group
        self.shards = all_shards(n, world)
        self.maxrows = max(b - a for a, b in self.shards)
        self.rank = dist.get_rank(group) if (world > 1 and dist.is_initialized()) else 0
        self.equal = all(b - a == self.maxrows for a, b in self.shards)
        self._bufs = {}
        self._index = None

    def _buf(self, r: int, dtype, device) -> torch.Tensor:
        key = (r, dtype, str(device))
        if key not in self._bufs:
            self._bufs[key] = torch.empty((self.world * self.maxrows, r), dtype=dtype, device=device)
        return self._bufs[key]

    def slot(self, r: int, dtype, device) -> torch.Tensor:
        """This rank's (rows, r) chunk of the gather buffer, for the kernel to write into."""
        a, b = self.shards[self.rank]
        off = self.rank * self.maxrows
        return self._buf(r, dtype, device)[off: off + (b - a)]

    def gather_slot(self, r: int, dtype, device) -> torch.Tensor:
        """All-gather the chunks written through ``slot``; returns the full (n, r) rows."""
        buf = self._buf(r, dtype, device)
        off = self.rank * self.maxrows
        dist.all_gather_into_tensor(buf, buf[off: off + self.maxrows], group=self.group)
        if self.equal:
            return buf[: self.n]
        if self._index is None or self._index.device != buf.device:
            self._index = torch.cat([torch.arange(i * self.maxrows, i * self.maxrows + (b - a), device=buf.device)
                                     for i, (a, b) in enumerate(self.shards)])
        return buf.index_select(0, self._index)

    def __call__(self, local: torch.Tensor) -> torch.Tensor:
        if self.world == 1:
            return local
        r = 1 if local.dim() == 1 else local.shape[1]
        self.slot(r, local.dtype, local.device).copy_(local.reshape(local.shape[0], r))
        out = self.gather_slot(r, local.dtype, local.device)
        if self.equal:
            out = out.clone()      # the buffer is reused by the next gather
        return out.reshape(self.n) if local.dim() == 1 else out


class ShardedDMAP:
    """DMAP operator M = diag(rscale) K diag(rscale) row-sharded over the process group.

    ``local_apply(V, col_scale, row_scale)`` is the rank's tile pass
    (``GaussianOperator.apply`` on its rows by default); it can be replaced by
    a host fake in tests.
    """

    def __init__(self, X: torch.Tensor, beta: float, alpha: float, precision: str = "f16", group=None,
                 local_apply: Optional[Callable] = None):
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.n = X.shape[0]
        self.rows = shard_rows(self.n, self.world, self.rank)
        self.gather = RowGather(self.n, self.world, group)
        if local_apply is None:
            from . import native
            from .kernel import GaussianOperator
            shift = native.mean_rows(X)
            a, b = self.rows
            self.op = GaussianOperator(X[a:b], X, beta, precision, shift=shift)
            self._apply = lambda V, cs, rs, dt: self.op.apply(V, col_scale=cs, row_scale=rs, out_dtype=dt)
            self._weights = native.dmap_weights
            self._rscale = native.dmap_rscale
        else:
            self._apply = local_apply
            self._weights = lambda D, a_: D.double().pow(-a_).to(D.dtype)
            self._rscale = lambda Kw, w: ((Kw.double() * w.double()).to(Kw.dtype),
                                          ((Kw.double() * w.double()).rsqrt() * w.double()).to(Kw.dtype))
        self.alpha = alpha
        self.D = self.D_alpha = self.rscale = None
        self.rscale_local = None

    def fit(self):
        """Two prepasses with a gather each: D = K 1, D_alpha = (K w) w, rscale."""
        Dl = self._apply(None, None, None, torch.float32)[:, 0].contiguous()
        D = self.gather(Dl).contiguous()
        w = self._weights(D, self.alpha)
        Kwl = self._apply(w, None, None, torch.float32)[:, 0].contiguous()
        Kw = self.gather(Kwl).contiguous()
        self.D = D
        self.D_alpha, self.rscale = self._rscale(Kw, w)
        a, b = self.rows
        self.rscale_local = self.rscale[a:b].contiguous()
        return self

    def matvec_local(self, v: torch.Tensor, out_dtype=torch.float64) -> torch.Tensor:
        squeeze = v.dim() == 1
        out = self._apply(v[:, None] if squeeze else v, self.rscale, self.rscale_local, out_dtype)
        return out[:, 0] if squeeze else out

    def matvec_device(self, v: torch.Tensor) -> torch.Tensor:
        """Full M v on every rank: local rows + one all-gather."""
        return self.gather(self.matvec_local(v))


class ShardedOperator:
    """Row-sharded operator for the three reference modes, with one all-gather per product.

    mode "dmap": Q = K = X, M = diag(rscale) K diag(rscale) (``FD/dmap.py:78-136``);
    mode "amap": Q != K, rscale_k from the DMAP normalisation of K and the
                 query scale of the reference's only Q != K normaliser
                 (``FD/utils.py:92-102``);
    mode "doob": DMAP with h: M_h v = M (h v) / (M h) (``FD/dmap.py:221-261``);
    mode "doob_sym": S M S with S = sqrt(h / (M h)), symmetric and similar to M_h
                 (same eigenvalues; eigenvectors y = x / sqrt(h M h)), the form a
                 symmetric Lanczos solves.
    Every rank holds all of K and owns a contiguous block of 256-row tiles of Q.
    """

    def __init__(self, Q: torch.Tensor, K: Optional[torch.Tensor], beta: float, alpha: float,
                 precision: str = "f16", mode: str = "dmap", h: Optional[torch.Tensor] = None, group=None):
        from . import native
        from .kernel import GaussianOperator
        if mode not in ("dmap", "amap", "doob", "doob_sym"):
            raise ValueError(f"mode must be dmap, amap, doob or doob_sym (got {mode!r})")
        if mode in ("doob", "doob_sym") and h is None:
            raise ValueError("mode 'doob' needs h")
        self.mode = mode
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.group = group
        self.alpha = alpha
        Kx = Q if K is None else K
        self.nq, self.nk = Q.shape[0], Kx.shape[0]
        self.rows = shard_rows(self.nq, self.world, self.rank)
        self.gather = RowGather(self.nq, self.world, group)
        shift = native.mean_rows(Kx)
        a, b = self.rows
        self.op = GaussianOperator(Q[a:b], Kx, beta, precision, shift=shift)
        if mode == "amap":
            self.krows = shard_rows(self.nk, self.world, self.rank)
            self.kgather = RowGather(self.nk, self.world, group)
            ka, kb = self.krows
            self.kop = GaussianOperator(Kx[ka:kb], Kx, beta, precision, shift=shift)
        self.h = None if h is None else h.to(torch.float32).contiguous()
        self.rscale_q = self.rscale_k = self.ph = None

    def fit(self):
        """Coifman-Lafon prepasses (two all-gathers each for the key side)."""
        from . import native
        if self.mode == "amap":
            Dk = self.kgather(self.kop.apply(out_dtype=torch.float32)[:, 0].contiguous()).contiguous()
            wk = native.dmap_weights(Dk, self.alpha)
            Kw = self.kgather(self.kop.apply(wk, out_dtype=torch.float32)[:, 0].contiguous()).contiguous()
            _, self.rscale_k = native.dmap_rscale(Kw, wk)
            Dq = self.op.apply(wk, out_dtype=torch.float32)[:, 0].contiguous()      # D_q = K(Q,K) w_k
            wq = native.dmap_weights(Dq, self.alpha)
            _, self.rscale_q = native.dmap_rscale(Dq, wq)                          # this rank's rows
        else:
            D = self.gather(self.op.apply(out_dtype=torch.float32)[:, 0].contiguous()).contiguous()
            w = native.dmap_weights(D, self.alpha)
            Kw = self.gather(self.op.apply(w, out_dtype=torch.float32)[:, 0].contiguous()).contiguous()
            _, rs = native.dmap_rscale(Kw, w)
            a, b = self.rows
            self.rscale_k, self.rscale_q = rs, rs[a:b].contiguous()
            if self.mode in ("doob", "doob_sym"):
                self.ph = self.op.apply(self.h, col_scale=rs, row_scale=self.rscale_q,
                                        out_dtype=torch.float32)[:, 0].contiguous()
            if self.mode == "doob_sym":
                ph = self.gather(self.ph).contiguous()
                s_full = (rs.double() * torch.sqrt(self.h.double() / ph.double())).float().contiguous()
                self.rscale_k, self.rscale_q = s_full, s_full[a:b].contiguous()
                self.h = None
                self.ph = None
        return self

    def matvec_local(self, v: torch.Tensor, out_dtype=torch.float64) -> torch.Tensor:
        squeeze = v.dim() == 1
        out = self.op.apply(v[:, None] if squeeze else v, col_scale=self.rscale_k, col_h=self.h,
                            row_scale=self.rscale_q, row_div=self.ph, out_dtype=out_dtype)
        return out[:, 0] if squeeze else out

    def _gather_dtype(self):
        return torch.float32 if self.op.precision in ("f16", "bf16") else torch.float64

    def matvec_shard(self, v: torch.Tensor):
        """This rank's rows of the product, written by the tile kernel straight
        into its chunk of the gather buffer (several GPUs), or returned (one)."""
        if self.world == 1:
            return self.matvec_local(v)
        r = 1 if v.dim() == 1 else v.shape[1]
        slot = self.gather.slot(r, self._gather_dtype(), v.device)
        self.op.apply(v[:, None] if v.dim() == 1 else v, col_scale=self.rscale_k, col_h=self.h,
                      row_scale=self.rscale_q, row_div=self.ph, out_dtype=slot.dtype, out=slot)
        return slot

    def gather_shards(self, shard: torch.Tensor, squeeze: bool) -> torch.Tensor:
        """The all-gather that completes ``matvec_shard``: the full fp64 product."""
        if self.world == 1:
            return shard
        r = shard.shape[1]
        full = self.gather.gather_slot(r, shard.dtype, shard.device)
        full = full.to(torch.float64) if full.dtype != torch.float64 else (full.clone() if self.gather.equal else full)
        return full.reshape(self.nq) if squeeze else full

    def matvec_device(self, v: torch.Tensor) -> torch.Tensor:
        """Full product on every rank: this rank's rows + one all-gather.  The
        16-bit tiles (error bound 2e-3) gather fp32, half the bytes of the fp64
        that the fp32-class tiles gather; the result is fp64 either way."""
        return self.gather_shards(self.matvec_shard(v), v.dim() == 1)

