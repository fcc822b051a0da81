"""fd_apply_noalloc: the operator with library-owned scratch, for callers that
cannot allocate device memory or pass a workspace (plugin / FFI hosts without
a device allocator, processes whose device memory is owned by a fixed pool,
loops that must avoid cudaMalloc's implicit synchronisation).

Checked through the C ABI against fd_apply (the workspace entry point) on two
calls in a row, with the 16-bit tile tolerance the parity tests use.  This
file is named to be collected last.
"""
import ctypes

import numpy as np
import pytest
import torch

TOL = 2e-3


def rel_l2(a, b):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-300))


def test_oversize_is_rejected_before_any_launch():
    from flashdiffusion_b200 import native
    lib = native.load()
    fake = ctypes.c_void_p(4096)
    nk = 4_000_000  # the prepared right-hand side alone exceeds the 8 MiB scratch
    rc = lib.fd_apply_noalloc(fake, 1000, fake, nk, 64, native.TILE_F16, fake, native.DTYPE_F32, 1,
                              None, None, None, None, fake, native.DTYPE_F32, None)
    assert rc == native.FD_ERR_WORKSPACE
    assert b"static scratch" in lib.fd_last_error()
    rc = lib.fd_apply_noalloc(fake, 10, fake, 10, 64, native.TILE_F32, fake, native.DTYPE_F32, 1,
                              None, None, None, None, fake, native.DTYPE_F32, None)
    assert rc == native.FD_ERR_ARG
    # 17 or more block columns: the block path's partial sums alone exceed the array
    rc = lib.fd_apply_noalloc(fake, 10, fake, 10, 64, native.TILE_F16, fake, native.DTYPE_F32, 17,
                              None, None, None, None, fake, native.DTYPE_F32, None)
    assert rc == native.FD_ERR_WORKSPACE
    assert b"r=17" in lib.fd_last_error()
    # r = 2..16 fits up to about 55,000 keys
    rc = lib.fd_apply_noalloc(fake, 10, fake, 60_000, 64, native.TILE_F16, fake, native.DTYPE_F32, 8,
                              None, None, None, None, fake, native.DTYPE_F32, None)
    assert rc == native.FD_ERR_WORKSPACE


@pytest.mark.gpu
def test_noalloc_matches_workspace_entry_point_twice():
    from flashdiffusion_b200 import native
    from flashdiffusion_b200.kernel import GaussianOperator
    dev = native.require_device()
    lib = native.load()
    rng = np.random.default_rng(5)
    nq, nk, d = 3000, 70_000, 64      # nk x rows > one CTA range: exercises the cross-CTA partials
    K = torch.from_numpy(rng.standard_normal((nk, d)).astype(np.float32)).to(dev)
    Q = K[:nq] + 0.05
    op = GaussianOperator(Q, K, 1.0 / d, "f16")
    rq = torch.from_numpy(rng.uniform(0.5, 2.0, nq).astype(np.float32)).to(dev)
    rk = torch.from_numpy(rng.uniform(0.5, 2.0, nk).astype(np.float32)).to(dev)
    stream = native._stream(dev)
    for call in range(2):
        V = torch.from_numpy(rng.standard_normal((nk, 1))).to(dev)
        ref = op.apply(V, col_scale=rk, row_scale=rq, out_dtype=torch.float64)
        out = torch.full((nq, 1), float("nan"), dtype=torch.float64, device=dev)
        rc = lib.fd_apply_noalloc(native._ptr(op.qop), nq, native._ptr(op.kop), nk, d, op.tile, native._ptr(V),
                                  native.DTYPE_F64, 1, native._ptr(rk), None, native._ptr(rq), None,
                                  native._ptr(out), native.DTYPE_F64, stream)
        native.check(rc)
        torch.cuda.synchronize()
        native.check_status(dev)
        o, r = out.cpu().numpy(), ref.cpu().numpy()
        assert np.isfinite(o).all(), f"call {call}: unwritten output"
        assert rel_l2(o, r) <= TOL, f"call {call}"


@pytest.mark.gpu
def test_noalloc_block_bf16_matches_workspace_entry_point_twice():
    """bf16 tiles and an 8-column block: the transposed fp16 right-hand side,
    its column scales and the block kernel's partial sums all come out of the
    static array."""
    from flashdiffusion_b200 import native
    from flashdiffusion_b200.kernel import GaussianOperator
    dev = native.require_device()
    lib = native.load()
    rng = np.random.default_rng(6)
    nq, nk, d, r = 2500, 40_000, 32, 8
    K = torch.from_numpy(rng.standard_normal((nk, d)).astype(np.float32)).to(dev)
    Q = K[:nq] + 0.05
    op = GaussianOperator(Q, K, 1.0 / d, "bf16")
    rk = torch.from_numpy(rng.uniform(0.5, 2.0, nk).astype(np.float32)).to(dev)
    stream = native._stream(dev)
    for call in range(2):
        V = torch.from_numpy(rng.standard_normal((nk, r))).to(dev)
        ref = op.apply(V, col_scale=rk, out_dtype=torch.float64)
        out = torch.full((nq, r), float("nan"), dtype=torch.float64, device=dev)
        rc = lib.fd_apply_noalloc(native._ptr(op.qop), nq, native._ptr(op.kop), nk, d, op.tile, native._ptr(V),
                                  native.DTYPE_F64, r, native._ptr(rk), None, None, None,
                                  native._ptr(out), native.DTYPE_F64, stream)
        native.check(rc)
        torch.cuda.synchronize()
        native.check_status(dev)
        o, ref_ = out.cpu().numpy(), ref.cpu().numpy()
        assert np.isfinite(o).all(), f"call {call}: unwritten output"
        for c in range(r):
            assert rel_l2(o[:, c], ref_[:, c]) <= TOL, f"call {call}, column {c}"
