"""C-ABI checks that need no GPU: the library builds, loads, exports every
symbol include/fd_sm100.h declares, and rejects bad arguments before any
launch.  No compute call is made here."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "fd_sm100.h")


def declared():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    out = {}
    for m in re.finditer(r"^\s*(?:const\s+)?\w+\s*\*?\s*(fd_\w+)\s*\(([^)]*)\)\s*;", src, flags=re.M):
        args = m.group(2).strip()
        out[m.group(1)] = 0 if args in ("", "void") else len(args.split(","))
    return out


@pytest.fixture(scope="module")
def lib():
    from flashdiffusion_b200 import build, native
    build.build()
    return native.load()


def test_header_parses():
    d = declared()
    assert "fd_apply" in d and "fd_matvec" in d and len(d) >= 15


def test_every_declared_symbol_is_exported(lib):
    from flashdiffusion_b200 import native
    d = declared()
    for name, nargs in d.items():
        assert hasattr(lib, name), name
        assert name in native.SIGNATURES, f"{name} missing from native.SIGNATURES"
        assert len(native.SIGNATURES[name][1]) == nargs, name
    assert set(native.SIGNATURES) == set(d)


def test_query_functions(lib):
    from flashdiffusion_b200 import native
    assert lib.fd_version() >= 100
    assert lib.fd_operand_bytes(1000, 64, native.TILE_BF16) == ((1000 * 80 * 2 + 255) // 256) * 256
    assert lib.fd_operand_bytes(1000, 3, native.TILE_F32) >= 1000 * 4 * 4 + 1000 * 4
    assert lib.fd_apply_workspace_bytes(10, 10, 1, native.TILE_BF16) > 0
    assert lib.fd_workspace_bytes(10, 10, 3, 1, native.TILE_F32) > 0
    assert lib.fd_workspace_bytes(-1, 10, 3, 1, native.TILE_F32) == 0


def test_argument_errors_before_launch(lib):
    from flashdiffusion_b200 import native
    P = ctypes.c_void_p
    fake = P(4096)
    # non-positive beta
    rc = lib.fd_pack_operand(fake, native.DTYPE_F32, 10, 3, None, 0.0, native.SIDE_QUERY, native.TILE_BF16, fake, None)
    assert rc == native.FD_ERR_ARG and b"beta" in lib.fd_last_error()
    # misaligned operand
    rc = lib.fd_pack_operand(fake, native.DTYPE_F32, 10, 3, None, 1.0, native.SIDE_QUERY, native.TILE_BF16, P(4100), None)
    assert rc == native.FD_ERR_ARG and b"aligned" in lib.fd_last_error()
    # bad dtype / tile / side
    assert lib.fd_pack_operand(fake, 9, 10, 3, None, 1.0, 0, 0, fake, None) == native.FD_ERR_ARG
    assert lib.fd_pack_operand(fake, 0, 10, 3, None, 1.0, 0, 7, fake, None) == native.FD_ERR_ARG
    assert lib.fd_pack_operand(fake, 0, 10, 3, None, 1.0, 5, 0, fake, None) == native.FD_ERR_ARG
    # negative sizes, zero r
    assert lib.fd_apply(fake, -1, fake, 4, 3, 0, fake, 0, 1, None, None, None, None, fake, 0, fake, 1 << 20, None) == native.FD_ERR_ARG
    assert lib.fd_apply(fake, 4, fake, 4, 3, 0, fake, 0, 0, None, None, None, None, fake, 0, fake, 1 << 20, None) == native.FD_ERR_ARG
    # workspace too small
    rc = lib.fd_apply(fake, 4, fake, 4, 3, 0, fake, 0, 1, None, None, None, None, fake, 0, fake, 16, None)
    assert rc == native.FD_ERR_WORKSPACE and b"workspace" in lib.fd_last_error()
    # bad V / out dtype
    assert lib.fd_apply(fake, 4, fake, 4, 3, 0, fake, native.DTYPE_F16, 1, None, None, None, None, fake, 0, fake, 1 << 20, None) == native.FD_ERR_ARG
    # reference trio: null rscale
    assert lib.fd_matvec(fake, 0, 4, 3, fake, None, 1.0, 0, fake, fake, 1 << 20, None) == native.FD_ERR_ARG
    # fp32-class split tiles: operand rows of at most 416 columns (d <= 136)
    rc = lib.fd_pack_operand(fake, native.DTYPE_F32, 10, 137, None, 1.0, native.SIDE_QUERY, native.TILE_F16X3, fake, None)
    assert rc == native.FD_ERR_ARG and b"416" in lib.fd_last_error()
    # bandwidth selection: k out of range, more neighbours than keys, bad d
    assert lib.fd_knn_sqdist(fake, 10, fake, 10, 3, 65, fake, None) == native.FD_ERR_ARG
    assert lib.fd_knn_sqdist(fake, 10, fake, 4, 3, 5, fake, None) == native.FD_ERR_ARG
    assert lib.fd_knn_sqdist(fake, 10, fake, 10, 0, 5, fake, None) == native.FD_ERR_ARG
    assert lib.fd_pairwise_sqdist(fake, 70000, 3, fake, None) == native.FD_ERR_ARG
    # RoPE windows: window sample index outside the window
    assert lib.fd_rope_windows(fake, 2, 2, fake, 1, 1, 10, 2, 3, 1, 3, 1.0, None, 0, fake, fake, fake, None) == native.FD_ERR_ARG
    # block options and the wait self-test validate their arguments
    assert lib.fd_set_block_options(65, 0) == native.FD_ERR_ARG
    assert lib.fd_set_block_options(0, 4) == native.FD_ERR_ARG
    assert lib.fd_set_block_options(0, 0) == native.FD_OK
    assert lib.fd_selftest_wait_timeout(10, None) == native.FD_ERR_ARG


def test_no_device_raises_loudly():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is visible")
    from flashdiffusion_b200 import native, FlashDiffusion
    import numpy as np
    with pytest.raises(RuntimeError, match="B200"):
        native.require_device()
    with pytest.raises(RuntimeError):
        FlashDiffusion(np.ones((3, 2)), np.ones((3, 2)), np.ones((3, 1)), 1.0)


def test_comm_rendezvous_id_without_a_gpu():
    """fd_comm_get_id needs only NCCL's host side: an id of fd_comm_id_bytes() bytes."""
    from flashdiffusion_b200 import native
    lib = native.load()
    n = int(lib.fd_comm_id_bytes())
    assert n == 128
    a, b = native.Comm.new_id(), native.Comm.new_id()
    assert len(a) == n and a != b
    assert lib.fd_comm_allgather(None, None, None, 0, None) == native.FD_ERR_ARG
