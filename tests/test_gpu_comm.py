"""fd_comm_* on one GPU: a one-rank communicator's in-place all-gather leaves
the buffer as it was, and a sharded product through it equals the plain
product.  Two ranks run in tests/test_multigpu.py."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_single_rank_comm_allgather_in_place():
    from flashdiffusion_b200 import native
    dev = native.require_device()
    comm = native.Comm(native.Comm.new_id(), 1, 0)
    try:
        buf = torch.arange(1000, dtype=torch.float64, device=dev)
        want = buf.clone()
        comm.allgather_(buf)
        torch.cuda.synchronize()
        comm.check()
        assert torch.equal(buf, want)
    finally:
        comm.close()
