"""The library's Lanczos reorthogonalisation (fd_lanczos_reorth) against the
same classical Gram-Schmidt applied twice in fp64 torch, plus determinism and
the breakdown signal.  The eigenvalue goldens (tests/test_gpu_parity.py) run
the whole solver through it."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _basis(n, rows, seed):
    g = torch.Generator(device="cpu").manual_seed(seed)
    A = torch.randn(n, rows, generator=g, dtype=torch.float64)
    return torch.linalg.qr(A)[0].T.contiguous()


@pytest.mark.parametrize("n,rows", [(1, 1), (257, 5), (200_001, 33), (100_000, 96)])
def test_reorth_matches_cgs2(n, rows):
    from flashdiffusion_b200 import native
    dev = native.require_device()
    rows = min(rows, n)
    Vh = _basis(n, rows, 1)
    V = torch.zeros((rows + 1, n), dtype=torch.float64, device=dev)
    V[:rows] = Vh.to(dev)
    w0 = torch.randn(n, dtype=torch.float64, generator=torch.Generator().manual_seed(2)).to(dev)
    if n > 1:
        w0 += 3.0 * V[0]          # a large component along the basis
    w = w0.clone()
    coef = torch.zeros(rows + 2, dtype=torch.float64, device=dev)
    ws = native.lanczos_workspace(n, rows, dev)
    native.lanczos_reorth(V, rows, w, V[rows], coef, ws)
    # reference CGS2
    Vb = V[:rows]
    r = w0.clone()
    h = Vb @ r
    r -= Vb.T @ h
    h2 = Vb @ r
    r -= Vb.T @ h2
    beta = torch.linalg.vector_norm(r)
    c = coef.cpu().numpy()
    if n == 1:      # the only direction is taken: breakdown, zeros out
        assert c[rows] <= 1e-12 * float(torch.linalg.vector_norm(w0))
        return
    assert np.allclose(c[:rows], (h + h2).cpu().numpy(), rtol=1e-12, atol=1e-12 * float(beta))
    assert abs(c[rows] - float(beta)) <= 1e-10 * float(beta)
    out = V[rows]
    assert float(torch.linalg.vector_norm(out - r / beta)) <= 1e-10
    assert float(torch.max(torch.abs(Vb @ out))) <= 1e-12


def test_reorth_is_bit_reproducible():
    from flashdiffusion_b200 import native
    dev = native.require_device()
    n, rows = 300_000, 40
    V = torch.zeros((rows + 1, n), dtype=torch.float64, device=dev)
    V[:rows] = _basis(n, rows, 3).to(dev)
    w0 = torch.randn(n, dtype=torch.float64, device=dev)
    ws = native.lanczos_workspace(n, rows, dev)
    outs = []
    for _ in range(2):
        w = w0.clone()
        coef = torch.zeros(rows + 2, dtype=torch.float64, device=dev)
        out = torch.empty(n, dtype=torch.float64, device=dev)
        native.lanczos_reorth(V, rows, w, out, coef, ws)
        outs.append((coef.cpu(), out.cpu()))
    assert torch.equal(outs[0][0], outs[1][0]) and torch.equal(outs[0][1], outs[1][1])


def test_reorth_argument_errors():
    from flashdiffusion_b200 import native
    dev = native.require_device()
    V = torch.zeros((98, 10), dtype=torch.float64, device=dev)
    w = torch.zeros(10, dtype=torch.float64, device=dev)
    coef = torch.zeros(99, dtype=torch.float64, device=dev)
    ws = native.lanczos_workspace(10, 97, dev)
    with pytest.raises(native.FDError):
        native.lanczos_reorth(V, 97, w, V[97], coef, ws)      # above the 96-row limit
