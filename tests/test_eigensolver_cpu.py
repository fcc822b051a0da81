"""Host logic of the eigensolvers (thick-restart Lanczos, LOBPCG) checked on CPU
tensors against dense LAPACK on small symmetric operators."""
import numpy as np
import torch

from flashdiffusion_b200.eigensolver import SolveInfo, lobpcg_core, trlan
from oracle import fd_oracle as O


def dmap_dense(n=400, seed=0):
    from tests.golden.make_golden import test_roll
    X = test_roll(n, seed)
    M, _ = O.dense_dmap_operator(X, 1.0, 0.5)
    return M


def test_trlan_matches_dense():
    M = dmap_dense()
    Mt = torch.from_numpy(M)
    info = SolveInfo()
    theta, vecs, res = trlan(lambda v: Mt @ v, M.shape[0], 8, 1e-12, 500, 20, None, torch.device("cpu"), info)
    ref = np.sort(np.linalg.eigvalsh(M))[::-1][:8]
    np.testing.assert_allclose(np.sort(theta)[::-1], ref, rtol=1e-10)
    assert info.converged
    # Ritz vectors are eigenvectors
    Y = vecs.numpy()
    R = M @ Y - Y * theta[None, :]
    assert np.linalg.norm(R, axis=0).max() < 1e-8


def test_trlan_restarts_and_counts():
    M = dmap_dense(300, 1)
    Mt = torch.from_numpy(M)
    info = SolveInfo()
    trlan(lambda v: Mt @ v, 300, 6, 1e-10, 500, 14, None, torch.device("cpu"), info)
    assert info.n_restart >= 2 and info.n_matvec >= 14


def test_trlan_stops_at_noise_floor():
    """A noisy operator stalls above tol; the solver must stop, not spin."""
    M = dmap_dense(200, 2)
    Mt = torch.from_numpy(M)
    g = torch.Generator().manual_seed(0)
    noisy = lambda v: Mt @ v + 1e-6 * torch.randn(v.shape[0], generator=g, dtype=torch.float64)
    info = SolveInfo()
    theta, _, _ = trlan(noisy, 200, 4, 1e-14, 200, 20, None, torch.device("cpu"), info)
    assert not info.converged and info.n_restart < 200
    ref = np.sort(np.linalg.eigvalsh(M))[::-1][:4]
    np.testing.assert_allclose(np.sort(theta)[::-1], ref, rtol=1e-5)


def test_lobpcg_matches_dense():
    M = dmap_dense(300, 3)
    Mt = torch.from_numpy(M)
    info = SolveInfo()
    vals, vecs = lobpcg_core(lambda B: Mt @ B, 300, 6, 1e-9, 500, 42, torch.device("cpu"), info)
    ref = np.sort(np.linalg.eigvalsh(M))[::-1][:6]
    np.testing.assert_allclose(vals, ref, rtol=1e-8)
    assert info.converged
