"""Pin the CPU oracle (oracle/fd_oracle.py) to outputs of the reference itself.

The fixtures under tests/golden/ were produced by running the reference
NumPy path (tests/golden/make_golden.py).  Every oracle function used as a
checker by the GPU parity tests is compared here first.  Reference test
tolerances (tests/test_kernel.py of the reference): prepass rtol 1e-5,
matvec rtol 2e-4, eigenvalues 1e-5.  The oracle restates the same fp32-GEMM /
fp64-exp algorithm, so it is held to 1e-10 relative.
"""
import numpy as np
import pytest

from oracle import fd_oracle as O

RT = 1e-10


def test_prepass_matches_reference(gold):
    g = gold("prepass.npz")
    X = g["X"]
    np.testing.assert_allclose(O.prepass_rowsum(X, X, 1.0, tile=64), g["D64"], rtol=RT)
    np.testing.assert_allclose(O.prepass_rowsum(X, X, 1.0, tile=256), g["D256"], rtol=RT)
    np.testing.assert_allclose(O.prepass_rowsum(X, X, 0.7, g["w"], tile=64), g["Dw"], rtol=RT)


def test_prepass_matches_dense():
    from tests.golden.make_golden import test_roll
    X = test_roll(150)
    np.testing.assert_allclose(O.prepass_rowsum(X, X, 1.0), O.dense_kernel(X, 1.0).sum(1), rtol=1e-5)


@pytest.mark.parametrize("n", [0, 1, 2])
def test_dmap_matvec_matches_reference(gold, n):
    g = gold("matvec.npz")
    beta, alpha = g["pairs"][n]
    D, Da, rs = O.dmap_fit(g["X"], beta, alpha, tile=64)
    np.testing.assert_allclose(rs, g[f"rscale{n}"], rtol=RT)
    np.testing.assert_allclose(O.dmap_matvec(g["X"], beta, g[f"rscale{n}"], g["v"]), g[f"out{n}"], rtol=RT, atol=1e-14)
    M, _ = O.dense_dmap_operator(g["X"], beta, alpha)
    np.testing.assert_allclose(g[f"out{n}"], M @ g["v"], rtol=2e-4, atol=1e-12)


def test_fit_matches_reference(gold):
    g = gold("fit.npz")
    D, Da, rs = O.dmap_fit(g["X"], 1.0, 0.5, tile=128)
    np.testing.assert_allclose(D, g["D"], rtol=RT)
    np.testing.assert_allclose(Da, g["D_alpha"], rtol=RT)
    np.testing.assert_allclose(rs, g["rscale"], rtol=RT)


def test_eigs_match_reference(gold):
    g = gold("eig.npz")
    X = g["X"]
    _, _, rs = O.dmap_fit(X, 1.0, 0.5, tile=128)
    vals, vecs = O.lanczos_eigsh(lambda v: O.dmap_matvec(X, 1.0, rs, v, tile=128), X.shape[0], k=6)
    np.testing.assert_allclose(vals, g["vals"], rtol=1e-9)
    coords = O.transform_coords(vals, vecs, rs)
    # eigenvectors are defined up to sign
    np.testing.assert_allclose(np.abs(coords), np.abs(g["coords"]), rtol=1e-5, atol=1e-8)


def test_doob_matches_reference(gold):
    g = gold("doob.npz")
    X = g["X"]
    Ph = O.doob_ph(X, 1.0, g["rscale"], g["h"], tile=64)
    np.testing.assert_allclose(Ph, g["Ph"], rtol=RT)
    np.testing.assert_allclose(O.doob_matvec(X, 1.0, g["rscale"], g["h"], Ph, g["v"], tile=64), g["out"], rtol=RT)


def test_amap_matches_reference(gold):
    g = gold("amap.npz")
    out = O.flash_diffusion(g["Q"], g["K"], g["V"], float(g["beta"]), g["rq"], g["rk"], g["h"], tile=64)
    np.testing.assert_allclose(out, g["out"], rtol=RT)
    np.testing.assert_allclose(O.flash_diffusion(g["Q"], g["K"], g["V"], float(g["beta"]), tile=64),
                               g["out_plain"], rtol=RT)


def test_nystrom_matches_reference(gold):
    g = gold("nystrom.npz")
    c = O.nystrom_extend(g["Xn"], g["Xt"], 1.0, 0.5, g["D"], g["rscale"], g["vals"], g["vecs"], tile=64)
    np.testing.assert_allclose(c, g["coords"], rtol=1e-9, atol=1e-14)


def test_gmm64_matches_reference(gold):
    g = gold("gmm64.npz")
    b = float(g["beta"])
    D, Da, rs = O.dmap_fit(g["X"], b, 0.5, tile=256)
    np.testing.assert_allclose(D, g["D"], rtol=RT)
    np.testing.assert_allclose(rs, g["rscale"], rtol=RT)
    np.testing.assert_allclose(O.dmap_matvec(g["X"], b, rs, g["v"], tile=256), g["out"], rtol=RT)


def test_c1_matches_reference(gold):
    g = gold("c1.npz")
    X, b = g["X"], float(g["beta"])
    D, Da, rs = O.dmap_fit(X, b, 0.5)
    np.testing.assert_allclose(D, g["D"], rtol=RT)
    np.testing.assert_allclose(rs, g["rscale"], rtol=RT)
    vals, _ = O.lanczos_eigsh(lambda v: O.dmap_matvec(X, b, rs, v), X.shape[0], k=8)
    np.testing.assert_allclose(vals, g["vals"], rtol=1e-8)


def test_synthetic_c1_is_the_fixture(gold):
    """The shipped generator still reproduces the configuration-1 fixture bit for bit."""
    from flashdiffusion_b200 import synthetic
    g = gold("c1.npz")
    X, b, _ = synthetic.swiss_roll(4096, seed=0)
    np.testing.assert_array_equal(X, g["X"])
    assert b == float(g["beta"])


def test_sym_doob_similarity():
    """S M S (S = sqrt(h/Ph)) has the spectrum of diag(1/Ph) M diag(h)."""
    from tests.golden.make_golden import test_roll
    X = test_roll(80)
    M, rs = O.dense_dmap_operator(X, 1.0, 0.5)
    h = np.exp(-(X ** 2).sum(1))
    Ph = M @ h
    Mh = M * h[None, :] / Ph[:, None]
    ev = np.sort(np.linalg.eigvals(Mh).real)[::-1]
    es = np.sort(np.linalg.eigvalsh(O.sym_doob_operator(M, h, Ph)))[::-1]
    np.testing.assert_allclose(ev[:6], es[:6], rtol=1e-9)


def test_bandwidth_rules_match_reference(gold):
    g = gold("bandwidth.npz")
    assert O.median_bandwidth(g["X"]) == pytest.approx(float(g["median_beta"]), rel=RT)
    assert O.median_bandwidth(g["X"][:500]) == pytest.approx(float(g["median_beta_small"]), rel=RT)
    np.testing.assert_allclose(O.knn_bandwidth(g["Xk"], k=7), g["sigma7"], rtol=RT)
    np.testing.assert_allclose(O.knn_bandwidth(g["Xk"], k=5), g["sigma5"], rtol=RT)


def test_carre_du_champ_matches_reference(gold):
    g = gold("cdc.npz")
    args = (g["X"], 1.0, 0.5, g["D"], g["D_alpha"])
    vals, phi = g["vals"], g["phi"]
    np.testing.assert_allclose(O.carre_du_champ(*args, phi[:, 1], phi[:, 3], vals[1], vals[3], tile=128),
                               g["gamma13"], rtol=1e-9, atol=1e-15)
    G, M = O.metric_tensor(*args, vals, phi, tile=128)
    np.testing.assert_allclose(G, g["G"], rtol=1e-9, atol=1e-15)
    np.testing.assert_allclose(M, g["M"], rtol=1e-9, atol=1e-15)
    Gp, Mp = O.metric_tensor(*args, vals, phi, pairs=[(1, 1), (1, 2), (0, 4)], tile=128)
    np.testing.assert_allclose(Gp, g["Gp"], rtol=1e-9, atol=1e-15)
    np.testing.assert_allclose(Mp, g["Mp"], rtol=1e-9, atol=1e-15)
