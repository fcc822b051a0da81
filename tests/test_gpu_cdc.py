"""Carre du Champ / metric tensor on the GPU against the reference's own outputs
(tests/golden/cdc.npz: the reference's fitted map, its eigenpairs and its G, M).

The map is refitted here with fp32 tiles (operator within 1e-5 of the
reference's); the eigenvectors are the reference's.  Gamma subtracts
(lambda_k + lambda_l) phi_k phi_l from P+(phi_k phi_l), so errors are judged
against max |G| (1e-5) rather than element-wise.
"""
import numpy as np
import pytest

from oracle import fd_oracle as O

pytestmark = pytest.mark.gpu


def _fitted(g, precision):
    from flashdiffusion_b200 import DiffusionMap
    return DiffusionMap(beta=1.0, alpha=0.5, n_components=5, precision=precision).fit(g["X"])


@pytest.mark.parametrize("precision", ["fp32", "f16x3"])
def test_metric_tensor_golden(gold, precision):
    from flashdiffusion_b200.cdc import metric_tensor, carre_du_champ
    g = gold("cdc.npz")
    dm = _fitted(g, precision)
    vals, phi = g["vals"], g["phi"]
    scale = np.abs(g["G"]).max()
    G, M = metric_tensor(dm, vals, phi)
    assert np.abs(G - g["G"]).max() <= 1e-5 * scale
    assert np.abs(M - g["M"]).max() <= 1e-5 * np.abs(g["M"]).max() * 4
    Gp, Mp = metric_tensor(dm, vals, phi, pairs=[(1, 1), (1, 2), (0, 4)])
    assert np.abs(Gp - g["Gp"]).max() <= 1e-5 * scale
    g13 = carre_du_champ(dm, phi[:, 1], phi[:, 3], vals[1], vals[3])
    assert np.abs(g13 - g["gamma13"]).max() <= 1e-5 * scale


def test_metric_tensor_16bit_and_many_pairs():
    """k = 10 (55 pairs: two block launches), 16-bit tiles, against the oracle's G."""
    from flashdiffusion_b200 import DiffusionMap
    from flashdiffusion_b200.cdc import metric_tensor
    from tests.golden.make_golden import test_roll
    X = test_roll(3000, seed=9)
    dm = DiffusionMap(beta=1.0, alpha=0.5, n_components=10, precision="f16").fit(X)
    rng = np.random.default_rng(0)
    phi = rng.standard_normal((3000, 10))
    vals = np.linspace(1.0, 0.5, 10)
    G, M = metric_tensor(dm, vals, phi)
    Gr, Mr = O.metric_tensor(X, 1.0, 0.5, dm.D_, dm.D_alpha_, vals, phi)
    assert np.abs(G - Gr).max() <= 2e-3 * np.abs(Gr).max()
    assert np.abs(M - Mr).max() <= 4e-3 * np.abs(Mr).max()
