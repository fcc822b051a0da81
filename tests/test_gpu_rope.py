"""RoPE-DMAP encoder on the GPU against the reference ROPE's own outputs
(tests/golden/rope.npz): sample mode (D=2, L=6) and window mode (odd D=3,
L=5, step 2, centre position, scaled features).

Eigenvectors are defined up to sign: each column is aligned to the
reference's before comparison, and the same signs carry over to the Nystrom
encodings.  Tolerances (the precision ramp ends on fp32-class tiles):
eigenvalues and beta 1e-6 relative, psi and encodings 2e-4 of the column's
largest entry (the first pair of eigenvalues is 3e-3 apart, which bounds how
well the individual vectors are determined).
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _aligned(got, ref):
    s = np.sign((got * ref).sum(0))
    s[s == 0] = 1
    return got * s[None, :], s


def _close(got, ref, tol):
    scale = np.abs(ref).max(0)
    assert np.all(np.abs(got - ref).max(0) <= tol * scale), (np.abs(got - ref).max(0) / scale)


def test_rope_sample_mode_golden(gold):
    from flashdiffusion_b200.rope import ROPE
    g = gold("rope.npz")
    a = ROPE(g["F"], L=6, rank=4, alpha=1.0, pos_scale=0.5, seed=3)
    assert a.beta_ == pytest.approx(float(g["a_beta"]), rel=1e-6)
    np.testing.assert_allclose(a.lam_, g["a_lam"], rtol=1e-6)
    psi, s = _aligned(a.psi_, g["a_psi"])
    _close(psi, g["a_psi"], 2e-4)
    _close(a.encode_series(g["Fn"]) * s, g["a_enc"], 2e-4)
    _close(a.encode_windows(g["Wq"], positions=g["Pq"]) * s, g["a_encw"], 2e-4)
    _close(a.encode_windows(g["Wq"]) * s, g["a_encw0"], 2e-4)
    assert a.Kmat_ is None and a.G_ is None


def test_rope_window_mode_golden(gold):
    from flashdiffusion_b200.rope import ROPE
    g = gold("rope.npz")
    b = ROPE(g["F3"], L=5, rank=3, alpha=0.5, step=2, rope_mode="window", window_position="center",
             pos_scale=0.2, scale=True, seed=7)
    assert b.beta_ == pytest.approx(float(g["b_beta"]), rel=1e-6)
    np.testing.assert_allclose(b.lam_, g["b_lam"], rtol=1e-6)
    psi, s = _aligned(b.psi_, g["b_psi"])
    _close(psi, g["b_psi"], 2e-4)
    _close(b.encode_series(g["Fn3"]) * s, g["b_enc"], 2e-4)


def test_rope_rejects_bad_windows(gold):
    from flashdiffusion_b200.rope import ROPE
    g = gold("rope.npz")
    a = ROPE(g["F"][:120], L=6, rank=2, pos_scale=0.5, precision="f16")
    with pytest.raises(ValueError):
        a.encode_windows(np.zeros((3, 5, 2)))
    with pytest.raises(ValueError):
        a.encode_windows(np.zeros((3, 6, 2)), positions=np.zeros((2, 6)))
