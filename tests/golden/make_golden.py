"""Generate golden fixtures by running the REFERENCE FlashDiffusion NumPy path.

Run once in a container that has the reference checkout (read-only)::

    python tests/golden/make_golden.py /path/to/FlashDiffusion

It imports the reference submodules ``flashdiffusion.kernel``, ``.dmap`` and
``.eigensolver`` directly (the reference package ``__init__`` is empty, so the
top-level names are not exported) and stores inputs and outputs as small
``.npz`` files next to this script.  Tests only read the ``.npz`` files; the
reference is never needed at test time.

Fixtures (reference call each one pins):
  prepass.npz     kernel.prepass_rowsum on the test_kernel.py Swiss roll, N=150, tiles 64/256
  matvec.npz      kernel.FlashDiffusion DMAP matvec, 3 (beta, alpha) pairs, N=150
  fit.npz         dmap.DiffusionMap.fit D_ / D_alpha_ / rscale_, N=300
  eig.npz         dmap.DiffusionMap.transform eigenvalues + coords, N=300, k=6
  doob.npz        dmap.DoobTransformedMap Ph_ and one matvec, N=100
  amap.npz        kernel.FlashDiffusion with Q != K, rscale_q != rscale_k, h, r=3
  nystrom.npz     utils.nystrom_extend (Q != K normalisation), 200 train / 40 new
  gmm64.npz       kernel.FlashDiffusion DMAP matvec at d=64, N=1024 (mixture)
  c1.npz          configuration 1 (Swiss roll N=4096, d=3): fit + Lanczos k=8 eigenvalues
  bandwidth.npz   utils.median_bandwidth (N=3000 > subsample) and utils.knn_bandwidth (k=7, 5)
  cdc.npz         cdc.carre_du_champ and cdc.metric_tensor on a fitted map (N=400, k=5)
  rope.npz        ROPE encoder: sample mode (D=2, L=6) and window mode (D=3, L=5, step=2, centre),
                  fitted eigenpairs, psi, beta, encode_series and encode_windows of new data
"""

from __future__ import annotations

import io
import os
import sys
import contextlib

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))


def _ref_modules(ref_root):
    sys.path.insert(0, os.path.join(ref_root, "src"))
    import flashdiffusion.kernel as K          # noqa: E402
    import flashdiffusion.dmap as D            # noqa: E402
    import flashdiffusion.eigensolver as E     # noqa: E402
    import flashdiffusion.utils as U           # noqa: E402
    # The reference dispatcher asks torch for a GPU; force its NumPy path.
    K._get_cuda_backend = lambda: None
    return K, D, E, U


def rope_series(n, D, seed):
    rng = np.random.default_rng(seed)
    t = np.arange(n) * 0.07
    cols = [np.sin(t * (1 + 0.3 * j)) + 0.05 * rng.standard_normal(n) for j in range(D)]
    return np.stack(cols, axis=1)


def rope(ref_root):
    sys.path.insert(0, os.path.join(ref_root, "src"))
    from flashdiffusion.ROPE import ROPE, make_hankel_windows   # noqa: E402
    F = rope_series(320, 2, 1)
    Fn = rope_series(120, 2, 2)
    a = ROPE(F, L=6, rank=4, alpha=1.0, pos_scale=0.5, seed=3)
    F3 = rope_series(300, 3, 4)
    Fn3 = rope_series(90, 3, 5)
    b = ROPE(F3, L=5, rank=3, alpha=0.5, step=2, rope_mode="window", window_position="center", pos_scale=0.2,
             scale=True, seed=7)
    Wq = make_hankel_windows(Fn, 6)[:7]
    Pq = np.arange(7)[:, None] + np.arange(6)[None, :] + 40.0
    np.savez_compressed(os.path.join(HERE, "rope.npz"), F=F, Fn=Fn, F3=F3, Fn3=Fn3,
                        a_lam=a.lam_, a_psi=a.psi_, a_beta=a.beta_, a_enc=a.encode_series(Fn),
                        a_encw=a.encode_windows(Wq, positions=Pq), a_encw0=a.encode_windows(Wq), Wq=Wq, Pq=Pq,
                        b_lam=b.lam_, b_psi=b.psi_, b_beta=b.beta_, b_enc=b.encode_series(Fn3))


def cdc(ref_root):
    K, D, _, _ = _ref_modules(ref_root)
    import flashdiffusion.cdc as C             # noqa: E402
    X = test_roll(400, seed=4)
    dm = D.DiffusionMap(beta=1.0, alpha=0.5, n_components=5, tile=128)
    with contextlib.redirect_stdout(io.StringIO()):
        dm.fit(X)
        dm.transform()
    vals = dm.eigenvalues_
    phi = dm.eigenvectors_ / dm.rscale_[:, None]
    phi = phi / np.linalg.norm(phi, axis=0, keepdims=True)
    g13 = C.carre_du_champ(dm, phi[:, 1], phi[:, 3], vals[1], vals[3])
    G, M = C.metric_tensor(dm, vals, phi)
    Gp, Mp = C.metric_tensor(dm, vals, phi, pairs=[(1, 1), (1, 2), (0, 4)])
    np.savez_compressed(os.path.join(HERE, "cdc.npz"), X=X, vals=vals, phi=phi, D=dm.D_, D_alpha=dm.D_alpha_,
                        gamma13=g13, G=G, M=M, Gp=Gp, Mp=Mp)


def test_roll(N, seed=0):
    """Swiss roll recipe of the reference test-suite fixture (t~U(0,4pi), height U(0,2), /std)."""
    rng = np.random.default_rng(seed)
    t = rng.uniform(0, 4 * np.pi, N)
    X = np.stack([t * np.cos(t), t * np.sin(t), rng.uniform(0, 2, N)], axis=1)
    return X / X.std()


def main(ref_root):
    K, D, E, U = _ref_modules(ref_root)
    sys.path.insert(0, REPO)
    from flashdiffusion_b200 import synthetic
    quiet = contextlib.redirect_stdout(io.StringIO())

    X = test_roll(150)
    np.savez_compressed(os.path.join(HERE, "prepass.npz"), X=X,
                        D64=K.prepass_rowsum(X, X, beta=1.0, tile=64),
                        D256=K.prepass_rowsum(X, X, beta=1.0, tile=256),
                        w=np.linspace(0.5, 1.5, 150),
                        Dw=K.prepass_rowsum(X, X, beta=0.7, weights_k=np.linspace(0.5, 1.5, 150), tile=64))

    v = np.random.default_rng(7).standard_normal(150)
    outs = {}
    for n, (beta, alpha) in enumerate([(1.0, 0.5), (0.5, 0.0), (2.0, 1.0)]):
        dm = D.DiffusionMap(beta=beta, alpha=alpha, tile=64)
        with quiet:
            dm.fit(X)
        outs[f"rscale{n}"] = dm.rscale_
        outs[f"out{n}"] = K.FlashDiffusion(X, X, v[:, None], beta=beta,
                                           rscale_q=dm.rscale_, rscale_k=dm.rscale_).ravel()
    np.savez_compressed(os.path.join(HERE, "matvec.npz"), X=X, v=v,
                        pairs=np.array([(1.0, 0.5), (0.5, 0.0), (2.0, 1.0)]), **outs)

    X3 = test_roll(300)
    dm = D.DiffusionMap(beta=1.0, alpha=0.5, n_components=6, tile=128)
    with quiet:
        dm.fit(X3)
        coords = dm.transform()
    np.savez_compressed(os.path.join(HERE, "fit.npz"), X=X3, D=dm.D_, D_alpha=dm.D_alpha_, rscale=dm.rscale_)
    np.savez_compressed(os.path.join(HERE, "eig.npz"), X=X3, vals=dm.eigenvalues_, coords=coords, k=6)

    X1 = test_roll(100)
    dm1 = D.DiffusionMap(beta=1.0, alpha=0.5, n_components=4, tile=64)
    with quiet:
        dm1.fit(X1)
    h = np.exp(-(X1 ** 2).sum(1))
    doob = dm1.doob_transform(h)
    vd = np.random.default_rng(3).standard_normal(100)
    np.savez_compressed(os.path.join(HERE, "doob.npz"), X=X1, h=h, rscale=dm1.rscale_,
                        Ph=doob.Ph_, v=vd, out=doob.matvec(vd))

    rng = np.random.default_rng(11)
    Qa = rng.standard_normal((130, 5)).astype(np.float32)
    Ka = rng.standard_normal((170, 5)).astype(np.float32)
    Va = rng.standard_normal((170, 3))
    rq = rng.uniform(0.5, 2.0, 130)
    rk = rng.uniform(0.5, 2.0, 170)
    ha = rng.uniform(0.1, 1.0, 170)
    np.savez_compressed(os.path.join(HERE, "amap.npz"), Q=Qa, K=Ka, V=Va, rq=rq, rk=rk, h=ha, beta=0.3,
                        out=K.FlashDiffusion(Qa, Ka, Va, beta=0.3, rscale_q=rq, rscale_k=rk, h=ha, tile=64),
                        out_plain=K.FlashDiffusion(Qa, Ka, Va, beta=0.3, tile=64))

    Xt = test_roll(200, seed=1)
    Xn = test_roll(40, seed=2)
    dmn = D.DiffusionMap(beta=1.0, alpha=0.5, n_components=5, tile=64)
    with quiet:
        dmn.fit(Xt)
        dmn.transform()
        cn = U.nystrom_extend(dmn, Xn, t=1)
    np.savez_compressed(os.path.join(HERE, "nystrom.npz"), Xt=Xt, Xn=Xn, D=dmn.D_, rscale=dmn.rscale_,
                        vals=dmn.eigenvalues_, vecs=dmn.eigenvectors_, coords=cn)

    Xg, bg = synthetic.gaussian_mixture(n=1024, d=64, seed=5)
    dmg = D.DiffusionMap(beta=bg, alpha=0.5, tile=256)
    with quiet:
        dmg.fit(Xg)
    vg = np.random.default_rng(9).standard_normal(1024)
    np.savez_compressed(os.path.join(HERE, "gmm64.npz"), X=Xg, beta=bg, D=dmg.D_, rscale=dmg.rscale_,
                        v=vg, out=dmg.matvec(vg))

    Xc, bc, _ = synthetic.swiss_roll(n=4096, seed=0)
    dmc = D.DiffusionMap(beta=bc, alpha=0.5, n_components=8, tile=512)
    with quiet:
        dmc.fit(Xc)
        dmc.transform()
    np.savez_compressed(os.path.join(HERE, "c1.npz"), X=Xc, beta=bc, D=dmc.D_, rscale=dmc.rscale_,
                        vals=dmc.eigenvalues_)
    bandwidth(U)
    cdc(ref_root)
    rope(ref_root)
    print("golden fixtures written to", HERE)


def bandwidth(U):
    Xb = np.random.default_rng(21).standard_normal((3000, 5)) * np.array([1.0, 2.0, 0.5, 1.0, 3.0])
    Xk = Xb[:1200]
    np.savez_compressed(os.path.join(HERE, "bandwidth.npz"), X=Xb, median_beta=U.median_bandwidth(Xb),
                        median_beta_small=U.median_bandwidth(Xb[:500]), Xk=Xk,
                        sigma7=U.knn_bandwidth(Xk, k=7), sigma5=U.knn_bandwidth(Xk, k=5))


if __name__ == "__main__":
    # usage: make_golden.py REFERENCE_ROOT [bandwidth|cdc|rope]   (the second form writes that fixture only)
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("FD_REFERENCE_ROOT", "")
    if len(sys.argv) > 2 and sys.argv[2] == "bandwidth":
        bandwidth(_ref_modules(root)[3])
    elif len(sys.argv) > 2 and sys.argv[2] == "cdc":
        cdc(root)
    elif len(sys.argv) > 2 and sys.argv[2] == "rope":
        rope(root)
    else:
        main(root)
