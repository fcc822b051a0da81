"""Time the reference's own SM100 kernels beside this package's (BASELINE INFRASTRUCTURE ONLY).

Loads the module built by ``oracle/build_ref_sm100.py`` from ``oracle/_ref`` and
runs, on the same seeded inputs, the reference's GPU precompute/matvec
(``FD/kernel_cuda_sm100.py:67-119``: fp16 X, sq norms, two prepasses, then the
matvec) and ``flashdiffusion_b200``'s equivalents, each
timed with CUDA events after a warm-up, and checks that the two matvecs agree.
Prints one JSON line.

Usage: python oracle/time_ref_sm100.py [N] [d]      (default the configuration-2 shape)
"""
import importlib.util
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))


def load_ref():
    path = os.path.join(HERE, "_ref", "flash_diffusion_sm100.so")
    spec = importlib.util.spec_from_file_location("flash_diffusion_sm100", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def timed(fn, reps=3):
    fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        out = fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / reps, out


def main(n=200_000, d=64):
    from flashdiffusion_b200 import synthetic, GaussianOperator
    from flashdiffusion_b200.kernel_cuda_sm100 import normalise
    ref = load_ref()
    X, beta = synthetic.gaussian_mixture(n=n, d=d, seed=0) if d == 64 else synthetic.tanh_manifold(n=n, d=d, seed=0)
    dev = torch.device("cuda", 0)
    Xh = torch.from_numpy(X).to(dev).half().contiguous()
    sq = ref.compute_sq_norms(Xh)
    ones = torch.ones(n, dtype=torch.float32, device=dev)
    t_pre_ref, D = timed(lambda: ref.prepass(Xh, ones, sq, float(beta)), reps=1)
    w = D.pow(-0.5)
    Da = ref.prepass(Xh, w, sq, float(beta)) * w
    rs = (Da.pow(-0.5) * w).contiguous()
    v = torch.from_numpy(np.random.default_rng(1).standard_normal(n).astype(np.float32)).to(dev)
    # the module's matvec forms u = rscale * v itself (flash_diffusion_sm100.cu:520-569)
    t_mv_ref, y_ref = timed(lambda: ref.matvec(Xh, v, rs, sq, float(beta)), reps=1)

    op = GaussianOperator(torch.from_numpy(X).to(dev), None, beta, "f16")
    t_pre_ours, _ = timed(lambda: normalise(op, 0.5))
    _, _, rs2 = normalise(op, 0.5)
    t_mv_ours, y = timed(lambda: op.apply(v[:, None], col_scale=rs2, row_scale=rs2, out_dtype=torch.float64))
    diff = float(torch.linalg.vector_norm(y[:, 0] - y_ref.double()) / torch.linalg.vector_norm(y_ref.double()))
    ev = float(n) * n
    print(json.dumps({"n": n, "d": d, "beta": float(beta),
                      "reference_sm100": {"prepass_ms": t_pre_ref, "matvec_ms": t_mv_ref,
                                          "matvec_evals_per_s": ev / (t_mv_ref / 1e3)},
                      "flashdiffusion_b200": {"two_prepasses_ms": t_pre_ours, "matvec_ms": t_mv_ours,
                                              "matvec_evals_per_s": ev / (t_mv_ours / 1e3)},
                      "matvec_rel_l2_between_the_two": diff}))


if __name__ == "__main__":
    main(*(int(a) for a in sys.argv[1:3]))
