"""The FMA-pipe exponential of the tensor-core epilogues against the fp64
exponential and CUDA's exp2: the degree-4 polynomial (fitted in
tests/test_exp2_poly.py) must stay within its fp32 Horner bound of 3.7e-6
relative over the whole exponent range the kernels feed it, [-125, 0]."""
import numpy as np
import pytest
import torch

BOUND = 3.7e-6


@pytest.mark.gpu
def test_exp2_poly_within_bound_over_the_exponent_range():
    from flashdiffusion_b200 import native
    dev = native.require_device()
    rng = np.random.default_rng(0)
    x = np.concatenate([np.linspace(-125.0, 0.0, 1_000_001), -125.0 * rng.random(1_000_000),
                        -rng.random(100_000), [0.0, -0.5, -1.5, -124.5, -125.0]]).astype(np.float32)
    xd = torch.from_numpy(x).to(dev)
    y = native.exp2_poly(xd).cpu().numpy().astype(np.float64)
    ref = np.exp2(x.astype(np.float64))
    rel = np.abs(y - ref) / ref
    assert np.isfinite(y).all()
    assert rel.max() < BOUND, (rel.max(), x[np.argmax(rel)])
    y_cuda = torch.exp2(xd).cpu().numpy().astype(np.float64)
    assert np.max(np.abs(y - y_cuda) / ref) < BOUND + 1e-6


@pytest.mark.gpu
def test_exp2_poly_clamp_and_odd_length():
    from flashdiffusion_b200 import native
    dev = native.require_device()
    x = torch.tensor([-200.0, -126.0, -125.0, -3.25, 0.0], dtype=torch.float32, device=dev)
    y = native.exp2_poly(x).cpu().numpy().astype(np.float64)
    ref = np.exp2(np.array([-125.0, -125.0, -125.0, -3.25, 0.0]))
    assert np.all(np.abs(y - ref) / ref < BOUND)
