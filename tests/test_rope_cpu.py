"""Host-side helpers of the RoPE-DMAP encoder (window and position builders)."""
import numpy as np
import pytest


def test_hankel_windows_and_positions():
    from flashdiffusion_b200.rope import make_hankel_windows, make_window_positions
    F = np.arange(20.0).reshape(10, 2)
    W = make_hankel_windows(F, L=3, step=2)
    assert W.shape == (6, 3, 2)
    np.testing.assert_array_equal(W[1, 2], F[5])
    P = make_window_positions(np.arange(10.0), 3, 2, "sample")
    np.testing.assert_array_equal(P[1], [1, 3, 5])
    np.testing.assert_array_equal(make_window_positions(np.arange(10.0), 3, 2, "window", "center"), np.arange(6) + 2)
    with pytest.raises(ValueError):
        make_hankel_windows(F, L=6, step=2)
    with pytest.raises(ValueError):
        make_window_positions(np.arange(10.0), 3, 2, "window", "middle")
