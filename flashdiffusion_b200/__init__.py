"""flashdiffusion_b200 — B200-native (sm_100a) FlashDiffusion Gaussian-kernel operator.

Drop-in for the reference package ``flashdiffusion`` on its hot path:
``FlashDiffusion``, ``prepass_rowsum``, ``DiffusionMap``, ``lanczos_eigsh``,
``lobpcg_eigsh`` keep their names and arguments; the O(N^2) work runs in
libfd_sm100.so (hand-written sm_100a kernels behind a C ABI, include/fd_sm100.h).
"""

from .kernel import FlashDiffusion, GaussianOperator, prepass_rowsum, _get_cuda_backend  # noqa: F401
from .dmap import DiffusionMap, DoobTransformedMap  # noqa: F401
from .eigensolver import lanczos_eigsh, lobpcg_eigsh  # noqa: F401
from . import cdc, rope, utils  # noqa: F401

__all__ = ["FlashDiffusion", "GaussianOperator", "prepass_rowsum", "DiffusionMap", "DoobTransformedMap",
           "lanczos_eigsh", "lobpcg_eigsh"]
