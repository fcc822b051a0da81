"""Wait-time breakdown of the block tile kernel (tc_block_kernel) on one GPU.

Loads ``libfd_sm100_prof.so`` (``build.build_profile()``: the library with
``-DFD_PROFILE_WAITS``), runs the configuration-5 block product (d = 128,
r = 32, fp16 tiles) on N seeded tanh-manifold points, and prints the cycles
that lane 0 of each warp of CTA 0 spent in each pipeline wait and inside the
MMA issue loops during one launch, per 128 x 128 tile of that CTA.

Usage: python -m flashdiffusion_b200.profile_waits [N] [products]   (products: 0 = default, 2 or 3)
"""
import ctypes
import os
import sys

NAMES = ["qempty (K producer)", "kempty (K producer)", "uempty (U producer)", "ufull (2 P.U issuers)",
         "pfull (2 P.U issuers)", "oempty (2 P.U issuers)", "qfull (2 Q.K issuers)", "kfull (2 Q.K issuers)",
         "sempty (2 Q.K issuers)", "sfull (12 epilogue warps)", "ofull (12 epilogue warps)", "done", "-",
         "P.U issue span (2 issuers)", "Q.K issue span (2 issuers)", "whole kernel (CTA 0)"]


def main(n: int = 131072, products: int = 0) -> None:
    import torch
    from . import build, native, synthetic
    from .kernel import GaussianOperator
    native.LIB_PATH = build.build_profile()
    lib = native.load()
    lib.fd_debug_wait_cycles.argtypes = [ctypes.c_void_p]
    X, beta = synthetic.tanh_manifold(n=n, d=128, seed=0)
    op = GaussianOperator(X, None, beta, "f16")
    native.set_block_options(0, products)
    V = torch.randn(n, 32, dtype=torch.float64, device="cuda")
    for _ in range(3):
        op.apply(V)
    torch.cuda.synchronize()
    buf = (ctypes.c_ulonglong * 16)()
    lib.fd_debug_wait_cycles(buf)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    op.apply(V)
    e1.record()
    torch.cuda.synchronize()
    lib.fd_debug_wait_cycles(buf)
    tiles = (n // 128) ** 2 / native.torch.cuda.get_device_properties(0).multi_processor_count
    print("N %d  products %d  launch %.3f ms  tiles per CTA %.0f" % (n, products, e0.elapsed_time(e1), tiles))
    for i, nm in enumerate(NAMES):
        if nm != "-":
            print("%-30s %14d cycles  %8.1f per tile" % (nm, buf[i], buf[i] / tiles))


if __name__ == "__main__":
    main(*(int(a) for a in sys.argv[1:3]))
