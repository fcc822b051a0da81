"""Build the reference's own SM100 kernel module (TEST / BASELINE INFRASTRUCTURE ONLY).

Compiles ``src/flashdiffusion/csrc/flash_diffusion_sm100.cu`` of the reference
checkout *where it lies* (nothing is copied) with torch's extension builder,
for sm_100a, into ``oracle/_ref/`` (git-ignored; it travels to the GPU box with
the other built libraries).  The result is the pybind module
``flash_diffusion_sm100`` with the reference's ``compute_sq_norms``,
``prepass`` and ``matvec``; ``oracle/time_ref_sm100.py`` times it.

Usage: python oracle/build_ref_sm100.py /path/to/FlashDiffusion
"""
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref")


def build(ref_root):
    from torch.utils.cpp_extension import load
    src = os.path.join(ref_root, "src", "flashdiffusion", "csrc", "flash_diffusion_sm100.cu")
    if not os.path.exists(src):
        raise FileNotFoundError(src)
    os.makedirs(OUT, exist_ok=True)
    os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0a")
    load(name="flash_diffusion_sm100", sources=[src], build_directory=OUT, verbose=False,
         extra_cuda_cflags=["-O3", "-gencode=arch=compute_100a,code=sm_100a"])
    return os.path.join(OUT, "flash_diffusion_sm100.so")


if __name__ == "__main__":
    print(build(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("FD_REFERENCE_ROOT", "")))
