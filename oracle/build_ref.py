"""Builds the REFERENCE's own CUDA sources into oracle/_ref/ (TEST INFRASTRUCTURE ONLY).

Compiles tbf16/csrc/gemm_sm75.cu and tbf16/csrc/small_kernels.cu of tech-cosmos/turing-bf16 where
they lie (TBF16_REFERENCE, default: a `reference` directory beside this repository), as torch
extensions for sm_100a, with the
reference's own arithmetic flags (-O3 --use_fast_math, reference tbf16/_ext.py:52-53) and only the
architecture changed. The reference's build system (its JIT loader) is not run. Outputs go only to
oracle/_ref/ (git-ignored; the .so files travel to the GPU box with the source tree), where the GPU
parity tests load them as the reference's fused-path oracle: its mma.sync kernel recompiled for
sm_100a, run on the same inputs as this build's tcgen05 kernel.

    python oracle/build_ref.py
"""
import os
import pathlib
import shutil
import sys

HERE = pathlib.Path(__file__).resolve().parent
OUT = HERE / "_ref"
REF = pathlib.Path(os.environ.get("TBF16_REFERENCE", str(HERE.parent.parent / "reference")))
TARGETS = {"tbf16_ref_gemm": "gemm_sm75.cu", "tbf16_ref_small": "small_kernels.cu"}
FLAGS = ["-O3", "-gencode=arch=compute_100a,code=sm_100a", "--use_fast_math"]


def built() -> bool:
    return all((OUT / f"{name}.so").exists() for name in TARGETS)


def build():
    src_dir = REF / "tbf16" / "csrc"
    if not src_dir.exists():
        print(f"reference sources not found at {src_dir}; oracle/_ref not built")
        return False
    os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0a")
    from torch.utils.cpp_extension import load
    OUT.mkdir(exist_ok=True)
    for name, src in TARGETS.items():
        work = OUT / f"build_{name}"
        work.mkdir(exist_ok=True)
        load(name=name, sources=[str(src_dir / src)], extra_cuda_cflags=FLAGS, build_directory=str(work),
             verbose=False, is_python_module=True)
        shutil.copy2(work / f"{name}.so", OUT / f"{name}.so")
    return True


def load_ref(name):
    """Import a built reference extension from oracle/_ref (torch must be imported first)."""
    import importlib.machinery
    import importlib.util
    import torch  # noqa: F401  (provides the libraries the extension links against)
    path = OUT / f"{name}.so"
    loader = importlib.machinery.ExtensionFileLoader(name, str(path))
    spec = importlib.util.spec_from_file_location(name, str(path), loader=loader)
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    return mod


if __name__ == "__main__":
    sys.exit(0 if build() else 1)
