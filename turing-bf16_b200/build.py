"""Builds libtbf16_sm100.so, the C-ABI library of the sm_100a kernels, from csrc/*.cu with nvcc.

    python turing-bf16_b200/build.py [--force]

Objects go to turing-bf16_b200/_build/, the library to turing-bf16_b200/tbf16/lib/ (in-tree, so it
travels with the source tree). Rebuilds only when a source or header is newer than the library.
"""
import concurrent.futures as cf
import os
import pathlib
import shutil
import subprocess
import sys

HERE = pathlib.Path(__file__).resolve().parent
ROOT = HERE.parent
CSRC = HERE / "csrc"
OBJ = HERE / "_build"
LIB = HERE / "tbf16" / "lib" / "libtbf16_sm100.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr", "-Xptxas", "-v"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found (set NVCC or put the CUDA toolkit on PATH)")


def sources():
    return sorted(CSRC.glob("*.cu"))


def deps():
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh")) + sorted((ROOT / "include").glob("*.h"))


def stale() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    return any(p.stat().st_mtime > t for p in deps())


def _compile(src: pathlib.Path):
    obj = OBJ / (src.stem + ".o")
    log = OBJ / (src.stem + ".log")
    cmd = [nvcc(), *ARCH, *FLAGS, "-c", str(src), "-o", str(obj)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    log.write_text(" ".join(cmd) + "\n" + r.stdout + r.stderr)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{r.stderr[-4000:]}")
    return obj


def build(force: bool = False, verbose: bool = False) -> pathlib.Path:
    if not force and not stale():
        return LIB
    OBJ.mkdir(exist_ok=True)
    LIB.parent.mkdir(parents=True, exist_ok=True)
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(_compile, sources()))
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH, "-shared", "-o", str(tmp), *map(str, objs)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stderr[-4000:]}")
    os.replace(tmp, LIB)
    if verbose:
        print(f"built {LIB}")
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
