"""Build recipe for the engine's shared libraries (run from anywhere; outputs land in this folder).

  libcuda_inference.so  the C ABI of include/cuda_inference.h: host engine + sm_100a kernels,
                        compiled by nvcc for `-gencode arch=compute_100a,code=sm_100a` only
  librandmodel.so       host-only writer of seeded random-init Qwen3 checkpoints

nvcc cross-compiles sm_100a on a machine without a GPU. The CUDA runtime is linked statically, so
the library does not depend on which libcudart another module of the process loaded.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent
CSRC = HERE / "csrc"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def _stale(out: Path, deps: list[Path]) -> bool:
    return not out.exists() or any(d.stat().st_mtime > out.stat().st_mtime for d in deps)


def build_engine(force: bool = False, verbose: bool = False) -> Path:
    out = HERE / "libcuda_inference.so"
    srcs = [CSRC / "engine.cu", CSRC / "micro_kernels.cu", CSRC / "prefill.cu", CSRC / "model_file.cpp"]
    deps = srcs + list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + [ROOT / "include" / "cuda_inference.h"]
    if not force and not _stale(out, deps):
        return out
    cmd = [nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-shared", "-Xcompiler", "-fPIC,-O2",
           "-cudart", "static", "-I", str(ROOT / "include"), *map(str, srcs), "-o", str(out) + ".tmp"]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    subprocess.run(cmd, check=True)
    os.replace(str(out) + ".tmp", out)
    return out


def build_randmodel(force: bool = False) -> Path:
    out = HERE / "librandmodel.so"
    src = CSRC / "randmodel.cpp"
    if force or _stale(out, [src]):
        subprocess.run(["g++", "-O2", "-std=c++17", "-fPIC", "-shared", "-pthread", str(src), "-o", str(out)], check=True)
    return out


def build_all(force: bool = False, verbose: bool = False) -> None:
    build_randmodel(force)
    build_engine(force, verbose)


if __name__ == "__main__":
    build_all(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print("built", HERE / "libcuda_inference.so", HERE / "librandmodel.so")
