"""Build the native parts of b200_gemm in-tree (no JIT cache outside the repo).

  python cuda-kernels_b200/b200_gemm/build.py   builds (this file imports nothing
  from the package, so it runs before the library exists):
    b200_gemm/libb200_gemm.so          C-ABI library (include/b200_gemm.h), sm_100a
    bf16_matmul/b200_matmul_ext.*.so   torch extension mirroring the reference's
                                       bf16_matmul/matmul.cpp binding
    flash_attn/b200_flash_attn_ext.so  torch extension mirroring the reference's
                                       flash_attn/flash_attn.cpp binding

Every CUDA compile targets sm_100a explicitly
(-gencode arch=compute_100a,code=sm_100a); nothing here depends on the GPU
being present, so the build runs on a CPU-only host.
"""
from __future__ import annotations

import glob
import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG_DIR)  # cuda-kernels_b200/
REPO = os.path.dirname(ROOT)
CSRC = os.path.join(ROOT, "csrc")
INCLUDE = os.path.join(REPO, "include")
LIB_PATH = os.path.join(PKG_DIR, "libb200_gemm.so")
EXT_DIR = os.path.join(ROOT, "bf16_matmul")
EXT_NAME = "b200_matmul_ext"
# Torch extensions: (name, directory, source), each linked against the C-ABI library.
EXTENSIONS = [
    (EXT_NAME, EXT_DIR, "matmul.cpp"),
    ("b200_flash_attn_ext", os.path.join(ROOT, "flash_attn"), "flash_attn.cpp"),
]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
]


def _nvcc() -> str:
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    cand = os.path.join(cuda_home, "bin", "nvcc")
    return cand if os.path.exists(cand) else "nvcc"


def _sources() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cuh"))
                  + [os.path.join(INCLUDE, "b200_gemm.h")])


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build_lib(force: bool = False, verbose: bool = False) -> str:
    """Compile csrc/*.cu into the C-ABI shared library."""
    if not force and not _stale(LIB_PATH, _sources()):
        return LIB_PATH
    cus = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    tmp = LIB_PATH + ".tmp"
    cmd = [_nvcc(), *NVCC_FLAGS, "-shared", "-I", INCLUDE, "-o", tmp, *cus]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


def ext_path(name: str = EXT_NAME, ext_dir: str = EXT_DIR) -> str | None:
    hits = sorted(glob.glob(os.path.join(ext_dir, name + "*.so")))
    return hits[0] if hits else None


def _build_one(name: str, ext_dir: str, source: str, force: bool, verbose: bool) -> str:
    src = os.path.join(ext_dir, source)
    cur = ext_path(name, ext_dir)
    if not force and cur is not None and not _stale(cur, [src, LIB_PATH, os.path.join(INCLUDE, "b200_gemm.h")]):
        return cur
    import torch.utils.cpp_extension as ce

    build_dir = os.path.join(ext_dir, "_build")
    os.makedirs(build_dir, exist_ok=True)
    rel = os.path.relpath(PKG_DIR, ext_dir)
    ce.load(
        name=name,
        sources=[src],
        extra_cflags=["-O3", "-std=c++17", f"-I{INCLUDE}"],
        extra_ldflags=[f"-L{PKG_DIR}", "-lb200_gemm", f"-Wl,-rpath,{PKG_DIR}", f"-Wl,-rpath,$ORIGIN/{rel}"],
        build_directory=build_dir,
        with_cuda=True,
        verbose=verbose,
        is_python_module=True,
    )
    built = os.path.join(build_dir, name + ".so")
    dst = os.path.join(ext_dir, name + ".so")
    shutil.copyfile(built, dst)
    shutil.rmtree(build_dir, ignore_errors=True)
    return dst


def build_ext(force: bool = False, verbose: bool = False) -> str:
    """Build the torch-extension bindings (bf16_matmul/matmul.cpp, flash_attn/flash_attn.cpp) against the
    C-ABI library; returns the GEMM extension's path."""
    paths = [_build_one(n, d, s, force, verbose) for n, d, s in EXTENSIONS]
    return paths[0]


def main(argv: list[str]) -> int:
    force = "--force" in argv
    verbose = "-v" in argv or "--verbose" in argv
    print(build_lib(force=force, verbose=verbose))
    if "--no-ext" not in argv:
        build_ext(force=force, verbose=verbose)
        for n, d, _ in EXTENSIONS:
            print(ext_path(n, d))
    return 0


if __name__ == "__main__":
    sys.exit(main(sys.argv[1:]))
