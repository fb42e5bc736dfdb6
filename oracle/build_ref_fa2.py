"""Build the reference's own attention operator as a checker (TEST INFRASTRUCTURE ONLY).

Compiles the reference's unmodified flash_attn/flash_attn.cpp and
flash_attn/fa2_tma_lazy_rescale.cu, read in place from the reference checkout
(never copied), into oracle/_ref/ref_fa2.so for sm_100a with torch's extension
builder — the same two sources and flags the reference's own
flash_attn/main.py:17-24 passes, plus the sm_100a target and the libcuda stub
for cuTensorMapEncodeTiled.  The module exposes the reference's
fa2_tma_lazy_rescale(Q, K, V) (flash_attn/flash_attn.cpp:28-30).  Only
tests/golden/make_golden_attn.py and tests/ load it.

    python oracle/build_ref_fa2.py [REF_FLASH_ATTN_DIR]

Skipped quietly when the reference checkout is absent (a GPU box uses the
prebuilt oracle/_ref copy that travels with the repository).
"""
import os
import shutil
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT_DIR = os.path.join(HERE, "_ref")
NAME = "ref_fa2"
DEFAULT_SRC = "/root/reference/flash_attn"


def out_path() -> str:
    return os.path.join(OUT_DIR, NAME + ".so")


def build(src_dir: str = DEFAULT_SRC, force: bool = False) -> str | None:
    srcs = [os.path.join(src_dir, "flash_attn.cpp"), os.path.join(src_dir, "fa2_tma_lazy_rescale.cu")]
    if not all(os.path.exists(p) for p in srcs):
        print(f"reference attention sources not found in {src_dir}; skipping oracle/_ref/{NAME}.so")
        return None
    dst = out_path()
    if not force and os.path.exists(dst) and all(os.path.getmtime(dst) >= os.path.getmtime(p) for p in srcs):
        return dst
    import torch.utils.cpp_extension as ce

    build_dir = os.path.join(OUT_DIR, NAME + "_build")
    os.makedirs(build_dir, exist_ok=True)
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    try:
        ce.load(
            name=NAME,
            sources=srcs,
            extra_cflags=["-std=c++20"],
            extra_cuda_cflags=["-O3", "-std=c++20", "-lineinfo", "-gencode", "arch=compute_100a,code=sm_100a"],
            extra_ldflags=[f"-L{cuda_home}/lib64/stubs", "-lcuda"],
            build_directory=build_dir,
            with_cuda=True,
            is_python_module=True,
            verbose=False,
        )
    except ImportError as e:
        # Built, but a host without a GPU driver has no libcuda.so.1 to import it with.
        if "libcuda" not in str(e) or not os.path.exists(os.path.join(build_dir, NAME + ".so")):
            raise
    shutil.copyfile(os.path.join(build_dir, NAME + ".so"), dst)
    shutil.rmtree(build_dir, ignore_errors=True)
    return dst


def load():
    """Import oracle/_ref/ref_fa2.so (needs a GPU to run, not to import)."""
    import importlib.machinery
    import importlib.util

    import torch  # noqa: F401  (the module links against libtorch)

    path = out_path()
    loader = importlib.machinery.ExtensionFileLoader(NAME, path)
    spec = importlib.util.spec_from_file_location(NAME, path, loader=loader)
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    return mod


if __name__ == "__main__":
    print(build(sys.argv[1] if len(sys.argv) > 1 else DEFAULT_SRC, force="--force" in sys.argv))
