"""Build the reference's own selective-scan CUDA extension (``selective_scan_cuda``) for
sm_100a from its sources where they lie, into ``oracle/_ref/``.  TEST INFRASTRUCTURE ONLY.

The sources, flags and module name follow the reference's ``setup.py:211-263``
(``csrc/selective_scan/selective_scan.cpp`` + the nine ``selective_scan_{fwd,bwd}_*.cu``
instantiations, ``-O3 --use_fast_math`` and the half/bf16 operator flags); only the
architecture is this machine's (``TORCH_CUDA_ARCH_LIST=10.0a``, i.e. sm_100a).  Nothing is
copied into the repository: the build reads the files under ``$MOTIF_REF`` (required: the
reference checkout's ``motifmamba`` project directory) and writes ``oracle/_ref/selective_scan_cuda*.so``, which is git-ignored
but travels with the working tree.  Used only by GPU tests (parity of this library against
the reference kernel) and by ``bench.py --workload refkernel``; the product never loads it.

    MOTIF_REF=<reference>/motifmamba python oracle/build_ref_scan.py   # ~10 min, 4 nvcc threads per file
"""
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref")
REF = os.environ.get("MOTIF_REF")  # the reference project directory; nothing is built without it
SOURCES = ["selective_scan.cpp"] + [f"selective_scan_fwd_{t}.cu" for t in ("fp32", "fp16", "bf16")] + [
    f"selective_scan_bwd_{t}_{k}.cu" for t in ("fp32", "fp16", "bf16") for k in ("real", "complex")]
NVCC_FLAGS = ["-O3", "-std=c++17", "-U__CUDA_NO_HALF_OPERATORS__", "-U__CUDA_NO_HALF_CONVERSIONS__",
              "-U__CUDA_NO_BFLOAT16_OPERATORS__", "-U__CUDA_NO_BFLOAT16_CONVERSIONS__",
              "-U__CUDA_NO_BFLOAT162_OPERATORS__", "-U__CUDA_NO_BFLOAT162_CONVERSIONS__",
              "--expt-relaxed-constexpr", "--expt-extended-lambda", "--use_fast_math", "-lineinfo",
              "--threads", "4"]


def built_path():
    """Path of the built extension, or None."""
    if not os.path.isdir(OUT):
        return None
    for f in sorted(os.listdir(OUT)):
        if f.startswith("selective_scan_cuda") and f.endswith(".so"):
            return os.path.join(OUT, f)
    return None


def load():
    """Import the prebuilt reference extension (no compilation); None when absent."""
    import importlib.machinery
    import importlib.util
    import torch  # noqa: F401  (the extension links against torch's libraries)
    path = built_path()
    if path is None:
        return None
    loader = importlib.machinery.ExtensionFileLoader("selective_scan_cuda", path)
    spec = importlib.util.spec_from_loader("selective_scan_cuda", loader)
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    return mod


def build():
    if not REF:
        raise SystemExit("set MOTIF_REF to the reference's motifmamba project directory")
    src_dir = os.path.join(REF, "csrc", "selective_scan")
    if not os.path.isdir(src_dir):
        print(f"reference sources not found under {src_dir}; nothing built")
        return None
    os.environ["TORCH_CUDA_ARCH_LIST"] = "10.0a"  # torch adds no other architectures
    from torch.utils.cpp_extension import load as cpp_load
    build_dir = os.path.join(OUT, "build")
    os.makedirs(build_dir, exist_ok=True)
    cpp_load(name="selective_scan_cuda", sources=[os.path.join(src_dir, s) for s in SOURCES],
             extra_cflags=["-O3", "-std=c++17"], extra_cuda_cflags=NVCC_FLAGS, extra_include_paths=[src_dir],
             build_directory=build_dir, verbose=False, is_python_module=True)
    so = os.path.join(build_dir, "selective_scan_cuda.so")
    dst = os.path.join(OUT, "selective_scan_cuda.so")
    os.replace(so, dst)
    print(dst)
    return dst


if __name__ == "__main__":
    os.environ.setdefault("MAX_JOBS", str(min(10, os.cpu_count() or 1)))
    sys.exit(0 if build() else 1)
