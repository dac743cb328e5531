"""Build the sm_100a shared library ``motif_ssm/libmotif_ssm.so`` from ``csrc/*.cu``.

nvcc cross-compiles for sm_100a without a GPU.  Objects are built in parallel under
``_build/`` (git-ignored) and linked into one shared library with the CUDA runtime
linked statically, so the library needs only the driver at run time.

    python motif-mamba_b200/build.py [--force] [--jobs N] [--ptxas-verbose]
"""
import argparse
import concurrent.futures as cf
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
OUT = os.path.join(HERE, "motif_ssm", "libmotif_ssm.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
         "--expt-relaxed-constexpr", "-I" + CSRC, "-I" + os.path.join(ROOT, "include")]


def _sources():
    return sorted(f for f in os.listdir(CSRC) if f.endswith(".cu"))


def _deps_mtime():
    return max(os.path.getmtime(os.path.join(d, f))
               for d in (CSRC, os.path.join(ROOT, "include"))
               for f in os.listdir(d) if f.endswith((".cu", ".cuh", ".h")))


def _compile(src, verbose):
    obj = os.path.join(BUILD, src[:-3] + ".o")
    cmd = [NVCC, *ARCH, *FLAGS, "-c", os.path.join(CSRC, src), "-o", obj]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    return obj, r.stderr


def build(force=False, jobs=None, verbose=False):
    if not force and os.path.exists(OUT) and os.path.getmtime(OUT) >= _deps_mtime():
        return OUT
    os.makedirs(BUILD, exist_ok=True)
    srcs = _sources()
    with cf.ThreadPoolExecutor(max_workers=jobs or min(8, len(srcs))) as ex:
        results = list(ex.map(lambda s: _compile(s, verbose), srcs))
    if verbose:
        for (_, log), s in zip(results, srcs):
            sys.stderr.write(f"== {s}\n{log}")
    objs = [o for o, _ in results]
    tmp = OUT + ".tmp"
    cmd = [NVCC, *ARCH, "-shared", "-cudart", "static", "-o", tmp, *objs]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, OUT)
    return OUT


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=None)
    ap.add_argument("--ptxas-verbose", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, jobs=a.jobs, verbose=a.ptxas_verbose))
