"""Build libmsda_b200.so (the C-ABI library) in-tree for sm_100a.

    python -m msda_triton_b200.build         # incremental
    python -m msda_triton_b200.build --force

Every .cu file in csrc/ is compiled by nvcc in parallel with
`-gencode arch=compute_100a,code=sm_100a` and linked into
msda_triton_b200/_lib/libmsda_b200.so (statically linked CUDA runtime, so
the library depends on nothing but the driver).

    python -m msda_triton_b200.build --checked

builds the checked variant (-DMSDA_CHECKED, include/msda_b200_checked.h)
into msda_triton_b200/_lib_checked/: the same kernels with bounds checks on
every value gather and value-gradient scatter, for tests and debugging.
Select it at run time with MSDA_B200_LIB=<path of that library>.
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import shutil
import subprocess

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
OBJ_DIR = os.path.join(PKG, "_build")
LIB_DIR = os.path.join(PKG, "_lib")
LIB = os.path.join(LIB_DIR, "libmsda_b200.so")
CHECKED_OBJ_DIR = os.path.join(PKG, "_build_checked")
CHECKED_LIB = os.path.join(PKG, "_lib_checked", "libmsda_b200.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "-Xptxas", "-warn-spills",
]


def _nvcc() -> str:
    cand = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")
    return cand if os.path.exists(cand) else (shutil.which("nvcc") or "nvcc")


def _deps_mtime() -> float:
    files = glob.glob(os.path.join(CSRC, "*")) + glob.glob(os.path.join(INCLUDE, "*.h"))
    return max(os.path.getmtime(f) for f in files)


def _compile(src: str, extra: list[str], obj_dir: str) -> str:
    obj = os.path.join(obj_dir, os.path.basename(src) + ".o")
    cmd = [_nvcc(), *ARCH, *NVCC_FLAGS, *extra, "-I", INCLUDE, "-c", src, "-o", obj]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src}:\n{res.stdout}\n{res.stderr}")
    return obj


def build(force: bool = False, verbose_ptxas: bool = False, checked: bool = False) -> str:
    """Compile every CUDA source and link the shared library; returns its path.
    checked=True builds the bounds-checked variant (-DMSDA_CHECKED)."""
    lib_path = CHECKED_LIB if checked else LIB
    obj_dir = CHECKED_OBJ_DIR if checked else OBJ_DIR
    if not force and os.path.exists(lib_path) and os.path.getmtime(lib_path) >= _deps_mtime():
        return lib_path
    os.makedirs(obj_dir, exist_ok=True)
    os.makedirs(os.path.dirname(lib_path), exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    extra = ["-Xptxas", "-v"] if verbose_ptxas else []
    if checked:
        extra = extra + ["-DMSDA_CHECKED"]
    with cf.ThreadPoolExecutor(max_workers=min(len(srcs), os.cpu_count() or 4)) as ex:
        objs = list(ex.map(lambda s: _compile(s, extra, obj_dir), srcs))
    tmp = lib_path + ".tmp"
    cmd = [_nvcc(), *ARCH, "-shared", "-cudart", "static", *objs, "-o", tmp]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, lib_path)
    return lib_path


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas-verbose", action="store_true")
    ap.add_argument("--checked", action="store_true",
                    help="build the bounds-checked variant into _lib_checked/")
    args = ap.parse_args()
    print(build(force=args.force, verbose_ptxas=args.ptxas_verbose, checked=args.checked))
