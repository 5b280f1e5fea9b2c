"""Build of the native library (libb200ops.so) and of the per-task drop-in sources.

Everything is compiled in-tree with nvcc for sm_100a only:

    nvcc -gencode arch=compute_100a,code=sm_100a -O3 -lineinfo -std=c++17 -shared -Xcompiler -fPIC
         -o <package>/libb200ops.so <package>/csrc/capi.cu

The build is skipped when the library is newer than every source under csrc/ and include/.
"""
import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
REPO = PKG.parent
CSRC = PKG / "csrc"
LIB = PKG / "libb200ops.so"
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-shared", "-Xcompiler", "-fPIC", "-Xcompiler", "-O3"]


def nvcc():
    cand = os.environ.get("NVCC")
    if cand:
        return cand
    for p in ("/usr/local/cuda/bin/nvcc",):
        if Path(p).exists():
            return p
    return "nvcc"


def _sources():
    srcs = [p for p in CSRC.rglob("*") if p.suffix in (".cu", ".cuh", ".h")]
    srcs += list((REPO / "include").glob("*.h"))
    return srcs


def up_to_date(lib=LIB):
    if not lib.exists():
        return False
    t = lib.stat().st_mtime
    return all(p.stat().st_mtime <= t for p in _sources())


def build_library(force=False, verbose=False):
    """Compile libb200ops.so in-tree; returns its path.  Raises on a compile error."""
    if not force and up_to_date():
        return LIB
    cmd = [nvcc(), *ARCH_FLAGS, *NVCC_FLAGS, "-o", str(LIB) + ".tmp", str(CSRC / "capi.cu")]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True, cwd=str(CSRC))
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError(f"nvcc failed building {LIB.name} (exit {r.returncode})")
    os.replace(str(LIB) + ".tmp", LIB)
    return LIB


def build_grader_libs(verbose=False):
    """Build every abi/<task>/solution.cu the way the reference grader does (in parallel)."""
    import importlib.util
    from concurrent.futures import ThreadPoolExecutor
    spec = importlib.util.spec_from_file_location("b200_amalgamate", PKG / "abi" / "amalgamate.py")
    am = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(am)
    if am.main(check=True) != 0:
        raise RuntimeError("abi/*/solution.cu are stale: run abi/amalgamate.py")
    with ThreadPoolExecutor(max_workers=6) as ex:
        paths = list(ex.map(lambda t: am.build_grader_lib(t, nvcc()), list(am.TASKS)))
    if verbose:
        for p in paths:
            print(p, flush=True)
    return paths


if __name__ == "__main__":
    print(build_library(force="--force" in sys.argv, verbose=True))
