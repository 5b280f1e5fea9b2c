"""Build recipe for the reference's own GPU kernels, used as a second checker.

TEST INFRASTRUCTURE, not product code: nothing under the package loads these libraries.

Each task's expert kernel (reference/<task>/solution.cu in the reference checkout, one
self-contained translation unit) is compiled where it lies, never copied, exactly the way the
reference grader builds a kernel (graders/grade.py:39,85-89,100-107): a shim that includes the
source and exposes `extern "C" void grader_entry(void** a)` (a[i] = address of argument i's value),
`nvcc -arch=sm_100a -O3 -shared -Xcompiler -fPIC -cudart shared -Xlinker -Bsymbolic`, and the
task's link libraries (tasks/<task>/tests/task.json "link": cuBLAS for efficient_kan, cuBLASLt for
fp8_linear).  Outputs go to oracle/_ref/<task>/expert.so (git-ignored; they travel with the tree to
the GPU box, where the reference checkout does not exist and this build is skipped).

tests/test_expert_gpu.py runs them on the same inputs as the B200 kernels: their results against
the fp64 oracle pin the oracle to the reference's own GPU implementation, and their times, taken
with the grader's timing rule, are the expert column beside the B200 kernels' times.

The reference grader's call counter (graders/interpose.c, an LD_PRELOAD library that counts the
CUDA runtime calls a graded call makes: allocations, host copies, device-wide synchronizations,
launches, work off the caller's stream) is compiled the same way, with the grader's own command
(graders/grade.py:256-262: gcc -O2 -shared -fPIC -I<cuda include> ... -ldl), into
oracle/_ref/interpose.so; tests/test_call_counts_gpu.py preloads it around the drop-ins.

    python oracle/ref_build.py          # build every task (skips when the checkout is absent)
"""
import importlib.util
import os
import subprocess
import sys
from pathlib import Path

ORACLE = Path(__file__).resolve().parent
REPO = ORACLE.parent
OUT = ORACLE / "_ref"
REFERENCE = Path(os.environ.get("B200_REFERENCE_ROOT", "/root/reference"))
LINK = {"efficient_kan": ["-lcublas"], "fp8_linear": ["-lcublasLt"]}
FLAGS = ["-arch=sm_100a", "-O3", "-shared", "-Xcompiler", "-fPIC", "-cudart", "shared", "-Xlinker", "-Bsymbolic"]


def _amalgamate():
    """The task signatures and the grader-style shim writer of abi/amalgamate.py."""
    path = REPO / "cuda-optimization-benchmark_b200" / "abi" / "amalgamate.py"
    spec = importlib.util.spec_from_file_location("b200_amalgamate_ref", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def tasks():
    return list(_amalgamate().TASKS)


def library(task):
    return OUT / task / "expert.so"


def available():
    return REFERENCE.joinpath("reference").is_dir()


def build_one(task, nvcc="nvcc", verbose=False):
    src = REFERENCE / "reference" / task / "solution.cu"
    if not src.exists():
        raise FileNotFoundError(src)
    d = OUT / task
    d.mkdir(parents=True, exist_ok=True)
    lib = library(task)
    shim = d / "shim.cu"
    text = _amalgamate().shim(task).replace('#include "solution.cu"', f'#include "{src}"')
    if lib.exists() and shim.exists() and shim.read_text() == text and lib.stat().st_mtime >= src.stat().st_mtime:
        return lib
    shim.write_text(text)
    cmd = [nvcc, *FLAGS, "-o", str(lib) + ".tmp", str(shim), *LINK.get(task, [])]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True, cwd=str(d))
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError(f"nvcc failed building the reference kernel of {task} (exit {r.returncode})")
    os.replace(str(lib) + ".tmp", lib)
    return lib


def counter_library():
    return OUT / "interpose.so"


def build_counter(nvcc="nvcc", verbose=False):
    """Compile graders/interpose.c from the reference checkout into oracle/_ref/interpose.so."""
    src = REFERENCE / "graders" / "interpose.c"
    if not src.exists():
        raise FileNotFoundError(src)
    OUT.mkdir(parents=True, exist_ok=True)
    lib = counter_library()
    if lib.exists() and lib.stat().st_mtime >= src.stat().st_mtime:
        return lib
    import shutil
    nv = shutil.which(nvcc) or "/usr/local/cuda/bin/nvcc"
    inc = Path(nv).resolve().parent.parent / "include"
    cmd = [os.environ.get("CC", "gcc"), "-O2", "-shared", "-fPIC", f"-I{inc}", "-o", str(lib) + ".tmp", str(src),
           "-ldl"]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError(f"gcc failed building the reference's call counter (exit {r.returncode})")
    os.replace(str(lib) + ".tmp", lib)
    return lib


def build(nvcc="nvcc", verbose=False):
    """Build every task's expert library when the reference checkout is present; returns the
    library paths (an empty list when it is absent)."""
    if not available():
        return []
    from concurrent.futures import ThreadPoolExecutor
    with ThreadPoolExecutor(max_workers=6) as ex:
        libs = list(ex.map(lambda t: build_one(t, nvcc, verbose), tasks()))
    return libs + [build_counter(nvcc, verbose)]


if __name__ == "__main__":
    for p in build(verbose=True):
        print(p)
