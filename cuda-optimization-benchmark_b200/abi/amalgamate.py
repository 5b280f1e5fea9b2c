"""Generate the per-task drop-in sources abi/<task>/solution.cu.

The reference grader builds a kernel from one file: it copies only `solution.cu` next to a shim
that includes it and calls the task's plain C++ `void reference(...)` (graders/grade.py:85-113).
Each solution.cu produced here is therefore a single self-contained translation unit: the task's
drop-in header (csrc/dropin/<task>.cuh) with every project header it includes inlined once, in
include order, followed by `void reference(...)` with the exact signature of
tasks/<task>/tests/task.json:3 forwarding to that drop-in body.

    python abi/amalgamate.py           # (re)write all six files
    python abi/amalgamate.py --check   # exit 1 if a committed file is stale
"""
import re
import sys
from pathlib import Path

ABI = Path(__file__).resolve().parent
CSRC = ABI.parent / "csrc"

TASKS = {
    "pow_abs_sqrt_mean": (
        "void reference(const float* inp, const float* target, int64_t batch_size, int64_t height, int64_t width, "
        "float* output)",
        "b200::dropin::pow_abs_sqrt_mean(inp, target, batch_size, height, width, output)"),
    "ppo_clip": (
        "void reference(const int32_t B, const int32_t T, const int32_t H, const float* current_log_prob, "
        "const float* old_log_prob, const float* advantage, const float clip_epsilon, float* output)",
        "b200::dropin::ppo_clip(B, T, H, current_log_prob, old_log_prob, advantage, nullptr, clip_epsilon, output)"),
    "reward_to_go": (
        "void reference(const float* reward, const bool* done, float gamma, int32_t B, int32_t T, float* output)",
        "b200::dropin::reward_to_go(reward, done, gamma, B, T, output)"),
    "leaky": (
        "void reference(const float* input_current, const float* mem0, const float* beta, const float* threshold, "
        "int32_t T, int32_t B, int32_t H, float* spikes, float* final_mem)",
        "b200::dropin::leaky(input_current, mem0, beta, threshold, T, B, H, spikes, final_mem)"),
    "efficient_kan": (
        "void reference(const float* x, const float* grid, const float* base_weight, const float* spline_weight, "
        "const float* spline_scaler, int32_t grid_size, int32_t spline_order, int32_t B, int32_t I, int32_t O, "
        "float* out)",
        "b200::dropin::efficient_kan(x, grid, base_weight, spline_weight, spline_scaler, grid_size, spline_order, B, "
        "I, O, out)"),
    "fp8_linear": (
        "void reference(const int32_t M, const int32_t K, const int32_t N, const __nv_fp8_e4m3* x_fp8, float scale_x, "
        "const __nv_fp8_e4m3* w_fp8, float scale_w, const __nv_bfloat16* bias, __nv_bfloat16* output)",
        "b200::dropin::fp8_linear(M, K, N, reinterpret_cast<const uint8_t*>(x_fp8), scale_x, "
        "reinterpret_cast<const uint8_t*>(w_fp8), scale_w, reinterpret_cast<const uint16_t*>(bias), "
        "reinterpret_cast<uint16_t*>(output))"),
}

INCLUDE = re.compile(r'^\s*#\s*include\s+"([^"]+)"')
BUILD = ABI / "_build"
# The reference grader's nvcc flags (graders/grade.py:40,104-107), arch for B200.
GRADER_FLAGS = ["-arch=sm_100a", "-O3", "-shared", "-Xcompiler", "-fPIC", "-cudart", "shared", "-Xlinker",
                "-Bsymbolic"]


def params(task):
    """[(c type, name)] of the task's `void reference(...)` signature."""
    inner = TASKS[task][0].split("(", 1)[1].rsplit(")", 1)[0]
    out = []
    for p in inner.split(","):
        p = " ".join(p.split())
        name = re.findall(r"[A-Za-z_]\w*", p)[-1]
        out.append((p[: p.rindex(name)].strip(), name))
    return out


def shim(task):
    """A grader-style shim: includes solution.cu and exposes extern "C" grader_entry(void** a),
    where a[i] is the address of argument i's value (the grader's calling protocol)."""
    args = []
    for i, (ctype, _) in enumerate(params(task)):
        t = ctype if "*" in ctype else ctype.replace("const ", "", 1)
        args.append(f"*({t}*)a[{i}]")
    return '#include "solution.cu"\nextern "C" void grader_entry(void** a) { reference(' + ", ".join(args) + "); }\n"


def build_grader_lib(task, nvcc="nvcc"):
    """Compile abi/<task>/solution.cu with the grader's command line into abi/_build/<task>/kernel.so."""
    import shutil
    import subprocess
    d = BUILD / task
    d.mkdir(parents=True, exist_ok=True)
    shutil.copyfile(ABI / task / "solution.cu", d / "solution.cu")
    (d / "shim.cu").write_text(shim(task))
    r = subprocess.run([nvcc, *GRADER_FLAGS, "-o", "kernel.so", "shim.cu"], cwd=d, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"grader-style build of {task} failed:\n{r.stderr[-3000:]}")
    return d / "kernel.so"


def inline(path, seen, out):
    path = path.resolve()
    if path in seen:
        return
    seen.add(path)
    out.append(f"// ---- {path.relative_to(CSRC).as_posix()}")
    for line in path.read_text().splitlines():
        m = INCLUDE.match(line)
        if m:
            inline(path.parent / m.group(1), seen, out)
            continue
        if line.strip() == "#pragma once":
            continue
        out.append(line)


def render(task):
    sig, call = TASKS[task]
    body = []
    inline(CSRC / "dropin" / f"{task}.cuh", set(), body)
    head = [
        f"// solution.cu for task {task}: B200 (sm_100a) drop-in for the reference's `void reference(...)`.",
        "// Generated by abi/amalgamate.py from csrc/ (one translation unit; do not edit by hand).",
        "// Build as the reference grader does, with -arch=sm_100a.",
        "#include <cuda_bf16.h>",
        "#include <cuda_fp8.h>",
        "#include <stdint.h>",
        "",
    ]
    tail = [
        "",
        f"{sig} {{",
        f"  (void){call};",
        "}",
        "",
    ]
    return "\n".join(head + body + tail)


def main(check=False):
    stale = []
    for task in TASKS:
        dst = ABI / task / "solution.cu"
        text = render(task)
        if check:
            if not dst.exists() or dst.read_text() != text:
                stale.append(task)
        else:
            dst.parent.mkdir(parents=True, exist_ok=True)
            dst.write_text(text)
    if check and stale:
        print("stale:", ", ".join(stale))
        return 1
    return 0


if __name__ == "__main__":
    sys.exit(main(check="--check" in sys.argv))
