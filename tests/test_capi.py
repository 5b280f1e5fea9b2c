"""CPU: the C-ABI library builds for sm_100a, loads without a GPU, and exports every function
that include/*.h declares, with a matching ctypes binding (no compute calls here)."""
import re
import subprocess
from pathlib import Path

import pytest

from conftest import REPO, pkg

HEADERS = sorted((REPO / "include").glob("*.h"))


def declared_functions():
    names = {}
    for h in HEADERS:
        text = h.read_text()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        text = re.sub(r"//[^\n]*", "", text)
        for m in re.finditer(r"\b([A-Za-z_][\w\s\*]*?)\b(b200_\w+)\s*\(([^;{]*?)\)\s*;", text, flags=re.S):
            args = m.group(3).strip()
            n = 0 if args in ("", "void") else len(args.split(","))
            names[m.group(2)] = n
    return names


@pytest.fixture(scope="module")
def lib():
    p = pkg()
    p._build.build_library()
    return p.load()


def test_header_declares_functions():
    d = declared_functions()
    assert len(d) >= 20
    assert "b200_pow_abs_sqrt_mean" in d and d["b200_pow_abs_sqrt_mean"] == 6


def test_library_exports_every_declared_symbol(lib):
    exported = subprocess.run(["nm", "-D", "--defined-only", str(pkg()._build.LIB)], capture_output=True,
                              text=True, check=True).stdout
    syms = {line.split()[-1] for line in exported.splitlines() if line.strip()}
    for name in declared_functions():
        assert name in syms, f"{name} declared in include/ but not exported"
        assert getattr(lib, name) is not None


def test_ctypes_bindings_match_header():
    sigs = pkg()._native.SIGNATURES
    decl = declared_functions()
    assert set(sigs) == set(decl), set(sigs) ^ set(decl)
    for name, nargs in decl.items():
        assert len(sigs[name][1]) == nargs, name


def test_no_host_only_queries_need_a_gpu(lib):
    """Pure size queries answer without a device."""
    assert lib.b200_robust_l1_chunk_elems() == 8192
    assert lib.b200_ppo_chunk_elems() == 4096
    assert lib.b200_ppo_partial_bytes() == 48
    assert lib.b200_robust_l1_workspace_bytes(1 << 26) == 256 + 8192 * 8
    assert lib.b200_status_string(0) == b"ok"


def test_chunked_reward_to_go_workspace_layout(lib):
    """The chunked reward-to-go's workspace: 256 bytes of control words (the grid-barrier count),
    then per 1056-step chunk its map (16 B), carry (8 B) and 32 lane suffix maps (512 B), and per
    block of 8 chunks its map (16 B) and carry (8 B); -1 for negative sizes, 0 for empty ones."""
    def expect(B, T):
        nch = (T + 1055) // 1056
        nblk = (nch + 7) // 8
        return 256 + B * nch * (16 + 8 + 512) + B * nblk * (16 + 8)
    for B, T in [(1, 1), (8, 1 << 21), (3, 9000), (4096, 1000), (1, 70_000_000)]:
        assert lib.b200_reward_to_go_chunked_workspace_bytes(B, T) == expect(B, T), (B, T)
    assert lib.b200_reward_to_go_chunked_workspace_bytes(0, 5) == 0
    assert lib.b200_reward_to_go_chunked_workspace_bytes(-1, 5) == -1


def test_built_for_sm100a_only():
    """The fatbinary holds sm_100a code (checked from the build command, not by reading binaries)."""
    b = pkg()._build
    assert b.ARCH_FLAGS == ["-gencode", "arch=compute_100a,code=sm_100a"]
    assert Path(b.LIB).exists()


def test_amalgamations_are_current():
    """abi/<task>/solution.cu (the grader drop-ins) match what abi/amalgamate.py generates now."""
    import importlib.util
    spec = importlib.util.spec_from_file_location("b200_amalgamate_c", REPO / "cuda-optimization-benchmark_b200" /
                                                  "abi" / "amalgamate.py")
    am = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(am)
    assert am.main(check=True) == 0
    for task in am.TASKS:
        text = (am.ABI / task / "solution.cu").read_text()
        assert am.TASKS[task][0] + " {" in text      # the verbatim reference signature
        assert "#include \"" not in text             # one self-contained translation unit
