"""GPU parity of the FP8 E4M3 linear layer through the C ABI.

- Every case of tests/task.json and public_cases.json under the grader's 3-call protocol on the
  drop-in entry point, against the fp64 oracle (tolerance 1e-2/1e-2, task.json) and against the
  reference oracle's outputs recorded in tests/golden/.
- The tensor-core path against the CUDA-core path on the same inputs, for each tile width (the
  256 x 256 tiles of the large-problem kernel included) and for the small-M path (M <= 64:
  swapped operands, K split over a cluster of CTAs).
- The BASELINE.json shapes: the two smaller ones against the full fp64 oracle, the two large ones
  against the oracle on a seeded subset of rows.
"""
import ctypes

import numpy as np
import pytest
import torch

from conftest import golden_cases, pkg
from harness import SET_B, three_call
from oracle import exact, inputs

pytestmark = pytest.mark.gpu
CASES = golden_cases("fp8_linear")
ATOL, RTOL = exact.TOLERANCE["fp8_linear"]


@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return pkg().load()


def bf16_bits(t):
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def call_dropin(lib, b, s):
    lib.b200_fp8_linear(s["M"], s["K"], s["N"], b["x_fp8"].ptr, s["scale_x"], b["w_fp8"].ptr, s["scale_w"],
                        b["bias"].ptr, b["output"].ptr)


@pytest.mark.parametrize("cid,rec", CASES, ids=[c for c, _ in CASES])
def test_case_parity(lib, cid, rec):
    case = rec["case"]
    sets = [inputs.task_inputs("fp8_linear", case, int(case["seed"])),
            inputs.task_inputs("fp8_linear", case, int(case["seed"]) + SET_B)]
    outs = {"output": (torch.bfloat16, (case["M"], case["N"]))}
    results, same = three_call(lambda b, s: call_dropin(lib, b, s), sets, ["x_fp8", "w_fp8", "bias"], outs)
    assert lib.b200_last_status() == 0
    assert same
    for s, r in zip(sets, results):
        ref = exact.fp8_linear(s)["output_f64"]
        got = exact.bf16_bits_to_f64(bf16_bits(r["output"]))
        bad, worst = exact.within(got, ref, ATOL, RTOL)
        assert bad == 0, f"{bad} bad, worst {worst:.3g}"
    o = rec["outputs"][0]
    got = exact.bf16_bits_to_f64(bf16_bits(results[0]["output"])).ravel()
    have = got[o["index"]] if "index" in o else got
    bad, worst = exact.within(have, o["values"], ATOL, RTOL)
    assert bad == 0, worst


def _run(lib, fn, s, dev="cuda"):
    x = s["x_fp8"].to(dev)
    w = s["w_fp8"].to(dev)
    bias = s["bias"].to(dev)
    out = torch.empty(s["M"], s["N"], dtype=torch.bfloat16, device=dev)
    st = fn(s["M"], s["K"], s["N"], x.data_ptr(), s["scale_x"], w.data_ptr(), s["scale_w"], bias.data_ptr(),
            out.data_ptr(), None)
    torch.cuda.synchronize()
    assert st == 0
    return out


@pytest.mark.parametrize("shape", [(1, 64, 64), (16, 4096, 512), (128, 256, 256), (300, 384, 1008),
                                   (1024, 2048, 4096), (257, 4096, 528),
                                   # M <= 64: swap-AB with K split over a cluster (split 1 to 8,
                                   # 16 / 32 / 64 columns, partial last W tile and K block)
                                   (5, 130, 4096), (17, 4096, 1040), (33, 1000, 2048), (64, 4096, 4096),
                                   (16, 28672, 1024), (2, 256, 16),
                                   # 256 x 256 tiles (at least four waves of them), exact and ragged
                                   (4096, 10240, 256), (4100, 10250, 272)])
def test_tensor_path_matches_cuda_core_path(lib, shape):
    M, N, K = shape
    s = inputs.baseline_inputs("fp8_linear", seed=7, shape=(M, N, K))
    plan = lib.b200_fp8_linear_plan(M, K, N, ctypes.c_void_p(256), ctypes.c_void_p(256))
    assert plan in (64, 128, 256, 512)
    tcore = _run(lib, lib.b200_fp8_linear_async, s)
    ccore = _run(lib, lib.b200_fp8_linear_cuda_core_async, s)
    a = exact.bf16_bits_to_f64(bf16_bits(tcore))
    b = exact.bf16_bits_to_f64(bf16_bits(ccore))
    bad, worst = exact.within(a, b, ATOL, RTOL)
    assert bad == 0, worst
    ref = exact.fp8_linear(s)["output_f64"]
    bad, worst = exact.within(a, ref, ATOL, RTOL)
    assert bad == 0, worst


def test_unaligned_k_takes_cuda_core_path(lib):
    assert lib.b200_fp8_linear_plan(333, 1000, 3000, ctypes.c_void_p(256), ctypes.c_void_p(256)) == 0
    assert lib.b200_fp8_linear_plan(333, 1024, 3000, ctypes.c_void_p(257), ctypes.c_void_p(256)) == 0


@pytest.mark.parametrize("shape", [(16, 4096, 4096), (1024, 4096, 4096)])
def test_baseline_small_shapes_full_oracle(lib, shape):
    s = inputs.baseline_inputs("fp8_linear", seed=0, shape=shape)
    out = _run(lib, lib.b200_fp8_linear_async, s)
    got = exact.bf16_bits_to_f64(bf16_bits(out))
    bad, worst = exact.within(got, exact.fp8_linear(s)["output_f64"], ATOL, RTOL)
    assert bad == 0, worst


@pytest.mark.parametrize("shape", [(8192, 8192, 8192), (16384, 28672, 8192)])
def test_baseline_large_shapes_row_subset(lib, shape):
    s = inputs.baseline_inputs("fp8_linear", seed=0, shape=shape)
    out = _run(lib, lib.b200_fp8_linear_async, s)
    rows = np.sort(np.random.default_rng(1).choice(shape[0], size=48, replace=False))
    got = exact.bf16_bits_to_f64(bf16_bits(out[torch.from_numpy(rows).cuda()]))
    ref = exact.fp8_linear(s, rows=rows)["output_f64"]
    bad, worst = exact.within(got, ref, ATOL, RTOL)
    assert bad == 0, worst
    assert pkg().load().b200_device_fault() == 0
