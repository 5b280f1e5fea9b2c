"""Per-tensor E4M3 quantisation (the step before fp8_linear, tasks/fp8_linear/reference.py:15-18).

CPU: the oracle's restatement (oracle.inputs._quantize_e4m3) reproduces the reference's own
`_quantize` on every case of tests/golden/fp8_quantize.json (inputs rebuilt bit for bit, scale and
every recorded E4M3 byte equal).

GPU, through the C ABI:
- the kernels give the recorded scale and bytes on every case, from fp32 sources and, for the
  bf16-representable cases, from bf16 sources; also from a source one element past a 16-byte
  boundary (scalar path);
- at the BASELINE.json sizes (bf16 sources of the four fp8 shapes' activations and weights) the
  bytes equal torch's own float8_e4m3fn conversion of the clamped product and the scale equals the
  oracle's;
- the fused bf16 linear layer is bit-identical to quantising and calling fp8_linear, and meets the
  fp64 oracle.
"""
import ctypes
import hashlib
import json

import numpy as np
import pytest
import torch

from conftest import REPO, pkg
from oracle import exact, inputs

GOLDEN = json.loads((REPO / "tests" / "golden" / "fp8_quantize.json").read_text())["cases"]
IDS = [c["name"] for c in GOLDEN]


def _recorded(case, q_bytes):
    """The recorded bytes of a case compared with q_bytes (uint8 numpy array)."""
    if "q" in case:
        return np.array_equal(q_bytes, np.frombuffer(bytes.fromhex(case["q"]), dtype=np.uint8))
    pos = np.asarray(case["positions"])
    return (np.array_equal(q_bytes[pos], np.frombuffer(bytes.fromhex(case["q_at"]), dtype=np.uint8))
            and hashlib.sha256(q_bytes.tobytes()).hexdigest() == case["q_sha256"])


@pytest.mark.parametrize("case", GOLDEN, ids=IDS)
def test_oracle_port_matches_reference(case):
    x = inputs.quant_input(case["name"])
    assert hashlib.sha256(x.numpy().tobytes()).hexdigest() == case["input_sha256"]
    q, scale = inputs._quantize_e4m3(x)
    assert float(scale).hex() == case["scale_hex"]
    assert _recorded(case, q.view(torch.uint8).numpy().ravel())


def test_golden_covers_the_edge_cases():
    names = set(IDS)
    assert {"zeros_16x16", "single", "tiny_17x33", "wide_31x129", "negative_8x64"} <= names
    assert any(c["bf16"] for c in GOLDEN) and any("positions" in c for c in GOLDEN)


# ---------------------------------------------------------------------------------------- GPU
@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return pkg().load()


def _quantize_dev(lib, x, bf16, offset=0):
    """Run the C-ABI quantisation on x (CPU fp32 tensor) placed `offset` elements into a buffer."""
    n = x.numel()
    dt = torch.bfloat16 if bf16 else torch.float32
    raw = torch.empty(n + offset + 1, dtype=dt, device="cuda")
    src = raw[offset:offset + n]
    src.copy_(x.reshape(-1).to(dt))
    qraw = torch.full((n + offset + 16,), 0xEE, dtype=torch.uint8, device="cuda")
    q = qraw[offset:offset + n]
    scale = torch.full((1,), float("nan"), device="cuda")
    ws = torch.zeros(lib.b200_fp8_quantize_workspace_bytes(), dtype=torch.uint8, device="cuda")
    st = lib.b200_fp8_quantize_async(src.data_ptr(), 1 if bf16 else 0, n, q.data_ptr(), scale.data_ptr(),
                                     ws.data_ptr(), ws.numel(), None)
    torch.cuda.synchronize()
    assert st == 0
    assert bool((qraw[offset + n:] == 0xEE).all()), "wrote past the output"
    assert bool((qraw[:offset] == 0xEE).all()), "wrote before the output"
    return q.cpu().numpy(), float(scale.item())


@pytest.mark.gpu
@pytest.mark.parametrize("case", GOLDEN, ids=IDS)
def test_kernel_matches_reference(lib, case):
    x = inputs.quant_input(case["name"])
    for bf16 in ([False, True] if case["bf16"] else [False]):
        for offset in (0, 1):
            q, scale = _quantize_dev(lib, x, bf16, offset)
            assert float(np.float32(scale)).hex() == case["scale_hex"], (bf16, offset)
            assert _recorded(case, q), (bf16, offset)


@pytest.mark.gpu
@pytest.mark.parametrize("rows,cols", [(16, 4096), (1024, 4096), (8192, 8192), (16384, 8192), (28672, 8192)])
def test_baseline_sizes_match_torch(lib, rows, cols):
    g = torch.Generator(device="cuda").manual_seed(rows + cols)
    x = torch.randn(rows, cols, device="cuda", generator=g).to(torch.bfloat16)
    x[0, 0] = 7.25  # a known maximum
    ops = pkg().ops
    q, scale = ops.fp8_quantize(x)
    torch.cuda.synchronize()
    amax = float(x.float().abs().max().item())
    want_scale = float(np.float32(448.0 / max(amax, 1e-9)))
    assert float(scale.item()) == want_scale
    want = (x.float() * want_scale).clamp(-448.0, 448.0).to(torch.float8_e4m3fn)
    assert torch.equal(q.view(torch.uint8), want.view(torch.uint8))


@pytest.mark.gpu
@pytest.mark.parametrize("shape", [(16, 4096, 4096), (1024, 4096, 4096), (300, 1000, 1008), (5, 130, 512)])
def test_fused_linear_matches_separate_calls(lib, shape):
    M, N, K = shape
    ops = pkg().ops
    g = torch.Generator(device="cpu").manual_seed(M * 7 + N)
    x = torch.randn(M, K, generator=g).to(torch.bfloat16).cuda()
    s = inputs.baseline_inputs("fp8_linear", seed=3, shape=shape)
    w, bias = s["w_fp8"].cuda(), s["bias"].cuda()
    scale_x = torch.empty(1, device="cuda")
    fused = ops.fp8_linear_bf16(x, w, s["scale_w"], bias, scale_x=scale_x)
    q, sx = ops.fp8_quantize(x)
    torch.cuda.synchronize()
    assert float(scale_x.item()) == float(sx.item())
    separate = ops.fp8_linear(q, float(sx.item()), w, s["scale_w"], bias)
    torch.cuda.synchronize()
    assert torch.equal(fused.view(torch.int16), separate.view(torch.int16))
    rows = slice(0, min(M, 64))
    ref = exact.fp8_linear({"M": M, "K": K, "N": N, "x_fp8": q.cpu(), "scale_x": float(sx.item()),
                            "w_fp8": s["w_fp8"], "scale_w": s["scale_w"], "bias": s["bias"]}, rows=rows)["output_f64"]
    have = exact.bf16_bits_to_f64(fused[rows].contiguous().view(torch.int16).cpu().numpy().view(np.uint16))
    bad, worst = exact.within(have, ref, *exact.TOLERANCE["fp8_linear"])
    assert bad == 0, worst


@pytest.mark.gpu
def test_status_codes(lib):
    ws = torch.zeros(64, dtype=torch.uint8, device="cuda")
    x = torch.zeros(16, device="cuda")
    # workspace too small, negative count
    assert lib.b200_fp8_quantize_async(x.data_ptr(), 0, 16, None, None, ws.data_ptr(), 8, None) == 4
    assert lib.b200_fp8_quantize_async(x.data_ptr(), 0, -1, None, None, ws.data_ptr(), 4096, None) == 1
    assert lib.b200_fp8_linear_bf16_async(4, 16, 8, x.data_ptr(), x.data_ptr(), 1.0, x.data_ptr(), x.data_ptr(),
                                          None, ws.data_ptr(), 8, None) == 4
