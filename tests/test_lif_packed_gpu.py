"""GPU: the LIF layer with bit-packed spikes (b200_leaky_packed_async).

Bit t % 32 of word [t / 32][n] must equal the fp32 spike of neuron n at step t from the reference-
layout entry point (itself bit-exact against the oracle, tests/test_stream_ops_gpu.py), with every
bit past T zero, and final_mem must be bit-identical: on the golden cases, on shapes that take the
one-neuron-per-thread path (B*H not a multiple of 4, unaligned pointers), on T that is not a
multiple of 32, and at the BASELINE.json size.
"""
import pytest
import torch

from conftest import golden_cases, pkg
from oracle import inputs

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    p = pkg()
    p.load()
    return p.ops


def pack(spikes):
    """fp32 spikes [T, B, H] -> int64 words [ceil(T/32), B, H] (bit t % 32 of word t // 32)."""
    T = spikes.shape[0]
    tb = (T + 31) // 32
    s = torch.zeros((tb * 32,) + tuple(spikes.shape[1:]), dtype=torch.int64, device=spikes.device)
    s[:T] = (spikes != 0).to(torch.int64)
    w = (torch.ones(32, dtype=torch.int64, device=spikes.device) << torch.arange(32, device=spikes.device))
    return (s.view(tb, 32, -1) * w.view(1, 32, 1)).sum(1).view((tb,) + tuple(spikes.shape[1:]))


def check(ops, x, m0, be, th, offset=0):
    if offset:
        def shift(t):
            raw = torch.empty(t.numel() + offset, dtype=t.dtype, device=t.device)
            v = raw[offset:].view(t.shape)
            v.copy_(t)
            return v
        x, m0, be, th = shift(x), shift(m0), shift(be), shift(th)
    sp, fm = ops.leaky(x, m0, be, th)
    bits, fm2 = ops.leaky_packed(x, m0, be, th)
    torch.cuda.synchronize()
    assert torch.equal(bits.to(torch.int64) & 0xFFFFFFFF, pack(sp))
    assert torch.equal(fm.view(torch.int32), fm2.view(torch.int32))


CASES = golden_cases("leaky")[:4]


@pytest.mark.parametrize("cid,rec", CASES, ids=[c for c, _ in CASES])
def test_golden_cases(ops, cid, rec):
    s = inputs.task_inputs("leaky", rec["case"], int(rec["case"]["seed"]))
    check(ops, *(s[k].cuda() for k in ("input_current", "mem0", "beta", "threshold")))


@pytest.mark.parametrize("T,B,H,offset", [(1, 3, 129, 0), (33, 5, 1021, 0), (64, 4, 256, 1), (95, 2, 512, 0),
                                          (31, 7, 1024, 0)])
def test_shapes(ops, T, B, H, offset):
    g = torch.Generator(device="cpu").manual_seed(T * 1000 + H)
    x = (torch.randn(T, B, H, generator=g) * 0.5 + 0.3).cuda()
    m0 = (torch.randn(B, H, generator=g) * 0.1).cuda()
    be = (torch.rand(H, generator=g) * 1.4 - 0.2).cuda()  # outside [0, 1] too: clamped
    th = (torch.rand(H, generator=g) + 0.5).cuda()
    check(ops, x, m0, be, th, offset)


def test_baseline_size(ops):
    s = inputs.baseline_inputs("lif", seed=0)
    check(ops, *(s[k].cuda() for k in ("input_current", "mem0", "beta", "threshold")))
