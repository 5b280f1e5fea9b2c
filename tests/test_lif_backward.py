"""Surrogate-gradient backward of the leaky layer (b200_leaky_train_async / _checkpoints_async /
_backward_async).

There is no backward in the reference repository (its leaky task restates the forward of snnTorch's
Leaky; snnTorch is not a dependency and is absent here).  The oracle (oracle.exact.leaky_backward)
runs the reference's own fp32 forward loop, so every reset and spike decision is the reference's,
then the hand-derived backward recursion in fp64.  It is pinned on the CPU two ways: its forward half
reproduces oracle.exact.leaky (the reference loop, checked against the golden cases elsewhere), and
its gradients equal torch autograd, in fp64, through the same forward written with a straight-
through arctangent surrogate and a detached reset.

GPU, through the C ABI:
- the training forward gives spikes and final_mem bit-identical to b200_leaky_async and checkpoints
  bit-identical to the oracle's fp32 states; the checkpoints-only entry gives the same bits;
- the backward meets the oracle on the golden leaky cases (beta outside [0, 1], H = 1021 and 129),
  T not a multiple of 16, B*H not a multiple of 4, no grad_final_mem, alpha 1 and 4: grad_input and
  grad_mem0 within atol 1e-5 + rtol 1e-4; grad_beta and grad_threshold within 1e-4 times the sum of
  their terms' magnitudes (plus 1e-6): an fp32 summation over T steps per neuron;
- the BASELINE.json LIF size (T=256, B=64, H=4096), every output;
- the outputs do not depend on the inputs' alignment (bit-identical from views one float off);
- torch.autograd through LeakyFunction returns the C-ABI backward's tensors;
- status codes.
"""
import math

import numpy as np
import pytest
import torch

from conftest import golden_cases, pkg
from oracle import exact, inputs

TOL_X = (1e-5, 1e-4)     # grad_input, grad_mem0: atol, rtol
TOL_SUM = (1e-6, 1e-4)   # grad_beta, grad_threshold: atol, fraction of the summed magnitudes


def make(T, B, H, seed, beta=None, th=None):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(T, B, H, generator=g) * 0.5 + 0.3
    mem0 = torch.randn(B, H, generator=g) * 0.5
    be = torch.rand(H, generator=g) * 0.4 + 0.7 if beta is None else beta
    t = torch.rand(H, generator=g) * 0.5 + 0.75 if th is None else th
    gs = torch.randn(T, B, H, generator=g)
    gf = torch.randn(B, H, generator=g)
    return {"input_current": x, "mem0": mem0, "beta": be, "threshold": t}, gs, gf


def autograd_reference(inp, gs, gf, alpha):
    """torch fp64 autograd through the reference forward with the surrogate and a detached reset."""
    class Spike(torch.autograd.Function):
        @staticmethod
        def forward(ctx, u):
            ctx.save_for_backward(u)
            return (u >= 0).double()

        @staticmethod
        def backward(ctx, go):
            (u,) = ctx.saved_tensors
            return go * (alpha / 2.0) / (1.0 + (math.pi / 2.0 * alpha * u) ** 2)

    x = inp["input_current"].double().requires_grad_()
    m0 = inp["mem0"].double().requires_grad_()
    be = inp["beta"].double().requires_grad_()
    th = inp["threshold"].double().requires_grad_()
    bc = be.clamp(0, 1)
    mem = m0
    loss = 0.0
    for t in range(x.shape[0]):
        reset = (mem >= th).double().detach()
        mem = bc * mem + x[t] - reset * th
        loss = loss + (Spike.apply(mem - th) * gs[t].double()).sum()
    if gf is not None:
        loss = loss + (mem * gf.double()).sum()
    loss.backward()
    return {"grad_input": x.grad.numpy(), "grad_mem0": m0.grad.numpy(), "grad_beta": be.grad.numpy(),
            "grad_threshold": th.grad.numpy()}


@pytest.mark.parametrize("T,B,H,alpha,with_final", [(37, 3, 5, 2.0, True), (70, 2, 7, 4.0, False),
                                                    (1, 4, 3, 1.0, True)])
def test_oracle_matches_autograd(T, B, H, alpha, with_final):
    inp, gs, gf = make(T, B, H, seed=T * 7 + H)
    inp["beta"][0] = 1.2   # clamped: no gradient
    inp["beta"][-1] = -0.1
    gf = gf if with_final else None
    o = exact.leaky_backward(inp, gs, gf, alpha)
    r = autograd_reference(inp, gs, gf, alpha)
    for k in r:
        scale = np.abs(r[k]).max() + 1.0
        assert np.abs(o[k] - r[k]).max() <= 1e-5 * scale, k
    assert o["grad_beta"][0] == 0.0 and o["grad_beta"][-1] == 0.0


@pytest.mark.parametrize("cid,rec", golden_cases("leaky")[:3], ids=[c for c, _ in golden_cases("leaky")[:3]])
def test_oracle_forward_is_the_reference(cid, rec):
    s = inputs.task_inputs("leaky", rec["case"], int(rec["case"]["seed"]))
    T, B, H = s["input_current"].shape
    o = exact.leaky_backward(s, torch.zeros(T, B, H))
    ref = exact.leaky(s)
    assert np.array_equal(o["spikes"], ref["spikes"])
    assert np.array_equal(o["final_mem"], ref["final_mem"])
    assert not o["grad_input"].any()


# ---------------------------------------------------------------------------------------- GPU
@pytest.fixture(scope="module")
def ops():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    p = pkg()
    p.load()
    return p.ops


KEYS = ("input_current", "mem0", "beta", "threshold")


def check_backward(ops, inp, gs, gf, alpha, got=None):
    if got is None:
        dev = {k: inp[k].cuda() for k in KEYS}
        _, _, ckpt = ops.leaky_train(dev["input_current"], dev["mem0"], dev["beta"], dev["threshold"])
        got = ops.leaky_backward(dev["input_current"], ckpt, dev["beta"], dev["threshold"], gs.cuda(),
                                 None if gf is None else gf.cuda(), alpha)
    torch.cuda.synchronize()
    ref = exact.leaky_backward(inp, gs, gf, alpha)
    for k, v in zip(("grad_input", "grad_mem0"), got[:2]):
        bad, worst = exact.within(v.cpu().double().numpy(), ref[k], *TOL_X)
        assert bad == 0, (k, worst)
    for k, v in zip(("grad_beta", "grad_threshold"), got[2:]):
        err = np.abs(v.cpu().double().numpy() - ref[k])
        lim = TOL_SUM[0] + TOL_SUM[1] * ref[k + "_abs"]
        assert (err <= lim).all(), (k, float((err / lim).max()))
    return ref


@pytest.mark.gpu
@pytest.mark.parametrize("cid,rec", golden_cases("leaky"), ids=[c for c, _ in golden_cases("leaky")])
def test_golden_cases(ops, cid, rec):
    s = inputs.task_inputs("leaky", rec["case"], int(rec["case"]["seed"]))
    T, B, H = s["input_current"].shape
    g = torch.Generator().manual_seed(int(rec["case"]["seed"]))
    gs = torch.randn(T, B, H, generator=g)
    gf = torch.randn(B, H, generator=g)
    check_backward(ops, s, gs, gf, 2.0)


SHAPES = [(1, 1, 1), (31, 2, 6), (33, 3, 5), (64, 4, 128), (100, 3, 129), (257, 2, 1021)]


@pytest.mark.gpu
@pytest.mark.parametrize("T,B,H", SHAPES, ids=[f"T{t}_B{b}_H{h}" for t, b, h in SHAPES])
@pytest.mark.parametrize("alpha,with_final", [(2.0, True), (1.0, False), (4.0, True)])
def test_shapes(ops, T, B, H, alpha, with_final):
    inp, gs, gf = make(T, B, H, seed=T * 1000 + B * 10 + H)
    inp["beta"][0] = 1.3
    check_backward(ops, inp, gs, gf if with_final else None, alpha)


@pytest.mark.gpu
@pytest.mark.parametrize("T,B,H", [(33, 4, 130), (64, 3, 256), (200, 2, 2052)])
def test_alignment_does_not_matter(ops, T, B, H):
    """Views one float off a 16-byte boundary give bit-identical outputs."""
    inp, gs, gf = make(T, B, H, seed=T * 3 + H)
    dev = {k: inp[k].cuda() for k in KEYS}
    _, _, ckpt = ops.leaky_train(dev["input_current"], dev["mem0"], dev["beta"], dev["threshold"])

    def shifted(t):
        raw = torch.empty(t.numel() + 1, dtype=t.dtype, device="cuda")
        v = raw[1:].view(t.shape)
        v.copy_(t)
        return v
    aligned = ops.leaky_backward(dev["input_current"], ckpt, dev["beta"], dev["threshold"], gs.cuda(), gf.cuda(), 2.0)
    aligned = [t.clone() for t in aligned]
    off = ops.leaky_backward(shifted(dev["input_current"]), ckpt, dev["beta"], dev["threshold"], shifted(gs.cuda()),
                             gf.cuda(), 2.0)
    torch.cuda.synchronize()
    for a, b in zip(aligned, off):
        assert torch.equal(a.view(torch.int32), b.view(torch.int32))
    check_backward(ops, inp, gs, gf, 2.0, got=aligned)


@pytest.mark.gpu
@pytest.mark.parametrize("T,B,H", [(1, 1, 1), (33, 3, 5), (100, 4, 256), (64, 2, 1021)])
def test_train_forward_and_checkpoints(ops, T, B, H):
    inp, _, _ = make(T, B, H, seed=T + B + H)
    args = tuple(inp[k].cuda() for k in KEYS)
    sp, fm = ops.leaky(*args)
    sp2, fm2, ckpt = ops.leaky_train(*args)
    ckpt2 = ops.leaky_checkpoints(*args)
    torch.cuda.synchronize()
    assert torch.equal(sp, sp2) and torch.equal(fm.view(torch.int32), fm2.view(torch.int32))
    want = exact.leaky_backward(inp, torch.zeros(T, B, H))["checkpoints"]
    assert np.array_equal(ckpt.cpu().numpy().view(np.int32), want.view(np.int32))
    assert torch.equal(ckpt.view(torch.int32), ckpt2.view(torch.int32))


@pytest.mark.gpu
def test_baseline_size(ops):
    T, B, H = 256, 64, 4096
    g = torch.Generator().manual_seed(11)
    x = torch.randn(T, B, H, generator=g) * 0.5 + 0.3
    inp = {"input_current": x, "mem0": torch.zeros(B, H), "beta": torch.full((H,), 0.9),
           "threshold": torch.ones(H)}
    gs = torch.randn(T, B, H, generator=g)
    gf = torch.randn(B, H, generator=g)
    check_backward(ops, inp, gs, gf, 2.0)


@pytest.mark.gpu
def test_autograd_function(ops):
    inp, gs, gf = make(45, 3, 33, seed=3)
    dev = {k: inp[k].cuda().requires_grad_() for k in KEYS}
    spikes, final_mem = ops.LeakyFunction.apply(dev["input_current"], dev["mem0"], dev["beta"], dev["threshold"],
                                                2.0)
    ((spikes * gs.cuda()).sum() + (final_mem * gf.cuda()).sum()).backward()
    got = [dev[k].grad for k in ("input_current", "mem0", "beta", "threshold")]
    check_backward(ops, inp, gs, gf, 2.0, got=got)


@pytest.mark.gpu
def test_status_codes(ops):
    lib = pkg().load()
    x = torch.zeros(64, device="cuda")
    y = torch.zeros(64, device="cuda")
    p, q = x.data_ptr(), y.data_ptr()
    assert lib.b200_leaky_checkpoint_bytes(33, 2, 3) == 3 * 2 * 3 * 4  # one checkpoint per 16 steps
    assert lib.b200_leaky_checkpoint_bytes(-1, 2, 3) == -1
    assert lib.b200_leaky_backward_workspace_bytes(2, 3) == 2 * 2 * 3 * 4
    # workspace too small for the parameter gradients; none needed without them
    assert lib.b200_leaky_backward_async(p, p, p, p, 1, 2, 3, p, None, 2.0, p, p, p, p, p, 8, None) == 4
    assert lib.b200_leaky_backward_async(p, p, p, p, 1, 2, 3, p, None, 2.0, q, q, None, None, None, 0, None) == 0
    # missing checkpoints / grad_spikes, negative sizes
    assert lib.b200_leaky_backward_async(p, None, p, p, 1, 2, 3, p, None, 2.0, p, p, None, None, None, 0, None) == 1
    assert lib.b200_leaky_backward_async(p, p, p, p, 1, 2, 3, None, None, 2.0, p, p, None, None, None, 0, None) == 1
    assert lib.b200_leaky_backward_async(p, p, p, p, -1, 2, 3, p, None, 2.0, p, p, None, None, None, 0, None) == 1
    assert lib.b200_leaky_train_async(p, p, p, p, 2, 2, 3, p, p, None, None) == 1
    torch.cuda.synchronize()
