"""Generalised advantage estimation (GAE): the step between the returns and the PPO loss.

There is no GAE implementation in the reference repository, so the oracle (oracle.exact.gae, fp64)
restates the published algorithm; it is pinned to the reference where the two meet: with value =
next_value = 0, terminated = done and lambda = 1 the recursion is the reward-to-go, and the oracle
reproduces oracle.exact.reward_to_go (itself pinned to the reference's reference_exact) on the
reward_to_go golden cases.

GPU, through the C ABI: against the fp64 oracle at the reward-to-go tolerance (1e-5 / 1e-5) on
ragged shapes, done / terminated patterns, misaligned pointers and lambda in {0, 0.95, 1}; lambda
= 0 gives delta itself; the reward-to-go special case is bit-identical to b200_reward_to_go_async;
and the BASELINE.json configs[1] batch size.
"""
import numpy as np
import pytest
import torch

from conftest import golden_cases, pkg
from oracle import exact, inputs

TOL = (1e-5, 1e-5)  # the reward-to-go task tolerance (tasks/reward_to_go/tests/task.json)


def make(B, T, seed, p_done=0.05, p_term=0.03, offset=0, dev="cpu"):
    g = torch.Generator(device="cpu").manual_seed(seed)
    r = torch.randn(B, T, generator=g)
    v = torch.randn(B, T, generator=g) * 0.5
    nv = torch.cat([v[:, 1:], torch.randn(B, 1, generator=g) * 0.5], dim=1)
    done = torch.rand(B, T, generator=g) < p_done
    term = done & (torch.rand(B, T, generator=g) < (p_term / max(p_done, 1e-9)))
    out = {"reward": r, "value": v, "next_value": nv, "done": done, "terminated": term}
    if dev != "cpu":
        def put(t):
            raw = torch.empty(t.numel() + offset + 1, dtype=t.dtype, device=dev)
            w = raw[offset:offset + t.numel()].view(t.shape)
            w.copy_(t)
            return w
        out = {k: put(t) for k, t in out.items()}
    return out


@pytest.mark.parametrize("cid,rec", golden_cases("reward_to_go")[:4], ids=[c for c, _ in golden_cases("reward_to_go")[:4]])
def test_oracle_reduces_to_reward_to_go(cid, rec):
    s = inputs.task_inputs("reward_to_go", rec["case"], int(rec["case"]["seed"]))
    zero = torch.zeros_like(s["reward"])
    got = exact.gae({"reward": s["reward"], "value": zero, "next_value": zero, "done": s["done"],
                     "terminated": s["done"], "gamma": s["gamma"], "lmbda": 1.0})["advantage"]
    want = exact.reward_to_go(s)["output"]
    np.testing.assert_allclose(got, want, rtol=1e-12, atol=1e-12)


# ---------------------------------------------------------------------------------------- GPU
@pytest.fixture(scope="module")
def ops():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    p = pkg()
    p.load()
    return p.ops


SHAPES = [(1, 1, 0), (3, 1, 0), (7, 2111, 0), (64, 1000, 0), (5, 333, 1), (33, 4096, 2), (200, 17, 3)]


@pytest.mark.gpu
@pytest.mark.parametrize("B,T,offset", SHAPES, ids=[f"B{b}_T{t}_o{o}" for b, t, o in SHAPES])
@pytest.mark.parametrize("gamma,lmbda", [(0.99, 0.95), (0.9, 1.0), (0.99, 0.0)])
def test_against_oracle(ops, B, T, offset, gamma, lmbda):
    host = make(B, T, seed=B * 131 + T, offset=0)
    dev = make(B, T, seed=B * 131 + T, offset=offset, dev="cuda")
    adv, tgt = ops.gae(dev["reward"], dev["value"], dev["next_value"], dev["done"], dev["terminated"], gamma, lmbda)
    torch.cuda.synchronize()
    ref = exact.gae(dict(host, gamma=gamma, lmbda=lmbda))
    for got, want in ((adv, ref["advantage"]), (tgt, ref["value_target"])):
        bad, worst = exact.within(got.cpu().double().numpy(), want, *TOL)
        assert bad == 0, worst


@pytest.mark.gpu
def test_reward_to_go_special_case_bit_identical(ops):
    s = make(64, 1000, seed=5, dev="cuda")
    zero = torch.zeros_like(s["reward"])
    adv, _ = ops.gae(s["reward"], zero, zero, s["done"], s["done"], 0.97, 1.0)
    rtg = ops.reward_to_go(s["reward"], s["done"], 0.97)
    torch.cuda.synchronize()
    assert torch.equal(adv.view(torch.int32), rtg.view(torch.int32))


@pytest.mark.gpu
def test_baseline_size(ops):
    s = inputs.baseline_inputs("rl_pipeline", seed=0)
    B, T = s["B"], s["T"]
    g = torch.Generator(device="cpu").manual_seed(9)
    v = torch.randn(B, T, generator=g) * 0.5
    nv = torch.cat([v[:, 1:], torch.zeros(B, 1)], dim=1)
    host = {"reward": s["reward"], "value": v, "next_value": nv, "done": s["done"], "terminated": s["done"]}
    dev = {k: t.cuda() for k, t in host.items()}
    adv, tgt = ops.gae(dev["reward"], dev["value"], dev["next_value"], dev["done"], dev["terminated"], 0.99, 0.95)
    torch.cuda.synchronize()
    rows = np.random.default_rng(0).choice(B, size=64, replace=False)
    sub = {k: t[rows] for k, t in host.items()}
    ref = exact.gae(dict(sub, gamma=0.99, lmbda=0.95))
    for got, want in ((adv, ref["advantage"]), (tgt, ref["value_target"])):
        bad, worst = exact.within(got.cpu()[rows].double().numpy(), want, *TOL)
        assert bad == 0, worst


@pytest.mark.gpu
def test_status_codes(ops):
    lib = pkg().load()
    x = torch.zeros(16, device="cuda")
    p = x.data_ptr()
    assert lib.b200_gae_async(p, p, p, p, p, 0.9, 0.9, -1, 4, p, p, None) == 1
    assert lib.b200_gae_async(p, p, p, p, p, 0.9, 0.9, 2, 4, p, None, None) == 1
    assert lib.b200_gae_async(p, p, p, p, p, 0.9, 0.9, 0, 4, p, p, None) == 0
