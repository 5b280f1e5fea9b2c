"""Done flags as bits: b200_pack_done_async, b200_reward_to_go_bits_async and the fused step with
B200_STEP_DONE_BITS (no reference counterpart: the reference ABI fixes one bool per step).

CPU: the packing oracle (oracle.exact.pack_done_bits) on a hand-written known answer.

GPU, through the C ABI:
- the pack kernel equals the oracle's words on ragged shapes (T below, at and past multiples of
  32 and of the scan's 1056-step pass) with done at byte offsets 0..3;
- reward-to-go from bits is bit-identical to reward-to-go from bytes on the same shapes, on the
  reward_to_go golden cases and at the BASELINE.json configs[1] size (so it inherits that entry's
  oracle parity);
- the fused step and the one-rank exchange step with bits are bit-identical to the same steps with
  bytes, with and without entropy and the inputs-ready declaration.
"""
import numpy as np
import pytest
import torch

from conftest import golden_cases, pkg
from oracle import exact, inputs


def test_pack_oracle_known_answer():
    d = np.zeros((2, 40), dtype=bool)
    d[0, 0] = d[0, 31] = d[0, 32] = True
    d[1, 39] = True
    assert exact.pack_done_bits(d).tolist() == [[0x80000001, 0x1], [0x0, 0x80]]
    assert exact.pack_done_bits(np.ones((1, 33), dtype=bool)).tolist() == [[0xFFFFFFFF, 0x1]]


# ---------------------------------------------------------------------------------------- GPU
@pytest.fixture(scope="module")
def ops():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    p = pkg()
    p.load()
    return p.ops


SHAPES = [(1, 1), (3, 31), (3, 32), (3, 33), (5, 1056), (2, 1057), (7, 2111), (64, 1000), (9, 3200), (40, 5)]


def make(B, T, seed, offset=0, p=0.05):
    g = torch.Generator().manual_seed(seed)
    reward = torch.randn(B, T, generator=g)
    done = torch.rand(B, T, generator=g) < p
    raw = torch.zeros(B * T + offset + 1, dtype=torch.bool, device="cuda")
    d = raw[offset:offset + B * T].view(B, T)
    d.copy_(done)
    return reward.cuda(), d, done


@pytest.mark.gpu
@pytest.mark.parametrize("B,T", SHAPES, ids=[f"B{b}_T{t}" for b, t in SHAPES])
@pytest.mark.parametrize("offset", [0, 1, 3])
def test_pack_matches_oracle(ops, B, T, offset):
    _, d, host = make(B, T, seed=B * 100 + T, offset=offset, p=0.3)
    words = ops.pack_done(d)
    torch.cuda.synchronize()
    assert np.array_equal(words.cpu().numpy().view(np.uint32), exact.pack_done_bits(host))


@pytest.mark.gpu
@pytest.mark.parametrize("B,T", SHAPES, ids=[f"B{b}_T{t}" for b, t in SHAPES])
@pytest.mark.parametrize("gamma", [0.99, 0.5])
def test_rtg_bits_match_bytes(ops, B, T, gamma):
    reward, d, _ = make(B, T, seed=B + T * 7)
    want = ops.reward_to_go(reward, d, gamma)
    got = ops.reward_to_go_bits(reward, ops.pack_done(d), gamma)
    torch.cuda.synchronize()
    assert torch.equal(got.view(torch.int32), want.view(torch.int32))


@pytest.mark.gpu
@pytest.mark.parametrize("cid,rec", golden_cases("reward_to_go"), ids=[c for c, _ in golden_cases("reward_to_go")])
def test_rtg_bits_golden(ops, cid, rec):
    s = inputs.task_inputs("reward_to_go", rec["case"], int(rec["case"]["seed"]))
    r, d = s["reward"].cuda(), s["done"].cuda()
    got = ops.reward_to_go_bits(r, ops.pack_done(d), s["gamma"])
    torch.cuda.synchronize()
    ref = exact.reward_to_go(s)["output"]
    bad, worst = exact.within(got.cpu().double().numpy(), ref, *exact.TOLERANCE["reward_to_go"])
    assert bad == 0, worst
    assert torch.equal(got.view(torch.int32), ops.reward_to_go(r, d, s["gamma"]).view(torch.int32))


@pytest.mark.gpu
def test_rtg_bits_baseline(ops):
    s = inputs.baseline_inputs("rl_pipeline", seed=0)
    r, d = s["reward"].cuda(), s["done"].cuda()
    got = ops.reward_to_go_bits(r, ops.pack_done(d), s["gamma"])
    want = ops.reward_to_go(r, d, s["gamma"])
    torch.cuda.synchronize()
    assert torch.equal(got.view(torch.int32), want.view(torch.int32))


STEP_SHAPES = [(4096, 1000, 4_096_000), (7, 2111, 12_345), (1000, 3, 4095), (3, 9000, 100_003), (12, 700, 0)]


@pytest.mark.gpu
@pytest.mark.parametrize("B,T,n", STEP_SHAPES, ids=[f"B{b}_T{t}_n{n}" for b, t, n in STEP_SHAPES])
@pytest.mark.parametrize("entropy", [True, False], ids=["ent", "noent"])
def test_step_bits_match_bytes(ops, B, T, n, entropy):
    g = torch.Generator().manual_seed(B + T + n)
    reward = torch.randn(B, T, generator=g).cuda()
    done = (torch.rand(B, T, generator=g) < 0.02).cuda()
    cur = (torch.randn(n, generator=g) * 0.1 - 1.0).cuda()
    old = cur + (torch.randn(n, generator=g) * 0.1).cuda()
    adv = torch.randn(n, generator=g).cuda()
    ent = (torch.rand(n, generator=g) * 2.0).cuda() if entropy else None
    words = ops.pack_done(done)
    want_r, want_p = ops.rl_step(reward, done, 0.99, cur, old, adv, 0.2, ent)
    want_r, want_p = want_r.clone(), want_p.clone()
    for ready in (False, True):
        got_r, got_p = ops.rl_step(reward, words, 0.99, cur, old, adv, 0.2, ent, inputs_ready=ready)
        torch.cuda.synchronize()
        assert torch.equal(got_r.view(torch.int32), want_r.view(torch.int32))
        assert torch.equal(got_p.view(torch.int32), want_p.view(torch.int32))


@pytest.mark.gpu
def test_exchange_one_rank_bits(ops):
    ex = ops.PeerExchange(1, 0, 500_001, swap=lambda h: [h])
    try:
        for step in range(3):
            g = torch.Generator().manual_seed(step)
            reward = torch.randn(50, 1500, generator=g).cuda()
            done = (torch.rand(50, 1500, generator=g) < 0.01).cuda()
            cur = (torch.randn(500_001, generator=g) * 0.1 - 1.0).cuda()
            old = cur + 0.05
            adv = torch.randn(500_001, generator=g).cuda()
            want_r, want_p = ops.rl_step(reward, done, 0.97, cur, old, adv, 0.2, None)
            want_r, want_p = want_r.clone(), want_p.clone()
            got_r, got_p = ops.rl_step_exchange(ex, reward, ops.pack_done(done), 0.97, cur, old, adv, 0.2, None)
            torch.cuda.synchronize()
            assert torch.equal(got_r.view(torch.int32), want_r.view(torch.int32))
            assert torch.equal(got_p.view(torch.int32), want_p.view(torch.int32))
        assert pkg().load().b200_device_fault() == 0
    finally:
        ex.close()


@pytest.mark.gpu
def test_status_codes(ops):
    lib = pkg().load()
    x = torch.zeros(16, device="cuda")
    p = x.data_ptr()
    assert lib.b200_pack_done_async(p, -1, 4, p, None) == 1
    assert lib.b200_pack_done_async(None, 2, 4, p, None) == 1
    assert lib.b200_pack_done_async(p, 0, 4, p, None) == 0
    assert lib.b200_reward_to_go_bits_async(p, None, 0.9, 2, 4, p, None) == 1
    assert lib.b200_reward_to_go_bits_async(p, p, 0.9, 2, -4, p, None) == 1
