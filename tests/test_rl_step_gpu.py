"""GPU: the fused RL loss step (reward-to-go and PPO in one launch, b200_rl_step_async) gives the
same bits as the two separate entry points, at the BASELINE.json configs[1] size and at ragged,
empty and misaligned shapes, with and without entropy; its shard form gives the same per-chunk
partials as b200_ppo_shard_partials.  Through that identity the fused step inherits the separate
ops' oracle parity (tests/test_stream_ops_gpu.py, tests/test_baseline_gpu.py), which is checked
again here at the full size.  Steps issued back to back with B200_STEP_INPUTS_READY (inputs read
while the previous step finishes) give the same bits, and so does the multi-GPU exchange step
run with one rank.
"""
import ctypes

import pytest
import torch

from conftest import pkg
from oracle import exact, inputs

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    p = pkg()
    p.load()
    return p.ops


def bits(t):
    return t.reshape(-1).contiguous().view(torch.uint8)


def make(B, T, n, seed, phase=0, entropy=True):
    """Reward-to-go inputs [B, T] and PPO inputs over n samples, each view `phase` floats (or
    bytes, for done) past a 256-byte boundary."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    dev = torch.device("cuda")

    def view(src, dtype=torch.float32):
        raw = torch.empty(src.numel() + phase + 1, dtype=dtype, device=dev)
        v = raw[phase:phase + src.numel()].view(src.shape)
        v.copy_(src)
        return v

    reward = view(torch.randn(B, T, generator=g))
    done = view(torch.rand(B, T, generator=g) < 0.02, torch.bool)
    cur = view(torch.randn(n, generator=g) * 0.1 - 1.0)
    old = view(cur.cpu() + torch.randn(n, generator=g) * 0.1)
    adv = view(torch.randn(n, generator=g))
    ent = view(torch.rand(n, generator=g) * 2.0) if entropy else None
    return reward, done, cur, old, adv, ent


SHAPES = [
    (4096, 1000, 4_096_000),   # configs[1]
    (1, 1, 1),
    (7, 2111, 12_345),
    (33, 64, 4096),
    (1000, 3, 4095),
    (0, 5, 100_000),           # no reward-to-go rows
    (5, 0, 1000),              # zero-length rows
    (12, 700, 0),              # no PPO samples
    (3, 9000, 2_000_003),      # long rows, ragged PPO tail
    (20_000, 17, 64),          # many short rows, tiny PPO
]


@pytest.mark.parametrize("B,T,n", SHAPES, ids=[f"B{b}_T{t}_n{n}" for b, t, n in SHAPES])
@pytest.mark.parametrize("entropy", [True, False], ids=["ent", "noent"])
def test_fused_matches_separate(ops, B, T, n, entropy):
    reward, done, cur, old, adv, ent = make(B, T, n, seed=B * 31 + T + n, entropy=entropy)
    rtg_sep = ops.reward_to_go(reward, done, 0.99)
    ppo_sep = ops.ppo_clip(cur, old, adv, 0.2, ent)
    rtg_f = torch.full_like(reward, float("nan"))
    ppo_f = torch.full_like(ppo_sep, float("nan"))
    for _ in range(2):  # twice: the completion counter is left ready for the next call
        ops.rl_step(reward, done, 0.99, cur, old, adv, 0.2, ent, rtg_out=rtg_f, ppo_out=ppo_f)
        torch.cuda.synchronize()
        assert torch.equal(bits(rtg_f), bits(rtg_sep))
        assert torch.equal(bits(ppo_f), bits(ppo_sep))


@pytest.mark.parametrize("phase", [1, 2, 3])
def test_fused_misaligned(ops, phase):
    """Unaligned PPO streams take the scalar path; the bits still match the separate ops."""
    reward, done, cur, old, adv, ent = make(61, 333, 100_001, seed=phase, phase=phase)
    rtg_f, ppo_f = ops.rl_step(reward, done, 0.95, cur, old, adv, 0.2, ent)
    assert torch.equal(bits(rtg_f), bits(ops.reward_to_go(reward, done, 0.95)))
    assert torch.equal(bits(ppo_f), bits(ops.ppo_clip(cur, old, adv, 0.2, ent)))


def test_fused_baseline_against_oracle(ops):
    """configs[1] inputs of the oracle's generator, checked against the fp64 oracle directly."""
    s = inputs.baseline_inputs("rl_pipeline", seed=0)
    g = {k: (v.cuda() if isinstance(v, torch.Tensor) else v) for k, v in s.items()}
    rtg, ppo = ops.rl_step(g["reward"], g["done"], g["gamma"], g["current_log_prob"], g["old_log_prob"],
                           g["advantage"], g["clip_epsilon"], g["entropy"])
    bad, worst = exact.within(rtg.cpu().double().numpy(), exact.reward_to_go(s)["output"], 1e-5, 1e-5)
    assert bad == 0, worst
    ref = exact.ppo_clip(s, entropy=s["entropy"])["output"]
    bad, worst = exact.within(ppo.cpu().double().numpy(), ref, 1e-5, 1e-4)
    assert bad == 0, worst


def test_fused_shard_form(ops):
    """The shard form's partials equal b200_ppo_shard_partials' and finish to the same bits."""
    lib = pkg().load()
    reward, done, cur, old, adv, ent = make(300, 500, 1_000_003, seed=5)
    n = cur.numel()
    want = ops.ppo_partials(cur, old, adv, 0.2, ent)
    got = torch.zeros_like(want)
    rtg = torch.empty_like(reward)
    st = lib.b200_rl_step_shard_async(reward.data_ptr(), done.data_ptr(), 0.9, 300, 500, rtg.data_ptr(),
                                      cur.data_ptr(), old.data_ptr(), adv.data_ptr(), ent.data_ptr(), n, 0.2,
                                      got.data_ptr(), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == 0
    torch.cuda.synchronize()
    assert torch.equal(got, want)
    assert torch.equal(bits(rtg), bits(ops.reward_to_go(reward, done, 0.9)))
    assert torch.equal(bits(ops.ppo_finish(got, n, True)), bits(ops.ppo_clip(cur, old, adv, 0.2, ent)))


def test_fused_status_codes(ops):
    lib = pkg().load()
    x = torch.zeros(64, device="cuda")
    out = torch.zeros(8, device="cuda")
    p = x.data_ptr()
    # negative sizes
    assert lib.b200_rl_step_async(p, p, 0.9, -1, 4, p, p, p, p, None, 16, 0.2, out.data_ptr(), p, 256, None) == 1
    assert lib.b200_rl_step_async(p, p, 0.9, 1, 4, p, p, p, p, None, -16, 0.2, out.data_ptr(), p, 256, None) == 1
    # workspace too small
    assert lib.b200_rl_step_async(p, p, 0.9, 1, 4, p, p, p, p, None, 16, 0.2, out.data_ptr(), p, 8, None) == 4
    # shard form without a partials buffer
    assert lib.b200_rl_step_shard_async(p, p, 0.9, 1, 4, p, p, p, p, None, 16, 0.2, None, None) == 1


def test_inputs_ready_back_to_back(ops):
    """Back-to-back steps over different resident batches, inputs declared ready: each step's
    outputs equal a step launched alone (the overlap with the previous step changes nothing)."""
    sets = [make(257, 900, 600_001, seed=40 + i) for i in range(3)]
    want = []
    for reward, done, cur, old, adv, ent in sets:
        r, p = ops.rl_step(reward, done, 0.97, cur, old, adv, 0.2, ent)
        torch.cuda.synchronize()
        want.append((r.clone(), p.clone()))
    outs = [(torch.full_like(sets[i][0], float("nan")), torch.full((7,), float("nan"), device="cuda"))
            for i in range(3)]
    for rep in range(4):
        for i, (reward, done, cur, old, adv, ent) in enumerate(sets):
            ops.rl_step(reward, done, 0.97, cur, old, adv, 0.2, ent, rtg_out=outs[i][0], ppo_out=outs[i][1],
                        inputs_ready=True)
    torch.cuda.synchronize()
    for (r, p), (wr, wp) in zip(outs, want):
        assert torch.equal(bits(r), bits(wr))
        assert torch.equal(bits(p), bits(wp))


def test_inputs_ready_after_producer(ops):
    """Without the declaration a step right after the kernel that writes its inputs reads them
    only after that kernel completes: the outputs follow the freshly written values."""
    reward, done, cur, old, adv, ent = make(64, 512, 300_000, seed=9)
    ref_r, ref_p = ops.rl_step(reward, done, 0.99, cur, old, adv, 0.2, ent)
    torch.cuda.synchronize()
    ref_r, ref_p = ref_r.clone(), ref_p.clone()
    saved_reward, saved_cur = reward.clone(), cur.clone()
    for _ in range(5):
        reward.zero_()  # producer kernels on the same stream, right before the step
        cur.zero_()
        reward.copy_(saved_reward)
        cur.copy_(saved_cur)
        r, p = ops.rl_step(reward, done, 0.99, cur, old, adv, 0.2, ent)
        torch.cuda.synchronize()
        assert torch.equal(bits(r), bits(ref_r))
        assert torch.equal(bits(p), bits(ref_p))


@pytest.mark.parametrize("entropy", [True, False], ids=["ent", "noent"])
def test_exchange_one_rank_matches_step(ops, entropy):
    """The multi-GPU exchange step with a world of one: the same bits as rl_step, over several
    epochs (alternating buffer halves), with and without the inputs-ready declaration."""
    ex = ops.PeerExchange(1, 0, 1_000_003, swap=lambda h: [h])
    try:
        for step in range(4):
            reward, done, cur, old, adv, ent = make(100, 777, 1_000_003, seed=70 + step, entropy=entropy)
            want_r, want_p = ops.rl_step(reward, done, 0.98, cur, old, adv, 0.2, ent)
            got_r, got_p = ops.rl_step_exchange(ex, reward, done, 0.98, cur, old, adv, 0.2, ent,
                                                inputs_ready=bool(step & 1))
            torch.cuda.synchronize()
            assert torch.equal(bits(got_r), bits(want_r))
            assert torch.equal(bits(got_p), bits(want_p))
        assert pkg().load().b200_device_fault() == 0
    finally:
        ex.close()


def test_step_flags_rejected(ops):
    lib = pkg().load()
    x = torch.zeros(64, device="cuda")
    out = torch.zeros(8, device="cuda")
    p = x.data_ptr()
    for flags in (4, 0x80000000):
        assert lib.b200_rl_step_ex_async(p, p, 0.9, 1, 4, p, p, p, p, None, 16, 0.2, out.data_ptr(), p, 4096, flags,
                                         None) == 1
