"""PyTorch-tensor front end of the native ops (device memory and streams come from torch; the
work is done by libb200ops.so on the current CUDA stream).

`reference(task, inp)` mirrors the reference's per-task `reference(inp) -> dict`
(tasks/<task>/reference.py): the same input dict keys (the C argument names), the same output
names and shapes, so a caller of the reference's PyTorch entry can switch to this one unchanged.
Every function raises on a non-CUDA tensor, a wrong dtype or a non-contiguous input, and on a
non-zero native status; there is no CPU fallback.
"""
import ctypes

import torch

from . import _native

_WS = {}


def _lib():
    return _native.load()


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else ctypes.c_void_p(0)


def _opt_ptr(t, stand_in):
    """Pointer of an optional input stream: NULL when absent.  torch gives an empty tensor a NULL
    data pointer, which the C ABI would read as "absent"; a present but empty stream passes a
    valid stand-in address instead (never dereferenced: there are no elements)."""
    if t is None:
        return ctypes.c_void_p(0)
    return ctypes.c_void_p(t.data_ptr() or stand_in.data_ptr())


def _stream(device):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _need(t, name, dtype, device=None):
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name}: expected a torch.Tensor")
    if not t.is_cuda:
        raise ValueError(f"{name}: expected a CUDA tensor (no CPU path)")
    if t.dtype != dtype:
        raise ValueError(f"{name}: expected {dtype}, got {t.dtype}")
    if not t.is_contiguous():
        raise ValueError(f"{name}: expected a contiguous tensor")
    if device is not None and t.device != device:
        raise ValueError(f"{name}: on {t.device}, expected {device}")
    return t


def workspace(op, nbytes, device):
    """Zero-initialised scratch for `op` on `device` and the current stream, grown on demand.

    The reduction kernels leave their control words ready for the next call, so one buffer serves
    every later call issued on the same stream (never two streams at once)."""
    key = (op, device.index, torch.cuda.current_stream(device).cuda_stream)
    buf = _WS.get(key)
    if buf is None or buf.numel() < nbytes:
        buf = torch.zeros(max(int(nbytes), 4096), dtype=torch.uint8, device=device)
        _WS[key] = buf
    return buf


# ----------------------------------------------------------------------------------- robust-L1
def robust_l1(inp, target, out=None):
    """mean(sqrt((inp - target)^2 + 1e-6)) as a 0-d fp32 tensor."""
    _need(inp, "inp", torch.float32)
    _need(target, "target", torch.float32, inp.device)
    if inp.numel() != target.numel():
        raise ValueError("inp and target differ in size")
    n = inp.numel()
    out = torch.empty((), dtype=torch.float32, device=inp.device) if out is None else out
    lib = _lib()
    ws = workspace("robust_l1", lib.b200_robust_l1_workspace_bytes(n), inp.device)
    _native.check(lib.b200_robust_l1_async(_ptr(inp), _ptr(target), n, _ptr(out), _ptr(ws), ws.numel(),
                                           _stream(inp.device)), "robust_l1")
    return out


def robust_l1_partials(inp, target):
    """Chunk partials (fp64, one per b200_robust_l1_chunk_elems() elements) of one shard."""
    _need(inp, "inp", torch.float32)
    _need(target, "target", torch.float32, inp.device)
    lib = _lib()
    n = inp.numel()
    chunk = lib.b200_robust_l1_chunk_elems()
    parts = torch.empty((n + chunk - 1) // chunk, dtype=torch.float64, device=inp.device)
    _native.check(lib.b200_robust_l1_shard_partials(_ptr(inp), _ptr(target), n, _ptr(parts),
                                                    _stream(inp.device)), "robust_l1_partials")
    return parts


def robust_l1_finish(partials, n_total, out=None):
    _need(partials, "partials", torch.float64)
    out = torch.empty((), dtype=torch.float32, device=partials.device) if out is None else out
    _native.check(_lib().b200_robust_l1_finish(_ptr(partials), partials.numel(), int(n_total), _ptr(out),
                                               _stream(partials.device)), "robust_l1_finish")
    return out


# ----------------------------------------------------------------------------------------- PPO
def ppo_clip(cur, old, adv, clip_epsilon, entropy=None, out=None):
    """[loss, clip_fraction, approx_kl, ess, max_ratio, mean_ratio] (+ mean entropy)."""
    _need(cur, "current_log_prob", torch.float32)
    _need(old, "old_log_prob", torch.float32, cur.device)
    _need(adv, "advantage", torch.float32, cur.device)
    if entropy is not None:
        _need(entropy, "entropy", torch.float32, cur.device)
    n = cur.numel()
    if old.numel() != n or adv.numel() != n or (entropy is not None and entropy.numel() != n):
        raise ValueError("PPO inputs differ in size")
    k = 7 if entropy is not None else 6
    out = torch.empty(k, dtype=torch.float32, device=cur.device) if out is None else out
    lib = _lib()
    ws = workspace("ppo", lib.b200_ppo_workspace_bytes(n), cur.device)
    _native.check(lib.b200_ppo_async(_ptr(cur), _ptr(old), _ptr(adv), _opt_ptr(entropy, out), n,
                                     float(clip_epsilon), _ptr(out), _ptr(ws), ws.numel(), _stream(cur.device)),
                  "ppo_clip")
    return out


def ppo_partials(cur, old, adv, clip_epsilon, entropy=None):
    """Per-chunk partial records (uint8 rows of b200_ppo_partial_bytes()) of one shard."""
    lib = _lib()
    n = cur.numel()
    chunk = lib.b200_ppo_chunk_elems()
    rec = lib.b200_ppo_partial_bytes()
    parts = torch.empty(((n + chunk - 1) // chunk, rec), dtype=torch.uint8, device=cur.device)
    _native.check(lib.b200_ppo_shard_partials(_ptr(cur), _ptr(old), _ptr(adv), _opt_ptr(entropy, parts), n,
                                              float(clip_epsilon), _ptr(parts), _stream(cur.device)),
                  "ppo_partials")
    return parts


def ppo_finish(partials, n_total, with_entropy, out=None):
    k = 7 if with_entropy else 6
    out = torch.empty(k, dtype=torch.float32, device=partials.device) if out is None else out
    _native.check(_lib().b200_ppo_finish(_ptr(partials), partials.shape[0], int(n_total), int(bool(with_entropy)),
                                         _ptr(out), _stream(partials.device)), "ppo_finish")
    return out


# -------------------------------------------------------------------------------- reward-to-go
def reward_to_go(reward, done, gamma, out=None):
    _need(reward, "reward", torch.float32)
    _need(done, "done", torch.bool, reward.device)
    if reward.dim() != 2 or done.shape != reward.shape:
        raise ValueError("reward and done must both be (B, T)")
    B, T = reward.shape
    out = torch.empty_like(reward) if out is None else out
    _native.check(_lib().b200_reward_to_go_async(_ptr(reward), _ptr(done), float(gamma), B, T, _ptr(out),
                                                 _stream(reward.device)), "reward_to_go")
    return out


def pack_done(done, out=None):
    """Done flags bool [B, T] -> bits int32 [B, ceil(T/32)]: bit t % 32 of word [b, t // 32] is
    done[b, t], bits past T zero."""
    _need(done, "done", torch.bool)
    if done.dim() != 2:
        raise ValueError("done must be (B, T)")
    B, T = done.shape
    out = torch.empty((B, (T + 31) // 32), dtype=torch.int32, device=done.device) if out is None else out
    _native.check(_lib().b200_pack_done_async(_ptr(done), B, T, _ptr(out), _stream(done.device)), "pack_done")
    return out


def reward_to_go_bits(reward, done_bits, gamma, out=None):
    """reward_to_go with the done flags as bits (pack_done): the same output bits."""
    _need(reward, "reward", torch.float32)
    if reward.dim() != 2:
        raise ValueError("reward must be (B, T)")
    B, T = reward.shape
    _need(done_bits, "done_bits", torch.int32, reward.device)
    if done_bits.shape != (B, (T + 31) // 32):
        raise ValueError("done_bits must be (B, ceil(T/32))")
    out = torch.empty_like(reward) if out is None else out
    _native.check(_lib().b200_reward_to_go_bits_async(_ptr(reward), _ptr(done_bits), float(gamma), B, T, _ptr(out),
                                                      _stream(reward.device)), "reward_to_go_bits")
    return out


def _done_layout(reward, done):
    """(is_bits, T) for a done tensor: bool [B, T] or int32 bits [B, ceil(T/32)]."""
    B, T = reward.shape
    if done.dtype == torch.int32:
        _need(done, "done_bits", torch.int32, reward.device)
        if done.shape != (B, (T + 31) // 32):
            raise ValueError("done bits must be (B, ceil(T/32))")
        return 1
    _need(done, "done", torch.bool, reward.device)
    if done.shape != reward.shape:
        raise ValueError("reward and done must both be (B, T)")
    return 0


def reward_to_go_chunked(reward, done, gamma, out=None):
    """reward_to_go parallel along T (for few, long rows); done: bool [B, T] or pack_done bits."""
    _need(reward, "reward", torch.float32)
    if reward.dim() != 2:
        raise ValueError("reward must be (B, T)")
    bits = _done_layout(reward, done)
    B, T = reward.shape
    out = torch.empty_like(reward) if out is None else out
    lib = _lib()
    ws = workspace("rtg_chunked", lib.b200_reward_to_go_chunked_workspace_bytes(B, T), reward.device)
    _native.check(lib.b200_reward_to_go_chunked_async(_ptr(reward), _ptr(done), bits, float(gamma), B, T, _ptr(out),
                                                      _ptr(ws), ws.numel(), _stream(reward.device)),
                  "reward_to_go_chunked")
    return out


def reward_to_go_slice_maps(reward, done, gamma, maps_out=None):
    """First half of reward-to-go sharded over time: this rank's [B, 2] fp64 slice maps (a, b)."""
    _need(reward, "reward", torch.float32)
    bits = _done_layout(reward, done)
    B, T = reward.shape
    maps_out = torch.empty((B, 2), dtype=torch.float64, device=reward.device) if maps_out is None else maps_out
    lib = _lib()
    ws = workspace("rtg_slice", lib.b200_reward_to_go_chunked_workspace_bytes(B, T), reward.device)
    _native.check(lib.b200_reward_to_go_slice_maps_async(_ptr(reward), _ptr(done), bits, float(gamma), B, T,
                                                         _ptr(maps_out), _ptr(ws), ws.numel(),
                                                         _stream(reward.device)), "reward_to_go_slice_maps")
    return maps_out


def reward_to_go_slice_scan(reward, done, gamma, all_maps, rank, out=None):
    """Second half: this rank's outputs from every rank's slice maps all_maps [world, B, 2] (rank
    order).  Uses the workspace reward_to_go_slice_maps filled on this stream."""
    _need(reward, "reward", torch.float32)
    bits = _done_layout(reward, done)
    B, T = reward.shape
    _need(all_maps, "all_maps", torch.float64, reward.device)
    world = all_maps.shape[0]
    if all_maps.shape != (world, B, 2):
        raise ValueError("all_maps must be (world, B, 2)")
    out = torch.empty_like(reward) if out is None else out
    lib = _lib()
    ws = workspace("rtg_slice", lib.b200_reward_to_go_chunked_workspace_bytes(B, T), reward.device)
    _native.check(lib.b200_reward_to_go_slice_scan_async(_ptr(reward), _ptr(done), bits, float(gamma), B, T,
                                                         _ptr(all_maps), int(world), int(rank), _ptr(out), _ptr(ws),
                                                         ws.numel(), _stream(reward.device)),
                  "reward_to_go_slice_scan")
    return out


def reward_to_go_time_sharded(reward, done, gamma, group=None, out=None):
    """reward_to_go over rows whose steps are sharded across the ranks of `group` in rank order
    (this rank holds steps [offset, offset + T_local) of every row): slice maps, one all-gather of
    16 bytes per row per rank, then this rank's outputs."""
    import torch.distributed as dist
    maps = reward_to_go_slice_maps(reward, done, gamma)
    world = dist.get_world_size(group)
    all_maps = torch.empty((world * maps.shape[0], 2), dtype=maps.dtype, device=maps.device)  # rank-major
    dist.all_gather_into_tensor(all_maps, maps, group=group)
    return reward_to_go_slice_scan(reward, done, gamma, all_maps.view(world, -1, 2), dist.get_rank(group), out=out)


# ---------------------------------------------------------------------------- fused RL loss step
STEP_INPUTS_READY = 1  # B200_STEP_INPUTS_READY
STEP_DONE_BITS = 2     # B200_STEP_DONE_BITS


def _step_done_flags(reward, done, dev):
    """The step's done argument: bool [B, T], or bits int32 [B, ceil(T/32)] (flag STEP_DONE_BITS)."""
    if reward.dim() != 2:
        raise ValueError("reward must be (B, T)")
    B, T = reward.shape
    if isinstance(done, torch.Tensor) and done.dtype == torch.int32:
        _need(done, "done", torch.int32, dev)
        if done.shape != (B, (T + 31) // 32):
            raise ValueError("done bits must be (B, ceil(T/32))")
        return STEP_DONE_BITS
    _need(done, "done", torch.bool, dev)
    if done.shape != reward.shape:
        raise ValueError("reward and done must both be (B, T)")
    return 0


def rl_step(reward, done, gamma, cur, old, adv, clip_epsilon, entropy=None, rtg_out=None, ppo_out=None,
            inputs_ready=False):
    """reward_to_go and ppo_clip on independent inputs in one launch; the same bits as the two
    separate calls.  Returns (returns [B, T], PPO outputs [6] or [7]).

    inputs_ready=True declares that the kernel launched just before on the stream writes none of
    the inputs, so the step reads them while that kernel finishes (programmatic dependent launch).
    done: bool [B, T], or the flags as bits (pack_done)."""
    _need(reward, "reward", torch.float32)
    dev = reward.device
    flags = _step_done_flags(reward, done, dev)
    for t, nm in ((cur, "current_log_prob"), (old, "old_log_prob"), (adv, "advantage")):
        _need(t, nm, torch.float32, dev)
    if entropy is not None:
        _need(entropy, "entropy", torch.float32, dev)
    n = cur.numel()
    if old.numel() != n or adv.numel() != n or (entropy is not None and entropy.numel() != n):
        raise ValueError("PPO inputs differ in size")
    B, T = reward.shape
    rtg_out = torch.empty_like(reward) if rtg_out is None else rtg_out
    k = 7 if entropy is not None else 6
    ppo_out = torch.empty(k, dtype=torch.float32, device=dev) if ppo_out is None else ppo_out
    lib = _lib()
    ws = workspace("ppo", lib.b200_ppo_workspace_bytes(n), dev)
    _native.check(lib.b200_rl_step_ex_async(_ptr(reward), _ptr(done), float(gamma), B, T, _ptr(rtg_out), _ptr(cur),
                                            _ptr(old), _ptr(adv), _opt_ptr(entropy, ppo_out), n, float(clip_epsilon),
                                            _ptr(ppo_out), _ptr(ws), ws.numel(),
                                            flags | (STEP_INPUTS_READY if inputs_ready else 0), _stream(dev)),
                  "rl_step")
    return rtg_out, ppo_out


def rl_step_shard(reward, done, gamma, cur, old, adv, clip_epsilon, entropy=None, rtg_out=None, partials_out=None):
    """The fused step of one shard: returns and the PPO per-chunk partial records (as
    ppo_partials), for a cross-GPU gather and ppo_finish."""
    _need(reward, "reward", torch.float32)
    dev = reward.device
    _need(done, "done", torch.bool, dev)
    if reward.dim() != 2 or done.shape != reward.shape:
        raise ValueError("reward and done must both be (B, T)")
    for t, nm in ((cur, "current_log_prob"), (old, "old_log_prob"), (adv, "advantage")):
        _need(t, nm, torch.float32, dev)
    if entropy is not None:
        _need(entropy, "entropy", torch.float32, dev)
    n = cur.numel()
    if old.numel() != n or adv.numel() != n or (entropy is not None and entropy.numel() != n):
        raise ValueError("PPO inputs differ in size")
    lib = _lib()
    chunk = lib.b200_ppo_chunk_elems()
    shape = ((n + chunk - 1) // chunk, lib.b200_ppo_partial_bytes())
    if partials_out is None:
        partials_out = torch.empty(shape, dtype=torch.uint8, device=dev)
    elif tuple(partials_out.shape) != shape or partials_out.dtype != torch.uint8:
        raise ValueError(f"partials_out must be uint8 {shape}")
    B, T = reward.shape
    rtg_out = torch.empty_like(reward) if rtg_out is None else rtg_out
    _native.check(lib.b200_rl_step_shard_async(_ptr(reward), _ptr(done), float(gamma), B, T, _ptr(rtg_out),
                                               _ptr(cur), _ptr(old), _ptr(adv), _opt_ptr(entropy, rtg_out), n,
                                               float(clip_epsilon), _ptr(partials_out), _stream(dev)),
                  "rl_step_shard")
    return rtg_out, partials_out


# ------------------------------------------------------- multi-GPU RL step over NVLink peer memory
class PeerExchange:
    """The per-rank exchange buffer of the fused multi-GPU RL step (one process per GPU).

    `swap(handle) -> list of handles` must return every rank's 64-byte handle in rank order; with
    torch.distributed initialised, the default does that with all_gather_object."""

    def __init__(self, world, rank, n, swap=None, slots=None, record_bytes=None):
        """An exchange for the RL step over n samples per rank (the default), or, with `slots` and
        `record_bytes`, for another op's records (e.g. RobustL1Exchange)."""
        lib = _lib()
        self._ptr = ctypes.c_void_p()
        handle = (ctypes.c_char * lib.b200_peer_handle_bytes())()
        slots = 1 if slots is None else int(slots)
        rec = lib.b200_rl_step_exchange_record_bytes() if record_bytes is None else int(record_bytes)
        _native.check(lib.b200_peer_exchange_create(int(world), int(rank), slots, rec, ctypes.byref(self._ptr),
                                                    handle), "peer_exchange_create")
        if swap is None:
            import torch.distributed as dist

            def swap(h):
                out = [None] * world
                dist.all_gather_object(out, h)
                return out
        handles = swap(bytes(handle))
        if len(handles) != world:
            raise ValueError("swap() must return one handle per rank")
        blob = b"".join(handles)
        _native.check(lib.b200_peer_exchange_open(self._ptr, blob), "peer_exchange_open")
        self.world, self.rank, self.n, self.epoch = world, rank, int(n), 0

    @property
    def handle(self):
        return self._ptr

    def close(self):
        if self._ptr:
            _native.check(_lib().b200_peer_exchange_destroy(self._ptr), "peer_exchange_destroy")
            self._ptr = ctypes.c_void_p()


class RobustL1Exchange(PeerExchange):
    """The NVLink exchange of the multi-GPU robust-L1 mean over n_total elements (one process per
    GPU; every rank builds one with the same n_total, collectively)."""

    def __init__(self, world, rank, n_total, swap=None):
        lib = _lib()
        super().__init__(world, rank, n_total, swap=swap, slots=lib.b200_robust_l1_exchange_slots(int(n_total), world),
                         record_bytes=lib.b200_robust_l1_exchange_record_bytes())

    def shard_range(self):
        """[lo, hi) global element range this rank holds (whole chunks, as dist.shard_range)."""
        lib = _lib()
        chunk = lib.b200_robust_l1_chunk_elems()
        n_chunks = (self.n + chunk - 1) // chunk
        c0, c1 = (n_chunks * self.rank) // self.world, (n_chunks * (self.rank + 1)) // self.world
        return min(c0 * chunk, self.n), min(c1 * chunk, self.n)


def robust_l1_exchange(exchange, inp_shard, tgt_shard, out=None):
    """The robust-L1 mean over every rank's elements, from this rank's shard (its
    exchange.shard_range() elements); every rank gets the same bits, those of robust_l1 over the
    whole range on one GPU.  Every rank must call it the same number of times."""
    _need(inp_shard, "inp", torch.float32)
    _need(tgt_shard, "target", torch.float32, inp_shard.device)
    lo, hi = exchange.shard_range()
    if inp_shard.numel() != hi - lo or tgt_shard.numel() != hi - lo:
        raise ValueError(f"this rank holds elements [{lo}, {hi}); got {inp_shard.numel()}")
    dev = inp_shard.device
    out = torch.empty((), dtype=torch.float32, device=dev) if out is None else out
    lib = _lib()
    ws = workspace("robust_l1_exchange", 256, dev)
    exchange.epoch = lib.b200_peer_next_epoch(exchange.epoch)
    _native.check(lib.b200_robust_l1_exchange_async(_opt_ptr(inp_shard, out), _opt_ptr(tgt_shard, out), exchange.n,
                                                    _ptr(out), _ptr(ws), ws.numel(), exchange.handle, exchange.epoch,
                                                    _stream(dev)), "robust_l1_exchange")
    return out


def rl_step_exchange(exchange, reward, done, gamma, cur, old, adv, clip_epsilon, entropy=None, rtg_out=None,
                     ppo_out=None, inputs_ready=False):
    """One rank's fused multi-GPU RL step: this rank's returns, and the PPO outputs over every
    rank's samples (the same bits on every rank).  Every rank must call it the same number of
    times.  inputs_ready and done as for rl_step."""
    _need(reward, "reward", torch.float32)
    dev = reward.device
    flags = _step_done_flags(reward, done, dev)
    for t, nm in ((cur, "current_log_prob"), (old, "old_log_prob"), (adv, "advantage")):
        _need(t, nm, torch.float32, dev)
    if entropy is not None:
        _need(entropy, "entropy", torch.float32, dev)
    n = cur.numel()
    if n != exchange.n:
        raise ValueError("the exchange was created for a different sample count")
    B, T = reward.shape
    rtg_out = torch.empty_like(reward) if rtg_out is None else rtg_out
    k = 7 if entropy is not None else 6
    ppo_out = torch.empty(k, dtype=torch.float32, device=dev) if ppo_out is None else ppo_out
    lib = _lib()
    ws = workspace("ppo", lib.b200_ppo_workspace_bytes(n), dev)
    exchange.epoch = lib.b200_peer_next_epoch(exchange.epoch)
    _native.check(lib.b200_rl_step_exchange_async(_ptr(reward), _ptr(done), float(gamma), B, T, _ptr(rtg_out),
                                                  _ptr(cur), _ptr(old), _ptr(adv), _opt_ptr(entropy, ppo_out), n,
                                                  float(clip_epsilon), _ptr(ppo_out), _ptr(ws), ws.numel(),
                                                  exchange.handle, exchange.epoch,
                                                  flags | (STEP_INPUTS_READY if inputs_ready else 0), _stream(dev)),
                  "rl_step_exchange")
    return rtg_out, ppo_out


# ----------------------------------------------------------------------------------------- GAE
def gae(reward, value, next_value, done, terminated, gamma, lmbda, advantage=None, value_target=None):
    """Generalised advantage estimation over [B, T] rows: returns (advantage, value_target)."""
    _need(reward, "reward", torch.float32)
    dev = reward.device
    for t, nm in ((value, "value"), (next_value, "next_value")):
        _need(t, nm, torch.float32, dev)
    for t, nm in ((done, "done"), (terminated, "terminated")):
        _need(t, nm, torch.bool, dev)
    if reward.dim() != 2 or any(t.shape != reward.shape for t in (value, next_value, done, terminated)):
        raise ValueError("gae: all inputs must be (B, T)")
    B, T = reward.shape
    advantage = torch.empty_like(reward) if advantage is None else advantage
    value_target = torch.empty_like(reward) if value_target is None else value_target
    _native.check(_lib().b200_gae_async(_ptr(reward), _ptr(value), _ptr(next_value), _ptr(done), _ptr(terminated),
                                        float(gamma), float(lmbda), B, T, _ptr(advantage), _ptr(value_target),
                                        _stream(dev)), "gae")
    return advantage, value_target


# ----------------------------------------------------------------------------------------- LIF
def leaky_packed(input_current, mem0, beta, threshold, spike_bits=None, final_mem=None):
    """The LIF layer with bit-packed spikes: returns (spike_bits int32 [ceil(T/32), B, H], bit t % 32
    of word [t // 32] being the spike at step t; final_mem [B, H])."""
    _need(input_current, "input_current", torch.float32)
    dev = input_current.device
    for t, nm in ((mem0, "mem0"), (beta, "beta"), (threshold, "threshold")):
        _need(t, nm, torch.float32, dev)
    T, B, H = input_current.shape
    if spike_bits is None:
        spike_bits = torch.empty(((T + 31) // 32, B, H), dtype=torch.int32, device=dev)
    final_mem = torch.empty((B, H), dtype=torch.float32, device=dev) if final_mem is None else final_mem
    _native.check(_lib().b200_leaky_packed_async(_ptr(input_current), _ptr(mem0), _ptr(beta), _ptr(threshold), T, B,
                                                 H, _ptr(spike_bits), _ptr(final_mem), _stream(dev)), "leaky_packed")
    return spike_bits, final_mem


def leaky(input_current, mem0, beta, threshold, spikes=None, final_mem=None):
    _need(input_current, "input_current", torch.float32)
    dev = input_current.device
    for t, nm in ((mem0, "mem0"), (beta, "beta"), (threshold, "threshold")):
        _need(t, nm, torch.float32, dev)
    T, B, H = input_current.shape
    spikes = torch.empty_like(input_current) if spikes is None else spikes
    final_mem = torch.empty((B, H), dtype=torch.float32, device=dev) if final_mem is None else final_mem
    _native.check(_lib().b200_leaky_async(_ptr(input_current), _ptr(mem0), _ptr(beta), _ptr(threshold), T, B, H,
                                          _ptr(spikes), _ptr(final_mem), _stream(dev)), "leaky")
    return spikes, final_mem


def _leaky_args(input_current, mem0, beta, threshold):
    _need(input_current, "input_current", torch.float32)
    dev = input_current.device
    for t, nm in ((mem0, "mem0"), (beta, "beta"), (threshold, "threshold")):
        _need(t, nm, torch.float32, dev)
    T, B, H = input_current.shape
    return dev, T, B, H


def _checkpoint_buffer(T, B, H, dev):
    return torch.empty(((T + 15) // 16, B, H), dtype=torch.float32, device=dev)


def leaky_train(input_current, mem0, beta, threshold):
    """The LIF forward for training: (spikes, final_mem, checkpoints), spikes and final_mem as leaky();
    checkpoints [ceil(T/16), B, H] are the membrane state before every 16th step, what
    leaky_backward recomputes the trajectory from."""
    dev, T, B, H = _leaky_args(input_current, mem0, beta, threshold)
    spikes = torch.empty_like(input_current)
    final_mem = torch.empty((B, H), dtype=torch.float32, device=dev)
    ckpt = _checkpoint_buffer(T, B, H, dev)
    _native.check(_lib().b200_leaky_train_async(_ptr(input_current), _ptr(mem0), _ptr(beta), _ptr(threshold), T, B,
                                                H, _ptr(spikes), _ptr(final_mem), _ptr(ckpt), _stream(dev)),
                  "leaky_train")
    return spikes, final_mem, ckpt


def leaky_checkpoints(input_current, mem0, beta, threshold):
    """The membrane checkpoints alone, for a forward that ran through leaky()."""
    dev, T, B, H = _leaky_args(input_current, mem0, beta, threshold)
    ckpt = _checkpoint_buffer(T, B, H, dev)
    _native.check(_lib().b200_leaky_checkpoints_async(_ptr(input_current), _ptr(mem0), _ptr(beta), _ptr(threshold),
                                                      T, B, H, _ptr(ckpt), _stream(dev)), "leaky_checkpoints")
    return ckpt


def leaky_backward(input_current, checkpoints, beta, threshold, grad_spikes, grad_final_mem=None, alpha=2.0,
                   need_params=True):
    """Surrogate-gradient backward (arctangent surrogate, reset detached): returns (grad_input,
    grad_mem0, grad_beta, grad_threshold); the last two are None unless need_params."""
    _need(input_current, "input_current", torch.float32)
    dev = input_current.device
    T, B, H = input_current.shape
    for t, nm in ((checkpoints, "checkpoints"), (beta, "beta"), (threshold, "threshold"),
                  (grad_spikes, "grad_spikes")):
        _need(t, nm, torch.float32, dev)
    if grad_final_mem is not None:
        _need(grad_final_mem, "grad_final_mem", torch.float32, dev)
    if checkpoints.numel() != ((T + 15) // 16) * B * H or grad_spikes.shape != input_current.shape:
        raise ValueError("leaky_backward: inconsistent shapes")
    lib = _lib()
    gx = torch.empty_like(input_current)
    gm = torch.empty((B, H), dtype=torch.float32, device=dev)
    gb = torch.empty(H, dtype=torch.float32, device=dev) if need_params else None
    gt = torch.empty(H, dtype=torch.float32, device=dev) if need_params else None
    ws = workspace("leaky_backward", lib.b200_leaky_backward_workspace_bytes(B, H), dev) if need_params else None
    _native.check(lib.b200_leaky_backward_async(_ptr(input_current), _ptr(checkpoints), _ptr(beta), _ptr(threshold),
                                                T, B, H, _ptr(grad_spikes),
                                                None if grad_final_mem is None else _ptr(grad_final_mem),
                                                float(alpha), _ptr(gx), _ptr(gm), _ptr(gb), _ptr(gt),
                                                None if ws is None else _ptr(ws), 0 if ws is None else ws.numel(),
                                                _stream(dev)), "leaky_backward")
    return gx, gm, gb, gt


class LeakyFunction(torch.autograd.Function):
    """torch.autograd form of the layer: forward through leaky_train (keeps the 1/4-byte-per-step
    checkpoints, not the trajectory), backward through leaky_backward."""

    @staticmethod
    def forward(ctx, input_current, mem0, beta, threshold, alpha=2.0):
        spikes, final_mem, ckpt = leaky_train(input_current, mem0, beta, threshold)
        ctx.save_for_backward(input_current, ckpt, beta, threshold)
        ctx.alpha = float(alpha)
        return spikes, final_mem

    @staticmethod
    def backward(ctx, grad_spikes, grad_final_mem):
        x, ckpt, beta, threshold = ctx.saved_tensors
        if grad_spikes is None:
            grad_spikes = torch.zeros_like(x)
        gs = grad_spikes.contiguous()
        gf = None if grad_final_mem is None else grad_final_mem.contiguous()
        need = ctx.needs_input_grad[2] or ctx.needs_input_grad[3]
        gx, gm, gb, gt = leaky_backward(x, ckpt, beta, threshold, gs, gf, ctx.alpha, need_params=need)
        return gx, gm, gb, gt, None


# ----------------------------------------------------------------------------------------- KAN
def efficient_kan(x, grid, base_weight, spline_weight, spline_scaler, grid_size, spline_order, out=None):
    """KANLinear forward: out[B, O] = silu(x) base_weight^T + bases(x) (spline_weight * scaler)^T."""
    _need(x, "x", torch.float32)
    dev = x.device
    for t, nm in ((grid, "grid"), (base_weight, "base_weight"), (spline_weight, "spline_weight"),
                  (spline_scaler, "spline_scaler")):
        _need(t, nm, torch.float32, dev)
    B, I = x.shape
    O = base_weight.shape[0]
    G, K = int(grid_size), int(spline_order)
    if grid.shape != (I, G + 2 * K + 1) or base_weight.shape != (O, I) or spline_weight.shape != (O, I, G + K) \
            or spline_scaler.shape != (O, I):
        raise ValueError("efficient_kan: inconsistent shapes")
    out = torch.empty((B, O), dtype=torch.float32, device=dev) if out is None else out
    lib = _lib()
    ws = workspace("kan", lib.b200_efficient_kan_workspace_bytes(G, K, B, I, O), dev)
    _native.check(lib.b200_efficient_kan_async(_ptr(x), _ptr(grid), _ptr(base_weight), _ptr(spline_weight),
                                               _ptr(spline_scaler), G, K, B, I, O, _ptr(out), _ptr(ws),
                                               ws.numel(), _stream(dev)), "efficient_kan")
    return out


def efficient_kan_backward(x, grid, base_weight, spline_weight, spline_scaler, grid_size, spline_order, grad_out,
                           need_x=True, need_weights=True):
    """Gradients of efficient_kan for grad_out [B, O]: (grad_x, grad_base_weight, grad_spline_weight,
    grad_spline_scaler); the input gradient is None unless need_x, the weight gradients None
    unless need_weights."""
    _need(x, "x", torch.float32)
    dev = x.device
    for t, nm in ((grid, "grid"), (base_weight, "base_weight"), (spline_weight, "spline_weight"),
                  (spline_scaler, "spline_scaler"), (grad_out, "grad_out")):
        _need(t, nm, torch.float32, dev)
    B, I = x.shape
    O = base_weight.shape[0]
    G, K = int(grid_size), int(spline_order)
    if grid.shape != (I, G + 2 * K + 1) or base_weight.shape != (O, I) or spline_weight.shape != (O, I, G + K) \
            or spline_scaler.shape != (O, I) or grad_out.shape != (B, O):
        raise ValueError("efficient_kan_backward: inconsistent shapes")
    gx = torch.empty_like(x) if need_x else None
    gwb = torch.empty_like(base_weight) if need_weights else None
    gsw = torch.empty_like(spline_weight) if need_weights else None
    gsc = torch.empty_like(spline_scaler) if need_weights else None
    lib = _lib()
    ws = workspace("kan_backward", lib.b200_efficient_kan_backward_workspace_bytes(G, K, B, I, O), dev)
    _native.check(lib.b200_efficient_kan_backward_async(_ptr(x), _ptr(grid), _ptr(base_weight), _ptr(spline_weight),
                                                        _ptr(spline_scaler), G, K, B, I, O, _ptr(grad_out), _ptr(gx),
                                                        _ptr(gwb), _ptr(gsw), _ptr(gsc), _ptr(ws), ws.numel(),
                                                        _stream(dev)), "efficient_kan_backward")
    return gx, gwb, gsw, gsc


class KANLinearFunction(torch.autograd.Function):
    """torch.autograd form of the KAN layer: forward through efficient_kan, backward through
    efficient_kan_backward (the knot grid gets no gradient, as a KANLinear buffer)."""

    @staticmethod
    def forward(ctx, x, grid, base_weight, spline_weight, spline_scaler, grid_size, spline_order):
        ctx.save_for_backward(x, grid, base_weight, spline_weight, spline_scaler)
        ctx.gk = (int(grid_size), int(spline_order))
        return efficient_kan(x, grid, base_weight, spline_weight, spline_scaler, grid_size, spline_order)

    @staticmethod
    def backward(ctx, grad_out):
        x, grid, wb, sw, sc = ctx.saved_tensors
        need_x = ctx.needs_input_grad[0]
        need_w = any(ctx.needs_input_grad[2:5])
        gx, gwb, gsw, gsc = efficient_kan_backward(x, grid, wb, sw, sc, *ctx.gk, grad_out.contiguous(), need_x, need_w)
        return gx, None, gwb, gsw, gsc, None, None


# ---------------------------------------------------------------------------------- FP8 linear
def fp8_quantize(x, q=None, scale=None):
    """Per-tensor E4M3 quantisation of an fp32 or bf16 tensor (tasks/fp8_linear/reference.py:15-18):
    returns (q as float8_e4m3fn with x's shape, scale as a 1-element fp32 device tensor)."""
    if x.dtype not in (torch.float32, torch.bfloat16):
        raise TypeError("fp8_quantize: x must be float32 or bfloat16")
    _need(x, "x", x.dtype)
    dev = x.device
    q = torch.empty(x.shape, dtype=torch.float8_e4m3fn, device=dev) if q is None else q
    scale = torch.empty(1, dtype=torch.float32, device=dev) if scale is None else scale
    lib = _lib()
    ws = workspace("fp8q", lib.b200_fp8_quantize_workspace_bytes(), dev)
    _native.check(lib.b200_fp8_quantize_async(_ptr(x), 1 if x.dtype == torch.bfloat16 else 0, x.numel(), _ptr(q),
                                              _ptr(scale), _ptr(ws), ws.numel(), _stream(dev)), "fp8_quantize")
    return q, scale


def fp8_linear_bf16(x, w_fp8, scale_w, bias, out=None, scale_x=None):
    """The linear layer from a bf16 activation x [M, K]: quantise x on the device, then the E4M3
    GEMM; the same bits as fp8_quantize followed by fp8_linear with the computed scale."""
    _need(x, "x", torch.bfloat16)
    dev = x.device
    _need(w_fp8, "w_fp8", torch.float8_e4m3fn, dev)
    _need(bias, "bias", torch.bfloat16, dev)
    M, K = x.shape
    N = w_fp8.shape[0]
    if w_fp8.shape[1] != K or bias.numel() != N:
        raise ValueError("fp8_linear_bf16: inconsistent shapes")
    out = torch.empty((M, N), dtype=torch.bfloat16, device=dev) if out is None else out
    lib = _lib()
    ws = workspace("fp8lin", lib.b200_fp8_linear_bf16_workspace_bytes(M, K), dev)
    _native.check(lib.b200_fp8_linear_bf16_async(M, K, N, _ptr(x), _ptr(w_fp8), float(scale_w), _ptr(bias),
                                                 _ptr(out), _opt_ptr(scale_x, None), _ptr(ws), ws.numel(),
                                                 _stream(dev)), "fp8_linear_bf16")
    return out


def fp8_linear(x_fp8, scale_x, w_fp8, scale_w, bias, out=None):
    """bf16 (x_fp8 / scale_x) (w_fp8 / scale_w)^T + bias with E4M3 operands [M, K] and [N, K]."""
    _need(x_fp8, "x_fp8", torch.float8_e4m3fn)
    dev = x_fp8.device
    _need(w_fp8, "w_fp8", torch.float8_e4m3fn, dev)
    _need(bias, "bias", torch.bfloat16, dev)
    M, K = x_fp8.shape
    N = w_fp8.shape[0]
    if w_fp8.shape[1] != K or bias.numel() != N:
        raise ValueError("fp8_linear: inconsistent shapes")
    out = torch.empty((M, N), dtype=torch.bfloat16, device=dev) if out is None else out
    _native.check(_lib().b200_fp8_linear_async(M, K, N, _ptr(x_fp8), float(scale_x), _ptr(w_fp8), float(scale_w),
                                               _ptr(bias), _ptr(out), _stream(dev)), "fp8_linear")
    return out


# ------------------------------------------------------------------- reference-interface mirror
def reference(task, inp):
    """Drop-in for tasks/<task>/reference.py:reference(inp): same keys in, same keys out."""
    if task == "pow_abs_sqrt_mean":
        return {"output": robust_l1(inp["inp"], inp["target"])}
    if task == "ppo_clip":
        return {"output": ppo_clip(inp["current_log_prob"], inp["old_log_prob"], inp["advantage"],
                                   inp["clip_epsilon"], inp.get("entropy"))}
    if task == "reward_to_go":
        return {"output": reward_to_go(inp["reward"], inp["done"], inp["gamma"])}
    if task == "leaky":
        s, m = leaky(inp["input_current"], inp["mem0"], inp["beta"], inp["threshold"])
        return {"spikes": s, "final_mem": m}
    if task == "efficient_kan":
        return {"out": efficient_kan(inp["x"], inp["grid"], inp["base_weight"], inp["spline_weight"],
                                     inp["spline_scaler"], inp["grid_size"], inp["spline_order"])}
    if task == "fp8_linear":
        return {"output": fp8_linear(inp["x_fp8"], inp["scale_x"], inp["w_fp8"], inp["scale_w"], inp["bias"])}
    raise KeyError(f"unknown or not yet built task: {task}")
