"""ctypes binding of libb200ops.so (declarations: include/b200ops.h).

There is no fallback: if the library is missing or fails to load, every op raises
`NativeLibraryError`.  The library is never rebuilt implicitly at import time; run
`__graft_entry__.build()` (or `python -m` on `_build.py`) first.
"""
import ctypes
from pathlib import Path

from . import _build

c_f = ctypes.c_float
c_i32 = ctypes.c_int32
c_i64 = ctypes.c_int64
c_sz = ctypes.c_size_t
c_int = ctypes.c_int
c_p = ctypes.c_void_p
c_str = ctypes.c_char_p

# name -> (restype, argtypes); one entry per function of include/b200ops.h.
SIGNATURES = {
    "b200_status_string": (c_str, [c_int]),
    "b200_last_status": (c_int, []),
    "b200_device_fault": (c_int, []),
    # robust-L1
    "b200_pow_abs_sqrt_mean": (None, [c_p, c_p, c_i64, c_i64, c_i64, c_p]),
    "b200_robust_l1_workspace_bytes": (c_sz, [c_i64]),
    "b200_robust_l1_async": (c_int, [c_p, c_p, c_i64, c_p, c_p, c_sz, c_p]),
    "b200_pow_abs_sqrt_mean_noalloc": (c_int, [c_p, c_p, c_i64, c_i64, c_i64, c_p, c_p]),
    "b200_robust_l1_chunk_elems": (c_i64, []),
    "b200_robust_l1_shard_partials": (c_int, [c_p, c_p, c_i64, c_p, c_p]),
    "b200_robust_l1_finish": (c_int, [c_p, c_i64, c_i64, c_p, c_p]),
    # PPO
    "b200_ppo_clip": (None, [c_i32, c_i32, c_i32, c_p, c_p, c_p, c_f, c_p]),
    "b200_ppo_clip_ext": (None, [c_i32, c_i32, c_i32, c_p, c_p, c_p, c_p, c_f, c_p]),
    "b200_ppo_workspace_bytes": (c_sz, [c_i64]),
    "b200_ppo_async": (c_int, [c_p, c_p, c_p, c_p, c_i64, c_f, c_p, c_p, c_sz, c_p]),
    "b200_ppo_chunk_elems": (c_i64, []),
    "b200_ppo_partial_bytes": (c_sz, []),
    "b200_ppo_shard_partials": (c_int, [c_p, c_p, c_p, c_p, c_i64, c_f, c_p, c_p]),
    "b200_ppo_finish": (c_int, [c_p, c_i64, c_i64, c_int, c_p, c_p]),
    # reward-to-go
    "b200_reward_to_go": (None, [c_p, c_p, c_f, c_i32, c_i32, c_p]),
    "b200_reward_to_go_async": (c_int, [c_p, c_p, c_f, c_i32, c_i32, c_p, c_p]),
    "b200_pack_done_async": (c_int, [c_p, c_i32, c_i32, c_p, c_p]),
    "b200_reward_to_go_bits_async": (c_int, [c_p, c_p, c_f, c_i32, c_i32, c_p, c_p]),
    "b200_reward_to_go_chunked_workspace_bytes": (c_i64, [c_i32, c_i32]),
    "b200_reward_to_go_chunked_async": (c_int, [c_p, c_p, c_int, c_f, c_i32, c_i32, c_p, c_p, c_i64, c_p]),
    "b200_reward_to_go_slice_maps_async": (c_int, [c_p, c_p, c_int, c_f, c_i32, c_i32, c_p, c_p, c_i64, c_p]),
    "b200_reward_to_go_slice_scan_async": (c_int, [c_p, c_p, c_int, c_f, c_i32, c_i32, c_p, c_int, c_int, c_p, c_p,
                                                   c_i64, c_p]),
    # fused RL step (reward-to-go + PPO in one launch)
    "b200_rl_step_async": (c_int, [c_p, c_p, c_f, c_i32, c_i32, c_p, c_p, c_p, c_p, c_p, c_i64, c_f, c_p, c_p, c_sz,
                                   c_p]),
    "b200_rl_step_ex_async": (c_int, [c_p, c_p, c_f, c_i32, c_i32, c_p, c_p, c_p, c_p, c_p, c_i64, c_f, c_p, c_p, c_sz,
                                      ctypes.c_uint, c_p]),
    "b200_rl_step_shard_async": (c_int, [c_p, c_p, c_f, c_i32, c_i32, c_p, c_p, c_p, c_p, c_p, c_i64, c_f, c_p,
                                         c_p]),
    # multi-GPU peer exchange
    "b200_peer_handle_bytes": (c_sz, []),
    "b200_rl_step_exchange_record_bytes": (c_sz, []),
    "b200_peer_next_epoch": (ctypes.c_uint, [ctypes.c_uint]),
    "b200_peer_exchange_create": (c_int, [c_int, c_int, c_i64, c_sz, c_p, c_p]),
    "b200_peer_exchange_open": (c_int, [c_p, c_p]),
    "b200_peer_exchange_destroy": (c_int, [c_p]),
    "b200_robust_l1_exchange_record_bytes": (c_sz, []),
    "b200_robust_l1_exchange_slots": (c_i64, [c_i64, c_int]),
    "b200_robust_l1_exchange_async": (c_int, [c_p, c_p, c_i64, c_p, c_p, c_sz, c_p, ctypes.c_uint, c_p]),
    "b200_rl_step_exchange_async": (c_int, [c_p, c_p, c_f, c_i32, c_i32, c_p, c_p, c_p, c_p, c_p, c_i64, c_f, c_p, c_p,
                                            c_sz, c_p, ctypes.c_uint, ctypes.c_uint, c_p]),
    # GAE
    "b200_gae_async": (c_int, [c_p, c_p, c_p, c_p, c_p, c_f, c_f, c_i32, c_i32, c_p, c_p, c_p]),
    # LIF
    "b200_leaky": (None, [c_p, c_p, c_p, c_p, c_i32, c_i32, c_i32, c_p, c_p]),
    "b200_leaky_async": (c_int, [c_p, c_p, c_p, c_p, c_i32, c_i32, c_i32, c_p, c_p, c_p]),
    "b200_leaky_packed_async": (c_int, [c_p, c_p, c_p, c_p, c_i32, c_i32, c_i32, c_p, c_p, c_p]),
    "b200_leaky_checkpoint_bytes": (c_i64, [c_i32, c_i32, c_i32]),
    "b200_leaky_train_async": (c_int, [c_p, c_p, c_p, c_p, c_i32, c_i32, c_i32, c_p, c_p, c_p, c_p]),
    "b200_leaky_checkpoints_async": (c_int, [c_p, c_p, c_p, c_p, c_i32, c_i32, c_i32, c_p, c_p]),
    "b200_leaky_backward_workspace_bytes": (c_i64, [c_i32, c_i32]),
    "b200_leaky_backward_async": (c_int, [c_p, c_p, c_p, c_p, c_i32, c_i32, c_i32, c_p, c_p, c_f, c_p, c_p, c_p,
                                          c_p, c_p, c_i64, c_p]),
    # KAN
    "b200_efficient_kan": (None, [c_p, c_p, c_p, c_p, c_p, c_i32, c_i32, c_i32, c_i32, c_i32, c_p]),
    "b200_efficient_kan_workspace_bytes": (c_sz, [c_i32, c_i32, c_i32, c_i32, c_i32]),
    "b200_efficient_kan_async": (c_int, [c_p, c_p, c_p, c_p, c_p, c_i32, c_i32, c_i32, c_i32, c_i32, c_p, c_p, c_sz,
                                         c_p]),
    "b200_efficient_kan_backward_workspace_bytes": (c_sz, [c_i32, c_i32, c_i32, c_i32, c_i32]),
    "b200_efficient_kan_backward_async": (c_int, [c_p, c_p, c_p, c_p, c_p, c_i32, c_i32, c_i32, c_i32, c_i32, c_p, c_p,
                                                  c_p, c_p, c_p, c_p, c_sz, c_p]),
    # FP8 linear
    "b200_fp8_linear": (None, [c_i32, c_i32, c_i32, c_p, c_f, c_p, c_f, c_p, c_p]),
    "b200_fp8_linear_async": (c_int, [c_i32, c_i32, c_i32, c_p, c_f, c_p, c_f, c_p, c_p, c_p]),
    "b200_fp8_linear_cuda_core_async": (c_int, [c_i32, c_i32, c_i32, c_p, c_f, c_p, c_f, c_p, c_p, c_p]),
    "b200_fp8_linear_plan": (c_int, [c_i32, c_i32, c_i32, c_p, c_p]),
    "b200_fp8_quantize_workspace_bytes": (c_sz, []),
    "b200_fp8_quantize_async": (c_int, [c_p, c_i32, c_i64, c_p, c_p, c_p, c_sz, c_p]),
    "b200_fp8_linear_bf16_workspace_bytes": (c_sz, [c_i32, c_i32]),
    "b200_fp8_linear_bf16_async": (c_int, [c_i32, c_i32, c_i32, c_p, c_p, c_f, c_p, c_p, c_p, c_p, c_sz, c_p]),
}


class NativeLibraryError(RuntimeError):
    pass


class OpError(RuntimeError):
    """A native entry point returned a non-zero status."""


_LIB = None


def library_path():
    return Path(_build.LIB)


def load():
    """Load libb200ops.so once and bind every entry point's signature."""
    global _LIB
    if _LIB is not None:
        return _LIB
    path = library_path()
    if not path.exists():
        raise NativeLibraryError(f"{path} is not built; run __graft_entry__.build() (needs nvcc) first")
    try:
        lib = ctypes.CDLL(str(path))
    except OSError as e:
        raise NativeLibraryError(f"cannot load {path}: {e}") from e
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _LIB = lib
    return lib


def check(status, what):
    if status != 0:
        msg = load().b200_status_string(status).decode()
        raise OpError(f"{what}: status {status} ({msg})")
