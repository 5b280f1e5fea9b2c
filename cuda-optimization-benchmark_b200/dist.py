"""Multi-GPU plumbing for the reductions (robust-L1, PPO): chunk-aligned shards, an all-gather of
per-chunk partials, and the same fixed-order finish on every rank.

The global element range is cut into fixed chunks (b200_*_chunk_elems()); rank r owns a contiguous
run of whole chunks (`shard_range`), computes one partial per local chunk on its GPU, and the ranks
all-gather the partials in rank order (`gather_rows`), which is the global chunk order.  Every rank
then runs the library's finish kernel over the same rows, so the result is bit-identical to the
single-GPU call for any number of ranks.  Works with NCCL (CUDA tensors) and gloo (CPU tensors).
"""
import torch
import torch.distributed as dist


def shard_range(n_total, chunk, world, rank):
    """[lo, hi) element range of `rank`: whole chunks, split as evenly as possible in chunk units."""
    n_chunks = (n_total + chunk - 1) // chunk
    c0 = (n_chunks * rank) // world
    c1 = (n_chunks * (rank + 1)) // world
    return min(c0 * chunk, n_total), min(c1 * chunk, n_total)


def shard_chunks(n_total, chunk, world):
    """Number of chunks each rank owns, in rank order."""
    out = []
    for r in range(world):
        lo, hi = shard_range(n_total, chunk, world, r)
        out.append((hi - lo + chunk - 1) // chunk)
    return out


def gather_rows(local, counts, group=None):
    """All-gather row blocks of different lengths (counts[r] rows from rank r) in rank order.

    Every rank pads its block to max(counts) rows, one all-gather moves the padded blocks, and the
    padding is dropped, so the result is the concatenation of the true blocks on every rank."""
    world = dist.get_world_size(group)
    rows = max(counts)
    pad = local.new_zeros((rows,) + tuple(local.shape[1:]))
    pad[: local.shape[0]] = local
    if local.is_cuda and dist.get_backend(group) == "nccl":
        out = local.new_empty((world * rows,) + tuple(local.shape[1:]))
        dist.all_gather_into_tensor(out, pad, group=group)
        blocks = [out[r * rows: r * rows + counts[r]] for r in range(world)]
    else:
        parts = [torch.empty_like(pad) for _ in range(world)]
        dist.all_gather(parts, pad, group=group)
        blocks = [parts[r][: counts[r]] for r in range(world)]
    return torch.cat(blocks, dim=0)


def robust_l1(ops, inp_shard, tgt_shard, n_total, group=None):
    """Global robust-L1 mean from this rank's chunk-aligned shard (CUDA tensors, NCCL group)."""
    lib = ops._lib()
    chunk = lib.b200_robust_l1_chunk_elems()
    world = dist.get_world_size(group)
    parts = ops.robust_l1_partials(inp_shard, tgt_shard)
    rows = gather_rows(parts, shard_chunks(n_total, chunk, world), group)
    return ops.robust_l1_finish(rows, n_total)


def ppo(ops, cur, old, adv, clip_epsilon, n_total, entropy=None, group=None):
    """Global PPO outputs from this rank's chunk-aligned shard of samples."""
    lib = ops._lib()
    chunk = lib.b200_ppo_chunk_elems()
    world = dist.get_world_size(group)
    parts = ops.ppo_partials(cur, old, adv, clip_epsilon, entropy)
    rows = gather_rows(parts, shard_chunks(n_total, chunk, world), group)
    return ops.ppo_finish(rows, n_total, entropy is not None)


def time_range(T, world, rank):
    """[t0, t1) steps of every row that `rank` holds when rows are sharded over time (contiguous,
    split as evenly as possible; every rank gets at least one step when T >= world)."""
    return (T * rank) // world, (T * (rank + 1)) // world
