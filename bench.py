"""Benchmark of the B200 kernels on the BASELINE.json workloads; prints one JSON line (rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

Headline workload ("RL loss pipeline"): per GPU a batch of
B=4096 trajectories x T=1000 steps; one step = discounted reward-to-go over the batch plus the
PPO clipped loss with its diagnostics and the mean entropy over the same 4,096,000 samples, both
in one launch of the fused kernel (b200_rl_step_async).  `value` is samples (trajectory steps)
per second over all GPUs, inputs resident in HBM; the per-op microseconds and roofline fractions
that BASELINE.json's metric names are reported beside it (the two ops also timed as separate
launches).  With N > 1 each rank processes its own batch (weak scaling) and the PPO reduction is
global: each rank's step kernel stores its PPO totals into every peer's buffer over NVLink (CUDA
IPC peer memory) and adds all ranks' totals in rank order, so every rank writes the same outputs;
where CUDA IPC cannot be set up, the shard kernel's chunk partials are all-gathered with NCCL and
finished on every rank instead.  After the timed steps the N > 1 results are checked on the same
box (`parity`: bitwise across ranks, against the finish over the gathered partials, returns
against the one-op entry); a failed check exits non-zero.  `exchange_us` is the step with no
samples (the exchange alone at N > 1, the step's fixed cost at N = 1).

`ops_sharded`: robust-L1, LIF, KAN and FP8 at their BASELINE sizes split over the N ranks (strong
scaling: element ranges whose chunk partials are exchanged, by an NCCL all-gather in a CUDA graph
or by the kernel's own pushes over NVLink, the faster form reported and both listed; batch rows;
batch rows; rows of M with W replicated), each checked against the same op run whole on one GPU.

Timing: W untimed warm-up steps, then exactly K steps between barriers and device syncs, timed
with CUDA events on the launching stream, max over ranks.  Each step reads a different one of
four input sets (4 x 102 MB, larger than the 126 MB L2), so every step streams from HBM.
`e2e` repeats the step through the same entry points with the inputs in pinned host memory:
host-to-device copies of that step's inputs and a device-to-host read of its results are inside
the timed region.  `--impl reference` times the CPU restatement of the reference's PyTorch-eager
implementation of the same step on all host cores (rank 0 only).
"""
import argparse
import importlib
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import torch

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

METRIC = "per-op µs and % of HBM or FP8-tensor roofline, 1–8 B200, vs CPU eager"
B, T = 4096, 1000
N_SAMPLES = B * T
ROTATE = 4
READY = 1  # B200_STEP_INPUTS_READY (include/b200ops.h)
REPEAT_BATCHES = 10  # extra timed batches of K steps after the headline region (run-to-run spread)
# Algorithmic bytes per call (reads + writes of each op's inputs and outputs).
RTG_BYTES = (4 + 1 + 4) * N_SAMPLES                 # reward f32 + done u8 -> output f32
PPO_BYTES = 16 * N_SAMPLES + 7 * 4                  # cur, old, adv, entropy f32 -> 7 f32
ROBUST_L1_BYTES = 2 * 4 * (1 << 26) + 4
LIF_BYTES = 4 * 2 * (256 * 64 * 4096) + 4 * 2 * (64 * 4096) + 4 * 2 * 4096


def peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def bf16_tflops(sustained=False):
    """Measured dense bf16 TFLOP/s of this pool's B200s (cuBLAS; burst, or sustained under the
    power cap for seconds-long loops), else the fallback figures."""
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["bf16_tflops_sustained" if sustained else "bf16_tflops"])
    return 1400.0 if sustained else 1590.0


# ------------------------------------------------------------------------------ distributed set-up
def dist_setup(n_gpus):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        # NCCL writes a version banner to file descriptor 1 when its communicator is created; this
        # run's stdout carries exactly one JSON line, so fd 1 points at stderr until then.
        sys.stdout.flush()
        saved = os.dup(1)
        os.dup2(2, 1)
        try:
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                    device_id=torch.device("cuda", local))
            dist.barrier()
            torch.cuda.synchronize()
        finally:
            os.dup2(saved, 1)
            os.close(saved)
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(x, world):
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ------------------------------------------------------------------------------------ clocks
class ClockSampler:
    """nvidia-smi samples (every 100 ms) of the SM clock and throttle reasons, collected by a
    reader thread from start to stop."""

    QUERY = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")

    def __init__(self, device):
        import threading
        self.proc = None
        self.lines = []
        ident = str(device)
        try:
            u = torch.cuda.get_device_properties(device).uuid
            ident = "GPU-" + str(u)
        except Exception:
            pass
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                                          "-lms", "100", "-i", ident], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
            return
        self.reader = threading.Thread(target=self._read, daemon=True)
        self.reader.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line)

    def wait_first(self, timeout=5.0):
        """Block until the first sample has arrived (nvidia-smi takes a moment to start)."""
        t0 = time.time()
        while self.proc is not None and not self.lines and time.time() - t0 < timeout:
            time.sleep(0.02)

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        time.sleep(0.15)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.reader.join(timeout=5)
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            f = [x.strip() for x in line.split(",")]
            if len(f) < 8:
                continue
            try:
                sm.append(float(f[0]))
                smax.append(float(f[1]))
            except ValueError:
                continue
            for nm, v in zip(names, f[4:8]):
                if v.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------------------------------ inputs
# ncu summaries under profiles/ that record dram__bytes_read.sum + dram__bytes_write.sum of one
# launch of a kernel at this workload, as a line "traffic_bytes_per_launch: <bytes>".
TRAFFIC_FILES = {"rl_step": "profiles/rl_step_B4096_T1000.txt"}


def profiled_traffic(kernel):
    import re
    p = REPO / TRAFFIC_FILES[kernel]
    if not p.exists():
        return None
    m = re.search(r"^traffic_bytes_per_launch:\s*(\d+)", p.read_text(), flags=re.M)
    return int(m.group(1)) if m else None


def bind_to_gpu_numa_node(dev):
    """Restrict this process to the CPUs of the NUMA node the GPU's PCIe link hangs off (from sysfs),
    so that pinned host memory allocated afterwards is local to that link.  Returns the node, or
    None when the machine does not say (single-node hosts, containers without sysfs)."""
    try:
        p = torch.cuda.get_device_properties(dev)
        bus = f"{p.pci_domain_id:04x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
        base = Path("/sys/bus/pci/devices") / bus
        node = int((base / "numa_node").read_text().strip())
        if node < 0:
            return None
        cpus = set()
        for part in (base / "local_cpulist").read_text().strip().split(","):
            lo, _, hi = part.partition("-")
            cpus.update(range(int(lo), int(hi or lo) + 1))
        cpus &= set(os.sched_getaffinity(0))
        if not cpus:
            return None
        os.sched_setaffinity(0, cpus)
        return node
    except (OSError, ValueError, AttributeError):
        return None


def workload_config(world):
    """The workload both arms run (identical dicts, so the two JSON lines name the same config)."""
    return {"workload": "rl_pipeline: reward_to_go + ppo_clip_ext", "B": B, "T": T, "H": 1,
            "samples_per_gpu": N_SAMPLES, "gamma": 0.99, "done_p": 0.01, "clip_epsilon": 0.2,
            "parallelism": f"dp{world}: one batch per rank, PPO outputs over all ranks' samples"
            if world > 1 else "1 GPU"}


def make_sets(dev, rank, n_sets):
    from oracle import inputs  # seeded synthetic inputs of BASELINE.json configs[1]
    sets = []
    for i in range(n_sets):
        s = inputs.baseline_inputs("rl_pipeline", seed=1000 * rank + i)
        sets.append({k: (v.to(dev) if isinstance(v, torch.Tensor) else v) for k, v in s.items()})
    return sets


# -------------------------------------------------------------------------------- GPU arm
def run_b200(args, world, rank, local):
    pkg = importlib.import_module("cuda-optimization-benchmark_b200")
    lib = pkg.load()
    ops = pkg.ops
    dev = torch.device("cuda", local)
    stream = torch.cuda.current_stream(dev)
    sets = make_sets(dev, rank, ROTATE)
    gamma, eps = sets[0]["gamma"], sets[0]["clip_epsilon"]
    rtg_out = torch.empty(B, T, device=dev)
    ppo_out = torch.empty(7, device=dev)
    exchange = None
    if world > 1:
        import torch.distributed as dist
        chunk = lib.b200_ppo_chunk_elems()
        n_parts = (N_SAMPLES + chunk - 1) // chunk
        rec = lib.b200_ppo_partial_bytes()
        local_parts = torch.empty((n_parts, rec), dtype=torch.uint8, device=dev)
        all_parts = torch.empty((world * n_parts, rec), dtype=torch.uint8, device=dev)
        # The fused step exchanges the PPO partials over NVLink peer memory inside the kernel; the
        # NCCL all-gather (graph-replayed) is the fallback where CUDA IPC cannot be set up.
        try:
            exchange = ops.PeerExchange(world, rank, N_SAMPLES)
        except Exception as e:  # noqa: BLE001 - any failure selects the fallback, reported below
            print(f"rank {rank}: peer exchange unavailable ({e}); using the NCCL all-gather", file=sys.stderr)
        ok = torch.tensor([1 if exchange is not None else 0], device=dev)
        dist.all_reduce(ok, op=dist.ReduceOp.MIN)
        if int(ok.item()) == 0 and exchange is not None:
            exchange.close()
            exchange = None

    # Pre-bound C-ABI argument tuples per input set: the timed loop is one ctypes call per step
    # (N = 1), or the fused shard launch, the NCCL all-gather and the finish launch (N > 1).
    import ctypes
    P = ctypes.c_void_p
    cs = P(stream.cuda_stream)
    ws = ops.workspace("ppo", lib.b200_ppo_workspace_bytes(N_SAMPLES), dev)
    step_args, rtg_args, ppo_args = [], [], []
    for s in sets:
        rtg_in = (P(s["reward"].data_ptr()), P(s["done"].data_ptr()), gamma, B, T, P(rtg_out.data_ptr()))
        ppo_in = (P(s["current_log_prob"].data_ptr()), P(s["old_log_prob"].data_ptr()),
                  P(s["advantage"].data_ptr()), P(s["entropy"].data_ptr()), N_SAMPLES, eps)
        # The timed steps run back to back over resident batches: no kernel writes their inputs,
        # so each step declares them ready and reads them while the previous step finishes.
        if world == 1:
            step_args.append(rtg_in + ppo_in + (P(ppo_out.data_ptr()), P(ws.data_ptr()), ws.numel(), READY, cs))
        elif exchange is not None:
            step_args.append(rtg_in + ppo_in + (P(ppo_out.data_ptr()), P(ws.data_ptr()), ws.numel(), exchange.handle))
        else:
            step_args.append(rtg_in + ppo_in + (P(local_parts.data_ptr()), cs))
        rtg_args.append(rtg_in + (cs,))
        ppo_args.append(ppo_in + (P(ppo_out.data_ptr()), P(ws.data_ptr()), ws.numel(), cs))
    f_rtg, f_ppo = lib.b200_reward_to_go_async, lib.b200_ppo_async
    f_step = lib.b200_rl_step_ex_async if world == 1 else lib.b200_rl_step_shard_async
    f_finish = lib.b200_ppo_finish
    f_exchange, f_next_epoch = lib.b200_rl_step_exchange_async, lib.b200_peer_next_epoch
    if world > 1:
        finish_args = (P(all_parts.data_ptr()), world * n_parts, world * N_SAMPLES, 1, P(ppo_out.data_ptr()), cs)
    status = [0]
    flags = [READY]  # the exchange step's flags (the one-GPU step carries them in step_args)

    def step(i):
        if world > 1 and exchange is not None:
            exchange.epoch = f_next_epoch(exchange.epoch)
            status[0] |= f_exchange(*step_args[i % ROTATE], exchange.epoch, flags[0], cs)
            return
        status[0] |= f_step(*step_args[i % ROTATE])
        if world > 1:
            dist.all_gather_into_tensor(all_parts, local_parts)
            status[0] |= f_finish(*finish_args)

    def loop_ms(fn, k):
        """Device ms per call of `fn` over k back-to-back calls between one pair of events."""
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for i in range(k):
            fn(i)
        b.record(stream)
        torch.cuda.synchronize(dev)
        return a.elapsed_time(b) / k

    clocks = ClockSampler(dev)  # from before the warm-up to the end of the timed steps
    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize(dev)
    if status[0] != 0:
        raise RuntimeError(f"rl_step returned status {status[0]}")
    # N > 1: each step (shard kernel -> NCCL all-gather of the chunk partials -> finish) is replayed
    # from a CUDA graph, one per input set, so the host issues one launch per step instead of three
    # (the Python cost of the collective call would otherwise exceed the step's device time).
    step_graphs = []
    if world > 1 and exchange is None:
        side = torch.cuda.Stream(dev)
        side.wait_stream(stream)
        for k in range(ROTATE):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=side):
                cs_side = P(torch.cuda.current_stream(dev).cuda_stream)
                status[0] |= f_step(*step_args[k][:-1], cs_side)
                dist.all_gather_into_tensor(all_parts, local_parts)
                status[0] |= f_finish(*finish_args[:-1], cs_side)
            step_graphs.append(g)
        torch.cuda.synchronize(dev)

        def step(i):  # noqa: F811 (the graphed step replaces the eager one)
            step_graphs[i % ROTATE].replay()
        for i in range(args.warmup):
            step(i)
        torch.cuda.synchronize(dev)
    # Untimed soak: about 0.3 s of the same back-to-back steps just before the timed ones, so the
    # clock samples (every 100 ms) cover the load the timed steps run under; the step count is the
    # same on every rank (each exchange step is a collective step).
    clocks.wait_first()
    t_cal = time.perf_counter()
    for i in range(50):
        step(i)
    torch.cuda.synchronize(dev)
    per_step = (time.perf_counter() - t_cal) / 50
    n_soak = int(max_over_ranks(float(min(200000, max(500, int(0.3 / max(per_step, 1e-7))))), world))
    for i in range(n_soak):
        step(i)
    barrier(world)
    torch.cuda.synchronize(dev)
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for i in range(args.steps):
        step(i)
    t1.record(stream)
    torch.cuda.synchronize(dev)
    barrier(world)
    clk = clocks.stop()
    if status[0] != 0:
        raise RuntimeError(f"rl_step returned status {status[0]}")
    ms = max_over_ranks(t0.elapsed_time(t1) / args.steps, world)

    # Run-to-run spread of the same measurement: REPEAT_BATCHES more batches of K steps, each timed
    # on its own between synchronizes (the region above stays the headline).
    batch_us = []
    for _ in range(REPEAT_BATCHES):
        barrier(world)
        batch_us.append(max_over_ranks(loop_ms(step, args.steps), world) * 1e3)
    if status[0] != 0:
        raise RuntimeError(f"rl_step returned status {status[0]}")

    parity = None
    exchange_us = None
    if world > 1:
        parity = multi_gpu_parity(ops, lib, dev, stream, world, sets, step, rtg_out, ppo_out, status)
        exchange_us = zero_work_step_us(lib, dev, stream, world, sets, ws, exchange, args, status, loop_ms)
    else:
        exchange_us = zero_work_step_us(lib, dev, stream, world, sets, ws, None, args, status, loop_ms)
    del step_graphs  # graphs holding NCCL work are released before the process group is destroyed

    # Average duration of the fused kernel alone (the roofline's kernel): at N = 1 the timed step is
    # exactly one launch of it; at N > 1 its shard form is timed in its own back-to-back loop.
    def fused_only(i):
        status[0] |= f_step(*step_args[i % ROTATE])
    if world == 1 or exchange is not None:
        fused_ms = ms  # the timed step is one launch of the fused kernel (exchange included at N > 1)
    else:
        fused_ms = max_over_ranks(loop_ms(fused_only, args.steps), world)

    # The same steps without the inputs-ready declaration: each waits for the previous kernel
    # before reading (the default of the API; only the launch latency overlaps).
    waitfirst_ms = None
    if world == 1 or exchange is not None:
        wf_args = [a[:-2] + (0, cs) for a in step_args] if world == 1 else None

        def waitfirst(i):
            if world == 1:
                status[0] |= f_step(*wf_args[i % ROTATE])
            else:
                flags[0] = 0
                step(i)
                flags[0] = READY
        for i in range(args.warmup):
            waitfirst(i)
        torch.cuda.synchronize(dev)
        barrier(world)
        waitfirst_ms = max_over_ranks(loop_ms(waitfirst, args.steps), world)
        if status[0] != 0:
            raise RuntimeError(f"rl_step returned status {status[0]}")

    # The same steps with the done flags as bits (B200_STEP_DONE_BITS, packed once per input set
    # outside the timed loop), and reward-to-go alone from bits: 1/8 instead of 1 byte per flag.
    bits_ms = rtg_bits_ms = None
    if world == 1:
        words = [ops.pack_done(s["done"]) for s in sets]
        torch.cuda.synchronize(dev)
        bits_args = [a[:1] + (P(w.data_ptr()),) + a[2:-2] + (READY | ops.STEP_DONE_BITS, cs)
                     for a, w in zip(step_args, words)]
        rtgb_args = [(a[0], P(w.data_ptr())) + a[2:] for a, w in zip(rtg_args, words)]
        f_rtgb = lib.b200_reward_to_go_bits_async

        def bits_step(i):
            status[0] |= f_step(*bits_args[i % ROTATE])

        def rtg_bits(i):
            status[0] |= f_rtgb(*rtgb_args[i % ROTATE])
        for i in range(args.warmup):
            bits_step(i)
            rtg_bits(i)
        torch.cuda.synchronize(dev)
        bits_ms = loop_ms(bits_step, args.steps)
        rtg_bits_ms = loop_ms(rtg_bits, args.steps)
        if status[0] != 0:
            raise RuntimeError(f"done-bits step returned status {status[0]}")
        rtgb_bytes = 8 * B * T + 4 * B * ((T + 31) // 32)
        bits_bytes = rtgb_bytes + PPO_BYTES

    # The two ops as separate launches on the same rotation (per-op breakdown, unfused step time).
    for i in range(args.warmup):
        f_rtg(*rtg_args[i % ROTATE])
        f_ppo(*ppo_args[i % ROTATE])
    torch.cuda.synchronize(dev)

    def rtg_only(i):
        status[0] |= f_rtg(*rtg_args[i % ROTATE])

    def ppo_only(i):
        status[0] |= f_ppo(*ppo_args[i % ROTATE])

    def both(i):
        rtg_only(i)
        ppo_only(i)
    rtg_ms = max_over_ranks(loop_ms(rtg_only, args.steps), world)
    ppo_ms = max_over_ranks(loop_ms(ppo_only, args.steps), world)
    unfused_ms = max_over_ranks(loop_ms(both, args.steps), world)
    if status[0] != 0:
        raise RuntimeError(f"reward_to_go / ppo returned status {status[0]}")

    # Same K steps replayed from a CUDA graph (one graph per input set), no events between kernels:
    # shows how much of the eager step time is host launch overhead.
    graph_ms = None
    if world == 1:
        graphs = []
        side = torch.cuda.Stream(dev)
        for k in range(ROTATE):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=side):
                cs_side = P(torch.cuda.current_stream(dev).cuda_stream)
                f_step(*step_args[k][:-1], cs_side)
            graphs.append(g)
        for i in range(args.warmup):
            graphs[i % ROTATE].replay()
        torch.cuda.synchronize(dev)
        g0 = torch.cuda.Event(enable_timing=True)
        g1 = torch.cuda.Event(enable_timing=True)
        g0.record(stream)
        for i in range(args.steps):
            graphs[i % ROTATE].replay()
        g1.record(stream)
        torch.cuda.synchronize(dev)
        graph_ms = g0.elapsed_time(g1) / args.steps
        del graphs

    # ---- e2e: the host buffers live on the CPU socket the GPU is attached to: with one process per
    # GPU, pinned buffers on the far socket would send every rank's copies across the socket link.
    all_cpus = os.sched_getaffinity(0)
    numa = bind_to_gpu_numa_node(dev)
    # ---- e2e: same entry points, inputs from pinned host memory, results read back each step.
    # PCIe is full duplex: a step's results are read back on a copy stream while the next step's
    # inputs go up, so the outputs and their host copies alternate between two buffers (step i + 2
    # writes buffer i % 2 only after step i's read-back of it has finished).
    host = []
    for s in sets[:2]:
        host.append({k: (v.cpu().pin_memory() if isinstance(v, torch.Tensor) else v) for k, v in s.items()})
    dbuf = {k: torch.empty_like(v) for k, v in sets[0].items() if isinstance(v, torch.Tensor)}
    rtg_o = [rtg_out, torch.empty_like(rtg_out)]
    ppo_o = [ppo_out, torch.empty_like(ppo_out)]
    rtg_host = [torch.empty(B, T).pin_memory() for _ in range(2)]
    ppo_host = [torch.empty(7).pin_memory() for _ in range(2)]
    names = ["reward", "done", "current_log_prob", "old_log_prob", "advantage", "entropy"]
    h2d = sum(dbuf[k].numel() * dbuf[k].element_size() for k in names)
    d2h = rtg_host[0].numel() * 4 + ppo_host[0].numel() * 4
    copy_stream = torch.cuda.Stream(dev)
    read_done = [None, None]

    def e2e_step(i):
        h = host[i % 2]
        j = i % 2
        for k in names:
            dbuf[k].copy_(h[k], non_blocking=True)
        if read_done[j] is not None:
            stream.wait_event(read_done[j])  # buffer j's previous results have reached the host
        if world == 1:
            ops.rl_step(dbuf["reward"], dbuf["done"], gamma, dbuf["current_log_prob"], dbuf["old_log_prob"],
                        dbuf["advantage"], eps, dbuf["entropy"], rtg_out=rtg_o[j], ppo_out=ppo_o[j])
        elif exchange is not None:
            ops.rl_step_exchange(exchange, dbuf["reward"], dbuf["done"], gamma, dbuf["current_log_prob"],
                                 dbuf["old_log_prob"], dbuf["advantage"], eps, dbuf["entropy"], rtg_out=rtg_o[j],
                                 ppo_out=ppo_o[j])
        else:
            ops.rl_step_shard(dbuf["reward"], dbuf["done"], gamma, dbuf["current_log_prob"], dbuf["old_log_prob"],
                              dbuf["advantage"], eps, dbuf["entropy"], rtg_out=rtg_o[j], partials_out=local_parts)
            dist.all_gather_into_tensor(all_parts, local_parts)
            ops.ppo_finish(all_parts, world * N_SAMPLES, True, out=ppo_o[j])
        computed = torch.cuda.Event()
        computed.record(stream)
        copy_stream.wait_event(computed)
        with torch.cuda.stream(copy_stream):
            rtg_host[j].copy_(rtg_o[j], non_blocking=True)
            ppo_host[j].copy_(ppo_o[j], non_blocking=True)
            read_done[j] = torch.cuda.Event()
            read_done[j].record(copy_stream)

    e2e_steps = max(3, min(args.steps, 50))
    for i in range(3):
        e2e_step(i)
    torch.cuda.synchronize(dev)
    barrier(world)
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for i in range(e2e_steps):
        e2e_step(i)
    stream.wait_stream(copy_stream)  # the last read-back is inside the timed region
    b.record(stream)
    torch.cuda.synchronize(dev)
    barrier(world)
    e2e_ms = max_over_ranks(a.elapsed_time(b) / e2e_steps, world)
    os.sched_setaffinity(0, all_cpus)  # the CPU baselines below use every core again

    extra, sharded, cpu_ops = {}, None, None
    if not args.no_ops:
        extra = other_ops(ops, dev, world, rank)
        sharded = sharded_ops(ops, lib, dev, world, rank)
        # The E4M3 peak is measured last: its 1.5 s sustained loop heats the part and runs into the
        # power cap, which would slow whatever were timed right after it.
        fp8_fractions(extra, dev)
        if rank == 0 and world == 1 and not args.no_cpu:
            cpu_ops = cpu_op_baselines()
            for name, cb in cpu_ops.items():
                if name in extra:
                    extra[name]["cpu_baseline"] = cb

    peak, peak_kind = peaks()
    step_bytes = RTG_BYTES + PPO_BYTES
    achieved = step_bytes / (fused_ms * 1e-3) / 1e9
    per_step_launches = 1 if (world == 1 or exchange is not None) else 2
    line = {
        "metric": METRIC,
        "value": world * N_SAMPLES / (ms * 1e-3),
        "unit": "samples/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms,
        "us_per_step": ms * 1e3,
        "graph_us_per_step": graph_ms * 1e3 if graph_ms is not None else None,
        "unfused_us_per_step": unfused_ms * 1e3,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded; BASELINE.json configs[1] distributions)",
        "config": workload_config(world),
        "launch": "programmatic dependent launch; back-to-back steps over resident batches declare their inputs "
                  "ready (B200_STEP_INPUTS_READY)",
        "l2": f"rotating {ROTATE} input sets of {(RTG_BYTES - 4 * N_SAMPLES + PPO_BYTES) / 1e6:.0f} MB (> 126 MB L2)",
        "exchange": (("PPO totals exchanged over NVLink peer memory inside the fused kernel" if exchange is not None
                      else "PPO chunk partials all-gathered (NCCL); each step replayed from a CUDA graph")
                     if world > 1 else None),
        "repeat_batches": {"n": len(batch_us), "steps_each": args.steps,
                           "median_us_per_step": statistics.median(batch_us),
                           "min_us_per_step": min(batch_us), "max_us_per_step": max(batch_us),
                           "spread": max(batch_us) / min(batch_us) - 1.0,
                           "how": "after the headline region, batches of K steps each timed alone between device "
                                  "synchronizes (max over ranks)"},
        "exchange_us": exchange_us,
        "exchange_us_note": ("the step with no samples (B = T = n = 0): at N > 1 one launch whose finishing CTA "
                             "stores this rank's totals to every peer and waits for every peer's; at N = 1 the "
                             "launch, election and finish alone"),
        "parity": parity,
        "per_op": {
            "rl_step (fused)": {"us": fused_ms * 1e3, "bytes": step_bytes,
                                "gbs": achieved, "frac_of_hbm": achieved / peak},
            "rl_step (fused, inputs not declared ready)": (
                {"us": waitfirst_ms * 1e3, "gbs": step_bytes / (waitfirst_ms * 1e-3) / 1e9,
                 "frac_of_hbm": step_bytes / (waitfirst_ms * 1e-3) / 1e9 / peak} if waitfirst_ms else None),
            "rl_step (fused, done as bits)": (
                {"us": bits_ms * 1e3, "bytes": bits_bytes, "gbs": bits_bytes / (bits_ms * 1e-3) / 1e9,
                 "frac_of_hbm": bits_bytes / (bits_ms * 1e-3) / 1e9 / peak} if bits_ms else None),
            "note": "each op timed alone, back to back on the same input rotation",
            "reward_to_go": {"us": rtg_ms * 1e3, "bytes": RTG_BYTES,
                             "gbs": RTG_BYTES / (rtg_ms * 1e-3) / 1e9,
                             "frac_of_hbm": RTG_BYTES / (rtg_ms * 1e-3) / 1e9 / peak},
            "ppo_clip_ext": {"us": ppo_ms * 1e3, "bytes": PPO_BYTES,
                             "gbs": PPO_BYTES / (ppo_ms * 1e-3) / 1e9,
                             "frac_of_hbm": PPO_BYTES / (ppo_ms * 1e-3) / 1e9 / peak},
            "reward_to_go, done as bits": (
                {"us": rtg_bits_ms * 1e3, "bytes": rtgb_bytes, "gbs": rtgb_bytes / (rtg_bits_ms * 1e-3) / 1e9,
                 "frac_of_hbm": rtgb_bytes / (rtg_bits_ms * 1e-3) / 1e9 / peak} if rtg_bits_ms else None),
        },
        "roofline": {"bound": "hbm", "kernel": "rl::step_kernel (reward_to_go + ppo_clip_ext, one launch)",
                     "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "algorithmic_bytes": step_bytes,
                     "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)"
                     if peak_kind == "measured" else "fallback 6650 GB/s",
                     "traffic": profiled_traffic("rl_step"),
                     "traffic_source": TRAFFIC_FILES["rl_step"]},
        "e2e": {"value": world * N_SAMPLES / (e2e_ms * 1e-3), "unit": "samples/s", "ms_per_step": e2e_ms,
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "pipeline": "each step's results are read back on a second stream while the next step's inputs "
                            "go up (PCIe full duplex)",
                "host_numa_node": numa},
        "gpu_launches": per_step_launches * args.steps,
        "clocks": {"sm_mhz": clk["sm_mhz"], "sm_max_mhz": clk["sm_max_mhz"], "reasons": clk["reasons"],
                   "samples": clk["samples"],
                   "window": "nvidia-smi every 100 ms over the warm-up, a 0.3 s soak of the same steps and the "
                             "timed steps"},
    }
    if extra:
        line["ops"] = extra
    if sharded:
        line["ops_sharded"] = sharded
    if cpu_ops:
        for name in ("reward_to_go", "ppo_clip_ext"):
            line["per_op"][name]["cpu_baseline"] = cpu_ops[name]
    if rank == 0 and world == 1 and not args.no_cpu:
        line["cpu_baseline"] = cpu_baseline(args)
    if exchange is not None:
        torch.cuda.synchronize(dev)
        barrier(world)  # no rank still stores into another's buffer
        exchange.close()
        barrier(world)
    return line


def multi_gpu_parity(ops, lib, dev, stream, world, sets, step, rtg_out, ppo_out, status):
    """Correctness of the N > 1 step on the box that times it.  One more step on input set 0, then:
    (a) every rank's 7 PPO outputs are the same bits (all-gathered and compared with rank 0's);
    (b) they meet, at the ppo_clip tolerance, the library's fixed-order finish over all ranks'
        chunk partials of the same batches, gathered with NCCL (the single-GPU semantics of
        reference/ppo_clip/solution.cu:66-74,112-161 over the concatenated samples);
    (c) each rank's returns are the bits of the one-op reward_to_go entry on its own batch.
    Every rank computes the verdict; a failure raises on every rank (exit status 1), never a hang."""
    import torch.distributed as dist
    step(0)
    torch.cuda.synchronize(dev)
    mine = ppo_out.clone()
    rtg_step = rtg_out.clone()
    s = sets[0]
    parts = ops.ppo_partials(s["current_log_prob"], s["old_log_prob"], s["advantage"], s["clip_epsilon"],
                             s["entropy"])
    allp = torch.empty((world * parts.shape[0], parts.shape[1]), dtype=torch.uint8, device=dev)
    dist.all_gather_into_tensor(allp, parts)
    ref = ops.ppo_finish(allp, world * N_SAMPLES, True)
    outs = torch.empty((world, 7), dtype=torch.float32, device=dev)
    dist.all_gather_into_tensor(outs, mine)
    rtg_single = ops.reward_to_go(s["reward"], s["done"], s["gamma"])
    torch.cuda.synchronize(dev)
    if status[0] != 0:
        raise RuntimeError(f"rl_step returned status {status[0]}")
    bits = outs.view(torch.int32)
    identical = bool((bits == bits[0:1]).all())
    atol, rtol = 1e-5, 1e-4  # tasks/ppo_clip/tests/task.json tolerance
    diff = (mine.double() - ref.double()).abs()
    within = bool((diff <= atol + rtol * ref.double().abs()).all())
    same_bits_as_finish = bool(torch.equal(mine.view(torch.int32), ref.view(torch.int32)))
    rtg_same = bool(torch.equal(rtg_step.view(torch.int32), rtg_single.view(torch.int32)))
    ok = torch.tensor([int(identical and within and rtg_same)], device=dev)
    dist.all_reduce(ok, op=dist.ReduceOp.MIN)
    res = {"ranks_identical": identical, "vs_gathered_finish": within,
           "vs_gathered_finish_bit_identical": same_bits_as_finish,
           "vs_gathered_finish_max_abs_diff": float(diff.max()),
           "rtg_matches_single_op_bits": rtg_same, "all_ranks_ok": bool(int(ok.item()) == 1),
           "tolerance": {"atol": atol, "rtol": rtol},
           "how": "one exchange step on input set 0 after the timed steps: the 7 outputs all-gathered and "
                  "compared bitwise across ranks; against b200_ppo_finish over the NCCL-gathered chunk partials "
                  "of every rank's batch; returns against b200_reward_to_go_async on the rank's own batch"}
    if not res["all_ranks_ok"]:
        raise RuntimeError(f"multi-GPU parity failed: {res}")
    return res


def zero_work_step_us(lib, dev, stream, world, sets, ws, exchange, args, status, loop_ms):
    """Device µs of the step with no samples: at N > 1 the exchange step alone (launch, the
    finishing CTA's record stores to every peer over NVLink, the wait for every peer's record and
    the rank-order sum); at N = 1 the one-GPU step's fixed cost (launch, election, finish).  The
    compute part of a full step is the one-GPU step time; this is the part added per step."""
    import ctypes
    P = ctypes.c_void_p
    cs = P(stream.cuda_stream)
    s = sets[0]
    tmp = torch.empty(7, device=dev)
    base = (P(s["reward"].data_ptr()), P(s["done"].data_ptr()), s["gamma"], 0, 0, P(tmp.data_ptr()),
            P(s["current_log_prob"].data_ptr()), P(s["old_log_prob"].data_ptr()), P(s["advantage"].data_ptr()),
            P(s["entropy"].data_ptr()), 0, s["clip_epsilon"], P(tmp.data_ptr()), P(ws.data_ptr()), ws.numel())
    if exchange is not None:
        f = lib.b200_rl_step_exchange_async

        def one(i):
            exchange.epoch = lib.b200_peer_next_epoch(exchange.epoch)
            status[0] |= f(*base, exchange.handle, exchange.epoch, READY, cs)
    elif world == 1:
        f = lib.b200_rl_step_ex_async

        def one(i):
            status[0] |= f(*base, READY, cs)
    else:
        return None
    for i in range(args.warmup):
        one(i)
    torch.cuda.synchronize(dev)
    barrier(world)
    us = max_over_ranks(loop_ms(one, args.steps), world) * 1e3
    if status[0] != 0:
        raise RuntimeError(f"zero-work step returned status {status[0]}")
    return us


def other_ops(ops, dev, world, rank):
    """Device-timed µs of the other BASELINE ops at their BASELINE sizes (one input set each,
    already larger than L2 for the streaming ops), with their roofline fractions."""
    from oracle import inputs
    peak, _ = peaks()
    res = {}

    def timeit(fn, reps=20):
        """Device ms per call: `reps` back-to-back calls captured in a CUDA graph and replayed, so
        the Python cost of a call (more than a small kernel's runtime) stays out of the number."""
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):  # warm-up on the capture stream: its scratch exists before capture
            for _ in range(3):
                fn()
        torch.cuda.synchronize(dev)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=side):
            for _ in range(reps):
                fn()
        g.replay()  # warm
        torch.cuda.synchronize(dev)
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        g.replay()
        b.record()
        torch.cuda.synchronize(dev)
        del g
        return a.elapsed_time(b) / reps

    s = inputs.baseline_inputs("robust_l1", seed=rank)
    x, y = s["inp"].to(dev), s["target"].to(dev)
    out = torch.empty((), device=dev)
    ms = timeit(lambda: ops.robust_l1(x, y, out=out))
    res["robust_l1"] = {"us": ms * 1e3, "bytes": ROBUST_L1_BYTES, "gbs": ROBUST_L1_BYTES / ms / 1e6,
                        "frac_of_hbm": ROBUST_L1_BYTES / ms / 1e6 / peak}
    del x, y
    s = inputs.baseline_inputs("lif", seed=rank)
    xs, m0, be, th = (s[k].to(dev) for k in ("input_current", "mem0", "beta", "threshold"))
    sp = torch.empty_like(xs)
    fm = torch.empty_like(m0)
    ms = timeit(lambda: ops.leaky(xs, m0, be, th, spikes=sp, final_mem=fm))
    res["leaky"] = {"us": ms * 1e3, "bytes": LIF_BYTES, "gbs": LIF_BYTES / ms / 1e6,
                    "frac_of_hbm": LIF_BYTES / ms / 1e6 / peak}
    bits = torch.empty(((xs.shape[0] + 31) // 32,) + tuple(xs.shape[1:]), dtype=torch.int32, device=dev)
    ms = timeit(lambda: ops.leaky_packed(xs, m0, be, th, spike_bits=bits, final_mem=fm))
    nbytes = LIF_BYTES - 4 * xs.numel() + bits.numel() * 4  # spikes as bits instead of fp32
    res["leaky bit-packed spikes"] = {"us": ms * 1e3, "bytes": nbytes, "gbs": nbytes / ms / 1e6,
                                      "frac_of_hbm": nbytes / ms / 1e6 / peak}
    del bits
    # Training: the forward that also stores the membrane checkpoints (one per 16 steps), then the
    # surrogate-gradient backward: x and grad_spikes in, grad_input out (12 bytes per neuron-step)
    # plus the checkpoints, grad_final_mem in and grad_mem0 out.
    import ctypes
    lib, P = ops._lib(), ctypes.c_void_p
    T_, B_, H_ = xs.shape
    ck = torch.empty(((T_ + 15) // 16, B_, H_), device=dev)
    gs, gx = torch.randn_like(xs), torch.empty_like(xs)
    gf, gm = torch.randn_like(m0), torch.empty_like(m0)
    gb, gt = torch.empty_like(be), torch.empty_like(th)
    wsb = torch.empty(lib.b200_leaky_backward_workspace_bytes(B_, H_), dtype=torch.uint8, device=dev)
    cur = lambda: P(torch.cuda.current_stream(dev).cuda_stream)
    ms = timeit(lambda: lib.b200_leaky_train_async(xs.data_ptr(), m0.data_ptr(), be.data_ptr(), th.data_ptr(), T_,
                                                   B_, H_, sp.data_ptr(), fm.data_ptr(), ck.data_ptr(), cur()))
    nbytes = LIF_BYTES + ck.numel() * 4
    res["leaky training forward (+checkpoints)"] = {"us": ms * 1e3, "bytes": nbytes, "gbs": nbytes / ms / 1e6,
                                                    "frac_of_hbm": nbytes / ms / 1e6 / peak}
    ms = timeit(lambda: lib.b200_leaky_backward_async(xs.data_ptr(), ck.data_ptr(), be.data_ptr(), th.data_ptr(), T_,
                                                      B_, H_, gs.data_ptr(), gf.data_ptr(), 2.0, gx.data_ptr(),
                                                      gm.data_ptr(), gb.data_ptr(), gt.data_ptr(), wsb.data_ptr(),
                                                      wsb.numel(), cur()))
    nbytes = 12 * xs.numel() + ck.numel() * 4 + 8 * m0.numel()
    res["leaky surrogate backward"] = {"us": ms * 1e3, "bytes": nbytes, "gbs": nbytes / ms / 1e6,
                                       "frac_of_hbm": nbytes / ms / 1e6 / peak}
    del xs, m0, be, th, sp, fm, ck, gs, gx, gf, gm, gb, gt, wsb

    # GAE over the configs[1] batch: reward, value, next_value (f32), done, terminated (u8) in,
    # advantage and value target (f32) out: 22 bytes per element of algorithmic traffic.  Two input
    # sets (2 x 74 MB of inputs, 2 x 33 MB of outputs) alternate, so a call never finds its inputs
    # in the 126 MB L2.
    s = inputs.baseline_inputs("rl_pipeline", seed=rank)
    gsets = []
    for k in range(2):
        r = s["reward"].to(dev) if k == 0 else torch.roll(s["reward"].to(dev), 1, dims=0)
        dn = s["done"].to(dev)
        vv = torch.randn(r.shape, device=dev) * 0.5
        nv = torch.roll(vv, -1, dims=1)
        gsets.append((r, vv, nv, dn, torch.empty_like(r), torch.empty_like(r)))
    it = [0]

    def gae_call():
        r, vv, nv, dn, adv, tgt = gsets[it[0] % 2]
        it[0] += 1
        ops.gae(r, vv, nv, dn, dn, 0.99, 0.95, advantage=adv, value_target=tgt)
    ms = timeit(gae_call)
    nbytes = 22 * s["reward"].numel()
    res["gae B4096 T1000"] = {"us": ms * 1e3, "bytes": nbytes, "gbs": nbytes / ms / 1e6,
                              "frac_of_hbm": nbytes / ms / 1e6 / peak, "l2": "2 alternating input sets (213 MB)"}
    del gsets, s

    # Long rows (T >> B): 8 rows of 2^21 steps (151 MB of reward and done flags), the one-warp-per-
    # row scan against the chunked one (a warp per 1056-step chunk, one cooperative launch).  9
    # algorithmic bytes per step; the chunked form's second read of the chunks is served in part by
    # L2 (DRAM bytes per call from ncu in profiles/rtg_chunked_B8_T2097152.txt).
    # Two input sets alternate (302 MB with the outputs), so no call finds its inputs in L2.
    g = torch.Generator(device=dev).manual_seed(rank)
    rs = [torch.rand(8, 1 << 21, device=dev, generator=g) for _ in range(2)]
    dns = [torch.rand(8, 1 << 21, device=dev, generator=g) < 0.001 for _ in range(2)]
    outs = [torch.empty_like(rs[0]) for _ in range(2)]
    nbytes = 9 * rs[0].numel()
    turn = [0]

    def long_rows(f):
        turn[0] ^= 1
        f(rs[turn[0]], dns[turn[0]], 0.99, out=outs[turn[0]])
    ms = timeit(lambda: long_rows(ops.reward_to_go), reps=3)
    res["reward_to_go B8 T2097152 (one warp per row)"] = {"us": ms * 1e3, "bytes": nbytes, "gbs": nbytes / ms / 1e6,
                                                          "frac_of_hbm": nbytes / ms / 1e6 / peak}
    ms = timeit(lambda: long_rows(ops.reward_to_go_chunked))
    res["reward_to_go B8 T2097152 (chunked along T)"] = {"us": ms * 1e3, "bytes": nbytes, "gbs": nbytes / ms / 1e6,
                                                         "frac_of_hbm": nbytes / ms / 1e6 / peak,
                                                         "l2": "two input sets alternating (302 MB with outputs)"}
    del rs, dns, outs

    # E4M3 quantisation of the largest BASELINE activation (bf16 16384 x 8192): a per-tensor amax
    # needs every value before the first byte can be written, so the op reads x twice (the second
    # pass partly from L2) and writes one byte per value; those 5 bytes per value are its traffic.
    # Two copies of x alternate (536 MB), so no call finds the previous call's x in L2; measured
    # before the tensor-core ops, whose long GEMMs leave the GPU at its power cap.
    xqs = [torch.randn(16384, 8192, device=dev, generator=g).to(torch.bfloat16) for _ in range(2)]
    qq = torch.empty(xqs[0].shape, dtype=torch.float8_e4m3fn, device=dev)
    sq = torch.empty(1, device=dev)
    turn = [0]

    def quant():
        turn[0] ^= 1
        ops.fp8_quantize(xqs[turn[0]], q=qq, scale=sq)
    ms = timeit(quant, reps=20)
    nbytes = 5 * xqs[0].numel()
    res["fp8_quantize bf16 16384x8192"] = {"us": ms * 1e3, "bytes": nbytes, "gbs": nbytes / ms / 1e6,
                                           "frac_of_hbm": nbytes / ms / 1e6 / peak,
                                           "l2": "two copies of x alternating (536 MB)"}
    del xqs, qq, sq
    torch.cuda.synchronize(dev)

    # Tensor-core ops against the measured dense bf16 peak, burst and sustained (the long GEMMs run
    # at the power-capped clock); FP8 against the dense E4M3 rate measured with torch._scaled_mm
    # after the timings (fp8_peaks).  KAN issues three fp16 GEMM passes per useful flop (the hi/lo
    # operand split), so both its useful and its issued rates are reported.
    bf16_peak, bf16_sus = bf16_tflops(), bf16_tflops(sustained=True)
    s = inputs.baseline_inputs("kan", seed=rank)
    t = {k: (v.to(dev) if isinstance(v, torch.Tensor) else v) for k, v in s.items()}
    kout = torch.empty((s["B"], s["O"]), device=dev)
    ms = timeit(lambda: ops.efficient_kan(t["x"], t["grid"], t["base_weight"], t["spline_weight"], t["spline_scaler"],
                                          t["grid_size"], t["spline_order"], out=kout), reps=10)
    flops = 2 * s["B"] * s["O"] * s["I"] * (s["grid_size"] + s["spline_order"] + 1)
    res["efficient_kan"] = {"us": ms * 1e3, "useful_tflops": flops / ms / 1e9,
                            "issued_tflops": 3 * flops / ms / 1e9,
                            "frac_of_bf16_peak_issued": 3 * flops / ms / 1e9 / bf16_peak,
                            "frac_of_bf16_sustained_issued": 3 * flops / ms / 1e9 / bf16_sus}
    # The backward at the same size: two GEMMs of the forward's size (grad_out . W' and
    # grad_out^T . A) plus the operand transposes and the basis derivatives.
    gy = torch.randn(s["B"], s["O"], device=dev)
    ms = timeit(lambda: ops.efficient_kan_backward(t["x"], t["grid"], t["base_weight"], t["spline_weight"],
                                                   t["spline_scaler"], t["grid_size"], t["spline_order"], gy),
                reps=5)
    res["efficient_kan backward"] = {"us": ms * 1e3, "useful_tflops": 2 * flops / ms / 1e9,
                                     "issued_tflops": 6 * flops / ms / 1e9,
                                     "frac_of_bf16_peak_issued": 6 * flops / ms / 1e9 / bf16_peak,
                                     "frac_of_bf16_sustained_issued": 6 * flops / ms / 1e9 / bf16_sus}
    del t, kout, gy
    # FP8 at the four BASELINE shapes; inputs drawn on the device (the values do not change the
    # timing; parity is tested on the oracle's own inputs).  Where one call's operands and output
    # fit in L2 (M = 16: 17 MB, M = 1024: 29 MB) the calls rotate over copies whose total exceeds it,
    # so the W stream comes from HBM.  Fractions are of the E4M3 dense peak measured on this GPU
    # (torch._scaled_mm, i.e. cuBLASLt, at 8192^3: best of 10 and sustained over 1.5 s).
    g = torch.Generator(device=dev).manual_seed(1234 + rank)
    fp8_rows = []
    for M, N, K in inputs.BASELINE_SHAPES["fp8_linear"]:
        one = M * K + N * K + 2 * N + 2 * M * N
        copies = 1 if one > (128 << 20) else (200 << 20) // one + 1
        sets8 = []
        for _ in range(copies):
            x8, w8 = (torch.randn(r, K, device=dev, generator=g).clamp_(-448, 448).to(torch.float8_e4m3fn)
                      for r in (M, N))
            bias = (torch.randn(N, device=dev, generator=g) * 0.02).to(torch.bfloat16)
            sets8.append((x8, w8, bias, torch.empty((M, N), dtype=torch.bfloat16, device=dev)))
        it = [0]

        def fp8_call():
            x8, w8, bias, yout = sets8[it[0] % copies]
            it[0] += 1
            ops.fp8_linear(x8, 1.0, w8, 1.0, bias, out=yout)
        ms = timeit(fp8_call, reps=10 if M * N * K > 1 << 36 else max(50, 2 * copies))
        fp8_rows.append((M, N, K, one, copies, ms))
        del sets8
    for M, N, K, one, copies, ms in fp8_rows:
        flops = 2 * M * N * K
        res[f"fp8_linear M{M} N{N} K{K}"] = {
            "us": ms * 1e3, "tflops": flops / ms / 1e9, "flops": flops, "bytes": one,
            "gbs": one / ms / 1e6, "frac_of_hbm": one / ms / 1e6 / peak,
            "l2": (f"{copies} rotating operand sets ({copies * one / 1e6:.0f} MB)" if copies > 1
                   else f"one operand set of {one / 1e6:.0f} MB (> L2)")}
    return res


def graph_ms(fn, dev, world, reps):
    """Device ms per call of `fn` on every rank, max over ranks: `reps` calls captured in one CUDA
    graph (collectives included, captured in the same order on every rank), replayed once between
    events after a warm replay, so the host cost of a call stays out of the number."""
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):  # warm-up on the capture stream: its scratch exists before capture
        for _ in range(3):
            fn()
    torch.cuda.synchronize(dev)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=side):
        for _ in range(reps):
            fn()
    g.replay()
    torch.cuda.synchronize(dev)
    barrier(world)
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    a.record()
    g.replay()
    b.record()
    torch.cuda.synchronize(dev)
    ms = a.elapsed_time(b) / reps
    del g  # graphs holding NCCL work are released before the process group is destroyed
    return max_over_ranks(ms, world)


def sharded_ops(ops, lib, dev, world, rank):
    """robust-L1, LIF, KAN and FP8 at their BASELINE sizes split over the ranks (strong scaling),
    each rank holding only its shard in its own tensors, against the same op run whole on one GPU.

    - robust-L1 2^26: contiguous chunk-aligned element ranges; each rank writes one fp64 partial per
      8192-element chunk, the ranks all-gather the partials (NCCL, rank order = chunk order) and
      every rank runs the same fixed-order finish: the result must be the bits of the one-GPU call.
    - LIF [256, 64, 4096]: batch rows split (neurons are independent): spikes and final membrane
      must be the bits of the one-GPU call's rows.
    - KAN B8192 I1024 O1024 G5: batch rows split, weights replicated (each rank prepares its own
      weight planes): within the task tolerance of the one-GPU call's rows.
    - FP8 8192^3 and 16384 x 28672 x 8192: rows of M split, W and bias replicated: within the task
      tolerance of the one-GPU call's rows.  (M = 16 does not shard: its cost is the W stream, which
      every rank would read whole.)
    Every rank draws the same full inputs from the same seed, keeps its shard, and also runs the
    whole op once for the check and for `us_whole_1gpu`.  Times: graph-replayed calls, max over
    ranks; `speedup` = whole-op µs / sharded µs, `efficiency` = speedup / N.  A failed check raises
    on every rank."""
    import importlib as _il
    pdist = _il.import_module("cuda-optimization-benchmark_b200.dist")
    if world > 1:
        import torch.distributed as dist
    g = torch.Generator(device=dev).manual_seed(4321)  # the same full inputs on every rank
    res, oks = {}, []

    def entry(name, us, us_whole, checks, partition, extra=None):
        sp = us_whole / us
        e = {"n_gpus": world, "us": us, "us_whole_1gpu": us_whole, "speedup": sp, "efficiency": sp / world,
             "partition": partition, "parity": checks}
        if extra:
            e.update(extra)
        res[name] = e
        oks.append(all(v for k, v in checks.items() if isinstance(v, bool)))

    # robust-L1
    n = 1 << 26
    x = torch.randn(n, device=dev, generator=g)
    y = torch.randn(n, device=dev, generator=g)
    whole = ops.robust_l1(x, y).clone()
    us_whole = graph_ms(lambda: ops.robust_l1(x, y), dev, 1, 20) * 1e3
    chunk = lib.b200_robust_l1_chunk_elems()
    counts = pdist.shard_chunks(n, chunk, world)
    if len(set(counts)) != 1:
        raise RuntimeError("robust-L1 shards must hold the same number of chunks")
    lo, hi = pdist.shard_range(n, chunk, world, rank)
    xs, ys = x[lo:hi].clone(), y[lo:hi].clone()
    del x, y
    parts = torch.empty(counts[rank], dtype=torch.float64, device=dev)
    allp = torch.empty(sum(counts), dtype=torch.float64, device=dev) if world > 1 else parts
    out = torch.empty((), device=dev)
    import ctypes
    P = ctypes.c_void_p

    def shard_step():
        cs = P(torch.cuda.current_stream(dev).cuda_stream)
        lib.b200_robust_l1_shard_partials(P(xs.data_ptr()), P(ys.data_ptr()), hi - lo, P(parts.data_ptr()), cs)
        if world > 1:
            dist.all_gather_into_tensor(allp, parts)
        lib.b200_robust_l1_finish(P(allp.data_ptr()), sum(counts), n, P(out.data_ptr()), cs)

    def partials_only():
        cs = P(torch.cuda.current_stream(dev).cuda_stream)
        lib.b200_robust_l1_shard_partials(P(xs.data_ptr()), P(ys.data_ptr()), hi - lo, P(parts.data_ptr()), cs)
    shard_step()
    torch.cuda.synchronize(dev)
    same = bool(torch.equal(out.view(torch.int32), whole.view(torch.int32)))
    # 100 calls per timing so the ranks' start skew after the barrier (tens of µs between
    # processes) is a small share of the per-call figure of the forms that wait for every rank.
    us_nccl = graph_ms(shard_step, dev, world, 100) * 1e3
    us_part = graph_ms(partials_only, dev, world, 100) * 1e3
    # The exchange fused into the kernel (each rank pushes its chunk partials to every rank over
    # NVLink, every rank runs the same finish): one launch per call.  Its epochs advance per call,
    # so it is timed as eager back-to-back launches with pre-bound arguments, not from a graph.
    us_x, same_x, ex = None, None, None
    if world > 1:
        try:
            ex = ops.RobustL1Exchange(world, rank, n)
        except Exception as e:  # noqa: BLE001 - any failure leaves the NCCL form as the result
            print(f"rank {rank}: robust-L1 peer exchange unavailable ({e})", file=sys.stderr)
        okx = torch.tensor([1 if ex is not None else 0], device=dev)
        dist.all_reduce(okx, op=dist.ReduceOp.MIN)
        if int(okx.item()) == 0 and ex is not None:
            ex.close()
            ex = None
    if ex is not None:
        out_x = torch.empty((), device=dev)
        ws_x = torch.zeros(256, dtype=torch.uint8, device=dev)
        fx = lib.b200_robust_l1_exchange_async
        cs = P(torch.cuda.current_stream(dev).cuda_stream)
        xargs = (P(xs.data_ptr()), P(ys.data_ptr()), n, P(out_x.data_ptr()), P(ws_x.data_ptr()), 256, ex.handle)
        st = [0]

        def xstep():
            ex.epoch = lib.b200_peer_next_epoch(ex.epoch)
            st[0] |= fx(*xargs, ex.epoch, cs)
        for _ in range(5):
            xstep()
        torch.cuda.synchronize(dev)
        same_x = bool(torch.equal(out_x.view(torch.int32), whole.view(torch.int32)))
        barrier(world)
        a_ev, b_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a_ev.record()
        for _ in range(100):
            xstep()
        b_ev.record()
        torch.cuda.synchronize(dev)
        us_x = max_over_ranks(a_ev.elapsed_time(b_ev) / 100, world) * 1e3
        if st[0] != 0:
            raise RuntimeError(f"robust_l1 exchange returned status {st[0]}")
        barrier(world)
        ex.close()
        barrier(world)
    checks = {"bit_identical_to_1gpu": same}
    if same_x is not None:
        checks["exchange_bit_identical_to_1gpu"] = same_x
    # The result is the faster of the two exchange forms, both reported: the NCCL all-gather of the
    # chunk partials inside a CUDA graph (three launches), and the in-kernel push of each partial
    # over NVLink (one launch, timed eagerly; its finishing CTA also waits out the ranks' skew).
    use_x = us_x is not None and us_x < us_nccl
    us = us_x if use_x else us_nccl
    entry("robust_l1 2^26", us, us_whole, checks,
          f"{counts[rank]} chunks of {chunk} elements per rank; "
          + ("chunk partials pushed to every rank over NVLink inside the kernel (one launch)" if use_x
             else "chunk partials all-gathered (NCCL, in a graph)" if world > 1 else "one rank: no exchange"),
          {"us_partials_kernel": us_part, "us_exchange_and_finish": us - us_part,
           "us_nccl_allgather_form": us_nccl if world > 1 else None,
           "us_in_kernel_exchange_form": us_x,
           "bytes_per_rank": 8 * (hi - lo), "frac_of_hbm_partials": 8 * (hi - lo) / (us_part * 1e-6) / 1e9
           / peaks()[0]})
    del xs, ys, parts, allp

    # LIF
    T_, B_, H_ = 256, 64, 4096
    xl = torch.randn(T_, B_, H_, device=dev, generator=g) * 0.5 + 0.3
    m0 = torch.zeros(B_, H_, device=dev)
    be, th = torch.full((H_,), 0.9, device=dev), torch.full((H_,), 1.0, device=dev)
    sp_w, fm_w = ops.leaky(xl, m0, be, th)
    us_whole = graph_ms(lambda: ops.leaky(xl, m0, be, th, spikes=sp_w, final_mem=fm_w), dev, 1, 10) * 1e3
    b0, b1 = (B_ * rank) // world, (B_ * (rank + 1)) // world
    xsl, m0s = xl[:, b0:b1].contiguous(), m0[b0:b1].contiguous()
    del xl
    sp_s, fm_s = ops.leaky(xsl, m0s, be, th)
    torch.cuda.synchronize(dev)
    same_sp = bool(torch.equal(sp_s, sp_w[:, b0:b1]))
    same_fm = bool(torch.equal(fm_s.view(torch.int32), fm_w[b0:b1].view(torch.int32)))
    del sp_w, fm_w
    us = graph_ms(lambda: ops.leaky(xsl, m0s, be, th, spikes=sp_s, final_mem=fm_s), dev, world, 10) * 1e3
    nb = 8 * xsl.numel() + 8 * m0s.numel() + 8 * H_
    entry("leaky T256 B64 H4096", us, us_whole, {"spikes_bit_identical_to_1gpu": same_sp,
                                                 "final_mem_bit_identical_to_1gpu": same_fm},
          f"batch rows [{b0}, {b1}) of {B_} on this rank", {"frac_of_hbm": nb / (us * 1e-6) / 1e9 / peaks()[0]})
    del xsl, m0s, sp_s, fm_s

    # KAN
    Bk, Ik, Ok, G, K = 8192, 1024, 1024, 5, 3
    xk = torch.rand(Bk, Ik, device=dev, generator=g) * 2.0 - 1.0
    knots = torch.arange(-K, G + K + 1, dtype=torch.float32, device=dev)
    grid = (knots * (2.0 / G) - 1.0).expand(Ik, -1).contiguous()
    std = 1.0 / Ik ** 0.5
    bw = torch.randn(Ok, Ik, device=dev, generator=g) * std
    sw = torch.randn(Ok, Ik, G + K, device=dev, generator=g) * std
    sc = torch.ones(Ok, Ik, device=dev)
    out_w = ops.efficient_kan(xk, grid, bw, sw, sc, G, K)
    us_whole = graph_ms(lambda: ops.efficient_kan(xk, grid, bw, sw, sc, G, K, out=out_w), dev, 1, 5) * 1e3
    b0, b1 = (Bk * rank) // world, (Bk * (rank + 1)) // world
    xks = xk[b0:b1].contiguous()
    del xk
    out_s = ops.efficient_kan(xks, grid, bw, sw, sc, G, K)
    torch.cuda.synchronize(dev)
    ref = out_w[b0:b1].double()
    ok_tol = bool(((out_s.double() - ref).abs() <= 1e-5 + 1e-5 * ref.abs()).all())
    same = bool(torch.equal(out_s.view(torch.int32), out_w[b0:b1].view(torch.int32)))
    del out_w, ref
    us = graph_ms(lambda: ops.efficient_kan(xks, grid, bw, sw, sc, G, K, out=out_s), dev, world, 5) * 1e3
    # The pass criterion is the tolerance: the one-GPU call splits its last partial round of tiles
    # into K halves (their fp32 partials added once more), which a shard's tile count may not.
    entry("efficient_kan B8192 I1024 O1024 G5", us, us_whole,
          {"within_task_tolerance_of_1gpu": ok_tol},
          f"batch rows [{b0}, {b1}) of {Bk} on this rank, weights replicated",
          {"bit_identical_to_1gpu": same})
    del xks, out_s, bw, sw, sc, grid

    # FP8
    for M, N, Kf in ((8192, 8192, 8192), (16384, 28672, 8192)):
        x8 = torch.randn(M, Kf, device=dev, generator=g).to(torch.float8_e4m3fn)
        w8 = torch.randn(N, Kf, device=dev, generator=g).to(torch.float8_e4m3fn)
        bias = (torch.randn(N, device=dev, generator=g) * 0.02).to(torch.bfloat16)
        y_w = ops.fp8_linear(x8, 1.0, w8, 1.0, bias)
        us_whole = graph_ms(lambda: ops.fp8_linear(x8, 1.0, w8, 1.0, bias, out=y_w), dev, 1, 5) * 1e3
        m0_, m1_ = (M * rank) // world, (M * (rank + 1)) // world
        xs8 = x8[m0_:m1_].contiguous()
        del x8
        y_s = ops.fp8_linear(xs8, 1.0, w8, 1.0, bias)
        torch.cuda.synchronize(dev)
        ref = y_w[m0_:m1_].float()
        ok_tol = bool(((y_s.float() - ref).abs() <= 1e-2 + 1e-2 * ref.abs()).all())
        same = bool(torch.equal(y_s.view(torch.int16), y_w[m0_:m1_].view(torch.int16)))
        del y_w, ref
        us = graph_ms(lambda: ops.fp8_linear(xs8, 1.0, w8, 1.0, bias, out=y_s), dev, world, 5) * 1e3
        entry(f"fp8_linear M{M} N{N} K{Kf}", us, us_whole,
              {"within_task_tolerance_of_1gpu": ok_tol, "bit_identical_to_1gpu": same},
              f"rows [{m0_}, {m1_}) of M = {M} on this rank, W and bias replicated",
              {"tflops_all_ranks": 2.0 * M * N * Kf / (us * 1e-6) / 1e12})
        del xs8, w8, bias, y_s
    torch.cuda.synchronize(dev)
    ok = torch.tensor([int(all(oks))], device=dev)
    if world > 1:
        dist.all_reduce(ok, op=dist.ReduceOp.MIN)
    if int(ok.item()) != 1:
        raise RuntimeError(f"sharded-op parity failed: {res}")
    res["note"] = ("strong scaling: the BASELINE size split over the N ranks; us = max over ranks of one sharded "
                   "call (exchange included), us_whole_1gpu = the whole op on one GPU; fp8 M16 is replicas only")
    return res


_FP8_PEAK = {}


def fp8_fractions(res, dev):
    """Roofline fractions of the FP8 lines against the E4M3 peak measured on this GPU."""
    fp8_peak, fp8_sus = fp8_peaks(dev)
    hbm = peaks()[0]
    for name, e in res.items():
        if not name.startswith("fp8_linear M"):
            continue
        flops, one = e["flops"], e["bytes"]
        e["frac_of_fp8_peak"] = e["tflops"] / fp8_peak
        e["frac_of_fp8_sustained"] = e["tflops"] / fp8_sus
        e["bound"] = "hbm" if flops / one < fp8_peak * 1e3 / hbm else "fp8 tensor"
        e["fp8_peak_tflops"] = {"burst": fp8_peak, "sustained": fp8_sus,
                                "source": "measured here after the timings: torch._scaled_mm (cuBLASLt) e4m3 "
                                          "8192^3 -> bf16, best of 10 / mean over 1.5 s"}


def fp8_peaks(dev):
    """Dense E4M3 TFLOP/s of this GPU, measured with the vendor library (torch._scaled_mm, which
    calls cuBLASLt) at 8192^3 into bf16: (best of 10 single calls, mean over 1.5 s back to back).
    The roofline denominator of the FP8 GEMM, measured the way MEASURED_PEAKS.json measures bf16."""
    if dev.index in _FP8_PEAK:
        return _FP8_PEAK[dev.index]
    n = 8192
    g = torch.Generator(device=dev).manual_seed(7)
    a = torch.randn(n, n, device=dev, generator=g).to(torch.float8_e4m3fn)
    b = torch.randn(n, n, device=dev, generator=g).to(torch.float8_e4m3fn)
    one = torch.ones((), device=dev)

    def mm():
        torch._scaled_mm(a, b.t(), scale_a=one, scale_b=one, out_dtype=torch.bfloat16)
    for _ in range(3):
        mm()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    best = None
    for _ in range(10):
        e0.record()
        mm()
        e1.record()
        e1.synchronize()
        t = e0.elapsed_time(e1)
        best = t if best is None else min(best, t)
    flops = 2.0 * n ** 3
    k = max(10, int(1500.0 / best))
    e0.record()
    for _ in range(k):
        mm()
    e1.record()
    e1.synchronize()
    sus = e0.elapsed_time(e1) / k
    _FP8_PEAK[dev.index] = (flops / best / 1e9, flops / sus / 1e9)
    del a, b
    return _FP8_PEAK[dev.index]


# -------------------------------------------------------------------------------- CPU baseline
def cpu_step_fn():
    from oracle import eager, inputs
    s = inputs.baseline_inputs("rl_pipeline", seed=0)

    def run():
        eager.reward_to_go(s["reward"], s["done"], s["gamma"])
        eager.ppo_clip(s["current_log_prob"], s["old_log_prob"], s["advantage"], s["clip_epsilon"], s["entropy"])
    return run


def cpu_op_baselines():
    """CPU-eager µs of each op at its BASELINE size on this host's cores: oracle/eager.py, the
    PyTorch-eager fp32 restatement of each task's reference() (tasks/<task>/reference.py), median of
    3 after one warm-up.  KAN and the large FP8 shapes run on a row subset and are scaled to the
    full batch linearly (each row's work is independent; the per-call weight preparation is then
    counted once per subset, so the scaled figure is an upper bound of a whole call)."""
    from oracle import eager
    cores = cpu_cores()
    torch.set_num_threads(cores)
    g = torch.Generator().manual_seed(99)
    res = {}

    def med(fn, reps=3):
        fn()
        ts = []
        for _ in range(reps):
            t = time.perf_counter()
            fn()
            ts.append(time.perf_counter() - t)
        return statistics.median(ts)

    def put(name, sec, scale, sample):
        res[name] = {"us": sec * scale * 1e6, "cores": cores, "kind": "port",
                     "sample": sample, "sample_us": sec * 1e6, "scale": scale,
                     "what": "oracle/eager.py (PyTorch-eager fp32 restatement of the reference's reference())"}

    from oracle import inputs
    r = inputs.baseline_inputs("rl_pipeline", seed=0)
    put("reward_to_go", med(lambda: eager.reward_to_go(r["reward"], r["done"], r["gamma"])), 1, "full [4096, 1000]")
    put("ppo_clip_ext", med(lambda: eager.ppo_clip(r["current_log_prob"], r["old_log_prob"], r["advantage"],
                                                    r["clip_epsilon"], r["entropy"])), 1, "full 4,096,000 samples")
    del r
    x = torch.randn(1 << 26, generator=g)
    y = torch.randn(1 << 26, generator=g)
    put("robust_l1", med(lambda: eager.pow_abs_sqrt_mean(x, y)), 1, "full 2^26 elements")
    del x, y
    xl = torch.randn(256, 64, 4096, generator=g) * 0.5 + 0.3
    m0 = torch.zeros(64, 4096)
    be, th = torch.full((4096,), 0.9), torch.full((4096,), 1.0)
    put("leaky", med(lambda: eager.leaky(xl, m0, be, th)), 1, "full [256, 64, 4096]")
    del xl
    def fitted(name, run, rows, full, reps=3):
        """Two row counts r and 2r: time = fixed + per_row * rows, extrapolated to the full batch
        (the per-call weight preparation is the fixed part, the rows' work the slope)."""
        t1 = med(lambda: run(rows), reps)
        t2 = med(lambda: run(2 * rows), reps)
        per_row = max(t2 - t1, 0.0) / rows
        fixed = max(t1 - per_row * rows, 0.0)
        sec = fixed + per_row * full
        res[name] = {"us": sec * 1e6, "cores": cores, "kind": "port",
                     "sample": f"{rows} and {2 * rows} of {full} rows, extrapolated linearly in rows "
                               f"(fixed {fixed * 1e3:.1f} ms + {per_row * 1e6:.1f} us per row)",
                     "sample_us": [t1 * 1e6, t2 * 1e6],
                     "what": "oracle/eager.py (PyTorch-eager fp32 restatement of the reference's reference())"}

    Bk, I, O, G, K = 8192, 1024, 1024, 5, 3
    xk = torch.rand(1024, I, generator=g) * 2 - 1
    knots = torch.arange(-K, G + K + 1, dtype=torch.float32)
    grid = (knots * (2.0 / G) - 1.0).expand(I, -1).contiguous()
    bw = torch.randn(O, I, generator=g) / 32
    sw = torch.randn(O, I, G + K, generator=g) / 32
    sc = torch.ones(O, I)
    fitted("efficient_kan", lambda r: eager.efficient_kan(xk[:r], grid, bw, sw, sc, K), 512, Bk)
    del xk, bw, sw, sc
    for (M, N, Kf), rows in (((16, 4096, 4096), 16), ((1024, 4096, 4096), 1024), ((8192, 8192, 8192), 256),
                             ((16384, 28672, 8192), 64)):
        xq = torch.randint(0, 0x7E, (min(M, 2 * rows), Kf), dtype=torch.uint8, generator=g).view(torch.float8_e4m3fn)
        wq = torch.randint(0, 0x7E, (N, Kf), dtype=torch.uint8, generator=g).view(torch.float8_e4m3fn)
        bias = torch.zeros(N, dtype=torch.bfloat16)
        name = f"fp8_linear M{M} N{N} K{Kf}"
        if rows == M:
            put(name, med(lambda: eager.fp8_linear(xq, 2.0, wq, 2.0, bias)), 1, "full call")
        else:
            fitted(name, lambda r: eager.fp8_linear(xq[:r], 2.0, wq, 2.0, bias), rows, M, reps=2)
        del xq, wq
    return res


def cpu_cores():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_baseline(args, reps=None):
    cores = cpu_cores()
    torch.set_num_threads(cores)
    run = cpu_step_fn()
    run()
    times = []
    reps = reps or 5
    for _ in range(reps):
        t = time.perf_counter()
        run()
        times.append(time.perf_counter() - t)
    sec = statistics.median(times)
    return {"value": N_SAMPLES / sec, "unit": "samples/s", "cores": cores, "kind": "port",
            "sample": f"full configs[1] batch (B={B}, T={T}); median of {reps} after 1 warm-up; "
                      f"PyTorch-eager fp32 restatement of the reference's reference() for reward_to_go and "
                      f"ppo_clip (+ entropy mean)",
            "ms_per_step": sec * 1e3}


def run_reference(args, world, rank):
    if rank != 0:
        return None
    cores = cpu_cores()
    torch.set_num_threads(cores)
    run = cpu_step_fn()
    for _ in range(args.warmup):
        run()
    t = time.perf_counter()
    for _ in range(args.steps):
        run()
    sec = (time.perf_counter() - t) / args.steps
    v = N_SAMPLES / sec
    return {"metric": METRIC, "value": v, "unit": "samples/s", "impl": "reference", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": sec * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded; BASELINE.json configs[1] distributions)",
            "config": workload_config(world),
            "cpu_baseline": {"value": v, "unit": "samples/s", "cores": cores, "kind": "port",
                             "sample": f"full configs[1] batch per step, {args.steps} steps after {args.warmup} "
                                       f"warm-up; PyTorch-eager fp32 restatement of the reference's reference()"},
            "e2e": {"value": v, "unit": "samples/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


PROFILE_FP8 = {"fp8_m16": (16, 4096, 4096), "fp8_m1024": (1024, 4096, 4096), "fp8_8192": (8192, 8192, 8192),
               "fp8_16384": (16384, 28672, 8192), "fp8_ref_timed": (2048, 4096, 1024)}


def run_profile(ops_list, reps):
    """Run each listed op `reps` times at its BASELINE size on cuda:0 and print nothing but the
    device fault word: the workload for `ncu` launch lists and captures (profiles/*.txt)."""
    from oracle import inputs
    pkg = importlib.import_module("cuda-optimization-benchmark_b200")
    lib = pkg.load()
    ops = pkg.ops
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    if "rl_step" in ops_list:
        s = {k: (v.to(dev) if isinstance(v, torch.Tensor) else v)
             for k, v in inputs.baseline_inputs("rl_pipeline", 0).items()}
        out = torch.empty(B, T, device=dev)
        po = torch.empty(7, device=dev)
        for _ in range(reps):
            ops.rl_step(s["reward"], s["done"], s["gamma"], s["current_log_prob"], s["old_log_prob"], s["advantage"],
                        0.2, s["entropy"], rtg_out=out, ppo_out=po)
    if "rtg" in ops_list or "ppo" in ops_list:
        s = {k: (v.to(dev) if isinstance(v, torch.Tensor) else v)
             for k, v in inputs.baseline_inputs("rl_pipeline", 0).items()}
        out = torch.empty(B, T, device=dev)
        po = torch.empty(7, device=dev)
        for _ in range(reps):
            if "rtg" in ops_list:
                ops.reward_to_go(s["reward"], s["done"], s["gamma"], out=out)
            if "ppo" in ops_list:
                ops.ppo_clip(s["current_log_prob"], s["old_log_prob"], s["advantage"], 0.2, s["entropy"], out=po)
    if "lif" in ops_list or "lif_packed" in ops_list or "lif_backward" in ops_list:
        s = {k: (v.to(dev) if isinstance(v, torch.Tensor) else v) for k, v in inputs.baseline_inputs("lif", 0).items()}
        if "lif_backward" in ops_list:
            _, _, ck = ops.leaky_train(s["input_current"], s["mem0"], s["beta"], s["threshold"])
            gs = torch.randn_like(s["input_current"])
        for _ in range(reps):
            if "lif" in ops_list:
                ops.leaky(s["input_current"], s["mem0"], s["beta"], s["threshold"])
            if "lif_packed" in ops_list:
                ops.leaky_packed(s["input_current"], s["mem0"], s["beta"], s["threshold"])
            if "lif_backward" in ops_list:
                ops.leaky_backward(s["input_current"], ck, s["beta"], s["threshold"], gs, None, 2.0)
    if "robust_l1" in ops_list:
        s = inputs.baseline_inputs("robust_l1", 0)
        a, b = s["inp"].to(dev), s["target"].to(dev)
        for _ in range(reps):
            ops.robust_l1(a, b)
    if "kan" in ops_list:
        s = inputs.baseline_inputs("kan", 0)
        t = {k: s[k].to(dev) for k in ["x", "grid", "base_weight", "spline_weight", "spline_scaler"]}
        out = torch.empty(s["B"], s["O"], device=dev)
        nb = lib.b200_efficient_kan_workspace_bytes(5, 3, s["B"], s["I"], s["O"])
        ws = torch.empty(nb, dtype=torch.uint8, device=dev)
        for _ in range(reps):
            lib.b200_efficient_kan_async(t["x"].data_ptr(), t["grid"].data_ptr(), t["base_weight"].data_ptr(),
                                         t["spline_weight"].data_ptr(), t["spline_scaler"].data_ptr(), 5, 3, s["B"],
                                         s["I"], s["O"], out.data_ptr(), ws.data_ptr(), nb, None)
    if "gae" in ops_list:  # configs[1] batch, as the bench's `ops` line
        s = inputs.baseline_inputs("rl_pipeline", seed=0)
        r, dn = s["reward"].to(dev), s["done"].to(dev)
        vv = torch.randn(r.shape, device=dev) * 0.5
        nv = torch.roll(vv, -1, dims=1)
        adv, tgt = torch.empty_like(r), torch.empty_like(r)
        for _ in range(reps):
            ops.gae(r, vv, nv, dn, dn, 0.99, 0.95, advantage=adv, value_target=tgt)
    if "rtg_long" in ops_list:  # 8 rows of 2^21 steps, chunked along T
        g = torch.Generator(device=dev).manual_seed(0)
        r = torch.rand(8, 1 << 21, device=dev, generator=g)
        dn = torch.rand(8, 1 << 21, device=dev, generator=g) < 0.001
        out = torch.empty_like(r)
        for _ in range(reps):
            ops.reward_to_go_chunked(r, dn, 0.99, out=out)
    if "fp8_quant" in ops_list:  # bf16 16384 x 8192, as the bench's `ops` line
        g = torch.Generator(device=dev).manual_seed(0)
        xq = torch.randn(16384, 8192, device=dev, generator=g).to(torch.bfloat16)
        qq = torch.empty(xq.shape, dtype=torch.float8_e4m3fn, device=dev)
        sq = torch.empty(1, device=dev)
        for _ in range(reps):
            ops.fp8_quantize(xq, q=qq, scale=sq)
    if "kan_timed" in ops_list:  # the reference's timed case (tasks/efficient_kan/tests/task.json, G = 8)
        s = inputs.task_inputs("efficient_kan", {"B": 4096, "I": 256, "O": 512}, 305)
        t = {k: s[k].to(dev) for k in ["x", "grid", "base_weight", "spline_weight", "spline_scaler"]}
        out = torch.empty(s["B"], s["O"], device=dev)
        for _ in range(reps):
            ops.efficient_kan(t["x"], t["grid"], t["base_weight"], t["spline_weight"], t["spline_scaler"], 8, 3,
                              out=out)
    if "kan_backward" in ops_list:
        s = inputs.baseline_inputs("kan", 0)
        t = {k: s[k].to(dev) for k in ["x", "grid", "base_weight", "spline_weight", "spline_scaler"]}
        gy = torch.randn(s["B"], s["O"], device=dev)
        for _ in range(reps):
            ops.efficient_kan_backward(t["x"], t["grid"], t["base_weight"], t["spline_weight"], t["spline_scaler"], 5, 3,
                                       gy)
    for name in [x for x in ops_list if x in PROFILE_FP8]:
        M, N, K = PROFILE_FP8[name]
        s = inputs.baseline_inputs("fp8_linear", 0, shape=(M, N, K))
        x, w, bb = s["x_fp8"].to(dev), s["w_fp8"].to(dev), s["bias"].to(dev)
        o = torch.empty(M, N, dtype=torch.bfloat16, device=dev)
        for _ in range(reps):
            lib.b200_fp8_linear_async(M, K, N, x.data_ptr(), s["scale_x"], w.data_ptr(), s["scale_w"], bb.data_ptr(),
                                      o.data_ptr(), None)
    torch.cuda.synchronize()
    print("device fault word:", lib.b200_device_fault(), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--no-ops", action="store_true", help="skip the per-op lines of the other streaming ops")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--profile", default=None,
                    help="comma list of ops (rl_step, rtg, ppo, gae, rtg_long, fp8_quant, lif, lif_packed, lif_backward, "
                         "robust_l1, kan, kan_timed, "
                         "kan_backward, fp8_m16, fp8_m1024, "
                         "fp8_8192, "
                         "fp8_16384, fp8_ref_timed): run each --steps times for ncu, no timing")
    args = ap.parse_args()
    if args.profile:
        run_profile(args.profile.split(","), args.steps)
        return
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        line = run_reference(args, world, rank)
        if line is not None:
            print(json.dumps(line), flush=True)
        return
    world, rank, local = dist_setup(args.gpus)
    line = run_b200(args, world, rank, local)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
