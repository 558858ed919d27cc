"""Benchmark of the tiered paged decode-attention path (one JSON line on rank 0).

Workload (benchmark configuration 5, Llama-3-8B attention shape, 32k context):
batch 32 sequences x 32768 tokens, 32 query / 8 KV heads, head_dim 128, block
16, HOT fraction 0.25 with the rest split 2:1 WARM:COLD (Format R, the
reference's uint8 layout).  One step = one decode-attention call for the
whole batch.  Inputs are seeded synthetic N(0, 1) data; the pools (2+ GB) are
far larger than the 126 MB L2, so no flush is needed between steps.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--hot-frac H] [--block-size BS] [--sweep]

For N > 1 the script runs under torchrun: each rank owns its own batch of 32
sequences (data-parallel, no collective on the data path; weak scaling) and
`value` is the bytes of all ranks over the slowest rank's device time.

On one GPU the line also carries `c1` (configuration 1, the parity op: us per
call, eager and graph-replayed), `c2` (configuration 2's attention at the
TinyLlama shape, 22 layers, L2 flushed per step), `demote` (2^20-tile
HOT->WARM demotion and promotion) and `sweep` (configuration 5's hot
fractions at block 16 and 32); `--no-single-extras` leaves them out.

The same line carries two strong-scaling objects (fixed total work split over
the N ranks, each replayed from a CUDA graph, max over ranks):
  c4 -- configuration 4, one 131072-token context over 32 layers, each layer's
        blocks split into time-balanced contiguous ranges; ms per step with
        the partials exchanged inside the decode launch over peer memory,
        the NCCL all-gather + merge variant beside it, the local shard decode
        alone, and layer-0 parity against the unsharded one-rank output;
  c3 -- configuration 3's attention, 64 sequences x 8192 tokens (20/60/20)
        split data-parallel; aggregate tokens/s and per-GPU GB/s.
(`--no-scaling-extras` leaves them out.)
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np
import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "tiered decode-attn HBM GB/s (Llama-3-8B attention shape, 32k ctx)"
PEAKS = os.path.join(ROOT, "MEASURED_PEAKS.json")
TRAFFIC = os.path.join(ROOT, "profiles", "ncu_traffic.json")
FALLBACK_HBM_GBS = 6650.0


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--batch", type=int, default=32)
    ap.add_argument("--ctx", type=int, default=32768)
    ap.add_argument("--hot-frac", type=float, default=0.25)
    ap.add_argument("--warm-frac", type=float, default=None,
                    help="WARM share of the blocks (default: the non-HOT blocks split 2:1 "
                         "WARM:COLD, configuration 5); 0.6 with --hot-frac 0.2 is configuration "
                         "3's 20/60/20 mix")
    ap.add_argument("--block-size", type=int, default=16)
    ap.add_argument("--sweep", action="store_true",
                    help="time hot fractions 1.0/0.5/0.25/0.1 at block 16 and 32 also on several "
                         "GPUs (one GPU: always, unless --no-single-extras)")
    ap.add_argument("--config", choices=["c5", "c4", "demote", "tick", "append", "prefill",
                                         "prefill_store"],
                    default="c5",
                    help="c5: data-parallel batches (default); c4: one 131k-token context "
                         "over 32 layers, sharded by block range across the GPUs; demote: "
                         "HOT->WARM demotion of 2^20 fp16 [16 x 128] tiles per GPU; tick: one "
                         "policy tick (storage sync) of a 2048-block layer; append: the "
                         "decode-time KV append of one token; prefill: exact prefill block "
                         "scores of one 8192-token layer")
    ap.add_argument("--layers", type=int, default=32)
    ap.add_argument("--demote-blocks", type=int, default=65536,
                    help="demote: demoted blocks per launch (x 8 kv heads x K/V tiles)")
    ap.add_argument("--exchange", choices=["p2p", "nccl"], default="p2p",
                    help="c4 on several GPUs: partials exchanged over peer memory inside the "
                         "decode launch (p2p) or NCCL all-gather + merge launch (nccl)")
    ap.add_argument("--no-graph", action="store_true",
                    help="c4: launch every layer from Python instead of replaying a CUDA graph")
    ap.add_argument("--no-scaling-extras", action="store_true",
                    help="leave out the c4 (one 131072-token context sharded over the GPUs) and "
                         "c3 (64 x 8192-token sequences split over the GPUs) strong-scaling "
                         "objects of the headline line")
    ap.add_argument("--no-single-extras", action="store_true",
                    help="one GPU: leave out the c1 (parity op), c2 (TinyLlama-shape attention), "
                         "demote and sweep objects of the headline line")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    return ap.parse_args()


# --------------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi samples of SM clock and throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines: list[str] = []
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()
        t0 = time.time()
        while not self.lines and time.time() - t0 < 10.0:  # wait for the first sample
            time.sleep(0.05)

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.thread:
            self.thread.join(timeout=2)
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm)}


# --------------------------------------------------------------------------- helpers
def hbm_peak():
    try:
        with open(PEAKS) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def ncu_traffic(key: str):
    try:
        with open(TRAFFIC) as f:
            return json.load(f).get(key)
    except Exception:
        return None


def workload_key(a) -> str:
    w = "" if getattr(a, "warm_frac", None) is None else f"_w{a.warm_frac:g}"
    return f"c5_b{a.batch}_ctx{a.ctx}_h{a.hot_frac:g}{w}_bs{a.block_size}"


# The headline workload's shape: Llama-3-8B attention heads, seeded.
Q_HEADS, KV_HEADS, HEAD_DIM, SEED = 32, 8, 128, 1234


def host_tier_counts(num_blocks: int, hot_frac: float, warm_frac: float | None = None):
    """(n_hot, n_warm, n_cold) of one sequence, computed on the host without
    importing the package: the same rule as workloads.tier_counts (a CPU test
    checks that they agree)."""
    n_hot = min(num_blocks, max(1, int(round(hot_frac * num_blocks))))
    rest = num_blocks - n_hot
    n_warm = int(round(rest * 2.0 / 3.0)) if warm_frac is None else \
        min(rest, int(round(warm_frac * num_blocks)))
    return n_hot, n_warm, rest - n_warm


def host_first_states(num_blocks: int, n_hot: int, n_warm: int, seed: int) -> np.ndarray:
    """Tier states of sequence 0 drawn exactly as workloads.assign_tiers draws
    them (the same CPU generator and permutation), on the host."""
    gen = torch.Generator().manual_seed(seed)
    states = np.full(num_blocks, 2, np.int32)
    states[0] = 0
    if n_hot > 1:
        states[num_blocks - (n_hot - 1):] = 0
    middle = np.arange(1, num_blocks - (n_hot - 1))
    pick = torch.randperm(middle.size, generator=gen)[:n_warm].numpy()
    states[middle[pick]] = 1
    return states


def host_bytes_per_step(batch, nb, n_hot, n_warm, bs, d, hkv, hq) -> int:
    """Algorithmic HBM bytes of one decode call (Workload.algorithmic_bytes on the host)."""
    per_seq_head = n_hot * bs * 4 * d + n_warm * (bs * 2 * d + 8 * bs)
    return batch * (hkv * per_seq_head + 12 * nb + 2 * hq * d * 2)


def bench_config(a, world: int) -> dict:
    """The `config` of the headline line, identical for both arms (it depends
    on the arguments and the world size only)."""
    nb = -(-a.ctx // a.block_size)
    n_hot, n_warm, n_cold = host_tier_counts(nb, a.hot_frac, getattr(a, "warm_frac", None))
    return {"workload": workload_key(a), "batch": a.batch, "q_heads": Q_HEADS,
            "kv_heads": KV_HEADS, "head_dim": HEAD_DIM, "block_size": a.block_size,
            "ctx_tokens": a.ctx, "hot_frac": a.hot_frac, "blocks_per_seq": nb,
            "hot_blocks": n_hot, "warm_blocks": n_warm, "cold_blocks": n_cold, "seed": SEED,
            "warm_format": "R (uint8 + fp16 scale/zero)",
            "parallelism": f"dp{world} (independent batches, no collective)",
            "l2": "inputs >> 126 MB L2; no flush needed",
            "bytes_per_step_per_gpu": host_bytes_per_step(a.batch, nb, n_hot, n_warm, a.block_size,
                                                          HEAD_DIM, KV_HEADS, Q_HEADS)}


def host_unit_sample(a, seed: int):
    """One (sequence, kv head) unit of the headline workload built on the host:
    sequence 0's tier layout (same seed and draws as our arm), N(0, 1) fp16
    K/V and query from a host generator, WARM blocks quantized by the oracle's
    restatement of quantize_fp16_to_int8 (bit-exact with the reference).
    Nothing here touches a GPU or this package."""
    from oracle import tierkv_oracle as orc
    bs, d, g = a.block_size, HEAD_DIM, Q_HEADS // KV_HEADS
    nb = -(-a.ctx // bs)
    n_hot, n_warm, _ = host_tier_counts(nb, a.hot_frac, getattr(a, "warm_frac", None))
    states = host_first_states(nb, n_hot, n_warm, seed)
    lengths = np.full(nb, bs, np.int32)
    lengths[-1] = a.ctx - (nb - 1) * bs
    rng = np.random.default_rng(seed)
    table = np.full(nb, -1, np.int32)
    hot_idx, warm_idx = np.nonzero(states == 0)[0], np.nonzero(states == 1)[0]
    table[hot_idx] = rng.permutation(hot_idx.size)
    table[warm_idx] = rng.permutation(warm_idx.size)
    f16 = lambda *shape: rng.standard_normal(shape, dtype=np.float32).astype(np.float16)  # noqa: E731
    hot_k, hot_v = f16(max(1, hot_idx.size), 1, bs, d), f16(max(1, hot_idx.size), 1, bs, d)
    wk, ks, kz = orc.quantize_rows_r(f16(max(1, warm_idx.size), 1, bs, d))
    wv, vs, vz = orc.quantize_rows_r(f16(max(1, warm_idx.size), 1, bs, d))
    return dict(query=f16(1, g, d), table=table[None], states=states[None], lengths=lengths[None],
                num_blocks=nb, hot_k=hot_k, hot_v=hot_v, warm_k=wk, warm_v=wv, k_scale=ks,
                k_zero=kz, v_scale=vs, v_zero=vz, groups=g, scaling=d ** -0.5)


def build_workload(a, seed, device):
    from paged_tierkv_b200 import workloads
    return workloads.make_workload(batch=a.batch, q_heads=Q_HEADS, kv_heads=KV_HEADS,
                                   head_dim=HEAD_DIM, block_size=a.block_size, ctx_tokens=a.ctx,
                                   hot_frac=a.hot_frac, warm_frac=getattr(a, "warm_frac", None),
                                   seed=seed, device=device)


def time_device(wl, steps, warmup, dist_on):
    """Device time of `steps` decode calls (events on the launching stream)."""
    from paged_tierkv_b200 import workloads
    stream = torch.cuda.current_stream()
    out = torch.empty(wl.query.shape, dtype=torch.float16, device=wl.query.device)
    for _ in range(warmup):
        workloads.decode(wl, out=out)
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    total0 = torch.cuda.Event(enable_timing=True)
    total1 = torch.cuda.Event(enable_timing=True)
    if dist_on:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    total0.record(stream)
    for i in range(steps):
        starts[i].record(stream)
        workloads.decode(wl, out=out)
        ends[i].record(stream)
    total1.record(stream)
    torch.cuda.synchronize()
    if dist_on:
        torch.distributed.barrier()
    total_ms = total0.elapsed_time(total1)
    per = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    return total_ms, per, out


def time_e2e(wl, steps, warmup):
    """Same metric through the public API with host buffers: every step's
    inputs (the query and the three block tables, packed back to back in
    pinned host memory) go host->device in one copy and its output comes back
    device->host, all inside the timed region.  The copies run on a second
    stream, double-buffered as a serving loop would run them: step i+1's
    inputs go up and step i-1's output comes down while step i computes;
    events order every buffer's reuse."""
    from paged_tierkv_b200 import ops
    dev = wl.query.device
    compute = torch.cuda.current_stream()
    copy = torch.cuda.Stream(device=dev)
    srcs = [wl.query, wl.block_table, wl.block_states, wl.block_lengths]
    sizes = [x.numel() * x.element_size() for x in srcs]
    offs = [0]
    for n in sizes:
        offs.append(offs[-1] + (n + 255) // 256 * 256)
    h_pack = torch.zeros(offs[-1], dtype=torch.uint8).pin_memory()
    for x, o, n in zip(srcs, offs, sizes):
        h_pack[o:o + n].view(x.dtype).view(x.shape).copy_(x.cpu())
    d_pack = [torch.empty(offs[-1], dtype=torch.uint8, device=dev) for _ in range(2)]
    views = [[d[o:o + n].view(x.dtype).view(x.shape) for x, o, n in zip(srcs, offs, sizes)]
             for d in d_pack]
    h_out = [torch.empty(wl.query.shape, dtype=torch.float16).pin_memory() for _ in range(2)]
    d_out = [torch.empty(wl.query.shape, dtype=torch.float16, device=dev) for _ in range(2)]

    def run(n):
        up = [torch.cuda.Event() for _ in range(n)]
        done = [torch.cuda.Event() for _ in range(n)]
        with torch.cuda.stream(copy):
            d_pack[0].copy_(h_pack, non_blocking=True)
            up[0].record(copy)
        for i in range(n):
            b = i % 2
            if i + 1 < n:
                with torch.cuda.stream(copy):
                    if i >= 1:
                        copy.wait_event(done[i - 1])  # buffer (i + 1) % 2 is free again
                    d_pack[1 - b].copy_(h_pack, non_blocking=True)
                    up[i + 1].record(copy)
            compute.wait_event(up[i])
            q, t, st, ln = views[b]
            ops.decode_attention(q, t, st, ln, wl.pools, wl.num_blocks, wl.groups, wl.scaling,
                                 out=d_out[b])
            done[i].record(compute)
            with torch.cuda.stream(copy):
                copy.wait_event(done[i])
                h_out[b].copy_(d_out[b], non_blocking=True)
        compute.wait_stream(copy)  # the last output is on the host

    run(max(2, warmup))
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(compute)
    copy.wait_event(e0)
    run(steps)
    e1.record(compute)
    torch.cuda.synchronize()
    h2d = h_pack.numel()
    d2h = h_out[0].numel() * h_out[0].element_size()
    return e0.elapsed_time(e1), h2d, d2h


def host_sample(wl, seqs):
    """Host copies of the pools/tables of the first `seqs` sequences (slots remapped)."""
    table = wl.block_table[:seqs].cpu().numpy()
    states = wl.block_states[:seqs].cpu().numpy()
    lengths = wl.block_lengths[:seqs].cpu().numpy()
    hot_ids = np.unique(table[states == 0])
    warm_ids = np.unique(table[states == 1])
    remap = table.copy()
    hmap = {int(s): i for i, s in enumerate(hot_ids)}
    wmap = {int(s): i for i, s in enumerate(warm_ids)}
    for idx in zip(*np.nonzero(states == 0)):
        remap[idx] = hmap[int(table[idx])]
    for idx in zip(*np.nonzero(states == 1)):
        remap[idx] = wmap[int(table[idx])]
    p = wl.pools
    hi = torch.from_numpy(hot_ids.astype(np.int64)).to(p.device)
    wi = torch.from_numpy(warm_ids.astype(np.int64)).to(p.device)
    g = lambda t, i: t.index_select(0, i).cpu().numpy()  # noqa: E731
    return dict(query=wl.query[:seqs].cpu().numpy(), table=remap, states=states, lengths=lengths,
                hot_k=g(p.hot_k, hi), hot_v=g(p.hot_v, hi), warm_k=g(p.warm_k, wi),
                warm_v=g(p.warm_v, wi), k_scale=g(p.k_scale, wi), k_zero=g(p.k_zero, wi),
                v_scale=g(p.v_scale, wi), v_zero=g(p.v_zero, wi))


def cpu_oracle_rate(s, seconds):
    """GB/s of the CPU restatement of the reference path on a bounded sample
    (``host_sample`` of the workload plus its byte count and geometry)."""
    from oracle import tierkv_oracle as orc
    bytes_per_call = s["bytes"]
    reps, t0 = 0, time.perf_counter()
    while True:
        orc.decode_attention(s["query"], s["table"], s["states"], s["lengths"], s["num_blocks"],
                             s["hot_k"], s["hot_v"], s["warm_k"], s["warm_v"], s["k_scale"],
                             s["k_zero"], s["v_scale"], s["v_zero"], s["groups"], s["scaling"],
                             dtype=np.float32)
        reps += 1
        el = time.perf_counter() - t0
        if el >= seconds and reps >= 2:
            break
    return bytes_per_call * reps / el / 1e9, el / reps, reps


def blas_threads() -> int:
    try:
        from threadpoolctl import threadpool_info
        return max((i.get("num_threads", 1) for i in threadpool_info()), default=1)
    except Exception:
        return os.cpu_count() or 1


# --------------------------------------------------------------------------- arms
def run_reference(a, rank, world):
    """The reference arm: the CPU restatement of the reference's PyTorch tiered
    path (tierkv_triton.py:708-820; the reference itself is Python, has no
    packaging and cannot travel to the GPU box), on the host cores.  Its
    inputs are built on the host (host_unit_sample); it imports nothing of
    this package and never touches a GPU."""
    if rank != 0:
        return
    from oracle import tierkv_oracle as orc
    # One step = one (sequence, kv head) unit over the full context (its G
    # query heads), 1/8 of a sequence, so that the default 2000 steps end in
    # about a minute; its bytes are the unit's share of the workload's.
    s = host_unit_sample(a, SEED)
    cfg = bench_config(a, world)
    bytes_per_step = cfg["bytes_per_step_per_gpu"] / a.batch / KV_HEADS

    def once():
        orc.decode_attention(s["query"], s["table"], s["states"], s["lengths"], s["num_blocks"],
                             s["hot_k"], s["hot_v"], s["warm_k"], s["warm_v"], s["k_scale"],
                             s["k_zero"], s["v_scale"], s["v_zero"], s["groups"], s["scaling"],
                             dtype=np.float32)
    for _ in range(a.warmup):
        once()
    t0 = time.perf_counter()
    for _ in range(a.steps):
        once()
    el = time.perf_counter() - t0
    gbs = bytes_per_step * a.steps / el / 1e9
    cores = blas_threads()
    sample = (f"1 (sequence, kv head) unit per step: {s['groups']} query heads over the full "
              f"{a.ctx}-token context of sequence 0 (its tier layout drawn with our arm's seed; "
              "N(0,1) K/V drawn on the host, WARM blocks quantized by the oracle's "
              "quantize_fp16_to_int8); GB/s = the unit's share of the step's bytes / time")
    line = {
        "metric": METRIC, "value": round(gbs, 3), "unit": "GB/s", "n_gpus": world,
        "steps": a.steps, "warmup": a.warmup, "ms_per_step": round(el / a.steps * 1e3, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp32",
        "data": "synthetic (seeded N(0,1) K/V/query)", "impl": "reference",
        "config": cfg,
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": cores, "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_ours(a, rank, world, dist_on, device):
    from paged_tierkv_b200 import _native, ops
    _native.load(build_if_missing=True)
    wl = build_workload(a, seed=1234 + rank, device=device)
    torch.cuda.synchronize()
    sampler = ClockSampler(torch.cuda.current_device()) if rank == 0 else None
    if sampler:
        sampler.start()
    total_ms, per, _ = time_device(wl, a.steps, a.warmup, dist_on)
    clocks = sampler.stop() if sampler else None
    e2e_ms, h2d, d2h = time_e2e(wl, a.steps, a.warmup)
    splits = ops.plan_splits(wl.pools, wl.batch, wl.query.shape[1], wl.groups, wl.num_blocks,
                             wl.num_blocks)
    t = torch.tensor([total_ms, e2e_ms], dtype=torch.float64, device=device)
    if dist_on:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    total_ms, e2e_ms = float(t[0]), float(t[1])
    bytes_step = wl.algorithmic_bytes()
    all_bytes = bytes_step * world * a.steps
    value = all_bytes / (total_ms * 1e-3) / 1e9
    e2e_val = all_bytes / (e2e_ms * 1e-3) / 1e9
    batch = wl.batch
    cpu_sample = None
    if rank == 0 and not a.no_cpu_baseline:
        cpu_sample = dict(host_sample(wl, 1), bytes=bytes_step / batch, num_blocks=wl.num_blocks,
                          groups=wl.groups, scaling=wl.scaling)
    del wl
    torch.cuda.empty_cache()
    extras = {}
    if not a.no_scaling_extras:
        # the two strong-scaling curves: fixed total work split over the ranks
        extras["c4"] = c4_object(a, rank, world, dist_on, device)
        extras["c3"] = c3_object(a, rank, world, dist_on, device)
    if world == 1 and not a.no_single_extras:
        # the other single-GPU measurements of the benchmark configurations
        extras["c1"] = c1_object(device)
        extras["c2"] = c2_object(device)
        extras["demote"] = demote_object(a, device)
    if (world == 1 and not a.no_single_extras) or a.sweep:
        extras["sweep"] = sweep_object(a, rank, dist_on, device)
    if rank != 0:
        return
    peak, peak_kind = hbm_peak()
    kernel_ms = statistics.mean(per)
    achieved = bytes_step / (kernel_ms * 1e-3) / 1e9
    cpu = None
    if cpu_sample is not None:
        gbs, sec_per, reps = cpu_oracle_rate(cpu_sample, a.cpu_seconds)
        cpu = {"value": round(gbs, 4), "unit": "GB/s", "cores": blas_threads(), "kind": "port",
               "sample": f"1 of {batch} sequences (8 kv heads, full context), {reps} reps, "
                         f"{sec_per:.2f} s each"}
    tr = ncu_traffic(workload_key(a))
    cfg = bench_config(a, world)
    if cfg["bytes_per_step_per_gpu"] != bytes_step:
        raise RuntimeError("host byte count disagrees with the workload's")
    line = {
        "metric": METRIC, "value": round(value, 1), "unit": "GB/s", "n_gpus": world,
        "steps": a.steps, "warmup": a.warmup, "ms_per_step": round(total_ms / a.steps, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp16",
        "data": "synthetic (seeded N(0,1) K/V/query; WARM blocks demoted on device)",
        "config": cfg,
        "splits": splits,
        "tokens_per_s": round(batch * world / (32 * total_ms / a.steps * 1e-3), 1),
        "tokens_per_s_note": "attention-only decode tokens/s for a 32-layer model (batch / (32 x step))",
        "e2e": {"value": round(e2e_val, 1), "unit": "GB/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h},
        "gpu_launches": a.steps,
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                     "traffic": tr,
                     "traffic_source": ("ncu dram__bytes_read.sum + dram__bytes_write.sum of one "
                                        "batch-4 launch of this mix, x 8 to batch 32 "
                                        "(profiles/decode_c5_h025_bs16.md)") if tr else None,
                     "kernel": "tkv::decode_kernel<128,16,R,f16>",
                     "kernel_ms": round(kernel_ms, 4)},
        "cpu_baseline": cpu,
        "clocks": clocks,
    }
    line.update(extras)
    print(json.dumps(line), flush=True)


def _timed_graph(step, steps, warmup, dist_on, device, graph=True, side=None, per_rank=False):
    """Device ms per call of `step`, captured once in a CUDA graph on a side
    stream (warm-up first, so nothing is allocated during capture) and
    replayed; max over ranks (with `per_rank`, also every rank's own time).
    Every rank makes the same collective calls."""
    side = side or torch.cuda.Stream(device=device)
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(max(1, warmup)):
            step()
    torch.cuda.synchronize()
    g = None
    if graph:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=side):
            step()
        torch.cuda.synchronize()
    run = g.replay if g is not None else step
    with torch.cuda.stream(side):
        for _ in range(warmup):
            run()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        if dist_on:
            torch.distributed.barrier()
        torch.cuda.synchronize()
        e0.record(side)
        for _ in range(steps):
            run()
        e1.record(side)
        torch.cuda.synchronize()
    if dist_on:
        torch.distributed.barrier()
    del g
    t = torch.tensor([e0.elapsed_time(e1) / steps], dtype=torch.float64, device=device)
    ranks = [float(t[0])]
    if dist_on:
        if per_rank:
            allt = torch.empty(torch.distributed.get_world_size(), dtype=torch.float64,
                               device=device)
            torch.distributed.all_gather_into_tensor(allt, t)
            ranks = allt.tolist()
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return (float(t[0]), ranks) if per_rank else float(t[0])


def c4_layers(a, rank, world, device, layers):
    """Configuration 4's per-rank shards: for each layer, the time-balanced
    contiguous block range of this rank, materialized as its own pools."""
    from paged_tierkv_b200 import workloads
    ctx, bs, d, hkv, hq = 131072, a.block_size, HEAD_DIM, KV_HEADS, Q_HEADS
    nb = ctx // bs
    n_hot, n_warm, _ = workloads.tier_counts(nb, 0.10, 0.60)
    out, total = [], 0
    for layer in range(layers):
        states = workloads.assign_tiers(1, nb, n_hot, n_warm, seed=5000 + layer)
        lengths = torch.full((1, nb), bs, dtype=torch.int32)
        s, e = workloads.balanced_block_ranges(states, world, bs, d)[rank]
        wl = workloads.materialize(states[:, s:e].contiguous(), lengths[:, s:e].contiguous(),
                                   q_heads=hq, kv_heads=hkv, head_dim=d, block_size=bs,
                                   seed=7000 + 97 * layer + rank, device=device)
        out.append(wl)
        total += wl.algorithmic_bytes()
    return out, total, (ctx, bs, nb, n_hot, n_warm)


def c4_parity(a, rank, world, device):
    """Layer-0 parity of the sharded decode against one rank: every rank
    builds the whole 131072-token layer from the same seed and decodes its
    time-balanced block range with the exchange (or, for one rank, the whole
    range); rank 0 also decodes the unsharded layer.  Returns the largest
    difference relative to the output's scale (rank 0), and whether any rank
    recorded a device error."""
    from paged_tierkv_b200 import ops, sharding, workloads
    bs, d = a.block_size, HEAD_DIM
    wl = workloads.make_workload(batch=1, q_heads=Q_HEADS, kv_heads=KV_HEADS, head_dim=d,
                                 block_size=bs, ctx_tokens=131072, hot_frac=0.10, warm_frac=0.60,
                                 seed=5000, device=device)
    s, e = workloads.balanced_block_ranges(wl.block_states.cpu(), world, bs, d)[rank]
    ex = None
    if world > 1:
        ex = sharding.PeerExchange(rows_cap=Q_HEADS, units_cap=KV_HEADS, head_dim=d)
        res = sharding.P2PContextDecode(ex)(
            wl.query, wl.block_table[:, s:e], wl.block_states[:, s:e], wl.block_lengths[:, s:e],
            wl.pools, e - s, wl.groups, wl.scaling, out_dtype=torch.float32)
        out = res.out
    else:
        out, _, _ = workloads.decode(wl, out_dtype=torch.float32)
    torch.cuda.synchronize()
    err = ops.read_device_errors()
    if ex is not None:
        ex.close()
    rel = 0.0
    if rank == 0:
        full, _, _ = workloads.decode(wl, out_dtype=torch.float32, num_splits=1)
        torch.cuda.synchronize()
        rel = float((out - full).abs().max() / full.abs().max())
    t = torch.tensor([rel, float(err)], dtype=torch.float64, device=device)
    if world > 1:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    del wl
    torch.cuda.empty_cache()
    return float(t[0]), int(t[1])


def c4_measure(a, rank, world, dist_on, device, steps, warmup, exchanges):
    """Configuration 4 (batch 1, 131072 tokens, 32 layers, 10 % HOT / 60 % WARM
    / 30 % COLD; block-range sharded over the ranks): ms per 32-layer step,
    replayed from a CUDA graph, for the local shard decode alone and for each
    exchange variant ("p2p": partials exchanged over peer memory inside the
    decode launch; "nccl": all-gather of the packed (o, LSE) + merge launch)."""
    from paged_tierkv_b200 import ops, sharding, workloads
    layers, total_bytes, (ctx, bs, nb, n_hot, n_warm) = c4_layers(a, rank, world, device, a.layers)
    out16 = torch.empty((1, Q_HEADS, HEAD_DIM), dtype=torch.float16, device=device)
    out32 = torch.empty((1, Q_HEADS, HEAD_DIM), dtype=torch.float32, device=device)
    lse = torch.empty((1, Q_HEADS), dtype=torch.float32, device=device)

    def local():
        for wl in layers:
            workloads.decode(wl, out=out32 if world > 1 else out16,
                             out_dtype=torch.float32 if world > 1 else None,
                             return_lse=lse if world > 1 else False)

    local_ms, local_ranks = _timed_graph(local, steps, warmup, dist_on, device, not a.no_graph,
                                         per_rank=True)
    res = {"local_ms": local_ms, "local_ms_per_rank": local_ranks}
    for kind in (exchanges if world > 1 else ()):
        ex = None
        if kind == "p2p":
            ex = sharding.PeerExchange(rows_cap=Q_HEADS, units_cap=KV_HEADS, head_dim=HEAD_DIM,
                                       device_epoch=True)
            dec = sharding.P2PContextDecode(ex)
        else:
            dec = sharding.ContextShardedDecode()

        def step(dec=dec, ex=ex):
            for wl in layers:
                args = (wl.query, wl.block_table, wl.block_states, wl.block_lengths, wl.pools,
                        wl.num_blocks, wl.groups, wl.scaling)
                if ex is not None:
                    dec(*args, out=out16)
                else:
                    dec(*args)
        side = torch.cuda.Stream(device=device)
        ops.read_device_errors(stream=side)
        res[f"{kind}_ms"] = _timed_graph(step, steps, warmup, dist_on, device, not a.no_graph,
                                         side=side)
        torch.cuda.synchronize()
        res[f"{kind}_device_errors"] = ops.read_device_errors(stream=side)
        if ex is not None:
            ex.close()
    t = torch.tensor([float(total_bytes)], dtype=torch.float64, device=device)
    if dist_on:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.SUM)
    del layers
    torch.cuda.empty_cache()
    return res, float(t[0]), (ctx, bs, nb, n_hot, n_warm)


def c4_object(a, rank, world, dist_on, device, steps=50, warmup=5):
    """The configuration-4 strong-scaling entry of the headline line."""
    res, all_bytes, (ctx, bs, nb, n_hot, n_warm) = c4_measure(
        a, rank, world, dist_on, device, steps, warmup, ("p2p", "nccl"))
    rel, perr = c4_parity(a, rank, world, device)
    ms = res.get("p2p_ms", res["local_ms"])
    obj = {"workload": f"c4_ctx{ctx}_bs{bs}_l{a.layers}", "hot_blocks": n_hot, "warm_blocks": n_warm,
           "partition": "contiguous block ranges balanced by estimated decode time (WARM bytes x 1.19), one per rank",
           "ms_per_step": round(ms, 4), "tokens_per_s": round(1000.0 / ms, 2),
           "GBps_all_gpus": round(all_bytes / (ms * 1e-3) / 1e9, 1),
           "local_decode_ms_per_step": round(res["local_ms"], 4),
           "steps": steps, "cuda_graph": not a.no_graph,
           "parity_layer0_max_rel_vs_1_rank": rel, "parity_device_errors": perr}
    if world > 1:
        obj.update({
            "exchange": "p2p: epoch-tagged peer-memory stores inside the decode launch",
            "exchange_us_per_layer": round((res["p2p_ms"] - res["local_ms"]) * 1e3 / a.layers, 2),
            "local_decode_ms_per_step_per_rank": [round(x, 4) for x in res["local_ms_per_rank"]],
            "nccl_ms_per_step": round(res["nccl_ms"], 4),
            "nccl_tokens_per_s": round(1000.0 / res["nccl_ms"], 2),
            "nccl_us_per_layer_over_local": round((res["nccl_ms"] - res["local_ms"]) * 1e3 / a.layers, 2),
            "device_errors": res["p2p_device_errors"] | res["nccl_device_errors"]})
    return obj


def c3_object(a, rank, world, dist_on, device, steps=20, warmup=5, distinct_layers=4):
    """Configuration 3's attention at fixed total work: 64 sequences x 8192
    tokens, 20 % HOT / 60 % WARM / 20 % COLD, split data-parallel over the
    ranks (no collective); one step = 32 layer calls per rank (cycling through
    `distinct_layers` separately materialized layers, so repeated calls do
    not find their layer in L2), replayed from a CUDA graph; max over ranks."""
    from paged_tierkv_b200 import sharding, workloads
    sl = sharding.dp_slice(64, rank, world)
    n = sl.stop - sl.start
    wls = [workloads.make_workload(batch=n, q_heads=Q_HEADS, kv_heads=KV_HEADS, head_dim=HEAD_DIM,
                                   block_size=16, ctx_tokens=8192, hot_frac=0.2, warm_frac=0.6,
                                   seed=600 + 31 * rank + i, device=device)
           for i in range(distinct_layers)]
    outs = [torch.empty((n, Q_HEADS, HEAD_DIM), dtype=torch.float16, device=device) for _ in wls]

    def step():
        for layer in range(32):
            k = layer % len(wls)
            workloads.decode(wls[k], out=outs[k])
    ms = _timed_graph(step, steps, warmup, dist_on, device, not a.no_graph)
    per_rank_bytes = 32 * wls[0].algorithmic_bytes()
    del wls, outs
    torch.cuda.empty_cache()
    return {"workload": "c3_b64_ctx8192_h0.2_w0.6_bs16_l32", "sequences_total": 64,
            "sequences_per_gpu": n, "ms_per_step": round(ms, 4),
            "tokens_per_s": round(64 / (ms * 1e-3), 1),
            "GBps_per_gpu": round(per_rank_bytes / (ms * 1e-3) / 1e9, 1),
            "steps": steps, "scaling": "strong", "distinct_layers": distinct_layers,
            "cuda_graph": not a.no_graph,
            "note": "attention only: the model's projections, MLP and weights are outside this path"}


def _flush_l2(buf):
    buf.add_(1)  # a write larger than the 126 MB L2 evicts it


def c1_object(device, calls=200):
    """Configuration 1 (the parity op): 4 sequences x 2048 tokens, 32 q / 8 kv
    heads, head_dim 128, block 16, 32 HOT / 64 WARM / 32 COLD blocks per
    sequence.  us per call as eager Python calls through the public API and
    as CUDA-graph replays of the same calls (the inputs, 17 MB, stay L2
    resident, as they would for a model layer)."""
    from paged_tierkv_b200 import workloads
    wl = workloads.make_workload(batch=4, q_heads=Q_HEADS, kv_heads=KV_HEADS, head_dim=HEAD_DIM,
                                 block_size=16, ctx_tokens=2048, hot_frac=0.25, warm_frac=0.5,
                                 seed=1, device=device)
    out = torch.empty(wl.query.shape, dtype=torch.float16, device=device)
    for _ in range(10):
        workloads.decode(wl, out=out)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(calls):
        workloads.decode(wl, out=out)
    e1.record()
    torch.cuda.synchronize()
    eager_us = e0.elapsed_time(e1) * 1e3 / calls

    def many():
        for _ in range(100):
            workloads.decode(wl, out=out)
    graph_ms = _timed_graph(many, 5, 2, False, device)
    b = wl.algorithmic_bytes()
    return {"workload": "c1_b4_ctx2048_bs16_32h_64w_32c", "bytes_per_call": b,
            "us_per_call_eager": round(eager_us, 2), "us_per_call_graph": round(graph_ms * 10, 2),
            "GBps_graph": round(b / (graph_ms * 1e-2 * 1e-3) / 1e9, 1),
            "l2": "inputs (17 MB) L2-resident across calls"}


def c2_object(device, steps=20):
    """Configuration 2's attention (TinyLlama shape: 22 layers, 32 q / 4 kv
    heads, head_dim 64, block 16, 25 % HOT / 50 % WARM / 25 % COLD) at its mid-
    generation context, 8 sequences x 1152 tokens (1024-token prompt + 128 of
    the 256 generated): ms per 22-layer step, each layer a separately
    materialised pool set, replayed from a CUDA graph after an L2 flush (the
    whole model's KV, 105 MB, would otherwise stay in L2, which the model's
    2.2 GB of weights evict in a real step).  Attention only: the model's
    other work is outside this path."""
    from paged_tierkv_b200 import workloads
    wls = [workloads.make_workload(batch=8, q_heads=32, kv_heads=4, head_dim=64, block_size=16,
                                   ctx_tokens=1152, hot_frac=0.25, warm_frac=0.5, seed=200 + i,
                                   device=device) for i in range(22)]
    outs = [torch.empty(w.query.shape, dtype=torch.float16, device=device) for w in wls]

    def step():
        for w, o in zip(wls, outs):
            workloads.decode(w, out=o)
    side = torch.cuda.Stream(device=device)
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        step()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=side):
        step()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=device)
    pairs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
             for _ in range(steps)]
    with torch.cuda.stream(side):
        for _ in range(3):
            _flush_l2(flush)
            g.replay()
        for e0, e1 in pairs:
            _flush_l2(flush)
            e0.record(side)
            g.replay()
            e1.record(side)
    torch.cuda.synchronize()
    ms = statistics.mean(e0.elapsed_time(e1) for e0, e1 in pairs)
    b = sum(w.algorithmic_bytes() for w in wls)
    del g, wls, outs, flush
    torch.cuda.empty_cache()
    return {"workload": "c2_b8_ctx1152_h0.25_w0.5_bs16_l22_kv4_d64", "ms_per_step": round(ms, 4),
            "attention_tokens_per_s": round(8 / (ms * 1e-3), 1),
            "GBps": round(b / (ms * 1e-3) / 1e9, 1), "bytes_per_step": b,
            "l2": "flushed (256 MB write) before every timed step", "cuda_graph": True,
            "note": "attention only: model-level tokens/s needs the reference's model code, "
                    "which does not run on the GPU box"}


def sweep_object(a, rank, dist_on, device):
    """Configuration 5's sweep: hot fractions 1.0 / 0.5 / 0.25 / 0.1 (the rest
    split 2:1 WARM:COLD) at block 16 and 32; per point the mean event time of
    a decode launch and its GB/s against the measured copy peak."""
    peak, _ = hbm_peak()
    out = []
    for bs in (16, 32):
        for h in (1.0, 0.5, 0.25, 0.1):
            a2 = argparse.Namespace(**{**vars(a), "hot_frac": h, "block_size": bs})
            w2 = build_workload(a2, seed=99 + rank, device=device)
            _, pl, _ = time_device(w2, max(20, min(a.steps, 200)), max(3, a.warmup), dist_on)
            b2 = w2.algorithmic_bytes()
            gbs = b2 / (statistics.mean(pl) * 1e-3) / 1e9
            out.append({"block_size": bs, "hot_frac": h, "bytes_per_call": b2,
                        "ms_per_call": round(statistics.mean(pl), 4), "GBps": round(gbs, 1),
                        "frac": round(gbs / peak, 4)})
            del w2
            torch.cuda.empty_cache()
    return out


def demote_object(a, device):
    """Configuration 5's demotion: 2^20 fp16 [16 x 128] N(0,1) tiles (65536
    blocks x 8 kv heads x K/V) quantized bit-exactly into the WARM pool in one
    launch, and promoted back; ms and GB/s against the measured copy peak."""
    a2 = argparse.Namespace(**{**vars(a), "demote_blocks": 65536})
    return _demote_measure(a2, 0, False, device)[0]


def run_c4(a, rank, world, dist_on, device):
    """`--config c4`: configuration 4 as its own line (strong scaling)."""
    from paged_tierkv_b200 import _native
    _native.load(build_if_missing=True)
    kinds = (a.exchange,)
    res, all_bytes, (ctx, bs, nb, n_hot, n_warm) = c4_measure(
        a, rank, world, dist_on, device, a.steps, a.warmup, kinds)
    ms = res.get(f"{a.exchange}_ms", res["local_ms"])
    if rank != 0:
        return
    line = {
        "metric": "tiered decode tokens/s (C4: 131072-token context, 32 layers, block-range sharded)",
        "value": round(1000.0 / ms, 2), "unit": "tokens/s", "n_gpus": world, "steps": a.steps,
        "warmup": a.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "fp16", "data": "synthetic",
        "config": {"workload": f"c4_ctx{ctx}_bs{bs}_l{a.layers}", "hot_blocks": n_hot,
                   "warm_blocks": n_warm, "partition": "contiguous block ranges balanced by estimated decode time",
                   "exchange": ("none" if world == 1 else
                                "epoch-tagged peer-memory stores inside the decode launch"
                                if a.exchange == "p2p" else
                                "NCCL all_gather of packed (o, lse) per layer"),
                   "cuda_graph": not a.no_graph},
        "local_decode_ms_per_step": round(res["local_ms"], 4),
        "local_decode_ms_per_step_per_rank": [round(x, 4) for x in res["local_ms_per_rank"]],
        "GBps_all_gpus": round(all_bytes / (ms * 1e-3) / 1e9, 1),
        "gpu_launches": a.steps * a.layers * (1 if (world == 1 or a.exchange == "p2p") else 2),
    }
    print(json.dumps(line), flush=True)


def _demote_measure(a, rank, dist_on, device):
    """Demotion of a.demote_blocks blocks x 8 kv heads x K/V tiles of [16 x 128]
    fp16 N(0,1) in one launch, then promotion back: mean event ms per launch."""
    from paged_tierkv_b200 import ops
    blocks, hkv, bs, d = a.demote_blocks, 8, 16, 128
    pools = ops.TieredPools.allocate(blocks, blocks, hkv, bs, d, device)
    gen = torch.Generator(device=device).manual_seed(11 + rank)
    pools.hot_k.normal_(generator=gen)
    pools.hot_v.normal_(generator=gen)
    src = torch.arange(blocks, dtype=torch.int32, device=device)
    dst = torch.flip(src, dims=[0]).contiguous()
    lens = torch.full((blocks,), bs, dtype=torch.int32, device=device)
    tiles = blocks * hkv * 2
    # read fp16, write codes + scale + zero (promotion moves the same bytes back)
    bytes_per = tiles * bs * d * 2 + tiles * bs * d + tiles * bs * 2 * 2
    steps = max(1, min(a.steps, 50))

    def timed(fn):
        for _ in range(max(1, a.warmup)):
            fn()
        starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
        ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
        if dist_on:
            torch.distributed.barrier()
        torch.cuda.synchronize()
        for i in range(steps):
            starts[i].record()
            fn()
            ends[i].record()
        torch.cuda.synchronize()
        return statistics.mean(s.elapsed_time(e) for s, e in zip(starts, ends))

    ms = timed(lambda: ops.demote_blocks_to_warm(pools, src, dst, lens))
    ms_p = timed(lambda: ops.promote_blocks_to_hot(pools, dst, src, lens))
    x = pools.hot_k[:128].cpu().numpy() if rank == 0 else None
    del pools
    torch.cuda.empty_cache()
    peak, _ = hbm_peak()
    return {"workload": f"demote_{tiles}_tiles", "tiles": tiles, "bytes_per_launch": bytes_per,
            "steps": steps, "ms": round(ms, 4), "GBps": round(bytes_per / (ms * 1e-3) / 1e9, 1),
            "frac": round(bytes_per / (ms * 1e-3) / 1e9 / peak, 4),
            "promote_ms": round(ms_p, 4),
            "promote_GBps": round(bytes_per / (ms_p * 1e-3) / 1e9, 1),
            "promote_frac": round(bytes_per / (ms_p * 1e-3) / 1e9 / peak, 4)}, x


def run_demote(a, rank, world, dist_on, device):
    """Configuration 5's demotion benchmark: 2^20 tiles of [16 x 128] fp16 N(0,1)
    (one tile = one (block, kv head) K or V), i.e. 65536 blocks x 8 kv heads x
    {K, V}, quantized bit-exactly (Format R) into the WARM pool in one launch.
    Bytes per launch: 4 GiB read, 2 GiB codes + 64 MiB scale/zero written."""
    from paged_tierkv_b200 import _native
    _native.load(build_if_missing=True)
    sampler = ClockSampler(torch.cuda.current_device()) if rank == 0 else None
    if sampler:
        sampler.start()
    res, x = _demote_measure(a, rank, dist_on, device)
    clocks = sampler.stop() if sampler else None
    t = torch.tensor([res["ms"], res["promote_ms"]], dtype=torch.float64, device=device)
    if dist_on:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    ms, ms_p = float(t[0]), float(t[1])
    if rank != 0:
        return
    tiles, bytes_per = res["tiles"], res["bytes_per_launch"]
    cpu = None
    if world == 1 and not a.no_cpu_baseline:
        # the oracle's restatement of quantize_fp16_to_int8 on a 2048-tile slice
        from oracle import tierkv_oracle as orc
        tiles_s = x.shape[0] * 8 * 2
        reps, t0 = 0, time.perf_counter()
        while True:
            orc.quantize_rows_r(x)
            orc.quantize_rows_r(x)  # K and V
            reps += 1
            el = time.perf_counter() - t0
            if el >= a.cpu_seconds / 2 and reps >= 2:
                break
        cpu = {"value": round(tiles_s * reps * (bytes_per / tiles) / el / 1e9, 4), "unit": "GB/s",
               "cores": 1, "kind": "port",
               "sample": f"{tiles_s} tiles (128 blocks x 8 kv heads x K/V), numpy, repeated"}
    peak, kind = hbm_peak()
    gbs = bytes_per / (ms * 1e-3) / 1e9
    gbs_p = bytes_per / (ms_p * 1e-3) / 1e9
    print(json.dumps({
        "metric": f"HOT->WARM demotion GB/s ({tiles} fp16 [16 x 128] tiles, Format R)",
        "value": round(gbs * world, 1), "unit": "GB/s", "n_gpus": world, "steps": res["steps"],
        "warmup": a.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
        "scaling": "weak", "dtype": "fp16->u8", "data": "synthetic N(0,1)",
        "config": {"workload": f"demote_{tiles}_tiles", "tiles": tiles,
                   "bytes_per_launch": bytes_per, "l2": "inputs larger than L2"},
        "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(gbs / peak, 4), "peak_kind": kind},
        "promote": {"value": round(gbs_p * world, 1), "unit": "GB/s", "ms_per_step": round(ms_p, 4),
                    "frac": round(gbs_p / peak, 4)},
        "clocks": clocks,
        "cpu_baseline": cpu,
        "gpu_launches": 2 * res["steps"],
    }), flush=True)


def _compact_pool_stand_in():
    """The test suite's stand-in for the reference's compact pool and block
    manager (tests/compact_pool.py): the reference's own classes are not
    installed on the GPU box."""
    tests = os.path.join(ROOT, "tests")
    if tests not in sys.path:
        sys.path.insert(0, tests)
    import compact_pool
    return compact_pool


def _tiering_layer(device, blocks=2048, n_hot=512, n_warm=1024, seed=17):
    """One layer of configuration 5's sequence shape in a CompactPool: 2048
    blocks appended through the fused append, then tiered by one tick into
    512 HOT (sink + recent) / 1024 WARM / 512 COLD."""
    import types
    from paged_tierkv_b200 import tiering
    compact_pool = _compact_pool_stand_in()
    bs, hkv, d = 16, 8, 128
    pool = compact_pool.CompactPool(num_layers=1, block_size=bs, kv_heads=hkv, head_dim=d,
                                    max_blocks_per_layer=blocks + 64, max_hot_slots=blocks + 64,
                                    max_warm_slots=blocks + 64, device=device)
    rt = types.SimpleNamespace(layer_states={0: compact_pool.LayerState()},
                               block_manager=compact_pool.BlockAllocator(blocks + 64),
                               kv_pool=pool, block_size=bs, max_blocks_per_layer=blocks + 64)
    gen = torch.Generator(device=device).manual_seed(seed)
    k = torch.randn((1, hkv, blocks * bs, d), generator=gen, device=device).to(torch.float16)
    v = torch.randn((1, hkv, blocks * bs, d), generator=gen, device=device).to(torch.float16)
    tiering.append_to_layer(rt, 0, k, v)
    rng = np.random.default_rng(seed)
    states = np.full(blocks, tiering.COLD_STATE, np.int32)
    states[0] = tiering.HOT_STATE
    states[blocks - (n_hot - 1):] = tiering.HOT_STATE
    mid = rng.permutation(np.arange(1, blocks - (n_hot - 1)))
    states[mid[:n_warm]] = tiering.WARM_STATE
    physical = list(range(blocks))
    tiering.apply_sync(pool, tiering.plan_sync(pool, 0, physical, states.tolist()))
    torch.cuda.synchronize()
    return rt, pool, physical, states


def run_tiering(a, rank, world, dist_on, device):
    """The survey's "next" rows measured on one layer of configuration 5's
    shape (2048 blocks x 8 kv heads x [16 x 128]):
      tick   -- sync_storage_states after the policy swaps 64 HOT and 64 WARM
                blocks (128 data moves), batched (one demotion + one promotion
                launch + staging + one table write) against the same moves done
                the reference's way, one launch per move and one element write
                per table cell;
      append -- one decode token appended to the open block, fused (one launch)
                against the reference's per-op sequence (two row copies, two
                tail fills, three table-element writes)."""
    from paged_tierkv_b200 import _native, ops, tiering
    _native.load(build_if_missing=True)
    rt, pool, physical, states = _tiering_layer(device)
    steps = max(3, min(a.steps, 200))
    warm = max(1, a.warmup)
    if a.config == "tick":
        rng = np.random.default_rng(5)
        warm_ids = rng.choice(np.nonzero(states == tiering.WARM_STATE)[0], 64, replace=False)
        recent = np.arange(len(states) - 511, len(states))
        hot_pick = rng.choice(recent[:-1], 64, replace=False)
        a_states = states.copy()
        b_states = states.copy()
        b_states[warm_ids] = tiering.HOT_STATE
        b_states[hot_pick] = tiering.WARM_STATE
        flip = [b_states, a_states]

        def batched(target):
            plan = tiering.plan_sync(pool, 0, physical, target.tolist())
            return tiering.apply_sync(pool, plan)

        def per_block(target):
            plan = tiering.plan_sync(pool, 0, physical, target.tolist())
            pools = tiering._pools(pool)
            for h, w, n in plan.demotions:
                ops.demote_blocks_to_warm(pools, [h], [w], [n])
            for w, h, n in plan.promotions:
                ops.promote_blocks_to_hot(pools, [w], [h], [n])
            for table, cells in tiering._table_groups(pool, plan):
                for (layer, logical), val in cells.items():
                    table[layer, logical] = val
            return plan

        def timed(fn):
            for i in range(warm * 2):
                fn(flip[i % 2])
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            t0 = time.perf_counter()
            e0.record()
            for i in range(steps * 2):
                fn(flip[i % 2])
            e1.record()
            torch.cuda.synchronize()
            return (time.perf_counter() - t0) * 1e3 / (steps * 2), e0.elapsed_time(e1) / (steps * 2)

        stats = batched(flip[0])
        batched(flip[1])
        wall, dev = timed(batched)
        wall_pb, dev_pb = timed(per_block)
        moves = stats["demotions"] + stats["promotions"]
        tile_bytes = 8 * 16 * 128 * 2 * 2 + 8 * 16 * 128 * 2 + 8 * 16 * 8
        line = {
            "metric": "policy tick ms (storage sync of one 2048-block layer, 64 HOT<->64 WARM swaps)",
            "value": round(wall, 3), "unit": "ms", "n_gpus": 1, "steps": steps * 2, "warmup": warm * 2,
            "ms_per_step": round(wall, 3), "higher_is_better": False, "scaling": "none",
            "dtype": "fp16<->u8", "data": "synthetic N(0,1)",
            "config": {"workload": "tick_2048_blocks_128_moves", "moves": moves,
                       "staged_moves": stats["staged_demotions"] + stats["staged_promotions"],
                       "bytes_moved": moves * tile_bytes},
            "device_ms": round(dev, 3),
            "per_block": {"ms": round(wall_pb, 3), "device_ms": round(dev_pb, 3),
                          "what": "same plan, one kernel launch per move, one element write "
                                  "per table cell (the reference's launch pattern)"},
            "gpu_launches": steps * 2 * (2 + int(stats["staged_demotions"] > 0)
                                         + int(stats["staged_promotions"] > 0)),
        }
        print(json.dumps(line), flush=True)
        return
    # append: one token per step into the open block of the layer
    hkv, d = pool.kv_heads, pool.head_dim
    gen = torch.Generator(device=device).manual_seed(3)
    toks = torch.randn((steps * 2 + warm * 4, 1, hkv, 1, d), generator=gen, device=device).to(torch.float16)
    cur = [0]

    def fused():
        t = toks[cur[0]]
        cur[0] += 1
        tiering.append_to_layer(rt, 0, t, t)

    def per_op():
        t = toks[cur[0]]
        cur[0] += 1
        steps_, _ = tiering.plan_append(rt, 0, t, t)
        for st in steps_:
            n = int(st.key.shape[-2])
            pool.hot_k_pool[st.slot, :, st.start:st.start + n, :].copy_(st.key[0])
            pool.hot_v_pool[st.slot, :, st.start:st.start + n, :].copy_(st.value[0])
            if st.start + n < pool.block_size:
                pool.hot_k_pool[st.slot, :, st.start + n:, :].zero_()
                pool.hot_v_pool[st.slot, :, st.start + n:, :].zero_()
            for table, cells in tiering._table_groups(pool, st.plan):
                for (layer, logical), val in cells.items():
                    table[layer, logical] = val

    def timed(fn, n):
        for _ in range(warm * 2):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0 = time.perf_counter()
        e0.record()
        for _ in range(n):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return (time.perf_counter() - t0) * 1e6 / n, e0.elapsed_time(e1) * 1e3 / n

    us, dev_us = timed(fused, steps)
    us_po, dev_po = timed(per_op, steps)
    line = {
        "metric": "decode KV append us per token (one layer, 8 kv heads x 128, block 16)",
        "value": round(us, 2), "unit": "us", "n_gpus": 1, "steps": steps, "warmup": warm * 2,
        "ms_per_step": round(us / 1e3, 5), "higher_is_better": False, "scaling": "none",
        "dtype": "fp16", "data": "synthetic N(0,1)",
        "config": {"workload": "append_1_token", "blocks": len(physical)},
        "device_us": round(dev_us, 2),
        "per_op": {"us": round(us_po, 2), "device_us": round(dev_po, 2),
                   "what": "same bookkeeping, then the reference's per-op sequence: two row copies, "
                           "two tail fills, one element write per table cell"},
        "gpu_launches": steps,
    }
    print(json.dumps(line), flush=True)


def _torch_quantize_r(x):
    """quantize_fp16_to_int8 (tierkv_policy.py:21-36) as the reference runs it:
    one fp16 torch op per step."""
    mn = x.amin(dim=-1, keepdim=True)
    mx = x.amax(dim=-1, keepdim=True)
    scale = (mx - mn) / 255.0
    scale = torch.where(scale == 0, torch.ones_like(scale), scale)
    zp = -torch.round(mn / scale)
    q = torch.clamp(torch.round(x / scale) + zp, 0, 255).to(torch.uint8)
    return q, scale, zp


def run_prefill_store(a, rank, device):
    """The storage half of a prefill with policy (append_prefill_with_policy,
    tierkv_policy.py:1722-1766) for one layer of an 8192-token prompt (512
    blocks of [16 x 128] x 8 kv heads; 25 % HOT, 50 % WARM, 25 % COLD by
    seeded scores): ours (bookkeeping replay, one store launch, one table
    copy) against the same bookkeeping followed by the reference's per-block
    tensor work (row copies and tail fills for HOT blocks, the torch
    quantizer's ops for WARM blocks, one element write per table cell)."""
    import types
    from paged_tierkv_b200 import _native, ops, tiering
    compact_pool = _compact_pool_stand_in()
    _native.load(build_if_missing=True)
    if rank != 0:
        return
    bs, hkv, d, tokens = 16, 8, 128, 8192
    nb = tokens // bs
    steps = max(3, min(a.steps, 20))
    warm = max(2, a.warmup)
    layers = 2 * (steps + warm) + 2
    pool = compact_pool.CompactPool(num_layers=layers, block_size=bs, kv_heads=hkv, head_dim=d,
                                    max_blocks_per_layer=nb, max_hot_slots=layers * nb,
                                    max_warm_slots=layers * nb, hot_chunk_slots=layers * nb,
                                    warm_chunk_slots=layers * nb, device=device)
    rt = types.SimpleNamespace(layer_states={i: compact_pool.LayerState() for i in range(layers)},
                               block_manager=compact_pool.BlockAllocator(layers * nb), kv_pool=pool,
                               block_size=bs, max_blocks_per_layer=nb)
    gen = torch.Generator(device=device).manual_seed(29)
    k = torch.randn((1, hkv, tokens, d), generator=gen, device=device).to(torch.float16)
    v = torch.randn((1, hkv, tokens, d), generator=gen, device=device).to(torch.float16)
    scores = torch.rand(nb, generator=torch.Generator().manual_seed(29))
    order = sorted(range(1, nb - 1), key=lambda i: float(scores[i]), reverse=True)
    desired = [2] * nb
    for i in [0, nb - 1] + order[:nb // 4 - 2]:
        desired[i] = 0
    for i in order[nb // 4 - 2:nb // 4 - 2 + nb // 2]:
        desired[i] = 1
    rt._desired_prefill_states = lambda n, sc: list(desired)
    layer = [0]

    def ours():
        tiering.append_prefill_with_policy(rt, layer[0], k, v, scores)
        layer[0] += 1

    def per_block():
        pp = tiering.plan_prefill(rt, layer[0], k, v, scores)
        layer[0] += 1
        key, val = pp.key, pp.value
        for state, slot, first, n in pp.entries:
            if state == 0:
                for src, dst in ((key, pool.hot_k_pool), (val, pool.hot_v_pool)):
                    dst[slot, :, :n, :].copy_(src[:, first:first + n, :])
                    if n < bs:
                        dst[slot, :, n:, :].zero_()
            else:
                for src, dst, sc, zp in ((key, pool.warm_k_pool, pool.k_scale, pool.k_zero),
                                         (val, pool.warm_v_pool, pool.v_scale, pool.v_zero)):
                    q, s_, z_ = _torch_quantize_r(src[:, first:first + n, :].contiguous())
                    dst[slot, :, :n, :].copy_(q)
                    sc[slot, :, :n, :].copy_(s_)
                    zp[slot, :, :n, :].copy_(z_)
        for table, cells in tiering._table_groups(pool, pp.plan):
            for (lay, logical), val_ in cells.items():
                table[lay, logical] = val_

    def timed(fn):
        for _ in range(warm):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0 = time.perf_counter()
        e0.record()
        for _ in range(steps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return (time.perf_counter() - t0) * 1e3 / steps, e0.elapsed_time(e1) / steps

    ms, dev_ms = timed(ours)
    # the store kernel alone: the last layer's entries stored again (same bytes)
    import ctypes
    from paged_tierkv_b200 import _native as N
    ents = torch.tensor(_last_entries(pool, layer[0] - 1, bs), dtype=torch.int32, device=device)
    ps = tiering._pools_struct(pool)
    kc, vc = k[0].contiguous(), v[0].contiguous()
    lib = N.load()

    def store():
        N.check(lib.tkv_store_prefill_blocks(ctypes.byref(ps), kc.data_ptr(), vc.data_ptr(), tokens,
                                              ents.data_ptr(), int(ents.shape[0]), ops._stream(None)),
                "tkv_store_prefill_blocks")

    for _ in range(5):
        store()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(50):
        store()
    e1.record()
    torch.cuda.synchronize()
    warm_ms = e0.elapsed_time(e1) / 50  # inputs L2-resident, as right after their projection
    # the HBM roofline: every launch after a 256 MB write that evicts L2
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=device)
    pairs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
             for _ in range(30)]
    for a0, a1 in pairs:
        flush.zero_()
        a0.record()
        store()
        a1.record()
    torch.cuda.synchronize()
    kernel_ms = sum(a0.elapsed_time(a1) for a0, a1 in pairs) / len(pairs)
    del flush
    ms_pb, dev_pb = timed(per_block)
    n_hot = desired.count(0)
    n_warm = desired.count(1)
    hbm_peak = None
    try:
        with open(PEAKS) as f:
            hbm_peak = float(json.load(f)["hbm_gbs"])
    except Exception:
        pass
    alg = 2 * hkv * d * 2 * tokens * (n_hot + n_warm) / nb + n_hot * 2 * hkv * bs * d * 2 \
        + n_warm * 2 * hkv * bs * (d + 4)
    line = {
        "metric": "prefill storage ms per layer (append_prefill_with_policy, 8192 tokens, "
                  "8 kv heads x 128, block 16)",
        "value": round(ms, 3), "unit": "ms", "n_gpus": 1, "steps": steps, "warmup": warm,
        "ms_per_step": round(ms, 3), "higher_is_better": False, "scaling": "none",
        "dtype": "fp16 -> fp16 / u8", "data": "synthetic N(0,1)",
        "config": {"workload": "prefill_store_8192", "blocks": nb, "hot": n_hot, "warm": n_warm,
                   "cold": nb - n_hot - n_warm, "algorithmic_bytes": int(alg)},
        "device_ms": round(dev_ms, 4),
        "roofline": {"bound": "hbm", "achieved": round(alg / (kernel_ms * 1e-3) / 1e9, 1),
                     "peak": hbm_peak, "unit": "GB/s",
                     "frac": round(alg / (kernel_ms * 1e-3) / 1e9 / hbm_peak, 4) if hbm_peak else None,
                     "kernel": "tkv::store_prefill_kernel<128>", "kernel_ms": round(kernel_ms, 4),
                     "traffic": None, "l2": "flushed before every timed launch",
                     "kernel_ms_l2_warm_inputs": round(warm_ms, 4)},
        "per_block": {"ms": round(ms_pb, 3), "device_ms": round(dev_pb, 3),
                      "what": "same bookkeeping, then the reference's per-block tensor work "
                              "(row copies, tail fills, torch quantizer ops, one element write "
                              "per table cell)"},
        "gpu_launches": steps,
    }
    print(json.dumps(line), flush=True)


def _last_entries(pool, layer, bs):
    """(state, slot, first token, length) of a stored layer's HOT / WARM blocks."""
    st = pool.block_states[layer].tolist()
    sl = pool.block_slot_indices[layer].tolist()
    ln = pool.block_lengths[layer].tolist()
    return [(s, q, i * bs, n) for i, (s, q, n) in enumerate(zip(st, sl, ln)) if s in (0, 1)]


def run_prefill(a, rank, device):
    """Exact prefill block scores of one layer of configuration 3's prompt
    (8192 tokens, 32 q / 8 kv heads, head_dim 128, block 16, causal):
    ours with the LSE pass, ours given the LSE of torch's flash SDPA (what a
    flash prefill returns), and the reference's way on the same GPU (eager
    weights materialised by torch: QK^T, fp32 softmax, fp16 cast, means)."""
    from paged_tierkv_b200 import _native, ops
    _native.load(build_if_missing=True)
    if rank != 0:
        return
    b, hq, hkv, t, d, bs = 1, 32, 8, 8192, 128, 16
    gen = torch.Generator(device=device).manual_seed(21)
    q = torch.randn((b, hq, t, d), generator=gen, device=device).to(torch.float16)
    k = torch.randn((b, hkv, t, d), generator=gen, device=device).to(torch.float16)
    v = torch.randn((b, hkv, t, d), generator=gen, device=device).to(torch.float16)
    scaling = d ** -0.5
    g = hq // hkv
    kr, vr = k.repeat_interleave(g, dim=1), v.repeat_interleave(g, dim=1)
    _, lse_flash = torch.ops.aten._scaled_dot_product_flash_attention(q, kr, vr, 0.0, True, False,
                                                                      scale=scaling)[:2]
    steps = max(3, min(a.steps, 20))

    def timed(fn):
        for _ in range(max(2, a.warmup)):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / steps

    def eager(cast=torch.float16):
        w = torch.matmul(q, kr.transpose(2, 3)) * scaling
        w = w + torch.full((t, t), float("-inf"), device=device).triu(1)
        w = torch.softmax(w, dim=-1, dtype=torch.float32).to(cast)
        tok = w.mean(dim=(0, 1, 2), dtype=torch.float32)
        return torch.stack([c.mean() for c in torch.split(tok, bs)])

    ms_full = timed(lambda: ops.prefill_block_scores(q, k, scaling, bs))
    ms_cols = timed(lambda: ops.prefill_block_scores(q, k, scaling, bs, lse=lse_flash))
    ms_eager = timed(eager)
    ours = ops.prefill_block_scores(q, k, scaling, bs)
    ref32 = eager(torch.float32)  # without the reference's fp16 rounding of the weights
    rel = float(((ours - ref32).abs() / ref32.abs().clamp_min(1e-12)).max())
    flops_pass = 2.0 * d * (t * (t + 1) / 2) * hq  # one causal Q K^T
    peak = None
    try:
        with open(PEAKS) as f:
            peak = float(json.load(f)["bf16_tflops"])
    except Exception:
        pass
    ach = 2 * flops_pass / (ms_full * 1e-3) / 1e12
    # exp2 evaluations the two passes make: every logit of every 128 x 128
    # (query tile, key tile) pair that the causal mask does not skip whole
    nt = (t + 127) // 128
    tiles = hq * nt * (nt + 1) // 2
    exps = 2 * tiles * 128 * 128
    exp_peak = 16 * 148 * 1.965e9  # MUFU: 16 exp2 per SM clock, 148 SMs, max SM clock
    line = {
        "metric": "prefill block-score ms (one 8192-token layer, 32 q / 8 kv heads, D 128, causal)",
        "value": round(ms_full, 3), "unit": "ms", "n_gpus": 1, "steps": steps, "warmup": a.warmup,
        "ms_per_step": round(ms_full, 3), "higher_is_better": False, "scaling": "none",
        "dtype": "fp16 mma, fp32 accumulate", "data": "synthetic N(0,1)",
        "config": {"workload": "prefill_scores_t8192", "block_size": bs,
                   "l2": "q and k (80 MB) stay L2-resident across steps, as after their "
                         "projection; the passes are exp2-bound (DRAM 2-3 % busy)"},
        "given_flash_lse_ms": round(ms_cols, 3),
        "torch_eager_weights_ms": round(ms_eager, 3),
        "max_rel_diff_vs_fp32_eager": rel,
        "roofline": {"bound": "tensor", "achieved": round(ach, 1), "peak": peak, "unit": "TFLOP/s",
                     "frac": round(ach / peak, 4) if peak else None,
                     "note": "tcgen05 UMMA; two causal Q K^T passes; the binding unit is the "
                             "exp2 unit (exp_roofline)"},
        "exp_roofline": {"exps": exps, "achieved": round(exps / (ms_full * 1e-3) / 1e12, 3),
                         "peak": round(exp_peak / 1e12, 3), "unit": "Texp2/s",
                         "frac": round(exps / (ms_full * 1e-3) / exp_peak, 4),
                         "note": "peak = 16 MUFU exp2 per SM clock x 148 SMs at the 1965 MHz "
                                 "max clock (nominal); 1/8 of the LSE pass's and 1/16 of the column "
                                 "pass's exps run on the FMA pipe instead"},
        "gpu_launches": steps * 3,
    }
    print(json.dumps(line), flush=True)


def main():
    a = parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dist_on = world > 1 and a.impl == "ours"
    if a.impl == "reference" and rank != 0:
        return  # the reference arm runs on rank 0's host cores only
    if dist_on:
        import datetime
        torch.cuda.set_device(local)
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=torch.device("cuda", local))
    device = torch.device("cuda", local)
    a.gpus = world
    try:
        if a.impl == "reference":
            run_reference(a, rank, world)
        elif a.config == "c4":
            run_c4(a, rank, world, dist_on, device)
        elif a.config == "demote":
            run_demote(a, rank, world, dist_on, device)
        elif a.config in ("tick", "append"):
            run_tiering(a, rank, world, dist_on, device)
        elif a.config == "prefill":
            run_prefill(a, rank, device)
        elif a.config == "prefill_store":
            run_prefill_store(a, rank, device)
        else:
            run_ours(a, rank, world, dist_on, device)
    finally:
        if dist_on:
            torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
