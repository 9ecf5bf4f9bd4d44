"""Benchmark of the paged KV hot path on B200: BASELINE config 2 (Llama-3.1-8B decode-attention shape).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config 2|3|4|5]
    torchrun --nproc-per-node N bench.py --gpus N ...      (KV-head sharding, NCCL all-gather)

Several GPUs (config 2): rank r of N owns KV heads [8r/N, 8(r+1)/N) of every sequence.  By default the
batch is 64 x N sequences (weak scaling: each rank reads one GPU's worth of KV bytes, as serving with N
GPUs runs N times the batch); --scaling strong keeps batch 64 and splits its heads.

The default (config 2) is the headline line.  At N=1 it also carries `configs` (4, 5:
the mixed continuous-batching step, the prefix-sharing step with copy-on-write, the long-context eviction
step with compaction, each described in its builder below), `flashinfer_decode` (the reference's CUDA
backend timed on the same pages) and `e2e_reference_metadata` (the end-to-end loop handing the backend an
object with only the reference's AttentionMetadata fields).  At N>1 it carries `strong`: KV-head sharding
of a fixed workload (config 2 at batch 64 and config 5) with each rank's attention time and the per-layer
gather + barrier time.  Every sub-object ends with a spot check of sampled rows against a plain torch fp32
attention over the same pages.  --config 3/4/5 print a line of their own for one workload.

Workload (config 2): bf16, 32 query heads, 8 KV heads, head_dim 128, block_size 16, batch 64, context
lengths U[512, 4096] (seeded), block tables a seeded shuffle of a pool sized 1.25x the blocks needed,
K/V ~ 0.5 N(0,1), Q ~ N(0,1).  One STEP = one decode step of all 32 layers: per layer, append one token
per sequence (K1) and run paged attention over the context (K2a + K2b), each layer on its own pool
(32 x 740 MB: every layer's reads are far larger than the 126 MB L2, so no flush is needed).
Synthetic data (no checkpoint or dataset): the kernels' cost depends only on shapes and lengths.

Metric: KV-read GB/s = algorithmic K+V bytes the attention must read (sum of contexts x 2 x Hkv x Dh x 2 B,
every layer) / step time, summed over ranks (value), with seqs/s and append GB/s alongside.  The
`reference` arm times the reference's CPU algorithm (the oracle port of paged_torch_ref.py) on the
host cores with the same metric.
"""

from __future__ import annotations

import argparse
import importlib
import json
import math
import os
import re
import statistics
import subprocess
import sys
import time
import types
from datetime import timedelta
from pathlib import Path

from dataclasses import dataclass, field

import numpy as np
import torch

REPO = Path(__file__).resolve().parent
PACKAGE = "mini-llm-inference-server_b200"
H, HKV, DH, BS = 32, 8, 128, 16
FALLBACK_HBM_GBS = 6650.0


# ----------------------------------------------------------------------------- workload


@dataclass
class Workload:
    """One benchmark step: rows whose k/v are appended, rows that attend, and block copies run first."""

    name: str
    describe: str
    append_rows: list  # (num_cached, num_new, block_ids)
    attend_rows: list  # (num_cached, num_new, block_ids): the rows that attend (decode or multi-token)
    num_blocks: int
    copy_src: list = field(default_factory=list)
    copy_dst: list = field(default_factory=list)
    kv_scale: float = 1.0
    layers: int = 32
    info: dict = field(default_factory=dict)

    @property
    def attend_ctx(self) -> np.ndarray:
        return np.array([c + n for c, n, _ in self.attend_rows], dtype=np.int64)

    def unique_pages(self) -> int:
        """Distinct pool blocks the attention reads (shared prefixes count once)."""
        return len({b for c, n, blk in self.attend_rows for b in blk[:-(-(c + n) // BS)]})


def _take(perm: np.ndarray, counts) -> list[list[int]]:
    offs = np.concatenate([[0], np.cumsum(counts)])
    return [perm[offs[i]:offs[i + 1]].tolist() for i in range(len(counts))]


def config2(batch: int = 64, seed: int = 1234) -> Workload:
    """batch 64, context U[512, 4096] after the append, pool 1.25x the blocks needed,
    tables a seeded shuffle, K/V 0.5 N(0,1); one decode token per sequence, 32 layer pools."""
    r = np.random.default_rng(seed)
    ctx = r.integers(512, 4097, size=batch).astype(np.int64)
    pages = -(-ctx // BS)
    nb = int(math.ceil(1.25 * int(pages.sum())))
    blocks = _take(r.permutation(nb), pages)
    rows = [(int(c) - 1, 1, b) for c, b in zip(ctx, blocks)]
    return Workload("config 2", f"Llama-3.1-8B decode attention (H32/Hkv8/Dh128, bs16), batch {batch}, "
                    "ctx U[512,4096], 32 layer pools, append 1 token/seq + paged attention", rows, rows, nb,
                    kv_scale=0.5)


def config3(seed: int = 33, attend_chunks: bool = False) -> Workload:
    """256 decode rows with context lognormal(median 1024, sigma 1) capped at 32768, and a
    varlen append of 8 prefill chunks of U[1, 2048] tokens.  Blocks come from a seeded random permutation of a
    pool 1.25x the need, so every table is scattered (a fragmented pool).  In BASELINE the chunks only append;
    with attend_chunks (--attend-chunks) they also attend causally over themselves, as an engine's chunked
    prefill does (multi-token rows, paged_torch_ref.py:61-73)."""
    r = np.random.default_rng(seed)
    ctx = np.clip(np.rint(1024.0 * np.exp(r.standard_normal(256))), 1, 32768).astype(np.int64)
    chunks = r.integers(1, 2049, size=8).astype(np.int64)
    pages, cpages = -(-ctx // BS), -(-chunks // BS)
    nb = int(math.ceil(1.25 * int(pages.sum() + cpages.sum())))
    perm = r.permutation(nb)
    blocks = _take(perm, np.concatenate([pages, cpages]))
    decode = [(int(c) - 1, 1, b) for c, b in zip(ctx, blocks[:256])]
    prefill = [(0, int(n), b) for n, b in zip(chunks, blocks[256:])]
    if attend_chunks:
        return Workload("config 3", "mixed step: 256 decode rows ctx lognormal(1024, 1.0) <= 32768 + 8 prefill "
                        "chunks U[1,2048] appended AND attending causally, fragmented pool, 32 layer pools",
                        decode + prefill, decode + prefill, nb,
                        info={"chunk_tokens": int(chunks.sum()), "decode_ctx_sum": int(ctx.sum()),
                              "chunks_attend": True})
    return Workload("config 3", "mixed step: 256 decode rows ctx lognormal(1024, 1.0) <= 32768 + varlen append of "
                    "8 prefill chunks U[1,2048], fragmented pool, 32 layer pools", decode + prefill, decode, nb,
                    info={"chunk_tokens": int(chunks.sum()), "decode_ctx_sum": int(ctx.sum())})


CONFIG4_PREFIX = 8200  # 512 full blocks + 8 tokens: the shared prefix ends mid-block, so its last block is COW'd


def config4(seed: int = 44) -> Workload:
    """128 sequences share one prefix (identical block ids, refcount 128) and each has a
    unique suffix of U[64, 512] tokens.  8192 tokens would fill the shared blocks exactly, so the prefix here
    is 8200 tokens: its last block holds 8 tokens, and every step first copies that shared partial block into
    each sequence's private block (copy-on-write: 128 copies) before appending one token per sequence and
    attending over shared + private blocks."""
    r = np.random.default_rng(seed)
    b = 128
    suffix = r.integers(64, 513, size=b).astype(np.int64)
    ctx = CONFIG4_PREFIX + suffix  # context after the append
    full = CONFIG4_PREFIX // BS
    private = -(-ctx // BS) - full  # the first private block is the COW copy of the shared partial block
    nb = full + 1 + int(private.sum())
    perm = r.permutation(nb)
    shared, partial = perm[:full].tolist(), int(perm[full])
    own = _take(perm[full + 1:], private)
    rows = [(int(c) - 1, 1, shared + o) for c, o in zip(ctx, own)]
    return Workload("config 4", "prefix sharing: 128 seqs share an 8200-token prefix (refcount 128; its partial last "
                    "block is COW-copied to each seq every step) + suffix U[64,512]; append 1 token/seq + attention, "
                    "32 layer pools", rows, rows, nb, copy_src=[partial] * b, copy_dst=[o[0] for o in own],
                    info={"prefix_tokens": CONFIG4_PREFIX})


def config5(seed: int = 55) -> Workload:
    """32 sequences of 131072 tokens in a pool with 64 spare blocks.  Each step evicts a
    seeded 10% (3 sequences), compacts the pool by copying every live block above the live count into the
    freed blocks below it (BlockManager.compact, one block-copy launch), then runs split-K decode for the 29
    survivors over their rewritten tables.  One layer (its K+V pool is 17 GB at one GPU)."""
    r = np.random.default_rng(seed)
    b, ctx = 32, 131072
    pages = ctx // BS
    nb = b * pages + 64
    tables = _take(r.permutation(nb), [pages] * b)
    evict = set(r.choice(b, size=3, replace=False).tolist())
    live = [t for i, t in enumerate(tables) if i not in evict]
    # compaction plan, as the block manager makes it: live blocks at ids >= n_live move to the free ids below
    n_live = len(live) * pages
    used = np.zeros(nb, dtype=bool)
    for t in live:
        used[t] = True
    holes = np.nonzero(~used[:n_live])[0]
    movers = np.nonzero(used[n_live:])[0] + n_live
    remap = np.arange(nb)
    remap[movers] = holes
    live = [remap[t].tolist() for t in live]
    rows = [(ctx - 1, 1, t) for t in live]
    return Workload("config 5", "long context: 32 x 131072 tokens, evict 3 (10%), compact by block copy into the "
                    "freed blocks, split-K decode of the 29 survivors; 1 layer", rows, rows, nb,
                    copy_src=movers.tolist(), copy_dst=holes.tolist(), layers=1,
                    info={"evicted": sorted(evict), "moved_blocks": int(len(movers))})


WORKLOADS = {2: config2, 3: config3, 4: config4, 5: config5}


def kv_bytes(ctx, hkv: int, elt: int = 2) -> int:
    return int(np.sum(ctx)) * 2 * hkv * DH * elt


# ----------------------------------------------------------------------------- clocks


class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int) -> None:
        self.idx = device_index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                                          "-lms", "20", "-i", str(self.idx)], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        time.sleep(0.25)
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc is not None:
            time.sleep(0.15)
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [ln for ln in out.splitlines() if ln.strip()]

    def summary(self) -> dict:
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in getattr(self, "lines", []):
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for name, val in zip(names, f[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


# ----------------------------------------------------------------------------- helpers


def measured_peak() -> tuple[float, str]:
    p = REPO / "MEASURED_PEAKS.json"
    try:
        return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return FALLBACK_HBM_GBS, "fallback"


def profiled_traffic() -> int | None:
    """DRAM bytes per attention launch from the committed ncu summary (None until one is captured)."""
    p = REPO / "profiles" / "paged_attention_cfg2.md"
    if not p.exists():
        return None
    m = re.search(r"traffic_bytes_per_launch:\s*([0-9]+)", p.read_text())
    return int(m.group(1)) if m else None


def bind_to_gpu_cpus(local_rank: int) -> list[int] | None:
    """Pin this process to the CPUs NVML reports as local to its GPU (reading the topology only), before any
    pinned host buffer is allocated, so the rank's host memory and threads sit on its GPU's NUMA node.
    Several ranks on one host otherwise float over both sockets and their host-device copies cross the
    socket link.  Returns the CPU list, or None where NVML or affinity is unavailable."""
    try:
        import pynvml

        pynvml.nvmlInit()
        try:
            handle = pynvml.nvmlDeviceGetHandleByIndex(local_rank)
            words = pynvml.nvmlDeviceGetCpuAffinity(handle, (os.cpu_count() + 63) // 64)
        finally:
            pynvml.nvmlShutdown()
        cpus = [64 * w + b for w, word in enumerate(words) for b in range(64) if (word >> b) & 1]
        cpus = [c for c in cpus if c < (os.cpu_count() or 0)]
        if not cpus:
            return None
        os.sched_setaffinity(0, cpus)
        return cpus
    except Exception:  # no NVML, no permission: run unbound
        return None


def dist_env() -> tuple[int, int, int]:
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


def max_over_ranks(x: float, world: int, device) -> float:
    if world == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ----------------------------------------------------------------------------- CPU reference leg


def cpu_reference_step(wl: Workload, nb_sample_seqs: int, seed: int = 7):
    """Build the oracle's inputs for a bounded sample of the config-2 step (first `nb_sample_seqs`
    sequences, one layer, pool holding just their blocks) and return a callable that runs one step."""
    sys.path.insert(0, str(REPO))
    import oracle  # the reference's CPU algorithm (paged_torch_ref.py restated): the baseline, not the product

    sel = list(range(nb_sample_seqs))
    sctx = [int(wl.attend_ctx[i]) for i in sel]
    sblocks, nxt = [], 0
    for i in sel:  # renumber the sample's blocks densely: a small pool, same access pattern per sequence
        n = len(wl.attend_rows[i][2])
        sblocks.append(list(range(nxt, nxt + n)))
        nxt += n
    g = torch.Generator().manual_seed(seed)
    sc = wl.kv_scale
    k_pool = (torch.randn(nxt, BS, HKV, DH, generator=g) * sc).to(torch.bfloat16)
    v_pool = (torch.randn(nxt, BS, HKV, DH, generator=g) * sc).to(torch.bfloat16)
    q = torch.randn(len(sel), H, DH, generator=g).to(torch.bfloat16)
    k = (torch.randn(len(sel), HKV, DH, generator=g) * sc).to(torch.bfloat16)
    v = (torch.randn(len(sel), HKV, DH, generator=g) * sc).to(torch.bfloat16)
    meta = oracle.build_metadata([(c - 1, 1, b) for c, b in zip(sctx, sblocks)], BS)

    def step():
        oracle.forward(q, k, v, k_pool, v_pool, meta, compute_dtype=None)  # the reference's own dtype: bf16

    return step, kv_bytes(sctx, HKV), (f"{len(sel)} of {len(wl.attend_rows)} sequences (sum ctx {sum(sctx)}), "
                                       "1 layer, bf16")


def host_info() -> dict:
    """The host the CPU legs ran on: logical cores, torch's thread count, CPU model."""
    model = None
    try:
        with open("/proc/cpuinfo") as f:
            for ln in f:
                if ln.startswith("model name"):
                    model = ln.split(":", 1)[1].strip()
                    break
    except OSError:
        pass
    return {"os_cpu_count": os.cpu_count(), "torch_threads": torch.get_num_threads(), "cpu_model": model}


def run_cpu_baseline(wl: Workload, seqs: int, reps: int, warmup: int = 1) -> dict:
    step, nbytes, sample = cpu_reference_step(wl, seqs)
    for _ in range(warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(reps):
        step()
    dt = (time.perf_counter() - t0) / reps
    return {"value": round(nbytes / dt / 1e9, 3), "unit": "GB/s", "cores": torch.get_num_threads(), "kind": "port",
            "sample": sample + f", {reps} reps", "ms_per_step": round(dt * 1e3, 2), "host": host_info()}


def run_reference_arm(args) -> None:
    rank, world, _ = dist_env()
    if rank != 0:
        return  # the CPU arm runs once, on rank 0 only
    torch.set_num_threads(os.cpu_count() or 1)
    # the same workload as our arm at this N (weak scaling: batch x N), timed on a bounded sample of it
    weak = args.gpus > 1 and args.scaling == "weak"
    wl = config2(args.batch * (args.gpus if weak else 1))
    step, nbytes, sample = cpu_reference_step(wl, args.cpu_sample_seqs)
    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = (time.perf_counter() - t0) / args.steps
    value = nbytes / dt / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt * 1e3, 3), "higher_is_better": True,
        "scaling": "weak" if weak else "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": f"{wl.name}: {wl.describe}", "sample": sample},
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": torch.get_num_threads(), "kind": "port",
                         "sample": sample, "host": host_info()},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


METRIC = "Llama-3.1-8B paged decode attn: KV-read GB/s vs HBM peak, seqs/s; append GB/s"


# ----------------------------------------------------------------------------- our arm


@dataclass
class Rig:
    """One workload's device state on this rank: its layer pools (this rank's KV heads), the step's q/k/v,
    metadata, plan, workspace and output transport."""

    wl: Workload
    layers: int
    rank: int
    world: int
    dev: torch.device
    hkv_l: int
    h_l: int
    qs: slice
    ks: slice
    k_pools: list
    v_pools: list
    q: torch.Tensor  # the step's full rows [n_q, H, Dh] (every rank holds the same)
    q_l: torch.Tensor  # this rank's heads
    k_l: torch.Tensor
    v_l: torch.Tensor
    meta_att: object
    meta_app: object
    plan: object
    ws: object
    out_l: torch.Tensor
    p2p: bool
    peers: object
    gathered: torch.Tensor | None
    copies: int
    ptrs: torch.Tensor | None
    src: torch.Tensor | None
    dst: torch.Tensor | None
    fused: bool
    n_q: int
    n_app: int
    ops: object
    pdl: bool = True

    @property
    def launches_per_layer(self) -> int:
        # [append,] attention (+ shared-prefix attention), split-K reduction (p2p: always, carrying the gather)
        # [+ p2p barrier after plain stores]
        return ((1 if self.fused else 2) + (1 if self.plan.num_shared_units else 0)
                + (1 if self.plan.num_partial_rows or self.p2p else 0)
                + (1 if self.p2p and not self.peers.use_packets(self.n_q) else 0))


def make_rig(args, mlb, sharding, wl: Workload, dev, rank: int, world: int, layers: int) -> Rig:
    ops = mlb.ops
    hkv_l, h_l = HKV // world, H // world
    n_app, n_q = sum(n for _, n, _ in wl.append_rows), sum(n for _, n, _ in wl.attend_rows)
    nb = wl.num_blocks
    g = torch.Generator(device=dev).manual_seed(100 + rank)
    k_pools, v_pools = [], []
    for l in range(layers):  # layer 0 drawn, the others copies of it (separate memory, the same cost to read)
        for pools in (k_pools, v_pools):
            p = torch.empty(nb, BS, hkv_l, DH, device=dev, dtype=torch.bfloat16)
            if l == 0:
                p.normal_(0.0, wl.kv_scale, generator=g)
            else:
                p.copy_(pools[0])
            pools.append(p)
    gq = torch.Generator(device=dev).manual_seed(7)  # the same full q/k/v on every rank
    q = torch.randn(n_q, H, DH, device=dev, generator=gq).to(torch.bfloat16)
    k = (torch.randn(n_app, HKV, DH, device=dev, generator=gq) * wl.kv_scale).to(torch.bfloat16)
    v = (torch.randn(n_app, HKV, DH, device=dev, generator=gq) * wl.kv_scale).to(torch.bfloat16)
    qs, ks = sharding.head_range(rank, world, H), sharding.head_range(rank, world, HKV)
    q_l, k_l, v_l = q[:, qs], k[:, ks], v[:, ks]

    def seqsteps(rows):
        return [mlb.SeqStep(c, n, b) for c, n, b in rows]

    meta_att = mlb.AttentionMetadata.build(seqsteps(wl.attend_rows), BS, dev)
    meta_app = meta_att if wl.append_rows is wl.attend_rows else mlb.AttentionMetadata.build(
        seqsteps(wl.append_rows), BS, dev)
    if args.no_query_tiles:  # every row on 8-column work units (no host tables: no query tiles, no cascade)
        plan = ops.plan_attention(meta_att.query_start_loc, meta_att.seq_lens, meta_att.block_tables_i32.shape[1],
                                  h_l, hkv_l, dev, pages_per_unit=args.pages_per_unit)
    else:
        plan = mlb.B200Backend(pages_per_unit=args.pages_per_unit).plan(meta_att, h_l, hkv_l, dev)
    p2p = world > 1 and args.transport == "p2p"
    copies = len(wl.copy_src)
    ptrs = src = dst = None
    if copies:
        ptrs = ops.pool_pointer_table(k_pools + v_pools)
        src = torch.tensor(wl.copy_src, dtype=torch.int32, device=dev)
        dst = torch.tensor(wl.copy_dst, dtype=torch.int32, device=dev)
    # the append rides in the attention launch when every written block is private to its row (the backend's
    # rule: B200Backend.forward); otherwise K1 runs first
    fused = (not args.no_fused_append and meta_app is meta_att and meta_att.append_private
             and ops.can_fuse_append(plan, k_pools[0], k_l, v_l))
    return Rig(wl, layers, rank, world, dev, hkv_l, h_l, qs, ks, k_pools, v_pools, q, q_l, k_l, v_l, meta_att,
               meta_app, plan, ops.Workspace(), torch.empty(n_q, h_l, DH, device=dev, dtype=torch.bfloat16), p2p,
               sharding.PeerOutputs(n_q, H, DH, torch.bfloat16, dev, exchange=args.exchange) if p2p else None,
               torch.empty(world * n_q, h_l, DH, device=dev, dtype=torch.bfloat16) if world > 1 and not p2p else None,
               copies, ptrs, src, dst, fused, n_q, n_app, ops, not args.no_pdl)


def attend(r: Rig, l: int) -> None:
    slot = l % r.peers.slots if r.p2p else 0
    r.ops.attention_partials(r.q_l, r.k_pools[l], r.v_pools[l], r.meta_att.block_tables_i32, r.meta_att.seq_lens_i32,
                             r.meta_att.qo_indptr, r.plan, r.ws, r.out_l,
                             targets=r.peers.local_targets(slot, r.qs.start) if r.p2p else None,
                             append=(r.k_l, r.v_l, r.meta_app.slot_mapping) if r.fused else None)


def gather_step(r: Rig, l: int) -> None:
    """The layer's split-K reduction and output all-gather: p2p = the reduction sending every row to every
    rank as flagged packets and receiving theirs (one launch), or storing every row into every rank's buffer
    followed by the flag barrier; NCCL = the local reduction + all_gather_into_tensor."""
    if r.p2p:
        slot = l % r.peers.slots
        if r.peers.use_packets(r.n_q):
            r.ops.splitk_reduce_exchange(r.plan, r.ws, r.peers, slot, torch.bfloat16, DH, r.dev)
            return
        r.ops.splitk_reduce_gather(r.plan, r.ws, r.peers.targets(slot, r.qs.start), r.peers.self_dest,
                                   torch.bfloat16, DH, r.dev)
        r.peers.barrier()
        return
    r.ops.splitk_reduce(r.plan, r.ws, r.out_l)
    if r.world > 1:
        import torch.distributed as dist

        dist.all_gather_into_tensor(r.gathered, r.out_l)


def layer_step(r: Rig, l: int, ev=None) -> None:
    if not r.fused:
        r.ops.kv_append(r.k_pools[l], r.v_pools[l], r.meta_app.slot_mapping, r.k_l, r.v_l)
    if ev is not None:
        ev[0].record()
    attend(r, l)
    if ev is not None:
        ev[1].record()
    gather_step(r, l)


def full_step(r: Rig) -> None:
    if r.copies:  # COW / compaction: one launch over every layer's K and V pools
        r.ops.block_copy(r.ptrs, r.k_pools[0], r.src, r.dst)
    for l in range(r.layers):
        layer_step(r, l)


def sync_all(world: int) -> None:
    torch.cuda.synchronize()
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
    torch.cuda.synchronize()


def events(n: int = 2):
    return [torch.cuda.Event(enable_timing=True) for _ in range(n)]


def measure(r: Rig, args, sample_clocks: bool = True) -> dict:
    """Device timings of one rig, max over ranks: the whole step as a replayed CUDA graph (value), every
    layer's attention launch back to back (the roofline's duration), the gather + barrier of every layer alone
    (several GPUs), and the block copy alone."""
    w = r.world
    for _ in range(args.warmup):  # NCCL communicators, kernel attributes, the workspace
        full_step(r)
    sync_all(w)
    step_graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(step_graph):
        full_step(r)
    step_graph.replay()
    sync_all(w)
    start, end = events()
    clocks = ClockSampler(r.dev.index) if sample_clocks else None
    if clocks:
        clocks.__enter__()
    start.record()
    for _ in range(args.steps):
        step_graph.replay()
    end.record()
    sync_all(w)
    if clocks:
        clocks.__exit__(None, None, None)
    res = {"ms_per_step": max_over_ranks(start.elapsed_time(end), w, r.dev) / args.steps,
           "clocks": clocks.summary() if clocks else None}
    del step_graph
    # every layer's attention launch back to back, nothing between them, bracketed by two events on the
    # launching stream: with programmatic dependent launch each launch's start hides behind its predecessor's
    # tail, so the mean is the kernel's own duration
    b0, b1 = events()
    sync_all(w)
    b0.record()
    for _ in range(args.kernel_steps):
        for l in range(r.layers):
            attend(r, l)
    b1.record()
    sync_all(w)
    res["attn_ms"] = max_over_ranks(b0.elapsed_time(b1), w, r.dev) / (args.kernel_steps * r.layers)
    if w > 1:  # the reduction + all-gather (+ barrier) of every layer alone, replayed from a graph
        gather_graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gather_graph):
            for l in range(r.layers):
                gather_step(r, l)
        gather_graph.replay()
        g0, g1 = events()
        sync_all(w)
        g0.record()
        for _ in range(args.kernel_steps):
            gather_graph.replay()
        g1.record()
        sync_all(w)
        res["gather_ms"] = max_over_ranks(g0.elapsed_time(g1), w, r.dev) / (args.kernel_steps * r.layers)
        del gather_graph
    if r.copies:
        c0, c1 = events()
        sync_all(w)
        c0.record()
        for _ in range(3):
            r.ops.block_copy(r.ptrs, r.k_pools[0], r.src, r.dst)
        c1.record()
        sync_all(w)
        res["copy_ms"] = max_over_ranks(c0.elapsed_time(c1) / 3, w, r.dev)
    return res


def spot_check(r: Rig, sample: list[int]) -> float:
    """Run the last layer's full step once more and compare `sample` sequences of this rank's heads of the
    (gathered) output with a plain torch fp32 attention over the same pages, read back from the device.  The
    pools already hold the step's appended rows (every timed step wrote the same rows).  Returns the max-abs
    error over ranks; the bar is 2e-2 (bf16)."""
    last = r.layers - 1
    if r.copies:
        r.ops.block_copy(r.ptrs, r.k_pools[0], r.src, r.dst)
    layer_step(r, last)
    torch.cuda.synchronize()
    if r.p2p:
        got = r.peers.output(last % r.peers.slots, r.n_q)[:, r.qs]
    elif r.world > 1:
        got = r.gathered.view(r.world, r.n_q, r.h_l, DH)[r.rank]
    else:
        got = r.out_l
    starts = r.meta_att.query_start_loc
    err = 0.0
    group = r.h_l // r.hkv_l
    for s in sample:
        c, n, blocks = r.wl.attend_rows[s]
        length = c + n
        ids = torch.tensor(blocks[:-(-length // BS)], device=r.dev, dtype=torch.long)
        kk = r.k_pools[last][ids].reshape(-1, r.hkv_l, DH)[:length].float()  # [L, hkv, Dh]
        vv = r.v_pools[last][ids].reshape(-1, r.hkv_l, DH)[:length].float()
        qq = r.q_l[starts[s]:starts[s + 1]].float()  # [n, h, Dh]
        kh = kk.repeat_interleave(group, dim=1).permute(1, 0, 2)  # [h, L, Dh]
        vh = vv.repeat_interleave(group, dim=1).permute(1, 0, 2)
        scores = torch.einsum("nhd,hld->hnl", qq, kh) / math.sqrt(DH)
        causal = torch.arange(length, device=r.dev)[None, :] <= (length - n + torch.arange(n, device=r.dev))[:, None]
        scores = scores.masked_fill(~causal[None], float("-inf"))
        want = torch.einsum("hnl,hld->nhd", torch.softmax(scores, dim=-1), vh)
        err = max(err, (got[starts[s]:starts[s + 1]].float() - want).abs().max().item())
    return max_over_ranks(err, r.world, r.dev)


def release(r: Rig) -> None:
    if r.peers is not None:
        r.peers.close()
    r.k_pools.clear()
    r.v_pools.clear()
    torch.cuda.synchronize()
    torch.cuda.empty_cache()


def workload_summary(r: Rig, t: dict, peak: float, check: float, sample: list[int]) -> dict:
    """One sub-object of the bench line: the workload's step, attention and (several GPUs) gather figures."""
    ctx = r.wl.attend_ctx
    per_rank = kv_bytes(ctx, r.hkv_l)
    achieved = per_rank / (t["attn_ms"] * 1e-3) / 1e9
    out = {"workload": f"{r.wl.name}: {r.wl.describe}", "layers": r.layers,
           "value": round(per_rank * r.layers * r.world / (t["ms_per_step"] * 1e-3) / 1e9, 2), "unit": "GB/s",
           "ms_per_step": round(t["ms_per_step"], 4), "attention_us_per_rank": round(t["attn_ms"] * 1e3, 2),
           "roofline_frac_per_rank": round(achieved / peak, 4), "kv_heads_per_rank": r.hkv_l,
           "attend_rows": len(r.wl.attend_rows), "sum_ctx": int(np.sum(ctx)),
           "units_per_layer": r.plan.num_units, "shared_units_per_layer": r.plan.num_shared_units,
           "append": "fused into the attention launch" if r.fused else "separate K1 launch",
           "spot_check_max_abs": round(check, 5), "spot_check_rows": sample, "spot_check_bar": 2e-2,
           "spot_check_passed": bool(check <= 2e-2), **{k: v for k, v in r.wl.info.items() if k != "evicted"}}
    if "gather_ms" in t:
        out["gather_barrier_us_per_layer"] = round(t["gather_ms"] * 1e3, 2)
        if r.p2p:
            out["gather"] = "flagged packets" if r.peers.use_packets(r.n_q) else "stores + flag barrier"
    if r.wl.name == "config 4":  # shared prefix: HBM sees each shared block once per launch, so the roofline
        unique = r.wl.unique_pages() * BS * 2 * r.hkv_l * DH * 2  # fraction counts unique bytes
        out["logical_gbs_per_rank"] = round(achieved, 1)
        out["roofline_frac_per_rank"] = round(unique / (t["attn_ms"] * 1e-3) / 1e9 / peak, 4)
        out["roofline_bytes"] = "unique pages (each shared block once)"
    if r.copies:
        moved = r.copies * 2 * r.layers * BS * r.hkv_l * DH * 2
        out["block_copy"] = {"pairs": r.copies, "us": round(t["copy_ms"] * 1e3, 2),
                             "gbs_read_plus_write_per_rank": round(2 * moved / (t["copy_ms"] * 1e-3) / 1e9, 1)}
    return out


def run_ours(args) -> None:
    rank, world, local = dist_env()
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    cpus = bind_to_gpu_cpus(local) if world > 1 else None
    if world > 1:
        import torch.distributed as dist

        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=120))
    mlb = importlib.import_module(PACKAGE)
    sharding = importlib.import_module(PACKAGE + ".sharding")
    ops = mlb.ops
    mlb._lib.lib().mlb_set_programmatic_launch(0 if args.no_pdl else 1)
    mlb._lib.lib().mlb_set_tensor_core_prefix(0 if args.no_tc_prefix else 1)
    mlb._lib.lib().mlb_set_concurrent_prefix(0 if args.serial_prefix else 1)

    weak = world > 1 and args.config == 2 and args.scaling == "weak"
    if args.config == 2:
        wl = config2(args.batch * (world if weak else 1))
    elif args.config == 3:
        wl = config3(attend_chunks=args.attend_chunks)
    else:
        wl = WORKLOADS[args.config]()
    layers = args.layers or wl.layers
    r = make_rig(args, mlb, sharding, wl, dev, rank, world, layers)
    peak, peak_kind = measured_peak()

    t = measure(r, args)
    ms_per_step = t["ms_per_step"]
    attn_avg_ms = t["attn_ms"]

    # --- the older per-launch figure: events around each attention launch inside eager steps (they also hold
    # the launch latency an event between two kernels exposes)
    evs = [[events() for _ in range(layers)] for _ in range(args.kernel_steps)]
    sync_all(world)
    for s in range(args.kernel_steps):
        for l in range(layers):
            layer_step(r, l, evs[s][l])
    sync_all(world)
    attn_launch_ms = max_over_ranks(statistics.mean(e0.elapsed_time(e1) for st in evs for e0, e1 in st), world, dev)

    # --- append kernel alone (append GB/s): K1 over the layer pools, captured in a CUDA graph so the
    # launch-bound kernel is timed on the device, not behind the Python launch path
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for l in range(layers):
            ops.kv_append(r.k_pools[l], r.v_pools[l], r.meta_app.slot_mapping, r.k_l, r.v_l)
    graph.replay()
    ap_s, ap_e = events()
    sync_all(world)
    reps = 20
    ap_s.record()
    for _ in range(reps):
        graph.replay()
    ap_e.record()
    sync_all(world)
    del graph
    append_ms = max_over_ranks(ap_s.elapsed_time(ap_e) / (reps * layers), world, dev)
    append_bytes = 2 * 2 * r.n_app * r.hkv_l * DH * 2  # K and V rows read + written, bf16
    if r.p2p:  # the kernels' NVLink stores must have assembled exactly what an NCCL all-gather does
        import torch.distributed as dist

        r.peers.raise_errors()
        last = layers - 1
        got = r.peers.output(last % r.peers.slots, r.n_q).clone()
        ops.attention_partials(r.q_l, r.k_pools[last], r.v_pools[last], r.meta_att.block_tables_i32,
                               r.meta_att.seq_lens_i32, r.meta_att.qo_indptr, r.plan, r.ws, r.out_l)
        ops.splitk_reduce(r.plan, r.ws, r.out_l)
        flat = torch.empty(world * r.n_q, r.h_l, DH, device=dev, dtype=torch.bfloat16)
        dist.all_gather_into_tensor(flat, r.out_l)
        want = flat.view(world, r.n_q, r.h_l, DH).movedim(0, 1).reshape(r.n_q, H, DH)
        if not torch.equal(got, want):
            raise SystemExit(f"rank {rank}: p2p-gathered output differs from the NCCL all-gather")
        del got, want, flat
    sample = [0, len(wl.attend_rows) // 2, len(wl.attend_rows) - 1]
    check = spot_check(r, sample)

    # --- GPU comparison: FlashInfer's paged decode on the same pools, called as the reference's FlashInfer
    # backend calls it (attention/flashinfer_backend.py:48-58: NHD, plan once, run per layer)
    flashinfer = None
    if world == 1 and args.config == 2 and not args.no_flashinfer:
        flashinfer = run_flashinfer(r.meta_att, r.q, r.k_pools, r.v_pools, wl.attend_ctx, layers, args.kernel_steps,
                                    dev, r.out_l, attn_avg_ms)

    # --- end to end through the public API with host buffers (metadata build + H2D in, D2H out)
    e2e = e2e_ref = None
    if not args.no_e2e and args.config == 2:
        e2e = run_e2e(args, mlb, sharding, wl, r.q_l, r.k_l, r.v_l, r.k_pools, r.v_pools, dev, world)
        if world == 1 and not args.no_reference_meta:  # the same loop with the reference's metadata object
            e2e_ref = run_e2e(args, mlb, sharding, wl, r.q_l, r.k_l, r.v_l, r.k_pools, r.v_pools, dev, world,
                              reference_meta=True)

    ctx = wl.attend_ctx
    bytes_rank_layer = kv_bytes(ctx, r.hkv_l)
    value = bytes_rank_layer * layers * world / (ms_per_step * 1e-3) / 1e9
    achieved = bytes_rank_layer / (attn_avg_ms * 1e-3) / 1e9
    headline = {"gather_ms": t.get("gather_ms"), "copy_ms": t.get("copy_ms")}
    launches = r.launches_per_layer * layers * args.steps + (args.steps if r.copies else 0)
    fused, plan, n_q, n_app, copies = r.fused, r.plan, r.n_q, r.n_app, r.copies
    gather_mode = (("flagged packets" if r.peers.use_packets(r.n_q) else "stores + flag barrier") if r.p2p
                   else "NCCL all-gather")
    release(r)
    del r

    # --- the other BASELINE configs (one GPU) and strong KV-head sharding (several GPUs), one rig at a time
    extra = {}
    if world == 1 and args.config == 2 and not args.no_configs:
        for c in (3, 4, 5):
            cwl = WORKLOADS[c]()
            cr = make_rig(args, mlb, sharding, cwl, dev, rank, world, cwl.layers)
            ct = measure(cr, args, sample_clocks=False)
            cs = [0, len(cwl.attend_rows) - 1]
            extra[f"config_{c}"] = workload_summary(cr, ct, peak, spot_check(cr, cs), cs)
            release(cr)
            del cr
    if world > 1 and args.config == 2 and not args.no_strong:
        for name, swl in (("config_2_batch_64", config2(args.batch)), ("config_5", config5())):
            sr = make_rig(args, mlb, sharding, swl, dev, rank, world, swl.layers)
            st = measure(sr, args, sample_clocks=False)
            ss = [0, len(swl.attend_rows) - 1]
            extra[name] = workload_summary(sr, st, peak, spot_check(sr, ss), ss)
            release(sr)
            del sr

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and args.config == 2:
        torch.set_num_threads(os.cpu_count() or 1)
        cpu = run_cpu_baseline(wl, args.cpu_sample_seqs, reps=args.cpu_reps)

    if rank == 0:
        p2p = world > 1 and args.transport == "p2p"
        line = {
            "metric": METRIC if args.config == 2 else f"{wl.name}: paged decode attn KV-read GB/s (step incl. "
                                                        f"appends{' and block copies' if copies else ''})",
            "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4), "higher_is_better": True,
            "scaling": "weak" if weak else "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": f"{wl.name}: {wl.describe}", "layers": layers, "attend_rows": len(wl.attend_rows),
                       "query_tokens": n_q, "appended_tokens": n_app, "sum_ctx": int(np.sum(ctx)),
                       "pool_blocks": wl.num_blocks,
                       "parallelism": (f"kv-head shard x{world}, output gather: "
                                       + ((f"kernel NVLink stores, exchange={args.exchange} (flagged packets up to "
                                           f"{sharding.PACKET_BYTES_PER_PEER >> 10} KB per peer, else stores + flag "
                                           "barrier)") if p2p else "NCCL all-gather"))
                                      if world > 1 else "single GPU",
                       "l2": "no flush: every layer's pool reads exceed the 126 MB L2",
                       "host_binding": (f"each rank pinned to its GPU's NVML-local CPUs ({len(cpus)} on rank 0)"
                                        if cpus else "unbound"),
                       "programmatic_launch": not args.no_pdl,
                       "append": "fused into the attention launch" if fused else "separate K1 launch",
                       "shared_prefix_kernel": "mma.sync" if args.no_tc_prefix else "tcgen05",
                       "shared_prefix_beside_per_sequence_kernel": not args.serial_prefix,
                       "pages_per_unit": args.pages_per_unit,
                       "units_per_layer": plan.num_units, "ctas_per_layer": plan.num_units * (HKV // world),
                       "partial_rows": plan.num_partial_rows, **wl.info},
            "seqs_per_s": round(len(wl.attend_rows) / (ms_per_step * 1e-3 / layers), 1),
            "append_gbs": round(append_bytes / (append_ms * 1e-3) / 1e9, 2),  # K1 alone (graph of its launches)
            "append_us": round(append_ms * 1e3, 2),
            "attention_us": round(attn_avg_ms * 1e3, 2),  # back-to-back launches (the roofline's duration)
            "attention_us_single_launch_events": round(attn_launch_ms * 1e3, 2),
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                         "traffic": profiled_traffic() if args.config == 2 and world == 1 else None,
                         "algorithmic_bytes": bytes_rank_layer,
                         "kernel": "paged_attn_mma_kernel<bf16, Dh 128, 2 slots, 4 warps>"},
            "spot_check_max_abs": round(check, 5), "spot_check_passed": bool(check <= 2e-2),
            "gpu_launches": launches,
            "timing": "value: CUDA-graph replays of the step; roofline: every layer's attention launch back to back "
                      "between two CUDA events (mean per launch); attention_us_single_launch_events: events around "
                      "each launch inside eager steps",
            "clocks": t["clocks"],
        }
        if world > 1:
            line["roofline"]["traffic_note"] = ("DRAM traffic is captured with ncu on one GPU (config 2, N=1); not "
                                                "captured per rank at N>1")
            line["gather_barrier_us_per_layer"] = round(headline["gather_ms"] * 1e3, 2)
            line["gather"] = gather_mode
        if args.config == 4:
            unique = wl.unique_pages() * BS * 2 * (HKV // world) * DH * 2
            line["roofline"]["unique_bytes"] = unique
            line["roofline"]["unique_gbs"] = round(unique / (attn_avg_ms * 1e-3) / 1e9, 1)
            line["roofline"]["unique_frac"] = round(unique / (attn_avg_ms * 1e-3) / 1e9 / peak, 4)
        if copies:
            moved = copies * 2 * layers * BS * (HKV // world) * DH * 2
            line["block_copy"] = {"pairs": copies, "us": round(headline["copy_ms"] * 1e3, 2),
                                  "gbs_read_plus_write": round(2 * moved / (headline["copy_ms"] * 1e-3) / 1e9, 1)}
        if e2e:
            line["e2e"] = e2e
        if e2e_ref:
            line["e2e_reference_metadata"] = e2e_ref
        if flashinfer:
            line["flashinfer_decode"] = flashinfer
        if world == 1 and extra:
            line["configs"] = extra
        if world > 1 and extra:
            line["strong"] = extra
        if cpu:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()


def run_e2e(args, mlb, sharding, wl: Workload, q, k, v, k_pools, v_pools, dev, world,
            reference_meta: bool = False) -> dict:
    """Each step, through the public API with pinned host buffers: the step's metadata
    (AttentionMetadata.build_arrays from the engine's block-table arrays) and the backend's plan, with their
    own H2D copies, issued on the loader stream ahead of the inputs; the q/k/v rows of every layer copied
    host-to-device on the loader stream in 4 growing chunks (layers [0,1), [1,3), [3,8), [8,L): each lands
    while the layers before it compute); per layer the backend's forward once its chunk is in; the outputs
    read back device-to-host on a copier stream in 4 chunks; the step ends when the last output is on the
    host.  Inputs, outputs and metadata are double-buffered, so step n + 1's uploads run while step n
    computes.  One GPU: the outputs go into a step-wide device buffer (forward's out_targets).  Several GPUs:
    each rank holds and uploads only its own heads (q [N, H/n, Dh], k / v [N, Hkv/n, Dh], as a column-parallel
    QKV projection leaves them), calls KVHeadShardedBackend.forward_local and reads back its own heads of the
    gathered output, so the job reads the whole result back once.
    reference_meta: hand the backend an object with only the reference's AttentionMetadata fields (what an
    unmodified reference engine passes), so it derives the host tables itself (one device-to-host copy and
    host synchronisation per step)."""
    layers = len(k_pools)
    rank = 0
    if world > 1:
        import torch.distributed as dist

        rank = dist.get_rank()
    q, k, v = q.contiguous(), k.contiguous(), v.contiguous()  # this rank's heads
    n_rows, h_full = q.shape[0], q.shape[1] * world
    sizes = [t.numel() * t.element_size() for t in (q, k, v)]
    per_layer = sum(sizes)
    host_in = torch.empty(layers * per_layer, dtype=torch.uint8).pin_memory()
    direct = world == 1
    p2p_ring = world > 1 and args.transport == "p2p"
    nbuf = 2
    dev_in = [torch.empty(layers * per_layer, dtype=torch.uint8, device=dev) for _ in range(nbuf)]

    def views(buf, l):
        out, off = [], l * per_layer
        for t, n in zip((q, k, v), sizes):
            out.append(buf[off:off + n].view(t.dtype).view(t.shape))
            off += n
        return out

    for l in range(layers):
        for dst, src in zip(views(host_in, l), (q, k, v)):
            dst.copy_(src.cpu())
    dev_views = [[views(dev_in[b], l) for l in range(layers)] for b in range(nbuf)]
    # the engine's block tables as arrays (AttentionMetadata.build_arrays skips the per-list conversion)
    rows = wl.attend_rows
    arrays = (np.array([c for c, _, _ in rows], dtype=np.int64), np.array([n for _, n, _ in rows], dtype=np.int64),
              np.concatenate([np.asarray(b, dtype=np.int64) for _, _, b in rows]),
              np.array([len(b) for _, _, b in rows], dtype=np.int64))
    fields = importlib.import_module(PACKAGE + ".attention.metadata").REFERENCE_FIELDS
    inner_backend = mlb.B200Backend(pages_per_unit=args.pages_per_unit)
    # p2p: one gathered-output slot per layer and step, two steps' worth: step n writes slots of parity n % 2
    backend = (sharding.KVHeadShardedBackend(inner_backend, transport=args.transport,
                                             slots=2 * layers if p2p_ring else 2, exchange=args.exchange)
               if world > 1 else inner_backend)
    # outputs come back in 4 shrinking chunks (a side-stream copy per layer costs ~60 us of host time: 32 per
    # step made the step host-bound)
    o_edges = sorted({0, layers} | {b for b in (layers // 2, layers - 4, layers - 1) if 0 < b < layers})
    o_chunks = list(zip(o_edges[:-1], o_edges[1:]))
    o_last = {hi - 1: (lo, hi) for lo, hi in o_chunks}
    host_out = [torch.empty((layers, *q.shape), dtype=q.dtype).pin_memory() for _ in range(nbuf)]
    # several GPUs: this rank's heads of the gathered rows are strided in the slots (a row of h/n heads every
    # H heads); they come back with one strided DMA per layer (cudaMemcpy2DAsync), no copy kernel.  Packing
    # them on the device first (torch's copy_ of the strided view, or a copy into a staging buffer) put a
    # kernel on the copier stream beside the attention kernel, and the layer after each read-back took
    # +80-130 us (a traced step, 2 GPUs: layers 16 and 28 of 32); the DMA alone costs nothing visible
    memcpy2d = None
    if world > 1:
        from cuda.bindings import runtime as cudart

        def memcpy2d(dst: int, dpitch: int, src: int, spitch: int, width: int, height: int) -> None:
            err, = cudart.cudaMemcpy2DAsync(dst, dpitch, src, spitch, width, height,
                                            cudart.cudaMemcpyKind.cudaMemcpyDeviceToHost, copier.cuda_stream)
            if int(err) != 0:
                raise RuntimeError(f"cudaMemcpy2DAsync: {err}")
    if direct:
        dev_out = [torch.empty((layers, *q.shape), dtype=q.dtype, device=dev) for _ in range(nbuf)]
        targets = [[mlb.ops.out_targets([dev_out[b][l].data_ptr()], 0, q.shape[1] * q.shape[2], q.shape[2])
                    for l in range(layers)] for b in range(nbuf)]
    state = {"step": 0, "host_ms": 0.0}
    compute = torch.cuda.current_stream(dev)
    loader, copier = torch.cuda.Stream(dev), torch.cuda.Stream(dev)  # H2D of inputs, D2H of outputs
    # chunk boundaries: layer 0's inputs alone, then chunks that land while the layers before them compute
    edges = sorted({0, layers} | {b for b in (1, 3, 8) if b < layers})
    chunks = list(zip(edges[:-1], edges[1:]))
    chunk_of = {lo: c for c, (lo, _) in enumerate(chunks)}
    loaded = [torch.cuda.Event() for _ in chunks]  # inputs of a chunk of layers on the device
    ready = [torch.cuda.Event() for _ in range(layers)]  # output l computed
    comp_done = [torch.cuda.Event() for _ in range(nbuf)]  # the last step on buffer b has finished computing
    io_done = [torch.cuda.Event() for _ in range(nbuf)]  # ... and its outputs are on the host
    for ev in comp_done + io_done:
        ev.record(compute)
    metas = [None] * nbuf  # each buffer's metadata, alive until the buffer's next turn
    inner = backend.inner if world > 1 else backend
    h_l, hkv_l = q.shape[1], k_pools[0].shape[2]
    own = slice(rank * h_l, (rank + 1) * h_l)  # this rank's query heads in the gathered output

    def step():
        b = state["step"] % nbuf
        prev = (state["step"] - 1) % nbuf
        loader.wait_event(comp_done[b])  # the last step on buffer b has read its inputs, metadata and plan
        t0 = time.perf_counter()
        with torch.cuda.stream(loader):
            # the step's metadata and plan go first in the loader's queue: on the compute stream their small
            # host-to-device copies queued behind the loader's input chunks (a measured ~0.48 ms at every
            # step start); layer 0 waits for the first chunk, so for them too
            meta = mlb.AttentionMetadata.build_arrays(*arrays, BS, dev)
            if reference_meta:
                meta = types.SimpleNamespace(**{f: getattr(meta, f) for f in fields})
            inner.plan(meta, h_l, hkv_l, dev, q.dtype)
            for c, (lo, hi) in enumerate(chunks):  # then the q/k/v rows in a few growing chunks
                dev_in[b][lo * per_layer:hi * per_layer].copy_(host_in[lo * per_layer:hi * per_layer],
                                                               non_blocking=True)
                loaded[c].record(loader)
        state["host_ms"] += (time.perf_counter() - t0) * 1e3
        metas[b] = meta  # the device tensors it holds (and the plan's) stay unreused until comp_done[b]
        compute.wait_event(io_done[b])  # buffer b's outputs of two steps back have been read back
        state["step"] += 1
        for l in range(layers):
            if l in chunk_of:
                compute.wait_event(loaded[chunk_of[l]])
            if p2p_ring and l == layers - 1:
                # the peers rewrite this rank's slots of the previous step's parity during the next step, which
                # none of them starts before this layer's barrier: the previous read-back must be done by then
                compute.wait_event(io_done[prev])
            qd, kd, vd = dev_views[b][l]
            if direct:
                backend.forward(qd, kd, vd, k_pools[l], v_pools[l], meta, out_targets=targets[b][l])
            elif p2p_ring:
                backend.forward_local(qd, kd, vd, k_pools[l], v_pools[l], meta)  # lands in slot b * layers + l
            else:
                out = backend.forward_local(qd, kd, vd, k_pools[l], v_pools[l], meta)  # NCCL: a fresh tensor
                ready[l].record(compute)
                copier.wait_event(ready[l])
                with torch.cuda.stream(copier):
                    host_out[b][l].copy_(out[:, own], non_blocking=True)
                out.record_stream(copier)  # from torch's allocator: keep it alive until the copy ran
                continue
            if l in o_last:  # a chunk of layers is complete: read it back on the side stream
                lo, hi = o_last[l]
                ready[l].record(compute)
                copier.wait_event(ready[l])
                with torch.cuda.stream(copier):
                    if direct:
                        host_out[b][lo:hi].copy_(dev_out[b][lo:hi], non_blocking=True)
                    else:
                        peers = backend.peers
                        eb = q.element_size()
                        width = h_l * q.shape[2] * eb  # this rank's heads of one token
                        for ll in range(lo, hi):
                            memcpy2d(host_out[b][ll].data_ptr(), width,
                                     peers.slot_address(b * layers + ll) + own.start * q.shape[2] * eb,
                                     h_full * q.shape[2] * eb, width, n_rows)
        io_done[b].record(copier)
        comp_done[b].record(compute)

    # warm-up as long as a timed window (and no synchronisation inside it): the host runs ahead of the device
    # by a growing number of steps, and torch's pinned staging buffers (metadata, plan) grow with that lead;
    # a short warm-up left their growth to the first timed window
    for _ in range(max(1, args.warmup) + args.steps):
        step()
    torch.cuda.synchronize()
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
    # three timed windows of `steps` steps each, the median reported: the eager path is the host's pace
    # when the host stalls (other jobs on the machine), and one stall must not stand for the path
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    windows, host_loop = [], []
    state["host_ms"] = 0.0
    for _ in range(3):
        s.record()
        t_loop = time.perf_counter()
        for _ in range(args.steps):
            step()
        host_loop.append((time.perf_counter() - t_loop) * 1e3 / args.steps)
        compute.wait_stream(copier)  # the window ends when the last step's outputs are on the host
        e.record()
        torch.cuda.synchronize()
        windows.append(max_over_ranks(s.elapsed_time(e), world, dev) / args.steps)
    ms = statistics.median(windows)
    host_build_ms = max_over_ranks(state["host_ms"] / (3 * args.steps), world, dev)
    d2h = layers * q.numel() * q.element_size()  # bytes read back (this rank's heads on several GPUs)
    if world > 1:
        backend.close()
    total = kv_bytes(wl.attend_ctx, HKV) * layers
    p = inner._plan
    plan_bytes = sum(a.nbytes for a in (p.units_host, p.shared_host, p.members_host, p.reduce_rows_host,
                                        p.reduce_chunks_host))
    h2d = layers * per_layer + _meta_upload_bytes(arrays) + plan_bytes
    return {"value": round(total / (ms * 1e-3) / 1e9, 2), "unit": "GB/s", "ms_per_step": round(ms, 4),
            "window_ms_per_step": [round(w, 4) for w in windows],
            "host_build_plan_ms_per_step": round(host_build_ms, 3),
            "host_issue_ms_per_step": round(max_over_ranks(statistics.median(host_loop), world, dev), 3),
            "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
            "metadata": ("reference-shaped object (the reference's AttentionMetadata fields only): host tables "
                         "derived by the backend" if reference_meta else "AttentionMetadata.build_arrays"),
            "path": (f"KVHeadShardedBackend(transport={args.transport!r}).forward_local" if world > 1
                     else "B200Backend.forward")
                    + " per layer; pinned host I/O on side streams, double-buffered: H2D of the step's q/k/v in 4 "
                      "chunks, D2H of the outputs " + ("in 4 chunks" if direct else
                                                       "as one strided DMA per layer, issued at 4 points" if p2p_ring
                                                       else "per layer")
                    + ("; each rank uploads and reads back its own heads" if world > 1 else "")}


def run_flashinfer(meta, q, k_pools, v_pools, ctx, layers, steps, dev, ours_out, ours_ms) -> dict:
    """FlashInfer BatchDecodeWithPagedKVCacheWrapper on the same pages, called as the reference's FlashInfer
    backend calls it (attention/flashinfer_backend.py:48-58): the reference's CUDA path, timed per launch with
    events, beside this build's attention on the same pools; its last layer's output is compared with ours."""
    try:
        import flashinfer
    except ImportError as e:
        return {"unavailable": f"flashinfer not importable: {e}"}
    try:
        return _time_flashinfer(flashinfer, meta, q, k_pools, v_pools, ctx, layers, steps, dev, ours_out, ours_ms)
    except Exception as e:  # a JIT build or plan failure of the library: reported, not fatal to the bench
        return {"unavailable": f"flashinfer {flashinfer.__version__}: {type(e).__name__}: {str(e)[:200]}"}


def _time_flashinfer(flashinfer, meta, q, k_pools, v_pools, ctx, layers, steps, dev, ours_out, ours_ms) -> dict:
    t0 = time.perf_counter()
    ws = torch.empty(128 * 2**20, dtype=torch.uint8, device=dev)
    w = flashinfer.BatchDecodeWithPagedKVCacheWrapper(ws, kv_layout="NHD")
    w.plan(meta.kv_indptr, meta.kv_indices, meta.kv_last_page_len, H, HKV, DH, BS, pos_encoding_mode="NONE",
           q_data_type=q.dtype, kv_data_type=k_pools[0].dtype)
    out = w.run(q, (k_pools[0], v_pools[0]))
    torch.cuda.synchronize()
    setup_s = time.perf_counter() - t0
    evs = []
    for _ in range(steps):
        for l in range(layers):
            e0, e1 = events()
            e0.record()
            w.run(q, (k_pools[l], v_pools[l]), out=out)
            e1.record()
            evs.append((e0, e1))
    torch.cuda.synchronize()
    us = statistics.mean(e0.elapsed_time(e1) for e0, e1 in evs) * 1e3
    nbytes = kv_bytes(ctx, HKV)
    diff = (out.float() - ours_out.float()).abs().max().item()  # out holds the last layer's output
    return {"attention_us": round(us, 2), "gbs": round(nbytes / us / 1e3, 1), "version": flashinfer.__version__,
            "ours_attention_us": round(ours_ms * 1e3, 2), "flashinfer_over_ours_time": round(us / (ours_ms * 1e3), 3),
            "max_abs_vs_ours": round(diff, 5), "setup_s": round(setup_s, 1),
            "timing": "events around each launch (ours: back to back, the roofline's duration)",
            "call": "BatchDecodeWithPagedKVCacheWrapper(NHD).plan(kv_indptr, kv_indices, kv_last_page_len, ...).run"}


def _meta_upload_bytes(arrays) -> int:
    """Host-to-device bytes of a step's metadata on the CUDA path: the compact int64 upload that
    mlb_build_metadata expands (block ids, their offsets and the per-sequence prefix arrays)."""
    cached, new, ids, nblk = arrays
    return 8 * (ids.size + 5 * cached.size + 3)


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", type=int, choices=sorted(WORKLOADS), default=2)
    ap.add_argument("--layers", type=int, default=0, help="layer pools (default: the config's, 32 or 1)")
    ap.add_argument("--kernel-steps", type=int, default=10, help="eager steps whose attention launches are timed")
    ap.add_argument("--batch", type=int, default=64, help="config 2 sequences per GPU-set (see --scaling)")
    ap.add_argument("--transport", choices=["p2p", "nccl"], default="p2p",
                    help="N>1: output all-gather by the kernels' own NVLink stores + a flag barrier (p2p), or NCCL")
    ap.add_argument("--exchange", choices=["auto", "packets", "barrier"], default="auto",
                    help="p2p: rows to the peers as flagged packets in the reduction's launch (packets), plain "
                         "stores followed by a flag-barrier launch (barrier), or by the step's size (auto)")
    ap.add_argument("--scaling", choices=["weak", "strong"], default="weak",
                    help="N>1, config 2: weak = batch x N sequences (each rank keeps one GPU's KV bytes); "
                         "strong = the same batch split by KV heads (configs 3-5 are always strong)")
    ap.add_argument("--cpu-sample-seqs", type=int, default=16)
    ap.add_argument("--cpu-reps", type=int, default=10)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-flashinfer", action="store_true",
                    help="N=1, config 2: skip timing FlashInfer's decode (the reference's CUDA backend) on the same pages")
    ap.add_argument("--no-configs", action="store_true",
                    help="N=1, config 2: skip the configs 3 / 4 / 5 sub-objects of the line")
    ap.add_argument("--no-strong", action="store_true",
                    help="N>1, config 2: skip the strong KV-head sharding sub-objects (config 2 batch 64, config 5)")
    ap.add_argument("--no-reference-meta", action="store_true",
                    help="N=1: skip the e2e run with the reference's metadata object")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-pdl", action="store_true", help="launch without programmatic dependent launch")
    ap.add_argument("--attend-chunks", action="store_true",
                    help="config 3: the prefill chunks also attend (multi-token rows on query tiles)")
    ap.add_argument("--no-query-tiles", action="store_true",
                    help="plan without host tables: every row on the decode kernel's 8-column units")
    ap.add_argument("--no-fused-append", action="store_true",
                    help="launch the append (K1) before attention even when it could ride in the attention launch")
    ap.add_argument("--pages-per-unit", type=int, default=0, help="split-K unit size in pages (0: the planner's)")
    ap.add_argument("--serial-prefix", action="store_true",
                    help="run the shared-prefix kernel before the per-sequence kernel instead of beside it")
    ap.add_argument("--no-tc-prefix", action="store_true",
                    help="shared-prefix units on the mma.sync kernel instead of tcgen05")
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference_arm(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
