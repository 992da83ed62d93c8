#!/usr/bin/env python
"""Benchmark of the FlashMap drafter hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload all|...]

The default line (``--workload all``) measures BASELINE config 5, the
workload quoted "at 1/2/4/8 B200": 512 requests of the Qwen3.8-27B-sized
drafter (hidden 2560, 10 DiT layers, SwiGLU 6912, a 32768-token state
vocabulary of 248320), contexts U[1024, 8192], K = 16, one jump.  Requests
are sharded over the N ranks by longest-processing-time on context length
with equal counts per rank (flashmap_b200.sharding); every rank drafts its
share in chunks of <= 64 with its own weight replica and no collective on the
data path.  A step drafts all 512 requests once: per chunk, W warm-up and K
timed replays of the CUDA-graph-captured pass (CUDA events, a barrier
before), summed over the rank's chunks, the maximum over ranks.  ``value`` is
512 x 16 drafted tokens / step time (strong scaling: the work is fixed as N
grows); ``e2e`` is the same through DraftSession.draft with anchors copied
from pinned host memory and tokens copied back on every call.  Each chunk
streams ~3 GB of context K/V per pass, more than the 126 MB L2.

Beside it: ``pass_us`` / ``batch1``, the BASELINE config-2 pass (Qwen3-8B
sizing: hidden 2048, 8 layers, 16 heads x 128, GELU 8192, LM head over
151936 rows of 4096), batch 1 per rank, a 2048-position context (2.5 GB of
weights and context streamed per pass), against its HBM floor; on one GPU
also configs 3 (batch 64 ragged, 1 and 2 jumps) and 4 (acceptance).  Weights
are seeded random-init (no checkpoint on the box), conditioning N(0, 1).

``--impl reference`` times the reference algorithm (the CPU oracle port of
modeling_flashmap.py) on the host cores over a bounded sample of the same
workload; under torchrun only rank 0 runs it.
"""

from __future__ import annotations

import argparse
import datetime
import json
import math
import os
import statistics
import subprocess
import sys
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

METRIC = "drafted tokens/sec (K=16) at 1/2/4/8 B200; batch-1 pass µs vs HBM floor"
CONFIG2 = dict(target_hidden_size=4096, vocab_size=151936, target_layer_ids=[1], block_size=16, hidden_size=2048,
               num_hidden_layers=8, num_attention_heads=16, intermediate_size=8192, mlp_type="gelu")
CONTEXT = 2048
# Config 5: the Qwen3.8-27B map (SwiGLU, 32768-token state vocabulary of 248320)
CONFIG5 = dict(target_hidden_size=5120, vocab_size=248320, state_vocab_size=32768, target_layer_ids=[1],
               block_size=16, hidden_size=2560, num_hidden_layers=10, num_attention_heads=20, intermediate_size=6912,
               mlp_type="swiglu")
FALLBACK_HBM_GBS = 6650.0


def log(*a):
    print(*a, file=sys.stderr, flush=True)


# ------------------------------------------------------------------ distributed plumbing

def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ------------------------------------------------------------------ workload

def algorithmic_bytes(c: dict, context: int) -> dict:
    """Bytes one batch-1 pass must move at least: every weight once, the context K/V once."""
    D, L, I, Ht, V = c["hidden_size"], c["num_hidden_layers"], c["intermediate_size"], c["target_hidden_size"], \
        c["vocab_size"]
    slot = L * (3 * D * D + D * D + D * D + D * D + 2 * D * I) + D * Ht + Ht * Ht + D * Ht
    anchor = Ht * D + L * 2 * D * D
    lm = V * Ht
    kv = (context + 1) * L * 2 * D * 2
    return {"weights": 2 * (slot + anchor + lm), "lm_head": 2 * lm, "kv": kv, "total": 2 * (slot + anchor + lm) + kv}


# the same per-layer shapes and kernels with 2 layers and a 32768-row LM head (< 2 GB on the device),
# for ncu captures that replay each kernel many times
PROFILE_SMALL = dict(CONFIG2, num_hidden_layers=2, vocab_size=32768)


def build_workload(seed: int = 0, small: bool = False, launch: str = "auto"):
    from flashmap_b200 import DraftSession, FlashMapCache, FlashMapConfig, FlashMapDraftModel
    from flashmap_b200.synthetic import synthetic_state_dict, synthetic_target_head
    from torch import nn

    config = FlashMapConfig(**(PROFILE_SMALL if small else CONFIG2))
    dev = torch.device("cuda", torch.cuda.current_device())
    with torch.device(dev):
        model = FlashMapDraftModel(config).to(torch.bfloat16).eval()
    model.launch_mode = launch
    model.load_state_dict(synthetic_state_dict(config, seed=seed, dtype=torch.bfloat16, device=dev), strict=True)
    emb_w, head_w = synthetic_target_head(config, seed=seed, dtype=torch.bfloat16, device=dev)
    embed, head = nn.Embedding(*emb_w.shape, device=dev, dtype=torch.bfloat16), nn.Linear(1, 1, bias=False)
    embed.weight = nn.Parameter(emb_w, requires_grad=False)
    head.weight = nn.Parameter(head_w, requires_grad=False)
    K = config.block_size
    cache = FlashMapCache(config, 1, CONTEXT + K + 2, device=dev, dtype=torch.bfloat16)
    g = torch.Generator(device=dev).manual_seed(seed + 2)
    hidden = torch.randn(1, CONTEXT, config.target_hidden_size, generator=g, device=dev).to(torch.bfloat16)
    model.extend_context(cache, hidden, embed, head)
    session = DraftSession(model, cache, embed, head, num_steps=1, seed=seed)
    session.embed_tokens, session.lm_head = embed, head
    return config, model, cache, session


# ------------------------------------------------------------------ clocks

class ClockSampler:
    """nvidia-smi samples every 200 ms while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.index = gpu_index
        self.proc = None
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "200", "-i", str(gpu_index)], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
        except (OSError, ValueError):
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=10)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sms, maxes, reasons, power = [], [], set(), []
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sms.append(float(f[1]))
                maxes.append(float(f[2]))
                power.append(float(f[3]))
            except ValueError:
                continue
            for name, val in zip(names, f[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sms) if sms else None, "sm_max_mhz": max(maxes) if maxes else None,
                "reasons": sorted(reasons), "samples": len(sms), "power_w_max": max(power) if power else None}


def physical_gpu_index(local: int) -> int:
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        ids = [v.strip() for v in vis.split(",") if v.strip()]
        if local < len(ids) and ids[local].isdigit():
            return int(ids[local])
    return local


def measured_peak_hbm():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return FALLBACK_HBM_GBS, "fallback"


def profiled_traffic_ratio(name: str, key: str = "traffic_ratio"):
    """DRAM traffic over algorithmic bytes of a kernel, from its committed ncu summary."""
    path = os.path.join(ROOT, "profiles", name)
    try:
        for line in open(path):
            if line.strip().startswith(key + ":"):
                return float(line.split(":", 1)[1].strip())
    except OSError:
        pass
    return None


def profiled_traffic():
    """DRAM bytes per LM-head launch from the committed ncu summary, if present."""
    path = os.path.join(ROOT, "profiles", "lm_head_gemm_config2.md")
    try:
        for line in open(path):
            if line.strip().startswith("traffic_bytes_per_launch:"):
                return int(float(line.split(":", 1)[1].strip()))
    except OSError:
        pass
    return None


# ------------------------------------------------------------------ CPU side (oracle port)

def tiled_target_head(config, seed: int):
    """Target embedding / head of the right shape filled with seeded N(0,1) and
    U(+-1/sqrt(H)) blocks of 8192 rows repeated down the vocabulary."""
    V, Ht = config.vocab_size, config.target_hidden_size
    g = torch.Generator().manual_seed(seed)
    e_blk = torch.randn(8192, Ht, generator=g).to(torch.bfloat16)
    h_blk = ((torch.rand(8192, Ht, generator=g) * 2 - 1) / Ht ** 0.5).to(torch.bfloat16)
    emb, head = torch.empty(V, Ht, dtype=torch.bfloat16), torch.empty(V, Ht, dtype=torch.bfloat16)
    for r in range(0, V, 8192):
        n = min(8192, V - r)
        emb[r:r + n] = e_blk[:n]
        head[r:r + n] = h_blk[:n]
    return emb, head


def cpu_reference(c: dict, context: int, seconds: float = 15.0, seed: int = 0, label: str = "config-2") -> dict:
    """The reference algorithm (CPU oracle port) on the host cores: a bounded
    sample of one-jump draft passes of the drafter `c`, bf16, batch 1, over a
    context of `context` positions."""
    from flashmap_b200 import FlashMapConfig
    from flashmap_b200.synthetic import synthetic_state_dict, synthetic_target_head
    from oracle.flashmap_oracle import Oracle, OracleCache

    threads = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
    torch.set_num_threads(threads)
    config = FlashMapConfig(**c)
    t0 = time.perf_counter()
    sd = synthetic_state_dict(config, seed=seed, dtype=torch.bfloat16)
    oracle = Oracle(config, sd, torch.bfloat16)
    if config.vocab_size * config.target_hidden_size > (1 << 30):
        # a timing sample: the target rows are seeded random 8192-row blocks repeated down the
        # vocabulary (drawing 2.5 G values one by one takes minutes on the host)
        emb, head = tiled_target_head(config, seed)
    else:
        emb, head = synthetic_target_head(config, seed=seed, dtype=torch.bfloat16)
    K = config.block_size
    cache = OracleCache(config, 1, context + K + 2, torch.bfloat16)
    width = len(config.target_layer_ids) * config.target_hidden_size
    hidden = torch.randn(1, context, width, generator=torch.Generator().manual_seed(2))
    oracle.extend_context(cache, hidden.to(torch.bfloat16))
    g = torch.Generator().manual_seed(3)
    z = torch.randn(1, K, config.target_hidden_size, generator=g).to(torch.bfloat16)
    anchor = torch.randint(0, config.vocab_size, (1,), generator=g)
    oracle.draft(anchor, cache, emb, head, num_steps=1, z=z)  # warm-up: includes the one-time Cholesky
    setup = time.perf_counter() - t0
    n, t1 = 0, time.perf_counter()
    while n < 3 or time.perf_counter() - t1 < seconds:
        oracle.draft(anchor, cache, emb, head, num_steps=1, z=z)
        n += 1
    el = time.perf_counter() - t1
    return {"value": K * n / el, "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"{n} {label} one-jump draft passes (bf16, batch 1, ctx {context}) of the CPU oracle port "
                      f"after one warm-up pass; {el:.1f} s timed, {setup:.1f} s setup",
            "ms_per_pass": 1000.0 * el / n}


def shard_context_median() -> int:
    return int(sorted(shard_lengths())[SHARD_REQUESTS // 2])


def workload_config(args, world: int) -> dict:
    """The ``config`` of both arms' JSON lines (the same workload, the same dict)."""
    if args.workload == "all":
        return {"workload": "config5: 512 requests of the Qwen3.8-27B-sized drafter (hidden 2560, 10 layers, 20 heads "
                            "x 128, SwiGLU 6912, 32768-of-248320 state vocabulary), contexts U[1024, 8192], K=16, "
                            "1 jump, sharded by request over the GPUs; beside it config2 (Qwen3-8B-sized drafter, "
                            "batch 1 per GPU, ctx 2048)",
                "requests": SHARD_REQUESTS, "chunk": SHARD_CHUNK, "block": 16, "num_steps": 1,
                "parallelism": f"request-sharded x{world} (LPT on context length, equal counts, no collective)",
                "l2": "inputs larger than L2: a 64-request chunk streams ~3 GB of context K/V per pass",
                "timing": "per chunk: CUDA events over K graph replays (ours), host clock over a bounded sample "
                          "(reference); a step drafts all 512 requests: sum over chunks, max over ranks",
                "launch": args.launch}
    nbytes = algorithmic_bytes(PROFILE_SMALL if args.profile_small else CONFIG2, CONTEXT)
    cfg = {"workload": "config2: Qwen3-8B-sized drafter pass, batch 1 per GPU, K=16, ctx 2048, 1 jump",
           "batch_per_gpu": 1, "block": 16, "context": CONTEXT, "num_steps": 1,
           "parallelism": f"replicas x{world} (request-sharded, no collective)",
           "l2": "inputs larger than L2: %.2f GB of weights + context streamed per pass" % (nbytes["total"] / 1e9),
           "timing": "per pass: CUDA events (ours), host clock (reference); max over ranks",
           "launch": args.launch}
    if args.profile_small:
        cfg["workload"] = "profiling case: config-2 layer shapes, 2 layers, 32768-row LM head"
    return cfg


def run_reference(args, world, rank):
    if rank != 0:
        return
    if args.workload == "all":
        ref = cpu_reference(CONFIG5, shard_context_median(), seconds=args.cpu_seconds, label="config-5")
    else:
        ref = cpu_reference(CONFIG2, CONTEXT, seconds=args.cpu_seconds)
    line = {"impl": "reference", "metric": METRIC, "value": ref["value"], "unit": "tokens/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ref["ms_per_pass"],
            "higher_is_better": True, "scaling": "strong" if args.workload == "all" else "weak",
            "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded random-init drafter, N(0,1) conditioning)",
            "config": workload_config(args, world),
            "cpu_baseline": {k: ref[k] for k in ("value", "unit", "cores", "kind", "sample")},
            "e2e": {"value": ref["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ secondary workloads (configs 3, 4)

def measured_peak_tensor():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["bf16_tflops"]), "measured"
    except (OSError, KeyError, ValueError):
        return 1590.0, "fallback"


def gemm_flops(c: dict, batch: int, block: int = 16) -> float:
    """Dense GEMM FLOPs of one one-jump draft of `batch` sequences (slot path
    and LM head per token, anchor path per sequence)."""
    D, L, I, Ht, V = c["hidden_size"], c["num_hidden_layers"], c["intermediate_size"], c["target_hidden_size"], \
        c["vocab_size"]
    mlp = (3 if c.get("mlp_type") == "swiglu" else 2) * D * I
    slot = L * (6 * D * D + mlp) + D * Ht + Ht * Ht + D * Ht
    lm = (c.get("state_vocab_size") or V) * Ht
    anchor = Ht * D + L * 2 * D * D
    return 2.0 * batch * (block * (slot + lm) + anchor)


def build_model(c: dict, seed: int):
    """A seeded random-init drafter of sizing `c` with its target embedding and head, on this GPU."""
    from flashmap_b200 import FlashMapConfig, FlashMapDraftModel
    from flashmap_b200.synthetic import synthetic_state_dict, synthetic_target_head
    from torch import nn

    config = FlashMapConfig(**c)
    dev = torch.device("cuda", torch.cuda.current_device())
    with torch.device(dev):
        model = FlashMapDraftModel(config).to(torch.bfloat16).eval()
    model.load_state_dict(synthetic_state_dict(config, seed=seed, dtype=torch.bfloat16, device=dev), strict=True)
    emb_w, head_w = synthetic_target_head(config, seed=seed, dtype=torch.bfloat16, device=dev)
    embed, head = nn.Embedding(*emb_w.shape, device=dev, dtype=torch.bfloat16), nn.Linear(1, 1, bias=False)
    embed.weight = nn.Parameter(emb_w, requires_grad=False)
    head.weight = nn.Parameter(head_w, requires_grad=False)
    return config, model, embed, head


def fill_contexts(config, model, embed, head, lengths: torch.Tensor, seed: int, num_steps: int = 1):
    """A cache of len(lengths) sequences whose contexts (N(0,1) conditioning
    rows, seeded) go through the varlen extend_context, and a DraftSession on it."""
    from flashmap_b200 import DraftSession, FlashMapCache

    dev = torch.device("cuda", torch.cuda.current_device())
    batch = int(lengths.numel())
    K = config.block_size
    cache = FlashMapCache(config, batch, int(lengths.max()) + K + 2, device=dev, dtype=torch.bfloat16)
    cu = torch.zeros(batch + 1, dtype=torch.int32)
    cu[1:] = torch.cumsum(lengths, 0)
    gd = torch.Generator(device=dev).manual_seed(seed + 6)
    width = len(config.target_layer_ids) * config.target_hidden_size
    rows = torch.randn(int(cu[-1]), width, generator=gd, device=dev).to(torch.bfloat16)
    model.extend_context_varlen(cache, rows, cu.to(dev), embed, head)
    del rows
    session = DraftSession(model, cache, embed, head, num_steps=num_steps, seed=seed)
    return cache, session


def build_batched(c: dict, batch: int, lo: int, hi: int, seed: int, num_steps: int):
    """A drafter with `batch` sequences whose contexts have ragged lengths
    uniform in [lo, hi] (seeded), filled through the varlen extend_context."""
    config, model, embed, head = build_model(c, seed)
    g = torch.Generator().manual_seed(seed + 5)
    lengths = torch.randint(lo, hi + 1, (batch,), generator=g)
    cache, session = fill_contexts(config, model, embed, head, lengths, seed, num_steps)
    return config, model, cache, session, lengths


# ------------------------------------------------------------------ config 5: 512 requests sharded by request

SHARD_REQUESTS = 512
SHARD_LENGTHS = (1024, 8192)
SHARD_CHUNK = 64


def shard_lengths() -> list:
    """The 512 context lengths of the config-5 workload (seeded, U[1024, 8192])."""
    g = torch.Generator().manual_seed(5)
    return torch.randint(SHARD_LENGTHS[0], SHARD_LENGTHS[1] + 1, (SHARD_REQUESTS,), generator=g).tolist()


def time_cross_attention(config, cache, reps: int = 20) -> dict:
    """The cross-attention kernel of one layer over a drafted chunk's cache, timed
    alone with CUDA events: the config-5 pass's dominant kernel (the K/V stream)."""
    from flashmap_b200 import _lib

    lib = _lib.load()
    L, _, Bc, H, T, hd = cache.kv.shape
    dev = cache.kv.device
    B = Bc
    nsplit = max(1, min((148 + B * H - 1) // (B * H), (T + 63) // 64))
    q = torch.randn(B * 16, H * hd, device=dev).to(torch.bfloat16)
    out = torch.empty_like(q)
    wsb = lib.fm_cross_attn_workspace_size(B, H, hd, nsplit)
    ws = torch.zeros(wsb, dtype=torch.uint8, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    p = lambda t: t.data_ptr()  # noqa: E731

    def launch(layer):
        _lib.call("fm_cross_attn", p(q), p(cache.kv), p(out), p(cache.lengths), B, H, hd, L, layer, Bc, T, nsplit,
                  p(ws), wsb, p(err), torch.cuda.current_stream().cuda_stream)

    for i in range(3):
        launch(i % L)
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for i in range(reps):
        launch(i % L)  # successive layers: each launch streams K/V rows not read by the one before
    b.record(stream)
    torch.cuda.synchronize()
    if int(err.item()) != 0:
        raise RuntimeError(f"cross-attention timing recorded device error {int(err.item())}")
    us = a.elapsed_time(b) / reps * 1000.0
    keys = int((cache.lengths.to(torch.int64) + 1).sum())
    nbytes = keys * H * hd * 2 * 2 + 2 * B * 16 * H * hd * 2
    return {"us": us, "bytes": nbytes}


def measure_sharded(args, world, rank, local) -> dict:
    """Config 5: 512 requests of the 27B map (contexts U[1024, 8192]) sharded by
    request over the ranks (LPT on context length with equal counts per rank),
    each rank drafting its share in chunks of <= 64 requests with one weight
    replica and no collective on the data path.  Per chunk: its contexts are
    filled (untimed), W warm-up replays, then K timed replays (CUDA events,
    barrier before), then K drafts through DraftSession.draft with host copies.
    A step drafts every request once: its time is the sum of the chunk times,
    the maximum over ranks."""
    from flashmap_b200 import _lib
    from flashmap_b200.sharding import balanced_capacity, chunks, lpt_assign, request_costs

    _lib.require_device()
    lengths = shard_lengths()
    shares = lpt_assign(request_costs(lengths), world, balanced_capacity(len(lengths), world))
    # chunks of similar lengths: less padding in each chunk's cache
    mine = sorted(shares[rank], key=lambda i: (lengths[i], i))
    config, model, embed, head = build_model(CONFIG5, seed=0)
    K = config.block_size
    stream = torch.cuda.current_stream()
    chunk_ms, e2e_ms, launches, h2d, d2h = [], [], 0, 0, 0
    xattn = None
    sampler = ClockSampler(physical_gpu_index(local))
    my_chunks = chunks(mine, SHARD_CHUNK)
    for ci, idx in enumerate(my_chunks):
        lens = torch.tensor([lengths[i] for i in idx])
        cache, session = fill_contexts(config, model, embed, head, lens, seed=1000 * rank + ci)
        for _ in range(args.warmup):
            session.replay()
        torch.cuda.synchronize()
        barrier(world)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(args.steps):
            session.replay()
        b.record(stream)
        torch.cuda.synchronize()
        chunk_ms.append(a.elapsed_time(b) / args.steps)
        launches += session.launches
        g = torch.Generator().manual_seed(7 + ci)
        anchors = torch.randint(0, config.vocab_size, (args.steps + 3, len(idx)), generator=g).pin_memory()
        for i in range(3):
            session.draft(anchors[args.steps + i])
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for i in range(args.steps):
            session.draft(anchors[i])
        e1.record(stream)
        torch.cuda.synchronize()
        e2e_ms.append(e0.elapsed_time(e1) / args.steps)
        h2d += len(idx) * 8
        d2h += len(idx) * K * 8
        session.plan.check_device_errors()
        if ci == len(my_chunks) - 1:
            xattn = time_cross_attention(config, cache)
        # the model's plans hold their caches: drop them before the next chunk's cache
        model._plans.clear()
        del session, cache
        torch.cuda.empty_cache()
    clocks = sampler.stop()
    step_ms = max_over_ranks(sum(chunk_ms), world)
    e2e_step_ms = max_over_ranks(sum(e2e_ms), world)
    peak_h, kind_h = measured_peak_hbm()
    peak_t, kind_t = measured_peak_tensor()
    flops = gemm_flops(CONFIG5, len(lengths))
    kv = float(sum(l + 1 for l in lengths) * CONFIG5["num_hidden_layers"] * 2 * CONFIG5["hidden_size"] * 2)
    total = SHARD_REQUESTS * K
    xa_gbs = xattn["bytes"] / (xattn["us"] * 1e-6) / 1e9
    ratio = profiled_traffic_ratio("cross_attention_config5.md")
    del model, embed, head
    torch.cuda.empty_cache()
    return {
        "value": total / (step_ms / 1000.0), "ms_per_step": step_ms, "chunk_ms": chunk_ms,
        "chunks_per_rank": len(my_chunks), "requests_per_rank": len(mine), "gpu_launches": launches * args.steps,
        "gpu_launches_per_step": launches, "clocks": clocks,
        "e2e": {"value": total / (e2e_step_ms / 1000.0), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "ms_per_step": e2e_step_ms,
                "api": "flashmap_b200.DraftSession.draft, one call per chunk"},
        "roofline": {"kernel": "cross_attn_kernel<128> (one layer over a 64-request chunk's context cache)",
                     "bound": "hbm", "achieved": xa_gbs, "peak": peak_h, "unit": "GB/s", "frac": xa_gbs / peak_h,
                     "peak_kind": f"{kind_h} (burst copy, kernel timed alone)",
                     "traffic": None if ratio is None else int(ratio * xattn["bytes"]),
                     "traffic_source": "profiles/cross_attention_config5.md: ncu DRAM bytes of an 8-request "
                                       "capture over its algorithmic bytes, times this launch's",
                     "launch_us": xattn["us"], "algorithmic_bytes": xattn["bytes"]},
        "pass_floor": {"kv_bytes": kv, "kv_floor_ms": kv / (peak_h * 1e9) * 1e3, "gemm_tflop": flops / 1e12,
                       "gemm_floor_ms": flops / (peak_t * 1e12) * 1e3,
                       "floor_ms_per_gpu": (kv / (peak_h * 1e9) + flops / (peak_t * 1e12)) * 1e3 / world,
                       "peak_kinds": [kind_h, kind_t]},
    }


def time_replays(session, steps: int, warmup: int, world: int) -> float:
    for _ in range(warmup):
        session.replay()
    torch.cuda.synchronize()
    barrier(world)
    stream = torch.cuda.current_stream()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(steps):
        session.replay()
    b.record(stream)
    torch.cuda.synchronize()
    return max_over_ranks(a.elapsed_time(b), world) / steps


def run_config3(args, world, rank, local):
    line = measure_config3(args, world, rank)
    if rank == 0:
        print(json.dumps(line), flush=True)


def measure_config3(args, world, rank):
    """Batched ragged drafting: config 3 (the config-2 map, 64 sequences
    per GPU, contexts U[512, 4096], one jump and two jumps) or config 5 (the
    27B map, SwiGLU and a state vocabulary, 64 requests per GPU — the per-GPU
    chunk of 512 requests over 8 GPUs — contexts U[1024, 8192], one jump).
    --profile-small keeps the GEMM shapes of config 3 (64 x 16 tokens) with 2
    layers, a 32768-row LM head and contexts U[64, 256], for ncu captures; with
    config5 it keeps the 27B map's cross-attention at its context lengths with
    8 requests and 2 layers (a 1.3 GB cache)."""
    from flashmap_b200 import _lib

    _lib.require_device()
    batch = 64
    five = args.workload == "config5"
    c = CONFIG5 if five else CONFIG2
    lo, hi = (1024, 8192) if five else (512, 4096)
    if args.profile_small and five:
        # the config-5 cross-attention at its real context lengths: 8 requests, 2 layers (a 1.3 GB cache)
        c = dict(CONFIG5, num_hidden_layers=2)
        batch = 8
    elif args.profile_small:
        c = dict(CONFIG2, num_hidden_layers=2, vocab_size=32768)
        lo, hi = 64, 256
    out = {}
    for steps_n in ((1,) if five or args.profile_small else (1, 2)):
        config, model, cache, session, lengths = build_batched(c, batch, lo, hi, seed=rank, num_steps=steps_n)
        ms = time_replays(session, args.steps, args.warmup, world)
        model._plans[next(iter(model._plans))].check_device_errors()
        out[steps_n] = (ms, lengths)
        del model, cache, session
        torch.cuda.empty_cache()
    ms1, lengths = out[1]
    ms2 = out[2][0] if 2 in out else None
    K = 16
    flops = gemm_flops(c, batch)
    kv = float(((lengths + 1).sum()) * c["num_hidden_layers"] * 2 * c["hidden_size"] * 2)
    peak_t, kind_t = measured_peak_tensor()
    peak_h, kind_h = measured_peak_hbm()
    achieved = flops / (ms1 / 1000.0) / 1e12
    name = "config5" if five else "config3"
    line = {
        "metric": "drafted tokens/sec (K=16), batch 64 ragged per GPU", "value": world * batch * K / (ms1 / 1000.0),
        "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms1,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": f"synthetic (seeded random-init {name} drafter, N(0,1) conditioning, context lengths U[{lo},{hi}])",
        "config": {"workload": (f"{name}: batch 64 ragged, K=16, one jump" + ("" if ms2 is None else
                                                                               " (and two jumps below)")
                                + (" [profile-small: 2 layers, 32768-row LM head]" if args.profile_small else "")),
                   "batch_per_gpu": batch, "context_mean": float(lengths.float().mean()), "launch": "kernel sequence"},
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak_t, "unit": "TFLOP/s",
                     "frac": achieved / peak_t, "peak_kind": kind_t, "gemm_tflop_per_pass": flops / 1e12,
                     "kv_bytes_per_pass": kv, "kv_floor_us": kv / (peak_h * 1e9) * 1e6,
                     "gemm_floor_us": flops / (peak_t * 1e12) * 1e6},
    }
    if ms2 is not None:
        line["two_jumps"] = {"ms_per_step": ms2, "value": world * batch * K / (ms2 / 1000.0), "unit": "tokens/s",
                             "ratio_to_one_jump": ms2 / ms1}
    return line


OPS_REF = os.path.join(os.path.dirname(os.path.abspath(__file__)), "baseline", "_ref")


def ops_cases(dev, sglang_kernels, vllm_kernels, ours: bool):
    """The serving operators at a serving batch of the config-2 map (64
    requests x 16 slots = 1024 token rows, 16 heads x 128, 8 layers; 4096 new
    context tokens into 16-token pages; greedy rows over a 151936-token
    vocabulary), seeded alike on both sides.  Returns name -> callable."""
    g = torch.Generator(device=dev).manual_seed(11)
    bf = torch.bfloat16
    T, H, hd, L, eps = 1024, 16, 128, 8, 1e-6
    rope = vllm_kernels.rope_table(4096, hd, 1e6, dev)  # each side's own table builder
    x = (2 * torch.randn(T, H, hd, generator=g, device=dev)).to(bf)
    w = (1 + 0.2 * torch.randn(hd, generator=g, device=dev)).to(bf)
    pos = torch.randint(0, 4096, (T,), generator=g, device=dev)
    qkv = torch.randn(T // 16, 16, 3, H, hd, generator=g, device=dev).to(bf)
    qn = (1 + 0.2 * torch.randn(hd, generator=g, device=dev)).to(bf)
    kn = (1 + 0.2 * torch.randn(hd, generator=g, device=dev)).to(bf)
    R, page = 4096, 16
    kv = torch.randn(R, L, 2, H, hd, generator=g, device=dev).to(bf)
    kvn = (1 + 0.2 * torch.randn(L, hd, generator=g, device=dev)).to(bf)
    caches = [torch.zeros(R // page + 8, H, page, 2 * hd, dtype=bf, device=dev) for _ in range(L)]
    ptrs = torch.tensor([c.data_ptr() for c in caches], dtype=torch.int64, device=dev)
    slots = torch.randperm(R + 8 * page, generator=g, device=dev)[:R]
    rpos = torch.randint(0, 4096, (R,), generator=g, device=dev)
    st = caches[0].stride()
    ang = torch.rand(64, 16, hd // 2, generator=g, device=dev) * 6.283
    freqs = torch.stack([ang.cos(), ang.sin()], -1).contiguous()
    xs = x.view(64, 16, H, hd)
    wf, qnf, knf = w.float(), qn.float(), kn.float()
    V = 151936
    logits = (3 * torch.randn(T, V, generator=g, device=dev)).to(bf)
    if ours:
        from flashmap_b200 import ops
        from flashmap_b200 import serving_ops as S

        return {
            "vllm rms_norm_rope (1024 x 16 x 128)": lambda: S.vllm_rms_norm_rope(x, w, rope, pos, eps),
            "vllm block_self_attention (64 blocks x 16, 16 x 128)": lambda: S.vllm_block_self_attention(
                qkv, qn, kn, rope, pos, eps),
            "vllm write_context_kv (4096 tokens x 8 layers, 16-token pages)": lambda: S.write_context_kv(
                kv, rpos, slots, kvn, rope, ptrs, (st[0], st[1], st[2], hd), page, eps),
            "sglang rms_norm_rope (64 x 16 x 16 x 128)": lambda: S.sglang_rms_norm_rope(xs, wf, freqs, eps),
            "sglang block_self_attention (64 blocks x 16, 16 x 128)": lambda: S.sglang_block_self_attention(
                qkv, qnf, knf, freqs, eps),
            "greedy rows (1024 x 151936)": lambda: ops.sample_rows(logits.view(1, T, V), None, 0.0, 0, 0),
        }
    temps = torch.ones(T, device=dev)
    greedy = torch.ones(T, dtype=torch.int32, device=dev)
    seed = torch.tensor(7, dtype=torch.int64, device=dev)
    vk, sk = vllm_kernels, sglang_kernels
    return {
        "vllm rms_norm_rope (1024 x 16 x 128)": lambda: vk.rms_norm_rope(x, w, rope, pos, eps),
        "vllm block_self_attention (64 blocks x 16, 16 x 128)": lambda: vk.block_self_attention(
            qkv, qn, kn, rope, pos, eps),
        "vllm write_context_kv (4096 tokens x 8 layers, 16-token pages)": lambda: vk.write_context_kv(
            kv, rpos, slots, kvn, rope, ptrs, (st[0], st[1], st[2], hd), page, eps),
        "sglang rms_norm_rope (64 x 16 x 16 x 128)": lambda: sk.rms_norm_rope(xs, wf, freqs, eps),
        "sglang block_self_attention (64 blocks x 16, 16 x 128)": lambda: sk.block_self_attention(
            qkv, qnf, knf, freqs, eps),
        "greedy rows (1024 x 151936)": lambda: sk.sample_rows(logits, temps, greedy, seed),
    }


def time_ops(cases, steps: int, warmup: int) -> dict:
    """Per operator: the time of one call through its Python entry (CUDA
    events around `steps` back-to-back calls after `warmup`; host dispatch
    included; the kernels' own device time comes from an ncu launch list of
    the same command)."""
    out = {}
    for name, fn in cases.items():
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(steps):
            fn()
        b.record()
        torch.cuda.synchronize()
        out[name] = {"call_us": a.elapsed_time(b) / steps * 1000.0}
    return out


def load_reference_module(sub: str, name: str):
    """A module of the reference's installed copy (baseline/_ref), loaded from
    its file: its package __init__ (plugin registration) is not run."""
    import importlib.util

    path = os.path.join(OPS_REF, "flashmap", sub, f"{name}.py")
    spec = importlib.util.spec_from_file_location(f"ref_{sub}_{name}", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def run_ops(args, world, rank, local):
    """The serving operators of flashmap_vllm / flashmap_sglang: this library's
    CUDA kernels beside the reference's own Triton kernels (the installed
    reference in baseline/_ref, run in a child process because both register
    the same torch.library names), same shapes and seeded inputs, each call
    through its Python entry on both sides."""
    if args.ops_side == "reference":
        vk, sk = load_reference_module("vllm", "kernels"), load_reference_module("sglang", "kernels")
        res = time_ops(ops_cases(torch.device("cuda", 0), sk, vk, ours=False), args.steps, args.warmup)
        print(json.dumps(res), flush=True)
        return
    from flashmap_b200 import _lib
    from flashmap_b200 import serving_ops as S

    _lib.require_device()
    ours = time_ops(ops_cases(torch.device("cuda", 0), None, S, ours=True), args.steps, args.warmup)
    ref, why = None, None
    if not os.path.isdir(os.path.join(OPS_REF, "flashmap")):
        why = "baseline/_ref holds no installed reference"
    else:
        p = subprocess.run([sys.executable, os.path.abspath(__file__), "--workload", "ops", "--ops-side", "reference",
                            "--steps", str(args.steps), "--warmup", str(args.warmup)], capture_output=True, text=True)
        lines = [l for l in p.stdout.splitlines() if l.startswith("{")]
        if p.returncode == 0 and lines:
            ref = json.loads(lines[-1])
        else:
            why = (p.stderr.strip().splitlines() or ["reference run failed"])[-1][:200]
    table = {}
    for name, o in ours.items():
        row = {"ours_call_us": o["call_us"]}
        r = (ref or {}).get(name)
        if r:
            row["reference_triton_call_us"] = r["call_us"]
            row["speedup"] = r["call_us"] / o["call_us"]
        table[name] = row
    ratios = [r["speedup"] for r in table.values() if "speedup" in r]
    geo = math.exp(sum(math.log(r) for r in ratios) / len(ratios)) if ratios else None
    line = {"metric": "serving operators: per-call speed-up over the reference's Triton kernels (geometric mean)",
            "value": geo, "unit": "x", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded)",
            "config": {"workload": "serving operators at 64 requests x 16 slots, config-2 map"}, "ops": table}
    if why:
        line["reference_unavailable"] = why
    print(json.dumps(line), flush=True)


def run_paged(args, world, rank, local):
    """The vLLM-layout paged cross-attention operator (flashmap_vllm::paged_cross_attention)
    at the config-2 map's shape: 64 requests x 16 query rows, 16 heads of 128,
    2048 context positions each in shuffled 16-token pages; HBM roofline on the
    K/V bytes (1.07 GB per call, larger than L2)."""
    from flashmap_b200 import _lib
    from flashmap_b200 import serving_ops as S

    _lib.require_device()
    R, H, hd, page, ctx = 64, 16, 128, 16, 2048
    dev = torch.device("cuda", torch.cuda.current_device())
    g = torch.Generator(device=dev).manual_seed(rank)
    cols = ctx // page
    cache = torch.randn(R * cols, H, page, 2 * hd, generator=g, device=dev).to(torch.bfloat16)
    table = torch.randperm(R * cols, generator=g, device=dev).view(R, cols).int()
    q = torch.randn(R * 16, H, hd, generator=g, device=dev).to(torch.bfloat16)
    cu = torch.arange(0, (R + 1) * 16, 16, dtype=torch.int32, device=dev)
    su = torch.full((R,), ctx, dtype=torch.int32, device=dev)

    def call():
        S.vllm_paged_cross_attention(q, cache, cu, su, table, None, None, 16, ctx, hd ** -0.5, 3)

    for _ in range(args.warmup):
        call()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        call()
    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()
    barrier(world)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(args.steps):
        graph.replay()
    b.record()
    torch.cuda.synchronize()
    us = max_over_ranks(a.elapsed_time(b), world) / args.steps * 1000.0
    del graph
    peak_h, kind_h = measured_peak_hbm()
    nbytes = R * ctx * H * hd * 2 * 2
    if rank != 0:
        return
    line = {
        "metric": "paged cross-attention (vLLM layout), us per call", "value": us, "unit": "us", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": us / 1000.0, "higher_is_better": False,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,1) cache and queries)",
        "config": {"workload": "paged: 64 requests x 16 queries, 16 heads x 128, ctx 2048, 16-token pages, shuffled",
                   "timing": "CUDA-graph replays (workspace allocation included), inputs larger than L2"},
        "roofline": {"bound": "hbm", "achieved": nbytes / (us * 1e-6) / 1e9, "peak": peak_h, "unit": "GB/s",
                     "frac": nbytes / (us * 1e-6) / 1e9 / peak_h, "peak_kind": kind_h, "algorithmic_bytes": nbytes},
    }
    print(json.dumps(line), flush=True)


def run_config4(args, world, rank, local):
    line = measure_config4(args, world, rank)
    if rank == 0:
        print(json.dumps(line), flush=True)


def measure_config4(args, world, rank):
    """Acceptance (config 4): target logits (64, 17, 151936) bf16 ~ N(0, 2^2),
    drafted tokens U[0, V), draft probabilities softmax(N(0,1)); greedy and
    rejection at T = 1 with Philox seed 1234."""
    import ctypes

    from flashmap_b200 import _lib

    _lib.require_device()
    lib = _lib.load()
    B, K, V = 64, 16, 151936
    dev = torch.device("cuda", torch.cuda.current_device())
    g = torch.Generator(device=dev).manual_seed(1234 + rank)
    target = (2.0 * torch.randn(B, K + 1, V, generator=g, device=dev)).to(torch.bfloat16)
    draft = torch.randint(0, V, (B, K), generator=g, device=dev)
    q = torch.softmax(torch.randn(B, K, V, generator=g, device=dev), -1)
    acc = torch.empty(B, dtype=torch.int64, device=dev)
    bonus = torch.empty_like(acc)
    wsb = lib.fm_accept_workspace_size(B, K)
    ws = torch.empty(wsb, dtype=torch.uint8, device=dev)
    p = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731

    def greedy():
        cur = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        _lib.check(lib.fm_accept_greedy(p(target), 0, p(draft), B, K, V, p(acc), p(bonus), p(ws), wsb, cur),
                   "fm_accept_greedy")

    def rejection():
        cur = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        _lib.check(lib.fm_accept_rejection(p(target), 0, p(draft), p(q), B, K, V, ctypes.c_float(1.0),
                                           ctypes.c_uint64(1234), ctypes.c_uint32(0), p(acc), p(bonus), p(ws), wsb,
                                           cur), "fm_accept_rejection")

    res = {}
    for name, fn in (("greedy", greedy), ("rejection", rejection)):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        # each call captured in a CUDA graph, so the timing is the device's and
        # not the host's ctypes round trip
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            fn()
        for _ in range(args.warmup):
            graph.replay()
        torch.cuda.synchronize()
        barrier(world)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(args.steps):
            graph.replay()
        b.record()
        torch.cuda.synchronize()
        res[name] = max_over_ranks(a.elapsed_time(b), world) / args.steps * 1000.0  # us
        del graph
    peak_h, kind_h = measured_peak_hbm()
    bytes_g = B * (K + 1) * V * 2
    bytes_r = bytes_g + B * V * 4
    line = {
        "metric": "acceptance of a (64 x 17 x 151936) block, us per call (greedy)", "value": res["greedy"],
        "unit": "us", "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": res["greedy"] / 1000,
        "higher_is_better": False, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded: logits 2*N(0,1), draft tokens U[0,V), Q = softmax(N(0,1)))",
        "config": {"workload": "config4: acceptance, B=64, K+1=17, V=151936, T=0 and T=1 (Philox seed 1234)"},
        "roofline": {"bound": "hbm", "achieved": bytes_g / (res["greedy"] * 1e-6) / 1e9, "peak": peak_h,
                     "unit": "GB/s", "frac": bytes_g / (res["greedy"] * 1e-6) / 1e9 / peak_h, "peak_kind": kind_h,
                     "algorithmic_bytes": bytes_g, "floor_us": bytes_g / (peak_h * 1e9) * 1e6},
        "rejection": {"us": res["rejection"], "algorithmic_bytes": bytes_r,
                      "achieved_gbs": bytes_r / (res["rejection"] * 1e-6) / 1e9,
                      "frac": bytes_r / (res["rejection"] * 1e-6) / 1e9 / peak_h,
                      "floor_us": bytes_r / (peak_h * 1e9) * 1e6},
    }
    return line


# ------------------------------------------------------------------ our arm

def run_ours(args, world, rank, local):
    """The config-2 batch-1 line alone (``--workload config2``)."""
    line = measure_batch1(args, world, rank, local)
    if world == 1 and not args.no_cpu_baseline and not args.profile_small:
        ref = cpu_reference(CONFIG2, CONTEXT, seconds=args.cpu_seconds)
        line["cpu_baseline"] = {k: ref[k] for k in ("value", "unit", "cores", "kind", "sample")}
    if rank == 0:
        print(json.dumps(line), flush=True)


def measure_batch1(args, world, rank, local):
    """The config-2 pass, batch 1 per rank (every rank drafts its own request)."""
    from flashmap_b200 import _lib

    _lib.require_device()
    config, model, cache, session = build_workload(seed=rank, small=args.profile_small, launch=args.launch)
    K = config.block_size
    stream = torch.cuda.current_stream()
    for _ in range(args.warmup):
        session.replay()
    torch.cuda.synchronize()
    launches = session.launches
    barrier(world)
    torch.cuda.synchronize()
    sampler = ClockSampler(physical_gpu_index(local))
    time.sleep(0.4)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(args.steps):
        session.replay()
    end.record(stream)
    torch.cuda.synchronize()
    clocks = sampler.stop()
    barrier(world)
    elapsed_ms = max_over_ranks(start.elapsed_time(end), world)
    ms_per_step = elapsed_ms / args.steps
    value = world * K * args.steps / (elapsed_ms / 1000.0)
    model._plans[next(iter(model._plans))].check_device_errors()

    # end to end through the public API: H2D anchor, replay, D2H tokens, every step
    e2e_steps = max(args.steps // 4, 10)
    anchors = torch.randint(0, config.vocab_size, (e2e_steps,), generator=torch.Generator().manual_seed(7))
    anchors = anchors.pin_memory()
    for i in range(5):
        session.draft(anchors[i : i + 1])
    barrier(world)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(e2e_steps):
        session.draft(anchors[i : i + 1])
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1), world)
    e2e_value = world * K * e2e_steps / (e2e_ms / 1000.0)

    # the dominant kernel: the LM-head GEMM (V x Ht weight stream) timed alone
    plan = session.plan
    for _ in range(3):
        plan.lm_head()
    torch.cuda.synchronize()
    n_lm = 50
    k0, k1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    k0.record(stream)
    for _ in range(n_lm):
        plan.lm_head()
    k1.record(stream)
    torch.cuda.synchronize()
    lm_ms = k0.elapsed_time(k1) / n_lm
    nbytes = algorithmic_bytes(PROFILE_SMALL if args.profile_small else CONFIG2, CONTEXT)
    peak, peak_kind = measured_peak_hbm()
    lm_gbs = nbytes["lm_head"] / (lm_ms / 1000.0) / 1e9
    pass_gbs = nbytes["total"] / (ms_per_step / 1000.0) / 1e9

    # the serving plugins' fast modes (changes rounding, outside parity), the same
    # draft reported beside the headline: the DiT head folded into the LM-head
    # rows, then that plus the eigen-folded noise
    folded = folded_all = None
    if not args.profile_small:
        from flashmap_b200 import DraftSession

        def time_folds(fold_head: bool, fold_noise: bool) -> float:
            # the folds run as the kernel sequence (the streamed pass serves the unfolded head)
            model.fold_head, model.fold_noise = fold_head, fold_noise
            mode, model.launch_mode = model.launch_mode, ("kernels" if model.launch_mode == "stream" else model.launch_mode)
            try:
                fsession = DraftSession(model, cache, session.embed_tokens, session.lm_head, num_steps=1, seed=rank)
            finally:
                model.launch_mode = mode
            for _ in range(args.warmup):
                fsession.replay()
            torch.cuda.synchronize()
            barrier(world)
            f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            f_steps = max(args.steps // 4, 10)
            f0.record(stream)
            for _ in range(f_steps):
                fsession.replay()
            f1.record(stream)
            torch.cuda.synchronize()
            model.fold_head = model.fold_noise = False
            del fsession
            return max_over_ranks(f0.elapsed_time(f1), world) / f_steps

        c2 = CONFIG2
        fbytes = nbytes["total"] - nbytes["lm_head"] - c2["target_hidden_size"] * c2["hidden_size"] * 2 \
            + c2["vocab_size"] * c2["hidden_size"] * 2
        f_ms = time_folds(True, False)
        folded = {"ms_per_step": f_ms, "value": world * K / (f_ms / 1000.0), "unit": "tokens/s",
                  "algorithmic_bytes": fbytes, "hbm_frac": fbytes / (f_ms / 1000.0) / 1e9 / peak,
                  "note": "fold_head fast mode (vllm/fold.py:76-100): outside parity with the HF path"}
        # the noise fold drops the [Ht, Ht] Cholesky factor (its [D, Ht] weight replaces x_embed's)
        abytes = fbytes - c2["target_hidden_size"] ** 2 * 2
        a_ms = time_folds(True, True)
        folded_all = {"ms_per_step": a_ms, "value": world * K / (a_ms / 1000.0), "unit": "tokens/s",
                      "algorithmic_bytes": abytes, "hbm_frac": abytes / (a_ms / 1000.0) / 1e9 / peak,
                      "note": "fold_head + fold_noise fast mode (vllm/fold.py:44-100, sglang/model.py:945-958): "
                              "outside parity with the HF path"}

    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded random-init config-2 drafter weights and target head, N(0,1) conditioning)",
        "config": workload_config(args, world),
        "pass_us": ms_per_step * 1000.0,
        "pass_roofline": {"bound": "hbm", "algorithmic_bytes": nbytes["total"], "achieved": pass_gbs, "peak": peak,
                          "unit": "GB/s", "frac": pass_gbs / peak, "peak_kind": peak_kind,
                          "floor_us": nbytes["total"] / (peak * 1e9) * 1e6},
        "roofline": {"kernel": "LM-head GEMM (tcgen05, 151936 x 4096 bf16 weight stream, N=16 tokens)",
                     "bound": "hbm", "achieved": lm_gbs, "peak": peak, "unit": "GB/s", "frac": lm_gbs / peak,
                     "peak_kind": f"{peak_kind} (burst copy, kernel timed alone)", "traffic": profiled_traffic(),
                     "launch_us": lm_ms * 1000.0, "algorithmic_bytes": nbytes["lm_head"]},
        "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": 8, "d2h_bytes_per_step": 8 * K,
                "ms_per_step": e2e_ms / e2e_steps, "api": "flashmap_b200.DraftSession.draft"},
        "gpu_launches": launches * args.steps,
        "gpu_launches_per_step": launches,
        "clocks": clocks,
    }
    if folded is not None:
        line["fast_mode_folded_head"] = folded
        line["fast_mode_folded_head_and_noise"] = folded_all
    del session, cache, model
    torch.cuda.empty_cache()
    return line


def run_all(args, world, rank, local):
    """The default line: config 5's 512 requests sharded over the ranks (the
    headline tokens/s), the config-2 batch-1 pass beside it (``pass_us``,
    ``batch1``), and at N = 1 configs 3 and 4 and the CPU baselines."""
    b1 = measure_batch1(args, world, rank, local)
    sh = measure_sharded(args, world, rank, local)
    extra = {}
    if world == 1:
        extra["config3"] = measure_config3(args, world, rank)
        extra["config4"] = measure_config4(args, world, rank)
    if rank != 0:
        return
    line = {
        "metric": METRIC, "value": sh["value"], "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": sh["ms_per_step"], "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded random-init config-5 and config-2 drafters and target heads, N(0,1) conditioning)",
        "config": workload_config(args, world),
        "e2e": sh["e2e"], "gpu_launches": sh["gpu_launches"], "gpu_launches_per_step": sh["gpu_launches_per_step"],
        "clocks": sh["clocks"], "roofline": sh["roofline"],
        "sharding": {"requests": SHARD_REQUESTS, "requests_per_rank": sh["requests_per_rank"],
                     "chunks_per_rank": sh["chunks_per_rank"], "chunk_ms_rank0": sh["chunk_ms"],
                     "pass_floor": sh["pass_floor"]},
        "pass_us": b1["pass_us"], "pass_roofline": b1["pass_roofline"],
        "batch1": {k: b1[k] for k in ("value", "ms_per_step", "pass_us", "e2e", "roofline", "clocks",
                                      "gpu_launches_per_step", "fast_mode_folded_head",
                                      "fast_mode_folded_head_and_noise") if k in b1},
    }
    line["batch1"]["workload"] = "config2: Qwen3-8B-sized drafter pass, batch 1 per GPU, K=16, ctx 2048, 1 jump"
    line.update(extra)
    if world == 1 and not args.no_cpu_baseline:
        ref = cpu_reference(CONFIG5, shard_context_median(), seconds=args.cpu_seconds, label="config-5")
        line["cpu_baseline"] = {k: ref[k] for k in ("value", "unit", "cores", "kind", "sample")}
        ref2 = cpu_reference(CONFIG2, CONTEXT, seconds=args.cpu_seconds)
        line["batch1"]["cpu_baseline"] = {k: ref2[k] for k in ("value", "unit", "cores", "kind", "sample")}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--launch", choices=["auto", "kernels", "stream"], default="auto",
                    help="launch structure of a draft: the kernel sequence (kernels), the streamed "
                         "single-launch pass (stream), or the library's choice (auto)")
    ap.add_argument("--workload", choices=["all", "config2", "config3", "config4", "config5", "paged", "ops"],
                    default="all",
                    help="all (the default line: config 5's 512 requests sharded over the GPUs, with the config-2 "
                         "batch-1 pass and, on one GPU, configs 3 and 4 beside it), config2 (batch 1 alone), "
                         "config3 (batch 64 ragged), config4 (acceptance), config5 (one 64-request chunk), "
                         "paged (vLLM paged cross-attention operator), ops (the serving operators beside the "
                         "reference's Triton kernels)")
    ap.add_argument("--ops-side", choices=["ours", "reference"], default="ours", help=argparse.SUPPRESS)
    ap.add_argument("--profile-small", action="store_true",
                    help="2 layers and a 32768-row LM head: the same kernels on < 2 GB, for ncu captures")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be at least 3")
    world, rank, local = dist_setup() if args.impl == "ours" else (int(os.environ.get("WORLD_SIZE", "1")),
                                                                   int(os.environ.get("RANK", "0")), 0)
    try:
        if args.impl == "reference":
            run_reference(args, world, rank)
        elif args.workload == "all" and not args.profile_small:
            run_all(args, world, rank, local)
        elif args.workload in ("config3", "config5"):
            run_config3(args, world, rank, local)
        elif args.workload == "paged":
            run_paged(args, world, rank, local)
        elif args.workload == "ops":
            run_ops(args, world, rank, local)
        elif args.workload == "config4":
            run_config4(args, world, rank, local)
        else:
            run_ours(args, world, rank, local)
    finally:
        if args.impl == "ours" and world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
