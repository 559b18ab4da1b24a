#!/usr/bin/env python
"""Benchmark of the B200 verify + accept round (benchmark config 3).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--batch 64] [--ctx 1000]

A step is one verify + accept round of a speculative decoder on a random-init Qwen3-8B-architecture target
(36 layers, hidden 4096, 32/8 heads of 128, FFN 12288, vocab 151936, bf16): B = 64 rows x (k = 7 drafts + 1)
verified positions over ~1000-token contexts in a paged KV cache (256-slot blocks, random block permutation),
the drafts and their q from a temperature-1 random-logit drafter.  The round is the target's verification
forward + LM head (one CUDA graph: cuBLAS GEMMs, this package's fused norm / RoPE / KV-store kernels and the
tcgen05 paged attention) followed by the fused sampler accepting straight from the bf16 logits with in-kernel
draws.  Data is synthetic; weights, the KV cache and the logits exceed L2 on every step (no flush needed).

One JSON line on rank 0: value = accepted tokens / s over all ranks (device-resident inputs), e2e = the same
through the public round API with the step's metadata copied from pinned host memory and the result read back,
plus the dominant kernel's roofline (paged attention, timed live with CUDA events), clocks sampled during the
timed region, and the CPU oracle baseline.  --impl reference runs the reference's algorithm for the path on
the host cores (the numpy oracle in oracle/, the reference being pure Python/ATen) on a bounded sample.
Multi-GPU (torchrun): every rank runs its own replica of 64 rows (weak scaling, no collective on the path).
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "nano-vllm-speculative-decoding_b200"))
sys.path.insert(0, str(ROOT))

V = 151936
K_DRAFTS = 7
METRIC = "verify+accept round: accepted tok/s at B=64, k=7 (8 verify positions)"


def parse_args():
    p = argparse.ArgumentParser(description=__doc__)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=100)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--batch", type=int, default=64)
    p.add_argument("--ctx", type=int, default=1000, help="mean context length (tokens before the verified ones)")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--kernel", choices=["attention", "accept", "accept_topk", "accept_greedy", "sample", "markov",
                                        "ctx_store", "after_verify", "attention_tp"],
                   default=None,
                   help="time one kernel alone on its benchmark config (attention: config 2, accept: config 3's "
                        "logits) instead of the round; used for profiling")
    return p.parse_args()


def peaks() -> dict:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return {"hbm_gbs": data["hbm_gbs"], "source": "measured"}
    return {"hbm_gbs": 6650.0, "source": "fallback"}


# ---------------------------------------------------------------------------------------------- clocks
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "200", "-i", str(self.index)], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
        except (OSError, ValueError):
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [line for line in out.splitlines() if line.strip()]
        return False

    def summary(self) -> dict:
        rows = []
        for line in self.lines:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append((float(parts[1]), float(parts[2]), float(parts[3]), parts[5:9]))
            except ValueError:
                continue
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        loaded = [r for r in rows if r[2] > 250.0] or rows
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in loaded for i, flag in enumerate(r[3]) if flag.lower().startswith("active")})
        return {"sm_mhz": statistics.median(r[0] for r in loaded), "sm_max_mhz": max(r[1] for r in loaded),
                "reasons": reasons, "samples": len(loaded)}


# ---------------------------------------------------------------------------------------------- workload
def build_workload(torch, device, batch: int, ctx: int, seed: int):
    from nanovllm_b200 import spec_sampler as S
    from nanovllm_b200.batch_metadata import RowState
    from nanovllm_b200.speculative import VerifyRound
    from nanovllm_b200.target import Qwen3Shape, Qwen3Target
    from types import SimpleNamespace

    shape = Qwen3Shape()
    block_size = 256
    gen = torch.Generator().manual_seed(seed)
    lengths = (torch.randint(ctx - 50, ctx + 51, (batch,), generator=gen) if ctx > 100
               else torch.full((batch,), ctx)).tolist()
    # each row holds its context plus the k + 1 verified positions
    blocks_per_row = [math.ceil((n + K_DRAFTS) / block_size) for n in lengths]
    num_blocks = sum(blocks_per_row) + 8
    width = max(blocks_per_row)
    perm = torch.randperm(num_blocks, generator=gen).tolist()
    target = Qwen3Target(shape, device, num_blocks, block_size, seed=seed)
    # the prompts' K/V (random, as from ~1000 random prompt ids); the pad block stays zero
    kv = target.kv_cache
    for layer in range(shape.layers):
        kv[:, layer, :num_blocks].normal_(generator=torch.Generator(device=device).manual_seed(seed + layer))
    rows, used = [], 0
    for n, nb in zip(lengths, blocks_per_row):
        rows.append(RowState(length=n, last_token=int(torch.randint(V, (1,), generator=gen)),
                             block_table=perm[used:used + nb]))
        used += nb
    rnd = VerifyRound(target, K_DRAFTS, [batch], width)
    dgen = torch.Generator(device=device).manual_seed(seed + 1)
    draft_logits = torch.randn(batch, K_DRAFTS, V, device=device, generator=dgen)
    sampling = S.sampling_tensors([SimpleNamespace(temperature=1.0, top_k=0, top_p=1.0)] * batch, device)
    q = S.probs_from_logits(draft_logits, sampling)                   # temperature-1 random-logit drafter
    drafts = S.sample(q, dgen)
    del draft_logits
    return SimpleNamespace(target=target, round=rnd, rows=rows, q=q, drafts=drafts, sampling=sampling,
                           lengths=lengths, width=width, shape=shape)


CFG2_TRAFFIC_BYTES = 141_530_624       # 136.830976 MB read + 4.699648 MB written, one launch
CFG2_ALGORITHMIC_BYTES = 135_319_552


def time_events(torch, fn, iters: int) -> float:
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    start.record()
    for _ in range(iters):
        fn()
    end.record()
    torch.cuda.synchronize()
    return start.elapsed_time(end) / iters * 1e3   # us


def attention_roofline(torch, w, hbm_peak: float) -> dict:
    """The dominant kernel of this package in a round: paged verify attention, 36 launches per round.  Timed
    live over every layer's cache (each launch reads a different 262 MB of K/V, beyond L2), as one CUDA graph of
    the 36 launches replayed (like the round's own graph)."""
    from nanovllm_b200 import attention
    t = w.target
    num_tokens = w.q.shape[0] * (K_DRAFTS + 1)
    graph, buffers = t.graphs[num_tokens]
    s = w.shape
    q = torch.randn(num_tokens, s.heads, s.head_dim, device=t.device).bfloat16()
    out = torch.empty_like(q)
    scale = s.head_dim ** -0.5

    def one_layer(layer):
        attention.paged_attention(q, t.kv_cache[0, layer], t.kv_cache[1, layer], buffers["block_tables"], scale,
                                  cu_seqlens_q=buffers["cu_seqlens_q"], cu_seqlens_k=buffers["cu_seqlens_k"],
                                  max_seqlen_q=K_DRAFTS + 1, out=out)

    def all_layers():
        for layer in range(s.layers):
            one_layer(layer)

    all_layers()                                   # warm-up (allocates the split workspace)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()                 # the 36 launches replayed as in the round: no host gaps
    with torch.cuda.graph(graph):
        all_layers()
    graph.replay()
    # five timings of 5 replays each; the median, so that one disturbed timing (seen as +10 us per launch now
    # and then) does not stand for the kernel
    samples = [time_events(torch, graph.replay, 5) / s.layers for _ in range(5)]
    per_launch_us = statistics.median(samples)
    keys = sum(n + K_DRAFTS for n in w.lengths)       # row r verifies positions len-1 .. len+6
    kv_bytes = keys * s.kv_heads * s.head_dim * 2 * 2
    qo_bytes = 2 * num_tokens * s.heads * s.head_dim * 2
    algorithmic = kv_bytes + qo_bytes
    achieved = algorithmic / (per_launch_us * 1e-6) / 1e9
    # DRAM traffic from one ncu capture of the config-2 launch (141.53 MB read + written for 135.32 MB
    # algorithmic), scaled to this launch by its algorithmic bytes (traffic grows with the keys)
    traffic = round(algorithmic * CFG2_TRAFFIC_BYTES / CFG2_ALGORITHMIC_BYTES)
    return {"kernel": "specdec::attention::verify_attention_kernel<4>", "bound": "hbm",
            "achieved": round(achieved, 1), "peak": hbm_peak, "unit": "GB/s",
            "frac": round(achieved / hbm_peak, 4), "traffic": traffic,
            "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of config 2, scaled by keys",
            "algorithmic_bytes_per_launch": algorithmic, "us_per_launch": round(per_launch_us, 2),
            "us_per_launch_samples": [round(x, 2) for x in samples],
            "timing": "median of 5 timings of 5 graph replays of the 36 layers' launches",
            "launches_per_step": s.layers}


def accept_timing(torch, w) -> dict:
    from nanovllm_b200 import spec_sampler as S
    num_tokens = w.q.shape[0] * (K_DRAFTS + 1)
    logits = w.target.graphs[num_tokens][1]["logits"]
    gen = torch.Generator(device=logits.device).manual_seed(3)
    us = statistics.median(time_events(torch, lambda: S.accept_from_logits(logits, w.q, w.drafts, w.sampling, None,
                                                                            gen), 20) for _ in range(3))
    batch = w.q.shape[0]
    algorithmic = logits.numel() * 2 + batch * V * (4 + 2)    # logits once + q and logits of the tail rows
    return {"us": round(us, 2), "algorithmic_bytes": algorithmic,
            "GBps": round(algorithmic / (us * 1e-6) / 1e9, 1)}


# ---------------------------------------------------------------------------------------------- CPU side
def cpu_round_sample(rows_sample: int, layers_sample: int, ctx: int, threads: int):
    """The reference's algorithm for the path on CPU (numpy oracle): paged attention of `rows_sample` rows over
    `layers_sample` layers and the sampler (probs_from_logits + accept_random) of the same rows; returns the
    seconds it took and the work it covered."""
    import numpy as np
    from oracle import attention as OA
    from oracle import spec_sampler as OS
    rng = np.random.default_rng(0)
    H, Hkv, D, bs = 32, 8, 128, 256
    nb = math.ceil((ctx + 8) / bs)
    k_cache = rng.standard_normal((rows_sample * nb, bs, Hkv, D), dtype=np.float32)
    v_cache = rng.standard_normal((rows_sample * nb, bs, Hkv, D), dtype=np.float32)
    tables = np.arange(rows_sample * nb).reshape(rows_sample, nb)
    q = rng.standard_normal((rows_sample * 8, H, D), dtype=np.float32)
    starts = np.arange(rows_sample) * 8
    logits = (rng.standard_normal((rows_sample * 8, V), dtype=np.float32) * 3).astype(np.float32)
    qd = OS.softmax(rng.standard_normal((rows_sample, 7, V), dtype=np.float32))
    drafts = rng.integers(0, V, (rows_sample, 7))
    u = rng.random((rows_sample, 7), dtype=np.float32)
    noise = OS.clamp_noise(rng.exponential(size=(rows_sample, V)).astype(np.float32))
    t0 = time.perf_counter()
    for _ in range(layers_sample):
        OA.paged_attention(q, k_cache, v_cache, tables, starts, [8] * rows_sample, [ctx + 8] * rows_sample, D ** -0.5)
    t1 = time.perf_counter()
    p = OS.probs_from_logits(logits, np.ones(rows_sample * 8, np.float32))
    n_accept, _tail = OS.accept_random(p.reshape(rows_sample, 8, V), qd, drafts, u, noise)
    t2 = time.perf_counter()
    return {"attn_s": t1 - t0, "accept_s": t2 - t1, "rows": rows_sample, "layers": layers_sample,
            "tokens_per_row": float(n_accept.mean() + 1)}


def cpu_round_seconds(sample: dict, batch: int, layers: int) -> float:
    per_row_layer = sample["attn_s"] / (sample["rows"] * sample["layers"])
    per_row_accept = sample["accept_s"] / sample["rows"]
    return batch * layers * per_row_layer + batch * per_row_accept


def _cpu_task(ctx: int) -> dict:
    """One reference-arm task in a worker process: four rows through two layers' attention plus their sampler."""
    from threadpoolctl import threadpool_limits
    with threadpool_limits(1):
        return cpu_round_sample(4, 2, ctx, 1)


def _cpu_warm(ctx: int) -> None:
    _cpu_task(ctx)               # first-call costs (imports, page faults) stay out of the timed tasks


def run_reference(args) -> int:
    """--impl reference: the reference's algorithm for the path (numpy oracle) on every host core, rank 0 only.
    A process pool (one single-threaded worker per core, spawned, each warmed up once) runs each step as one task
    per worker: four rows through two layers' paged attention plus those rows' sampler.  The whole job of the
    config (batch x n_gpus rows, 36 layers) is costed from the step's per-task times and the pool's measured
    parallelism; the host has the same cores whatever the GPU count, so the whole-job time grows with the rows.
    Steps beyond 10 are not run (the median of 10 bounded samples already settles)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    import concurrent.futures as cf
    import multiprocessing as mp
    workers = os.cpu_count() or 1
    os.environ.setdefault("OMP_NUM_THREADS", "1")
    rows = args.batch * args.gpus
    values, round_times, par, tasks = [], [], [], 0
    with cf.ProcessPoolExecutor(max_workers=workers, mp_context=mp.get_context("spawn"), initializer=_cpu_warm,
                                initargs=(args.ctx,)) as pool:
        for _ in range(max(1, min(args.steps, 10))):
            t0 = time.perf_counter()
            results = list(pool.map(_cpu_task, [args.ctx] * workers))
            wall = time.perf_counter() - t0
            tasks += len(results)
            attn = statistics.mean(r["attn_s"] / (r["rows"] * r["layers"]) for r in results)   # per row, layer
            accept = statistics.mean(r["accept_s"] / r["rows"] for r in results)               # per row
            parallelism = sum(r["attn_s"] + r["accept_s"] for r in results) / wall
            round_s = rows * (36 * attn + accept) / parallelism
            tokens = rows * statistics.mean(r["tokens_per_row"] for r in results)
            values.append(tokens / round_s)
            round_times.append(round_s)
            par.append(parallelism)
    value = statistics.median(values)
    line = {"impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "tok/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(statistics.median(round_times) * 1e3, 1),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "config": {"workload": "cfg3 round path on CPU (numpy oracle)", "global_batch": rows,
                                             "seq_len": args.ctx, "parallelism": f"cpu x{workers} processes"},
            "cpu_baseline": {"value": round(value, 3), "unit": "tok/s", "cores": workers, "kind": "port",
                             "sample": f"{tasks} tasks of 4 rows x 2 layers of paged attention at ctx {args.ctx} + "
                                       f"those rows' sampler on {workers} single-threaded processes (median "
                                       f"parallelism {statistics.median(par):.1f}), costed to {rows} rows x 36 "
                                       f"layers; GEMMs excluded"},
            "e2e": {"value": round(value, 3), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------------------------- one kernel
def run_kernel(args) -> int:
    """Times one kernel alone (CUDA events, W warm-up launches, K timed launches) on its benchmark config:
    attention = config 2 (32 rows x 8 queries, contexts U[900, 1100], 32/8 heads, random block permutation);
    accept = config 3's fused accept (64 rows x 8 positions of bf16 logits, temperature 1, in-kernel draws)."""
    import torch
    from types import SimpleNamespace
    device = torch.device("cuda", 0)
    g = torch.Generator().manual_seed(0)
    if args.kernel == "attention":
        from nanovllm_b200 import attention
        R, H, Hkv, D, bs = 32, 32, 8, 128, 256
        k_lens = torch.randint(900, 1101, (R,), generator=g).tolist()
        nb = [math.ceil(k / bs) for k in k_lens]
        NB = sum(nb) + 1
        perm = torch.randperm(NB - 1, generator=g).tolist()
        tables = torch.full((R, max(nb)), NB - 1, dtype=torch.int32)
        used = 0
        for r, n in enumerate(nb):
            tables[r, :n] = torch.tensor(perm[used:used + n])
            used += n
        copies = 4      # distinct caches so consecutive launches read beyond L2
        caches = [(torch.randn(NB, bs, Hkv, D, device=device).bfloat16(),
                   torch.randn(NB, bs, Hkv, D, device=device).bfloat16()) for _ in range(copies)]
        q = torch.randn(R * 8, H, D, device=device).bfloat16()
        cu_q = torch.arange(0, 8 * R + 1, 8, dtype=torch.int32, device=device)
        cu_k = torch.tensor([0] + torch.tensor(k_lens).cumsum(0).tolist(), dtype=torch.int32, device=device)
        tables = tables.to(device)
        state = {"i": 0}

        def fn():
            kc, vc = caches[state["i"] % copies]
            state["i"] += 1
            attention.paged_attention(q, kc, vc, tables, D ** -0.5, cu_seqlens_q=cu_q, cu_seqlens_k=cu_k,
                                      max_seqlen_q=8)
        algorithmic = sum(k_lens) * Hkv * D * 2 * 2 + 2 * R * 8 * H * D * 2
    elif args.kernel == "markov":
        # config 4's drafter: 64 rows x 7 in-block steps, V = 151936, rank-256 Markov head, top_k 128 (192 candidates)
        from nanovllm_b200 import spec_sampler as S
        from nanovllm_b200.markov import MarkovHeadWeights, MarkovQBuffer, markov_rows, num_candidates
        B, k, r = 64, 7, 256
        gg = torch.Generator(device=device).manual_seed(0)
        logits = (torch.randn(B, k, V, device=device, generator=gg) * 2).bfloat16()
        head = MarkovHeadWeights((torch.randn(V, r, device=device, generator=gg) * 0.1).bfloat16(),
                                 (torch.randn(V, r, device=device, generator=gg) * 0.1).bfloat16())
        samp = S.sampling_tensors([SimpleNamespace(temperature=1.0, top_k=128, top_p=1.0)] * B, device)
        cand = num_candidates(samp.max_top_k, samp.all_top_k, V)
        noise = torch.empty(B, k, cand, device=device).exponential_(generator=gg).clamp_min_(1e-10)
        prev = torch.randint(V, (B,), device=device, generator=gg)
        drafts = torch.empty(B, k, dtype=torch.int64, device=device)
        qbuf = MarkovQBuffer(B, k, V, cand, device)     # persistent q: only the last call's candidates cleared

        def fn():
            markov_rows(logits, prev, samp, noise, drafts, qbuf, cand, head)
        # per step: W2 (77.8 MB) + the row's logits (19.4 MB); q is scattered (C values per row), not zero-filled
        algorithmic = k * (V * r * 2 + B * V * 2)
    elif args.kernel == "ctx_store":
        # config 4's ctx_store: T = 288 verified tokens, 5 draft layers, hidden 4096, 8 KV heads of 128
        from nanovllm_b200.dflash import store_context_kv
        from nanovllm_b200.fused import rope_cache
        T, layers, hidden, hkv, bs = 288, 5, 4096, 8, 256
        gg = torch.Generator(device=device).manual_seed(0)
        features = torch.randn(T, hidden, device=device, generator=gg).bfloat16()
        w = (torch.randn(layers * 2 * hkv * 128, hidden, device=device, generator=gg) * 0.02).bfloat16()
        k_norm = torch.ones(layers, 128, device=device).bfloat16()
        cos_sin = rope_cache(128, 8192, 1000000.0, device)
        positions = torch.randint(0, 8192, (T,), device=device, generator=gg)
        slots = torch.randperm(64 * 16 * bs, device=device, generator=gg)[:T].to(torch.int32)
        cache = torch.zeros(2, layers, 64 * 16, bs, hkv, 128, dtype=torch.bfloat16, device=device)
        kv = torch.empty(T, layers * 2 * hkv * 128, dtype=torch.bfloat16, device=device)

        def fn():
            store_context_kv(features, w, k_norm, cos_sin, positions, slots, cache, 1e-6, kv_out=kv)
        # weights (GEMM) + features + projection write/read + cache writes
        algorithmic = w.numel() * 2 + features.numel() * 2 + 2 * kv.numel() * 2 + T * layers * 2 * hkv * 128 * 2
    elif args.kernel == "after_verify":
        # config 4's whole after_verify: context features (fc 20480 -> 4096 + hidden_norm) of T = 288 verified
        # tokens, then the 5 draft layers' context K/V (W_kv GEMM + k_norm / RoPE / paged store)
        from nanovllm_b200.dflash import after_verify
        from nanovllm_b200.fused import rope_cache
        T, layers, hidden, hkv, bs = 288, 5, 4096, 8, 256
        gg = torch.Generator(device=device).manual_seed(0)
        aux = torch.randn(T, 5 * hidden, device=device, generator=gg).bfloat16()
        w_fc = (torch.randn(hidden, 5 * hidden, device=device, generator=gg) * 0.01).bfloat16()
        hidden_norm = torch.ones(hidden, device=device).bfloat16()
        w = (torch.randn(layers * 2 * hkv * 128, hidden, device=device, generator=gg) * 0.02).bfloat16()
        k_norm = torch.ones(layers, 128, device=device).bfloat16()
        cos_sin = rope_cache(128, 8192, 1000000.0, device)
        positions = torch.randint(0, 8192, (T,), device=device, generator=gg)
        slots = torch.randperm(64 * 16 * bs, device=device, generator=gg)[:T].to(torch.int32)
        cache = torch.zeros(2, layers, 64 * 16, bs, hkv, 128, dtype=torch.bfloat16, device=device)
        bufs = {"fc": torch.empty(T, hidden, dtype=torch.bfloat16, device=device),
                "features": torch.empty(T, hidden, dtype=torch.bfloat16, device=device),
                "kv": torch.empty(T, layers * 2 * hkv * 128, dtype=torch.bfloat16, device=device)}

        def fn():
            after_verify(aux, w_fc, hidden_norm, w, k_norm, cos_sin, positions, slots, cache, 1e-6, buffers=bufs)
        # both weights + aux + fc / features / projection writes and reads + cache writes
        algorithmic = (w_fc.numel() + w.numel() + aux.numel() + 4 * T * hidden + 2 * bufs["kv"].numel()
                       + T * layers * 2 * hkv * 128) * 2
    elif args.kernel == "accept_greedy":
        # config 3's greedy accept: 64 requests x 8 verified rows of bf16 logits, argmax prefix match
        from nanovllm_b200 import spec_sampler as S
        B = 64
        logits = (torch.randn(B * 8, V, device=device) * 3).bfloat16()
        drafts = torch.randint(V, (B, 7), device=device)

        def fn():
            S.accept_greedy(logits.view(B, 8, V), drafts)
        algorithmic = logits.numel() * 2                       # the logits once
    elif args.kernel == "sample":
        # the exponential race of a [64, V] fp32 distribution with in-kernel Exp(1) draws (spec_sampler.sample)
        from nanovllm_b200 import spec_sampler as S
        B = 64
        w = torch.softmax(torch.randn(B, V, device=device) * 3, -1)
        gen = torch.Generator(device=device).manual_seed(0)

        def fn():
            S.sample(w, gen)
        algorithmic = w.numel() * 4                            # the weights once (the draws are generated)
    else:
        from nanovllm_b200 import spec_sampler as S
        B = 64
        logits = (torch.randn(B * 8, V, device=device) * 3).bfloat16()
        q = torch.softmax(torch.randn(B, 7, V, device=device), -1)
        drafts = torch.randint(V, (B, 7), device=device)
        params = (0.7, 20, 0.8) if args.kernel == "accept_topk" else (1.0, 0, 1.0)   # protocol sampling
        samp = S.sampling_tensors([SimpleNamespace(temperature=params[0], top_k=params[1], top_p=params[2])] * B,
                                  device)
        gen = torch.Generator(device=device).manual_seed(0)

        def fn():
            S.accept_from_logits(logits, q, drafts, samp, None, gen)
        # logits once, plus the tail rows' q and logits for the full-row race (a truncating batch races only its
        # rows' kept tokens: a few KB)
        algorithmic = logits.numel() * 2 + (B * V * (4 + 2) if args.kernel == "accept" else 0)
    for _ in range(args.warmup):
        fn()
    timing = "events"
    if args.kernel in ("attention", "ctx_store", "after_verify", "markov"):
        # K calls captured in one CUDA graph and replayed, so the host's per-call work (tensor map encoding,
        # Python) does not pace the device; the reference captures its Markov rows in a graph the same way
        # (speculative.py:216-231)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for _ in range(args.steps):
                fn()
        graph.replay()
        us = time_events(torch, graph.replay, 3) / args.steps
        timing = f"CUDA graph of {args.steps} calls, 3 replays"
    else:
        us = time_events(torch, fn, args.steps)
    pk = peaks()
    achieved = algorithmic / (us * 1e-6) / 1e9
    print(json.dumps({"kernel": args.kernel, "us_per_launch": round(us, 2), "timing": timing,
                      "algorithmic_bytes": algorithmic,
                      "achieved_GBps": round(achieved, 1), "peak_GBps": pk["hbm_gbs"],
                      "frac": round(achieved / pk["hbm_gbs"], 4), "peak_source": pk["source"]}), flush=True)
    return 0


def run_attention_tp(args) -> int:
    """KV-head tensor-parallel verify attention (benchmark config 5's TP mode), one rank per GPU under torchrun:
    B rows x 8 verify positions (T = 8B), 32 / 8 heads of 128, contexts ~ctx in 256-slot blocks (random block
    permutation); each of N ranks holds Hkv/N KV heads of every row.  One layer = this rank's K/V store + the
    paged attention over its heads + the in-place NCCL all-gather of the outputs + the head interleave; with N > 1
    also the peer-store exchange (the kernel stores every tile into all ranks' symmetric output buffers, then one
    bounded cross-GPU barrier).  Timed as a CUDA graph of K layers over 4 rotating caches (beyond L2), 3 replays,
    max over ranks; the local store + attention alone is timed the same way, so the difference is the exchange."""
    import datetime
    import torch
    import torch.distributed as dist
    from nanovllm_b200.context import reset_context, set_context
    from nanovllm_b200.replicas import barrier, reduce_scalar
    from nanovllm_b200.tp_attention import TPAttention
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)
    B, H, Hkv, D, bs, nq = args.batch, 32, 8, 128, 256, K_DRAFTS + 1
    g = torch.Generator().manual_seed(0)                 # the same rows on every rank
    ctx = torch.randint(max(args.ctx - 50, 1), args.ctx + 51, (B,), generator=g).tolist()
    k_lens = [c + nq for c in ctx]
    nb = [math.ceil(k / bs) for k in k_lens]
    NB = sum(nb) + 1
    perm = torch.randperm(NB - 1, generator=g).tolist()
    tables = torch.full((B, max(nb)), NB - 1, dtype=torch.int32)
    used = 0
    for r, n in enumerate(nb):
        tables[r, :n] = torch.tensor(perm[used:used + n])
        used += n
    slots = [int(tables[r, p // bs]) * bs + p % bs for r in range(B) for p in range(ctx[r], k_lens[r])]
    T = B * nq
    m = TPAttention(H, D, D ** -0.5, Hkv)
    modules = {"tp": m}
    if m.world > 1:        # the fused exchange: stores into the peers' symmetric buffers + bounded barrier
        modules["tp_peer"] = TPAttention(H, D, D ** -0.5, Hkv, exchange="peer", max_tokens=T, device=device)
    Hl, Hkl = H // m.world, Hkv // m.world
    copies = 4
    caches = []
    for _ in range(copies):
        pair = []
        for _kv in range(2):
            c = torch.empty(NB, bs, Hkl, D, dtype=torch.bfloat16, device=device)
            c.normal_()
            pair.append(c)
        caches.append(pair)
    q = torch.randn(T, Hl, D, device=device).bfloat16()
    k_new = torch.randn(T, Hkl, D, device=device).bfloat16()
    v_new = torch.randn(T, Hkl, D, device=device).bfloat16()
    cu_q = torch.arange(0, T + 1, nq, dtype=torch.int32, device=device)
    cu_k = torch.tensor([0] + torch.tensor(k_lens).cumsum(0).tolist(), dtype=torch.int32, device=device)
    set_context(True, cu_q, cu_k, nq, max(k_lens), torch.tensor(slots, dtype=torch.int32, device=device), None,
                tables.to(device))
    state = {"i": 0}

    def bind(module):
        module.k_cache, module.v_cache = caches[state["i"] % copies]
        state["i"] += 1

    def layer_fn(module):
        def layer():
            bind(module)
            module(q, k_new, v_new)
        return layer

    def local_only():
        bind(m)
        m.local(q, k_new, v_new, out=m.gather_buffer(T, device)[m.rank])

    fns = {name: layer_fn(module) for name, module in modules.items()}
    fns["local"] = local_only
    for _ in range(max(args.warmup, 3)):
        for fn in fns.values():
            fn()
    barrier()
    steps = args.steps
    graphs = {}
    for name, fn in fns.items():
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, capture_error_mode="thread_local"):
            for _ in range(steps):
                fn()
        graphs[name] = graph
    barrier()
    times = {}
    with ClockSampler(local_rank) as clocks:
        for name in list(fns) * 2:                       # each timed twice; the second timing is kept
            graphs[name].replay()
            barrier()
            times[name] = reduce_scalar(time_events(torch, graphs[name].replay, 3) / steps, "max")
    barrier()
    peer_status = modules["tp_peer"].peer_error() if "tp_peer" in modules else 0
    reset_context()
    graphs.clear()                                       # graphs holding NCCL calls go before the group
    keys = sum(k_lens)
    local_bytes = keys * Hkl * D * 2 * 2 + 2 * T * Hl * D * 2 + 2 * T * Hkl * D * 2   # K/V + q, out + stores
    pk = peaks()
    achieved = local_bytes / (times["local"] * 1e-6) / 1e9
    if rank == 0:
        print(json.dumps({
            "kernel": "attention_tp", "n_gpus": world, "rows": B, "verify_positions": nq, "ctx_mean": args.ctx,
            "heads": H, "kv_heads_per_gpu": Hkl, "us_per_layer": round(times["tp"], 2),
            "local_attention_us": round(times["local"], 2),
            "exchange_us": round(times["tp"] - times["local"], 2),
            "peer_store_us_per_layer": round(times["tp_peer"], 2) if "tp_peer" in times else None,
            "peer_store_exchange_us": round(times["tp_peer"] - times["local"], 2) if "tp_peer" in times else None,
            "peer_barrier_status": peer_status,
            "per_gpu_algorithmic_bytes": local_bytes, "local_achieved_GBps": round(achieved, 1),
            "peak_GBps": pk["hbm_gbs"], "local_frac": round(achieved / pk["hbm_gbs"], 4), "peak_source": pk["source"],
            "nvlink_bytes_in_per_gpu": 2 * T * H * D * (world - 1) // world,
            "timing": f"CUDA graph of {steps} layers over {copies} rotating caches, 3 replays, max over ranks",
            "clocks": clocks.summary()}), flush=True)
    del caches
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


# ---------------------------------------------------------------------------------------------- our arm
def main() -> int:
    args = parse_args()
    if args.impl == "reference":
        return run_reference(args)
    if args.kernel == "attention_tp":
        return run_attention_tp(args)
    if args.kernel is not None:
        return run_kernel(args)
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=device)

    w = build_workload(torch, device, args.batch, args.ctx, seed=1234 + rank)
    rnd, batch = w.round, args.batch
    gen = torch.Generator(device=device).manual_seed(99 + rank)
    num_tokens = rnd.load(w.rows)

    def step_device():
        return rnd.verify_and_accept(num_tokens, batch, w.drafts, w.q, w.sampling, gen)

    from nanovllm_b200.replicas import barrier, reduce_scalar

    def max_over_ranks(x: float) -> float:
        return reduce_scalar(x, "max")

    def sum_over_ranks(x: float) -> float:
        return reduce_scalar(x, "sum")

    for _ in range(args.warmup):
        step_device()
    barrier()
    accepted = torch.zeros((), dtype=torch.int64, device=device)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clocks:
        barrier()
        torch.cuda.nvtx.range_push("timed")     # lets a profiler keep to the timed launches (--nvtx-include)
        start.record()
        for _ in range(args.steps):
            n_accept, _tail = step_device()
            accepted += n_accept.sum() + batch
        end.record()
        torch.cuda.nvtx.range_pop()
        barrier()
        device_ms = start.elapsed_time(end)
        # e2e: metadata H2D from pinned host buffers + the round's D2H payload, every step
        for _ in range(args.warmup):
            rnd.run_round(w.rows, w.drafts, w.q, w.sampling, gen)
        barrier()
        e2e_tokens = 0
        start.record()
        for _ in range(args.steps):
            out = rnd.run_round(w.rows, w.drafts, w.q, w.sampling, gen)
            e2e_tokens += sum(len(r) for r in out)
        end.record()
        barrier()
        e2e_ms = start.elapsed_time(end)
    device_ms = max_over_ranks(device_ms)
    e2e_ms = max_over_ranks(e2e_ms)
    total_accepted = sum_over_ranks(float(accepted.item()))
    total_e2e_tokens = sum_over_ranks(float(e2e_tokens))
    value = total_accepted / (device_ms / 1e3)
    e2e_value = total_e2e_tokens / (e2e_ms / 1e3)
    ms_per_step = device_ms / args.steps

    pk = peaks()
    roofline = attention_roofline(torch, w, pk["hbm_gbs"])
    roofline["peak_source"] = pk["source"]
    accept = accept_timing(torch, w)
    launches_per_step = w.shape.layers * 5 + 1 + 2      # per layer: 2 norms, qk-norm/rope/store, attention,
                                                        # silu; final norm; sampler stats + tail
    h2d = (num_tokens * (8 + 8 + 4) + 2 * (batch + 1) * 4 + batch * w.width * 4)
    d2h = batch * (K_DRAFTS + 2) * 8
    line = None
    if rank == 0:
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            from threadpoolctl import threadpool_limits
            with threadpool_limits(1):                    # the reported core count is the one used
                sample = cpu_round_sample(8, 16, args.ctx, 1)
            cpu_round_s = cpu_round_seconds(sample, batch, w.shape.layers)
            tokens_per_round = total_accepted / args.steps / world
            cpu = {"value": round(tokens_per_round / cpu_round_s, 3), "unit": "tok/s", "cores": 1, "kind": "port",
                   "sample": f"numpy oracle: paged attention of {sample['rows']} rows x {sample['layers']} layers at ctx {args.ctx} "
                             f"({sample['attn_s']:.2f} s) + sampler of the same rows ({sample['accept_s']:.2f} s), "
                             f"scaled to {batch} rows x {w.shape.layers} layers; GEMMs excluded"}
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": f"cfg3: verify+accept round, random-init Qwen3-8B target, B={batch} rows x 8 "
                                   f"verify positions, ctx ~{args.ctx} (U[ctx-50, ctx+50]), temperature 1, "
                                   f"in-kernel draws",
                       "model": "Qwen3-8B architecture (random init)", "global_batch": batch * world,
                       "seq_len": args.ctx, "parallelism": f"dp{world} (row-sharded replicas)",
                       "l2": "no flush: weights 16.4 GB + KV > L2 every step"},
            "e2e": {"value": round(e2e_value, 1), "unit": "tok/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "ms_per_step": round(e2e_ms / args.steps, 4)},
            "roofline": roofline,
            "cpu_baseline": cpu,
            "clocks": clocks.summary(),
            "gpu_launches": launches_per_step * args.steps,
            "extra": {"round_us": round(ms_per_step * 1e3, 1),
                      "verified_tok_s": round(batch * (K_DRAFTS + 1) * world / (ms_per_step / 1e3), 1),
                      "tokens_per_round_per_row": round(total_accepted / args.steps / world / batch, 4),
                      "accept_kernel": accept},
        }
        print(json.dumps(line), flush=True)
    w.target.close()
    del w
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
