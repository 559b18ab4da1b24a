"""Generates the golden fixtures under tests/golden/ by running the reference itself on CPU torch.

    python tests/golden/make_golden.py [--reference /path/to/nano-vllm-speculative-decoding]

Needs the reference checkout (default: $SPECDEC_REFERENCE or ../reference next to this repository's parent);
the fixtures it writes are committed, so nothing at test time reads the reference.

Every random draw the reference makes is recorded next to its outputs: the generator's state is cloned before
the call and the same draws are replayed in the reference's order (uniforms [B, k] first, then the [B, V]
exponential noise of the tail race, clamped at 1e-10), and the script asserts that the replay leaves the
generator where the reference left it.
"""
from __future__ import annotations

import argparse
import os
import sys
import zlib
from pathlib import Path
from types import SimpleNamespace

import numpy as np

# The reference's RMSNorm / RoPE / SiLU are torch.compile'd methods; the fixtures use their eager bodies.
os.environ.setdefault("TORCHDYNAMO_DISABLE", "1")
import torch  # noqa: E402

HERE = Path(__file__).resolve().parent


def import_reference(path: Path):
    sys.path.insert(0, str(path))
    sys.path.insert(0, str(path / "tests"))
    import gpu_import_stubs  # noqa: F401  (flash_attn / triton stand-ins so nanovllm imports on CPU)
    from nanovllm.layers import spec_sampler
    return spec_sampler


def sampling(ss, temps, top_k, top_p):
    seqs = [SimpleNamespace(temperature=t, top_k=k, top_p=p) for t, k, p in zip(temps, top_k, top_p)]
    return ss.sampling_tensors(seqs, torch.device("cpu"))


def draws(generator: torch.Generator, batch: int, k: int, vocab: int):
    clone = torch.Generator().manual_seed(0)
    clone.set_state(generator.get_state())
    u = torch.rand(batch, k, generator=clone)
    noise = torch.empty(batch, vocab).exponential_(1.0, generator=clone).clamp_min_(1e-10)
    return u, noise, clone


def random_lens(rng: np.random.Generator, batch: int, k: int) -> np.ndarray:
    return rng.integers(1, k + 2, size=batch).astype(np.int64)


def accept_cases(ss) -> dict[str, np.ndarray]:
    """accept_random[_varlen] on given probabilities (the reference functions' own inputs)."""
    out: dict[str, np.ndarray] = {}
    cases = []
    # the pre-varlen equivalence cases of the reference's tests (B=6, k=7, V=5, seeds 0-4)
    for seed in range(5):
        torch.manual_seed(seed)
        p = torch.softmax(torch.randn(6, 8, 5), dim=-1)
        q = torch.softmax(torch.randn(6, 7, 5), dim=-1)
        drafts = torch.randint(5, (6, 7))
        cases.append((f"m3_seed{seed}", p.flatten(0, 1), q, drafts, None, seed))
    # varlen point masses: rows verify 1, 2, 4 positions
    point = torch.eye(4)
    cases.append(("varlen_points", point[[3, 1, 2, 1, 2, 3, 0]], torch.eye(4)[torch.tensor([[1, 2, 3]] * 3)],
                  torch.tensor([[1, 2, 3]] * 3), torch.tensor([1, 2, 4]), 0))
    # random varlen / fixed cases at moderate vocabulary
    rng = np.random.default_rng(7)
    for name, batch, k, vocab, varlen, seed in [("fixed_b16_v600", 16, 7, 600, False, 11),
                                                  ("varlen_b24_v377", 24, 7, 377, True, 12),
                                                  ("varlen_b9_k3_v64", 9, 3, 64, True, 13),
                                                  ("fixed_b4_k1_v33", 4, 1, 33, False, 14)]:
        g = torch.Generator().manual_seed(seed)
        lens = torch.from_numpy(random_lens(rng, batch, k)) if varlen else torch.full((batch,), k + 1)
        total = int(lens.sum())
        p = torch.softmax(torch.randn(total, vocab, generator=g) * 3, dim=-1)
        q = torch.softmax(torch.randn(batch, k, vocab, generator=g) * 3, dim=-1)
        # half the rows propose from p itself so long prefixes get accepted
        starts = torch.cumsum(lens, 0) - lens
        for b in range(0, batch, 2):
            for j in range(k):
                pos = int(starts[b]) + min(j, int(lens[b]) - 1)
                q[b, j] = p[pos]
        drafts = torch.stack([torch.multinomial(q[b], 1, generator=g).squeeze(-1) for b in range(batch)])
        cases.append((name, p, q, drafts, lens if varlen else None, seed))
    for name, p, q, drafts, lens, seed in cases:
        batch, k = drafts.shape
        g = torch.Generator().manual_seed(1000 + seed)
        u, noise, clone = draws(g, batch, k, p.shape[-1])
        if lens is None:
            n_accept, tail = ss.accept_random(p.view(batch, k + 1, -1), q, drafts, g)
            lens_out = torch.full((batch,), k + 1)
        else:
            n_accept, tail = ss.accept_random_varlen(p, q, drafts, lens, g)
            lens_out = lens
        assert torch.equal(g.get_state(), clone.get_state()), name
        prefix = f"accept/{name}/"
        for key, value in dict(p=p, q=q, drafts=drafts, lens=lens_out, u=u, noise=noise, n_accept=n_accept,
                               tail=tail, fixed=torch.tensor(lens is None)).items():
            out[prefix + key] = value.numpy()
    return out


def logits_cases(ss) -> dict[str, np.ndarray]:
    """probs_from_logits + accept on logits: the fused _accept path (speculative.py:450-462)."""
    out: dict[str, np.ndarray] = {}
    rng = np.random.default_rng(21)
    configs = [
        # name, batch, k, vocab, dtype, temps, top_k, top_p, varlen
        ("t1_fp32_v800", 8, 7, 800, torch.float32, [1.0] * 8, [0] * 8, [1.0] * 8, False),
        ("protocol_fp32_v900", 8, 7, 900, torch.float32, [0.7] * 8, [20] * 8, [0.8] * 8, False),
        ("mixed_bf16_v700", 6, 7, 700, torch.bfloat16, [1.0, 0.7, 0.5, 1.3, 0.9, 1.0], [0, 20, 5, 0, 64, 1],
         [1.0, 0.8, 0.5, 1.0, 0.95, 1.0], True),
        ("topk_only_fp16_v999", 5, 4, 999, torch.float16, [0.8] * 5, [3, 10, 50, 7, 1], [1.0] * 5, True),
    ]
    for name, batch, k, vocab, dtype, temps, top_k, top_p, varlen in configs:
        g = torch.Generator().manual_seed(zlib.crc32(name.encode()) % 100000)
        lens = torch.from_numpy(random_lens(rng, batch, k)) if varlen else torch.full((batch,), k + 1)
        total = int(lens.sum())
        logits = (torch.randn(total, vocab, generator=g) * 3).to(dtype)
        samp = sampling(ss, temps, top_k, top_p)
        per_token = ss.sampling_per_token(samp, lens, total)
        p = ss.probs_from_logits(logits, per_token)
        q_logits = torch.randn(batch, k, vocab, generator=g) * 3
        q = ss.probs_from_logits(q_logits, samp)
        drafts = ss.sample(q, g)
        u, noise, clone = draws(g, batch, k, vocab)
        n_accept, tail = ss.accept_random_varlen(p, q, drafts, lens, g)
        assert torch.equal(g.get_state(), clone.get_state()), name
        prefix = f"logits/{name}/"
        for key, value in dict(logits=logits.float(), p=p, q=q, drafts=drafts, lens=lens, u=u, noise=noise,
                               n_accept=n_accept, tail=tail, temperature=samp.temperatures, top_k=samp.top_k,
                               top_p=samp.top_p).items():
            out[prefix + key] = value.numpy()
        out[prefix + "dtype"] = np.array(str(dtype).replace("torch.", ""))
        out[prefix + "max_top_k"] = np.array(samp.max_top_k)
        out[prefix + "has_top_p"] = np.array(samp.has_top_p)
    return out


def truncation_cases(ss) -> dict[str, np.ndarray]:
    """probs_from_logits known answers, including the reference tests' tie and nucleus cases."""
    out: dict[str, np.ndarray] = {}
    g = torch.Generator().manual_seed(5)
    tied = torch.randn(1, 200, generator=g).clamp(max=2.5)
    tied[0, :32] = torch.tensor([5.0, 4.0] + [3.0] * 30)
    cases = [
        ("temperature", torch.tensor([[1.0, 0.0]]), [0.5], [0], [1.0]),
        ("top_k_two", torch.tensor([[1.0, 3.0, 2.0, 0.0]]), [1.0], [2], [1.0]),
        ("top_k_tie", torch.tensor([[2.0, 2.0, 1.0, 0.0]]), [1.0], [1], [1.0]),
        ("top_p_half", torch.tensor([[0.4, 0.3, 0.2, 0.1]]).log(), [1.0], [4], [0.5]),
        ("top_p_within_k", torch.tensor([[0.4, 0.3, 0.2, 0.1]]).log(), [1.0], [2], [0.99]),
        ("mixed_rows", torch.tensor([[1.0, 2.0, 3.0], [1.0, 2.0, 3.0]]), [1.0, 1.0], [0, 1], [1.0, 1.0]),
        ("thirty_tied_at_cut", tied, [0.7], [3], [1.0]),
        ("top_k_above_vocab", torch.randn(2, 50, generator=g), [1.0, 0.9], [80, 3], [1.0, 0.7]),
        ("wide_random", torch.randn(7, 1500, generator=g) * 4, [0.7, 1.0, 0.3, 2.0, 1.0, 0.7, 0.9],
         [20, 0, 128, 1, 1000, 64, 7], [0.8, 1.0, 0.9, 1.0, 0.99, 0.3, 0.05]),
    ]
    for name, logits, temps, top_k, top_p in cases:
        samp = sampling(ss, temps, top_k, top_p)
        probs = ss.probs_from_logits(logits, samp)
        prefix = f"trunc/{name}/"
        out[prefix + "logits"] = logits.numpy()
        out[prefix + "temperature"] = samp.temperatures.numpy()
        out[prefix + "top_k"] = samp.top_k.numpy()
        out[prefix + "top_p"] = samp.top_p.numpy()
        out[prefix + "max_top_k"] = np.array(samp.max_top_k)
        out[prefix + "has_top_p"] = np.array(samp.has_top_p)
        out[prefix + "probs"] = probs.numpy()
    return out


def greedy_cases(ss) -> dict[str, np.ndarray]:
    out: dict[str, np.ndarray] = {}
    rng = np.random.default_rng(3)
    for name, batch, k, vocab, varlen in [("fixed_b8_v500", 8, 7, 500, False), ("varlen_b12_v300", 12, 7, 300, True)]:
        g = torch.Generator().manual_seed(batch)
        lens = torch.from_numpy(random_lens(rng, batch, k)) if varlen else torch.full((batch,), k + 1)
        total = int(lens.sum())
        logits = torch.randn(total, vocab, generator=g)
        target = logits.argmax(-1)
        starts = torch.cumsum(lens, 0) - lens
        drafts = torch.randint(vocab, (batch, k), generator=g)
        for b in range(batch):   # agree with the target for a random prefix
            agree = int(rng.integers(0, k + 1))
            for j in range(min(agree, int(lens[b]) - 1)):
                drafts[b, j] = target[int(starts[b]) + j]
        n_accept, tail = ss.accept_greedy_varlen(logits, drafts, lens)
        prefix = f"greedy/{name}/"
        for key, value in dict(logits=logits, drafts=drafts, lens=lens, n_accept=n_accept, tail=tail).items():
            out[prefix + key] = value.numpy()
    # a tie: two equal maxima, the first index wins
    logits = torch.zeros(2, 6)
    logits[0, [2, 4]] = 1.0
    logits[1, [1, 5]] = 2.0
    n_accept, tail = ss.accept_greedy(logits.view(1, 2, 6), torch.tensor([[2]]))
    for key, value in dict(logits=logits, drafts=torch.tensor([[2]]), lens=torch.tensor([2]), n_accept=n_accept,
                           tail=tail).items():
        out["greedy/ties/" + key] = value.numpy()
    return out


def ctx_store_cases(reference: Path) -> dict[str, np.ndarray]:
    """DFlashDraftModel.store_context_kv (dflash.py:88-96) on a small random draft: 2 layers, hidden 256, 4/2
    heads of 128, bf16, with the CPU store_kvcache stand-in (tests/fake_paged_attention.py)."""
    import torch.distributed as dist
    from nanovllm.layers import attention as ref_attention
    from nanovllm.models.dflash import DFlashDraftModel
    import fake_paged_attention
    if not dist.is_initialized():
        dist.init_process_group("gloo", init_method="tcp://127.0.0.1:29517", world_size=1, rank=0)
    config = SimpleNamespace(block_size=7, mask_token_id=99, target_layer_ids=[0, 1], vocab_size=128,
                             hidden_size=256, num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
                             head_dim=128, rms_norm_eps=1e-6, intermediate_size=512, hidden_act="silu",
                             max_position_embeddings=4096, markov_rank=0, enable_confidence_head=False,
                             attention_bias=False, rope_theta=1000000, rope_scaling=None)
    torch.manual_seed(0)
    default_dtype = torch.get_default_dtype()
    torch.set_default_dtype(torch.bfloat16)
    try:
        model = DFlashDraftModel(config)
    finally:
        torch.set_default_dtype(default_dtype)
    with torch.no_grad():
        for name, param in model.named_parameters():
            if name.endswith("norm.weight"):
                param.copy_(1.0 + 0.1 * torch.randn(param.shape))
            else:
                param.copy_(0.05 * torch.randn(param.shape))
    blocks, block_size, hkv = 4, 256, 2
    kv_cache = torch.zeros(2, 2, blocks, block_size, hkv, 128, dtype=torch.bfloat16)
    for layer_id, layer in enumerate(model.layers):
        layer.self_attn.attn.k_cache = kv_cache[0, layer_id]
        layer.self_attn.attn.v_cache = kv_cache[1, layer_id]
    T = 40
    g = torch.Generator().manual_seed(3)
    features = torch.randn(T, 256, generator=g).bfloat16()
    positions = torch.randint(0, 3000, (T,), generator=g)
    slots = torch.randperm(blocks * block_size, generator=g)[:T].to(torch.int32)
    slots[[5, 17]] = -1                                   # padding rows are skipped
    original = ref_attention.store_kvcache
    ref_attention.store_kvcache = fake_paged_attention.store_kvcache
    try:
        with torch.no_grad():
            model.store_context_kv(features, positions, slots)
    finally:
        ref_attention.store_kvcache = original
    attn = model.layers[0].self_attn
    model.requires_grad_(False)
    w_kv = torch.cat([layer.self_attn.qkv_proj.weight[attn.q_size:] for layer in model.layers])
    k_norm = torch.stack([layer.self_attn.k_norm.weight for layer in model.layers])
    out = {"ctx/features": features.float().numpy(), "ctx/w_kv": w_kv.float().numpy(),
           "ctx/k_norm": k_norm.float().numpy(), "ctx/positions": positions.numpy(),
           "ctx/slots": slots.numpy(), "ctx/kv_cache": kv_cache.float().numpy(),
           "ctx/eps": np.array(1e-6), "ctx/rope_base": np.array(1000000.0), "ctx/max_position": np.array(4096)}
    # the target's q path: q_norm + RoPE of random queries (qwen3.py:77-84)
    q = torch.randn(T, 4, 128, generator=g).bfloat16()
    with torch.no_grad():
        qn = attn.q_norm(q)
        q_rot, _ = attn.rotary_emb(positions, qn, qn.clone())
    out.update({"ctx/q": q.float().numpy(), "ctx/q_norm": attn.q_norm.weight.float().numpy(),
                "ctx/q_out": q_rot.float().numpy()})
    return out


def markov_cases(reference: Path) -> dict[str, np.ndarray]:
    """DFlashDrafter._markov_rows (speculative.py:163-184) with a lookup-table Markov head, as the reference's
    tests/test_dspark_propose.py builds it: greedy, candidate rows (every row truncates) and whole-vocabulary
    rows.  fp32 logits and a rank-1 bias a[prev] * c[v] (one fp32 product, reproduced exactly by any
    implementation), so no two candidates tie."""
    from nanovllm.engine.speculative import DFlashDrafter, num_candidates
    from nanovllm.layers import spec_sampler as ss
    out: dict[str, np.ndarray] = {}
    configs = [
        # name, B, k, V, temps (None = greedy), top_k, top_p
        ("greedy_v300", 5, 7, 300, None, [0] * 5, [1.0] * 5),
        ("candidates_v500", 6, 7, 500, [1.0, 0.7, 0.5, 1.3, 0.9, 1.0], [3, 10, 20, 5, 1, 64],
         [1.0, 0.8, 0.5, 1.0, 0.95, 1.0]),
        ("whole_vocab_v400", 4, 7, 400, [1.0, 0.7, 1.0, 0.8], [0, 5, 0, 3], [1.0, 0.9, 1.0, 0.7]),
        ("candidates_v5000_k128", 3, 7, 5000, [1.0, 1.0, 0.7], [128, 20, 128], [1.0, 0.8, 1.0]),
    ]
    for name, batch, k, vocab, temps, top_k, top_p in configs:
        g = torch.Generator().manual_seed(zlib.crc32(name.encode()) % 100000)
        logits = torch.randn(batch, k, vocab, generator=g) * 2
        bias_a = torch.randn(vocab, generator=g)
        bias_c = torch.randn(vocab, generator=g)
        prev = torch.randint(vocab, (batch,), generator=g)
        drafter = object.__new__(DFlashDrafter)
        drafter.model = SimpleNamespace(markov_head=lambda p, a=bias_a, c=bias_c: a[p][:, None] * c[None, :])
        drafts = torch.empty(batch, k, dtype=torch.int64)
        if temps is None:
            samp, noise, probs, cand = None, None, None, 0
            drafter._markov_rows(logits, prev.clone(), None, None, drafts, None, 0)
        else:
            samp = sampling(ss, temps, top_k, top_p)
            cand = num_candidates(samp.max_top_k, samp.all_top_k, vocab)
            noise = ss.exponential_noise_(torch.empty(batch, k, cand or vocab), g)
            probs = torch.empty(batch, k, vocab)
            drafter._markov_rows(logits, prev.clone(), samp, noise, drafts, probs, cand)
        prefix = f"markov/{name}/"
        out[prefix + "logits"] = logits.numpy()
        out[prefix + "bias_a"] = bias_a.numpy()
        out[prefix + "bias_c"] = bias_c.numpy()
        out[prefix + "prev"] = prev.numpy()
        out[prefix + "drafts"] = drafts.numpy()
        out[prefix + "candidates"] = np.array(cand)
        if samp is not None:
            out[prefix + "temperature"] = samp.temperatures.numpy()
            out[prefix + "top_k"] = samp.top_k.numpy()
            out[prefix + "top_p"] = samp.top_p.numpy()
            out[prefix + "max_top_k"] = np.array(samp.max_top_k)
            out[prefix + "has_top_p"] = np.array(samp.has_top_p)
            out[prefix + "noise"] = noise.numpy()
            out[prefix + "probs"] = probs.numpy()
    return out


def markov_bf16_cases(reference: Path) -> dict[str, np.ndarray]:
    """_markov_rows on the production dtypes: bf16 logits and a bf16 head output, summed in bf16 (the fp32 sum
    rounded once).  Greedy rows use random values (a tied maximum takes its first index on both sides).  torch.topk
    leaves the order of equal values open and that order assigns the candidates' noise, so the candidate rows are
    built tie-free: each row's logits are a permutation of a grid 2^-3 apart and the head's products stay below
    2^-5, so sums round to bf16 (in the binades where the grid is the bf16 spacing) without two ever meeting."""
    from nanovllm.engine.speculative import DFlashDrafter, num_candidates
    from nanovllm.layers import spec_sampler as ss
    out: dict[str, np.ndarray] = {}
    configs = [
        # name, B, k, V, temps (None = greedy), top_k, top_p
        ("greedy_bf16_v4096", 4, 7, 4096, None, [0] * 4, [1.0] * 4),
        ("candidates_bf16_v512", 4, 7, 512, [1.0, 0.7, 0.9, 1.2], [8, 3, 20, 5], [1.0, 0.8, 0.9, 1.0]),
    ]
    for name, batch, k, vocab, temps, top_k, top_p in configs:
        g = torch.Generator().manual_seed(zlib.crc32(name.encode()) % 100000)
        if temps is None:
            logits = (torch.randn(batch, k, vocab, generator=g) * 4).bfloat16()
            bias_a = torch.randn(vocab, generator=g).bfloat16()
            bias_c = torch.randn(vocab, generator=g).bfloat16()
        else:
            grid = (torch.arange(vocab) - vocab // 2).float() * 0.125           # exact in bf16 (|x| < 32)
            logits = torch.stack([grid[torch.randperm(vocab, generator=g)] for _ in range(batch * k)])
            logits = logits.view(batch, k, vocab).bfloat16()
            signs = lambda: torch.randint(0, 2, (vocab,), generator=g).float() * 2 - 1   # noqa: E731
            bias_a = (signs() * 0.125).bfloat16()                                  # |a| = 2^-3
            bias_c = (signs() * torch.randint(1, 4, (vocab,), generator=g).float() * 0.0625).bfloat16()  # < 2^-2
        prev = torch.randint(vocab, (batch,), generator=g)
        drafter = object.__new__(DFlashDrafter)
        drafter.model = SimpleNamespace(markov_head=lambda p, a=bias_a, c=bias_c: a[p][:, None] * c[None, :])
        drafts = torch.empty(batch, k, dtype=torch.int64)
        samp = noise = probs = None
        cand = 0
        if temps is None:
            drafter._markov_rows(logits, prev.clone(), None, None, drafts, None, 0)
        else:
            samp = sampling(ss, temps, top_k, top_p)
            cand = num_candidates(samp.max_top_k, samp.all_top_k, vocab)
            noise = ss.exponential_noise_(torch.empty(batch, k, cand), g)
            probs = torch.empty(batch, k, vocab)
            drafter._markov_rows(logits, prev.clone(), samp, noise, drafts, probs, cand)
            p_row = prev                               # tie-free check on the rows the reference drew
            for row in range(k):
                values = (logits[:, row] + drafter.model.markov_head(p_row)).float()
                top = values.sort(dim=-1, descending=True).values[:, :cand + 1]
                assert not bool((top[:, 1:] == top[:, :-1]).any()), name
                p_row = drafts[:, row]
        prefix = f"markov_bf16/{name}/"
        for key, value in dict(logits=logits.float(), bias_a=bias_a.float(), bias_c=bias_c.float(), prev=prev,
                               drafts=drafts).items():
            out[prefix + key] = value.numpy()
        out[prefix + "candidates"] = np.array(cand)
        if samp is not None:
            for key, value in dict(temperature=samp.temperatures, top_k=samp.top_k, top_p=samp.top_p,
                                   noise=noise, probs=probs).items():
                out[prefix + key] = value.numpy()
            out[prefix + "max_top_k"] = np.array(samp.max_top_k)
            out[prefix + "has_top_p"] = np.array(samp.has_top_p)
    return out


def masked_cases(ss) -> dict[str, np.ndarray]:
    """Masked vocabularies: rows whose finite logits are fewer than their top_k (the rest -inf), through
    probs_from_logits and the fused accept, with the draws recorded as in logits_cases."""
    out: dict[str, np.ndarray] = {}
    rng = np.random.default_rng(33)
    configs = [
        # name, batch, k, vocab, dtype, temps, top_k, top_p, finite logits per masked row
        ("few_finite_bf16_v640", 6, 7, 640, torch.bfloat16, [0.7] * 6, [20] * 6, [0.8] * 6, 12),
        ("few_finite_fp32_v640", 5, 4, 640, torch.float32, [1.0, 0.7, 0.9, 1.0, 0.5], [20, 3, 64, 0, 7],
         [1.0, 0.8, 0.9, 1.0, 0.6], 5),
    ]
    for name, batch, k, vocab, dtype, temps, top_k, top_p, n_finite in configs:
        g = torch.Generator().manual_seed(zlib.crc32(name.encode()) % 100000)
        lens = torch.from_numpy(random_lens(rng, batch, k))
        total = int(lens.sum())
        logits = torch.randn(total, vocab, generator=g) * 3
        starts = (torch.cumsum(lens, 0) - lens).tolist()
        for b in range(1, batch, 2):                       # odd requests: every verified row masked
            for r in range(starts[b], starts[b] + int(lens[b])):
                keep = torch.randperm(vocab, generator=g)[:n_finite]
                row = torch.full((vocab,), float("-inf"))
                row[keep] = logits[r, keep]
                logits[r] = row
        logits = logits.to(dtype)
        samp = sampling(ss, temps, top_k, top_p)
        per_token = ss.sampling_per_token(samp, lens, total)
        p = ss.probs_from_logits(logits, per_token)
        q = ss.probs_from_logits(torch.randn(batch, k, vocab, generator=g) * 3, samp)
        drafts = ss.sample(q, g)
        u, noise, clone = draws(g, batch, k, vocab)
        n_accept, tail = ss.accept_random_varlen(p, q, drafts, lens, g)
        assert torch.equal(g.get_state(), clone.get_state()), name
        prefix = f"masked/{name}/"
        for key, value in dict(logits=logits.float(), p=p, q=q, drafts=drafts, lens=lens, u=u, noise=noise,
                               n_accept=n_accept, tail=tail, temperature=samp.temperatures, top_k=samp.top_k,
                               top_p=samp.top_p).items():
            out[prefix + key] = value.numpy()
        out[prefix + "max_top_k"] = np.array(samp.max_top_k)
        out[prefix + "has_top_p"] = np.array(samp.has_top_p)
    return out


def greedy_edge_cases(ss) -> dict[str, np.ndarray]:
    """Greedy accept on rows of few distinct values (many tied maxima: the first index wins), rows whose maximum
    is +inf (twice), a row of -inf only and a constant row, in fp32 and bf16."""
    out: dict[str, np.ndarray] = {}
    batch, k, vocab = 6, 3, 4099
    for dtype in (torch.float32, torch.bfloat16):
        g = torch.Generator().manual_seed(vocab)
        rows = batch * (k + 1)
        logits = torch.randint(-3, 4, (rows, vocab), generator=g).to(torch.float32)
        logits[1, vocab // 2] = float("inf")
        logits[1, vocab - 1] = float("inf")
        logits[5] = float("-inf")
        logits[9, :] = 2.0
        logits[13, -1] = 7.0
        logits = logits.to(dtype)
        target = logits.float().argmax(-1).view(batch, k + 1)
        drafts = torch.randint(0, vocab, (batch, k), generator=g)
        for b in range(batch):      # agree with the target on a prefix of length b % (k + 1)
            drafts[b, : b % (k + 1)] = target[b, : b % (k + 1)]
        n_accept, tail = ss.accept_greedy(logits.view(batch, k + 1, vocab), drafts)
        prefix = f"greedy_edge/{str(dtype).replace('torch.', '')}/"
        for key, value in dict(logits=logits.float(), drafts=drafts, n_accept=n_accept, tail=tail).items():
            out[prefix + key] = value.numpy()
    return out


def attention_cases(reference: Path) -> dict[str, np.ndarray]:
    """The reference's paged-attention stand-in (tests/fake_paged_attention.py: store_kvcache, then SDPA over the
    keys gathered through the block table) in its decode layout: query_len_per_seq queries per row, causal
    (queries at the end of the context, the verify rule) and non-causal (the DFlash draft block), fp32 math on
    values exact in fp16 (stored as fp16 to keep the fixture small), GQA group 4, shuffled block tables, a padding
    token at slot -1; of the updated caches only the rows at the stored slots are kept."""
    sys.path.insert(0, str(reference / "tests"))
    import fake_paged_attention as fpa
    from nanovllm.utils.context import reset_context, set_context
    out: dict[str, np.ndarray] = {}
    H, Hkv, D, bs = 4, 1, 128, 256
    for name, q_per_seq, causal, context_lens in [("verify_causal", 8, True, [300, 129, 600, 8, 257]),
                                                   ("draft_block", 7, False, [7, 260, 40, 390])]:
        g = torch.Generator().manual_seed(zlib.crc32(name.encode()) % 100000)
        R = len(context_lens)
        nblk = [-(-n // bs) for n in context_lens]
        num_blocks = sum(nblk) + 2
        perm = torch.randperm(num_blocks, generator=g)
        tables = torch.full((R, max(nblk)), num_blocks - 1, dtype=torch.int32)
        used = 0
        for r, n in enumerate(nblk):
            tables[r, :n] = perm[used:used + n].to(torch.int32)
            used += n
        exact = lambda *shape: torch.randn(*shape, generator=g).half().float()   # noqa: E731
        k_cache = exact(num_blocks, bs, Hkv, D)
        v_cache = exact(num_blocks, bs, Hkv, D)
        T = R * q_per_seq
        q = exact(T, H, D)
        k = exact(T, Hkv, D)
        v = exact(T, Hkv, D)
        slots = []
        for r, n in enumerate(context_lens):          # the row's last q_per_seq positions are its new tokens
            for j in range(q_per_seq):
                pos = n - q_per_seq + j
                slots.append(int(tables[r, pos // bs]) * bs + pos % bs if pos >= 0 else -1)
        slots[1] = -1                                   # a padding token: not stored
        cache_in = (k_cache.clone(), v_cache.clone())
        layer = SimpleNamespace(k_cache=k_cache, v_cache=v_cache, num_heads=H, num_kv_heads=Hkv, head_dim=D,
                                scale=D ** -0.5)
        set_context(False, slot_mapping=torch.tensor(slots), context_lens=torch.tensor(context_lens),
                    block_tables=tables, query_len_per_seq=q_per_seq, causal=causal)
        try:
            o = fpa.attention_forward(layer, q, k, v)
        finally:
            reset_context()
        prefix = f"attention/{name}/"
        stored = torch.tensor([x for x in slots if x >= 0])
        for key, value in dict(q=q.half(), k=k.half(), v=v.half(), k_cache_in=cache_in[0].half(),
                               v_cache_in=cache_in[1].half(), tables=tables, slots=torch.tensor(slots),
                               context_lens=torch.tensor(context_lens), out=o,
                               k_stored=k_cache.view(-1, Hkv, D)[stored].half(),
                               v_stored=v_cache.view(-1, Hkv, D)[stored].half()).items():
            out[prefix + key] = value.numpy()
        out[prefix + "q_per_seq"] = np.array(q_per_seq)
        out[prefix + "causal"] = np.array(causal)
    return out


def forward_helper_cases() -> dict[str, np.ndarray]:
    """The verify forward's RMSNorm (plain and with residual, nanovllm/layers/layernorm.py) and SiluAndMul
    (nanovllm/layers/activation.py), the reference's modules on bf16 CPU tensors (their eager bodies: this script
    disables torch.compile)."""
    from nanovllm.layers.activation import SiluAndMul
    from nanovllm.layers.layernorm import RMSNorm
    g = torch.Generator().manual_seed(17)
    rows, hidden, inter = 16, 4096, 1024
    x = torch.randn(rows, hidden, generator=g).bfloat16()
    residual = torch.randn(rows, hidden, generator=g).bfloat16()
    norm = RMSNorm(hidden, 1e-6)
    norm.weight.data = (1.0 + 0.1 * torch.randn(hidden, generator=g)).bfloat16()
    gate_up = (torch.randn(rows, 2 * inter, generator=g) * 2).bfloat16()
    with torch.no_grad():
        y = norm(x)
        y_res, res_out = norm(x, residual)
        act = SiluAndMul()(gate_up)
    out = dict(x=x, residual=residual, weight=norm.weight.data, y=y, y_res=y_res, res_out=res_out,
               gate_up=gate_up, act=act)
    return {"forward/" + key: value.float().numpy() for key, value in out.items()} | {"forward/eps": np.array(1e-6)}


class _Seq:
    """The Sequence fields verify_varlen_metadata reads: len(seq), last_token, target_kv.block_table."""

    def __init__(self, length: int, last_token: int, block_table: list[int]):
        self.length, self.last_token = length, last_token
        self.target_kv = SimpleNamespace(block_table=block_table)

    def __len__(self) -> int:
        return self.length


def metadata_cases() -> dict[str, np.ndarray]:
    """nanovllm/engine/batch_metadata.py verify_varlen_metadata on random batches: ragged block tables, fixed and
    variable verified lengths, padding rows and empty row slots.  Ragged inputs are stored padded with -1."""
    from nanovllm.engine.batch_metadata import verify_varlen_metadata
    import random
    out: dict[str, np.ndarray] = {}
    for case in range(24):
        rng = random.Random(1000 + case)
        k, block_size, width, pad = 7, 256, 8, 999
        # cases 12-23: no rows at all (12, 13), every row verifying its last token only (14, 15), and row slots
        # left empty after the padding rows' tokens (every other case from 16)
        n = 0 if case in (12, 13) else rng.randint(1, 10)
        lengths, tokens, tables, lens = [], [], [], []
        next_block = 0
        for _ in range(n):
            length = rng.randint(1, 1500)
            ln = 1 if case in (14, 15) else rng.randint(1, k + 1) if case % 2 else k + 1
            blocks = -(-(length - 1 + ln) // block_size)
            lengths.append(length)
            tokens.append(rng.randint(0, 150000))
            tables.append(list(range(next_block, next_block + blocks)))
            next_block += blocks
            lens.append(ln)
        num_rows = n + rng.randint(1 if case >= 12 else 0, 3)
        extra = rng.randint(0, (num_rows - n) * (k + 1))
        if case >= 16 and case % 2 == 0:
            extra = rng.randint(0, (num_rows - n - 1) * (k + 1))   # at least one row slot stays empty
        num_tokens = sum(lens) + extra
        seqs = [_Seq(a, b, c) for a, b, c in zip(lengths, tokens, tables)]
        m = verify_varlen_metadata(seqs, lens, k, block_size, num_rows, num_tokens, pad, width)
        prefix = f"meta/{case:02d}/"
        padded = np.full((n, width), -1, dtype=np.int64)
        for r, t in enumerate(tables):
            padded[r, :len(t)] = t
        params = dict(lengths=lengths, last_tokens=tokens, verified_lens=lens,
                      scalars=[k, block_size, num_rows, num_tokens, pad, width])
        for key, value in params.items():
            out[prefix + key] = np.array(value, dtype=np.int64)
        out[prefix + "tables"] = padded
        for key in ("input_ids", "positions", "slot_mapping", "cu_seqlens_q", "cu_seqlens_k", "draft_index",
                    "draft_source"):
            out[prefix + key] = np.array(getattr(m, key), dtype=np.int64)
        out[prefix + "block_tables"] = np.array(m.block_tables, dtype=np.int64)
    return out


def draft_block_cases() -> dict[str, np.ndarray]:
    """nanovllm/engine/batch_metadata.py draft_block_metadata on random batches (ragged block tables, padded batch
    sizes, no rows); ragged inputs stored padded with -1."""
    from nanovllm.engine.batch_metadata import draft_block_metadata
    import random
    out: dict[str, np.ndarray] = {}
    for case in range(12):
        rng = random.Random(2000 + case)
        k, block_size, width, pad, mask = 7, 256, 8, 999, 151669
        n = 0 if case == 0 else rng.randint(1, 10)
        lengths, tokens, tables = [], [], []
        next_block = 0
        for _ in range(n):
            length = rng.randint(1, 1500)
            blocks = -(-(length - 1 + k) // block_size)
            lengths.append(length)
            tokens.append(rng.randint(0, 150000))
            tables.append(list(range(next_block, next_block + blocks)))
            next_block += blocks
        padded_rows = n + rng.randint(0 if n else 1, 4)
        seqs = [_Seq(a, b, c) for a, b, c in zip(lengths, tokens, tables)]
        m = draft_block_metadata(seqs, block_size, k, mask, padded_rows, pad, width)
        prefix = f"draft/{case:02d}/"
        padded = np.full((n, width), -1, dtype=np.int64)
        for r, t in enumerate(tables):
            padded[r, :len(t)] = t
        out[prefix + "lengths"] = np.array(lengths, dtype=np.int64)
        out[prefix + "last_tokens"] = np.array(tokens, dtype=np.int64)
        out[prefix + "scalars"] = np.array([k, block_size, mask, padded_rows, pad, width], dtype=np.int64)
        out[prefix + "tables"] = padded
        for key in ("input_ids", "positions", "slot_mapping", "context_lens"):
            out[prefix + key] = np.array(getattr(m, key), dtype=np.int64)
        out[prefix + "block_tables"] = np.array(m.block_tables, dtype=np.int64)
    return out


def qwen3_forward_cases(reference: Path) -> dict[str, np.ndarray]:
    """The reference's Qwen3ForCausalLM (nanovllm/models/qwen3.py) on CPU bf16 over the inputs of
    tests/golden/qwen3_case.py: the verify layout (8 tokens at the end of each row's context, causal) through the
    reference's paged-attention stand-in (tests/fake_paged_attention.py, whose decode branch with 8 queries per
    row applies the verify rule), the aux layers' outputs exported (qwen3.py:186-190), all logits.  The fixture
    holds the outputs, the stored K/V rows and checksums of the inputs (regenerated from seeds by the tests)."""
    import torch.distributed as dist
    from transformers import Qwen3Config
    sys.path.insert(0, str(reference / "tests"))
    sys.path.insert(0, str(HERE))
    import fake_paged_attention as fpa
    import qwen3_case as Q
    from nanovllm.layers import attention as attention_module
    from nanovllm.models.qwen3 import Qwen3ForCausalLM
    from nanovllm.utils.context import reset_context, set_context
    if not dist.is_initialized():
        dist.init_process_group("gloo", init_method="tcp://127.0.0.1:29517", world_size=1, rank=0)
    case = Q.inputs()
    config = Qwen3Config(vocab_size=Q.VOCAB, hidden_size=Q.HIDDEN, intermediate_size=Q.FFN,
                         num_hidden_layers=Q.LAYERS, num_attention_heads=Q.HEADS, num_key_value_heads=Q.KV_HEADS,
                         head_dim=Q.HEAD_DIM, max_position_embeddings=Q.MAX_POSITION, rms_norm_eps=Q.EPS,
                         rope_theta=Q.ROPE_THETA, attention_bias=False, tie_word_embeddings=False,
                         hidden_act="silu")
    default = torch.get_default_dtype()
    torch.set_default_dtype(torch.bfloat16)
    try:
        model = Qwen3ForCausalLM(config)
    finally:
        torch.set_default_dtype(default)
    m = model.model
    m.embed_tokens.weight.data.copy_(case["embed"])
    m.norm.weight.data.copy_(case["final_norm"])
    model.lm_head.weight.data.copy_(case["lm_head"])
    for layer, w, (k_cache, v_cache) in zip(m.layers, case["layers"], case["caches"]):
        attn = layer.self_attn
        for module, key in ((attn.qkv_proj, "w_qkv"), (attn.o_proj, "w_o"), (attn.q_norm, "q_norm"),
                            (attn.k_norm, "k_norm"), (layer.mlp.gate_up_proj, "w_gate_up"),
                            (layer.mlp.down_proj, "w_down"), (layer.input_layernorm, "in_norm"),
                            (layer.post_attention_layernorm, "post_norm")):
            module.weight.data.copy_(w[key])
        attn.attn.k_cache, attn.attn.v_cache = k_cache.clone(), v_cache.clone()
    m.aux_layer_ids = Q.AUX_LAYER_IDS
    T = case["input_ids"].shape[0]
    original = attention_module.Attention.forward
    attention_module.Attention.forward = fpa.attention_forward
    set_context(False, slot_mapping=case["slot_mapping"], context_lens=case["key_lens"],
                block_tables=case["tables"], query_len_per_seq=Q.QUERY_LEN, causal=True)
    try:
        with torch.inference_mode():
            aux = torch.zeros(T, len(Q.AUX_LAYER_IDS) * Q.HIDDEN, dtype=torch.bfloat16)
            hidden = model(case["input_ids"], case["positions"], aux)
            logits = model.compute_logits(hidden, all_logits=True)
    finally:
        attention_module.Attention.forward = original
        reset_context()
    slots = case["slot_mapping"].long()
    out = {"qwen3/hidden": hidden.float().numpy(), "qwen3/aux": aux.float().numpy(),
           "qwen3/logits": logits.float().numpy(), "qwen3/checksums": np.array(Q.checksums(case))}
    for i, layer in enumerate(m.layers):
        cache_k, cache_v = layer.self_attn.attn.k_cache, layer.self_attn.attn.v_cache
        out[f"qwen3/k_stored{i}"] = cache_k.view(-1, Q.KV_HEADS, Q.HEAD_DIM)[slots].float().numpy()
        out[f"qwen3/v_stored{i}"] = cache_v.view(-1, Q.KV_HEADS, Q.HEAD_DIM)[slots].float().numpy()
    return out


def main() -> int:
    parser = argparse.ArgumentParser(description=__doc__)
    default_ref = os.environ.get("SPECDEC_REFERENCE", str(HERE.parents[2] / "reference"))
    parser.add_argument("--reference", default=default_ref)
    parser.add_argument("--only", choices=["metadata", "qwen3"], default=None, help="write only this fixture file")
    args = parser.parse_args()
    if args.only == "qwen3":
        import_reference(Path(args.reference))
        fx = qwen3_forward_cases(Path(args.reference))
        np.savez_compressed(HERE / "qwen3.npz", **fx)
        print(f"wrote {len(fx)} arrays to {HERE / 'qwen3.npz'}")
        return 0
    if args.only == "metadata":
        import_reference(Path(args.reference))
        meta = metadata_cases() | draft_block_cases()
        np.savez_compressed(HERE / "metadata.npz", **meta)
        print(f"wrote {len(meta)} arrays to {HERE / 'metadata.npz'}")
        return 0
    ss = import_reference(Path(args.reference))
    fixtures = {}
    fixtures.update(accept_cases(ss))
    fixtures.update(logits_cases(ss))
    fixtures.update(truncation_cases(ss))
    fixtures.update(greedy_cases(ss))
    np.savez_compressed(HERE / "sampler.npz", **fixtures)
    print(f"wrote {len(fixtures)} arrays to {HERE / 'sampler.npz'}")
    edges = {**masked_cases(ss), **greedy_edge_cases(ss)}
    np.savez_compressed(HERE / "sampler_edges.npz", **edges)
    print(f"wrote {len(edges)} arrays to {HERE / 'sampler_edges.npz'}")
    markov = markov_cases(Path(args.reference))
    np.savez_compressed(HERE / "markov.npz", **markov)
    print(f"wrote {len(markov)} arrays to {HERE / 'markov.npz'}")
    markov16 = markov_bf16_cases(Path(args.reference))
    np.savez_compressed(HERE / "markov_bf16.npz", **markov16)
    print(f"wrote {len(markov16)} arrays to {HERE / 'markov_bf16.npz'}")
    attn = attention_cases(Path(args.reference))
    np.savez_compressed(HERE / "attention.npz", **attn)
    print(f"wrote {len(attn)} arrays to {HERE / 'attention.npz'}")
    meta = metadata_cases() | draft_block_cases()
    np.savez_compressed(HERE / "metadata.npz", **meta)
    print(f"wrote {len(meta)} arrays to {HERE / 'metadata.npz'}")
    fwd = forward_helper_cases()
    np.savez_compressed(HERE / "forward.npz", **fwd)
    print(f"wrote {len(fwd)} arrays to {HERE / 'forward.npz'}")
    ctx = ctx_store_cases(Path(args.reference))
    np.savez_compressed(HERE / "ctx_store.npz", **ctx)
    print(f"wrote {len(ctx)} arrays to {HERE / 'ctx_store.npz'}")
    fx = qwen3_forward_cases(Path(args.reference))
    np.savez_compressed(HERE / "qwen3.npz", **fx)
    print(f"wrote {len(fx)} arrays to {HERE / 'qwen3.npz'}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
