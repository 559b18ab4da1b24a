"""The variable-length DSpark round of benchmark config 4 (SpeculativeDecoder.run_round with verified_lens,
nanovllm/engine/speculative.py:411-462), end to end on the B200 path, checked stage by stage against the oracle:

  propose       the drafter's block graph + Markov sampling graph: drafts bit-exact against oracle/markov.py run on
                the graph's draft logits with the same noise (a row may diverge only after a near-tie step), q
                within 1e-5 relative;
  verify        the verification graph at the round's token bucket: the drafts sit where the reference's
                metadata puts them;
  after_verify  inside that graph: fc and W_kv projections against fp32 products (bf16 rounding), hidden_norm and
                the draft cache rows at every verified slot against oracle/ctx_store.py (99.9 % within one bf16
                ulp, all within 2e-2; V rows exact);
  accept        each row's accepted drafts and tail bit-exact against oracle/spec_sampler.py on the graph's
                logits with the generator's draws, except near-tie requests, counted by kind.

Shapes: B = 64 rows, k = 7, contexts ~3000 tokens (U[2950, 3050]) in 256-slot blocks (random block permutation),
verified lengths uniform on {1..8} (mean 4.5), a random-init Qwen3-8B-architecture target (36 layers) exporting
its 5 aux layers, a random-init 5-layer draft of the same widths with a rank-256 Markov head, top_k 128
(192 candidates), vocabulary 151936, bf16."""
import math
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from oracle import ctx_store as OC
from oracle import markov as OM
from oracle import spec_sampler as O

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
B, K, CTX, BS = 64, 7, 3000, 256
ULP = 2 ** -7          # one bf16 step relative to the value


def close_bf16(got: np.ndarray, want: np.ndarray, frac: float = 0.999) -> None:
    """The ctx_store tolerance of tests/test_ctx_store_gpu.py: at least 99.9 % of the values within one bf16 ulp
    of the larger magnitude (rsqrt and accumulation order may move the last bit, and RoPE's differences of
    products near zero move it further in relative terms), every value within 2e-2 absolute."""
    ok = np.abs(got - want) <= ULP * np.maximum(np.abs(got), np.abs(want)) + 1e-6
    assert ok.mean() >= frac, f"{(~ok).sum()} of {ok.size} beyond one bf16 ulp"
    np.testing.assert_allclose(got, want, atol=2e-2, rtol=0)


def gemm_close(got: np.ndarray, want: np.ndarray) -> None:
    """A bf16 GEMM output against the fp32 product: one bf16 rounding plus summation order."""
    assert np.all(np.abs(got - want) <= np.abs(want) * 2 ** -8 + 1e-3 * np.abs(want).max())


@pytest.fixture(scope="module")
def dspark():
    from nanovllm_b200.batch_metadata import RowState
    from nanovllm_b200.dflash import DFlashDraftModel
    from nanovllm_b200.speculative import DFlashDrafter, SpeculativeDecoder
    from nanovllm_b200.target import Qwen3Shape, Qwen3Target
    gen = torch.Generator().manual_seed(4)
    lengths = torch.randint(CTX - 50, CTX + 51, (B,), generator=gen).tolist()
    lens = torch.randint(1, K + 2, (B,), generator=gen).tolist()
    blocks = [math.ceil((n + K) / BS) for n in lengths]
    num_blocks = sum(blocks) + 4
    width = max(blocks)
    perm = torch.randperm(num_blocks, generator=gen).tolist()
    shape = Qwen3Shape()
    target = Qwen3Target(shape, DEV, num_blocks, BS, seed=40)
    model = DFlashDraftModel(Qwen3Shape(layers=5), shape.aux_layer_ids, DEV, num_blocks, BS, markov_rank=256,
                             seed=41)
    for cache, seed in ((target.kv_cache, 42), (model.kv_cache, 43)):
        g = torch.Generator(device=DEV).manual_seed(seed)
        for layer in range(cache.shape[1]):
            cache[:, layer, :num_blocks].normal_(generator=g)     # the contexts' K/V; the pad block stays zero
    rows, used = [], 0
    for n, nb in zip(lengths, blocks):
        rows.append(RowState(length=n, last_token=int(torch.randint(shape.vocab, (1,), generator=gen)),
                             block_table=perm[used:used + nb]))
        used += nb
    drafter = DFlashDrafter(model, K, [B], width, target.pad_block_id)
    bucket = -(-sum(lens) // (K + 1)) * (K + 1)
    dec = SpeculativeDecoder(target, drafter, K, width, token_counts=[bucket])
    yield SimpleNamespace(target=target, model=model, drafter=drafter, dec=dec, rows=rows, lens=lens, bucket=bucket,
                          V=shape.vocab)
    dec.close()


def sampling_of(temps, top_k, top_p):
    from nanovllm_b200 import spec_sampler as S
    seqs = [SimpleNamespace(temperature=t, top_k=k, top_p=p) for t, k, p in zip(temps, top_k, top_p)]
    return S.sampling_tensors(seqs, DEV)


def markov_oracle(c, sampling, noise, candidates):
    """oracle/markov.py on the sampling graph's draft logits, each step's Markov bias recomputed with the same
    cuBLAS product the round runs (W1[prev] . W2^T for the previous step's drafted token)."""
    from nanovllm_b200.speculative import sampling_graph_key
    from oracle.ctx_store import bf16
    key = sampling_graph_key(sampling)
    logits = c.drafter.logits[key, B].float().cpu().numpy()
    drafts = c.drafter.drafts[:B].clone()
    anchors = torch.tensor([row.last_token for row in c.rows], device=DEV)
    head = c.model.markov_head
    prevs = [anchors] + [drafts[:, j] for j in range(K - 1)]
    biases = iter([torch.matmul(head.w1[p].contiguous(), head.w2.t()).float().cpu().numpy() for p in prevs])
    params = None if sampling.temperatures is None else dict(
        temps=sampling.temperatures.cpu().numpy(), top_k=sampling.top_k.cpu().numpy(),
        top_p=sampling.top_p.cpu().numpy(), max_top_k=sampling.max_top_k, has_top_p=sampling.has_top_p)
    want, want_q = OM.markov_rows(logits, anchors.cpu().numpy(), lambda _prev: next(biases), params,
                                  None if noise is None else noise.cpu().numpy(), candidates, round_fn=bf16)
    return drafts.cpu().numpy(), want, want_q


def check_after_verify(c, num_tokens):
    """The draft cache rows the verification graph's after_verify wrote at the verified tokens' slots."""
    buffers = c.target.graphs[num_tokens][1]
    T = sum(c.lens)
    aux = buffers["aux"][:T]
    fc = buffers["context_fc"][:T]
    gemm_close(fc.float().cpu().numpy(), (aux.float() @ c.model.w_fc.float().t()).cpu().numpy())
    features = buffers["context_features"][:T].float().cpu().numpy()
    close_bf16(features, OC.rmsnorm(fc.float().cpu().numpy(), c.model.hidden_norm.float().cpu().numpy(), 1e-6))
    kv = buffers["context_kv"][:T]
    gemm_close(kv.float().cpu().numpy(), (buffers["context_features"][:T].float() @ c.model.w_kv.float().t())
               .cpu().numpy())
    kv = kv.float().cpu().numpy()
    positions = buffers["positions"][:T].cpu().numpy()
    slots = buffers["slot_mapping"][:T].to(torch.int64)
    assert (slots >= 0).all()
    s = c.model.shape
    width = 2 * s.kv_heads * 128
    cos_sin = c.model.cos_sin.cpu().numpy()
    local = np.arange(T)
    for layer in range(s.layers):
        want_k = np.zeros((T, s.kv_heads, 128), np.float32)
        want_v = np.zeros((T, s.kv_heads, 128), np.float32)
        OC.norm_rope_store(kv[:, layer * width:(layer + 1) * width], s.kv_heads,
                           c.model.k_norm[layer].float().cpu().numpy(), cos_sin, positions, local, want_k, want_v,
                           1e-6)
        got_k = c.model.kv_cache[0, layer].view(-1, s.kv_heads, 128)[slots].float().cpu().numpy()
        got_v = c.model.kv_cache[1, layer].view(-1, s.kv_heads, 128)[slots].float().cpu().numpy()
        close_bf16(got_k, want_k)
        assert np.array_equal(got_v, want_v)


def test_config4_round_matches_the_oracle_stage_by_stage(dspark):
    c = dspark
    temps = [1.0] * (B // 2) + [0.8] * (B // 2)
    top_p = [1.0, 0.9] * (B // 2)
    sampling = sampling_of(temps, [128] * B, top_p)
    gen = torch.Generator(device=DEV).manual_seed(11)
    replay = torch.Generator(device=DEV)
    replay.set_state(gen.get_state())
    appended = c.dec.run_round(c.rows, sampling, gen, verified_lens=c.lens)
    num_tokens = c.dec.verify.graph_for(B, sum(c.lens))
    assert num_tokens == c.bucket
    # the round's draws, replayed in the reference's order: Markov noise [B, k, C] (speculative.py:225-238),
    # then the accept's u [B, k] and tail noise [B, V] (spec_sampler.py:141, 149)
    candidates = OM.num_candidates(128, True, c.V)
    noise = torch.empty(B, K, candidates, device=DEV).exponential_(1.0, generator=replay).clamp_min_(1e-10)
    u = torch.rand(B, K, device=DEV, generator=replay).cpu().numpy()
    tail_noise = torch.empty(B, c.V, device=DEV).exponential_(1.0, generator=replay).clamp_min_(1e-10)
    assert gen.get_offset() == replay.get_offset()
    # propose: Markov rows
    from nanovllm_b200.speculative import sampling_graph_key
    q_buf = c.drafter.q[sampling_graph_key(sampling)].probs[:B]
    drafts, want_drafts, want_q = markov_oracle(c, sampling, noise, candidates)
    diverged = (drafts != want_drafts).any(axis=1)
    assert diverged.sum() <= 1, f"{int(diverged.sum())} rows diverge from the oracle's Markov rows"
    q = q_buf.cpu().numpy()
    np.testing.assert_allclose(q[~diverged], want_q[~diverged], rtol=1e-5, atol=1e-8)
    # verify: the drafts where the reference's metadata puts them (speculative.py:514-517)
    ids = c.target.graphs[num_tokens][1]["input_ids"].cpu().numpy()
    start = 0
    for r, (row, ln) in enumerate(zip(c.rows, c.lens)):
        assert ids[start:start + ln].tolist() == [row.last_token] + drafts[r, :ln - 1].tolist()
        start += ln
    # after_verify inside the verification graph
    check_after_verify(c, num_tokens)
    # accept, on the graph's logits and the GPU's drafts / q
    logits = c.dec.verify.logits(num_tokens).float().cpu().numpy()
    lens = np.asarray(c.lens, dtype=np.int64)
    p = O.probs_from_logits(logits, np.repeat(np.asarray(temps, np.float32), lens),
                            np.repeat(np.full(B, 128, np.int64), lens), np.repeat(np.asarray(top_p, np.float32), lens),
                            128, True)
    n_accept, tail = O.accept_random_varlen(p, q, drafts, lens, u, tail_noise.cpu().numpy())
    accept_flags, race_flags = O.near_tie_kinds(p, q, drafts, lens, u, tail_noise.cpu().numpy())
    flagged = accept_flags | race_flags
    assert flagged.sum() <= 2, (int(accept_flags.sum()), int(race_flags.sum()))
    for r in range(B):
        if not flagged[r]:
            assert appended[r] == drafts[r, :n_accept[r]].tolist() + [int(tail[r])], r
    assert all(1 <= len(a) <= ln for a, ln in zip(appended, c.lens))
    assert c.dec.stats["rounds"] == 1 and sum(v for key, v in c.dec.stats.items() if key.startswith("verified_")) == B
    print(f"config-4 round: {int(accept_flags.sum())} accept-draw and {int(race_flags.sum())} race near ties "
          f"of {B} requests; {int(diverged.sum())} Markov rows diverged after a near tie")


def test_config4_greedy_round_matches_the_oracle(dspark):
    """Greedy rows (temperature 0): Markov argmax rows and the greedy varlen accept, both bit-exact."""
    c = dspark
    sampling = sampling_of([0.0] * B, [0] * B, [1.0] * B)
    appended = c.dec.run_round(c.rows, sampling, None, verified_lens=c.lens)
    drafts, want_drafts, _ = markov_oracle(c, sampling, None, 0)
    assert np.array_equal(drafts, want_drafts)
    num_tokens = c.dec.verify.graph_for(B, sum(c.lens))
    logits = c.dec.verify.logits(num_tokens).float().cpu().numpy()
    n_accept, tail = O.accept_greedy_varlen(logits, drafts, np.asarray(c.lens, dtype=np.int64))
    for r in range(B):
        assert appended[r] == drafts[r, :n_accept[r]].tolist() + [int(tail[r])]
    check_after_verify(c, num_tokens)


def test_draft_block_graph_equals_its_eager_forward(dspark):
    """The drafter's captured block forward reproduces the eager forward bit for bit (same kernels, same
    inputs): the block's hidden states and its K/V stored at the block's slots."""
    c = dspark
    padded = c.drafter.load(c.rows)
    c.drafter.graphs[padded].replay()
    graph_out = c.drafter.outputs[:B * K].clone()
    v = c.drafter.views[padded]
    eager = c.model.forward(v["input_ids"], v["positions"], v["slot_mapping"], v["context_lens"], v["block_tables"],
                            K)
    assert torch.isfinite(eager).all()
    assert torch.equal(graph_out, eager)
    # the block's K/V sit at positions anchor .. anchor + k - 1 of the draft cache
    slots = v["slot_mapping"][:B * K].cpu().tolist()
    for r, row in enumerate(c.rows):
        p = row.length - 1
        assert slots[r * K] == row.block_table[p // BS] * BS + p % BS
