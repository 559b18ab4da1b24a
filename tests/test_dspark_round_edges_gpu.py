"""Edge paths of the variable-length round (nanovllm_b200.speculative) on a small Qwen3 target and DSpark draft:
the drafter's batch padded past the real rows (5 rows in graphs of 8), rounds whose rows all verify only their
last token (nothing placed), all verify every draft, or mix the extremes, greedy and sampled; several rounds in a
row on the same graphs.  Each round is checked stage by stage against the oracle as in
tests/test_dspark_round_gpu.py: Markov drafts and q, the drafts' places among the input ids, the accepted tokens,
and the draft cache rows after_verify wrote."""
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
B, K, BS, V = 5, 7, 256, 1000


@pytest.fixture(scope="module")
def small():
    from nanovllm_b200.batch_metadata import RowState
    from nanovllm_b200.dflash import DFlashDraftModel
    from nanovllm_b200.speculative import DFlashDrafter, SpeculativeDecoder, verify_token_counts
    from nanovllm_b200.target import Qwen3Shape, Qwen3Target
    gen = torch.Generator().manual_seed(9)
    lengths = [300, 17, 513, 256, 90]
    blocks = [math.ceil((n + K) / BS) for n in lengths]
    num_blocks = sum(blocks) + 2
    width = max(blocks)
    perm = torch.randperm(num_blocks, generator=gen).tolist()
    tshape = Qwen3Shape(hidden=256, layers=3, heads=4, kv_heads=1, intermediate=512, vocab=V, max_position=4096,
                        aux_layer_ids=(0, 1, 2))
    target = Qwen3Target(tshape, DEV, num_blocks, BS, seed=5, init_scale=0.08)
    dshape = Qwen3Shape(hidden=256, layers=2, heads=4, kv_heads=1, intermediate=512, vocab=V, max_position=4096,
                        aux_layer_ids=(0, 1, 2))
    model = DFlashDraftModel(dshape, tshape.aux_layer_ids, DEV, num_blocks, BS, markov_rank=64, mask_token_id=V - 1,
                             seed=6, init_scale=0.08, markov_scale=0.3)
    for cache, seed in ((target.kv_cache, 7), (model.kv_cache, 8)):
        g = torch.Generator(device=DEV).manual_seed(seed)
        for layer in range(cache.shape[1]):
            cache[:, layer, :num_blocks].normal_(generator=g)
    rows, used = [], 0
    for n, nb in zip(lengths, blocks):
        rows.append(RowState(length=n, last_token=int(torch.randint(V, (1,), generator=gen)),
                             block_table=perm[used:used + nb]))
        used += nb
    drafter = DFlashDrafter(model, K, [8], width, target.pad_block_id)
    dec = SpeculativeDecoder(target, drafter, K, width, token_counts=verify_token_counts(8, K + 1))
    yield SimpleNamespace(target=target, model=model, drafter=drafter, dec=dec, rows=rows)
    dec.close()


def sampling_of(params):
    from nanovllm_b200 import spec_sampler as S
    return S.sampling_tensors([SimpleNamespace(temperature=t, top_k=k, top_p=p) for t, k, p in params], DEV)


def check_round(c, sampling, lens, seed):
    from nanovllm_b200.markov import num_candidates
    from nanovllm_b200.speculative import sampling_graph_key
    from oracle.ctx_store import bf16
    greedy = sampling.temperatures is None
    gen = None if greedy else torch.Generator(device=DEV).manual_seed(seed)
    replay = None
    if gen is not None:
        replay = torch.Generator(device=DEV)
        replay.set_state(gen.get_state())
    appended = c.dec.run_round(c.rows, sampling, gen, verified_lens=lens)
    key = sampling_graph_key(sampling)
    cand = 0 if greedy else num_candidates(sampling.max_top_k, sampling.all_top_k, V)
    noise = u = tail_noise = None
    if not greedy:
        noise = torch.empty(B, K, cand or V, device=DEV).exponential_(1.0, generator=replay).clamp_min_(1e-10)
        u = torch.rand(B, K, device=DEV, generator=replay).cpu().numpy()
        tail_noise = torch.empty(B, V, device=DEV).exponential_(1.0, generator=replay).clamp_min_(1e-10)
        assert gen.get_offset() == replay.get_offset()
    # propose: the Markov rows of the real rows (the padded batch's first B rows)
    drafts = c.drafter.drafts[:B].clone()
    logits = c.drafter.logits[key, 8][:B].float().cpu().numpy()
    head = c.model.markov_head
    anchors = torch.tensor([row.last_token for row in c.rows], device=DEV)
    prevs = [anchors] + [drafts[:, j] for j in range(K - 1)]
    biases = iter([torch.matmul(head.w1[p].contiguous(), head.w2.t()).float().cpu().numpy() for p in prevs])
    params = None if greedy else dict(temps=sampling.temperatures.cpu().numpy(), top_k=sampling.top_k.cpu().numpy(),
                                      top_p=sampling.top_p.cpu().numpy(), max_top_k=sampling.max_top_k,
                                      has_top_p=sampling.has_top_p)
    want_d, want_q = OM.markov_rows(logits, anchors.cpu().numpy(), lambda _p: next(biases), params,
                                    None if noise is None else noise.cpu().numpy(), cand, round_fn=bf16)
    d = drafts.cpu().numpy()
    diverged = (d != want_d).any(axis=1)
    assert diverged.sum() <= 1
    q = None
    if not greedy:
        q = c.drafter.q[key].probs[:B].cpu().numpy() if cand else c.drafter.q[key][:B].cpu().numpy()
        np.testing.assert_allclose(q[~diverged], want_q[~diverged], rtol=1e-5, atol=1e-8)
    # verify: the drafts' places
    num_tokens = c.dec.verify.graph_for(B, sum(lens))
    buffers = c.target.graphs[num_tokens][1]
    ids = buffers["input_ids"].cpu().numpy()
    start = 0
    for r, (row, ln) in enumerate(zip(c.rows, lens)):
        assert ids[start:start + ln].tolist() == [row.last_token] + d[r, :ln - 1].tolist()
        start += ln
    # accept
    target_logits = c.dec.verify.logits(num_tokens).float().cpu().numpy()
    ln = np.asarray(lens, dtype=np.int64)
    if greedy:
        n, tail = O.accept_greedy_varlen(target_logits, d, ln)
        flagged = np.zeros(B, bool)
    else:
        tk = sampling.top_k.cpu().numpy()
        p = O.probs_from_logits(target_logits, np.repeat(sampling.temperatures.cpu().numpy(), ln), np.repeat(tk, ln),
                                np.repeat(sampling.top_p.cpu().numpy(), ln), sampling.max_top_k, sampling.has_top_p)
        n, tail = O.accept_random_varlen(p, q, d, ln, u, tail_noise.cpu().numpy())
        flagged = O.near_tie_flags(p, q, d, ln, u, tail_noise.cpu().numpy())
    assert flagged.sum() <= 1
    for r in range(B):
        if not flagged[r]:
            assert appended[r] == d[r, :n[r]].tolist() + [int(tail[r])]
    # after_verify: the draft cache rows at the verified slots, from the graph's own projection
    T = sum(lens)
    kv = buffers["context_kv"][:T].float().cpu().numpy()
    positions = buffers["positions"][:T].cpu().numpy()
    slots = buffers["slot_mapping"][:T].to(torch.int64)
    s = c.model.shape
    width = 2 * s.kv_heads * 128
    for layer in range(s.layers):
        want_k = np.zeros((T, s.kv_heads, 128), np.float32)
        want_v = np.zeros((T, s.kv_heads, 128), np.float32)
        OC.norm_rope_store(kv[:, layer * width:(layer + 1) * width], s.kv_heads,
                           c.model.k_norm[layer].float().cpu().numpy(), c.model.cos_sin.cpu().numpy(), positions,
                           np.arange(T), want_k, want_v, 1e-6)
        got_k = c.model.kv_cache[0, layer].view(-1, s.kv_heads, 128)[slots].float().cpu().numpy()
        got_v = c.model.kv_cache[1, layer].view(-1, s.kv_heads, 128)[slots].float().cpu().numpy()
        ok = np.abs(got_k - want_k) <= 2.0 ** -7 * np.maximum(np.abs(got_k), np.abs(want_k)) + 1e-6
        assert ok.mean() >= 0.999 and np.abs(got_k - want_k).max() < 2e-2
        assert np.array_equal(got_v, want_v)
    return appended


LENS = {"mixed": [1, 8, 3, 8, 1], "last_token_only": [1] * B, "all_drafts": [K + 1] * B}


@pytest.mark.parametrize("lens", list(LENS))
@pytest.mark.parametrize("mode", ["greedy", "sampled"])
def test_round_edges_match_the_oracle(small, lens, mode):
    params = ([(0.0, 0, 1.0)] * B if mode == "greedy" else
              [(1.0, 20, 1.0), (0.8, 20, 0.9), (1.2, 20, 1.0), (0.7, 20, 0.95), (1.0, 20, 1.0)])
    out = check_round(small, sampling_of(params), LENS[lens], seed=len(lens) * 7 + (mode == "greedy"))
    assert all(1 <= len(o) <= ln for o, ln in zip(out, LENS[lens]))


def test_whole_vocabulary_rows_and_rounds_in_a_row(small):
    """A batch where some row does not truncate draws its Markov rows over the whole vocabulary (dense q); three
    rounds in a row on the same graphs, each against the oracle."""
    params = [(1.0, 0, 1.0), (0.9, 30, 1.0), (1.0, 0, 0.8), (1.1, 5, 1.0), (1.0, 0, 1.0)]
    for i, lens in enumerate([[2, 8, 5, 1, 7], [8, 8, 1, 1, 4], [3, 3, 3, 3, 3]]):
        check_round(small, sampling_of(params), lens, seed=100 + i)


def test_keys_past_the_graph_limit_sample_eagerly_and_alike(small, monkeypatch):
    """A drafter that may capture no sampling graph (MAX_SAMPLING_KEYS = 0) runs the graphs' body eagerly
    (speculative.py:41-43): the same drafts, q and generator offset as the captured graph, bit for bit."""
    from nanovllm_b200 import speculative
    from nanovllm_b200.speculative import DFlashDrafter, sampling_graph_key
    params = [(1.0, 20, 1.0), (0.8, 20, 0.9), (1.2, 20, 1.0), (0.7, 20, 0.95), (1.0, 20, 1.0)]
    sampling = sampling_of(params)
    g1 = torch.Generator(device=DEV).manual_seed(55)
    d1, q1 = small.drafter.propose(small.rows, sampling, g1)
    d1, q1 = d1.clone(), q1.clone()
    monkeypatch.setattr(speculative, "MAX_SAMPLING_KEYS", 0)
    eager = DFlashDrafter(small.model, K, [8], small.drafter.max_num_blocks, small.drafter.pad_block_id)
    g2 = torch.Generator(device=DEV).manual_seed(55)
    d2, q2 = eager.propose(small.rows, sampling, g2)
    assert eager.stats["eager_proposals"] == 1 and not eager.sampling_graphs
    assert sampling_graph_key(sampling) in eager.noise
    assert torch.equal(d1, d2) and torch.equal(q1, q2)
    assert g1.get_offset() == g2.get_offset()
