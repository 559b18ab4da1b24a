"""The verify + accept round (speculative.py:411-512 restated in nanovllm_b200.speculative) on a small
Qwen3-shaped target: the captured graph reproduces the eager forward bit for bit, the paged KV store of the
verified positions lands where the metadata says, and the accepted drafts / tail equal the oracle's on the
graph's logits with the generator's draws."""
import math
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from oracle import spec_sampler as O

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


@pytest.fixture(scope="module")
def small_round():
    from nanovllm_b200 import spec_sampler as S
    from nanovllm_b200.batch_metadata import RowState
    from nanovllm_b200.speculative import VerifyRound
    from nanovllm_b200.target import Qwen3Shape, Qwen3Target
    shape = Qwen3Shape(hidden=256, layers=2, heads=4, kv_heads=2, intermediate=512, vocab=1000,
                       max_position=4096, aux_layer_ids=(0, 1))
    lengths = [300, 17, 513, 256]
    bs, k = 256, 7
    blocks = [math.ceil((n + k) / bs) for n in lengths]
    target = Qwen3Target(shape, DEV, sum(blocks) + 2, bs, seed=5, init_scale=0.05)
    target.kv_cache[:, :, :-1].normal_()
    perm = torch.randperm(sum(blocks) + 2, generator=torch.Generator().manual_seed(0)).tolist()
    rows, used = [], 0
    for n, nb in zip(lengths, blocks):
        rows.append(RowState(length=n, last_token=n % 997, block_table=perm[used:used + nb]))
        used += nb
    rnd = VerifyRound(target, k, [4], max(blocks))
    samp = S.sampling_tensors([SimpleNamespace(temperature=1.0, top_k=0, top_p=1.0)] * 4, DEV)
    g = torch.Generator(device=DEV).manual_seed(1)
    q = torch.softmax(torch.randn(4, k, shape.vocab, device=DEV, generator=g) * 2, -1)
    drafts = S.sample(q, g)
    return SimpleNamespace(S=S, target=target, rnd=rnd, rows=rows, samp=samp, q=q, drafts=drafts, k=k, shape=shape)


def test_graph_replay_equals_eager_forward(small_round):
    c = small_round
    num_tokens = c.rnd.load(c.rows)
    c.rnd.place_drafts(num_tokens, c.drafts)
    graph_logits = c.target.replay(num_tokens).clone()
    b = c.target.graphs[num_tokens][1]
    hidden = c.target.forward(b["input_ids"], b["positions"], b["slot_mapping"], b["cu_seqlens_q"],
                              b["cu_seqlens_k"], c.k + 1, b["block_tables"])
    eager_logits = c.target.compute_logits(hidden)
    assert torch.isfinite(eager_logits).all()
    assert torch.equal(graph_logits, eager_logits)
    # the verified positions' K/V were stored at their slots: position len-1+j of row r
    slots = b["slot_mapping"].cpu().tolist()
    for r, row in enumerate(c.rows):
        assert slots[r * 8] == row.block_table[(row.length - 1) // 256] * 256 + (row.length - 1) % 256


def test_round_accepts_like_the_oracle(small_round):
    c = small_round
    gen = torch.Generator(device=DEV).manual_seed(7)
    replay = torch.Generator(device=DEV)
    replay.set_state(gen.get_state())
    appended = c.rnd.run_round(c.rows, c.drafts, c.q, c.samp, gen)
    logits = c.target.graphs[32][1]["logits"].float().cpu().numpy()
    u = torch.rand(4, c.k, device=DEV, generator=replay).cpu().numpy()
    noise = c.S.exponential_noise_(torch.empty(4, c.shape.vocab, device=DEV), replay).cpu().numpy()
    p = O.probs_from_logits(logits, np.ones(32, np.float32))
    args = (c.q.cpu().numpy(), c.drafts.cpu().numpy(), np.full(4, 8), u, noise)
    n_accept, tail = O.accept_random_varlen(p, *args)
    flags = O.near_tie_flags(p, *args)
    for r in range(4):
        if flags[r]:
            continue
        want = c.drafts[r, :n_accept[r]].tolist() + [int(tail[r])]
        assert appended[r] == want
    assert gen.get_offset() == replay.get_offset()
    assert c.rnd.stats["rounds"] == 1
