"""The properties the reference's own sampler and DSpark suites pin, restated with cases of this file's own and run
on CUDA through the B200 modules (the reference's test files do not travel to the GPU box):

  tests/test_spec_sampler.py:208-221         fixed-length accept_random / accept_greedy keep the pre-varlen rule:
                                             same accepts, same tails, same generator state;
  tests/test_accept_random_multistep.py      the output distribution of rounds of k drafts (sample + accept_random,
                                             and accept_random_varlen with per-row lengths) is the target's, every
                                             output sequence's frequency within a Hoeffding bound (its cuda
                                             parameter, :22);
  tests/test_dspark_propose.py:39-133        DSpark's rows: greedy drafts follow the Markov chain, q is each row's
                                             distribution after its bias, a zero bias draws what DFlash draws (same
                                             generator state), candidate rows give the whole-vocabulary
                                             distribution with ties at the cut kept, and the sampling graph draws
                                             what the eager rows draw.
"""
import itertools
import math
from collections import Counter
from types import SimpleNamespace

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


@pytest.fixture(scope="module")
def S():
    from nanovllm_b200 import spec_sampler
    return spec_sampler


def sampling_of(S, params):
    seqs = [SimpleNamespace(temperature=t, top_k=k, top_p=p) for t, k, p in params]
    return S.sampling_tensors(seqs, DEV)


# ---------------------------------------------------------------------------------------------- the fixed-length rule
def rule_accept_random(p, q, drafts, generator):
    """The rejection rule of a batch verifying all k drafts, in plain torch (spec_sampler.py:114-150 at k + 1
    positions per row): u [B, k] drawn first, accept while u q_d < p_d, then the residual (p - q)+ or the bonus row
    raced with Exp(1) noise [B, V] drawn second, clamped at 1e-10."""
    B, k = drafts.shape
    rows = torch.arange(B, device=p.device)
    u = torch.rand(B, k, device=p.device, generator=generator)
    p_d = p[:, :k].gather(-1, drafts.unsqueeze(-1)).squeeze(-1)
    q_d = q.gather(-1, drafts.unsqueeze(-1)).squeeze(-1)
    n = ((u * q_d) < p_d).long().cumprod(-1).sum(-1)
    p_next = p[rows, n]
    q_next = q[rows, n.clamp(max=k - 1)]
    w = torch.where((n == k).unsqueeze(-1), p_next, (p_next - q_next).clamp_min(0))
    noise = torch.empty_like(w).exponential_(1.0, generator=generator).clamp_min_(1e-10)
    return n, (w / noise).argmax(-1)


@pytest.mark.parametrize("seed", range(5))
def test_every_row_verifying_all_drafts_keeps_the_fixed_length_rule(S, seed):
    g = torch.Generator(device=DEV).manual_seed(100 + seed)
    B, k, V = 6, 7, 5
    p = torch.softmax(torch.randn(B, k + 1, V, device=DEV, generator=g), -1)
    q = torch.softmax(torch.randn(B, k, V, device=DEV, generator=g), -1)
    drafts = torch.randint(V, (B, k), device=DEV, generator=g)
    ours = torch.Generator(device=DEV).manual_seed(seed)
    theirs = torch.Generator(device=DEV).manual_seed(seed)
    got = S.accept_random(p, q, drafts, ours)
    want = rule_accept_random(p, q, drafts, theirs)
    assert torch.equal(got[0], want[0]) and torch.equal(got[1], want[1])
    assert ours.get_offset() == theirs.get_offset()
    logp = p.log()
    n, tail = S.accept_greedy(logp, drafts)
    target = logp.argmax(-1)
    want_n = (target[:, :k] == drafts).long().cumprod(-1).sum(-1)
    assert torch.equal(n, want_n) and torch.equal(tail, target[torch.arange(B, device=DEV), want_n])


# ---------------------------------------------------------------------------------------------- output distribution
# A four-token Markov source: token 3 is EOS, outputs stop at EOS or after MAX_TOKENS tokens.  State 0 precedes the
# first token, state x + 1 follows token x.  The draft's rows differ from the target's, so rejections and residual
# draws happen often.
TARGET_ROWS = [[0.50, 0.25, 0.15, 0.10], [0.10, 0.60, 0.20, 0.10], [0.30, 0.10, 0.40, 0.20],
               [0.20, 0.20, 0.20, 0.40], [0.25, 0.25, 0.25, 0.25]]
DRAFT_ROWS = [[0.20, 0.50, 0.20, 0.10], [0.40, 0.30, 0.20, 0.10], [0.25, 0.25, 0.25, 0.25],
              [0.10, 0.70, 0.10, 0.10], [0.60, 0.10, 0.20, 0.10]]
EOS, MAX_TOKENS, TRIALS, FAILURE = 3, 3, 100_000, 1e-3


def exact_distribution() -> dict:
    """Every output sequence's probability under the target alone."""
    out = {}
    for length in range(1, MAX_TOKENS + 1):
        for seq in itertools.product(range(4), repeat=length):
            if EOS in seq[:-1] or (length < MAX_TOKENS and seq[-1] != EOS):
                continue
            prob, state = 1.0, 0
            for token in seq:
                prob *= TARGET_ROWS[state][token]
                state = token + 1
            out[seq] = prob
    assert abs(sum(out.values()) - 1.0) < 1e-9
    return out


def run_rounds(S, k: int, generator, lengths=None) -> list[tuple]:
    """TRIALS rows, round by round until each stops (in chunks of 1024 requests, the sampler's batch cap):
    drafts sampled from the draft's rows, accepted against the target's (all k positions, or the first
    lengths(rows) - 1 through accept_random_varlen)."""
    p_rows = torch.tensor(TARGET_ROWS, device=DEV)
    q_rows = torch.tensor(DRAFT_ROWS, device=DEV)
    outputs = []
    for start in range(0, TRIALS, 1024):
        n = min(1024, TRIALS - start)
        out = [[] for _ in range(n)]
        state = [0] * n
        active = list(range(n))
        while active:
            states, drafts = [torch.tensor([state[r] for r in active], device=DEV)], []
            for _ in range(k):
                drafts.append(S.sample(q_rows[states[-1]], generator))
                states.append(drafts[-1] + 1)
            p = torch.stack([p_rows[s] for s in states], 1)
            q = torch.stack([q_rows[s] for s in states[:-1]], 1)
            drafts = torch.stack(drafts, 1)
            if lengths is None:
                n_accept, tail = S.accept_random(p, q, drafts, generator)
            else:
                lens = lengths(len(active))
                verified = torch.arange(k + 1, device=DEV) < lens.unsqueeze(1)
                n_accept, tail = S.accept_random_varlen(p[verified], q, drafts, lens, generator)
            rounds = torch.cat([drafts, tail[:, None]], 1).tolist()
            still = []
            for row, tokens, count in zip(active, rounds, n_accept.tolist()):
                for token in tokens[:count] + [tokens[k]]:
                    out[row].append(token)
                    if token == EOS or len(out[row]) == MAX_TOKENS:
                        break
                if out[row][-1] != EOS and len(out[row]) < MAX_TOKENS:
                    still.append(row)
                    state[row] = out[row][-1] + 1
            active = still
        outputs += [tuple(o) for o in out]
    return outputs


@pytest.mark.parametrize("mode", ["all_drafts", "varlen"])
def test_output_distribution_is_the_targets(S, mode):
    expected = exact_distribution()
    bound = math.sqrt(math.log(2 * len(expected) / FAILURE) / (2 * TRIALS))      # Hoeffding, union over sequences
    generator = torch.Generator(device=DEV).manual_seed(7 if mode == "all_drafts" else 8)
    len_gen = torch.Generator(device=DEV).manual_seed(9)
    lengths = None if mode == "all_drafts" else (
        lambda n: torch.randint(1, 4, (n,), device=DEV, generator=len_gen))         # lengths drawn apart from drafts
    counts = Counter(run_rounds(S, 2, generator, lengths))
    assert set(counts) <= set(expected)
    worst = max(abs(counts.get(seq, 0) / TRIALS - prob) for seq, prob in expected.items())
    assert worst <= bound, (worst, bound)


# ---------------------------------------------------------------------------------------------- DSpark rows
class LookupHead:
    """A Markov head whose bias is a row of a table by previous token."""

    def __init__(self, table):
        self.table = table

    def __call__(self, prev):
        return self.table[prev]


def test_greedy_drafts_follow_the_markov_chain(S):
    from nanovllm_b200.markov import markov_rows
    # every row's base logits pick token 0; after token 0 the bias lifts token 1 above it, after token 1 it does not
    bias = torch.tensor([[0.0, 2.0, 0.0], [0.0, 0.0, 0.0], [0.0, 0.0, 0.0]], device=DEV)
    logits = torch.tensor([2.0, 1.0, 0.0], device=DEV).expand(2, 3, 3).contiguous()
    drafts = torch.empty(2, 3, dtype=torch.int64, device=DEV)
    markov_rows(logits, torch.tensor([0, 1], device=DEV), None, None, drafts, None, 0, LookupHead(bias))
    assert drafts.tolist() == [[1, 0, 1], [0, 1, 0]]


def test_q_is_each_rows_distribution_after_its_bias(S):
    from nanovllm_b200.markov import markov_rows
    bias = torch.randn(3, 3, device=DEV, generator=torch.Generator(device=DEV).manual_seed(11))
    sampling = sampling_of(S, [(1.0, 0, 1.0), (0.7, 2, 1.0)])
    g = torch.Generator(device=DEV).manual_seed(1)
    logits = torch.randn(2, 4, 3, device=DEV, generator=g)
    noise = S.exponential_noise_(torch.empty(2, 4, 3, device=DEV), g)
    drafts = torch.empty(2, 4, dtype=torch.int64, device=DEV)
    probs = torch.empty(2, 4, 3, device=DEV)
    markov_rows(logits, torch.tensor([0, 1], device=DEV), sampling, noise, drafts, probs, 0, LookupHead(bias))
    prev = torch.tensor([0, 1], device=DEV)
    for row in range(4):
        assert torch.equal(probs[:, row], S.probs_from_logits(logits[:, row] + bias[prev], sampling))
        prev = drafts[:, row]


def test_without_a_bias_the_rows_draw_what_dflash_draws(S):
    from nanovllm_b200.markov import markov_rows
    sampling = sampling_of(S, [(1.0, 0, 1.0), (0.7, 3, 0.9)])       # one row does not truncate: whole vocabulary
    logits = torch.randn(2, 4, 6, device=DEV, generator=torch.Generator(device=DEV).manual_seed(2))
    ours = torch.Generator(device=DEV).manual_seed(0)
    noise = S.exponential_noise_(torch.empty(2, 4, 6, device=DEV), ours)   # all k rows' noise, drawn at once
    drafts = torch.empty(2, 4, dtype=torch.int64, device=DEV)
    probs = torch.empty(2, 4, 6, device=DEV)
    markov_rows(logits, torch.tensor([2, 0], device=DEV), sampling, noise, drafts, probs, 0,
                LookupHead(torch.zeros(6, 6, device=DEV)))
    dflash = torch.Generator(device=DEV).manual_seed(0)
    dflash_probs = S.probs_from_logits(logits, sampling)
    assert torch.equal(probs, dflash_probs)
    assert torch.equal(drafts, S.sample(dflash_probs, dflash))
    assert ours.get_offset() == dflash.get_offset()


def test_candidate_rows_give_the_whole_vocabulary_distribution(S):
    from nanovllm_b200.markov import markov_rows, num_candidates
    V, k = 200, 4
    sampling = sampling_of(S, [(0.7, 3, 1.0), (1.0, 20, 0.8)])
    g = torch.Generator(device=DEV).manual_seed(5)
    logits = torch.randn(2, k, V, device=DEV, generator=g)
    logits[0] = logits[0].clamp(max=2.5)
    logits[0, :, :32] = torch.tensor([5.0, 4.0] + [3.0] * 30, device=DEV)   # 30 tokens tie with the top-3 cut
    candidates = num_candidates(sampling.max_top_k, sampling.all_top_k, V)
    assert candidates == 84
    noise = S.exponential_noise_(torch.empty(2, k, candidates, device=DEV), g)
    drafts = torch.empty(2, k, dtype=torch.int64, device=DEV)
    probs = torch.full((2, k, V), 9.0, device=DEV)
    markov_rows(logits, torch.tensor([1, 3], device=DEV), sampling, noise, drafts, probs, candidates,
                LookupHead(torch.zeros(V, V, device=DEV)))
    whole = S.probs_from_logits(logits, sampling)
    assert torch.equal(probs > 0, whole > 0)
    assert torch.allclose(probs, whole, rtol=0, atol=1e-6)
    assert bool((probs.gather(-1, drafts.unsqueeze(-1)) > 0).all())


@pytest.mark.parametrize("params", [
    [(0.0, 0, 1.0), (0.0, 0, 1.0)],
    [(1.0, 0, 1.0), (0.7, 3, 0.9)],
    [(1.0, 4, 1.0), (0.7, 3, 0.9)],
], ids=["greedy", "random", "candidates"])
def test_sampling_graph_draws_what_the_eager_rows_draw(S, params):
    """A small DFlashDrafter: two rows padded to four; the captured block + sampling graphs against the same
    bodies run eagerly from the same generator state (drafts, q and the generator's offset)."""
    from nanovllm_b200.batch_metadata import RowState
    from nanovllm_b200.dflash import DFlashDraftModel
    from nanovllm_b200.markov import MarkovQBuffer, markov_rows, num_candidates
    from nanovllm_b200.spec_sampler import SamplingTensors
    from nanovllm_b200.speculative import DFlashDrafter, sampling_graph_key
    from nanovllm_b200.target import Qwen3Shape
    shape = Qwen3Shape(hidden=128, layers=1, heads=4, kv_heads=1, intermediate=256, vocab=600, max_position=4096,
                       aux_layer_ids=(0,))
    model = DFlashDraftModel(shape, (0,), DEV, num_blocks=4, block_size=256, markov_rank=16, mask_token_id=599,
                             seed=3, init_scale=0.2, markov_scale=0.5)
    model.kv_cache.normal_()
    k = 3
    rows = [RowState(length=40, last_token=17, block_table=[2]), RowState(length=300, last_token=5,
                                                                          block_table=[0, 3])]
    drafter = DFlashDrafter(model, k, [4], max_num_blocks=2, pad_block_id=4)
    sampling = sampling_of(S, params)
    key = sampling_graph_key(sampling)
    start = torch.Generator(device=DEV).manual_seed(21)
    gen = torch.Generator(device=DEV)
    gen.set_state(start.get_state())
    drafts, q = drafter.propose(rows, sampling, gen)
    drafts, q = drafts.clone(), None if q is None else q.clone()
    # eager: the same block forward and rows over the same padded batch (padding rows' parameters and noise are
    # whatever the buffers hold, as in the graph), the real rows' noise checked against the generator's draws
    padded = drafter.load(rows)
    drafter._block_forward(padded)
    logits = model.compute_logits(drafter.outputs[:padded * k]).view(padded, k, -1)
    prev = drafter.views[padded]["input_ids"].view(padded, k)[:, 0]
    assert prev[:2].tolist() == [17, 5]
    got = torch.empty(padded, k, dtype=torch.int64, device=DEV)
    if key is None:
        markov_rows(logits, prev, None, None, got, None, 0, model.markov_head)
        assert q is None
    else:
        candidates = num_candidates(sampling.max_top_k, sampling.all_top_k, shape.vocab)
        noise = drafter.noise[key][:padded].clone()
        eager = torch.Generator(device=DEV)
        eager.set_state(start.get_state())
        drawn = S.exponential_noise_(torch.empty(2, k, candidates or shape.vocab, device=DEV), eager)
        assert torch.equal(noise[:2], drawn) and gen.get_offset() == eager.get_offset()
        params = SamplingTensors(temperatures=drafter.temperatures[:padded], top_k=drafter.top_k[:padded],
                                 top_p=drafter.top_p[:padded], max_top_k=sampling.max_top_k,
                                 has_top_p=sampling.has_top_p, all_top_k=sampling.all_top_k)
        probs = (MarkovQBuffer(padded, k, shape.vocab, candidates, DEV) if candidates else
                 torch.empty(padded, k, shape.vocab, device=DEV))
        markov_rows(logits, prev, params, noise, got, probs, candidates, model.markov_head)
        probs = probs.probs if candidates else probs
        assert torch.equal(q, probs[:2])
    assert torch.equal(drafts, got[:2])
