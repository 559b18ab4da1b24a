"""Kernel (3), DSpark's in-block Markov rows, against oracle/markov.py and the reference's golden vectors.
Drafts bit-exact (candidate ties ordered by ascending token id on both sides), q within 1e-5 relative; at full
size, a row whose race is within 1e-5 of a tie is compared only up to that step."""
from pathlib import Path
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from oracle import markov as OM

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
G = np.load(Path(__file__).parent / "golden" / "markov.npz")
NAMES = sorted({key.split("/")[1] for key in G.files if key.startswith("markov/")})


def case(name):
    prefix = f"markov/{name}/"
    return {key[len(prefix):]: G[key] for key in G.files if key.startswith(prefix)}


def sampling_of(temps, top_k, top_p):
    from nanovllm_b200 import spec_sampler as S
    seqs = [SimpleNamespace(temperature=float(t), top_k=int(k), top_p=float(p)) for t, k, p in zip(temps, top_k, top_p)]
    return S.sampling_tensors(seqs, DEV)


@pytest.mark.parametrize("name", NAMES)
def test_golden_markov_rows(name):
    from nanovllm_b200.markov import markov_rows
    c = case(name)
    a = torch.from_numpy(c["bias_a"]).to(DEV)
    cc = torch.from_numpy(c["bias_c"]).to(DEV)
    head = lambda prev: a[prev][:, None] * cc[None, :]
    logits = torch.from_numpy(c["logits"]).to(DEV)
    B, k, V = logits.shape
    drafts = torch.empty(B, k, dtype=torch.int64, device=DEV)
    samp = probs = noise = None
    if "temperature" in c:
        samp = sampling_of(c["temperature"], c["top_k"], c["top_p"])
        probs = torch.full((B, k, V), 7.0, device=DEV)     # garbage: the call must zero / overwrite it
        noise = torch.from_numpy(c["noise"]).to(DEV)
    markov_rows(logits, torch.from_numpy(c["prev"]).to(DEV), samp, noise, drafts, probs, int(c["candidates"]), head)
    assert drafts.cpu().numpy().tolist() == c["drafts"].tolist()
    if probs is not None:
        got = probs.cpu().numpy()
        assert np.array_equal(got > 0, c["probs"] > 0)
        np.testing.assert_allclose(got, c["probs"], rtol=1e-5, atol=1e-7)


class RecordingHead:
    """The production Markov head (W2 . W1[prev], cuBLAS) that records every step's bias for the oracle."""

    def __init__(self, w1, w2):
        self.w1, self.w2, self.biases = w1, w2, []

    def __call__(self, prev):
        bias = torch.matmul(self.w1[prev], self.w2.t())
        self.biases.append(bias.clone())
        return bias


@pytest.mark.parametrize("greedy", [False, True])
def test_config4_markov_rows_match_oracle(greedy):
    """benchmark config 4's drafter: B = 64 rows, k = 7, V = 151936, rank 256, bf16, top_k = 128 (192 candidates)."""
    from nanovllm_b200.markov import markov_rows, num_candidates
    B, k, V, r = 64, 7, 151936, 256
    g = torch.Generator(device=DEV).manual_seed(4)
    logits = (torch.randn(B, k, V, device=DEV, generator=g) * 2).bfloat16()
    w1 = (torch.randn(V, r, device=DEV, generator=g) * 0.1).bfloat16()
    w2 = (torch.randn(V, r, device=DEV, generator=g) * 0.1).bfloat16()
    prev = torch.randint(V, (B,), device=DEV, generator=g)
    head = RecordingHead(w1, w2)
    drafts = torch.empty(B, k, dtype=torch.int64, device=DEV)
    if greedy:
        samp, cand, noise, probs = None, 0, None, None
    else:
        samp = sampling_of([1.0] * (B // 2) + [0.7] * (B // 2), [128] * B, [1.0] * (B // 2) + [0.9] * (B // 2))
        cand = num_candidates(samp.max_top_k, samp.all_top_k, V)
        noise = torch.empty(B, k, cand, device=DEV).exponential_(generator=g).clamp_min_(1e-10)
        probs = torch.empty(B, k, V, device=DEV)
    markov_rows(logits, prev, samp, noise, drafts, probs, cand, head)
    biases = [b.float().cpu().numpy() for b in head.biases]
    step = {"i": 0}

    def bias_fn(_prev):
        out = biases[step["i"]]
        step["i"] += 1
        return out

    from oracle.ctx_store import bf16
    sampling = None if greedy else dict(temps=samp.temperatures.cpu().numpy(), top_k=samp.top_k.cpu().numpy(),
                                        top_p=samp.top_p.cpu().numpy(), max_top_k=samp.max_top_k,
                                        has_top_p=samp.has_top_p)
    want, want_probs = OM.markov_rows(logits.float().cpu().numpy(), prev.cpu().numpy(), bias_fn, sampling,
                                      None if noise is None else noise.cpu().numpy(), cand, round_fn=bf16)
    got = drafts.cpu().numpy()
    # rows agree step by step; a row may only diverge after a step whose race is a near tie
    mismatched = (got != want).any(axis=1)
    assert mismatched.sum() <= 1, f"{mismatched.sum()} rows diverge"
    if not greedy:
        same = ~mismatched
        gp = probs.cpu().numpy()[same]
        np.testing.assert_allclose(gp, want_probs[same], rtol=1e-5, atol=1e-8)


def test_whole_vocabulary_rows_use_the_sampler_kernels():
    """A batch where one row does not truncate draws every row over the whole vocabulary (candidates = 0)."""
    from nanovllm_b200.markov import markov_rows
    B, k, V = 3, 4, 3000
    g = torch.Generator(device=DEV).manual_seed(9)
    logits = torch.randn(B, k, V, device=DEV, generator=g)
    a = torch.randn(V, device=DEV, generator=g)
    cvec = torch.randn(V, device=DEV, generator=g)
    head = lambda prev: a[prev][:, None] * cvec[None, :]
    samp = sampling_of([1.0, 0.8, 1.2], [0, 20, 5], [1.0, 0.9, 1.0])
    noise = torch.empty(B, k, V, device=DEV).exponential_(generator=g).clamp_min_(1e-10)
    drafts = torch.empty(B, k, dtype=torch.int64, device=DEV)
    probs = torch.empty(B, k, V, device=DEV)
    prev = torch.tensor([1, 2, 3], device=DEV)
    markov_rows(logits, prev, samp, noise, drafts, probs, 0, head)
    an, cn = a.cpu().numpy(), cvec.cpu().numpy()
    sampling = dict(temps=samp.temperatures.cpu().numpy(), top_k=samp.top_k.cpu().numpy(),
                    top_p=samp.top_p.cpu().numpy(), max_top_k=samp.max_top_k, has_top_p=samp.has_top_p)
    want, want_probs = OM.markov_rows(logits.cpu().numpy(), prev.cpu().numpy(),
                                      lambda p: an[p][:, None] * cn[None, :], sampling, noise.cpu().numpy(), 0)
    assert drafts.cpu().numpy().tolist() == want.tolist()
    np.testing.assert_allclose(probs.cpu().numpy(), want_probs, rtol=1e-5, atol=1e-8)


@pytest.mark.parametrize("top_k", [5, 500])
def test_candidate_selection_paths(top_k):
    """C = top_k + 64 candidates: <= 512 takes the thread-maxima selection, > 512 the exact radix fallback; both
    must give the oracle's drafts and q (bf16 logits and bias, so many candidates tie)."""
    from nanovllm_b200.markov import markov_rows, num_candidates
    from oracle.ctx_store import bf16
    B, k, V = 5, 3, 6000
    g = torch.Generator(device=DEV).manual_seed(top_k)
    logits = (torch.randn(B, k, V, device=DEV, generator=g) * 2).bfloat16()
    table = (torch.randn(64, V, device=DEV, generator=g)).bfloat16()
    head = lambda prev: table[prev % 64]
    samp = sampling_of([1.0, 0.8, 1.0, 0.6, 1.2], [top_k] * B, [1.0, 0.9, 1.0, 0.5, 1.0])
    cand = num_candidates(samp.max_top_k, samp.all_top_k, V)
    noise = torch.empty(B, k, cand, device=DEV).exponential_(generator=g).clamp_min_(1e-10)
    drafts = torch.empty(B, k, dtype=torch.int64, device=DEV)
    probs = torch.empty(B, k, V, device=DEV)
    prev = torch.randint(V, (B,), device=DEV, generator=g)
    markov_rows(logits, prev, samp, noise, drafts, probs, cand, head)
    tab = table.float().cpu().numpy()
    sampling = dict(temps=samp.temperatures.cpu().numpy(), top_k=samp.top_k.cpu().numpy(),
                    top_p=samp.top_p.cpu().numpy(), max_top_k=samp.max_top_k, has_top_p=samp.has_top_p)
    want, want_probs = OM.markov_rows(logits.float().cpu().numpy(), prev.cpu().numpy(), lambda p: tab[p % 64],
                                      sampling, noise.cpu().numpy(), cand, round_fn=bf16)
    assert drafts.cpu().numpy().tolist() == want.tolist()
    np.testing.assert_allclose(probs.cpu().numpy(), want_probs, rtol=1e-5, atol=1e-8)


@pytest.mark.parametrize("top_k", [100, 500, 0])
def test_rows_split_over_many_ctas_keep_ties_by_id(top_k):
    """V = 40000 rows are split over several CTAs (9 pieces at C = 164, 7 at C = 564); values drawn from a
    handful of levels tie across piece boundaries, and the merged candidates must still be the oracle's (ties by
    ascending token id).  top_k = 0 runs the greedy rows (argmax, first index)."""
    from nanovllm_b200.markov import markov_rows, num_candidates
    from oracle.ctx_store import bf16
    B, k, V = 2, 3, 40000
    g = torch.Generator(device=DEV).manual_seed(100 + top_k)
    logits = (torch.randint(-3, 4, (B, k, V), device=DEV, generator=g).float() * 0.5).bfloat16()
    table = (torch.randint(-2, 3, (8, V), device=DEV, generator=g).float() * 0.25).bfloat16()
    head = lambda prev: table[prev % 8]
    drafts = torch.empty(B, k, dtype=torch.int64, device=DEV)
    prev = torch.randint(V, (B,), device=DEV, generator=g)
    tab = table.float().cpu().numpy()
    if top_k == 0:
        markov_rows(logits, prev, None, None, drafts, None, 0, head)
        want, _ = OM.markov_rows(logits.float().cpu().numpy(), prev.cpu().numpy(), lambda p: tab[p % 8], None, None,
                                 0, round_fn=bf16)
        assert drafts.cpu().numpy().tolist() == want.tolist()
        return
    samp = sampling_of([1.0, 0.8], [top_k] * B, [1.0, 0.9])
    cand = num_candidates(samp.max_top_k, samp.all_top_k, V)
    noise = torch.empty(B, k, cand, device=DEV).exponential_(generator=g).clamp_min_(1e-10)
    probs = torch.empty(B, k, V, device=DEV)
    markov_rows(logits, prev, samp, noise, drafts, probs, cand, head)
    sampling = dict(temps=samp.temperatures.cpu().numpy(), top_k=samp.top_k.cpu().numpy(),
                    top_p=samp.top_p.cpu().numpy(), max_top_k=samp.max_top_k, has_top_p=samp.has_top_p)
    want, want_probs = OM.markov_rows(logits.float().cpu().numpy(), prev.cpu().numpy(), lambda p: tab[p % 8],
                                      sampling, noise.cpu().numpy(), cand, round_fn=bf16)
    assert drafts.cpu().numpy().tolist() == want.tolist()
    np.testing.assert_allclose(probs.cpu().numpy(), want_probs, rtol=1e-5, atol=1e-8)


def test_persistent_q_buffer_matches_fresh_zeroed_buffers():
    """A MarkovQBuffer clears only the previous call's candidates: two calls in a row give exactly the drafts and
    q of two calls on freshly zeroed tensors, and the buffer stays zero outside the current candidates."""
    from nanovllm_b200.markov import MarkovQBuffer, markov_rows, num_candidates
    B, k, V = 6, 4, 20000
    g = torch.Generator(device=DEV).manual_seed(77)
    table = (torch.randn(16, V, device=DEV, generator=g)).bfloat16()
    head = lambda prev: table[prev % 16]
    samp = sampling_of([1.0, 0.8, 1.0, 0.6, 1.2, 0.9], [40] * B, [1.0, 0.9, 1.0, 0.5, 1.0, 0.95])
    cand = num_candidates(samp.max_top_k, samp.all_top_k, V)
    qbuf = MarkovQBuffer(B, k, V, cand, DEV)
    for call in range(3):
        logits = (torch.randn(B, k, V, device=DEV, generator=g) * 2).bfloat16()
        noise = torch.empty(B, k, cand, device=DEV).exponential_(generator=g).clamp_min_(1e-10)
        prev = torch.randint(V, (B,), device=DEV, generator=g)
        d_ref = torch.empty(B, k, dtype=torch.int64, device=DEV)
        q_ref = torch.full((B, k, V), float("nan"), device=DEV)      # garbage: markov_rows zero-fills it
        markov_rows(logits, prev, samp, noise, d_ref, q_ref, cand, head)
        d = torch.empty(B, k, dtype=torch.int64, device=DEV)
        markov_rows(logits, prev, samp, noise, d, qbuf, cand, head)
        assert torch.equal(d, d_ref)
        assert torch.equal(qbuf.probs, q_ref)
        assert int((qbuf.probs != 0).sum(dim=-1).max()) <= cand


@pytest.mark.parametrize("dtype,V", [(torch.float32, 6001), (torch.bfloat16, 6001), (torch.float32, 8000)])
def test_markov_rows_fp32_and_ragged_vocab(dtype, V):
    """fp32 logits and bias (no rounding of the biased row, 3-digit radix keys) and rows whose length is not a
    multiple of 8 (the scalar load path) against the oracle."""
    from nanovllm_b200.markov import markov_rows, num_candidates
    from oracle.ctx_store import bf16
    B, k = 4, 3
    g = torch.Generator(device=DEV).manual_seed(V)
    logits = (torch.randn(B, k, V, device=DEV, generator=g) * 2).to(dtype)
    table = (torch.randn(16, V, device=DEV, generator=g)).to(dtype)
    head = lambda prev: table[prev % 16]
    samp = sampling_of([1.0, 0.8, 1.3, 0.6], [50] * B, [1.0, 0.9, 1.0, 0.7])
    cand = num_candidates(samp.max_top_k, samp.all_top_k, V)
    noise = torch.empty(B, k, cand, device=DEV).exponential_(generator=g).clamp_min_(1e-10)
    drafts = torch.empty(B, k, dtype=torch.int64, device=DEV)
    probs = torch.empty(B, k, V, device=DEV)
    prev = torch.randint(V, (B,), device=DEV, generator=g)
    markov_rows(logits, prev, samp, noise, drafts, probs, cand, head)
    tab = table.float().cpu().numpy()
    sampling = dict(temps=samp.temperatures.cpu().numpy(), top_k=samp.top_k.cpu().numpy(),
                    top_p=samp.top_p.cpu().numpy(), max_top_k=samp.max_top_k, has_top_p=samp.has_top_p)
    want, want_probs = OM.markov_rows(logits.float().cpu().numpy(), prev.cpu().numpy(), lambda p: tab[p % 16],
                                      sampling, noise.cpu().numpy(), cand,
                                      round_fn=bf16 if dtype == torch.bfloat16 else (lambda x: x))
    assert drafts.cpu().numpy().tolist() == want.tolist()
    np.testing.assert_allclose(probs.cpu().numpy(), want_probs, rtol=1e-5, atol=1e-8)


def test_markov_workspace_shared_by_batches_of_different_sizes():
    """One Markov workspace (zeroed once) serves batches of different sizes: the per-row tickets and greedy keys
    sit at fixed offsets, so a call never finds another call's candidate keys in its tickets."""
    from nanovllm_b200.markov import markov_rows, num_candidates
    k, V = 3, 20000
    g = torch.Generator(device=DEV).manual_seed(12)
    table = (torch.randn(16, V, device=DEV, generator=g)).bfloat16()
    head = lambda prev: table[prev % 16]
    runs = {}
    for B in (3, 40, 3, 40):
        gB = torch.Generator(device=DEV).manual_seed(B)
        logits = (torch.randn(B, k, V, device=DEV, generator=gB) * 2).bfloat16()
        samp = sampling_of([1.0] * B, [30] * B, [1.0] * B)
        cand = num_candidates(samp.max_top_k, samp.all_top_k, V)
        noise = torch.empty(B, k, cand, device=DEV).exponential_(generator=gB).clamp_min_(1e-10)
        prev = torch.randint(V, (B,), device=DEV, generator=gB)
        drafts = torch.empty(B, k, dtype=torch.int64, device=DEV)
        probs = torch.empty(B, k, V, device=DEV)
        markov_rows(logits, prev, samp, noise, drafts, probs, cand, head)
        greedy = torch.empty(B, k, dtype=torch.int64, device=DEV)
        markov_rows(logits, prev, None, None, greedy, None, 0, head)
        torch.cuda.synchronize()
        if B in runs:
            assert torch.equal(drafts, runs[B][0]) and torch.equal(greedy, runs[B][1])
        runs[B] = (drafts, greedy)


# ---------------------------------------------------------------------------------------------- fused bias GEMM
def test_markov_bias_gemm_against_the_fp32_product():
    """specdec_markov_bias: bf16(bf16(e . W2^T) + logits) on the tensor cores, at config 4's shape (64 rows, rank
    256, V = 151936) and a ragged one (37 rows: a partial column tile), against the fp32 product: the bias within
    one bf16 rounding plus summation order, then one rounding of the sum."""
    from nanovllm_b200.markov import markov_bias
    for B, V in [(64, 151936), (37, 1280)]:
        g = torch.Generator(device=DEV).manual_seed(B)
        r = 256
        w2 = (torch.randn(V, r, device=DEV, generator=g) * 0.1).bfloat16()
        e = (torch.randn(B, r, device=DEV, generator=g) * 0.1).bfloat16()
        logits = (torch.randn(B, 3, V, device=DEV, generator=g) * 2).bfloat16()
        out = torch.full((B, V), float("nan"), dtype=torch.bfloat16, device=DEV)
        markov_bias(w2, e, logits[:, 1], out)
        bias = e.float() @ w2.float().t()
        want = logits[:, 1].float() + bias
        got = out.float()
        assert torch.isfinite(got).all()
        tol = bias.abs() * 2 ** -8 + want.abs() * 2 ** -8 + 1e-3 * bias.abs().max()
        assert bool(((got - want).abs() <= tol).all())


def fused_case(B, k, V, r, seed):
    from nanovllm_b200.markov import MarkovHeadWeights
    g = torch.Generator(device=DEV).manual_seed(seed)
    logits = (torch.randn(B, k, V, device=DEV, generator=g) * 2).bfloat16()
    head = MarkovHeadWeights((torch.randn(V, r, device=DEV, generator=g) * 0.1).bfloat16(),
                             (torch.randn(V, r, device=DEV, generator=g) * 0.1).bfloat16())
    prev = torch.randint(V, (B,), device=DEV, generator=g)
    return g, logits, head, prev


@pytest.mark.parametrize("greedy", [False, True])
def test_fused_bias_rows_match_oracle(greedy):
    """Config 4's drafter through the fused-bias path (MarkovHeadWeights, bf16, fused_bias=True): each step's biased
    rows recomputed with the same kernel from the drafted tokens, and oracle/markov.py run on them (bias 0): drafts
    bit-exact (at most one row diverging after a near-tie race), q within 1e-5."""
    from nanovllm_b200.markov import fused_bias_eligible, markov_bias, markov_rows, num_candidates
    from oracle.ctx_store import bf16
    B, k, V, r = 64, 7, 151936, 256
    g, logits, head, prev = fused_case(B, k, V, r, 44)
    assert fused_bias_eligible(logits, head)
    drafts = torch.empty(B, k, dtype=torch.int64, device=DEV)
    if greedy:
        samp, cand, noise, probs = None, 0, None, None
    else:
        samp = sampling_of([1.0] * (B // 2) + [0.7] * (B // 2), [128] * B, [1.0] * (B // 2) + [0.9] * (B // 2))
        cand = num_candidates(samp.max_top_k, samp.all_top_k, V)
        noise = torch.empty(B, k, cand, device=DEV).exponential_(generator=g).clamp_min_(1e-10)
        probs = torch.empty(B, k, V, device=DEV)
    markov_rows(logits, prev, samp, noise, drafts, probs, cand, head, fused_bias=True)
    prevs = [prev] + [drafts[:, j] for j in range(k - 1)]
    biased = torch.empty(B, k, V, dtype=torch.bfloat16, device=DEV)
    for j, p in enumerate(prevs):
        markov_bias(head.w2, head.w1[p].contiguous(), logits[:, j], biased[:, j])
    zero = np.zeros((B, V), np.float32)
    sampling = None if greedy else dict(temps=samp.temperatures.cpu().numpy(), top_k=samp.top_k.cpu().numpy(),
                                        top_p=samp.top_p.cpu().numpy(), max_top_k=samp.max_top_k,
                                        has_top_p=samp.has_top_p)
    want, want_probs = OM.markov_rows(biased.float().cpu().numpy(), prev.cpu().numpy(), lambda _p: zero, sampling,
                                      None if noise is None else noise.cpu().numpy(), cand, round_fn=bf16)
    got = drafts.cpu().numpy()
    mismatched = (got != want).any(axis=1)
    assert mismatched.sum() <= 1, f"{mismatched.sum()} rows diverge"
    if not greedy:
        same = ~mismatched
        np.testing.assert_allclose(probs.cpu().numpy()[same], want_probs[same], rtol=1e-5, atol=1e-8)


def test_fused_and_unfused_bias_agree_where_the_bias_rounds_alike():
    """The fused path against the path that adds a given bias in the selection kernel, fed the fused kernel's own
    biased rows as logits with a zero bias: identical drafts and q (the selection is the same code either way)."""
    from nanovllm_b200.markov import MarkovQBuffer, markov_bias, markov_rows, num_candidates
    B, k, V, r = 16, 4, 12800, 64
    g, logits, head, prev = fused_case(B, k, V, r, 45)
    samp = sampling_of([0.9] * B, [20] * B, [0.95] * B)
    cand = num_candidates(samp.max_top_k, samp.all_top_k, V)
    noise = torch.empty(B, k, cand, device=DEV).exponential_(generator=g).clamp_min_(1e-10)
    d1 = torch.empty(B, k, dtype=torch.int64, device=DEV)
    q1 = MarkovQBuffer(B, k, V, cand, DEV)
    markov_rows(logits, prev, samp, noise, d1, q1, cand, head, fused_bias=True)
    prevs = [prev] + [d1[:, j] for j in range(k - 1)]
    biased = torch.empty(B, k, V, dtype=torch.bfloat16, device=DEV)
    for j, p in enumerate(prevs):
        markov_bias(head.w2, head.w1[p].contiguous(), logits[:, j], biased[:, j])
    zero = torch.zeros(B, V, dtype=torch.bfloat16, device=DEV)
    d2 = torch.empty(B, k, dtype=torch.int64, device=DEV)
    q2 = torch.empty(B, k, V, device=DEV)
    markov_rows(biased, prev, samp, noise, d2, q2, cand, lambda _p: zero)
    assert torch.equal(d1, d2)
    assert torch.equal(q1.probs, q2)
