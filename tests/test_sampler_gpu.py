"""Kernel (1), the batched speculative sampler, against the CPU oracle and the reference's golden vectors.

Tolerances (north star): accepted lengths and tail tokens bit-exact, except requests whose accept draw or tail
race is within 1e-6 of a tie under the probability uncertainty (oracle.spec_sampler.near_tie_flags), which are
counted and skipped; probabilities within 1e-5 relative.
"""
from pathlib import Path
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from oracle import spec_sampler as O

pytestmark = pytest.mark.gpu

GOLDEN = np.load(Path(__file__).parent / "golden" / "sampler.npz")
DEV = torch.device("cuda", 0)
V_FULL = 151936
RTOL = 1e-5


@pytest.fixture(scope="module")
def S():
    from nanovllm_b200 import spec_sampler
    return spec_sampler


def case(kind, name):
    prefix = f"{kind}/{name}/"
    return {key[len(prefix):]: GOLDEN[key] for key in GOLDEN.files if key.startswith(prefix)}


def names(kind):
    return sorted({key.split("/")[1] for key in GOLDEN.files if key.startswith(kind + "/")})


def cuda(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a))
    return t.to(DEV, dtype=dtype) if dtype is not None else t.to(DEV)


def sampling_of(S, temps, top_k, top_p):
    seqs = [SimpleNamespace(temperature=float(t), top_k=int(k), top_p=float(p)) for t, k, p in zip(temps, top_k, top_p)]
    return S.sampling_tensors(seqs, DEV)


# ------------------------------------------------------------------------------------------- golden fixtures
@pytest.mark.parametrize("name", names("accept"))
def test_golden_accept_on_probabilities(S, name):
    c = case("accept", name)
    draws = (cuda(c["u"]), cuda(c["noise"]))
    n_accept, tail = S.accept_random_varlen(cuda(c["p"]), cuda(c["q"]), cuda(c["drafts"]), cuda(c["lens"]), None,
                                            draws=draws)
    assert n_accept.cpu().numpy().tolist() == c["n_accept"].tolist()
    assert tail.cpu().numpy().tolist() == c["tail"].tolist()


@pytest.mark.parametrize("name", names("logits"))
def test_golden_fused_accept_on_logits(S, name):
    c = case("logits", name)
    dtype = getattr(torch, str(c["dtype"]))
    samp = sampling_of(S, c["temperature"], c["top_k"], c["top_p"])
    draws = (cuda(c["u"]), cuda(c["noise"]))
    n_accept, tail = S.accept_from_logits(cuda(c["logits"], dtype), cuda(c["q"]), cuda(c["drafts"]), samp,
                                          cuda(c["lens"]), None, draws=draws)
    flags = O.near_tie_flags(c["p"], c["q"], c["drafts"], c["lens"], c["u"], c["noise"])
    keep = ~flags
    assert np.array_equal(n_accept.cpu().numpy()[keep], c["n_accept"][keep])
    assert np.array_equal(tail.cpu().numpy()[keep], c["tail"][keep])


@pytest.mark.parametrize("name", names("logits"))
def test_golden_probs_from_logits_per_token(S, name):
    c = case("logits", name)
    dtype = getattr(torch, str(c["dtype"]))
    samp = sampling_of(S, c["temperature"], c["top_k"], c["top_p"])
    lens = cuda(c["lens"])
    per_token = S.sampling_per_token(samp, lens, int(c["lens"].sum()))
    probs = S.probs_from_logits(cuda(c["logits"], dtype), per_token).cpu().numpy()
    assert np.array_equal(probs > 0, c["p"] > 0)
    np.testing.assert_allclose(probs, c["p"], rtol=RTOL, atol=1e-7)


@pytest.mark.parametrize("name", names("trunc"))
def test_golden_truncation(S, name):
    c = case("trunc", name)
    samp = sampling_of(S, c["temperature"], c["top_k"], c["top_p"])
    probs = S.probs_from_logits(cuda(c["logits"]), samp).cpu().numpy()
    assert np.array_equal(probs > 0, c["probs"] > 0)
    np.testing.assert_allclose(probs, c["probs"], rtol=RTOL, atol=1e-7)


@pytest.mark.parametrize("name", names("greedy"))
def test_golden_greedy(S, name):
    c = case("greedy", name)
    n_accept, tail = S.accept_greedy_varlen(cuda(c["logits"]), cuda(c["drafts"]), cuda(c["lens"]))
    assert n_accept.cpu().tolist() == c["n_accept"].tolist()
    assert tail.cpu().tolist() == c["tail"].tolist()


# ------------------------------------------------------------------------------------------- in-kernel draws
@pytest.mark.parametrize("rows,vocab", [(1, 5), (3, 100), (8, 7777), (64, V_FULL), (37, 50021)])
def test_in_kernel_noise_reproduces_torch_exponential(S, rows, vocab):
    g = torch.Generator(device=DEV).manual_seed(1234 + rows)
    g.set_offset(8 * rows)
    w = torch.rand(rows, vocab, device=DEV, generator=torch.Generator(device=DEV).manual_seed(7)) ** 4
    g_torch = torch.Generator(device=DEV)
    g_torch.set_state(g.get_state())
    expected = S.race(w, S.exponential_noise_(torch.empty_like(w), g_torch))
    got = S.sample(w, g)
    assert torch.equal(got, expected)
    assert g.get_offset() == g_torch.get_offset()


MIXED_TOPK = ([0.7, 1.0, 1.3, 0.9] * 16, [20, 0, 128, 600] * 16, [0.8, 1.0, 1.0, 0.95] * 16)


@pytest.mark.parametrize("batch,k,vocab,varlen,params", [
    (8, 7, V_FULL, False, None), (64, 7, V_FULL, True, None), (5, 3, 1000, True, None),
    (64, 7, V_FULL, True, ([0.7] * 64, [20] * 64, [0.8] * 64)),       # every tail raced among its kept tokens
    (64, 7, V_FULL, True, MIXED_TOPK),                                 # rows without a kept set: full-row race
])
def test_in_kernel_draws_match_torch_draws(S, batch, k, vocab, varlen, params):
    gen = torch.Generator(device=DEV).manual_seed(99)
    temps, top_k, top_p = params or (None, None, None)
    logits, q, drafts, lens, samp = synthetic_round(S, batch, k, vocab, torch.float32, varlen, seed=3,
                                                    temps=temps, top_k=top_k, top_p=top_p)
    g1 = torch.Generator(device=DEV).manual_seed(5)
    g2 = torch.Generator(device=DEV).manual_seed(5)
    a = S.accept_from_logits(logits, q, drafts, samp, lens, g1, draws="kernel")
    b = S.accept_from_logits(logits, q, drafts, samp, lens, g2, draws="torch")
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])
    assert g1.get_offset() == g2.get_offset()
    del gen


# ------------------------------------------------------------------------------------------- full vocabulary
def synthetic_round(S, batch, k, vocab, dtype, varlen, seed, temps=None, top_k=None, top_p=None):
    g = torch.Generator(device=DEV).manual_seed(seed)
    lens = (torch.randint(1, k + 2, (batch,), device=DEV, generator=g) if varlen
            else torch.full((batch,), k + 1, device=DEV))
    total = int(lens.sum())
    logits = (torch.randn(total, vocab, device=DEV, generator=g) * 3).to(dtype)
    temps = temps or [1.0] * batch
    samp = sampling_of(S, temps, top_k or [0] * batch, top_p or [1.0] * batch)
    q = torch.softmax(torch.randn(batch, k, vocab, device=DEV, generator=g) * 3, dim=-1)
    # every other request proposes from the target itself so long prefixes get accepted
    starts = torch.cumsum(lens, 0) - lens
    p = S.probs_from_logits(logits, S.sampling_per_token(samp, lens, total))
    for b in range(0, batch, 2):
        pos = starts[b] + torch.clamp(torch.arange(k, device=DEV), max=int(lens[b]) - 1)
        q[b] = p[pos]
    drafts = S.sample(q, g)
    return logits, q, drafts, lens, samp


@pytest.mark.parametrize("batch,k,dtype,varlen,params", [
    (8, 7, torch.float32, False, None),                                     # benchmark config 1
    (64, 7, torch.bfloat16, False, None),                                   # config 3's accept
    (64, 7, torch.bfloat16, True, None),                                    # config 4's varlen lengths
    (16, 7, torch.bfloat16, True, ([0.7] * 16, [20] * 16, [0.8] * 16)),    # protocol sampling
    (64, 7, torch.bfloat16, True, ([0.7] * 64, [20] * 64, [0.8] * 64)),    # tails raced among kept tokens
    (64, 7, torch.bfloat16, True, MIXED_TOPK),                             # top-k off / radix rows mixed in
])
def test_full_vocab_accept_matches_oracle(S, batch, k, dtype, varlen, params):
    temps, top_k, top_p = params or (None, None, None)
    logits, q, drafts, lens, samp = synthetic_round(S, batch, k, V_FULL, dtype, varlen, seed=batch + k,
                                                    temps=temps, top_k=top_k, top_p=top_p)
    gen = torch.Generator(device=DEV).manual_seed(11)
    u = torch.rand(batch, k, device=DEV, generator=gen)
    noise = S.exponential_noise_(torch.empty(batch, V_FULL, device=DEV), gen)
    n_accept, tail = S.accept_from_logits(logits, q, drafts, samp, lens, None, draws=(u, noise))
    lens_np = lens.cpu().numpy()
    per = lambda t: np.repeat(t.cpu().numpy(), lens_np)
    p = O.probs_from_logits(logits.float().cpu().numpy(), per(samp.temperatures), per(samp.top_k),
                            per(samp.top_p), samp.max_top_k, samp.has_top_p)
    args = (q.cpu().numpy(), drafts.cpu().numpy(), lens_np, u.cpu().numpy(), noise.cpu().numpy())
    want_n, want_tail = O.accept_random_varlen(p, *args)
    flags = O.near_tie_flags(p, *args)
    keep = ~flags
    assert flags.sum() <= max(1, batch // 16), f"{flags.sum()} near-tie rows"
    assert np.array_equal(n_accept.cpu().numpy()[keep], want_n[keep])
    assert np.array_equal(tail.cpu().numpy()[keep], want_tail[keep])
    # probabilities of the same rows through specdec_probs
    p_gpu = S.probs_from_logits(logits, S.sampling_per_token(samp, lens, int(lens_np.sum()))).cpu().numpy()
    assert np.array_equal(p_gpu > 0, p > 0)
    np.testing.assert_allclose(p_gpu, p, rtol=RTOL, atol=1e-9)


def test_full_vocab_greedy_matches_oracle(S):
    batch, k = 64, 7
    logits, q, drafts, lens, samp = synthetic_round(S, batch, k, V_FULL, torch.bfloat16, True, seed=2)
    target = logits.float().argmax(-1)
    starts = torch.cumsum(lens, 0) - lens
    for b in range(batch):       # agree with the target on a prefix of length b % (k + 1)
        for j in range(min(b % (k + 1), int(lens[b]) - 1)):
            drafts[b, j] = target[starts[b] + j]
    n_accept, tail = S.accept_greedy_varlen(logits, drafts, lens)
    want_n, want_tail = O.accept_greedy_varlen(logits.float().cpu().numpy(), drafts.cpu().numpy(), lens.cpu().numpy())
    assert n_accept.cpu().numpy().tolist() == want_n.tolist()
    assert tail.cpu().numpy().tolist() == want_tail.tolist()


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("vocab", [4096, 4099, V_FULL])
def test_greedy_ties_and_infinities(S, dtype, vocab):
    """Rows of few distinct values (many tied maxima, the first index wins), rows whose maximum is +inf, rows of
    -inf only; 16-byte groups when V * size is a multiple of 16, elementwise loads otherwise."""
    batch, k = 6, 3
    gen = torch.Generator().manual_seed(vocab)
    rows = batch * (k + 1)
    logits = torch.randint(-3, 4, (rows, vocab), generator=gen).to(torch.float32)
    logits[1, vocab // 2] = float("inf")
    logits[1, vocab - 1] = float("inf")
    logits[5] = float("-inf")
    logits[9, :] = 2.0
    logits[13, -1] = 7.0
    logits = logits.to(DEV, dtype)
    target = logits.float().argmax(-1).view(batch, k + 1)
    drafts = torch.randint(0, vocab, (batch, k), generator=gen).to(DEV)
    for b in range(batch):      # agree with the target on a prefix of length b % (k + 1)
        drafts[b, : b % (k + 1)] = target[b, : b % (k + 1)]
    n_accept, tail = S.accept_greedy(logits.view(batch, k + 1, vocab), drafts)
    want_n, want_tail = O.accept_greedy_varlen(logits.float().cpu().numpy(), drafts.cpu().numpy(),
                                               np.full(batch, k + 1))
    assert n_accept.cpu().numpy().tolist() == want_n.tolist()
    assert tail.cpu().numpy().tolist() == want_tail.tolist()


def test_fixed_length_entry_points(S):
    batch, k = 8, 7
    logits, q, drafts, lens, samp = synthetic_round(S, batch, k, 4099, torch.float32, False, seed=8)
    p = S.probs_from_logits(logits.view(batch, k + 1, -1), samp)
    gen = torch.Generator(device=DEV).manual_seed(3)
    u = torch.rand(batch, k, device=DEV, generator=gen)
    noise = S.exponential_noise_(torch.empty(batch, 4099, device=DEV), gen)
    a = S.accept_random(p, q, drafts, None, draws=(u, noise))
    b = S.accept_from_logits(logits.view(batch, k + 1, -1), q, drafts, samp, None, None, draws=(u, noise))
    want = O.accept_random(p.cpu().numpy(), q.cpu().numpy(), drafts.cpu().numpy(), u.cpu().numpy(),
                           noise.cpu().numpy())
    assert a[0].cpu().tolist() == want[0].tolist() and a[1].cpu().tolist() == want[1].tolist()
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])
    g1 = S.accept_greedy(logits.view(batch, k + 1, -1), drafts)
    want_g = O.accept_greedy(logits.view(batch, k + 1, -1).cpu().numpy(), drafts.cpu().numpy())
    assert g1[0].cpu().tolist() == want_g[0].tolist() and g1[1].cpu().tolist() == want_g[1].tolist()


def test_repeated_calls_reuse_the_workspace(S):
    """The workspace's tickets and keys must return to zero after every call of every shape."""
    for batch, vocab, varlen in [(64, V_FULL, True), (3, 17, False), (64, V_FULL, False), (1, 1, False)]:
        k = 7
        logits, q, drafts, lens, samp = synthetic_round(S, batch, k, vocab, torch.bfloat16, varlen, seed=vocab)
        gen = torch.Generator(device=DEV).manual_seed(1)
        u = torch.rand(batch, k, device=DEV, generator=gen)
        noise = S.exponential_noise_(torch.empty(batch, vocab, device=DEV), gen)
        first = S.accept_from_logits(logits, q, drafts, samp, lens, None, draws=(u, noise))
        second = S.accept_from_logits(logits, q, drafts, samp, lens, None, draws=(u, noise))
        assert torch.equal(first[0], second[0]) and torch.equal(first[1], second[1])
        g1 = S.accept_greedy_varlen(logits, drafts, lens)
        g2 = S.accept_greedy_varlen(logits, drafts, lens)
        assert torch.equal(g1[0], g2[0]) and torch.equal(g1[1], g2[1])


def test_host_errors_are_raised_before_launch(S):
    from nanovllm_b200._lib import SpecdecError
    q = torch.rand(2000, 1, 8, device=DEV)
    with pytest.raises(SpecdecError, match="batch"):
        S.accept_random_varlen(torch.rand(2000, 8, device=DEV), q, torch.zeros(2000, 1, dtype=torch.int64,
                                                                                 device=DEV),
                               torch.ones(2000, dtype=torch.int64, device=DEV), None)
    with pytest.raises(ValueError):
        S.accept_greedy(torch.rand(1, 2, 8), torch.zeros(1, 1, dtype=torch.int64))


def test_inconsistent_lengths_and_drafts_are_reported_not_read(S):
    """Lengths that do not sum to T, or a draft id outside the vocabulary, stop the kernels before any
    out-of-range read and leave a status code in the workspace."""
    from nanovllm_b200._lib import device_status
    batch, k, vocab = 4, 3, 64
    logits = torch.randn(10, vocab, device=DEV)
    q = torch.softmax(torch.randn(batch, k, vocab, device=DEV), -1)
    samp = sampling_of(S, [1.0] * batch, [0] * batch, [1.0] * batch)
    drafts = torch.randint(vocab, (batch, k), device=DEV)
    bad_lens = torch.tensor([4, 4, 4, 4], device=DEV)            # sums to 16, not 10
    S.accept_from_logits(logits, q, drafts, samp, bad_lens, None)
    assert device_status(DEV) == 1
    lens = torch.tensor([1, 2, 3, 4], device=DEV)
    bad_drafts = drafts.clone()
    bad_drafts[2, 0] = vocab + 5
    S.accept_from_logits(logits, q, bad_drafts, samp, lens, None)
    assert device_status(DEV) == 2
    S.accept_from_logits(logits, q, drafts, samp, lens, None)
    assert device_status(DEV) == 0


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("vocab", [32000, 4099])          # 16-byte vectors / a ragged row (scalar paths)
@pytest.mark.parametrize("params", [None, ([0.7] * 16, [20] * 16, [0.8] * 16), MIXED_TOPK])
def test_accept_dtypes_and_vocab_shapes(S, dtype, vocab, params):
    """Every logits dtype the kernels take, on vectorised and ragged rows, without and with truncation (the
    packed 16-bit selection, the scalar fallback, the kept-token and full-row tail races)."""
    batch = 16
    if params is MIXED_TOPK:
        params = tuple(p[:batch] for p in MIXED_TOPK)
    temps, top_k, top_p = params or (None, None, None)
    logits, q, drafts, lens, samp = synthetic_round(S, batch, 7, vocab, dtype, True, seed=vocab + batch,
                                                    temps=temps, top_k=top_k, top_p=top_p)
    gen = torch.Generator(device=DEV).manual_seed(23)
    u = torch.rand(batch, 7, device=DEV, generator=gen)
    noise = S.exponential_noise_(torch.empty(batch, vocab, device=DEV), gen)
    n_accept, tail = S.accept_from_logits(logits, q, drafts, samp, lens, None, draws=(u, noise))
    lens_np = lens.cpu().numpy()
    per = lambda t: np.repeat(t.cpu().numpy(), lens_np)
    p = O.probs_from_logits(logits.float().cpu().numpy(), per(samp.temperatures), per(samp.top_k),
                            per(samp.top_p), samp.max_top_k, samp.has_top_p)
    args = (q.cpu().numpy(), drafts.cpu().numpy(), lens_np, u.cpu().numpy(), noise.cpu().numpy())
    want_n, want_tail = O.accept_random_varlen(p, *args)
    keep = ~O.near_tie_flags(p, *args)
    assert keep.sum() >= batch - 1
    assert np.array_equal(n_accept.cpu().numpy()[keep], want_n[keep])
    assert np.array_equal(tail.cpu().numpy()[keep], want_tail[keep])


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_truncation_with_fewer_finite_logits_than_top_k(S, dtype):
    """Masked vocabularies: odd rows keep only 12 finite logits (the rest -inf) under top_k = 20, so the
    selection bound is -inf (fewer than top_k finite thread maxima) and every element, -inf ones included, ties
    into the kept set; probabilities stay zero off the finite entries and the accept matches the oracle."""
    batch, k, vocab = 16, 7, 32000
    temps, top_k, top_p = [0.7] * batch, [20] * batch, [0.8] * batch
    logits, q, drafts, lens, samp = synthetic_round(S, batch, k, vocab, dtype, True, seed=77, temps=temps,
                                                    top_k=top_k, top_p=top_p)
    starts = (torch.cumsum(lens, 0) - lens).tolist()
    gen_mask = torch.Generator(device=DEV).manual_seed(5)
    for b in range(1, batch, 2):
        for r in range(starts[b], starts[b] + int(lens[b])):
            keep = torch.randperm(vocab, device=DEV, generator=gen_mask)[:12]
            row = torch.full((vocab,), float("-inf"), device=DEV, dtype=dtype)
            row[keep] = logits[r, keep]
            logits[r] = row
    gen = torch.Generator(device=DEV).manual_seed(29)
    u = torch.rand(batch, k, device=DEV, generator=gen)
    noise = S.exponential_noise_(torch.empty(batch, vocab, device=DEV), gen)
    n_accept, tail = S.accept_from_logits(logits, q, drafts, samp, lens, None, draws=(u, noise))
    lens_np = lens.cpu().numpy()
    per = lambda t: np.repeat(t.cpu().numpy(), lens_np)
    p = O.probs_from_logits(logits.float().cpu().numpy(), per(samp.temperatures), per(samp.top_k),
                            per(samp.top_p), samp.max_top_k, samp.has_top_p)
    args = (q.cpu().numpy(), drafts.cpu().numpy(), lens_np, u.cpu().numpy(), noise.cpu().numpy())
    want_n, want_tail = O.accept_random_varlen(p, *args)
    keep = ~O.near_tie_flags(p, *args)
    assert keep.sum() >= batch - 1
    assert np.array_equal(n_accept.cpu().numpy()[keep], want_n[keep])
    assert np.array_equal(tail.cpu().numpy()[keep], want_tail[keep])
    assert (tail.cpu().numpy() < vocab).all()
    p_gpu = S.probs_from_logits(logits, S.sampling_per_token(samp, lens, int(lens_np.sum()))).cpu().numpy()
    assert np.array_equal(p_gpu > 0, p > 0)
    np.testing.assert_allclose(p_gpu, p, rtol=RTOL, atol=1e-9)
