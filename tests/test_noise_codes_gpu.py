"""The accept tail race over noise codes (specdec_accept with specdec_accept_workspace_bytes of workspace).

Two properties make it exact, and both are checked here on the GPU:
1. the in-kernel draws are torch's own exponential_ values, bit for bit (ATen's transform takes the logarithm with
   __logf), and every 16-bit code brackets its element's value: lo <= E < hi, over draws of up to 2^26 elements
   at several seeds and Philox offsets;
2. the race over codes finds the same tail as the race that regenerates every draw (the workspace of
   specdec_sampler_workspace_bytes), bit for bit, over logits of every dtype, temperatures, verified lengths,
   probability inputs, bonus rows, ragged and small vocabularies and rows whose weights are all zero.
The second race is itself pinned to the oracle by tests/test_sampler_gpu.py."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def lib():
    from nanovllm_b200 import _lib
    return _lib.load()


def torch_noise(seed, offset, numel):
    g = torch.Generator(device=DEV).manual_seed(seed)
    g.set_offset(offset)
    return torch.empty(numel, device=DEV).exponential_(1.0, generator=g).clamp_min_(1e-10)


@pytest.mark.parametrize("seed,offset,numel", [(0, 0, 64 * 151936), (7, 4, 1 << 26), (123456789, 4096, 1000003),
                                               (2 ** 40 + 5, 8, 1), (99, 12, 151936)])
def test_in_kernel_draws_are_torch_exponential_and_codes_bracket_them(seed, offset, numel):
    L = lib()
    stream = torch.cuda.current_stream().cuda_stream
    values = torch.empty(numel, device=DEV)
    codes = torch.empty(numel, dtype=torch.int16, device=DEV)
    assert L.specdec_exponential_codes(seed, offset, numel, None, values.data_ptr(), stream) == 0, \
        L.specdec_last_error()
    assert L.specdec_exponential_codes(seed, offset, numel, codes.data_ptr(), None, stream) == 0, \
        L.specdec_last_error()
    e = torch_noise(seed, offset, numel)
    assert torch.equal(values, e), f"{int((values != e).sum())} of {numel} draws differ from torch's"
    c = codes.to(torch.int32) & 0xffff
    lo = (c << 16).view(torch.float32)
    hi = ((c + 1) << 16).view(torch.float32)
    assert bool((e >= lo).all()) and bool((e < hi).all())


def test_codes_entry_point_rejects_bad_arguments():
    L = lib()
    buf = torch.empty(16, dtype=torch.float32, device=DEV)
    stream = torch.cuda.current_stream().cuda_stream
    assert L.specdec_exponential_codes(0, 2, 16, buf.data_ptr(), None, stream) != 0     # offset not a multiple of 4
    assert L.specdec_exponential_codes(0, 0, 0, buf.data_ptr(), None, stream) != 0
    assert L.specdec_exponential_codes(0, 0, 16, None, None, stream) != 0
    assert L.specdec_exponential_codes(0, 0, 16, buf.data_ptr(), buf.data_ptr(), stream) != 0
    assert L.specdec_accept_workspace_bytes(512, 64, 151936) == (L.specdec_sampler_workspace_bytes(512)
                                                                 + 64 * 151936 * 2)
    assert L.specdec_accept_workspace_bytes(0, 64, 151936) == 0


def accept(x, x_is_probs, q, drafts, lens, temps, seed, offsets, workspace_bytes):
    L = lib()
    batch, k = drafts.shape
    V = x.shape[-1]
    rows = x.shape[0]
    ws = torch.zeros(workspace_bytes, dtype=torch.uint8, device=DEV)
    n_accept = torch.full((batch,), -1, dtype=torch.int64, device=DEV)
    tail = torch.full((batch,), -1, dtype=torch.int64, device=DEV)
    dtype_code = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}[x.dtype]
    st = L.specdec_accept(x.data_ptr(), int(x_is_probs), dtype_code, rows, V, q.data_ptr(), drafts.data_ptr(),
                          batch, k, None if lens is None else lens.data_ptr(),
                          None if temps is None else temps.data_ptr(), None, None, 0, 0, None, None, seed,
                          offsets[0], offsets[1], n_accept.data_ptr(), tail.data_ptr(), ws.data_ptr(), ws.numel(),
                          torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert st == 0, L.specdec_last_error()
    return n_accept.cpu(), tail.cpu()


def both(x, x_is_probs, q, drafts, lens, temps, seed, offsets=(0, 8)):
    L = lib()
    batch = drafts.shape[0]
    rows, V = x.shape
    small = accept(x, x_is_probs, q, drafts, lens, temps, seed, offsets, L.specdec_sampler_workspace_bytes(rows))
    big = accept(x, x_is_probs, q, drafts, lens, temps, seed, offsets,
                 L.specdec_accept_workspace_bytes(rows, batch, V))
    assert torch.equal(small[0], big[0]), "n_accept differs"
    assert torch.equal(small[1], big[1]), f"tails differ: {small[1].tolist()} vs {big[1].tolist()}"
    return big


def make(seed, batch, k, V, dtype, varlen, scale=3.0, draft_from_p=False, temp=1.0):
    g = torch.Generator(device=DEV).manual_seed(seed)
    lens = torch.randint(1, k + 2, (batch,), device=DEV, generator=g) if varlen else None
    rows = int(lens.sum()) if varlen else batch * (k + 1)
    logits = (torch.randn(rows, V, device=DEV, generator=g) * scale).to(dtype)
    q = torch.softmax(torch.randn(batch, k, V, device=DEV, generator=g) * scale, dim=-1)
    if draft_from_p:   # drafts the target likes and a draft q of ~0: long accepted prefixes, bonus rows
        assert not varlen
        drafts = logits.float().view(batch, k + 1, V)[:, :k].argmax(-1)
        q = torch.full_like(q, 1e-9)
    else:
        drafts = torch.randint(V, (batch, k), device=DEV, generator=g)
    temps = torch.full((batch,), temp, device=DEV)
    return logits, q, drafts, lens, temps


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32, torch.float16])
@pytest.mark.parametrize("varlen", [False, True])
def test_code_race_matches_the_full_race_at_config_3(dtype, varlen):
    for seed in range(3):
        x, q, d, lens, temps = make(seed, 64, 7, 151936, dtype, varlen)
        n, t = both(x, False, q, d, lens, temps, 1000 + seed, (0, 4 * (seed + 1)))
        assert (t >= 0).all() and (t < 151936).all()


@pytest.mark.parametrize("V", [1000, 1001, 8, 7, 513, 32000])
def test_code_race_matches_on_small_and_ragged_vocabularies(V):
    for seed, temp in [(1, 1.0), (2, 0.7), (3, 1.3)]:
        x, q, d, lens, temps = make(seed, 17, 5, V, torch.bfloat16, True, temp=temp)
        both(x, False, q, d, lens, temps, 77 + seed)


def test_code_race_matches_at_the_request_limit():
    """1024 requests: the descriptors fill the race's 32 KB of shared memory."""
    x, q, d, lens, temps = make(11, 1024, 2, 1000, torch.bfloat16, True, temp=0.8)
    both(x, False, q, d, lens, temps, 12)


def test_code_race_matches_with_bonus_rows_and_one_request():
    x, q, d, lens, temps = make(4, 64, 7, 151936, torch.bfloat16, False, draft_from_p=True)
    n, t = both(x, False, q, d, lens, temps, 5)
    assert (n == 7).any()    # some bonus rows (plain p, no residual)
    x, q, d, lens, temps = make(5, 1, 3, 151936, torch.float32, False)
    both(x, False, q, d, lens, temps, 6)


def test_code_race_matches_on_probability_inputs_with_zero_rows():
    """accept_random_varlen on given probabilities, with rows whose residual is zero on whole items and
    requests whose tail weights are all zero (the first index wins)."""
    V = 151936
    for seed in range(3):
        g = torch.Generator(device=DEV).manual_seed(50 + seed)
        batch, k = 16, 4
        lens = torch.randint(1, k + 2, (batch,), device=DEV, generator=g)
        rows = int(lens.sum())
        p = torch.softmax(torch.randn(rows, V, device=DEV, generator=g) * 4, dim=-1)
        # sparse rows: only a few hundred tokens carry mass
        keep = torch.rand(rows, V, device=DEV, generator=g) < 0.002
        p = torch.where(keep | (torch.arange(rows, device=DEV)[:, None] % 2 == 0), p, torch.zeros_like(p))
        p = p / p.sum(-1, keepdim=True)
        q = torch.softmax(torch.randn(batch, k, V, device=DEV, generator=g) * 4, dim=-1)
        q[::3] = 1.0   # q >= p everywhere: residual weights all zero for these requests
        d = torch.randint(V, (batch, k), device=DEV, generator=g)
        both(p, True, q, d, lens, None, 300 + seed)


def test_code_race_repeats_and_leaves_the_workspace_clean():
    """Back-to-back calls on one workspace (self-cleaning keys and tickets) give the same tails as fresh ones."""
    L = lib()
    x, q, d, lens, temps = make(9, 64, 7, 151936, torch.bfloat16, True)
    rows, V = x.shape
    ws = torch.zeros(L.specdec_accept_workspace_bytes(rows, 64, V), dtype=torch.uint8, device=DEV)
    outs = []
    for rep in range(3):
        n_accept = torch.empty(64, dtype=torch.int64, device=DEV)
        tail = torch.empty(64, dtype=torch.int64, device=DEV)
        st = L.specdec_accept(x.data_ptr(), 0, 1, rows, V, q.data_ptr(), d.data_ptr(), 64, 7, lens.data_ptr(),
                              temps.data_ptr(), None, None, 0, 0, None, None, 42 + rep % 2, 0, 8,
                              n_accept.data_ptr(), tail.data_ptr(), ws.data_ptr(), ws.numel(),
                              torch.cuda.current_stream().cuda_stream)
        assert st == 0
        outs.append((n_accept.cpu(), tail.cpu()))
    torch.cuda.synchronize()
    assert torch.equal(outs[0][1], outs[2][1]) and torch.equal(outs[0][0], outs[2][0])
    fresh = accept(x, False, q, d, lens, temps, 43, (0, 8), L.specdec_sampler_workspace_bytes(rows))
    assert torch.equal(fresh[1], outs[1][1])


def oracle_accept(logits, q, drafts, lens, temps, u, noise):
    from oracle import spec_sampler as O
    ln = lens.cpu().numpy()
    p = O.probs_from_logits(logits.float().cpu().numpy(), np.repeat(temps.cpu().numpy(), ln))
    args = (q.cpu().numpy(), drafts.cpu().numpy(), ln, u.cpu().numpy(), noise.cpu().numpy())
    n, tail = O.accept_random_varlen(p, *args)
    keep = ~O.near_tie_flags(p, *args)
    return n, tail, keep


@pytest.mark.parametrize("batch,k,V,accepting", [
    (700, 2, 512, False),     # more requests than one wave holds: every row reduced (the full pass 1)
    (64, 7, 151936, True),    # drafts the target likes: long walks of the early-exit pass
    (64, 7, 151936, False),
    (5, 4, 1001, True),       # ragged vocabulary, few requests: many chunks per row
    (300, 3, 4096, True),     # one CTA per request (clusters of 1)
    (148, 5, 8192, True),     # clusters of 3: one row in the first step, then three
])
def test_accept_passes_match_the_oracle(batch, k, V, accepting):
    """specdec_accept's pass 1 in both forms against the oracle: the early-exit walk (each request's rows only up
    to its first rejection, its chunks waiting on each other) and the full pass for batches past one wave."""
    from nanovllm_b200 import spec_sampler as S
    from types import SimpleNamespace
    g = torch.Generator(device=DEV).manual_seed(batch + V)
    lens = torch.randint(1, k + 2, (batch,), device=DEV, generator=g)
    rows = int(lens.sum())
    logits = (torch.randn(rows, V, device=DEV, generator=g) * 3).bfloat16()
    q = torch.softmax(torch.randn(batch, k, V, device=DEV, generator=g) * 3, dim=-1)
    drafts = torch.randint(V, (batch, k), device=DEV, generator=g)
    if accepting:   # drafts = the target's argmax at each verified position, q ~ 0 there: most drafts accepted
        starts = torch.cumsum(lens, 0) - lens
        for b in range(batch):
            for j in range(int(lens[b]) - 1):
                drafts[b, j] = logits[starts[b] + j].float().argmax()
        q = torch.full_like(q, 1e-9)
    temps = torch.full((batch,), 0.9, device=DEV)
    samp = S.sampling_tensors([SimpleNamespace(temperature=0.9, top_k=0, top_p=1.0)] * batch, DEV)
    g1 = torch.Generator(device=DEV).manual_seed(7)
    g2 = torch.Generator(device=DEV).manual_seed(7)
    n, tail = S.accept_from_logits(logits, q, drafts, samp, lens, g1, draws="kernel")
    u = torch.rand(batch, k, device=DEV, generator=g2)
    noise = S.exponential_noise_(torch.empty(batch, V, device=DEV), g2)
    from nanovllm_b200 import _lib
    assert _lib.device_status(DEV) == 0
    want_n, want_tail, keep = oracle_accept(logits, q, drafts, lens, temps, u, noise)
    assert keep.mean() > 0.9
    assert np.array_equal(n.cpu().numpy()[keep], want_n[keep])
    assert np.array_equal(tail.cpu().numpy()[keep], want_tail[keep])
    if accepting:
        assert (n.cpu().numpy() == lens.cpu().numpy() - 1).mean() > 0.5
