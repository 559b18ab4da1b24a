"""specdec_accept_noalloc: the fused accept for callers that cannot allocate device memory (a plugin whose host
process owns the device memory budget, or a latency-critical caller that may not call cudaMalloc).  Its scratch
is a fixed array inside the library, so this checks, through the C ABI, that two calls in a row give exactly
what the workspace entry point gives on the same inputs, and that sizes beyond its limit are refused.  The
file sorts last so that a run stopping at the first failure has run every other test first."""
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
V = 151936


def case(seed, batch, k, dtype, varlen):
    g = torch.Generator(device=DEV).manual_seed(seed)
    lens = (torch.randint(1, k + 2, (batch,), device=DEV, generator=g) if varlen
            else torch.full((batch,), k + 1, device=DEV))
    total = int(lens.sum())
    logits = (torch.randn(total, V, device=DEV, generator=g) * 3).to(dtype)
    q = torch.softmax(torch.randn(batch, k, V, device=DEV, generator=g) * 3, dim=-1)
    drafts = torch.randint(V, (batch, k), device=DEV, generator=g)
    temps = torch.full((batch,), 0.9, device=DEV)
    return logits, q, drafts, (lens if varlen else None), temps


def call(lib, name, logits, q, drafts, lens, temps, seed, workspace=None, top_k=None, top_p=None):
    batch, k = drafts.shape
    max_top_k = 0 if top_k is None else int(top_k.max())
    has_top_p = 0 if top_p is None else int((top_p < 1).any())
    n_accept = torch.full((batch,), -1, dtype=torch.int64, device=DEV)
    tail = torch.full((batch,), -1, dtype=torch.int64, device=DEV)
    dtype_code = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}[logits.dtype]
    args = [logits.data_ptr(), 0, dtype_code, logits.shape[0], V, q.data_ptr(), drafts.data_ptr(), batch, k,
            None if lens is None else lens.data_ptr(), temps.data_ptr(), None if top_k is None else top_k.data_ptr(),
            None if top_p is None else top_p.data_ptr(), max_top_k, has_top_p, None, None, seed, 0, 4,
            n_accept.data_ptr(), tail.data_ptr()]
    if workspace is not None:
        args += [workspace.data_ptr(), workspace.numel()]
    status = getattr(lib, name)(*args, torch.cuda.current_stream().cuda_stream)
    return status, n_accept, tail


def test_no_alloc_accept_matches_the_workspace_entry_point_twice():
    from nanovllm_b200 import _lib
    lib = _lib.load()
    calls = [case(1, 64, 7, torch.bfloat16, False), case(2, 40, 7, torch.float32, True)]
    for i, (logits, q, drafts, lens, temps) in enumerate(calls):
        workspace = torch.zeros(lib.specdec_sampler_workspace_bytes(logits.shape[0]), dtype=torch.uint8,
                                device=DEV)
        st_ref, n_ref, t_ref = call(lib, "specdec_accept", logits, q, drafts, lens, temps, 100 + i, workspace)
        st, n, t = call(lib, "specdec_accept_noalloc", logits, q, drafts, lens, temps, 100 + i)
        torch.cuda.synchronize()
        assert st_ref == 0 and st == 0, lib.specdec_last_error()
        assert torch.equal(n, n_ref) and torch.equal(t, t_ref)
        assert (n >= 0).all() and (t >= 0).all()


def test_no_alloc_accept_with_truncation_matches_the_workspace_entry_point():
    """Top-k / top-p rows: the kept-token tail race (every row truncated) and the gated full-row race (rows
    without top-k mixed in) through the fixed scratch, twice in a row."""
    from nanovllm_b200 import _lib
    lib = _lib.load()
    for i, mixed in enumerate([False, True]):
        logits, q, drafts, lens, temps = case(10 + i, 32, 7, torch.bfloat16, True)
        top_k = torch.full((32,), 20, dtype=torch.int64, device=DEV)
        if mixed:
            top_k[::3] = 0
        top_p = torch.where(top_k > 0, 0.8, 1.0).float()
        workspace = torch.zeros(lib.specdec_sampler_workspace_bytes(logits.shape[0]), dtype=torch.uint8,
                                device=DEV)
        ref = call(lib, "specdec_accept", logits, q, drafts, lens, temps, 50 + i, workspace, top_k, top_p)
        for _ in range(2):
            got = call(lib, "specdec_accept_noalloc", logits, q, drafts, lens, temps, 50 + i, None, top_k, top_p)
            torch.cuda.synchronize()
            assert ref[0] == 0 and got[0] == 0, lib.specdec_last_error()
            assert torch.equal(got[1], ref[1]) and torch.equal(got[2], ref[2])


def test_no_alloc_accept_refuses_more_rows_than_its_scratch_holds():
    from nanovllm_b200 import _lib
    lib = _lib.load()
    logits, q, drafts, lens, temps = case(3, 129, 7, torch.bfloat16, False)     # 1032 rows > 1024
    st, n, _ = call(lib, "specdec_accept_noalloc", logits, q, drafts, lens, temps, 7)
    assert st == 3
    assert b"at most 1024 verified rows" in lib.specdec_last_error()
    assert (n == -1).all()                      # nothing was launched


def test_no_alloc_accept_allocates_no_device_memory():
    """The entry point's contract: after a first call on the device (which looks up the array's address), a call
    leaves the device's free memory exactly where it was, and a call the host rejects launches nothing."""
    from nanovllm_b200 import _lib
    lib = _lib.load()
    logits, q, drafts, lens, temps = case(4, 48, 7, torch.bfloat16, True)
    assert call(lib, "specdec_accept_noalloc", logits, q, drafts, lens, temps, 11)[0] == 0
    n_accept = torch.full((48,), -1, dtype=torch.int64, device=DEV)
    tail = torch.full((48,), -1, dtype=torch.int64, device=DEV)
    torch.cuda.synchronize()
    free_before, _ = torch.cuda.mem_get_info(DEV)
    stream = torch.cuda.current_stream().cuda_stream
    args = [logits.data_ptr(), 0, 1, logits.shape[0], V, q.data_ptr(), drafts.data_ptr(), 48, 7, lens.data_ptr(),
            temps.data_ptr(), None, None, 0, 0, None, None, 12, 0, 4, n_accept.data_ptr(), tail.data_ptr(), stream]
    assert lib.specdec_accept_noalloc(*args) == 0
    rejected = list(args)
    rejected[2] = 9                                       # an unknown dtype code
    assert lib.specdec_accept_noalloc(*rejected) == 1
    torch.cuda.synchronize()
    free_after, _ = torch.cuda.mem_get_info(DEV)
    assert free_after == free_before
    assert (n_accept >= 0).all() and (tail >= 0).all()
