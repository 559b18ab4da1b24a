"""KV-head tensor-parallel verify attention on the GPU.  Ranks emulated in one process on cuda:0 (each with
its own cache of its KV heads, storing its new K/V through the kernel) must reassemble to the single-GPU
output; with two GPUs visible, two NCCL ranks run the whole TPAttention forward (all-gather included).
Tolerance: bf16 outputs within 2e-2 absolute of the oracle; the emulated ranks within 2e-2 of the single-GPU
kernel (split items may merge in a different number of pieces)."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from test_attention_gpu import ATOL, DEV, oracle_out, paged_case

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_emulated_ranks_reassemble_the_single_gpu_output(world):
    from nanovllm_b200 import attention as A
    from nanovllm_b200.context import reset_context, set_context
    from nanovllm_b200.tp_attention import TPAttention, interleave_heads

    rng = np.random.default_rng(world)
    q_lens = [8] * 20 + [5, 1, 3]
    k_lens = rng.integers(400, 1300, size=len(q_lens)).tolist()
    c = paged_case(q_lens, k_lens, seed=10 + world, pad_rows=1)
    T, H, D = c["q"].shape
    Hkv = c["k_cache"].shape[2]
    local_caches = []
    for r in range(world):
        ks = slice(r * Hkv // world, (r + 1) * Hkv // world)
        local_caches.append((c["k_cache"][:, :, ks].contiguous(), c["v_cache"][:, :, ks].contiguous()))
    A.reset_device_error(DEV)
    A.store_kvcache(c["k"], c["v"], c["k_cache"], c["v_cache"], c["slots"])
    single = A.paged_attention(c["q"], c["k_cache"], c["v_cache"], c["tables"], c["scale"], cu_seqlens_q=c["cu_q"],
                               cu_seqlens_k=c["cu_k"], max_seqlen_q=8)
    set_context(True, c["cu_q"], c["cu_k"], 8, max(c["k_lens"]), c["slots"], None, c["tables"])
    try:
        gathered = torch.full((world, T, H // world, D), float("nan"), dtype=torch.bfloat16, device=DEV)
        for r in range(world):
            m = TPAttention(H, D, c["scale"], Hkv, world=world, rank=r)
            m.k_cache, m.v_cache = local_caches[r]
            qs, ks = m.q_heads, m.kv_heads
            m.local(c["q"][:, qs], c["k"][:, ks], c["v"][:, ks], out=gathered[r])
        got = interleave_heads(gathered)
        torch.cuda.synchronize()
        assert A.device_error(DEV) == 0
    finally:
        reset_context()
    for r in range(world):      # each rank stored exactly its heads of the new tokens
        ks = slice(r * Hkv // world, (r + 1) * Hkv // world)
        assert torch.equal(local_caches[r][0].view(torch.int16), c["k_cache"][:, :, ks].view(torch.int16))
        assert torch.equal(local_caches[r][1].view(torch.int16), c["v_cache"][:, :, ks].view(torch.int16))
    valid = sum(q_lens)
    got_np = got.float().cpu().numpy()[:valid]
    np.testing.assert_allclose(got_np, single.float().cpu().numpy()[:valid], atol=ATOL, rtol=0)
    np.testing.assert_allclose(got_np, oracle_out(c)[:valid], atol=ATOL, rtol=0)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _nccl_worker(rank, world, port, out):
    import torch.distributed as dist
    from test_tp_attention import _case
    from nanovllm_b200.context import set_context
    from nanovllm_b200.tp_attention import TPAttention

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        q, k_cache, v_cache, tables, starts, q_lens, k_lens, scale = _case(seed=3)
        T, H, D = q.shape
        m = TPAttention(H, D, scale, k_cache.shape[2])
        qs, ks = m.q_heads, m.kv_heads
        on = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev).bfloat16()   # noqa: E731
        m.k_cache, m.v_cache = on(k_cache[:, :, ks]), on(v_cache[:, :, ks])
        cu_q = torch.tensor(np.concatenate([[0], np.cumsum(q_lens)]), dtype=torch.int32, device=dev)
        cu_k = torch.tensor(np.concatenate([[0], np.cumsum(k_lens)]), dtype=torch.int32, device=dev)
        slots = torch.full((T,), -1, dtype=torch.int32, device=dev)        # keys already in the caches
        set_context(True, cu_q, cu_k, int(q_lens.max()), int(k_lens.max()), slots, None,
                    torch.from_numpy(tables).to(dev))
        kv_new = torch.zeros(T, ks.stop - ks.start, D, dtype=torch.bfloat16, device=dev)
        got = m(on(q[:, qs]).reshape(T, -1), kv_new, kv_new)
        for _ in range(3):                                                  # repeated calls reuse the buffer
            again = m(on(q[:, qs]).reshape(T, -1), kv_new, kv_new)
        torch.cuda.synchronize()
        out[rank] = (got.float().cpu().numpy(), bool(torch.equal(got, again)))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(300)
@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_nccl_ranks_all_gather_the_heads():
    from oracle import attention as OA
    from test_tp_attention import _case
    world, port = 2, _free_port()
    manager = mp.get_context("spawn").Manager()
    out = manager.dict()
    mp.start_processes(_nccl_worker, args=(world, port, out), nprocs=world, join=True, start_method="spawn")
    q, k_cache, v_cache, tables, starts, q_lens, k_lens, scale = _case(seed=3)
    want = OA.paged_attention(q, k_cache, v_cache, tables, starts, q_lens, k_lens, scale)
    assert np.array_equal(out[0][0], out[1][0]) and out[0][1] and out[1][1]
    np.testing.assert_allclose(out[0][0], want, atol=ATOL, rtol=0)
