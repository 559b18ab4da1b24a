"""Host logic of the KV-head tensor-parallel verify attention on CPU: the head split (the reference's rank-order
chunks), the interleave of the gathered chunks, and the in-place all-gather over two gloo ranks, each rank's
local heads computed by the numpy oracle.  Tolerance: outputs are bf16, compared within 2e-2 absolute."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from nanovllm_b200.tp_attention import TPAttention, interleave_heads, shard_heads
from oracle import attention as OA


@pytest.mark.parametrize("heads,kv_heads,world", [(32, 8, 1), (32, 8, 2), (32, 8, 4), (32, 8, 8), (16, 2, 2)])
def test_shards_cover_every_head_once_with_whole_groups(heads, kv_heads, world):
    group = heads // kv_heads
    q_seen, kv_seen = [], []
    for rank in range(world):
        qs, ks = shard_heads(heads, kv_heads, world, rank)
        q_seen += list(range(heads))[qs]
        kv_seen += list(range(kv_heads))[ks]
        # the query heads of a rank are exactly the GQA groups of its KV heads
        assert list(range(heads))[qs] == [h for kh in range(kv_heads)[ks] for h in range(kh * group, (kh + 1) * group)]
    assert q_seen == list(range(heads)) and kv_seen == list(range(kv_heads))


@pytest.mark.parametrize("heads,kv_heads,world,rank", [(32, 8, 16, 0), (32, 8, 3, 0), (30, 8, 2, 0), (32, 8, 2, 2)])
def test_uneven_splits_raise(heads, kv_heads, world, rank):
    with pytest.raises(ValueError):
        shard_heads(heads, kv_heads, world, rank)


def test_interleave_places_rank_chunks_at_their_heads():
    N, T, Hl, D = 4, 5, 3, 2
    gathered = torch.arange(N * T * Hl * D, dtype=torch.float32).view(N, T, Hl, D)
    out = interleave_heads(gathered)
    for r in range(N):
        for j in range(Hl):
            assert torch.equal(out[:, r * Hl + j], gathered[r, :, j])
    into = torch.empty(T, N * Hl, D)
    assert interleave_heads(gathered, into) is into and torch.equal(into, out)


def _case(seed=0, H=32, Hkv=8, D=128, bs=256, q_lens=(8, 8, 5, 1), k_lens=(300, 129, 1000, 40)):
    rng = np.random.default_rng(seed)
    nblk = [-(-k // bs) for k in k_lens]
    tables = np.zeros((len(k_lens), max(nblk)), np.int32)
    perm = rng.permutation(sum(nblk))
    used = 0
    for r, n in enumerate(nblk):
        tables[r, :n] = perm[used:used + n]
        used += n
    bf16 = lambda a: torch.from_numpy(a.astype(np.float32)).bfloat16().float().numpy()   # noqa: E731
    k_cache = bf16(rng.standard_normal((sum(nblk), bs, Hkv, D)))
    v_cache = bf16(rng.standard_normal((sum(nblk), bs, Hkv, D)))
    q = bf16(rng.standard_normal((sum(q_lens), H, D)))
    starts = np.concatenate([[0], np.cumsum(q_lens)[:-1]])
    return q, k_cache, v_cache, tables, starts, np.array(q_lens), np.array(k_lens), D ** -0.5


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        q, k_cache, v_cache, tables, starts, q_lens, k_lens, scale = _case()
        T, H, D = q.shape
        m = TPAttention(H, D, scale, k_cache.shape[2])
        assert (m.world, m.rank) == (world, rank)
        qs, ks = m.q_heads, m.kv_heads
        # this rank's heads, over its own cache (its KV heads only), by the oracle in place of the kernel
        local = OA.paged_attention(q[:, qs], np.ascontiguousarray(k_cache[:, :, ks]),
                                   np.ascontiguousarray(v_cache[:, :, ks]), tables, starts, q_lens, k_lens, scale)
        gathered = m.gather_buffer(T, torch.device("cpu"))
        gathered[rank] = torch.from_numpy(local).bfloat16()
        got = interleave_heads(m.all_gather(gathered))
        out[rank] = got.float().numpy()
    finally:
        dist.destroy_process_group()


def test_all_gather_over_two_gloo_ranks_matches_full_attention():
    world, port = 2, _free_port()
    manager = mp.get_context("spawn").Manager()
    out = manager.dict()
    mp.start_processes(_worker, args=(world, port, out), nprocs=world, join=True, start_method="spawn")
    q, k_cache, v_cache, tables, starts, q_lens, k_lens, scale = _case()
    want = OA.paged_attention(q, k_cache, v_cache, tables, starts, q_lens, k_lens, scale)
    assert np.array_equal(out[0], out[1])
    np.testing.assert_allclose(out[0], want, atol=2e-2, rtol=0)


def test_module_validates_its_exchange_on_the_host():
    with pytest.raises(ValueError):
        TPAttention(32, 128, 0.088, 8, exchange="allreduce")
    with pytest.raises(ValueError):          # the peer exchange needs a process group (and a CUDA device)
        TPAttention(32, 128, 0.088, 8, exchange="peer", max_tokens=512, device=torch.device("cuda", 0))
    with pytest.raises(ValueError):
        TPAttention(32, 128, 0.088, 8, exchange="peer", max_tokens=0, device=torch.device("cuda", 0))


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_emulated_rank_modules_hold_their_heads_and_one_growing_buffer(world):
    for rank in range(world):
        m = TPAttention(32, 128, 0.088, 8, world=world, rank=rank)
        assert (m.world, m.rank) == (world, rank)
        assert (m.local.num_heads, m.local.num_kv_heads) == (32 // world, 8 // world)
        assert m.q_heads == slice(rank * 32 // world, (rank + 1) * 32 // world)
        big = m.gather_buffer(64, torch.device("cpu"))
        assert big.shape == (world, 64, 32 // world, 128) and big.dtype == torch.bfloat16
        small = m.gather_buffer(16, torch.device("cpu"))
        assert small.shape == (world, 16, 32 // world, 128)
        assert small.data_ptr() == big.data_ptr()        # smaller calls reuse the persistent storage
        m.k_cache = torch.zeros(2, 256, 8 // world, 128)
        assert m.local.k_cache is m.k_cache


def test_grown_buffers_keep_their_predecessors_alive():
    """A CUDA graph captured before a buffer grows keeps addressing the old storage: growth retires, never
    frees, the previous buffer (the gather buffer here, the library workspaces alike)."""
    from nanovllm_b200._lib import Workspace
    m = TPAttention(32, 128, 0.088, 8, world=2, rank=0)
    small = m.gather_buffer(8, torch.device("cpu"))
    big = m.gather_buffer(64, torch.device("cpu"))
    assert big.data_ptr() != small.data_ptr()
    assert any(t.data_ptr() == small.data_ptr() for t in m._retired)
    dev = torch.device("cpu", 0)
    first = Workspace.get(dev, 16, name="growth-test")
    grown = Workspace.get(dev, (2 << 20), name="growth-test")
    assert grown.numel() >= (2 << 20) and not grown.any()
    assert any(t.data_ptr() == first.data_ptr() for t in Workspace._retired)
