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


def _nccl_worker(rank, world, port, out, exchange):
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
        m = TPAttention(H, D, scale, k_cache.shape[2], exchange=exchange, max_tokens=T, device=dev)
        qs, ks = m.q_heads, m.kv_heads
        on = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev).bfloat16()   # noqa: E731
        m.k_cache, m.v_cache = on(k_cache[:, :, ks]), on(v_cache[:, :, ks])
        cu_q = torch.tensor(np.concatenate([[0], np.cumsum(q_lens)]), dtype=torch.int32, device=dev)
        cu_k = torch.tensor(np.concatenate([[0], np.cumsum(k_lens)]), dtype=torch.int32, device=dev)
        slots = torch.full((T,), -1, dtype=torch.int32, device=dev)        # keys already in the caches
        set_context(True, cu_q, cu_k, int(q_lens.max()), int(k_lens.max()), slots, None,
                    torch.from_numpy(tables).to(dev))
        kv_new = torch.zeros(T, ks.stop - ks.start, D, dtype=torch.bfloat16, device=dev)
        got = m(on(q[:, qs]).reshape(T, -1), kv_new, kv_new).clone()
        for _ in range(3):                                                  # repeated calls reuse the buffers
            again = m(on(q[:, qs]).reshape(T, -1), kv_new, kv_new)
        torch.cuda.synchronize()
        status = m.peer_error() if exchange == "peer" else 0
        out[rank] = (got.float().cpu().numpy(), bool(torch.equal(got, again)), status)
        dist.barrier()
    finally:
        dist.destroy_process_group()


def _gpus() -> int:
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


@pytest.mark.timeout(300)
@pytest.mark.parametrize("exchange", ["nccl", "peer"])
@pytest.mark.parametrize("world", [2, 4, 8])
def test_ranks_gather_the_heads(world, exchange):
    """world ranks, one per GPU, each holding 8 / world KV heads (one per GPU at 8, as benchmark config 5's TP
    mode): every rank ends with the same [T, H, D] output, equal to the oracle's single-GPU attention."""
    if _gpus() < world:
        pytest.skip(f"needs {world} GPUs")
    from oracle import attention as OA
    from test_tp_attention import _case
    port = _free_port()
    manager = mp.get_context("spawn").Manager()
    out = manager.dict()
    mp.start_processes(_nccl_worker, args=(world, port, out, exchange), nprocs=world, join=True,
                       start_method="spawn")
    q, k_cache, v_cache, tables, starts, q_lens, k_lens, scale = _case(seed=3)
    want = OA.paged_attention(q, k_cache, v_cache, tables, starts, q_lens, k_lens, scale)
    for r in range(world):
        assert out[r][2] == 0 and out[r][1]
        assert np.array_equal(out[0][0], out[r][0])
    np.testing.assert_allclose(out[0][0], want, atol=ATOL, rtol=0)


def test_multi_destination_outputs_match_the_single_output_bit_for_bit():
    """specdec_paged_attention_multi with three destinations (each at a head offset of a wider output, as the
    peer-store mode writes every rank's buffer) stores exactly the single-output result in each."""
    from nanovllm_b200 import attention as A
    c = paged_case([8, 8, 3, 1], [700, 129, 1000, 40], seed=21, pad_rows=1)
    T, H, D = c["q"].shape
    A.reset_device_error(DEV)
    A.store_kvcache(c["k"], c["v"], c["k_cache"], c["v_cache"], c["slots"])
    single = A.paged_attention(c["q"], c["k_cache"], c["v_cache"], c["tables"], c["scale"], cu_seqlens_q=c["cu_q"],
                               cu_seqlens_k=c["cu_k"], max_seqlen_q=8)
    wide = [torch.full((T, 3 * H, D), float("nan"), dtype=torch.bfloat16, device=DEV) for _ in range(3)]
    ptrs = [w.data_ptr() + (i * H * D) * 2 for i, w in enumerate(wide)]   # destination i at head offset i*H
    A.paged_attention_to(c["q"], c["k_cache"], c["v_cache"], c["tables"], c["scale"], ptrs, 3 * H * D,
                         cu_seqlens_q=c["cu_q"], cu_seqlens_k=c["cu_k"], max_seqlen_q=8)
    torch.cuda.synchronize()
    assert A.device_error(DEV) == 0
    for i, w in enumerate(wide):
        got = w[:, i * H:(i + 1) * H]
        assert torch.equal(got.view(torch.int16), single.view(torch.int16))
        rest = torch.cat([w[:, :i * H], w[:, (i + 1) * H:]], dim=1)
        assert torch.isnan(rest.float()).all()          # nothing written outside the destination's heads


def _barrier(flags, world, rank, epoch, timeout_ns, err):
    import ctypes
    from nanovllm_b200 import _lib
    from nanovllm_b200._lib import check, stream_of
    arr = (ctypes.c_void_p * world)(*[f.data_ptr() for f in flags])
    check(_lib.lib().specdec_peer_barrier(arr, world, rank, epoch.data_ptr(), timeout_ns, err.data_ptr(),
                                          stream_of(DEV)))


def test_peer_barrier_passes_when_every_rank_has_arrived():
    """One rank's barrier on one GPU: alone (world 1), and in a world of 2 whose peer already signalled the
    epoch (its word pre-set, as the peer's own barrier would have stored it).  No second waiting kernel runs."""
    epoch = torch.zeros(1, dtype=torch.int32, device=DEV)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    mine = torch.zeros(8, dtype=torch.int32, device=DEV)
    _barrier([mine], 1, 0, epoch, 10**9, err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0 and int(epoch.item()) == 1 and int(mine[0].item()) == 1
    epoch.zero_()
    mine.zero_()
    peer = torch.zeros(8, dtype=torch.int32, device=DEV)
    mine[1] = 1                              # rank 1 has arrived at epoch 1
    _barrier([mine, peer], 2, 0, epoch, 10**9, err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0 and int(epoch.item()) == 1
    assert peer.tolist()[:2] == [1, 0]       # rank 0 signalled rank 1 at epoch 1


def test_peer_barrier_wait_is_bounded_and_reports_a_status():
    """A peer that never arrives (its word is never set): the wait gives up after its 50 ms limit, records 21
    and returns; the context stays usable."""
    epoch = torch.zeros(1, dtype=torch.int32, device=DEV)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    mine = torch.zeros(8, dtype=torch.int32, device=DEV)
    peer = torch.zeros(8, dtype=torch.int32, device=DEV)
    _barrier([mine, peer], 2, 0, epoch, 50_000_000, err)
    torch.cuda.synchronize()
    assert int(err.item()) == 21
    assert float(torch.ones(4, device=DEV).sum().item()) == 4.0
