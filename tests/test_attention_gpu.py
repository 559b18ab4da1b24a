"""Kernel (2), paged verify / decode attention and the paged K/V store, against the numpy oracle
(oracle/attention.py, the reference's tests/fake_paged_attention.py rule).  Tolerance (north star): bf16
attention outputs within 2e-2 absolute; the K/V store is a bit-exact copy."""
import math

import numpy as np
import pytest
import torch

from oracle import attention as OA

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
ATOL = 2e-2


@pytest.fixture(scope="module")
def A():
    from nanovllm_b200 import attention
    return attention


def paged_case(q_lens, k_lens, H=32, Hkv=8, D=128, block_size=256, seed=0, stale_nan=True, pad_rows=0):
    """Rows with q_lens queries and k_lens keys (the last q_len keys are the new tokens, stored through
    store_kvcache), blocks drawn from a random permutation; unused slots hold NaN (stale cache)."""
    g = torch.Generator(device=DEV).manual_seed(seed)
    R = len(q_lens)
    blocks_per_row = [math.ceil(k / block_size) for k in k_lens]
    W = max(blocks_per_row)
    num_blocks = sum(blocks_per_row) + 3 + 1                         # + spare blocks + the pad block
    perm = torch.randperm(num_blocks - 1, generator=torch.Generator().manual_seed(seed)).tolist()
    pad_block = num_blocks - 1
    k_cache = torch.full((num_blocks, block_size, Hkv, D), float("nan") if stale_nan else 0.0, dtype=torch.bfloat16,
                         device=DEV)
    v_cache = k_cache.clone()
    k_cache[pad_block] = 0
    v_cache[pad_block] = 0
    tables = torch.full((R + pad_rows, W), pad_block, dtype=torch.int32)
    used = 0
    for r, nb in enumerate(blocks_per_row):
        tables[r, :nb] = torch.tensor(perm[used:used + nb], dtype=torch.int32)
        used += nb
    # context keys / values (positions < k_len - q_len) written directly
    for r, (ql, kl) in enumerate(zip(q_lens, k_lens)):
        pos = torch.arange(kl - ql)
        slots = tables[r, pos // block_size].long() * block_size + pos % block_size
        k_cache.view(-1, Hkv, D)[slots.to(DEV)] = torch.randn(len(pos), Hkv, D, device=DEV, generator=g).bfloat16()
        v_cache.view(-1, Hkv, D)[slots.to(DEV)] = torch.randn(len(pos), Hkv, D, device=DEV, generator=g).bfloat16()
    # new tokens: q / k / v of every query position, slot mapping for the store
    q_lens_all = list(q_lens) + [1] * pad_rows
    k_lens_all = list(k_lens) + [1] * pad_rows
    T = sum(q_lens_all)
    q = torch.randn(T, H, D, device=DEV, generator=g).bfloat16()
    k = torch.randn(T, Hkv, D, device=DEV, generator=g).bfloat16()
    v = torch.randn(T, Hkv, D, device=DEV, generator=g).bfloat16()
    slot_mapping = []
    for r, (ql, kl) in enumerate(zip(q_lens_all, k_lens_all)):
        for j in range(ql):
            position = kl - ql + j
            slot_mapping.append(int(tables[r, position // block_size]) * block_size + position % block_size
                                if r < R else -1)
    cu_q = torch.tensor([0] + np.cumsum(q_lens_all).tolist(), dtype=torch.int32, device=DEV)
    cu_k = torch.tensor([0] + np.cumsum(k_lens_all).tolist(), dtype=torch.int32, device=DEV)
    return dict(q=q, k=k, v=v, k_cache=k_cache, v_cache=v_cache, tables=tables.to(DEV), cu_q=cu_q, cu_k=cu_k,
                slots=torch.tensor(slot_mapping, dtype=torch.int32, device=DEV), q_lens=q_lens_all,
                k_lens=k_lens_all, scale=D ** -0.5)


def oracle_out(c, causal=True):
    k_cache = c["k_cache"].float().cpu().numpy()
    v_cache = c["v_cache"].float().cpu().numpy()
    starts = np.concatenate([[0], np.cumsum(c["q_lens"])[:-1]])
    return OA.paged_attention(c["q"].float().cpu().numpy(), k_cache, v_cache, c["tables"].cpu().numpy(), starts,
                              c["q_lens"], c["k_lens"], c["scale"], causal)


def run_verify(A, c):
    A.reset_device_error(DEV)
    A.store_kvcache(c["k"], c["v"], c["k_cache"], c["v_cache"], c["slots"])
    out = A.paged_attention(c["q"], c["k_cache"], c["v_cache"], c["tables"], c["scale"], cu_seqlens_q=c["cu_q"],
                            cu_seqlens_k=c["cu_k"], max_seqlen_q=max(c["q_lens"]))
    torch.cuda.synchronize()
    assert A.device_error(DEV) == 0
    return out


def test_store_kvcache_is_an_exact_copy(A):
    c = paged_case([3, 8], [40, 300], stale_nan=False)
    expected_k = c["k_cache"].float().cpu().numpy()
    expected_v = c["v_cache"].float().cpu().numpy()
    A.store_kvcache(c["k"], c["v"], c["k_cache"], c["v_cache"], c["slots"])
    OA.store_kvcache(c["k"].float().cpu().numpy(), c["v"].float().cpu().numpy(), expected_k, expected_v,
                     c["slots"].cpu().numpy())
    assert np.array_equal(c["k_cache"].float().cpu().numpy(), expected_k)
    assert np.array_equal(c["v_cache"].float().cpu().numpy(), expected_v)


def test_baseline_config2_verify_attention(A):
    """benchmark config 2: 32 rows x 8 queries, 32/8 heads, head_dim 128, contexts U[900, 1100], block size 256,
    random block permutation, stale NaN in unused slots."""
    rng = np.random.default_rng(0)
    k_lens = rng.integers(900, 1101, size=32).tolist()
    c = paged_case([8] * 32, k_lens, seed=1)
    out = run_verify(A, c)
    want = oracle_out(c)
    got = out.float().cpu().numpy()
    assert np.isfinite(got).all()
    np.testing.assert_allclose(got, want, atol=ATOL, rtol=0)


@pytest.mark.parametrize("k_lens", [[1, 2, 8], [127, 128, 129], [255, 256, 257], [383, 512, 640],
                                    [31, 32, 33], [159, 160, 161], [191, 192, 193], [223, 224, 225]])
def test_ragged_rows_and_tile_edges(A, k_lens):
    """Row ends at every 32-key sub-box edge of a last tile (a partial last tile loads only its sub-boxes)."""
    q_lens = [min(k, q) for k, q in zip(k_lens, [1, 5, 8])]
    c = paged_case(q_lens, k_lens, seed=sum(k_lens))
    out = run_verify(A, c)
    np.testing.assert_allclose(out.float().cpu().numpy(), oracle_out(c), atol=ATOL, rtol=0)


def test_padding_rows_read_the_pad_block(A):
    c = paged_case([8, 3], [700, 1000], pad_rows=2, seed=4)
    out = run_verify(A, c)
    got = out.float().cpu().numpy()
    np.testing.assert_allclose(got[:11], oracle_out(c)[:11], atol=ATOL, rtol=0)
    assert np.abs(got[11:]).max() == 0      # attention over the zero pad block


@pytest.mark.parametrize("H,Hkv,ql", [(8, 8, 8), (16, 8, 8), (64, 8, 4), (32, 4, 4)])
def test_gqa_groups(A, H, Hkv, ql):
    c = paged_case([ql, ql, ql], [300, 129, 800], H=H, Hkv=Hkv, seed=H + Hkv)
    out = run_verify(A, c)
    np.testing.assert_allclose(out.float().cpu().numpy(), oracle_out(c), atol=ATOL, rtol=0)


@pytest.mark.parametrize("causal", [False, True])
def test_decode_branch_draft_block(A, causal):
    """The decode branch: query_len_per_seq = 7 queries per row over context_lens (the DFlash draft block is
    non-causal)."""
    k_lens = [7, 100, 300, 1000]
    c = paged_case([7] * 4, k_lens, seed=9)
    A.store_kvcache(c["k"], c["v"], c["k_cache"], c["v_cache"], c["slots"])
    ctx = torch.tensor(k_lens, dtype=torch.int32, device=DEV)
    A.reset_device_error(DEV)
    out = A.paged_attention(c["q"], c["k_cache"], c["v_cache"], c["tables"], c["scale"], context_lens=ctx,
                            query_len_per_seq=7, causal=causal)
    torch.cuda.synchronize()
    assert A.device_error(DEV) == 0
    np.testing.assert_allclose(out.float().cpu().numpy(), oracle_out(c, causal=causal), atol=ATOL, rtol=0)


def test_attention_module_reads_the_context(A):
    from nanovllm_b200.attention import Attention
    from nanovllm_b200.context import reset_context, set_context
    c = paged_case([8, 5], [600, 257], seed=12)
    layer = Attention(32, 128, c["scale"], 8)
    layer.k_cache, layer.v_cache = c["k_cache"], c["v_cache"]
    set_context(True, c["cu_q"], c["cu_k"], 8, 4096, c["slots"], None, c["tables"])
    out = layer(c["q"].view(-1, 32 * 128), c["k"], c["v"])
    reset_context()
    np.testing.assert_allclose(out.float().cpu().numpy(), oracle_out(c), atol=ATOL, rtol=0)


def test_unsupported_shapes_raise(A):
    from nanovllm_b200._lib import SpecdecError
    c = paged_case([8], [100], seed=3)
    with pytest.raises(SpecdecError):
        A.paged_attention(c["q"], c["k_cache"], c["v_cache"], c["tables"], c["scale"], cu_seqlens_q=c["cu_q"],
                          cu_seqlens_k=c["cu_k"], max_seqlen_q=9)


@pytest.mark.parametrize("k_lens", [[20000], [15000, 3000, 40]])
def test_long_rows_split_over_many_ctas(A, k_lens):
    """Rows far longer than one CTA's share of the tile sequence: every item is cut into many pieces that the
    last-arriving CTA merges."""
    c = paged_case([8] * len(k_lens), k_lens, seed=len(k_lens) + 20)
    out = run_verify(A, c)
    got = out.float().cpu().numpy()
    assert np.isfinite(got).all()
    np.testing.assert_allclose(got, oracle_out(c), atol=ATOL, rtol=0)


def test_repeated_launches_are_bitwise_identical(A):
    """Split-item counters clean themselves and pieces merge in a fixed order: three launches agree bit for bit."""
    rng = np.random.default_rng(5)
    c = paged_case([8] * 24, rng.integers(500, 3000, size=24).tolist(), seed=31)
    first = run_verify(A, c)
    for _ in range(2):
        again = A.paged_attention(c["q"], c["k_cache"], c["v_cache"], c["tables"], c["scale"],
                                  cu_seqlens_q=c["cu_q"], cu_seqlens_k=c["cu_k"], max_seqlen_q=8)
        torch.cuda.synchronize()
        assert torch.equal(again, first)
    assert A.device_error(DEV) == 0
    np.testing.assert_allclose(first.float().cpu().numpy(), oracle_out(c), atol=ATOL, rtol=0)


def test_workspace_query(A):
    from nanovllm_b200 import _lib
    lib = _lib.lib()
    need = lib.specdec_attention_workspace_bytes(64, 8)
    sms = torch.cuda.get_device_properties(DEV).multi_processor_count
    assert need == (64 * 8 * 4 + 255) // 256 * 256 + 2 * sms * (32 * 128 + 64) * 4
    assert lib.specdec_attention_workspace_bytes(0, 8) == -1


def test_early_launch_after_the_qk_store(A):
    """An early (programmatic dependent) launch right after the kernel that writes q and the new K/V rows reads
    what that kernel wrote: the same bits as an ordinary launch, and the oracle's values."""
    from nanovllm_b200.fused import qk_norm_rope_store, rope_cache
    rng = np.random.default_rng(7)
    c = paged_case([8] * 16, rng.integers(300, 2000, size=16).tolist(), seed=41)
    T, H, Hkv = c["q"].shape[0], 32, 8
    g = torch.Generator(device=DEV).manual_seed(9)
    qkv = torch.randn(T, (H + 2 * Hkv) * 128, device=DEV, generator=g).bfloat16()
    q_norm = (1.0 + 0.1 * torch.randn(128, device=DEV, generator=g)).bfloat16()
    k_norm = (1.0 + 0.1 * torch.randn(128, device=DEV, generator=g)).bfloat16()
    cos_sin = rope_cache(128, 8192, 1000000.0, DEV)
    positions = torch.tensor([kl - ql + j for ql, kl in zip(c["q_lens"], c["k_lens"]) for j in range(ql)],
                             device=DEV)
    outs, caches = [], []
    for early in (False, True):
        kc, vc = c["k_cache"].clone(), c["v_cache"].clone()
        q = qk_norm_rope_store(qkv, H, Hkv, q_norm, k_norm, cos_sin, positions, c["slots"], kc, vc, 1e-6)
        outs.append(A.paged_attention(q, kc, vc, c["tables"], c["scale"], cu_seqlens_q=c["cu_q"],
                                      cu_seqlens_k=c["cu_k"], max_seqlen_q=8, early_launch=early))
        caches.append((q, kc, vc))
    torch.cuda.synchronize()
    assert A.device_error(DEV) == 0
    assert torch.equal(outs[0], outs[1])
    q, kc, vc = caches[1]
    c2 = dict(c, q=q, k_cache=kc, v_cache=vc)
    np.testing.assert_allclose(outs[1].float().cpu().numpy(), oracle_out(c2), atol=ATOL, rtol=0)


def test_workspace_shared_by_calls_of_different_shapes(A):
    """One workspace, zeroed once, serves calls with different row counts: the split-item counters sit at a fixed
    offset, past the pieces of every call, so a larger call's counters never land on a smaller call's pieces."""
    rng = np.random.default_rng(11)
    big = paged_case([8] * 64, rng.integers(800, 1200, size=64).tolist(), seed=61)
    small = paged_case([8] * 9, rng.integers(2000, 4000, size=9).tolist(), seed=62)

    def attend(c):
        return A.paged_attention(c["q"], c["k_cache"], c["v_cache"], c["tables"], c["scale"], cu_seqlens_q=c["cu_q"],
                                 cu_seqlens_k=c["cu_k"], max_seqlen_q=8)

    first_big = run_verify(A, big)                   # zeroes the workspace, stores the new K/V, attends
    A.store_kvcache(small["k"], small["v"], small["k_cache"], small["v_cache"], small["slots"])
    for _ in range(2):
        out_small = attend(small)
        again_big = attend(big)
        torch.cuda.synchronize()
        assert torch.equal(again_big, first_big)
    assert A.device_error(DEV) == 0
    np.testing.assert_allclose(out_small.float().cpu().numpy(), oracle_out(small), atol=ATOL, rtol=0)
