"""numpy restatement of the reference's paged attention -- test infrastructure only.

store_kvcache            nanovllm/layers/attention.py:10-40 (and tests/fake_paged_attention.py:14-17)
paged attention          nanovllm/layers/attention.py:59-77 restated by tests/fake_paged_attention.py:20-41: keys
                         gathered through the block table up to the row's key length, SDPA in fp32, causal
                         bottom-right aligned (query j of L_q sees keys 0 .. L_k - L_q + j).
"""
from __future__ import annotations

import numpy as np


def store_kvcache(key, value, k_cache, v_cache, slot_mapping) -> None:
    """attention.py:33-40: key/value [N, Hkv, D] rows to flat slots; slot -1 skipped (in place)."""
    rows = slot_mapping >= 0
    k_cache.reshape(-1, *key.shape[1:])[slot_mapping[rows]] = key[rows]
    v_cache.reshape(-1, *value.shape[1:])[slot_mapping[rows]] = value[rows]


def paged_attention(q, k_cache, v_cache, block_tables, q_starts, q_lens, k_lens, scale: float, causal: bool = True):
    """q [T, H, D]; k_cache / v_cache [blocks, block_size, Hkv, D]; per row r: queries q[q_starts[r] :
    q_starts[r] + q_lens[r]], keys 0 .. k_lens[r]-1 through block_tables[r].  Returns out [T, H, D] fp32 (rows
    not covered stay 0)."""
    q = np.asarray(q, dtype=np.float32)
    T, H, D = q.shape
    block_size, Hkv = k_cache.shape[1], k_cache.shape[2]
    group = H // Hkv
    keys_all = np.asarray(k_cache, dtype=np.float32).reshape(-1, Hkv, D)       # no copy when already fp32
    values_all = np.asarray(v_cache, dtype=np.float32).reshape(-1, Hkv, D)
    out = np.zeros((T, H, D), dtype=np.float32)
    for r in range(len(q_lens)):
        ql, kl, qs = int(q_lens[r]), int(k_lens[r]), int(q_starts[r])
        if ql == 0:
            continue
        positions = np.arange(kl)
        slots = block_tables[r, positions // block_size].astype(np.int64) * block_size + positions % block_size
        keys = keys_all[slots].transpose(1, 2, 0)                 # [Hkv, D, L]
        values = values_all[slots].transpose(1, 0, 2)             # [Hkv, L, D]
        # query head h reads KV head h // group: per KV head, its group's queries as (g, n) rows
        queries = q[qs:qs + ql].reshape(ql, Hkv, group, D).transpose(1, 2, 0, 3).reshape(Hkv, group * ql, D)
        scores = np.matmul(queries, keys) * np.float32(scale)     # [Hkv, G n, L]
        if causal:
            allowed = positions[None, :] <= (kl - ql + np.arange(ql))[:, None]
            scores = np.where(np.tile(allowed, (group, 1))[None], scores, -np.inf)
        scores = scores - scores.max(axis=-1, keepdims=True)
        weights = np.exp(scores)
        weights /= weights.sum(axis=-1, keepdims=True)
        o = np.matmul(weights, values)                            # [Hkv, G n, D]
        out[qs:qs + ql] = o.reshape(Hkv, group, ql, D).transpose(2, 0, 1, 3).reshape(ql, H, D)
    return out
