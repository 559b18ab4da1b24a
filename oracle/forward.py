"""numpy restatement of the Qwen3 verify forward -- test infrastructure only (the checker of the B200 forward at
small sizes, and the timed CPU baseline of bench.py).

Qwen3Model.forward         nanovllm/models/qwen3.py:176-191 (aux export hidden + residual, :186-190)
Qwen3DecoderLayer.forward  nanovllm/models/qwen3.py:147-160
Qwen3Attention.forward     nanovllm/models/qwen3.py:70-86   (qkv split, q_norm / k_norm, RoPE, paged attention,
                                                             o_proj)
Qwen3MLP.forward           nanovllm/models/qwen3.py:105-109 (gate_up, SiluAndMul, down)
RMSNorm                    nanovllm/layers/layernorm.py:16-38 (with a residual: the sum in fp32, the residual
                                                             output rounded, the norm of the fp32 sum)
ParallelLMHead (all logits) nanovllm/layers/embed_head.py, qwen3.py:221-226
Linear layers are bf16 GEMMs with fp32 accumulation: here an fp32 product rounded once to bf16.
"""
from __future__ import annotations

import numpy as np

from .attention import paged_attention, store_kvcache
from .ctx_store import apply_rope, bf16, rmsnorm, silu_and_mul


def rmsnorm_residual(x: np.ndarray, residual: np.ndarray, weight: np.ndarray, eps: float):
    """layernorm.py:28-38: (norm(x + residual), bf16(x + residual)) with the sum kept in fp32 for the norm."""
    s = x.astype(np.float32) + residual.astype(np.float32)
    return rmsnorm(s, weight, eps), bf16(s)


def linear(x: np.ndarray, w: np.ndarray) -> np.ndarray:
    """x [T, in] . w [out, in]^T, fp32 accumulation, one bf16 rounding."""
    return bf16(np.matmul(np.asarray(x, dtype=np.float32), np.asarray(w, dtype=np.float32).T))


def decoder_layer(w: dict, h: np.ndarray, residual: np.ndarray | None, positions: np.ndarray,
                  slot_mapping: np.ndarray, k_cache: np.ndarray, v_cache: np.ndarray, block_tables: np.ndarray,
                  q_starts, q_lens, k_lens, cos_sin: np.ndarray, heads: int, kv_heads: int, eps: float,
                  causal: bool = True, attend=paged_attention):
    """qwen3.py:147-160 for one layer (weights as in nanovllm_b200.target.random_layer_weights, bf16 values in
    fp32 arrays); stores the layer's K/V rows at slot_mapping into k_cache / v_cache [blocks, block_size, Hkv, D]
    (in place) and attends per row r to keys 0 .. k_lens[r] - 1 (attend: oracle.attention.paged_attention or a
    function with its signature and results, e.g. the same split over threads).  Returns (hidden, residual)."""
    T = h.shape[0]
    D = 128
    if residual is None:
        x, residual = rmsnorm(h, w["in_norm"], eps), h
    else:
        x, residual = rmsnorm_residual(h, residual, w["in_norm"], eps)
    qkv = linear(x, w["w_qkv"])                                                         # :74
    q = qkv[:, :heads * D].reshape(T, heads, D)
    k = qkv[:, heads * D:(heads + kv_heads) * D].reshape(T, kv_heads, D)
    v = qkv[:, (heads + kv_heads) * D:].reshape(T, kv_heads, D)
    q = apply_rope(rmsnorm(q, w["q_norm"], eps), cos_sin, positions)                   # :79-82
    k = apply_rope(rmsnorm(k, w["k_norm"], eps), cos_sin, positions)
    store_kvcache(k, v, k_cache, v_cache, slot_mapping)                                 # attention.py:62-63
    o = bf16(attend(q, k_cache, v_cache, block_tables, q_starts, q_lens, k_lens, D ** -0.5, causal))
    h = linear(o.reshape(T, heads * D), w["w_o"])                                       # :85
    x, residual = rmsnorm_residual(h, residual, w["post_norm"], eps)                    # :158
    h = linear(silu_and_mul(linear(x, w["w_gate_up"])), w["w_down"])                    # :107-109
    return h, residual


def forward(embed: np.ndarray, layers: list[dict], final_norm: np.ndarray, input_ids: np.ndarray,
            positions: np.ndarray, slot_mapping: np.ndarray, kv_caches: list[tuple[np.ndarray, np.ndarray]],
            block_tables: np.ndarray, q_starts, q_lens, k_lens, cos_sin: np.ndarray, heads: int, kv_heads: int,
            eps: float, aux_layer_ids=(), causal: bool = True):
    """qwen3.py:176-191: hidden states after the final norm, and the aux layers' outputs (hidden + residual,
    bf16) concatenated in aux_layer_ids order ([T, 0] without aux layers)."""
    h = embed[input_ids].astype(np.float32)
    residual = None
    aux = []
    for layer_id, w in enumerate(layers):
        k_cache, v_cache = kv_caches[layer_id]
        h, residual = decoder_layer(w, h, residual, positions, slot_mapping, k_cache, v_cache, block_tables, q_starts,
                                    q_lens, k_lens, cos_sin, heads, kv_heads, eps, causal)
        if layer_id in aux_layer_ids:
            aux.append(bf16(h + residual))
    hidden, _ = rmsnorm_residual(h, residual, final_norm, eps)
    aux_out = np.concatenate(aux, axis=-1) if aux else np.zeros((h.shape[0], 0), np.float32)
    return hidden, aux_out


def compute_logits(hidden: np.ndarray, lm_head: np.ndarray) -> np.ndarray:
    """qwen3.py:221-226 with all_logits: [T, V] bf16 values."""
    return linear(hidden, lm_head)
