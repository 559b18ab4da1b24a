"""numpy restatement of the draft context store and the target's q/k norm + RoPE -- test infrastructure only.

DFlashDraftModel.store_context_kv   nanovllm/models/dflash.py:88-96
RMSNorm.rms_forward                 nanovllm/layers/layernorm.py:16-26  (fp32 stats; cast to bf16, times weight)
apply_rotary_emb / RotaryEmbedding   nanovllm/layers/rotary_embedding.py:6-27
store_kvcache                       nanovllm/layers/attention.py:33-40
SiluAndMul                          nanovllm/layers/activation.py:8-11  (compiled: fp32 math, one bf16 rounding)
bf16 arithmetic is emulated with round-to-nearest-even on the fp32 bit patterns.
"""
from __future__ import annotations

import numpy as np


def bf16(x: np.ndarray) -> np.ndarray:
    """Rounds fp32 values to bf16 (nearest, ties to even), returned as fp32."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    rounded = (u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))) & np.uint32(0xFFFF0000)
    return rounded.view(np.float32)


def rope_cache(head_dim: int, max_position: int, base: float) -> np.ndarray:
    """rotary_embedding.py:17-27 in fp32: [max_position, head_dim] = cos | sin of t * inv_freq."""
    inv_freq = (1.0 / (base ** (np.arange(0, head_dim, 2, dtype=np.float32) / head_dim))).astype(np.float32)
    t = np.arange(max_position, dtype=np.float32)
    freqs = np.outer(t, inv_freq).astype(np.float32)
    return np.concatenate([np.cos(freqs), np.sin(freqs)], axis=-1).astype(np.float32)


def silu_and_mul(gate_up: np.ndarray) -> np.ndarray:
    """activation.py:8-11: silu(x) * y over the two halves of the last dim, in fp32, rounded once to bf16 (the
    reference's torch.compile'd forward fuses the two ops; its eager body rounds after each, within one bf16 ulp
    of this)."""
    gate_up = gate_up.astype(np.float32)
    a, b = np.split(gate_up, 2, axis=-1)
    return bf16(a / (np.float32(1.0) + np.exp(-a)) * b)


def rmsnorm(x: np.ndarray, weight: np.ndarray, eps: float) -> np.ndarray:
    """layernorm.py:16-26 over the last dim; x and weight hold bf16 values; result bf16 (as fp32)."""
    x = x.astype(np.float32)
    var = np.mean(x * x, axis=-1, keepdims=True, dtype=np.float32)
    y = bf16(x * (np.float32(1.0) / np.sqrt(var + np.float32(eps))))
    return bf16(y * weight.astype(np.float32))


def apply_rope(x: np.ndarray, cos_sin: np.ndarray, positions: np.ndarray) -> np.ndarray:
    """rotary_embedding.py:6-14: x [T, heads, D] bf16 values -> bf16 (as fp32)."""
    half = x.shape[-1] // 2
    cs = cos_sin[positions][:, None, :]
    cos, sin = cs[..., :half], cs[..., half:]
    x1, x2 = x[..., :half], x[..., half:]
    return bf16(np.concatenate([x1 * cos - x2 * sin, x2 * cos + x1 * sin], axis=-1))


def norm_rope_store(kv: np.ndarray, num_kv_heads: int, k_norm: np.ndarray, cos_sin: np.ndarray,
                    positions: np.ndarray, slot_mapping: np.ndarray, k_cache: np.ndarray, v_cache: np.ndarray,
                    eps: float) -> None:
    """dflash.py:93-96 for one layer given its projection kv [T, 2 Hkv D] (bf16 values): k_norm, RoPE(k), then
    store_kvcache into k_cache / v_cache [slots, Hkv, D] (in place; slot -1 skipped)."""
    T = kv.shape[0]
    k = kv[:, : num_kv_heads * 128].reshape(T, num_kv_heads, 128)
    v = kv[:, num_kv_heads * 128:].reshape(T, num_kv_heads, 128)
    k = apply_rope(rmsnorm(k, k_norm, eps), cos_sin, positions)
    rows = slot_mapping >= 0
    k_cache.reshape(-1, num_kv_heads, 128)[slot_mapping[rows]] = k[rows]
    v_cache.reshape(-1, num_kv_heads, 128)[slot_mapping[rows]] = v[rows]


def q_norm_rope(q: np.ndarray, q_norm: np.ndarray, cos_sin: np.ndarray, positions: np.ndarray,
                eps: float) -> np.ndarray:
    """qwen3.py:77-84 for the query heads: q_norm then RoPE; q [T, H, D] bf16 values."""
    return apply_rope(rmsnorm(q, q_norm, eps), cos_sin, positions)
