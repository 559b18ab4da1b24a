"""Fused elementwise kernels around the verify forward (libspecdec_b200.so), mirroring the reference layers:

    rmsnorm(x, weight, eps[, residual])     nanovllm/layers/layernorm.py:16-40  -> specdec_rmsnorm
    silu_and_mul(gate_up)                   nanovllm/layers/activation.py:8-11  -> specdec_silu_mul
    qk_norm_rope_store(...)                 nanovllm/models/qwen3.py:77-86 + attention.py:62-63
                                            (q_norm, k_norm, RoPE, store_kvcache in one launch) -> specdec_norm_rope_store
    rope_cache(head_dim, max_position, base) nanovllm/layers/rotary_embedding.py:17-27 (the cos|sin table)
"""
from __future__ import annotations

import torch

from . import _lib
from ._lib import Workspace, check, ptr, require_cuda, stream_of


def err_word(device: torch.device) -> torch.Tensor:
    return Workspace.get(device, 256, name="fused")[:4].view(torch.int32)


def rope_cache(head_dim: int, max_position: int, base: float, device: torch.device) -> torch.Tensor:
    """rotary_embedding.py:17-27: [max_position, head_dim] fp32 = cat(cos(t * inv_freq), sin(t * inv_freq))."""
    inv_freq = 1.0 / (base ** (torch.arange(0, head_dim, 2, dtype=torch.float) / head_dim))
    t = torch.arange(max_position, dtype=torch.float)
    freqs = torch.einsum("i,j -> ij", t, inv_freq)
    return torch.cat((freqs.cos(), freqs.sin()), dim=-1).contiguous().to(device)


def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float, residual: torch.Tensor | None = None, *,
            out: torch.Tensor | None = None):
    """layernorm.py:16-40: without residual returns norm(x); with it returns (norm(x + residual), x + residual)."""
    device = require_cuda(x, weight, residual)
    width = x.shape[-1]
    T = x.numel() // width
    x = x.contiguous()
    out = torch.empty_like(x) if out is None else out
    res_out = torch.empty_like(x) if residual is not None else None
    check(_lib.lib().specdec_rmsnorm(ptr(x), ptr(None if residual is None else residual.contiguous()), ptr(weight),
                                     ptr(out), ptr(res_out), T, width, float(eps), stream_of(device)))
    return out if residual is None else (out, res_out)


def silu_and_mul(gate_up: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """activation.py:8-11: silu(x) * y over the two halves of the last dim (fp32 math, one rounding)."""
    device = require_cuda(gate_up)
    two_i = gate_up.shape[-1]
    T = gate_up.numel() // two_i
    if out is None:
        out = torch.empty(*gate_up.shape[:-1], two_i // 2, dtype=gate_up.dtype, device=device)
    check(_lib.lib().specdec_silu_mul(ptr(gate_up.contiguous()), ptr(out), T, two_i // 2, stream_of(device)))
    return out


def qk_norm_rope_store(qkv: torch.Tensor, num_heads: int, num_kv_heads: int, q_norm: torch.Tensor,
                       k_norm: torch.Tensor, cos_sin: torch.Tensor, positions: torch.Tensor,
                       slot_mapping: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, eps: float,
                       q_out: torch.Tensor | None = None) -> torch.Tensor:
    """The verify forward's qkv [T, (H + 2 Hkv) * 128] -> q [T, H, 128] (q_norm, RoPE); k_norm + RoPE'd K and V
    rows go straight to their slots of the layer's paged caches (slot -1 skipped)."""
    device = require_cuda(qkv, positions, slot_mapping, k_cache, v_cache)
    T = qkv.shape[0]
    head_dim = 128
    if q_out is None:
        q_out = torch.empty(T, num_heads, head_dim, dtype=qkv.dtype, device=device)
    num_slots = k_cache.numel() // (num_kv_heads * head_dim)
    check(_lib.lib().specdec_norm_rope_store(
        ptr(qkv), 0, qkv.stride(0), T, 1, num_heads, num_kv_heads, ptr(q_norm), ptr(k_norm), 0, ptr(cos_sin),
        cos_sin.shape[0], ptr(positions), ptr(slot_mapping), ptr(k_cache), ptr(v_cache), 0, num_slots, ptr(q_out),
        float(eps), ptr(err_word(device)), stream_of(device)))
    return q_out
