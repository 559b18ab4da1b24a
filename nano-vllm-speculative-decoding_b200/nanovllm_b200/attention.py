"""The reference's attention layer (nanovllm/layers/attention.py) on the B200 kernels of libspecdec_b200.so.

    store_kvcache(key, value, k_cache, v_cache, slot_mapping)   attention.py:33-40   -> specdec_store_kvcache
    Attention(num_heads, head_dim, scale, num_kv_heads).forward  attention.py:43-77   -> specdec_paged_attention

Attention.forward reads the module-global context (nanovllm_b200.context, the reference's nanovllm/utils/context.py)
and serves the two paged branches of the reference:
  - verify (is_prefill with block_tables): varlen over cu_seqlens_q / cu_seqlens_k, causal bottom-right aligned;
  - decode (not is_prefill): query_len_per_seq queries per row over context_lens, causal or not (the DFlash
    draft block).
Plain prefill without a block table is not on the verify/accept path and raises NotImplementedError.

Shapes: q [T, H, 128], k / v [T, Hkv, 128] bf16; k_cache / v_cache [blocks, block_size, Hkv, 128] bf16 with
block_size a multiple of 128; rows of at most 32 / (H / Hkv) queries (8 for Qwen3's GQA group of 4).
"""
from __future__ import annotations

import ctypes

import torch
from torch import nn

from . import _lib
from ._lib import Workspace, check, ptr, require_cuda, stream_of
from .context import get_context


def _err_word(device: torch.device) -> torch.Tensor:
    return Workspace.get(device, 256, name="attention")[:4].view(torch.int32)


def device_error(device: torch.device) -> int:
    """First error code a paged-attention / K-V store kernel recorded on this device since the last reset
    (synchronises): 0 none, 2 row metadata inconsistent with the block table width, 3 a slot past the cache,
    11-17 a bounded pipeline wait gave up."""
    return int(_err_word(device).item())


def reset_device_error(device: torch.device) -> None:
    """Clears the error word and the split-item counters (a launch that gave up may leave counters behind)."""
    _err_word(device).zero_()
    Workspace.get(device, _SPLIT_MIN_BYTES, name="attention_split").zero_()


# Split-item workspace of the persistent attention kernel (arrival counters + two piece slots per SM), shared by
# every launch on the device; allocated once at a size covering R * Hkv up to ~1.3M so that a captured CUDA graph
# keeps a valid pointer.
_SPLIT_MIN_BYTES = 8 << 20


def _split_workspace(device: torch.device, R: int, Hkv: int, name: str = "attention_split") -> torch.Tensor:
    with torch.cuda.device(device):
        need = int(_lib.lib().specdec_attention_workspace_bytes(R, Hkv))
    if need < 0:
        raise _lib.SpecdecError(_lib.lib().specdec_last_error().decode())
    return Workspace.get(device, max(need, _SPLIT_MIN_BYTES), name=name)


def store_kvcache(key: torch.Tensor, value: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                  slot_mapping: torch.Tensor) -> None:
    """attention.py:33-40: key/value [N, Hkv, D] rows to slot_mapping[N] of the paged caches; slot -1 skipped."""
    device = require_cuda(key, value, k_cache, v_cache, slot_mapping)
    N, num_heads, head_dim = key.shape
    assert key.stride(-1) == 1 and value.stride(-1) == 1
    assert key.stride(1) == head_dim and value.stride(1) == head_dim
    assert slot_mapping.numel() == N
    if key.dtype != torch.bfloat16 or k_cache.dtype != torch.bfloat16:
        raise ValueError("the B200 K/V store takes bf16 keys, values and caches")
    slots = slot_mapping.to(torch.int32).contiguous()
    num_slots = k_cache.numel() // (num_heads * head_dim)
    check(_lib.lib().specdec_store_kvcache(ptr(key), key.stride(0), ptr(value), value.stride(0), ptr(k_cache),
                                           ptr(v_cache), ptr(slots), N, num_heads, head_dim, num_slots,
                                           ptr(_err_word(device)), stream_of(device)))


EARLY_LAUNCH = 1   # SPECDEC_ATTN_EARLY_LAUNCH
CTAS_SHIFT = 8     # SPECDEC_ATTN_CTAS_SHIFT: bits 8..15 of the flags cap the persistent grid


def _row_metadata(block_tables, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, context_lens, query_len_per_seq):
    tables = block_tables.to(torch.int32).contiguous()
    if cu_seqlens_q is not None:
        if max_seqlen_q is None:
            raise ValueError("varlen attention needs max_seqlen_q")
        cq = cu_seqlens_q.to(torch.int32).contiguous()
        ck = cu_seqlens_k.to(torch.int32).contiguous()
        return tables, cq, ck, None, cq.numel() - 1, 0, int(max_seqlen_q)
    ctx = context_lens.to(torch.int32).contiguous()
    return tables, None, None, ctx, ctx.numel(), query_len_per_seq, query_len_per_seq


def _output(out: torch.Tensor | None, shape, device: torch.device) -> torch.Tensor:
    """out itself after checking it is a bf16 [T, H, D] tensor on `device` with dense heads (rows may be strided),
    or a new one."""
    T, H, D = shape
    if out is None:
        return torch.empty(T, H, D, dtype=torch.bfloat16, device=device)
    if (out.shape != (T, H, D) or out.dtype != torch.bfloat16 or out.device != device or out.stride(2) != 1
            or out.stride(1) != D):
        raise ValueError(f"out must be a bf16 [{T}, {H}, {D}] tensor on {device} with dense heads "
                         f"(got {out.dtype} {tuple(out.shape)} strides {out.stride()})")
    return out


def paged_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, block_tables: torch.Tensor,
                    scale: float, *, cu_seqlens_q: torch.Tensor | None = None,
                    cu_seqlens_k: torch.Tensor | None = None, max_seqlen_q: int | None = None,
                    context_lens: torch.Tensor | None = None, query_len_per_seq: int = 1, causal: bool = True,
                    out: torch.Tensor | None = None, early_launch: bool = False, max_ctas: int = 0,
                    workspace: str = "attention_split") -> torch.Tensor:
    """Attention of q [T, H, D] over the paged caches.  Varlen (cu_seqlens_q/k, the verify forward) or decode
    (context_lens with query_len_per_seq queries per row).  Returns out [T, H, D] bf16.  early_launch: launch as a
    programmatic dependent of the preceding kernel (its prologue overlaps that kernel's end); only when that kernel
    does not write the row metadata (cu_seqlens / context_lens / block_tables).  max_ctas (1..255, 0 = one per SM):
    cap the persistent grid, leaving SMs to work on another stream.  workspace: the name of the split-item
    workspace; launches that may run at the same time on different streams need different names."""
    device = require_cuda(q, k_cache, v_cache, block_tables)
    out = _output(out, q.shape, device)
    paged_attention_to(q, k_cache, v_cache, block_tables, scale, [out.data_ptr()], out.stride(0),
                       cu_seqlens_q=cu_seqlens_q, cu_seqlens_k=cu_seqlens_k, max_seqlen_q=max_seqlen_q,
                       context_lens=context_lens, query_len_per_seq=query_len_per_seq, causal=causal,
                       early_launch=early_launch, max_ctas=max_ctas, workspace=workspace)
    return out


def paged_attention_to(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, block_tables: torch.Tensor,
                       scale: float, out_ptrs: list[int], out_row_stride: int, *,
                       cu_seqlens_q: torch.Tensor | None = None, cu_seqlens_k: torch.Tensor | None = None,
                       max_seqlen_q: int | None = None, context_lens: torch.Tensor | None = None,
                       query_len_per_seq: int = 1, causal: bool = True, early_launch: bool = False,
                       max_ctas: int = 0, workspace: str = "attention_split") -> None:
    """paged_attention writing its [T, H, D] bf16 output to every device address in out_ptrs (1 to 8; this GPU's
    memory or a peer's mapped into this process), all with row stride out_row_stride elements.  The caller owns
    the destinations' extent: each must hold T rows of out_row_stride elements from its address."""
    device = require_cuda(q, k_cache, v_cache, block_tables)
    T, H, D = q.shape
    blocks, block_size, Hkv, Dc = k_cache.shape
    if Dc != D or v_cache.shape != k_cache.shape:
        raise ValueError("q, k_cache and v_cache disagree on head_dim or shape")
    if not 1 <= len(out_ptrs) <= 8 or out_row_stride < H * D:
        raise ValueError(f"{len(out_ptrs)} destinations with row stride {out_row_stride}: 1 to 8, stride >= H * D")
    if q.stride(-1) != 1 or q.stride(1) != D:
        q = q.contiguous()
    tables, cq, ck, ctx, R, q_per_seq, max_q = _row_metadata(block_tables, cu_seqlens_q, cu_seqlens_k, max_seqlen_q,
                                                              context_lens, query_len_per_seq)
    W = tables.shape[1]
    if not 0 <= max_ctas <= 255:
        raise ValueError(f"max_ctas {max_ctas}: 0 (one CTA per SM) to 255")
    ws = _split_workspace(device, R, Hkv, workspace)
    flags = (EARLY_LAUNCH if early_launch else 0) | (max_ctas << CTAS_SHIFT)
    if len(out_ptrs) == 1:
        check(_lib.lib().specdec_paged_attention_ex(
            ptr(q), T, q.stride(0), H, Hkv, D, ptr(k_cache), ptr(v_cache), blocks * block_size, block_size, ptr(cq),
            ptr(ck), ptr(ctx), q_per_seq, R, ptr(tables), W, max_q, float(scale), int(causal), out_ptrs[0],
            out_row_stride, ptr(ws), ws.numel(), ptr(_err_word(device)), flags, stream_of(device)))
        return
    outs = (ctypes.c_void_p * len(out_ptrs))(*out_ptrs)
    check(_lib.lib().specdec_paged_attention_multi(
        ptr(q), T, q.stride(0), H, Hkv, D, ptr(k_cache), ptr(v_cache), blocks * block_size, block_size, ptr(cq),
        ptr(ck), ptr(ctx), q_per_seq, R, ptr(tables), W, max_q, float(scale), int(causal), outs, len(out_ptrs),
        out_row_stride, ptr(ws), ws.numel(), ptr(_err_word(device)), flags, stream_of(device)))


class Attention(nn.Module):
    """attention.py:43-77: paged attention over this layer's k_cache / v_cache (bound by the model runner)."""

    def __init__(self, num_heads, head_dim, scale, num_kv_heads):
        super().__init__()
        self.num_heads = num_heads
        self.head_dim = head_dim
        self.scale = scale
        self.num_kv_heads = num_kv_heads
        self.k_cache = self.v_cache = torch.tensor([])

    def forward(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, out: torch.Tensor | None = None
                ) -> torch.Tensor:
        """The reference's forward(q, k, v); out optionally names the [T, H, D] bf16 tensor to write (rows may be
        strided)."""
        q = q.view(-1, self.num_heads, self.head_dim)
        out = _output(out, q.shape, q.device)
        self.forward_to(q, k, v, [out.data_ptr()], out.stride(0))
        return out

    def forward_to(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, out_ptrs: list[int],
                   out_row_stride: int) -> None:
        """forward writing the output to every address in out_ptrs (see paged_attention_to): the store of k / v
        into this layer's caches at the context's slot_mapping, then the paged branch the context selects."""
        context = get_context()
        k_cache, v_cache = self.k_cache, self.v_cache
        if k_cache.numel() and v_cache.numel():
            store_kvcache(k, v, k_cache, v_cache, context.slot_mapping)
        q = q.view(-1, self.num_heads, self.head_dim)
        if context.is_prefill:
            if context.block_tables is None:
                raise NotImplementedError("prefill without a block table is outside the B200 verify/accept path")
            paged_attention_to(q, k_cache, v_cache, context.block_tables, self.scale, out_ptrs, out_row_stride,
                               cu_seqlens_q=context.cu_seqlens_q, cu_seqlens_k=context.cu_seqlens_k,
                               max_seqlen_q=context.max_seqlen_q, causal=True)
        else:
            paged_attention_to(q, k_cache, v_cache, context.block_tables, self.scale, out_ptrs, out_row_stride,
                               context_lens=context.context_lens, query_len_per_seq=context.query_len_per_seq,
                               causal=context.causal)
