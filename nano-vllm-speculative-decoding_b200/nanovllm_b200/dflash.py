"""DFlash / DSpark draft context store (kernel 4, "ctx_store") on libspecdec_b200.so.

Reference: DFlashDraftModel.store_context_kv (nanovllm/models/dflash.py:88-96), called by
DFlashDrafter.after_verify (nanovllm/engine/speculative.py:326-337) for every verified position:

    for layer in draft layers:
        k, v = F.linear(features, W_kv[layer]).split(...)
        k = RoPE(positions, k_norm[layer](k))
        store_kvcache(k, v, kv_cache[0, layer], kv_cache[1, layer], slot_mapping)

store_context_kv projects with one cuBLAS GEMM against the layers' stacked W_kv and then runs every layer's
k_norm + RoPE + paged scatter of K and V as one kernel over (token, layer, head) rows (specdec_norm_rope_store with
no query heads); slot -1 rows (padding) are skipped.  context_features (dflash.py:84-86, hidden_norm(fc(aux))) is
the cuBLAS fc GEMM then this library's RMSNorm; after_verify chains the two.  store_context_kv_fused and
context_gemm run the same projections on this library's tcgen05 stream-K GEMM (the former with the norm / RoPE /
store epilogue); both are verified against the oracle but slower than the cuBLAS path on these shapes.
"""
from __future__ import annotations

import torch

from . import _lib
from ._lib import check, ptr, require_cuda, stream_of
from .fused import err_word
from .fused import rmsnorm as fused_rmsnorm


CONTEXT_GEMM_MAX_TOKENS = 288


def context_gemm(x: torch.Tensor, w: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """x [T, K] bf16 . w [O, K]^T -> [T, O] bf16 on this library's tcgen05 stream-K kernel (fp32 accumulation,
    one rounding, deterministic); tokens go through in calls of at most 288.  Measured slower than cuBLAS on the
    draft's shapes (the split tiles' fp32 pieces dominate), so the production path keeps cuBLAS."""
    device = require_cuda(x, w, out)
    if x.dtype != torch.bfloat16 or w.dtype != torch.bfloat16:
        raise ValueError("the context GEMM takes bf16 operands")
    T, K = x.shape
    O = w.shape[0]
    if x.stride(1) != 1 or w.stride(1) != 1:
        raise ValueError("rows must be contiguous")
    if out is None:
        out = torch.empty(T, O, dtype=torch.bfloat16, device=device)
    lib = _lib.lib()
    with torch.cuda.device(device):
        need = int(lib.specdec_context_gemm_workspace_bytes(min(T, CONTEXT_GEMM_MAX_TOKENS), O))
    if need < 0:
        raise _lib.SpecdecError(lib.specdec_last_error().decode())
    ws = _lib.Workspace.get(device, need, name="context_gemm")
    for t0 in range(0, T, CONTEXT_GEMM_MAX_TOKENS):
        n = min(CONTEXT_GEMM_MAX_TOKENS, T - t0)
        check(lib.specdec_context_gemm(ptr(x[t0:]), x.stride(0), ptr(w), w.stride(0), n, O, K, ptr(out[t0:]),
                                       out.stride(0), ptr(ws), ws.numel(), ptr(err_word(device)),
                                       stream_of(device)))
    return out


def context_features(aux: torch.Tensor, w_fc: torch.Tensor, norm_weight: torch.Tensor, eps: float, *,
                     fc_out: torch.Tensor | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
    """DFlashDraftModel.context_features (dflash.py:84-86): hidden_norm(fc(aux)).  aux [T, len(aux layers) * H]
    bf16, w_fc [H, len(aux layers) * H] bf16, norm_weight [H]; returns the normalised features [T, H] bf16.  The fc
    projection is a cuBLAS GEMM (faster here than this library's context_gemm), the RMSNorm this library's kernel."""
    require_cuda(aux, w_fc, norm_weight)
    x = torch.matmul(aux, w_fc.t(), out=fc_out)
    return fused_rmsnorm(x, norm_weight, eps, out=out)


def store_context_kv_fused(features: torch.Tensor, w_kv_stacked: torch.Tensor, k_norm: torch.Tensor,
                           cos_sin: torch.Tensor, positions: torch.Tensor, slot_mapping: torch.Tensor,
                           kv_cache: torch.Tensor, eps: float) -> None:
    """store_context_kv (dflash.py:88-96) as one tcgen05 kernel: the stacked W_kv projection with the k_norm,
    RoPE and paged store in its epilogue (the projection never goes to memory).  Arguments as store_context_kv.
    Correct, but measured ~9x slower than store_context_kv at T = 288 (its per-16-token epilogue and the split
    tiles' merges are latency-bound), so the production path keeps store_context_kv."""
    device = require_cuda(features, w_kv_stacked, k_norm, cos_sin, positions, slot_mapping, kv_cache)
    T, hidden = features.shape
    _, layers, blocks, block_size, num_kv_heads, head_dim = kv_cache.shape
    if head_dim != 128 or k_norm.shape != (layers, 128):
        raise ValueError("ctx_store expects 128-dim heads and one k_norm row per layer")
    if w_kv_stacked.shape != (layers * 2 * num_kv_heads * 128, hidden):
        raise ValueError(f"stacked W_kv of shape {tuple(w_kv_stacked.shape)} does not match the cache")
    if features.dtype != torch.bfloat16 or w_kv_stacked.dtype != torch.bfloat16:
        raise ValueError("the fused context store takes bf16 features and weights")
    features = features.contiguous()
    k_norm = k_norm.contiguous()
    positions = positions.to(torch.int64).contiguous()
    slots = slot_mapping.to(torch.int32).contiguous()
    k_cache, v_cache = kv_cache[0], kv_cache[1]
    O = layers * 2 * num_kv_heads * 128
    lib = _lib.lib()
    with torch.cuda.device(device):
        need = int(lib.specdec_context_gemm_workspace_bytes(min(T, CONTEXT_GEMM_MAX_TOKENS), O))
    if need < 0:
        raise _lib.SpecdecError(lib.specdec_last_error().decode())
    ws = _lib.Workspace.get(device, need, name="context_gemm")
    for t0 in range(0, T, CONTEXT_GEMM_MAX_TOKENS):
        n = min(CONTEXT_GEMM_MAX_TOKENS, T - t0)
        check(lib.specdec_context_kv_store(
            ptr(features[t0:]), features.stride(0), ptr(w_kv_stacked), w_kv_stacked.stride(0), n, layers,
            num_kv_heads, hidden, ptr(k_norm), k_norm.stride(0), ptr(cos_sin), cos_sin.shape[0], ptr(positions[t0:]),
            ptr(slots[t0:]), ptr(k_cache), ptr(v_cache), k_cache.stride(0), blocks * block_size, float(eps), ptr(ws),
            ws.numel(), ptr(err_word(device)), stream_of(device)))


def after_verify(aux: torch.Tensor, w_fc: torch.Tensor, norm_weight: torch.Tensor, w_kv_stacked: torch.Tensor,
                 k_norm: torch.Tensor, cos_sin: torch.Tensor, positions: torch.Tensor, slot_mapping: torch.Tensor,
                 kv_cache: torch.Tensor, eps: float, *, buffers: dict | None = None) -> None:
    """DFlashDrafter.after_verify's device work (speculative.py:326-337 -> dflash.py:84-96): the context features
    of every verified position from the aux layers the verification exported, then every draft layer's context
    K/V at slot_mapping.  buffers (optional, e.g. for CUDA graph capture): preallocated "fc" and "features" [T, H]
    and "kv" [T, L * 2 * Hkv * 128] bf16."""
    buffers = buffers or {}
    features = context_features(aux, w_fc, norm_weight, eps, fc_out=buffers.get("fc"), out=buffers.get("features"))
    store_context_kv(features, w_kv_stacked, k_norm, cos_sin, positions, slot_mapping, kv_cache, eps,
                     kv_out=buffers.get("kv"))


def stacked_kv_weight(layer_kv_weights: list[torch.Tensor]) -> torch.Tensor:
    """[layers * 2 * Hkv * 128, hidden]: each draft layer's K then V rows of its packed qkv_proj
    (qkv_proj.weight[q_size:] in dflash.py:92), stacked so one GEMM projects every layer."""
    return torch.cat(layer_kv_weights, dim=0).contiguous()


def store_context_kv(features: torch.Tensor, w_kv_stacked: torch.Tensor, k_norm: torch.Tensor,
                     cos_sin: torch.Tensor, positions: torch.Tensor, slot_mapping: torch.Tensor,
                     kv_cache: torch.Tensor, eps: float, *, kv_out: torch.Tensor | None = None) -> None:
    """dflash.py:88-96 for all layers.  features [T, hidden] bf16; w_kv_stacked [L * 2 * Hkv * 128, hidden];
    k_norm [L, 128] bf16; cos_sin [max_position, 128] fp32; positions [T] int64; slot_mapping [T] int32;
    kv_cache [2, L, blocks, block_size, Hkv, 128] bf16 (the drafter's cache, sharing the target's block ids)."""
    device = require_cuda(features, w_kv_stacked, k_norm, cos_sin, positions, slot_mapping, kv_cache)
    T = features.shape[0]
    _, layers, blocks, block_size, num_kv_heads, head_dim = kv_cache.shape
    if head_dim != 128 or k_norm.shape != (layers, 128):
        raise ValueError("ctx_store expects 128-dim heads and one k_norm row per layer")
    width = 2 * num_kv_heads * head_dim
    if w_kv_stacked.shape[0] != layers * width:
        raise ValueError(f"stacked W_kv has {w_kv_stacked.shape[0]} rows, expected {layers * width}")
    kv = torch.matmul(features, w_kv_stacked.t(), out=kv_out)        # [T, L * 2 * Hkv * 128] (cuBLAS)
    k_cache, v_cache = kv_cache[0], kv_cache[1]
    num_slots = blocks * block_size
    check(_lib.lib().specdec_norm_rope_store(
        ptr(kv), width, kv.stride(0), T, layers, 0, num_kv_heads, None, ptr(k_norm.contiguous()), 128,
        ptr(cos_sin), cos_sin.shape[0], ptr(positions), ptr(slot_mapping.to(torch.int32)), ptr(k_cache),
        ptr(v_cache), k_cache.stride(0), num_slots, None, float(eps), ptr(err_word(device)), stream_of(device)))


class DFlashDraftModel:
    """DFlashDraftModel (nanovllm/models/dflash.py:55-115) with random-initialised weights (no checkpoints here):
    embed_tokens, Qwen3 decoder layers, the final norm and LM head, the context projection fc + hidden_norm, and
    DSpark's Markov head (markov_w1 / markov_w2 of rank markov_rank; 0 = DFlash, no head).  Its paged KV cache
    [2, layers, blocks + 1, block_size, Hkv, 128] shares the target's block ids and pad block
    (speculative.py:80-91).

    forward runs a draft block: every row's anchor and mask tokens through the layers, each layer storing the
    block's K/V at slot_mapping and attending, non-causally, to the context below the anchor and the whole block
    (the decode branch of the paged attention with query_len_per_seq = block length, causal off)."""

    def __init__(self, shape, aux_layer_ids: tuple[int, ...], device: torch.device, num_blocks: int,
                 block_size: int = 256, markov_rank: int = 256, mask_token_id: int = 151669, seed: int = 1,
                 init_scale: float = 0.02, markov_scale: float = 0.1):
        from .target import random_layer_weights
        self.shape = s = shape
        self.device = device
        self.aux_layer_ids = tuple(aux_layer_ids)
        self.aux_width = len(self.aux_layer_ids) * s.hidden
        self.mask_token_id = mask_token_id
        self.block_size = block_size
        g = torch.Generator(device=device).manual_seed(seed)
        bf = torch.bfloat16

        def rand(*dims, scale=init_scale):
            return (torch.randn(*dims, device=device, generator=g, dtype=torch.float32) * scale).to(bf)

        def norm_weight(n):
            return (1.0 + 0.05 * torch.randn(n, device=device, generator=g)).to(bf)

        self.embed = rand(s.vocab, s.hidden)
        self.layers = [random_layer_weights(s, rand, norm_weight) for _ in range(s.layers)]
        self.final_norm = norm_weight(s.hidden)
        self.lm_head = rand(s.vocab, s.hidden)
        self.w_fc = rand(s.hidden, self.aux_width, scale=init_scale / 2)
        self.hidden_norm = norm_weight(s.hidden)
        q_rows = s.heads * s.head_dim
        # each layer's W_k | W_v rows (qkv_proj.weight[q_size:], dflash.py:92), stacked for one projection GEMM
        self.w_kv = stacked_kv_weight([w["w_qkv"][q_rows:] for w in self.layers])
        self.k_norm = torch.stack([w["k_norm"] for w in self.layers]).contiguous()
        self.markov_head = None
        if markov_rank:
            from .markov import MarkovHeadWeights
            self.markov_head = MarkovHeadWeights(rand(s.vocab, markov_rank, scale=markov_scale),
                                                 rand(s.vocab, markov_rank, scale=markov_scale))
        self.kv_cache = torch.zeros(2, s.layers, num_blocks + 1, block_size, s.kv_heads, s.head_dim, dtype=bf,
                                    device=device)
        from .fused import rope_cache
        self.cos_sin = rope_cache(s.head_dim, s.max_position, s.rope_theta, device)
        self.scale = s.head_dim ** -0.5

    def forward(self, input_ids: torch.Tensor, positions: torch.Tensor, slot_mapping: torch.Tensor,
                context_lens: torch.Tensor, block_tables: torch.Tensor, query_len: int) -> torch.Tensor:
        """dflash.py:98-105 over block rows, sequence-major ([B * query_len]): hidden states after the final norm."""
        from . import attention
        from .target import decoder_layer
        s = self.shape

        def attend(q, layer_id):
            return attention.paged_attention(q, self.kv_cache[0, layer_id], self.kv_cache[1, layer_id], block_tables,
                                             self.scale, context_lens=context_lens, query_len_per_seq=query_len,
                                             causal=False, early_launch=True)

        h = torch.nn.functional.embedding(input_ids, self.embed)
        residual = None
        for layer_id, w in enumerate(self.layers):
            h, residual = decoder_layer(s, w, layer_id, h, residual, positions, slot_mapping, self.kv_cache,
                                        self.cos_sin, attend)
        h, _ = fused_rmsnorm(h, self.final_norm, s.eps, residual=residual)
        return h

    def compute_logits(self, hidden: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """dflash.py:107-108: [rows, vocab] bf16 over every row."""
        return torch.matmul(hidden, self.lm_head.t(), out=out)

    def context_features(self, aux: torch.Tensor, *, fc_out: torch.Tensor | None = None,
                         out: torch.Tensor | None = None) -> torch.Tensor:
        """dflash.py:84-86: hidden_norm(fc(aux))."""
        return context_features(aux, self.w_fc, self.hidden_norm, self.shape.eps, fc_out=fc_out, out=out)

    def store_context_kv(self, features: torch.Tensor, positions: torch.Tensor, slot_mapping: torch.Tensor, *,
                         kv_out: torch.Tensor | None = None) -> None:
        """dflash.py:88-96: every layer's context K/V of the features at slot_mapping (slot -1 skipped)."""
        store_context_kv(features, self.w_kv, self.k_norm, self.cos_sin, positions, slot_mapping, self.kv_cache,
                         self.shape.eps, kv_out=kv_out)
