"""A Qwen3-architecture target for the verify forward of a speculative round, on B200.

Mirrors the reference's target model and verification (nano-vllm-speculative-decoding):
    Qwen3DecoderLayer / Qwen3Model.forward     nanovllm/models/qwen3.py:133-213  (aux-layer export :174-191)
    compute_logits (all positions)             nanovllm/models/qwen3.py:221-226
    SpeculativeDecoder.verify_logits / graphs  nanovllm/engine/speculative.py:471-582
    verify_varlen_metadata                     nanovllm/engine/batch_metadata.py:149-181

The projections and the LM head are plain cuBLAS GEMMs (torch.matmul); everything between them runs on this
package's kernels: RMSNorm(+residual), q/k norm + RoPE + paged K/V store, paged verify attention (kernel 2) and
SiLU*mul.  Weights are random-initialised (no checkpoints here); the paged KV cache is [2, layers, blocks + 1,
block_size, Hkv, 128] with the last block the zeroed pad block, as ModelRunner.allocate_kv_cache lays it out
(nanovllm/engine/model_runner.py:142-169).  A whole verification (forward + logits) is captured as one CUDA
graph per token count, replayed with the round's metadata copied into its static buffers.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from . import attention, fused


@dataclass
class Qwen3Shape:
    hidden: int = 4096
    layers: int = 36
    heads: int = 32
    kv_heads: int = 8
    head_dim: int = 128
    intermediate: int = 12288
    vocab: int = 151936
    eps: float = 1e-6
    rope_theta: float = 1000000.0
    max_position: int = 40960
    aux_layer_ids: tuple[int, ...] = (1, 9, 17, 25, 33)    # DSpark / DFlash Qwen3-8B target_layer_ids


def random_layer_weights(s: Qwen3Shape, rand, norm_weight) -> dict:
    """One Qwen3DecoderLayer's weights (qwen3.py:120-145): packed qkv_proj, o_proj, packed gate_up_proj, down_proj,
    the two RMSNorm weights and the per-head q_norm / k_norm."""
    qkv_rows = (s.heads + 2 * s.kv_heads) * s.head_dim
    return dict(w_qkv=rand(qkv_rows, s.hidden), w_o=rand(s.hidden, s.heads * s.head_dim),
                w_gate_up=rand(2 * s.intermediate, s.hidden), w_down=rand(s.hidden, s.intermediate),
                in_norm=norm_weight(s.hidden), post_norm=norm_weight(s.hidden),
                q_norm=norm_weight(s.head_dim), k_norm=norm_weight(s.head_dim))


def decoder_layer(s: Qwen3Shape, w: dict, layer_id: int, h: torch.Tensor, residual: torch.Tensor | None,
                  positions: torch.Tensor, slot_mapping: torch.Tensor, kv_cache: torch.Tensor,
                  cos_sin: torch.Tensor, attend) -> tuple[torch.Tensor, torch.Tensor]:
    """Qwen3DecoderLayer.forward (qwen3.py:147-160) on this package's kernels: input RMSNorm (+residual), the
    qkv GEMM, q/k norm + RoPE with the K/V rows stored at slot_mapping into layer `layer_id` of kv_cache, then
    attend(q, layer_id) (the paged branch the caller picks: varlen verify or the draft block), o_proj, the
    post-attention RMSNorm and the SiLU-gated MLP.  Returns (hidden, residual) like the reference's layer."""
    T = h.shape[0]
    if residual is None:
        x, residual = fused.rmsnorm(h, w["in_norm"], s.eps), h
    else:
        x, residual = fused.rmsnorm(h, w["in_norm"], s.eps, residual=residual)
    qkv = torch.matmul(x, w["w_qkv"].t())
    q = fused.qk_norm_rope_store(qkv, s.heads, s.kv_heads, w["q_norm"], w["k_norm"], cos_sin, positions,
                                 slot_mapping, kv_cache[0, layer_id], kv_cache[1, layer_id], s.eps)
    o = attend(q, layer_id)
    h = torch.matmul(o.view(T, -1), w["w_o"].t())
    x, residual = fused.rmsnorm(h, w["post_norm"], s.eps, residual=residual)
    h = torch.matmul(fused.silu_and_mul(torch.matmul(x, w["w_gate_up"].t())), w["w_down"].t())
    return h, residual


class Qwen3Target:
    def __init__(self, shape: Qwen3Shape, device: torch.device, num_blocks: int, block_size: int = 256,
                 seed: int = 0, init_scale: float = 0.02):
        self.shape = s = shape
        self.device = device
        self.block_size = block_size
        self.num_blocks = num_blocks
        self.pad_block_id = num_blocks
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
        self.kv_cache = torch.zeros(2, s.layers, num_blocks + 1, block_size, s.kv_heads, s.head_dim, dtype=bf,
                                    device=device)
        self.cos_sin = fused.rope_cache(s.head_dim, s.max_position, s.rope_theta, device)
        self.scale = s.head_dim ** -0.5
        # error words / workspaces exist before any graph capture
        fused.err_word(device)
        attention.reset_device_error(device)
        self.graphs: dict[int, tuple[torch.cuda.CUDAGraph, dict]] = {}
        self.graph_pool = None

    # ------------------------------------------------------------------ eager forward
    def forward(self, input_ids, positions, slot_mapping, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, block_tables,
                aux_out: torch.Tensor | None = None) -> torch.Tensor:
        """qwen3.py:201-213: hidden states [T, hidden] after the final norm; aux_out [T, 5 * hidden] receives the
        aux layers' outputs (hidden + residual, qwen3.py:186-190)."""
        s = self.shape

        def attend(q, layer_id):
            # launched early: its predecessor (the q/k norm, RoPE and K/V store) writes q and the caches only
            return attention.paged_attention(q, self.kv_cache[0, layer_id], self.kv_cache[1, layer_id], block_tables,
                                             self.scale, cu_seqlens_q=cu_seqlens_q, cu_seqlens_k=cu_seqlens_k,
                                             max_seqlen_q=max_seqlen_q, early_launch=True)

        h = torch.nn.functional.embedding(input_ids, self.embed)
        residual = None
        for layer_id, w in enumerate(self.layers):
            h, residual = decoder_layer(s, w, layer_id, h, residual, positions, slot_mapping, self.kv_cache,
                                        self.cos_sin, attend)
            if aux_out is not None and layer_id in s.aux_layer_ids:
                seg = s.aux_layer_ids.index(layer_id)
                aux_out[:, seg * s.hidden:(seg + 1) * s.hidden].copy_(h + residual)
        h, _ = fused.rmsnorm(h, self.final_norm, s.eps, residual=residual)
        return h

    def compute_logits(self, hidden: torch.Tensor) -> torch.Tensor:
        """qwen3.py:221-226 with all_logits: [T, vocab] bf16."""
        return torch.matmul(hidden, self.lm_head.t())

    # ------------------------------------------------------------------ graphs
    def static_buffers(self, num_rows: int, num_tokens: int, width: int) -> dict:
        """The graph's metadata inputs as views of one int64 and one int32 device buffer, so a round's metadata
        arrives in two host-to-device copies (batch_metadata.packed_views gives the layout)."""
        from .batch_metadata import packed_sizes, packed_views
        n64, n32 = packed_sizes(num_rows, num_tokens, width)
        packed64 = torch.zeros(n64, dtype=torch.int64, device=self.device)
        packed32 = torch.zeros(n32, dtype=torch.int32, device=self.device)
        buffers = packed_views(packed64, packed32, num_rows, num_tokens, width)
        buffers["slot_mapping"].fill_(-1)
        buffers["block_tables"].fill_(self.pad_block_id)
        buffers["_packed64"], buffers["_packed32"] = packed64, packed32
        return buffers

    def capture(self, num_rows: int, num_tokens: int, width: int, max_seqlen_q: int, load_padding,
                aux_width: int = 0, epilogue=None) -> dict:
        """Captures forward + logits for one (rows, tokens) shape; load_padding(buffers) fills a valid
        all-padding metadata first (speculative.py:559-571).  aux_width > 0: the forward also exports the aux
        layers' outputs into buffers["aux"] [num_tokens, aux_width] (speculative.py:547-549); epilogue(buffers),
        when given, is captured after the logits (the drafter's after_verify reads the aux buffer there).
        Returns the graph's buffers (with "logits")."""
        buffers = self.static_buffers(num_rows, num_tokens, width)
        if aux_width:
            buffers["aux"] = torch.zeros(num_tokens, aux_width, dtype=torch.bfloat16, device=self.device)
        load_padding(buffers)

        def body():
            hidden = self.forward(buffers["input_ids"], buffers["positions"], buffers["slot_mapping"],
                                  buffers["cu_seqlens_q"], buffers["cu_seqlens_k"], max_seqlen_q,
                                  buffers["block_tables"], aux_out=buffers.get("aux"))
            logits = self.compute_logits(hidden)
            if epilogue is not None:
                epilogue(buffers)
            return logits

        body()   # warm-up (also configures the kernels' shared-memory attributes)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, self.graph_pool):
            buffers["logits"] = body()
        if self.graph_pool is None:
            self.graph_pool = graph.pool()
        torch.cuda.synchronize()
        self.graphs[num_tokens] = (graph, buffers)
        return buffers

    def replay(self, num_tokens: int) -> torch.Tensor:
        graph, buffers = self.graphs[num_tokens]
        graph.replay()
        return buffers["logits"]

    def close(self) -> None:
        self.graphs.clear()
