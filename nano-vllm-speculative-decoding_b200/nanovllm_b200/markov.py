"""DSpark's in-block Markov sampling (kernel 3) on libspecdec_b200.so.

    markov_rows(logits, prev, sampling, noise, drafts, draft_probs, candidates, markov_head)

mirrors DFlashDrafter._markov_rows (nanovllm/engine/speculative.py:163-184) with the Markov head passed in:
k sequential steps, each `bias = markov_head(prev)` (for MarkovHeadWeights a cuBLAS GEMM of the W1 rows the
previous step's kernel gathered against W2) followed by ONE kernel launch that, for every batch row at once,
adds the bias, selects the top `candidates` logits (ties by ascending token id), applies the row's temperature /
top-k / top-p over them, races them against that row's noise, scatters q and gathers the next W1 rows.  With
fused_bias=True the bias GEMM is this library's tcgen05 kernel with the logits added in its epilogue
(specdec_markov_bias), and the selection reads the biased rows; verified, slower than cuBLAS here.  Greedy batches take the argmax.
Rows drawn over the whole vocabulary (candidates == 0: some row does not truncate) use the sampler's
probs_from_logits + race kernels.  drafts [B, k] and draft_probs [B, k, V] are written in place, as in the
reference; noise [B, k, candidates or V] is drawn by the caller before row 0 (speculative.py:156-159).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _lib, spec_sampler
from ._lib import DTYPE_CODES, Workspace, check, ptr, require_cuda, stream_of
from .fused import err_word

TIE_MARGIN = 64


def num_candidates(max_top_k: int, all_top_k: bool, vocab_size: int) -> int:
    """speculative.py:46-50: a row is drawn among its top max_top_k + 64 logits when every row truncates."""
    return min(max_top_k + TIE_MARGIN, vocab_size) if all_top_k else 0


@dataclass
class MarkovHeadWeights:
    """MarkovHead (nanovllm/models/dflash.py:26-41): markov_w1 [V, r] embeds the previous token, markov_w2 [V, r]
    projects it to a bias over the vocabulary."""
    w1: torch.Tensor
    w2: torch.Tensor

    def embed(self, prev: torch.Tensor) -> torch.Tensor:
        return self.w1[prev]

    def __call__(self, prev: torch.Tensor) -> torch.Tensor:
        return torch.matmul(self.embed(prev), self.w2.t())


def fused_bias_eligible(logits: torch.Tensor, weights) -> bool:
    """Whether a step's bias can come from specdec_markov_bias: a MarkovHeadWeights head and bf16 logits, the
    vocabulary a multiple of 128, the rank a multiple of 64 and at most 288 rows (the tensor-core GEMM's shape)."""
    if not isinstance(weights, MarkovHeadWeights):
        return False
    batch, _, vocab = logits.shape
    rank = weights.w2.shape[1]
    return (logits.dtype == torch.bfloat16 and weights.w1.dtype == torch.bfloat16 and weights.w2.dtype ==
            torch.bfloat16 and vocab % 128 == 0 and rank % 64 == 0 and batch <= 288 and weights.w2.stride(1) == 1
            and (weights.w2.stride(0) * 2) % 16 == 0)


def _bias_workspace(device: torch.device, batch: int, vocab: int) -> torch.Tensor:
    lib = _lib.lib()
    with torch.cuda.device(device):
        need = int(lib.specdec_context_gemm_workspace_bytes(batch, vocab))
    if need < 0:
        raise _lib.SpecdecError(lib.specdec_last_error().decode())
    return Workspace.get(device, need, name="markov_bias")


def markov_bias(w2: torch.Tensor, e: torch.Tensor, row_logits: torch.Tensor, out: torch.Tensor,
                workspace: torch.Tensor | None = None) -> torch.Tensor:
    """speculative.py:173 with MarkovHead (dflash.py:39-41): out [B, V] = bf16(bf16(e . w2^T) + row_logits), the
    bias GEMM on the tensor cores with the logits added in its epilogue.  e [B, rank] (the markov_w1 rows of the
    previous tokens), w2 [V, rank], row_logits [B, V] (rows may be strided), all bf16."""
    device = require_cuda(w2, e, row_logits, out)
    batch, rank = e.shape
    vocab = w2.shape[0]
    if row_logits.stride(1) != 1 or out.stride(1) != 1 or e.stride(1) != 1:
        raise ValueError("the Markov bias GEMM needs unit-stride rows")
    ws = workspace if workspace is not None else _bias_workspace(device, batch, vocab)
    check(_lib.lib().specdec_markov_bias(ptr(w2), w2.stride(0), ptr(e), e.stride(0), batch, vocab, rank,
                                         ptr(row_logits), row_logits.stride(0), ptr(out), out.stride(0), ptr(ws),
                                         ws.numel(), ptr(err_word(device)), stream_of(device)))
    return out


def _round_flag(logits: torch.Tensor, bias: torch.Tensor) -> int:
    if logits.dtype == torch.bfloat16 and bias.dtype == torch.bfloat16:
        return 1
    if logits.dtype == torch.float16 or bias.dtype == torch.float16:
        raise ValueError("fp16 Markov rows are not implemented (bf16 and fp32 are)")
    return 0


class MarkovQBuffer:
    """A persistent q buffer for markov_rows: probs [B, k, V] fp32 is zero except where each row scattered q on the
    previous call, recorded in ids [B, k, C] int32 (-1: none), so a call clears just those entries instead of
    zero-filling the whole buffer (the reference zero-fills a fresh [B, k, V] tensor every call,
    speculative.py:170-171).  Pass it as draft_probs; read q from .probs.  Tied to one (B, k, V, C)."""

    def __init__(self, batch: int, k: int, vocab: int, candidates: int, device: torch.device):
        if candidates < 1:
            raise ValueError("a persistent q buffer needs candidate rows (candidates >= 1)")
        self.probs = torch.zeros(batch, k, vocab, dtype=torch.float32, device=device)
        self.ids = torch.full((batch, k, candidates), -1, dtype=torch.int32, device=device)
        self.candidates = candidates

    def rows(self, batch: int) -> "MarkovQBuffer":
        """The same buffer's first `batch` rows (views), for a smaller padded batch."""
        view = object.__new__(MarkovQBuffer)
        view.probs, view.ids, view.candidates = self.probs[:batch], self.ids[:batch], self.candidates
        return view


def markov_rows(logits: torch.Tensor, prev: torch.Tensor, sampling, noise: torch.Tensor | None,
                drafts: torch.Tensor, draft_probs: torch.Tensor | None, candidates: int, markov_head, *,
                fused_bias: bool = False) -> None:
    """speculative.py:163-184: draw the k rows left to right into drafts (and q into draft_probs unless greedy);
    prev holds the anchors.  logits [B, k, V]; markov_head(prev [B]) -> bias [B, V].  fused_bias (MarkovHeadWeights,
    bf16, shapes as fused_bias_eligible): each step's bias from specdec_markov_bias with the logits added in the
    GEMM's epilogue; verified, but measured slower than the cuBLAS bias GEMM at config 4 (31 vs 17 us per step), so
    off by default."""
    device = require_cuda(logits, prev, drafts)
    batch, k, vocab = logits.shape
    logits = logits.contiguous()
    qbuf = None
    if isinstance(draft_probs, MarkovQBuffer):
        qbuf, draft_probs = draft_probs, draft_probs.probs
        if candidates != qbuf.candidates or tuple(draft_probs.shape) != (batch, k, vocab):
            raise ValueError("the persistent q buffer was made for another batch shape or candidate count")
    greedy = draft_probs is None
    if not greedy and candidates and qbuf is None:
        draft_probs.zero_()                     # q is zero outside each row's candidates (speculative.py:171)
    prev_buf = prev.to(torch.int64).clone(memory_format=torch.contiguous_format)   # the kernel writes it
    weights = markov_head if isinstance(markov_head, MarkovHeadWeights) else None
    e_buf = None
    if weights is not None:
        e_buf = weights.embed(prev_buf).contiguous()
    temps = top_k = top_p = None
    max_top_k = has_top_p = 0
    if not greedy:
        temps = sampling.temperatures.contiguous()
        top_k = sampling.top_k.contiguous()
        top_p = sampling.top_p.contiguous() if sampling.has_top_p else None
        max_top_k, has_top_p = sampling.max_top_k, int(sampling.has_top_p)
        noise = noise.float().contiguous()
    lib = _lib.lib()
    stream = stream_of(device)
    ws = None
    if greedy or candidates:
        with torch.cuda.device(device):
            need = int(lib.specdec_markov_workspace_bytes(batch, vocab, max(candidates, 1), int(greedy)))
        if need < 0:
            raise _lib.SpecdecError(lib.specdec_last_error().decode())
        ws = Workspace.get(device, need, name="markov")    # zeroed once; the kernel keeps its counters zeroed
    fused = fused_bias and (greedy or candidates) and fused_bias_eligible(logits, weights)
    if fused:
        # the bias GEMM with the logits added in its epilogue (one tcgen05 kernel per row), then the selection
        # reads the biased rows: the [B, V] bias is never written
        biased = torch.empty(batch, vocab, dtype=torch.bfloat16, device=device)
        gemm_ws = _bias_workspace(device, batch, vocab)
    for row in range(k):
        if fused:
            markov_bias(weights.w2, e_buf, logits[:, row], biased, gemm_ws)
            check(lib.specdec_markov_step(
                ptr(biased), DTYPE_CODES[torch.bfloat16], None, 0, batch, k, vocab, row, candidates, int(greedy), 1,
                ptr(temps), ptr(top_k), ptr(top_p), max_top_k, has_top_p, ptr(noise),
                0 if noise is None else noise.shape[-1], ptr(drafts), ptr(draft_probs), ptr(prev_buf), ptr(weights.w1),
                weights.w1.shape[1], ptr(e_buf), ptr(None if qbuf is None else qbuf.ids), ptr(ws), ws.numel(),
                ptr(err_word(device)), stream))
            continue
        bias = torch.matmul(e_buf, weights.w2.t()) if weights is not None else markov_head(prev_buf)
        bias = bias.contiguous()
        if greedy or candidates:
            check(lib.specdec_markov_step(
                ptr(logits), DTYPE_CODES[logits.dtype], ptr(bias), DTYPE_CODES[bias.dtype], batch, k, vocab, row,
                candidates, int(greedy), _round_flag(logits, bias), ptr(temps), ptr(top_k), ptr(top_p), max_top_k,
                has_top_p, ptr(noise), 0 if noise is None else noise.shape[-1], ptr(drafts), ptr(draft_probs),
                ptr(prev_buf), ptr(None if weights is None else weights.w1), 0 if weights is None else
                weights.w1.shape[1], ptr(e_buf), ptr(None if qbuf is None else qbuf.ids), ptr(ws), ws.numel(),
                ptr(err_word(device)), stream))
        else:
            row_logits = logits[:, row] + bias  # torch's dtype promotion and rounding, as the reference
            probs = spec_sampler.probs_from_logits(row_logits, sampling)
            draft_probs[:, row] = probs
            prev_buf = spec_sampler.race(probs, noise[:, row])
            drafts[:, row] = prev_buf
            if weights is not None:
                e_buf = weights.embed(prev_buf).contiguous()
