"""The reference's attention context (nanovllm/utils/context.py:5-31): a module-global record of the current
forward's paged-attention metadata, set by the runner before a forward and read by Attention.forward."""
from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass(slots=True)
class Context:
    is_prefill: bool = False
    cu_seqlens_q: torch.Tensor | None = None
    cu_seqlens_k: torch.Tensor | None = None
    max_seqlen_q: int = 0
    max_seqlen_k: int = 0
    slot_mapping: torch.Tensor | None = None
    context_lens: torch.Tensor | None = None
    block_tables: torch.Tensor | None = None
    query_len_per_seq: int = 1    # query rows per sequence in the decode branch (k for a draft block)
    causal: bool = True           # False lets every query row see every key of its block (the draft block)


_CONTEXT = Context()


def get_context() -> Context:
    return _CONTEXT


def set_context(is_prefill, cu_seqlens_q=None, cu_seqlens_k=None, max_seqlen_q=0, max_seqlen_k=0, slot_mapping=None,
                context_lens=None, block_tables=None, query_len_per_seq=1, causal=True) -> None:
    global _CONTEXT
    _CONTEXT = Context(is_prefill, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k, slot_mapping, context_lens,
                       block_tables, query_len_per_seq, causal)


def reset_context() -> None:
    global _CONTEXT
    _CONTEXT = Context()
