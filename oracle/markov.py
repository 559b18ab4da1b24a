"""numpy restatement of DSpark's in-block Markov sampling -- test infrastructure only.

DFlashDrafter._markov_rows   nanovllm/engine/speculative.py:163-184
num_candidates               nanovllm/engine/speculative.py:46-50   (max_top_k + TIE_MARGIN(64) when every row
                             truncates, else 0 = the whole vocabulary)
MarkovHead                   nanovllm/models/dflash.py:26-41         (bias = W2 . W1[prev]; here any bias(prev))

Candidate order: descending value, ties by ascending token id.  torch.topk leaves the order of equal values
unspecified; the order decides which noise value (noise[:, row, c] belongs to the c-th candidate) a tied token
meets, so this restatement fixes the order and the kernels follow it.
"""
from __future__ import annotations

import numpy as np

from .spec_sampler import probs_from_logits, race

TIE_MARGIN = 64


def num_candidates(max_top_k: int, all_top_k: bool, vocab_size: int) -> int:
    """speculative.py:46-50."""
    return min(max_top_k + TIE_MARGIN, vocab_size) if all_top_k else 0


def top_candidates(row_logits: np.ndarray, count: int) -> np.ndarray:
    """Indices of each row's `count` largest values, descending, ties by ascending index."""
    order = np.argsort(-row_logits, axis=-1, kind="stable")
    return order[..., :count]


def markov_rows(logits: np.ndarray, prev: np.ndarray, bias_fn, sampling: dict | None, noise: np.ndarray | None,
                candidates: int, round_fn=lambda x: x):
    """speculative.py:163-184.  logits [B, k, V] (values); bias_fn(prev [B]) -> [B, V]; sampling = dict(temps,
    top_k, top_p, max_top_k, has_top_p) or None for greedy; noise [B, k, C or V]; round_fn rounds the biased
    logits to the logits' dtype (bf16 in the drafter).  Returns drafts [B, k] and q [B, k, V] (None if greedy)."""
    batch, k, vocab = logits.shape
    drafts = np.zeros((batch, k), dtype=np.int64)
    draft_probs = None if sampling is None else np.zeros((batch, k, vocab), dtype=np.float32)
    prev = np.asarray(prev, dtype=np.int64)
    rows = np.arange(batch)
    for row in range(k):
        row_logits = round_fn(logits[:, row].astype(np.float32) + bias_fn(prev).astype(np.float32))   # :173
        if sampling is None:
            prev = np.argmax(row_logits, axis=-1)                                                          # :175
        elif candidates:
            ids = top_candidates(row_logits, candidates)                                                   # :177
            values = np.take_along_axis(row_logits, ids, axis=-1)
            probs = probs_from_logits(values, sampling["temps"], sampling["top_k"], sampling["top_p"],
                                      sampling["max_top_k"], sampling["has_top_p"])                        # :178
            prev = ids[rows, race(probs, noise[:, row, :candidates])]                                     # :179
            draft_probs[rows[:, None], row, ids] = probs                                                   # :180
        else:
            probs = probs_from_logits(row_logits, sampling["temps"], sampling["top_k"], sampling["top_p"],
                                      sampling["max_top_k"], sampling["has_top_p"])                        # :182
            draft_probs[:, row] = probs
            prev = race(probs, noise[:, row])                                                             # :183
        drafts[:, row] = prev
    return drafts, draft_probs
