"""numpy restatement of the reference sampler (nanovllm/layers/spec_sampler.py) -- test infrastructure only.

All arithmetic is float32 like the reference's fp32 tensors; draws (u, E) are explicit inputs.
"""
from __future__ import annotations

import numpy as np

EXPONENTIAL_NOISE_FLOOR = np.float32(1e-10)   # spec_sampler.py:13


def _per_row(values: np.ndarray, ndim: int) -> np.ndarray:
    """spec_sampler.py:60-62: [B] -> broadcastable against ndim dims."""
    return values.reshape(values.shape[0], *([1] * (ndim - 1)))


def softmax(x: np.ndarray) -> np.ndarray:
    """torch.softmax over the last dim in fp32: exp(x - max) / sum."""
    x = x.astype(np.float32, copy=False)
    m = np.max(x, axis=-1, keepdims=True)
    with np.errstate(invalid="ignore", over="ignore"):
        e = np.exp((x - m).astype(np.float32)).astype(np.float32)
        return (e / np.sum(e, axis=-1, keepdims=True, dtype=np.float32)).astype(np.float32)


def truncate_logits(scaled: np.ndarray, top_k: np.ndarray, top_p: np.ndarray, max_top_k: int,
                    has_top_p: bool) -> np.ndarray:
    """spec_sampler.py:72-96: -inf outside each row's top-k (ties at the k-th value kept), then outside the
    top-p nucleus of those candidates; rows with top_k == 0 unchanged."""
    if max_top_k == 0:
        return scaled
    ndim = scaled.ndim
    tk = _per_row(top_k.astype(np.int64), ndim)
    effective_k = np.maximum(tk, 1)                                          # :82
    num_candidates = min(max_top_k, scaled.shape[-1])                        # :83
    candidates = -np.sort(-scaled, axis=-1)[..., :num_candidates]            # :84 topk values, descending
    ranks = np.arange(num_candidates)
    candidates = np.where(ranks >= effective_k, np.float32(-np.inf), candidates).astype(np.float32)   # :86
    k_index = np.minimum(effective_k - 1, num_candidates - 1)                # :87
    k_index = np.broadcast_to(k_index, (*candidates.shape[:-1], 1))
    threshold = np.take_along_axis(candidates, k_index, axis=-1)             # :88
    if has_top_p:
        nucleus = softmax(candidates)                                        # :90
        mass_before = (np.cumsum(nucleus, axis=-1, dtype=np.float32) - nucleus).astype(np.float32)   # :91
        num_kept = np.sum(mass_before < _per_row(top_p.astype(np.float32), ndim), axis=-1, keepdims=True)  # :92
        p_threshold = np.take_along_axis(candidates, num_kept - 1, axis=-1)  # :93
        threshold = np.maximum(threshold, p_threshold)                       # :94
    threshold = np.where(tk > 0, threshold, np.float32(-np.inf))             # :95
    return np.where(scaled < threshold, np.float32(-np.inf), scaled).astype(np.float32)   # :96


def probs_from_logits(logits: np.ndarray, temperatures: np.ndarray, top_k: np.ndarray | None = None,
                      top_p: np.ndarray | None = None, max_top_k: int = 0, has_top_p: bool = False) -> np.ndarray:
    """spec_sampler.py:65-69: softmax(truncate(logits.float() / T))."""
    scaled = (logits.astype(np.float32) / _per_row(temperatures.astype(np.float32), logits.ndim)).astype(np.float32)
    if top_k is None:
        top_k = np.zeros(logits.shape[0], dtype=np.int64)
    if top_p is None:
        top_p = np.ones(logits.shape[0], dtype=np.float32)
    return softmax(truncate_logits(scaled, top_k, top_p, max_top_k, has_top_p))


def clamp_noise(raw_exponential: np.ndarray) -> np.ndarray:
    """spec_sampler.py:99-101: Exp(1) noise clamped at 1e-10."""
    return np.maximum(raw_exponential.astype(np.float32), EXPONENTIAL_NOISE_FLOOR)


def race(weights: np.ndarray, noise: np.ndarray) -> np.ndarray:
    """spec_sampler.py:104-106: argmax(w / E) over the last dim, first index on ties."""
    ratio = (weights.astype(np.float32) / noise.astype(np.float32)).astype(np.float32)
    return np.argmax(ratio, axis=-1).astype(np.int64)


def verified_positions(verified_lens: np.ndarray, num_drafts: int):
    """spec_sampler.py:172-180: starts [B], positions [B, k] clamped to the bonus position, verified [B, k]."""
    lens = verified_lens.astype(np.int64)
    starts = np.cumsum(lens) - lens
    max_drafts = (lens - 1)[:, None]
    steps = np.arange(num_drafts)[None, :]
    return starts, starts[:, None] + np.minimum(steps, max_drafts), steps < max_drafts


def accept_random_varlen(p: np.ndarray, q: np.ndarray, drafts: np.ndarray, verified_lens: np.ndarray,
                         u: np.ndarray, noise: np.ndarray):
    """spec_sampler.py:123-150 with the draws given: u [B, k] (torch.rand, drawn first) and noise [B, V] (the
    clamped Exp(1) of the tail race, drawn second).  Returns n_accept [B], tail [B]."""
    batch_size, num_drafts = drafts.shape
    starts, positions, verified = verified_positions(verified_lens, num_drafts)
    rows = np.arange(batch_size)
    p_draft = p[positions, drafts]                                          # :139
    q_draft = np.take_along_axis(q, drafts[..., None], axis=-1)[..., 0]     # :140
    accepted = ((u.astype(np.float32) * q_draft).astype(np.float32) < p_draft) & verified   # :142
    n_accept = np.cumprod(accepted.astype(np.int64), axis=-1).sum(axis=-1)  # :143
    p_next = p[starts + n_accept]                                           # :145
    q_next = q[rows, np.minimum(n_accept, num_drafts - 1)]                  # :146
    residual = np.maximum((p_next - q_next).astype(np.float32), np.float32(0))   # :147
    is_bonus = (n_accept == verified_lens - 1)[:, None]                      # :148
    weights = np.where(is_bonus, p_next, residual).astype(np.float32)        # :149
    return n_accept.astype(np.int64), race(weights, noise)


def accept_random(p: np.ndarray, q: np.ndarray, drafts: np.ndarray, u: np.ndarray, noise: np.ndarray):
    """spec_sampler.py:114-120: every row verifies k + 1 positions; p [B, k+1, V]."""
    batch_size, num_drafts = drafts.shape
    lens = np.full(batch_size, num_drafts + 1, dtype=np.int64)
    return accept_random_varlen(p.reshape(-1, p.shape[-1]), q, drafts, lens, u, noise)


def accept_greedy_varlen(target_logits: np.ndarray, drafts: np.ndarray, verified_lens: np.ndarray):
    """spec_sampler.py:161-169."""
    target_tokens = np.argmax(target_logits.astype(np.float32), axis=-1)
    starts, positions, verified = verified_positions(verified_lens, drafts.shape[1])
    accepted = (target_tokens[positions] == drafts) & verified
    n_accept = np.cumprod(accepted.astype(np.int64), axis=-1).sum(axis=-1)
    return n_accept.astype(np.int64), target_tokens[starts + n_accept].astype(np.int64)


def accept_greedy(target_logits: np.ndarray, drafts: np.ndarray):
    """spec_sampler.py:153-158: target_logits [B, k+1, V]."""
    batch_size, num_drafts = drafts.shape
    lens = np.full(batch_size, num_drafts + 1, dtype=np.int64)
    return accept_greedy_varlen(target_logits.reshape(-1, target_logits.shape[-1]), drafts, lens)


# ------------------------------------------------------------------------------------------ parity flags
def near_tie_kinds(p: np.ndarray, q: np.ndarray, drafts: np.ndarray, verified_lens: np.ndarray, u: np.ndarray,
                   noise: np.ndarray, eps: float = 1e-6) -> tuple[np.ndarray, np.ndarray]:
    """Requests [B] whose outcome may legitimately differ between two correct fp32 implementations whose p agree
    to `eps` relative, by kind: (accept, race).  accept: an accept draw with |u q_d - p_d| <= eps * max(p_d, u q_d)
    (the exemption the parity rule states).  race: the tail race's winner is within the p uncertainty of another
    candidate (two softmaxes summing in different orders disagree in the last bits of p, so such a race may pick
    either).  Tests compare the other requests bit for bit and count each kind."""
    batch_size, num_drafts = drafts.shape
    starts, positions, verified = verified_positions(verified_lens, num_drafts)
    p_draft = p[positions, drafts].astype(np.float64)
    q_draft = np.take_along_axis(q, drafts[..., None], axis=-1)[..., 0].astype(np.float64)
    uq = u.astype(np.float64) * q_draft
    close = (np.abs(uq - p_draft) <= eps * np.maximum(p_draft, uq)) & verified
    accept_flags = close.any(axis=-1)
    n_accept, _ = accept_random_varlen(p, q, drafts, verified_lens, u, noise)
    rows = np.arange(batch_size)
    p_next = p[starts + n_accept].astype(np.float64)
    q_next = q[rows, np.minimum(n_accept, num_drafts - 1)].astype(np.float64)
    bonus = (n_accept == verified_lens - 1)[:, None]
    w = np.where(bonus, p_next, np.maximum(p_next - q_next, 0.0))
    e = noise.astype(np.float64)
    ratio = w / e
    slack = eps * p_next / e + 1e-7 * ratio
    win = np.argmax(ratio, axis=-1)
    lower = ratio[rows, win] - slack[rows, win]
    upper = ratio + slack
    upper[rows, win] = -np.inf
    race_flags = (upper.max(axis=-1) >= lower) & ~accept_flags
    return accept_flags, race_flags


def near_tie_flags(p: np.ndarray, q: np.ndarray, drafts: np.ndarray, verified_lens: np.ndarray, u: np.ndarray,
                   noise: np.ndarray, eps: float = 1e-6) -> np.ndarray:
    """Requests [B] flagged by either kind of near_tie_kinds."""
    accept_flags, race_flags = near_tie_kinds(p, q, drafts, verified_lens, u, noise, eps)
    return accept_flags | race_flags
