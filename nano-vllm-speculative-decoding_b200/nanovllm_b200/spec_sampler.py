"""The reference's sampler API (nanovllm/layers/spec_sampler.py) on the B200 kernels of libspecdec_b200.so.

Same names, arguments and results as the reference module, so callers and tests switch by import:

    SamplingTensors, sampling_tensors, sampling_per_token   spec_sampler.py:17-52   (host bookkeeping, unchanged)
    probs_from_logits                                       spec_sampler.py:65-69   -> specdec_probs
    exponential_noise_                                      spec_sampler.py:99-101  (torch draw, unchanged)
    race / sample                                           spec_sampler.py:104-111 -> specdec_race
    accept_random / accept_random_varlen                    spec_sampler.py:114-150 -> specdec_accept (probs)
    accept_greedy / accept_greedy_varlen                    spec_sampler.py:153-169 -> specdec_accept_greedy
plus the fused entry the round driver uses, accept_from_logits (SpeculativeDecoder._accept's body without the
[T, V] probability tensor, speculative.py:450-462) -> specdec_accept on logits.

Random draws.  With draws="kernel" (default) the kernels regenerate, in-kernel, exactly the numbers torch's CUDA
generator would have produced for the reference's draws - the [B, k] uniforms of torch.rand, then the [B, V]
Exp(1) noise of exponential_ - and the generator's offset is advanced by what torch would have consumed, so the
generator ends where the reference leaves it.  With draws="torch" the wrapper draws u and E with those torch
calls and the kernels read them (the same numbers, at the cost of writing and reading the noise).  Inside CUDA
graph capture, use draws="torch".  Tests may pass draws=(u, noise), the two draws as tensors.

Limits of this build (checked on the host, errors raise SpecdecError): B <= 1024 requests, k <= 32 drafts,
T <= 16384 verified rows, B * V < 2^31, top_k <= 1024 when truncating.
"""
from __future__ import annotations

from dataclasses import dataclass, replace

import torch

from . import _lib
from ._lib import DTYPE_CODES, Workspace, check, ptr, require_cuda, stream_of

EXPONENTIAL_NOISE_FLOOR = 1e-10
NEGATIVE_INFINITY = float("-inf")


@dataclass
class SamplingTensors:
    temperatures: torch.Tensor | None  # [B] fp32; None when every row is greedy
    top_k: torch.Tensor                # [B] int64; 0 disables top-k for that row
    top_p: torch.Tensor                # [B] fp32; 1.0 disables top-p for that row
    max_top_k: int                     # host copy of max(top_k); 0 means no row truncates
    has_top_p: bool                    # host: some row has top_p < 1
    all_top_k: bool                    # host: every row has top_k > 0


def sampling_tensors(seqs, device: torch.device) -> SamplingTensors:
    """spec_sampler.py:27-41: per-row parameters of a batch; mixed greedy/random batches are rejected."""
    temperatures = [seq.temperature for seq in seqs]
    is_greedy = temperatures[0] == 0
    if any((temperature == 0) != is_greedy for temperature in temperatures):
        raise ValueError("mixed greedy and random sampling is not supported")
    top_k = [seq.top_k for seq in seqs]
    top_p = [seq.top_p for seq in seqs]
    return SamplingTensors(
        temperatures=None if is_greedy else _to_device(temperatures, torch.float32, device),
        top_k=_to_device(top_k, torch.int64, device),
        top_p=_to_device(top_p, torch.float32, device),
        max_top_k=max(top_k),
        has_top_p=any(value < 1.0 for value in top_p),
        all_top_k=min(top_k) > 0,
    )


def sampling_per_token(sampling: SamplingTensors, verified_lens: torch.Tensor, num_tokens: int) -> SamplingTensors:
    """spec_sampler.py:44-52: each row's parameters repeated over its verified positions."""
    temperatures = sampling.temperatures
    return replace(sampling,
                   temperatures=None if temperatures is None else
                   temperatures.repeat_interleave(verified_lens, output_size=num_tokens),
                   top_k=sampling.top_k.repeat_interleave(verified_lens, output_size=num_tokens),
                   top_p=sampling.top_p.repeat_interleave(verified_lens, output_size=num_tokens))


def _to_device(values: list, dtype: torch.dtype, device: torch.device) -> torch.Tensor:
    host = torch.tensor(values, dtype=dtype, pin_memory=device.type == "cuda")
    return host.to(device, non_blocking=True)


def _workspace(device: torch.device, rows: int) -> torch.Tensor:
    return Workspace.get(device, _lib.lib().specdec_sampler_workspace_bytes(rows))


def _generator(generator: torch.Generator | None, device: torch.device) -> torch.Generator:
    if generator is not None:
        if generator.device.type != "cuda":
            raise ValueError("in-kernel draws need a CUDA generator (use draws='torch' for others)")
        return generator
    index = device.index if device.index is not None else torch.cuda.current_device()
    return torch.cuda.default_generators[index]


def _claim_draws(generator: torch.Generator | None, device: torch.device, *numels: int) -> tuple[int, list[int]]:
    """Reserves the Philox offsets torch would consume for draws of these sizes, in order; returns the seed and
    the offset each draw starts at, and advances the generator past them."""
    if torch.cuda.is_current_stream_capturing():
        raise RuntimeError("in-kernel draws read the generator on the host; use draws='torch' under graph capture")
    gen = _generator(generator, device)
    seed = gen.initial_seed()
    offset = gen.get_offset()
    starts = []
    for numel in numels:
        starts.append(offset)
        offset += int(_lib.lib().specdec_philox_increment(numel))
    gen.set_offset(offset)
    return seed, starts


def _params_per_row(sampling: SamplingTensors):
    top_k = sampling.top_k.contiguous() if sampling.max_top_k > 0 else None
    top_p = sampling.top_p.contiguous() if sampling.has_top_p else None
    return top_k, top_p


def probs_from_logits(logits: torch.Tensor, sampling: SamplingTensors) -> torch.Tensor:
    """spec_sampler.py:65-69: fp32 probabilities after temperature, top-k and top-p, in two kernel passes.
    logits [B, n, V] with [B] parameters, or [T, V] with [T] parameters."""
    assert sampling.temperatures is not None
    device = require_cuda(logits)
    logits = logits.contiguous()
    vocab = logits.shape[-1]
    rows = logits.numel() // vocab
    params = sampling.temperatures.shape[0]
    if rows % params:
        raise ValueError(f"{rows} rows do not split over {params} parameter rows")
    out = torch.empty(logits.shape, dtype=torch.float32, device=device)
    top_k, top_p = _params_per_row(sampling)
    ws = _workspace(device, rows)
    check(_lib.lib().specdec_probs(ptr(logits), DTYPE_CODES[logits.dtype], rows, vocab, rows // params,
                                   ptr(sampling.temperatures.contiguous()), ptr(top_k), ptr(top_p),
                                   sampling.max_top_k, int(sampling.has_top_p), ptr(out), ptr(ws), ws.numel(),
                                   stream_of(device)))
    return out


def exponential_noise_(out: torch.Tensor, generator: torch.Generator | None) -> torch.Tensor:
    """spec_sampler.py:99-101: Exp(1) noise clamped at 1e-10, in place (the reference's own draw)."""
    return out.exponential_(1.0, generator=generator).clamp_min_(EXPONENTIAL_NOISE_FLOOR)


def race(weights: torch.Tensor, noise: torch.Tensor) -> torch.Tensor:
    """spec_sampler.py:104-106: argmax(w / E) over the last dim, first index on ties."""
    device = require_cuda(weights, noise)
    w = weights.float().contiguous()
    vocab = w.shape[-1]
    rows = w.numel() // vocab
    e = noise.float().contiguous()
    out = torch.empty(w.shape[:-1], dtype=torch.int64, device=device)
    ws = _workspace(device, rows)
    check(_lib.lib().specdec_race(ptr(w), rows, vocab, ptr(e), 0, 0, ptr(out), ptr(ws), ws.numel(),
                                  stream_of(device)))
    return out


def sample(weights: torch.Tensor, generator: torch.Generator | None, *, draws: str = "kernel") -> torch.Tensor:
    """spec_sampler.py:109-111: the exponential race with fresh Exp(1) noise from `generator`."""
    if draws == "torch":
        return race(weights, exponential_noise_(torch.empty_like(weights, dtype=torch.float32), generator))
    device = require_cuda(weights)
    w = weights.float().contiguous()
    vocab = w.shape[-1]
    rows = w.numel() // vocab
    seed, (offset,) = _claim_draws(generator, device, rows * vocab)
    out = torch.empty(w.shape[:-1], dtype=torch.int64, device=device)
    ws = _workspace(device, rows)
    check(_lib.lib().specdec_race(ptr(w), rows, vocab, None, seed, offset, ptr(out), ptr(ws), ws.numel(),
                                  stream_of(device)))
    return out


def _accept(x: torch.Tensor, x_is_probs: bool, q: torch.Tensor, drafts: torch.Tensor,
            verified_lens: torch.Tensor | None, sampling: SamplingTensors | None,
            generator: torch.Generator | None, draws: str) -> tuple[torch.Tensor, torch.Tensor]:
    device = require_cuda(x, q, drafts, verified_lens)
    batch, k = drafts.shape
    vocab = x.shape[-1]
    x = x.contiguous()
    rows = x.numel() // vocab
    q = q.float().contiguous()
    drafts = drafts.to(torch.int64).contiguous()
    lens = None if verified_lens is None else verified_lens.to(torch.int64).contiguous()
    n_accept = torch.empty(batch, dtype=torch.int64, device=device)
    tail = torch.empty(batch, dtype=torch.int64, device=device)
    if isinstance(draws, tuple):
        u, noise = (t.to(device=device, dtype=torch.float32).contiguous() for t in draws)
        if u.shape != (batch, k) or noise.shape != (batch, vocab):
            raise ValueError(f"explicit draws must be u [{batch}, {k}] and noise [{batch}, {vocab}]")
        seed, offsets = 0, [0, 0]
    elif draws == "torch":
        u = torch.rand(batch, k, device=device, generator=generator)
        noise = exponential_noise_(torch.empty(batch, vocab, device=device), generator)
        seed, offsets = 0, [0, 0]
    elif draws == "kernel":
        u = noise = None
        seed, offsets = _claim_draws(generator, device, batch * k, batch * vocab)
    else:
        raise ValueError(f"draws must be 'kernel', 'torch' or a (u, noise) pair, not {draws!r}")
    temps = top_k = top_p = None
    max_top_k, has_top_p = 0, False
    if sampling is not None:
        temps = sampling.temperatures.contiguous()
        top_k, top_p = _params_per_row(sampling)
        max_top_k, has_top_p = sampling.max_top_k, sampling.has_top_p
    if noise is None:   # in-kernel draws: room for the noise codes the tail race streams
        ws = Workspace.get(device, _lib.lib().specdec_accept_workspace_bytes(rows, batch, vocab))
    else:
        ws = _workspace(device, rows)
    check(_lib.lib().specdec_accept(ptr(x), int(x_is_probs), DTYPE_CODES[x.dtype], rows, vocab, ptr(q), ptr(drafts),
                                    batch, k, ptr(lens), ptr(temps), ptr(top_k), ptr(top_p), max_top_k,
                                    int(has_top_p), ptr(u), ptr(noise), seed, offsets[0], offsets[1],
                                    ptr(n_accept), ptr(tail), ptr(ws), ws.numel(), stream_of(device)))
    return n_accept, tail


def accept_random(p: torch.Tensor, q: torch.Tensor, drafts: torch.Tensor, generator: torch.Generator | None,
                  *, draws: str = "kernel") -> tuple[torch.Tensor, torch.Tensor]:
    """spec_sampler.py:114-120: every row verifies all k drafts; p [B, k+1, V]."""
    return _accept(p.float(), True, q, drafts, None, None, generator, draws)


def accept_random_varlen(p: torch.Tensor, q: torch.Tensor, drafts: torch.Tensor, verified_lens: torch.Tensor,
                         generator: torch.Generator | None, *, draws: str = "kernel"
                         ) -> tuple[torch.Tensor, torch.Tensor]:
    """spec_sampler.py:123-150: rejection sampling of each row's first verified_lens - 1 drafts over the flat
    [T, V] probabilities; returns n_accept [B] and tail [B]."""
    return _accept(p.float(), True, q, drafts, verified_lens, None, generator, draws)


def accept_from_logits(logits: torch.Tensor, q: torch.Tensor, drafts: torch.Tensor, sampling: SamplingTensors,
                       verified_lens: torch.Tensor | None, generator: torch.Generator | None, *,
                       draws: str = "kernel") -> tuple[torch.Tensor, torch.Tensor]:
    """speculative.py:450-462 (random branch) fused: accept_random[_varlen](probs_from_logits(logits), ...) with
    the probabilities computed inside the kernels and never written.  logits [B, k+1, V] or flat [T, V] (bf16,
    fp16 or fp32); sampling holds the per-request [B] parameters."""
    if sampling.temperatures is None:
        raise ValueError("greedy batches go through accept_greedy[_varlen]")
    return _accept(logits, False, q, drafts, verified_lens, sampling, generator, draws)


def accept_greedy(target_logits: torch.Tensor, drafts: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """spec_sampler.py:153-158: target_logits [B, k+1, V]."""
    return accept_greedy_varlen(target_logits.flatten(0, 1), drafts, None)


def accept_greedy_varlen(target_logits: torch.Tensor, drafts: torch.Tensor,
                         verified_lens: torch.Tensor | None) -> tuple[torch.Tensor, torch.Tensor]:
    """spec_sampler.py:161-169: a draft is accepted iff it equals the target's argmax at its position."""
    device = require_cuda(target_logits, drafts, verified_lens)
    batch, k = drafts.shape
    logits = target_logits.contiguous()
    vocab = logits.shape[-1]
    rows = logits.numel() // vocab
    drafts = drafts.to(torch.int64).contiguous()
    lens = None if verified_lens is None else verified_lens.to(torch.int64).contiguous()
    n_accept = torch.empty(batch, dtype=torch.int64, device=device)
    tail = torch.empty(batch, dtype=torch.int64, device=device)
    ws = _workspace(device, rows)
    check(_lib.lib().specdec_accept_greedy(ptr(logits), DTYPE_CODES[logits.dtype], rows, vocab, ptr(drafts), batch, k,
                                           ptr(lens), ptr(n_accept), ptr(tail), ptr(ws), ws.numel(),
                                           stream_of(device)))
    return n_accept, tail
