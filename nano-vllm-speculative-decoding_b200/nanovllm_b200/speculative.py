"""The verify + accept round (SpeculativeDecoder.run_round / verify_logits / _accept,
nanovllm/engine/speculative.py:411-512) on the B200 kernels.

    round = VerifyRound(target, num_drafts=7, graph_rows=[64])
    appended = round.run_round(rows, drafts, draft_probs, sampling, generator=gen)   # list[list[int]]

A round: the rows' metadata (batch_metadata.pack_verify_metadata: the values of verify_varlen_metadata, built
with array operations into a pinned staging copy of the graph's two packed metadata buffers) reaches the device in
two host-to-device copies, the drafts are placed on the device, the graph replays the
target's verification forward and LM head (logits [T, V] bf16), the fused sampler (kernel 1) accepts straight
from the logits - probabilities, uniforms and the race noise never materialise - and the single D2H copy of
[drafts | n_accept | tail] returns each row's accepted drafts followed by its tail token.
"""
from __future__ import annotations

from collections import Counter

import torch

from . import spec_sampler
from .batch_metadata import RowState, pack_verify_metadata
from .spec_sampler import SamplingTensors
from .target import Qwen3Target


class VerifyRound:
    def __init__(self, target: Qwen3Target, num_drafts: int, graph_rows: list[int], max_num_blocks: int):
        self.target = target
        self.num_drafts = num_drafts
        self.block_size = target.block_size
        self.max_num_blocks = max_num_blocks
        self.stats: Counter = Counter()
        self.pinned: dict[int, tuple[torch.Tensor, torch.Tensor]] = {}
        query_len = num_drafts + 1
        for rows in sorted(graph_rows):
            tokens = rows * query_len
            target.capture(rows, tokens, max_num_blocks, query_len,
                           lambda b, r=rows, t=tokens: self._load(b, [], [], r, t))

    # ------------------------------------------------------------------ metadata
    def _load(self, buffers: dict, rows: list[RowState], lens: list[int], num_rows: int, num_tokens: int) -> None:
        """speculative.py:519-527: the metadata (batch_metadata.py:149-181) into the graph's two packed buffers:
        built in a pinned staging copy (one per graph), then two non-blocking host-to-device copies.  The staging
        copy is rewritten only after the previous round's D2H read, which follows these copies on the stream."""
        dev64, dev32 = buffers["_packed64"], buffers["_packed32"]
        staging = self.pinned.get(num_tokens)
        if staging is None:
            staging = (torch.empty(dev64.shape, dtype=torch.int64, pin_memory=True),
                       torch.empty(dev32.shape, dtype=torch.int32, pin_memory=True))
            self.pinned[num_tokens] = staging
        host64, host32 = staging
        pack_verify_metadata(rows, lens, self.num_drafts, self.block_size, num_rows, num_tokens,
                             self.target.pad_block_id, self.max_num_blocks, host64.numpy(), host32.numpy())
        dev64.copy_(host64, non_blocking=True)
        dev32.copy_(host32, non_blocking=True)

    def load(self, rows: list[RowState], verified_lens: list[int] | None = None) -> int:
        """Loads a round's metadata into the smallest fitting graph; returns its token count."""
        lens = [self.num_drafts + 1] * len(rows) if verified_lens is None else verified_lens
        num_verified = sum(lens)
        num_tokens = next(t for t in sorted(self.target.graphs) if t >= num_verified)
        num_rows = num_tokens // (self.num_drafts + 1)
        self._load(self.target.graphs[num_tokens][1], rows, lens, num_rows, num_tokens)
        return num_tokens

    def place_drafts(self, num_tokens: int, drafts: torch.Tensor) -> None:
        """speculative.py:514-517 for fixed-length rows: drafts [B, k] after each row's last token."""
        buffers = self.target.graphs[num_tokens][1]
        batch, k = drafts.shape
        buffers["input_ids"][:batch * (k + 1)].view(batch, k + 1)[:, 1:].copy_(drafts)

    # ------------------------------------------------------------------ the round
    def verify_and_accept(self, num_tokens: int, batch: int, drafts: torch.Tensor, draft_probs: torch.Tensor | None,
                          sampling: SamplingTensors, generator: torch.Generator | None
                          ) -> tuple[torch.Tensor, torch.Tensor]:
        """Graph replay (forward + logits) then acceptance of every row's k drafts (speculative.py:430-434)."""
        self.place_drafts(num_tokens, drafts)
        logits = self.target.replay(num_tokens)[:batch * (self.num_drafts + 1)]
        if sampling.temperatures is None:
            return spec_sampler.accept_greedy_varlen(logits, drafts, None)
        return spec_sampler.accept_from_logits(logits, draft_probs, drafts, sampling, None, generator)

    def run_round(self, rows: list[RowState], drafts: torch.Tensor, draft_probs: torch.Tensor | None,
                  sampling: SamplingTensors, generator: torch.Generator | None = None) -> list[list[int]]:
        """speculative.py:411-448 for fixed-length rows, drafts given: accepted drafts + tail per row."""
        num_tokens = self.load(rows)
        n_accept, tail = self.verify_and_accept(num_tokens, len(rows), drafts, draft_probs, sampling, generator)
        payload = torch.cat([drafts, n_accept.unsqueeze(1), tail.unsqueeze(1)], dim=1).tolist()   # the one D2H
        appended = []
        for row in payload:
            count, tail_token = row[self.num_drafts], row[self.num_drafts + 1]
            appended.append(row[:count] + [tail_token])
            self.stats[f"accepted_{count}"] += 1
        self.stats["rounds"] += 1
        return appended
