"""The speculative round (nanovllm/engine/speculative.py) on the B200 kernels.

    VerifyRound        verify + accept of given drafts: SpeculativeDecoder.verify_logits / _accept
                       (speculative.py:450-582), fixed-length rows or variable verified lengths
    DFlashDrafter      the block draft: propose (block forward + DSpark's Markov rows) and after_verify
                       (speculative.py:63-337)
    SpeculativeDecoder propose -> verify -> after_verify -> accept -> one D2H (run_round, speculative.py:411-448)

A verification replays one CUDA graph per token count.  The rows' metadata (batch_metadata.pack_verify_metadata:
the values of the reference's verify_varlen_metadata, built with array operations into a pinned staging copy of
the graph's two packed metadata buffers) reaches the device in two host-to-device copies, a third carries the
verified lengths and the draft placement of a variable-length round; the graph replays the target's
verification forward and LM head (logits [T, V] bf16) and, when a drafter is attached, its after_verify (the
context features of the aux layers the forward exported, then every draft layer's context K/V at the verified
positions' slots); the fused sampler (kernel 1) accepts straight from the logits - probabilities, uniforms and
the race noise never materialise - and the single D2H copy of [drafts | n_accept | tail] returns each row's
accepted drafts followed by its tail token.
"""
from __future__ import annotations

from collections import Counter

import numpy as np
import torch

from . import spec_sampler
from .batch_metadata import (RowState, draft_packed_sizes, draft_packed_views, draft_placement,
                             pack_draft_block_metadata, pack_verify_metadata)
from .markov import MarkovQBuffer, markov_rows, num_candidates
from .spec_sampler import SamplingTensors
from .target import Qwen3Target

# DSpark captures sampling graphs for at most this many sampling keys, the first ones it meets; a batch with any
# other key samples eagerly (speculative.py:41-43).
MAX_SAMPLING_KEYS = 4


def verify_token_counts(max_batch_size: int, query_len: int) -> list[int]:
    """The token counts of the variable-length verification graphs (verify_schedule.py:18-23): 1, 2 and 4 when
    below query_len, then every multiple of query_len up to max_batch_size * query_len, so B rows of at most
    query_len tokens always fit the graph of B * query_len tokens."""
    small = [count for count in (1, 2, 4) if count < query_len]
    return small + [query_len * rows for rows in range(1, max_batch_size + 1)]


def sampling_graph_key(sampling: SamplingTensors) -> tuple[int, bool, bool] | None:
    """speculative.py:53-57: what a sampling graph depends on besides the batch size."""
    return None if sampling.temperatures is None else (sampling.max_top_k, sampling.has_top_p, sampling.all_top_k)


class VerifyRound:
    """Verify + accept of given drafts.  graph_rows: fixed-length graphs of B rows x (k + 1) tokens; token_counts:
    variable-length graphs of T tokens with min(T, max_rows) row slots (speculative.py:538-543).  drafter: a
    DFlashDrafter whose after_verify each graph runs after the logits (its aux features exported by the
    forward)."""

    def __init__(self, target: Qwen3Target, num_drafts: int, graph_rows=(), max_num_blocks: int = 0, *,
                 token_counts=(), max_rows: int = 512, drafter: "DFlashDrafter | None" = None):
        self.target = target
        self.num_drafts = num_drafts
        self.block_size = target.block_size
        self.max_num_blocks = max_num_blocks
        self.drafter = drafter
        self.stats: Counter = Counter()
        self.pinned: dict[int, tuple[torch.Tensor, torch.Tensor]] = {}
        self.placement: dict[int, tuple[torch.Tensor, torch.Tensor]] = {}   # pinned host | device, per graph
        self.loaded: dict[int, tuple[int, int, int]] = {}   # per graph: verified tokens, rows, drafts placed
        query_len = num_drafts + 1
        self.shapes: dict[int, int] = {}
        for rows in graph_rows:
            self.shapes[rows * query_len] = rows
        for tokens in token_counts:
            rows = min(tokens, max_rows)
            if self.shapes.get(tokens, rows) != rows:
                raise ValueError(f"graphs of {tokens} tokens with {self.shapes[tokens]} and {rows} row slots")
            if rows * query_len < tokens:
                raise ValueError(f"{rows} row slots cannot hold {tokens} tokens")
            self.shapes[tokens] = rows
        aux_width = drafter.model.aux_width if drafter is not None else 0
        epilogue = drafter.after_verify_graph if drafter is not None else None
        for tokens in sorted(self.shapes):
            rows = self.shapes[tokens]
            target.capture(rows, tokens, max_num_blocks, query_len,
                           lambda b, r=rows, t=tokens: self._load(b, [], [], r, t), aux_width, epilogue)
            self.placement[tokens] = (torch.zeros(rows + 2 * tokens, dtype=torch.int64, pin_memory=True),
                                      torch.zeros(rows + 2 * tokens, dtype=torch.int64, device=target.device))

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

    def graph_for(self, num_rows: int, num_verified: int) -> int:
        """The smallest graph whose row slots and tokens hold num_rows rows verifying num_verified tokens, the
        tokens left filling padding rows of at most k + 1 tokens (speculative.py:503-506)."""
        query_len = self.num_drafts + 1
        for tokens in sorted(self.shapes):
            slots = self.shapes[tokens]
            if tokens >= num_verified and slots >= num_rows and (slots - num_rows) * query_len >= tokens - num_verified:
                return tokens
        raise ValueError(f"no verification graph holds {num_rows} rows verifying {num_verified} tokens")

    def load(self, rows: list[RowState], verified_lens: list[int] | None = None) -> int:
        """Loads a round's metadata into the smallest fitting graph; returns its token count.  With verified_lens
        (row r verifies its last token and its first verified_lens[r] - 1 drafts) the lengths and the draft
        placement go to the device too, in one more copy."""
        k = self.num_drafts
        lens = [k + 1] * len(rows) if verified_lens is None else [int(x) for x in verified_lens]
        if len(lens) != len(rows):
            raise ValueError(f"{len(lens)} verified lengths for {len(rows)} rows")
        num_verified = sum(lens)
        num_tokens = self.graph_for(len(rows), num_verified)
        self._load(self.target.graphs[num_tokens][1], rows, lens, self.shapes[num_tokens], num_tokens)
        placed = -1                                            # fixed-length: rows are contiguous k + 1 blocks
        if verified_lens is not None:
            index, source = draft_placement(lens, k)
            host, dev = self.placement[num_tokens]
            n, placed = len(rows), index.shape[0]
            host_np = host.numpy()
            host_np[:n] = lens
            host_np[n:n + placed] = index
            host_np[n + placed:n + 2 * placed] = source
            dev[:n + 2 * placed].copy_(host[:n + 2 * placed], non_blocking=True)
        self.loaded[num_tokens] = (num_verified, len(rows), placed)
        return num_tokens

    def place_drafts(self, num_tokens: int, drafts: torch.Tensor) -> torch.Tensor | None:
        """speculative.py:514-517: the verified drafts into the graph's input ids where the loaded metadata puts
        them.  Returns the device verified lengths of a variable-length round (None for fixed-length rows)."""
        buffers = self.target.graphs[num_tokens][1]
        _num_verified, n, placed = self.loaded[num_tokens]
        batch, k = drafts.shape
        if batch != n:
            raise ValueError(f"drafts for {batch} rows, metadata loaded for {n}")
        if placed < 0:
            buffers["input_ids"][:batch * (k + 1)].view(batch, k + 1)[:, 1:].copy_(drafts)
            return None
        dev = self.placement[num_tokens][1]
        if placed:
            index, source = dev[n:n + placed], dev[n + placed:n + 2 * placed]
            buffers["input_ids"].index_copy_(0, index, drafts.reshape(-1).index_select(0, source))
        return dev[:n]

    # ------------------------------------------------------------------ the round
    def verify_and_accept(self, num_tokens: int, batch: int, drafts: torch.Tensor, draft_probs: torch.Tensor | None,
                          sampling: SamplingTensors, generator: torch.Generator | None
                          ) -> tuple[torch.Tensor, torch.Tensor]:
        """Graph replay (forward + logits [+ after_verify]) then acceptance of every row's verified drafts
        (speculative.py:430-434, _accept :450-462)."""
        lens = self.place_drafts(num_tokens, drafts)
        num_verified = self.loaded[num_tokens][0]
        logits = self.target.replay(num_tokens)[:num_verified]
        if sampling.temperatures is None:
            return spec_sampler.accept_greedy_varlen(logits, drafts, lens)
        return spec_sampler.accept_from_logits(logits, draft_probs, drafts, sampling, lens, generator)

    def logits(self, num_tokens: int) -> torch.Tensor:
        """The last replay's logits of the verified tokens, [T, V] bf16 (valid until the next replay)."""
        return self.target.graphs[num_tokens][1]["logits"][:self.loaded[num_tokens][0]]

    def commit(self, drafts: torch.Tensor, n_accept: torch.Tensor, tail: torch.Tensor,
               verified_lens: list[int] | None) -> list[list[int]]:
        """speculative.py:436-446: the one D2H copy, then each row's accepted drafts followed by its tail."""
        payload = torch.cat([drafts, n_accept.unsqueeze(1), tail.unsqueeze(1)], dim=1).tolist()   # the one D2H
        appended = []
        for row in payload:
            count, tail_token = row[self.num_drafts], row[self.num_drafts + 1]
            appended.append(row[:count] + [tail_token])
            self.stats[f"accepted_{count}"] += 1
        for length in verified_lens or ():
            self.stats[f"verified_{length}"] += 1
        self.stats["rounds"] += 1
        return appended

    def run_round(self, rows: list[RowState], drafts: torch.Tensor, draft_probs: torch.Tensor | None,
                  sampling: SamplingTensors, generator: torch.Generator | None = None,
                  verified_lens: list[int] | None = None) -> list[list[int]]:
        """speculative.py:411-448 with the drafts given: accepted drafts + tail per row; with verified_lens row r
        verifies only its last token and its first verified_lens[r] - 1 drafts."""
        num_tokens = self.load(rows, verified_lens)
        n_accept, tail = self.verify_and_accept(num_tokens, len(rows), drafts, draft_probs, sampling, generator)
        return self.commit(drafts, n_accept, tail, verified_lens)


class DFlashDrafter:
    """DFlashDrafter (speculative.py:63-337) over a DFlashDraftModel: one block forward proposes k drafts per row,
    DSpark's Markov rows drawing them left to right (kernel 3).  The block forward replays one graph per padded
    batch size (speculative.py:296-324); the logits and the k rows replay a sampling graph per padded batch size
    and sampling key, captured when the key first appears, for the first MAX_SAMPLING_KEYS keys
    (speculative.py:211-266); a key past those runs the same body without a graph; the noise of all k rows is
    drawn outside the graphs, before row 0, from the round's generator.  q lives in a persistent buffer per key whose previous candidates are cleared by the kernel
    (MarkovQBuffer) instead of zero-filling [B, k, V] every round.  after_verify_graph is what a verification
    graph runs after its logits (speculative.py:326-337)."""

    def __init__(self, model, num_drafts: int, graph_batch_sizes, max_num_blocks: int, pad_block_id: int):
        self.model = model
        self.num_drafts = k = num_drafts
        self.batch_sizes = sorted(graph_batch_sizes)
        self.max_num_blocks = max_num_blocks
        self.pad_block_id = pad_block_id
        device = model.device
        bmax = self.batch_sizes[-1]
        s = model.shape
        self.outputs = torch.zeros(bmax * k, s.hidden, dtype=torch.bfloat16, device=device)
        self.drafts = torch.zeros(bmax, k, dtype=torch.int64, device=device)
        self.temperatures = torch.ones(bmax, dtype=torch.float32, device=device)
        self.top_k = torch.zeros(bmax, dtype=torch.int64, device=device)
        self.top_p = torch.ones(bmax, dtype=torch.float32, device=device)
        self.noise: dict = {}
        self.q: dict = {}
        self.logits: dict = {}
        self.views: dict[int, dict] = {}
        self.pinned: dict[int, tuple[torch.Tensor, torch.Tensor]] = {}
        self.graphs: dict[int, torch.cuda.CUDAGraph] = {}
        self.sampling_graphs: dict = {}
        self.graph_pool = None
        self.stats: Counter = Counter()
        for b in reversed(self.batch_sizes):
            n64, n32 = draft_packed_sizes(b, k, max_num_blocks)
            dev64 = torch.zeros(n64, dtype=torch.int64, device=device)
            dev32 = torch.zeros(n32, dtype=torch.int32, device=device)
            self.views[b] = dict(draft_packed_views(dev64, dev32, b, k, max_num_blocks), _packed64=dev64,
                                 _packed32=dev32)
            self.pinned[b] = (torch.empty(n64, dtype=torch.int64, pin_memory=True),
                              torch.empty(n32, dtype=torch.int32, pin_memory=True))
            self._load_block([], b)
            self._capture(self.graphs, b, lambda b=b: self._block_forward(b))

    # ------------------------------------------------------------------ graphs
    def _capture(self, table: dict, b: int, body) -> None:
        body()                                  # warm-up (workspaces, kernel attributes)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, self.graph_pool):
            body()
        if self.graph_pool is None:
            self.graph_pool = graph.pool()
        torch.cuda.synchronize()
        table[b] = graph

    def _load_block(self, rows: list[RowState], b: int) -> None:
        """speculative.py:276-294: draft_block_metadata (batch_metadata.py:99-117) into the graph's buffers
        through a pinned staging copy, two host-to-device copies."""
        host64, host32 = self.pinned[b]
        pack_draft_block_metadata(rows, self.model.block_size, self.num_drafts, self.model.mask_token_id, b,
                                  self.pad_block_id, self.max_num_blocks, host64.numpy(), host32.numpy())
        v = self.views[b]
        v["_packed64"].copy_(host64, non_blocking=True)
        v["_packed32"].copy_(host32, non_blocking=True)

    def _block_forward(self, b: int) -> None:
        v, k = self.views[b], self.num_drafts
        hidden = self.model.forward(v["input_ids"], v["positions"], v["slot_mapping"], v["context_lens"],
                                    v["block_tables"], k)
        self.outputs[:b * k].copy_(hidden)

    def _q_buffer(self, key, b: int):
        q = self.q[key]
        return q.rows(b) if isinstance(q, MarkovQBuffer) else q[:b]

    def _sampling_forward(self, b: int, key) -> None:
        """speculative.py:240-266: the logits of the block outputs, then the k rows into the buffers; row 0's
        previous token is each block's first input, the anchor."""
        k, model = self.num_drafts, self.model
        logits = model.compute_logits(self.outputs[:b * k]).view(b, k, -1)
        self.logits[key, b] = logits         # kept for inspection: the last replay's draft logits
        prev = self.views[b]["input_ids"].view(b, k)[:, 0]
        drafts = self.drafts[:b]
        if key is None:
            markov_rows(logits, prev, None, None, drafts, None, 0, model.markov_head)
            return
        max_top_k, has_top_p, all_top_k = key
        sampling = SamplingTensors(temperatures=self.temperatures[:b], top_k=self.top_k[:b], top_p=self.top_p[:b],
                                   max_top_k=max_top_k, has_top_p=has_top_p, all_top_k=all_top_k)
        candidates = num_candidates(max_top_k, all_top_k, logits.shape[-1])
        markov_rows(logits, prev, sampling, self.noise[key][:b], drafts, self._q_buffer(key, b), candidates,
                    model.markov_head)

    def _key_buffers(self, key) -> None:
        """A random key's noise [max batch, k, candidates or V] (finite padding rows) and q buffer
        (speculative.py:268-275)."""
        if key is None or key in self.noise:
            return
        bmax, k, vocab = self.batch_sizes[-1], self.num_drafts, self.model.shape.vocab
        device = self.model.device
        max_top_k, _, all_top_k = key
        candidates = num_candidates(max_top_k, all_top_k, vocab)
        self.noise[key] = torch.ones(bmax, k, candidates or vocab, dtype=torch.float32, device=device)
        self.q[key] = (MarkovQBuffer(bmax, k, vocab, candidates, device) if candidates else
                       torch.zeros(bmax, k, vocab, dtype=torch.float32, device=device))

    def _capture_sampling_graphs(self, key) -> None:
        self._key_buffers(key)
        graphs: dict = {}
        for b in reversed(self.batch_sizes):
            self._capture(graphs, b, lambda b=b: self._sampling_forward(b, key))
        self.sampling_graphs[key] = graphs

    # ------------------------------------------------------------------ propose
    def load(self, rows: list[RowState]) -> int:
        """The rows' draft-block metadata into the smallest graph that holds them; returns its batch size."""
        padded = next(size for size in self.batch_sizes if size >= len(rows))
        self._load_block(rows, padded)
        return padded

    def draw(self, batch: int, padded: int, sampling: SamplingTensors, generator: torch.Generator | None = None
             ) -> tuple[torch.Tensor, torch.Tensor | None]:
        """The loaded rows' block forward and k Markov rows; returns drafts [B, k] and q [B, k, V] (None when
        greedy), views of the drafter's buffers valid until the next draw."""
        if self.model.markov_head is None:
            raise NotImplementedError("this drafter samples DSpark's Markov rows; a DFlash draft has no Markov head")
        self.graphs[padded].replay()
        key = sampling_graph_key(sampling)
        eager = key not in self.sampling_graphs and len(self.sampling_graphs) >= MAX_SAMPLING_KEYS
        if eager:
            self._key_buffers(key)          # a key past the first MAX_SAMPLING_KEYS samples without a graph
        elif key not in self.sampling_graphs:
            self._capture_sampling_graphs(key)
        if key is not None:                       # speculative.py:225-238; padding rows keep earlier values
            self.temperatures[:batch].copy_(sampling.temperatures)
            self.top_k[:batch].copy_(sampling.top_k)
            self.top_p[:batch].copy_(sampling.top_p)
            spec_sampler.exponential_noise_(self.noise[key][:batch], generator)
        if eager:
            self._sampling_forward(padded, key)
            self.stats["eager_proposals"] += 1
        else:
            self.sampling_graphs[key][padded].replay()
        self.stats["proposals"] += 1
        if key is None:
            return self.drafts[:batch], None
        q = self._q_buffer(key, batch)
        return self.drafts[:batch], q.probs if isinstance(q, MarkovQBuffer) else q

    def propose(self, rows: list[RowState], sampling: SamplingTensors, generator: torch.Generator | None = None
                ) -> tuple[torch.Tensor, torch.Tensor | None]:
        """speculative.py:113-122 without the confidence head: load, then draw."""
        return self.draw(len(rows), self.load(rows), sampling, generator)

    # ------------------------------------------------------------------ after_verify
    def after_verify_graph(self, buffers: dict) -> None:
        """DFlashDrafter.after_verify (speculative.py:326-337) inside a verification graph: the context features of
        every token's aux features, then every draft layer's context K/V at the token's slot (padding tokens have
        slot -1 and store nothing).  The intermediate tensors stay in `buffers` for inspection."""
        aux = buffers["aux"]
        T, hidden = aux.shape[0], self.model.shape.hidden
        device = aux.device
        fc = torch.empty(T, hidden, dtype=torch.bfloat16, device=device)
        features = torch.empty(T, hidden, dtype=torch.bfloat16, device=device)
        kv = torch.empty(T, self.model.w_kv.shape[0], dtype=torch.bfloat16, device=device)
        self.model.context_features(aux, fc_out=fc, out=features)
        self.model.store_context_kv(features, buffers["positions"], buffers["slot_mapping"], kv_out=kv)
        buffers.update(context_fc=fc, context_features=features, context_kv=kv)

    def after_verify(self, rows: list[RowState], aux: torch.Tensor, verified_lens: list[int] | None = None) -> None:
        """speculative.py:326-337 eagerly: context K/V of every verified position from aux [T, aux width]."""
        k = self.num_drafts
        lens = [k + 1] * len(rows) if verified_lens is None else list(verified_lens)
        from .batch_metadata import packed_sizes, packed_views
        n64, n32 = packed_sizes(len(rows), sum(lens), self.max_num_blocks)
        host64 = np.zeros(n64, dtype=np.int64)
        host32 = np.zeros(n32, dtype=np.int32)
        pack_verify_metadata(rows, lens, k, self.model.block_size, len(rows), sum(lens), self.pad_block_id,
                             self.max_num_blocks, host64, host32)
        v = packed_views(host64, host32, len(rows), sum(lens), self.max_num_blocks)
        device = self.model.device
        positions = torch.from_numpy(v["positions"].copy()).to(device)
        slots = torch.from_numpy(v["slot_mapping"].copy()).to(device)
        self.model.store_context_kv(self.model.context_features(aux), positions, slots)


class SpeculativeDecoder:
    """SpeculativeDecoder.run_round (speculative.py:411-448) over a Qwen3Target and a DFlashDrafter: propose, one
    verification (graph: forward, logits, after_verify), acceptance, one D2H copy.  variable_length: the
    verification graphs are one per token count of verify_token_counts (speculative.py:538-541) and a round may
    pass verified_lens; otherwise one per batch size of B rows x (k + 1) tokens."""

    def __init__(self, target: Qwen3Target, drafter: DFlashDrafter, num_drafts: int, max_num_blocks: int, *,
                 variable_length: bool = True, token_counts=None, max_rows: int = 512):
        self.target, self.drafter, self.num_drafts = target, drafter, num_drafts
        batch_sizes = drafter.batch_sizes
        if variable_length:
            counts = verify_token_counts(batch_sizes[-1], num_drafts + 1) if token_counts is None else token_counts
            self.verify = VerifyRound(target, num_drafts, (), max_num_blocks, token_counts=counts, max_rows=max_rows,
                                      drafter=drafter)
        else:
            self.verify = VerifyRound(target, num_drafts, batch_sizes, max_num_blocks, drafter=drafter)
        self.stats = self.verify.stats

    def run_round(self, rows: list[RowState], sampling: SamplingTensors, generator: torch.Generator | None = None,
                  verified_lens: list[int] | None = None) -> list[list[int]]:
        """Per row, the accepted drafts followed by the tail token.  With verified_lens row r verifies only its
        last token and its first verified_lens[r] - 1 drafts."""
        drafts, draft_probs = self.drafter.propose(rows, sampling, generator)
        num_tokens = self.verify.load(rows, verified_lens)
        n_accept, tail = self.verify.verify_and_accept(num_tokens, len(rows), drafts, draft_probs, sampling,
                                                       generator)
        return self.verify.commit(drafts, n_accept, tail, verified_lens)

    def close(self) -> None:
        self.target.close()
        self.drafter.graphs.clear()
        self.drafter.sampling_graphs.clear()
