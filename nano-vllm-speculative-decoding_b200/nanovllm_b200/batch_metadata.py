"""Host-side verification metadata (nanovllm/engine/batch_metadata.py:140-181), as plain lists.

A row needs only what the reference reads from a Sequence: its length (len(seq)), its last token and its
block table (seq.target_kv.block_table).  PAD_SLOT rows store nothing; padding rows read the pad block.
"""
from __future__ import annotations

from dataclasses import dataclass, field

PAD_SLOT = -1


@dataclass
class RowState:
    """The fields of a Sequence a verification reads (sequence.py): token count, last token, block table."""
    length: int
    last_token: int
    block_table: list[int]


def slot_of(block_table: list[int], block_size: int, position: int) -> int:
    """batch_metadata.py:14-15."""
    return block_table[position // block_size] * block_size + position % block_size


@dataclass
class VerifyMetadata:
    input_ids: list[int] = field(default_factory=list)      # draft positions hold 0, filled on device
    positions: list[int] = field(default_factory=list)
    slot_mapping: list[int] = field(default_factory=list)
    cu_seqlens_q: list[int] = field(default_factory=lambda: [0])
    cu_seqlens_k: list[int] = field(default_factory=lambda: [0])
    block_tables: list[list[int]] = field(default_factory=list)
    draft_index: list[int] = field(default_factory=list)    # where each verified draft goes in input_ids
    draft_source: list[int] = field(default_factory=list)   # and where it is in the drafts [B, k], flattened


def verify_varlen_metadata(rows: list[RowState], verified_lens: list[int], num_drafts: int, block_size: int,
                           num_rows: int, num_tokens: int, pad_block_id: int, width: int) -> VerifyMetadata:
    """batch_metadata.py:149-181: row r verifies its last token and its first verified_lens[r] - 1 drafts at
    positions len-1 onward; the tokens left of num_tokens fill padding rows (<= k + 1 tokens each, positions 0
    onward of the pad block); the row slots left of num_rows are empty."""
    query_len = num_drafts + 1
    m = VerifyMetadata()
    for r, (row, length) in enumerate(zip(rows, verified_lens)):
        table = row.block_table
        start = row.length - 1
        assert 1 <= length <= query_len
        assert len(table) <= width and len(table) * block_size >= start + length
        first = len(m.input_ids)
        m.input_ids.extend([row.last_token] + [0] * (length - 1))
        m.positions.extend(range(start, start + length))
        m.slot_mapping.extend(slot_of(table, block_size, p) for p in range(start, start + length))
        m.draft_index.extend(range(first + 1, first + length))
        m.draft_source.extend(range(r * num_drafts, r * num_drafts + length - 1))
        m.cu_seqlens_q.append(m.cu_seqlens_q[-1] + length)
        m.cu_seqlens_k.append(m.cu_seqlens_k[-1] + start + length)
        m.block_tables.append(table + [pad_block_id] * (width - len(table)))
    left = num_tokens - len(m.input_ids)
    for _ in range(num_rows - len(rows)):
        length = min(left, query_len)
        left -= length
        m.input_ids.extend([0] * length)
        m.positions.extend(range(length))
        m.slot_mapping.extend([PAD_SLOT] * length)
        m.cu_seqlens_q.append(m.cu_seqlens_q[-1] + length)
        m.cu_seqlens_k.append(m.cu_seqlens_k[-1] + length)
        m.block_tables.append([pad_block_id] * width)
    assert left == 0, "the padding rows cannot hold the tokens left"
    return m
