"""Host-side verification metadata (nanovllm/engine/batch_metadata.py:140-181): as plain lists
(verify_varlen_metadata, the reference's shape) and packed into two arrays (pack_verify_metadata, what a round
copies to the device).

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


# ---------------------------------------------------------------------------------------------- packed arrays
def packed_sizes(num_rows: int, num_tokens: int, width: int) -> tuple[int, int]:
    """Elements of the int64 part (input_ids | positions) and the int32 part (slot_mapping | cu_seqlens_q |
    cu_seqlens_k | block_tables) of a round's metadata, in that order."""
    return 2 * num_tokens, num_tokens + 2 * (num_rows + 1) + num_rows * width


def packed_views(buf64, buf32, num_rows: int, num_tokens: int, width: int) -> dict:
    """The named metadata arrays as views of the two packed buffers (numpy arrays or torch tensors)."""
    t, r = num_tokens, num_rows
    return dict(input_ids=buf64[:t], positions=buf64[t:2 * t], slot_mapping=buf32[:t],
                cu_seqlens_q=buf32[t:t + r + 1], cu_seqlens_k=buf32[t + r + 1:t + 2 * (r + 1)],
                block_tables=buf32[t + 2 * (r + 1):t + 2 * (r + 1) + r * width].reshape(r, width))


def pack_verify_metadata(rows: list[RowState], verified_lens: list[int], num_drafts: int, block_size: int,
                         num_rows: int, num_tokens: int, pad_block_id: int, width: int, buf64, buf32) -> None:
    """verify_varlen_metadata written straight into the packed numpy buffers (int64 [2 T], int32 [...]): the
    same values, built with array operations instead of per-token Python lists."""
    import numpy as np
    query_len = num_drafts + 1
    v = packed_views(buf64, buf32, num_rows, num_tokens, width)
    n = len(rows)
    lens = np.asarray(verified_lens, dtype=np.int64)
    assert lens.shape == (n,) and ((lens >= 1) & (lens <= query_len)).all()
    starts = np.fromiter((row.length - 1 for row in rows), dtype=np.int64, count=n)
    tables = v["block_tables"]
    tables.fill(pad_block_id)
    for i, row in enumerate(rows):
        table = row.block_table
        assert len(table) <= width and len(table) * block_size >= starts[i] + lens[i]
        tables[i, :len(table)] = table
    # the rows' tokens: row r's tokens are positions starts[r] .. starts[r] + lens[r] - 1
    n_real = int(lens.sum())
    first = np.zeros(n, dtype=np.int64)
    np.cumsum(lens[:-1], out=first[1:])
    row_of = np.repeat(np.arange(n), lens)
    pos = starts[row_of] + (np.arange(n_real) - first[row_of])
    ids, positions, slots = v["input_ids"], v["positions"], v["slot_mapping"]
    ids.fill(0)
    ids[first] = np.fromiter((row.last_token for row in rows), dtype=np.int64, count=n)
    positions[:n_real] = pos
    slots[:n_real] = tables[row_of, pos // block_size].astype(np.int64) * block_size + pos % block_size
    # padding rows: <= query_len tokens each at positions 0 onward of the pad block, nothing stored
    left = num_tokens - n_real
    pad_lens = []
    for _ in range(num_rows - n):
        length = min(left, query_len)
        left -= length
        pad_lens.append(length)
    assert left == 0, "the padding rows cannot hold the tokens left"
    pad_lens = np.asarray(pad_lens, dtype=np.int64)
    n_pad = int(pad_lens.sum())
    if n_pad:
        pfirst = np.zeros(len(pad_lens), dtype=np.int64)
        np.cumsum(pad_lens[:-1], out=pfirst[1:])
        prow = np.repeat(np.arange(len(pad_lens)), pad_lens)
        positions[n_real:] = np.arange(n_pad) - pfirst[prow]
        slots[n_real:] = PAD_SLOT
    all_q = np.concatenate([lens, pad_lens])
    all_k = np.concatenate([starts + lens, pad_lens])
    v["cu_seqlens_q"][0] = 0
    v["cu_seqlens_q"][1:] = np.cumsum(all_q)
    v["cu_seqlens_k"][0] = 0
    v["cu_seqlens_k"][1:] = np.cumsum(all_k)
