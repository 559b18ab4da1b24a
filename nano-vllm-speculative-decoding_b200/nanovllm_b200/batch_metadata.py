"""Host-side verification metadata (nanovllm/engine/batch_metadata.py:140-181), built with array operations
straight into the two packed arrays a round copies to the device (pack_verify_metadata), plus where each
verified draft goes among the round's input ids (draft_placement).  The values are those of the reference's
verify_varlen_metadata; tests/golden/metadata.npz holds that function's output on random batches.

A row needs only what the reference reads from a Sequence: its length (len(seq)), its last token and its
block table (seq.target_kv.block_table).  PAD_SLOT rows store nothing; padding rows read the pad block.
"""
from __future__ import annotations

from dataclasses import dataclass

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


def draft_placement(verified_lens, num_drafts: int):
    """Where a round's verified drafts go: row r's drafts 0 .. verified_lens[r] - 2 sit right after its last token
    in the flat input ids.  Returns (index into the input ids, index into the flattened drafts [B, k]), both int64
    numpy arrays in row order (the draft_index / draft_source lists of batch_metadata.py:135-136, 167-168)."""
    import numpy as np
    lens = np.asarray(verified_lens, dtype=np.int64)
    n = lens.shape[0]
    first = np.zeros(n, dtype=np.int64)
    if n:
        np.cumsum(lens[:-1], out=first[1:])
    drafts_per_row = lens - 1
    row_of = np.repeat(np.arange(n, dtype=np.int64), drafts_per_row)
    row_start = np.zeros(n, dtype=np.int64)
    if n:
        np.cumsum(drafts_per_row[:-1], out=row_start[1:])
    j = np.arange(row_of.shape[0], dtype=np.int64) - row_start[row_of]
    return first[row_of] + 1 + j, row_of * num_drafts + j


# ---------------------------------------------------------------------------------------------- draft blocks
def draft_packed_sizes(num_rows: int, query_len: int, width: int) -> tuple[int, int]:
    """Elements of the int64 part (input_ids | positions) and the int32 part (slot_mapping | context_lens |
    block_tables) of a draft block forward's metadata, in that order."""
    t = num_rows * query_len
    return 2 * t, t + num_rows + num_rows * width


def draft_packed_views(buf64, buf32, num_rows: int, query_len: int, width: int) -> dict:
    t, r = num_rows * query_len, num_rows
    return dict(input_ids=buf64[:t], positions=buf64[t:2 * t], slot_mapping=buf32[:t], context_lens=buf32[t:t + r],
                block_tables=buf32[t + r:t + r + r * width].reshape(r, width))


def pack_draft_block_metadata(rows: list[RowState], block_size: int, query_len: int, mask_token_id: int,
                              num_rows: int, pad_block_id: int, width: int, buf64, buf32) -> None:
    """The values of the reference's draft_block_metadata (batch_metadata.py:99-117) written into the packed
    numpy buffers: row r's block is its last token (the anchor, position len-1) then query_len - 1 mask tokens at
    the following positions, stored at their block-table slots, reading len-1 + query_len keys; padding rows are
    query_len mask tokens at positions 0 onward that store nothing and read the pad block."""
    import numpy as np
    v = draft_packed_views(buf64, buf32, num_rows, query_len, width)
    n = len(rows)
    assert n <= num_rows
    ids, positions, slots = (v[key].reshape(num_rows, query_len) for key in ("input_ids", "positions",
                                                                           "slot_mapping"))
    tables = v["block_tables"]
    tables.fill(pad_block_id)
    ids.fill(mask_token_id)
    positions[:] = np.arange(query_len, dtype=np.int64)
    slots.fill(PAD_SLOT)
    v["context_lens"].fill(query_len)
    if not n:
        return
    anchors = np.fromiter((row.length - 1 for row in rows), dtype=np.int64, count=n)
    for i, row in enumerate(rows):
        table = row.block_table
        assert len(table) <= width and len(table) * block_size >= anchors[i] + query_len
        tables[i, :len(table)] = table
    ids[:n, 0] = np.fromiter((row.last_token for row in rows), dtype=np.int64, count=n)
    pos = anchors[:, None] + np.arange(query_len, dtype=np.int64)[None, :]
    positions[:n] = pos
    slots[:n] = tables[np.arange(n)[:, None], pos // block_size].astype(np.int64) * block_size + pos % block_size
    v["context_lens"][:n] = anchors + query_len
