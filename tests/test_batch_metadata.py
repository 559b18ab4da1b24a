"""Verification metadata (nanovllm/engine/batch_metadata.py:149-181): the packed array builder a round copies to
the device, checked against the reference's verify_varlen_metadata run on the same batches (tests/golden/
metadata.npz, written by tests/golden/make_golden.py), and against the layout's invariants on random batches."""
import random
from pathlib import Path

import numpy as np
import pytest

from nanovllm_b200.batch_metadata import (PAD_SLOT, RowState, draft_packed_sizes, draft_packed_views,
                                          draft_placement, pack_draft_block_metadata, pack_verify_metadata,
                                          packed_sizes, packed_views)

META = np.load(Path(__file__).parent / "golden" / "metadata.npz")
CASES = sorted({key.split("/")[1] for key in META.files if key.startswith("meta/")})
DRAFT_CASES = sorted({key.split("/")[1] for key in META.files if key.startswith("draft/")})


def golden_case(case):
    c = {key.split("/")[2]: META[key] for key in META.files if key.startswith(f"meta/{case}/")}
    k, bs, num_rows, num_tokens, pad, width = (int(x) for x in c["scalars"])
    rows = [RowState(length=int(n), last_token=int(t), block_table=[int(b) for b in table if b >= 0])
            for n, t, table in zip(c["lengths"], c["last_tokens"], c["tables"])]
    return c, rows, [int(x) for x in c["verified_lens"]], k, bs, num_rows, num_tokens, pad, width


def packed(rows, lens, k, bs, num_rows, num_tokens, pad, width):
    n64, n32 = packed_sizes(num_rows, num_tokens, width)
    buf64 = np.full(n64, -7, dtype=np.int64)          # poison: every element must be written
    buf32 = np.full(n32, -7, dtype=np.int32)
    pack_verify_metadata(rows, lens, k, bs, num_rows, num_tokens, pad, width, buf64, buf32)
    return packed_views(buf64, buf32, num_rows, num_tokens, width)


def test_golden_cases_cover_the_layouts():
    kinds = set()
    for case in CASES:
        c, rows, lens, k, *_rest, num_rows, num_tokens, _pad, _width = golden_case(case)
        kinds.add("varlen" if any(x != k + 1 for x in lens) else "fixed")
        if num_rows > len(rows):
            kinds.add("padding rows")
        cq = c["cu_seqlens_q"].tolist()
        if any(cq[r + 1] == cq[r] for r in range(len(rows), num_rows)):
            kinds.add("empty row slots")
        if not rows:
            kinds.add("no rows")
    assert {"varlen", "fixed", "padding rows", "empty row slots", "no rows"} <= kinds, kinds


@pytest.mark.parametrize("case", CASES)
def test_packed_metadata_matches_the_reference(case):
    """Every array the round copies, padding rows and empty row slots included, equals the reference's."""
    c, rows, lens, k, bs, num_rows, num_tokens, pad, width = golden_case(case)
    v = packed(rows, lens, k, bs, num_rows, num_tokens, pad, width)
    for key in ("input_ids", "positions", "slot_mapping", "cu_seqlens_q", "cu_seqlens_k"):
        assert v[key].tolist() == c[key].tolist(), key
    assert v["block_tables"].tolist() == c["block_tables"].tolist()


@pytest.mark.parametrize("case", CASES)
def test_draft_placement_matches_the_reference(case):
    c, _rows, lens, k, *_ = golden_case(case)
    index, source = draft_placement(lens, k)
    assert index.tolist() == c["draft_index"].tolist()
    assert source.tolist() == c["draft_source"].tolist()


def random_case(seed):
    rng = random.Random(seed)
    k, block_size, width = 7, 256, 8
    n = rng.randint(0, 12)
    rows, lens, next_block = [], [], 0
    for _ in range(n):
        length = rng.randint(1, 1500)
        ln = rng.randint(1, k + 1)
        blocks = -(-(length - 1 + ln) // block_size)
        rows.append(RowState(length=length, last_token=rng.randint(0, 150000),
                             block_table=list(range(next_block, next_block + blocks))))
        next_block += blocks
        lens.append(ln)
    num_rows = n + rng.randint(0, 4)
    num_tokens = sum(lens) + rng.randint(0, (num_rows - n) * (k + 1))
    return rows, lens, k, block_size, num_rows, num_tokens, 999, width


@pytest.mark.parametrize("seed", range(40))
def test_packed_metadata_invariants(seed):
    """The layout's rules on random batches: row r's tokens are its last token then zeros (drafts are placed on
    the device) at positions len-1 onward, stored at their block-table slots; padding rows hold at most k + 1
    tokens at positions 0 onward, store nothing and read only the pad block; row slots past the tokens are empty."""
    rows, lens, k, bs, num_rows, num_tokens, pad, width = random_case(seed)
    v = packed(rows, lens, k, bs, num_rows, num_tokens, pad, width)
    cq, ck = v["cu_seqlens_q"].tolist(), v["cu_seqlens_k"].tolist()
    assert cq[0] == 0 and ck[0] == 0 and cq[-1] == num_tokens
    for r, (row, ln) in enumerate(zip(rows, lens)):
        a = cq[r]
        assert cq[r + 1] - a == ln
        assert ck[r + 1] - ck[r] == row.length - 1 + ln
        assert v["input_ids"][a:a + ln].tolist() == [row.last_token] + [0] * (ln - 1)
        for j in range(ln):
            p = row.length - 1 + j
            assert v["positions"][a + j] == p
            assert v["slot_mapping"][a + j] == row.block_table[p // bs] * bs + p % bs
        table = v["block_tables"][r].tolist()
        assert table == row.block_table + [pad] * (width - len(row.block_table))
    for r in range(len(rows), num_rows):
        ln = cq[r + 1] - cq[r]
        assert 0 <= ln <= k + 1 and ck[r + 1] - ck[r] == ln
        assert v["positions"][cq[r]:cq[r + 1]].tolist() == list(range(ln))
        assert (v["block_tables"][r] == pad).all()
    assert (v["slot_mapping"][sum(lens):] == PAD_SLOT).all()
    assert (v["input_ids"][sum(lens):] == 0).all()
    index, source = draft_placement(lens, k)
    assert index.shape == source.shape == (sum(lens) - len(lens),)
    assert (np.asarray(v["input_ids"])[index] == 0).all()


def test_packed_metadata_rejects_overfull_padding():
    rows = [RowState(length=10, last_token=3, block_table=[0])]
    n64, n32 = packed_sizes(2, 20, 4)
    with pytest.raises(AssertionError):
        pack_verify_metadata(rows, [8], 7, 256, 2, 20, 9, 4, np.zeros(n64, np.int64), np.zeros(n32, np.int32))


@pytest.mark.parametrize("case", DRAFT_CASES)
def test_draft_block_metadata_matches_the_reference(case):
    """The draft block forward's packed metadata against the reference's draft_block_metadata (batch_metadata.py:
    99-117): anchors and mask tokens, positions, slots, context lengths and block tables, padding rows included."""
    c = {key.split("/")[2]: META[key] for key in META.files if key.startswith(f"draft/{case}/")}
    k, bs, mask, num_rows, pad, width = (int(x) for x in c["scalars"])
    rows = [RowState(length=int(n), last_token=int(t), block_table=[int(b) for b in table if b >= 0])
            for n, t, table in zip(c["lengths"], c["last_tokens"], c["tables"])]
    n64, n32 = draft_packed_sizes(num_rows, k, width)
    buf64 = np.full(n64, -7, dtype=np.int64)
    buf32 = np.full(n32, -7, dtype=np.int32)
    pack_draft_block_metadata(rows, bs, k, mask, num_rows, pad, width, buf64, buf32)
    v = draft_packed_views(buf64, buf32, num_rows, k, width)
    for key in ("input_ids", "positions", "slot_mapping", "context_lens"):
        assert v[key].tolist() == c[key].tolist(), key
    assert v["block_tables"].tolist() == c["block_tables"].tolist()
