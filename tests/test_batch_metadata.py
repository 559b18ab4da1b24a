"""Verification metadata (nanovllm/engine/batch_metadata.py:149-181): the packed array builder a round copies to
the device gives exactly the values of the list builder that mirrors the reference, for fixed and variable
verified lengths, padding rows and ragged block tables."""
import random

import numpy as np
import pytest

from nanovllm_b200.batch_metadata import (PAD_SLOT, RowState, pack_verify_metadata, packed_sizes, packed_views,
                                          verify_varlen_metadata)


def build_case(seed):
    rng = random.Random(seed)
    k, block_size, width = 7, 256, 8
    n = rng.randint(0, 12)
    rows, lens = [], []
    next_block = 0
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
def test_packed_metadata_equals_the_list_builder(seed):
    rows, lens, k, bs, num_rows, num_tokens, pad, width = build_case(seed)
    m = verify_varlen_metadata(rows, lens, k, bs, num_rows, num_tokens, pad, width)
    n64, n32 = packed_sizes(num_rows, num_tokens, width)
    buf64 = np.full(n64, -7, dtype=np.int64)
    buf32 = np.full(n32, -7, dtype=np.int32)
    pack_verify_metadata(rows, lens, k, bs, num_rows, num_tokens, pad, width, buf64, buf32)
    v = packed_views(buf64, buf32, num_rows, num_tokens, width)
    assert v["input_ids"].tolist() == m.input_ids
    assert v["positions"].tolist() == m.positions
    assert v["slot_mapping"].tolist() == m.slot_mapping
    assert v["cu_seqlens_q"].tolist() == m.cu_seqlens_q
    assert v["cu_seqlens_k"].tolist() == m.cu_seqlens_k
    assert v["block_tables"].tolist() == m.block_tables
    assert (v["slot_mapping"][sum(lens):] == PAD_SLOT).all()


def test_packed_metadata_rejects_overfull_padding():
    rows = [RowState(length=10, last_token=3, block_table=[0])]
    n64, n32 = packed_sizes(2, 20, 4)
    with pytest.raises(AssertionError):
        pack_verify_metadata(rows, [8], 7, 256, 2, 20, 9, 4, np.zeros(n64, np.int64), np.zeros(n32, np.int32))


META = np.load(__import__("pathlib").Path(__file__).parent / "golden" / "metadata.npz")


@pytest.mark.parametrize("case", sorted({key.split("/")[1] for key in META.files}))
def test_list_builder_matches_the_reference(case):
    """The list builder against the reference's verify_varlen_metadata run on the same batches
    (tests/golden/make_golden.py): every list, padding rows and empty row slots included."""
    c = {key.split("/")[2]: META[key] for key in META.files if key.startswith(f"meta/{case}/")}
    k, bs, num_rows, num_tokens, pad, width = (int(x) for x in c["scalars"])
    rows = [RowState(length=int(n), last_token=int(t), block_table=[int(b) for b in table if b >= 0])
            for n, t, table in zip(c["lengths"], c["last_tokens"], c["tables"])]
    m = verify_varlen_metadata(rows, [int(x) for x in c["verified_lens"]], k, bs, num_rows, num_tokens, pad, width)
    for key in ("input_ids", "positions", "slot_mapping", "cu_seqlens_q", "cu_seqlens_k", "draft_index",
                "draft_source"):
        assert getattr(m, key) == c[key].tolist(), key
    assert m.block_tables == c["block_tables"].tolist()
