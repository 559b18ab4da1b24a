"""Host logic of the round (nanovllm_b200/speculative.py) on CPU: the variable-length graphs' token counts
(verify_schedule.py:18-23), the choice of the graph a round's rows fit (speculative.py:503-506), the sampling
graph key (speculative.py:53-57) and the draft placement of verified drafts (batch_metadata.py:135-136)."""
from types import SimpleNamespace

import numpy as np
import pytest

from nanovllm_b200.batch_metadata import draft_placement
from nanovllm_b200.speculative import VerifyRound, sampling_graph_key, verify_token_counts


def test_token_counts_are_the_small_sizes_then_every_multiple_of_the_query_length():
    assert verify_token_counts(4, 8) == [1, 2, 4, 8, 16, 24, 32]
    assert verify_token_counts(3, 2) == [1, 2, 4, 6]
    assert verify_token_counts(2, 4) == [1, 2, 4, 8]
    counts = verify_token_counts(64, 8)
    assert counts[-1] == 512 and len(counts) == 3 + 64
    # B rows of at most query_len tokens always fit the graph of B * query_len tokens
    for rows in range(1, 65):
        assert rows * 8 in counts


def chooser(shapes, k=7):
    """VerifyRound.graph_for on a bare object holding only the graph shapes (tokens -> row slots)."""
    rnd = object.__new__(VerifyRound)
    rnd.num_drafts, rnd.shapes = k, shapes
    return rnd.graph_for


@pytest.mark.parametrize("rows,verified,want", [
    (64, 280, 280), (64, 281, 288), (64, 512, 512), (1, 1, 1), (2, 3, 4), (64, 64, 64)])
def test_the_smallest_graph_holding_the_rows_is_chosen(rows, verified, want):
    shapes = {t: min(t, 512) for t in verify_token_counts(64, 8)}
    assert chooser(shapes)(rows, verified) == want


def test_padding_rows_must_hold_the_tokens_left():
    # fixed-length graphs (B slots of 8 tokens): 3 rows of 8 tokens leave one padding row of 8 in the 32-token
    # graph; 3 rows verifying only 10 tokens would leave 22 (or 54) tokens for 1 (or 5) padding rows of at most 8:
    # no fixed-length graph holds them (variable-length rounds use the token-count graphs)
    graph_for = chooser({32: 4, 64: 8})
    assert graph_for(3, 24) == 32
    assert graph_for(4, 32) == 32
    assert graph_for(5, 40) == 64
    with pytest.raises(ValueError):
        graph_for(3, 10)
    with pytest.raises(ValueError):
        graph_for(9, 72)


def test_sampling_graph_key_follows_the_host_flags():
    greedy = SimpleNamespace(temperatures=None, max_top_k=0, has_top_p=False, all_top_k=False)
    assert sampling_graph_key(greedy) is None
    rnd = SimpleNamespace(temperatures=object(), max_top_k=128, has_top_p=True, all_top_k=True)
    assert sampling_graph_key(rnd) == (128, True, True)


def test_draft_placement_puts_each_rows_drafts_after_its_last_token():
    index, source = draft_placement([3, 1, 8, 2], 7)
    # row 0: tokens 0-2 (drafts 0, 1 at 1, 2); row 1: token 3 (none); row 2: tokens 4-11; row 3: tokens 12-13
    assert index.tolist() == [1, 2] + list(range(5, 12)) + [13]
    assert source.tolist() == [0, 1] + list(range(14, 21)) + [21]
    empty = draft_placement([], 7)
    assert empty[0].shape == (0,) and empty[1].shape == (0,)
    assert np.all(np.diff(draft_placement([8] * 5, 7)[0]) >= 1)
