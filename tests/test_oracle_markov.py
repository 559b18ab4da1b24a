"""Pins the Markov-rows oracle (oracle/markov.py) to the reference's DFlashDrafter._markov_rows run on CPU
(tests/golden/make_golden.py): greedy, candidate and whole-vocabulary rows."""
from pathlib import Path

import numpy as np
import pytest

from oracle import markov as OM

G = np.load(Path(__file__).parent / "golden" / "markov.npz")
NAMES = sorted({key.split("/")[1] for key in G.files if key.startswith("markov/")})


def case(name):
    prefix = f"markov/{name}/"
    return {key[len(prefix):]: G[key] for key in G.files if key.startswith(prefix)}


@pytest.mark.parametrize("name", NAMES)
def test_markov_rows_match_reference(name):
    c = case(name)
    bias = lambda prev: c["bias_a"][prev][:, None] * c["bias_c"][None, :]
    sampling = None
    if "temperature" in c:
        sampling = dict(temps=c["temperature"], top_k=c["top_k"], top_p=c["top_p"], max_top_k=int(c["max_top_k"]),
                        has_top_p=bool(c["has_top_p"]))
    drafts, probs = OM.markov_rows(c["logits"], c["prev"], bias, sampling, c.get("noise"), int(c["candidates"]))
    assert np.array_equal(drafts, c["drafts"])
    if sampling is not None:
        assert np.array_equal(probs > 0, c["probs"] > 0)
        np.testing.assert_allclose(probs, c["probs"], rtol=1e-5, atol=1e-7)


def test_num_candidates_rule():
    assert OM.num_candidates(128, True, 151936) == 192
    assert OM.num_candidates(128, False, 151936) == 0
    assert OM.num_candidates(100, True, 120) == 120


G16 = np.load(Path(__file__).parent / "golden" / "markov_bf16.npz")


@pytest.mark.parametrize("name", sorted({key.split("/")[1] for key in G16.files}))
def test_markov_rows_on_bf16_match_reference(name):
    """The production dtypes: bf16 logits + a bf16 head product, the sum rounded once to bf16 (the reference's
    bf16 add); greedy on random values, candidates on a tie-free construction."""
    from oracle.ctx_store import bf16
    prefix = f"markov_bf16/{name}/"
    c = {key[len(prefix):]: G16[key] for key in G16.files if key.startswith(prefix)}
    bias = lambda prev: bf16(c["bias_a"][prev][:, None] * c["bias_c"][None, :])   # noqa: E731
    sampling = None
    if "temperature" in c:
        sampling = dict(temps=c["temperature"], top_k=c["top_k"], top_p=c["top_p"], max_top_k=int(c["max_top_k"]),
                        has_top_p=bool(c["has_top_p"]))
    drafts, probs = OM.markov_rows(c["logits"], c["prev"], bias, sampling, c.get("noise"), int(c["candidates"]),
                                   round_fn=bf16)
    assert np.array_equal(drafts, c["drafts"])
    if sampling is not None:
        assert np.array_equal(probs > 0, c["probs"] > 0)
        np.testing.assert_allclose(probs, c["probs"], rtol=1e-5, atol=1e-7)
