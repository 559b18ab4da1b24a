"""Pins the CPU oracle (oracle/spec_sampler.py) to golden vectors produced by the reference itself
(tests/golden/make_golden.py running nanovllm/layers/spec_sampler.py on CPU torch)."""
from pathlib import Path

import numpy as np
import pytest

from oracle import spec_sampler as O

GOLDEN = np.load(Path(__file__).parent / "golden" / "sampler.npz")


def cases(kind):
    names = sorted({key.split("/")[1] for key in GOLDEN.files if key.startswith(kind + "/")})
    return names


def case(kind, name):
    prefix = f"{kind}/{name}/"
    return {key[len(prefix):]: GOLDEN[key] for key in GOLDEN.files if key.startswith(prefix)}


@pytest.mark.parametrize("name", cases("accept"))
def test_accept_random_matches_reference_bit_exact(name):
    c = case("accept", name)
    n_accept, tail = O.accept_random_varlen(c["p"], c["q"], c["drafts"], c["lens"], c["u"], c["noise"])
    assert np.array_equal(n_accept, c["n_accept"])
    assert np.array_equal(tail, c["tail"])


@pytest.mark.parametrize("name", cases("accept"))
def test_fixed_length_entry_point_matches_varlen(name):
    c = case("accept", name)
    if not bool(c["fixed"]):
        pytest.skip("variable-length case")
    batch, k = c["drafts"].shape
    n_accept, tail = O.accept_random(c["p"].reshape(batch, k + 1, -1), c["q"], c["drafts"], c["u"], c["noise"])
    assert np.array_equal(n_accept, c["n_accept"]) and np.array_equal(tail, c["tail"])


@pytest.mark.parametrize("name", cases("trunc"))
def test_probs_from_logits_matches_reference(name):
    c = case("trunc", name)
    probs = O.probs_from_logits(c["logits"], c["temperature"], c["top_k"], c["top_p"], int(c["max_top_k"]),
                                bool(c["has_top_p"]))
    assert np.array_equal(probs > 0, c["probs"] > 0)            # the kept set is exact
    np.testing.assert_allclose(probs, c["probs"], rtol=1e-5, atol=1e-7)


@pytest.mark.parametrize("name", cases("logits"))
def test_fused_logits_accept_matches_reference(name):
    c = case("logits", name)
    lens = c["lens"]
    per_token = lambda v: np.repeat(v, lens)   # sampling_per_token (spec_sampler.py:44-52)
    p = O.probs_from_logits(c["logits"], per_token(c["temperature"]), per_token(c["top_k"]),
                            per_token(c["top_p"]), int(c["max_top_k"]), bool(c["has_top_p"]))
    assert np.array_equal(p > 0, c["p"] > 0)
    np.testing.assert_allclose(p, c["p"], rtol=1e-5, atol=1e-7)
    n_accept, tail = O.accept_random_varlen(p, c["q"], c["drafts"], lens, c["u"], c["noise"])
    flags = O.near_tie_flags(c["p"], c["q"], c["drafts"], lens, c["u"], c["noise"])
    keep = ~flags
    assert np.array_equal(n_accept[keep], c["n_accept"][keep])
    assert np.array_equal(tail[keep], c["tail"][keep])
    assert flags.sum() <= 1


@pytest.mark.parametrize("name", cases("greedy"))
def test_greedy_matches_reference(name):
    c = case("greedy", name)
    n_accept, tail = O.accept_greedy_varlen(c["logits"], c["drafts"], c["lens"])
    assert np.array_equal(n_accept, c["n_accept"]) and np.array_equal(tail, c["tail"])


def test_race_first_index_on_ties():
    weights = np.array([[0.0, 1.0, 1.0, 0.5]], dtype=np.float32)
    noise = np.ones((1, 4), dtype=np.float32)
    assert O.race(weights, noise).tolist() == [1]


def test_near_tie_flags_catch_an_exact_tie():
    p = np.array([[0.5, 0.5], [0.5, 0.5]], dtype=np.float32)
    q = np.array([[[0.5, 0.5]]], dtype=np.float32)
    drafts = np.array([[0]])
    u = np.array([[1.0]], dtype=np.float32)            # u * q_d == p_d: the accept test is on the knife edge
    noise = np.ones((1, 2), dtype=np.float32)
    assert O.near_tie_flags(p, q, drafts, np.array([2]), u, noise).tolist() == [True]


EDGES = np.load(Path(__file__).parent / "golden" / "sampler_edges.npz")


def edge_cases(kind):
    return sorted({key.split("/")[1] for key in EDGES.files if key.startswith(kind + "/")})


@pytest.mark.parametrize("name", edge_cases("masked"))
def test_masked_vocabulary_accept_matches_reference(name):
    """Rows with fewer finite logits than top_k (the rest -inf): probabilities, the kept set and the accept
    against the reference's own outputs (the kernel is held to the oracle on such rows by the GPU tests)."""
    prefix = f"masked/{name}/"
    c = {key[len(prefix):]: EDGES[key] for key in EDGES.files if key.startswith(prefix)}
    lens = c["lens"]
    per_token = lambda v: np.repeat(v, lens)   # noqa: E731  (sampling_per_token, spec_sampler.py:44-52)
    p = O.probs_from_logits(c["logits"], per_token(c["temperature"]), per_token(c["top_k"]),
                            per_token(c["top_p"]), int(c["max_top_k"]), bool(c["has_top_p"]))
    assert np.array_equal(p > 0, c["p"] > 0)
    np.testing.assert_allclose(p, c["p"], rtol=1e-5, atol=1e-7)
    n_accept, tail = O.accept_random_varlen(p, c["q"], c["drafts"], lens, c["u"], c["noise"])
    keep = ~O.near_tie_flags(c["p"], c["q"], c["drafts"], lens, c["u"], c["noise"])
    assert keep.sum() >= len(lens) - 1
    assert np.array_equal(n_accept[keep], c["n_accept"][keep])
    assert np.array_equal(tail[keep], c["tail"][keep])


@pytest.mark.parametrize("name", edge_cases("greedy_edge"))
def test_greedy_ties_and_infinities_match_reference(name):
    """Tied maxima (first index), +inf maxima, an all -inf row and a constant row, as the reference decides
    them (the kernel is held to the oracle on the same construction by the GPU tests)."""
    prefix = f"greedy_edge/{name}/"
    c = {key[len(prefix):]: EDGES[key] for key in EDGES.files if key.startswith(prefix)}
    batch, k = c["drafts"].shape
    n_accept, tail = O.accept_greedy_varlen(c["logits"], c["drafts"], np.full(batch, k + 1))
    assert np.array_equal(n_accept, c["n_accept"]) and np.array_equal(tail, c["tail"])


@pytest.mark.parametrize("name", cases("logits"))
def test_host_sampling_tensors_match_reference(name):
    """sampling_tensors / sampling_per_token (the host bookkeeping feeding the kernels) give the reference's
    per-row tensors and host flags for the same per-request parameters, on CPU."""
    import torch
    from types import SimpleNamespace
    from nanovllm_b200 import spec_sampler as S
    c = case("logits", name)
    seqs = [SimpleNamespace(temperature=float(t), top_k=int(k), top_p=float(p))
            for t, k, p in zip(c["temperature"], c["top_k"], c["top_p"])]
    samp = S.sampling_tensors(seqs, torch.device("cpu"))
    assert np.array_equal(samp.temperatures.numpy(), c["temperature"])
    assert np.array_equal(samp.top_k.numpy(), c["top_k"]) and np.array_equal(samp.top_p.numpy(), c["top_p"])
    assert (samp.max_top_k, samp.has_top_p) == (int(c["max_top_k"]), bool(c["has_top_p"]))
    lens = torch.from_numpy(c["lens"])
    per = S.sampling_per_token(samp, lens, int(lens.sum()))
    assert np.array_equal(per.top_k.numpy(), np.repeat(c["top_k"], c["lens"]))
    assert np.array_equal(per.temperatures.numpy(), np.repeat(c["temperature"], c["lens"]))
    with pytest.raises(ValueError):                     # the reference rejects mixed greedy and random rows
        S.sampling_tensors(seqs + [SimpleNamespace(temperature=0.0, top_k=0, top_p=1.0)], torch.device("cpu"))
