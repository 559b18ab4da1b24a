"""oracle/forward.py (the numpy Qwen3 verify forward) against the reference's Qwen3ForCausalLM run on the inputs
of tests/golden/qwen3_case.py (fixture tests/golden/qwen3.npz, written by tests/golden/make_golden.py): the
stored K/V rows, the aux layers' outputs, the hidden states after the final norm and the logits.

Tolerance: the reference's CPU bf16 GEMMs round once like the oracle's fp32 products but sum in another order, so
a value may land one bf16 step away, and from the second layer on those steps mix through the GEMMs.  The first
layer's stored K/V: 99.9 % within one bf16 ulp.  Everything after it: relative Frobenius error at most 1e-2 (one
bf16 rounding of random sign is ~2e-3) and every value within 3e-2 of the output's largest magnitude."""
import sys
from pathlib import Path

import numpy as np
import pytest

HERE = Path(__file__).parent
sys.path.insert(0, str(HERE / "golden"))
import qwen3_case as Q  # noqa: E402

from oracle import ctx_store as OC  # noqa: E402
from oracle import forward as OF  # noqa: E402

G = np.load(HERE / "golden" / "qwen3.npz")


def within_ulp(got, want, frac=0.999):
    ok = np.abs(got - want) <= 2.0 ** -7 * np.maximum(np.abs(got), np.abs(want)) + 1e-6
    assert ok.mean() >= frac, f"{(~ok).sum()} of {ok.size} beyond one bf16 ulp"


def close(got, want, rel=1e-2, atol_scale=3e-2):
    err = float(np.linalg.norm(got - want) / np.linalg.norm(want))
    assert err <= rel, err
    np.testing.assert_allclose(got, want, atol=atol_scale * np.abs(want).max(), rtol=0)


def oracle_run(case):
    f = lambda t: t.float().numpy()                            # noqa: E731
    layers = [{key: f(value) for key, value in w.items()} for w in case["layers"]]
    caches = [(f(k).copy(), f(v).copy()) for k, v in case["caches"]]
    n = len(Q.KEY_LENS)
    q_starts = np.arange(n) * Q.QUERY_LEN
    cos_sin = OC.rope_cache(Q.HEAD_DIM, Q.MAX_POSITION, Q.ROPE_THETA)
    hidden, aux = OF.forward(f(case["embed"]), layers, f(case["final_norm"]), case["input_ids"].numpy(),
                             case["positions"].numpy(), case["slot_mapping"].numpy(), caches, case["tables"].numpy(),
                             q_starts, [Q.QUERY_LEN] * n, list(Q.KEY_LENS), cos_sin, Q.HEADS, Q.KV_HEADS, Q.EPS,
                             aux_layer_ids=Q.AUX_LAYER_IDS)
    logits = OF.compute_logits(hidden, f(case["lm_head"]))
    return hidden, aux, logits, caches


def test_regenerated_inputs_are_the_ones_the_reference_ran_on():
    assert np.allclose(Q.checksums(Q.inputs()), G["qwen3/checksums"], rtol=0, atol=0)


def test_oracle_forward_matches_the_reference():
    case = Q.inputs()
    hidden, aux, logits, caches = oracle_run(case)
    slots = case["slot_mapping"].numpy()
    for i, (k_cache, v_cache) in enumerate(caches):
        k_got = k_cache.reshape(-1, Q.KV_HEADS, Q.HEAD_DIM)[slots]
        v_got = v_cache.reshape(-1, Q.KV_HEADS, Q.HEAD_DIM)[slots]
        if i == 0:
            within_ulp(k_got, G[f"qwen3/k_stored{i}"])
            within_ulp(v_got, G[f"qwen3/v_stored{i}"])
        close(k_got, G[f"qwen3/k_stored{i}"])
        close(v_got, G[f"qwen3/v_stored{i}"])
    close(aux, G["qwen3/aux"])
    close(hidden, G["qwen3/hidden"])
    close(logits, G["qwen3/logits"])
    # the greedy tokens too, wherever the reference's top two logits are more than a few ulps apart
    want = G["qwen3/logits"]
    top2 = np.sort(want, axis=-1)[:, -2:]
    clear = (top2[:, 1] - top2[:, 0]) > 4 * 2.0 ** -7 * np.abs(top2[:, 1])
    assert clear.sum() >= len(clear) // 2
    assert np.array_equal(np.argmax(logits, -1)[clear], np.argmax(want, -1)[clear])
