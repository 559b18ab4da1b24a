"""The B200 Qwen3 verify forward (nanovllm_b200.target.Qwen3Target.forward: cuBLAS GEMMs, this library's RMSNorm,
q/k norm + RoPE + paged K/V store, tcgen05 paged attention and SiLU * mul) against the reference's
Qwen3ForCausalLM run on the same inputs (tests/golden/qwen3.npz, from tests/golden/make_golden.py over
tests/golden/qwen3_case.py), with the tolerance tests/test_oracle_forward.py states for the oracle: the first
layer's stored K/V 99.9 % within one bf16 ulp; everything after it within 1e-2 relative Frobenius error and 3e-2
of the output's largest magnitude (bf16 roundings of other summation orders mixing through the layers)."""
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

HERE = Path(__file__).parent
sys.path.insert(0, str(HERE / "golden"))
import qwen3_case as Q  # noqa: E402

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
G = np.load(HERE / "golden" / "qwen3.npz")


def within_ulp(got, want, frac=0.999):
    ok = np.abs(got - want) <= 2.0 ** -7 * np.maximum(np.abs(got), np.abs(want)) + 1e-6
    assert ok.mean() >= frac, f"{(~ok).sum()} of {ok.size} beyond one bf16 ulp"


def close(got, want, rel=1e-2, atol_scale=3e-2):
    err = float(np.linalg.norm(got - want) / np.linalg.norm(want))
    assert err <= rel, err
    np.testing.assert_allclose(got, want, atol=atol_scale * np.abs(want).max(), rtol=0)


def test_b200_forward_matches_the_reference_qwen3():
    from nanovllm_b200.target import Qwen3Shape, Qwen3Target
    case = Q.inputs()
    assert np.allclose(Q.checksums(case), G["qwen3/checksums"], rtol=0, atol=0)
    shape = Qwen3Shape(hidden=Q.HIDDEN, layers=Q.LAYERS, heads=Q.HEADS, kv_heads=Q.KV_HEADS, head_dim=Q.HEAD_DIM,
                       intermediate=Q.FFN, vocab=Q.VOCAB, eps=Q.EPS, rope_theta=Q.ROPE_THETA,
                       max_position=Q.MAX_POSITION, aux_layer_ids=Q.AUX_LAYER_IDS)
    num_blocks = case["caches"][0][0].shape[0] - 1              # the pad block is the cache's last
    target = Qwen3Target(shape, DEV, num_blocks, Q.BLOCK)
    target.embed = case["embed"].to(DEV)
    target.final_norm = case["final_norm"].to(DEV)
    target.lm_head = case["lm_head"].to(DEV)
    target.layers = [{key: value.to(DEV) for key, value in w.items()} for w in case["layers"]]
    for i, (k_cache, v_cache) in enumerate(case["caches"]):
        target.kv_cache[0, i].copy_(k_cache)
        target.kv_cache[1, i].copy_(v_cache)
    n = len(Q.KEY_LENS)
    cu_q = torch.arange(0, Q.QUERY_LEN * (n + 1), Q.QUERY_LEN, dtype=torch.int32, device=DEV)
    cu_k = torch.tensor([0] + np.cumsum(Q.KEY_LENS).tolist(), dtype=torch.int32, device=DEV)
    T = case["input_ids"].shape[0]
    aux = torch.zeros(T, len(Q.AUX_LAYER_IDS) * Q.HIDDEN, dtype=torch.bfloat16, device=DEV)
    slots = case["slot_mapping"].to(DEV)
    hidden = target.forward(case["input_ids"].to(DEV), case["positions"].to(DEV), slots, cu_q, cu_k, Q.QUERY_LEN,
                            case["tables"].to(DEV), aux_out=aux)
    logits = target.compute_logits(hidden)
    torch.cuda.synchronize()
    for i in range(Q.LAYERS):
        k_got = target.kv_cache[0, i].reshape(-1, Q.KV_HEADS, Q.HEAD_DIM)[slots.long()].float().cpu().numpy()
        v_got = target.kv_cache[1, i].reshape(-1, Q.KV_HEADS, Q.HEAD_DIM)[slots.long()].float().cpu().numpy()
        if i == 0:
            within_ulp(k_got, G[f"qwen3/k_stored{i}"])
            within_ulp(v_got, G[f"qwen3/v_stored{i}"])
        close(k_got, G[f"qwen3/k_stored{i}"])
        close(v_got, G[f"qwen3/v_stored{i}"])
    close(aux.float().cpu().numpy(), G["qwen3/aux"])
    close(hidden.float().cpu().numpy(), G["qwen3/hidden"])
    got_logits = logits.float().cpu().numpy()
    want = G["qwen3/logits"]
    close(got_logits, want)
    top2 = np.sort(want, axis=-1)[:, -2:]
    clear = (top2[:, 1] - top2[:, 0]) > 4 * 2.0 ** -7 * np.abs(top2[:, 1])
    assert np.array_equal(np.argmax(got_logits, -1)[clear], np.argmax(want, -1)[clear])
    target.close()
