"""Pins the ctx_store / q-norm-RoPE oracle (oracle/ctx_store.py) to the reference's own
DFlashDraftModel.store_context_kv and Qwen3Attention q path run on CPU (tests/golden/make_golden.py)."""
from pathlib import Path

import numpy as np

from oracle import ctx_store as OC

G = np.load(Path(__file__).parent / "golden" / "ctx_store.npz")
BF16_ULP = 2.0 ** -7   # relative spacing of bf16 values


def within_one_bf16_ulp(got, want):
    return np.abs(got - want) <= BF16_ULP * np.maximum(np.abs(want), np.abs(got)) + 1e-6


def oracle_cache():
    features, w_kv, k_norm = G["ctx/features"], G["ctx/w_kv"], G["ctx/k_norm"]
    cache = np.zeros_like(G["ctx/kv_cache"])
    cos_sin = OC.rope_cache(128, int(G["ctx/max_position"]), float(G["ctx/rope_base"]))
    layers = k_norm.shape[0]
    width = w_kv.shape[0] // layers
    for layer in range(layers):
        kv = OC.bf16(features @ w_kv[layer * width:(layer + 1) * width].T)
        OC.norm_rope_store(kv, 2, k_norm[layer], cos_sin, G["ctx/positions"], G["ctx/slots"], cache[0, layer],
                           cache[1, layer], float(G["ctx/eps"]))
    return cache


def test_rope_cache_matches_reference_table():
    # the cos|sin table the reference builds in fp32 (rotary_embedding.py:17-27): numpy's float32 cos/sin differ
    # from torch's by a few 1e-6 at large angles, far below bf16 resolution (the product builds it with torch)
    import torch
    inv_freq = 1.0 / (1000000.0 ** (torch.arange(0, 128, 2, dtype=torch.float) / 128))
    t = torch.arange(64, dtype=torch.float)
    freqs = torch.einsum("i,j -> ij", t, inv_freq)
    want = torch.cat((freqs.cos(), freqs.sin()), dim=-1).numpy()
    got = OC.rope_cache(128, 64, 1000000.0)
    np.testing.assert_allclose(got, want, rtol=0, atol=1e-5)


def test_store_context_kv_matches_reference():
    got, want = oracle_cache(), G["ctx/kv_cache"]
    ok = within_one_bf16_ulp(got, want)
    assert ok.mean() > 0.999, f"{(~ok).sum()} entries beyond one bf16 ulp"
    np.testing.assert_allclose(got, want, atol=2e-2, rtol=0)
    # slots of padding rows (-1) were never written: the untouched cache stays zero in both
    written = np.zeros(want.shape[2] * want.shape[3], dtype=bool)
    written[G["ctx/slots"][G["ctx/slots"] >= 0]] = True
    assert not want[:, :, ~written.reshape(want.shape[2], want.shape[3])].any()


def test_q_norm_rope_matches_reference():
    cos_sin = OC.rope_cache(128, int(G["ctx/max_position"]), float(G["ctx/rope_base"]))
    got = OC.q_norm_rope(G["ctx/q"], G["ctx/q_norm"], cos_sin, G["ctx/positions"], float(G["ctx/eps"]))
    ok = within_one_bf16_ulp(got, G["ctx/q_out"])
    assert ok.mean() > 0.999
    np.testing.assert_allclose(got, G["ctx/q_out"], atol=2e-2, rtol=0)


F = np.load(Path(__file__).parent / "golden" / "forward.npz")


def test_rmsnorm_matches_reference():
    """layernorm.py rms_forward / add_rms_forward: the residual sum bit-exact, the normed rows within one bf16 ulp
    (fp32 rsqrt of the variance may differ in its last bits)."""
    x, r, w, eps = F["forward/x"], F["forward/residual"], F["forward/weight"], float(F["forward/eps"])
    got = OC.rmsnorm(x, w, eps)
    assert within_one_bf16_ulp(got, F["forward/y"]).all()
    s = OC.bf16(x + r)
    assert np.array_equal(s, F["forward/res_out"])
    assert within_one_bf16_ulp(OC.rmsnorm(x + r, w, eps), F["forward/y_res"]).all()


def test_silu_and_mul_matches_reference():
    got = OC.silu_and_mul(F["forward/gate_up"])
    ok = within_one_bf16_ulp(got, F["forward/act"])
    assert ok.all(), f"{(~ok).sum()} entries beyond one bf16 ulp"
