"""Pins the attention oracle (oracle/attention.py) to the reference's own paged-attention stand-in
(tests/fake_paged_attention.py in the reference, run by tests/golden/make_golden.py): the K/V store by slot
(-1 skipped) and SDPA over the keys gathered through the block table, in the decode layout, causal (queries at
the end of the context: the verify rule) and not (the DFlash draft block).  fp32 on fp16-exact inputs; the store
bit-exact, the outputs within 1e-5."""
from pathlib import Path

import numpy as np
import pytest

from oracle import attention as OA

GOLDEN = np.load(Path(__file__).parent / "golden" / "attention.npz")
NAMES = sorted({key.split("/")[1] for key in GOLDEN.files})


@pytest.mark.parametrize("name", NAMES)
def test_store_and_paged_attention_match_reference(name):
    prefix = f"attention/{name}/"
    c = {key[len(prefix):]: GOLDEN[key] for key in GOLDEN.files if key.startswith(prefix)}
    f32 = lambda a: a.astype(np.float32)   # noqa: E731
    k_cache, v_cache = f32(c["k_cache_in"]), f32(c["v_cache_in"])
    slots = c["slots"].astype(np.int64)
    OA.store_kvcache(f32(c["k"]), f32(c["v"]), k_cache, v_cache, slots)
    Hkv, D = k_cache.shape[2], k_cache.shape[3]
    stored = slots[slots >= 0]
    assert np.array_equal(k_cache.reshape(-1, Hkv, D)[stored], f32(c["k_stored"]))
    assert np.array_equal(v_cache.reshape(-1, Hkv, D)[stored], f32(c["v_stored"]))
    lens = c["context_lens"].astype(np.int64)
    q_per = int(c["q_per_seq"])
    R = len(lens)
    out = OA.paged_attention(f32(c["q"]), k_cache, v_cache, c["tables"], np.arange(R) * q_per, np.full(R, q_per),
                             lens, D ** -0.5, bool(c["causal"]))
    np.testing.assert_allclose(out, c["out"], atol=1e-5, rtol=1e-5)
