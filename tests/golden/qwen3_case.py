"""The inputs of the golden Qwen3 verify-forward case (tests/golden/qwen3.npz), regenerated from fixed seeds with
torch's CPU generator, so the fixture holds only the reference's outputs and checksums of these inputs.

A small Qwen3 (hidden 128, 2 layers, 4 query heads / 1 KV head of 128 - the GQA group of 4 the B200 attention
packs -, FFN 256, vocabulary 500) with random bf16 weights, paged KV caches [blocks, 256, 1, 128] holding
random contexts, and three rows verifying 8 tokens each at the end of contexts of 300, 129 and 260 keys (block
tables shuffled, the last block the zeroed pad block).  Imported by make_golden.py (which runs the reference on
it) and by the tests (which run the oracle and the B200 forward on it)."""
from __future__ import annotations

import torch

HIDDEN, LAYERS, HEADS, KV_HEADS, HEAD_DIM, FFN, VOCAB = 128, 2, 4, 1, 128, 256, 500
EPS, ROPE_THETA, MAX_POSITION, BLOCK = 1e-6, 1000000.0, 4096, 256
AUX_LAYER_IDS = (0, 1)
KEY_LENS = (300, 129, 260)       # keys per row, the last 8 being the verified tokens
QUERY_LEN = 8


def inputs() -> dict:
    """Weights (bf16), caches (bf16, contexts filled, pad block zero), the rows' metadata (verify layout)."""
    g = torch.Generator().manual_seed(2024)

    def rand(*shape, scale=0.05):
        return (torch.randn(*shape, generator=g) * scale).bfloat16()

    def norm_weight(n):
        return (1.0 + 0.1 * torch.randn(n, generator=g)).bfloat16()

    layers = []
    for _ in range(LAYERS):
        layers.append(dict(
            w_qkv=rand((HEADS + 2 * KV_HEADS) * HEAD_DIM, HIDDEN), w_o=rand(HIDDEN, HEADS * HEAD_DIM),
            w_gate_up=rand(2 * FFN, HIDDEN), w_down=rand(HIDDEN, FFN), in_norm=norm_weight(HIDDEN),
            post_norm=norm_weight(HIDDEN), q_norm=norm_weight(HEAD_DIM), k_norm=norm_weight(HEAD_DIM)))
    embed = rand(VOCAB, HIDDEN, scale=1.0)
    final_norm = norm_weight(HIDDEN)
    lm_head = rand(VOCAB, HIDDEN)
    blocks = [-(-n // BLOCK) for n in KEY_LENS]
    num_blocks = sum(blocks) + 1                                   # + the pad block, last
    perm = torch.randperm(num_blocks - 1, generator=g).tolist()
    tables = torch.full((len(KEY_LENS), max(blocks)), num_blocks - 1, dtype=torch.int32)
    used = 0
    for r, nb in enumerate(blocks):
        tables[r, :nb] = torch.tensor(perm[used:used + nb], dtype=torch.int32)
        used += nb
    caches = []
    for _ in range(LAYERS):
        k_cache = torch.randn(num_blocks, BLOCK, KV_HEADS, HEAD_DIM, generator=g).bfloat16()
        v_cache = torch.randn(num_blocks, BLOCK, KV_HEADS, HEAD_DIM, generator=g).bfloat16()
        k_cache[-1].zero_()
        v_cache[-1].zero_()
        caches.append((k_cache, v_cache))
    positions, slots = [], []
    for r, n in enumerate(KEY_LENS):
        for p in range(n - QUERY_LEN, n):
            positions.append(p)
            slots.append(int(tables[r, p // BLOCK]) * BLOCK + p % BLOCK)
    input_ids = torch.randint(VOCAB, (len(positions),), generator=g)
    return dict(layers=layers, embed=embed, final_norm=final_norm, lm_head=lm_head, caches=caches, tables=tables,
                positions=torch.tensor(positions), slot_mapping=torch.tensor(slots, dtype=torch.int32),
                input_ids=input_ids, key_lens=torch.tensor(KEY_LENS, dtype=torch.int32))


def checksums(case: dict) -> list[float]:
    """Sums of every input tensor in a fixed order (float64), stored in the fixture so a test notices when its
    regenerated inputs are not the ones the reference ran on."""
    tensors = [case["embed"], case["final_norm"], case["lm_head"], case["tables"], case["positions"],
               case["slot_mapping"], case["input_ids"]]
    for w in case["layers"]:
        tensors += [w[key] for key in sorted(w)]
    for k_cache, v_cache in case["caches"]:
        tensors += [k_cache, v_cache]
    return [float(t.double().sum()) for t in tensors]
