"""B200-native verify/accept hot path of nano-vllm-speculative-decoding.

Python mirrors of the reference's interfaces on top of libspecdec_b200.so (a C-ABI library of sm_100a CUDA
kernels, built by nano-vllm-speculative-decoding_b200/build.py):

    nanovllm_b200.spec_sampler    nanovllm/layers/spec_sampler.py          batched rejection sampler (kernel 1)
    nanovllm_b200.attention       nanovllm/layers/attention.py             paged verify / draft-block attention (kernel 2)
    nanovllm_b200.context         nanovllm/utils/context.py                the attention context record
    nanovllm_b200.markov          speculative.py _markov_rows + MarkovHead DSpark in-block Markov rows (kernel 3)
    nanovllm_b200.dflash          nanovllm/models/dflash.py                draft model, context features, ctx_store (kernel 4)
    nanovllm_b200.fused           nanovllm/layers/{layernorm,activation}   RMSNorm, SiLU*mul, q/k norm + RoPE + KV store
    nanovllm_b200.target          nanovllm/models/qwen3.py                 Qwen3 verify forward (graphs per token count)
    nanovllm_b200.batch_metadata  nanovllm/engine/batch_metadata.py        packed verification metadata
    nanovllm_b200.speculative     nanovllm/engine/speculative.py           the verify + accept round, fixed or varlen
    nanovllm_b200.tp_attention    qwen3.py head split + model_runner.py    KV-head tensor-parallel verify attention
    nanovllm_b200.replicas        (bench plumbing)                         row-sharded replicas: barrier, reductions
"""
from . import _lib  # noqa: F401

__all__ = ["_lib"]
