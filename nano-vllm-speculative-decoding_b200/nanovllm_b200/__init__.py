"""B200-native verify/accept hot path of nano-vllm-speculative-decoding.

Python mirrors of the reference's interfaces on top of libspecdec_b200.so (a C-ABI library of sm_100a CUDA
kernels, built by nano-vllm-speculative-decoding_b200/build.py):

    nanovllm_b200.spec_sampler   nanovllm/layers/spec_sampler.py   batched rejection sampler (kernel 1)
"""
from . import _lib  # noqa: F401

__all__ = ["_lib"]
