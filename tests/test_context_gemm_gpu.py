"""Kernel (5), the draft context path's tcgen05 projection GEMM, against an fp32 reference of the same product.
Tolerance: bf16 outputs within one bf16 rounding of the fp32 product (plus summation-order noise)."""
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


@pytest.mark.parametrize("T,O,K", [(288, 4096, 20480), (288, 10240, 4096), (1, 128, 64), (17, 384, 192),
                                   (256, 1024, 2048), (288, 2048, 1024), (700, 512, 256)])
def test_context_gemm_matches_fp32_product(T, O, K):
    from nanovllm_b200.dflash import context_gemm
    g = torch.Generator(device=DEV).manual_seed(T + O + K)
    x = torch.randn(T, K, device=DEV, generator=g).bfloat16()
    w = (torch.randn(O, K, device=DEV, generator=g) * 0.02).bfloat16()
    out = context_gemm(x, w)
    torch.cuda.synchronize()
    ref = x.float() @ w.float().t()
    err = (out.float() - ref).abs()
    tol = ref.abs() * 2 ** -8 + 1e-3 * ref.abs().max()
    assert bool((err <= tol).all()), float((err - tol).max())
    # cuBLAS's bf16 GEMM rounds the same fp32 sums: the two differ only where summation order moves a sum across a
    # bf16 rounding boundary (about 1 % of the outputs at K = 20480)
    cublas = torch.matmul(x, w.t())
    assert float((out != cublas).float().mean()) < 0.05


def test_context_gemm_is_deterministic_and_leaves_counters_clean():
    from nanovllm_b200.dflash import context_gemm
    g = torch.Generator(device=DEV).manual_seed(5)
    x = torch.randn(288, 20480, device=DEV, generator=g).bfloat16()
    w = (torch.randn(4096, 20480, device=DEV, generator=g) * 0.01).bfloat16()
    first = context_gemm(x, w)
    for _ in range(2):
        assert torch.equal(context_gemm(x, w), first)


def test_context_gemm_workspace_shared_by_calls_of_different_shapes():
    """Calls with different output widths share one workspace zeroed once (fixed counter offsets)."""
    from nanovllm_b200.dflash import context_gemm
    g = torch.Generator(device=DEV).manual_seed(8)
    x = torch.randn(288, 4096, device=DEV, generator=g).bfloat16()
    w_small = (torch.randn(4096, 4096, device=DEV, generator=g) * 0.02).bfloat16()
    w_big = (torch.randn(10240, 4096, device=DEV, generator=g) * 0.02).bfloat16()
    ref = x.float() @ w_big.float().t()
    outs = []
    for _ in range(3):
        context_gemm(x, w_small)
        outs.append(context_gemm(x, w_big))
    torch.cuda.synchronize()
    assert all(torch.equal(o, outs[0]) for o in outs)
    err = (outs[0].float() - ref).abs()
    assert bool((err <= ref.abs() * 2 ** -8 + 1e-3 * ref.abs().max()).all())
