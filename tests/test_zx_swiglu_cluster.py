"""Cluster split-K decode GEMM with the SwiGLU epilogue (each tile pairs 64 gate
rows with the matching 64 up rows; SwiGLU after the DSMEM reduction), against
a plain fp32 torch reference, and against the split-K SwiGLU GEMM."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("T,K,I", [(1, 2048, 768), (16, 4096, 1536), (64, 2048, 6144), (128, 1024, 512),
                                   (37, 512, 192)])
@pytest.mark.parametrize("cs", [0, 1, 4])
def test_swiglu_cluster_matches_fp32(cuda, T, K, I, cs):
    from mod_b200.ops import check_status, native

    if cs and (K // 64) // cs < 1:
        pytest.skip("fewer K blocks than CTAs")
    torch.manual_seed(T + K + I + cs)
    x = torch.randn(T, K, device=cuda).bfloat16()
    w = (torch.randn(2 * I, K, device=cuda) * 0.02).bfloat16()
    y = native.swiglu_cluster(x, w, cs=cs)
    g = x.float() @ w[:I].float().t()
    u = x.float() @ w[I:].float().t()
    ref = torch.nn.functional.silu(g) * u
    torch.cuda.synchronize()
    check_status()
    torch.testing.assert_close(y.float(), ref, rtol=2e-2, atol=2e-2 * max(1.0, ref.abs().max().item()) / 8)
    if I % 128 == 0 and T <= 128:  # the split-K dual-accumulator form gives the same values
        y2 = native.swiglu_linear(x, w)
        torch.testing.assert_close(y.float(), y2.float(), rtol=2e-2, atol=2e-2 * max(1.0, ref.abs().max().item()) / 8)
