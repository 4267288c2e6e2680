"""The tcgen05 dense layer (g1_gemm_bf16_tc) against a torch fp32 reference of the same op on
the same bf16 inputs.  Only the accumulation order differs (fp32 accumulators in tensor
memory), so the tolerance is 1e-5 relative to the output scale, plus the activation."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (200, 256, 100), (57, 30, 256), (300, 1024, 1024), (1000, 512, 1024)])
@pytest.mark.parametrize("act", [-1, 0, 1])
def test_dense_tc_matches_fp32(M, N, K, act):
    import g1env
    g = torch.Generator(device="cpu").manual_seed(M * 7 + N + K)
    X = torch.randn(M, K, generator=g).to(torch.bfloat16).cuda()
    W = (torch.randn(N, K, generator=g) / K ** 0.5).to(torch.bfloat16).cuda()
    b = torch.randn(N, generator=g).cuda()
    out = g1env.gemm_bf16_tc(X, W, b, act)
    ref = X.float() @ W.float().T + b
    if act == 0:
        ref = torch.tanh(ref)
    elif act == 1:
        ref = torch.nn.functional.elu(ref)
    err = (out - ref).abs().max().item()
    assert err <= 1e-5 * max(1.0, ref.abs().max().item()) + 1e-5, err
