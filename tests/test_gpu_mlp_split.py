"""The fp32 policy layer of the fused rollout on the tensor cores (operands split into three
bf16 words, six cross products on tcgen05 kind::f16, fp32 accumulation in TMEM;
g1_dense_bf16x3) against an fp64 matmul.

Gate: fp32-class accuracy -- per element |out - ref64| <= 1e-6 * (|X| |W|^T) + 1e-7, and the
largest error no worse than 2x that of torch's fp32 matmul on the same inputs (+1e-7)."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _ref(X, W, b, act):
    y = X.double() @ W.double().T + (b.double() if b is not None else 0)
    if act == 0:
        y = torch.tanh(y)
    elif act == 1:
        y = torch.nn.functional.elu(y)
    return y


@pytest.mark.parametrize("rows,K,N,act", [
    (56, 100, 256, -1), (56, 256, 256, -1), (56, 256, 32, -1), (64, 256, 256, 0), (56, 256, 256, 1),
    (1, 16, 16, -1), (37, 40, 48, -1), (64, 200, 128, 1), (13, 7, 64, 0), (56, 256, 32, 0),
])
def test_dense_bf16x3(rows, K, N, act):
    import g1env
    g = torch.Generator(device="cuda").manual_seed(rows * 1000 + K + N)
    X = torch.randn(rows, K, device="cuda", generator=g) * 2
    W = torch.randn(N, K, device="cuda", generator=g) / K ** 0.5
    b = torch.randn(N, device="cuda", generator=g) * 0.1
    out = g1env.dense_bf16x3(X, W, b, act)
    ref = _ref(X, W, b, act)
    scale = (X.double().abs() @ W.double().abs().T)
    err = (out.double() - ref).abs()
    assert torch.isfinite(out).all()
    assert (err <= 1e-6 * scale + 1e-7).all(), float((err - 1e-6 * scale).max())
    f32 = X @ W.T + b
    if act == 0:
        f32 = torch.tanh(f32)
    elif act == 1:
        f32 = torch.nn.functional.elu(f32)
    e32 = (f32.double() - ref).abs().max().item()
    assert err.max().item() <= 2 * e32 + 1e-7, (err.max().item(), e32)
