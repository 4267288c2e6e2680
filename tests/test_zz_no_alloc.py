"""g1_rollout_noalloc: the rollout entry point that allocates no device memory, for callers
that cannot allocate on their hot path (e.g. a host framework that owns all device memory or
has reserved its budget up front, or code running while a stream is being captured).  It
keeps the repacked policy weights in a fixed device area of the library instead of an
env-owned buffer, and computes the fp32 policy on the FFMA path (the tensor-core path of
g1_rollout needs an env-owned weight image).  Checked through the C-ABI against g1_rollout
with the same policy arithmetic (precision "fp32-ffma") on two calls in a row.

This file is collected last on purpose: it runs after every other test, and it must also
pass when run alone in a fresh process."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _bufs(H, N):
    z = lambda *s: torch.zeros(*s, device="cuda")
    return [z(H, N, 100), z(H, N, 29), z(H, N), z(H, N), z(H, N), z(H, N), z(N)]


def test_noalloc_rollout_matches_rollout_twice():
    import g1env
    g1env.load_library()
    N, H = 200, 3
    ac = g1env.init_policy_normal(g1env.AC(100, 29).cuda(), seed=4)
    W = g1env.pack_weights(ac).detach()
    mean = torch.zeros(100, device="cuda")
    var = torch.ones(100, device="cuda")
    ref = g1env.G1Env(N, 10, 8, seed=21)
    new = g1env.G1Env(N, 10, 8, seed=21)
    ref.set_policy((256, 256), "tanh", precision="fp32-ffma")
    ref.reset()
    new.reset()
    for call in range(2):
        a, b = _bufs(H, N), _bufs(H, N)
        ref.rollout(H, W, mean, var, *a)
        new.rollout_noalloc(H, W, mean, var, *b)
        torch.cuda.synchronize()
        for k, (x, y) in enumerate(zip(a, b)):
            x, y = x.cpu().numpy(), y.cpu().numpy()
            assert np.abs(x - y).max() <= 1e-4, (call, k)
        assert np.array_equal(a[5].cpu().numpy(), b[5].cpu().numpy())   # done flags exact
        sr, sn = ref.get_state(), new.get_state()
        assert np.array_equal(sr[3], sn[3]) and sr[4] == sn[4]          # counters and RNG tick
    ref.close()
    new.close()


def test_noalloc_rejects_policy_beyond_static_area():
    import g1env
    lib = g1env.load_library()
    env = g1env.G1Env(8, 10, 8, seed=1)
    env.set_policy((300, 300, 300, 300), "elu")   # 310,864 repacked floats > 131,072
    H = 1
    ac = g1env.init_policy_normal(g1env.AC(100, 29, (300, 300, 300, 300), "elu").cuda(), seed=0)
    W = g1env.pack_weights(ac).detach()
    b = _bufs(H, 8)
    with pytest.raises(g1env.G1Error, match="static area"):
        env.rollout_noalloc(H, W, torch.zeros(100, device="cuda"), torch.ones(100, device="cuda"), *b)
    lib.g1_env_clear_error()
    env.close()


def test_noalloc_rejects_bf16_policy_and_value_net():
    """The static area only backs the fp32 in-kernel policy: an env set to the bf16
    tensor-core policy, or given a separate value network, is rejected with an error rather
    than run with a mismatched weight layout."""
    import g1env
    lib = g1env.load_library()
    N, H = 16, 1
    env = g1env.G1Env(N, 10, 8, seed=2)
    env.reset()
    mean, var = torch.zeros(100, device="cuda"), torch.ones(100, device="cuda")
    env.set_policy((512,), "elu", precision="bf16")
    W = g1env.pack_weights(g1env.init_policy_normal(g1env.AC(100, 29, (512,), "elu").cuda(), seed=0)).detach()
    with pytest.raises(g1env.G1Error, match="fp32 in-kernel policy"):
        env.rollout_noalloc(H, W, mean, var, *_bufs(H, N))
    lib.g1_env_clear_error()
    env.set_policy((256, 256), "elu", precision="bf16")
    env.set_value_net((64,))
    with pytest.raises(g1env.G1Error, match="fp32 in-kernel policy"):
        env.rollout_noalloc(H, W, mean, var, *_bufs(H, N))
    lib.g1_env_clear_error()
    env.close()


def test_noalloc_leaves_free_device_memory_unchanged():
    """After a first call (which looks up the area's address), further calls change the
    device's free memory by nothing: no allocation by the library or the CUDA runtime."""
    import g1env
    g1env.load_library()
    N, H = 64, 2
    env = g1env.G1Env(N, 10, 8, seed=5)
    env.reset()
    W = g1env.pack_weights(g1env.init_policy_normal(g1env.AC(100, 29).cuda(), seed=3)).detach()
    mean, var = torch.zeros(100, device="cuda"), torch.ones(100, device="cuda")
    b = _bufs(H, N)
    env.rollout_noalloc(H, W, mean, var, *b)
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    for _ in range(3):
        env.rollout_noalloc(H, W, mean, var, *b)
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free0
    assert np.isfinite(b[0].cpu().numpy()).all()
    env.close()
