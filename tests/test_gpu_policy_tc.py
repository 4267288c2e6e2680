"""The wide-policy rollout path (100 -> 1024 -> 1024 -> 512 -> 29 ELU,
bf16 weights, fp32 accumulation on tcgen05 tensor cores), through g1_rollout.

* policy outputs vs a torch fp32 reference of the same actor-critic on the same observations:
  relative error <= 1e-2 on the means (config 3's stated tolerance; log_std is set to -20 so
  the sampled actions equal the means to 1e-8).  The value head of a random-init net is a
  small, cancelling sum (|v| ~ 0.04), so its bf16 rounding shows as ~2e-2 relative to fp32:
  it is held to 1e-2 against a torch reference that rounds weights and activations to bf16
  where the kernel does, and to 5e-2 against fp32;
* physics: replaying the GPU's own actions through the CPU oracle reproduces rewards, done
  flags, episode counters and observations (the fp32 rollout tolerances)."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

HID = (1024, 1024, 512)


def test_config3_policy_means_and_physics():
    import g1env
    from oracle.oracle import Oracle, OracleEnv
    N, H = 300, 2
    env = g1env.G1Env(N, 10, 8, seed=13)
    env.set_policy(HID, "elu", precision="bf16")
    env.reset()
    oenv = OracleEnv(Oracle("f32"), N, 10, 8, seed=13)
    st = env.get_state()
    oenv.set_state(*st[:4], tick=st[4])
    ac = g1env.init_policy_normal(g1env.AC(100, 29, HID, "elu").cuda(), seed=2)
    with torch.no_grad():
        ac.log_std.fill_(-20.0)
    W = g1env.pack_weights(ac).detach()
    rng = np.random.default_rng(1)
    mean = torch.tensor(rng.normal(0, 0.1, 100), dtype=torch.float32).cuda()
    var = torch.tensor(rng.uniform(0.5, 2.0, 100), dtype=torch.float32).cuda()
    z = lambda *s: torch.zeros(*s, device="cuda")
    O, A, LP, V, R, D, Vl = z(H, N, 100), z(H, N, 29), z(H, N), z(H, N), z(H, N), z(H, N), z(N)
    env.rollout(H, W, mean, var, O, A, LP, V, R, D, Vl)
    torch.cuda.synchronize()
    assert env.tc_status() == 0
    with torch.no_grad():
        for t in range(H):
            x = torch.clamp((O[t] - mean) / torch.sqrt(var + 1e-8), -10, 10)
            mu, _, v = ac(x)
            assert ((A[t] - mu).norm() / mu.norm()).item() <= 1e-2
            assert ((V[t] - v).norm() / v.norm()).item() <= 5e-2
            h = x.to(torch.bfloat16).float()
            for m in ac.body:
                if isinstance(m, torch.nn.Linear):
                    h = h @ m.weight.to(torch.bfloat16).float().T + m.bias
                else:
                    h = torch.nn.functional.elu(h).to(torch.bfloat16).float()
            vb = (h @ ac.v.weight.to(torch.bfloat16).float().T + ac.v.bias).squeeze(-1)
            assert ((V[t] - vb).norm() / vb.norm()).item() <= 1e-2
    assert torch.isfinite(LP).all()
    # physics on the GPU's own actions
    Ah, Oh, Rh, Dh = A.cpu().numpy(), O.cpu().numpy(), R.cpu().numpy(), D.cpu().numpy()
    for t in range(H):
        o2, r2, d2 = oenv.step(Ah[t])
        assert np.abs(r2 - Rh[t]).max() < 1e-4
        assert np.array_equal(d2, Dh[t])
        if t + 1 < H:
            assert np.abs(o2 - Oh[t + 1]).max() < 1e-3
    g, o = env.get_state(), oenv.get_state()
    assert np.array_equal(g[3], o[3]) and g[4] == o[4] == H
    env.close()



def test_config4_separate_value_network():
    """BASELINE config 4's networks: the config-3 policy plus a separate 100-512-512-512-1 value
    MLP (g1_env_set_value_net).  Means within 1e-2 of fp32; the value within 1e-2 of a torch
    reference rounding weights and activations to bf16 where the kernel does."""
    import g1env
    N, H, VH = 300, 2, (512, 512, 512)
    env = g1env.G1Env(N, 10, 8, seed=17)
    env.set_policy(HID, "elu", precision="bf16")
    env.set_value_net(VH)
    env.reset()
    ac = g1env.init_policy_normal(g1env.AC(100, 29, HID, "elu", value_hidden=VH).cuda(), seed=5)
    with torch.no_grad():
        ac.log_std.fill_(-20.0)
        ac.v.bias.fill_(0.3)
    W = g1env.pack_weights(ac).detach()
    mean, var = torch.zeros(100, device="cuda"), torch.ones(100, device="cuda")
    z = lambda *s: torch.zeros(*s, device="cuda")
    O, A, LP, V, R, D, Vl = z(H, N, 100), z(H, N, 29), z(H, N), z(H, N), z(H, N), z(H, N), z(N)
    env.rollout(H, W, mean, var, O, A, LP, V, R, D, Vl)
    torch.cuda.synchronize()
    assert env.tc_status() == 0
    with torch.no_grad():
        for t in range(H):
            x = torch.clamp((O[t] - mean) / torch.sqrt(var + 1e-8), -10, 10)
            mu, _, v = ac(x)
            assert ((A[t] - mu).norm() / mu.norm()).item() <= 1e-2
            h = x.to(torch.bfloat16).float()
            for m in ac.v_body:
                if isinstance(m, torch.nn.Linear):
                    h = h @ m.weight.to(torch.bfloat16).float().T + m.bias
                else:
                    h = torch.nn.functional.elu(h).to(torch.bfloat16).float()
            vb = (h @ ac.v.weight.to(torch.bfloat16).float().T + ac.v.bias).squeeze(-1)
            assert ((V[t] - vb).norm() / vb.norm()).item() <= 1e-2
            assert ((V[t] - v).norm() / v.norm()).item() <= 5e-2
    env.set_value_net(())
    env.close()
