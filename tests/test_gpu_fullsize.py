"""The fused rollout at BASELINE's full sizes (config 2: N = 8192, H = 32; config 3: N = 32768),
where the grid is the production one (147 CTAs of 56 worlds, two rounds of groups per CTA):
size-independent properties plus oracle parity on a block of worlds.

* determinism: two rollouts from the same state and tick are bitwise identical;
* every output finite; done flags exactly 0/1; episode counters advance by one per control
  step and restart at 0 after a done (g1_env.cu:193-210); the RNG tick advances by H;
* config 2, H = 4: the first 64 worlds (all of CTA 0 and part of CTA 1) against the fp32 CPU
  oracle with the rollout tolerances (O 1e-3, A/LP/V/R/Vlast 1e-4, done flags and counters
  exact)."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _bufs(H, N):
    z = lambda *s: torch.zeros(*s, device="cuda")
    return dict(O=z(H, N, 100), A=z(H, N, 29), LP=z(H, N), V=z(H, N), R=z(H, N), D=z(H, N), Vlast=z(N))


def _run(env, st, H, W, mean, var):
    env.set_state(*st[:4], st[4])
    b = _bufs(H, env.N)
    env.rollout(H, W, mean, var, *b.values())
    torch.cuda.synchronize()
    return b, env.get_state()


def _check_rollout_properties(b, st0, st1, H):
    for k, v in b.items():
        assert torch.isfinite(v).all(), k
    D = b["D"].cpu().numpy()
    assert np.isin(D, (0.0, 1.0)).all()
    steps = st0[3].astype(np.int64)
    for t in range(H):
        steps = np.where(D[t] > 0.5, 0, steps + 1)
    assert np.array_equal(steps, st1[3])
    assert st1[4] == st0[4] + H


@pytest.mark.parametrize("cfg", ["config2", "config3"])
def test_fullsize_determinism_and_invariants(cfg):
    import g1env
    if cfg == "config2":
        N, H, hid, prec = 8192, 32, (256, 256), "fp32"
    else:
        N, H, hid, prec = 32768, 4, (1024, 1024, 512), "bf16"
    env = g1env.G1Env(N, 10, 8, seed=31)
    env.set_policy(hid, "elu", precision=prec)
    env.reset()
    st0 = env.get_state()
    ac = g1env.init_policy_normal(g1env.AC(100, 29, hid, "elu").cuda(), seed=3)
    W = g1env.pack_weights(ac).detach()
    mean, var = torch.zeros(100, device="cuda"), torch.ones(100, device="cuda")
    b1, s1 = _run(env, st0, H, W, mean, var)
    b2, s2 = _run(env, st0, H, W, mean, var)
    for k in b1:
        assert torch.equal(b1[k], b2[k]), k
    for x, y in zip(s1[:4], s2[:4]):
        assert np.array_equal(x, y)
    _check_rollout_properties(b1, st0, s1, H)
    assert env.tc_status() == 0
    env.close()


def test_fullsize_config2_block_vs_oracle():
    import g1env
    from oracle.oracle import Oracle, OracleEnv
    N, H, NB = 8192, 4, 64
    env = g1env.G1Env(N, 10, 8, seed=9)
    env.set_policy((256, 256), "elu")
    env.reset()
    st = env.get_state()
    oenv = OracleEnv(Oracle("f32"), N, 10, 8, seed=9)
    oenv.set_state(*st[:4], tick=st[4])
    ac = g1env.init_policy_normal(g1env.AC(100, 29, (256, 256), "elu").cuda(), seed=6)
    W = g1env.pack_weights(ac).detach()
    mean, var = torch.zeros(100, device="cuda"), torch.ones(100, device="cuda")
    b = _bufs(H, N)
    env.rollout(H, W, mean, var, *b.values())
    torch.cuda.synchronize()
    ro = oenv.rollout(H, W.cpu().numpy(), mean.cpu().numpy(), var.cpu().numpy(), act="elu", nworlds=NB)
    tol = dict(O=1e-3, A=1e-4, LP=1e-4, V=1e-4, R=1e-4)
    for k, t in tol.items():
        g = b[k].cpu().numpy()[:, :NB]
        assert np.abs(g - ro[k][:, :NB]).max() <= t, k
    assert np.abs(b["Vlast"].cpu().numpy()[:NB] - ro["Vlast"][:NB]).max() <= 1e-4
    assert np.array_equal(b["D"].cpu().numpy()[:, :NB], ro["D"][:, :NB])
    gs, os_ = env.get_state(), oenv.get_state()
    assert np.array_equal(gs[3][:NB], os_[3][:NB])
    env.close()
