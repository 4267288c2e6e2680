"""Host-side trainer pieces on CPU: the closed-form PPO objective against the same objective
built from torch.distributions (the form of the reference trainer, ppo_fused.py:121-140),
and the running observation normaliser against the moments of all rows at once."""
import os
import sys

import numpy as np
import torch

sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "g1.cu_b200"))


def test_ppo_loss_matches_distribution_form():
    from g1env import AC
    from ppo_fused import ppo_loss
    torch.manual_seed(3)
    ac = AC(100, 29)
    with torch.no_grad():
        ac.log_std.uniform_(-1.0, 0.3)
    obs, act = torch.randn(64, 100), torch.randn(64, 29)
    old, adv, ret = torch.randn(64) - 30.0, torch.randn(64), torch.randn(64)
    got = ppo_loss(ac, obs, act, old, adv, ret)
    mu, std, val = ac(obs)
    d = torch.distributions.Normal(mu, std)
    r = (d.log_prob(act).sum(-1) - old).exp()
    want = (-torch.min(r * adv, torch.clamp(r, 0.8, 1.2) * adv).mean() + 0.5 * (val - ret).pow(2).mean()
            - 0.01 * d.entropy().sum(-1).mean())
    assert torch.allclose(got, want, rtol=1e-5, atol=1e-5), (got.item(), want.item())


def test_runnorm_batches_equal_all_rows():
    from g1env import RunNorm
    g = torch.Generator().manual_seed(0)
    xs = [torch.randn(n, 100, generator=g) * (1 + i) + i for i, n in enumerate((37, 200, 5))]
    rn = RunNorm(100, "cpu")
    for x in xs:
        rn.update(x)
    allx = torch.cat(xs).double().numpy()
    n0 = 1e-4   # the initial pseudo-count with mean 0, var 1
    n = allx.shape[0]
    m = allx.mean(0) * n / (n + n0)
    # merged variance of {prior (mean 0, var 1, count n0), all rows}
    v = (n0 * 1.0 + n * allx.var(0) + (allx.mean(0) ** 2) * n0 * n / (n0 + n)) / (n0 + n)
    assert np.allclose(rn.mean.numpy(), m, atol=1e-5)
    assert np.allclose(rn.var.numpy(), v, rtol=1e-5, atol=1e-5)
    assert abs(rn.count - (n + n0)) < 1e-9
