"""Trainer batch preparation on the GPU (g1_gae, g1_obs_prep, g1_adv_normalize,
g1_runnorm_update) against the reference trainer's own torch code for the same step
(scripts/ppo_fused.py:104-119, scripts/ppo.py:71-79), restated here verbatim in operation order.

Gates: adv, ret and nobs bit-identical to the torch loop / expression (the kernels round each
operation once in the same order); the RunNorm update and the normalised advantages, whose
reductions the kernels take in fp64 where torch reduces in fp32, within 1e-5 (absolute on
mean, relative on var, absolute on the normalised advantages, which are O(1))."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def ref_gae(R, V, D, Vlast, gamma=0.99, lam=0.95):
    """ppo_fused.py:108-116"""
    H, N = R.shape
    adv = torch.zeros_like(R)
    gae = torch.zeros(N, device=R.device)
    for t in reversed(range(H)):
        nextv = Vlast if t == H - 1 else V[t + 1]
        delta = R[t] + gamma * nextv * (1 - D[t]) - V[t]
        gae = delta + gamma * lam * (1 - D[t]) * gae
        adv[t] = gae
    return adv, adv + V


class RefRunNorm:
    """ppo.py:63-81"""

    def __init__(self, dim, dev):
        self.mean = torch.zeros(dim, device=dev)
        self.var = torch.ones(dim, device=dev)
        self.count = 1e-4

    def update(self, x):
        b = x.shape[0]
        bm = x.mean(0); bv = x.var(0, unbiased=False)
        tot = self.count + b
        delta = bm - self.mean
        self.mean += delta * b / tot
        self.var = (self.var * self.count + bv * b + delta ** 2 * self.count * b / tot) / tot
        self.count = tot


def _traj(H, N, dim, seed, p_done=0.03):
    g = torch.Generator(device="cuda").manual_seed(seed)
    O = torch.randn(H, N, dim, device="cuda", generator=g) * 2.0 + 0.5
    O[..., :4] = torch.tensor([0.8, 0.0, 0.0, 0.0], device="cuda")[: min(4, dim)]  # constant command slot
    V = torch.randn(H, N, device="cuda", generator=g)
    R = torch.rand(H, N, device="cuda", generator=g) * 3 - 1
    D = (torch.rand(H, N, device="cuda", generator=g) < p_done).float()
    Vlast = torch.randn(N, device="cuda", generator=g)
    return O, V, R, D, Vlast


@pytest.mark.parametrize("H,N", [(32, 8192), (1, 1), (5, 37), (64, 1000)])
def test_gae_bit_exact(H, N):
    import g1env
    _, V, R, D, Vlast = _traj(H, N, 4, seed=H * 1000 + N)
    adv, ret, mom = g1env.gae_device(R, V, D, Vlast)
    radv, rret = ref_gae(R, V, D, Vlast)
    torch.cuda.synchronize()
    assert torch.equal(adv, radv)
    assert torch.equal(ret, rret)
    a = radv.double()
    assert mom[0].item() == H * N
    assert abs(mom[1].item() - a.sum().item()) <= 1e-9 * max(1.0, a.abs().sum().item())
    assert abs(mom[2].item() - (a * a).sum().item()) <= 1e-9 * max(1.0, (a * a).sum().item())
    # advantage normalisation (ppo_fused.py:119)
    b_ref = radv.reshape(-1)
    b_ref = (b_ref - b_ref.mean()) / (b_ref.std() + 1e-8) if H * N > 1 else (b_ref - b_ref.mean()) / 1e-8
    if H * N > 1:
        g1env.adv_normalize_device(adv, mom)
        torch.cuda.synchronize()
        assert (adv.reshape(-1) - b_ref).abs().max().item() <= 1e-5


@pytest.mark.parametrize("H,N,dim", [(32, 8192, 100), (3, 37, 100), (2, 50, 7), (1, 1, 100), (4, 300, 1024)])
def test_obs_prep_and_runnorm(H, N, dim):
    import g1env
    O, *_ = _traj(H, N, dim, seed=7 + dim)
    fmean = torch.randn(dim, device="cuda") * 0.3
    fvar = torch.rand(dim, device="cuda") * 4 + 0.01
    fvar[:2] = 0.0  # constant dimensions: sqrt(0 + 1e-8)
    nobs, mom = g1env.obs_prep_device(O, fmean, fvar)
    ref = torch.clamp((O - fmean) / torch.sqrt(fvar + 1e-8), -10.0, 10.0)
    torch.cuda.synchronize()
    assert torch.equal(nobs, ref)
    # RunNorm update from the moments, twice (the second from a non-trivial state)
    norm = g1env.RunNorm(dim, "cuda")
    rn = RefRunNorm(dim, "cuda")
    rows = H * N
    for k in range(2):
        x = O.reshape(-1, dim) * (1 + k)
        _, m = g1env.obs_prep_device(x, fmean, fvar)
        g1env.runnorm_update_device(norm, m, rows)
        rn.update(x)
        torch.cuda.synchronize()
        assert abs(norm.count - rn.count) < 1e-9 * rn.count
        assert (norm.mean - rn.mean).abs().max().item() <= 1e-5
        assert ((norm.var - rn.var).abs() / rn.var.abs().clamp_min(1e-3)).max().item() <= 1e-5


def test_prepare_batch_on_rollout():
    """The trainer's prepare_batch on a real rollout equals the reference trainer's torch code."""
    import g1env
    import ppo_fused
    N, H = 512, 8
    env = g1env.G1Env(N, 10, 8, seed=5, device=0)
    env.reset()
    ac = g1env.init_policy_normal(g1env.AC(100, 29).cuda(), seed=2)
    W = g1env.pack_weights(ac).detach()
    norm = g1env.RunNorm(100, "cuda")
    rn = RefRunNorm(100, "cuda")
    z = lambda *s: torch.zeros(*s, device="cuda")
    O, A, LP, V, R, D, Vlast = z(H, N, 100), z(H, N, 29), z(H, N), z(H, N), z(H, N), z(H, N), z(N)
    for _ in range(2):
        fmean, fvar = norm.mean.clone(), norm.var.clone()
        env.rollout(H, W, fmean, fvar, O, A, LP, V, R, D, Vlast)
        nobs, b_adv, ret = ppo_fused.prepare_batch(norm, O, V, R, D, Vlast, fmean, fvar)
        # reference: ppo_fused.py:104-119
        r_nobs = torch.clamp((O - fmean) / torch.sqrt(fvar + 1e-8), -10.0, 10.0)
        rn.update(O.reshape(-1, 100))
        radv, rret = ref_gae(R, V, D, Vlast)
        rb = radv.reshape(-1)
        rb = (rb - rb.mean()) / (rb.std() + 1e-8)
        torch.cuda.synchronize()
        assert torch.equal(nobs, r_nobs)
        assert torch.equal(ret, rret)
        assert (b_adv.reshape(-1) - rb).abs().max().item() <= 1e-5
        assert (norm.mean - rn.mean).abs().max().item() <= 1e-5
        assert ((norm.var - rn.var).abs() / rn.var.abs().clamp_min(1e-3)).max().item() <= 1e-5
        norm.mean.copy_(rn.mean); norm.var.copy_(rn.var)  # keep both trainers on the same stats
    env.close()
