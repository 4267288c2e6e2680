"""Multi-rank host logic of the PPO update on CPU (gloo, world size 2): the RunNorm moments,
advantage normalisation and gradient averaging that cross NCCL on GPUs give the same result
as one process holding all ranks' data."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def runnorm_from_moments(norm, mom):
    """the arithmetic of k_runnorm (g1_ppo_prep.cuh) in torch fp64"""
    dim = norm.mean.numel()
    b = mom[0]
    bm = mom[1:1 + dim] / b
    bv = (mom[1 + dim:] / b - bm ** 2).clamp_min(0)
    tot = norm.count + b
    m0, v0 = norm.mean.double(), norm.var.double()
    delta = bm - m0
    norm.mean = (m0 + delta * b / tot).float()
    norm.var = ((v0 * norm.count + bv * b + delta ** 2 * norm.count * b / tot) / tot).float()
    norm.count = float(tot)


def adv_norm_from_moments(adv, mom):
    """the arithmetic of k_adv_norm (g1_ppo_prep.cuh)"""
    n, mean = mom[0], mom[1] / mom[0]
    std = ((mom[2] - n * mean * mean) / max(float(n) - 1.0, 1.0)).clamp_min(0).sqrt()
    return (adv - mean.float()) / (std.float() + 1e-8)


def _worker(rank, world, port, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import sys
    sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
    from test_dist_cpu import adv_norm_from_moments, runnorm_from_moments
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import ppo_fused
    from g1env import AC, RunNorm
    g = torch.Generator().manual_seed(100 + rank)
    x = torch.randn(50 + 30 * rank, 100, generator=g) * (1 + rank)
    norm = RunNorm(100, "cpu")
    adv = torch.randn(40 + 10 * rank, generator=g)
    # the moment layouts g1_obs_prep / g1_gae produce, summed over ranks by the trainer
    omom = torch.cat([torch.tensor([float(x.shape[0])], dtype=torch.float64), x.double().sum(0), (x.double() ** 2).sum(0)])
    amom = torch.tensor([float(adv.numel()), adv.double().sum().item(), (adv.double() ** 2).sum().item()],
                        dtype=torch.float64)
    ppo_fused.allreduce_moments(omom, amom)
    runnorm_from_moments(norm, omom)
    nadv = adv_norm_from_moments(adv, amom)
    torch.manual_seed(0)
    ac = AC(100, 29)
    ppo_fused.broadcast_params(ac)
    out = ac(x[:8])[0].sum() * (rank + 1)
    out.backward()
    ppo_fused.allreduce_grads(list(ac.parameters()))
    # tensors travel as numpy arrays (pickled by value): a tensor would be passed as a shared
    # memory handle, which breaks when this process exits before the parent unpickles it
    q.put(tuple(t.detach().numpy().copy() if torch.is_tensor(t) else t
                for t in (rank, x, norm.mean, norm.var, norm.count, adv, nadv, ac.mu.weight.grad)))
    dist.barrier()
    dist.destroy_process_group()


def test_distributed_stats_match_single_process():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in ps:
        p.start()
    res = sorted([q.get(timeout=120) for _ in range(world)], key=lambda r: r[0])
    res = [tuple(torch.from_numpy(v) if hasattr(v, "dtype") and hasattr(v, "shape") else v for v in r) for r in res]
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    import sys
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "g1.cu_b200"))
    from g1env import AC, RunNorm
    xs = torch.cat([r[1] for r in res])
    ref = RunNorm(100, "cpu")
    ref.update(xs)
    for r in res:
        assert torch.allclose(r[2], ref.mean, atol=1e-5) and torch.allclose(r[3], ref.var, atol=1e-4)
        assert abs(r[4] - ref.count) < 1e-6
    adv = torch.cat([r[5] for r in res])
    nadv = (adv - adv.mean()) / (adv.std() + 1e-8)
    assert torch.allclose(torch.cat([r[6] for r in res]), nadv, atol=1e-5)
    # gradient average: mean over ranks of (rank+1) * d sum(mu(x_rank[:8])) / dW
    torch.manual_seed(0)
    ac = AC(100, 29)
    g_sum = 0
    for r in res:
        ac.zero_grad()
        (ac(r[1][:8])[0].sum() * (r[0] + 1)).backward()
        g_sum = g_sum + ac.mu.weight.grad.clone()
    for r in res:
        assert torch.allclose(r[7], g_sum / world, atol=1e-5)
