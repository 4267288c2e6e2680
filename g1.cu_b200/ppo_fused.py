"""PPO on the fused GPU rollout, one process per GPU (the reference's scripts/ppo_fused.py
training loop, ppo_fused.py:47-171, with world sharding across ranks).

    python g1.cu_b200/ppo_fused.py [iters] [n_worlds_per_gpu] [--smoke] [--tag=name] [--config4] [--no-eval] [--tf32]
    torchrun --nproc-per-node 8 g1.cu_b200/ppo_fused.py 1500 8192
    torchrun --nproc-per-node 8 g1.cu_b200/ppo_fused.py 3 65536 --config4 --no-eval

--config4: policy 100-1024-1024-512-29 ELU on the bf16 tensor-core path plus a separate
100-512-512-512-1 value network; each iteration prints its wall time split into rollout and
update (and the rollout's substeps/s).

The rollout runs in the CUDA library (g1_rollout); torch does only the PPO update, reading
the trajectory buffers in place.  With WORLD_SIZE > 1 each rank owns its own worlds (global
world ids rank*N + i, so RNG streams are disjoint) and two things cross NCCL:
  * one fp64 buffer of batch moments -- the raw-observation sums for the RunNorm update (so
    every rank keeps the same frozen normaliser, ppo_fused.py:104-106) and the advantage sums
    for advantage normalisation (ppo_fused.py:119) -- produced and consumed by the batch
    preparation kernels (g1_obs_prep, g1_gae, g1_runnorm_update, g1_adv_normalize),
  * the gradients, once per minibatch step (summed then divided by the world size).
"""
import os
import sys
import time

import torch
import torch.nn as nn

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
from g1env import (AC, G1Env, RunNorm, adv_normalize_device, evaluate, gae_device, obs_prep_device,  # noqa: E402
                   pack_weights, runnorm_update_device)


# ---------------------------------------------------------------- distributed helpers
def _dist():
    import torch.distributed as dist
    return dist if dist.is_available() and dist.is_initialized() else None


def allreduce_moments(*bufs):
    """Sum the fp64 moment buffers of the batch preparation over ranks, in place, in one
    all-reduce (obs moments [rows, sum o, sum o^2] and advantage moments [n, sum, sumsq])."""
    dist = _dist()
    if dist is None:
        return bufs
    flat = torch.cat([b.reshape(-1) for b in bufs])
    dist.all_reduce(flat)
    off = 0
    for b in bufs:
        b.copy_(flat[off:off + b.numel()].view_as(b))
        off += b.numel()
    return bufs


def prepare_batch(norm, O, V, R, D, Vlast, fmean, fvar, gamma=0.99, lam=0.95):
    """ppo_fused.py:104-119 on the GPU, straight from the rollout buffers:
    nobs (frozen-stat renormalisation), RunNorm update from the raw observations, GAE, returns
    and normalised advantages.  Only the moment buffers cross ranks."""
    nobs, omom = obs_prep_device(O, fmean, fvar)
    adv, ret, amom = gae_device(R, V, D, Vlast, gamma, lam)
    allreduce_moments(omom, amom)
    dist = _dist()
    rows = (O.numel() // O.shape[-1]) * (dist.get_world_size() if dist is not None else 1)
    runnorm_update_device(norm, omom, rows)
    adv_normalize_device(adv, amom)
    return nobs, adv, ret


def allreduce_grads(params):
    """Average the gradients of `params` over ranks in one flat bucket."""
    dist = _dist()
    if dist is None:
        return
    grads = [p.grad for p in params if p.grad is not None]
    flat = torch.cat([g.reshape(-1) for g in grads])
    dist.all_reduce(flat)
    flat /= dist.get_world_size()
    off = 0
    for g in grads:
        n = g.numel()
        g.copy_(flat[off:off + n].view_as(g))
        off += n


def broadcast_params(module):
    dist = _dist()
    if dist is None:
        return
    for p in module.parameters():
        dist.broadcast(p.data, 0)


HALF_LOG_2PI = 0.9189385332046727


def ppo_loss(ac, obs, act, old_logp, adv, ret, clip=0.2, vf_coef=0.5, ent_coef=0.01):
    """The clipped-surrogate PPO objective the reference trainer minimises
    (ppo_fused.py:121-140): policy term -E[min(r A, clip(r, 1 +- eps) A)], value term
    vf_coef E[(V - R)^2], entropy bonus ent_coef E[H].  The diagonal Gaussian's log-density
    and entropy are written in closed form from the mean and log-std:
        log p(a) = sum_i [-(a_i - mu_i)^2 / (2 s_i^2) - log s_i - log sqrt(2 pi)],
        H = sum_i [log s_i + 1/2 + log sqrt(2 pi)]."""
    mu, std, val = ac(obs)
    log_std = torch.log(std).expand_as(mu)
    z = (act - mu) / std
    logp = (-0.5 * z * z - log_std - HALF_LOG_2PI).sum(-1)
    ratio = torch.exp(logp - old_logp)
    surrogate = torch.minimum(ratio * adv, ratio.clamp(1.0 - clip, 1.0 + clip) * adv)
    entropy = (log_std + 0.5 + HALF_LOG_2PI).sum(-1)
    return -surrogate.mean() + vf_coef * (val - ret).square().mean() - ent_coef * entropy.mean()


def ppo_update(ac, opt, b_o, b_a, b_lp, b_adv, b_ret, epochs=5, mb=4, clip=0.2):
    """Epochs x minibatches of ppo_loss over a shuffled batch, with the gradients averaged
    over ranks before clipping (max norm 0.5) and the optimiser step."""
    n = b_o.shape[0]
    size = n // mb
    params = list(ac.parameters())
    last = 0.0
    for _ in range(epochs):
        perm = torch.randperm(n, device=b_o.device)
        for j in perm[: size * mb].view(mb, size).unbind(0):
            loss = ppo_loss(ac, b_o[j], b_a[j], b_lp[j], b_adv[j], b_ret[j], clip)
            opt.zero_grad()
            loss.backward()
            allreduce_grads(params)
            nn.utils.clip_grad_norm_(params, 0.5)
            opt.step()
            last = float(loss.item())
    return last


def main():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=dev)
    smoke = "--smoke" in sys.argv
    args = [a for a in sys.argv[1:] if not a.startswith("--")]
    iters = int(args[0]) if args else (3 if smoke else 1500)
    N = int(args[1]) if len(args) > 1 else (256 if smoke else 8192)
    H = 16 if smoke else 32
    config4 = "--config4" in sys.argv
    do_eval = "--no-eval" not in sys.argv
    if "--tf32" in sys.argv:
        # opt-in: the update's matmuls on the tensor cores in TF32 (10-bit mantissa products,
        # fp32 accumulation); off by default, so the update's arithmetic is the reference's fp32
        torch.backends.cuda.matmul.allow_tf32 = True
        torch.backends.cudnn.allow_tf32 = True
    tag = next((a.split("=", 1)[1] for a in sys.argv if a.startswith("--tag=")), "fused")
    out_dir = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "runs")
    os.makedirs(out_dir, exist_ok=True)

    env = G1Env(N, substeps=10, pgs_iters=8, seed=1, device=local, world0=rank * N)
    O_dim, A_dim = env.obs_dim, env.act_dim
    torch.manual_seed(0)
    if config4:
        env.set_policy((1024, 1024, 512), "elu", precision="bf16")
        env.set_value_net((512, 512, 512))
        ac = AC(O_dim, A_dim, (1024, 1024, 512), "elu", value_hidden=(512, 512, 512)).to(dev)
    else:
        ac = AC(O_dim, A_dim).to(dev)
    broadcast_params(ac)
    norm = RunNorm(O_dim, dev)
    opt = torch.optim.Adam(ac.parameters(), lr=3e-4)
    z = lambda *s: torch.zeros(*s, device=dev)
    O, A, LP, V, R, D, Vlast = z(H, N, O_dim), z(H, N, A_dim), z(H, N), z(H, N), z(H, N), z(H, N), z(N)
    env.reset()
    logf = open(os.path.join(out_dir, f"reward_curve_{tag}.csv"), "w") if rank == 0 else None
    if logf:
        logf.write("iter,mean_ep_rew_step,ret,loss,fwd_mean,ep_len,fall_rate,vx_mean,sps\n")
    t0 = time.time()
    for it in range(iters):
        torch.cuda.synchronize()
        t_it = time.time()
        fmean, fvar = norm.mean.clone(), norm.var.clone()
        W = pack_weights(ac).detach()
        env.rollout(H, W, fmean, fvar, O, A, LP, V, R, D, Vlast)
        torch.cuda.synchronize()
        t_roll = time.time() - t_it
        with torch.no_grad():
            nobs, b_adv, ret = prepare_batch(norm, O, V, R, D, Vlast, fmean, fvar)
        loss = ppo_update(ac, opt, nobs.reshape(-1, O_dim), A.reshape(-1, A_dim), LP.reshape(-1), b_adv.reshape(-1),
                          ret.reshape(-1))
        torch.cuda.synchronize()
        t_iter = time.time() - t_it
        if rank == 0 and config4:
            print(f"iter {it}: wall {t_iter:.3f} s (rollout {t_roll:.3f} s = {world * N * H * 10 / t_roll:.3e} "
                  f"substeps/s, batch prep + PPO update {t_iter - t_roll:.3f} s)", flush=True)
        sps = world * (it + 1) * H * N / (time.time() - t0)
        ev = {"fwd_mean": float("nan"), "ep_len_mean": float("nan"), "fall_rate": float("nan"), "vx_mean": float("nan")}
        if rank == 0 and do_eval and ((it % 25 == 0) or it == iters - 1):
            ev = evaluate(env, ac, norm, dev, steps=400 if not smoke else 20)
            torch.save(dict(model=ac.state_dict(), obs_mean=norm.mean, obs_var=norm.var),
                       os.path.join(out_dir, f"{tag}_last.pt"))
        if rank == 0:
            print(f"iter {it:4d} rew/step={R.mean().item():7.3f} loss={loss:7.3f} sps={sps:.2e}", flush=True)
            logf.write(f"{it},{R.mean().item():.4f},{ret.mean().item():.4f},{loss:.4f},{ev['fwd_mean']:.4f},"
                       f"{ev['ep_len_mean']:.2f},{ev['fall_rate']:.4f},{ev['vx_mean']:.4f},{sps:.3e}\n")
            logf.flush()
    env.close()
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    if smoke and rank == 0:
        print("SMOKE OK: fused rollout + PPO update ran end-to-end.")


if __name__ == "__main__":
    main()
