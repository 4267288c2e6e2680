"""Checkpoint / weight-format round trip and playback of the reference's trained walker on the
CPU oracle (the reference's models/ppo_ckpt/finish_best.pt, exported to
tests/golden/finish_policy.npz by tests/golden/make_golden.py).

* The reference's state_dict loads strictly into this repo's AC (same module names/shapes,
  scripts/ppo.py:85-99), and pack_weights lays it out in the g1_rollout order
  (scripts/ppo_fused.py:35-44): per hidden layer W, b; then Wmu, bmu, Wv, bv, log_std.
* The trainer's checkpoint format {model, obs_mean, obs_var} (ppo_fused.py:150-154)
  survives a torch.save / torch.load round trip bit for bit.
* Playback: the reference documents that this policy, run deterministically (mean action,
  scripts/play_finish.py) from reset for up to 480 control steps, takes 256/256 worlds across
  x = 5 m (DEVLOG.md:421-422).  The fp32 CPU oracle (the reference's physics arithmetic) does
  the same for every world of a 16-world sample."""
import io
import os

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def load_finish_policy():
    from g1env import AC
    z = np.load(os.path.join(HERE, "golden", "finish_policy.npz"))
    sd = {k[len("param."):]: torch.tensor(z[k]) for k in z.files if k.startswith("param.")}
    ac = AC(100, 29)
    ac.load_state_dict(sd, strict=True)
    ac.eval()
    return ac, torch.tensor(z["obs_mean"]), torch.tensor(z["obs_var"]), z


def test_reference_checkpoint_packs_in_rollout_order():
    from g1env import pack_weights
    ac, _, _, z = load_finish_policy()
    W = pack_weights(ac).detach().numpy()
    p = lambda k: z["param." + k].reshape(-1)
    ref = np.concatenate([p("body.0.weight"), p("body.0.bias"), p("body.2.weight"), p("body.2.bias"),
                          p("mu.weight"), p("mu.bias"), p("v.weight"), p("v.bias"), p("log_std")])
    assert W.shape == (99387,)
    assert np.array_equal(W, ref)


def test_trainer_checkpoint_roundtrip():
    from g1env import AC, RunNorm
    ac, mean, var, _ = load_finish_policy()
    norm = RunNorm(100, "cpu")
    norm.mean, norm.var = mean.clone(), var.clone()
    buf = io.BytesIO()
    torch.save(dict(model=ac.state_dict(), obs_mean=norm.mean, obs_var=norm.var), buf)
    buf.seek(0)
    ck = torch.load(buf)
    ac2 = AC(100, 29)
    ac2.load_state_dict(ck["model"], strict=True)
    for (k, a), (_, b) in zip(ac.state_dict().items(), ac2.state_dict().items()):
        assert torch.equal(a, b), k
    assert torch.equal(ck["obs_mean"], mean) and torch.equal(ck["obs_var"], var)


def playback(env, ac, mean, var, N, steps):
    """Deterministic playback (scripts/play_finish.py): returns per world the first done step
    (-1 if none) and whether that done was a win (the +50 finish bonus is in its reward)."""
    obs = torch.tensor(np.asarray(env.reset()), dtype=torch.float32)
    first = np.full(N, -1)
    won = np.zeros(N, bool)
    with torch.no_grad():
        for t in range(steps):
            nobs = torch.clamp((obs - mean) / torch.sqrt(var + 1e-8), -10.0, 10.0)
            mu, _, _ = ac(nobs)
            o, r, d = env.step(mu.numpy())
            new = (np.asarray(d) > 0.5) & (first < 0)
            first[new] = t + 1
            won[new] = np.asarray(r)[new] > 25.0
            obs = torch.tensor(np.asarray(o), dtype=torch.float32)
            if (first > 0).all():
                break
    return first, won


def test_oracle_playback_reaches_finish_line():
    from oracle.oracle import Oracle, OracleEnv
    ac, mean, var, z = load_finish_policy()
    N = 16
    env = OracleEnv(Oracle("f32"), N, 10, 8, seed=0)
    first, won = playback(env, ac, mean, var, N, int(z["playback_max_steps"]))
    env.close()
    assert won.all(), (first, won)
