"""Playback of the reference's trained finish-line walker (models/ppo_ckpt/finish_best.pt,
exported to tests/golden/finish_policy.npz) through the CUDA env's host-loop step path
(g1_env_step, the path scripts/play_finish.py drives).

* The reference reports 256/256 worlds across x = 5 m within 480 deterministic control steps
  (DEVLOG.md:421-422).  Reset noise here comes from Philox, not curand, so the worlds start
  from different (equally distributed) perturbations: the gate is >= 252/256, the measured
  count is printed.
* Closed-loop parity with the CPU oracle from identical reset states.  Over ~370 control
  steps (3,700 substeps of walking with contacts) rounding differences grow chaotically, so
  finishing steps are compared against the oracle's own fp32-vs-fp64 spread on the same
  worlds: the same worlds win, and the mean |step(GPU) - step(fp32 oracle)| is at most
  2x the mean |step(fp64 oracle) - step(fp32 oracle)| + 1 (and the mean finishing step
  differs by at most 5)."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_trained_walker_reaches_finish_line():
    import g1env
    from test_checkpoint import load_finish_policy, playback
    ac, mean, var, z = load_finish_policy()
    N = int(z["playback_worlds"])
    env = g1env.G1Env(N, 10, 8, seed=0)
    first, won = playback(env, ac, mean, var, N, int(z["playback_max_steps"]))
    env.close()
    print(f"trained walker: {int(won.sum())}/{N} worlds reached x = 5 m; "
          f"median finishing step {int(np.median(first[won])) if won.any() else -1}")
    assert won.sum() >= 252


def test_playback_matches_oracle():
    import g1env
    from oracle.oracle import Oracle, OracleEnv
    from test_checkpoint import load_finish_policy, playback
    ac, mean, var, z = load_finish_policy()
    N, steps = 32, int(z["playback_max_steps"])
    genv = g1env.G1Env(N, 10, 8, seed=4)

    class Started:  # an env already placed in its start state: reset() returns that state's obs
        def __init__(self, env, obs0):
            self.env, self.obs0 = env, obs0

        def reset(self):
            return self.obs0

        def step(self, a):
            return self.env.step(a)

    g_obs0 = genv.reset()
    st = genv.get_state()
    res = {}
    for tag in ("f32", "f64"):
        oenv = OracleEnv(Oracle(tag), N, 10, 8, seed=4)
        oenv.set_state(*st[:4], tick=st[4])
        res[tag] = playback(Started(oenv, g_obs0), ac, mean, var, N, steps)
        oenv.close()
    gf, gw = playback(Started(genv, g_obs0), ac, mean, var, N, steps)
    genv.close()
    of, ow = res["f32"]
    df, dw = res["f64"]
    d_gpu = np.abs(gf - of).mean()
    d_ref = np.abs(df - of).mean()
    print(f"finishing steps: gpu mean {gf.mean():.1f}, oracle fp32 {of.mean():.1f}, fp64 {df.mean():.1f}; "
          f"mean |gpu - fp32| {d_gpu:.2f}, mean |fp64 - fp32| {d_ref:.2f}")
    assert gw.all() and np.array_equal(gw, ow) and np.array_equal(dw, ow)
    assert d_gpu <= 2 * d_ref + 1
    assert abs(gf.mean() - of.mean()) <= 5
