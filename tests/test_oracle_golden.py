"""Pin the CPU oracle (oracle/g1_oracle.c) against the reference's MuJoCo goldens and
against the reference's own arithmetic (its physics headers compiled for the host),
with the thresholds of the reference's own gates:
  tests/test_m0.py:43-71 (bias 1e-5, qacc 1e-4, trajectory 1e-4),
  scripts/test_implicit.py:53-56 (single-step qvel 1e-3),
  src/test_envqacc.cu:76-90 (env_qacc vs the frozen fp32 reference, 1e-5)."""
import numpy as np
import pytest

from oracle.oracle import NQ, Oracle, RefHost


def rel(a, b):
    return np.linalg.norm(a - b) / np.linalg.norm(b)


@pytest.fixture(scope="module")
def o64():
    return Oracle("f64")


@pytest.fixture(scope="module")
def o32():
    return Oracle("f32")


@pytest.mark.parametrize("prec", ["f64", "f32"])
def test_smooth_bias_and_qacc_vs_mujoco(golden, prec):
    o = Oracle(prec)
    z = golden["mujoco_smooth"]
    r = o.qacc(z["qpos_at_q"][:1], z["qvel_at_q"][:1], None, None, 8)  # step 0 (test_m0.py:49-56)
    assert rel(r["bias"][0], z["qfrc_bias"][0]) < 1e-5
    assert rel(r["qacc"][0], z["qacc"][0]) < 1e-4


@pytest.mark.parametrize("prec", ["f64", "f32"])
def test_smooth_trajectory_vs_mujoco(golden, prec):
    o = Oracle(prec)
    z = golden["mujoco_smooth"]
    qp, _, _ = o.smooth_traj(z["qpos"][0], z["qvel"][0], 300)
    q = qp[z["steps"]]
    rq = z["qpos"]
    assert np.abs(q[:, :3] - rq[:, :3]).max() < 1e-4
    assert np.abs(q[:, 7:] - rq[:, 7:]).max() < 1e-4
    dq = np.minimum(np.abs(q[:, 3:7] - rq[:, 3:7]).sum(1), np.abs(q[:, 3:7] + rq[:, 3:7]).sum(1)).max()
    assert dq < 1e-4


@pytest.mark.parametrize("prec,tol", [("f64", 1e-5), ("f32", 3e-5)])
def test_contact_qacc_vs_mujoco(golden, prec, tol):
    """Pure foot-ground states at 2000 PGS iterations vs MuJoCo's converged qacc (the
    reference's sim_contact validate mode measured fp32 2.24e-5, DEVLOG.md:251,272)."""
    o = Oracle(prec)
    c = golden["mujoco_contact"]
    r = o.qacc(c["qpos"], c["qvel"], None, None, 2000)
    assert (r["ncon"] == c["ncon"]).all()
    for i in range(len(c["ncon"])):
        assert rel(r["qacc"][i], c["qacc"][i]) < tol, (i, c["label"][i])


@pytest.mark.parametrize("prec", ["f64", "f32"])
def test_implicit_pd_vs_mujoco(golden, prec):
    o = Oracle(prec)
    m = golden["mujoco_implicit"]
    qp, qv = o.pd_traj(m["qpos"][0], m["qvel"][0], m["targets"], pgs=8)
    assert np.abs(qv[1] - m["qvel"][1]).max() < 1e-3          # test_implicit.py:53-56
    assert np.isfinite(qv).all()
    assert np.abs(qp[-1] - m["qpos"][-1]).max() < 1e-4


def test_oracle_f32_is_bit_exact_with_reference_fp32(golden, o32):
    """The fp32 oracle reproduces the reference's host-compiled fp32 env_qacc bit for bit."""
    z = golden["ref_envqacc"]
    r = o32.qacc(z["qpos"], z["qvel"], z["tau"], z["bdt"], 8)
    assert np.array_equal(r["qacc"], z["qacc_f32"])
    assert np.array_equal(r["bias"], z["bias_f32"])
    r = o32.qacc(z["qpos"], z["qvel"], z["tau"], z["bdt"], 200)
    assert np.array_equal(r["qacc"], z["qacc_f32_pgs200"])
    r = o32.qacc(z["qpos"], z["qvel"], z["tau"], z["bdt"], 8, mu=1.0)
    assert np.array_equal(r["qacc"], z["qacc_f32_mu1"])
    c = golden["ref_config1"]
    r = o32.qacc(c["qpos"], c["qvel"], None, z["bdt"], 8)
    assert np.array_equal(r["qacc"], c["qacc_f32"])


def test_oracle_f64_close_to_reference_fp64(golden, o64):
    z = golden["ref_envqacc"]
    r = o64.qacc(z["qpos"], z["qvel"], z["tau"], z["bdt"], 8)
    e = np.linalg.norm(r["qacc"] - z["qacc_f64"], axis=1) / np.linalg.norm(z["qacc_f64"], axis=1)
    assert e.max() < 1e-5


@pytest.mark.skipif(not RefHost.available("f32"), reason="reference host build (oracle/_ref) not present")
def test_oracle_live_vs_reference_build(o32):
    from oracle.oracle import envqacc_states, default_bdt
    qp, qv = envqacc_states(256, seed=4242)
    r = RefHost("f32").qacc(qp, qv, None, default_bdt(), 8)
    assert np.array_equal(o32.qacc(qp, qv, None, default_bdt(), 8)["qacc"], r)


def test_env_step_done_and_counters(o32):
    """Integer logic of env_advance (g1_env.cu:193-210): the episode counter, the timeout at
    step 1000 and the auto-reset are exact."""
    from oracle.oracle import OracleEnv, stand_pose
    env = OracleEnv(o32, 4, substeps=2, pgs_iters=8, seed=3)
    env.reset()
    qp, qv, pa, st, tick = env.get_state()
    st[:] = [0, 998, 999, 500]
    env.set_state(qp, qv, pa, st, tick)
    _, _, done = env.step(np.zeros((4, 29)))
    _, _, _, st2, tick2 = env.get_state()
    assert tick2 == tick + 1
    assert done[2] == 1.0 and st2[2] == 0               # timeout -> reset counter
    assert st2[0] == 1 and st2[1] == 999 and st2[3] == 501
    assert done[0] == 0.0 and done[1] == 0.0
    # a fallen world (base height below 0.45) terminates and respawns at the stand pose
    qp, qv, pa, st, tick = env.get_state()
    qp[0, 2] = 0.3
    env.set_state(qp, qv, pa, st, tick)
    _, rew, done = env.step(np.zeros((4, 29)))
    assert done[0] == 1.0 and rew[0] == -5.0
    qp2, qv2, _, st3, _ = env.get_state()
    assert st3[0] == 0 and np.all(qv2[0] == 0)
    assert abs(qp2[0, 2] - stand_pose()[2]) < 1e-6
