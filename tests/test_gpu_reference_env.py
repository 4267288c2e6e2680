"""The env step, observation, reward, done flags and policy MLP against the reference's OWN
env code: oracle/_ref/libg1env_ref.so is the reference's src/g1_env.cu compiled unchanged
for sm_100a (oracle/build_oracle.py), driven through its own C-ABI (g1_env.cu:405-467).

The reference draws curand numbers only on a reset (g1_env.cu:97-111, 206) and for the
action noise (:310).  So both tests start from the reference's own reset state (read back
with g1_env_qpos_all; qvel, prev_act and the step counters are zero after a reset) and avoid
every other draw:
  * host-loop steps (g1_env_step, :431-441) with fixed actions: no world is done within
    the few steps run, so no reset noise is drawn;
  * the fused rollout (g1_rollout, :446-453) with log-std -20: the sampled action is the
    mean to ~1e-9, whatever the noise stream.  LP carries the noise term and is left out.
The same states and actions also go through the fp32 CPU oracle, which pins the oracle's
restatement of the reward and observation (oracle/g1_oracle.c) to the reference itself.

Tolerances: the first step's observation within relative L2 1e-5 per world (one control
step of the same fp32 arithmetic, differently rounded); later observations within 1e-3
absolute (rounding differences grow over contact-rich substeps, as in the rollout gates);
reward within 1e-4; done flags exact.  Rollouts run H = 4 control steps at N = 128, as the
rollout gates against the oracle, and H = 2 at the full N = 8192."""
import ctypes
import os

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_ENV = os.path.join(ROOT, "oracle", "_ref", "libg1env_ref.so")
NQ, NV, ACT, OBS = 36, 35, 29, 100
_vp = ctypes.c_void_p


@pytest.fixture(scope="module")
def ref():
    if not os.path.exists(REF_ENV):
        pytest.fail("oracle/_ref/libg1env_ref.so is missing: build it with oracle/build_oracle.py "
                    "where the reference tree is present")
    lib = ctypes.CDLL(REF_ENV)
    lib.g1_env_create.restype = _vp
    lib.g1_env_create.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_ulong]
    lib.g1_env_reset.argtypes = [_vp, _vp]
    lib.g1_env_step.argtypes = [_vp] * 5
    lib.g1_rollout.argtypes = [_vp, ctypes.c_int] + [_vp] * 10
    lib.g1_env_qpos_all.argtypes = [_vp, _vp]
    lib.g1_env_destroy.argtypes = [_vp]
    return lib


@pytest.fixture(scope="module")
def g1():
    import g1env
    g1env.load_library()
    return g1env


def _np(a):
    return a.ctypes.data_as(_vp)


def _ref_reset(ref, N, seed):
    h = ref.g1_env_create(N, 10, 8, seed)
    obs0 = np.zeros((N, OBS), np.float32)
    ref.g1_env_reset(h, _np(obs0))
    qp = np.zeros((N, NQ), np.float32)
    ref.g1_env_qpos_all(h, _np(qp))
    return h, qp, obs0


def _relrows(a, b):
    return np.linalg.norm(a - b, axis=1) / (np.linalg.norm(b, axis=1) + 1e-30)


def test_host_step_obs_reward_done_vs_reference_env(ref, g1):
    from oracle.oracle import Oracle, OracleEnv
    N, K = 64, 8
    h, qp, obs_ref0 = _ref_reset(ref, N, seed=11)
    zv, zp, zs = np.zeros((N, NV), np.float32), np.zeros((N, ACT), np.float32), np.zeros(N, np.int32)
    env = g1.G1Env(N, 10, 8, seed=11)
    env.set_state(qp, zv, zp, zs)
    oenv = OracleEnv(Oracle("f32"), N, 10, 8, seed=11)
    oenv.set_state(qp, zv, zp, zs)
    rng = np.random.default_rng(5)
    acts = rng.uniform(-0.6, 0.6, (K, N, ACT)).astype(np.float32)
    ro, rr, rd = np.zeros((N, OBS), np.float32), np.zeros(N, np.float32), np.zeros(N, np.float32)
    for k in range(K):
        a = np.ascontiguousarray(acts[k])
        ref.g1_env_step(h, _np(a), _np(ro), _np(rr), _np(rd))
        go, gr, gd = env.step(a)
        oo, orr, od = oenv.step(a)
        assert not rd.any(), "a world finished its episode: the reference would draw reset noise"
        for name, o in (("cuda", go), ("oracle", oo)):
            if k == 0:
                assert _relrows(o, ro).max() <= 1e-5, (name, "obs", _relrows(o, ro).max())
            assert np.abs(o - ro).max() <= 1e-3, (name, "obs", k, np.abs(o - ro).max())
        assert np.abs(gr - rr).max() <= 1e-4, ("cuda reward", k, np.abs(gr - rr).max())
        assert np.abs(orr - rr).max() <= 1e-4, ("oracle reward", k, np.abs(orr - rr).max())
        assert np.array_equal(gd, rd) and np.array_equal(od, rd)
    qref = np.zeros((N, NQ), np.float32)
    ref.g1_env_qpos_all(h, _np(qref))
    assert np.abs(env.get_state()[0] - qref).max() <= 1e-3
    assert env.get_state()[3].tolist() == [K] * N          # episode counters
    ref.g1_env_destroy(h)
    env.close()
    oenv.close()


@pytest.mark.parametrize("precision,N,H", [("fp32", 128, 4), ("fp32-ffma", 128, 4), ("fp32", 8192, 2)])
def test_fused_rollout_vs_reference_env(ref, g1, precision, N, H):
    """N = 8192 runs the production grid (147 CTAs, two rounds of groups per CTA)."""
    from oracle.oracle import Oracle, OracleEnv
    h, qp, _ = _ref_reset(ref, N, seed=23)
    zv, zp, zs = np.zeros((N, NV), np.float32), np.zeros((N, ACT), np.float32), np.zeros(N, np.int32)
    env = g1.G1Env(N, 10, 8, seed=23)
    env.set_policy((256, 256), "tanh", precision=precision)
    env.set_state(qp, zv, zp, zs)
    ac = g1.init_policy_normal(g1.AC(100, 29).cuda(), seed=9)
    with torch.no_grad():
        ac.log_std.fill_(-20.0)        # sampled action == mean to ~1e-9 (g1_env.cu:308-312)
    W = g1.pack_weights(ac).detach().contiguous()
    rng = np.random.default_rng(1)
    mean = torch.tensor(rng.normal(0, 0.1, OBS), dtype=torch.float32).cuda()
    var = torch.tensor(rng.uniform(0.5, 2.0, OBS), dtype=torch.float32).cuda()
    z = lambda *s: torch.zeros(*s, device="cuda")
    mk = lambda: dict(O=z(H, N, OBS), A=z(H, N, ACT), LP=z(H, N), V=z(H, N), R=z(H, N), D=z(H, N), Vlast=z(N))
    rb, gb = mk(), mk()
    torch.cuda.synchronize()
    ref.g1_rollout(h, H, *[_vp(t.data_ptr()) for t in (W, mean, var)], *[_vp(t.data_ptr()) for t in rb.values()])
    torch.cuda.synchronize()
    env.rollout(H, W, mean, var, *gb.values())
    torch.cuda.synchronize()
    r = {k: v.cpu().numpy() for k, v in rb.items()}
    g = {k: v.cpu().numpy() for k, v in gb.items()}
    assert not r["D"].any(), "a world finished its episode: the reference would draw reset noise"
    assert _relrows(g["O"][0], r["O"][0]).max() <= 1e-5
    tol = dict(O=1e-3, A=1e-4, V=1e-4, R=1e-4, Vlast=1e-4)
    # The reference's k_rollout, built for sm_100a here, writes NaN into every Vlast entry
    # (its O/A/LP/V/R/D are finite and agree); Vlast is then pinned to the oracle, whose
    # bootstrap value restates g1_env.cu:323-330, and compared with the reference only where
    # the reference's is finite.
    ref_vlast_ok = np.isfinite(r["Vlast"]).all()
    if not ref_vlast_ok:
        print("reference Vlast is not finite on this build; Vlast checked against the oracle only")
        tol_ref = {k: v for k, v in tol.items() if k != "Vlast"}
    else:
        tol_ref = tol
    for k, t in tol_ref.items():
        print(f"{precision} {k}: max |cuda - reference| {np.abs(g[k] - r[k]).max():.2e}")
        assert np.abs(g[k] - r[k]).max() <= t, (k, np.abs(g[k] - r[k]).max())
    assert np.array_equal(g["D"], r["D"])
    # the oracle's restatement of the same rollout
    oenv = OracleEnv(Oracle("f32"), N, 10, 8, seed=23)
    oenv.set_state(qp, zv, zp, zs)
    ro = oenv.rollout(H, W.cpu().numpy(), mean.cpu().numpy(), var.cpu().numpy(), act="tanh")
    for k, t in tol_ref.items():
        assert np.abs(ro[k] - r[k]).max() <= t, ("oracle", k, np.abs(ro[k] - r[k]).max())
    assert np.abs(g["Vlast"] - ro["Vlast"]).max() <= tol["Vlast"]
    qref = np.zeros((N, NQ), np.float32)
    ref.g1_env_qpos_all(h, _np(qref))
    assert np.abs(env.get_state()[0] - qref).max() <= 1e-3
    ref.g1_env_destroy(h)
    env.close()
    oenv.close()
