"""ctypes front-end of the CPU oracle (oracle/g1_oracle.c) and of the reference's host
builds (oracle/_ref).  TEST INFRASTRUCTURE: imported only by tests/, __graft_entry__.smoke()
and bench.py's CPU-baseline legs, always as the checker.
"""
import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
NQ, NV, NB, OBS, ACT, MAXEFC = 36, 35, 31, 100, 29, 32

_c_int, _c_u64, _c_u32 = ctypes.c_int, ctypes.c_uint64, ctypes.c_uint32
_vp = ctypes.c_void_p


def _ptr(a):
    return None if a is None else a.ctypes.data_as(_vp)


class Oracle:
    """The C restatement, fp32 ('f32') or fp64 ('f64')."""

    def __init__(self, prec="f64"):
        path = os.path.join(HERE, f"liboracle_{prec}.so")
        if not os.path.exists(path):
            from oracle.build_oracle import build_oracle  # noqa: local build on demand
            build_oracle()
        self.lib = ctypes.CDLL(path)
        self.dt = np.float32 if prec == "f32" else np.float64
        real = ctypes.c_float if prec == "f32" else ctypes.c_double
        self._real = real
        L = self.lib
        L.orc_qacc.argtypes = [_c_int, _vp, _vp, _vp, _vp, _c_int, real, _vp, _vp, _vp, _vp, _vp]
        L.orc_fk.argtypes = [_c_int, _vp, _vp, _vp, _vp]
        L.orc_smooth_traj.argtypes = [_vp, _vp, _vp, _c_int, _vp, _vp, _vp]
        L.orc_pd_traj.argtypes = [_vp, _vp, _vp, _c_int, _c_int, real, _vp, _vp]
        L.orc_philox_block.argtypes = [_vp, _vp, _vp]
        L.orc_env_create.restype = _vp
        L.orc_env_create.argtypes = [_c_int, _c_int, _c_int, _c_u64, _c_u32, real]
        L.orc_env_destroy.argtypes = [_vp]
        L.orc_env_set_state.argtypes = [_vp, _vp, _vp, _vp, _vp, _c_u64]
        L.orc_env_get_state.argtypes = [_vp, _vp, _vp, _vp, _vp, _vp]
        L.orc_env_reset.argtypes = [_vp, _vp]
        L.orc_env_step.argtypes = [_vp, _vp, _vp, _vp, _vp]
        L.orc_env_bench_phys.argtypes = [_vp, _c_int, _c_int]
        L.orc_rollout.argtypes = [_vp, _c_int, _vp, _vp, _vp, _c_int, _vp, _c_int] + [_vp] * 7 + [_c_int]

    def _a(self, x, shape=None):
        a = np.ascontiguousarray(x, dtype=self.dt)
        if shape is not None:
            a = a.reshape(shape)
        return a

    def fk(self, qpos):
        qpos = self._a(qpos, (-1, NQ)); n = qpos.shape[0]
        xp = np.zeros((n, NB, 3), self.dt); xq = np.zeros((n, NB, 4), self.dt); xi = np.zeros((n, NB, 3), self.dt)
        self.lib.orc_fk(n, _ptr(qpos), _ptr(xp), _ptr(xq), _ptr(xi))
        return xp, xq, xi

    def qacc(self, qpos, qvel, tau=None, bdt=None, pgs=8, mu=0.6):
        """FK + env_qacc per state.  Returns dict(qacc, qacc_s, bias, f, ncon)."""
        qpos = self._a(qpos, (-1, NQ)); n = qpos.shape[0]
        qvel = self._a(qvel, (n, NV))
        tau = self._a(np.zeros((n, NV)) if tau is None else tau, (n, NV))
        bdt = None if bdt is None else self._a(np.broadcast_to(bdt, (n, NV)), (n, NV))
        out = {k: np.zeros((n, NV), self.dt) for k in ("qacc", "qacc_s", "bias")}
        out["f"] = np.zeros((n, MAXEFC), self.dt)
        out["ncon"] = np.zeros(n, np.int32)
        self.lib.orc_qacc(n, _ptr(qpos), _ptr(qvel), _ptr(tau), _ptr(bdt), pgs, mu,
                          _ptr(out["qacc"]), _ptr(out["qacc_s"]), _ptr(out["bias"]), _ptr(out["f"]), _ptr(out["ncon"]))
        return out

    def smooth_traj(self, qpos0, qvel0, nsteps, tau=None):
        qp = np.zeros((nsteps + 1, NQ), self.dt); qv = np.zeros((nsteps + 1, NV), self.dt)
        qa = np.zeros((nsteps, NV), self.dt)
        t = None if tau is None else self._a(tau, (NV,))
        self.lib.orc_smooth_traj(_ptr(self._a(qpos0)), _ptr(self._a(qvel0)), _ptr(t), nsteps, _ptr(qp), _ptr(qv), _ptr(qa))
        return qp, qv, qa

    def pd_traj(self, qpos0, qvel0, targets, pgs=8, mu=0.6):
        targets = self._a(targets, (-1, ACT)); n = targets.shape[0]
        qp = np.zeros((n + 1, NQ), self.dt); qv = np.zeros((n + 1, NV), self.dt)
        self.lib.orc_pd_traj(_ptr(self._a(qpos0)), _ptr(self._a(qvel0)), _ptr(targets), n, pgs, mu, _ptr(qp), _ptr(qv))
        return qp, qv

    def philox(self, ctr, key):
        c = np.ascontiguousarray(ctr, np.uint32); k = np.ascontiguousarray(key, np.uint32)
        o = np.zeros(4, np.uint32)
        self.lib.orc_philox_block(_ptr(c), _ptr(k), _ptr(o))
        return o


class OracleEnv:
    """Oracle twin of the env handle (g1_env_create semantics, g1_env.cu:405-422)."""

    def __init__(self, oracle, N, substeps=10, pgs_iters=8, seed=1, world0=0, mu=0.6):
        self.o, self.N = oracle, N
        self.h = oracle.lib.orc_env_create(N, substeps, pgs_iters, seed, world0, mu)

    def close(self):
        if self.h:
            self.o.lib.orc_env_destroy(self.h)
            self.h = None

    __del__ = close

    def set_state(self, qp, qv, pa, steps, tick=0):
        o = self.o
        self._keep = [o._a(qp, (self.N, NQ)), o._a(qv, (self.N, NV)), o._a(pa, (self.N, ACT)),
                      np.ascontiguousarray(steps, np.int32)]
        o.lib.orc_env_set_state(self.h, *[_ptr(a) for a in self._keep], tick)

    def get_state(self):
        o = self.o
        qp = np.zeros((self.N, NQ), o.dt); qv = np.zeros((self.N, NV), o.dt); pa = np.zeros((self.N, ACT), o.dt)
        st = np.zeros(self.N, np.int32); tick = np.zeros(1, np.uint64)
        o.lib.orc_env_get_state(self.h, _ptr(qp), _ptr(qv), _ptr(pa), _ptr(st), _ptr(tick))
        return qp, qv, pa, st, int(tick[0])

    def reset(self):
        obs = np.zeros((self.N, OBS), self.o.dt)
        self.o.lib.orc_env_reset(self.h, _ptr(obs))
        return obs

    def step(self, act):
        o = self.o
        act = o._a(act, (self.N, ACT))
        obs = np.zeros((self.N, OBS), o.dt); rew = np.zeros(self.N, o.dt); done = np.zeros(self.N, o.dt)
        o.lib.orc_env_step(self.h, _ptr(act), _ptr(obs), _ptr(rew), _ptr(done))
        return obs, rew, done

    def bench_phys(self, K, nworlds=0):
        self.o.lib.orc_env_bench_phys(self.h, K, nworlds)

    def rollout(self, H, W, mean, var, hidden=(256, 256), act="tanh", nworlds=0):
        o, N = self.o, self.N
        W = np.ascontiguousarray(W, np.float32); mean = np.ascontiguousarray(mean, np.float32)
        var = np.ascontiguousarray(var, np.float32)
        hid = np.ascontiguousarray(hidden, np.int32)
        out = dict(O=np.zeros((H, N, OBS), o.dt), A=np.zeros((H, N, ACT), o.dt), LP=np.zeros((H, N), o.dt),
                   V=np.zeros((H, N), o.dt), R=np.zeros((H, N), o.dt), D=np.zeros((H, N), o.dt),
                   Vlast=np.zeros(N, o.dt))
        o.lib.orc_rollout(self.h, H, _ptr(W), _ptr(mean), _ptr(var), len(hidden), _ptr(hid), 0 if act == "tanh" else 1,
                          *[_ptr(out[k]) for k in ("O", "A", "LP", "V", "R", "D", "Vlast")], nworlds)
        return out


class RefHost:
    """The reference's own physics headers compiled for the host (oracle/_ref)."""

    def __init__(self, tag="f32"):
        path = os.path.join(HERE, "_ref", f"libg1ref_host_{tag}.so")
        self.lib = ctypes.CDLL(path)
        self.dt = np.float64 if tag == "f64" else np.float32
        L = self.lib
        L.ref_fk.argtypes = [_c_int, _vp, _vp, _vp, _vp]
        L.ref_bias.argtypes = [_c_int, _vp, _vp, _vp]
        L.ref_qacc.argtypes = [_c_int, _vp, _vp, _vp, _vp, _c_int, _vp]
        L.ref_integrate.argtypes = [_c_int, _vp, _vp]

    @staticmethod
    def available(tag="f32"):
        return os.path.exists(os.path.join(HERE, "_ref", f"libg1ref_host_{tag}.so"))

    def qacc(self, qpos, qvel, tau=None, bdt=None, pgs=8):
        qpos = np.ascontiguousarray(qpos, self.dt).reshape(-1, NQ); n = qpos.shape[0]
        qvel = np.ascontiguousarray(qvel, self.dt).reshape(n, NV)
        tau = np.ascontiguousarray(np.zeros((n, NV)) if tau is None else tau, self.dt).reshape(n, NV)
        bd = None if bdt is None else np.ascontiguousarray(np.broadcast_to(bdt, (n, NV)), self.dt)
        out = np.zeros((n, NV), self.dt)
        self.lib.ref_qacc(n, _ptr(qpos), _ptr(qvel), _ptr(tau), _ptr(bd), pgs, _ptr(out))
        return out

    def bias(self, qpos, qvel):
        qpos = np.ascontiguousarray(qpos, self.dt).reshape(-1, NQ); n = qpos.shape[0]
        out = np.zeros((n, NV), self.dt)
        self.lib.ref_bias(n, _ptr(qpos), _ptr(np.ascontiguousarray(qvel, self.dt).reshape(n, NV)), _ptr(out))
        return out

    def fk(self, qpos):
        qpos = np.ascontiguousarray(qpos, self.dt).reshape(-1, NQ); n = qpos.shape[0]
        xp = np.zeros((n, NB, 3), self.dt); xq = np.zeros((n, NB, 4), self.dt); xi = np.zeros((n, NB, 3), self.dt)
        self.lib.ref_fk(n, _ptr(qpos), _ptr(xp), _ptr(xq), _ptr(xi))
        return xp, xq, xi


# ----------------------------------------------------------------- shared seeded inputs
def stand_pose():
    """The stand keyframe (reference g1_model.h:377-414), read from the committed model data."""
    import re
    txt = open(os.path.join(HERE, "..", "g1.cu_b200", "csrc", "g1_model_data.h")).read()
    body = re.search(r"G1M_QPOS_STAND\[36\] = \{(.*?)\};", txt, re.S).group(1)
    return np.array([float(v.strip().rstrip("f")) for v in body.split(",") if v.strip()])


def envqacc_states(n, seed=999):
    """Random states with the distribution of the reference's env_qacc gate
    (src/test_envqacc.cu:33-39): stand +-0.2 on every qpos entry, base z lowered by
    U(0,0.15), unit base quaternion, qvel U(-1,1).  Drawn with numpy (not curand)."""
    rng = np.random.default_rng(seed)
    stand = stand_pose()
    qpos = stand[None, :] + 0.2 * (rng.random((n, NQ)) * 2 - 1)
    qpos[:, 2] -= 0.15 * rng.random(n)
    qpos[:, 3:7] /= np.linalg.norm(qpos[:, 3:7], axis=1, keepdims=True)
    qvel = rng.random((n, NV)) * 2 - 1
    return qpos.astype(np.float32), qvel.astype(np.float32)


def config0_states(n, seed=0):
    """Config 0/1 seeded states: stand + N(0,0.05) joint noise, unit base quat,
    qvel ~ N(0,0.5); base z ~ U(0.75,0.8) (config 1)."""
    rng = np.random.default_rng(seed)
    stand = stand_pose()
    qpos = np.tile(stand, (n, 1))
    qpos[:, 7:] += rng.normal(0, 0.05, (n, NQ - 7))
    qpos[:, 3:7] /= np.linalg.norm(qpos[:, 3:7], axis=1, keepdims=True)
    qpos[:, 2] = rng.uniform(0.75, 0.8, n)
    qvel = rng.normal(0, 0.5, (n, NV))
    return qpos, qvel


def default_bdt():
    """dt * kd on the actuated dofs (g1_env.cu:137-139)."""
    import re
    txt = open(os.path.join(HERE, "..", "g1.cu_b200", "csrc", "g1_model_data.h")).read()
    kd = re.search(r"G1M_ACT_KD\[29\] = \{(.*?)\};", txt, re.S).group(1)
    kd = np.array([float(v.strip().rstrip("f")) for v in kd.split(",") if v.strip()], np.float32)
    b = np.zeros(NV, np.float32)
    b[6:] = np.float32(0.002) * kd
    return b
