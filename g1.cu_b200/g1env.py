"""Python host side of the B200 G1 rollout: the ctypes binding of libg1env.so plus the
trainer-facing classes, under the names the reference's scripts use
(scripts/ppo.py:24-125: the ctypes binding, G1Env, RunNorm, AC, evaluate;
scripts/ppo_fused.py:27-44: the g1_rollout binding and pack_weights).

The CUDA library is required: importing works on a CPU-only machine, but creating an env
or calling a kernel entry point raises if libg1env.so is missing or no GPU is visible --
there is no CPU fallback.
"""
import ctypes
import os

import numpy as np
import torch
import torch.nn as nn

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "libg1env.so")
OBS_DIM, ACT_DIM, NQ, NV = 100, 29, 36, 35

_fp = ctypes.POINTER(ctypes.c_float)
_vp = ctypes.c_void_p
_lib = None

# exported symbols and their ctypes signatures (include/g1env.h)
SIGNATURES = {
    "g1_env_create": (_vp, [ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_ulong]),
    "g1_env_create_ex": (_vp, [ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_ulong, ctypes.c_int, ctypes.c_uint,
                               ctypes.c_float]),
    "g1_env_destroy": (None, [_vp]),
    "g1_env_reset": (None, [_vp, _fp]),
    "g1_env_step": (None, [_vp, _fp, _fp, _fp, _fp]),
    "g1_env_step_device": (None, [_vp] + [_vp] * 4),
    "g1_rollout": (None, [_vp, ctypes.c_int] + [_vp] * 10),
    "g1_rollout_noalloc": (None, [_vp, ctypes.c_int] + [_vp] * 10),
    "g1_env_bench_phys": (None, [_vp, ctypes.c_int]),
    "g1_env_phys_async": (None, [_vp, ctypes.c_int]),
    "g1_env_phys_actions": (None, [_vp, ctypes.c_int, _vp]),
    "g1_env_qpos": (None, [_vp, _fp]),
    "g1_env_qpos_all": (None, [_vp, _fp]),
    "g1_env_obs_dim": (ctypes.c_int, []),
    "g1_env_act_dim": (ctypes.c_int, []),
    "g1_occupancy_report": (None, []),
    "g1_env_last_error": (ctypes.c_char_p, []),
    "g1_env_last_error_code": (ctypes.c_int, []),
    "g1_env_clear_error": (None, []),
    "g1_env_set_stream": (None, [_vp, _vp]),
    "g1_env_set_policy": (ctypes.c_int, [_vp, ctypes.c_int, _vp, ctypes.c_int]),
    "g1_env_set_friction": (None, [_vp, ctypes.c_float]),
    "g1_env_set_policy_ex": (ctypes.c_int, [_vp, ctypes.c_int, _vp, ctypes.c_int, ctypes.c_int]),
    "g1_env_tc_status": (ctypes.c_int, [_vp]),
    "g1_env_set_value_net": (ctypes.c_int, [_vp, ctypes.c_int, _vp]),
    "g1_env_get_state": (None, [_vp, _vp, _vp, _vp, _vp, _vp]),
    "g1_env_set_state": (None, [_vp, _vp, _vp, _vp, _vp, ctypes.c_ulonglong]),
    "g1_env_ncon_hist": (None, [_vp, ctypes.c_int, _vp]),
    "g1_gemm_bf16_tc": (ctypes.c_int, [ctypes.c_int, ctypes.c_int, ctypes.c_int, _vp, ctypes.c_int, _vp, _vp, ctypes.c_int,
                                       _vp]),
    "g1_dense_bf16x3": (ctypes.c_int, [ctypes.c_int] * 3 + [_vp] * 3 + [ctypes.c_int, _vp]),
    "g1_gae": (ctypes.c_int, [ctypes.c_int, ctypes.c_int] + [_vp] * 4 + [ctypes.c_double, ctypes.c_double] + [_vp] * 4),
    "g1_obs_prep": (ctypes.c_int, [ctypes.c_longlong, ctypes.c_int] + [_vp] * 6),
    "g1_adv_normalize": (ctypes.c_int, [ctypes.c_longlong, _vp, _vp, _vp]),
    "g1_runnorm_update": (ctypes.c_int, [ctypes.c_int, _vp, _vp, ctypes.c_double, _vp, _vp]),
    "g1_qacc_batch": (ctypes.c_int, [ctypes.c_int] + [_vp] * 4 + [ctypes.c_int, ctypes.c_float] + [_vp] * 5),
}


class G1Error(RuntimeError):
    pass


def load_library(path=LIB):
    """Load libg1env.so and bind every exported symbol (raises if it is missing)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise G1Error(f"{path} not built: run `python g1.cu_b200/build.py` (nvcc, sm_100a); "
                      "there is no CPU fallback")
    lib = ctypes.CDLL(path)
    for name, (res, args) in SIGNATURES.items():
        f = getattr(lib, name)
        f.restype = res
        f.argtypes = args
    _lib = lib
    return lib


def _check():
    code = _lib.g1_env_last_error_code()
    if code:
        msg = _lib.g1_env_last_error()
        _lib.g1_env_clear_error()
        raise G1Error(f"libg1env: {msg.decode() if msg else code}")


def _p(a):
    return a.ctypes.data_as(_fp)


def _dp(t):
    """device (or host numpy) pointer as c_void_p (ppo_fused.py:31-32)"""
    if t is None:
        return None
    if isinstance(t, np.ndarray):
        return t.ctypes.data_as(_vp)
    return ctypes.c_void_p(t.data_ptr())


def _require_gpu():
    if not torch.cuda.is_available():
        raise G1Error("no CUDA device visible: the G1 rollout runs only on the GPU (no CPU fallback)")


class G1Env:
    """Batched G1 env on one GPU (ppo.py:39-60).  All N worlds stay resident on the device."""

    def __init__(self, n_worlds, substeps=10, pgs_iters=2000, seed=0, device=None, world0=0, mu=0.6):
        _require_gpu()
        lib = load_library()
        self.N = n_worlds
        self.obs_dim = lib.g1_env_obs_dim()
        self.act_dim = lib.g1_env_act_dim()
        dev = torch.cuda.current_device() if device is None else int(device)
        self.device = dev
        self.h = lib.g1_env_create_ex(n_worlds, substeps, pgs_iters, seed, dev, world0, mu)
        if not self.h:
            _check()
            raise G1Error("g1_env_create failed")
        self._obs = np.zeros((n_worlds, self.obs_dim), np.float32)
        self._rew = np.zeros(n_worlds, np.float32)
        self._done = np.zeros(n_worlds, np.float32)

    def reset(self):
        _lib.g1_env_reset(self.h, _p(self._obs)); _check()
        return self._obs.copy()

    def step(self, act):
        act = np.ascontiguousarray(act, np.float32)
        _lib.g1_env_step(self.h, _p(act), _p(self._obs), _p(self._rew), _p(self._done)); _check()
        return self._obs.copy(), self._rew.copy(), self._done.copy()

    def step_device(self, act, obs, rew, done):
        """g1_env_step_device: one control step on CUDA tensors (act [N, 29] -> obs [N, 100],
        rew [N], done [N]), asynchronous on the env's stream."""
        _lib.g1_env_step_device(self.h, _dp(act), _dp(obs), _dp(rew), _dp(done)); _check()

    def set_stream(self, stream):
        _lib.g1_env_set_stream(self.h, ctypes.c_void_p(stream.cuda_stream if stream is not None else 0))

    def set_policy(self, hidden=(256, 256), activation="tanh", precision="fp32"):
        """precision "fp32": the in-kernel fp32-accurate policy (split-bf16 on the tensor cores when
        every hidden width is a multiple of 16 up to 256, else FFMA); "fp32-ffma": always FFMA;
        "bf16": tensor-core policy for wide MLPs."""
        hid = np.ascontiguousarray(hidden, np.int32)
        code = {"fp32": 0, "bf16": 1, "fp32-ffma": 2}[precision]
        rc = _lib.g1_env_set_policy_ex(self.h, len(hidden), _dp(hid), 0 if activation == "tanh" else 1, code)
        if rc:
            _check()

    def tc_status(self):
        return _lib.g1_env_tc_status(self.h)

    def set_value_net(self, hidden=()):
        """Separate value network for the bf16 tensor-core policy path;
        () returns to the shared trunk's value head."""
        hid = np.ascontiguousarray(hidden if len(hidden) else [0], np.int32)
        if _lib.g1_env_set_value_net(self.h, len(hidden), _dp(hid)):
            _check()

    def set_friction(self, mu):
        _lib.g1_env_set_friction(self.h, float(mu))

    def rollout(self, H, W, mean, var, O, A, LP, V, R, D, Vlast):
        """g1_rollout on torch-owned device tensors (ppo_fused.py:101-102)."""
        _lib.g1_rollout(self.h, H, _dp(W), _dp(mean), _dp(var), _dp(O), _dp(A), _dp(LP), _dp(V), _dp(R), _dp(D),
                        _dp(Vlast))
        _check()

    def rollout_noalloc(self, H, W, mean, var, O, A, LP, V, R, D, Vlast):
        """g1_rollout_noalloc: the same rollout without any device allocation (weights repacked
        into the library's fixed device area)."""
        _lib.g1_rollout_noalloc(self.h, H, _dp(W), _dp(mean), _dp(var), _dp(O), _dp(A), _dp(LP), _dp(V), _dp(R),
                                _dp(D), _dp(Vlast))
        _check()

    def bench_phys(self, K):
        _lib.g1_env_bench_phys(self.h, K); _check()

    def phys_async(self, K):
        _lib.g1_env_phys_async(self.h, K); _check()

    def phys_actions(self, K, act=None):
        """g1_env_phys_actions: K control steps of physics with a constant action per world
        (act: CUDA tensor [N, 29], None = zero), asynchronous."""
        _lib.g1_env_phys_actions(self.h, K, _dp(act.contiguous() if act is not None else None)); _check()

    def get_state(self):
        N = self.N
        qp = np.zeros((N, NQ), np.float32); qv = np.zeros((N, NV), np.float32); pa = np.zeros((N, ACT_DIM), np.float32)
        st = np.zeros(N, np.int32); tick = np.zeros(1, np.uint64)
        _lib.g1_env_get_state(self.h, _dp(qp), _dp(qv), _dp(pa), _dp(st), _dp(tick)); _check()
        return qp, qv, pa, st, int(tick[0])

    def set_state(self, qp, qv, pa, steps, tick=0):
        N = self.N
        a = [np.ascontiguousarray(qp, np.float32).reshape(N, NQ), np.ascontiguousarray(qv, np.float32).reshape(N, NV),
             np.ascontiguousarray(pa, np.float32).reshape(N, ACT_DIM), np.ascontiguousarray(steps, np.int32).reshape(N)]
        _lib.g1_env_set_state(self.h, *[_dp(x) for x in a], int(tick)); _check()

    def qpos(self):
        out = np.zeros(NQ, np.float32)
        _lib.g1_env_qpos(self.h, _p(out)); _check()
        return out

    def qpos_all(self):
        out = np.zeros((self.N, NQ), np.float32)
        _lib.g1_env_qpos_all(self.h, _p(out)); _check()
        return out

    def ncon_hist(self, enable=True):
        out = np.zeros(9, np.uint64)
        _lib.g1_env_ncon_hist(self.h, 1 if enable else 0, _dp(out)); _check()
        return out

    def close(self):
        if getattr(self, "h", None):
            _lib.g1_env_destroy(self.h)
            self.h = None


def qacc_batch(qpos, qvel, tau=None, bdt=None, pgs_iters=8, mu=0.6):
    """Per-state FK + generalized acceleration on the GPU (g1_qacc_batch).  Takes CUDA
    tensors; returns dict of CUDA tensors qacc, qacc_smooth, bias [n,35], f [n,32], ncon [n]."""
    _require_gpu()
    lib = load_library()
    n = qpos.shape[0]
    dev = qpos.device
    f32 = dict(dtype=torch.float32, device=dev)
    out = dict(qacc=torch.zeros(n, NV, **f32), qacc_smooth=torch.zeros(n, NV, **f32), bias=torch.zeros(n, NV, **f32),
               f=torch.zeros(n, 32, **f32), ncon=torch.zeros(n, dtype=torch.int32, device=dev))
    qpos = qpos.contiguous().float(); qvel = qvel.contiguous().float()
    tau = None if tau is None else tau.contiguous().float()
    bdt = None if bdt is None else bdt.expand(n, NV).contiguous().float()
    rc = lib.g1_qacc_batch(n, _dp(qpos), _dp(qvel), _dp(tau), _dp(bdt), pgs_iters, float(mu),
                           *[_dp(out[k]) for k in ("qacc", "qacc_smooth", "bias", "f", "ncon")])
    if rc:
        _check()
    return out


def gemm_bf16_tc(X, W, bias=None, act=-1):
    """out = act(X W^T + b) on the tensor cores (tcgen05).  X [M,K], W [N,K] bf16 CUDA tensors."""
    _require_gpu()
    lib = load_library()
    M, K = X.shape
    N = W.shape[0]
    out = torch.empty(M, N, dtype=torch.float32, device=X.device)
    X = X.contiguous(); W = W.contiguous()
    b = None if bias is None else bias.float().contiguous()
    rc = lib.g1_gemm_bf16_tc(M, N, K, _dp(X), K, _dp(W), _dp(b), act, _dp(out))
    if rc:
        _check()
    return out


def dense_bf16x3(X, W, bias=None, act=-1):
    """out = act(X W^T + b) with the rollout kernel's split-bf16 tensor-core layer (rows <= 64)."""
    _require_gpu()
    lib = load_library()
    X = X.float().contiguous(); W = W.float().contiguous()
    rows, K = X.shape
    N = W.shape[0]
    out = torch.empty(rows, N, dtype=torch.float32, device=X.device)
    b = None if bias is None else bias.float().contiguous()
    if lib.g1_dense_bf16x3(rows, K, N, _dp(X), _dp(W), _dp(b), act, _dp(out)):
        _check()
    return out


# ---------------- trainer batch preparation (ppo_fused.py:104-119, ppo.py:71-79) ----------------
def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def gae_device(R, V, D, Vlast, gamma=0.99, lam=0.95):
    """adv, ret [H,N] and the fp64 advantage moments [count, sum, sumsq] (g1_gae), on torch's
    current stream.  adv/ret are bit-identical to the reference's torch GAE loop."""
    _require_gpu()
    lib = load_library()
    H, N = R.shape
    adv, ret = torch.empty_like(R), torch.empty_like(R)
    mom = torch.empty(3, dtype=torch.float64, device=R.device)
    Rc, Vc, Dc, Lc = (t.contiguous() for t in (R, V, D, Vlast))
    if lib.g1_gae(H, N, _dp(Rc), _dp(Vc), _dp(Dc), _dp(Lc), gamma, lam, _dp(adv), _dp(ret), _dp(mom), _stream()):
        _check()
    return adv, ret, mom


def obs_prep_device(O, fmean, fvar):
    """nobs = clamp((O - fmean)/sqrt(fvar + 1e-8), -10, 10) and the fp64 raw-observation
    moments [rows, sum[dim], sumsq[dim]] in one pass (g1_obs_prep)."""
    _require_gpu()
    lib = load_library()
    dim = O.shape[-1]
    Oc = O.contiguous()
    rows = Oc.numel() // dim
    nobs = torch.empty_like(Oc)
    mom = torch.empty(1 + 2 * dim, dtype=torch.float64, device=O.device)
    fm, fv = fmean.float().contiguous(), fvar.float().contiguous()
    if lib.g1_obs_prep(rows, dim, _dp(Oc), _dp(fm), _dp(fv), _dp(nobs), _dp(mom), _stream()):
        _check()
    return nobs, mom


def adv_normalize_device(adv, adv_mom):
    """In place: adv = (adv - mean)/(std + 1e-8) from (possibly all-reduced) moments."""
    lib = load_library()
    assert adv.is_contiguous()
    if lib.g1_adv_normalize(adv.numel(), _dp(adv), _dp(adv_mom), _stream()):
        _check()
    return adv


def runnorm_update_device(norm, obs_mom, rows_total):
    """RunNorm.update (ppo.py:71-79) on the device from (possibly all-reduced) moments;
    rows_total = obs_mom[0], known on the host so nothing synchronises."""
    lib = load_library()
    assert norm.mean.is_contiguous() and norm.var.is_contiguous()
    if lib.g1_runnorm_update(norm.mean.numel(), _dp(norm.mean), _dp(norm.var), float(norm.count), _dp(obs_mom),
                             _stream()):
        _check()
    norm.count = norm.count + rows_total


# ---------------- running obs normalizer (the state of ppo.py:63-81) ----------------
class RunNorm:
    """Running mean / variance of the raw observations and the clipped normalisation
    z = clamp((o - mean) / sqrt(var + 1e-8), +-10) that the rollout kernel applies.

    The state (mean, var, count) and its merge rule are the reference's (a batch of b rows
    with moments (m_b, v_b) merged into (mean, var, count) by the parallel-variance formula).
    Batches are reduced here in fp64 -- the same moments the device batch preparation
    (g1_obs_prep + g1_runnorm_update) accumulates -- so a host update and a device update of
    the same rows agree to fp32 rounding."""

    def __init__(self, dim, dev):
        self.mean = torch.zeros(dim, device=dev)
        self.var = torch.ones(dim, device=dev)
        self.count = 1e-4

    def merge(self, m_b, v_b, b):
        """Merge a batch of b rows with per-dimension mean m_b and (biased) variance v_b."""
        n0, n = float(self.count), float(b)
        tot = n0 + n
        m0, v0 = self.mean.double(), self.var.double()
        d = m_b.double() - m0
        self.mean = (m0 + d * (n / tot)).float()
        self.var = ((v0 * n0 + v_b.double() * n + d * d * (n0 * n / tot)) / tot).float()
        self.count = tot

    def update(self, x):
        """Merge the rows of x [B, dim] (fp64 moments)."""
        xd = x.detach().double()
        m_b = xd.mean(0)
        self.merge(m_b, (xd * xd).mean(0) - m_b * m_b, x.shape[0])

    def norm(self, x):
        return torch.clamp((x - self.mean) / torch.sqrt(self.var + 1e-8), -10.0, 10.0)


# ---------------- actor-critic (ppo.py:85-99) ----------------
class AC(nn.Module):
    """The reference's actor-critic (shared trunk, value head on the last hidden layer).
    value_hidden: a separate value network of those widths instead."""

    def __init__(self, obs_dim, act_dim, hidden=(256, 256), activation="tanh", value_hidden=None):
        super().__init__()
        act = (lambda: nn.Tanh()) if activation == "tanh" else (lambda: nn.ELU())
        layers, d = [], obs_dim
        for h in hidden:
            layers += [nn.Linear(d, h), act()]
            d = h
        self.hidden = tuple(hidden)
        self.activation = activation
        self.value_hidden = tuple(value_hidden) if value_hidden else None
        self.body = nn.Sequential(*layers)
        self.mu = nn.Linear(d, act_dim)
        if self.value_hidden:
            vl, dv = [], obs_dim
            for h in self.value_hidden:
                vl += [nn.Linear(dv, h), act()]
                dv = h
            self.v_body = nn.Sequential(*vl)
            self.v = nn.Linear(dv, 1)
        else:
            self.v = nn.Linear(d, 1)
        self.log_std = nn.Parameter(-0.5 * torch.ones(act_dim))

    def forward(self, x):
        z = self.body(x)
        v = self.v(self.v_body(x)) if self.value_hidden else self.v(z)
        return self.mu(z), self.log_std.exp(), v.squeeze(-1)


def pack_weights(ac):
    """Flatten AC params in the order the kernel unpacks (ppo_fused.py:35-44): per hidden
    layer W,b; then Wmu,bmu, Wv,bv, log_std.  nn.Linear weight is [out,in] row-major.
    With a separate value network (g1_env_set_value_net): per policy hidden layer W,b; Wmu,
    bmu, log_std; per value hidden layer W,b; Wv, bv."""
    lin = lambda seq: [t for m in seq if isinstance(m, nn.Linear) for t in (m.weight.reshape(-1), m.bias)]
    parts = lin(ac.body)
    if getattr(ac, "value_hidden", None):
        parts += [ac.mu.weight.reshape(-1), ac.mu.bias, ac.log_std] + lin(ac.v_body) + [ac.v.weight.reshape(-1), ac.v.bias]
    else:
        parts += [ac.mu.weight.reshape(-1), ac.mu.bias, ac.v.weight.reshape(-1), ac.v.bias, ac.log_std]
    return torch.cat(parts).contiguous()


def init_policy_normal(ac, seed=0):
    """Config-2 style random init: N(0, 1/fan_in) weights, zero bias, log_std = -0.5."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    with torch.no_grad():
        for m in ac.modules():
            if isinstance(m, nn.Linear):
                m.weight.copy_(torch.randn(m.weight.shape, generator=g) / np.sqrt(m.weight.shape[1]))
                m.bias.zero_()
        ac.log_std.fill_(-0.5)
    return ac


@torch.no_grad()
def evaluate(env, ac, norm, dev, steps=200):
    """Deterministic (mean-action) evaluation on the device-resident host-loop step path
    (g1_env_step_device), reporting the metrics of the reference trainer's evaluate
    (ppo.py:103-125): distance walked (base forward velocity, obs[:, 0], integrated over
    the 0.02 s control step) until the first episode end, its mean and max over worlds, the
    mean number of live steps, the fraction of worlds that ended an episode, and the mean
    forward velocity while live.  Everything stays on the GPU; one host sync at the end."""
    N, ctrl_dt = env.N, 0.02
    obs = torch.as_tensor(env.reset(), device=dev)
    rew = torch.zeros(N, device=dev)
    done = torch.zeros(N, device=dev)
    live = torch.ones(N, device=dev)
    dist = torch.zeros(N, device=dev)
    vsum = torch.zeros(N, device=dev)
    nlive = torch.zeros(N, device=dev)
    for _ in range(steps):
        mu = ac(norm.norm(obs))[0].contiguous()
        env.step_device(mu, obs, rew, done)
        vx = obs[:, 0]
        dist += live * vx * ctrl_dt
        vsum += live * vx
        nlive += live
        live = live * (done == 0).float()
    fallen = 1.0 - live
    out = torch.stack([dist.mean(), dist.max(), nlive.mean(), fallen.mean(),
                       (vsum / nlive.clamp_min(1.0)).mean()]).tolist()
    return dict(zip(("fwd_mean", "fwd_max", "ep_len_mean", "fall_rate", "vx_mean"), out))
