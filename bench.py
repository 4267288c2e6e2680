"""Benchmark of the fused G1 rollout (BASELINE.json metric: fused-rollout substeps/s per
box, N=8192 worlds per GPU, H=32 control steps, S=10 substeps).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]
    torchrun --nproc-per-node N bench.py --gpus N ...        (one rank per GPU)

A step is one fused rollout (g1_rollout) of every world on this rank: N*H*S substeps.  The
policy is the config-2 actor-critic (100 -> 256 -> 256 ELU -> 29 means + value, weights
N(0, 1/fan_in), zero bias, log_std -0.5), observation stats mean 0 / var 1; data are
synthetic (there is no dataset in this workload: the env generates its own states).
Worlds are sharded across ranks (weak scaling); the rollout needs no communication, the
timing is the max over ranks of CUDA-event time.

Between timed steps the L2 is flushed (a 256 MiB write, outside the timed events).
`--impl reference` times the reference implementation of the path on the host cores: the
CPU oracle (oracle/g1_oracle.c, bit-identical to the reference's fp32 physics), OpenMP on
all host threads, rank 0 only.
"""
import argparse
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "g1.cu_b200"))

N_PER_GPU, H, S, PGS = 8192, 32, 10, 8
OBS, ACT = 100, 29
# DRAM traffic of one config-2 k_g1 launch (H = 32), dram__bytes_read.sum + dram__bytes_write.sum
# from one ncu capture of the full-size launch (profiles/k_g1_rollout_n8192_h32.md)
TRAFFIC_PER_LAUNCH = 6.55e6 + 91.92e6
TRAFFIC_SOURCE = ("ncu --metrics dram__bytes_read.sum,dram__bytes_write.sum (1 pass) of one full-size H=32 k_g1 "
                  "launch: 6.55 MB read + 91.92 MB written; below the algorithmic bytes because ~48 MB of "
                  "trajectory stores are still dirty in the 126 MB L2 when the kernel ends")
METRIC = "fused-rollout substeps/s per box at 1/2/4/8 B200 (N=8192/GPU, H=32); % roofline"
CONFIG = {"workload": "config2: fused PPO rollout, N=8192 worlds/GPU, H=32, S=10, PGS 8, "
                      "policy 100-256-256(ELU)-29+value fp32 random-init",
          "worlds_per_gpu": N_PER_GPU, "horizon": H, "substeps": S, "pgs_iters": PGS,
          "mlp": [100, 256, 256, 29], "activation": "elu", "l2": "flushed between timed steps (256 MiB write)"}

# algorithmic FLOPs per world-substep by contact count (FK + env_qacc at PGS 8; mul and add
# counted separately, FMA = 2), from the op-count of the reference physics at ncon 0/4/8
# (35/72/122 kFLOP incl. FK); intermediate counts interpolated linearly between those.
FLOP_NCON_ANCHORS = {0: 5673 + 29071, 4: 5673 + 65948, 8: 5673 + 116400}
MLP_FLOP_PER_WORLD_STEP = 2 * (100 * 256 + 256 * 256 + 256 * 30)  # config-2 MLP incl. value head


def flops_per_ncon():
    a = FLOP_NCON_ANCHORS
    out = []
    for n in range(9):
        lo, hi = (0, 4) if n <= 4 else (4, 8)
        out.append(a[lo] + (a[hi] - a[lo]) * (n - lo) / (hi - lo))
    return np.array(out)


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        return json.load(open(p)), "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}, "fallback"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 50 ms during the timed region."""
    Q = ("timestamp,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.idx, self.rows, self.proc = gpu_index, [], None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.idx), f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "50"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append((time.time(), [x.strip() for x in line.split(",")]))

    def stop(self, t0=None, t1=None):
        """Stop sampling; summarise the samples that arrived inside [t0, t1] (host time of the
        timed region; the nearest sample if none did)."""
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        self.proc.wait()
        self.t.join(timeout=2)
        ok = [(t, r) for t, r in self.rows if len(r) > 7 and r[1].replace(".", "").isdigit()]
        sel = [r for t, r in ok if t0 is None or (t0 <= t <= t1 + 0.25)]
        if not sel and ok:
            sel = [min(ok, key=lambda x: abs(x[0] - (t0 or 0)))[1]]
        sm = [float(r[1]) for r in sel]
        mx = [float(r[2]) for r in sel if r[2].replace(".", "").isdigit()]
        pw = [float(r[3]) for r in sel if r[3].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in sel for i in range(4) if r[4 + i] == "Active"})
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "power_w_max": max(pw) if pw else None, "reasons": reasons, "samples": len(sm)}


def dist_setup(args):
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import torch.distributed as dist
        if args.impl == "reference":
            dist.init_process_group("gloo")
        else:
            torch.cuda.set_device(local)
            dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    return world, rank, local


def max_over_ranks(x, world):
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda" if dist.get_backend() == "nccl" else "cpu")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def all_ranks(x, world):
    """x of every rank (rank order)."""
    if world == 1:
        return [x]
    import torch
    import torch.distributed as dist
    dev = "cuda" if dist.get_backend() == "nccl" else "cpu"
    out = [torch.zeros(1, dtype=torch.float64, device=dev) for _ in range(world)]
    dist.all_gather(out, torch.tensor([x], dtype=torch.float64, device=dev))
    return [float(t.item()) for t in out]


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def cpu_baseline(steps_sample=None, worlds_sample=None, target_s=10.0):
    """The CPU oracle rollout on a bounded sample of the config-2 workload (worlds_sample
    worlds x steps_sample control steps; by default sized from a short calibration run to
    about target_s seconds), OpenMP over all host threads."""
    if steps_sample is None or worlds_sample is None:
        cal = cpu_baseline(2, 1024)
        worlds_sample = 2048
        steps_sample = int(np.clip(target_s * cal["value"] / (worlds_sample * S), 1, 512))
    import torch  # noqa: F401  (policy init uses torch)
    import g1env
    from oracle.oracle import Oracle, OracleEnv
    o = Oracle("f32")
    cores = os.cpu_count() or 1
    env = OracleEnv(o, worlds_sample, S, PGS, seed=1)
    env.reset()
    ac = g1env.init_policy_normal(g1env.AC(100, 29, (256, 256), "elu"), seed=0)
    W = g1env.pack_weights(ac).detach().numpy()
    mean, var = np.zeros(100, np.float32), np.ones(100, np.float32)
    env.rollout(1, W, mean, var, act="elu")  # warm (thread pool)
    t0 = time.perf_counter()
    env.rollout(steps_sample, W, mean, var, act="elu")
    dt = time.perf_counter() - t0
    env.close()
    sub = worlds_sample * steps_sample * S
    return {"value": sub / dt, "unit": "substeps/s", "cores": cores, "kind": "port",
            "sample": f"{worlds_sample} worlds x {steps_sample} control steps x {S} substeps "
                      f"({sub} substeps, {dt:.1f} s) of the config-2 rollout, CPU oracle fp32 "
                      f"(bit-identical to the reference's fp32 physics), OpenMP {cores} threads"}


def run_reference(args, world, rank):
    """The reference arm: the CPU implementation of the path (the oracle port, bit-identical
    to the reference's fp32 physics; the reference has no CPU rollout of its own besides
    MuJoCo, which is not installed) on all host threads.  Each timed step is the FULL
    config-2 workload -- one rollout of N_PER_GPU worlds x H control steps x S substeps,
    continuing from the previous step's state, as the GPU arm does -- timed by wall clock
    (one process, no GPU).  Warm-up steps are one control step each (thread-pool start)."""
    if rank != 0:
        return
    import torch  # noqa: F401  (policy init uses torch)
    import g1env
    from oracle.oracle import Oracle, OracleEnv
    cores = os.cpu_count() or 1
    env = OracleEnv(Oracle("f32"), N_PER_GPU, S, PGS, seed=1)
    env.reset()
    ac = g1env.init_policy_normal(g1env.AC(100, 29, (256, 256), "elu"), seed=0)
    W = g1env.pack_weights(ac).detach().numpy()
    mean, var = np.zeros(100, np.float32), np.ones(100, np.float32)
    for _ in range(args.warmup):
        env.rollout(1, W, mean, var, act="elu")
    ts = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        env.rollout(H, W, mean, var, act="elu")
        ts.append(time.perf_counter() - t0)
    env.close()
    ms = 1e3 * float(np.mean(ts))
    v = N_PER_GPU * H * S / (ms * 1e-3)  # the host's rate: its cores are the same at any N
    cb = {"value": v, "unit": "substeps/s", "cores": cores, "kind": "port",
          "sample": f"the full config-2 workload per step: {N_PER_GPU} worlds x {H} control steps x {S} substeps "
                    f"with the ELU policy, CPU oracle fp32 (bit-identical to the reference's fp32 physics), "
                    f"OpenMP {cores} threads; {args.steps} steps, mean {ms:.0f} ms"}
    line = {"impl": "reference", "metric": METRIC, "value": v, "unit": "substeps/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic (env-generated states, random-init policy)",
            "config": dict(CONFIG, parallelism=f"world shards x{world}, no rollout communication"),
            "cpu_baseline": cb,
            "e2e": {"value": v, "unit": "substeps/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    if world > 1:
        line["note"] = "rank 0 alone ran (one host, the same cores at any N): value is the host's rate on one rank's share"
    print(json.dumps(line), flush=True)


def reference_kernel_time(N, mean, var, W, reps=2):
    """The reference's own k_rollout (src/g1_env.cu compiled for sm_100a, oracle/_ref), same
    workload, for the per-GPU speed-up target.  Returns ms per rollout or None."""
    import ctypes
    import torch
    path = os.path.join(ROOT, "oracle", "_ref", "libg1env_ref.so")
    if not os.path.exists(path):
        return None
    R = ctypes.CDLL(path)
    R.g1_env_create.restype = ctypes.c_void_p
    R.g1_env_create.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_ulong]
    R.g1_env_reset.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
    R.g1_rollout.argtypes = [ctypes.c_void_p, ctypes.c_int] + [ctypes.c_void_p] * 10
    R.g1_env_destroy.argtypes = [ctypes.c_void_p]
    h = R.g1_env_create(N, S, PGS, 1)
    ob = np.zeros((N, 100), np.float32)
    R.g1_env_reset(h, ob.ctypes.data_as(ctypes.c_void_p))
    z = lambda *s: torch.zeros(*s, device="cuda")
    bufs = [z(H, N, 100), z(H, N, 29), z(H, N), z(H, N), z(H, N), z(H, N), z(N)]
    vp = lambda t: ctypes.c_void_p(t.data_ptr())
    args = [vp(W), vp(mean), vp(var)] + [vp(b) for b in bufs]
    R.g1_rollout(h, H, *args)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        R.g1_rollout(h, H, *args)
    e1.record()
    torch.cuda.synchronize()
    R.g1_env_destroy(h)
    return e0.elapsed_time(e1) / reps


def profile_case(h):
    """Two g1_rollout calls of the config-2 workload with horizon h (the second is the one to
    capture with ncu -s 1 -c 1)."""
    import torch
    import g1env
    env = g1env.G1Env(N_PER_GPU, S, PGS, seed=1)
    env.set_policy((256, 256), "elu")
    env.reset()
    ac = g1env.init_policy_normal(g1env.AC(100, 29, (256, 256), "elu"), seed=0).cuda()
    W = g1env.pack_weights(ac).detach()
    mean, var = torch.zeros(100, device="cuda"), torch.ones(100, device="cuda")
    z = lambda *s: torch.zeros(*s, device="cuda")
    bufs = [z(h, N_PER_GPU, 100), z(h, N_PER_GPU, 29)] + [z(h, N_PER_GPU) for _ in range(4)] + [z(N_PER_GPU)]
    for _ in range(2):
        env.rollout(h, W, mean, var, *bufs)
    torch.cuda.synchronize()
    env.close()
    print("profile case done")


def profile_case3(h):
    """Two g1_rollout calls of the config-3 workload (N = 32768, 100-1024-1024-512-29 ELU,
    bf16 on the tensor cores) with horizon h: the small case for ncu captures of k_gemm."""
    import torch
    import g1env
    N3 = 32768
    env = g1env.G1Env(N3, S, PGS, seed=3)
    env.set_policy((1024, 1024, 512), "elu", precision="bf16")
    env.reset()
    ac = g1env.init_policy_normal(g1env.AC(100, 29, (1024, 1024, 512), "elu"), seed=0).cuda()
    W = g1env.pack_weights(ac).detach().contiguous()
    mean, var = torch.zeros(100, device="cuda"), torch.ones(100, device="cuda")
    z = lambda *sh: torch.zeros(*sh, device="cuda")
    bufs = [z(h, N3, 100), z(h, N3, 29), z(h, N3), z(h, N3), z(h, N3), z(h, N3), z(N3)]
    for _ in range(2):
        env.rollout(h, W, mean, var, *bufs)
    torch.cuda.synchronize()
    if env.tc_status():
        raise RuntimeError("tensor-core wait timed out in the config-3 rollout")
    env.close()
    print("profile case 3 done")


PHASES = ["policy", "F1", "B1", "base", "F2", "contact_setup", "back_solves", "gram", "pgs", "dq", "pd_torque",
          "end_of_step_wait", "integrate", "detect", "mlp_layer0", "sampling", "mlp_layer1", "mlp_head",
          "substep_barrier_wait", "energy", "mlp_mma_wait", "mlp_epilogue", "step_state_load", "reward_done",
          "state_store_reset", "contact_sort", "kernel_total", "solve_leaf_to_root", "solve_base",
          "solve_root_to_leaf", "mlp_epilogue_stage", "mlp_epilogue_act", "F1_pass2", "base_pull_U6",
          "base_Dm_q6", "midbar_wait"]
# sub-phases: counted inside another phase, left out of the unattributed remainder
SUBPHASES = {"mlp_layer0", "mlp_layer1", "mlp_head", "sampling", "mlp_mma_wait", "mlp_epilogue",
             "mlp_epilogue_stage", "mlp_epilogue_act", "solve_leaf_to_root", "solve_base", "solve_root_to_leaf"}


def phase_profile(h):
    """Per-phase cycle attribution of k_g1 (attribution only, not a benchmark): builds the
    -DG1_PROF variant of the library (clock64 counters around each phase, summed per warp)
    into _build/libg1env_prof.so, runs one warm-up and one measured config-2 rollout of
    horizon h, and prints the mean cycles per warp per control step of each phase."""
    import ctypes
    import torch
    import g1env
    from build import ARCH, CSRC, FLAGS
    out_dir = os.path.join(ROOT, "_build")
    os.makedirs(out_dir, exist_ok=True)
    lib_path = os.path.join(out_dir, "libg1env_prof.so")
    r = subprocess.run(["nvcc"] + ARCH + FLAGS + ["-DG1_PROF", os.path.join(CSRC, "g1_env.cu"), "-o", lib_path],
                       capture_output=True, text=True)
    if r.returncode:
        raise RuntimeError(r.stderr)
    g1env.load_library(lib_path)
    lib = g1env._lib
    lib.g1_prof_read.argtypes = [ctypes.c_void_p]
    N = N_PER_GPU
    env = g1env.G1Env(N, S, PGS, seed=1)
    env.set_policy((256, 256), "elu")
    env.reset()
    ac = g1env.init_policy_normal(g1env.AC(100, 29, (256, 256), "elu").cuda(), seed=0)
    W = g1env.pack_weights(ac).detach()
    mean, var = torch.zeros(100, device="cuda"), torch.ones(100, device="cuda")
    z = lambda *sh: torch.zeros(*sh, device="cuda")
    bufs = [z(h, N, 100), z(h, N, 29), z(h, N), z(h, N), z(h, N), z(h, N), z(N)]
    env.rollout(h, W, mean, var, *bufs)
    cnt = (ctypes.c_ulonglong * 64)()
    lib.g1_prof_read(cnt)  # clears the counters
    env.rollout(h, W, mean, var, *bufs)
    lib.g1_prof_read(cnt)
    sm = torch.cuda.get_device_properties(0).multi_processor_count
    wb = (N + sm - 1) // sm
    nwarps = ((N + wb - 1) // wb) * 7
    per = {n: round(cnt[i] / nwarps / h) for i, n in enumerate(PHASES)}
    per["unattributed"] = per["kernel_total"] - sum(v for k, v in per.items() if k != "kernel_total" and k not in SUBPHASES)
    batches = [round(cnt[47 + c] / h / (nwarps // 7), 2) for c in range(1, 9)]
    print(json.dumps({"N": N, "H": h, "cycles_per_warp_per_control_step": per,
                      "contact_batches_per_cta_per_control_step_by_size_1_to_8": batches}))
    env.close()


def other_configs(dev):
    """Informational timings of BASELINE configs 1 and 3 on this GPU (CUDA events, L2 flushed
    between timed calls); the headline metric is config 2."""
    import torch
    import g1env
    out = {}
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)

    def timed(fn, reps):
        ts = []
        for _ in range(reps):
            flush.fill_(1.0)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            ts.append((e0, e1))
        torch.cuda.synchronize()
        return sum(a.elapsed_time(b) for a, b in ts) / reps

    # config 1: physics only, N = 8192, mu = 1.0, 32 control steps x 10 substeps, a constant
    # action U(-1,1) per world through the PD-target path; state = the reset pose with base
    # height U(0.75, 0.8) m and qvel ~ N(0, 0.5)
    rng = np.random.default_rng(11)
    N1, K1 = 8192, 32
    env = g1env.G1Env(N1, S, PGS, seed=11, device=dev.index, mu=1.0)
    env.reset()
    st = env.get_state()
    qp, qv = st[0].copy(), rng.normal(0, 0.5, (N1, 35)).astype(np.float32)
    qp[:, 2] = rng.uniform(0.75, 0.8, N1)
    act = torch.tensor(rng.uniform(-1, 1, (N1, 29)).astype(np.float32), device=dev)

    def c1():
        env.set_state(qp, qv, st[2], st[3], st[4])
        env.phys_actions(K1, act)
    c1()
    torch.cuda.synchronize()
    ms1 = timed(c1, 3)
    env.close()
    out["config1"] = {"value": N1 * K1 * S / (ms1 * 1e-3), "unit": "substeps/s", "ms": ms1,
                      "what": "physics only, N=8192, mu=1.0, 32 control steps x 10 substeps, constant U(-1,1) "
                              "action per world (state upload included in the timed call)"}
    # config 3: N = 32768, H = 32, policy 100-1024-1024-512-29 ELU on the tensor cores (bf16)
    N3, H3 = 32768, 32
    env = g1env.G1Env(N3, S, PGS, seed=3, device=dev.index)
    env.set_policy((1024, 1024, 512), "elu", precision="bf16")
    env.reset()
    ac = g1env.init_policy_normal(g1env.AC(100, 29, (1024, 1024, 512), "elu"), seed=0).to(dev)
    W = g1env.pack_weights(ac).detach().contiguous()
    mean, var = torch.zeros(100, device=dev), torch.ones(100, device=dev)
    z = lambda *sh: torch.zeros(*sh, device=dev)
    bufs = [z(H3, N3, 100), z(H3, N3, 29), z(H3, N3), z(H3, N3), z(H3, N3), z(H3, N3), z(N3)]
    env.rollout(H3, W, mean, var, *bufs)
    torch.cuda.synchronize()
    ms3 = timed(lambda: env.rollout(H3, W, mean, var, *bufs), 2)
    if env.tc_status():
        raise RuntimeError("tensor-core wait timed out in the config-3 rollout")
    env.close()
    out["config3"] = {"value": N3 * H3 * S / (ms3 * 1e-3), "unit": "substeps/s", "ms": ms3,
                      "what": "fused rollout N=32768, H=32, S=10, policy 100-1024-1024-512-29 ELU, bf16 on tcgen05"}
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-ref-kernel", action="store_true")
    ap.add_argument("--no-other-configs", action="store_true")
    ap.add_argument("--profile-case", type=int, default=0, metavar="H",
                    help="run two H-step rollouts of the config-2 worlds and exit (small case for ncu captures)")
    ap.add_argument("--profile-case3", type=int, default=0, metavar="H",
                    help="run two H-step rollouts of the config-3 workload and exit (small case for ncu captures)")
    ap.add_argument("--phase-profile", type=int, default=0, metavar="H",
                    help="per-phase cycle attribution of k_g1 from a -DG1_PROF build (horizon H) and exit")
    args = ap.parse_args()
    if args.phase_profile:
        phase_profile(args.phase_profile)
        return
    if args.profile_case3:
        profile_case3(args.profile_case3)
        return
    if args.profile_case:
        profile_case(args.profile_case)
        return
    args.warmup = max(args.warmup, 3)
    world, rank, local = dist_setup(args)
    if args.impl == "reference":
        run_reference(args, world, rank)
        return
    import torch
    import g1env
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    N = N_PER_GPU
    env = g1env.G1Env(N, S, PGS, seed=1, device=local, world0=rank * N)
    env.set_policy((256, 256), "elu")
    env.reset()
    stream = torch.cuda.current_stream(dev)
    env.set_stream(stream)
    ac = g1env.init_policy_normal(g1env.AC(100, 29, (256, 256), "elu"), seed=0).to(dev)
    W = g1env.pack_weights(ac).detach().contiguous()
    mean = torch.zeros(100, device=dev)
    var = torch.ones(100, device=dev)
    z = lambda *s: torch.zeros(*s, device=dev)
    bufs = [z(H, N, 100), z(H, N, 29), z(H, N), z(H, N), z(H, N), z(H, N), z(N)]
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)

    for _ in range(args.warmup):
        env.rollout(H, W, mean, var, *bufs)
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    clocks.start()
    # two rollouts keep the GPU busy while the sampler spins up; they also record the
    # contact-count histogram that the FLOP count uses (the timed rollouts run without it)
    env.ncon_hist(True)
    for _ in range(2):
        env.rollout(H, W, mean, var, *bufs)
    hist = env.ncon_hist(False).astype(np.float64)
    barrier(world)
    torch.cuda.synchronize()
    t_start = time.time()
    times = []
    for _ in range(args.steps):
        flush.fill_(1.0)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        env.rollout(H, W, mean, var, *bufs)
        e1.record(stream)
        times.append((e0, e1))
    torch.cuda.synchronize()
    t_end = time.time()
    barrier(world)
    ck = clocks.stop(t_start, t_end)
    ms_local = sum(a.elapsed_time(b) for a, b in times) / args.steps
    ms = max_over_ranks(ms_local, world)
    per_rank_ms = all_ranks(ms_local, world)
    substeps = N * H * S
    value = world * substeps / (ms * 1e-3)

    # --- e2e through the public API with host buffers: pinned W/mean/var in, rewards/dones/
    # bootstrap values out, every step
    hW = W.cpu().pin_memory(); hm = mean.cpu().pin_memory(); hv = var.cpu().pin_memory()
    dW, dm, dv = torch.empty_like(W), torch.empty_like(mean), torch.empty_like(var)
    hR = torch.empty(H, N).pin_memory(); hD = torch.empty(H, N).pin_memory(); hVl = torch.empty(N).pin_memory()
    barrier(world)
    torch.cuda.synchronize()
    e_times = []
    for _ in range(args.steps):
        flush.fill_(1.0)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        dW.copy_(hW, non_blocking=True); dm.copy_(hm, non_blocking=True); dv.copy_(hv, non_blocking=True)
        env.rollout(H, dW, dm, dv, *bufs)
        hR.copy_(bufs[4], non_blocking=True); hD.copy_(bufs[5], non_blocking=True); hVl.copy_(bufs[6], non_blocking=True)
        e1.record(stream)
        e_times.append((e0, e1))
    torch.cuda.synchronize()
    ems = max_over_ranks(sum(a.elapsed_time(b) for a, b in e_times) / args.steps, world)
    h2d = (W.numel() + 200) * 4
    d2h = (2 * H * N + N) * 4

    # --- roofline of the dominant kernel (k_g1): algorithmic FP32 FLOPs / kernel time
    flop_sub = float((hist * flops_per_ncon()).sum() / max(hist.sum(), 1))
    phys_flops = substeps * flop_sub
    mlp_flops = N * (H + 1) * MLP_FLOP_PER_WORLD_STEP
    flops_launch = phys_flops + mlp_flops
    peaks, peak_src = load_peaks()
    sm_count = torch.cuda.get_device_properties(dev).multi_processor_count
    clk = ck.get("sm_max_mhz") or peaks.get("sm_max_mhz", 1965.0)
    fp32_peak = sm_count * 128 * 2 * clk * 1e6 / 1e12  # nominal FP32 FMA peak at max SM clock
    achieved = flops_launch / (ms * 1e-3) / 1e12
    phys_achieved = phys_flops / (ms * 1e-3) / 1e12
    mlp_achieved = mlp_flops / (ms * 1e-3) / 1e12
    bf16_peak = float(peaks.get("bf16_tflops_sustained", peaks.get("bf16_tflops", 1590.0)))
    # algorithmic HBM bytes of one launch: trajectory O/A/LP/V/R/D written once (133 floats per
    # world-step), Vlast, the state read and written once, the packed weights and obs stats read
    algo_bytes = 4 * (N * H * (OBS + ACT + 4) + N + 2 * N * (36 + 35 + 29 + 1) + W.numel() + 200)
    ref_ms = None
    if rank == 0 and not args.no_ref_kernel:
        try:
            ref_ms = reference_kernel_time(N, mean, var, W)
        except Exception:  # the reference kernel is a comparison only
            ref_ms = None
    cpu = cpu_baseline() if (rank == 0 and world == 1) else None
    others = None
    if rank == 0 and world == 1 and not args.no_other_configs:
        try:
            others = other_configs(dev)
        except Exception as e:  # informational only
            others = {"error": str(e)[:200]}
    env.close()
    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": "substeps/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "f32", "data": "synthetic (env-generated states, random-init policy)",
                "config": dict(CONFIG, parallelism=f"world shards x{world}, no rollout communication"),
                "e2e": {"value": world * substeps / (ems * 1e-3), "unit": "substeps/s", "h2d_bytes_per_step": h2d,
                        "d2h_bytes_per_step": d2h,
                        "note": "policy weights and obs stats copied in, rewards / dones / bootstrap values copied "
                                "out every step; the trajectory stays on the device, where the trainer reads it "
                                "in place (ppo_fused.py)"},
                "gpu_launches": 2 * args.steps,
                "roofline": {"bound": "fp32", "achieved": phys_achieved, "peak": fp32_peak, "unit": "TFLOP/s",
                             "frac": phys_achieved / fp32_peak,
                             "what": "k_g1 physics: algorithmic FP32 FLOPs of the substeps (FK + env_qacc by contact "
                                     "count) / k_g1 launch time (CUDA events) vs the nominal FP32 rate",
                             "traffic": TRAFFIC_PER_LAUNCH, "algorithmic_bytes": algo_bytes,
                             "traffic_source": TRAFFIC_SOURCE,
                             "peak_source": f"nominal FP32 FMA rate: {sm_count} SMs x 128 lanes x 2 x {clk:.0f} MHz "
                                            f"(MEASURED_PEAKS.json has no FP32 figure)",
                             "flop_per_substep": flop_sub, "ncon_hist": hist.tolist(),
                             "ncon_hist_source": "the 2 untimed rollouts just before the timed ones",
                             "policy_mlp": {"bound": "tensor", "achieved": mlp_achieved, "peak": bf16_peak,
                                            "unit": "TFLOP/s", "frac": mlp_achieved / bf16_peak,
                                            "what": "config-2 MLP FLOPs (fp32 semantics, run as split-bf16 tcgen05 "
                                                    "MMAs inside k_g1) over the whole k_g1 launch time, vs "
                                                    f"MEASURED_PEAKS.json bf16_tflops_sustained ({peak_src})"},
                             "all_flops": {"achieved": achieved, "frac_of_fp32": achieved / fp32_peak}},
                "clocks": ck,
                "per_rank_ms": per_rank_ms,
                "reference_kernel": None if ref_ms is None else {
                    "ms_per_step": ref_ms, "value": substeps / (ref_ms * 1e-3), "unit": "substeps/s",
                    "what": "reference k_rollout (src/g1_env.cu) built for sm_100a, same N/H/S, 1 GPU"}}
        if cpu is not None:
            line["cpu_baseline"] = cpu
        if others is not None:
            line["other_configs"] = others
        print(json.dumps(line), flush=True)
    barrier(world)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
