"""Per-phase cycle profile of the fused rollout kernel (k_g1).

    python g1.cu_b200/phase_profile.py [N] [H]

Builds a profiling variant of the library (-DG1_PROF: clock64 counters around each phase of
the policy and physics code, summed per phase by lane 0 of every warp) as
g1.cu_b200/libg1env_prof.so, runs one H-step config-2 rollout of N worlds (ELU 256-256
policy) after a warm-up, and prints the mean cycles per warp per control step of each phase.
The substep-barrier wait is measured by a shared-memory load right after the barrier (the
barrier blocks lazily).  Timings of this build are for attribution only, not benchmarks.
"""
import ctypes
import json
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
LIB = os.path.join(HERE, "libg1env_prof.so")
NAMES = ["policy", "F1", "B1", "base", "F2", "contact_setup", "back_solves", "gram", "pgs", "dq", "pd_torque",
         "end_of_step_wait", "integrate", "detect", "mlp_layer0", "sampling", "mlp_layer1", "mlp_head",
         "substep_barrier_wait", "energy", "mlp_mma_wait", "mlp_epilogue", "step_state_load", "reward_done",
         "state_store_reset", "contact_sort", "kernel_total", "solve_leaf_to_root", "solve_base", "solve_root_to_leaf", "mlp_epilogue_stage",
         "mlp_epilogue_act"]


def build():
    from build import ARCH, FLAGS, CSRC
    cmd = ["nvcc"] + ARCH + FLAGS + ["-DG1_PROF", os.path.join(CSRC, "g1_env.cu"), "-o", LIB]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode:
        raise RuntimeError(r.stderr)


def main():
    N = int(sys.argv[1]) if len(sys.argv) > 1 else 8192
    H = int(sys.argv[2]) if len(sys.argv) > 2 else 8
    build()
    import torch
    import g1env
    g1env.load_library(LIB)
    lib = g1env._lib
    lib.g1_prof_read.argtypes = [ctypes.c_void_p]
    env = g1env.G1Env(N, 10, 8, seed=1)
    env.set_policy((256, 256), "elu")
    env.reset()
    ac = g1env.init_policy_normal(g1env.AC(100, 29, (256, 256), "elu").cuda(), seed=0)
    W = g1env.pack_weights(ac).detach()
    mean, var = torch.zeros(100, device="cuda"), torch.ones(100, device="cuda")
    z = lambda *s: torch.zeros(*s, device="cuda")
    bufs = [z(H, N, 100), z(H, N, 29), z(H, N), z(H, N), z(H, N), z(H, N), z(N)]
    env.rollout(H, W, mean, var, *bufs)
    out = (ctypes.c_ulonglong * 64)()
    lib.g1_prof_read(out)  # clear
    env.rollout(H, W, mean, var, *bufs)
    lib.g1_prof_read(out)
    nwarps = torch.cuda.get_device_properties(0).multi_processor_count * 7
    nw_live = ((N + 55) // 56) * 7  # warps of the launched CTAs (56-world blocks)
    per = {n: round(out[i] / nw_live / H) for i, n in enumerate(NAMES)}
    per["unattributed"] = per["kernel_total"] - sum(v for k, v in per.items()
                                                    if k not in ("kernel_total", "mlp_layer0", "mlp_layer1", "mlp_head",
                                                                 "sampling", "mlp_mma_wait", "mlp_epilogue",
                                                                 "mlp_epilogue_stage", "mlp_epilogue_act", "solve_leaf_to_root", "solve_base", "solve_root_to_leaf"))
    batches = [round(out[47 + c] / H / (nw_live // 7), 2) for c in range(1, 9)]
    print(json.dumps({"N": N, "H": H, "cycles_per_warp_per_control_step": per,
                      "contact_batches_per_cta_per_control_step_by_size_1_to_8": batches}))
    env.close()


if __name__ == "__main__":
    main()
