"""Generate the committed golden fixtures under tests/golden/ (run where the reference tree
is present; the fixtures are committed, nothing at test time reads the reference).

Sources:
  * the reference's own MuJoCo 3.9.0 goldens (Infatoshi/g1.cu bench/):
      ref_traj.npz          smooth fp64 trajectory, base lifted 5 m (scripts/gen_reference.py)
      contact_solve_ref.npz foot-ground contact states (scripts/gen_contact_solve_ref.py);
                            only the pure foot-ground ones (scripts/gen_contact_validate.py:25-30)
      implicit_ref.npz      implicit-PD trajectory, contacts off (scripts/gen_implicit_ref.py)
  * the reference's physics headers compiled for the host (oracle/_ref, built by
    oracle/build_oracle.py): FK + env_qacc outputs on seeded states in fp32 (the
    reference's arithmetic) and fp64, at mu = 0.6 and mu = 1.0.
  * the reference's trained finish-line walker (models/ppo_ckpt/finish_best.pt, a torch
    checkpoint {model: AC state_dict, obs_mean, obs_var}) as plain arrays in
    finish_policy.npz, with the playback result the reference documents for it
    (DEVLOG.md:421-422, scripts/play_finish.py: 256 worlds, deterministic actions, <= 480
    control steps -> 256/256 reach x = 5 m).

    python tests/golden/make_golden.py [reference-root] [--policy-only]
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

FOOT_GEOMS = {15, 16, 17, 18, 30, 31, 32, 33}


def export_finish_policy(ref_root):
    import torch
    ck = torch.load(os.path.join(ref_root, "models", "ppo_ckpt", "finish_best.pt"), map_location="cpu")
    arrays = {"param." + k: v.numpy().astype(np.float32) for k, v in ck["model"].items()}
    np.savez_compressed(os.path.join(HERE, "finish_policy.npz"), obs_mean=ck["obs_mean"].numpy().astype(np.float32),
                        obs_var=ck["obs_var"].numpy().astype(np.float32), playback_worlds=np.int32(256),
                        playback_max_steps=np.int32(480), playback_reached=np.int32(256), x_fin=np.float32(5.0),
                        **arrays)


def main(ref_root):
    from oracle.build_oracle import build_ref
    from oracle.oracle import RefHost, envqacc_states, default_bdt, config0_states
    build_ref(ref_root, cuda=False)
    bench = os.path.join(ref_root, "bench")

    # --- smooth MuJoCo trajectory (every 10th step kept for qpos/qvel, qacc/bias at 0..300 step 25)
    z = np.load(os.path.join(bench, "ref_traj.npz"))
    keep = np.arange(0, 301, 10)
    kq = np.arange(0, 301, 25)
    np.savez_compressed(os.path.join(HERE, "mujoco_smooth.npz"), qpos=z["qpos"][keep], qvel=z["qvel"][keep],
                        steps=keep, qacc=z["qacc"][kq], qfrc_bias=z["qfrc_bias"][kq], qsteps=kq,
                        qpos_at_q=z["qpos"][kq], qvel_at_q=z["qvel"][kq], xpos0=z["xpos"][0], xquat0=z["xquat"][0])

    # --- pure foot-ground contact states
    c = np.load(os.path.join(bench, "contact_solve_ref.npz"), allow_pickle=True)
    sel = []
    for k in range(len(c["label"])):
        g1, g2 = c["cgeom1"][k], c["cgeom2"][k]
        if len(g1) == 0 or all((a == 0 and b in FOOT_GEOMS) or (b == 0 and a in FOOT_GEOMS)
                               for a, b in zip(np.asarray(g1).tolist(), np.asarray(g2).tolist())):
            sel.append(k)
    np.savez_compressed(os.path.join(HERE, "mujoco_contact.npz"),
                        label=np.array([str(c["label"][k]) for k in sel]),
                        qpos=np.array([np.asarray(c["qpos"][k], np.float64) for k in sel]),
                        qvel=np.array([np.asarray(c["qvel"][k], np.float64) for k in sel]),
                        qacc=np.array([np.asarray(c["qacc"][k], np.float64) for k in sel]),
                        qacc_smooth=np.array([np.asarray(c["qacc_smooth"][k], np.float64) for k in sel]),
                        ncon=np.array([int(c["ncon"][k]) for k in sel]))

    # --- implicit PD trajectory (contacts off in MuJoCo; base 2 m up so none occur)
    z = np.load(os.path.join(bench, "implicit_ref.npz"))
    np.savez_compressed(os.path.join(HERE, "mujoco_implicit.npz"), qpos=z["qpos"], qvel=z["qvel"],
                        targets=z["targets"], Bdiag=z["Bdiag"], dt=z["dt"])

    # --- reference host arithmetic on seeded env_qacc states (test_envqacc.cu distribution)
    qp, qv = envqacc_states(512, seed=999)
    bdt = default_bdt()
    rng = np.random.default_rng(5)
    tau = np.zeros((512, 35), np.float32)
    tau[256:, 6:] = rng.uniform(-40, 40, (256, 29)).astype(np.float32)  # half with joint torques
    r32, r64, r32m1 = RefHost("f32"), RefHost("f64"), RefHost("f32_mu1")
    np.savez_compressed(os.path.join(HERE, "ref_envqacc.npz"), qpos=qp, qvel=qv, tau=tau, bdt=bdt,
                        qacc_f32=r32.qacc(qp, qv, tau, bdt, 8), qacc_f64=r64.qacc(qp, qv, tau, bdt, 8),
                        qacc_f32_mu1=r32m1.qacc(qp, qv, tau, bdt, 8),
                        qacc_f32_pgs200=r32.qacc(qp, qv, tau, bdt, 200),
                        bias_f32=r32.bias(qp, qv), bias_f64=r64.bias(qp, qv))
    # config-1 states (stand + N(0,0.05), base z U(0.75,0.8), qvel N(0,0.5))
    qp1, qv1 = config0_states(256, seed=11)
    np.savez_compressed(os.path.join(HERE, "ref_config1.npz"), qpos=qp1.astype(np.float32), qvel=qv1.astype(np.float32),
                        qacc_f32=r32.qacc(qp1.astype(np.float32), qv1.astype(np.float32), None, bdt, 8),
                        qacc_f64=r64.qacc(qp1, qv1, None, bdt, 8))
    export_finish_policy(ref_root)
    for f in sorted(os.listdir(HERE)):
        if f.endswith(".npz"):
            print(f, os.path.getsize(os.path.join(HERE, f)))


if __name__ == "__main__":
    args = [a for a in sys.argv[1:] if not a.startswith("--")]
    root = args[0] if args else os.environ.get("G1_REFERENCE_ROOT", "/root/reference")
    if "--policy-only" in sys.argv:
        export_finish_policy(root)
    else:
        main(root)
