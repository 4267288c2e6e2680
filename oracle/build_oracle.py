"""Build the CPU oracle (and, where the reference tree is present, the reference builds
used only as checkers and as the timed reference arm).  TEST INFRASTRUCTURE.

Outputs (all git-ignored, all travel with the repository snapshot to a GPU box):
  oracle/liboracle_f32.so, oracle/liboracle_f64.so   -- this repository's C restatement
  oracle/_ref/libg1ref_host_f32.so / _f64.so / _f32_mu1.so
                                                     -- reference physics headers, host C++
  oracle/_ref/libg1ref_cuda.so, _mu1.so              -- reference physics, CUDA sm_100a harness
                                                        (model friction 0.6, and 1.0)
  oracle/_ref/libg1env_ref.so                        -- the reference's g1_env.cu as shipped,
                                                        compiled for sm_100a (its own C-ABI)
  oracle/_ref/trainer/scripts/ppo.py, ppo_fused.py   -- the reference's trainer, staged
                                                        unchanged for the drop-in test

The reference pieces are compiled from the sources where they lie (-I<ref>/src); nothing is
copied into this repository.
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REF_DEFAULT = os.environ.get("G1_REFERENCE_ROOT", "/root/reference")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _run(cmd):
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("build failed: " + " ".join(cmd) + "\n" + r.stdout + r.stderr)


def _stale(out, srcs):
    if not os.path.exists(out):
        return True
    t = os.path.getmtime(out)
    return any(os.path.getmtime(s) > t for s in srcs if os.path.exists(s))


def build_oracle(force=False):
    src = os.path.join(HERE, "g1_oracle.c")
    hdr = os.path.join(HERE, "..", "g1.cu_b200", "csrc", "g1_model_data.h")
    outs = {}
    for tag, real in (("f32", "float"), ("f64", "double")):
        out = os.path.join(HERE, f"liboracle_{tag}.so")
        if force or _stale(out, [src, hdr, __file__]):
            _run(["gcc", "-O2", "-fopenmp", "-shared", "-fPIC", "-ffp-contract=off", f"-DREAL={real}", src, "-o", out, "-lm"])
        outs[tag] = out
    return outs


def build_ref(ref_root=None, force=False, cuda=True):
    ref_root = ref_root or REF_DEFAULT
    src_dir = os.path.join(ref_root, "src")
    if not os.path.isdir(src_dir):
        return None
    out_dir = os.path.join(HERE, "_ref")
    os.makedirs(out_dir, exist_ok=True)
    shim = os.path.join(HERE, "ref_host_shim.cpp")
    ref_srcs = [os.path.join(src_dir, f) for f in os.listdir(src_dir)]
    for tag, flags in (("f32", []), ("f64", ["-DREF_F64"]), ("f32_mu1", ["-DREF_MU=1.0f"])):
        out = os.path.join(out_dir, f"libg1ref_host_{tag}.so")
        if force or _stale(out, [shim] + ref_srcs):
            _run(["g++", "-O2", "-shared", "-fPIC", "-ffp-contract=off", "-w", "-I", src_dir] + flags + [shim, "-o", out])
    if cuda:
        harness = os.path.join(HERE, "ref_cuda_harness.cu")
        for tag, flags in (("", []), ("_mu1", ["-DREF_MU=1.0f"])):
            out = os.path.join(out_dir, f"libg1ref_cuda{tag}.so")
            if force or _stale(out, [harness] + ref_srcs):
                _run(["nvcc"] + ARCH + ["-O3", "-Xcompiler", "-fPIC", "--shared", "-w", "-I", src_dir] + flags +
                     [harness, "-o", out])
        out = os.path.join(out_dir, "libg1env_ref.so")
        env_src = os.path.join(src_dir, "g1_env.cu")
        if force or _stale(out, [env_src] + ref_srcs):
            _run(["nvcc"] + ARCH + ["-O3", "-Xcompiler", "-fPIC", "--shared", "-w", env_src, "-lcurand", "-o", out])
    stage_ref_trainer(ref_root, out_dir)
    return out_dir


def stage_ref_trainer(ref_root, out_dir):
    """Stage the reference's own trainer scripts, byte for byte, into oracle/_ref/trainer/
    (git-ignored, like the reference builds; it travels with the snapshot to a GPU box,
    which has no reference tree).  The drop-in test runs them unmodified against this
    repository's libg1env.so."""
    import shutil
    dst = os.path.join(out_dir, "trainer", "scripts")
    os.makedirs(dst, exist_ok=True)
    for f in ("ppo.py", "ppo_fused.py"):
        src = os.path.join(ref_root, "scripts", f)
        if os.path.exists(src) and _stale(os.path.join(dst, f), [src]):
            shutil.copyfile(src, os.path.join(dst, f))


if __name__ == "__main__":
    print(build_oracle(force="--force" in sys.argv))
    print(build_ref(force="--force" in sys.argv, cuda="--no-cuda" not in sys.argv))
