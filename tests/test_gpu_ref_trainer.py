"""Drop-in proof: the reference's own trainers, unmodified, run against this repository's
libg1env.so.

oracle/build_oracle.py stages the reference's scripts/ppo.py (host-loop env, ctypes binding
of g1_env_create / reset / step / destroy, ppo.py:19-58) and scripts/ppo_fused.py (the fused
g1_rollout, ppo_fused.py:24-28, 101-102) byte for byte into oracle/_ref/trainer/scripts.  The
test lays them out as the reference tree expects (scripts/ beside build/libg1env.so), with
build/libg1env.so a symlink to this repository's library, and runs each trainer's --smoke
mode in a fresh process.  Done = exit 0, the trainer's "SMOKE OK" line, and finite losses in
every iteration line."""
import os
import re
import shutil
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
STAGED = os.path.join(ROOT, "oracle", "_ref", "trainer", "scripts")
LIB = os.path.join(ROOT, "g1.cu_b200", "libg1env.so")


@pytest.mark.parametrize("script", ["ppo_fused.py", "ppo.py"])
def test_reference_trainer_smoke_on_this_library(tmp_path, script):
    if not os.path.exists(os.path.join(STAGED, script)):
        pytest.fail("the reference trainer is not staged: run oracle/build_oracle.py where the reference tree is present")
    assert os.path.exists(LIB), "libg1env.so is not built"
    shutil.copytree(STAGED, tmp_path / "scripts")
    (tmp_path / "build").mkdir()
    os.symlink(LIB, tmp_path / "build" / "libg1env.so")
    r = subprocess.run([sys.executable, os.path.join("scripts", script), "--smoke"], cwd=tmp_path,
                       capture_output=True, text=True, timeout=600)
    out = r.stdout + r.stderr
    print(out[-3000:])
    assert r.returncode == 0, out[-3000:]
    assert "SMOKE OK" in out
    losses = [float(x) for x in re.findall(r"loss=\s*(\S+)", r.stdout)]
    assert losses and all(abs(x) < 1e6 for x in losses), losses
    # the library the trainer loaded is this repository's (it exports the extensions)
    assert "g1_env_create_ex" in subprocess.run(["nm", "-D", os.path.join(tmp_path, "build", "libg1env.so")],
                                                capture_output=True, text=True).stdout
