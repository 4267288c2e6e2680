"""The C-ABI library loads on a CPU-only machine and exports every symbol include/g1env.h
declares (no compute calls here)."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB = os.path.join(ROOT, "g1.cu_b200", "libg1env.so")


def declared_symbols():
    txt = open(os.path.join(ROOT, "include", "g1env.h")).read()
    txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
    return sorted(set(re.findall(r"\b(g1_\w+)\s*\(", txt)))


@pytest.fixture(scope="module")
def lib():
    if not os.path.exists(LIB):
        from build import build  # g1.cu_b200/build.py (nvcc cross-compiles without a GPU)
        build()
    return ctypes.CDLL(LIB)


def test_exports_every_declared_symbol(lib):
    syms = declared_symbols()
    assert "g1_rollout" in syms and "g1_env_create" in syms and len(syms) >= 20
    for s in syms:
        assert hasattr(lib, s), s


def test_reference_ctypes_surface(lib):
    """The names and dims the reference's scripts bind (scripts/ppo.py:24-33, ppo_fused.py:27-28)."""
    for s in ("g1_env_create", "g1_env_reset", "g1_env_step", "g1_env_destroy", "g1_rollout", "g1_env_bench_phys",
              "g1_env_qpos", "g1_env_qpos_all", "g1_env_obs_dim", "g1_env_act_dim", "g1_occupancy_report"):
        assert hasattr(lib, s)
    lib.g1_env_obs_dim.restype = ctypes.c_int
    lib.g1_env_act_dim.restype = ctypes.c_int
    assert lib.g1_env_obs_dim() == 100 and lib.g1_env_act_dim() == 29


def test_binding_signatures_cover_header():
    import g1env
    assert set(g1env.SIGNATURES) == set(declared_symbols())


def test_no_gpu_fails_loudly():
    """The product path has no CPU fallback: without a GPU it raises."""
    import torch
    import g1env
    if torch.cuda.is_available():
        pytest.skip("GPU present")
    with pytest.raises(g1env.G1Error):
        g1env.G1Env(8)
