"""Failure detection of the tensor-core pipeline without a GPU fault: a bounded mbarrier wait
that runs out.  The test entry g1_env_test_wait_timeout sets up the policy pipeline as the
rollout does (barriers, TMEM), waits on a barrier nothing arrives at with a spin limit of a
few thousand iterations (no bulk copy or MMA in flight), sets the device error flag and
frees TMEM.  The host reads the flag with g1_env_tc_status, and the device stays usable: a
rollout afterwards still matches the CPU oracle and reports no error."""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_timed_out_wait_is_reported_and_device_stays_usable():
    import g1env
    from oracle.oracle import Oracle, OracleEnv
    lib = g1env.load_library()
    lib.g1_env_test_wait_timeout.restype = ctypes.c_int
    lib.g1_env_test_wait_timeout.argtypes = [ctypes.c_void_p, ctypes.c_uint]
    N, H = 37, 2
    env = g1env.G1Env(N, 10, 8, seed=4)
    env.reset()
    assert env.tc_status() == 0
    assert lib.g1_env_test_wait_timeout(env.h, 4096) == 0      # the launch itself succeeds
    assert env.tc_status() == 2                                 # the wait ran out and said so
    assert env.tc_status() == 0                                 # reading clears the flag
    # the context is intact: a tensor-core rollout still matches the oracle
    oenv = OracleEnv(Oracle("f32"), N, 10, 8, seed=4)
    st = env.get_state()
    oenv.set_state(*st[:4], tick=st[4])
    W = g1env.pack_weights(g1env.init_policy_normal(g1env.AC(100, 29).cuda(), seed=2)).detach()
    mean, var = torch.zeros(100, device="cuda"), torch.ones(100, device="cuda")
    z = lambda *s: torch.zeros(*s, device="cuda")
    b = dict(O=z(H, N, 100), A=z(H, N, 29), LP=z(H, N), V=z(H, N), R=z(H, N), D=z(H, N), Vlast=z(N))
    env.rollout(H, W, mean, var, *b.values())
    torch.cuda.synchronize()
    assert env.tc_status() == 0
    ro = oenv.rollout(H, W.cpu().numpy(), mean.cpu().numpy(), var.cpu().numpy())
    for k, tol in dict(O=1e-3, A=1e-4, LP=1e-4, V=1e-4, R=1e-4, Vlast=1e-4).items():
        assert np.abs(b[k].cpu().numpy() - ro[k]).max() <= tol, k
    env.close()
    oenv.close()
