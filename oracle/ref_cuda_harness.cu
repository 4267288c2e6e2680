// ref_cuda_harness.cu -- the REFERENCE's own CUDA fp32 physics (Infatoshi/g1.cu headers,
// included unchanged from the reference tree) compiled for sm_100a, exposing one batched
// FK + env_qacc kernel per state.  TEST INFRASTRUCTURE: it is the "reference's own CUDA
// fp32 path" the per-substep parity gate compares against on identical states (the harness
// pattern of the reference's src/test_envqacc.cu:29-51, with caller-supplied states instead
// of curand ones).  Built by oracle/build_oracle.py into oracle/_ref/ only where the
// reference tree is present; never shipped.
#include <cstdio>
#include <cuda_runtime.h>
// -DREF_MU=x overrides the model friction G1_FOOT_MU (the reference hard-codes 0.6); the
// model header is included first so the override holds in every physics header after it
#include "g1_model.h"
#ifdef REF_MU
#undef G1_FOOT_MU
#define G1_FOOT_MU REF_MU
#endif
#include "dynamics.cuh"
#include "aba.cuh"
#include "aba_factor.cuh"
#include "aba_bias.cuh"
#include "contact.cuh"
#include "env_qacc.cuh"
#include "g1_model.h"

__global__ void __launch_bounds__(64, 1)
k_ref_qacc(int n, const float* qpos, const float* qvel, const float* tau, const float* bdt, int pgs, float* qacc_out) {
    int w = blockIdx.x * blockDim.x + threadIdx.x;
    if (w >= n) return;
    float qp[G1_NQ], qv[G1_NV], tq[G1_NV], bd[G1_NV];
    for (int i = 0; i < G1_NQ; ++i) qp[i] = qpos[(size_t)w * G1_NQ + i];
    for (int i = 0; i < G1_NV; ++i) { qv[i] = qvel[(size_t)w * G1_NV + i]; tq[i] = tau[(size_t)w * G1_NV + i];
                                      bd[i] = bdt ? bdt[(size_t)w * G1_NV + i] : 0.f; }
    float xpos[G1_NBODY * 3], xquat[G1_NBODY * 4], xipos[G1_NBODY * 3], S[G1_NV * 6], q[G1_NV];
    forward_kinematics(qp, xpos, xquat, xipos);
    env_qacc(qp, qv, xpos, xquat, xipos, tq, bd, S, q, pgs);
    for (int i = 0; i < G1_NV; ++i) qacc_out[(size_t)w * G1_NV + i] = q[i];
}

extern "C" int ref_cuda_qacc(int n, const float* qpos, const float* qvel, const float* tau, const float* bdt, int pgs,
                             float* qacc_out) {
    // all pointers are device pointers
    k_ref_qacc<<<(n + 63) / 64, 64>>>(n, qpos, qvel, tau, bdt, pgs, qacc_out);
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) { fprintf(stderr, "ref_cuda_qacc: %s\n", cudaGetErrorString(e)); return (int)e; }
    return 0;
}

// One full physics substep of the reference's env_advance (src/g1_env.cu:118-161) from
// caller states and actions: PD target = stand + 0.5 a clamped to the ctrl range (:123-131),
// implicit-damping diagonal dt*kd (:137-139), FK, PD torque clamped to the force range
// (:143-152), env_qacc, semi-implicit velocity update with the NaN / +-50 guard (:154-160),
// integrate_pos (dynamics.cuh:345-355).  The statements follow the reference's order so the
// compiled arithmetic is the reference's own; the per-substep qpos / qvel gate compares
// against this.  (S = 1: the reward and done logic after the substep loop is not run.)
__global__ void __launch_bounds__(64, 1)
k_ref_substep(int n, const float* qpos, const float* qvel, const float* act, int pgs, float* qpos_out,
              float* qvel_out) {
    int w = blockIdx.x * blockDim.x + threadIdx.x;
    if (w >= n) return;
    float lp[G1_NQ], lv[G1_NV], target[G1_NU];
    for (int i = 0; i < G1_NQ; ++i) lp[i] = qpos[(size_t)w * G1_NQ + i];
    for (int i = 0; i < G1_NV; ++i) lv[i] = qvel[(size_t)w * G1_NV + i];
    for (int i = 0; i < G1_NU; ++i) {
        float t = g1_qpos_stand[g1_act_qadr[i]] + 0.5f * act[(size_t)w * G1_NU + i];
        if (t < g1_act_ctrl_lo[i]) t = g1_act_ctrl_lo[i];
        if (t > g1_act_ctrl_hi[i]) t = g1_act_ctrl_hi[i];
        target[i] = t;
    }
    float xpos[G1_NBODY * 3], xquat[G1_NBODY * 4], xipos[G1_NBODY * 3];
    float Sm[G1_NV * 6], qacc[G1_NV], tau[G1_NV], Bdt[G1_NV];
    const float dt = G1_DT;
    for (int i = 0; i < G1_NV; ++i) Bdt[i] = 0.f;
    for (int i = 0; i < G1_NU; ++i) Bdt[g1_act_dof[i]] = dt * g1_act_kd[i];
    forward_kinematics(lp, xpos, xquat, xipos);
    for (int i = 0; i < G1_NV; ++i) tau[i] = 0.f;
    for (int i = 0; i < G1_NU; ++i) {
        int d = g1_act_dof[i];
        float pdt = g1_act_kp[i] * (target[i] - lp[g1_act_qadr[i]]) - g1_act_kd[i] * lv[d];
        if (pdt < g1_act_frc_lo[i]) pdt = g1_act_frc_lo[i];
        else if (pdt > g1_act_frc_hi[i]) pdt = g1_act_frc_hi[i];
        tau[d] = pdt;
    }
    env_qacc(lp, lv, xpos, xquat, xipos, tau, Bdt, Sm, qacc, pgs);
    for (int i = 0; i < G1_NV; ++i) {
        float v = lv[i] + dt * qacc[i];
        if (!isfinite(v)) v = 0.f;
        if (v > 50.f) v = 50.f; else if (v < -50.f) v = -50.f;
        lv[i] = v;
    }
    integrate_pos(lp, lv, dt);
    for (int i = 0; i < G1_NQ; ++i) qpos_out[(size_t)w * G1_NQ + i] = lp[i];
    for (int i = 0; i < G1_NV; ++i) qvel_out[(size_t)w * G1_NV + i] = lv[i];
}

extern "C" int ref_cuda_substep(int n, const float* qpos, const float* qvel, const float* act, int pgs,
                                float* qpos_out, float* qvel_out) {
    // all pointers are device pointers
    k_ref_substep<<<(n + 63) / 64, 64>>>(n, qpos, qvel, act, pgs, qpos_out, qvel_out);
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) { fprintf(stderr, "ref_cuda_substep: %s\n", cudaGetErrorString(e)); return (int)e; }
    return 0;
}
