// ref_cuda_harness.cu -- the REFERENCE's own CUDA fp32 physics (Infatoshi/g1.cu headers,
// included unchanged from the reference tree) compiled for sm_100a, exposing one batched
// FK + env_qacc kernel per state.  TEST INFRASTRUCTURE: it is the "reference's own CUDA
// fp32 path" the per-substep parity gate compares against on identical states (the harness
// pattern of the reference's src/test_envqacc.cu:29-51, with caller-supplied states instead
// of curand ones).  Built by oracle/build_oracle.py into oracle/_ref/ only where the
// reference tree is present; never shipped.
#include <cstdio>
#include <cuda_runtime.h>
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
