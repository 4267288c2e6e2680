// ref_host_shim.cpp -- compiles the REFERENCE's own physics headers (Infatoshi/g1.cu,
// src/dynamics.cuh, aba.cuh, aba_factor.cuh, aba_solvem_multi.cuh, aba_bias.cuh,
// contact.cuh, env_qacc.cuh, g1_model.h) unchanged as host C++ and exports a few C entry
// points so the tests can check this repository's oracle restatement against the
// reference's own arithmetic.  TEST INFRASTRUCTURE: built only where the reference tree is
// present (oracle/build_oracle.py adds -I<reference>/src) into oracle/_ref/, never shipped.
//
// Variants (compile-time):
//   -DREF_F64   : every `float` in the headers becomes `double` (fp64 restatement)
//   -DREF_MU=x  : overrides the model friction G1_FOOT_MU (the reference hard-codes 0.6)
#include <cmath>
#include <cstring>

#define __device__
#define __constant__
#define __forceinline__ inline
#define __host__
#ifdef REF_F64
#define float double
#define sqrtf sqrt
#define sinf sin
#define cosf cos
#define powf pow
#define fabsf fabs
#define expf exp
static inline double rsqrtf(double x) { return 1.0 / sqrt(x); }
#else
static inline float rsqrtf(float x) { return 1.0f / sqrtf(x); }
#endif

#include "g1_model.h"
#ifdef REF_MU
#undef G1_FOOT_MU
#define G1_FOOT_MU REF_MU
#endif
#include "dynamics.cuh"
#include "aba.cuh"
#include "aba_factor.cuh"
#include "aba_solvem_multi.cuh"
#include "aba_bias.cuh"
#include "contact.cuh"
#include "env_qacc.cuh"

typedef float RT;  // float, or double under REF_F64

extern "C" {

int ref_real_size(void) { return (int)sizeof(RT); }

// forward_kinematics per state: qpos[n*NQ] -> xpos[n*NB*3], xquat[n*NB*4], xipos[n*NB*3]
void ref_fk(int n, const RT* qpos, RT* xpos, RT* xquat, RT* xipos) {
    for (int w = 0; w < n; ++w)
        forward_kinematics(qpos + (size_t)w * G1_NQ, xpos + (size_t)w * G1_NBODY * 3,
                           xquat + (size_t)w * G1_NBODY * 4, xipos + (size_t)w * G1_NBODY * 3);
}

// compute_bias per state (RNE, qacc=0): -> bias[n*NV]
void ref_bias(int n, const RT* qpos, const RT* qvel, RT* bias) {
    for (int w = 0; w < n; ++w) {
        RT xpos[G1_NBODY * 3], xquat[G1_NBODY * 4], xipos[G1_NBODY * 3], S[G1_NV * 6];
        const RT* qp = qpos + (size_t)w * G1_NQ;
        forward_kinematics(qp, xpos, xquat, xipos);
        compute_bias(qp, qvel + (size_t)w * G1_NV, xpos, xquat, xipos, S, bias + (size_t)w * G1_NV);
    }
}

// forward_kinematics + env_qacc per state (the test_envqacc.cu harness semantics).
// bdt may be null (then zero damping).
void ref_qacc(int n, const RT* qpos, const RT* qvel, const RT* tau, const RT* bdt, int pgs, RT* qacc) {
    for (int w = 0; w < n; ++w) {
        RT xpos[G1_NBODY * 3], xquat[G1_NBODY * 4], xipos[G1_NBODY * 3], S[G1_NV * 6], zero[G1_NV];
        for (int i = 0; i < G1_NV; ++i) zero[i] = 0;
        const RT* qp = qpos + (size_t)w * G1_NQ;
        forward_kinematics(qp, xpos, xquat, xipos);
        env_qacc(qp, qvel + (size_t)w * G1_NV, xpos, xquat, xipos, tau + (size_t)w * G1_NV,
                 bdt ? bdt + (size_t)w * G1_NV : zero, S, qacc + (size_t)w * G1_NV, pgs);
    }
}

// semi-implicit Euler position update (integrate_pos) for n states, in place.
void ref_integrate(int n, RT* qpos, const RT* qvel) {
    for (int w = 0; w < n; ++w) integrate_pos(qpos + (size_t)w * G1_NQ, qvel + (size_t)w * G1_NV, G1_DT);
}

}  // extern "C"
