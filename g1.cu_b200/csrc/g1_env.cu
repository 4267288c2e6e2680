// g1_env.cu -- the B200 fused G1 rollout and its C-ABI (libg1env.so).
//
// Drop-in for the reference's build/libg1env.so (Infatoshi/g1.cu src/g1_env.cu:361-476):
// same exported names, argument types, buffer layouts and ownership, so the reference's
// ctypes trainer (scripts/ppo.py, scripts/ppo_fused.py) loads this library unchanged.
//
// Execution model (sm_100a):
//   * one persistent kernel per call; a CTA owns a contiguous block of worlds for the whole
//     horizon (a CTA per SM: the grid is sized to the SM count);
//   * per control step the CTA first runs the POLICY phase over its whole world block --
//     observations, normalisation, the actor-critic MLP (tcgen05 split-bf16 or FFMA),
//     Philox Gaussian sampling, trajectory writes -- then the PHYSICS phase: the block's
//     worlds are sorted by their last contact count and dealt in snake order into groups of
//     4, one group per warp, and each warp advances its group S substeps with the worlds'
//     frames in shared memory (g1_physics.cuh);
//   * world state (qpos, qvel, previous action, episode step) stays in HBM/L2 between
//     control steps ([N,36], [N,35], [N,29], [N] like the reference's EnvState).
// Errors: C-ABI functions keep the reference's void returns; failures are recorded and
// read with g1_env_last_error() instead of exit(1) (the reference's CK, g1_env.cu:33-34).
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <mutex>
#include <string>

#include "g1_physics.cuh"
#include "g1_mlp_tc.cuh"
#include "g1_gemm_tma.cuh"
#include "../../include/g1env.h"

using namespace g1;

#define OBS_DIM 100
#define ACT_DIM 29
#define CMD_VX 0.8f
#define X_FIN 5.0f
#define FINISH_BONUS 50.0f
#define ACT_SCALE 0.5f

#define NWARPS 7
#define NTHREADS (NWARPS * 32)
#define MAX_WB 64          // worlds per CTA block, upper bound (MLP activations in smem)
#define MAX_HIDDEN 4
#define XSTR 104           // normalized-obs row stride (floats)
// Barrier schedule of the physics phase, fixed at build time.  G1_LOCKSTEP > 0: the CTA's
// warps meet at a named barrier every G1_LOCKSTEP substeps (they then run the same code, and
// instruction fetch stays in cache).  G1_MIDBAR bit 1: a second barrier per substep, after
// the contact solve (measured 0.8 % faster: the warps integrate on the same code too).
#ifndef G1_LOCKSTEP
#define G1_LOCKSTEP 1
#endif
#ifndef G1_MIDBAR
#define G1_MIDBAR 2
#endif

__constant__ G1Tables c_tab;

// ------------------------------------------------------------------ error state
static std::mutex g_err_mu;
static std::string g_last_error;
static int g_last_code = 0;
static void set_error(int code, const char* where, const char* what) {
    std::lock_guard<std::mutex> lk(g_err_mu);
    g_last_code = code;
    char buf[512];
    snprintf(buf, sizeof buf, "%s: %s", where, what);
    g_last_error = buf;
}
#define CKR(call, ret)                                                       \
    do {                                                                     \
        cudaError_t e_ = (call);                                             \
        if (e_ != cudaSuccess) {                                             \
            set_error((int)e_, __func__, cudaGetErrorString(e_));            \
            return ret;                                                      \
        }                                                                    \
    } while (0)

// ------------------------------------------------------------------ Philox4x32-10
// Salmon et al., SC'11.  Counter = {world id, tick lo, tick hi, purpose<<16 | index},
// key = seed (lo, hi).  Identical layout in the CPU oracle.
__device__ __forceinline__ uint4 philox(uint4 c, uint2 k) {
#pragma unroll
    for (int r = 0; r < 10; ++r) {
        if (r) { k.x += 0x9E3779B9u; k.y += 0xBB67AE85u; }
        uint32_t hi0 = __umulhi(0xD2511F53u, c.x), lo0 = 0xD2511F53u * c.x;
        uint32_t hi1 = __umulhi(0xCD9E8D57u, c.z), lo1 = 0xCD9E8D57u * c.z;
        c = make_uint4(hi1 ^ c.y ^ k.x, lo1, hi0 ^ c.w ^ k.y, lo0);
    }
    return c;
}
enum : uint32_t { RNG_ACTION = 1, RNG_AUTORESET = 2, RNG_RESET = 3 };
__device__ __forceinline__ uint4 rng_draw(uint64_t seed, uint32_t world, uint64_t tick, uint32_t purpose, uint32_t idx) {
    return philox(make_uint4(world, (uint32_t)tick, (uint32_t)(tick >> 32), (purpose << 16) | idx),
                  make_uint2((uint32_t)seed, (uint32_t)(seed >> 32)));
}
__device__ __forceinline__ float u01_open(uint32_t x) { return (float)((x >> 8) + 1u) * (1.0f / 16777216.0f); }
__device__ __forceinline__ float u01(uint32_t x) { return (float)(x >> 8) * (1.0f / 16777216.0f); }

// ------------------------------------------------------------------ kernel parameters
enum Mode : int { MODE_ROLLOUT = 0, MODE_STEP = 1, MODE_PHYS = 2 };

struct Params {
    int N, S, pgs, H, K, mode, wb;
    float mu;
    float *qp, *qv, *pa;
    int* steps;
    uint64_t seed;
    uint32_t world0;
    uint64_t tick0;
    // policy (repacked: per layer W^T [nin][nout] then bias; head W^T [nlast][32], bias[32], log_std[32])
    const float* WT;
    int nh, hid[MAX_HIDDEN], act;
    const float *mean, *var;
    float *O, *A, *LP, *V, *R, *D, *Vlast;
    // host-loop step
    const float* act_in;
    float *obs_out, *rew_out, *done_out;
    int* ncon_hist;  // [MAXCON+1] contact-count histogram (substeps), may be null
    int lockstep;    // > 0: the CTA's warps meet at a named barrier every `lockstep` substeps
    int midbar;      // extra barriers inside a substep (group_qacc's midbar bits; with lockstep only)
    int* ncon_last;  // [N] contact count of each world's last substep (load balancing)
    int t0;          // trajectory row of the first control step of this launch
    int ext_policy;  // actions already in A[t0..]: skip the in-kernel policy phase
    // fp32 policy on the tensor cores (split-bf16, g1_mlp_tc.cuh tf_layer): chunk images and
    // biases from k_repack_tf; 0 = the FFMA path (cta_dense) over WT
    int tf_mlp;
    const __nv_bfloat16* tf_img;
    const float* tf_bias;
    long long tf_woff[MAX_HIDDEN + 1];
    int tf_boff[MAX_HIDDEN + 1], tf_lsoff;
    int* tf_err;
    int o_vec;  // O is 16-byte aligned: 128-bit observation stores
};

// ------------------------------------------------------------------ observations
// compute_obs (g1_env.cu:46-53, 69-81) for one world by one warp; returns element i.
__device__ __forceinline__ float obs_elem(int i, const float* qp, const float* qv, const float* pa, const G1Tables& T) {
    if (i < 6) return qv[i];
    if (i < 9) {
        float m[9];
        qmat(ld4(qp + 3), m);
        return -m[i];  // -third row of R_base
    }
    if (i < 38) return qp[T.act_qadr[i - 9]];
    if (i < 67) return qv[T.act_dof[i - 38]];
    if (i < 96) return pa[i - 67];
    return i == 96 ? CMD_VX : 0.f;
}

// Raw observations k0 .. k0+7 (k0 % 8 == 0) of one world, the same values as obs_elem, with
// every global load issued before the first is used (one L2 round trip per call instead of
// one per element).
__device__ __forceinline__ void obs8(int k0, const float* qp, const float* qv, const float* pa, const G1Tables& T,
                                     float* o) {
    float x[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const int i = k0 + j;
        const float* src = i < 6 ? qv + i
                         : i < 9 ? qp
                         : i < 38 ? qp + T.act_qadr[i - 9]
                         : i < 67 ? qv + T.act_dof[i - 38]
                         : i < 96 ? pa + (i - 67) : nullptr;
        x[j] = (src && (i < 6 || i >= 9)) ? *src : 0.f;
    }
    Q4 q = {0.f, 0.f, 0.f, 0.f};
    if (k0 < 16) q = ld4(qp + 3);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const int i = k0 + j;
        if (i >= 6 && i < 9) {
            float m[9];
            qmat(q, m);
            x[j] = -m[i];  // -third row of R_base
        } else if (i >= 96) {
            x[j] = i == 96 ? CMD_VX : 0.f;
        }
        o[j] = x[j];
    }
}

// ------------------------------------------------------------------ policy phase
// out[w][o] = act(b[o] + sum_i W[o][i] in[w][i]), i ascending (the mlp_forward order,
// g1_env.cu:230-237), for the nw worlds of the block.  WT is [nin][wstr] (W transposed);
// weights are staged through shared memory in tiles of KT inputs x OC outputs (coalesced
// loads, reused by every world of the block); a thread owns 2 outputs x 4 worlds of an
// output chunk.  nin must be a multiple of 4 (inputs are read as float4).
#define KT 64
#define OC 64
#define TILE_PER ((KT * OC + NTHREADS - 1) / NTHREADS)
__device__ __noinline__ void cta_dense(const float* __restrict__ WT, int wstr, const float* __restrict__ bias, int nin, int nout,
                                       const float* in, int istr, float* out, int ostr, int nw, int act, float* wtile) {
    const int nwg = (nw + 3) >> 2;
    constexpr int NOG = OC / 2;
    const int nitems = NOG * nwg;
    constexpr int MAXIT = (NOG * (MAX_WB / 4) + NTHREADS - 1) / NTHREADS;
    for (int oc0 = 0; oc0 < nout; oc0 += OC) {
        float acc[MAXIT][4][2];
#pragma unroll
        for (int j = 0; j < MAXIT; ++j) {
            const int it = threadIdx.x + j * NTHREADS;
            const int o0 = oc0 + 2 * (it % NOG);
            const float b0 = (it < nitems && o0 < nout) ? bias[o0] : 0.f;
            const float b1 = (it < nitems && o0 + 1 < nout) ? bias[o0 + 1] : 0.f;
#pragma unroll
            for (int k = 0; k < 4; ++k) { acc[j][k][0] = b0; acc[j][k][1] = b1; }
        }
        // weight tiles are fetched one tile ahead into registers, so the global loads of tile
        // k+1 are in flight while tile k is multiplied
        float pre[TILE_PER];
        auto fetch = [&](int k0) {
            const int kt = min(KT, nin - k0);
#pragma unroll
            for (int q = 0; q < TILE_PER; ++q) {
                const int e = threadIdx.x + q * NTHREADS, kk = e / OC, oo = e % OC;
                pre[q] = (e < KT * OC && kk < kt && oc0 + oo < nout) ? __ldg(WT + (size_t)(k0 + kk) * wstr + oc0 + oo) : 0.f;
            }
        };
        fetch(0);
        for (int k0 = 0; k0 < nin; k0 += KT) {
            const int kt = min(KT, nin - k0);
            __syncthreads();  // previous tile consumed
#pragma unroll
            for (int q = 0; q < TILE_PER; ++q) {
                const int e = threadIdx.x + q * NTHREADS;
                if (e < KT * OC) wtile[e] = pre[q];
            }
            __syncthreads();
            if (k0 + KT < nin) fetch(k0 + KT);
#pragma unroll
            for (int j = 0; j < MAXIT; ++j) {
                const int it = threadIdx.x + j * NTHREADS;
                if (it >= nitems) break;
                const int og = it % NOG, w0 = 4 * (it / NOG);
                const float* xr[4];
#pragma unroll
                for (int k = 0; k < 4; ++k) xr[k] = in + (size_t)min(w0 + k, nw - 1) * istr + k0;
                const float* wt = wtile + 2 * og;
                for (int kk = 0; kk < kt; kk += 4) {
                    const float2 wa = *reinterpret_cast<const float2*>(wt + (kk + 0) * OC);
                    const float2 wb = *reinterpret_cast<const float2*>(wt + (kk + 1) * OC);
                    const float2 wc = *reinterpret_cast<const float2*>(wt + (kk + 2) * OC);
                    const float2 wd = *reinterpret_cast<const float2*>(wt + (kk + 3) * OC);
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        const float4 x = *reinterpret_cast<const float4*>(xr[k] + kk);
                        acc[j][k][0] += wa.x * x.x; acc[j][k][1] += wa.y * x.x;
                        acc[j][k][0] += wb.x * x.y; acc[j][k][1] += wb.y * x.y;
                        acc[j][k][0] += wc.x * x.z; acc[j][k][1] += wc.y * x.z;
                        acc[j][k][0] += wd.x * x.w; acc[j][k][1] += wd.y * x.w;
                    }
                }
            }
        }
#pragma unroll
        for (int j = 0; j < MAXIT; ++j) {
            const int it = threadIdx.x + j * NTHREADS;
            if (it >= nitems) break;
            const int o0 = oc0 + 2 * (it % NOG), w0 = 4 * (it / NOG);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                if (w0 + k >= nw) break;
#pragma unroll
                for (int q = 0; q < 2; ++q) {
                    if (o0 + q >= nout) break;
                    float v = acc[j][k][q];
                    if (act == 0) v = tanhf(v);
                    else if (act == 1) v = v > 0.f ? v : expm1f(v);
                    out[(size_t)(w0 + k) * ostr + o0 + q] = v;
                }
            }
        }
    }
    __syncthreads();
}

// Policy phase for the CTA's world block: obs -> normalise -> MLP -> sample -> writes.
// The block's actions go to A[t] (the physics phase reads them back from there).
// k_rollout body, g1_env.cu:296-318.
// final_value: only the value head is used (bootstrap Vlast, g1_env.cu:325-332).
__device__ __forceinline__ void policy_sample(const Params& P, const float* HD, const float* lsp, float* tmp, int wbeg,
                                              int nbw, int t, bool final_value);

// tfs (shared memory, tensor-core path only): the g1tc::TfShared pipeline state (mbarriers,
// TMEM address, phases), kept outside `work`, which the physics phases reuse.
__device__ __noinline__ void policy_phase(const Params& P, const G1Tables& T, float* work, int wbeg, int nbw, int t,
                             bool final_value, float* tfs) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int maxw = 0;
    for (int l = 0; l < P.nh; ++l) maxw = max(maxw, P.hid[l]);
    const int hstr = ((maxw + 3) & ~3) + 4;
    // FFMA path: X [nbw][XSTR], H0/H1 [nbw][hstr], weight tile.  Tensor-core path
    // (g1_mlp_tc.cuh): split-bf16 activations A, weight stages, head outputs; the pipeline
    // state lives in tfs.
    uint8_t* tf_A = reinterpret_cast<uint8_t*>(((uintptr_t)work + 127) & ~(uintptr_t)127);
    uint8_t* tf_stages = tf_A + g1tc::TF_ABYTES;
    float* tf_hd = reinterpret_cast<float*>(tf_stages + g1tc::TF_NSTAGE * g1tc::TF_STAGE);
    g1tc::TfShared* TS = reinterpret_cast<g1tc::TfShared*>(tfs);
    auto tf_L = [&](int l) -> g1tc::TfLayer {
        return g1tc::TfLayer{P.tf_img + P.tf_woff[l], P.tf_bias + P.tf_boff[l], l == 0 ? OBS_DIM : P.hid[l - 1],
                             l == P.nh ? 32 : P.hid[l]};
    };
    if (P.tf_mlp) {
        // first layer's weights stream in while the observations are built
        if (threadIdx.x == g1tc::TF_COPY_WARP * 32) {
            const g1tc::TfLayer L0 = tf_L(0);
            if (!g1tc::tf_prefetch(TS, tf_stages, L0, TS->st[1])) atomicExch(P.tf_err, 1);
        }
        // observations: raw to O, normalised straight into the three bf16 parts of A (8
        // inputs per thread; inputs 100..111 zero)
        // consecutive threads take consecutive worlds (contiguous stores into A; see tf_layer)
        for (int e = threadIdx.x; e < nbw * 14; e += NTHREADS) {
            const int w = e % nbw, k0 = (e / nbw) * 8, gw = wbeg + w;
            const float* qp = P.qp + (size_t)gw * NQ;
            const float* qv = P.qv + (size_t)gw * NV;
            const float* pa = P.pa + (size_t)gw * NU;
            float v[8], o[8], mu[8], va[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int i = k0 + j;
                mu[j] = i < OBS_DIM ? P.mean[i] : 0.f;
                va[j] = i < OBS_DIM ? P.var[i] : 0.f;
            }
            obs8(k0, qp, qv, pa, T, o);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int i = k0 + j;
                float z = 0.f;
                if (i < OBS_DIM) {
                    z = (o[j] - mu[j]) / sqrtf(va[j] + 1e-8f);
                    if (z < -10.f) z = -10.f; else if (z > 10.f) z = 10.f;
                } else {
                    o[j] = 0.f;
                }
                v[j] = z;
            }
            if (!final_value && k0 < OBS_DIM) {
                float* row = P.O + ((size_t)t * P.N + gw) * OBS_DIM + k0;
                if (P.o_vec) {  // raw obs: 16-byte stores (rows are 400 B; O is 16-byte aligned)
                    float4* dst = reinterpret_cast<float4*>(row);
                    dst[0] = make_float4(o[0], o[1], o[2], o[3]);
                    if (k0 + 8 <= OBS_DIM) dst[1] = make_float4(o[4], o[5], o[6], o[7]);
                } else {
#pragma unroll
                    for (int j = 0; j < 8; ++j)
                        if (k0 + j < OBS_DIM) row[j] = o[j];
                }
            }
            g1tc::tf_store8(tf_A, w, k0, v);
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncthreads();
        PROF_BEGIN();
        for (int l = 0; l <= P.nh; ++l) {
            const g1tc::TfLayer L = tf_L(l), Ln = l < P.nh ? tf_L(l + 1) : L;
            g1tc::tf_layer<NTHREADS>(TS, tf_A, tf_stages, L, l < P.nh ? &Ln : nullptr, nbw, l < P.nh ? P.act : -1, tf_hd,
                                     P.tf_err);
            PROF_MARK(l == 0 ? P_MLP : (l < P.nh ? P_MLP_L1 : P_MLP_HEAD));
        }
        policy_sample(P, tf_hd, P.tf_bias + P.tf_lsoff, tf_hd + g1tc::TF_ROWS * 32, wbeg, nbw, t, final_value);
        PROF_MARK(P_SAMPLE);
        return;
    }
    float* X = work;
    float* H0 = X + MAX_WB * XSTR;
    float* H1 = H0 + MAX_WB * hstr;
    float* WTILE = H1 + MAX_WB * hstr;  // [KT][OC]
    // observations (raw to O, normalised to X)
    for (int w = warp; w < nbw; w += NWARPS) {
        const int gw = wbeg + w;
        const float* qp = P.qp + (size_t)gw * NQ;
        const float* qv = P.qv + (size_t)gw * NV;
        const float* pa = P.pa + (size_t)gw * NU;
        for (int i = lane; i < OBS_DIM; i += 32) {
            float o = obs_elem(i, qp, qv, pa, T);
            if (!final_value) P.O[((size_t)t * P.N + gw) * OBS_DIM + i] = o;
            float z = (o - P.mean[i]) / sqrtf(P.var[i] + 1e-8f);
            if (z < -10.f) z = -10.f; else if (z > 10.f) z = 10.f;
            X[w * XSTR + i] = z;
        }
        if (lane < XSTR - OBS_DIM) X[w * XSTR + OBS_DIM + lane] = 0.f;
    }
    __syncthreads();
    PROF_BEGIN();
    // hidden layers
    const float* wp = P.WT;
    const float* in = X;
    int nin = OBS_DIM, istr = XSTR;
    float* bufs[2] = {H0, H1};
    for (int l = 0; l < P.nh; ++l) {
        const int no = P.hid[l];
        float* out = bufs[l & 1];
        cta_dense(wp, no, wp + (size_t)nin * no, nin, no, in, istr, out, hstr, nbw, P.act, WTILE);
        wp += (size_t)nin * no + no;
        in = out; nin = no; istr = hstr;
        __syncthreads();
        PROF_MARK(l == 0 ? P_MLP : P_MLP_L1);
    }
    // heads: 29 means + value (+2 pad) -> scratch row of 32 in X (X is dead now)
    float* HD = X;
    cta_dense(wp, 32, wp + (size_t)nin * 32, nin, 30, in, istr, HD, 32, nbw, -1, WTILE);
    const float* lsp = wp + (size_t)nin * 32 + 32;
    __syncthreads();
    PROF_MARK(P_MLP_HEAD);
    policy_sample(P, HD, lsp, WTILE, wbeg, nbw, t, final_value);  // the weight tile is dead after the head
    PROF_MARK(P_SAMPLE);
}

// sampling (g1_env.cu:308-318): one thread per (world, action) draws the Gaussian and writes
// the action; the log-prob terms go to tmp [nbw][32] and one thread per world adds them in
// action order.  HD [nbw][32] holds the 29 means and the value, lsp the 29 log-stds.
__device__ __forceinline__ void policy_sample(const Params& P, const float* HD, const float* lsp, float* tmp, int wbeg,
                                              int nbw, int t, bool final_value) {
    const size_t sb0 = (size_t)t * P.N + wbeg;
    if (!final_value) {
        const float LOG2PI = 1.8378770664093453f;
        const uint64_t tick = P.tick0 + (uint64_t)t;
        for (int e = threadIdx.x; e < nbw * ACT_DIM; e += NTHREADS) {
            const int w = e / ACT_DIM, i = e % ACT_DIM;
            const uint4 rb = rng_draw(P.seed, P.world0 + (uint32_t)(wbeg + w), tick, RNG_ACTION, (uint32_t)i);
            const float nz = sqrtf(-2.f * logf(u01_open(rb.x))) * cosf(6.283185307179586f * u01(rb.y));
            const float ls = lsp[i];
            P.A[sb0 * ACT_DIM + e] = HD[w * 32 + i] + expf(ls) * nz;
            tmp[w * 32 + i] = -0.5f * nz * nz - ls - 0.5f * LOG2PI;
        }
        __syncthreads();
    }
    if (threadIdx.x < nbw) {
        const int w = threadIdx.x, gw = wbeg + w;
        const float* hd = HD + w * 32;
        if (final_value) {
            P.Vlast[gw] = hd[29];
        } else {
            float lps = 0.f;
            for (int i = 0; i < ACT_DIM; ++i) lps += tmp[w * 32 + i];
            P.LP[sb0 + w] = lps;
            P.V[sb0 + w] = hd[29];
        }
    }
    __syncthreads();
}

// ------------------------------------------------------------------ physics phase
// Named barrier that keeps the CTA's warps on the same substep (so they fetch the same code).
__device__ __forceinline__ void substep_barrier() { asm volatile("bar.sync 1, %0;" ::"r"(NTHREADS) : "memory"); }
// The one place the substep barrier is taken: every warp of the CTA -- with or without a group
// of worlds this round -- calls this for each substep s, so all warps reach the same barriers.
__device__ __forceinline__ void lockstep_barrier(const Params& P, int s) {
    if (P.lockstep > 0 && s % P.lockstep == 0) substep_barrier();
}
// the barriers group_qacc takes inside a substep, for a warp without a group this round
__device__ __forceinline__ void idle_midbar(const Params& P) {
    if (P.lockstep > 0) {
        if (P.midbar & 1) substep_barrier();
        PROF_BEGIN();
        if (P.midbar & 2) substep_barrier();
        PROF_MARK(P_MIDBAR);
    }
}

// The global world ids of a group's GW slots.  Indexed through unrolled selects, so the ids
// stay in registers (a run-time array index would put them in local memory).
struct Slots {
    int v[GW];
    __device__ __forceinline__ int operator[](int w) const {
        int r = v[0];
#pragma unroll
        for (int k = 1; k < GW; ++k) r = (w == k) ? v[k] : r;
        return r;
    }
    __device__ __forceinline__ void set(int w, int id) {
#pragma unroll
        for (int k = 0; k < GW; ++k)
            if (k == w) v[k] = id;
    }
};

// One control step of GW worlds (global ids wid[0 .. nvalid-1]; the remaining slots carry a
// stand pose and are not written back) by one warp: PD targets, S substeps, reward, done,
// auto-reset.  env_advance, g1_env.cu:118-212.  `acts_base`: actions indexed by global world
// id (row-major [N,29]; null = zero action).
__device__ void group_control_step(const Params& P, const G1Tables& T, float* grp, float* cw, const Slots& wid, int nvalid,
                                   const float* acts_base, uint64_t tick, float& r_out, float& d_out) {
    const int lane = threadIdx.x & 31;
    PROF_BEGIN();
    // slot w < nvalid holds world wid[w]; its actions are acts_base[wid[w]] (null = zero)
    // load state
    for (int it = lane; it < GW * NQ; it += 32) {
        const int w = it / NQ, i = it % NQ;
        grp[w * WFLOATS + WL::QP + i] = w < nvalid ? P.qp[(size_t)wid[w] * NQ + i] : T.qpos_stand[i];
    }
    for (int it = lane; it < GW * 36; it += 32) {
        const int w = it / 36, i = it % 36;
        float* fr = grp + w * WFLOATS;
        fr[WL::QV + i] = (w < nvalid && i < NV) ? P.qv[(size_t)wid[w] * NV + i] : 0.f;
        fr[WL::TAU + i] = 0.f;
    }
    for (int it = lane; it < GW * ACT_DIM; it += 32) {
        const int w = it / ACT_DIM, i = it % ACT_DIM;
        const float a = (acts_base && w < nvalid) ? acts_base[(size_t)wid[w] * ACT_DIM + i] : 0.f;
        float t = T.target0[i] + ACT_SCALE * a;
        if (t < T.ctrl_lo[i]) t = T.ctrl_lo[i];
        if (t > T.ctrl_hi[i]) t = T.ctrl_hi[i];
        grp[w * WFLOATS + WL::TGT + i] = t;
    }
    float energy = 0.f, vx_sum = 0.f;  // lane w < GW: world w
    QaccOpts opt;
    opt.pgs_iters = P.pgs; opt.mu = P.mu; opt.bdt = nullptr; opt.bdt_all = T.bdt;
    PROF_MARK(P_CS_LOAD);
    // PD torque, clamped to the actuator range, and |tau qd| accumulated into the energy
    // actuator by actuator in index order (g1_env.cu:143-152).  The torque of substep s + 1 is
    // computed right after substep s integrates (same values; it keeps this small piece of code
    // next to the integration code, which is still in the instruction cache).
    auto pd_torque = [&]() {
        for (int it = lane; it < GW * ACT_DIM; it += 32) {
            const int w = it / ACT_DIM, i = it % ACT_DIM;
            float* fr = grp + w * WFLOATS;
            const int d = T.act_dof[i];
            float pdt = T.kp[i] * (fr[WL::TGT + i] - fr[WL::QP + T.act_qadr[i]]) - T.kd[i] * fr[WL::QV + d];
            if (pdt < T.frc_lo[i]) pdt = T.frc_lo[i];
            else if (pdt > T.frc_hi[i]) pdt = T.frc_hi[i];
            fr[WL::TAU + d] = pdt;
            fr[WL::CON + i] = fabsf(pdt * fr[WL::QV + d]);
        }
        __syncwarp();
        if (lane < GW) {
            const float* e = grp + lane * WFLOATS + WL::CON;
            for (int i = 0; i < ACT_DIM; ++i) energy += e[i];
        }
        __syncwarp();
    };
    __syncwarp();
    pd_torque();
    for (int s = 0; s < P.S; ++s) {
        PROF_BEGIN();
        lockstep_barrier(P, s);
#ifdef G1_PROF
        (void)*(volatile const float*)grp;  // bar.sync blocks lazily: make the wait land here
#endif
        PROF_MARK(P_BAR);
        int ncon[GW];
        group_qacc(grp, cw, T, lane, opt, nullptr, nullptr, ncon, nullptr, P.lockstep > 0 ? P.midbar : 0, NTHREADS, 1);
        if (P.ncon_hist && lane == 0)
#pragma unroll
            for (int w = 0; w < GW; ++w)
                if (w < nvalid) atomicAdd(&P.ncon_hist[ncon[w]], 1);
        if (s == P.S - 1 && P.ncon_last && lane < nvalid) {
            int nc = 0;
#pragma unroll
            for (int w = 0; w < GW; ++w) nc = (w == lane) ? ncon[w] : nc;
            P.ncon_last[wid[lane]] = nc;
        }
        {
            PROF_BEGIN();
            group_integrate(grp, T, lane, true);
            if (lane < GW) vx_sum += grp[lane * WFLOATS + WL::QV];
            PROF_MARK(P_INTEG);
            if (s + 1 < P.S) pd_torque();
            PROF_MARK(P_STEP);
        }
    }
    // reward / termination per world (g1_env.cu:164-197), lane w
    PROF_RESTART();
    int d_flag = 0;
    if (lane < nvalid) {
        const int w = lane, gw = wid[w];
        const float* fr = grp + w * WFLOATS;
        const float* qp = fr + WL::QP;
        const float* qv = fr + WL::QV;
        const float vx = vx_sum / (float)P.S, height = qp[2];
        float m[9];
        qmat(ld4(qp + 3), m);
        const float up = m[8];
        const int alive = (height < 0.45f || up < 0.5f) ? 0 : 1;
        const float upc = up < 0.f ? 0.f : (up > 1.f ? 1.f : up);
        float vxc = vx > CMD_VX ? CMD_VX : vx;
        if (vxc < 0.f) vxc = 0.f;
        const float r_vel = 1.0f * vxc * upc;
        const float r_lat = -0.2f * fabsf(qv[1]) - 0.05f * fabsf(qv[5]);
        const float r_up = 0.3f * upc;
        const float r_h = -0.5f * fabsf(height - 0.78f);
        float act_pen = 0.f;
        for (int i = 0; i < ACT_DIM; ++i) {
            const float da = (acts_base ? acts_base[(size_t)gw * ACT_DIM + i] : 0.f) - P.pa[(size_t)gw * NU + i];
            act_pen += da * da;
        }
        if (act_pen > 10.f) act_pen = 10.f;
        float r = alive ? 1.0f + r_vel + r_lat + r_up + r_h - 0.005f * act_pen - 1e-4f * energy : -5.0f;
        const int step = P.steps[gw] + 1;
        const int won = (alive && qp[0] >= X_FIN);
        if (won) r += FINISH_BONUS;
        d_flag = (!alive || won || step >= 1000) ? 1 : 0;
        P.steps[gw] = d_flag ? 0 : step;
        r_out = r;
        d_out = (float)d_flag;
    }
    unsigned dmask = __ballot_sync(FULLMASK, d_flag != 0);
    __syncwarp();
    PROF_MARK(P_CS_REWARD);
    // auto-reset (g1_env.cu:202-210), store state and previous action
    for (int it = lane; it < GW * NQ; it += 32) {
        const int w = it / NQ, i = it % NQ;
        if ((dmask >> w) & 1u) grp[w * WFLOATS + WL::QP + i] = T.qpos_stand[i];
    }
    __syncwarp();
    for (int it = lane; it < GW * ACT_DIM; it += 32) {
        const int w = it / ACT_DIM, i = it % ACT_DIM;
        if (w >= nvalid) continue;
        const int gw = wid[w];
        if ((dmask >> w) & 1u) {
            const uint4 rb = rng_draw(P.seed, P.world0 + (uint32_t)gw, tick, RNG_AUTORESET, (uint32_t)i);
            grp[w * WFLOATS + WL::QP + T.act_qadr[i]] += 0.05f * (u01_open(rb.x) * 2.f - 1.f);
            P.pa[(size_t)gw * NU + i] = 0.f;
        } else {
            P.pa[(size_t)gw * NU + i] = acts_base ? acts_base[(size_t)gw * ACT_DIM + i] : 0.f;
        }
    }
    __syncwarp();
    for (int it = lane; it < GW * NQ; it += 32) {
        const int w = it / NQ, i = it % NQ;
        if (w < nvalid) P.qp[(size_t)wid[w] * NQ + i] = grp[w * WFLOATS + WL::QP + i];
    }
    for (int it = lane; it < GW * NV; it += 32) {
        const int w = it / NV, i = it % NV;
        if (w < nvalid) P.qv[(size_t)wid[w] * NV + i] = ((dmask >> w) & 1u) ? 0.f : grp[w * WFLOATS + WL::QV + i];
    }
    __syncwarp();
    PROF_MARK(P_CS_STORE);
}

// ------------------------------------------------------------------ the kernel
struct SmemPlan {
    int tab_floats, group_floats, tf_floats, total_bytes;
};
// [tables][NWARPS frames][4 + MAX_WB: perm][16: tensor-core MLP barriers, TMEM slot, context]
__host__ __device__ inline SmemPlan smem_plan() {
    SmemPlan p;
    p.tab_floats = ((int)((sizeof(G1Tables) + 15) / 16)) * 4;
    p.group_floats = GROUP_FLOATS;
    p.tf_floats = p.tab_floats + NWARPS * p.group_floats + 4 + MAX_WB;
    p.total_bytes = (p.tf_floats + 16 + 2 * 16) * 4;
    return p;
}
static_assert(((((int)((sizeof(G1Tables) + 15) / 16)) * 4 + NWARPS * GROUP_FLOATS + 4 + MAX_WB) & 1) == 0,
              "mbarriers need 8-byte alignment");
// policy scratch of the tensor-core MLP inside the frames (g1_mlp_tc.cuh: activations,
// weight stages, head outputs), 128 bytes of alignment slack
static_assert(128 + g1tc::TF_SCRATCH + g1tc::TF_ROWS * 32 * 4 <= NWARPS * GROUP_FLOATS * 4,
              "tensor-core MLP scratch and the sampling terms must fit in the frames");
static_assert(sizeof(g1tc::TfShared) <= (16 + 2 * 16) * 4, "tensor-core MLP state must fit its smem slot");
static_assert(MAX_WB * XSTR + 2 * MAX_WB * 260 + KT * OC <= NWARPS * GROUP_FLOATS, "MLP activations must fit in the frames");

__device__ __forceinline__ void load_tables(float* smem) {
    const int4* src = reinterpret_cast<const int4*>(&c_tab);
    int4* dst = reinterpret_cast<int4*>(smem);
    for (int i = threadIdx.x; i < (int)(sizeof(G1Tables) / 16); i += blockDim.x) dst[i] = src[i];
}

__global__ void __launch_bounds__(NTHREADS, 1) k_g1(const __grid_constant__ Params P) {
#ifdef G1_PROF
    const long long t_kernel0 = clock64();
#endif
    extern __shared__ float4 smem4[];
    float* smem = reinterpret_cast<float*>(smem4);
    const SmemPlan plan = smem_plan();
    load_tables(smem);
    const G1Tables& T = *reinterpret_cast<const G1Tables*>(smem);
    float* frames = smem + plan.tab_floats;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float* grp = frames + warp * plan.group_floats;
    float* cw = grp + GW * WFLOATS;
    __syncthreads();

    const int wbeg = blockIdx.x * P.wb;
    const int nbw = min(P.wb, P.N - wbeg);
    if (nbw <= 0) return;
    // tensor-core MLP: barriers + 256 TMEM columns for the life of this (persistent) CTA
    float* tfs = smem + plan.tf_floats;
    const bool use_tf = P.tf_mlp && P.mode == MODE_ROLLOUT && !P.ext_policy;
    if (use_tf) g1tc::tf_init(reinterpret_cast<g1tc::TfShared*>(tfs));
    const int nsteps = P.mode == MODE_ROLLOUT ? P.H : (P.mode == MODE_PHYS ? P.K : 1);
    const int nrounds = (nbw + GW * NWARPS - 1) / (GW * NWARPS);
    int* perm = reinterpret_cast<int*>(frames + NWARPS * plan.group_floats + 4);
    for (int t = 0; t < nsteps; ++t) {
        const uint64_t tick = P.tick0 + (uint64_t)t;
        const int trow = P.t0 + t;
        if (P.mode == MODE_ROLLOUT && !P.ext_policy) {
            PROF_BEGIN();
            policy_phase(P, T, frames, wbeg, nbw, t, false, tfs);
            PROF_MARK(P_POLICY);
        }
        __syncthreads();
        // physics.  Worlds are dealt into groups of GW: sorted by their last contact count
        // (descending, stable) and dealt in snake order over the groups, so every warp gets a
        // similar contact load.  Warp takes groups warp, warp + NWARPS, ...; a warp with no
        // group in a round still passes the substep barriers.
        const int ngroups = (nbw + GW - 1) / GW;
        PROF_BEGIN();
        if (warp == 0) {
            int v0 = -1, v1 = -1;  // this lane's two worlds (nbw <= 64)
            if (lane < nbw) v0 = P.ncon_last ? P.ncon_last[wbeg + lane] : 0;
            if (lane + 32 < nbw) v1 = P.ncon_last ? P.ncon_last[wbeg + lane + 32] : 0;
            int base = 0;
            for (int v = MAXCON; v >= 0; --v) {
                const unsigned m0 = __ballot_sync(FULLMASK, v0 == v), m1 = __ballot_sync(FULLMASK, v1 == v);
                const unsigned below = (1u << lane) - 1u;
                if (v0 == v) perm[base + __popc(m0 & below)] = lane;
                if (v1 == v) perm[base + __popc(m0) + __popc(m1 & below)] = lane + 32;
                base += __popc(m0) + __popc(m1);
            }
        }
        __syncthreads();
        PROF_MARK(P_SORT);
        for (int round = 0; round < nrounds; ++round) {
            const int g = warp + round * NWARPS;
            Slots wid;
            int nvalid = 0;
#pragma unroll
            for (int sl = 0; sl < GW; ++sl) {
                const int pidx = sl * ngroups + ((sl & 1) ? ngroups - 1 - g : g);
                wid.v[sl] = wbeg;
                if (g < ngroups && pidx < nbw) wid.set(nvalid++, wbeg + perm[pidx]);
            }
            if (nvalid == 0) {
                if (P.lockstep)
                    for (int s = 0; s < P.S; ++s) { lockstep_barrier(P, s); idle_midbar(P); }
                continue;
            }
            const float* acts = P.mode == MODE_ROLLOUT ? P.A + (size_t)trow * P.N * ACT_DIM
                              : P.act_in;  // MODE_STEP: this step's actions; MODE_PHYS: constant actions (may be null = zero)
            float my_r = 0.f, my_d = 0.f;  // lane w < nvalid: reward and done of slot w
            group_control_step(P, T, grp, cw, wid, nvalid, acts, tick, my_r, my_d);
            const int my_w = wid[lane < GW ? lane : 0];
            if (lane < nvalid) {
                if (P.mode == MODE_ROLLOUT) {
                    P.R[(size_t)trow * P.N + my_w] = my_r;
                    P.D[(size_t)trow * P.N + my_w] = my_d;
                } else if (P.mode == MODE_STEP) {
                    P.rew_out[my_w] = my_r;
                    P.done_out[my_w] = my_d;
                }
            }
            if (P.mode == MODE_STEP) {  // k_step's obs after the step (g1_env.cu:265-266)
                __syncwarp();
                for (int it = lane; it < nvalid * OBS_DIM; it += 32) {
                    const int sl = it / OBS_DIM, i = it % OBS_DIM;
                    const int gw = wid[sl];
                    P.obs_out[(size_t)gw * OBS_DIM + i] =
                        obs_elem(i, P.qp + (size_t)gw * NQ, P.qv + (size_t)gw * NV, P.pa + (size_t)gw * NU, T);
                }
            }
            __syncwarp();
        }
        {
            PROF_BEGIN();
            __syncthreads();
            PROF_MARK(P_WAIT);
        }
    }
    if (P.mode == MODE_ROLLOUT && !P.ext_policy) policy_phase(P, T, frames, wbeg, nbw, 0, true, tfs);
    if (use_tf) g1tc::tf_release(reinterpret_cast<g1tc::TfShared*>(tfs));
#ifdef G1_PROF
    if (lane == 0) atomicAdd(&g_prof[P_TOTAL], (unsigned long long)(clock64() - t_kernel0));
#endif
}
// Per-state FK + generalised acceleration (the reference's test_envqacc.cu harness
// semantics, with caller states): a warp takes GW states at a time.
__global__ void __launch_bounds__(NTHREADS, 1) k_qacc(int n, const float* qpos, const float* qvel, const float* tau,
                                                      const float* bdt, int pgs, float mu, float* qacc_out,
                                                      float* qacc_s_out, float* bias_out, float* f_out, int* ncon_out) {
    extern __shared__ float4 smem4[];
    float* smem = reinterpret_cast<float*>(smem4);
    const SmemPlan plan = smem_plan();
    load_tables(smem);
    __syncthreads();
    const G1Tables& T = *reinterpret_cast<const G1Tables*>(smem);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float* grp = smem + plan.tab_floats + warp * plan.group_floats;
    float* cw = grp + GW * WFLOATS;
    for (int s0 = (blockIdx.x * NWARPS + warp) * GW; s0 < n; s0 += gridDim.x * NWARPS * GW) {
        const int nvalid = min(GW, n - s0);
        for (int it = lane; it < GW * 36; it += 32) {
            const int w = it / 36, i = it % 36;
            float* fr = grp + w * WFLOATS;
            const bool ok = w < nvalid;
            const size_t st = (size_t)(s0 + (ok ? w : 0));
            fr[WL::QP + i] = ok && i < NQ ? qpos[st * NQ + i] : (i < NQ ? T.qpos_stand[i] : 0.f);
            fr[WL::QV + i] = ok && i < NV ? qvel[st * NV + i] : 0.f;
            fr[WL::TAU + i] = ok && i < NV && tau ? tau[st * NV + i] : 0.f;
        }
        __syncwarp();
        const float* bdt_w[GW];
        float* bias_w[GW];
        float* f_w[GW];
        float* qs_w[GW];
#pragma unroll
        for (int w = 0; w < GW; ++w) {
            const bool ok = w < nvalid;
            bdt_w[w] = (ok && bdt) ? bdt + (size_t)(s0 + w) * NV : nullptr;  // damping rows read from global
            bias_w[w] = (ok && bias_out) ? bias_out + (size_t)(s0 + w) * NV : nullptr;
            f_w[w] = (ok && f_out) ? f_out + (size_t)(s0 + w) * MAXEFC : nullptr;
            qs_w[w] = (ok && qacc_s_out) ? qacc_s_out + (size_t)(s0 + w) * NV : nullptr;
        }
        QaccOpts opt;
        opt.pgs_iters = pgs; opt.mu = mu; opt.bdt = bdt_w; opt.bdt_all = nullptr;
        int ncon[GW];
        group_qacc(grp, cw, T, lane, opt, bias_w, f_w, ncon, qs_w);
        for (int it = lane; it < nvalid * NV; it += 32) {
            const int w = it / NV, i = it % NV;
            const float* fr = grp + w * WFLOATS;
            if (qacc_out) qacc_out[(size_t)(s0 + w) * NV + i] = fr[WL::QACC + i];
        }
        if (ncon_out && lane < nvalid) ncon_out[s0 + lane] = ncon[lane];
        __syncwarp();
    }
}

// ------------------------------------------------------------------ large-policy pipeline
// For policies run on the tensor cores the control step is split into launches: observations
// (k_obs_norm) -> one tcgen05 dense layer per MLP layer (bf16 activations in HBM/L2) -> head
// -> sampling (k_sample) -> one physics step of k_g1 with the actions already in A[t].
#define XK 104  // padded observation width of the bf16 activations (multiple of 8)

// raw obs -> O[row] (row >= 0), normalised + clipped obs -> Xb [N][XK] bf16 (g1_env.cu:297-304)
__global__ void k_obs_norm(Params P, int row, __nv_bfloat16* Xb) {
    const int w = blockIdx.x * blockDim.y + threadIdx.y;
    if (w >= P.N) return;
    const G1Tables& T = c_tab;
    const float* qp = P.qp + (size_t)w * NQ;
    const float* qv = P.qv + (size_t)w * NV;
    const float* pa = P.pa + (size_t)w * NU;
    for (int i = threadIdx.x; i < XK; i += blockDim.x) {
        float z = 0.f;
        if (i < OBS_DIM) {
            const float o = obs_elem(i, qp, qv, pa, T);
            if (row >= 0) P.O[((size_t)row * P.N + w) * OBS_DIM + i] = o;
            z = (o - P.mean[i]) / sqrtf(P.var[i] + 1e-8f);
            if (z < -10.f) z = -10.f; else if (z > 10.f) z = 10.f;
        }
        Xb[(size_t)w * XK + i] = __float2bfloat16(z);
    }
}

// Gaussian actions and log-probabilities from the head outputs HD [N][32] (29 means, value)
// (g1_env.cu:308-318); row < 0: only the bootstrap value -> Vlast
// HV: the [N][32] head output whose column 29 is the value (HD itself for the shared trunk)
__global__ void k_sample(Params P, int row, const float* HD, const float* HV, const float* ls, uint64_t tick) {
    const int w = blockIdx.x * blockDim.x + threadIdx.x;
    if (w >= P.N) return;
    const float* hd = HD + (size_t)w * 32;
    const float val = HV[(size_t)w * 32 + 29];
    if (row < 0) { P.Vlast[w] = val; return; }
    const float LOG2PI = 1.8378770664093453f;
    const size_t sb = (size_t)row * P.N + w;
    float lps = 0.f;
    for (int i = 0; i < ACT_DIM; ++i) {
        const uint4 rb = rng_draw(P.seed, P.world0 + (uint32_t)w, tick, RNG_ACTION, (uint32_t)i);
        const float nz = sqrtf(-2.f * logf(u01_open(rb.x))) * cosf(6.283185307179586f * u01(rb.y));
        const float a = hd[i] + expf(ls[i]) * nz;
        lps += -0.5f * nz * nz - ls[i] - 0.5f * LOG2PI;
        P.A[sb * ACT_DIM + i] = a;
    }
    P.LP[sb] = lps;
    P.V[sb] = val;
}

// torch-ordered fp32 weights (ppo_fused.py:35-44) -> bf16 [out][in] per layer (layer 0's
// inputs padded to XK with zeros), fp32 biases; head: 29 mean rows, the value row, 2 zero
// rows; log_std.  seg: per layer {src W offset, src b offset, dst W offset, nin, nout,
// nin_pad}, the head as layer nh.
struct RepackPlan {
    int nl;
    long long srcW[MAX_HIDDEN + 1], srcB[MAX_HIDDEN + 1], dstW[MAX_HIDDEN + 1], dstB[MAX_HIDDEN + 1];
    int nin[MAX_HIDDEN + 1], nout[MAX_HIDDEN + 1], ninp[MAX_HIDDEN + 1];
    long long srcLS;
    int novalue;  // separate value network: the policy head's value row is zero
};
// fp32 policy -> split-bf16 chunk images for the in-kernel tensor-core MLP (g1_mlp_tc.cuh,
// tf_layer): per layer, ceil(nin/16) chunks of [w1 | w2 | w3] in the canonical K-major
// layout; fp32 biases; the head as 32 outputs (29 means, value, 2 zero rows); log_std [32].
__device__ __forceinline__ void tf_put(__nv_bfloat16* dst, int N, int n, int kk, float v) {
    __nv_bfloat16 p0, p1, p2;
    g1tc::split3(v, p0, p1, p2);
    const int bi = g1tc::tf_bidx(N, n, kk), per = N * g1tc::tf_kc(N);
    dst[bi] = p0;
    dst[per + bi] = p1;
    dst[2 * per + bi] = p2;
}
__global__ void k_repack_tf(const float* W, __nv_bfloat16* img, float* bias, float* LS, RepackPlan R) {
    const size_t tid = blockIdx.x * (size_t)blockDim.x + threadIdx.x, nth = (size_t)gridDim.x * blockDim.x;
    for (int l = 0; l <= R.nl; ++l) {
        const bool head = l == R.nl;
        const int nin = R.nin[l], N = head ? 32 : R.nout[l], kc = g1tc::tf_kc(N), nch = g1tc::tf_nchunk(nin, N);
        const int per = N * kc;
        for (size_t e = tid; e < (size_t)nch * per; e += nth) {
            const int c = (int)(e / per), n = (int)(e % per) / kc, kk = (int)(e % kc);
            const int k = c * kc + kk;
            float v = 0.f;
            if (k < nin) {
                if (!head || n < ACT_DIM) v = W[R.srcW[l] + (size_t)n * nin + k];
                else if (n == ACT_DIM) v = W[R.srcW[l] + (size_t)ACT_DIM * nin + ACT_DIM + k];  // Wv after bmu
            }
            tf_put(img + R.dstW[l] + (size_t)c * g1tc::tf_chunk_elems(N), N, n, kk, v);
        }
        for (size_t e = tid; e < (size_t)N; e += nth) {
            float b = 0.f;
            if (!head) b = W[R.srcB[l] + e];
            else if (e < ACT_DIM) b = W[R.srcB[l] + e];
            else if (e == ACT_DIM) b = W[R.srcB[l] + ACT_DIM + nin];  // bv
            bias[R.dstB[l] + e] = b;
        }
    }
    for (size_t e = tid; e < 32; e += nth) LS[e] = e < ACT_DIM ? W[R.srcLS + e] : 0.f;
}

// one layer W [N][K] (torch layout) -> chunk images + bias copy (the standalone test entry)
__global__ void k_tf_image_layer(const float* W, const float* b, int K, int N, __nv_bfloat16* img, float* bias) {
    const size_t tid = blockIdx.x * (size_t)blockDim.x + threadIdx.x, nth = (size_t)gridDim.x * blockDim.x;
    const int kc = g1tc::tf_kc(N), nch = g1tc::tf_nchunk(K, N), per = N * kc;
    for (size_t e = tid; e < (size_t)nch * per; e += nth) {
        const int c = (int)(e / per), n = (int)(e % per) / kc, kk = (int)(e % kc);
        const int k = c * kc + kk;
        tf_put(img + (size_t)c * g1tc::tf_chunk_elems(N), N, n, kk, k < K ? W[(size_t)n * K + k] : 0.f);
    }
    for (size_t e = tid; e < (size_t)N; e += nth) bias[e] = b ? b[e] : 0.f;
}

// separate value network: per hidden layer W, b, then the output row
// (1 x last) placed as row 29 of a 32-row head (so the value lands where the shared-trunk
// head puts it); layer 0's inputs padded to XK
__global__ void k_repack_bf16_value(const float* W, __nv_bfloat16* Wb, float* Bf, RepackPlan R) {
    const size_t tid = blockIdx.x * (size_t)blockDim.x + threadIdx.x, nth = (size_t)gridDim.x * blockDim.x;
    for (int l = 0; l <= R.nl; ++l) {
        const bool head = l == R.nl;
        const int nin = R.nin[l], ninp = R.ninp[l], nout = head ? 32 : R.nout[l];
        for (size_t e = tid; e < (size_t)nout * ninp; e += nth) {
            const int o = (int)(e / ninp), i = (int)(e % ninp);
            float v = 0.f;
            if (i < nin) {
                if (!head) v = W[R.srcW[l] + (size_t)o * nin + i];
                else if (o == ACT_DIM) v = W[R.srcW[l] + i];
            }
            Wb[R.dstW[l] + e] = __float2bfloat16(v);
        }
        for (size_t e = tid; e < (size_t)nout; e += nth) {
            float b = 0.f;
            if (!head) b = W[R.srcB[l] + e];
            else if (e == ACT_DIM) b = W[R.srcB[l]];
            Bf[R.dstB[l] + e] = b;
        }
    }
}

__global__ void k_repack_bf16(const float* W, __nv_bfloat16* Wb, float* Bf, float* LS, RepackPlan R) {
    const size_t tid = blockIdx.x * (size_t)blockDim.x + threadIdx.x, nth = (size_t)gridDim.x * blockDim.x;
    for (int l = 0; l <= R.nl; ++l) {
        const bool head = l == R.nl;
        const int nin = R.nin[l], ninp = R.ninp[l], nout = head ? 32 : R.nout[l];
        for (size_t e = tid; e < (size_t)nout * ninp; e += nth) {
            const int o = (int)(e / ninp), i = (int)(e % ninp);
            float v = 0.f;
            if (i < nin) {
                if (!head) v = W[R.srcW[l] + (size_t)o * nin + i];
                else if (o < ACT_DIM) v = W[R.srcW[l] + (size_t)o * nin + i];
                else if (o == ACT_DIM && !R.novalue) v = W[R.srcW[l] + (size_t)ACT_DIM * nin + ACT_DIM + i];  // Wv after bmu
            }
            Wb[R.dstW[l] + e] = __float2bfloat16(v);
        }
        for (size_t e = tid; e < (size_t)nout; e += nth) {
            float b = 0.f;
            if (!head) b = W[R.srcB[l] + e];
            else if (e < ACT_DIM) b = W[R.srcB[l] + e];
            else if (e == ACT_DIM && !R.novalue) b = W[R.srcB[l] + ACT_DIM + nin];  // bv
            Bf[R.dstB[l] + e] = b;
        }
    }
    for (size_t e = tid; e < 32; e += nth) LS[e] = e < ACT_DIM ? W[R.srcLS + e] : 0.f;
}

// Reset: stand pose + U(+-0.02) joint noise (k_reset, g1_env.cu:97-111); obs optional.
__global__ void k_reset(Params P, float* obs) {
    const int w = blockIdx.x * blockDim.x + threadIdx.x;
    if (w >= P.N) return;
    G1Tables const& T = c_tab;
    float* qp = P.qp + (size_t)w * NQ;
    float* qv = P.qv + (size_t)w * NV;
    float* pa = P.pa + (size_t)w * NU;
    for (int i = 0; i < NQ; ++i) qp[i] = T.qpos_stand[i];
    for (int i = 0; i < ACT_DIM; ++i) {
        uint4 rb = rng_draw(P.seed, P.world0 + (uint32_t)w, P.tick0, RNG_RESET, (uint32_t)i);
        qp[T.act_qadr[i]] += 0.02f * (u01_open(rb.x) * 2.f - 1.f);
    }
    for (int i = 0; i < NV; ++i) qv[i] = 0.f;
    for (int i = 0; i < ACT_DIM; ++i) pa[i] = 0.f;
    P.steps[w] = 0;
    if (obs)
        for (int i = 0; i < OBS_DIM; ++i) obs[(size_t)w * OBS_DIM + i] = obs_elem(i, qp, qv, pa, T);
}

// Repack the torch-ordered actor-critic weights (ppo_fused.py:35-44: per hidden layer
// W[out,in], b; Wmu, bmu, Wv, bv, log_std) into the kernel layout (per layer W^T[in][out],
// b; head W^T[nlast][32] with 29 mean rows + value row, b[32], log_std[32]).
__global__ void k_repack(const float* W, float* WT, int nh, int h0, int h1, int h2, int h3) {
    const int hid[4] = {h0, h1, h2, h3};
    size_t src = 0, dst = 0;
    int nin = OBS_DIM;
    const size_t tid = blockIdx.x * (size_t)blockDim.x + threadIdx.x, nth = (size_t)gridDim.x * blockDim.x;
    for (int l = 0; l < nh; ++l) {
        const int no = hid[l];
        for (size_t e = tid; e < (size_t)nin * no; e += nth) {
            size_t o = e / nin, i = e % nin;
            WT[dst + i * no + o] = W[src + e];
        }
        for (size_t e = tid; e < (size_t)no; e += nth) WT[dst + (size_t)nin * no + e] = W[src + (size_t)nin * no + e];
        src += (size_t)nin * no + no;
        dst += (size_t)nin * no + no;
        nin = no;
    }
    // head
    for (size_t e = tid; e < (size_t)nin * 32; e += nth) {
        size_t i = e / 32, o = e % 32;
        float v = 0.f;
        if (o < ACT_DIM) v = W[src + o * nin + i];
        else if (o == ACT_DIM) v = W[src + (size_t)ACT_DIM * nin + ACT_DIM + i];
        WT[dst + e] = v;
    }
    for (size_t e = tid; e < 32; e += nth) {
        float b = 0.f, ls = 0.f;
        if (e < ACT_DIM) { b = W[src + (size_t)ACT_DIM * nin + e]; ls = W[src + (size_t)ACT_DIM * nin + ACT_DIM + nin + 1 + e]; }
        else if (e == ACT_DIM) b = W[src + (size_t)ACT_DIM * nin + ACT_DIM + nin];
        WT[dst + (size_t)nin * 32 + e] = b;
        WT[dst + (size_t)nin * 32 + 32 + e] = ls;
    }
}

// ------------------------------------------------------------------ host side
struct EnvState {
    int N, S, pgs, device;
    float mu;
    uint64_t seed;
    uint32_t world0;
    uint64_t tick;
    float *qp, *qv, *pa;
    int* steps;
    float *dact, *dobs, *drew, *ddone;  // host-loop staging (g1_env.cu:88-89)
    float* WT;                          // repacked policy weights
    size_t WT_cap;
    int nh, hid[MAX_HIDDEN], act;
    int sm_count;
    int* ncon_hist;
    int* ncon_last;
    int prec;                           // 0: fp32 in-kernel policy, 1: bf16 tensor-core policy
    __nv_bfloat16 *Xb, *Hb[2], *Wb;     // large-policy activations and weights
    float *Bf, *LS, *HD;
    int* derr;
    size_t tc_N, tc_w, tc_wb;
    int vnh, vhid[MAX_HIDDEN];          // separate value network (bf16 path), vnh = 0: shared trunk
    __nv_bfloat16* Wvb;
    float *Bvf, *HDv;
    size_t tc_wvb, tc_hdv;
    uint8_t* tf_img;                    // fp32 policy on the tensor cores: chunk images + biases
    size_t tf_cap;
    int ffma_only;                      // 1: keep the fp32 policy on the FFMA path
    cudaStream_t stream;                // 0 = legacy default stream (the reference's)
};

static std::once_flag g_tab_once[64];
static int upload_tables(int dev) {
    int rc = 0;
    std::call_once(g_tab_once[dev & 63], [&]() {
        G1Tables T;
        g1_build_tables(&T);
        if (cudaMemcpyToSymbol(c_tab, &T, sizeof(T)) != cudaSuccess) rc = -1;
        SmemPlan p = smem_plan();
        if (cudaFuncSetAttribute(k_g1, cudaFuncAttributeMaxDynamicSharedMemorySize, p.total_bytes) != cudaSuccess) rc = -2;
        if (cudaFuncSetAttribute(k_qacc, cudaFuncAttributeMaxDynamicSharedMemorySize, p.total_bytes) != cudaSuccess) rc = -3;
        if (T.nchain > CPW) rc = -4;  // the chain-lane mapping holds at most CPW chains
        for (int c = 0; c < T.nchain; ++c)
            if (T.chain_len[c] > G1_MAXCLEN) rc = -5;  // the per-step table holds G1_MAXCLEN bodies
    });
    return rc;
}

static Params base_params(EnvState* E) {
    Params P;
    memset(&P, 0, sizeof P);
    P.N = E->N; P.S = E->S; P.pgs = E->pgs; P.mu = E->mu;
    P.qp = E->qp; P.qv = E->qv; P.pa = E->pa; P.steps = E->steps;
    P.seed = E->seed; P.world0 = E->world0; P.tick0 = E->tick;
    P.nh = E->nh; P.act = E->act;
    for (int i = 0; i < MAX_HIDDEN; ++i) P.hid[i] = E->hid[i];
    P.ncon_hist = E->ncon_hist;
    P.ncon_last = E->ncon_last;
    P.lockstep = G1_LOCKSTEP;
    P.midbar = G1_MIDBAR;
    // worlds per CTA: spread over all SMs, at most MAX_WB (then CTAs run in waves)
    int wb = (E->N + E->sm_count - 1) / E->sm_count;
    if (wb > 2 * GW * NWARPS) wb = 2 * GW * NWARPS;  // large N: blocks of two full rounds of groups
    if (wb < 1) wb = 1;
    P.wb = wb;
    return P;
}

static bool launch_g1(EnvState* E, const Params& P) {
    const int grid = (P.N + P.wb - 1) / P.wb;
    const SmemPlan plan = smem_plan();
    k_g1<<<grid, NTHREADS, plan.total_bytes, E->stream>>>(P);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) { set_error((int)e, "k_g1 launch", cudaGetErrorString(e)); return false; }
    return true;
}

static size_t policy_floats(int nh, const int* hid) {
    size_t n = 0;
    int nin = OBS_DIM;
    for (int l = 0; l < nh; ++l) { n += (size_t)nin * hid[l] + hid[l]; nin = hid[l]; }
    return n + (size_t)nin * 32 + 64;
}

// ------------------------------------------------------------------ tensor-core dense layer
// out = act(X W^T + b) on tcgen05 (g1_mlp_tc.cuh); N tiles of BN = 256 (smaller for narrow
// layers).  Asynchronous on `stream`; *err (device) is set if an MMA wait timed out.
template <int BN>
static cudaError_t launch_dense_tc(int M, int N, int K, const __nv_bfloat16* X, int ldx, const __nv_bfloat16* W,
                                   const float* bias, int act, float* of, int ldo, __nv_bfloat16* ob, int ldob, int* err,
                                   cudaStream_t stream) {
    static bool attr = false;  // per process: the attribute is per function, set before first launch
    const int smem = g1tc::dense_tc_smem<BN>();
    if (!attr) {
        cudaError_t e = cudaFuncSetAttribute(g1tc::k_dense_tc<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        attr = true;
    }
    dim3 grid((M + g1tc::TM - 1) / g1tc::TM, (N + BN - 1) / BN);
    g1tc::k_dense_tc<BN><<<grid, g1tc::NTH, smem, stream>>>(M, N, K, X, ldx, W, bias, act, of, ldo, ob, ldob, err);
    return cudaGetLastError();
}
// cuTensorMapEncodeTiled through the runtime's driver entry point (no libcuda link)
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
static EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, []() {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = (EncodeTiledFn)p;
    });
    return fn;
}

// 2-D bf16 row-major [rows][ld] tensor, box {64 columns, box_rows}, 128-byte swizzle,
// out-of-range elements read as zero
static bool make_map(CUtensorMap* m, const void* base, int cols, int rows, int ld, int box_rows) {
    EncodeTiledFn f = encode_fn();
    if (!f) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
    const cuuint32_t box[2] = {(cuuint32_t)g1gemm::BK, (cuuint32_t)box_rows};
    const cuuint32_t es[2] = {1, 1};
    return f(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, es,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int BN>
static cudaError_t launch_gemm_tma(int M, int N, int K, const __nv_bfloat16* X, int ldx, const __nv_bfloat16* W,
                                   const float* bias, int act, float* of, int ldo, __nv_bfloat16* ob, int ldob, int* err,
                                   cudaStream_t stream) {
    static int attr_dev = -1;
    int dev = 0, nsm = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
    const int smem = g1gemm::smem_bytes<BN>();
    if (attr_dev != dev) {
        cudaError_t e = cudaFuncSetAttribute(g1gemm::k_gemm<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        attr_dev = dev;
    }
    CUtensorMap mx, mw;
    if (!make_map(&mx, X, K, M, ldx, g1gemm::BM) || !make_map(&mw, W, K, N, K, BN)) return cudaErrorInvalidValue;
    const int tiles = ((M + g1gemm::BM - 1) / g1gemm::BM) * ((N + BN - 1) / BN);
    const int grid = tiles < nsm ? tiles : nsm;
    g1gemm::k_gemm<BN><<<grid, g1gemm::nth<BN>(), smem, stream>>>(mx, mw, M, N, K, bias, act, ob, of, of ? ldo : ldob, err);
    return cudaGetLastError();
}

static cudaError_t dense_tc(int M, int N, int K, const __nv_bfloat16* X, int ldx, const __nv_bfloat16* W, const float* bias,
                            int act, float* of, int ldo, __nv_bfloat16* ob, int ldob, int* err, cudaStream_t stream) {
    // TMA path: 16-byte aligned operands with 16-byte row pitches
    const bool tma = (K % 8 == 0) && (ldx % 8 == 0) && ((((uintptr_t)X) | ((uintptr_t)W)) % 16 == 0) && encode_fn();
    if (tma) {
        if (N <= 32) return launch_gemm_tma<32>(M, N, K, X, ldx, W, bias, act, of, ldo, ob, ldob, err, stream);
        if (N <= 64) return launch_gemm_tma<64>(M, N, K, X, ldx, W, bias, act, of, ldo, ob, ldob, err, stream);
        if (N <= 128) return launch_gemm_tma<128>(M, N, K, X, ldx, W, bias, act, of, ldo, ob, ldob, err, stream);
        return launch_gemm_tma<256>(M, N, K, X, ldx, W, bias, act, of, ldo, ob, ldob, err, stream);
    }
    if (N <= 32) return launch_dense_tc<32>(M, N, K, X, ldx, W, bias, act, of, ldo, ob, ldob, err, stream);
    if (N <= 64) return launch_dense_tc<64>(M, N, K, X, ldx, W, bias, act, of, ldo, ob, ldob, err, stream);
    return launch_dense_tc<256>(M, N, K, X, ldx, W, bias, act, of, ldo, ob, ldob, err, stream);
}

// The large-policy rollout: per control step obs -> tcgen05 layers -> sampling -> physics.
static void rollout_tc(EnvState* E, int H, const float* W, const float* mean, const float* var, float* O, float* A,
                       float* LP, float* V, float* R, float* D, float* Vlast) {
    const int N = E->N, nh = E->nh;
    int maxw = 32;
    for (int l = 0; l < nh; ++l) maxw = E->hid[l] > maxw ? E->hid[l] : maxw;
    RepackPlan RP;
    memset(&RP, 0, sizeof RP);
    RP.nl = nh;
    long long src = 0, dw = 0, db = 0;
    int nin = OBS_DIM;
    for (int l = 0; l <= nh; ++l) {
        const bool head = l == nh;
        const int no = head ? 32 : E->hid[l];
        RP.srcW[l] = src; RP.nin[l] = nin; RP.ninp[l] = l == 0 ? XK : nin; RP.nout[l] = no;
        RP.srcB[l] = src + (long long)(head ? ACT_DIM : no) * nin;
        RP.dstW[l] = dw; RP.dstB[l] = db;
        dw += (long long)no * RP.ninp[l];
        db += no;
        if (!head) { src += (long long)nin * no + no; nin = no; }
    }
    // separate value network: the policy part ends [.. Wmu, bmu, log_std], the value
    // network's layers and its 1-row output follow (g1env.pack_weights with value_hidden)
    const bool vnet = E->vnh > 0;
    RP.novalue = vnet;
    RP.srcLS = vnet ? src + (long long)ACT_DIM * nin + ACT_DIM : src + (long long)ACT_DIM * nin + ACT_DIM + nin + 1;
    RepackPlan VP;
    memset(&VP, 0, sizeof VP);
    long long vdw = 0, vdb = 0;
    if (vnet) {
        long long vs = RP.srcLS + ACT_DIM;
        int vin = OBS_DIM;
        VP.nl = E->vnh;
        for (int l = 0; l <= E->vnh; ++l) {
            const bool head = l == E->vnh;
            const int no = head ? 32 : E->vhid[l];
            VP.srcW[l] = vs; VP.nin[l] = vin; VP.ninp[l] = l == 0 ? XK : vin; VP.nout[l] = no;
            VP.srcB[l] = vs + (long long)(head ? 1 : no) * vin;
            VP.dstW[l] = vdw; VP.dstB[l] = vdb;
            vdw += (long long)no * VP.ninp[l];
            vdb += no;
            if (!head) { vs += (long long)vin * no + no; vin = no; }
            if (E->vhid[l] > maxw && !head) maxw = E->vhid[l];
        }
        if (E->tc_wvb < (size_t)vdw || E->tc_hdv < (size_t)N) {
            cudaFree(E->Wvb); cudaFree(E->Bvf); cudaFree(E->HDv);
            E->Wvb = nullptr; E->Bvf = nullptr; E->HDv = nullptr; E->tc_wvb = 0; E->tc_hdv = 0;
            CKR(cudaMalloc(&E->Wvb, (size_t)vdw * 2), );
            CKR(cudaMalloc(&E->Bvf, (size_t)vdb * 4), );
            CKR(cudaMalloc(&E->HDv, (size_t)N * 32 * 4), );
            E->tc_wvb = vdw; E->tc_hdv = N;
        }
    }
    // buffers (allocated on first use, kept by the env)
    if (E->tc_N < (size_t)N || E->tc_w < (size_t)maxw) {
        cudaFree(E->Xb); cudaFree(E->Hb[0]); cudaFree(E->Hb[1]); cudaFree(E->HD);
        E->Xb = E->Hb[0] = E->Hb[1] = nullptr; E->HD = nullptr;
        CKR(cudaMalloc(&E->Xb, (size_t)N * XK * 2), );
        CKR(cudaMalloc(&E->Hb[0], (size_t)N * maxw * 2), );
        CKR(cudaMalloc(&E->Hb[1], (size_t)N * maxw * 2), );
        CKR(cudaMalloc(&E->HD, (size_t)N * 32 * 4), );
        E->tc_N = N; E->tc_w = maxw;
    }
    if (E->tc_wb < (size_t)dw) {
        cudaFree(E->Wb); cudaFree(E->Bf); cudaFree(E->LS);
        CKR(cudaMalloc(&E->Wb, (size_t)dw * 2), );
        CKR(cudaMalloc(&E->Bf, (size_t)db * 4), );
        CKR(cudaMalloc(&E->LS, 32 * 4), );
        E->tc_wb = dw;
    }
    if (!E->derr) { CKR(cudaMalloc(&E->derr, sizeof(int)), ); CKR(cudaMemset(E->derr, 0, sizeof(int)), ); }
    k_repack_bf16<<<240, 256, 0, E->stream>>>(W, E->Wb, E->Bf, E->LS, RP);
    CKR(cudaGetLastError(), );
    if (vnet) {
        k_repack_bf16_value<<<240, 256, 0, E->stream>>>(W, E->Wvb, E->Bvf, VP);
        CKR(cudaGetLastError(), );
    }
    Params P = base_params(E);
    P.mode = MODE_ROLLOUT; P.H = 1; P.ext_policy = 1;
    P.mean = mean; P.var = var;
    P.O = O; P.A = A; P.LP = LP; P.V = V; P.R = R; P.D = D; P.Vlast = Vlast;
    P.o_vec = ((uintptr_t)O & 15) == 0;
    const dim3 oblk(32, 8);
    const int ogrid = (N + 7) / 8;
    auto policy = [&](int row, uint64_t tick) -> bool {
        k_obs_norm<<<ogrid, oblk, 0, E->stream>>>(P, row, E->Xb);
        if (cudaGetLastError() != cudaSuccess) return false;
        const __nv_bfloat16* in = E->Xb;
        int k = XK;
        for (int l = 0; l < nh; ++l) {
            __nv_bfloat16* out = E->Hb[l & 1];
            cudaError_t e = dense_tc(N, E->hid[l], k, in, k, E->Wb + RP.dstW[l], E->Bf + RP.dstB[l], E->act, nullptr, 0,
                                     out, E->hid[l], E->derr, E->stream);
            if (e != cudaSuccess) { set_error((int)e, "rollout_tc", cudaGetErrorString(e)); return false; }
            in = out;
            k = E->hid[l];
        }
        cudaError_t e = dense_tc(N, 32, k, in, k, E->Wb + RP.dstW[nh], E->Bf + RP.dstB[nh], -1, E->HD, 32, nullptr, 0,
                                 E->derr, E->stream);
        if (e != cudaSuccess) { set_error((int)e, "rollout_tc", cudaGetErrorString(e)); return false; }
        if (vnet) {  // value network on the same normalised observations
            in = E->Xb;
            k = XK;
            for (int l = 0; l < E->vnh; ++l) {
                __nv_bfloat16* out = E->Hb[l & 1];
                e = dense_tc(N, E->vhid[l], k, in, k, E->Wvb + VP.dstW[l], E->Bvf + VP.dstB[l], E->act, nullptr, 0, out,
                             E->vhid[l], E->derr, E->stream);
                if (e != cudaSuccess) { set_error((int)e, "rollout_tc", cudaGetErrorString(e)); return false; }
                in = out;
                k = E->vhid[l];
            }
            e = dense_tc(N, 32, k, in, k, E->Wvb + VP.dstW[E->vnh], E->Bvf + VP.dstB[E->vnh], -1, E->HDv, 32, nullptr, 0,
                         E->derr, E->stream);
            if (e != cudaSuccess) { set_error((int)e, "rollout_tc", cudaGetErrorString(e)); return false; }
        }
        k_sample<<<(N + 127) / 128, 128, 0, E->stream>>>(P, row, E->HD, vnet ? E->HDv : E->HD, E->LS, tick);
        return cudaGetLastError() == cudaSuccess;
    };
    for (int t = 0; t < H; ++t) {
        const uint64_t tick = E->tick + (uint64_t)t;
        if (!policy(t, tick)) { set_error(-1, "rollout_tc", "policy launch failed"); return; }
        P.t0 = t; P.tick0 = tick;
        if (!launch_g1(E, P)) return;
    }
    P.tick0 = E->tick + (uint64_t)H;
    if (!policy(-1, 0)) { set_error(-1, "rollout_tc", "policy launch failed"); return; }
    E->tick += (uint64_t)H;
}

// Device error flag of the tensor-core path (a timed-out MMA wait); read and cleared.
static int tc_error(EnvState* E) {
    if (!E->derr) return 0;
    int herr = 0;
    if (cudaMemcpy(&herr, E->derr, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return -1;
    if (herr) cudaMemset(E->derr, 0, sizeof(int));
    return herr;
}

// Test entry (not part of the public header): runs k_wait_probe on the env's stream with a
// spin limit of `spin_limit` iterations; the timed-out wait is reported through the same
// device flag as the rollout's, read with g1_env_tc_status.  Returns the CUDA status.
extern "C" int g1_env_test_wait_timeout(void* h, unsigned spin_limit) {
    EnvState* E = (EnvState*)h;
    if (!E->derr) {
        CKR(cudaMalloc(&E->derr, sizeof(int)), -1);
        CKR(cudaMemset(E->derr, 0, sizeof(int)), -1);
    }
    g1tc::k_wait_probe<<<1, 224, 0, E->stream>>>(E->derr, spin_limit);
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) e = cudaStreamSynchronize(E->stream);
    if (e != cudaSuccess) set_error((int)e, "g1_env_test_wait_timeout", cudaGetErrorString(e));
    return (int)e;
}

// ------------------------------------------------------------------ allocation-free rollout
// g1_rollout repacks the policy weights into a buffer the env allocates on first use (and
// reallocates when the policy grows).  g1_rollout_noalloc keeps that repacked copy in this
// fixed device array instead, so it never allocates.  Every GPU that loads the library holds
// the array until the process exits.  All calls share it: each call rewrites the part it
// uses before reading it, and calls that overlap on the GPU (other streams, other threads)
// race on it.
#define G1_NOALLOC_WT_FLOATS (128 * 1024)  // 512 KiB: fits the reference's 100-256-256 policy (99,904 floats)
static __device__ __align__(256) float g_noalloc_wt[G1_NOALLOC_WT_FLOATS];
static std::mutex g_noalloc_mu;
static float* g_noalloc_ptr[64];  // device address of g_noalloc_wt, per device ordinal

// Device address of the static weight area on device `dev`, looked up once per device
// (cudaGetSymbolAddress; the host-side name g_noalloc_wt is not a device address).  The
// symbol resolves on the CURRENT device, so the lookup makes `dev` current for its duration
// and restores the caller's device afterwards.
static float* noalloc_area(int dev) {
    if (dev < 0 || dev >= 64) { set_error(-22, "g1_rollout_noalloc", "device ordinal out of range"); return nullptr; }
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
        int prev = -1;
        CKR(cudaGetDevice(&prev), nullptr);
        if (prev != dev) CKR(cudaSetDevice(dev), nullptr);
        float* ptr = nullptr;
        const cudaError_t e = cudaGetSymbolAddress((void**)&ptr, g_noalloc_wt);
        if (prev != dev) cudaSetDevice(prev);
        if (e != cudaSuccess) { set_error((int)e, "g1_rollout_noalloc", cudaGetErrorString(e)); return nullptr; }
        g_noalloc_ptr[dev] = ptr;
    }
    return g_noalloc_ptr[dev];
}

extern "C" {

const char* g1_env_last_error(void) {
    std::lock_guard<std::mutex> lk(g_err_mu);
    return g_last_code ? g_last_error.c_str() : nullptr;
}
int g1_env_last_error_code(void) { return g_last_code; }
void g1_env_clear_error(void) {
    std::lock_guard<std::mutex> lk(g_err_mu);
    g_last_code = 0;
    g_last_error.clear();
}

int g1_env_obs_dim(void) { return OBS_DIM; }
int g1_env_act_dim(void) { return ACT_DIM; }

void* g1_env_create_ex(int N, int substeps, int pgs_iters, unsigned long seed, int device, unsigned int world0, float mu) {
    if (N <= 0 || substeps <= 0 || pgs_iters < 0) { set_error(-22, "g1_env_create", "invalid argument"); return nullptr; }
    if (device >= 0) CKR(cudaSetDevice(device), nullptr);
    int dev = 0;
    CKR(cudaGetDevice(&dev), nullptr);
    if (upload_tables(dev) != 0) { set_error(-1, "g1_env_create", "table upload / smem attribute failed"); return nullptr; }
    EnvState* E = new EnvState();
    memset(E, 0, sizeof *E);
    E->N = N; E->S = substeps; E->pgs = pgs_iters; E->device = dev; E->seed = seed; E->world0 = world0; E->mu = mu;
    E->nh = 2; E->hid[0] = 256; E->hid[1] = 256; E->act = 0;  // the reference's AC (ppo.py:85-99)
    cudaDeviceGetAttribute(&E->sm_count, cudaDevAttrMultiProcessorCount, dev);
    bool ok = cudaMalloc(&E->qp, (size_t)N * NQ * 4) == cudaSuccess && cudaMalloc(&E->qv, (size_t)N * NV * 4) == cudaSuccess &&
              cudaMalloc(&E->pa, (size_t)N * NU * 4) == cudaSuccess && cudaMalloc(&E->steps, (size_t)N * 4) == cudaSuccess &&
              cudaMalloc(&E->dact, (size_t)N * ACT_DIM * 4) == cudaSuccess &&
              cudaMalloc(&E->dobs, (size_t)N * OBS_DIM * 4) == cudaSuccess && cudaMalloc(&E->drew, (size_t)N * 4) == cudaSuccess &&
              cudaMalloc(&E->ddone, (size_t)N * 4) == cudaSuccess && cudaMalloc(&E->ncon_last, (size_t)N * 4) == cudaSuccess &&
              cudaMemset(E->ncon_last, 0, (size_t)N * 4) == cudaSuccess;
    if (!ok) {
        set_error(2, "g1_env_create", "cudaMalloc failed");
        cudaFree(E->qp); cudaFree(E->qv); cudaFree(E->pa); cudaFree(E->steps);
        cudaFree(E->dact); cudaFree(E->dobs); cudaFree(E->drew); cudaFree(E->ddone); cudaFree(E->ncon_last);
        delete E;
        return nullptr;
    }
    // a valid state before the first reset: the stand pose without noise
    Params P = base_params(E);
    k_reset<<<(N + 127) / 128, 128>>>(P, nullptr);
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) { set_error((int)e, "g1_env_create", cudaGetErrorString(e)); }
    return E;
}

// g1_env.cu:405-422
void* g1_env_create(int N, int substeps, int pgs_iters, unsigned long seed) {
    return g1_env_create_ex(N, substeps, pgs_iters, seed, -1, 0u, G1M_FOOT_MU_MODEL);
}

void g1_env_destroy(void* h) {  // g1_env.cu:469-474
    EnvState* E = (EnvState*)h;
    if (!E) return;
    cudaFree(E->qp); cudaFree(E->qv); cudaFree(E->pa); cudaFree(E->steps);
    cudaFree(E->dact); cudaFree(E->dobs); cudaFree(E->drew); cudaFree(E->ddone);
    cudaFree(E->WT); cudaFree(E->ncon_hist); cudaFree(E->ncon_last);
    cudaFree(E->Xb); cudaFree(E->Hb[0]); cudaFree(E->Hb[1]); cudaFree(E->Wb); cudaFree(E->Bf); cudaFree(E->LS);
    cudaFree(E->HD); cudaFree(E->derr); cudaFree(E->tf_img); cudaFree(E->Wvb); cudaFree(E->Bvf); cudaFree(E->HDv);
    delete E;
}

void g1_env_set_stream(void* h, void* stream) { ((EnvState*)h)->stream = (cudaStream_t)stream; }

int g1_env_set_policy(void* h, int nh, const int* hidden, int activation) {
    EnvState* E = (EnvState*)h;
    if (nh < 1 || nh > MAX_HIDDEN || activation < 0 || activation > 1) { set_error(-22, "g1_env_set_policy", "invalid"); return -22; }
    for (int i = 0; i < nh; ++i)
        if (hidden[i] < 4 || hidden[i] > 1024 || (hidden[i] & 3)) { set_error(-22, "g1_env_set_policy", "bad width"); return -22; }
    // MLP activations for MAX_WB worlds must fit in the physics frames it aliases
    int maxw = 0;
    for (int i = 0; i < nh; ++i) maxw = hidden[i] > maxw ? hidden[i] : maxw;
    size_t need = (size_t)MAX_WB * XSTR + 2 * (size_t)MAX_WB * (((maxw + 3) & ~3) + 4) + KT * OC;
    if (need > (size_t)NWARPS * GROUP_FLOATS) { set_error(-22, "g1_env_set_policy", "hidden width too large for this build"); return -22; }
    E->nh = nh; E->act = activation;
    for (int i = 0; i < MAX_HIDDEN; ++i) E->hid[i] = i < nh ? hidden[i] : 0;
    return 0;
}

// extension: policy precision 1 runs the MLP on the tensor cores in bf16 (fp32 accumulation)
// as separate launches per control step; widths multiple of 8, up to 1024.
int g1_env_set_policy_ex(void* h, int nh, const int* hidden, int activation, int precision) {
    EnvState* E = (EnvState*)h;
    if (precision == 0 || precision == 2) {  // fp32: tensor cores (3xTF32) where eligible / FFMA only
        int rc = g1_env_set_policy(h, nh, hidden, activation);
        if (rc == 0) { E->prec = 0; E->ffma_only = precision == 2; }
        return rc;
    }
    if (precision != 1 || nh < 1 || nh > MAX_HIDDEN || activation < 0 || activation > 1) {
        set_error(-22, "g1_env_set_policy_ex", "invalid");
        return -22;
    }
    for (int i = 0; i < nh; ++i)
        if (hidden[i] < 8 || hidden[i] > 1024 || (hidden[i] & 7)) {
            set_error(-22, "g1_env_set_policy_ex", "bf16 widths must be multiples of 8 in [8, 1024]");
            return -22;
        }
    E->nh = nh; E->act = activation; E->prec = 1;
    for (int i = 0; i < MAX_HIDDEN; ++i) E->hid[i] = i < nh ? hidden[i] : 0;
    return 0;
}

// extension: a separate value network of nh hidden layers (widths
// multiples of 8 in [8, 1024], the policy's activation) on the tensor-core policy path;
// nh = 0 returns to the shared trunk's value head.  Returns 0 on success.
int g1_env_set_value_net(void* h, int nh, const int* hidden) {
    EnvState* E = (EnvState*)h;
    if (nh < 0 || nh > MAX_HIDDEN) { set_error(-22, "g1_env_set_value_net", "invalid"); return -22; }
    for (int i = 0; i < nh; ++i)
        if (hidden[i] < 8 || hidden[i] > 1024 || (hidden[i] & 7)) {
            set_error(-22, "g1_env_set_value_net", "widths must be multiples of 8 in [8, 1024]");
            return -22;
        }
    E->vnh = nh;
    for (int i = 0; i < MAX_HIDDEN; ++i) E->vhid[i] = i < nh ? hidden[i] : 0;
    return 0;
}

void g1_env_set_friction(void* h, float mu) { ((EnvState*)h)->mu = mu; }

// g1_env.cu:424-429 (host obs_out [N x 100], synchronous)
void g1_env_reset(void* h, float* obs_out) {
    EnvState* E = (EnvState*)h;
    Params P = base_params(E);
    k_reset<<<(E->N + 127) / 128, 128, 0, E->stream>>>(P, E->dobs);
    CKR(cudaGetLastError(), );
    if (obs_out) CKR(cudaMemcpyAsync(obs_out, E->dobs, (size_t)E->N * OBS_DIM * 4, cudaMemcpyDeviceToHost, E->stream), );
    CKR(cudaStreamSynchronize(E->stream), );
}

// g1_env.cu:431-441 (host pointers; synchronous).  Advances the control tick.
void g1_env_step(void* h, const float* act, float* obs, float* rew, float* done) {
    EnvState* E = (EnvState*)h;
    CKR(cudaMemcpyAsync(E->dact, act, (size_t)E->N * ACT_DIM * 4, cudaMemcpyHostToDevice, E->stream), );
    Params P = base_params(E);
    P.mode = MODE_STEP;
    P.act_in = E->dact; P.obs_out = E->dobs; P.rew_out = E->drew; P.done_out = E->ddone;
    if (!launch_g1(E, P)) return;
    E->tick += 1;
    CKR(cudaMemcpyAsync(obs, E->dobs, (size_t)E->N * OBS_DIM * 4, cudaMemcpyDeviceToHost, E->stream), );
    CKR(cudaMemcpyAsync(rew, E->drew, (size_t)E->N * 4, cudaMemcpyDeviceToHost, E->stream), );
    CKR(cudaMemcpyAsync(done, E->ddone, (size_t)E->N * 4, cudaMemcpyDeviceToHost, E->stream), );
    CKR(cudaStreamSynchronize(E->stream), );
}

// Device-pointer variant of g1_env_step (no host copies, asynchronous on the env stream).
void g1_env_step_device(void* h, const float* act, float* obs, float* rew, float* done) {
    EnvState* E = (EnvState*)h;
    Params P = base_params(E);
    P.mode = MODE_STEP;
    P.act_in = act; P.obs_out = obs; P.rew_out = rew; P.done_out = done;
    if (launch_g1(E, P)) E->tick += 1;
}

// g1_env.cu:446-453: the fused rollout into caller-owned DEVICE buffers, asynchronous.
// The fp32 policy runs on the tensor cores (3xTF32) when every hidden width is a multiple of
// 16 in [16, 256]; other widths, or ffma_only, keep the FFMA path.
static bool tf_eligible(const EnvState* E) {
    if (E->ffma_only || E->nh < 1) return false;
    for (int l = 0; l < E->nh; ++l)
        if (E->hid[l] < 16 || E->hid[l] > 256 || (E->hid[l] & 15)) return false;
    return true;
}

// Builds the chunk images of W (k_repack_tf, on the env stream) and fills the tensor-core
// fields of P.  Returns false (error set) on allocation failure.
static bool prepare_tf(EnvState* E, const float* W, Params& P) {
    RepackPlan RP;
    memset(&RP, 0, sizeof RP);
    RP.nl = E->nh;
    long long src = 0, dw = 0;
    int db = 0, nin = OBS_DIM;
    for (int l = 0; l <= E->nh; ++l) {
        const bool head = l == E->nh;
        const int no = head ? 32 : E->hid[l];
        RP.srcW[l] = src; RP.nin[l] = nin; RP.nout[l] = no;
        RP.srcB[l] = src + (long long)(head ? ACT_DIM : no) * nin;
        RP.dstW[l] = dw; RP.dstB[l] = db;
        P.tf_woff[l] = dw; P.tf_boff[l] = db;
        dw += (long long)g1tc::tf_nchunk(nin, no) * g1tc::tf_chunk_elems(no);
        db += no;
        if (!head) { src += (long long)nin * no + no; nin = no; }
    }
    RP.srcLS = src + (long long)ACT_DIM * nin + ACT_DIM + nin + 1;
    const size_t img_bytes = ((size_t)dw * 2 + 255) & ~(size_t)255;
    const size_t need = img_bytes + ((size_t)db + 32) * 4;
    if (need > E->tf_cap) {
        cudaFree(E->tf_img);
        E->tf_img = nullptr;
        E->tf_cap = 0;
        CKR(cudaMalloc(&E->tf_img, need), false);
        E->tf_cap = need;
    }
    if (!E->derr) {
        CKR(cudaMalloc(&E->derr, sizeof(int)), false);
        CKR(cudaMemset(E->derr, 0, sizeof(int)), false);
    }
    __nv_bfloat16* img = reinterpret_cast<__nv_bfloat16*>(E->tf_img);
    float* bias = reinterpret_cast<float*>(E->tf_img + img_bytes);
    k_repack_tf<<<148, 256, 0, E->stream>>>(W, img, bias, bias + db, RP);
    CKR(cudaGetLastError(), false);
    P.tf_mlp = 1;
    P.tf_img = img;
    P.tf_bias = bias;
    P.tf_lsoff = db;
    P.tf_err = E->derr;
    return true;
}

void g1_rollout(void* h, int H, const float* W, const float* mean, const float* var, float* O, float* A, float* LP,
                float* V, float* R, float* D, float* Vlast) {
    EnvState* E = (EnvState*)h;
    if (H <= 0) return;
    if (E->prec == 1) {
        rollout_tc(E, H, W, mean, var, O, A, LP, V, R, D, Vlast);
        return;
    }
    if (E->vnh > 0) {
        set_error(-22, "g1_rollout", "a separate value network needs the tensor-core policy (precision 1)");
        return;
    }
    size_t need = policy_floats(E->nh, E->hid);
    if (need > E->WT_cap) {
        cudaFree(E->WT);
        E->WT = nullptr;
        CKR(cudaMalloc(&E->WT, need * 4), );
        E->WT_cap = need;
    }
    Params P = base_params(E);
    if (tf_eligible(E)) {
        if (!prepare_tf(E, W, P)) return;
    } else {
        k_repack<<<120, 256, 0, E->stream>>>(W, E->WT, E->nh, E->hid[0], E->hid[1], E->hid[2], E->hid[3]);
        CKR(cudaGetLastError(), );
    }
    P.mode = MODE_ROLLOUT; P.H = H;
    P.WT = E->WT; P.mean = mean; P.var = var;
    P.O = O; P.A = A; P.LP = LP; P.V = V; P.R = R; P.D = D; P.Vlast = Vlast;
    P.o_vec = ((uintptr_t)O & 15) == 0;
    if (launch_g1(E, P)) E->tick += (uint64_t)H;
}

// Same as g1_rollout, but allocates nothing: the repacked policy weights go to the fixed
// device area g_noalloc_wt (G1_NOALLOC_WT_FLOATS floats) instead of an env-owned buffer.
// Rejects a policy whose repacked size exceeds that area.  The first call on a device looks
// up the area's device address; make that first call before any stream capture.
void g1_rollout_noalloc(void* h, int H, const float* W, const float* mean, const float* var, float* O, float* A,
                        float* LP, float* V, float* R, float* D, float* Vlast) {
    EnvState* E = (EnvState*)h;
    if (H <= 0) return;
    // only the in-kernel FFMA policy path reads its weights from this area: the bf16
    // tensor-core policy (precision 1) and a separate value network keep env-owned buffers
    if (E->prec == 1 || E->vnh > 0) {
        set_error(-22, "g1_rollout_noalloc", "supports the fp32 in-kernel policy only (not precision 1, not a separate value network)");
        return;
    }
    const size_t need = policy_floats(E->nh, E->hid);
    if (need > (size_t)G1_NOALLOC_WT_FLOATS) {
        char msg[160];
        snprintf(msg, sizeof msg, "policy needs %zu floats of repacked weights; the static area holds %d", need,
                 G1_NOALLOC_WT_FLOATS);
        set_error(-22, "g1_rollout_noalloc", msg);
        return;
    }
    float* wt = noalloc_area(E->device);
    if (!wt) return;
    // k_repack writes all `need` floats of the area, so no clearing is needed
    k_repack<<<120, 256, 0, E->stream>>>(W, wt, E->nh, E->hid[0], E->hid[1], E->hid[2], E->hid[3]);
    CKR(cudaGetLastError(), );
    Params P = base_params(E);
    P.mode = MODE_ROLLOUT; P.H = H;
    P.WT = wt; P.mean = mean; P.var = var;
    P.O = O; P.A = A; P.LP = LP; P.V = V; P.R = R; P.D = D; P.Vlast = Vlast;
    P.o_vec = ((uintptr_t)O & 15) == 0;
    if (launch_g1(E, P)) E->tick += (uint64_t)H;
}

// g1_env.cu:385-389: K control steps with zero action, synchronous.
void g1_env_bench_phys(void* h, int K) {
    EnvState* E = (EnvState*)h;
    if (K <= 0) return;
    Params P = base_params(E);
    P.mode = MODE_PHYS; P.K = K;
    if (!launch_g1(E, P)) return;
    E->tick += (uint64_t)K;
    CKR(cudaStreamSynchronize(E->stream), );
}

// extension: K control steps of physics only with a constant action per
// world, act = DEVICE [N, 29] (null = zero, as g1_env_bench_phys); asynchronous on the env
// stream.  The actions go through the same PD-target path as the rollout's.
void g1_env_phys_actions(void* h, int K, const float* act) {
    EnvState* E = (EnvState*)h;
    if (K <= 0) return;
    Params P = base_params(E);
    P.mode = MODE_PHYS; P.K = K; P.act_in = act;
    if (launch_g1(E, P)) E->tick += (uint64_t)K;
}

// Asynchronous variant of g1_env_bench_phys (for timing with events on the env stream).
void g1_env_phys_async(void* h, int K) {
    EnvState* E = (EnvState*)h;
    if (K <= 0) return;
    Params P = base_params(E);
    P.mode = MODE_PHYS; P.K = K;
    if (launch_g1(E, P)) E->tick += (uint64_t)K;
}

// g1_env.cu:457-467
void g1_env_qpos(void* h, float* out) {
    EnvState* E = (EnvState*)h;
    CKR(cudaMemcpyAsync(out, E->qp, (size_t)NQ * 4, cudaMemcpyDeviceToHost, E->stream), );
    CKR(cudaStreamSynchronize(E->stream), );
}
void g1_env_qpos_all(void* h, float* out) {
    EnvState* E = (EnvState*)h;
    CKR(cudaMemcpyAsync(out, E->qp, (size_t)E->N * NQ * 4, cudaMemcpyDeviceToHost, E->stream), );
    CKR(cudaStreamSynchronize(E->stream), );
}

// Host state access (for checkpoint/parity): qp [N*36], qv [N*35], pa [N*29] float,
// steps [N] int, tick.  Any pointer may be null.  Synchronous.
void g1_env_get_state(void* h, float* qp, float* qv, float* pa, int* steps, unsigned long long* tick) {
    EnvState* E = (EnvState*)h;
    if (qp) CKR(cudaMemcpyAsync(qp, E->qp, (size_t)E->N * NQ * 4, cudaMemcpyDeviceToHost, E->stream), );
    if (qv) CKR(cudaMemcpyAsync(qv, E->qv, (size_t)E->N * NV * 4, cudaMemcpyDeviceToHost, E->stream), );
    if (pa) CKR(cudaMemcpyAsync(pa, E->pa, (size_t)E->N * NU * 4, cudaMemcpyDeviceToHost, E->stream), );
    if (steps) CKR(cudaMemcpyAsync(steps, E->steps, (size_t)E->N * 4, cudaMemcpyDeviceToHost, E->stream), );
    CKR(cudaStreamSynchronize(E->stream), );
    if (tick) *tick = E->tick;
}
void g1_env_set_state(void* h, const float* qp, const float* qv, const float* pa, const int* steps, unsigned long long tick) {
    EnvState* E = (EnvState*)h;
    if (qp) CKR(cudaMemcpyAsync(E->qp, qp, (size_t)E->N * NQ * 4, cudaMemcpyHostToDevice, E->stream), );
    if (qv) CKR(cudaMemcpyAsync(E->qv, qv, (size_t)E->N * NV * 4, cudaMemcpyHostToDevice, E->stream), );
    if (pa) CKR(cudaMemcpyAsync(E->pa, pa, (size_t)E->N * NU * 4, cudaMemcpyHostToDevice, E->stream), );
    if (steps) CKR(cudaMemcpyAsync(E->steps, steps, (size_t)E->N * 4, cudaMemcpyHostToDevice, E->stream), );
    CKR(cudaStreamSynchronize(E->stream), );
    E->tick = tick;
}

// Contact-count histogram over all substeps since enabled (ncon 0..8), for the roofline
// FLOP tally.  enable=1 allocates/zeroes, enable=0 disables.  out[9] host.
void g1_env_ncon_hist(void* h, int enable, unsigned long long* out) {
    EnvState* E = (EnvState*)h;
    if (out && E->ncon_hist) {
        int tmp[MAXCON + 1];
        CKR(cudaMemcpyAsync(tmp, E->ncon_hist, sizeof tmp, cudaMemcpyDeviceToHost, E->stream), );
        CKR(cudaStreamSynchronize(E->stream), );
        for (int i = 0; i <= MAXCON; ++i) out[i] = (unsigned long long)tmp[i];
    }
    if (enable) {
        if (!E->ncon_hist) CKR(cudaMalloc(&E->ncon_hist, (MAXCON + 1) * sizeof(int)), );
        CKR(cudaMemsetAsync(E->ncon_hist, 0, (MAXCON + 1) * sizeof(int), E->stream), );
    } else if (E->ncon_hist) {
        cudaFree(E->ncon_hist);
        E->ncon_hist = nullptr;
    }
}

// Per-state FK + generalized acceleration on DEVICE buffers (the per-substep parity gate;
// test_envqacc.cu:29-51 semantics with caller states).  Outputs may be null.  Synchronous.
int g1_qacc_batch(int n, const float* qpos, const float* qvel, const float* tau, const float* bdt, int pgs_iters, float mu,
                  float* qacc, float* qacc_smooth, float* bias, float* f, int* ncon) {
    int dev = 0;
    CKR(cudaGetDevice(&dev), -1);
    if (upload_tables(dev) != 0) { set_error(-1, "g1_qacc_batch", "table upload failed"); return -1; }
    int sms = 148;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const SmemPlan plan = smem_plan();
    int grid = (n + NWARPS - 1) / NWARPS;
    if (grid > sms * 4) grid = sms * 4;
    if (grid < 1) grid = 1;
    k_qacc<<<grid, NTHREADS, plan.total_bytes>>>(n, qpos, qvel, tau, bdt, pgs_iters, mu, qacc, qacc_smooth, bias, f, ncon);
    CKR(cudaGetLastError(), -1);
    CKR(cudaDeviceSynchronize(), -1);
    return 0;
}

#ifdef G1_PROF
// profiling builds only (-DG1_PROF, not part of the shipped ABI): per-phase warp cycles
// since the last call (64 counters: phases from 0, contact batches by size at 48..55).
int g1_prof_read(unsigned long long* out) {
    CKR(cudaDeviceSynchronize(), -1);
    CKR(cudaMemcpyFromSymbol(out, g_prof, sizeof(unsigned long long) * 64), -1);
    unsigned long long z[64] = {0};
    CKR(cudaMemcpyToSymbol(g_prof, z, sizeof z), -1);
    return 0;
}
#endif

// extension: one dense layer out = act(X W^T + b) on the tensor cores (tcgen05, bf16 inputs,
// fp32 accumulation).  DEVICE pointers: X [M][K] bf16 (row stride ldx), W [N][K] bf16, bias
// [N] f32 (may be null), out [M][N] f32.  act: 0 tanh, 1 ELU, -1 identity.  Synchronous;
// returns 0, or nonzero with the last error set.
// extension (test entry of the in-kernel fp32 policy layer): out = act(X W^T + b) for
// rows <= 64, N % 16 == 0, N <= 256, K <= 256, with the split-bf16 tensor-core layer the
// fused rollout uses (one CTA).  DEVICE pointers X [rows][K], W [N][K], b [N] (may be null),
// out [rows][N]; act 0 tanh, 1 ELU, -1 identity; synchronous; 0 on success.
int g1_dense_bf16x3(int rows, int K, int N, const float* X, const float* W, const float* b, int act, float* out) {
    if (rows < 1 || rows > g1tc::TF_ROWS || K < 1 || K > g1tc::TF_KMAX || N < 16 || N > 256 || (N & 15) || act < -1 ||
        act > 1) {
        set_error(-22, "g1_dense_bf16x3", "invalid shape");
        return -22;
    }
    const int nch = g1tc::tf_nchunk(K, N);
    __nv_bfloat16* img = nullptr;
    float* bias = nullptr;
    int* derr = nullptr;
    CKR(cudaMalloc(&img, (size_t)nch * g1tc::tf_chunk_elems(N) * 2), -1);
    CKR(cudaMalloc(&bias, (size_t)N * 4), -1);
    CKR(cudaMalloc(&derr, sizeof(int)), -1);
    CKR(cudaMemset(derr, 0, sizeof(int)), -1);
    k_tf_image_layer<<<64, 256>>>(W, b, K, N, img, bias);
    const int smem = g1tc::tf_test_smem();
    // identity on a wide layer goes through the hidden-layer epilogue (act 2)
    const int kact = (act < 0 && N > 32) ? 2 : act;
    cudaError_t e = cudaFuncSetAttribute(g1tc::k_tf_layer_test<224>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e == cudaSuccess) {
        g1tc::k_tf_layer_test<224><<<1, 224, smem>>>(rows, K, N, X, img, bias, kact, out, derr);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    int herr = 0;
    if (e == cudaSuccess) e = cudaMemcpy(&herr, derr, sizeof(int), cudaMemcpyDeviceToHost);
    cudaFree(img); cudaFree(bias); cudaFree(derr);
    if (e != cudaSuccess) { set_error((int)e, "g1_dense_bf16x3", cudaGetErrorString(e)); return -1; }
    if (herr) { set_error(-62, "g1_dense_bf16x3", "tensor-core wait timed out"); return -62; }
    return 0;
}

int g1_gemm_bf16_tc(int M, int N, int K, const void* X, int ldx, const void* W, const float* bias, int act, float* out) {
    if (M <= 0 || N <= 0 || K <= 0 || ldx < K) { set_error(-22, "g1_gemm_bf16_tc", "invalid shape"); return -22; }
    int* derr = nullptr;
    CKR(cudaMalloc(&derr, sizeof(int)), -1);
    CKR(cudaMemset(derr, 0, sizeof(int)), -1);
    cudaError_t e = dense_tc(M, N, K, (const __nv_bfloat16*)X, ldx, (const __nv_bfloat16*)W, bias, act, out, N, nullptr, 0,
                             derr, 0);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    int herr = 0;
    if (e == cudaSuccess) e = cudaMemcpy(&herr, derr, sizeof(int), cudaMemcpyDeviceToHost);
    cudaFree(derr);
    if (e != cudaSuccess) { set_error((int)e, "g1_gemm_bf16_tc", cudaGetErrorString(e)); return -1; }
    if (herr) { set_error(-62, "g1_gemm_bf16_tc", "tensor-core wait timed out"); return -62; }
    return 0;
}

// extension: nonzero if a tensor-core wait of this env's bf16 policy path timed out since
// the last call (synchronises the env's device work; the flag is cleared).
int g1_env_tc_status(void* h) { return tc_error((EnvState*)h); }

// g1_env.cu:365-382
void g1_occupancy_report(void) {
    cudaDeviceProp p;
    if (cudaGetDeviceProperties(&p, 0) != cudaSuccess) return;
    printf("SM count %d, regs/SM %d, smem/SM %zu, maxThreads/SM %d\n", p.multiProcessorCount, p.regsPerMultiprocessor,
           p.sharedMemPerMultiprocessor, p.maxThreadsPerMultiProcessor);
    struct { const char* nm; const void* fn; } ks[] = {{"k_g1", (const void*)k_g1}, {"k_qacc", (const void*)k_qacc}};
    const SmemPlan plan = smem_plan();
    for (auto& k : ks) {
        cudaFuncAttributes fa;
        cudaFuncGetAttributes(&fa, k.fn);
        int mb = 0;
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&mb, k.fn, NTHREADS, plan.total_bytes);
        printf("  %-8s regs=%d localFrame=%zuB smem=%dB maxActiveBlocks/SM=%d warps/SM=%d\n", k.nm, fa.numRegs,
               fa.localSizeBytes, plan.total_bytes, mb, mb * NWARPS);
    }
}

}  // extern "C"

// trainer batch preparation (GAE, observation renormalisation, RunNorm update)
#include "g1_ppo_prep.cuh"
