// g1_mlp_tc.cuh -- the policy MLP as a tensor-core contraction on sm_100a (tcgen05 + TMEM).
//
// One CTA computes a 128 x BN tile of  out = act(X W^T + b)  for one dense layer:
//   X  [M][K]  bf16 row-major (rows = worlds),
//   W  [N][K]  bf16 row-major (torch Linear layout, i.e. K-major for the MMA's B operand),
//   b  [N]     fp32, accumulation in fp32 in tensor memory.
// K is walked in chunks of KC = 64: 128 threads copy the A and B chunks from global memory
// into shared memory in the canonical K-major, no-swizzle UMMA layout (8-row x 16-byte core
// matrices), one thread issues KC/16 = 4 `tcgen05.mma.cta_group::1.kind::f16` (M = 128,
// N = BN, K = 16 each) and commits them to an mbarrier; the chunks are double-buffered so the
// copy of chunk c+1 overlaps the MMAs of chunk c.  The epilogue reads the accumulator with
// `tcgen05.ld.32x32b` (warp w owns TMEM lanes 32w..32w+31 = rows), adds the bias, applies the
// activation and writes fp32 and/or bf16 outputs.
//
// Every wait on an mbarrier is bounded; a timeout sets *err and the CTA finishes without
// touching its accumulator.
#pragma once
#include <cuda_bf16.h>
#include <stdint.h>

namespace g1tc {

constexpr int TM = 128;   // rows (worlds) per CTA tile
constexpr int KC = 64;    // K per chunk
constexpr int NTH = 128;  // threads per CTA
constexpr uint32_t SPIN_LIMIT = 1u << 22;

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

// byte offset of element (r, k) of a [rows][KC] bf16 chunk in the canonical K-major,
// no-swizzle layout: 8x8 core matrices (8 rows x 16 bytes), core matrices adjacent along K
// (LBO = 128 B), 8-row groups KC/8 core matrices apart (SBO = KC/8 * 128 B = 1024 B)
__device__ __forceinline__ uint32_t canon_off(int r, int k) {
    return (uint32_t)((r >> 3) * (KC / 8) * 128 + (k >> 3) * 128 + (r & 7) * 16 + (k & 7) * 2);
}

// UMMA shared-memory descriptor (SWIZZLE_NONE, K-major): start, LBO, SBO in 16-byte units,
// version 1 (bit 46)
__device__ __forceinline__ uint64_t make_desc(uint32_t saddr) {
    const uint64_t lbo = 128 >> 4, sbo = (KC / 8 * 128) >> 4;
    return (uint64_t)((saddr >> 4) & 0x3FFF) | (lbo << 16) | (sbo << 32) | (1ull << 46);
}

// instruction descriptor: kind::f16 with bf16 A/B, f32 accumulator, both K-major
__host__ __device__ constexpr uint32_t make_idesc(int M, int N) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t phase, uint32_t limit = SPIN_LIMIT) {
    for (uint32_t it = 0; it < limit; ++it) {
        uint32_t done;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(done)
            : "r"(bar), "r"(phase)
            : "memory");
        if (done) return true;
    }
    return false;
}

// act: 0 tanh, 1 ELU, -1 identity
template <int BN>
__global__ void __launch_bounds__(NTH, 1)
k_dense_tc(int M, int N, int K, const __nv_bfloat16* __restrict__ X, int ldx, const __nv_bfloat16* __restrict__ W,
           const float* __restrict__ bias, int act, float* __restrict__ out_f32, int ldo,
           __nv_bfloat16* __restrict__ out_bf16, int ldob, int* err) {
    extern __shared__ __align__(1024) uint8_t smem[];
    constexpr int ABYTES = TM * KC * 2, BBYTES = BN * KC * 2;
    uint8_t* As[2] = {smem, smem + ABYTES + BBYTES};
    uint8_t* Bs[2] = {smem + ABYTES, smem + 2 * ABYTES + BBYTES};
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 2 * (ABYTES + BBYTES));  // [2]
    uint32_t* tslot = reinterpret_cast<uint32_t*>(bars + 2);
    __shared__ int s_fail;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int m0 = blockIdx.x * TM, n0 = blockIdx.y * BN;
    if (tid == 0) {
        s_fail = 0;
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(&bars[0])));
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(&bars[1])));
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tslot)),
                     "r"(BN));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    asm volatile("tcgen05.fence::before_thread_sync;");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;");
    const uint32_t tmem = *tslot;
    const uint32_t idesc = make_idesc(TM, BN);
    const int nchunk = (K + KC - 1) / KC;
    uint32_t phase[2] = {0u, 0u};
    bool ok = true;

    auto load_chunk = [&](int c, int buf) {
        const int k0 = c * KC;
        // A: TM rows x KC, 8 bf16 (16 bytes) per item
        for (int it = tid; it < TM * (KC / 8); it += NTH) {
            const int r = it / (KC / 8), kg = (it % (KC / 8)) * 8;
            const int gm = m0 + r, gk = k0 + kg;
            uint4 v = make_uint4(0, 0, 0, 0);
            if (gm < M) {
                if (gk + 8 <= K && ((ldx & 7) == 0)) v = *reinterpret_cast<const uint4*>(X + (size_t)gm * ldx + gk);
                else {
                    __nv_bfloat16 t[8];
#pragma unroll
                    for (int q = 0; q < 8; ++q) t[q] = (gk + q < K) ? X[(size_t)gm * ldx + gk + q] : __float2bfloat16(0.f);
                    v = *reinterpret_cast<uint4*>(t);
                }
            }
            *reinterpret_cast<uint4*>(As[buf] + canon_off(r, kg)) = v;
        }
        for (int it = tid; it < BN * (KC / 8); it += NTH) {
            const int r = it / (KC / 8), kg = (it % (KC / 8)) * 8;
            const int gn = n0 + r, gk = k0 + kg;
            uint4 v = make_uint4(0, 0, 0, 0);
            if (gn < N) {
                if (gk + 8 <= K && ((K & 7) == 0)) v = *reinterpret_cast<const uint4*>(W + (size_t)gn * K + gk);
                else {
                    __nv_bfloat16 t[8];
#pragma unroll
                    for (int q = 0; q < 8; ++q) t[q] = (gk + q < K) ? W[(size_t)gn * K + gk + q] : __float2bfloat16(0.f);
                    v = *reinterpret_cast<uint4*>(t);
                }
            }
            *reinterpret_cast<uint4*>(Bs[buf] + canon_off(r, kg)) = v;
        }
        // make the generic-proxy smem writes visible to the tensor core (async proxy)
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    };

    load_chunk(0, 0);
    for (int c = 0; c < nchunk; ++c) {
        const int buf = c & 1;
        __syncthreads();
        if (tid == 0) {
            asm volatile("tcgen05.fence::after_thread_sync;");
            const uint32_t a0 = smem_u32(As[buf]), b0 = smem_u32(Bs[buf]);
#pragma unroll
            for (int ks = 0; ks < KC / 16; ++ks) {
                const uint64_t ad = make_desc(a0 + ks * 256), bd = make_desc(b0 + ks * 256);
                const uint32_t accum = (c > 0 || ks > 0) ? 1u : 0u;
                asm volatile(
                    "{\n\t.reg .pred p;\n\t"
                    "setp.ne.b32 p, %4, 0;\n\t"
                    "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
                    ::"r"(tmem), "l"(ad), "l"(bd), "r"(idesc), "r"(accum));
            }
            asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                             smem_u32(&bars[buf]))
                         : "memory");
        }
        // copy the next chunk into the other buffer while these MMAs run; that buffer's
        // previous MMAs (chunk c-1) must have finished first
        if (c + 1 < nchunk) {
            if (c >= 1) {
                if (!mbar_wait(smem_u32(&bars[buf ^ 1]), phase[buf ^ 1])) ok = false;
                phase[buf ^ 1] ^= 1u;
            }
            load_chunk(c + 1, buf ^ 1);
        }
    }
    // wait for the last chunk's MMAs (and the one before it if not yet waited)
    if (nchunk >= 2) {
        const int b = (nchunk - 2) & 1;
        if (!mbar_wait(smem_u32(&bars[b]), phase[b])) ok = false;
        phase[b] ^= 1u;
    }
    {
        const int b = (nchunk - 1) & 1;
        if (!mbar_wait(smem_u32(&bars[b]), phase[b])) ok = false;
    }
    if (!ok) atomicExch(&s_fail, 1);
    asm volatile("tcgen05.fence::before_thread_sync;");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;");
    if (s_fail) {
        if (tid == 0) atomicExch(err, 1);
    } else {
        // epilogue: warp w reads TMEM lanes 32w.. (rows), 8 columns per load
        const int row = m0 + warp * 32 + lane;
        for (int c0 = 0; c0 < BN; c0 += 8) {
            uint32_t r[8];
            const uint32_t taddr = tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)c0;
            asm volatile(
                "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                : "r"(taddr));
            asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
            if (row < M) {
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                    const int n = n0 + c0 + q;
                    if (n >= N) break;
                    float v = __uint_as_float(r[q]) + (bias ? bias[n] : 0.f);
                    if (act == 0) v = tanhf(v);
                    else if (act == 1) v = v > 0.f ? v : expm1f(v);
                    if (out_f32) out_f32[(size_t)row * ldo + n] = v;
                    if (out_bf16) out_bf16[(size_t)row * ldob + n] = __float2bfloat16(v);
                }
            }
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;");
    __syncthreads();
    if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(BN));
}

template <int BN>
constexpr int dense_tc_smem() {
    return 2 * (TM * KC * 2 + BN * KC * 2) + 64;
}

// ======================================================================================
// fp32-accurate dense layers inside a CTA on the tensor cores (the fp32 policy MLP of the
// fused rollout kernel).
//
// out[r][n] = act(b[n] + sum_k x[r][k] W[n][k]) for r < nrows <= 64, N <= 256 (N % 16 == 0),
// K <= 256.  Each fp32 operand is split into three bf16 parts, v = v1 + v2 + v3 with
// v1 = bf16(v), v2 = bf16(v - v1), v3 = bf16(v - v1 - v2) (the differences are exact in fp32;
// the split keeps 24+ significant bits), and the six products whose size is at least
// 2^-18 of x*w -- x3w1, x1w3, x2w2, x2w1, x1w2, x1w1, smallest first -- are accumulated in
// fp32 in tensor memory by `tcgen05.mma.kind::f16` (M = 128, N, K = 16).  The dropped terms
// are below 2^-26 |x w|, under fp32 rounding (the multi-word split is the classical way to
// carry a wider mantissa through a narrower multiplier).  The tensor core aligns each MMA's
// addends to the accumulator it adds into, so small terms added into the running full sum
// would lose their low bits (measured: ~6x the error of an fp32 dot product at K = 256).  The
// five small products therefore accumulate in their own TMEM accumulator (columns 256..511)
// and x1w1 in another (columns 0..N-1); the epilogue adds the two in fp32 -- the result is as
// accurate as an fp32 FFMA dot product.
//
// Activations stay resident in shared memory as the three bf16 parts of the whole input
// row (A, canonical K-major no-swizzle layout, 64 rows stored); the previous layer's
// epilogue writes them directly.  Weights come from global memory pre-split: one contiguous
// image per 16-wide K chunk ([w1 | w2 | w3], canonical), fetched by a single `cp.async.bulk`
// (no multicast) into one of TF_NSTAGE stages, completing on the stage's `full` mbarrier.
// One thread walks the chunks (wait full, six MMAs, commit to the stage's `empty` barrier,
// refill the stage behind), so there is no CTA-wide synchronisation per chunk; a final
// commit to `done` releases the epilogue.  Every mbarrier wait is bounded; a timeout sets
// *err (the results are then garbage, nothing faults).
//
// Byte layouts:
//   A part p: p * TF_APART + (k>>3)*1024 + (r>>3)*128 + (r&7)*16 + (k&7)*2.  The M = 128 MMA
//       also reads rows 64..127 through the row stride; those land in the next 1 KB
//       (garbage rows, never read back).
//   B chunk part p (N-wide layer): p * 32N + (k>>3)*16N + (n>>3)*128 + (n&7)*16 + (k&7)*2.
// Descriptors: LBO = distance between core matrices along K, SBO = 128 (next 8 rows).
#ifdef G1_PROF  // phase counters of the profiling build (g1_physics.cuh)
using ::g1::g_prof;
using ::g1::P_TF_MMA;
using ::g1::P_TF_EPI;
using ::g1::P_TF_EPI1;
using ::g1::P_TF_EPI2;
#endif
constexpr int TF_ROWS = 64;
constexpr int TF_KMAX = 256;
constexpr int TF_APART = TF_ROWS * TF_KMAX * 2;  // 32 KB per bf16 part
constexpr int TF_ABYTES = 3 * TF_APART;
constexpr int TF_STAGE = 3 * 4096 * 2;           // 24 KB: one chunk of N x kc weights, N kc = 4096
constexpr int TF_NSTAGE = 4;
constexpr int TF_HDBYTES = TF_ROWS * 32 * 4;     // head outputs, fp32 [64][32]
constexpr int TF_SCRATCH = TF_ABYTES + TF_NSTAGE * TF_STAGE + TF_HDBYTES;
static_assert(TF_ROWS * (TF_KMAX + 4) * 4 <= TF_NSTAGE * TF_STAGE, "hidden-layer epilogue staging must fit in the stages");
constexpr int TF_MMA_WARP = 2, TF_COPY_WARP = 3;  // lane 0 of each; idle in the epilogue (rows < 64)

// K width of one weight chunk of an N-wide layer: the largest multiple of 16 with N kc <= 4096
__host__ __device__ constexpr int tf_kc(int N) { return ((4096 / N) & ~15) < TF_KMAX ? ((4096 / N) & ~15) : TF_KMAX; }

__device__ __forceinline__ uint64_t make_desc_lbo(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
    return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)((lbo_bytes >> 4) & 0x3FFF) << 16) |
           ((uint64_t)((sbo_bytes >> 4) & 0x3FFF) << 32) | (1ull << 46);
}

__device__ __forceinline__ void mbar_init(uint64_t* b, int count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(count));
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* b, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)), "r"(bytes) : "memory");
}
// global -> shared bulk copy of `bytes` (multiple of 16, both addresses 16-byte aligned),
// completing on mbarrier `bar`; plain (non-multicast) form
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}

// split of an fp32 value into three bf16 words (v = p0 + p1 + p2 to 2^-27)
__device__ __forceinline__ void split3(float v, __nv_bfloat16& p0, __nv_bfloat16& p1, __nv_bfloat16& p2) {
    p0 = __float2bfloat16_rn(v);
    const float r1 = v - __bfloat162float(p0);
    p1 = __float2bfloat16_rn(r1);
    p2 = __float2bfloat16_rn(r1 - __bfloat162float(p1));
}
__device__ __forceinline__ uint32_t pack2(__nv_bfloat16 a, __nv_bfloat16 b) {
    return (uint32_t)__bfloat16_as_ushort(a) | ((uint32_t)__bfloat16_as_ushort(b) << 16);
}
// byte offset of (row r, input k) inside one A part
__host__ __device__ inline uint32_t tf_aoff(int r, int k) {
    return (uint32_t)((k >> 3) * 1024 + (r >> 3) * 128 + (r & 7) * 16 + (k & 7) * 2);
}
// element index of (n, kk) inside one part of a chunk image of an N-wide layer
__host__ __device__ inline int tf_bidx(int N, int n, int kk) {
    return (kk >> 3) * (8 * N) + (n >> 3) * 64 + (n & 7) * 8 + (kk & 7);
}
// bf16 elements of one chunk image of an N-wide layer ([w1 | w2 | w3])
__host__ __device__ constexpr int tf_chunk_elems(int N) { return 3 * N * tf_kc(N); }
__host__ __device__ constexpr int tf_nchunk(int K, int N) { return (K + tf_kc(N) - 1) / tf_kc(N); }

// writes the 3 parts of 8 consecutive inputs k0..k0+7 (k0 % 8 == 0) of row r
__device__ __forceinline__ void tf_store8(uint8_t* A, int r, int k0, const float* v) {
    __nv_bfloat16 p[3][8];
#pragma unroll
    for (int j = 0; j < 8; ++j) split3(v[j], p[0][j], p[1][j], p[2][j]);
    const uint32_t off = tf_aoff(r, k0);
#pragma unroll
    for (int q = 0; q < 3; ++q)
        *reinterpret_cast<uint4*>(A + q * TF_APART + off) =
            make_uint4(pack2(p[q][0], p[q][1]), pack2(p[q][2], p[q][3]), pack2(p[q][4], p[q][5]), pack2(p[q][6], p[q][7]));
}

// Shared-memory pipeline state (outlives the caller's other uses of the scratch).  Weight
// chunks are numbered globally (st[1] = chunks consumed so far); chunk g uses stage g % NSTAGE
// and is that stage's (g / NSTAGE)-th use, so its full / empty phase parity is (g/NSTAGE) & 1.
// st = {tmem, chunks consumed, -, -, done phase, chunks of the next layer already issued}.
struct TfShared {
    uint64_t bars[2 * TF_NSTAGE + 1];  // full[4], empty[4], done
    uint32_t st[6];
};
// TMEM: 512 columns -- [0, 256) the x1w1 accumulator, [256, 512) the small-product one

struct TfLayer {
    const __nv_bfloat16* img;  // chunk images
    const float* bias;         // [N]
    int K, N;
};

__device__ __forceinline__ void tf_init(TfShared* S) {
    if (threadIdx.x == 0) {
        for (int i = 0; i < 2 * TF_NSTAGE + 1; ++i) mbar_init(&S->bars[i], 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        for (int i = 1; i < 6; ++i) S->st[i] = 0;
    }
    if ((threadIdx.x >> 5) == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&S->st[0])),
                     "r"(512));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    asm volatile("tcgen05.fence::before_thread_sync;");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;");
}

__device__ __forceinline__ void tf_release(TfShared* S) {
    asm volatile("tcgen05.fence::before_thread_sync;");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;");
    if ((threadIdx.x >> 5) == 0)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(S->st[0]), "r"(512));
}

// Failure-path check of the bounded waits (test entry g1_env_test_wait_timeout): sets up the
// policy pipeline exactly as k_g1 does (barriers, 512 TMEM columns), then the MMA-issuing
// thread waits on a stage's `full` barrier that nothing arrives at -- no bulk copy and no
// MMA is in flight -- with a spin limit given at launch.  The wait runs out, the error flag
// is set as in the rollout, and TMEM is released before the CTA exits.
__global__ void __launch_bounds__(224, 1) k_wait_probe(int* err, uint32_t limit) {
    __shared__ TfShared S;
    tf_init(&S);
    bool ok = true;
    if (threadIdx.x == 64) ok = mbar_wait(smem_u32(&S.bars[0]), 0u, limit);
    if (!ok) atomicExch(err, 2);
    tf_release(&S);
}

// copy thread: bring chunk c of layer L in as global chunk g, once the stage's previous
// chunk (g - NSTAGE) has been consumed by its MMAs
__device__ __forceinline__ bool tf_issue(TfShared* S, uint8_t* stages, const TfLayer& L, int c, uint32_t g) {
    const uint32_t s = g % TF_NSTAGE;
    bool ok = true;
    if (g >= TF_NSTAGE) ok = mbar_wait(smem_u32(&S->bars[TF_NSTAGE + s]), ((g / TF_NSTAGE) - 1) & 1u);
    const uint32_t bytes = (uint32_t)tf_chunk_elems(L.N) * 2;
    mbar_expect_tx(&S->bars[s], bytes);
    bulk_g2s(stages + s * TF_STAGE, L.img + (size_t)c * tf_chunk_elems(L.N), bytes, &S->bars[s]);
    return ok;
}

// copy thread: queue the first chunks of layer L, which starts at global chunk g0
__device__ __forceinline__ bool tf_prefetch(TfShared* S, uint8_t* stages, const TfLayer& L, uint32_t g0) {
    const int n = tf_nchunk(L.K, L.N), m = n < TF_NSTAGE ? n : TF_NSTAGE;
    bool ok = true;
    for (int c = 0; c < m; ++c) ok &= tf_issue(S, stages, L, c, g0 + c);
    S->st[5] = (uint32_t)m;
    return ok;
}

// One layer.  All threads call it; on entry the A parts of the input are in place (visible
// to the async proxy: the writers ran fence.proxy.async before the CTA barrier that
// preceded this call) and tf_prefetch queued the first chunks of L.  The MMA thread walks
// the chunks (wait full, six MMAs, commit to the stage's empty barrier); the copy thread
// refills stages as they empty and then queues the first chunks of nxt (if any).  Epilogue:
// hidden layers (act 0 tanh / 1 ELU / 2 identity) write the 3 parts of their output into A,
// in place; the head (act -1, N <= 32) writes fp32 to hd [rows][32].
template <int NT>
__device__ void tf_layer(TfShared* S, uint8_t* A, uint8_t* stages, const TfLayer& L, const TfLayer* nxt, int nrows, int act,
                         float* hd, int* err) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int N = L.N, kc = tf_kc(N), nchunk = tf_nchunk(L.K, N);
    const uint32_t tmem = S->st[0], g0 = S->st[1];
    bool ok = true;
#ifdef G1_PROF
    PROF_BEGIN();
#endif
    if (warp == TF_MMA_WARP && lane == 0) {
        const uint32_t idesc = make_idesc(128, N);
        const uint32_t pbytes = (uint32_t)N * kc * 2;
        const uint32_t a0 = smem_u32(A);
        // operand pairs (A part, B part), smallest product first
        const int pa[6] = {2, 0, 1, 1, 0, 0}, pb[6] = {0, 2, 1, 0, 1, 0};
        for (int c = 0; c < nchunk; ++c) {
            const uint32_t g = g0 + c, s = g % TF_NSTAGE;
            if (!mbar_wait(smem_u32(&S->bars[s]), (g / TF_NSTAGE) & 1u)) ok = false;
            asm volatile("tcgen05.fence::after_thread_sync;");
            const uint32_t b0 = smem_u32(stages + s * TF_STAGE);
            for (int j = 0; j < kc / 16; ++j) {
                const int kg = c * (kc / 16) + j;  // 16-wide K step within the layer
                if (kg * 16 >= L.K) break;  // all-zero weights past K (A is zero-padded to 16)
#pragma unroll
                for (int m = 0; m < 6; ++m) {
                    const uint64_t ad = make_desc_lbo(a0 + pa[m] * TF_APART + kg * 2048, 1024, 128);
                    const uint64_t bd = make_desc_lbo(b0 + pb[m] * pbytes + j * 2 * (16 * N), 16 * N, 128);
                    // m < 5: small products -> columns 256..; m == 5: x1 w1 -> columns 0..
                    const uint32_t dst = tmem + (m < 5 ? 256u : 0u);
                    const uint32_t accum = (kg > 0 || (m > 0 && m < 5)) ? 1u : 0u;
                    asm volatile(
                        "{\n\t.reg .pred p;\n\t"
                        "setp.ne.b32 p, %4, 0;\n\t"
                        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(dst),
                        "l"(ad), "l"(bd), "r"(idesc), "r"(accum));
                }
            }
            asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                             smem_u32(&S->bars[TF_NSTAGE + s]))
                         : "memory");
        }
        asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                         smem_u32(&S->bars[2 * TF_NSTAGE]))
                     : "memory");
    } else if (warp == TF_COPY_WARP && lane == 0) {
        for (int c = (int)S->st[5]; c < nchunk; ++c) ok &= tf_issue(S, stages, L, c, g0 + c);
        // a hidden layer's epilogue stages its sums in the weight stages: the next layer's
        // chunks are queued by that layer itself
        if (nxt && act < 0) ok &= tf_prefetch(S, stages, *nxt, g0 + nchunk);
        else S->st[5] = 0;
    }
    // every thread: wait for the layer's MMAs
    if (!mbar_wait(smem_u32(&S->bars[2 * TF_NSTAGE]), S->st[4] & 1u)) ok = false;
    if (!ok) atomicExch(err, 1);
    asm volatile("tcgen05.fence::after_thread_sync;");
#ifdef G1_PROF
    PROF_MARK(P_TF_MMA);
#endif
    // epilogue.  TMEM lane r = row r: only warps w with 32 (w & 3) < rows can read it, and
    // they sit on two of the SM's four sub-partitions.  Phase 1: those warps (w and w + 4
    // split the columns) move accumulator sums + bias to fp32 rows in the weight stages
    // (hidden layers) or straight to hd (the head).  Phase 2 (hidden layers): every warp
    // applies the activation and writes the three bf16 parts of the next layer's input.
    const int q = warp & 3;
    const int nshare = (q + 4 < NT / 32) ? 2 : 1;
    float* stg = reinterpret_cast<float*>(stages);
    const int sld = N + 4;
    if (32 * q < nrows) {
        const int half = N / nshare, c_beg = (warp >> 2) * half, row = 32 * q + lane;
        for (int c0 = c_beg; c0 < c_beg + half; c0 += 8) {
            uint32_t r[8], u[8];
            const uint32_t taddr = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)c0;
            asm volatile(
                "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                : "r"(taddr));
            asm volatile(
                "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                : "=r"(u[0]), "=r"(u[1]), "=r"(u[2]), "=r"(u[3]), "=r"(u[4]), "=r"(u[5]), "=r"(u[6]), "=r"(u[7])
                : "r"(taddr + 256u));
            asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
            float v[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) v[j] = (__uint_as_float(r[j]) + __uint_as_float(u[j])) + L.bias[c0 + j];
            if (row < nrows) {
                if (act < 0) {
#pragma unroll
                    for (int j = 0; j < 8; ++j) hd[row * 32 + c0 + j] = v[j];
                } else {
                    float4* dst = reinterpret_cast<float4*>(stg + row * sld + c0);
                    dst[0] = make_float4(v[0], v[1], v[2], v[3]);
                    dst[1] = make_float4(v[4], v[5], v[6], v[7]);
                }
            }
        }
    }
    if (act >= 0) {
        __syncthreads();
#ifdef G1_PROF
        PROF_MARK(P_TF_EPI1);
#endif
        const int ng = N / 8;
        // consecutive threads take consecutive rows: their 16-byte stores into A are then
        // contiguous (a row's column groups are 1024 bytes apart, one bank group)
        for (int e = tid; e < nrows * ng; e += NT) {
            const int row = e % nrows, c0 = (e / nrows) * 8;
            const float4* src = reinterpret_cast<const float4*>(stg + row * sld + c0);
            const float4 a = src[0], b = src[1];
            float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                if (act == 0) v[j] = tanhf(v[j]);
                else if (act == 1) v[j] = v[j] > 0.f ? v[j] : expm1f(v[j]);
            }
            tf_store8(A, row, c0, v);
        }
#ifdef G1_PROF
        PROF_MARK(P_TF_EPI2);
#endif
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    asm volatile("tcgen05.fence::before_thread_sync;");
    __syncthreads();
#ifdef G1_PROF
    PROF_MARK(P_TF_EPI);
#endif
    if (tid == 0) { S->st[1] = g0 + nchunk; S->st[4] ^= 1u; }
    __syncthreads();
}

// Standalone test of tf_layer: one CTA of NT threads, rows <= 64; X [rows][K] fp32 global,
// W image / bias as built for one layer, out [rows][N] fp32 global.  Runs the layer twice
// (the second pass exercises the later barrier phases); hidden activations are read back
// from the A parts (sum of the three words), identity from the head buffer (N <= 32).
template <int NT>
__global__ void __launch_bounds__(NT, 1)
k_tf_layer_test(int rows, int K, int N, const float* X, const __nv_bfloat16* img, const float* bias, int act, float* out,
                int* err) {
    extern __shared__ __align__(1024) uint8_t smem[];
    uint8_t* A = smem;
    uint8_t* stages = smem + TF_ABYTES;
    float* hd = reinterpret_cast<float*>(stages + TF_NSTAGE * TF_STAGE);
    TfShared* S = reinterpret_cast<TfShared*>(smem + TF_SCRATCH);
    tf_init(S);
    TfLayer L{img, bias, K, N};
    for (int rep = 0; rep < 2; ++rep) {
        const int kpad = tf_nchunk(K, N) * tf_kc(N) < TF_KMAX ? tf_nchunk(K, N) * tf_kc(N) : TF_KMAX;
        for (int e = threadIdx.x; e < rows * (kpad / 8); e += NT) {
            const int r = e / (kpad / 8), k0 = (e % (kpad / 8)) * 8;
            float v[8];
            for (int j = 0; j < 8; ++j) v[j] = k0 + j < K ? X[r * K + k0 + j] : 0.f;
            tf_store8(A, r, k0, v);
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncthreads();
        if (threadIdx.x == TF_COPY_WARP * 32) tf_prefetch(S, stages, L, S->st[1]);
        tf_layer<NT>(S, A, stages, L, nullptr, rows, act, hd, err);
    }
    for (int e = threadIdx.x; e < rows * N; e += NT) {
        const int r = e / N, n = e % N;
        float v;
        if (act < 0) v = hd[r * 32 + n];
        else {
            const uint32_t off = tf_aoff(r, n);
            v = __bfloat162float(*reinterpret_cast<const __nv_bfloat16*>(A + off)) +
                __bfloat162float(*reinterpret_cast<const __nv_bfloat16*>(A + TF_APART + off)) +
                __bfloat162float(*reinterpret_cast<const __nv_bfloat16*>(A + 2 * TF_APART + off));
        }
        out[e] = v;
    }
    tf_release(S);
}
__host__ __device__ constexpr int tf_test_smem() { return TF_SCRATCH + (int)sizeof(TfShared); }

}  // namespace g1tc
