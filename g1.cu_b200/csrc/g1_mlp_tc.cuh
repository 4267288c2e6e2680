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
constexpr uint32_t SPIN_LIMIT = 1u << 26;

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

__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t phase) {
    for (uint32_t it = 0; it < SPIN_LIMIT; ++it) {
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

}  // namespace g1tc
