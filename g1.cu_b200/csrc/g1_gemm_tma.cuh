// g1_gemm_tma.cuh -- the wide-policy dense layer as a persistent, warp-specialised tcgen05
// GEMM fed by TMA:  out = act(X W^T + b),  X [M][K] bf16 (rows = worlds), W [N][K] bf16,
// fp32 accumulation in tensor memory, bf16 or fp32 output.
//
// * Tiles of 128 (worlds) x BN (outputs); a CTA per SM walks tiles m-fastest, so the CTAs in
//   flight share a weight tile in L2.
// * K in chunks of 64 (128 bytes of bf16): one TMA tiled load per operand per chunk
//   (`cp.async.bulk.tensor.2d`, 128-byte swizzle, out-of-range rows / columns zero-filled,
//   no multicast) into one of STAGES shared-memory stages, completing on the stage's `full`
//   mbarrier.  The operands land in the canonical K-major SWIZZLE_128B layout the MMA reads
//   directly (8-row groups 1024 bytes apart; the 16-wide K steps 32 bytes apart inside the
//   swizzle atom).
// * Warp 0 lane 0 issues the loads; warp 1 lane 0 issues `tcgen05.mma.cta_group::1.kind::f16`
//   (M = 128, N = BN, K = 16) and commits each stage to its `empty` barrier; the other warps
//   run the epilogue (four per TMEM lane quarter for BN >= 128, two otherwise, each on an
//   equal share of the columns): `tcgen05.ld`, bias,
//   activation, store.  The accumulator is double-buffered in TMEM (2 x BN columns) so the
//   epilogue of one tile overlaps the MMAs of the next.
// * Every mbarrier wait is bounded; a timeout sets *err and the CTA stops waiting (results are
//   then garbage, nothing faults).  X and W must be 16-byte aligned with K % 8 == 0 (TMA row
//   pitch); the host falls back to the thread-copy kernel otherwise.
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <stdint.h>

// Each CTA walks a tile's K chunks starting at chunk blockIdx.x (mod the chunk count): the
// CTAs working on tiles of one weight block then read different chunks of it at any moment
// instead of all 148 reading the same 16 KB from the same L2 slices.  The fp32 accumulation
// order depends only on the CTA index, so results stay deterministic for a given grid.
#ifndef G1_GEMM_KROT
#define G1_GEMM_KROT 1
#endif

namespace g1gemm {

constexpr int BM = 128, BK = 64, STAGES = 4;
// epilogue warps: four per TMEM lane quarter for wide tiles (each a quarter of the columns),
// two for narrow ones
template <int BN>
__host__ __device__ constexpr int nepi() { return BN >= 128 ? 16 : 8; }
template <int BN>
__host__ __device__ constexpr int nth() { return 64 + 32 * nepi<BN>(); }
constexpr uint32_t SPIN = 1u << 22;

__device__ __forceinline__ uint32_t s32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ bool wait(uint64_t* bar, uint32_t parity) {
    const uint32_t a = s32(bar);
    for (uint32_t it = 0; it < SPIN; ++it) {
        uint32_t done;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(done)
            : "r"(a), "r"(parity)
            : "memory");
        if (done) return true;
    }
    return false;
}

// K-major SWIZZLE_128B UMMA descriptor: SBO = 1024 B (next 8 rows), LBO unused (16 B),
// version 1, layout type 2
__device__ __forceinline__ uint64_t desc_sw128(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) | (1ull << 46) |
           (2ull << 61);
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            s32(dst)),
        "l"(map), "r"(x), "r"(y), "r"(s32(bar))
        : "memory");
}

template <int BN>
struct Smem {
    uint8_t a[STAGES][BM * BK * 2];  // 16 KB each, 1024-byte aligned
    uint8_t b[STAGES][BN * BK * 2];
    uint64_t full[STAGES], empty[STAGES], tfull[2], tempty[2];
    uint32_t tslot;
};
template <int BN>
constexpr int smem_bytes() {
    return (int)sizeof(Smem<BN>) + 1024;
}

// act: 0 tanh, 1 ELU, -1 identity; out_b (bf16, ld ldo) or out_f (fp32, ld ldo)
template <int BN>
__global__ void __launch_bounds__(nth<BN>(), 1)
k_gemm(const __grid_constant__ CUtensorMap tmx, const __grid_constant__ CUtensorMap tmw, int M, int N, int K,
       const float* __restrict__ bias, int act, __nv_bfloat16* __restrict__ out_b, float* __restrict__ out_f, int ldo,
       int* err) {
    extern __shared__ uint8_t smem_raw[];
    Smem<BN>& S = *reinterpret_cast<Smem<BN>*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int ntm = (M + BM - 1) / BM, ntn = (N + BN - 1) / BN, ntiles = ntm * ntn, nk = (K + BK - 1) / BK;
    if (tid == 0) {
        for (int i = 0; i < STAGES; ++i) {
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(s32(&S.full[i])));
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(s32(&S.empty[i])));
        }
        for (int i = 0; i < 2; ++i) {
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(s32(&S.tfull[i])));
            asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(s32(&S.tempty[i])), "r"(nepi<BN>()));
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(s32(&S.tslot)),
                     "r"(2 * BN));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    asm volatile("tcgen05.fence::before_thread_sync;");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;");
    const uint32_t tmem = S.tslot;
    bool ok = true;

    if (warp == 0 && lane == 0) {  // TMA producer
        asm volatile("prefetch.tensormap [%0];" ::"l"(&tmx) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(&tmw) : "memory");
        int stage = 0;
        uint32_t phase = 0;
        for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x) {
            const int m0 = (tile % ntm) * BM, n0 = (tile / ntm) * BN;
            for (int kb = 0; kb < nk; ++kb) {
                if (!wait(&S.empty[stage], phase ^ 1u)) { ok = false; break; }
                asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(s32(&S.full[stage])),
                             "r"((BM + BN) * BK * 2)
                             : "memory");
#if G1_GEMM_KROT
                const int kc = (kb + (int)blockIdx.x) % nk;
#else
                const int kc = kb;
#endif
                tma_load_2d(S.a[stage], &tmx, kc * BK, m0, &S.full[stage]);
                tma_load_2d(S.b[stage], &tmw, kc * BK, n0, &S.full[stage]);
                if (++stage == STAGES) { stage = 0; phase ^= 1u; }
            }
        }
    } else if (warp == 1 && lane == 0) {  // MMA issuer
        constexpr uint32_t idesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
        int stage = 0;
        uint32_t phase = 0, acc = 0, accph = 0;
        for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x) {
            if (!wait(&S.tempty[acc], accph ^ 1u)) { ok = false; break; }
            asm volatile("tcgen05.fence::after_thread_sync;");
            const uint32_t d = tmem + acc * BN;
            for (int kb = 0; kb < nk; ++kb) {
                if (!wait(&S.full[stage], phase)) { ok = false; break; }
                asm volatile("tcgen05.fence::after_thread_sync;");
                const uint32_t a0 = s32(S.a[stage]), b0 = s32(S.b[stage]);
#pragma unroll
                for (int k = 0; k < BK / 16; ++k) {
                    const uint64_t ad = desc_sw128(a0 + k * 32), bd = desc_sw128(b0 + k * 32);
                    const uint32_t accum = (kb > 0 || k > 0) ? 1u : 0u;
                    asm volatile(
                        "{\n\t.reg .pred p;\n\t"
                        "setp.ne.b32 p, %4, 0;\n\t"
                        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
                        "l"(ad), "l"(bd), "r"(idesc), "r"(accum));
                }
                asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                                 s32(&S.empty[stage]))
                             : "memory");
                if (++stage == STAGES) { stage = 0; phase ^= 1u; }
            }
            asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                             s32(&S.tfull[acc]))
                         : "memory");
            if (++acc == 2) { acc = 0; accph ^= 1u; }
        }
    } else if (warp >= 2) {  // epilogue: warp w reads TMEM lanes 32 (w & 3) .., part (w - 2) / 4 of the columns
        const int q = warp & 3, half = (warp - 2) >> 2;
        constexpr int CW = BN / (nepi<BN>() / 4);  // columns per epilogue warp
        static_assert(CW % 16 == 0, "16-column TMEM loads");
        uint32_t acc = 0, accph = 0;
        for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
            const int m0 = (tile % ntm) * BM, n0 = (tile / ntm) * BN;
            if (!wait(&S.tfull[acc], accph)) { ok = false; break; }
            asm volatile("tcgen05.fence::after_thread_sync;");
            const int row = m0 + 32 * q + lane;
#pragma unroll 1
            for (int cc = 0; cc < CW; cc += 16) {
                const int c0 = half * CW + cc, nb = n0 + c0;
                uint32_t r[16];
                const uint32_t taddr = tmem + ((uint32_t)(32 * q) << 16) + acc * BN + (uint32_t)c0;
                asm volatile(
                    "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
                    : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
                      "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
                    : "r"(taddr));
                // the bias of these 16 columns (same for every lane) while the load is in flight
                float bv[16];
                if (bias && nb + 16 <= N && (((uintptr_t)(bias + nb)) & 15) == 0) {
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const float4 t = __ldg(reinterpret_cast<const float4*>(bias + nb) + j);
                        bv[4 * j] = t.x; bv[4 * j + 1] = t.y; bv[4 * j + 2] = t.z; bv[4 * j + 3] = t.w;
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < 16; ++j) bv[j] = (bias && nb + j < N) ? __ldg(bias + nb + j) : 0.f;
                }
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                if (row < M && nb < N) {
                    float v[16];
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        float x = __uint_as_float(r[j]) + bv[j];
                        if (act == 0) x = tanhf(x);
                        else if (act == 1) x = x > 0.f ? x : expm1f(x);
                        v[j] = x;
                    }
                    if (out_f) {
#pragma unroll
                        for (int j = 0; j < 16; ++j)
                            if (nb + j < N) out_f[(size_t)row * ldo + nb + j] = v[j];
                    } else if (nb + 16 <= N && (ldo & 7) == 0) {
                        uint32_t pk[8];
#pragma unroll
                        for (int j = 0; j < 8; ++j) {
                            const __nv_bfloat162 h2 = __floats2bfloat162_rn(v[2 * j], v[2 * j + 1]);
                            pk[j] = *reinterpret_cast<const uint32_t*>(&h2);
                        }
                        uint4* dst = reinterpret_cast<uint4*>(out_b + (size_t)row * ldo + nb);
                        dst[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
                        dst[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
                    } else {
#pragma unroll
                        for (int j = 0; j < 16; ++j)
                            if (nb + j < N) out_b[(size_t)row * ldo + nb + j] = __float2bfloat16(v[j]);
                    }
                }
            }
            asm volatile("tcgen05.fence::before_thread_sync;");
            __syncwarp();
            if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(s32(&S.tempty[acc])) : "memory");
            if (++acc == 2) { acc = 0; accph ^= 1u; }
        }
    }
    if (!ok) atomicExch(err, 1);
    asm volatile("tcgen05.fence::before_thread_sync;");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;");
    if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2 * BN));
}

}  // namespace g1gemm
