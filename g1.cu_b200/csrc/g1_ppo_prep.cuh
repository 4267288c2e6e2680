// g1_ppo_prep.cuh -- the trainer's per-iteration batch preparation on the GPU, fed directly
// from the rollout's trajectory buffers (the Python H-loop and torch reductions of the
// reference trainer, scripts/ppo_fused.py:104-119, and RunNorm.update, scripts/ppo.py:71-79).
//
//   k_gae          one thread per world walks t = H-1 .. 0: delta, gae, adv, ret, in the exact
//                  fp32 operation order of ppo_fused.py:110-115 (each op rounded once, no FMA
//                  contraction), so adv/ret are bit-identical to the torch loop; fp64 block
//                  sums of adv and adv^2 for the advantage normalisation.
//   k_obs_prep     one HBM pass over O[H*N][dim]: nobs = clamp((o - fmean)/sqrt(fvar + 1e-8),
//                  -10, 10) (ppo_fused.py:104-105, bit-identical: IEEE sqrt and divide) and the
//                  fp64 per-dimension sums of o and o^2 of the RAW observations (the moments
//                  norm.update needs, ppo_fused.py:106).  Each thread owns one 16-byte column
//                  group and strides over rows, so a warp's loads and stores are contiguous.
//   k_adv_norm     adv = (adv - mean) / (std + 1e-8), unbiased std (ppo_fused.py:119).
//   k_runnorm      RunNorm.update from the batch moments (ppo.py:71-79), in fp64.
//
// Moment buffers are fp64 [count, sum[dim], sumsq[dim]] so that several ranks can add theirs
// with one all-reduce before the finalising kernels; the entry points zero them first.
#pragma once

namespace g1prep {

constexpr int PREP_THREADS = 256;

__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// gl = (float)(gamma * lam) computed on the host in double, as Python does before torch sees it
__global__ void __launch_bounds__(PREP_THREADS) k_gae(int H, int N, const float* __restrict__ R,
                                                      const float* __restrict__ V, const float* __restrict__ D,
                                                      const float* __restrict__ Vlast, float g, float gl,
                                                      float* __restrict__ adv, float* __restrict__ ret,
                                                      double* __restrict__ mom) {
    __shared__ double s_sum[PREP_THREADS / 32], s_sq[PREP_THREADS / 32];
    const int w = blockIdx.x * blockDim.x + threadIdx.x;
    double a1 = 0.0, a2 = 0.0;
    if (w < N) {
        float gae = 0.f;
        float nextv = Vlast[w];
        for (int t = H - 1; t >= 0; --t) {
            const size_t i = (size_t)t * N + w;
            const float vt = V[i];
            const float nd = __fsub_rn(1.f, D[i]);
            // delta = R[t] + gamma * nextv * (1 - D[t]) - V[t]
            const float delta = __fsub_rn(__fadd_rn(R[i], __fmul_rn(__fmul_rn(g, nextv), nd)), vt);
            // gae = delta + gamma * lam * (1 - D[t]) * gae
            gae = __fadd_rn(delta, __fmul_rn(__fmul_rn(gl, nd), gae));
            adv[i] = gae;
            ret[i] = __fadd_rn(gae, vt);
            a1 += (double)gae;
            a2 += (double)gae * (double)gae;
            nextv = vt;
        }
    }
    a1 = warp_sum_d(a1);
    a2 = warp_sum_d(a2);
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    if (lane == 0) { s_sum[wid] = a1; s_sq[wid] = a2; }
    __syncthreads();
    if (threadIdx.x == 0) {
        double t1 = 0.0, t2 = 0.0;
        for (int k = 0; k < PREP_THREADS / 32; ++k) { t1 += s_sum[k]; t2 += s_sq[k]; }
        atomicAdd(&mom[1], t1);
        atomicAdd(&mom[2], t2);
        if (blockIdx.x == 0) atomicAdd(&mom[0], (double)H * (double)N);
    }
}

__device__ __forceinline__ float norm1(float o, float m, float v) {
    float x = __fdiv_rn(__fsub_rn(o, m), __fsqrt_rn(__fadd_rn(v, 1e-8f)));
    return fminf(fmaxf(x, -10.f), 10.f);
}

// VEC = 4: dim % 4 == 0 and 16-byte aligned O / nobs; VEC = 1 otherwise.
// Dynamic shared memory: 2*dim doubles.
template <int VEC>
__global__ void __launch_bounds__(PREP_THREADS) k_obs_prep(long long rows, int dim, const float* __restrict__ O,
                                                           const float* __restrict__ fmean,
                                                           const float* __restrict__ fvar, float* __restrict__ nobs,
                                                           double* __restrict__ mom) {
    extern __shared__ double s_acc[];  // [2*dim]
    const int ncol = dim / VEC;
    const int rpb = PREP_THREADS / ncol;  // rows per block pass
    for (int i = threadIdx.x; i < 2 * dim; i += PREP_THREADS) s_acc[i] = 0.0;
    __syncthreads();
    const int c = threadIdx.x % ncol, rl = threadIdx.x / ncol;
    if (rl < rpb) {
        float m[VEC], v[VEC];
        double s1[VEC], s2[VEC];
#pragma unroll
        for (int q = 0; q < VEC; ++q) { m[q] = fmean[c * VEC + q]; v[q] = fvar[c * VEC + q]; s1[q] = 0.0; s2[q] = 0.0; }
        const long long step = (long long)gridDim.x * rpb;
        for (long long r = (long long)blockIdx.x * rpb + rl; r < rows; r += step) {
            const size_t off = (size_t)r * dim + (size_t)c * VEC;
            float o[VEC], y[VEC];
            if (VEC == 4) {
                const float4 t = __ldcs(reinterpret_cast<const float4*>(O + off));
                o[0] = t.x; o[1] = t.y; o[2] = t.z; o[3] = t.w;
            } else {
                o[0] = __ldcs(O + off);
            }
#pragma unroll
            for (int q = 0; q < VEC; ++q) {
                y[q] = norm1(o[q], m[q], v[q]);
                s1[q] += (double)o[q];
                s2[q] += (double)o[q] * (double)o[q];
            }
            if (VEC == 4) __stcs(reinterpret_cast<float4*>(nobs + off), make_float4(y[0], y[1], y[2], y[3]));
            else __stcs(nobs + off, y[0]);
        }
#pragma unroll
        for (int q = 0; q < VEC; ++q) {
            atomicAdd(&s_acc[c * VEC + q], s1[q]);
            atomicAdd(&s_acc[dim + c * VEC + q], s2[q]);
        }
    }
    __syncthreads();
    for (int i = threadIdx.x; i < 2 * dim; i += PREP_THREADS) atomicAdd(&mom[1 + i], s_acc[i]);
    if (blockIdx.x == 0 && threadIdx.x == 0) atomicAdd(&mom[0], (double)rows);
}

__global__ void __launch_bounds__(PREP_THREADS) k_adv_norm(long long n, float* __restrict__ adv,
                                                           const double* __restrict__ mom) {
    const double cnt = mom[0], mean = mom[1] / cnt;
    double var = (mom[2] - cnt * mean * mean) / fmax(cnt - 1.0, 1.0);  // unbiased (torch.std)
    const float std = (float)sqrt(fmax(var, 0.0));
    const float mf = (float)mean, den = std + 1e-8f;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
        adv[i] = (adv[i] - mf) / den;
}

// RunNorm.update (ppo.py:71-79) with the batch mean/var from the moments; count = the
// normaliser's count before this update (kept by the host, as the reference's is)
__global__ void k_runnorm(int dim, float* __restrict__ mean, float* __restrict__ var, double count,
                          const double* __restrict__ mom) {
    const int d = blockIdx.x * blockDim.x + threadIdx.x;
    if (d >= dim) return;
    const double b = mom[0];
    const double bm = mom[1 + d] / b;
    const double bv = fmax(mom[1 + dim + d] / b - bm * bm, 0.0);
    const double tot = count + b;
    const double m0 = (double)mean[d], v0 = (double)var[d];
    const double delta = bm - m0;
    mean[d] = (float)(m0 + delta * b / tot);
    var[d] = (float)((v0 * count + bv * b + delta * delta * count * b / tot) / tot);
}

}  // namespace g1prep

extern "C" {

// extension: GAE (ppo_fused.py:108-116).  DEVICE pointers R/V/D [H,N], Vlast [N] -> adv, ret
// [H,N]; adv_mom (fp64 [3]) <- [H*N, sum adv, sum adv^2].  Asynchronous on `stream`.
int g1_gae(int H, int N, const float* R, const float* V, const float* D, const float* Vlast, double gamma, double lam,
           float* adv, float* ret, double* adv_mom, void* stream) {
    if (H <= 0 || N <= 0) { set_error(-22, "g1_gae", "invalid shape"); return -22; }
    cudaStream_t s = (cudaStream_t)stream;
    cudaError_t e = cudaMemsetAsync(adv_mom, 0, 3 * sizeof(double), s);
    if (e == cudaSuccess) {
        g1prep::k_gae<<<(N + g1prep::PREP_THREADS - 1) / g1prep::PREP_THREADS, g1prep::PREP_THREADS, 0, s>>>(
            H, N, R, V, D, Vlast, (float)gamma, (float)(gamma * lam), adv, ret, adv_mom);
        e = cudaGetLastError();
    }
    if (e != cudaSuccess) { set_error((int)e, "g1_gae", cudaGetErrorString(e)); return -1; }
    return 0;
}

// extension: observation renormalisation with the frozen statistics plus the raw moments
// (ppo_fused.py:104-106).  O, nobs [rows][dim]; obs_mom (fp64 [1 + 2*dim]) <- [rows, sum o,
// sum o^2].  nobs may not alias O.  Asynchronous on `stream`.
int g1_obs_prep(long long rows, int dim, const float* O, const float* fmean, const float* fvar, float* nobs,
                double* obs_mom, void* stream) {
    if (rows <= 0 || dim <= 0 || dim > g1prep::PREP_THREADS * 4) {
        set_error(-22, "g1_obs_prep", "invalid shape");
        return -22;
    }
    cudaStream_t s = (cudaStream_t)stream;
    int dev = 0, nsm = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
    cudaError_t e = cudaMemsetAsync(obs_mom, 0, (1 + 2 * (size_t)dim) * sizeof(double), s);
    const bool vec = (dim % 4 == 0) && (((uintptr_t)O | (uintptr_t)nobs) % 16 == 0) && dim / 4 <= g1prep::PREP_THREADS;
    const int ncol = vec ? dim / 4 : dim;
    if (!vec && dim > g1prep::PREP_THREADS) { set_error(-22, "g1_obs_prep", "dim too large for the scalar path"); return -22; }
    const int rpb = g1prep::PREP_THREADS / ncol;
    long long want = (rows + rpb - 1) / rpb;
    // enough blocks to fill every SM several times; each block's partial sums cost 2*dim atomics
    long long grid = std::min<long long>(want, (long long)nsm * 8);
    const size_t smem = 2 * (size_t)dim * sizeof(double);
    if (e == cudaSuccess) {
        if (vec)
            g1prep::k_obs_prep<4><<<(int)grid, g1prep::PREP_THREADS, smem, s>>>(rows, dim, O, fmean, fvar, nobs, obs_mom);
        else
            g1prep::k_obs_prep<1><<<(int)grid, g1prep::PREP_THREADS, smem, s>>>(rows, dim, O, fmean, fvar, nobs, obs_mom);
        e = cudaGetLastError();
    }
    if (e != cudaSuccess) { set_error((int)e, "g1_obs_prep", cudaGetErrorString(e)); return -1; }
    return 0;
}

// extension: b_adv = (adv - mean) / (std + 1e-8) in place (ppo_fused.py:119), mean and the
// unbiased std from adv_mom (possibly summed over ranks).  Asynchronous on `stream`.
int g1_adv_normalize(long long n, float* adv, const double* adv_mom, void* stream) {
    if (n <= 0) { set_error(-22, "g1_adv_normalize", "invalid size"); return -22; }
    long long grid = std::min<long long>((n + g1prep::PREP_THREADS - 1) / g1prep::PREP_THREADS, 148 * 8);
    g1prep::k_adv_norm<<<(int)grid, g1prep::PREP_THREADS, 0, (cudaStream_t)stream>>>(n, adv, adv_mom);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) { set_error((int)e, "g1_adv_normalize", cudaGetErrorString(e)); return -1; }
    return 0;
}

// extension: RunNorm.update (ppo.py:71-79) in place on mean/var [dim] from obs_mom (possibly
// summed over ranks); `count` is the normaliser's count before the update -- the caller adds
// the batch size to its own copy, as the reference's host-side count does.
int g1_runnorm_update(int dim, float* mean, float* var, double count, const double* obs_mom, void* stream) {
    if (dim <= 0) { set_error(-22, "g1_runnorm_update", "invalid size"); return -22; }
    g1prep::k_runnorm<<<(dim + 127) / 128, 128, 0, (cudaStream_t)stream>>>(dim, mean, var, count, obs_mom);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) { set_error((int)e, "g1_runnorm_update", cudaGetErrorString(e)); return -1; }
    return 0;
}

}  // extern "C"
