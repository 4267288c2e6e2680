/*
 * g1env.h -- C-ABI of libg1env.so, the B200 (sm_100a) fused G1 rollout.
 *
 * Drop-in for the reference's ctypes library build/libg1env.so (Infatoshi/g1.cu,
 * src/g1_env.cu:361-476): every reference export keeps its name, argument types, buffer
 * layouts and ownership, so scripts/ppo.py and scripts/ppo_fused.py bind it unchanged.
 * Additions (g1_env_*_ex / _device / _last_error / state access / g1_qacc_batch) are
 * marked "extension".
 *
 * Conventions (as the reference):
 *   - N worlds; OBS = 100, ACT = 29; NQ = 36, NV = 35 (MuJoCo qpos/qvel order).
 *   - Trajectory buffers are world-major rows: O[H,N,100], A[H,N,29], LP/V/R/D[H,N],
 *     Vlast[N], float32, done flags stored as 0.0/1.0.
 *   - Policy weights W: one float32 buffer in torch parameter order, per hidden layer
 *     W[out,in] row-major then bias; then Wmu[29,h], bmu[29], Wv[1,h], bv[1], log_std[29]
 *     (ppo_fused.py:35-44).
 *   - Errors: functions keep the reference's void returns; a failure is recorded and can be
 *     read with g1_env_last_error() (the reference prints and calls exit(1),
 *     g1_env.cu:33-34).  Functions returning int return 0 on success.
 */
#ifndef G1ENV_H
#define G1ENV_H
#ifdef __cplusplus
extern "C" {
#endif

/* replaces g1_env_create, g1_env.cu:405-422.  Allocates device state on the current
 * device and places every world at the stand pose; returns NULL on failure. */
void* g1_env_create(int n_worlds, int substeps, int pgs_iters, unsigned long seed);

/* extension: explicit device ordinal (-1 = current), global id of world 0 (world shards of
 * a multi-GPU job draw disjoint RNG streams), and foot friction mu (the reference
 * hard-codes 0.6 in g1_model.h:420). */
void* g1_env_create_ex(int n_worlds, int substeps, int pgs_iters, unsigned long seed, int device,
                       unsigned int world0, float mu);

/* replaces g1_env_destroy, g1_env.cu:469-474 */
void g1_env_destroy(void* h);

/* replaces g1_env_reset, g1_env.cu:424-429.  obs_out: HOST [N*100] (may be NULL). */
void g1_env_reset(void* h, float* obs_out);

/* replaces g1_env_step, g1_env.cu:431-441.  HOST pointers: act [N*29] -> obs [N*100],
 * rew [N], done [N]; synchronous. */
void g1_env_step(void* h, const float* act, float* obs, float* rew, float* done);

/* extension: g1_env_step on DEVICE pointers, asynchronous on the env stream. */
void g1_env_step_device(void* h, const float* act, float* obs, float* rew, float* done);

/* replaces g1_rollout, g1_env.cu:446-453.  DEVICE pointers (torch-owned); asynchronous on
 * the env stream (default: the legacy default stream, as the reference). */
void g1_rollout(void* h, int H, const float* W, const float* mean, const float* var, float* O, float* A,
                float* LP, float* V, float* R, float* D, float* Vlast);

/* extension, no counterpart in the reference: g1_rollout that allocates nothing, for callers
 * that must not allocate device memory on their hot path (a host allocator that owns all
 * device memory, a pre-reserved memory budget, or code running while a stream is captured).
 * The repacked policy weights live in a fixed 512 KiB device area (131,072 floats) shared by
 * all calls and all envs on a device: policies needing more are rejected (last error set),
 * and calls that overlap on the GPU race on the area.  The first call on each device looks
 * up the area's address; make it before any stream capture.  Arguments as g1_rollout.
 * The policy always runs on the in-kernel FFMA contraction, so results equal g1_rollout's
 * under precision 2 ("fp32-ffma") and differ slightly (rounding) from its default tensor-core
 * MLP.  Envs set to precision 1 or given a separate value network are rejected. */
void g1_rollout_noalloc(void* h, int H, const float* W, const float* mean, const float* var, float* O, float* A,
                        float* LP, float* V, float* R, float* D, float* Vlast);

/* replaces g1_env_bench_phys, g1_env.cu:385-389: K control steps with zero action, synchronous. */
void g1_env_bench_phys(void* h, int K);

/* extension: asynchronous g1_env_bench_phys (timing with events on the env stream). */
void g1_env_phys_async(void* h, int K);

/* extension: K control steps of physics only with a constant action per
 * world, act = DEVICE [N, 29] (NULL = zero actions, as g1_env_bench_phys); asynchronous on the
 * env's stream.  The actions go through the rollout's PD-target path (g1_env.cu:123-152). */
void g1_env_phys_actions(void* h, int K, const float* act);

/* replaces g1_env_qpos / g1_env_qpos_all, g1_env.cu:457-467 (HOST out [36] / [N*36]). */
void g1_env_qpos(void* h, float* out);
void g1_env_qpos_all(void* h, float* out);

/* replaces g1_env_obs_dim / g1_env_act_dim, g1_env.cu:391-392 */
int g1_env_obs_dim(void);
int g1_env_act_dim(void);

/* replaces g1_occupancy_report, g1_env.cu:365-382 (prints) */
void g1_occupancy_report(void);

/* extension: error reporting in place of exit(1).  NULL / 0 when no error is pending. */
const char* g1_env_last_error(void);
int g1_env_last_error_code(void);
void g1_env_clear_error(void);

/* extension: stream for all asynchronous work of this env (a cudaStream_t; NULL = legacy default). */
void g1_env_set_stream(void* h, void* stream);

/* extension: policy architecture used by g1_rollout: nh hidden layers (1..4, even widths
 * <= 1024), activation 0 = tanh (the reference's AC, ppo.py:85-99), 1 = ELU. */
int g1_env_set_policy(void* h, int nh, const int* hidden, int activation);

/* extension: policy_precision 1 runs the MLP on the tensor cores (tcgen05, bf16 weights and
 * activations, fp32 accumulation) as separate launches per control step, for wide policies
 * (widths multiple of 8, up to 1024); 0 = the fp32 in-kernel policy of
 * g1_env_set_policy (computed with split-bf16 operands on the tensor cores -- fp32-class
 * accuracy -- when
 * every hidden width is a multiple of 16 in [16, 256], on FFMA otherwise); 2 = the fp32
 * in-kernel policy always on FFMA.  Returns 0 on success. */
int g1_env_set_policy_ex(void* h, int nh, const int* hidden, int activation, int policy_precision);

/* extension: a separate value network of nh hidden layers (widths multiples
 * of 8 in [8, 1024], the policy's activation), used by g1_rollout with policy_precision 1;
 * nh = 0 returns to the shared trunk's value head (the reference's AC, ppo.py:85-99).  With a
 * value network the packed weights are [policy hidden layers W, b][Wmu][bmu][log_std][value
 * hidden layers W, b][Wv (1 x last)][bv].  Returns 0 on success. */
int g1_env_set_value_net(void* h, int nh, const int* hidden);

/* extension: nonzero if a tensor-core wait of the bf16 policy path timed out since the last
 * call (synchronous; clears the flag). */
int g1_env_tc_status(void* h);

/* extension: foot friction coefficient mu of the pyramidal cone (default 0.6). */
void g1_env_set_friction(void* h, float mu);

/* extension: HOST state access: qp [N*36], qv [N*35], prev_act [N*29], steps [N], control
 * tick (the RNG counter).  NULL pointers are skipped.  Synchronous. */
void g1_env_get_state(void* h, float* qp, float* qv, float* pa, int* steps, unsigned long long* tick);
void g1_env_set_state(void* h, const float* qp, const float* qv, const float* pa, const int* steps,
                      unsigned long long tick);

/* extension: contact-count histogram over substeps (ncon 0..8).  enable=1 (re)starts
 * counting; out (HOST [9], may be NULL) receives the counts so far. */
void g1_env_ncon_hist(void* h, int enable, unsigned long long* out);

/* extension: per-state forward kinematics + generalized acceleration (the per-substep
 * parity gate; semantics of the reference's src/test_envqacc.cu:29-51 with caller states).
 * DEVICE pointers: qpos [n*36], qvel/tau/bdt [n*35] (tau, bdt may be NULL = 0) ->
 * qacc, qacc_smooth, bias [n*35], f [n*32] contact impulses, ncon [n] (outputs may be NULL). */
int g1_qacc_batch(int n, const float* qpos, const float* qvel, const float* tau, const float* bdt, int pgs_iters,
                  float mu, float* qacc, float* qacc_smooth, float* bias, float* f, int* ncon);

/* extension: one dense policy layer out = act(X W^T + b) on the tensor cores (tcgen05, bf16
 * X [M][K] (row stride ldx) and W [N][K], fp32 bias [N] or NULL, fp32 out [M][N]; act 0 tanh,
 * 1 ELU, -1 identity).  DEVICE pointers; synchronous; 0 on success.  The building block of
 * the large-policy rollout (reference counterpart: the per-world mlp_forward layers,
 * g1_env.cu:229-237, batched over worlds). */
int g1_gemm_bf16_tc(int M, int N, int K, const void* X, int ldx, const void* W, const float* bias, int act, float* out);

/* extension: the fp32 policy layer of the fused rollout as a standalone call -- out = act(X W^T
 * + b) on the tensor cores with both operands split into three bf16 words (tcgen05 kind::f16,
 * the six significant cross products, fp32 accumulation: fp32-class accuracy), rows <= 64,
 * 16 <= N <= 256 with N % 16 == 0, K <= 256.  DEVICE pointers X
 * [rows][K], W [N][K], b [N] or NULL, out [rows][N]; act 0 tanh, 1 ELU, -1 identity;
 * synchronous; 0 on success.  Reference counterpart: one mlp_forward layer (g1_env.cu:229-237)
 * for a block of worlds. */
int g1_dense_bf16x3(int rows, int K, int N, const float* X, const float* W, const float* b, int act, float* out);

/* extension: the trainer's batch preparation on the GPU, fed from the rollout buffers
 * (reference counterpart: the Python GAE loop and torch reductions of scripts/ppo_fused.py:104-119
 * and RunNorm.update, scripts/ppo.py:71-79).  DEVICE pointers, asynchronous on `stream`
 * (a cudaStream_t; NULL = legacy default stream), 0 on success.  Moment buffers are fp64 and
 * zeroed by the producing call; several ranks may sum theirs (all-reduce) before the
 * finalising calls.
 *   g1_gae            adv/ret [H,N] from R/V/D [H,N], Vlast [N]; bit-identical to the torch loop;
 *                     adv_mom[3] = {H*N, sum adv, sum adv^2}
 *   g1_obs_prep       nobs = clamp((O - fmean)/sqrt(fvar + 1e-8), -10, 10) over O [rows][dim];
 *                     obs_mom[1 + 2*dim] = {rows, sum o[dim], sum o^2[dim]} of the raw O
 *   g1_adv_normalize  adv = (adv - mean)/(std + 1e-8), unbiased std, in place
 *   g1_runnorm_update mean/var [dim] updated in place; count = the count before the update */
int g1_gae(int H, int N, const float* R, const float* V, const float* D, const float* Vlast, double gamma, double lam,
           float* adv, float* ret, double* adv_mom, void* stream);
int g1_obs_prep(long long rows, int dim, const float* O, const float* fmean, const float* fvar, float* nobs,
                double* obs_mom, void* stream);
int g1_adv_normalize(long long n, float* adv, const double* adv_mom, void* stream);
int g1_runnorm_update(int dim, float* mean, float* var, double count, const double* obs_mom, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* G1ENV_H */
