// g1_physics.cuh -- per-substep G1 dynamics, GW worlds per warp, frames in shared memory.
//
// The reference runs a world per thread and keeps its ~25 KB working set in local memory
// (g1_env.cu:245, "255 regs, ~25-31 KB local frame").  Here a warp advances GW = 4 worlds
// together with their frames in shared memory, and splits the work over independent items:
//   tree sweeps (FK, RNE, factor, smooth solve)  one lane per (world, chain of the tree)
//   contact detection                            one lane per (world, foot sphere)
//   contact solve, one world at a time:
//     M^-1 of the contact basis                  one lane per basis column (<= 24)
//     Gram / Delassus blocks                     one lane per (contact pair, entry)
//     PGS                                        one lane per constraint row, rows in order
//   integration                                  one lane per (world, dof / joint)
// Within each item the arithmetic follows the reference's order (citations per function),
// so results agree with it to fp32 rounding.
#pragma once
#include "g1_tables.cuh"

#define FULLMASK 0xffffffffu

namespace g1 {

constexpr int NB = G1_NB, NV = G1_NV_, NQ = G1_NQ_, NJ = G1_NJ, NU = G1_NU_, NFOOT = G1_NFOOT_;
constexpr int MAXCON = G1_MAXCON, MAXEFC = G1_MAXEFC, CDS = G1_CDS, NRHS = G1_NRHS;

// ------------------------------------------------------------------ small algebra
struct V3 { float x, y, z; };
struct Q4 { float w, x, y, z; };
__device__ __forceinline__ V3 mk3(float x, float y, float z) { return {x, y, z}; }
__device__ __forceinline__ V3 add3(V3 a, V3 b) { return {a.x + b.x, a.y + b.y, a.z + b.z}; }
__device__ __forceinline__ V3 sub3(V3 a, V3 b) { return {a.x - b.x, a.y - b.y, a.z - b.z}; }
__device__ __forceinline__ V3 cross3(V3 a, V3 b) {
    return {a.y * b.z - a.z * b.y, a.z * b.x - a.x * b.z, a.x * b.y - a.y * b.x};
}
__device__ __forceinline__ float dot3(V3 a, V3 b) { return a.x * b.x + a.y * b.y + a.z * b.z; }
__device__ __forceinline__ V3 ld3(const float* p) { return {p[0], p[1], p[2]}; }
__device__ __forceinline__ void st3(float* p, V3 v) { p[0] = v.x; p[1] = v.y; p[2] = v.z; }
__device__ __forceinline__ Q4 ld4(const float* p) { return {p[0], p[1], p[2], p[3]}; }
// six floats [a; b] at an 8-byte aligned address, as three float2 stores
__device__ __forceinline__ void st6(float* p, V3 a, V3 b) {
    float2* q = reinterpret_cast<float2*>(p);
    q[0] = make_float2(a.x, a.y); q[1] = make_float2(a.z, b.x); q[2] = make_float2(b.y, b.z);
}
__device__ __forceinline__ void st4(float* p, Q4 q) { p[0] = q.w; p[1] = q.x; p[2] = q.y; p[3] = q.z; }
// Hamilton product (dynamics.cuh:17-24)
__device__ __forceinline__ Q4 qmul(Q4 a, Q4 b) {
    return {a.w * b.w - a.x * b.x - a.y * b.y - a.z * b.z, a.w * b.x + a.x * b.w + a.y * b.z - a.z * b.y,
            a.w * b.y - a.x * b.z + a.y * b.w + a.z * b.x, a.w * b.z + a.x * b.y - a.y * b.x + a.z * b.w};
}
// rotate v by q (dynamics.cuh:26-35)
__device__ __forceinline__ V3 qrot(Q4 q, V3 v) {
    float tx = 2.f * (q.y * v.z - q.z * v.y), ty = 2.f * (q.z * v.x - q.x * v.z), tz = 2.f * (q.x * v.y - q.y * v.x);
    return {v.x + q.w * tx + (q.y * tz - q.z * ty), v.y + q.w * ty + (q.z * tx - q.x * tz),
            v.z + q.w * tz + (q.x * ty - q.y * tx)};
}
__device__ __forceinline__ Q4 qnormalize(Q4 q) {  // dynamics.cuh:36-39
    float n = rsqrtf(q.w * q.w + q.x * q.x + q.y * q.y + q.z * q.z);
    return {q.w * n, q.x * n, q.y * n, q.z * n};
}
__device__ __forceinline__ void qmat(Q4 q, float* m) {  // dynamics.cuh:99-106
    float w = q.w, x = q.x, y = q.y, z = q.z;
    m[0] = 1 - 2 * (y * y + z * z); m[1] = 2 * (x * y - w * z);     m[2] = 2 * (x * z + w * y);
    m[3] = 2 * (x * y + w * z);     m[4] = 1 - 2 * (x * x + z * z); m[5] = 2 * (y * z - w * x);
    m[6] = 2 * (x * z - w * y);     m[7] = 2 * (y * z + w * x);     m[8] = 1 - 2 * (x * x + y * y);
}
__device__ __forceinline__ int sym6(int i, int j) {  // aba.cuh:20-23
    if (i > j) { int t = i; i = j; j = t; }
    return i * 6 - (i * (i - 1)) / 2 + (j - i);
}
// (Iw, c, m) applied to motion [w; v]  (dynamics.cuh:126-139)
__device__ __forceinline__ void inertia_apply(const float* Iw, V3 c, float m, V3 sw, V3 sv, V3& fw, V3& fv) {
    V3 A = {Iw[0] * sw.x + Iw[1] * sw.y + Iw[2] * sw.z, Iw[3] * sw.x + Iw[4] * sw.y + Iw[5] * sw.z,
            Iw[6] * sw.x + Iw[7] * sw.y + Iw[8] * sw.z};
    float cc = dot3(c, c), csw = dot3(c, sw);
    A = {A.x + m * (cc * sw.x - csw * c.x), A.y + m * (cc * sw.y - csw * c.y), A.z + m * (cc * sw.z - csw * c.z)};
    V3 a = cross3(c, sv);
    fw = {A.x + m * a.x, A.y + m * a.y, A.z + m * a.z};
    V3 b = cross3(c, sw);
    fv = {-m * b.x + m * sv.x, -m * b.y + m * sv.y, -m * b.z + m * sv.z};
}

// ------------------------------------------------------------------ tree sweeps
// Spatial inertia of body b about the pelvis origin p, packed symmetric 6x6 (21), from its
// world rotational inertia Iw and com offset c (aba_factor.cuh:53-74).
__device__ __forceinline__ void spatial_inertia21(const float* Iw, V3 c, float m, float* X) {
    float cc = dot3(c, c);
    float A[9];
#pragma unroll
    for (int i = 0; i < 9; ++i) A[i] = Iw[i];
    A[0] += m * (cc - c.x * c.x); A[1] += m * (-c.x * c.y); A[2] += m * (-c.x * c.z);
    A[3] += m * (-c.y * c.x);     A[4] += m * (cc - c.y * c.y); A[5] += m * (-c.y * c.z);
    A[6] += m * (-c.z * c.x);     A[7] += m * (-c.z * c.y); A[8] += m * (cc - c.z * c.z);
    const float sk[9] = {0, -c.z, c.y, c.z, 0, -c.x, -c.y, c.x, 0};
#pragma unroll
    for (int i = 0; i < 3; ++i)
#pragma unroll
        for (int j = i; j < 3; ++j) X[sym6(i, j)] = A[3 * i + j];
#pragma unroll
    for (int i = 0; i < 3; ++i)
#pragma unroll
        for (int j = 0; j < 3; ++j) X[sym6(i, j + 3)] = m * sk[3 * i + j];
#pragma unroll
    for (int i = 0; i < 3; ++i)
#pragma unroll
        for (int j = i; j < 3; ++j) X[sym6(i + 3, j + 3)] = (i == j) ? m : 0.f;
}

// world rotational inertia R diag(d) R^T and com offset (dynamics.cuh:108-115,
// aba_bias.cuh:400-410)
__device__ __forceinline__ void world_inertia(const G1Tables& T, int b, Q4 quat, V3 xip, V3 p, float* Iw, V3& c) {
    float Rm[9];
    qmat(qmul(quat, ld4(T.body_iquat + 4 * b)), Rm);
    const float d0 = T.body_inertia[3 * b], d1 = T.body_inertia[3 * b + 1], d2 = T.body_inertia[3 * b + 2];
#pragma unroll
    for (int i = 0; i < 3; ++i)
#pragma unroll
        for (int k = 0; k < 3; ++k)
            Iw[3 * i + k] = Rm[3 * i] * d0 * Rm[3 * k] + Rm[3 * i + 1] * d1 * Rm[3 * k + 1] + Rm[3 * i + 2] * d2 * Rm[3 * k + 2];
    c = sub3(xip, p);
}

// body force f = I a + v x* (I v)  (aba_bias.cuh:458-466)
__device__ __forceinline__ void body_force(const float* Iw, V3 c, float m, V3 vw, V3 vv, V3 aw, V3 av, V3& fw, V3& fv) {
    V3 Iaw, Iav, Ivw, Ivv;
    inertia_apply(Iw, c, m, aw, av, Iaw, Iav);
    inertia_apply(Iw, c, m, vw, vv, Ivw, Ivv);
    V3 cn = add3(cross3(vw, Ivw), cross3(vv, Ivv)), cf = cross3(vw, Ivv);
    fw = add3(Iaw, cn);
    fv = add3(Iav, cf);
}

// ------------------------------------------------------------------ frame layouts
// A warp advances GW worlds together.  Each world has its own frame (WL) in shared memory;
// the warp has one contact workspace (CL) that its worlds use one after another.
constexpr int GW = 4;        // worlds per warp
constexpr int CPW = 4;       // chain lanes per world in the tree sweeps (lane = 4 w + chain)
static_assert(GW * CPW <= 32, "lanes");

struct WL {  // per-world frame, offsets in floats
    enum : int {
        QP = 0,               // qpos [36]
        QV = 36,              // qvel [35] (+1)
        TGT = 72,             // PD targets [29] (+3)
        TAU = 104,            // generalised force [35] (+1)
        QACC = 140,           // qacc_smooth, then qacc [35] (+1)
        S = 176,              // motion axes [35][6]
        FU = 386,             // factor U [31][6]
        FINVD = 572,          // factor 1/D [31] (+1)
        FU6 = 604,            // base U6 [36]
        FL6 = 640,            // base Dm -> Cholesky factor [36]
        XS = 676,             // kept body frames (pelvis, feet): quat [4] + pos [3] (+1) per slot
        BQ = 708,             // per body (F1 -> B1): world rotational inertia, upper triangle
                              // [xx xy xz yy yz zz], then xipos - p [3]
        FOWN = BQ + 280,      // per body: own force, then subtree force [31][6]
        HF = FOWN + 186,      // F1 branch hand-off: pos, quat, w, v, aw, av [19] (+1) per branch slot
        HA = HF + 20 * G1_MAXBRANCH,   // F2 branch hand-off: spatial acceleration [6] (+2)
        HB = HA + 8 * G1_MAXBRANCH,    // B1 chain-head contributions: IA [21], f [6], pA [6] (+3)
        A1 = HB + 36 * 4,     // base spatial acceleration [6] (+2)
        CON = A1 + 8,         // contacts: sphere (int) [8], pt [8][3], pen [8]
        MISC = CON + 40,      // [0] ncon (int)
        SIZE = MISC + 4
    };
};
struct CL {  // per-warp contact workspace, offsets in floats
    enum : int {
        MM = 0,                       // M^-1 of the 3 ncon basis rows [24][35]
        EB = MM + 3 * G1_MAXCON * 35, // basis rows [8][3][12]
        RR = EB + 288,                // R [32]
        BV = RR + 32,                 // b [32]
        FF = BV + 32,                 // f [32]
        GRAM = FF + 32,               // 3x3 Gram blocks [36][9]
        AP = GRAM + 324,              // Delassus matrix, packed upper triangle [528]
        SCR_END = GRAM + 24 * 36,     // per-lane back-solve scratch aliases GRAM/AP (24 lanes x 36)
        SIZE = (AP + 528 > SCR_END) ? AP + 528 : SCR_END
    };
};
constexpr int WFLOATS = (WL::SIZE + 3) & ~3;
static_assert(WL::S % 2 == 0 && WL::FU % 2 == 0 && WL::FOWN % 2 == 0,
              "S, U and force rows are accessed as float2 (frames are 16-byte aligned)");
constexpr int CFLOATS = (CL::SIZE + 3) & ~3;
constexpr int GROUP_FLOATS = GW * WFLOATS + CFLOATS;
constexpr int MSTR = 35;
constexpr int SOLVE_SCRATCH = 6 * (4 + G1_MAXBRANCH);  // per solving lane, aliases GRAM/AP
static_assert(3 * G1_MAXCON * SOLVE_SCRATCH <= CL::SIZE - CL::GRAM, "solve scratch must fit in GRAM/AP");
__device__ __forceinline__ int apidx(int i, int j) {  // packed upper triangle of a 32x32 symmetric matrix
    int a = min(i, j), b = max(i, j);
    return a * 32 - (a * (a - 1)) / 2 + (b - a);
}

// ------------------------------------------------------------------ profiling (G1_PROF builds)
#ifdef G1_PROF
__device__ unsigned long long g_prof[64];
#define PROF_BEGIN() long long _pt = clock64();
#define PROF_RESTART() _pt = clock64();
#define PROF_MARK(i)                                                                          \
    do {                                                                                      \
        long long _n = clock64();                                                             \
        if ((threadIdx.x & 31) == 0) atomicAdd(&g_prof[i], (unsigned long long)(_n - _pt));   \
        _pt = _n;                                                                             \
    } while (0)
#else
#define PROF_BEGIN()
#define PROF_RESTART()
#define PROF_MARK(i) do { } while (0)
#endif
enum ProfPhase { P_POLICY = 0, P_F1, P_B1, P_BASE, P_F2, P_CSETUP, P_SOLVE, P_GRAM, P_PGS, P_DQ, P_STEP, P_WAIT, P_INTEG, P_DETECT, P_MLP, P_SAMPLE, P_MLP_L1, P_MLP_HEAD, P_BAR, P_ENERGY, P_TF_MMA, P_TF_EPI, P_CS_LOAD, P_CS_REWARD, P_CS_STORE, P_SORT, P_TOTAL, P_LS_BACK, P_LS_BASE, P_LS_FWD, P_TF_EPI1, P_TF_EPI2, P_F1B, P_BASE_PULL, P_BASE_DM, P_MIDBAR, P_NPHASE };

// pyramid coefficients d_k = DC[k] of the 3-basis (env_qacc.cuh:98-100,154-155)
__device__ __forceinline__ float dcoef(int k, int a) {
    if (a == 0) return 1.f;
    if (a == 1) return k == 0 ? 1.f : (k == 1 ? -1.f : 0.f);
    return k == 2 ? 1.f : (k == 3 ? -1.f : 0.f);
}

// ------------------------------------------------------------------ tree sweeps
// body force of body b from its frame and spatial velocity / acceleration, also keeping the
// upper triangle of its world inertia and its com offset in bi[9] for the leaf -> root sweep
__device__ __forceinline__ void body_force_keep(const G1Tables& T, int b, Q4 quat, V3 cpos, V3 w, V3 v, V3 aw, V3 av,
                                                float* f_out, float* bi) {
    float Iw[9];
    V3 c;
    world_inertia(T, b, quat, cpos, mk3(0, 0, 0), Iw, c);
    bi[0] = Iw[0]; bi[1] = Iw[1]; bi[2] = Iw[2]; bi[3] = Iw[4]; bi[4] = Iw[5]; bi[5] = Iw[8];
    st3(bi + 6, c);
    V3 fw, fv;
    body_force(Iw, c, T.body_mass[b], w, v, aw, av, fw, fv);
    st6(f_out, fw, fv);
}
// spatial inertia (packed 21) of body b from the kept world inertia (upper triangle -- the
// only entries spatial_inertia21 reads) and com offset
__device__ __forceinline__ void body_ia_kept(const G1Tables& T, int b, const float* bi, float* ia) {
    const float Iw[9] = {bi[0], bi[1], bi[2], bi[1], bi[3], bi[4], bi[2], bi[4], bi[5]};
    spatial_inertia21(Iw, ld3(bi + 6), T.body_mass[b], ia);
}

// F1's hand-off to its second pass for body b: orientation to qs[4], position and spatial
// velocity to bi[9] (the body's kept-inertia row), spatial acceleration to f[6] (its force row)
__device__ __forceinline__ void stash_body(float* qs, Q4 quat, V3 pos, V3 w, V3 v, V3 aw, V3 av, float* f, float* bi) {
    st4(qs, quat);
    st3(bi, pos); st3(bi + 3, w); st3(bi + 6, v);
    st6(f, aw, av);
}
static_assert(4 * GW * NB <= CL::SIZE, "F1's orientation stash must fit in the contact workspace");

// The smooth part of the per-substep dynamics for the GW worlds of a warp (qp, qv, tau in each
// world frame): forward kinematics, motion axes S, RNE bias, the articulated-inertia factor
// of M + dtB and qacc_smooth = (M + dtB)^-1 (-bias + tau) into QACC.
//
// Lane 4w + l walks chain l of world w with the running body state in registers; hand-offs
// through shared memory only at branch bodies.  Sweeps:
//   F1 (root->leaf): FK (dynamics.cuh:47-88), S (aba_bias.cuh:380-398), RNE partial
//      velocities / cdof_dot / accelerations (aba_bias.cuh:419-457); then a second pass, one
//      lane per (world, body), for the body forces (:458-466) and kept world inertias;
//   contact detection (group_detect: it needs only F1's kept body frames);
//   B1 (leaf->root): subtree forces -> bias (aba_bias.cuh:467-475), the articulated-inertia
//      factor (aba_factor.cuh:76-88) and, fused, the bias-force pass of the smooth solve
//      (aba_factor.cuh:128-136).  A body adds its children's contributions in descending
//      child index -- the order in which the reference's b-descending loops push them;
//   base: the floating base's 6x6 block, its Cholesky solve (aba_factor.cuh:90-108,138-155);
//   F2 (root->leaf): qdd per hinge body (aba_factor.cuh:156-164).
// B1 parks u_b in qacc[d]; the base solve and F2 turn it into qacc_smooth.  With allow_defer
// and a contact in the group, those two steps are skipped here (the base block leaves its
// right-hand side in qacc[0..5]) and the function returns 1: batch_contact finishes them in
// its lane_solve step.  Otherwise it returns 0 with qacc_smooth in QACC.
// bias_out (optional, per world slot, global memory) receives qfrc_bias.  bdt_all, when
// non-null, is the dt*B diagonal of every world slot (else bdt_w per slot).
__device__ void group_detect(float* grp, const G1Tables& T, int lane);
__device__ int group_smooth(float* grp, const G1Tables& T, int lane, const float* const* bdt_w, float* const* bias_out,
                            const float* bdt_all = nullptr, int allow_defer = 0) {
    const int w = lane >> 2, cl = lane & 3;
    const float* bdt = nullptr;  // world w's entry, by unrolled select (no run-time index)
    if (bdt_all) {
        bdt = w < GW ? bdt_all : nullptr;
    } else if (bdt_w && w < GW) {
#pragma unroll
        for (int k = 0; k < GW; ++k) bdt = (w == k) ? bdt_w[k] : bdt;
    }
    const bool on = w < GW && cl < T.nchain;
    // this lane's chain bounds and the sweep lengths, in registers for all three sweeps (the
    // frame stores inside the sweeps would otherwise make the compiler reload them each step)
    const int c_start = on ? T.chain_start[cl] : 0, c_len = on ? T.chain_len[cl] : 0;
    const int c_bstart = on ? T.chain_bstart[cl] : 0;
    const int n_fwd = T.nsteps, n_back = T.nsteps_back;
    float* fr = grp + (w < GW ? w : 0) * WFLOATS;
    const float *qp = fr + WL::QP, *qv = fr + WL::QV, *tau = fr + WL::TAU;
    float *S = fr + WL::S, *BQ = fr + WL::BQ, *FOWN = fr + WL::FOWN;
    float *FU = fr + WL::FU, *FINVD = fr + WL::FINVD, *qacc = fr + WL::QACC, *XS = fr + WL::XS;
    float* bias = (bias_out && w < GW) ? bias_out[w] : nullptr;
    float* QS = grp + GW * WFLOATS;  // the group's contact workspace, idle until the contact solve
    PROF_BEGIN();

    // ---- floating base (body 1): the chain lanes of a world compute it redundantly
    const V3 p = ld3(qp);
    const Q4 q1 = qnormalize(ld4(qp + 3));
    V3 bw = mk3(0, 0, 0), bv = mk3(0, 0, 0), baw = mk3(0, 0, 0), bav = mk3(-T.gravity[0], -T.gravity[1], -T.gravity[2]);
    if (on) {
        float R1[9];
        qmat(q1, R1);
        // base motion axes: translation e_k, rotation = columns of R1
        V3 Sw[6], Sv[6];
#pragma unroll
        for (int k = 0; k < 3; ++k) {
            Sw[k] = mk3(0, 0, 0);
            Sv[k] = mk3(k == 0 ? 1.f : 0.f, k == 1 ? 1.f : 0.f, k == 2 ? 1.f : 0.f);
            Sw[3 + k] = mk3(R1[k], R1[3 + k], R1[6 + k]);
            Sv[3 + k] = mk3(0, 0, 0);
        }
        // RNE through the 6 base dofs (aba_bias.cuh:423-440)
        V3 Sdw[6], Sdv[6];
        V3 wv = bw, vv = bv;
#pragma unroll
        for (int a = 0; a < 3; ++a) {
            const float qd = qv[a];
            Sdw[a] = cross3(wv, Sw[a]);
            Sdv[a] = add3(cross3(wv, Sv[a]), cross3(vv, Sw[a]));
            wv = {wv.x + Sw[a].x * qd, wv.y + Sw[a].y * qd, wv.z + Sw[a].z * qd};
            vv = {vv.x + Sv[a].x * qd, vv.y + Sv[a].y * qd, vv.z + Sv[a].z * qd};
        }
        const V3 wr = wv, vr = vv;
#pragma unroll
        for (int a = 3; a < 6; ++a) {
            Sdw[a] = cross3(wr, Sw[a]);
            Sdv[a] = add3(cross3(wr, Sv[a]), cross3(vr, Sw[a]));
        }
#pragma unroll
        for (int a = 3; a < 6; ++a) {
            const float qd = qv[a];
            wv = {wv.x + Sw[a].x * qd, wv.y + Sw[a].y * qd, wv.z + Sw[a].z * qd};
            vv = {vv.x + Sv[a].x * qd, vv.y + Sv[a].y * qd, vv.z + Sv[a].z * qd};
        }
        V3 ea = baw, eb = bav;
#pragma unroll
        for (int a = 0; a < 6; ++a) {
            const float qd = qv[a];
            ea = {ea.x + Sdw[a].x * qd, ea.y + Sdw[a].y * qd, ea.z + Sdw[a].z * qd};
            eb = {eb.x + Sdv[a].x * qd, eb.y + Sdv[a].y * qd, eb.z + Sdv[a].z * qd};
        }
        bw = wv; bv = vv; baw = ea; bav = eb;
        if (cl == 0) {
#pragma unroll
            for (int k = 0; k < 6; ++k) { st3(S + 6 * k, Sw[k]); st3(S + 6 * k + 3, Sv[k]); }
            float* xs = XS + 8 * T.xslot[1];
            st4(xs, q1); st3(xs + 4, p);
            stash_body(QS + 4 * (w * NB + 1), q1, p, bw, bv, baw, bav, FOWN + 6, BQ + 9);
        }
    }

    // ---- F1: root -> leaf along the chains
    {
        V3 pos = p, wv = bw, vv = bv, aw = baw, av = bav;
        Q4 quat = q1;
        int4 cs_nx = T.cstep[cl & 3][0];  // the next step's entry, loaded one step ahead
        for (int s = 0; s < n_fwd; ++s) {
            const int k = on ? s - c_start : -1;
            if (k >= 0 && k < c_len) {
                const int4 cs = cs_nx;
                cs_nx = T.cstep[cl][min(k + 1, G1_MAXCLEN - 1)];
                const int b = cs.x;
                if (k == 0) {
                    const int par = cstep_parent(cs.y);
                    if (par == 1) {
                        pos = p; quat = q1; wv = bw; vv = bv; aw = baw; av = bav;
                    } else {
                        const float* st = fr + WL::HF + 20 * T.branch_slot[par];
                        pos = ld3(st); quat = ld4(st + 3); wv = ld3(st + 7); vv = ld3(st + 10); aw = ld3(st + 13); av = ld3(st + 16);
                    }
                }
                const int j = cstep_jnt(cs.y), d = cs.w;
                const int xsl = cstep_xslot(cs.y), bsl = cstep_bslot(cs.y);
                pos = add3(pos, qrot(quat, ld3(T.body_pos + 3 * b)));
                quat = qmul(quat, ld4(T.body_quat + 4 * b));
                const V3 an = ld3(T.jnt_pos + 3 * j), ax = ld3(T.jnt_axis + 3 * j);
                const V3 anchor = add3(pos, qrot(quat, an));
                float sn, csn;
                sincosf(0.5f * qp[cs.z], &sn, &csn);
                quat = qmul(quat, Q4{csn, ax.x * sn, ax.y * sn, ax.z * sn});
                pos = sub3(anchor, qrot(quat, an));
                if (xsl >= 0) {
                    float* xs = XS + 8 * xsl;
                    st4(xs, quat); st3(xs + 4, pos);
                }
                const V3 sw = qrot(quat, ax);
                const V3 sv = cross3(sub3(add3(pos, qrot(quat, an)), p), sw);
                st6(S + 6 * d, sw, sv);
                const float qd = qv[d];
                const V3 sdw = cross3(wv, sw), sdv = add3(cross3(wv, sv), cross3(vv, sw));
                wv = {wv.x + sw.x * qd, wv.y + sw.y * qd, wv.z + sw.z * qd};
                vv = {vv.x + sv.x * qd, vv.y + sv.y * qd, vv.z + sv.z * qd};
                aw = {aw.x + sdw.x * qd, aw.y + sdw.y * qd, aw.z + sdw.z * qd};
                av = {av.x + sdv.x * qd, av.y + sdv.y * qd, av.z + sdv.z * qd};
                stash_body(QS + 4 * (w * NB + b), quat, pos, wv, vv, aw, av, FOWN + 6 * b, BQ + 9 * b);
                if (bsl >= 0) {
                    float* st = fr + WL::HF + 20 * bsl;
                    st3(st, pos); st4(st + 3, quat); st3(st + 7, wv); st3(st + 10, vv); st3(st + 13, aw); st3(st + 16, av);
                }
            }
            __syncwarp();
        }
    }
    PROF_MARK(P_F1);
    // F1, second pass: the body forces and kept world inertias, one lane per (world, body),
    // from the kinematics the chain walk stashed (in place: a body's stash sits in its own
    // BQ / FOWN rows, its orientation in the idle contact workspace)
#pragma unroll 1
    for (int it = lane; it < GW * (NB - 1); it += 32) {
        const int ww = it / (NB - 1), b = 1 + it % (NB - 1);
        float* fw = grp + ww * WFLOATS;
        float* bq = fw + WL::BQ + 9 * b;
        float* fo = fw + WL::FOWN + 6 * b;
        const Q4 quat = ld4(QS + 4 * (ww * NB + b));
        // com offset xipos - p, rounded as the reference does it (the pelvis's pos is p itself)
        const V3 cpos = sub3(add3(ld3(bq), qrot(quat, ld3(T.body_ipos + 3 * b))), ld3(fw + WL::QP));
        const V3 vw = ld3(bq + 3), vv = ld3(bq + 6);
        const float2* f2 = reinterpret_cast<const float2*>(fo);
        const float2 a01 = f2[0], a23 = f2[1], a45 = f2[2];
        body_force_keep(T, b, quat, cpos, vw, vv, mk3(a01.x, a01.y, a23.x), mk3(a23.y, a45.x, a45.y), fo, bq);
    }
    __syncwarp();
    PROF_MARK(P_F1B);
    // contact detection needs only F1's kept frames.  With contacts in the group (and
    // allow_defer), the base solve and F2 are left to the contact solve's back-solve step
    // (lane_solve, four more lanes), off the path to the contact batch.
    group_detect(grp, T, lane);
    PROF_MARK(P_DETECT);
    int anycon = 0;
#pragma unroll
    for (int ww = 0; ww < GW; ++ww) anycon |= reinterpret_cast<const int*>(grp + ww * WFLOATS + WL::MISC)[0];
    const bool defer = allow_defer && anycon != 0;

    // ---- B1: leaf -> root along the chains.  The contribution of the previous (child) body
    // of the chain is carried in registers; other children (chain heads below a branch body)
    // left theirs in HB.
    {
        float cia[21], cf[6], cpa[6];
        int carried = -1;
        int4 cs_nx = T.cstep[cl & 3][max(c_len - 1, 0)];  // the next step's entry, one step ahead
        for (int s = 0; s < n_back; ++s) {
            const int len = c_len;
            const int k = on ? s - c_bstart : -1;
            if (k >= 0 && k < len) {
                const int4 cs = cs_nx;
                cs_nx = T.cstep[cl][max(len - 2 - k, 0)];
                const int b = cs.x, d = cs.w;
                float ia[21], f[6], pa[6];
                body_ia_kept(T, b, BQ + 9 * b, ia);
                {
                    const float2* f2 = reinterpret_cast<const float2*>(FOWN + 6 * b);
                    const float2 f01 = f2[0], f23 = f2[1], f45 = f2[2];
                    f[0] = f01.x; f[1] = f01.y; f[2] = f23.x; f[3] = f23.y; f[4] = f45.x; f[5] = f45.y;
                }
#pragma unroll
                for (int i = 0; i < 6; ++i) pa[i] = 0.f;
                if (cstep_bslot(cs.y) < 0) {  // one child -- the walk's previous body -- or a leaf
                    if (k > 0) {
#pragma unroll
                        for (int i = 0; i < 21; ++i) ia[i] += cia[i];
#pragma unroll
                        for (int i = 0; i < 6; ++i) { f[i] += cf[i]; pa[i] += cpa[i]; }
                    }
                } else
                for (int q = T.child_start[b]; q < T.child_start[b + 1]; ++q) {
                    const int c = T.child_list[q];
                    if (c == carried) {
#pragma unroll
                        for (int i = 0; i < 21; ++i) ia[i] += cia[i];
#pragma unroll
                        for (int i = 0; i < 6; ++i) { f[i] += cf[i]; pa[i] += cpa[i]; }
                    } else {
                        const float* hb = fr + WL::HB + 36 * T.head_chain[c];
#pragma unroll
                        for (int i = 0; i < 21; ++i) ia[i] += hb[i];
#pragma unroll
                        for (int i = 0; i < 6; ++i) { f[i] += hb[21 + i]; pa[i] += hb[27 + i]; }
                    }
                }
                float sd[6];
                {
                    const float2* s2 = reinterpret_cast<const float2*>(S + 6 * d);
                    const float2 s01 = s2[0], s23 = s2[1], s45 = s2[2];
                    sd[0] = s01.x; sd[1] = s01.y; sd[2] = s23.x; sd[3] = s23.y; sd[4] = s45.x; sd[5] = s45.y;
                }
                const float bd = sd[0] * f[0] + sd[1] * f[1] + sd[2] * f[2] + sd[3] * f[3] + sd[4] * f[4] + sd[5] * f[5];
                if (bias) bias[d] = bd;
                const float rhs = -bd + tau[d];
                float U[6];
#pragma unroll
                for (int r = 0; r < 6; ++r) {
                    float acc = 0.f;
#pragma unroll
                    for (int c = 0; c < 6; ++c) acc += ia[sym6(r, c)] * sd[c];
                    U[r] = acc;
                }
                float D = 0.f;
#pragma unroll
                for (int i = 0; i < 6; ++i) D += sd[i] * U[i];
                D = D + T.armature[d];
                if (bdt) D += bdt[d];
                const float invD = 1.f / D;
                float sp = 0.f;
#pragma unroll
                for (int i = 0; i < 6; ++i) sp += sd[i] * pa[i];
                const float u = rhs - sp;
                const float ud = u * invD;
                {
                    float2* u2 = reinterpret_cast<float2*>(FU + 6 * b);
                    u2[0] = make_float2(U[0], U[1]); u2[1] = make_float2(U[2], U[3]); u2[2] = make_float2(U[4], U[5]);
                }
                FINVD[b] = invD;
                qacc[d] = u;  // u_b parks in qacc[d] until the root -> leaf pass
#pragma unroll
                for (int r = 0; r < 6; ++r)
#pragma unroll
                    for (int c = r; c < 6; ++c) cia[sym6(r, c)] = ia[sym6(r, c)] - U[r] * U[c] * invD;
#pragma unroll
                for (int i = 0; i < 6; ++i) { cpa[i] = pa[i] + U[i] * ud; cf[i] = f[i]; }
                carried = b;
                if (k == len - 1) {  // chain head: leave the contribution for its parent
                    float* hb = fr + WL::HB + 36 * cl;
#pragma unroll
                    for (int i = 0; i < 21; ++i) hb[i] = cia[i];
#pragma unroll
                    for (int i = 0; i < 6; ++i) { hb[21 + i] = cf[i]; hb[27 + i] = cpa[i]; }
                }
            }
            __syncwarp();
        }
    }
    PROF_MARK(P_B1);

    // ---- floating base: 8 lanes per world, lanes 4w + c and 16 + 4w + c (c = 0..3) of
    // world w, sub-lane k8 = c (+4).  Same arithmetic, entry by entry, as one lane doing it all
    // (aba_factor.cuh:90-108, 128-155); only the lower triangle of Dm is formed (the Cholesky
    // and the solves read nothing else).
    const int wb = (lane & 15) >> 2, k8 = (lane & 3) + ((lane >> 4) << 2);
    float* frb = grp + wb * WFLOATS;
    const float* Sb = frb + WL::S;
    float* U6 = frb + WL::FU6;
    float* L6 = frb + WL::FL6;
    float* BA = frb + WL::HF;  // pelvis IA [21], f [6], pA [6] (F1's hand-off area is dead now)
    const float* bdtb = bdt_all;
    float* biasb = nullptr;
    if (!bdt_all && bdt_w) {
#pragma unroll
        for (int k = 0; k < GW; ++k) bdtb = (wb == k) ? bdt_w[k] : bdtb;
    }
    if (bias_out) {
#pragma unroll
        for (int k = 0; k < GW; ++k) biasb = (wb == k) ? bias_out[k] : biasb;
    }
    static_assert(20 * G1_MAXBRANCH >= 33, "the pelvis accumulators fit in the F1 hand-off area");
    // the pelvis's own IA / f, then its children's contributions in descending child index
    {
        // the pelvis's children (at most 4: the G1 has 3), their chain-head hand-offs in HB
        const int q0 = T.child_start[1], nch = T.child_start[2] - q0;
        int hoff[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) hoff[c] = c < nch ? WL::HB + 36 * T.head_chain[T.child_list[q0 + c]] : 0;
        float ia1[21];
        body_ia_kept(T, 1, frb + WL::BQ + 9, ia1);
#pragma unroll
        for (int m = 0; m < 5; ++m) {
            const int e = k8 + 8 * m;
            if (e < 33) {
                float v = (e >= 21 && e < 27) ? frb[WL::FOWN + 6 + (e - 21)] : 0.f;
#pragma unroll
                for (int j = 0; j < 8; ++j)
                    if (8 * m + j < 21) v = (k8 == j) ? ia1[8 * m + j] : v;
#pragma unroll
                for (int c = 0; c < 4; ++c)
                    if (c < nch) v += frb[hoff[c] + e];
                BA[e] = v;
            }
        }
    }
    __syncwarp();
    // U6[i*6+l] = (IA S_l)[i]: 36 entries over the 8 lanes
    for (int e = k8; e < 36; e += 8) {
        const int i = e / 6, l = e % 6;
        float acc = 0.f;
#pragma unroll
        for (int j = 0; j < 6; ++j) acc += BA[sym6(i, j)] * Sb[6 * l + j];
        U6[i * 6 + l] = acc;
    }
    __syncwarp();
    PROF_MARK(P_BASE_PULL);
    // Dm[k*6+l] = S_k . U6_l (+ diag) for l <= k: 21 entries; u = (-bias + tau) - S^T pA: 6
    for (int e = k8; e < 27; e += 8) {
        if (e < 21) {
            int k = 0;
#pragma unroll
            for (int r = 1; r < 6; ++r) k += (e >= r * (r + 1) / 2) ? 1 : 0;
            const int l = e - k * (k + 1) / 2;
            float acc = 0.f;
#pragma unroll
            for (int i = 0; i < 6; ++i) acc += Sb[6 * k + i] * U6[i * 6 + l];
            L6[k * 6 + l] = acc + (k == l ? (T.armature[k] + (bdtb ? bdtb[k] : 0.f)) : 0.f);
        } else {
            const int kk = e - 21;
            const float* sd = Sb + 6 * kk;
            const float* bf = BA + 21;
            const float bd = sd[0] * bf[0] + sd[1] * bf[1] + sd[2] * bf[2] + sd[3] * bf[3] + sd[4] * bf[4] + sd[5] * bf[5];
            if (biasb) biasb[kk] = bd;
            float sp = 0.f;
#pragma unroll
            for (int i = 0; i < 6; ++i) sp += sd[i] * BA[27 + i];
            frb[WL::QACC + kk] = (-bd + frb[WL::TAU + kk]) - sp;  // u of the base dofs, parked in qacc
        }
    }
    __syncwarp();
    PROF_MARK(P_BASE_DM);
    if (w < GW && cl == 0) {
        // 6x6 Cholesky of Dm and the base solve in registers (aba_factor.cuh:103-107,
        // 148-152); one lane per world
        float Dm[36], q6[6];
#pragma unroll
        for (int i = 0; i < 6; ++i)
#pragma unroll
            for (int j = 0; j <= i; ++j) Dm[i * 6 + j] = L6[i * 6 + j];
#pragma unroll
        for (int k = 0; k < 6; ++k) q6[k] = qacc[k];
#pragma unroll
        for (int i = 0; i < 6; ++i)
#pragma unroll
            for (int j = 0; j <= i; ++j) {
                float acc = Dm[i * 6 + j];
#pragma unroll
                for (int k = 0; k < j; ++k) acc -= Dm[i * 6 + k] * Dm[j * 6 + k];
                if (i == j) Dm[i * 6 + i] = sqrtf(acc); else Dm[i * 6 + j] = acc / Dm[j * 6 + j];
            }
#pragma unroll
        for (int i = 0; i < 6; ++i)
#pragma unroll
            for (int j = 0; j <= i; ++j) L6[i * 6 + j] = Dm[i * 6 + j];
      if (!defer) {  // else the base solve and the root -> leaf pass run later, in lane_solve
#pragma unroll
        for (int i = 0; i < 6; ++i) {
            float acc = q6[i];
#pragma unroll
            for (int k = 0; k < i; ++k) acc -= Dm[i * 6 + k] * q6[k];
            q6[i] = acc / Dm[i * 6 + i];
        }
#pragma unroll
        for (int i = 5; i >= 0; --i) {
            float acc = q6[i];
#pragma unroll
            for (int k = i + 1; k < 6; ++k) acc -= Dm[k * 6 + i] * q6[k];
            q6[i] = acc / Dm[i * 6 + i];
        }
#pragma unroll
        for (int k = 0; k < 6; ++k) qacc[k] = q6[k];
        float* A1 = fr + WL::A1;
#pragma unroll
        for (int i = 0; i < 6; ++i) {
            float acc = 0.f;
#pragma unroll
            for (int k = 0; k < 6; ++k) acc += S[6 * k + i] * q6[k];
            A1[i] = acc;
        }
      }
    }
    __syncwarp();
    PROF_MARK(P_BASE);
    if (defer) return 1;

    // ---- F2: root -> leaf, qdd per hinge body
    {
        float a[6];
        int4 cs_nx = T.cstep[cl & 3][0];  // the next step's entry, loaded one step ahead
        for (int s = 0; s < n_fwd; ++s) {
            const int k = on ? s - c_start : -1;
            if (k >= 0 && k < c_len) {
                const int4 cs = cs_nx;
                cs_nx = T.cstep[cl][min(k + 1, G1_MAXCLEN - 1)];
                const int b = cs.x, d = cs.w;
                const int bsl = cstep_bslot(cs.y);
                if (k == 0) {
                    const int par = cstep_parent(cs.y);
                    const float* src = par == 1 ? fr + WL::A1 : fr + WL::HA + 8 * T.binfo[par].y;
#pragma unroll
                    for (int i = 0; i < 6; ++i) a[i] = src[i];
                }
                const float2* U2 = reinterpret_cast<const float2*>(FU + 6 * b);
                const float2 u01 = U2[0], u23 = U2[1], u45 = U2[2];
                float s2 = 0.f;
                s2 += u01.x * a[0]; s2 += u01.y * a[1]; s2 += u23.x * a[2];
                s2 += u23.y * a[3]; s2 += u45.x * a[4]; s2 += u45.y * a[5];
                const float qdd = (qacc[d] - s2) * FINVD[b];
                qacc[d] = qdd;
                const float2* S2 = reinterpret_cast<const float2*>(S + 6 * d);
                const float2 s01 = S2[0], s23 = S2[1], s45 = S2[2];
                a[0] = a[0] + s01.x * qdd; a[1] = a[1] + s01.y * qdd; a[2] = a[2] + s23.x * qdd;
                a[3] = a[3] + s23.y * qdd; a[4] = a[4] + s45.x * qdd; a[5] = a[5] + s45.y * qdd;
                if (bsl >= 0) {
                    float* st = fr + WL::HA + 8 * bsl;
#pragma unroll
                    for (int i = 0; i < 6; ++i) st[i] = a[i];
                }
            }
            __syncwarp();
        }
    }
    PROF_MARK(P_F2);
    return 0;
}

// ------------------------------------------------------------------ M^-1 apply, one lane
// y = (M + dtB)^-1 x in place on xy[0..NV), one lane per right-hand side, reading the factor
// of world frame `fr` (a shared-memory broadcast: every lane reads the same entry).
// aba_factor.cuh:121-165.  The lane walks the chains with the articulated bias force of the
// current body in registers; leaf->root the chains go last-to-first and a chain head leaves
// its contribution in hand[chain]; a body adds its children in descending child index.
// u_b = x_d - S_d.pA_b parks in xy[d] between the sweeps; root->leaf a branch body leaves
// its acceleration in fwd[slot].  `scratch`: SOLVE_SCRATCH floats of this lane.
// The factor (frame), the right-hand side (contact workspace row) and the scratch are
// disjoint shared-memory arrays: the restrict qualifiers let the compiler move a body's loads
// ahead of the previous body's stores.
__device__ __noinline__ void lane_solve(const float* __restrict__ fr, const G1Tables& T, float* __restrict__ xy,
                                       float* __restrict__ scratch, int chains) {
    const float* __restrict__ S = fr + WL::S;
    const float* __restrict__ FU = fr + WL::FU;
    const float* __restrict__ FINVD = fr + WL::FINVD;
    const float* __restrict__ L6 = fr + WL::FL6;
    float* __restrict__ hand = scratch;
    float* __restrict__ fwd = scratch + 6 * 4;
#ifdef G1_PROF
    long long _pt = clock64();
    const bool _lead = (threadIdx.x & 31) == (__ffs(__activemask()) - 1);
#define LS_MARK(i) do { long long _n = clock64(); if (_lead) atomicAdd(&g_prof[i], (unsigned long long)(_n - _pt)); _pt = _n; } while (0)
#else
#define LS_MARK(i) do { } while (0)
#endif
    // leaf -> root, chains last-to-first; the next body's index is fetched one body ahead.
    // Chains outside `chains` have a zero right-hand side: their pass would produce exact
    // zeros, so it is skipped (their hand-off is zero).
    for (int c = T.nchain - 1; c >= 0; --c) {
        if (!((chains >> c) & 1)) {
#pragma unroll
            for (int i = 0; i < 6; ++i) hand[6 * c + i] = 0.f;
            continue;
        }
        const int len = T.chain_len[c];
        float pa[6] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        int b = T.chain_body[c][len - 1], prev = -1;
        for (int k = len - 1; k >= 0; --k) {
            const int bn = k > 0 ? T.chain_body[c][k - 1] : 0;
            const int4 bi = T.binfo[b];
            const int d = bi.x;
            float acc[6];
            if (bi.y >= 0) {  // branch body: children in descending index
#pragma unroll
                for (int i = 0; i < 6; ++i) acc[i] = 0.f;
                for (int q = T.child_start[b]; q < T.child_start[b + 1]; ++q) {
                    const int ch = T.child_list[q];
                    if (ch == prev) {
#pragma unroll
                        for (int i = 0; i < 6; ++i) acc[i] += pa[i];
                    } else {
                        const float* src = hand + 6 * T.head_chain[ch];
#pragma unroll
                        for (int i = 0; i < 6; ++i) acc[i] += src[i];
                    }
                }
            } else {  // one child (the previous body of the walk) or a leaf
#pragma unroll
                for (int i = 0; i < 6; ++i) acc[i] = pa[i];
            }
            const float2* S2 = reinterpret_cast<const float2*>(S + 6 * d);
            const float2 s01 = S2[0], s23 = S2[1], s45 = S2[2];
            const float sp = ((((0.f + s01.x * acc[0]) + s01.y * acc[1]) + s23.x * acc[2]) + s23.y * acc[3]) + s45.x * acc[4] + s45.y * acc[5];
            const float u = xy[d] - sp;
            xy[d] = u;
            const float ud = u * FINVD[b];
            const float2* U2 = reinterpret_cast<const float2*>(FU + 6 * b);
            const float2 u01 = U2[0], u23 = U2[1], u45 = U2[2];
            pa[0] = acc[0] + u01.x * ud; pa[1] = acc[1] + u01.y * ud; pa[2] = acc[2] + u23.x * ud;
            pa[3] = acc[3] + u23.y * ud; pa[4] = acc[4] + u45.x * ud; pa[5] = acc[5] + u45.y * ud;
            prev = b;
            b = bn;
        }
#pragma unroll
        for (int i = 0; i < 6; ++i) hand[6 * c + i] = pa[i];
    }
    LS_MARK(P_LS_BACK);
    float pa1[6] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int q = T.child_start[1]; q < T.child_start[2]; ++q) {
        const float* src = hand + 6 * T.head_chain[T.child_list[q]];
#pragma unroll
        for (int i = 0; i < 6; ++i) pa1[i] += src[i];
    }
    float q6[6];
#pragma unroll
    for (int k = 0; k < 6; ++k) {
        const float* sd = S + 6 * k;
        q6[k] = xy[k] - (((((0.f + sd[0] * pa1[0]) + sd[1] * pa1[1]) + sd[2] * pa1[2]) + sd[3] * pa1[3]) + sd[4] * pa1[4] + sd[5] * pa1[5]);
    }
    float Lr[21];  // lower triangle of the base Cholesky factor
#pragma unroll
    for (int i = 0; i < 6; ++i)
#pragma unroll
        for (int k = 0; k <= i; ++k) Lr[i * (i + 1) / 2 + k] = L6[i * 6 + k];
#pragma unroll
    for (int i = 0; i < 6; ++i) {
        float acc = q6[i];
#pragma unroll
        for (int k = 0; k < i; ++k) acc -= Lr[i * (i + 1) / 2 + k] * q6[k];
        q6[i] = acc / Lr[i * (i + 1) / 2 + i];
    }
#pragma unroll
    for (int i = 5; i >= 0; --i) {
        float acc = q6[i];
#pragma unroll
        for (int k = i + 1; k < 6; ++k) acc -= Lr[k * (k + 1) / 2 + i] * q6[k];
        q6[i] = acc / Lr[i * (i + 1) / 2 + i];
    }
    float a1[6];
#pragma unroll
    for (int i = 0; i < 6; ++i) {
        float acc = 0.f;
#pragma unroll
        for (int k = 0; k < 6; ++k) acc += S[6 * k + i] * q6[k];
        a1[i] = acc;
    }
#pragma unroll
    for (int k = 0; k < 6; ++k) xy[k] = q6[k];
    LS_MARK(P_LS_BASE);
    // root -> leaf, chains first-to-last (U and S rows read as float2: 6-float rows of an
    // 8-byte aligned frame; the body's dof, branch slot and parent in one 16-byte load)
    for (int c = 0; c < T.nchain; ++c) {
        const int len = T.chain_len[c];
        int b = T.chain_body[c][0];
        const int par = T.binfo[b].z;
        float a[6];
        if (par == 1) {
#pragma unroll
            for (int i = 0; i < 6; ++i) a[i] = a1[i];
        } else {
            const float* src = fwd + 6 * T.binfo[par].y;
#pragma unroll
            for (int i = 0; i < 6; ++i) a[i] = src[i];
        }
        for (int k = 0; k < len; ++k) {
            const int bn = k + 1 < len ? T.chain_body[c][k + 1] : 0;
            const int4 bi = T.binfo[b];
            const int d = bi.x;
            const float2* U2 = reinterpret_cast<const float2*>(FU + 6 * b);
            const float2 u01 = U2[0], u23 = U2[1], u45 = U2[2];
            const float s2 = ((((0.f + u01.x * a[0]) + u01.y * a[1]) + u23.x * a[2]) + u23.y * a[3]) + u45.x * a[4] + u45.y * a[5];
            const float qdd = (xy[d] - s2) * FINVD[b];
            xy[d] = qdd;
            const float2* S2 = reinterpret_cast<const float2*>(S + 6 * d);
            const float2 s01 = S2[0], s23 = S2[1], s45 = S2[2];
            a[0] = a[0] + s01.x * qdd; a[1] = a[1] + s01.y * qdd; a[2] = a[2] + s23.x * qdd;
            a[3] = a[3] + s23.y * qdd; a[4] = a[4] + s45.x * qdd; a[5] = a[5] + s45.y * qdd;
            if (bi.y >= 0) {
                float* dst = fwd + 6 * bi.y;
#pragma unroll
                for (int i = 0; i < 6; ++i) dst[i] = a[i];
            }
            b = bn;
        }
    }
    LS_MARK(P_LS_FWD);
#undef LS_MARK
}

// ------------------------------------------------------------------ contact
// MuJoCo solimp impedance (contact.cuh:97-109)
__device__ __forceinline__ float foot_impedance(const G1Tables& T, float pos) {
    float dmin = T.solimp[0], dmax = T.solimp[1], width = T.solimp[2], mid = T.solimp[3], power = T.solimp[4];
    float x = fabsf(pos) / width, y;
    if (x >= 1.f) y = 1.f;
    else {
        float a = 1.f / powf(mid, power - 1.f), b = 1.f / powf(1.f - mid, power - 1.f);
        y = (x < mid) ? a * powf(x, power) : 1.f - b * powf(1.f - x, power);
    }
    return dmin + y * (dmax - dmin);
}

struct QaccOpts {
    int pgs_iters;
    float mu;
    const float* const* bdt;  // per world slot: shared-memory dt*B diagonal (entries may be null)
    const float* bdt_all;     // if non-null: the dt*B diagonal of every world slot (bdt unused)
};

// Foot-sphere contacts of the GW worlds (contact.cuh:31-46), lane = 8 (w - w0) + sphere in
// passes of 32 / 8 worlds, compacted in sphere order into each world's CON; ncon in MISC[0].
__device__ void group_detect(float* grp, const G1Tables& T, int lane) {
    constexpr int WPP = 32 / G1_NFOOT_;  // worlds per pass
    static_assert(WPP * G1_NFOOT_ == 32, "one lane per (world, sphere) in a pass");
#pragma unroll 1
    for (int w0 = 0; w0 < GW; w0 += WPP) {
        const int wl = lane / NFOOT, w = w0 + wl, s = lane % NFOOT;
        float* fr = grp + (w < GW ? w : 0) * WFLOATS;
        bool hit = false;
        float cx = 0.f, cy = 0.f, pen = 0.f;
        if (w < GW) {
            const float* xs = fr + WL::XS + 8 * T.xslot[T.foot_body[s]];
            const V3 c = add3(ld3(xs + 4), qrot(ld4(xs), ld3(T.foot_lpos + 3 * s)));
            pen = c.z - G1M_FOOT_RADIUS;
            hit = pen < 0.f;
            cx = c.x; cy = c.y;
        }
        const unsigned m = __ballot_sync(FULLMASK, hit);
        const unsigned wm = (m >> (NFOOT * wl)) & ((1u << NFOOT) - 1u);
        if (hit) {
            const int k = __popc(wm & ((1u << s) - 1u));
            int* con_s = reinterpret_cast<int*>(fr + WL::CON);
            con_s[k] = s;
            fr[WL::CON + 8 + 3 * k] = cx; fr[WL::CON + 9 + 3 * k] = cy; fr[WL::CON + 10 + 3 * k] = pen * 0.5f;
            fr[WL::CON + 32 + k] = pen;
        }
        if (w < GW && s == 0) reinterpret_cast<int*>(fr + WL::MISC)[0] = __popc(wm);
    }
    __syncwarp();
}

// A contact batch: worlds of the group (slot ids) whose contacts are solved together,
// at most MAXCON contacts in total; contact gc of the batch belongs to world slot
// wid[x] with coff[x] <= gc < coff[x+1].  The accessors index with unrolled selects, so a
// batch lives in registers (a run-time array index would put it in local memory).
struct Batch {
    int nw, wid[GW], coff[GW + 1];
    __device__ __forceinline__ int world_of(int gc) const {
        int x = 0;
#pragma unroll
        for (int k = 1; k < GW; ++k) x += (k < nw && gc >= coff[k]) ? 1 : 0;
        return x;
    }
    __device__ __forceinline__ int wof(int x) const {
        int r = wid[0];
#pragma unroll
        for (int k = 1; k < GW; ++k) r = (x == k) ? wid[k] : r;
        return r;
    }
    __device__ __forceinline__ int cof(int x) const {
        int r = coff[0];
#pragma unroll
        for (int k = 1; k <= GW; ++k) r = (x == k) ? coff[k] : r;
        return r;
    }
    // appends world slot w with n contacts
    __device__ __forceinline__ void append(int w, int n) {
#pragma unroll
        for (int k = 0; k < GW; ++k)
            if (k == nw) { wid[k] = w; coff[k + 1] = coff[k] + n; }
        ++nw;
    }
};

// Contact correction for the worlds of a batch by the whole warp, using the workspace cw:
// qacc += M^-1 J' f per world  (env_qacc.cuh:53-211).  The worlds' constraint rows sit side
// by side; the Delassus matrix is block diagonal over worlds and each world's PGS sweeps
// its own rows in order, all worlds in the same pass.  f -> cw[FF] (world x's rows start at
// 4*coff[x]).
// smooth_lanes: lanes 32 - GW .. 31 also finish the deferred smooth solves of the group's
// worlds (qacc_smooth = (M + dtB)^-1 (tau - bias) from the u_b parked in QACC), in the same
// lane_solve step as the contact-basis columns (at most 24).
__device__ __noinline__ void batch_contact(float* grp, float* cw, const G1Tables& T, int lane, int pgs_iters, float mu,
                                          const Batch B, int smooth_lanes) {
    float* MM = cw + CL::MM;
    float* EB = cw + CL::EB;
    const int nc = B.cof(B.nw), nb = 3 * nc, nefc_all = 4 * nc;
    PROF_BEGIN();
    for (int e = lane; e < nb * MSTR; e += 32) MM[e] = 0.f;
    __syncwarp();
    // basis rows e0 = n, e1 = mu t1, e2 = mu t2 over the ancestor dofs (env_qacc.cuh:113-126)
    for (int it = lane; it < nc * CDS; it += 32) {
        const int gc = it / CDS, k = it % CDS, x = B.world_of(gc), c = gc - B.cof(x);
        const float* fr = grp + B.wof(x) * WFLOATS;
        const int s = reinterpret_cast<const int*>(fr + WL::CON)[c];
        if (k < T.foot_ndof[s]) {
            const int a = T.foot_dofs[s][k];
            const float* S = fr + WL::S;
            const V3 p = ld3(fr + WL::XS + 8 * T.xslot[1] + 4);
            const V3 r = sub3(ld3(fr + WL::CON + 8 + 3 * c), p);
            const V3 t = add3(cross3(ld3(S + 6 * a), r), ld3(S + 6 * a + 3));
            const float e0 = t.z, e1 = mu * t.y, e2 = -mu * t.x;
            EB[gc * 36 + k] = e0; EB[gc * 36 + 12 + k] = e1; EB[gc * 36 + 24 + k] = e2;
            MM[(3 * gc) * MSTR + a] = e0; MM[(3 * gc + 1) * MSTR + a] = e1; MM[(3 * gc + 2) * MSTR + a] = e2;
        }
    }
    __syncwarp();
    PROF_MARK(P_CSETUP);
    static_assert(3 * MAXCON <= 32 - GW, "contact-basis columns and smooth lanes share the warp");
    const bool sm = smooth_lanes && lane >= 32 - GW;
    if (lane < nb || sm) {
        float* fr;
        float *xy, *scr;
        int chains;
        if (sm) {  // world slot lane - (32 - GW): rhs = u_b in QACC, no leaf -> root pass
            fr = grp + (lane - (32 - GW)) * WFLOATS;
            xy = fr + WL::QACC;
            scr = fr + WL::HB;  // B1's hand-off area, dead after the base block
            chains = 0;
        } else {
            const int gc = lane / 3, x = B.world_of(gc);
            fr = grp + B.wof(x) * WFLOATS;
            const int s = reinterpret_cast<const int*>(fr + WL::CON)[gc - B.cof(x)];
            xy = MM + lane * MSTR;
            scr = cw + CL::GRAM + lane * SOLVE_SCRATCH;
            chains = T.foot_chains[s];
        }
        lane_solve(fr, T, xy, scr, chains);
    }
    __syncwarp();
    PROF_MARK(P_SOLVE);
    // per contact: bb = e.qacc_smooth, e.qvel -> R, aref, b  (env_qacc.cuh:113-136, 188-191)
    float *RR = cw + CL::RR, *BV = cw + CL::BV;
    if (lane < nc) {
        const int gc = lane, x = B.world_of(gc), c = gc - B.cof(x);
        const float* fr = grp + B.wof(x) * WFLOATS;
        const int s = reinterpret_cast<const int*>(fr + WL::CON)[c], nd = T.foot_ndof[s];
        const float *qs = fr + WL::QACC, *qv = fr + WL::QV;
        float b0 = 0, b1 = 0, b2 = 0, v0 = 0, v1 = 0, v2 = 0;
        for (int k = 0; k < nd; ++k) {
            const int a = T.foot_dofs[s][k];
            const float e0 = EB[gc * 36 + k], e1 = EB[gc * 36 + 12 + k], e2 = EB[gc * 36 + 24 + k];
            const float qa = qs[a], qd = qv[a];
            b0 += e0 * qa; b1 += e1 * qa; b2 += e2 * qa;
            v0 += e0 * qd; v1 += e1 * qd; v2 += e2 * qd;
        }
        const float dmax = T.solimp[1], tc = T.solref[0], dr = T.solref[1];
        const float bcoef = 2.f / (dmax * tc);
        const float kcoef = 1.f / (dmax * dmax * tc * tc * dr * dr);
        const float pyr = (1.f + mu * mu) * (2.f * mu * mu / G1M_FOOT_IMPRATIO);
        const float pn = fr[WL::CON + 32 + c], imp = foot_impedance(T, pn);
        const float Rc = T.foot_invw0[s] * pyr * (1.f - imp) / imp;
        const float kip = kcoef * imp * pn;
        const float dv[4] = {v0 + v1, v0 - v1, v0 + v2, v0 - v2};
        const float db[4] = {b0 + b1, b0 - b1, b0 + b2, b0 - b2};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const float aref = -bcoef * dv[k] - kip;
            RR[4 * gc + k] = Rc;
            BV[4 * gc + k] = db[k] - aref;
        }
    }
    // pairs (c <= c') inside each world of the batch
    int poff[GW + 1];
    poff[0] = 0;
#pragma unroll
    for (int x = 0; x < GW; ++x) {
        const int n = x < B.nw ? B.cof(x + 1) - B.cof(x) : 0;
        poff[x + 1] = poff[x] + n * (n + 1) / 2;
    }
    auto pof = [&](int x) {
        int r = poff[0];
#pragma unroll
        for (int k = 1; k <= GW; ++k) r = (x == k) ? poff[k] : r;
        return r;
    };
    // the world of pair pr: count the worlds whose pairs start at or before it
    auto pair_world = [&](int pr) {
        int x = 0;
#pragma unroll
        for (int k = 1; k < GW; ++k) x += (k < B.nw && pr >= poff[k]) ? 1 : 0;
        return x;
    };
    const int npair = pof(B.nw);
    // 3x3 Gram blocks G[a][b] = e_{c,a} . m_{c',b} over c's dofs (env_qacc.cuh:161-171)
    float* G = cw + CL::GRAM;
    for (int it = lane; it < npair * 9; it += 32) {
        const int pr = it / 9, ab = it % 9, a = ab / 3, bb = ab % 3;
        const int x = pair_world(pr);
        const int n = B.cof(x + 1) - B.cof(x);
        int c = 0, rem = pr - pof(x);
        while (rem >= n - c) { rem -= n - c; ++c; }
        const int gc = B.cof(x) + c, gcp = B.cof(x) + c + rem;
        const float* fr = grp + B.wof(x) * WFLOATS;
        const int s = reinterpret_cast<const int*>(fr + WL::CON)[c], nd = T.foot_ndof[s];
        const float* ea = EB + gc * 36 + 12 * a;
        const float* mcp = MM + (3 * gcp + bb) * MSTR;
        float g = 0.f;
        for (int k = 0; k < nd; ++k) g += ea[k] * mcp[T.foot_dofs[s][k]];
        G[pr * 9 + ab] = g;
    }
    __syncwarp();
    // A = J M^-1 J' + diag R: each Gram block expanded to its 4x4 pyramid block
    // (env_qacc.cuh:172-187), packed upper triangle
    float* AP = cw + CL::AP;
    for (int it = lane; it < npair * 4; it += 32) {
        const int pr = it >> 2, k = it & 3;
        const int x = pair_world(pr);
        const int n = B.cof(x + 1) - B.cof(x);
        int c = 0, rem = pr - pof(x);
        while (rem >= n - c) { rem -= n - c; ++c; }
        const int cp = c + rem;
        const float* g = G + 9 * pr;
        const float c0 = dcoef(k, 0), c1 = dcoef(k, 1), c2 = dcoef(k, 2);
        const float t0 = c0 * g[0] + c1 * g[3] + c2 * g[6];
        const float t1 = c0 * g[1] + c1 * g[4] + c2 * g[7];
        const float t2 = c0 * g[2] + c1 * g[5] + c2 * g[8];
        const int i = 4 * (B.cof(x) + c) + k;
        // inside a diagonal block the reference's later (larger k) write of (k,kp)/(kp,k) wins
        const int kpmax = (c == cp) ? k : 3;
#pragma unroll
        for (int kp = 0; kp < 4; ++kp) {
            if (kp > kpmax) break;
            float aij = t0 * dcoef(kp, 0) + t1 * dcoef(kp, 1) + t2 * dcoef(kp, 2);
            const int j = 4 * (B.cof(x) + cp) + kp;
            if (i == j) aij += RR[i];
            AP[apidx(i, j)] = aij;
        }
    }
    __syncwarp();
    PROF_MARK(P_GRAM);
    // projected Gauss-Seidel, each world's rows in order (contact.cuh:159-171), the worlds side
    // by side.  Lane j keeps the residual r_j = b_j + sum_k A_jk f_k of its row; after row i of
    // its world moves by delta, it adds A_ji delta.
    const int xj = lane < nefc_all ? B.world_of(lane / 4) : 0;
    const int r0 = 4 * B.cof(xj), nrow = lane < nefc_all ? 4 * (B.cof(xj + 1) - B.cof(xj)) : 0;
    int maxrow = 0;
#pragma unroll
    for (int x = 0; x < GW; ++x)
        if (x < B.nw) maxrow = max(maxrow, 4 * (B.cof(x + 1) - B.cof(x)));
    float fj = 0.f, rj = lane < nefc_all ? BV[lane] : 0.f;
    const float ajj = lane < nefc_all ? AP[apidx(lane, lane)] : 1.f;
    const float inv = 1.f / ajj;
    const int lj = lane - r0;
    // this lane's column of its world's block, in registers (off the row-to-row chain)
    float acol[4 * MAXCON];
#pragma unroll
    for (int i = 0; i < 4 * MAXCON; ++i) {
        if (i >= maxrow) break;  // rows past the batch's largest world are never read
        acol[i] = i < nrow ? AP[apidx(r0 + i, lane)] : 0.f;
    }
    for (int itr = 0; itr < pgs_iters; ++itr) {
#pragma unroll
        for (int i = 0; i < 4 * MAXCON; ++i) {
            if (i >= maxrow) break;
            const bool live = i < nrow;
            const float aji = acol[i];
            // every lane evaluates the update; the lane of row i of its world keeps it
            // (branch-free: no divergence on the row-to-row chain)
            const float ri = rj - ajj * fj;
            float fn = -ri * inv;
            fn = fn > 0.f ? fn : 0.f;
            const bool mine = live && lj == i;
            float delta = mine ? fn - fj : 0.f;
            fj = mine ? fn : fj;
            delta = __shfl_sync(FULLMASK, delta, live ? r0 + i : lane);
            rj += aji * delta;
        }
    }
    float* F = cw + CL::FF;
    if (lane < nefc_all) F[lane] = fj;
    __syncwarp();
    PROF_MARK(P_PGS);
    // qacc = qacc_smooth + sum_c sum_a fb_c[a] m_{c,a}, per world  (env_qacc.cuh:199-211)
    for (int it = lane; it < B.nw * NV; it += 32) {
        const int x = it / NV, d = it % NV;
        float* qacc = grp + B.wof(x) * WFLOATS + WL::QACC;
        float dq = 0.f;
        for (int gc = B.cof(x); gc < B.cof(x + 1); ++gc) {
            const float f0 = F[4 * gc], f1 = F[4 * gc + 1], f2 = F[4 * gc + 2], f3 = F[4 * gc + 3];
            const float fb0 = f0 + f1 + f2 + f3, fb1 = f0 - f1, fb2 = f2 - f3;
            const float* mc = MM + 3 * gc * MSTR;
            dq += fb0 * mc[d] + fb1 * mc[MSTR + d] + fb2 * mc[2 * MSTR + d];
        }
        qacc[d] = qacc[d] + dq;
    }
    __syncwarp();
    PROF_MARK(P_DQ);
}

// Smooth dynamics and contact detection for the GW worlds of the warp; ncon per world.
// returns 1 when the base solve and F2 were deferred to the contact solve (allow_defer)
__device__ int group_smooth_detect(float* grp, const G1Tables& T, int lane, const QaccOpts& opt, float* const* bias_out,
                                   int* ncon, float* const* qs_out = nullptr, int allow_defer = 0) {
    const int defer = group_smooth(grp, T, lane, opt.bdt, bias_out, opt.bdt_all, allow_defer && !qs_out);
    if (qs_out)
        for (int it = lane; it < GW * NV; it += 32) {
            const int w = it / NV, d = it % NV;
            if (qs_out[w]) qs_out[w][d] = grp[w * WFLOATS + WL::QACC + d];
        }
#pragma unroll
    for (int w = 0; w < GW; ++w) ncon[w] = reinterpret_cast<const int*>(grp + w * WFLOATS + WL::MISC)[0];
    return defer;
}

// Full per-substep generalised acceleration for the GW worlds of the warp (qp, qv, tau
// filled in each frame), the warp solving its own contact batches.  env_qacc.cuh:27-212.
// qacc -> each frame's QACC; per-world outputs for k_qacc through the optional arrays.
// midbar (fused rollout only): bit 0 -- the CTA's warps (bar_threads threads) meet at named
// barrier 1 after the smooth dynamics, bit 1 -- after the contact solve.
__device__ void group_qacc(float* grp, float* cw, const G1Tables& T, int lane, const QaccOpts& opt, float* const* bias_out,
                           float* const* f_out, int* ncon_out, float* const* qs_out = nullptr, int midbar = 0,
                           int bar_threads = 0, int allow_defer = 0) {
    int ncon[GW];
    int smooth_lanes = group_smooth_detect(grp, T, lane, opt, bias_out, ncon, qs_out, allow_defer);
    if (midbar & 1) asm volatile("bar.sync 1, %0;" ::"r"(bar_threads) : "memory");
#pragma unroll
    for (int w = 0; w < GW; ++w) {
        if (ncon_out) ncon_out[w] = ncon[w];
        if (f_out && f_out[w] && ncon[w] == 0) f_out[w][lane] = 0.f;
    }
    // contact batches, formed greedily in slot order (at most MAXCON contacts each; worlds
    // without contacts skipped) and solved as they close
    auto solve = [&](const Batch& B) {
#ifdef G1_PROF
        if (lane == 0) atomicAdd(&g_prof[47 + B.cof(B.nw)], 1ull);  // batches by contact count 1..8
#endif
        batch_contact(grp, cw, T, lane, opt.pgs_iters, opt.mu, B, smooth_lanes);
        smooth_lanes = 0;  // the first batch finished the deferred smooth solves
        if (f_out)
#pragma unroll
            for (int x = 0; x < GW; ++x)
                if (x < B.nw && f_out[B.wof(x)]) {
                    const int n4 = 4 * (B.cof(x + 1) - B.cof(x));
                    f_out[B.wof(x)][lane] = lane < n4 ? cw[CL::FF + 4 * B.cof(x) + lane] : 0.f;
                }
    };
    Batch B;
    B.nw = 0;
    B.coff[0] = 0;
#pragma unroll
    for (int w = 0; w < GW; ++w) {
        if (ncon[w] > 0) {
            if (B.cof(B.nw) + ncon[w] > MAXCON) {
                solve(B);
                B.nw = 0;
            }
            B.append(w, ncon[w]);
        }
    }
    if (B.nw > 0) solve(B);
    PROF_BEGIN();
    if (midbar & 2) asm volatile("bar.sync 1, %0;" ::"r"(bar_threads) : "memory");
#ifdef G1_PROF
    (void)*(volatile const float*)grp;  // bar.sync blocks lazily: make the wait land here
#endif
    PROF_MARK(P_MIDBAR);
}

// ------------------------------------------------------------------ integration
// qvel += dt qacc (non-finite -> 0, clamp +-50), then the semi-implicit position update with
// the base quaternion exponential, for the GW worlds.  g1_env.cu:154-162, dynamics.cuh:333-355
__device__ void group_integrate(float* grp, const G1Tables& T, int lane, bool guard) {
    const float dt = G1M_DT;
    for (int it = lane; it < GW * NV; it += 32) {
        const int w = it / NV, d = it % NV;
        float* fr = grp + w * WFLOATS;
        float v = fr[WL::QV + d] + dt * fr[WL::QACC + d];
        if (guard) {
            if (!isfinite(v)) v = 0.f;
            if (v > 50.f) v = 50.f; else if (v < -50.f) v = -50.f;
        }
        fr[WL::QV + d] = v;
    }
    __syncwarp();
    // hinge joints in one uniform pass; the free joint of each world (the heavier quaternion
    // update) on lanes 0..GW-1 in a second pass
    for (int it = lane; it < GW * NJ; it += 32) {
        const int w = it / NJ, j = it % NJ;
        if (T.jnt_type[j] != 3) continue;
        float* fr = grp + w * WFLOATS;
        fr[WL::QP + T.jnt_qposadr[j]] += dt * fr[WL::QV + T.jnt_dofadr[j]];
    }
    if (lane < GW) {
        const int w = lane, j = T.free_jnt;
        float* fr = grp + w * WFLOATS;
        float *qp = fr + WL::QP;
        const float* qv = fr + WL::QV;
        const int qa = T.jnt_qposadr[j], da = T.jnt_dofadr[j];
        {
            qp[qa] += dt * qv[da]; qp[qa + 1] += dt * qv[da + 1]; qp[qa + 2] += dt * qv[da + 2];
            const V3 v = {qv[da + 3] * dt, qv[da + 4] * dt, qv[da + 5] * dt};
            const float ang = sqrtf(v.x * v.x + v.y * v.y + v.z * v.z);
            Q4 dq;
            if (ang < 1e-9f) dq = {1.f, 0.5f * v.x, 0.5f * v.y, 0.5f * v.z};
            else {
                float sn, cs;
                sincosf(0.5f * ang, &sn, &cs);
                sn = sn / ang;
                dq = {cs, v.x * sn, v.y * sn, v.z * sn};
            }
            st4(qp + qa + 3, qnormalize(qmul(ld4(qp + qa + 3), dq)));
        }
    }
    __syncwarp();
}

}  // namespace g1
