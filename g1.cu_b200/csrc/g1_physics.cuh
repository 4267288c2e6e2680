// g1_physics.cuh -- per-substep G1 dynamics for ONE world, executed by ONE warp.
//
// The reference runs a world per thread and keeps its ~25 KB working set in local memory
// (g1_env.cu:245, "255 regs, ~25-31 KB local frame").  Here a warp owns a world and its
// frame lives in shared memory; lanes split every step of the algorithm over the
// independent items it offers:
//   forward kinematics / RNE        one lane per body of a tree level  (root->leaf)
//   motion axes, body inertias      one lane per dof / per body
//   articulated-inertia factor      one lane per body of a level       (leaf->root, pull)
//   M^-1 back-solves                one lane per right-hand side: the smooth solve and the
//                                   3*ncon contact basis columns run together (25 lanes)
//   Gram / Delassus blocks          one lane per (contact pair, basis entry)
//   PGS                             one lane per constraint row, rows swept in order
// Within each item the arithmetic follows the reference's order (citations per function),
// so results agree with it to fp32 rounding.
#pragma once
#include "g1_tables.cuh"

#define FULLMASK 0xffffffffu

namespace g1 {

constexpr int NB = G1_NB, NV = G1_NV_, NQ = G1_NQ_, NJ = G1_NJ, NU = G1_NU_, NFOOT = G1_NFOOT_;
constexpr int MAXCON = G1_MAXCON, MAXEFC = G1_MAXEFC, CDS = G1_CDS, NRHS = G1_NRHS;
constexpr int ASTR = 33;   // row stride of the Delassus matrix in shared memory
constexpr int MSTR = 35;   // row stride of the back-solve buffer (35 is odd: conflict-free per lane row)

// compile-time tree for the fully unrolled per-lane back-solve
__device__ constexpr int kParent[NB] = {G1M_BODY_PARENT_LIST};
__device__ constexpr int kDofAdr[NB] = {G1M_BODY_DOFADR_LIST};

// ------------------------------------------------------------------ frame layout
// Offsets (in floats) inside one warp's shared-memory frame.
struct FrameLayout {
    enum : int {
        QP = 0,                    // qpos[36]
        QV = QP + 36,              // qvel[35] (+1)
        TGT = QV + 36,             // PD targets [29] (+3)
        TAU = TGT + 32,            // generalized force [35] (+1)
        QACC = TAU + 36,           // result qacc [35] (+1)
        MISC = QACC + 36,          // 16 scalars
        S = MISC + 16,             // motion axes [35*6]
        FU = S + 210,              // factor: U [31*6]
        FINVD = FU + 186,          // factor: 1/D [31] (+1)
        FU6 = FINVD + 32,          // base: U6 [36]
        FL6 = FU6 + 36,            // base: Dm, then its Cholesky factor [36]
        BIAS = FL6 + 36,           // qfrc_bias [35] (+1)
        CON = BIAS + 36,           // contacts: sphere(int) [8], pt [8*3], pen [8]
        EB = CON + 40,             // basis rows [8][3][12]
        BB = EB + 288,             // (spare) [24]
        RR = BB + 24,              // R [32]
        AREF = RR + 32,            // (spare) [32]
        BV = AREF + 32,            // b [32]
        FF = BV + 32,              // impulses f [32]
        MM = FF + 32,              // [25][35]: row 0 qacc_smooth, rows 1+3c+a contact basis solves
        UNION = MM + NRHS * MSTR,  // tree sweep scratch | Gram + Delassus matrix
        // union part 1: tree sweeps (dead once the contact basis is built)
        XPOS = UNION,              // body positions [31*3] (+3)
        XQUAT = XPOS + 96,         // body orientations [31*4]
        IAB = XQUAT + 124,         // per body: own articulated inertia, then its contribution [31*21]
        FOWN = IAB + NB * 21,      // per body: own force, then subtree force [31*6]
        PAC = FOWN + NB * 6,       // per body: articulated bias-force contribution [31*6]
        UB = PAC + NB * 6,         // per body: u_b = x_d - S_d.pA_b [31] (+1)
        BST = UB + 32,             // branch hand-off slots: pos,quat,w,v,aw,av (19) + a (6) -> 26 each
        A1 = BST + G1_MAXBRANCH * 26,  // base spatial acceleration [6] (+2)
        U1_END = A1 + 8,
        // union part 2
        GRAM = UNION,              // [36 pairs][9]
        AMAT = GRAM + 324,         // [32][33]
        U2_END = AMAT + MAXEFC * ASTR,
        SIZE = (U1_END > U2_END ? U1_END : U2_END)
    };
};

constexpr int FRAME_FLOATS = (FrameLayout::SIZE + 3) & ~3;

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

// Spatial inertia (-> ia_out[21]) and body force (-> f_out[6]) of body b from its frame and
// its spatial velocity / acceleration (shared by the base and the hinge bodies).
__device__ __noinline__ void body_inertia_force(const G1Tables& T, int b, Q4 quat, V3 pos, V3 p, V3 w, V3 v, V3 aw, V3 av,
                                                float* ia_out, float* f_out) {
    const V3 xip = add3(pos, qrot(quat, ld3(T.body_ipos + 3 * b)));
    float Iw[9];
    V3 c;
    world_inertia(T, b, quat, xip, p, Iw, c);
    const float m = T.body_mass[b];
    spatial_inertia21(Iw, c, m, ia_out);
    V3 fw, fv;
    body_force(Iw, c, m, w, v, aw, av, fw, fv);
    st3(f_out, fw);
    st3(f_out + 3, fv);
}

// The smooth part of the per-substep dynamics for the world in `fr` (qp, qv, tau filled):
// forward kinematics, motion axes S, RNE bias, the articulated-inertia factor of M + dtB
// and qacc_smooth = (M + dtB)^-1 (-bias + tau), written to MM row 0.
//
// Three sweeps over the chain decomposition of the tree, lane l walking chain l with the
// running body state in registers (hand-offs through shared memory only at branch bodies):
//   F1 (root->leaf): FK (dynamics.cuh:47-88), S (aba_bias.cuh:380-398), spatial inertias,
//      RNE partial velocities / cdof_dot / accelerations (aba_bias.cuh:419-457) and body
//      forces (aba_bias.cuh:458-466);
//   B1 (leaf->root): subtree forces and bias (aba_bias.cuh:467-475), the articulated
//      inertia factor (aba_factor.cuh:76-88) and, fused into the same pass, the bias-force
//      sweep of the smooth solve (aba_factor.cuh:128-136); a body pulls its children's
//      contributions in descending child index -- the order the reference pushes them;
//   base: the floating base's 6x6 block and Cholesky solve (aba_factor.cuh:90-108,138-155);
//   F2 (root->leaf): qdd per body (aba_factor.cuh:156-164).
__device__ void warp_smooth(float* fr, const G1Tables& T, int lane, const float* bdt) {
    using L = FrameLayout;
    const float *qp = fr + L::QP, *qv = fr + L::QV, *tau = fr + L::TAU;
    float *S = fr + L::S, *XPOS = fr + L::XPOS, *XQUAT = fr + L::XQUAT, *IAB = fr + L::IAB, *FOWN = fr + L::FOWN;
    float *PAC = fr + L::PAC, *UB = fr + L::UB, *BST = fr + L::BST, *FU = fr + L::FU, *FINVD = fr + L::FINVD;
    float* bias = fr + L::BIAS;
    float* qacc_s = fr + L::MM;
    const bool chain_lane = lane < T.nchain;

    // ---- floating base (body 1): every chain lane computes it (identical values)
    const V3 p = ld3(qp);
    const Q4 q1 = qnormalize(ld4(qp + 3));
    V3 bw = mk3(0, 0, 0), bv = mk3(0, 0, 0), baw = mk3(0, 0, 0), bav = mk3(-T.gravity[0], -T.gravity[1], -T.gravity[2]);
    if (chain_lane) {
        float R1[9];
        qmat(q1, R1);
        float Sb[6][6];
#pragma unroll
        for (int k = 0; k < 6; ++k)
#pragma unroll
            for (int i = 0; i < 6; ++i) Sb[k][i] = 0.f;
        Sb[0][3] = 1.f; Sb[1][4] = 1.f; Sb[2][5] = 1.f;
#pragma unroll
        for (int k = 0; k < 3; ++k) { Sb[3 + k][0] = R1[k]; Sb[3 + k][1] = R1[3 + k]; Sb[3 + k][2] = R1[6 + k]; }
        // RNE through the 6 base dofs (aba_bias.cuh:423-440)
        V3 Sdw[6], Sdv[6];
        V3 w = bw, v = bv;
#pragma unroll
        for (int a = 0; a < 3; ++a) {
            const float qd = qv[a];
            V3 sw = mk3(Sb[a][0], Sb[a][1], Sb[a][2]), sv = mk3(Sb[a][3], Sb[a][4], Sb[a][5]);
            Sdw[a] = cross3(w, sw);
            Sdv[a] = add3(cross3(w, sv), cross3(v, sw));
            w = {w.x + sw.x * qd, w.y + sw.y * qd, w.z + sw.z * qd};
            v = {v.x + sv.x * qd, v.y + sv.y * qd, v.z + sv.z * qd};
        }
        const V3 wr = w, vr = v;
#pragma unroll
        for (int a = 3; a < 6; ++a) {
            V3 sw = mk3(Sb[a][0], Sb[a][1], Sb[a][2]), sv = mk3(Sb[a][3], Sb[a][4], Sb[a][5]);
            Sdw[a] = cross3(wr, sw);
            Sdv[a] = add3(cross3(wr, sv), cross3(vr, sw));
        }
#pragma unroll
        for (int a = 3; a < 6; ++a) {
            const float qd = qv[a];
            w = {w.x + Sb[a][0] * qd, w.y + Sb[a][1] * qd, w.z + Sb[a][2] * qd};
            v = {v.x + Sb[a][3] * qd, v.y + Sb[a][4] * qd, v.z + Sb[a][5] * qd};
        }
        V3 ea = baw, eb = bav;
#pragma unroll
        for (int a = 0; a < 6; ++a) {
            const float qd = qv[a];
            ea = {ea.x + Sdw[a].x * qd, ea.y + Sdw[a].y * qd, ea.z + Sdw[a].z * qd};
            eb = {eb.x + Sdv[a].x * qd, eb.y + Sdv[a].y * qd, eb.z + Sdv[a].z * qd};
        }
        bw = w; bv = v; baw = ea; bav = eb;
        if (lane == 0) {
#pragma unroll
            for (int k = 0; k < 6; ++k)
#pragma unroll
                for (int i = 0; i < 6; ++i) S[6 * k + i] = Sb[k][i];
            st3(XPOS + 3, p);
            st4(XQUAT + 4, q1);
            body_inertia_force(T, 1, q1, p, p, bw, bv, baw, bav, IAB + 21, FOWN + 6);
        }
    }

    // ---- F1: root -> leaf along the chains
    {
        V3 pos = p, w = bw, v = bv, aw = baw, av = bav;
        Q4 quat = q1;
        for (int s = 0; s < T.nsteps; ++s) {
            const int k = chain_lane ? s - T.chain_start[lane] : -1;
            if (k >= 0 && k < T.chain_len[lane]) {
                const int b = T.chain_body[lane][k];
                if (k == 0 && T.parent[b] != 1) {  // head below a branch body: its state from the slot
                    const float* st = BST + 26 * T.branch_slot[T.parent[b]];
                    pos = ld3(st); quat = ld4(st + 3); w = ld3(st + 7); v = ld3(st + 10); aw = ld3(st + 13); av = ld3(st + 16);
                } else if (k == 0) {
                    pos = p; quat = q1; w = bw; v = bv; aw = baw; av = bav;
                }
                const int j = T.body_jnt[b], d = T.dofadr[b];
                // kinematics (hinge)
                pos = add3(pos, qrot(quat, ld3(T.body_pos + 3 * b)));
                quat = qmul(quat, ld4(T.body_quat + 4 * b));
                const V3 an = ld3(T.jnt_pos + 3 * j), ax = ld3(T.jnt_axis + 3 * j);
                const V3 anchor = add3(pos, qrot(quat, an));
                float sn, cs;
                sincosf(0.5f * qp[T.jnt_qposadr[j]], &sn, &cs);
                quat = qmul(quat, Q4{cs, ax.x * sn, ax.y * sn, ax.z * sn});
                pos = sub3(anchor, qrot(quat, an));
                st3(XPOS + 3 * b, pos);
                st4(XQUAT + 4 * b, quat);
                // motion axis of the hinge dof
                const V3 sw = qrot(quat, ax);
                const V3 sv = cross3(sub3(add3(pos, qrot(quat, an)), p), sw);
                st3(S + 6 * d, sw); st3(S + 6 * d + 3, sv);
                // RNE forward (one dof)
                const float qd = qv[d];
                const V3 sdw = cross3(w, sw), sdv = add3(cross3(w, sv), cross3(v, sw));
                w = {w.x + sw.x * qd, w.y + sw.y * qd, w.z + sw.z * qd};
                v = {v.x + sv.x * qd, v.y + sv.y * qd, v.z + sv.z * qd};
                aw = {aw.x + sdw.x * qd, aw.y + sdw.y * qd, aw.z + sdw.z * qd};
                av = {av.x + sdv.x * qd, av.y + sdv.y * qd, av.z + sdv.z * qd};
                body_inertia_force(T, b, quat, pos, p, w, v, aw, av, IAB + 21 * b, FOWN + 6 * b);
                if (T.branch_slot[b] >= 0) {
                    float* st = BST + 26 * T.branch_slot[b];
                    st3(st, pos); st4(st + 3, quat); st3(st + 7, w); st3(st + 10, v); st3(st + 13, aw); st3(st + 16, av);
                }
            }
            __syncwarp();
        }
    }

    // ---- B1: leaf -> root along the chains (bias, factor, smooth-solve bias forces).  A body
    // leaves its contributions (subtree force, IA - U U^T / D, pA + U ud) in its own slots,
    // where its parent pulls them.
    for (int s = 0; s < T.nsteps_back; ++s) {
        const int k = chain_lane ? s - T.chain_bstart[lane] : -1;
        const int len = chain_lane ? T.chain_len[lane] : 0;
        if (k >= 0 && k < len) {
            const int b = T.chain_body[lane][len - 1 - k], d = T.dofadr[b];
            float f[6], ia[21], pa[6];
#pragma unroll
            for (int i = 0; i < 6; ++i) { f[i] = FOWN[6 * b + i]; pa[i] = 0.f; }
#pragma unroll
            for (int i = 0; i < 21; ++i) ia[i] = IAB[21 * b + i];
            for (int q = T.child_start[b]; q < T.child_start[b + 1]; ++q) {
                const int c = T.child_list[q];
#pragma unroll
                for (int i = 0; i < 6; ++i) { f[i] += FOWN[6 * c + i]; pa[i] += PAC[6 * c + i]; }
#pragma unroll
                for (int i = 0; i < 21; ++i) ia[i] += IAB[21 * c + i];
            }
            float sd[6];
#pragma unroll
            for (int i = 0; i < 6; ++i) sd[i] = S[6 * d + i];
            const float bd = sd[0] * f[0] + sd[1] * f[1] + sd[2] * f[2] + sd[3] * f[3] + sd[4] * f[4] + sd[5] * f[5];
            bias[d] = bd;
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
#pragma unroll
            for (int i = 0; i < 6; ++i) FU[6 * b + i] = U[i];
            FINVD[b] = invD;
            UB[b] = u;
#pragma unroll
            for (int r = 0; r < 6; ++r)
#pragma unroll
                for (int c = r; c < 6; ++c) IAB[21 * b + sym6(r, c)] = ia[sym6(r, c)] - U[r] * U[c] * invD;
#pragma unroll
            for (int i = 0; i < 6; ++i) { PAC[6 * b + i] = pa[i] + U[i] * ud; FOWN[6 * b + i] = f[i]; }
        }
        __syncwarp();
    }

    // ---- floating base: pull the pelvis children (descending), 6x6 block, Cholesky, qdd
    const int b1 = 1;
    if (lane < 21) {
        float acc = IAB[21 * b1 + lane];
        for (int q = T.child_start[b1]; q < T.child_start[b1 + 1]; ++q) acc += IAB[21 * T.child_list[q] + lane];
        IAB[21 * b1 + lane] = acc;
    } else if (lane < 27) {
        const int i = lane - 21;
        float acc = FOWN[6 * b1 + i];
        for (int q = T.child_start[b1]; q < T.child_start[b1 + 1]; ++q) acc += FOWN[6 * T.child_list[q] + i];
        FOWN[6 * b1 + i] = acc;
    }
    if (lane < 6) {
        float acc = 0.f;
        for (int q = T.child_start[b1]; q < T.child_start[b1 + 1]; ++q) acc += PAC[6 * T.child_list[q] + lane];
        PAC[6 * b1 + lane] = acc;
    }
    __syncwarp();
    float *U6 = fr + L::FU6, *L6 = fr + L::FL6;
    for (int e = lane; e < 36; e += 32) {  // U6[i*6+l] = (IA S_l)[i]
        const int i = e / 6, l = e % 6;
        float acc = 0.f;
#pragma unroll
        for (int j = 0; j < 6; ++j) acc += IAB[21 * b1 + sym6(i, j)] * S[6 * l + j];
        U6[e] = acc;
    }
    float ub = 0.f;
    if (lane < 6) {  // base bias and u = (-bias + tau) - S^T pA
        const float* f = FOWN + 6 * b1;
        const float* sd = S + 6 * lane;
        const float bd = sd[0] * f[0] + sd[1] * f[1] + sd[2] * f[2] + sd[3] * f[3] + sd[4] * f[4] + sd[5] * f[5];
        bias[lane] = bd;
        float sp = 0.f;
#pragma unroll
        for (int i = 0; i < 6; ++i) sp += sd[i] * PAC[6 * b1 + i];
        ub = (-bd + tau[lane]) - sp;
    }
    __syncwarp();
    for (int e = lane; e < 36; e += 32) {  // Dm[k*6+l] = S_k . U6_l (+ diag)
        const int kk = e / 6, l = e % 6;
        float acc = 0.f;
#pragma unroll
        for (int i = 0; i < 6; ++i) acc += S[6 * kk + i] * U6[i * 6 + l];
        L6[e] = acc + (kk == l ? (T.armature[kk] + (bdt ? bdt[kk] : 0.f)) : 0.f);
    }
    __syncwarp();
    float q[6];
#pragma unroll
    for (int k = 0; k < 6; ++k) q[k] = __shfl_sync(FULLMASK, ub, k);
    if (lane == 0) {
        float* Dm = L6;  // in place (aba_factor.cuh:103-107), rolled loops: one lane, once per substep
#pragma unroll 1
        for (int i = 0; i < 6; ++i)
#pragma unroll 1
            for (int j = 0; j <= i; ++j) {
                float acc = Dm[i * 6 + j];
                for (int k = 0; k < j; ++k) acc -= Dm[i * 6 + k] * Dm[j * 6 + k];
                if (i == j) Dm[i * 6 + i] = sqrtf(acc); else Dm[i * 6 + j] = acc / Dm[j * 6 + j];
            }
#pragma unroll 1
        for (int i = 0; i < 6; ++i) {
            float acc = q[i];
            for (int k = 0; k < i; ++k) acc -= Dm[i * 6 + k] * q[k];
            q[i] = acc / Dm[i * 6 + i];
        }
#pragma unroll 1
        for (int i = 5; i >= 0; --i) {
            float acc = q[i];
            for (int k = i + 1; k < 6; ++k) acc -= Dm[k * 6 + i] * q[k];
            q[i] = acc / Dm[i * 6 + i];
        }
#pragma unroll
        for (int k = 0; k < 6; ++k) qacc_s[k] = q[k];
        float* A1 = fr + L::A1;
#pragma unroll
        for (int i = 0; i < 6; ++i) {
            float acc = 0.f;
#pragma unroll
            for (int k = 0; k < 6; ++k) acc += S[6 * k + i] * q[k];
            A1[i] = acc;
        }
    }
    __syncwarp();

    // ---- F2: root -> leaf, qdd per hinge body
    {
        float a[6];
        for (int s = 0; s < T.nsteps; ++s) {
            const int k = chain_lane ? s - T.chain_start[lane] : -1;
            if (k >= 0 && k < T.chain_len[lane]) {
                const int b = T.chain_body[lane][k], d = T.dofadr[b];
                if (k == 0) {
                    const int par = T.parent[b];
                    const float* src = par == 1 ? fr + L::A1 : BST + 26 * T.branch_slot[par] + 19;
#pragma unroll
                    for (int i = 0; i < 6; ++i) a[i] = src[i];
                }
                float s2 = 0.f;
#pragma unroll
                for (int i = 0; i < 6; ++i) s2 += FU[6 * b + i] * a[i];
                const float qdd = (UB[b] - s2) * FINVD[b];
                qacc_s[d] = qdd;
#pragma unroll
                for (int i = 0; i < 6; ++i) a[i] = a[i] + S[6 * d + i] * qdd;
                if (T.branch_slot[b] >= 0) {
                    float* st = BST + 26 * T.branch_slot[b] + 19;
#pragma unroll
                    for (int i = 0; i < 6; ++i) st[i] = a[i];
                }
            }
            __syncwarp();
        }
    }
}

// ------------------------------------------------------------------ M^-1 apply, one lane
// y = (M + dtB)^-1 x in place on xy[0..NV), one lane per right-hand side, reading the factor
// from the frame (every lane touches the same factor entry at the same time: a shared-memory
// broadcast).  aba_factor.cuh:121-165.
// The lane walks the chains with the articulated bias force of the current body in
// registers.  Leaf->root, chains go last-to-first; a chain's head leaves its contribution in
// hand[chain] and a body pulls its children's contributions in descending child index (the
// order in which the reference's b-descending loop pushes them).  u_b = x_d - S_d.pA_b parks
// in xy[d] between the sweeps.  Root->leaf, chains go first-to-last and a branch body leaves
// its spatial acceleration in fwd[slot] for the chains below it.
// `scratch`: this lane's 6*(MAXCHAIN + MAXBRANCH) floats.
constexpr int SOLVE_SCRATCH = 6 * (G1_MAXCHAIN + G1_MAXBRANCH);
static_assert(3 * MAXCON * SOLVE_SCRATCH <= FrameLayout::U1_END - FrameLayout::UNION,
              "per-lane solve scratch must fit in the tree-sweep part of the frame union");
__device__ __noinline__ void lane_solve(const float* fr, const G1Tables& T, float* xy, float* scratch) {
    using L = FrameLayout;
    const float *S = fr + L::S, *FU = fr + L::FU, *FINVD = fr + L::FINVD, *L6 = fr + L::FL6;
    float* hand = scratch;
    float* fwd = scratch + 6 * G1_MAXCHAIN;
    // leaf -> root
    for (int c = T.nchain - 1; c >= 0; --c) {
        const int len = T.chain_len[c];
        float pa[6] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        int carried = -1;
        for (int k = len - 1; k >= 0; --k) {
            const int b = T.chain_body[c][k], d = T.dofadr[b];
            float acc[6] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
            for (int q = T.child_start[b]; q < T.child_start[b + 1]; ++q) {
                const int ch = T.child_list[q];
                if (ch == carried) {
#pragma unroll
                    for (int i = 0; i < 6; ++i) acc[i] += pa[i];
                } else {
                    const float* src = hand + 6 * T.head_chain[ch];
#pragma unroll
                    for (int i = 0; i < 6; ++i) acc[i] += src[i];
                }
            }
            const float* sd = S + 6 * d;
            const float sp = ((((0.f + sd[0] * acc[0]) + sd[1] * acc[1]) + sd[2] * acc[2]) + sd[3] * acc[3]) + sd[4] * acc[4] + sd[5] * acc[5];
            const float u = xy[d] - sp;
            xy[d] = u;
            const float ud = u * FINVD[b];
            const float* U = FU + 6 * b;
#pragma unroll
            for (int i = 0; i < 6; ++i) pa[i] = acc[i] + U[i] * ud;
            carried = b;
        }
#pragma unroll
        for (int i = 0; i < 6; ++i) hand[6 * c + i] = pa[i];
    }
    // floating base: pull the pelvis children, 6x6 Cholesky solve, base acceleration
    const int d1 = T.dofadr[1];
    float pa1[6] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int q = T.child_start[1]; q < T.child_start[2]; ++q) {
        const float* src = hand + 6 * T.head_chain[T.child_list[q]];
#pragma unroll
        for (int i = 0; i < 6; ++i) pa1[i] += src[i];
    }
    float q6[6];
#pragma unroll
    for (int k = 0; k < 6; ++k) {
        const float* sd = S + 6 * (d1 + k);
        q6[k] = xy[d1 + k] - (((((0.f + sd[0] * pa1[0]) + sd[1] * pa1[1]) + sd[2] * pa1[2]) + sd[3] * pa1[3]) + sd[4] * pa1[4] + sd[5] * pa1[5]);
    }
#pragma unroll
    for (int i = 0; i < 6; ++i) {
        float acc = q6[i];
#pragma unroll
        for (int k = 0; k < i; ++k) acc -= L6[i * 6 + k] * q6[k];
        q6[i] = acc / L6[i * 6 + i];
    }
#pragma unroll
    for (int i = 5; i >= 0; --i) {
        float acc = q6[i];
#pragma unroll
        for (int k = i + 1; k < 6; ++k) acc -= L6[k * 6 + i] * q6[k];
        q6[i] = acc / L6[i * 6 + i];
    }
    float a1[6];
#pragma unroll
    for (int i = 0; i < 6; ++i) {
        float acc = 0.f;
#pragma unroll
        for (int k = 0; k < 6; ++k) acc += S[6 * (d1 + k) + i] * q6[k];
        a1[i] = acc;
    }
#pragma unroll
    for (int k = 0; k < 6; ++k) xy[d1 + k] = q6[k];
    // root -> leaf
    for (int c = 0; c < T.nchain; ++c) {
        const int par = T.parent[T.chain_body[c][0]];
        float a[6];
        if (par == 1) {
#pragma unroll
            for (int i = 0; i < 6; ++i) a[i] = a1[i];
        } else {
            const float* src = fwd + 6 * T.branch_slot[par];
#pragma unroll
            for (int i = 0; i < 6; ++i) a[i] = src[i];
        }
        for (int k = 0; k < T.chain_len[c]; ++k) {
            const int b = T.chain_body[c][k], d = T.dofadr[b];
            const float* U = FU + 6 * b;
            const float s2 = ((((0.f + U[0] * a[0]) + U[1] * a[1]) + U[2] * a[2]) + U[3] * a[3]) + U[4] * a[4] + U[5] * a[5];
            const float qdd = (xy[d] - s2) * FINVD[b];
            xy[d] = qdd;
            const float* sd = S + 6 * d;
#pragma unroll
            for (int i = 0; i < 6; ++i) a[i] = a[i] + sd[i] * qdd;
            if (T.branch_slot[b] >= 0) {
                float* dst = fwd + 6 * T.branch_slot[b];
#pragma unroll
                for (int i = 0; i < 6; ++i) dst[i] = a[i];
            }
        }
    }
}

// ------------------------------------------------------------------ profiling (G1_PROF builds)
#ifdef G1_PROF
__device__ unsigned long long g_prof[16];
#define PROF_BEGIN() long long _pt = clock64();
#define PROF_MARK(i)                                                                          \
    do {                                                                                      \
        long long _n = clock64();                                                             \
        if ((threadIdx.x & 31) == 0) atomicAdd(&g_prof[i], (unsigned long long)(_n - _pt));   \
        _pt = _n;                                                                             \
    } while (0)
#else
#define PROF_BEGIN()
#define PROF_MARK(i) do { } while (0)
#endif
enum ProfPhase { P_POLICY = 0, P_FK, P_AXES, P_BIAS, P_FACTOR, P_CSETUP, P_SOLVE, P_GRAM, P_PGS, P_DQ, P_STEP, P_WAIT, P_NPHASE };

// pyramid coefficients d_k = DC[k] of the 3-basis (env_qacc.cuh:98-100,154-155)
__device__ __forceinline__ float dcoef(int k, int a) {
    if (a == 0) return 1.f;
    if (a == 1) return k == 0 ? 1.f : (k == 1 ? -1.f : 0.f);
    return k == 2 ? 1.f : (k == 3 ? -1.f : 0.f);
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
    const float* bdt;  // shared-memory dt*B diagonal (may be null)
};

// Full per-substep generalized acceleration for the world in `fr` (qp, qv, tau filled);
// FK must have run.  env_qacc.cuh:27-212.  Writes qacc to fr[QACC]; f / ncon stay in the
// frame.  Returns ncon.
__device__ int warp_qacc(float* fr, const G1Tables& T, int lane, const QaccOpts& opt) {
    using L = FrameLayout;
    PROF_BEGIN();
    warp_smooth(fr, T, lane, opt.bdt);
    PROF_MARK(P_FACTOR);
    const float* S = fr + L::S;
    float* MM = fr + L::MM;
    int* con_s = reinterpret_cast<int*>(fr + L::CON);
    float *con_pt = fr + L::CON + 8, *con_pen = fr + L::CON + 32;
    // foot spheres vs z=0, compacted in sphere order (contact.cuh:31-46)
    bool hit = false;
    float cx = 0, cy = 0, pen = 0;
    if (lane < NFOOT) {
        int b = T.foot_body[lane];
        const float* xp = fr + L::XPOS + 3 * b;
        V3 c = add3(ld3(xp), qrot(ld4(fr + L::XQUAT + 4 * b), ld3(T.foot_lpos + 3 * lane)));
        pen = c.z - G1M_FOOT_RADIUS;
        hit = pen < 0.f;
        cx = c.x; cy = c.y;
    }
    unsigned m = __ballot_sync(FULLMASK, hit);
    int ncon = __popc(m);
    if (hit) {
        int k = __popc(m & ((1u << lane) - 1u));
        con_s[k] = lane;
        con_pt[3 * k] = cx; con_pt[3 * k + 1] = cy; con_pt[3 * k + 2] = pen * 0.5f;
        con_pen[k] = pen;
    }
    V3 p = ld3(fr + L::XPOS + 3);
    // contact basis right-hand sides: rows 1..3ncon (zero-filled; row 0 holds qacc_smooth)
    const int nrhs = 1 + 3 * ncon;
    for (int e = MSTR + lane; e < nrhs * MSTR; e += 32) MM[e] = 0.f;
    __syncwarp();
    // contact basis rows e0 = n, e1 = mu t1, e2 = mu t2 over the ancestor dofs
    // (env_qacc.cuh:113-126), one lane per (contact, dof)
    float* EB = fr + L::EB;
    for (int it = lane; it < ncon * CDS; it += 32) {
        int c = it / CDS, k = it % CDS, s = con_s[c];
        if (k < T.foot_ndof[s]) {
            int a = T.foot_dofs[s][k];
            V3 r = sub3(ld3(con_pt + 3 * c), p);
            V3 t = add3(cross3(ld3(S + 6 * a), r), ld3(S + 6 * a + 3));
            float e0 = t.z, e1 = opt.mu * t.y, e2 = -opt.mu * t.x;
            EB[c * 36 + k] = e0; EB[c * 36 + 12 + k] = e1; EB[c * 36 + 24 + k] = e2;
            MM[(1 + 3 * c) * MSTR + a] = e0; MM[(2 + 3 * c) * MSTR + a] = e1; MM[(3 + 3 * c) * MSTR + a] = e2;
        }
    }
    __syncwarp();
    PROF_MARK(P_CSETUP);
    // all basis back-solves at once: lane r solves basis column r
    if (lane < nrhs - 1) lane_solve(fr, T, MM + (lane + 1) * MSTR, fr + L::UNION + lane * SOLVE_SCRATCH);
    __syncwarp();
    PROF_MARK(P_SOLVE);
    float* qacc = fr + L::QACC;
    if (ncon == 0) {
        for (int d = lane; d < NV; d += 32) qacc[d] = MM[d];
        __syncwarp();
        return 0;
    }
    // per contact: bb = e.qacc_smooth, e.qvel -> R, aref, b  (env_qacc.cuh:113-136, 188-191)
    float *RR = fr + L::RR, *BV = fr + L::BV;
    if (lane < ncon) {
        int c = lane, s = con_s[c], nd = T.foot_ndof[s];
        const float* qv = fr + L::QV;
        float b0 = 0, b1 = 0, b2 = 0, v0 = 0, v1 = 0, v2 = 0;
        for (int k = 0; k < nd; ++k) {
            int a = T.foot_dofs[s][k];
            float e0 = EB[c * 36 + k], e1 = EB[c * 36 + 12 + k], e2 = EB[c * 36 + 24 + k];
            float qa = MM[a], qd = qv[a];
            b0 += e0 * qa; b1 += e1 * qa; b2 += e2 * qa;
            v0 += e0 * qd; v1 += e1 * qd; v2 += e2 * qd;
        }
        float dmax = T.solimp[1], tc = T.solref[0], dr = T.solref[1];
        float bcoef = 2.f / (dmax * tc);
        float kcoef = 1.f / (dmax * dmax * tc * tc * dr * dr);
        float pyr = (1.f + opt.mu * opt.mu) * (2.f * opt.mu * opt.mu / G1M_FOOT_IMPRATIO);
        float pn = con_pen[c], imp = foot_impedance(T, pn);
        float Rc = T.foot_invw0[s] * pyr * (1.f - imp) / imp;
        float kip = kcoef * imp * pn;
        float dv[4] = {v0 + v1, v0 - v1, v0 + v2, v0 - v2};
        float db[4] = {b0 + b1, b0 - b1, b0 + b2, b0 - b2};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            float aref = -bcoef * dv[k] - kip;
            RR[4 * c + k] = Rc;
            BV[4 * c + k] = db[k] - aref;
        }
    }
    // 3x3 Gram blocks G[a][b] = e_{c,a} . m_{c',b} over c's dofs, c <= c'
    // (env_qacc.cuh:161-171), one lane per (pair, a, b)
    float* G = fr + L::GRAM;
    const int npair = ncon * (ncon + 1) / 2;
    for (int it = lane; it < npair * 9; it += 32) {
        int pr = it / 9, ab = it % 9, a = ab / 3, bb = ab % 3;
        int c = 0, rem = pr;
        while (rem >= ncon - c) { rem -= ncon - c; ++c; }
        int cp = c + rem, s = con_s[c], nd = T.foot_ndof[s];
        const float* ea = EB + c * 36 + 12 * a;
        const float* mcp = MM + (1 + 3 * cp + bb) * MSTR;
        float g = 0.f;
        for (int k = 0; k < nd; ++k) g += ea[k] * mcp[T.foot_dofs[s][k]];
        G[pr * 9 + ab] = g;
    }
    __syncwarp();
    // Delassus A = J M^-1 J' + diag R: expand each Gram block to the 4x4 pyramid block
    // (env_qacc.cuh:172-187), one lane per (pair, k)
    float* A = fr + L::AMAT;
    const int nefc = 4 * ncon;
    for (int it = lane; it < npair * 4; it += 32) {
        int pr = it >> 2, k = it & 3;
        int c = 0, rem = pr;
        while (rem >= ncon - c) { rem -= ncon - c; ++c; }
        int cp = c + rem;
        const float* g = G + 9 * pr;
        const float c0 = dcoef(k, 0), c1 = dcoef(k, 1), c2 = dcoef(k, 2);
        float t0 = c0 * g[0] + c1 * g[3] + c2 * g[6];
        float t1 = c0 * g[1] + c1 * g[4] + c2 * g[7];
        float t2 = c0 * g[2] + c1 * g[5] + c2 * g[8];
        int i = 4 * c + k;
        // inside a diagonal block (c == cp) the reference writes (k,kp) and (kp,k) from both
        // iterations and the later one (larger k) wins; this lane owns kp <= k only
        const int kpmax = (c == cp) ? k : 3;
#pragma unroll
        for (int kp = 0; kp < 4; ++kp) {
            if (kp > kpmax) break;
            float aij = t0 * dcoef(kp, 0) + t1 * dcoef(kp, 1) + t2 * dcoef(kp, 2);
            int j = 4 * cp + kp;
            if (i == j) aij += RR[i];
            A[i * ASTR + j] = aij;
            A[j * ASTR + i] = aij;
        }
    }
    __syncwarp();
    PROF_MARK(P_GRAM);
    // projected Gauss-Seidel, rows in order (contact.cuh:159-171).  Lane j keeps the
    // residual r_j = b_j + sum_k A_jk f_k; after row i moves by delta, every lane updates
    // its residual with column i of A.
    float fj = 0.f, rj = lane < nefc ? BV[lane] : 0.f, ajj = lane < nefc ? A[lane * ASTR + lane] : 1.f;
    float inv = 1.f / ajj;
    for (int itr = 0; itr < opt.pgs_iters; ++itr) {
        for (int i = 0; i < nefc; ++i) {
            float aji = lane < nefc ? A[i * ASTR + lane] : 0.f;
            float delta = 0.f;
            if (lane == i) {
                float ri = rj - ajj * fj;
                float fn = -ri * inv;
                fn = fn > 0.f ? fn : 0.f;
                delta = fn - fj;
                fj = fn;
            }
            delta = __shfl_sync(FULLMASK, delta, i);
            rj += aji * delta;
        }
    }
    float* F = fr + L::FF;
    if (lane < nefc) F[lane] = fj;
    __syncwarp();
    PROF_MARK(P_PGS);
    // qacc = qacc_smooth + sum_c sum_a fb_c[a] m_{c,a}  (env_qacc.cuh:199-211)
    for (int d = lane; d < NV; d += 32) {
        float dq = 0.f;
        for (int c = 0; c < ncon; ++c) {
            float f0 = F[4 * c], f1 = F[4 * c + 1], f2 = F[4 * c + 2], f3 = F[4 * c + 3];
            float fb0 = f0 + f1 + f2 + f3, fb1 = f0 - f1, fb2 = f2 - f3;
            const float* mc = MM + (1 + 3 * c) * MSTR;
            dq += fb0 * mc[d] + fb1 * mc[MSTR + d] + fb2 * mc[2 * MSTR + d];
        }
        qacc[d] = MM[d] + dq;
    }
    __syncwarp();
    PROF_MARK(P_DQ);
    return ncon;
}

// ------------------------------------------------------------------ integration
// qvel += dt qacc (non-finite -> 0, clamp +-50), then the semi-implicit position update
// with the base quaternion exponential.  g1_env.cu:154-162, dynamics.cuh:333-355
__device__ void warp_integrate(float* fr, const G1Tables& T, int lane, bool guard) {
    using L = FrameLayout;
    float *qp = fr + L::QP, *qv = fr + L::QV;
    const float* qacc = fr + L::QACC;
    const float dt = G1M_DT;
    for (int d = lane; d < NV; d += 32) {
        float v = qv[d] + dt * qacc[d];
        if (guard) {
            if (!isfinite(v)) v = 0.f;
            if (v > 50.f) v = 50.f; else if (v < -50.f) v = -50.f;
        }
        qv[d] = v;
    }
    __syncwarp();
    for (int j = lane; j < NJ; j += 32) {
        int qa = T.jnt_qposadr[j], da = T.jnt_dofadr[j];
        if (T.jnt_type[j] == 3) {
            qp[qa] += dt * qv[da];
        } else {
            qp[qa] += dt * qv[da]; qp[qa + 1] += dt * qv[da + 1]; qp[qa + 2] += dt * qv[da + 2];
            V3 v = {qv[da + 3] * dt, qv[da + 4] * dt, qv[da + 5] * dt};
            float ang = sqrtf(v.x * v.x + v.y * v.y + v.z * v.z);
            Q4 dq;
            if (ang < 1e-9f) dq = {1.f, 0.5f * v.x, 0.5f * v.y, 0.5f * v.z};
            else {
                float s, c;
                sincosf(0.5f * ang, &s, &c);
                s = s / ang;
                dq = {c, v.x * s, v.y * s, v.z * s};
            }
            Q4 qn = qnormalize(qmul(ld4(qp + qa + 3), dq));
            st4(qp + qa + 3, qn);
        }
    }
    __syncwarp();
}

}  // namespace g1
