/*
 * g1_oracle.c -- CPU ORACLE for the fused G1 rollout.  TEST INFRASTRUCTURE ONLY.
 *
 * This file is the checker, never the product: only tests/, __graft_entry__.smoke() and
 * bench.py's CPU-baseline legs load it.  The shipped library (g1.cu_b200/libg1env.so) has
 * no CPU path and never links this file.
 *
 * It restates, in plain C, the algorithm of the reference's rollout hot path
 * (Infatoshi/g1.cu).  Every function names the reference file:line it follows.  The
 * arithmetic order inside each function follows the reference so that the fp32 build
 * reproduces the reference's host-compiled fp32 numbers to rounding level, and the fp64
 * build (REAL=double) serves as the high-precision oracle.
 *
 * Build (oracle/build_oracle.py):  gcc -O2 -fopenmp -shared -fPIC -DREAL=float|double
 *
 * Parity is pinned by tests/test_oracle_golden.py against the MuJoCo-generated goldens the
 * reference commits (bench/ref_traj.npz, bench/contact_solve_ref.npz, bench/implicit_ref.npz,
 * copied as fixtures under tests/golden/) and, where the reference tree is present, against
 * the reference's own physics headers compiled for the host (oracle/_ref).
 *
 * RNG: the reference draws from curand XORWOW (g1_env.cu:92-95,206,310).  This build uses
 * Philox4x32-10 (Salmon, Moraes, Dror, Shaw, SC'11) with the counter layout documented at
 * orc_philox() below; the GPU kernel uses the same layout, so RNG streams are bit-identical
 * between oracle and kernel (pinned by the paper's known-answer vectors in the tests).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include "../g1.cu_b200/csrc/g1_model_data.h"

#ifndef REAL
#define REAL float
#endif
typedef REAL R;

#define NB G1M_NBODY
#define NQ G1M_NQ
#define NV G1M_NV
#define NJ G1M_NJNT
#define NU G1M_NU
#define NFOOT G1M_NFOOT
#define MAXCON NFOOT
#define MAXEFC (4 * MAXCON)
#define OBS 100
#define ACT 29
#define CDS 12 /* ancestor dofs of a foot body: 6 base + 6 leg hinges (env_qacc.cuh:80-83) */

/* math wrappers: float or double flavour chosen by sizeof(R) at compile time */
#define ISF (sizeof(R) == sizeof(float))
static inline R r_sqrt(R x) { return ISF ? (R)sqrtf((float)x) : (R)sqrt((double)x); }
static inline R r_sin(R x) { return ISF ? (R)sinf((float)x) : (R)sin((double)x); }
static inline R r_cos(R x) { return ISF ? (R)cosf((float)x) : (R)cos((double)x); }
static inline R r_exp(R x) { return ISF ? (R)expf((float)x) : (R)exp((double)x); }
static inline R r_expm1(R x) { return ISF ? (R)expm1f((float)x) : (R)expm1((double)x); }
static inline R r_log(R x) { return ISF ? (R)logf((float)x) : (R)log((double)x); }
static inline R r_tanh(R x) { return ISF ? (R)tanhf((float)x) : (R)tanh((double)x); }
static inline R r_pow(R x, R y) { return ISF ? (R)powf((float)x, (float)y) : (R)pow((double)x, (double)y); }
static inline R r_abs(R x) { return x < 0 ? -x : x; }
static inline int r_finite(R x) { return isfinite(x); }

/* ----------------------------------------------------------------- small vector algebra */
typedef struct { R x, y, z; } V3;
typedef struct { R w, x, y, z; } Q4;

static inline V3 v3(R x, R y, R z) { V3 r = {x, y, z}; return r; }
static inline V3 vadd(V3 a, V3 b) { return v3(a.x + b.x, a.y + b.y, a.z + b.z); }
static inline V3 vsub(V3 a, V3 b) { return v3(a.x - b.x, a.y - b.y, a.z - b.z); }
static inline V3 vcross(V3 a, V3 b) {
    return v3(a.y * b.z - a.z * b.y, a.z * b.x - a.x * b.z, a.x * b.y - a.y * b.x);
}
static inline R vdot(V3 a, V3 b) { return a.x * b.x + a.y * b.y + a.z * b.z; }
static inline V3 vload(const R* p) { return v3(p[0], p[1], p[2]); }
static inline V3 vloadf(const float* p) { return v3(p[0], p[1], p[2]); }
static inline Q4 qloadf(const float* p) { Q4 q = {p[0], p[1], p[2], p[3]}; return q; }
static inline Q4 qload(const R* p) { Q4 q = {p[0], p[1], p[2], p[3]}; return q; }

/* Hamilton product, dynamics.cuh:17-24 */
static inline Q4 qmul(Q4 a, Q4 b) {
    Q4 r;
    r.w = a.w * b.w - a.x * b.x - a.y * b.y - a.z * b.z;
    r.x = a.w * b.x + a.x * b.w + a.y * b.z - a.z * b.y;
    r.y = a.w * b.y - a.x * b.z + a.y * b.w + a.z * b.x;
    r.z = a.w * b.z + a.x * b.y - a.y * b.x + a.z * b.w;
    return r;
}
/* v' = v + w t + u x t, t = 2 u x v  (dynamics.cuh:26-35) */
static inline V3 qrot(Q4 q, V3 v) {
    R tx = 2 * (q.y * v.z - q.z * v.y), ty = 2 * (q.z * v.x - q.x * v.z), tz = 2 * (q.x * v.y - q.y * v.x);
    return v3(v.x + q.w * tx + (q.y * tz - q.z * ty),
              v.y + q.w * ty + (q.z * tx - q.x * tz),
              v.z + q.w * tz + (q.x * ty - q.y * tx));
}
/* dynamics.cuh:36-39 (rsqrt) */
static inline Q4 qnormalize(Q4 q) {
    R n = (R)1 / r_sqrt(q.w * q.w + q.x * q.x + q.y * q.y + q.z * q.z);
    Q4 r = {q.w * n, q.x * n, q.y * n, q.z * n};
    return r;
}
/* rotation matrix, row-major (dynamics.cuh:99-106) */
static inline void qmat(Q4 q, R m[9]) {
    R w = q.w, x = q.x, y = q.y, z = q.z;
    m[0] = 1 - 2 * (y * y + z * z); m[1] = 2 * (x * y - w * z);     m[2] = 2 * (x * z + w * y);
    m[3] = 2 * (x * y + w * z);     m[4] = 1 - 2 * (x * x + z * z); m[5] = 2 * (y * z - w * x);
    m[6] = 2 * (x * z - w * y);     m[7] = 2 * (y * z + w * x);     m[8] = 1 - 2 * (x * x + y * y);
}

/* ----------------------------------------------------------------- kinematics */
/* Body frames from qpos.  dynamics.cuh:47-88 */
static void orc_fk_one(const R* qpos, R* xpos, R* xquat, R* xipos) {
    xpos[0] = xpos[1] = xpos[2] = 0;
    xquat[0] = 1; xquat[1] = xquat[2] = xquat[3] = 0;
    for (int b = 1; b < NB; ++b) {
        int p = G1M_BODY_PARENT[b];
        Q4 qp = qload(&xquat[4 * p]);
        V3 pos = vadd(vload(&xpos[3 * p]), qrot(qp, vloadf(&G1M_BODY_POS[3 * b])));
        Q4 quat = qmul(qp, qloadf(&G1M_BODY_QUAT[4 * b]));
        for (int jj = 0; jj < G1M_BODY_JNTNUM[b]; ++jj) {
            int j = G1M_BODY_JNTADR[b] + jj, qa = G1M_JNT_QPOSADR[j];
            if (G1M_JNT_TYPE[j] == 0) {
                pos = v3(qpos[qa], qpos[qa + 1], qpos[qa + 2]);
                Q4 q = {qpos[qa + 3], qpos[qa + 4], qpos[qa + 5], qpos[qa + 6]};
                quat = qnormalize(q);
            } else if (G1M_JNT_TYPE[j] == 3) {
                V3 ax = vloadf(&G1M_JNT_AXIS[3 * j]), an = vloadf(&G1M_JNT_POS[3 * j]);
                V3 anchor = vadd(pos, qrot(quat, an));
                R h = (R)0.5 * qpos[qa], s = r_sin(h);
                Q4 loc = {r_cos(h), ax.x * s, ax.y * s, ax.z * s};
                quat = qmul(quat, loc);
                pos = vsub(anchor, qrot(quat, an));
            }
        }
        xpos[3 * b] = pos.x; xpos[3 * b + 1] = pos.y; xpos[3 * b + 2] = pos.z;
        xquat[4 * b] = quat.w; xquat[4 * b + 1] = quat.x; xquat[4 * b + 2] = quat.y; xquat[4 * b + 3] = quat.z;
        V3 cw = vadd(pos, qrot(quat, vloadf(&G1M_BODY_IPOS[3 * b])));
        xipos[3 * b] = cw.x; xipos[3 * b + 1] = cw.y; xipos[3 * b + 2] = cw.z;
    }
    xipos[0] = xipos[1] = xipos[2] = 0;
}

/* ----------------------------------------------------------------- spatial inertia */
/* Body inertia about the pelvis origin p, world axes: rotational part Iw (row-major 3x3)
 * and com offset c.  dynamics.cuh:108-115 (world_inertia) and aba_bias.cuh:400-410. */
static void body_inertia_world(const R* xquat, const R* xipos, V3 p, int b, R Iw[9], V3* c) {
    R Rm[9];
    qmat(qmul(qload(&xquat[4 * b]), qloadf(&G1M_BODY_IQUAT[4 * b])), Rm);
    R d0 = G1M_BODY_INERTIA[3 * b], d1 = G1M_BODY_INERTIA[3 * b + 1], d2 = G1M_BODY_INERTIA[3 * b + 2];
    for (int i = 0; i < 3; ++i)
        for (int j = 0; j < 3; ++j)
            Iw[3 * i + j] = Rm[3 * i] * d0 * Rm[3 * j] + Rm[3 * i + 1] * d1 * Rm[3 * j + 1] +
                            Rm[3 * i + 2] * d2 * Rm[3 * j + 2];
    *c = v3(xipos[3 * b] - p.x, xipos[3 * b + 1] - p.y, xipos[3 * b + 2] - p.z);
}

/* apply (Iw,c,m) to a spatial motion [w;v]  (dynamics.cuh:126-139) */
static void inertia_apply(const R Iw[9], V3 c, R m, V3 sw, V3 sv, V3* fw, V3* fv) {
    V3 A = v3(Iw[0] * sw.x + Iw[1] * sw.y + Iw[2] * sw.z, Iw[3] * sw.x + Iw[4] * sw.y + Iw[5] * sw.z,
              Iw[6] * sw.x + Iw[7] * sw.y + Iw[8] * sw.z);
    R cc = vdot(c, c), csw = vdot(c, sw);
    A = v3(A.x + m * (cc * sw.x - csw * c.x), A.y + m * (cc * sw.y - csw * c.y), A.z + m * (cc * sw.z - csw * c.z));
    V3 a = vcross(c, sv);
    *fw = v3(A.x + m * a.x, A.y + m * a.y, A.z + m * a.z);
    V3 b = vcross(c, sw);
    *fv = v3(-m * b.x + m * sv.x, -m * b.y + m * sv.y, -m * b.z + m * sv.z);
}

/* 6x6 packed-symmetric index (aba.cuh:20-23) */
static inline int sym6(int i, int j) {
    if (i > j) { int t = i; i = j; j = t; }
    return i * 6 - (i * (i - 1)) / 2 + (j - i);
}

/* ----------------------------------------------------------------- RNE bias + motion axes */
/* qfrc_bias by RNE with qacc=0 and base acceleration -g, plus the motion axes S[NV*6]
 * (world axes about the pelvis origin).  aba_bias.cuh:17-121 */
static void orc_bias_one(const R* qvel, const R* xpos, const R* xquat, const R* xipos, R* S, R* bias) {
    V3 p = vload(&xpos[3]);
    R R1[9];
    qmat(qload(&xquat[4]), R1);
    for (int i = 0; i < NV * 6; ++i) S[i] = 0;
    for (int j = 0; j < NJ; ++j) {
        int b = G1M_JNT_BODY[j], d = G1M_JNT_DOFADR[j];
        if (G1M_JNT_TYPE[j] == 0) {
            S[(d + 0) * 6 + 3] = 1; S[(d + 1) * 6 + 4] = 1; S[(d + 2) * 6 + 5] = 1;
            for (int k = 0; k < 3; ++k) {
                S[(d + 3 + k) * 6 + 0] = R1[k]; S[(d + 3 + k) * 6 + 1] = R1[3 + k]; S[(d + 3 + k) * 6 + 2] = R1[6 + k];
            }
        } else if (G1M_JNT_TYPE[j] == 3) {
            Q4 qb = qload(&xquat[4 * b]);
            V3 aw = qrot(qb, vloadf(&G1M_JNT_AXIS[3 * j]));
            V3 anchor = vadd(vload(&xpos[3 * b]), qrot(qb, vloadf(&G1M_JNT_POS[3 * j])));
            V3 rxa = vcross(vsub(anchor, p), aw);
            S[d * 6 + 0] = aw.x; S[d * 6 + 1] = aw.y; S[d * 6 + 2] = aw.z;
            S[d * 6 + 3] = rxa.x; S[d * 6 + 4] = rxa.y; S[d * 6 + 5] = rxa.z;
        }
    }
    R Iw[NB][9]; V3 cb[NB];
    for (int b = 1; b < NB; ++b) body_inertia_world(xquat, xipos, p, b, Iw[b], &cb[b]);

    V3 vw[NB], vv[NB], aw[NB], av[NB], Sdw[NV], Sdv[NV];
    vw[0] = v3(0, 0, 0); vv[0] = v3(0, 0, 0); aw[0] = v3(0, 0, 0);
    av[0] = v3(-(R)G1M_GRAVITY[0], -(R)G1M_GRAVITY[1], -(R)G1M_GRAVITY[2]);
    for (int b = 1; b < NB; ++b) {
        int par = G1M_BODY_PARENT[b], da = G1M_BODY_DOFADR[b], dn = G1M_BODY_DOFNUM[b];
        V3 w = vw[par], v = vv[par];
        /* cdof_dot = (partial velocity) x_m S_a; the free joint's three rotational dofs all
         * use the post-translation partial velocity (aba_bias.cuh:423-440) */
        int nseq = (dn == 6) ? 3 : dn;
        for (int a = da; a < da + nseq; ++a) {
            R qd = qvel[a];
            V3 sw = vload(&S[a * 6]), sv = vload(&S[a * 6 + 3]);
            Sdw[a] = vcross(w, sw);
            Sdv[a] = vadd(vcross(w, sv), vcross(v, sw));
            w = v3(w.x + sw.x * qd, w.y + sw.y * qd, w.z + sw.z * qd);
            v = v3(v.x + sv.x * qd, v.y + sv.y * qd, v.z + sv.z * qd);
        }
        if (dn == 6) {
            V3 wr = w, vr = v;
            for (int a = da + 3; a < da + 6; ++a) {
                V3 sw = vload(&S[a * 6]), sv = vload(&S[a * 6 + 3]);
                Sdw[a] = vcross(wr, sw);
                Sdv[a] = vadd(vcross(wr, sv), vcross(vr, sw));
            }
            for (int a = da + 3; a < da + 6; ++a) {
                R qd = qvel[a];
                w = v3(w.x + S[a * 6 + 0] * qd, w.y + S[a * 6 + 1] * qd, w.z + S[a * 6 + 2] * qd);
                v = v3(v.x + S[a * 6 + 3] * qd, v.y + S[a * 6 + 4] * qd, v.z + S[a * 6 + 5] * qd);
            }
        }
        vw[b] = w; vv[b] = v;
        V3 ea = aw[par], eb = av[par];
        for (int a = da; a < da + dn; ++a) {
            R qd = qvel[a];
            ea = v3(ea.x + Sdw[a].x * qd, ea.y + Sdw[a].y * qd, ea.z + Sdw[a].z * qd);
            eb = v3(eb.x + Sdv[a].x * qd, eb.y + Sdv[a].y * qd, eb.z + Sdv[a].z * qd);
        }
        aw[b] = ea; av[b] = eb;
    }
    V3 fw[NB], fv[NB];
    for (int b = 1; b < NB; ++b) {
        R m = G1M_BODY_MASS[b];
        V3 Iaw, Iav, Ivw, Ivv;
        inertia_apply(Iw[b], cb[b], m, aw[b], av[b], &Iaw, &Iav);
        inertia_apply(Iw[b], cb[b], m, vw[b], vv[b], &Ivw, &Ivv);
        /* v x* (I v) = [w x n + vv x f ; w x f]  (dynamics.cuh:148-152) */
        V3 cn = vadd(vcross(vw[b], Ivw), vcross(vv[b], Ivv)), cf = vcross(vw[b], Ivv);
        fw[b] = vadd(Iaw, cn); fv[b] = vadd(Iav, cf);
    }
    for (int a = 0; a < NV; ++a) bias[a] = 0;
    for (int b = NB - 1; b >= 1; --b) {
        int da = G1M_BODY_DOFADR[b], dn = G1M_BODY_DOFNUM[b];
        for (int a = da; a < da + dn; ++a)
            bias[a] = S[a * 6 + 0] * fw[b].x + S[a * 6 + 1] * fw[b].y + S[a * 6 + 2] * fw[b].z +
                      S[a * 6 + 3] * fv[b].x + S[a * 6 + 4] * fv[b].y + S[a * 6 + 5] * fv[b].z;
        int par = G1M_BODY_PARENT[b];
        if (par >= 1) { fw[par] = vadd(fw[par], fw[b]); fv[par] = vadd(fv[par], fv[b]); }
    }
}

/* ----------------------------------------------------------------- ABA factor / M^-1 */
typedef struct {
    R U[NB * 6]; R invD[NB]; R U6[36]; R L6[36];
} Factor;

/* Articulated-inertia factorisation of (M + diag(bdt)), leaf->root.
 * aba_factor.cuh:44-109 */
static void orc_factor(const R* xpos, const R* xquat, const R* xipos, const R* S, const R* bdt, Factor* F) {
    V3 p = vload(&xpos[3]);
    R IA[NB][21];
    for (int b = 1; b < NB; ++b) {
        R Iw[9]; V3 c;
        body_inertia_world(xquat, xipos, p, b, Iw, &c);
        R m = G1M_BODY_MASS[b], cc = vdot(c, c);
        R A[9];
        for (int i = 0; i < 9; ++i) A[i] = Iw[i];
        A[0] += m * (cc - c.x * c.x); A[1] += m * (-c.x * c.y); A[2] += m * (-c.x * c.z);
        A[3] += m * (-c.y * c.x);     A[4] += m * (cc - c.y * c.y); A[5] += m * (-c.y * c.z);
        A[6] += m * (-c.z * c.x);     A[7] += m * (-c.z * c.y); A[8] += m * (cc - c.z * c.z);
        R sk[9] = {0, -c.z, c.y, c.z, 0, -c.x, -c.y, c.x, 0};
        R M6[36];
        for (int i = 0; i < 3; ++i)
            for (int j = 0; j < 3; ++j) {
                M6[6 * i + j] = A[3 * i + j];
                M6[6 * i + j + 3] = m * sk[3 * i + j];
                M6[6 * (i + 3) + j] = -m * sk[3 * i + j];
                M6[6 * (i + 3) + j + 3] = (i == j) ? m : 0;
            }
        for (int i = 0; i < 6; ++i)
            for (int j = i; j < 6; ++j) IA[b][sym6(i, j)] = M6[6 * i + j];
    }
    for (int b = NB - 1; b >= 2; --b) {
        int par = G1M_BODY_PARENT[b], d = G1M_BODY_DOFADR[b];
        R U[6];
        for (int i = 0; i < 6; ++i) {
            R s = 0;
            for (int j = 0; j < 6; ++j) s += IA[b][sym6(i, j)] * S[d * 6 + j];
            U[i] = s;
        }
        R D = 0;
        for (int i = 0; i < 6; ++i) D += S[d * 6 + i] * U[i];
        D = D + (R)G1M_DOF_ARMATURE[d];
        if (bdt) D += bdt[d];
        R invD = (R)1 / D;
        for (int k = 0; k < 6; ++k) F->U[b * 6 + k] = U[k];
        F->invD[b] = invD;
        for (int i = 0; i < 6; ++i)
            for (int j = i; j < 6; ++j) IA[par][sym6(i, j)] += IA[b][sym6(i, j)] - U[i] * U[j] * invD;
    }
    int d = G1M_BODY_DOFADR[1];
    for (int l = 0; l < 6; ++l)
        for (int i = 0; i < 6; ++i) {
            R s = 0;
            for (int j = 0; j < 6; ++j) s += IA[1][sym6(i, j)] * S[(d + l) * 6 + j];
            F->U6[i * 6 + l] = s;
        }
    R Dm[36];
    for (int k = 0; k < 6; ++k)
        for (int l = 0; l < 6; ++l) {
            R s = 0;
            for (int i = 0; i < 6; ++i) s += S[(d + k) * 6 + i] * F->U6[i * 6 + l];
            Dm[k * 6 + l] = s + (k == l ? ((R)G1M_DOF_ARMATURE[d + k] + (bdt ? bdt[d + k] : 0)) : 0);
        }
    for (int i = 0; i < 6; ++i)
        for (int j = 0; j <= i; ++j) {
            R s = Dm[i * 6 + j];
            for (int k = 0; k < j; ++k) s -= Dm[i * 6 + k] * Dm[j * 6 + k];
            if (i == j) Dm[i * 6 + i] = r_sqrt(s); else Dm[i * 6 + j] = s / Dm[j * 6 + j];
        }
    for (int i = 0; i < 36; ++i) F->L6[i] = Dm[i];
}

/* y = (M + diag bdt)^-1 x using the stored factor.  aba_factor.cuh:121-165 (and the
 * identical per-column math of aba_solvem_multi.cuh:21-125). */
static void orc_solve(const Factor* F, const R* S, const R* x, R* y) {
    R pA[NB * 6], a6[NB * 6];
    for (int i = 0; i < NB * 6; ++i) pA[i] = 0;
    for (int b = NB - 1; b >= 2; --b) {
        int par = G1M_BODY_PARENT[b], d = G1M_BODY_DOFADR[b];
        R s = 0;
        for (int i = 0; i < 6; ++i) s += S[d * 6 + i] * pA[b * 6 + i];
        R ud = (x[d] - s) * F->invD[b];
        for (int k = 0; k < 6; ++k) pA[par * 6 + k] += pA[b * 6 + k] + F->U[b * 6 + k] * ud;
    }
    int d = G1M_BODY_DOFADR[1];
    R q[6];
    for (int k = 0; k < 6; ++k) {
        R s = 0;
        for (int i = 0; i < 6; ++i) s += S[(d + k) * 6 + i] * pA[6 + i];
        q[k] = x[d + k] - s;
    }
    const R* L = F->L6;
    for (int i = 0; i < 6; ++i) { R s = q[i]; for (int k = 0; k < i; ++k) s -= L[i * 6 + k] * q[k]; q[i] = s / L[i * 6 + i]; }
    for (int i = 5; i >= 0; --i) { R s = q[i]; for (int k = i + 1; k < 6; ++k) s -= L[k * 6 + i] * q[k]; q[i] = s / L[i * 6 + i]; }
    for (int k = 0; k < 6; ++k) y[d + k] = q[k];
    for (int i = 0; i < 6; ++i) {
        R s = 0;
        for (int k = 0; k < 6; ++k) s += S[(d + k) * 6 + i] * q[k];
        a6[6 + i] = s;
    }
    for (int b = 2; b < NB; ++b) {
        int par = G1M_BODY_PARENT[b], db = G1M_BODY_DOFADR[b];
        R s1 = 0, s2 = 0;
        for (int i = 0; i < 6; ++i) s1 += S[db * 6 + i] * pA[b * 6 + i];
        for (int i = 0; i < 6; ++i) s2 += F->U[b * 6 + i] * a6[par * 6 + i];
        R qdd = ((x[db] - s1) - s2) * F->invD[b];
        y[db] = qdd;
        for (int i = 0; i < 6; ++i) a6[b * 6 + i] = a6[par * 6 + i] + S[db * 6 + i] * qdd;
    }
}

/* The same apply in the column form of aba_solvem_multi.cuh:21-125 with K=1, which the
 * reference's contact pass uses (env_qacc.cuh:143-152): the hinge terms are subtracted one
 * at a time from the right-hand side instead of summed first. */
static void orc_solve_multi1(const Factor* F, const R* S, const R* x, R* y) {
    R pA[NB * 6], a6[NB * 6];
    for (int i = 0; i < NB * 6; ++i) pA[i] = 0;
    for (int b = NB - 1; b >= 2; --b) {
        int par = G1M_BODY_PARENT[b], d = G1M_BODY_DOFADR[b];
        R ud = x[d];
        for (int i = 0; i < 6; ++i) ud -= S[d * 6 + i] * pA[b * 6 + i];
        ud *= F->invD[b];
        for (int k = 0; k < 6; ++k) pA[par * 6 + k] += pA[b * 6 + k] + F->U[b * 6 + k] * ud;
    }
    int d = G1M_BODY_DOFADR[1];
    R q[6];
    for (int k = 0; k < 6; ++k) {
        R s = 0;
        for (int j = 0; j < 6; ++j) s += S[(d + k) * 6 + j] * pA[6 + j];
        q[k] = x[d + k] - s;
    }
    const R* L = F->L6;
    for (int i = 0; i < 6; ++i) { R s = q[i]; for (int k = 0; k < i; ++k) s -= L[i * 6 + k] * q[k]; q[i] = s / L[i * 6 + i]; }
    for (int i = 5; i >= 0; --i) { R s = q[i]; for (int k = i + 1; k < 6; ++k) s -= L[k * 6 + i] * q[k]; q[i] = s / L[i * 6 + i]; }
    for (int k = 0; k < 6; ++k) y[d + k] = q[k];
    for (int i = 0; i < 6; ++i) {
        R s = 0;
        for (int k = 0; k < 6; ++k) s += S[(d + k) * 6 + i] * q[k];
        a6[6 + i] = s;
    }
    for (int b = 2; b < NB; ++b) {
        int par = G1M_BODY_PARENT[b], db = G1M_BODY_DOFADR[b];
        R qdd = x[db];
        for (int i = 0; i < 6; ++i) qdd -= S[db * 6 + i] * pA[b * 6 + i] + F->U[b * 6 + i] * a6[par * 6 + i];
        qdd *= F->invD[b];
        y[db] = qdd;
        for (int i = 0; i < 6; ++i) a6[b * 6 + i] = a6[par * 6 + i] + S[db * 6 + i] * qdd;
    }
}

/* ----------------------------------------------------------------- contact */
/* MuJoCo solimp impedance.  contact.cuh:97-109 */
static R foot_impedance(R pos) {
    R dmin = G1M_FOOT_SOLIMP[0], dmax = G1M_FOOT_SOLIMP[1], width = G1M_FOOT_SOLIMP[2];
    R mid = G1M_FOOT_SOLIMP[3], power = G1M_FOOT_SOLIMP[4];
    R x = r_abs(pos) / width, y;
    if (x >= 1) y = 1;
    else {
        R a = (R)1 / r_pow(mid, power - 1), b = (R)1 / r_pow(1 - mid, power - 1);
        y = (x < mid) ? a * r_pow(x, power) : 1 - b * r_pow(1 - x, power);
    }
    return dmin + y * (dmax - dmin);
}

typedef struct {
    int ncon;
    int body[MAXCON];
    R pt[MAXCON][3];
    R pen[MAXCON];
    R invw0[MAXCON];
} Contacts;

/* 8 foot spheres vs the plane z=0.  contact.cuh:31-46 (+ invweight0, env_qacc.cuh:59-65) */
static void detect_contacts(const R* xpos, const R* xquat, Contacts* C) {
    C->ncon = 0;
    for (int s = 0; s < NFOOT; ++s) {
        int b = G1M_FOOT_BODY[s];
        V3 c = vadd(vload(&xpos[3 * b]), qrot(qload(&xquat[4 * b]), vloadf(&G1M_FOOT_LPOS[3 * s])));
        R pen = c.z - (R)G1M_FOOT_RADIUS;
        if (pen < 0) {
            int k = C->ncon++;
            C->body[k] = b; C->pen[k] = pen;
            C->pt[k][0] = c.x; C->pt[k][1] = c.y; C->pt[k][2] = pen * (R)0.5;
            C->invw0[k] = G1M_FOOT_INVWEIGHT0[s];
        }
    }
}

/* Ancestor dof list of a body in the reference's walk order (env_qacc.cuh:89-96). */
static int ancestor_dofs(int body, unsigned char* out) {
    int n = 0;
    for (int b = body; b >= 1; b = G1M_BODY_PARENT[b])
        for (int a = G1M_BODY_DOFADR[b]; a < G1M_BODY_DOFADR[b] + G1M_BODY_DOFNUM[b]; ++a) out[n++] = (unsigned char)a;
    return n;
}

/* Projected Gauss-Seidel on min 1/2 f'Af + f'b, f>=0, rows in order.  contact.cuh:159-171 */
static void solve_pgs(const R* A, const R* b, R* f, int n, int iters) {
    for (int i = 0; i < n; ++i) f[i] = 0;
    for (int it = 0; it < iters; ++it)
        for (int i = 0; i < n; ++i) {
            R Aii = A[i * n + i], r = b[i];
            for (int j = 0; j < n; ++j) r += A[i * n + j] * f[j];
            r -= Aii * f[i];
            R fi = -r / Aii;
            f[i] = fi > 0 ? fi : 0;
        }
}

/* Per-substep generalized acceleration: (M+dtB)^-1(-bias+tau) plus the foot-contact
 * correction in the reference's 3-basis pyramidal formulation.  env_qacc.cuh:27-212.
 * Optional outputs: S (motion axes), f (contact impulses, 4*ncon), ncon, qacc_smooth, bias. */
typedef struct {
    R S[NV * 6];
    R bias[NV];
    R qacc_s[NV];
    R f[MAXEFC];
    int ncon;
} QaccAux;

static void orc_qacc_one(const R* qp, const R* qv, const R* xpos, const R* xquat, const R* xipos,
                         const R* tau, const R* bdt, int pgs_iters, R mu, R* qacc, QaccAux* X) {
    R* S = X->S;
    orc_bias_one(qv, xpos, xquat, xipos, S, X->bias);
    Factor F;
    orc_factor(xpos, xquat, xipos, S, bdt, &F);
    R rhs[NV];
    for (int i = 0; i < NV; ++i) rhs[i] = -X->bias[i] + tau[i];
    orc_solve(&F, S, rhs, X->qacc_s);
    (void)qp;
    Contacts C;
    detect_contacts(xpos, xquat, &C);
    X->ncon = C.ncon;
    for (int i = 0; i < MAXEFC; ++i) X->f[i] = 0;
    if (C.ncon == 0) { for (int i = 0; i < NV; ++i) qacc[i] = X->qacc_s[i]; return; }
    int ncon = C.ncon, nefc = 4 * ncon;
    V3 p = vload(&xpos[3]);
    /* R / aref coefficients (env_qacc.cuh:69-72) */
    R dmax = G1M_FOOT_SOLIMP[1], tc = G1M_FOOT_SOLREF[0], dr = G1M_FOOT_SOLREF[1];
    R bcoef = 2 / (dmax * tc);
    R kcoef = 1 / (dmax * dmax * tc * tc * dr * dr);
    R pyr = (1 + mu * mu) * (2 * mu * mu / (R)G1M_FOOT_IMPRATIO);

    unsigned char cdof[MAXCON][CDS]; int cnd[MAXCON];
    R Eb[MAXCON][3][CDS], bb[MAXCON][3], Rr[MAXEFC], aref[MAXEFC];
    /* PASS 1: sparse 3-basis rows e0=n, e1=mu t1, e2=mu t2 from the point Jacobian
     * (env_qacc.cuh:113-136) */
    for (int c = 0; c < ncon; ++c) {
        cnd[c] = ancestor_dofs(C.body[c], cdof[c]);
        V3 pt = v3(C.pt[c][0], C.pt[c][1], C.pt[c][2]), r = vsub(pt, p);
        R b0 = 0, b1 = 0, b2 = 0, u0 = 0, u1 = 0, u2 = 0;
        for (int k = 0; k < cnd[c]; ++k) {
            int a = cdof[c][k];
            V3 t = vadd(vcross(vload(&S[a * 6]), r), vload(&S[a * 6 + 3]));
            R e0 = t.z, e1 = mu * t.y, e2 = -mu * t.x;
            Eb[c][0][k] = e0; Eb[c][1][k] = e1; Eb[c][2][k] = e2;
            R qa = X->qacc_s[a]; b0 += e0 * qa; b1 += e1 * qa; b2 += e2 * qa;
            R qd = qv[a];        u0 += e0 * qd; u1 += e1 * qd; u2 += e2 * qd;
        }
        bb[c][0] = b0; bb[c][1] = b1; bb[c][2] = b2;
        R pen = C.pen[c], imp = foot_impedance(pen);
        R Rc = C.invw0[c] * pyr * (1 - imp) / imp, kip = kcoef * imp * pen;
        R dv[4] = {u0 + u1, u0 - u1, u0 + u2, u0 - u2};
        for (int k = 0; k < 4; ++k) { Rr[4 * c + k] = Rc; aref[4 * c + k] = -bcoef * dv[k] - kip; }
    }
    /* PASS 2: M^-1 of each basis row (env_qacc.cuh:143-152) */
    R Mm[MAXCON][3][NV];
    for (int c = 0; c < ncon; ++c)
        for (int a = 0; a < 3; ++a) {
            R e[NV];
            for (int i = 0; i < NV; ++i) e[i] = 0;
            for (int k = 0; k < cnd[c]; ++k) e[cdof[c][k]] = Eb[c][a][k];
            orc_solve_multi1(&F, S, e, Mm[c][a]);
        }
    /* A = J M^-1 J' + diag R via 3x3 Gram blocks expanded to the 4x4 pyramid, and
     * b = d.bb - aref (env_qacc.cuh:155-192) */
    static const R DC[4][3] = {{1, 1, 0}, {1, -1, 0}, {1, 0, 1}, {1, 0, -1}};
    R A[MAXEFC * MAXEFC], bv[MAXEFC];
    for (int c = 0; c < ncon; ++c) {
        for (int cp = c; cp < ncon; ++cp) {
            R G[3][3];
            for (int a = 0; a < 3; ++a) {
                R g0 = 0, g1 = 0, g2 = 0;
                for (int k = 0; k < cnd[c]; ++k) {
                    R v = Eb[c][a][k]; int dd = cdof[c][k];
                    g0 += v * Mm[cp][0][dd]; g1 += v * Mm[cp][1][dd]; g2 += v * Mm[cp][2][dd];
                }
                G[a][0] = g0; G[a][1] = g1; G[a][2] = g2;
            }
            for (int k = 0; k < 4; ++k) {
                const R* dk = DC[k];
                R t0 = dk[0] * G[0][0] + dk[1] * G[1][0] + dk[2] * G[2][0];
                R t1 = dk[0] * G[0][1] + dk[1] * G[1][1] + dk[2] * G[2][1];
                R t2 = dk[0] * G[0][2] + dk[1] * G[1][2] + dk[2] * G[2][2];
                int i = 4 * c + k;
                for (int kp = 0; kp < 4; ++kp) {
                    R aij = t0 * DC[kp][0] + t1 * DC[kp][1] + t2 * DC[kp][2];
                    int j = 4 * cp + kp;
                    if (i == j) aij += Rr[i];
                    A[i * nefc + j] = aij; A[j * nefc + i] = aij;
                }
            }
        }
        for (int k = 0; k < 4; ++k)
            bv[4 * c + k] = DC[k][0] * bb[c][0] + DC[k][1] * bb[c][1] + DC[k][2] * bb[c][2] - aref[4 * c + k];
    }
    R f[MAXEFC];
    solve_pgs(A, bv, f, nefc, pgs_iters);
    for (int i = 0; i < nefc; ++i) X->f[i] = f[i];
    /* dq = sum_c sum_a fb_c[a] * Mm[c][a]  (env_qacc.cuh:199-211) */
    R dq[NV];
    for (int a = 0; a < NV; ++a) dq[a] = 0;
    for (int c = 0; c < ncon; ++c) {
        R f0 = f[4 * c], f1 = f[4 * c + 1], f2 = f[4 * c + 2], f3 = f[4 * c + 3];
        R fb0 = f0 + f1 + f2 + f3, fb1 = f0 - f1, fb2 = f2 - f3;
        for (int a = 0; a < NV; ++a) dq[a] += fb0 * Mm[c][0][a] + fb1 * Mm[c][1][a] + fb2 * Mm[c][2][a];
    }
    for (int i = 0; i < NV; ++i) qacc[i] = X->qacc_s[i] + dq[i];
}

/* ----------------------------------------------------------------- integration */
/* q <- q (x) exp(w dt) with w in the body frame.  dynamics.cuh:333-342 */
static void quat_step(R* q, V3 w, R dt) {
    V3 v = v3(w.x * dt, w.y * dt, w.z * dt);
    R ang = r_sqrt(v.x * v.x + v.y * v.y + v.z * v.z);
    Q4 dq;
    if (ang < (R)1e-9) { dq.w = 1; dq.x = (R)0.5 * v.x; dq.y = (R)0.5 * v.y; dq.z = (R)0.5 * v.z; }
    else { R s = r_sin((R)0.5 * ang) / ang; dq.w = r_cos((R)0.5 * ang); dq.x = v.x * s; dq.y = v.y * s; dq.z = v.z * s; }
    Q4 qn = qnormalize(qmul(qload(q), dq));
    q[0] = qn.w; q[1] = qn.x; q[2] = qn.y; q[3] = qn.z;
}
/* semi-implicit Euler position update.  dynamics.cuh:345-355 */
static void integrate_pos(R* qpos, const R* qvel, R dt) {
    for (int j = 0; j < NJ; ++j) {
        int qa = G1M_JNT_QPOSADR[j], da = G1M_JNT_DOFADR[j];
        if (G1M_JNT_TYPE[j] == 0) {
            qpos[qa] += dt * qvel[da]; qpos[qa + 1] += dt * qvel[da + 1]; qpos[qa + 2] += dt * qvel[da + 2];
            quat_step(&qpos[qa + 3], v3(qvel[da + 3], qvel[da + 4], qvel[da + 5]), dt);
        } else if (G1M_JNT_TYPE[j] == 3) {
            qpos[qa] += dt * qvel[da];
        }
    }
}

/* ----------------------------------------------------------------- Philox4x32-10 RNG */
/* Philox4x32 with 10 rounds (Salmon et al., SC'11, "Parallel random numbers: as easy as
 * 1, 2, 3").  Round: (hi0,lo0)=M0*x0, (hi1,lo1)=M1*x2; x <- {hi1^x1^k0, lo1, hi0^x3^k1, lo0};
 * key bumped by the Weyl constants between rounds. */
void orc_philox(const uint32_t ctr[4], const uint32_t key[2], uint32_t out[4]) {
    uint32_t x0 = ctr[0], x1 = ctr[1], x2 = ctr[2], x3 = ctr[3], k0 = key[0], k1 = key[1];
    for (int r = 0; r < 10; ++r) {
        if (r) { k0 += 0x9E3779B9u; k1 += 0xBB67AE85u; }
        uint64_t p0 = (uint64_t)0xD2511F53u * x0, p1 = (uint64_t)0xCD9E8D57u * x2;
        uint32_t hi0 = (uint32_t)(p0 >> 32), lo0 = (uint32_t)p0, hi1 = (uint32_t)(p1 >> 32), lo1 = (uint32_t)p1;
        x0 = hi1 ^ x1 ^ k0; x1 = lo1; x2 = hi0 ^ x3 ^ k1; x3 = lo0;
    }
    out[0] = x0; out[1] = x1; out[2] = x2; out[3] = x3;
}
/* Counter layout shared with the CUDA kernel:
 *   ctr = {global world id, tick low 32, tick high 32, (purpose << 16) | index}
 *   key = {seed low 32, seed high 32}
 * purpose 1 = action noise (index = action i), 2 = auto-reset joint noise (index = actuator),
 * 3 = g1_env_reset joint noise.  'tick' is the env's control-step counter. */
#define RNG_ACTION 1u
#define RNG_AUTORESET 2u
#define RNG_RESET 3u
static void rng_draw(uint64_t seed, uint32_t world, uint64_t tick, uint32_t purpose, uint32_t idx, uint32_t out[4]) {
    uint32_t c[4] = {world, (uint32_t)tick, (uint32_t)(tick >> 32), (purpose << 16) | idx};
    uint32_t k[2] = {(uint32_t)seed, (uint32_t)(seed >> 32)};
    orc_philox(c, k, out);
}
/* uniform in (0,1]  (as curand_uniform's range) from the top 24 bits */
static inline float u01_open(uint32_t x) { return (float)((x >> 8) + 1u) * (1.0f / 16777216.0f); }
static inline float u01(uint32_t x) { return (float)(x >> 8) * (1.0f / 16777216.0f); }
/* standard normal by Box-Muller (cosine branch) from one Philox block */
static inline R normal_from(const uint32_t o[4]) {
    R u1 = u01_open(o[0]), u2 = u01(o[1]);
    return r_sqrt(-2 * r_log(u1)) * r_cos((R)6.283185307179586 * u2);
}

/* ----------------------------------------------------------------- env step */
typedef struct {
    int N, S, pgs;
    R mu;
    uint64_t seed;
    uint32_t world0;   /* global id of world 0 (multi-GPU sharding) */
    uint64_t tick;
    R* qp; R* qv; R* pa; int* steps;
} OrcEnv;

#define ACT_SCALE 0.5
#define CMD_VX 0.8
#define X_FIN 5.0
#define FINISH_BONUS 50.0

/* observation vector (g1_env.cu:46-53, 69-81) */
static void compute_obs(const R* qp, const R* qv, const R* pa, R* o) {
    for (int i = 0; i < 6; ++i) o[i] = qv[i];
    R m[9];
    Q4 qb = {qp[3], qp[4], qp[5], qp[6]};
    qmat(qb, m);
    o[6] = -m[6]; o[7] = -m[7]; o[8] = -m[8];
    for (int i = 0; i < ACT; ++i) o[9 + i] = qp[G1M_ACT_QADR[i]];
    for (int i = 0; i < ACT; ++i) o[38 + i] = qv[G1M_ACT_DOF[i]];
    for (int i = 0; i < ACT; ++i) o[67 + i] = pa[i];
    o[96] = (R)CMD_VX; o[97] = 0; o[98] = 0; o[99] = 0;
}

/* one control step of one world: PD targets, S substeps, reward, done, auto-reset.
 * g1_env.cu:118-212 */
static void env_advance(OrcEnv* E, int w, uint64_t tick, R* lp, R* lv, R* pa, int* step, const R* a, R* r_out, int* done_out) {
    R target[ACT];
    for (int i = 0; i < ACT; ++i) {
        R t = (R)G1M_QPOS_STAND[G1M_ACT_QADR[i]] + (R)ACT_SCALE * a[i];
        if (t < (R)G1M_ACT_CTRL_LO[i]) t = G1M_ACT_CTRL_LO[i];
        if (t > (R)G1M_ACT_CTRL_HI[i]) t = G1M_ACT_CTRL_HI[i];
        target[i] = t;
    }
    R bdt[NV];
    for (int i = 0; i < NV; ++i) bdt[i] = 0;
    for (int i = 0; i < ACT; ++i) bdt[G1M_ACT_DOF[i]] = (R)G1M_DT * (R)G1M_ACT_KD[i];
    R xpos[NB * 3], xquat[NB * 4], xipos[NB * 3], tau[NV], qacc[NV];
    R dt = (R)G1M_DT, vx_sum = 0, energy = 0;
    QaccAux X;
    for (int s = 0; s < E->S; ++s) {
        orc_fk_one(lp, xpos, xquat, xipos);
        for (int i = 0; i < NV; ++i) tau[i] = 0;
        for (int i = 0; i < ACT; ++i) {
            int d = G1M_ACT_DOF[i];
            R pd = (R)G1M_ACT_KP[i] * (target[i] - lp[G1M_ACT_QADR[i]]) - (R)G1M_ACT_KD[i] * lv[d];
            if (pd < (R)G1M_ACT_FRC_LO[i]) pd = G1M_ACT_FRC_LO[i];
            else if (pd > (R)G1M_ACT_FRC_HI[i]) pd = G1M_ACT_FRC_HI[i];
            tau[d] = pd;
            energy += r_abs(pd * lv[d]);
        }
        orc_qacc_one(lp, lv, xpos, xquat, xipos, tau, bdt, E->pgs, E->mu, qacc, &X);
        for (int i = 0; i < NV; ++i) {
            R v = lv[i] + dt * qacc[i];
            if (!r_finite(v)) v = 0;
            if (v > 50) v = 50; else if (v < -50) v = -50;
            lv[i] = v;
        }
        integrate_pos(lp, lv, dt);
        vx_sum += lv[0];
    }
    R vx = vx_sum / (R)E->S, height = lp[2];
    R m[9];
    Q4 qb = {lp[3], lp[4], lp[5], lp[6]};
    qmat(qb, m);
    R up = m[8];
    int alive = !(height < (R)0.45 || up < (R)0.5);
    R upc = up < 0 ? 0 : (up > 1 ? 1 : up);
    R vxc = vx > (R)CMD_VX ? (R)CMD_VX : vx;
    if (vxc < 0) vxc = 0;
    R r_vel = 1 * vxc * upc;
    R r_lat = (R)-0.2 * r_abs(lv[1]) - (R)0.05 * r_abs(lv[5]);
    R r_up = (R)0.3 * upc;
    R r_h = (R)-0.5 * r_abs(height - (R)0.78);
    R pen = 0;
    for (int i = 0; i < ACT; ++i) { R da = a[i] - pa[i]; pen += da * da; }
    if (pen > 10) pen = 10;
    R r = alive ? 1 + r_vel + r_lat + r_up + r_h - (R)0.005 * pen - (R)1e-4 * energy : (R)-5;
    *step += 1;
    int won = alive && lp[0] >= (R)X_FIN;
    if (won) r += (R)FINISH_BONUS;
    int d_flag = (!alive || won || *step >= 1000) ? 1 : 0;
    for (int i = 0; i < ACT; ++i) pa[i] = a[i];
    if (d_flag) {
        for (int i = 0; i < NQ; ++i) lp[i] = G1M_QPOS_STAND[i];
        for (int i = 0; i < ACT; ++i) {
            uint32_t o[4];
            rng_draw(E->seed, E->world0 + (uint32_t)w, tick, RNG_AUTORESET, (uint32_t)i, o);
            lp[G1M_ACT_QADR[i]] += (R)0.05 * ((R)u01_open(o[0]) * 2 - 1);
        }
        for (int i = 0; i < NV; ++i) lv[i] = 0;
        for (int i = 0; i < ACT; ++i) pa[i] = 0;
        *step = 0;
    }
    *r_out = r; *done_out = d_flag;
}

/* ----------------------------------------------------------------- policy MLP */
/* Actor-critic forward (g1_env.cu:214-239 for the 2-layer tanh default; generalised to any
 * hidden widths and to ELU).  Packed weights, torch Linear [out,in] row-major, in order:
 * for each hidden layer W,b; then Wmu,bmu, Wv,bv, log_std[ACT]  (ppo_fused.py:35-44). */
typedef struct { int nh; int h[4]; int act; /* 0 tanh, 1 elu */ } Policy;

static void mlp_forward(const Policy* P, const float* W, const R* x, R* mu, R* ls, R* val) {
    R buf0[1024], buf1[1024];
    const R* in = x; int nin = OBS;
    const float* w = W;
    R* outs[2] = {buf0, buf1};
    for (int l = 0; l < P->nh; ++l) {
        int no = P->h[l];
        const float* bias = w + (size_t)no * nin;
        R* out = outs[l & 1];
        for (int o = 0; o < no; ++o) {
            R s = bias[o];
            const float* row = w + (size_t)o * nin;
            for (int i = 0; i < nin; ++i) s += (R)row[i] * in[i];
            out[o] = P->act == 0 ? r_tanh(s) : (s > 0 ? s : r_expm1(s));
        }
        w = bias + no; in = out; nin = no;
    }
    const float* Wmu = w; const float* bmu = Wmu + (size_t)ACT * nin;
    const float* Wv = bmu + ACT; const float* bv = Wv + nin; const float* lsp = bv + 1;
    for (int o = 0; o < ACT; ++o) {
        R s = bmu[o];
        for (int i = 0; i < nin; ++i) s += (R)Wmu[(size_t)o * nin + i] * in[i];
        mu[o] = s;
    }
    R sv = bv[0];
    for (int i = 0; i < nin; ++i) sv += (R)Wv[i] * in[i];
    *val = sv;
    for (int o = 0; o < ACT; ++o) ls[o] = lsp[o];
}

static void normalize_obs(const R* o, const float* mean, const float* var, R* no) {
    for (int i = 0; i < OBS; ++i) {
        R z = (o[i] - (R)mean[i]) / r_sqrt((R)var[i] + (R)1e-8);
        if (z < -10) z = -10; else if (z > 10) z = 10;
        no[i] = z;
    }
}

/* =================================================================== exported C-ABI
 * (ctypes entry points used by the tests and the CPU baseline).  All buffers are host
 * pointers of type R (float in liboracle_f32.so, double in liboracle_f64.so) unless noted. */

void orc_fk(int n, const R* qpos, R* xpos, R* xquat, R* xipos) {
#pragma omp parallel for schedule(static)
    for (int w = 0; w < n; ++w)
        orc_fk_one(qpos + (size_t)w * NQ, xpos + (size_t)w * NB * 3, xquat + (size_t)w * NB * 4, xipos + (size_t)w * NB * 3);
}

/* per-state env_qacc (the reference's test_envqacc.cu harness semantics: FK then env_qacc).
 * bdt may be NULL (plain M).  Any output pointer may be NULL. */
void orc_qacc(int n, const R* qpos, const R* qvel, const R* tau, const R* bdt, int pgs, R mu,
              R* qacc, R* qacc_s, R* bias, R* f, int* ncon) {
#pragma omp parallel for schedule(dynamic, 16)
    for (int w = 0; w < n; ++w) {
        R xpos[NB * 3], xquat[NB * 4], xipos[NB * 3], q[NV];
        QaccAux X;
        const R* qp = qpos + (size_t)w * NQ;
        orc_fk_one(qp, xpos, xquat, xipos);
        orc_qacc_one(qp, qvel + (size_t)w * NV, xpos, xquat, xipos, tau + (size_t)w * NV, bdt ? bdt + (size_t)w * NV : NULL,
                     pgs, mu, q, &X);
        if (qacc) memcpy(qacc + (size_t)w * NV, q, sizeof(R) * NV);
        if (qacc_s) memcpy(qacc_s + (size_t)w * NV, X.qacc_s, sizeof(R) * NV);
        if (bias) memcpy(bias + (size_t)w * NV, X.bias, sizeof(R) * NV);
        if (f) memcpy(f + (size_t)w * MAXEFC, X.f, sizeof(R) * MAXEFC);
        if (ncon) ncon[w] = X.ncon;
    }
}

/* plain semi-implicit Euler trajectory with direct joint torques, no contact, no damping
 * (the MuJoCo-Euler golden regime of gen_reference.py:62-66).  Writes (nsteps+1) states. */
void orc_smooth_traj(const R* qpos0, const R* qvel0, const R* tau, int nsteps, R* qpos_out, R* qvel_out, R* qacc_out) {
    R lp[NQ], lv[NV], xpos[NB * 3], xquat[NB * 4], xipos[NB * 3];
    memcpy(lp, qpos0, sizeof lp); memcpy(lv, qvel0, sizeof lv);
    memcpy(qpos_out, lp, sizeof lp); memcpy(qvel_out, lv, sizeof lv);
    for (int t = 0; t < nsteps; ++t) {
        R S[NV * 6], bias[NV], rhs[NV], qacc[NV];
        Factor F;
        orc_fk_one(lp, xpos, xquat, xipos);
        orc_bias_one(lv, xpos, xquat, xipos, S, bias);
        orc_factor(xpos, xquat, xipos, S, NULL, &F);
        for (int i = 0; i < NV; ++i) rhs[i] = -bias[i] + (tau ? tau[i] : 0);
        orc_solve(&F, S, rhs, qacc);
        if (qacc_out) memcpy(qacc_out + (size_t)t * NV, qacc, sizeof qacc);
        for (int i = 0; i < NV; ++i) lv[i] += (R)G1M_DT * qacc[i];
        integrate_pos(lp, lv, (R)G1M_DT);
        memcpy(qpos_out + (size_t)(t + 1) * NQ, lp, sizeof lp);
        memcpy(qvel_out + (size_t)(t + 1) * NV, lv, sizeof lv);
    }
}

/* implicit-PD trajectory with given per-step joint targets, contacts evaluated as in the env
 * (test_implicit.cu:42-72 semantics, pgs iterations as given). */
void orc_pd_traj(const R* qpos0, const R* qvel0, const R* targets, int nsteps, int pgs, R mu, R* qpos_out, R* qvel_out) {
    R lp[NQ], lv[NV], xpos[NB * 3], xquat[NB * 4], xipos[NB * 3], bdt[NV], tau[NV], qacc[NV];
    QaccAux X;
    memcpy(lp, qpos0, sizeof lp); memcpy(lv, qvel0, sizeof lv);
    memcpy(qpos_out, lp, sizeof lp); memcpy(qvel_out, lv, sizeof lv);
    for (int i = 0; i < NV; ++i) bdt[i] = 0;
    for (int i = 0; i < ACT; ++i) bdt[G1M_ACT_DOF[i]] = (R)G1M_DT * (R)G1M_ACT_KD[i];
    for (int t = 0; t < nsteps; ++t) {
        const R* tg = targets + (size_t)t * ACT;
        orc_fk_one(lp, xpos, xquat, xipos);
        for (int i = 0; i < NV; ++i) tau[i] = 0;
        for (int i = 0; i < ACT; ++i) {
            int d = G1M_ACT_DOF[i];
            R pd = (R)G1M_ACT_KP[i] * (tg[i] - lp[G1M_ACT_QADR[i]]) - (R)G1M_ACT_KD[i] * lv[d];
            if (pd < (R)G1M_ACT_FRC_LO[i]) pd = G1M_ACT_FRC_LO[i];
            else if (pd > (R)G1M_ACT_FRC_HI[i]) pd = G1M_ACT_FRC_HI[i];
            tau[d] = pd;
        }
        orc_qacc_one(lp, lv, xpos, xquat, xipos, tau, bdt, pgs, mu, qacc, &X);
        for (int i = 0; i < NV; ++i) lv[i] += (R)G1M_DT * qacc[i];
        integrate_pos(lp, lv, (R)G1M_DT);
        memcpy(qpos_out + (size_t)(t + 1) * NQ, lp, sizeof lp);
        memcpy(qvel_out + (size_t)(t + 1) * NV, lv, sizeof lv);
    }
}

void orc_philox_block(const uint32_t* ctr, const uint32_t* key, uint32_t* out) { orc_philox(ctr, key, out); }

/* --- env handle mirroring the reference's EnvState (g1_env.cu:83-90) --- */
void* orc_env_create(int N, int S, int pgs, uint64_t seed, uint32_t world0, R mu) {
    OrcEnv* E = (OrcEnv*)calloc(1, sizeof(OrcEnv));
    E->N = N; E->S = S; E->pgs = pgs; E->seed = seed; E->world0 = world0; E->mu = mu; E->tick = 0;
    E->qp = (R*)calloc((size_t)N * NQ, sizeof(R));
    E->qv = (R*)calloc((size_t)N * NV, sizeof(R));
    E->pa = (R*)calloc((size_t)N * ACT, sizeof(R));
    E->steps = (int*)calloc((size_t)N, sizeof(int));
    return E;
}
void orc_env_destroy(void* h) {
    OrcEnv* E = (OrcEnv*)h;
    free(E->qp); free(E->qv); free(E->pa); free(E->steps); free(E);
}
/* state access (host arrays of R; steps int; tick uint64) */
void orc_env_set_state(void* h, const R* qp, const R* qv, const R* pa, const int* steps, uint64_t tick) {
    OrcEnv* E = (OrcEnv*)h;
    memcpy(E->qp, qp, sizeof(R) * (size_t)E->N * NQ);
    memcpy(E->qv, qv, sizeof(R) * (size_t)E->N * NV);
    memcpy(E->pa, pa, sizeof(R) * (size_t)E->N * ACT);
    memcpy(E->steps, steps, sizeof(int) * (size_t)E->N);
    E->tick = tick;
}
void orc_env_get_state(void* h, R* qp, R* qv, R* pa, int* steps, uint64_t* tick) {
    OrcEnv* E = (OrcEnv*)h;
    memcpy(qp, E->qp, sizeof(R) * (size_t)E->N * NQ);
    memcpy(qv, E->qv, sizeof(R) * (size_t)E->N * NV);
    memcpy(pa, E->pa, sizeof(R) * (size_t)E->N * ACT);
    memcpy(steps, E->steps, sizeof(int) * (size_t)E->N);
    *tick = E->tick;
}
/* stand pose + U(+-0.02) joint noise, zero velocity / previous action / step (k_reset,
 * g1_env.cu:97-111).  obs_out [N*OBS] may be NULL.  Does not advance the tick. */
void orc_env_reset(void* h, R* obs_out) {
    OrcEnv* E = (OrcEnv*)h;
#pragma omp parallel for schedule(static)
    for (int w = 0; w < E->N; ++w) {
        R* qp = E->qp + (size_t)w * NQ; R* qv = E->qv + (size_t)w * NV; R* pa = E->pa + (size_t)w * ACT;
        for (int i = 0; i < NQ; ++i) qp[i] = G1M_QPOS_STAND[i];
        for (int i = 0; i < ACT; ++i) {
            uint32_t o[4];
            rng_draw(E->seed, E->world0 + (uint32_t)w, E->tick, RNG_RESET, (uint32_t)i, o);
            qp[G1M_ACT_QADR[i]] += (R)0.02 * ((R)u01_open(o[0]) * 2 - 1);
        }
        for (int i = 0; i < NV; ++i) qv[i] = 0;
        for (int i = 0; i < ACT; ++i) pa[i] = 0;
        E->steps[w] = 0;
        if (obs_out) compute_obs(qp, qv, pa, obs_out + (size_t)w * OBS);
    }
}
/* host-loop control step with given actions (k_step, g1_env.cu:245-268).  Advances tick. */
void orc_env_step(void* h, const R* act, R* obs, R* rew, R* done) {
    OrcEnv* E = (OrcEnv*)h;
    uint64_t tick = E->tick;
#pragma omp parallel for schedule(dynamic, 4)
    for (int w = 0; w < E->N; ++w) {
        R* qp = E->qp + (size_t)w * NQ; R* qv = E->qv + (size_t)w * NV; R* pa = E->pa + (size_t)w * ACT;
        R r; int d;
        env_advance(E, w, tick, qp, qv, pa, &E->steps[w], act + (size_t)w * ACT, &r, &d);
        if (obs) compute_obs(qp, qv, pa, obs + (size_t)w * OBS);
        if (rew) rew[w] = r;
        if (done) done[w] = (R)d;
    }
    E->tick = tick + 1;
}
/* K control steps with zero action (k_phys_bench, g1_env.cu:343-359).  Advances tick by K.
 * Only worlds [0, nw) are stepped when nw > 0 (bounded CPU-baseline samples). */
void orc_env_bench_phys(void* h, int K, int nw) {
    OrcEnv* E = (OrcEnv*)h;
    int n = nw > 0 && nw < E->N ? nw : E->N;
    uint64_t tick = E->tick;
#pragma omp parallel for schedule(dynamic, 1)
    for (int w = 0; w < n; ++w) {
        R a[ACT];
        for (int i = 0; i < ACT; ++i) a[i] = 0;
        R* qp = E->qp + (size_t)w * NQ; R* qv = E->qv + (size_t)w * NV; R* pa = E->pa + (size_t)w * ACT;
        for (int k = 0; k < K; ++k) {
            R r; int d;
            env_advance(E, w, tick + (uint64_t)k, qp, qv, pa, &E->steps[w], a, &r, &d);
        }
    }
    E->tick = tick + (uint64_t)K;
}
/* Fused rollout (k_rollout, g1_env.cu:278-338).  W/mean/var are float arrays; trajectory
 * outputs O[H,N,OBS], A[H,N,ACT], LP/V/R/D[H,N], Vlast[N] are R arrays.  hidden/nh/act
 * describe the MLP (tanh=0, elu=1).  Worlds [0, nw) only when nw > 0.  Advances tick by H. */
void orc_rollout(void* h, int H, const float* W, const float* mean, const float* var, int nh, const int* hidden, int act,
                 R* O, R* A, R* LP, R* V, R* Rw, R* D, R* Vlast, int nw) {
    OrcEnv* E = (OrcEnv*)h;
    Policy P; P.nh = nh; P.act = act;
    for (int i = 0; i < nh; ++i) P.h[i] = hidden[i];
    int N = E->N, n = nw > 0 && nw < N ? nw : N;
    uint64_t tick0 = E->tick;
    const R LOG2PI = (R)1.8378770664093453;
#pragma omp parallel for schedule(dynamic, 1)
    for (int w = 0; w < n; ++w) {
        R* qp = E->qp + (size_t)w * NQ; R* qv = E->qv + (size_t)w * NV; R* pa = E->pa + (size_t)w * ACT;
        R o[OBS], no[OBS], mu[ACT], ls[ACT], val, a[ACT];
        for (int t = 0; t < H; ++t) {
            uint64_t tick = tick0 + (uint64_t)t;
            compute_obs(qp, qv, pa, o);
            normalize_obs(o, mean, var, no);
            size_t sb = (size_t)t * N + w;
            for (int i = 0; i < OBS; ++i) O[sb * OBS + i] = o[i];
            mlp_forward(&P, W, no, mu, ls, &val);
            R lps = 0;
            for (int i = 0; i < ACT; ++i) {
                uint32_t rb[4];
                rng_draw(E->seed, E->world0 + (uint32_t)w, tick, RNG_ACTION, (uint32_t)i, rb);
                R nz = normal_from(rb);
                a[i] = mu[i] + r_exp(ls[i]) * nz;
                lps += (R)-0.5 * nz * nz - ls[i] - (R)0.5 * LOG2PI;
            }
            for (int i = 0; i < ACT; ++i) A[sb * ACT + i] = a[i];
            LP[sb] = lps; V[sb] = val;
            R r; int d;
            env_advance(E, w, tick, qp, qv, pa, &E->steps[w], a, &r, &d);
            Rw[sb] = r; D[sb] = (R)d;
        }
        compute_obs(qp, qv, pa, o);
        normalize_obs(o, mean, var, no);
        mlp_forward(&P, W, no, mu, ls, &val);
        Vlast[w] = val;
    }
    E->tick = tick0 + (uint64_t)H;
}

int orc_real_size(void) { return (int)sizeof(R); }
