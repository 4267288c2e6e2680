// g1_tables.cuh -- the G1 model as the kernels see it: a flat POD struct built once on the
// host from the exported model tables (g1_model_data.h), uploaded to __constant__ memory,
// and copied by every CTA into its shared memory so lane-divergent lookups (lane = body,
// lane = dof) hit shared-memory banks instead of serialising on the constant cache.
//
// Derived tables replace the reference's run-time tree walks:
//   * level order of the kinematic tree (FK and RNE forward, root->leaf; the factor and the
//     RNE force pass walk it backwards).  The reference iterates bodies in index order
//     (dynamics.cuh:53, aba_factor.cuh:77); bodies at one tree depth are independent, so a
//     warp processes a whole level at once, one lane per body.
//   * children lists in DESCENDING index order, so a parent "pulls" its children's
//     contributions in the same order the reference "pushes" them while b descends
//     (aba_factor.cuh:86-87, aba_bias.cuh:473-474, aba_factor.cuh:135).
//   * per foot sphere, the ancestor dof list in the reference's walk order
//     (env_qacc.cuh:89-96).
#pragma once
#include <stdint.h>
#include "g1_model_data.h"

#define G1_NB G1M_NBODY
#define G1_NQ_ G1M_NQ
#define G1_NV_ G1M_NV
#define G1_NJ G1M_NJNT
#define G1_NU_ G1M_NU
#define G1_NFOOT_ G1M_NFOOT
#define G1_MAXCON G1M_NFOOT
#define G1_MAXEFC (4 * G1M_NFOOT)
#define G1_CDS 12
#define G1_OBS 100
#define G1_ACT 29
#define G1_NRHS (1 + 3 * G1_MAXCON)
#define G1_MAXCHAIN 6
#define G1_MAXBRANCH 2
#define G1_MAXCLEN 12  // bodies per chain (the G1's longest chain, waist + left arm, has 10)
#define G1_MAXXSLOT 4

// cstep's packed field: joint (bits 0-7), branch slot + 1 (8-11), kept-frame slot + 1
// (12-15), parent body (16-23)
__host__ __device__ constexpr int cstep_pack(int jnt, int bslot, int xslot, int parent) {
    return jnt | ((bslot + 1) << 8) | ((xslot + 1) << 12) | (parent << 16);
}
__host__ __device__ __forceinline__ int cstep_jnt(int y) { return y & 0xFF; }
__host__ __device__ __forceinline__ int cstep_bslot(int y) { return ((y >> 8) & 0xF) - 1; }
__host__ __device__ __forceinline__ int cstep_xslot(int y) { return ((y >> 12) & 0xF) - 1; }
__host__ __device__ __forceinline__ int cstep_parent(int y) { return (y >> 16) & 0xFF; }
static_assert(G1_NJ <= 256 && G1_MAXBRANCH < 15 && G1_MAXXSLOT < 15 && G1_NB <= 256, "cstep packing");

struct alignas(16) G1Tables {
    float body_pos[G1_NB * 3], body_quat[G1_NB * 4], body_ipos[G1_NB * 3], body_iquat[G1_NB * 4];
    float body_mass[G1_NB], body_inertia[G1_NB * 3];
    float jnt_axis[G1_NJ * 3], jnt_pos[G1_NJ * 3];
    float armature[G1_NV_ + 1];
    float qpos_stand[G1_NQ_];
    float foot_lpos[G1_NFOOT_ * 3], foot_invw0[G1_NFOOT_];
    float kp[G1_NU_], kd[G1_NU_], ctrl_lo[G1_NU_], ctrl_hi[G1_NU_], frc_lo[G1_NU_], frc_hi[G1_NU_];
    float target0[G1_NU_];  // stand pose at the actuated joints
    float bdt[G1_NV_ + 1];  // dt * kd on actuated dofs (g1_env.cu:137-139)
    float solimp[5], solref[2], gravity[3];
    int parent[G1_NB], dofadr[G1_NB], dofnum[G1_NB], body_jnt[G1_NB];
    int jnt_type[G1_NJ], jnt_qposadr[G1_NJ], jnt_dofadr[G1_NJ], jnt_body[G1_NJ];
    int dof_jnt[G1_NV_ + 1];
    int act_dof[G1_NU_], act_qadr[G1_NU_];
    int foot_body[G1_NFOOT_];
    int nlev;
    int lev_start[G1_NB + 1];
    int lev_body[G1_NB];
    int child_start[G1_NB + 1];
    int child_list[G1_NB];
    int foot_ndof[G1_NFOOT_];
    unsigned char foot_dofs[G1_NFOOT_][G1_CDS];
    int foot_chains[G1_NFOOT_];  // bit c: chain c holds an ancestor of the sphere's body
    int free_jnt;                // the floating base's free joint (the only non-hinge joint)
    int4 binfo[G1_NB];           // per body {dofadr, branch_slot, parent, 0}: one 16-byte load
    // chain decomposition of the hinge bodies (root->leaf order inside a chain); lane l of
    // a warp walks chain l.  A chain starts at a child of the floating base or of a branch
    // body; f1_start is the sweep step of its head (its parent is done by then).
    int nchain, nsteps, nsteps_back;
    int chain_len[G1_MAXCHAIN], chain_start[G1_MAXCHAIN];
    int chain_bstart[G1_MAXCHAIN];  // leaf->root sweep: step at which the chain's leaf is processed
    int chain_body[G1_MAXCHAIN][G1_NB];
    // step k of chain c as one 16-byte load: {body, packed (joint, branch slot, kept-frame
    // slot, parent) -- cstep_pack --, the joint's qpos address, the body's dof}: a sweep step
    // needs no dependent index loads after it
    int4 cstep[G1_MAXCHAIN][G1_MAXCLEN];
    int branch_slot[G1_NB];  // bodies other than the base with >1 child: hand-off slot, else -1
    int head_chain[G1_NB];   // chain whose head is this body, else -1
    int xslot[G1_NB];        // pelvis and foot bodies: slot of their kept frame, else -1
    int nxslot;
};

#ifndef __CUDACC_RTC__
#include <string.h>
// Host: fill the tables from the exported model (and the derived orders above).
static inline void g1_build_tables(G1Tables* T) {
    memset(T, 0, sizeof(*T));
    memcpy(T->body_pos, G1M_BODY_POS, sizeof(T->body_pos));
    memcpy(T->body_quat, G1M_BODY_QUAT, sizeof(T->body_quat));
    memcpy(T->body_ipos, G1M_BODY_IPOS, sizeof(T->body_ipos));
    memcpy(T->body_iquat, G1M_BODY_IQUAT, sizeof(T->body_iquat));
    memcpy(T->body_mass, G1M_BODY_MASS, sizeof(T->body_mass));
    memcpy(T->body_inertia, G1M_BODY_INERTIA, sizeof(T->body_inertia));
    memcpy(T->jnt_axis, G1M_JNT_AXIS, sizeof(T->jnt_axis));
    memcpy(T->jnt_pos, G1M_JNT_POS, sizeof(T->jnt_pos));
    memcpy(T->armature, G1M_DOF_ARMATURE, sizeof(G1M_DOF_ARMATURE));
    memcpy(T->qpos_stand, G1M_QPOS_STAND, sizeof(T->qpos_stand));
    memcpy(T->foot_lpos, G1M_FOOT_LPOS, sizeof(T->foot_lpos));
    memcpy(T->foot_invw0, G1M_FOOT_INVWEIGHT0, sizeof(T->foot_invw0));
    memcpy(T->kp, G1M_ACT_KP, sizeof(T->kp));
    memcpy(T->kd, G1M_ACT_KD, sizeof(T->kd));
    memcpy(T->ctrl_lo, G1M_ACT_CTRL_LO, sizeof(T->ctrl_lo));
    memcpy(T->ctrl_hi, G1M_ACT_CTRL_HI, sizeof(T->ctrl_hi));
    memcpy(T->frc_lo, G1M_ACT_FRC_LO, sizeof(T->frc_lo));
    memcpy(T->frc_hi, G1M_ACT_FRC_HI, sizeof(T->frc_hi));
    memcpy(T->solimp, G1M_FOOT_SOLIMP, sizeof(T->solimp));
    memcpy(T->solref, G1M_FOOT_SOLREF, sizeof(T->solref));
    memcpy(T->gravity, G1M_GRAVITY, sizeof(T->gravity));
    memcpy(T->parent, G1M_BODY_PARENT, sizeof(T->parent));
    memcpy(T->dofadr, G1M_BODY_DOFADR, sizeof(T->dofadr));
    memcpy(T->dofnum, G1M_BODY_DOFNUM, sizeof(T->dofnum));
    memcpy(T->jnt_type, G1M_JNT_TYPE, sizeof(T->jnt_type));
    memcpy(T->jnt_qposadr, G1M_JNT_QPOSADR, sizeof(T->jnt_qposadr));
    memcpy(T->jnt_dofadr, G1M_JNT_DOFADR, sizeof(T->jnt_dofadr));
    memcpy(T->jnt_body, G1M_JNT_BODY, sizeof(T->jnt_body));
    memcpy(T->act_dof, G1M_ACT_DOF, sizeof(T->act_dof));
    memcpy(T->act_qadr, G1M_ACT_QADR, sizeof(T->act_qadr));
    memcpy(T->foot_body, G1M_FOOT_BODY, sizeof(T->foot_body));
    for (int b = 0; b < G1_NB; ++b) T->body_jnt[b] = G1M_BODY_JNTNUM[b] > 0 ? G1M_BODY_JNTADR[b] : -1;
    for (int j = 0; j < G1_NJ; ++j) {
        int n = G1M_JNT_TYPE[j] == 0 ? 6 : 1;
        for (int k = 0; k < n; ++k) T->dof_jnt[G1M_JNT_DOFADR[j] + k] = j;
    }
    for (int i = 0; i < G1_NU_; ++i) {
        T->target0[i] = G1M_QPOS_STAND[G1M_ACT_QADR[i]];
        T->bdt[G1M_ACT_DOF[i]] = G1M_DT * G1M_ACT_KD[i];
    }
    // level order: depth of body b (body 1 at depth 0)
    int depth[G1_NB];
    depth[0] = -1;
    int maxd = 0;
    for (int b = 1; b < G1_NB; ++b) {
        depth[b] = depth[G1M_BODY_PARENT[b]] + 1;
        if (depth[b] > maxd) maxd = depth[b];
    }
    int n = 0;
    T->nlev = maxd + 1;
    for (int l = 0; l <= maxd; ++l) {
        T->lev_start[l] = n;
        for (int b = 1; b < G1_NB; ++b)
            if (depth[b] == l) T->lev_body[n++] = b;
    }
    T->lev_start[maxd + 1] = n;
    // children in descending index order
    n = 0;
    for (int p = 0; p < G1_NB; ++p) {
        T->child_start[p] = n;
        for (int b = G1_NB - 1; b >= 1; --b)
            if (G1M_BODY_PARENT[b] == p && b != p) T->child_list[n++] = b;
    }
    T->child_start[G1_NB] = n;
    // chains: follow the child with the deepest subtree (lowest index on ties); every
    // other child of a body heads a new chain.  Heads of chains are children of the base
    // (body 1) or of branch bodies.
    {
        int height[G1_NB];
        for (int b = G1_NB - 1; b >= 1; --b) {
            height[b] = 0;
            for (int c = b + 1; c < G1_NB; ++c)
                if (G1M_BODY_PARENT[c] == b && height[c] + 1 > height[b]) height[b] = height[c] + 1;
        }
        int pos_step[G1_NB];  // sweep step at which a body is processed
        for (int b = 0; b < G1_NB; ++b) { pos_step[b] = -1; T->branch_slot[b] = -1; T->head_chain[b] = -1; }
        int nch = 0, nslot = 0;
        // heads in ascending index order, processed in order (a head's parent precedes it)
        for (int h = 2; h < G1_NB; ++h) {
            int p = G1M_BODY_PARENT[h];
            bool is_head = (p == 1);
            if (!is_head) {  // head if not the chosen continuation of its parent
                int best = -1;
                for (int c = p + 1; c < G1_NB; ++c)
                    if (G1M_BODY_PARENT[c] == p && (best < 0 || height[c] > height[best])) best = c;
                is_head = (best != h);
            }
            if (!is_head || nch >= G1_MAXCHAIN) continue;
            int start = (p == 1) ? 0 : pos_step[p] + 1;
            int len = 0;
            for (int b = h; b >= 0;) {
                T->chain_body[nch][len] = b;
                pos_step[b] = start + len;
                ++len;
                int best = -1;
                for (int c = b + 1; c < G1_NB; ++c)
                    if (G1M_BODY_PARENT[c] == b && (best < 0 || height[c] > height[best])) best = c;
                b = best;
            }
            T->chain_len[nch] = len;
            T->head_chain[h] = nch;
            T->chain_start[nch] = start;
            ++nch;
        }
        T->nchain = nch;
        int ns = 0;
        for (int c = 0; c < nch; ++c)
            if (T->chain_start[c] + T->chain_len[c] > ns) ns = T->chain_start[c] + T->chain_len[c];
        T->nsteps = ns;
        // leaf->root: a chain walks its bodies leaf first; a branch body must come after the
        // last (head) body of every other chain hanging off it
        int chain_of[G1_NB], pos_in[G1_NB];
        for (int b = 0; b < G1_NB; ++b) chain_of[b] = -1;
        for (int c = 0; c < nch; ++c)
            for (int k = 0; k < T->chain_len[c]; ++k) { chain_of[T->chain_body[c][k]] = c; pos_in[T->chain_body[c][k]] = k; }
        for (int c = nch - 1; c >= 0; --c) {
            int bs = 0;
            for (int k = 0; k < T->chain_len[c]; ++k) {
                int b = T->chain_body[c][k];
                for (int c2 = c + 1; c2 < nch; ++c2) {
                    int h = T->chain_body[c2][0];
                    if (G1M_BODY_PARENT[h] != b) continue;
                    int done = T->chain_bstart[c2] + T->chain_len[c2];           // first free step
                    int at = T->chain_len[c] - 1 - k;                              // b's offset
                    if (done - at > bs) bs = done - at;
                }
            }
            T->chain_bstart[c] = bs;
        }
        int nb2 = 0;
        for (int c = 0; c < nch; ++c)
            if (T->chain_bstart[c] + T->chain_len[c] > nb2) nb2 = T->chain_bstart[c] + T->chain_len[c];
        T->nsteps_back = nb2;
        (void)chain_of; (void)pos_in;
        for (int b = 2; b < G1_NB; ++b) {
            int nc = 0;
            for (int c = b + 1; c < G1_NB; ++c) nc += G1M_BODY_PARENT[c] == b;
            if (nc > 1 && nslot < G1_MAXBRANCH) T->branch_slot[b] = nslot++;
        }
    }
    for (int b = 0; b < G1_NB; ++b) T->xslot[b] = -1;
    T->xslot[1] = 0;
    T->nxslot = 1;
    for (int s = 0; s < G1_NFOOT_; ++s)
        if (T->xslot[G1M_FOOT_BODY[s]] < 0) T->xslot[G1M_FOOT_BODY[s]] = T->nxslot++;
    for (int s = 0; s < G1_NFOOT_; ++s) {
        int k = 0;
        for (int b = G1M_FOOT_BODY[s]; b >= 1; b = G1M_BODY_PARENT[b])
            for (int a = G1M_BODY_DOFADR[b]; a < G1M_BODY_DOFADR[b] + G1M_BODY_DOFNUM[b]; ++a)
                if (k < G1_CDS) T->foot_dofs[s][k++] = (unsigned char)a;
        T->foot_ndof[s] = k;
        int mask = 0;
        for (int b = G1M_FOOT_BODY[s]; b >= 2; b = G1M_BODY_PARENT[b])
            for (int c = 0; c < T->nchain; ++c)
                for (int q = 0; q < T->chain_len[c]; ++q)
                    if (T->chain_body[c][q] == b) mask |= 1 << c;
        T->foot_chains[s] = mask;
    }
    for (int b = 0; b < G1_NB; ++b) T->binfo[b] = make_int4(T->dofadr[b], T->branch_slot[b], T->parent[b], 0);
    for (int c = 0; c < T->nchain; ++c)
        for (int k = 0; k < T->chain_len[c] && k < G1_MAXCLEN; ++k) {
            const int bb = T->chain_body[c][k], j = T->body_jnt[bb];
            T->cstep[c][k] = make_int4(bb, cstep_pack(j, T->branch_slot[bb], T->xslot[bb], T->parent[bb]),
                                       T->jnt_qposadr[j], T->dofadr[bb]);
        }
    T->free_jnt = 0;
    for (int j = G1_NJ - 1; j >= 0; --j)
        if (G1M_JNT_TYPE[j] == 0) T->free_jnt = j;
}
#endif
