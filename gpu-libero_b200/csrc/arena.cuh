// Per-world shared-memory arena of the fused control-step kernel.
//
// A world (one or four warps of a CTA) owns its arena for a whole control
// step; every array the substep touches lives here, so HBM is read once
// (state in) and written once (state and outputs out) per control step.  The layout is computed identically on
// the host (to size the dynamic shared memory) and on the device.
#pragma once
#include <cstddef>
#include "b200phys.h"

namespace b200 {

// Per-contact record, in reals (solref / solimp are recomputed from the
// geom pair where rows are built).
enum ContactField { kCDist = 0, kCPos = 1, kCFrame = 4, kCMargin = 13, kCFriction = 14, kCWidth = 19 };

struct Carve {
  size_t at = 0;
  template <class T> __host__ __device__ size_t take(size_t count) {
    at = (at + 15) & ~size_t(15);
    size_t offset = at;
    at += count * sizeof(T);
    return offset;
  }
};

template <class R> struct Arena {
  // state
  R *qpos, *qvel, *warm, *ctrl, *goal_pos, *goal_rot, *gripper, *action;
  // position stage
  R *xpos, *xquat, *xmat, *xipos, *ximat, *anchor, *axis, *gxpos, *gxmat, *sxpos, *sxmat;
  R *com, *cinert, *crb, *cdof, *M, *L;
  // velocity stage
  R *cvel, *cacc, *cfrc, *cdof_dot, *act_length, *act_moment;
  // dof vectors
  R *qfrc_bias, *qfrc_passive, *qfrc_actuator, *qfrc_smooth, *qacc_smooth, *qacc, *Ma, *Mv;
  R *grad, *search, *qfrc_constraint, *ee_vel;
  // contacts and rows
  R *con;
  int *con_dim, *con_g1, *con_g2, *con_key, *con_order, *con_adr;
  // constraint rows: Jacobian values over at most two kinematic trees
  // (row_t[2r], row_t[2r+1]; -1 = none), kmax_dof values per row
  R *J, *efc_D, *efc_aref, *efc_floss, *efc_force, *efc_jaref, *efc_jv, *efc_quad;
  int *efc_type, *efc_id, *efc_state, *row_t;
  // islands: trees coupled by constraint rows; the Hessian is block diagonal
  // over islands, each block dense in island-local dof order
  int *tree_isl, *isl_n, *isl_off, *isl_dofstart, *isl_dof, *dof_isl, *dof_loc;
  // per-tree segment lists, rebuilt with the rows every substep: the
  // single-dof rows and the contacts (row ranges) acting on tree t are
  // tree_seg[tree_segadr[t] .. tree_segadr[t + 1]), in ascending row order;
  // entry = first row | rows << 16 | (column of the tree's first dof in the
  // row's Jacobian values) << 24
  int *tree_segadr;
  unsigned *tree_seg;
  R *xs, *colbuf;  // permuted solve vector; Cholesky column buffers (2 x nv) / per-warp 6 x 6 contact scratch
  // Newton Hessian, reused as OSC scratch (double) before the solve
  R *H;
  double *osc;
  // scalars and reduction scratch
  R *scal;   // [0] alpha [1] improvement [2] search_dot [3] grad_dot [4] decrement [5] time
  int *iscal;  // [0] ncon [1] nefc [2] nf [3] overflow [4] niter [5] done [6] error [7] ls evals
               // [8] raw contact count [9] ls evals at previous substep [10] profiling on
               // [11] islands [12] largest island [13] single-dof rows [14] refactor Newton H
               // [15] sum of row widths k_r [16..19] OSC factor flags [20..22] pinv flags
               // [23] sum of k_r^2 [24] factored block work (n^3 + 6 n^2)
               // [25] GJK / EPA pairs past the broadphase this substep
  R *red;    // reduction scratch: up to 9 values per warp of the world
  long long *prof;  // [0] last stamp, [1..15] per-stage cycle sums (stage profiling only)
  int ubytes;       // size of the stage-scoped union region (H, OSC and kinematics scratch)

  static constexpr int kOscDoubles = 400;
  // single-dof rows appear in one tree's list, contacts in at most two
  __host__ __device__ static int seg_capacity(const B200Model &m) { return m.nfric + m.nlimited + 2 * m.ncon_max; }
  // colbuf holds the Cholesky column buffers (2 x nv) or one 6 x 6 contact
  // coupling matrix per warp of a world (at most four warps)
  static constexpr int kColbufWarps = 4, kColbufMin = 160, kRed = 9 * kColbufWarps;
  static_assert(kColbufWarps * 36 <= kColbufMin, "colbuf holds a 6 x 6 matrix per warp");

  // Stage-scoped arrays share one region (U): kinematics -> CRB scratch
  // (xipos, ximat, joint anchors/axes, crb), the RNE scratch (cvel, cacc,
  // cfrc, cdof_dot), the FP64 OSC scratch, and finally the Newton/Euler
  // factorization blocks (H).  Each use ends before the next begins.
  __host__ __device__ static size_t layout(const B200Model &m, int threads, Arena *a, unsigned char *base) {
    Carve c;
    c.at = sizeof(Arena);  // the descriptor itself heads the world's region
    const int nq = m.nq, nv = m.nv, nu = m.nu, nb = m.nbody, nj = m.njnt, ng = m.ngeom, ns = m.nsite;
    const int nc = m.ncon_max, ne = m.nefc_max, nt = m.ntree;
    size_t o[96];
    int k = 0;
    o[k++] = c.take<R>(nq); o[k++] = c.take<R>(nv); o[k++] = c.take<R>(nv); o[k++] = c.take<R>(nu);
    o[k++] = c.take<R>(3); o[k++] = c.take<R>(9); o[k++] = c.take<R>(2); o[k++] = c.take<R>(7);
    o[k++] = c.take<R>(nb * 3); o[k++] = c.take<R>(nb * 4); o[k++] = c.take<R>(nb * 9);
    o[k++] = c.take<R>(ng * 3); o[k++] = c.take<R>(ng * 9); o[k++] = c.take<R>(ns * 3); o[k++] = c.take<R>(ns * 9);
    o[k++] = c.take<R>(nb * 3); o[k++] = c.take<R>(nb * 10); o[k++] = c.take<R>(nv * 6);
    o[k++] = c.take<R>(m.nM); o[k++] = c.take<R>(m.nL);  // M (dense tree blocks), L (packed)
    o[k++] = c.take<R>(nu); o[k++] = c.take<R>(nu);
    for (int i = 0; i < 11; ++i) o[k++] = c.take<R>(nv);
    o[k++] = c.take<R>(6);
    o[k++] = c.take<R>((size_t)nc * kCWidth);
    for (int i = 0; i < 6; ++i) o[k++] = c.take<int>(nc);
    o[k++] = c.take<R>((size_t)ne * m.kmax_dof);
    for (int i = 0; i < 6; ++i) o[k++] = c.take<R>(ne);
    o[k++] = c.take<R>((size_t)ne * 3);
    for (int i = 0; i < 3; ++i) o[k++] = c.take<int>(ne);
    o[k++] = c.take<int>(2 * ne);
    o[k++] = c.take<int>(nt); o[k++] = c.take<int>(nt); o[k++] = c.take<int>(nt);
    o[k++] = c.take<int>(nt + 1);
    o[k++] = c.take<int>(nv); o[k++] = c.take<int>(nv); o[k++] = c.take<int>(nv);
    o[k++] = c.take<int>(nt + 1); o[k++] = c.take<unsigned>(seg_capacity(m));
    o[k++] = c.take<R>(nv);
    o[k++] = c.take<R>(2 * nv > kColbufMin ? 2 * nv : kColbufMin);  // colbuf
    o[k++] = c.take<R>(8); o[k++] = c.take<int>(32); o[k++] = c.take<R>(kRed);
    o[k++] = c.take<long long>(16);
    // union region
    const size_t kin = (size_t)(nb * 3 + nb * 9 + nj * 3 + nj * 3 + nb * 10) * sizeof(R) + 5 * 16;
    const size_t rne = (size_t)(nb * 6 * 3 + nv * 6) * sizeof(R) + 4 * 16;
    const size_t osc = (size_t)kOscDoubles * sizeof(double);
    const size_t hes = (size_t)nv * (nv + 1) / 2 * sizeof(R);  // packed island blocks, one island at worst
    size_t ubytes = kin > rne ? kin : rne;
    ubytes = ubytes > osc ? ubytes : osc;
    ubytes = ubytes > hes ? ubytes : hes;
    const size_t u = c.take<unsigned char>(ubytes);
    size_t total = (c.at + 15) & ~size_t(15);
    if (a) {
      int i = 0;
#define B200_P(field, T) a->field = (T *)(base + o[i++])
      B200_P(qpos, R); B200_P(qvel, R); B200_P(warm, R); B200_P(ctrl, R);
      B200_P(goal_pos, R); B200_P(goal_rot, R); B200_P(gripper, R); B200_P(action, R);
      B200_P(xpos, R); B200_P(xquat, R); B200_P(xmat, R);
      B200_P(gxpos, R); B200_P(gxmat, R); B200_P(sxpos, R); B200_P(sxmat, R);
      B200_P(com, R); B200_P(cinert, R); B200_P(cdof, R); B200_P(M, R); B200_P(L, R);
      B200_P(act_length, R); B200_P(act_moment, R);
      B200_P(qfrc_bias, R); B200_P(qfrc_passive, R); B200_P(qfrc_actuator, R); B200_P(qfrc_smooth, R);
      B200_P(qacc_smooth, R); B200_P(qacc, R); B200_P(Ma, R); B200_P(Mv, R); B200_P(grad, R); B200_P(search, R);
      B200_P(qfrc_constraint, R);
      B200_P(ee_vel, R);
      B200_P(con, R);
      B200_P(con_dim, int); B200_P(con_g1, int); B200_P(con_g2, int); B200_P(con_key, int); B200_P(con_order, int);
      B200_P(con_adr, int);
      B200_P(J, R); B200_P(efc_D, R); B200_P(efc_aref, R); B200_P(efc_floss, R); B200_P(efc_force, R);
      B200_P(efc_jaref, R); B200_P(efc_jv, R); B200_P(efc_quad, R);
      B200_P(efc_type, int); B200_P(efc_id, int); B200_P(efc_state, int); B200_P(row_t, int);
      B200_P(tree_isl, int); B200_P(isl_n, int); B200_P(isl_off, int); B200_P(isl_dofstart, int);
      B200_P(isl_dof, int); B200_P(dof_isl, int); B200_P(dof_loc, int);
      B200_P(tree_segadr, int); B200_P(tree_seg, unsigned);
      B200_P(xs, R); B200_P(colbuf, R);
      B200_P(scal, R); B200_P(iscal, int); B200_P(red, R); B200_P(prof, long long);
#undef B200_P
      unsigned char *ub = base + u;
      Carve kc;
      a->xipos = (R *)(ub + kc.take<R>(nb * 3));
      a->ximat = (R *)(ub + kc.take<R>(nb * 9));
      a->anchor = (R *)(ub + kc.take<R>(nj * 3));
      a->axis = (R *)(ub + kc.take<R>(nj * 3));
      a->crb = (R *)(ub + kc.take<R>(nb * 10));
      Carve vc;
      a->cvel = (R *)(ub + vc.take<R>(nb * 6));
      a->cacc = (R *)(ub + vc.take<R>(nb * 6));
      a->cfrc = (R *)(ub + vc.take<R>(nb * 6));
      a->cdof_dot = (R *)(ub + vc.take<R>(nv * 6));
      a->osc = (double *)ub;
      a->H = (R *)ub;
      a->ubytes = (int)ubytes;
    }
    return total;
  }
};

}  // namespace b200
