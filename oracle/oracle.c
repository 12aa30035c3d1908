/* Portions restate MuJoCo Warp formulas: Copyright 2025 The Newton Developers,
 * SPDX-License-Identifier: Apache-2.0 (see NOTICE). */
/*
 * CPU ORACLE — test infrastructure only.
 *
 * Serial C restatement of the reference's FP32 physics substep (MJWarp
 * semantics at commit c384ac51, as ported by GPU-LIBERO's cuda_fp32 engine),
 * one world at a time, in the order of the reference's captured substep
 * (libero/libero/gpu/host/backends/cuda_fp32/runtime.py:40-56,
 * physics.py:161-210).  It is the checker for the CUDA kernels: only tests/,
 * __graft_entry__.smoke() and bench.py's CPU-baseline leg may load it.  It
 * is never part of the product path.
 *
 * Compiled twice: -DREAL=float (mirrors the FP32 engine) and -DREAL=double
 * (the FP64 configuration).  The OSC controller always computes in double,
 * as the reference promotes it (cuda/control/osc_solver.cu, compute_t).
 *
 * Parity pinning: the leaves are checked against the reference's own NumPy
 * oracles (tools/validation/mjwarp_*_reference.py) through fixtures in
 * tests/golden/, and against the reference's geometric fixtures
 * (tests/fixtures/boxbox_*.json, tests/data/gjk_tuned_direction.json).
 */
#include <math.h>
#include <stdlib.h>
#include <string.h>
#include <float.h>
#include "../include/b200phys.h"

#ifndef REAL
#define REAL float
#endif
typedef REAL real;
#define IS_F32 (sizeof(real) == 4)
#define R(x) ((real)(x))

#define MF(name) ((const real *)m->real + m->off_##name)
#define MI(name) (m->ints + m->off_##name)

#define MAXB 64
#define MAXV 128
#define MAXG 64
#define MAXC 256
#define MAXE 1024

static real rmax(real a, real b) { return a > b ? a : b; }
static real rmin(real a, real b) { return a < b ? a : b; }
static real rabs(real a) { return a < 0 ? -a : a; }
static real rsqrt_(real a) { return IS_F32 ? (real)sqrtf((float)a) : (real)sqrt((double)a); }
static real rclamp(real x, real lo, real hi) { return rmax(lo, rmin(hi, x)); }
static real safe_div(real x, real y) { return x / (y != 0 ? y : R(1e-15)); }

/* ------------------------------------------------------------ vector math */
typedef struct { real v[3]; } V3;
typedef struct { real w, x, y, z; } Q4;
static V3 v3(real x, real y, real z) { V3 r = {{x, y, z}}; return r; }
static V3 vload(const real *p) { return v3(p[0], p[1], p[2]); }
static void vstore(real *p, V3 a) { p[0] = a.v[0]; p[1] = a.v[1]; p[2] = a.v[2]; }
static V3 vadd(V3 a, V3 b) { return v3(a.v[0] + b.v[0], a.v[1] + b.v[1], a.v[2] + b.v[2]); }
static V3 vsub(V3 a, V3 b) { return v3(a.v[0] - b.v[0], a.v[1] - b.v[1], a.v[2] - b.v[2]); }
static V3 vscale(V3 a, real s) { return v3(a.v[0] * s, a.v[1] * s, a.v[2] * s); }
static V3 vneg(V3 a) { return v3(-a.v[0], -a.v[1], -a.v[2]); }
static real vdot(V3 a, V3 b) { return a.v[0] * b.v[0] + a.v[1] * b.v[1] + a.v[2] * b.v[2]; }
static V3 vcross(V3 a, V3 b) {
  return v3(a.v[1] * b.v[2] - a.v[2] * b.v[1], a.v[2] * b.v[0] - a.v[0] * b.v[2],
            a.v[0] * b.v[1] - a.v[1] * b.v[0]);
}
static V3 vnormalize(V3 a) { real n = rsqrt_(vdot(a, a)); return n > 0 ? vscale(a, R(1) / n) : v3(0, 0, 0); }
/* R * x for row-major 3x3 */
static V3 mrot(const real *r, V3 x) {
  return v3(r[0] * x.v[0] + r[1] * x.v[1] + r[2] * x.v[2], r[3] * x.v[0] + r[4] * x.v[1] + r[5] * x.v[2],
            r[6] * x.v[0] + r[7] * x.v[1] + r[8] * x.v[2]);
}
/* R^T * x */
static V3 mrotT(const real *r, V3 x) {
  return v3(r[0] * x.v[0] + r[3] * x.v[1] + r[6] * x.v[2], r[1] * x.v[0] + r[4] * x.v[1] + r[7] * x.v[2],
            r[2] * x.v[0] + r[5] * x.v[1] + r[8] * x.v[2]);
}
static V3 mcol(const real *r, int k) { return v3(r[k], r[3 + k], r[6 + k]); }

static Q4 qload(const real *p) { Q4 q = {p[0], p[1], p[2], p[3]}; return q; }
static void qstore(real *p, Q4 q) { p[0] = q.w; p[1] = q.x; p[2] = q.y; p[3] = q.z; }
static Q4 qnormalize(Q4 q) {
  real n = rsqrt_(q.w * q.w + q.x * q.x + q.y * q.y + q.z * q.z);
  if (n > 0) { real r = R(1) / n; Q4 o = {q.w * r, q.x * r, q.y * r, q.z * r}; return o; }
  { Q4 o = {0, 0, 0, 1}; return o; } /* Warp storage fallback (mjwarp_kinematics.cu:58-61) */
}
static Q4 qmul(Q4 a, Q4 b) {
  Q4 o = {a.w * b.w - a.x * b.x - a.y * b.y - a.z * b.z, a.w * b.x + a.x * b.w + a.y * b.z - a.z * b.y,
          a.w * b.y - a.x * b.z + a.y * b.w + a.z * b.x, a.w * b.z + a.x * b.y - a.y * b.x + a.z * b.w};
  return o;
}
/* mjwarp_kinematics.cu:69-73 rotate(v,q) */
static V3 qrot(V3 v, Q4 q) {
  V3 u = v3(q.x, q.y, q.z);
  V3 r = vadd(vscale(u, R(2) * vdot(u, v)), vscale(v, q.w * q.w - vdot(u, u)));
  return vadd(r, vscale(vcross(u, v), R(2) * q.w));
}
static Q4 axis_angle(V3 a, real angle) {
  real s, c;
  if (IS_F32) { s = (real)sinf((float)(angle * R(0.5))); c = (real)cosf((float)(angle * R(0.5))); }
  else { s = (real)sin((double)(angle * R(0.5))); c = (real)cos((double)(angle * R(0.5))); }
  Q4 q = {c, a.v[0] * s, a.v[1] * s, a.v[2] * s};
  return q;
}
static void qmat(real *p, Q4 q) { /* mjwarp_kinematics.cu:79-92 */
  real a = q.w * q.w, b = q.w * q.x, c = q.w * q.y, d = q.w * q.z;
  real e = q.x * q.x, f = q.x * q.y, h = q.x * q.z, j = q.y * q.y, k = q.y * q.z, l = q.z * q.z;
  p[0] = a + e - j - l; p[1] = R(2) * (f - d); p[2] = R(2) * (h + c);
  p[3] = R(2) * (f + d); p[4] = a - e + j - l; p[5] = R(2) * (k - b);
  p[6] = R(2) * (h - c); p[7] = R(2) * (k + b); p[8] = a - e - j + l;
}

/* ------------------------------------------------------------ per-world work */
typedef struct {
  int dim, g1, g2;
  real dist, pos[3], frame[9], margin, friction[5], solref[2], solreffriction[2], solimp[5];
} Contact;

typedef struct {
  /* position stage */
  real xpos[MAXB][3], xquat[MAXB][4], xmat[MAXB][9], xipos[MAXB][3], ximat[MAXB][9];
  real anchor[MAXB][3], axis[MAXB][3]; /* per joint */
  real gxpos[MAXG][3], gxmat[MAXG][9], sxpos[8][3], sxmat[8][9];
  real com[MAXB][3], cinert[MAXB][10], crb[MAXB][10], cdof[MAXV][6];
  real M[MAXV * MAXV];  /* dense per-tree blocks at tree_madr */
  real L[MAXV * MAXV];  /* upper Cholesky factors, same layout */
  /* velocity stage */
  real cvel[MAXB][6], cdof_dot[MAXV][6], qfrc_bias[MAXV], qfrc_passive[MAXV];
  real act_length[16], act_moment[16], act_force[16], qfrc_actuator[MAXV];
  real qfrc_smooth[MAXV], qacc_smooth[MAXV];
  /* collision / constraints: rows [0, ne) are equality rows (none in the
   * scenes; the Newton-piece leaves use them), [ne, ne + nf) friction loss */
  int ncon, nefc, ne, nf, overflow;
  Contact con[MAXC];
  int con_adr[MAXC];
  real J[MAXE][MAXV];
  real efc_D[MAXE], efc_aref[MAXE], efc_frictionloss[MAXE], efc_force[MAXE], efc_jaref[MAXE], efc_jv[MAXE];
  real quad[MAXE][3];
  int efc_type[MAXE], efc_id[MAXE], efc_state[MAXE];
  /* Newton */
  real qacc[MAXV], Ma[MAXV], Mv[MAXV], grad[MAXV], search[MAXV], qfrc_constraint[MAXV];
  real H[MAXV * MAXV];
  real grad_dot, search_dot, decrement, improvement, alpha;
  int niter, done, ls_evals;
  real U[MAXV * MAXV], Md[MAXV * MAXV], Ld[MAXV * MAXV];
} Work;

static int tree_of(const B200Model *m, int dof) { return MI(dof_treeid)[dof]; }

/* M[i][j] for dofs i, j (0 across trees) */
static real mass_at(const B200Model *m, const real *M, int i, int j) {
  int t = tree_of(m, i);
  if (t != tree_of(m, j)) return 0;
  int a = MI(tree_dofadr)[t], n = MI(tree_dofnum)[t];
  return M[MI(tree_madr)[t] + (i - a) * n + (j - a)];
}

/* ============================================================ kinematics
 * mjwarp_kinematics.cu:95-212 (body_poses .. site_frames) */
static void kinematics(const B200Model *m, Work *k, const real *qpos) {
  int nb = m->nbody;
  const int *parent = MI(body_parentid), *jadr = MI(body_jntadr), *jnum = MI(body_jntnum);
  const int *jtype = MI(jnt_type), *qadr = MI(jnt_qposadr);
  k->xpos[0][0] = k->xpos[0][1] = k->xpos[0][2] = 0;
  k->xquat[0][0] = 1; k->xquat[0][1] = k->xquat[0][2] = k->xquat[0][3] = 0;
  for (int b = 1; b < nb; ++b) {
    int first = jadr[b], count = jnum[b], p = parent[b];
    V3 pos; Q4 quat;
    if (count == 1 && jtype[first] == B200_JNT_FREE) {
      const real *q = qpos + qadr[first];
      pos = v3(q[0], q[1], q[2]);
      Q4 raw = {q[3], q[4], q[5], q[6]};
      quat = qnormalize(raw);
      vstore(k->anchor[first], pos);
      vstore(k->axis[first], vload(MF(jnt_axis) + 3 * first));
    } else {
      V3 pp = vload(k->xpos[p]);
      Q4 pq = qload(k->xquat[p]);
      pos = vadd(qrot(vload(MF(body_pos) + 3 * b), pq), pp);
      quat = qmul(pq, qload(MF(body_quat) + 4 * b));
      for (int j = first; j < first + count; ++j) {
        int kind = jtype[j], q = qadr[j];
        V3 lpos = vload(MF(jnt_pos) + 3 * j), lax = vload(MF(jnt_axis) + 3 * j);
        V3 anchor = vadd(qrot(lpos, quat), pos), axis = qrot(lax, quat);
        if (kind == B200_JNT_BALL) {
          Q4 raw = {qpos[q], qpos[q + 1], qpos[q + 2], qpos[q + 3]};
          quat = qmul(quat, qnormalize(raw));
          pos = vsub(anchor, qrot(lpos, quat));
        } else if (kind == B200_JNT_SLIDE) {
          pos = vadd(pos, vscale(axis, qpos[q] - MF(qpos0)[q]));
        } else if (kind == B200_JNT_HINGE) {
          quat = qmul(quat, axis_angle(lax, qpos[q] - MF(qpos0)[q]));
          pos = vsub(anchor, qrot(lpos, quat));
        }
        vstore(k->anchor[j], anchor);
        vstore(k->axis[j], axis);
      }
      quat = qnormalize(quat);
    }
    vstore(k->xpos[b], pos);
    qstore(k->xquat[b], quat);
  }
  for (int b = 0; b < nb; ++b) {
    Q4 q = qload(k->xquat[b]);
    qmat(k->xmat[b], q);
    vstore(k->xipos[b], vadd(vload(k->xpos[b]), qrot(vload(MF(body_ipos) + 3 * b), q)));
    qmat(k->ximat[b], qmul(q, qload(MF(body_iquat) + 4 * b)));
  }
  for (int g = 0; g < m->ngeom; ++g) {
    int b = MI(geom_bodyid)[g];
    Q4 q = qload(k->xquat[b]);
    vstore(k->gxpos[g], vadd(vload(k->xpos[b]), qrot(vload(MF(geom_pos) + 3 * g), q)));
    qmat(k->gxmat[g], qmul(q, qload(MF(geom_quat) + 4 * g)));
  }
  for (int s = 0; s < m->nsite; ++s) {
    int b = MI(site_bodyid)[s];
    Q4 q = qload(k->xquat[b]);
    vstore(k->sxpos[s], vadd(vload(k->xpos[b]), qrot(vload(MF(site_pos) + 3 * s), q)));
    qmat(k->sxmat[s], qmul(q, qload(MF(site_quat) + 4 * s)));
  }
}

/* ============================================================ com_pos
 * mjwarp_com_pos.cu:7-88 (subtree com, centered inertia, motion axes) */
static void com_pos(const B200Model *m, Work *k) {
  int nb = m->nbody;
  const int *parent = MI(body_parentid), *root = MI(body_rootid);
  const real *mass = MF(body_mass), *stm = MF(body_subtreemass);
  for (int b = 0; b < nb; ++b)
    for (int c = 0; c < 3; ++c) k->com[b][c] = k->xipos[b][c] * mass[b];
  for (int b = nb - 1; b > 0; --b)
    for (int c = 0; c < 3; ++c) k->com[parent[b]][c] += k->com[b][c];
  for (int b = 0; b < nb; ++b)
    if (stm[b] != 0)
      for (int c = 0; c < 3; ++c) k->com[b][c] /= stm[b];
  for (int b = 0; b < nb; ++b) {
    const real *r = k->ximat[b], *in = MF(body_inertia) + 3 * b, *com = k->com[root[b]];
    real dx = k->xipos[b][0] - com[0], dy = k->xipos[b][1] - com[1], dz = k->xipos[b][2] - com[2];
    real sc[9];
    for (int i = 0; i < 3; ++i)
      for (int j = 0; j < 3; ++j) sc[3 * i + j] = r[3 * i + j] * in[j];
    static const int rows[6] = {0, 1, 2, 0, 0, 1}, cols[6] = {0, 1, 2, 1, 2, 2};
    real *o = k->cinert[b], ms = mass[b];
    for (int i = 0; i < 6; ++i) {
      int a = 3 * rows[i], c = 3 * cols[i];
      o[i] = sc[a] * r[c] + sc[a + 1] * r[c + 1] + sc[a + 2] * r[c + 2];
    }
    o[0] += ms * (dy * dy + dz * dz); o[1] += ms * (dx * dx + dz * dz); o[2] += ms * (dx * dx + dy * dy);
    o[3] -= ms * dx * dy; o[4] -= ms * dx * dz; o[5] -= ms * dy * dz;
    o[6] = ms * dx; o[7] = ms * dy; o[8] = ms * dz; o[9] = ms;
  }
  for (int j = 0; j < m->njnt; ++j) {
    int b = MI(jnt_bodyid)[j], kind = MI(jnt_type)[j];
    real *out = k->cdof[MI(jnt_dofadr)[j]];
    const real *com = k->com[root[b]];
    real dx = com[0] - k->anchor[j][0], dy = com[1] - k->anchor[j][1], dz = com[2] - k->anchor[j][2];
    if (kind == B200_JNT_FREE) {
      for (int a = 0; a < 3; ++a)
        for (int c = 0; c < 6; ++c) out[6 * a + c] = (real)(c == a + 3);
      out += 18;
    }
    if (kind == B200_JNT_FREE || kind == B200_JNT_BALL) {
      const real *r = k->xmat[b];
      for (int a = 0; a < 3; ++a) {
        real x = r[a], y = r[3 + a], z = r[6 + a];
        real *o = out + 6 * a;
        o[0] = x; o[1] = y; o[2] = z;
        o[3] = y * dz - z * dy; o[4] = z * dx - x * dz; o[5] = x * dy - y * dx;
      }
    } else if (kind == B200_JNT_SLIDE) {
      for (int c = 0; c < 3; ++c) { out[c] = 0; out[c + 3] = k->axis[j][c]; }
    } else {
      real x = k->axis[j][0], y = k->axis[j][1], z = k->axis[j][2];
      out[0] = x; out[1] = y; out[2] = z;
      out[3] = y * dz - z * dy; out[4] = z * dx - x * dz; out[5] = x * dy - y * dx;
    }
  }
}

/* spatial inertia (vec10) times motion (angular, linear): mjwarp_mass_matrix.cu:33-39 */
static void inert_mul(const real *i, const real *v, real *r) {
  r[0] = i[0] * v[0] + i[3] * v[1] + i[4] * v[2] - i[8] * v[4] + i[7] * v[5];
  r[1] = i[3] * v[0] + i[1] * v[1] + i[5] * v[2] + i[8] * v[3] - i[6] * v[5];
  r[2] = i[4] * v[0] + i[5] * v[1] + i[2] * v[2] - i[7] * v[3] + i[6] * v[4];
  r[3] = i[8] * v[1] - i[7] * v[2] + i[9] * v[3];
  r[4] = i[6] * v[2] - i[8] * v[0] + i[9] * v[4];
  r[5] = i[7] * v[0] - i[6] * v[1] + i[9] * v[5];
}

/* ============================================================ CRB mass matrix
 * mjwarp_mass_matrix.cu:52-104 (world_mass): composite inertia, then each dof
 * row walks its dof ancestors.  Stored as dense per-tree blocks. */
static void mass_matrix(const B200Model *m, Work *k) {
  int nb = m->nbody;
  memcpy(k->crb, k->cinert, sizeof(real) * 10 * nb);
  for (int b = nb - 1; b > 0; --b) {
    int p = MI(body_parentid)[b];
    if (p == 0) continue; /* world composite inertia is held */
    for (int c = 0; c < 10; ++c) k->crb[p][c] += k->crb[b][c];
  }
  memset(k->M, 0, sizeof(real) * m->nM);
  for (int i = 0; i < m->nv; ++i) {
    real f[6];
    inert_mul(k->crb[MI(dof_bodyid)[i]], k->cdof[i], f);
    int t = tree_of(m, i), a = MI(tree_dofadr)[t], n = MI(tree_dofnum)[t], base = MI(tree_madr)[t];
    for (int j = i; j >= 0; j = MI(dof_parentid)[j]) {
      real v = 0;
      for (int c = 0; c < 6; ++c) v += k->cdof[j][c] * f[c];
      if (j == i) v = MF(dof_armature)[i] + v;
      k->M[base + (i - a) * n + (j - a)] = v;
      k->M[base + (j - a) * n + (i - a)] = v;
    }
  }
}

/* dense upper Cholesky U^T U = A of one n x n block (row-major), the
 * per-tree factor of mjwarp_mass_factor.cu:19-61 (scalar_factor) */
static int chol_upper(const real *A, real *U, int n, int lda) {
  for (int i = 0; i < n; ++i)
    for (int j = 0; j < n; ++j) U[i * lda + j] = 0;
  for (int i = 0; i < n; ++i) {
    real v = A[i * lda + i];
    for (int kk = 0; kk < i; ++kk) v -= U[kk * lda + i] * U[kk * lda + i];
    real d = rsqrt_(v);
    U[i * lda + i] = d;
    real inv = R(1) / d;
    for (int j = i + 1; j < n; ++j) {
      real e = A[j * lda + i];
      for (int kk = 0; kk < i; ++kk) e -= U[kk * lda + i] * U[kk * lda + j];
      U[i * lda + j] = e * inv;
    }
  }
  return 0;
}
/* solve U^T U x = b in place */
static void chol_solve(const real *U, real *x, int n, int lda) {
  for (int i = 0; i < n; ++i) {
    real v = x[i];
    for (int kk = 0; kk < i; ++kk) v -= U[kk * lda + i] * x[kk];
    x[i] = v / U[i * lda + i];
  }
  for (int i = n - 1; i >= 0; --i) {
    real v = x[i];
    for (int kk = i + 1; kk < n; ++kk) v -= U[i * lda + kk] * x[kk];
    x[i] = v / U[i * lda + i];
  }
}
static void factor_mass(const B200Model *m, const real *M, real *L) {
  for (int t = 0; t < m->ntree; ++t) {
    int n = MI(tree_dofnum)[t], base = MI(tree_madr)[t];
    chol_upper(M + base, L + base, n, n);
  }
}
static void solve_mass(const B200Model *m, const real *L, const real *b, real *x) {
  for (int i = 0; i < m->nv; ++i) x[i] = b[i];
  for (int t = 0; t < m->ntree; ++t) {
    int n = MI(tree_dofnum)[t], base = MI(tree_madr)[t], a = MI(tree_dofadr)[t];
    chol_solve(L + base, x + a, n, n);
  }
}
static void mul_mass(const B200Model *m, const real *M, const real *x, real *y) {
  for (int i = 0; i < m->nv; ++i) {
    int t = tree_of(m, i), a = MI(tree_dofadr)[t], n = MI(tree_dofnum)[t];
    const real *row = M + MI(tree_madr)[t] + (i - a) * n;
    real s = 0;
    for (int j = 0; j < n; ++j) s += row[j] * x[a + j];
    y[i] = s;
  }
}

/* ============================================================ collision */
static void contact_frame(V3 a, real *f) { /* mjwarp_contact.cuh:42-48 */
  a = vnormalize(a);
  V3 b = (R(-0.5) < a.v[1] && a.v[1] < R(0.5)) ? v3(0, 1, 0) : v3(0, 0, 1);
  b = vnormalize(vsub(b, vscale(a, vdot(a, b))));
  if (rsqrt_(vdot(a, a)) == 0) b = v3(0, 0, 0);
  V3 c = vcross(a, b);
  vstore(f, a); vstore(f + 3, b); vstore(f + 6, c);
}

typedef struct { int dim; real margin, gap, friction[5], solref[2], solreffriction[2], solimp[5]; } Material;

/* mjwarp_contact.cuh:60-98 contact_material (no explicit <pair>s here) */
static Material material(const B200Model *m, int g1, int g2) {
  Material p;
  memset(&p, 0, sizeof(p));
  p.margin = MF(geom_margin)[g1] + MF(geom_margin)[g2];
  p.gap = MF(geom_gap)[g1] + MF(geom_gap)[g2];
  real m1 = MF(geom_solmix)[g1], m2 = MF(geom_solmix)[g2], mix;
  const real *f1 = MF(geom_friction) + 3 * g1, *f2 = MF(geom_friction) + 3 * g2;
  real f[3];
  int p1 = MI(geom_priority)[g1], p2 = MI(geom_priority)[g2];
  if (p1 > p2) { mix = 1; p.dim = MI(geom_condim)[g1]; for (int c = 0; c < 3; ++c) f[c] = f1[c]; }
  else if (p2 > p1) { mix = 0; p.dim = MI(geom_condim)[g2]; for (int c = 0; c < 3; ++c) f[c] = f2[c]; }
  else {
    mix = m1 + m2 != 0 ? m1 / (m1 + m2) : 0;
    if (m1 < R(1e-15) && m2 < R(1e-15)) mix = R(0.5);
    if (m1 < R(1e-15) && m2 >= R(1e-15)) mix = 0;
    if (m1 >= R(1e-15) && m2 < R(1e-15)) mix = 1;
    p.dim = MI(geom_condim)[g1] > MI(geom_condim)[g2] ? MI(geom_condim)[g1] : MI(geom_condim)[g2];
    for (int c = 0; c < 3; ++c) f[c] = rmax(f1[c], f2[c]);
  }
  p.friction[0] = f[0]; p.friction[1] = f[0]; p.friction[2] = f[1]; p.friction[3] = f[2]; p.friction[4] = f[2];
  const real *r1 = MF(geom_solref) + 2 * g1, *r2 = MF(geom_solref) + 2 * g2;
  const real *i1 = MF(geom_solimp) + 5 * g1, *i2 = MF(geom_solimp) + 5 * g2;
  for (int c = 0; c < 2; ++c) p.solref[c] = r1[0] > 0 && r2[0] > 0 ? mix * r1[c] + (1 - mix) * r2[c] : rmin(r1[c], r2[c]);
  for (int c = 0; c < 5; ++c) p.solimp[c] = mix * i1[c] + (1 - mix) * i2[c];
  for (int c = 0; c < 5; ++c) p.friction[c] = rmax(R(1e-5), p.friction[c]);
  return p;
}

static void publish(Work *k, const B200Model *m, const Material *p, int g1, int g2, real dist, V3 pos,
                    const real *frame) {
  if (!(dist < p->margin + p->gap)) return; /* mjwarp_contact.cuh:100-104 */
  if (k->ncon >= m->ncon_max || k->ncon >= MAXC) { k->overflow |= B200_OVERFLOW_NARROWPHASE; return; }
  Contact *c = &k->con[k->ncon++];
  c->dim = p->dim; c->g1 = g1; c->g2 = g2; c->dist = dist; c->margin = p->margin;
  vstore(c->pos, pos);
  for (int i = 0; i < 9; ++i) c->frame[i] = frame[i];
  for (int i = 0; i < 5; ++i) { c->friction[i] = p->friction[i]; c->solimp[i] = p->solimp[i]; }
  for (int i = 0; i < 2; ++i) { c->solref[i] = p->solref[i]; c->solreffriction[i] = p->solreffriction[i]; }
}

/* ---- broadphase filters: mjwarp_broadphase.cu:21-96 */
static int plane_filter(real r1, real r2, real m1, real m2, V3 p1, V3 p2, const real *R1, const real *R2) {
  if (r1 == 0) return vdot(vsub(p2, p1), mcol(R1, 2)) <= r2 + m1 + m2;
  if (r2 == 0) return vdot(vsub(p1, p2), mcol(R2, 2)) <= r1 + m1 + m2;
  return 1;
}
static int sphere_filter(real r1, real r2, real m1, real m2, V3 p1, V3 p2) {
  real bound = r1 + r2 + m1 + m2;
  V3 d = vsub(p2, p1);
  return vdot(d, d) <= bound * bound;
}
static int obb_filter(V3 c1, V3 c2, V3 s1, V3 s2, real m1, real m2, V3 p1, V3 p2, const real *R1, const real *R2) {
  V3 centers[2] = {vadd(mrot(R1, c1), p1), vadd(mrot(R2, c2), p2)};
  V3 normals[6] = {mcol(R1, 0), mcol(R1, 1), mcol(R1, 2), mcol(R2, 0), mcol(R2, 1), mcol(R2, 2)};
  V3 sizes[2] = {s1, s2};
  real margin = m1 + m2;
  for (int j = 0; j < 2; ++j)
    for (int a = 0; a < 3; ++a) {
      real proj[2], rad[2];
      for (int i = 0; i < 2; ++i) {
        proj[i] = vdot(centers[i], normals[3 * j + a]);
        rad[i] = rabs(sizes[i].v[0] * vdot(normals[3 * i], normals[3 * j + a])) +
                 rabs(sizes[i].v[1] * vdot(normals[3 * i + 1], normals[3 * j + a])) +
                 rabs(sizes[i].v[2] * vdot(normals[3 * i + 2], normals[3 * j + a]));
      }
      if (rad[0] + rad[1] + margin < rabs(proj[1] - proj[0])) return 0;
    }
  return 1;
}
static int broadphase(const B200Model *m, const Work *k, int g1, int g2) {
  const real *aabb = MF(geom_aabb);
  V3 c1 = vload(aabb + 6 * g1), c2 = vload(aabb + 6 * g2), s1 = vload(aabb + 6 * g1 + 3), s2 = vload(aabb + 6 * g2 + 3);
  real r1 = MF(geom_rbound)[g1], r2 = MF(geom_rbound)[g2];
  real m1 = MF(geom_margin)[g1] + MF(geom_gap)[g1], m2 = MF(geom_margin)[g2] + MF(geom_gap)[g2];
  V3 p1 = vload(k->gxpos[g1]), p2 = vload(k->gxpos[g2]);
  const real *R1 = k->gxmat[g1], *R2 = k->gxmat[g2];
  if (r1 == 0 || r2 == 0) return plane_filter(r1, r2, m1, m2, p1, p2, R1, R2);
  if (!sphere_filter(r1, r2, m1, m2, p1, p2)) return 0;
  if (!obb_filter(c1, c2, s1, s2, m1, m2, p1, p2, R1, R2)) return 0;
  return 1;
}

/* ---- plane narrowphase: mjwarp_plane.cu:18-60 */
static void plane_sphere_one(Work *k, const B200Model *m, const Material *p, int g1, int g2, V3 n, V3 o, V3 c,
                             real r, const real *frame) {
  real d = vdot(vsub(c, o), n) - r;
  publish(k, m, p, g1, g2, d, vsub(c, vscale(n, r + R(0.5) * d)), frame);
}
static void plane_mesh(Work *k, const B200Model *m, const Material *p, int g1, int g2, V3 n, V3 origin);
static void plane_collide(Work *k, const B200Model *m, int g1, int g2) {
  Material p = material(m, g1, g2);
  V3 o = vload(k->gxpos[g1]), c = vload(k->gxpos[g2]), n = mcol(k->gxmat[g1], 2);
  const real *Rg = k->gxmat[g2];
  V3 size = vload(MF(geom_size) + 3 * g2);
  int type = MI(geom_type)[g2];
  real frame[9];
  if (type == B200_GEOM_SPHERE) {
    contact_frame(n, frame);
    plane_sphere_one(k, m, &p, g1, g2, n, o, c, size.v[0], frame);
  } else if (type == B200_GEOM_CAPSULE) {
    V3 axis = mcol(Rg, 2);
    V3 tangent = vsub(axis, vscale(n, vdot(n, axis)));
    real len = rsqrt_(vdot(tangent, tangent));
    V3 b = len == 0 ? tangent : vscale(tangent, R(1) / len);
    if (len < R(0.5)) b = (R(-0.5) < n.v[1] && n.v[1] < R(0.5)) ? v3(0, 1, 0) : v3(0, 0, 1);
    vstore(frame, n); vstore(frame + 3, b); vstore(frame + 6, vcross(n, b));
    plane_sphere_one(k, m, &p, g1, g2, n, o, vadd(c, vscale(axis, size.v[1])), size.v[0], frame);
    plane_sphere_one(k, m, &p, g1, g2, n, o, vsub(c, vscale(axis, size.v[1])), size.v[0], frame);
  } else if (type == B200_GEOM_BOX) {
    contact_frame(n, frame);
    real cd = vdot(vsub(c, o), n);
    for (int i = 0; i < 8; ++i) {
      V3 corner = mrot(Rg, v3(i & 1 ? size.v[0] : -size.v[0], i & 2 ? size.v[1] : -size.v[1],
                              i & 4 ? size.v[2] : -size.v[2]));
      real d = cd + vdot(n, corner);
      publish(k, m, &p, g1, g2, d, vsub(vadd(corner, c), vscale(n, R(0.5) * d)), frame);
    }
  } else if (type == B200_GEOM_MESH)
    plane_mesh(k, m, &p, g1, g2, n, o);
}

/* ---- sphere/capsule/box - box: mjwarp_box.cu:14-176 */
typedef struct { int count; real dist[8]; V3 pos[8], normal[8]; } BoxOut;
static void box_init(BoxOut *o, int count) { o->count = count; for (int i = 0; i < 8; ++i) o->dist[i] = R(1e10); }

static void sphere_box(BoxOut *o, int id, V3 sphere, real radius, V3 center, const real *Rb, V3 size) {
  V3 local = mrotT(Rb, vsub(sphere, center)), clamped;
  for (int c = 0; c < 3; ++c) clamped.v[c] = rclamp(local.v[c], -size.v[c], size.v[c]);
  V3 dir = vsub(clamped, local);
  real dist = rsqrt_(vdot(dir, dir));
  dir = dist == 0 ? dir : vscale(dir, R(1) / dist);
  V3 pos, normal;
  if (dist <= R(1e-15)) {
    real closest = R(2) * (size.v[0] + size.v[1] + size.v[2]);
    int face = 0;
    for (int i = 0; i < 6; ++i) {
      real d = rabs((i % 2 ? R(1) : R(-1)) * size.v[i / 2] - local.v[i / 2]);
      if (closest > d) { closest = d; face = i; }
    }
    V3 nearest = v3(0, 0, 0);
    nearest.v[face / 2] = face % 2 ? R(-1) : R(1);
    pos = vadd(local, vscale(nearest, (radius - closest) * R(0.5)));
    normal = mrot(Rb, nearest);
    o->dist[id] = -closest - radius;
  } else {
    V3 deepest = vadd(local, vscale(dir, radius));
    pos = vscale(vadd(clamped, deepest), R(0.5));
    normal = mrot(Rb, dir);
    o->dist[id] = dist - radius;
  }
  o->pos[id] = vadd(center, mrot(Rb, pos));
  o->normal[id] = normal;
}

static void capsule_box(BoxOut *o, V3 center, V3 axis, real radius, real half_length, V3 bc, const real *Rb, V3 size) {
  box_init(o, 2);
  V3 pos = mrotT(Rb, vsub(center, bc));
  axis = mrotT(Rb, axis);
  V3 ha = vscale(axis, half_length);
  int axisdir = (int)(ha.v[0] > 0) + 2 * (int)(ha.v[1] > 0) + 4 * (int)(ha.v[2] > 0);
  real bestdist = R(1e32), bestseg = R(-12), bestbox = 0;
  int type = -4, face = -12, corner = -123, edge = -123;
  for (int i = -1; i <= 1; i += 2) {
    V3 tip = vadd(pos, vscale(ha, (real)i)), point = tip;
    int outside = 0, ax = -1;
    for (int j = 0; j < 3; ++j) {
      if (point.v[j] < -size.v[j]) { ++outside; ax = j; point.v[j] = -size.v[j]; }
      else if (point.v[j] > size.v[j]) { ++outside; ax = j; point.v[j] = size.v[j]; }
    }
    if (outside > 1) continue;
    V3 dif = vsub(point, tip);
    real dist = vdot(dif, dif);
    if (dist < bestdist) { bestdist = dist; bestseg = (real)i; type = -2 + i; face = ax; }
  }
  for (int i = 0; i < 8; ++i)
    for (int j = 0; j < 3; ++j) {
      if (i & (1 << j)) continue;
      V3 point = v3((i & 1 ? R(1) : R(-1)) * size.v[0], (i & 2 ? R(1) : R(-1)) * size.v[1], (i & 4 ? R(1) : R(-1)) * size.v[2]);
      point.v[j] = 0;
      V3 dif = vsub(point, pos);
      real u = -size.v[j] * dif.v[j], v = vdot(ha, dif), ma = size.v[j] * size.v[j], mb = -size.v[j] * ha.v[j],
           mc = half_length * half_length;
      real det = ma * mc - mb * mb;
      if (rabs(det) < R(1e-15)) continue;
      real inv = R(1) / det, x1 = (mc * u - mb * v) * inv, x2 = (ma * v - mb * u) * inv;
      int s1 = 1, s2 = 1;
      if (x1 > 1) { x1 = 1; s1 = 2; x2 = safe_div(v - mb, mc); }
      else if (x1 < -1) { x1 = -1; s1 = 0; x2 = safe_div(v + mb, mc); }
      int over = x2 > 1;
      if (over || x2 < -1) {
        if (over) { x2 = 1; s2 = 2; x1 = safe_div(u - mb, ma); }
        else { x2 = -1; s2 = 0; x1 = safe_div(u + mb, ma); }
        if (x1 > 1) { x1 = 1; s1 = 2; } else if (x1 < -1) { x1 = -1; s1 = 0; }
      }
      dif = vsub(dif, vscale(ha, x2));
      dif.v[j] += size.v[j] * x1;
      real distance = vdot(dif, dif);
      int config = s1 * 3 + s2;
      if (distance < bestdist - R(1e-15)) {
        bestdist = distance; bestseg = x2; bestbox = x1; corner = i + (1 << j) * (config / 6); edge = j; type = config;
      }
    }
  if (type == -4) return;
  real second = -4;
  if (type >= 0 && type / 3 != 1) {
    int config = axisdir ^ corner;
    if (config != 0 && config != 7) {
      int mul;
      if (config == 1 || config == 2 || config == 4) mul = 1; else { mul = -1; config = 7 - config; }
      int ax = config == 1 ? 0 : config == 2 ? 1 : 2, ax1 = (ax + 1) % 3, ax2 = (ax + 2) % 3;
      if (axis.v[ax] * axis.v[ax] > R(0.5)) {
        real mm = R(2) * safe_div(size.v[ax], rabs(ha.v[ax]));
        second = rmin(R(1) - (real)mul * bestseg, mm);
      } else {
        real mm = R(2) * rmin(safe_div(size.v[ax1], rabs(ha.v[ax1])), safe_div(size.v[ax2], rabs(ha.v[ax2])));
        second = -rmin(R(1) + (real)mul * bestseg, mm);
      }
      second *= (real)mul;
    }
  } else if (type >= 0 && type / 3 == 1) {
    int config = (axisdir ^ corner) & (7 - (1 << edge));
    if (config == 1 || config == 2 || config == 4) {
      int ax = edge, ax1 = (edge + 1) % 3, ax2 = (edge + 2) % 3;
      if (rabs(axis.v[ax1]) > rabs(axis.v[ax2])) ax1 = ax2;
      ax2 = 3 - ax - ax1;
      int mul;
      if (config & (1 << ax2)) { mul = 1; second = R(1) - bestseg; } else { mul = -1; second = R(1) + bestseg; }
      real e1 = R(2) * safe_div(size.v[ax2], rabs(ha.v[ax2]));
      second = rmin(e1, second);
      real e2 = (!!(axisdir & (1 << ax))) == (!!(config & (1 << ax2))) ? R(1) - bestbox : R(1) + bestbox;
      e1 = size.v[ax] * safe_div(e2, rabs(ha.v[ax]));
      second = rmin(e1, second);
      second *= (real)mul;
    }
  } else if (type < 0 && face != -1) {
    int mul = type == -3 ? 1 : -1;
    second = 2;
    V3 tmp = vsub(pos, vscale(ha, (real)mul));
    for (int i = 0; i < 3; ++i)
      if (i != face) {
        real inv = safe_div((real)mul, ha.v[i]);
        real e1 = (size.v[i] - tmp.v[i]) * inv;
        if (0 < e1 && e1 < second) second = e1;
        e1 = (-size.v[i] - tmp.v[i]) * inv;
        if (0 < e1 && e1 < second) second = e1;
      }
    second *= (real)mul;
  }
  sphere_box(o, 0, vadd(mrot(Rb, vadd(pos, vscale(ha, bestseg))), bc), radius, bc, Rb, size);
  if (second > -3) sphere_box(o, 1, vadd(mrot(Rb, vadd(pos, vscale(ha, second + bestseg))), bc), radius, bc, Rb, size);
}

static int clip_face(int count, V3 *poly, int coord, real sign, real limit) {
  real d[8];
  int inside = 1;
  for (int i = 0; i < count; ++i) { d[i] = sign * poly[i].v[coord] - limit; if (!(d[i] <= 0)) inside = 0; }
  if (inside) return count;
  V3 clipped[8];
  memset(clipped, 0, sizeof(clipped));
  int n = 0;
  for (int i = 0; i < count; ++i) {
    int nx = i + 1 == count ? 0 : i + 1;
    real dp = d[i], dq = d[nx];
    if (dp <= 0 && n < 8) clipped[n++] = poly[i];
    if (((dp < 0 && dq > 0) || (dp > 0 && dq < 0)) && n < 8) {
      real t = dp / (dp - dq);
      clipped[n++] = vadd(poly[i], vscale(vsub(poly[nx], poly[i]), t));
    }
  }
  for (int i = 0; i < 8; ++i) poly[i] = clipped[i];
  return n;
}

static void box_box(BoxOut *o, V3 p1, const real *R1, V3 size1, V3 p2, const real *R2, V3 size2, real margin) {
  box_init(o, 0);
  V3 pos21 = mrotT(R1, vsub(p2, p1)), pos12 = mrotT(R2, vsub(p1, p2));
  real rot[9], ab[9];
  for (int i = 0; i < 3; ++i)
    for (int j = 0; j < 3; ++j) { rot[3 * i + j] = vdot(mcol(R1, i), mcol(R2, j)); ab[3 * i + j] = rabs(rot[3 * i + j]); }
  real septol = margin + R(1e-6) * (size1.v[0] + size1.v[1] + size1.v[2] + size2.v[0] + size2.v[1] + size2.v[2]);
  real best = R(-1e10);
  int code = -1;
  for (int i = 0; i < 3; ++i) {
    real radius = ab[3 * i] * size2.v[0] + ab[3 * i + 1] * size2.v[1] + ab[3 * i + 2] * size2.v[2];
    real sep = rabs(pos21.v[i]) - size1.v[i] - radius;
    if (sep > septol) return;
    if (sep > best) { best = sep; code = i; }
  }
  for (int j = 0; j < 3; ++j) {
    real radius = ab[j] * size1.v[0] + ab[3 + j] * size1.v[1] + ab[6 + j] * size1.v[2];
    real sep = rabs(pos12.v[j]) - size2.v[j] - radius;
    if (sep > septol) return;
    if (sep > best) { best = sep; code = 3 + j; }
  }
  real face_best = best;
  int face_code = code;
  for (int i = 0; i < 3; ++i)
    for (int j = 0; j < 3; ++j) {
      int i1 = (i + 1) % 3, i2 = (i + 2) % 3;
      real x = -rot[3 * i2 + j], y = rot[3 * i1 + j], n2 = x * x + y * y;
      if (n2 < R(1e-7)) continue;
      real inv = R(1) / rsqrt_(n2);
      x *= inv; y *= inv;
      real rad1 = size1.v[i1] * rabs(x) + size1.v[i2] * rabs(y);
      int j1 = (j + 1) % 3, j2 = (j + 2) % 3;
      real a1 = x * rot[3 * i1 + j1] + y * rot[3 * i2 + j1], a2 = x * rot[3 * i1 + j2] + y * rot[3 * i2 + j2];
      real rad2 = size2.v[j1] * rabs(a1) + size2.v[j2] * rabs(a2);
      real sep = rabs(x * pos21.v[i1] + y * pos21.v[i2]) - rad1 - rad2;
      if (sep > septol) return;
      if (sep - R(1e-6) * rabs(sep) > best && sep > face_best) { best = sep; code = 6 + 3 * i + j; }
    }
  if (code < 0) return;
  int ei = 0, ej = 0, i1 = 0, i2 = 0;
  V3 axis = v3(0, 0, 0);
  if (code >= 6) {
    ei = (code - 6) / 3; ej = (code - 6) % 3; i1 = (ei + 1) % 3; i2 = (ei + 2) % 3;
    axis.v[i1] = -rot[3 * i2 + ej]; axis.v[i2] = rot[3 * i1 + ej];
    axis = vnormalize(axis);
    real align = face_code < 3 ? rabs(axis.v[face_code]) : rabs(vdot(axis, mcol(rot, face_code - 3)));
    if (align > R(0.99) && best < face_best + R(0.05) * rabs(face_best) + R(1e-15)) { code = face_code; best = face_best; }
  }
  if (code >= 6) {
    int j1 = (ej + 1) % 3, j2 = (ej + 2) % 3;
    if (vdot(axis, pos21) < 0) axis = vneg(axis);
    V3 a2 = mrotT(rot, axis);
    int amb1 = -1, amb2 = -1;
    if (rabs(axis.v[i1]) < R(1e-5)) amb1 = i1; else if (rabs(axis.v[i2]) < R(1e-5)) amb1 = i2;
    if (rabs(a2.v[j1]) < R(1e-5)) amb2 = j1; else if (rabs(a2.v[j2]) < R(1e-5)) amb2 = j2;
    V3 d2 = mcol(rot, ej);
    real b = d2.v[ei], denom = R(1) - b * b, best_dist = R(1e10);
    V3 w1 = v3(0, 0, 0), w2 = v3(0, 0, 0);
    for (int u1 = 0; u1 < (amb1 >= 0 ? 2 : 1); ++u1)
      for (int u2 = 0; u2 < (amb2 >= 0 ? 2 : 1); ++u2) {
        V3 c1 = v3(0, 0, 0);
        c1.v[i1] = axis.v[i1] >= 0 ? size1.v[i1] : -size1.v[i1];
        c1.v[i2] = axis.v[i2] >= 0 ? size1.v[i2] : -size1.v[i2];
        if (amb1 >= 0 && u1) c1.v[amb1] = -c1.v[amb1];
        V3 cr = v3(0, 0, 0);
        cr.v[j1] = a2.v[j1] >= 0 ? -size2.v[j1] : size2.v[j1];
        cr.v[j2] = a2.v[j2] >= 0 ? -size2.v[j2] : size2.v[j2];
        if (amb2 >= 0 && u2) cr.v[amb2] = -cr.v[amb2];
        V3 c2 = vadd(mrot(rot, cr), pos21), e = vsub(c2, c1);
        real d1e = e.v[ei], d2e = vdot(d2, e), s = denom >= R(1e-15) ? (d1e - b * d2e) / denom : 0;
        s = rclamp(s, -size1.v[ei], size1.v[ei]);
        real t = rclamp(b * s - d2e, -size2.v[ej], size2.v[ej]);
        s = rclamp(d1e + b * t, -size1.v[ei], size1.v[ei]);
        V3 q1 = c1;
        q1.v[ei] = s;
        V3 q2 = vadd(c2, vscale(d2, t)), gap = vsub(q2, q1);
        real dd = vdot(gap, gap);
        if (dd < best_dist) { best_dist = dd; w1 = q1; w2 = q2; }
      }
    real dist = vdot(vsub(w2, w1), axis);
    if (dist > septol) return;
    o->count = 1; o->dist[0] = dist;
    o->pos[0] = vadd(mrot(R1, vscale(vadd(w1, w2), R(0.5))), p1);
    o->normal[0] = mrot(R1, axis);
    return;
  }
  int ref1 = code < 3, a = ref1 ? code : code - 3;
  V3 size_ref = ref1 ? size1 : size2, size_inc = ref1 ? size2 : size1, pos_ref = ref1 ? p1 : p2, posoi = ref1 ? pos21 : pos12;
  const real *matref = ref1 ? R1 : R2;
  real rinc[9];
  for (int i = 0; i < 3; ++i)
    for (int j = 0; j < 3; ++j) rinc[3 * i + j] = ref1 ? rot[3 * i + j] : rot[3 * j + i];
  real sign = posoi.v[a] >= 0 ? R(1) : R(-1);
  int inc = 0;
  for (int c = 1; c < 3; ++c)
    if (rabs(rinc[3 * a + c]) > rabs(rinc[3 * a + inc])) inc = c;
  real incsign = sign * rinc[3 * a + inc] > 0 ? R(-1) : R(1);
  int ax = (a + 1) % 3, ay = (a + 2) % 3, bu = (inc + 1) % 3, bv = (inc + 2) % 3, coords[3] = {ax, ay, a};
  V3 cx, du, dv;
  for (int r = 0; r < 3; ++r) {
    int c = coords[r];
    cx.v[r] = posoi.v[c] + incsign * size_inc.v[inc] * rinc[3 * c + inc];
    du.v[r] = size_inc.v[bu] * rinc[3 * c + bu];
    dv.v[r] = size_inc.v[bv] * rinc[3 * c + bv];
  }
  cx.v[2] = sign * cx.v[2] - size_ref.v[a];
  du.v[2] *= sign; dv.v[2] *= sign;
  V3 poly[8];
  memset(poly, 0, sizeof(poly));
  for (int c = 0; c < 4; ++c) {
    real su = c == 0 || c == 3 ? R(1) : R(-1), sv = c < 2 ? R(1) : R(-1);
    poly[c] = vadd(vadd(cx, vscale(du, su)), vscale(dv, sv));
  }
  int count = 4;
  count = clip_face(count, poly, 0, 1, size_ref.v[ax]);
  count = clip_face(count, poly, 0, -1, size_ref.v[ax]);
  count = clip_face(count, poly, 1, 1, size_ref.v[ay]);
  count = clip_face(count, poly, 1, -1, size_ref.v[ay]);
  int accepted = 0;
  real dup = R(1e-10) * (size_ref.v[ax] * size_ref.v[ax] + size_ref.v[ay] * size_ref.v[ay]);
  for (int c = 0; c < count; ++c) {
    if (poly[c].v[2] > margin) continue;
    int dupe = 0;
    for (int q = 0; q < accepted; ++q) {
      real dx = o->pos[q].v[0] - poly[c].v[0], dy = o->pos[q].v[1] - poly[c].v[1];
      if (dx * dx + dy * dy < dup) { dupe = 1; break; }
    }
    if (!dupe) o->pos[accepted++] = poly[c];
  }
  if (!accepted) return;
  V3 normal = vscale(mcol(matref, a), ref1 ? sign : -sign);
  for (int c = 0; c < accepted; ++c) {
    V3 v = o->pos[c], local = v3(0, 0, 0);
    local.v[ax] = v.v[0]; local.v[ay] = v.v[1]; local.v[a] = sign * (size_ref.v[a] + R(0.5) * v.v[2]);
    o->dist[c] = v.v[2];
    o->pos[c] = vadd(mrot(matref, local), pos_ref);
    o->normal[c] = normal;
  }
  o->count = accepted;
}

static void box_collide(Work *k, const B200Model *m, int g1, int g2) {
  int t1 = MI(geom_type)[g1];
  Material p = material(m, g1, g2);
  V3 p1 = vload(k->gxpos[g1]), p2 = vload(k->gxpos[g2]);
  V3 s1 = vload(MF(geom_size) + 3 * g1), s2 = vload(MF(geom_size) + 3 * g2);
  const real *R1 = k->gxmat[g1], *R2 = k->gxmat[g2];
  BoxOut o;
  box_init(&o, 1);
  if (t1 == B200_GEOM_SPHERE) sphere_box(&o, 0, p1, s1.v[0], p2, R2, s2);
  else if (t1 == B200_GEOM_CAPSULE) capsule_box(&o, p1, mcol(R1, 2), s1.v[0], s1.v[1], p2, R2, s2);
  else box_box(&o, p1, R1, s1, p2, R2, s2, p.margin + p.gap);
  for (int c = 0; c < o.count; ++c) {
    real frame[9];
    contact_frame(o.normal[c], frame);
    publish(k, m, &p, g1, g2, o.dist[c], o.pos[c], frame);
  }
}

#include "narrow.c"

static void collision(const B200Model *m, Work *k) {
  k->ncon = 0;
  if (m->disable_flags & (B200_DSBL_CONSTRAINT | B200_DSBL_CONTACT)) return;
  const int *pg = MI(pair_geom), *gt = MI(geom_type);
  for (int i = 0; i < m->npair; ++i) {
    int g1 = pg[2 * i], g2 = pg[2 * i + 1];
    if (!broadphase(m, k, g1, g2)) continue;
    int t1 = gt[g1], t2 = gt[g2];
    if (t1 == B200_GEOM_PLANE && t2 >= 2 && t2 <= 7) plane_collide(k, m, g1, g2);
    else if (t2 == B200_GEOM_MESH) convex_collide(k, m, g1, g2);
    /* box-box on the convex path when no box pair has a margin (physics.py:89-90) */
    else if (t1 == B200_GEOM_BOX && t2 == B200_GEOM_BOX && m->boxbox_convex) convex_collide(k, m, g1, g2);
    else if (t2 == B200_GEOM_BOX && (t1 == B200_GEOM_SPHERE || t1 == B200_GEOM_CAPSULE || t1 == B200_GEOM_BOX))
      box_collide(k, m, g1, g2);
    else if ((t1 == B200_GEOM_SPHERE || t1 == B200_GEOM_CAPSULE) && (t2 == B200_GEOM_SPHERE || t2 == B200_GEOM_CAPSULE))
      prim_collide(k, m, g1, g2);
  }
}

/* ============================================================ constraints
 * mjwarp_constraint_build.cu:24-196 */
typedef struct { real k, b, imp; } KBI;
static real rpow(real a, real b) { return IS_F32 ? (real)powf((float)a, (float)b) : (real)pow((double)a, (double)b); }
static KBI impedance(const B200Model *m, const real *ref, const real *imp, real position) {
  const real minval = R(1e-15), minimp = R(0.0001), maximp = R(0.9999);
  int refsafe = !(m->disable_flags & B200_DSBL_REFSAFE);
  real ts = (real)m->timestep;
  real time = refsafe ? rmax(ref[0], R(2) * ts) : ref[0];
  real lo = rclamp(imp[0], minimp, maximp), hi = rclamp(imp[1], minimp, maximp);
  real width = rmax(minval, imp[2]), mid = rclamp(imp[3], minimp, maximp), power = rmax(R(1), imp[4]);
  KBI o;
  o.k = ref[0] <= 0 ? -ref[0] / rmax(minval, hi * hi) : R(1) / rmax(minval, hi * hi * time * time * ref[1] * ref[1]);
  o.b = ref[1] <= 0 ? -ref[1] / rmax(minval, hi) : R(2) / rmax(minval, hi * time);
  real x = rabs(position) / width;
  if (lo == hi || imp[2] <= minval) o.imp = R(0.5) * (lo + hi);
  else if (x <= 0) o.imp = lo;
  else if (x >= 1) o.imp = hi;
  else if (power == 1) o.imp = lo + x * (hi - lo);
  else if (x <= mid) o.imp = rclamp(lo + (R(1) / rpow(mid, power - R(1))) * rpow(x, power) * (hi - lo), lo, hi);
  else o.imp = rclamp(lo + (R(1) - (R(1) / rpow(R(1) - mid, power - R(1))) * rpow(R(1) - x, power)) * (hi - lo), lo, hi);
  return o;
}

static void publish_row(const B200Model *m, Work *k, int r, real pos, real imp_pos, real weight, const real *ref,
                        const real *imp, real velocity, real friction, int type, int id) {
  KBI kbi = impedance(m, ref, imp, imp_pos);
  real kk = type == 1 ? 0 : kbi.k;
  k->efc_D[r] = R(1) / rmax(weight * (R(1) - kbi.imp) / kbi.imp, R(1e-15));
  k->efc_aref[r] = -kk * kbi.imp * pos - kbi.b * velocity;
  k->efc_frictionloss[r] = friction;
  k->efc_type[r] = type;
  k->efc_id[r] = id;
}

static void jac_point(const B200Model *m, const Work *k, int body, int dof, V3 point, real *lin, real *ang) {
  const int *mask = MI(body_dofmask) + 4 * body;
  if (!((((unsigned)mask[dof >> 5]) >> (dof & 31)) & 1u)) {
    lin[0] = lin[1] = lin[2] = ang[0] = ang[1] = ang[2] = 0;
    return;
  }
  const real *mo = k->cdof[dof];
  V3 a = v3(mo[0], mo[1], mo[2]), l = v3(mo[3], mo[4], mo[5]);
  V3 off = vsub(point, vload(k->com[MI(body_rootid)[body]]));
  V3 r = vadd(l, vcross(a, off));
  vstore(lin, r); vstore(ang, a);
}

static void build_constraints(const B200Model *m, Work *k, const real *qpos, const real *qvel) {
  int nv = m->nv, cap = m->nefc_max < MAXE ? m->nefc_max : MAXE;
  k->nefc = 0; k->nf = 0;
  if (m->disable_flags & B200_DSBL_CONSTRAINT) return;
  /* dof friction rows (dof_friction_rows) */
  if (!(m->disable_flags & B200_DSBL_FRICTIONLOSS))
    for (int d = 0; d < nv; ++d) {
      real fl = MF(dof_frictionloss)[d];
      if (fl <= 0) continue;
      if (k->nefc >= cap) { k->overflow |= B200_OVERFLOW_NEFC; continue; }
      int r = k->nefc++;
      k->nf++;
      for (int i = 0; i < nv; ++i) k->J[r][i] = 0;
      k->J[r][d] = 1;
      publish_row(m, k, r, 0, 0, MF(dof_invweight0)[d], MF(dof_solref) + 2 * d, MF(dof_solimp) + 5 * d, qvel[d], fl, 1, d);
    }
  /* joint limit rows (scalar_limit_rows) */
  if (!(m->disable_flags & B200_DSBL_LIMIT))
    for (int l = 0; l < m->nlimited; ++l) {
      int j = MI(limited_jnt)[l], d = MI(jnt_dofadr)[j];
      const real *range = MF(jnt_range) + 2 * j;
      real q = qpos[MI(jnt_qposadr)[j]], margin = MF(jnt_margin)[j];
      real lower = q - range[0], upper = range[1] - q, position = rmin(lower, upper) - margin;
      if (!(position < 0)) continue;
      if (k->nefc >= cap) { k->overflow |= B200_OVERFLOW_NEFC; continue; }
      int r = k->nefc++;
      real sign = (real)(lower < upper) * R(2) - R(1);
      for (int i = 0; i < nv; ++i) k->J[r][i] = 0;
      k->J[r][d] = sign;
      publish_row(m, k, r, position, position, MF(dof_invweight0)[d], MF(jnt_solref) + 2 * j, MF(jnt_solimp) + 5 * j,
                  sign * qvel[d], 0, 3, j);
    }
  /* contact rows (allocate_contacts, contact_jacobian, contact_reference_rows) */
  int elliptic = m->cone == 1;
  for (int c = 0; c < k->ncon; ++c) {
    Contact *ct = &k->con[c];
    k->con_adr[c] = -1;
    if (m->disable_flags & B200_DSBL_CONTACT) continue;
    real position = ct->dist - ct->margin;
    if (!(position < 0)) continue;
    int dim = ct->dim, count = elliptic || dim == 1 ? dim : 2 * (dim - 1);
    if (k->nefc + count > cap) { k->overflow |= B200_OVERFLOW_NEFC; continue; }
    int base = k->nefc;
    k->nefc += count;
    k->con_adr[c] = base;
    int b1 = MI(geom_bodyid)[ct->g1], b2 = MI(geom_bodyid)[ct->g2];
    V3 point = vload(ct->pos);
    real weight = MF(body_invweight0)[2 * b1] + MF(body_invweight0)[2 * b2];
    real ratio = (real)m->impratio_invsqrt;
    for (int comp = 0; comp < count; ++comp) {
      int r = base + comp;
      real jqv = 0;
      for (int d = 0; d < nv; ++d) {
        real l1[3], a1[3], l2[3], a2[3];
        jac_point(m, k, b2, d, point, l2, a2);
        jac_point(m, k, b1, d, point, l1, a1);
        V3 lin = v3(l2[0] - l1[0], l2[1] - l1[1], l2[2] - l1[2]), ang = v3(a2[0] - a1[0], a2[1] - a1[1], a2[2] - a1[2]);
        real v;
        if (elliptic) v = vdot(comp < 3 ? lin : ang, vload(ct->frame + 3 * (comp % 3)));
        else {
          v = vdot(lin, vload(ct->frame));
          if (dim > 1) {
            int dir = comp / 2 + 1;
            real fr = ct->friction[dir - 1] * (R(1) - R(2) * (real)(comp & 1));
            v += vdot(dir < 3 ? lin : ang, vload(ct->frame + 3 * (dir % 3))) * fr;
          }
        }
        k->J[r][d] = v;
        jqv += v * qvel[d];
      }
      real w = weight, scale = 1, pos_aref = position;
      if (elliptic && comp > 0) {
        scale = ratio * ratio;
        if (comp > 1) scale *= ct->friction[0] * ct->friction[0] / (ct->friction[comp - 1] * ct->friction[comp - 1]);
        pos_aref = 0;
      } else if (!elliptic && dim > 1) {
        w = w + ct->friction[0] * ct->friction[0] * w;
        w = w * R(2) * ct->friction[0] * ct->friction[0] * ratio * ratio;
      }
      int type = dim == 1 ? 5 : elliptic ? 7 : 6;
      publish_row(m, k, r, pos_aref, position, w, ct->solref, ct->solimp, jqv, 0, type, c);
      if (elliptic && comp > 0) {
        k->efc_D[r] /= scale;
        const real *ref = ct->solref;
        if (ct->solreffriction[0] != 0 || ct->solreffriction[1] != 0) ref = ct->solreffriction;
        real damping = impedance(m, ref, ct->solimp, position).b;
        k->efc_aref[r] = -damping * jqv;
      }
    }
  }
}

/* ============================================================ velocity stage
 * fused_motion.cu:13-186 (cvel, cdof_dot, RNE bias), mjwarp_passive.cu:12-48 */
static void motion_cross(const real *v, const real *u, real *out) { /* v x u, spatial motion */
  out[0] = -v[2] * u[1] + v[1] * u[2];
  out[1] = v[2] * u[0] - v[0] * u[2];
  out[2] = -v[1] * u[0] + v[0] * u[1];
  out[3] = -v[2] * u[4] + v[1] * u[5] - v[5] * u[1] + v[4] * u[2];
  out[4] = v[2] * u[3] - v[0] * u[5] + v[5] * u[0] - v[3] * u[2];
  out[5] = -v[1] * u[3] + v[0] * u[4] - v[4] * u[0] + v[3] * u[1];
}
static void force_cross(const real *v, const real *f, real *out) { /* v x* f */
  out[0] = -v[2] * f[1] + v[1] * f[2] - v[5] * f[4] + v[4] * f[5];
  out[1] = v[2] * f[0] - v[0] * f[2] + v[5] * f[3] - v[3] * f[5];
  out[2] = -v[1] * f[0] + v[0] * f[1] - v[4] * f[3] + v[3] * f[4];
  out[3] = -v[2] * f[4] + v[1] * f[5];
  out[4] = v[2] * f[3] - v[0] * f[5];
  out[5] = -v[1] * f[3] + v[0] * f[4];
}

static void velocity_stage(const B200Model *m, Work *k, const real *qpos, const real *qvel) {
  int nb = m->nbody, nv = m->nv;
  real cacc[MAXB][6], cfrc[MAXB][6];
  for (int c = 0; c < 6; ++c) { k->cvel[0][c] = 0; cacc[0][c] = 0; }
  if (!(m->disable_flags & B200_DSBL_GRAVITY)) {
    cacc[0][3] = -(real)m->gravity_x; cacc[0][4] = -(real)m->gravity_y; cacc[0][5] = -(real)m->gravity_z;
  }
  for (int b = 1; b < nb; ++b) {
    int p = MI(body_parentid)[b];
    real vel[6], acc[6];
    for (int c = 0; c < 6; ++c) { vel[c] = k->cvel[p][c]; acc[c] = cacc[p][c]; }
    int dof = MI(body_dofadr)[b];
    for (int j = MI(body_jntadr)[b]; j < MI(body_jntadr)[b] + MI(body_jntnum)[b]; ++j) {
      int type = MI(jnt_type)[j];
      if (type == B200_JNT_FREE) {
        for (int i = 0; i < 3; ++i) {
          for (int c = 0; c < 6; ++c) vel[c] += k->cdof[dof + i][c] * qvel[dof + i];
          for (int c = 0; c < 6; ++c) k->cdof_dot[dof + i][c] = 0;
        }
        dof += 3;
      }
      int width = type == B200_JNT_FREE || type == B200_JNT_BALL ? 3 : 1;
      /* derivatives use the velocity before this joint's contribution */
      for (int i = 0; i < width; ++i) {
        real dd[6];
        motion_cross(vel, k->cdof[dof + i], dd);
        for (int c = 0; c < 6; ++c) { k->cdof_dot[dof + i][c] = dd[c]; acc[c] += dd[c] * qvel[dof + i]; }
      }
      for (int i = 0; i < width; ++i)
        for (int c = 0; c < 6; ++c) vel[c] += k->cdof[dof + i][c] * qvel[dof + i];
      dof += width;
    }
    for (int c = 0; c < 6; ++c) { k->cvel[b][c] = vel[c]; cacc[b][c] = acc[c]; }
  }
  for (int c = 0; c < 6; ++c) cfrc[0][c] = 0;
  for (int b = 1; b < nb; ++b) {
    real f[6], mom[6], corr[6];
    inert_mul(k->cinert[b], cacc[b], f);
    inert_mul(k->cinert[b], k->cvel[b], mom);
    force_cross(k->cvel[b], mom, corr);
    for (int c = 0; c < 6; ++c) cfrc[b][c] = f[c] + corr[c];
  }
  for (int b = nb - 1; b > 0; --b) {
    int p = MI(body_parentid)[b];
    for (int c = 0; c < 6; ++c) cfrc[p][c] += cfrc[b][c];
  }
  for (int d = 0; d < nv; ++d) {
    const real *f = cfrc[MI(dof_bodyid)[d]];
    real v = 0;
    for (int c = 0; c < 6; ++c) v += k->cdof[d][c] * f[c];
    k->qfrc_bias[d] = v;
  }
  /* passive: damper (and hinge/slide springs) */
  for (int j = 0; j < m->njnt; ++j) {
    int d = MI(jnt_dofadr)[j], kind = MI(jnt_type)[j], p = MI(jnt_qposadr)[j];
    int width = kind == B200_JNT_FREE ? 6 : kind == B200_JNT_BALL ? 3 : 1;
    for (int i = 0; i < width; ++i) {
      real damping = MF(dof_damping)[d + i], force = 0;
      if (!(m->disable_flags & B200_DSBL_DAMPER) && damping != 0) force = -qvel[d + i] * damping;
      k->qfrc_passive[d + i] = force;
    }
    real stiff = MF(jnt_stiffness)[j];
    if (!(m->disable_flags & B200_DSBL_SPRING) && stiff != 0 && (kind == B200_JNT_SLIDE || kind == B200_JNT_HINGE)) {
      real delta = qpos[p] - MF(qpos_spring)[p];
      k->qfrc_passive[d] += -delta * stiff;
    }
  }
  /* transmission (joint, gear): length and moment */
  for (int u = 0; u < m->nu; ++u) {
    int j = MI(actuator_trnid)[u];
    real gear = MF(actuator_gear)[u];
    k->act_length[u] = gear * qpos[MI(jnt_qposadr)[j]];
    k->act_moment[u] = gear;
  }
}

/* ============================================================ OSC controller
 * FP64 robosuite OSC_POSE: fused_control_drive.cu:35-111 (gather),
 * osc_solver.cu:309-676 (control), rotation_delta osc_solver.cu:279-306,
 * action_component osc_solver.cu:36-45, pinv_group osc_solver.cu:120-253 */
static int inverse7(const double *A, double *inv) {
  double lu[49];
  int piv[7];
  memcpy(lu, A, sizeof(lu));
  for (int c = 0; c < 7; ++c) {
    int p = c;
    for (int r = c + 1; r < 7; ++r) if (fabs(lu[r * 7 + c]) > fabs(lu[p * 7 + c])) p = r;
    piv[c] = p;
    if (lu[p * 7 + c] == 0) return 1;
    if (p != c) for (int k = 0; k < 7; ++k) { double t = lu[c * 7 + k]; lu[c * 7 + k] = lu[p * 7 + k]; lu[p * 7 + k] = t; }
    for (int r = c + 1; r < 7; ++r) {
      double f = lu[r * 7 + c] / lu[c * 7 + c];
      lu[r * 7 + c] = f;
      for (int k = c + 1; k < 7; ++k) lu[r * 7 + k] -= f * lu[c * 7 + k];
    }
  }
  for (int col = 0; col < 7; ++col) {
    double x[7];
    for (int i = 0; i < 7; ++i) x[i] = i == col;
    for (int c = 0; c < 7; ++c) if (piv[c] != c) { double t = x[c]; x[c] = x[piv[c]]; x[piv[c]] = t; }
    for (int i = 0; i < 7; ++i) for (int k = 0; k < i; ++k) x[i] -= lu[i * 7 + k] * x[k];
    for (int i = 6; i >= 0; --i) {
      for (int k = i + 1; k < 7; ++k) x[i] -= lu[i * 7 + k] * x[k];
      x[i] /= lu[i * 7 + i];
    }
    for (int i = 0; i < 7; ++i) inv[i * 7 + col] = x[i];
  }
  return 0;
}

/* one-sided Jacobi pseudoinverse of the leading n x n block of a 6-stride matrix */
static int pinv_jacobi(const double *in, double *out, int n) {
  double scale = 0, B[6][6], V[6][6];
  for (int i = 0; i < 36; ++i) out[i] = 0;
  for (int r = 0; r < n; ++r) for (int c = 0; c < n; ++c) scale = fmax(scale, fabs(in[r * 6 + c]));
  if (!(scale > 0)) return 1;
  for (int r = 0; r < n; ++r) for (int c = 0; c < n; ++c) { B[r][c] = in[r * 6 + c] / scale; V[r][c] = r == c; }
  int converged = 0;
  for (int sweep = 0; sweep < 64; ++sweep) {
    int rotations = 0;
    for (int p = 0; p < n - 1; ++p)
      for (int q = p + 1; q < n; ++q) {
        double alpha = 0, beta = 0, gamma = 0;
        for (int r = 0; r < n; ++r) { alpha += B[r][p] * B[r][p]; beta += B[r][q] * B[r][q]; gamma += B[r][p] * B[r][q]; }
        if (fabs(gamma) > DBL_EPSILON * sqrt(alpha) * sqrt(beta)) {
          double zeta = (beta - alpha) / (2 * gamma);
          double t = (zeta < 0 ? -1.0 : 1.0) / (fabs(zeta) + sqrt(1 + zeta * zeta));
          double c = 1 / sqrt(1 + t * t), s = c * t;
          for (int r = 0; r < n; ++r) {
            double bp = B[r][p], bq = B[r][q], vp = V[r][p], vq = V[r][q];
            B[r][p] = c * bp - s * bq; B[r][q] = s * bp + c * bq;
            V[r][p] = c * vp - s * vq; V[r][q] = s * vp + c * vq;
          }
          ++rotations;
        }
      }
    if (rotations == 0) { converged = 1; break; }
  }
  double norms[6], sing[6], maxn = 0;
  int keep[6];
  for (int p = 0; p < n; ++p) {
    double s = 0;
    for (int r = 0; r < n; ++r) s += B[r][p] * B[r][p];
    norms[p] = s; sing[p] = sqrt(s); maxn = fmax(maxn, sing[p]);
  }
  for (int p = 0; p < n; ++p) keep[p] = sing[p] > 1e-15 * maxn;
  double maxcorr = 0;
  for (int p = 0; p < n; ++p)
    for (int q = p + 1; q < n; ++q)
      if (keep[p] && keep[q]) {
        double g = 0;
        for (int r = 0; r < n; ++r) g += B[r][p] * B[r][q];
        maxcorr = fmax(maxcorr, fabs(g) / (sing[p] * sing[q]));
      }
  if (maxcorr < 2e-15) converged = 1;
  for (int r = 0; r < n; ++r)
    for (int c = 0; c < n; ++c) {
      double v = 0;
      for (int k = 0; k < n; ++k) if (keep[k]) v += V[r][k] * B[c][k] * ((1 / norms[k]) / scale);
      out[r * 6 + c] = v;
    }
  return !converged;
}

static real action_component(const B200Model *m, real action, int axis) {
  const real *p = MF(osc_action_config);
  real scale = rabs(p[18 + axis] - p[12 + axis]) / rabs(p[6 + axis] - p[axis]);
  real a = action != action ? action : rmin(p[6 + axis], rmax(p[axis], action));
  return (a - (p[6 + axis] + p[axis]) * R(0.5)) * scale + (p[18 + axis] + p[12 + axis]) * R(0.5);
}

static void rotation_delta(real x, real y, real z, double *r) {
  real angle = rsqrt_(x * x + y * y + z * z);
  real f = angle == 0 ? 0 : (IS_F32 ? (real)sinf((float)(angle * R(0.5))) : (real)sin((double)(angle * R(0.5)))) / angle;
  real raw[4] = {x * f, y * f, z * f,
                 angle == 0 ? R(1) : (IS_F32 ? (real)cosf((float)(angle * R(0.5))) : (real)cos((double)(angle * R(0.5))))};
  float q[4] = {(float)raw[3], (float)raw[0], (float)raw[1], (float)raw[2]};
  real acc = 0;
  for (int i = 0; i < 4; ++i) acc += (real)(q[i] * q[i]);
  float norm = (float)acc;
  real factor = rsqrt_(R(2) / (real)norm);
  for (int i = 0; i < 4; ++i) q[i] = (float)((real)q[i] * factor);
  r[0] = (double)(R(1) - (real)(q[2] * q[2]) - (real)(q[3] * q[3]));
  r[4] = (double)(R(1) - (real)(q[1] * q[1]) - (real)(q[3] * q[3]));
  r[8] = (double)(R(1) - (real)(q[1] * q[1]) - (real)(q[2] * q[2]));
  r[1] = (double)(real)(q[1] * q[2] - q[3] * q[0]);
  r[2] = (double)(real)(q[1] * q[3] + q[2] * q[0]);
  r[3] = (double)(real)(q[1] * q[2] + q[3] * q[0]);
  r[5] = (double)(real)(q[2] * q[3] - q[1] * q[0]);
  r[6] = (double)(real)(q[1] * q[3] - q[2] * q[0]);
  r[7] = (double)(real)(q[2] * q[3] + q[1] * q[0]);
}

typedef struct {
  real *goal_pos, *goal_rot, *gripper, *ctrl;
  const real *action;
  int *error;
} OscState;

static void osc(const B200Model *m, Work *k, const real *qpos, const real *qvel, OscState *s, int policy) {
  if (*s->error) return;
  int nv = m->nv, site = m->ee_site, body = MI(site_bodyid)[site];
  const int *qi = MI(osc_qposadr), *vi = MI(osc_dofadr);
  V3 point = vload(k->sxpos[site]);
  real jp[3][MAXV], jr[3][MAXV];
  for (int d = 0; d < nv; ++d) {
    real l[3], a[3];
    jac_point(m, k, body, d, point, l, a);
    for (int c = 0; c < 3; ++c) { jp[c][d] = l[c]; jr[c][d] = a[c]; }
  }
  real ee_vel[6];
  for (int ax = 0; ax < 6; ++ax) {
    real v = 0;
    for (int d = 0; d < nv; ++d) v += (ax < 3 ? jp[ax][d] : jr[ax - 3][d]) * qvel[d];
    ee_vel[ax] = v;
  }
  double M7[49], J[42], JT[42], q[7], qd[7], bias[7];
  for (int r = 0; r < 7; ++r) {
    for (int c = 0; c < 7; ++c) M7[r * 7 + c] = (double)mass_at(m, k->M, vi[r], vi[c]);
    q[r] = (double)qpos[qi[r]]; qd[r] = (double)qvel[vi[r]]; bias[r] = (double)k->qfrc_bias[vi[r]];
  }
  for (int ax = 0; ax < 6; ++ax)
    for (int c = 0; c < 7; ++c) {
      J[ax * 7 + c] = (double)(ax < 3 ? jp[ax][vi[c]] : jr[ax - 3][vi[c]]);
      JT[c * 6 + ax] = J[ax * 7 + c];
    }
  double Mi[49];
  if (inverse7(M7, Mi)) { *s->error = 2; return; }
  double MJT[42], A[36], Ap[36], Ar[36], Lf[36], Lp[36], Lr[36];
  for (int r = 0; r < 7; ++r)
    for (int c = 0; c < 6; ++c) { double v = 0; for (int k2 = 0; k2 < 7; ++k2) v += Mi[r * 7 + k2] * JT[k2 * 6 + c]; MJT[r * 6 + c] = v; }
  for (int r = 0; r < 6; ++r)
    for (int c = 0; c < 6; ++c) { double v = 0; for (int k2 = 0; k2 < 7; ++k2) v += J[r * 7 + k2] * MJT[k2 * 6 + c]; A[r * 6 + c] = v; }
  for (int z = 0; z < 36; ++z) {
    int r = z / 6, c = z % 6;
    Ap[z] = r < 3 && c < 3 ? A[z] : 0;
    Ar[z] = r < 3 && c < 3 ? A[(r + 3) * 6 + c + 3] : 0;
  }
  int bad = pinv_jacobi(A, Lf, 6);
  bad |= pinv_jacobi(Ap, Lp, 3);
  bad |= pinv_jacobi(Ar, Lr, 3);
  if (bad) { *s->error = 4; return; }
  double Jbar[42], N[49];
  for (int r = 0; r < 7; ++r)
    for (int c = 0; c < 6; ++c) { double v = 0; for (int k2 = 0; k2 < 6; ++k2) v += MJT[r * 6 + k2] * Lf[k2 * 6 + c]; Jbar[r * 6 + c] = v; }
  for (int r = 0; r < 7; ++r)
    for (int c = 0; c < 7; ++c) {
      double v = 0;
      for (int k2 = 0; k2 < 6; ++k2) v += Jbar[r * 6 + k2] * J[k2 * 7 + c];
      N[r * 7 + c] = (r == c ? 1.0 : 0.0) - v;
    }
  /* goal */
  double gp[3], gr[9], cur[9];
  for (int r = 0; r < 3; ++r) {
    gp[r] = (double)s->goal_pos[r];
    for (int c = 0; c < 9 / 3; ++c) { gr[r * 3 + c] = (double)s->goal_rot[r * 3 + c]; cur[r * 3 + c] = (double)k->sxmat[site][r * 3 + c]; }
  }
  if (policy) {
    for (int r = 0; r < 3; ++r) gp[r] = (double)(real)(k->sxpos[site][r] + action_component(m, s->action[r], r));
    real x = action_component(m, s->action[3], 3), y = action_component(m, s->action[4], 4), z = action_component(m, s->action[5], 5);
    if (x != 0 || y != 0 || z != 0) {
      double d[9], g2[9];
      rotation_delta(x, y, z, d);
      for (int r = 0; r < 3; ++r)
        for (int c = 0; c < 3; ++c) { double v = 0; for (int k2 = 0; k2 < 3; ++k2) v += d[r * 3 + k2] * cur[k2 * 3 + c]; g2[r * 3 + c] = v; }
      for (int i = 0; i < 9; ++i) gr[i] = IS_F32 ? (double)(float)g2[i] : g2[i];
    }
  }
  const real *gains = MF(osc_gains);
  double desired[6];
  for (int r = 0; r < 3; ++r) {
    int nx = (r + 1) % 3, ls = (r + 2) % 3;
    double er = 0;
    for (int c = 0; c < 3; ++c) er += 0.5 * (cur[nx * 3 + c] * gr[ls * 3 + c] - cur[ls * 3 + c] * gr[nx * 3 + c]);
    double ep = gp[r] - (double)k->sxpos[site][r];
    desired[r] = (double)gains[r] * ep - (double)gains[r + 6] * (double)ee_vel[r];
    desired[r + 3] = (double)gains[r + 3] * er - (double)gains[r + 9] * (double)ee_vel[r + 3];
  }
  double pd[7], op[6], opm[7];
  const real *q0 = MF(osc_q0), *nul = MF(osc_null);
  for (int c = 0; c < 7; ++c) pd[c] = (double)nul[0] * ((double)q0[c] - q[c]) - (double)nul[1] * qd[c];
  for (int l = 0; l < 6; ++l) {
    double v = 0;
    if (m->osc_uncouple) {
      int row = l % 3, off = l < 3 ? 0 : 3;
      const double *lam = l < 3 ? Lp : Lr;
      for (int k2 = 0; k2 < 3; ++k2) v += lam[row * 6 + k2] * desired[off + k2];
    } else
      for (int k2 = 0; k2 < 6; ++k2) v += Lf[l * 6 + k2] * desired[k2];
    op[l] = v;
  }
  for (int r = 0; r < 7; ++r) { double v = 0; for (int k2 = 0; k2 < 7; ++k2) v += M7[r * 7 + k2] * pd[k2]; opm[r] = v; }
  const int *ids = MI(osc_actuator);
  for (int i = 0; i < 7; ++i) {
    double task = 0, post = 0;
    for (int k2 = 0; k2 < 6; ++k2) task += JT[i * 6 + k2] * op[k2];
    for (int k2 = 0; k2 < 7; ++k2) post += N[k2 * 7 + i] * opm[k2];
    double t = task + bias[i] + post;
    const real *rg = MF(actuator_ctrlrange) + 2 * ids[i];
    double lim = t != t ? t : fmin((double)rg[1], fmax((double)rg[0], t));
    s->ctrl[ids[i]] = (real)lim;
  }
  for (int r = 0; r < 3; ++r) s->goal_pos[r] = (real)gp[r];
  for (int i = 0; i < 9; ++i) s->goal_rot[i] = (real)gr[i];
  real a6 = s->action[6], sgn = a6 != a6 ? a6 : (a6 > 0 ? R(1) : (a6 < 0 ? R(-1) : R(0)));
  real speed = MF(osc_action_config)[24];
  for (int i = 0; i < 2; ++i) {
    real v = s->gripper[i] + speed * (i == 0 ? R(-1) : R(1)) * sgn;
    v = v != v ? v : rmin(R(1), rmax(R(-1), v));
    s->gripper[i] = v;
    const real *rg = MF(actuator_ctrlrange) + 2 * ids[7 + i];
    s->ctrl[ids[7 + i]] = (rg[1] + rg[0]) * R(0.5) + (rg[1] - rg[0]) * R(0.5) * v;
  }
}

/* ============================================================ actuation
 * mjwarp_actuation.cu:14-55, mjwarp_smooth_force.cu:35-45, mass_solve */
static void actuation(const B200Model *m, Work *k, const real *qpos, const real *qvel, const real *ctrl) {
  int nv = m->nv;
  for (int d = 0; d < nv; ++d) k->qfrc_actuator[d] = 0;
  for (int u = 0; u < m->nu; ++u) {
    real c = ctrl[u];
    if (MI(actuator_ctrllimited)[u] && !(m->disable_flags & B200_DSBL_CLAMPCTRL)) {
      const real *rg = MF(actuator_ctrlrange) + 2 * u;
      c = rmin(rmax(rg[0], c), rg[1]);
    }
    const real *gp = MF(actuator_gainprm) + 3 * u, *bp = MF(actuator_biasprm) + 3 * u;
    int j = MI(actuator_trnid)[u], d = MI(jnt_dofadr)[j];
    real vel = k->act_moment[u] * qvel[d];
    real gain = gp[0];
    if (MI(actuator_gaintype)[u] == 1) gain = gp[0] + gp[1] * k->act_length[u] + gp[2] * vel;
    real bias = 0;
    if (MI(actuator_biastype)[u] == 1) bias = bp[0] + bp[1] * k->act_length[u] + bp[2] * vel;
    real force = gain * c + bias;
    if (MI(actuator_forcelimited)[u]) {
      const real *fr = MF(actuator_forcerange) + 2 * u;
      force = rmin(rmax(fr[0], force), fr[1]);
    }
    k->act_force[u] = force;
    k->qfrc_actuator[d] += k->act_moment[u] * force;
  }
  for (int d = 0; d < nv; ++d)
    k->qfrc_smooth[d] = k->qfrc_passive[d] - k->qfrc_bias[d] + k->qfrc_actuator[d];
  solve_mass(m, k->L, k->qfrc_smooth, k->qacc_smooth);
}

/* ============================================================ Newton solver
 * mjwarp_solver_state.cu, mjwarp_constraint.cu, mjwarp_hessian.cu,
 * mjwarp_direction.cu, mjwarp_linesearch.cu */
enum { kSatisfied = 0, kQuadratic = 1, kLinearNegative = 2, kLinearPositive = 3, kCone = 4 };

static void eval_constraints(const B200Model *m, Work *k) {
  int nv = m->nv;
  real impratio = (real)m->impratio_invsqrt;
  for (int r = 0; r < k->nefc; ++r) {
    real d = k->efc_D[r], res = k->efc_jaref[r], force;
    int state;
    int friction = r >= k->ne && r < k->ne + k->nf;
    if (r < k->ne) { force = -d * res; state = kQuadratic; }
    else if (friction) {
      real loss = k->efc_frictionloss[r], radius = safe_div(loss, d);
      if (res <= -radius) { force = loss; state = kLinearNegative; }
      else if (res >= radius) { force = -loss; state = kLinearPositive; }
      else { force = -d * res; state = kQuadratic; }
    } else if (k->efc_type[r] == 7) {
      const Contact *ct = &k->con[k->efc_id[r]];
      int head = k->con_adr[k->efc_id[r]];
      real mu = ct->friction[0] * impratio, normal = k->efc_jaref[head], d0 = k->efc_D[head];
      real tt = 0, tscale = 0;
      for (int j = 1; j < ct->dim; ++j) {
        real u = k->efc_jaref[head + j] * ct->friction[j - 1];
        tt += u * u;
        if (r == head + j) tscale = u * ct->friction[j - 1];
      }
      real n = normal * mu, t = tt <= 0 ? 0 : rsqrt_(tt);
      if (n >= mu * t || (t <= 0 && n >= 0)) { force = 0; state = kSatisfied; }
      else if (mu * n + t <= 0 || (t <= 0 && n < 0)) { force = -d * res; state = kQuadratic; }
      else {
        real dm = safe_div(d0, mu * mu * (R(1) + mu * mu));
        real fn = -dm * (n - mu * t) * mu;
        force = r == head ? fn : -safe_div(fn, t) * tscale;
        state = kCone;
      }
    } else if (res >= 0) { force = 0; state = kSatisfied; }
    else { force = -d * res; state = kQuadratic; }
    k->efc_force[r] = force;
    k->efc_state[r] = state;
  }
  k->grad_dot = 0;
  for (int i = 0; i < nv; ++i) {
    real tot = 0;
    for (int r = 0; r < k->nefc; ++r) tot += k->J[r][i] * k->efc_force[r];
    k->qfrc_constraint[i] = tot;
    real g = k->Ma[i] - k->qfrc_smooth[i] - tot;
    k->grad[i] = g;
    k->grad_dot += g * g;
  }
}

static void hessian(const B200Model *m, Work *k) {
  int nv = m->nv;
  real impratio = (real)m->impratio_invsqrt;
  for (int i = 0; i < nv; ++i)
    for (int j = 0; j < nv; ++j) {
      real v = mass_at(m, k->M, i, j);
      for (int r = 0; r < k->nefc; ++r)
        if (k->efc_state[r] == kQuadratic) v += k->J[r][i] * k->efc_D[r] * k->J[r][j];
      k->H[i * nv + j] = v;
    }
  if (m->cone != 1) return;
  for (int c = 0; c < k->ncon; ++c) {
    const Contact *ct = &k->con[c];
    int head = k->con_adr[c];
    if (head < 0 || ct->dim == 1 || k->efc_state[head] != kCone) continue;
    real mu = ct->friction[0] * impratio, mu2 = mu * mu;
    real den = mu2 * (R(1) + mu2);
    real dm = k->efc_D[head] / (den != 0 ? den : R(1e-15));
    if (dm == 0) continue;
    real n = k->efc_jaref[head] * mu, tt = 0;
    for (int d = 1; d < ct->dim; ++d) { real u = k->efc_jaref[head + d] * ct->friction[d - 1]; tt += u * u; }
    real t = rmax(rsqrt_(tt), R(1e-15)), it = R(1) / t, mnt = mu * n * it;
    for (int i = 0; i < nv; ++i)
      for (int j = i; j < nv; ++j) {
        real z01 = mu * k->J[head][i], z02 = mu * k->J[head][j], p1 = 0, p2 = 0, td = 0;
        for (int d = 1; d < ct->dim; ++d) {
          real s = ct->friction[d - 1], u = k->efc_jaref[head + d] * s;
          real z1 = s * k->J[head + d][i], z2 = s * k->J[head + d][j];
          p1 += u * z1; p2 += u * z2; td += z1 * z2;
        }
        p1 *= it; p2 *= it;
        real cv = dm * (z01 * z02 - mu * (z01 * p2 + z02 * p1) + mnt * p1 * p2 + (mu2 - mnt) * td);
        k->H[i * nv + j] += cv;
        if (j != i) k->H[j * nv + i] += cv;
      }
  }
}

static void direction(const B200Model *m, Work *k) {
  int nv = m->nv;
  real *U = k->U;
  chol_upper(k->H, U, nv, nv);
  real x[MAXV];
  for (int i = 0; i < nv; ++i) x[i] = k->grad[i];
  chol_solve(U, x, nv, nv);
  real sq = 0, dec = 0;
  for (int i = 0; i < nv; ++i) { k->search[i] = -x[i]; sq += x[i] * x[i]; dec += k->grad[i] * x[i]; }
  k->search_dot = sq;
  k->decrement = dec;
}

/* ---- exact line search: mjwarp_linesearch.cu:80-365 (Point algebra) */
typedef struct { real cost, slope, curv; } Pt;
static Pt padd(Pt a, Pt b) { Pt o = {a.cost + b.cost, a.slope + b.slope, a.curv + b.curv}; return o; }
static Pt quadratic(real q1, real q2, real alpha) { real aq2 = alpha * q2; Pt o = {alpha * aq2 + alpha * q1, R(2) * aq2 + q1, R(2) * q2}; return o; }
static int in_bracket(Pt x, Pt y) { return (x.slope < y.slope && y.slope < 0) || (x.slope > y.slope && y.slope > 0); }

typedef struct {
  int kind; /* 0 equality, 1 frictionloss, 2 inequality, 3 primary cone, 4 secondary */
  real x, v, d, loss, q0, q1, q2, u0, v0, uu, uv, vv, dm, mu, cost0, t0, r0;
  int state0;
} Row;

static Row load_row(const B200Model *m, const Work *k, int r) {
  Row o;
  memset(&o, 0, sizeof(o));
  if (r < k->ne) o.kind = 0; /* equality: always quadratic */
  else if (r < k->ne + k->nf) o.kind = 1;
  else if (k->efc_type[r] != 7) o.kind = 2;
  else {
    int c = k->efc_id[r], head = k->con_adr[c];
    if (r != head) { o.kind = 4; return o; }
    o.kind = 3;
    const real *qa = k->quad[r], *qb = k->quad[head + 1], *qc = k->quad[head + 2];
    o.q0 = qa[0]; o.q1 = qa[1]; o.q2 = qa[2];
    o.u0 = qb[0]; o.v0 = qb[1]; o.uu = qb[2];
    o.uv = qc[0]; o.vv = qc[1]; o.dm = qc[2];
    o.mu = k->con[c].friction[0] * (real)m->impratio_invsqrt;
    if (o.uu <= 0) { o.state0 = o.u0 < 0 ? 1 : 0; o.cost0 = o.state0 == 1 ? o.q0 : 0; }
    else {
      o.t0 = rsqrt_(o.uu);
      if (o.u0 >= o.mu * o.t0) o.state0 = 0;
      else if (o.mu * o.u0 + o.t0 <= 0) { o.state0 = 1; o.cost0 = o.q0; }
      else { o.state0 = 4; o.r0 = o.u0 - o.mu * o.t0; o.cost0 = R(0.5) * o.dm * o.r0 * o.r0; }
    }
    return o;
  }
  o.x = k->efc_jaref[r]; o.v = k->efc_jv[r]; o.d = k->efc_D[r];
  if (o.kind == 1) o.loss = k->efc_frictionloss[r];
  return o;
}
static Pt friction_point(const Row *r, real x) {
  real rf = safe_div(r->loss, r->d);
  if (-rf < x && x < rf) { real vd = r->v * r->d; Pt o = {R(0.5) * r->d * x * x, vd * x, r->v * vd}; return o; }
  if (x <= -rf) { Pt o = {r->loss * (R(-0.5) * rf - x), -r->loss * r->v, 0}; return o; }
  { Pt o = {r->loss * (R(-0.5) * rf + x), r->loss * r->v, 0}; return o; }
}
static Pt eval_zero(const Row *r) {
  Pt z = {0, 0, 0};
  if (r->kind == 4) return z;
  if (r->kind == 3) {
    if (r->state0 == 1) { Pt o = {r->q0, r->q1, R(2) * r->q2}; return o; }
    if (r->state0 == 4) {
      real ti = R(1) / r->t0, t1 = r->uv * ti, t2 = (r->vv - t1 * t1) * ti, r1 = r->v0 - r->mu * t1;
      Pt o = {r->cost0, r->dm * r->r0 * r1, r->dm * (r1 * r1 - r->mu * r->r0 * t2)};
      return o;
    }
    return z;
  }
  if (r->kind == 1) return friction_point(r, r->x);
  if (r->kind == 2 && r->x >= 0) return z;
  { real vd = r->v * r->d; Pt o = {R(0.5) * r->d * r->x * r->x, vd * r->x, r->v * vd}; return o; }
}
static Pt cone_quad_shift(const Row *r, real alpha, real n, real tsqr) {
  real aq2 = alpha * r->q2, cost = alpha * (aq2 + r->q1);
  if (r->state0 == 4) { real bd = r->mu * r->u0 + r->t0; cost += R(0.5) * r->dm * bd * bd; }
  else if (r->state0 == 0) cost = R(0.5) * r->dm * (R(1) + r->mu * r->mu) * (n * n + rmax(tsqr, 0));
  Pt o = {cost, R(2) * aq2 + r->q1, R(2) * r->q2};
  return o;
}
static Pt eval_shift(const Row *r, real alpha) {
  Pt z = {0, 0, 0};
  if (r->kind == 4) return z;
  if (r->kind == 3) {
    real n = r->u0 + alpha * r->v0, tsd = alpha * (R(2) * r->uv + alpha * r->vv), tsqr = r->uu + tsd;
    if (tsqr <= 0) {
      if (n < 0) return cone_quad_shift(r, alpha, n, tsqr);
    } else {
      real t = rsqrt_(tsqr);
      if (n >= r->mu * t) {
      } else if (r->mu * n + t <= 0) return cone_quad_shift(r, alpha, n, tsqr);
      else {
        real ti = R(1) / t, t1 = (r->uv + alpha * r->vv) * ti, t2 = (r->vv - t1 * t1) * ti;
        real res = n - r->mu * t, r1 = r->v0 - r->mu * t1, cost;
        if (r->state0 == 4) {
          real tdelta = tsd / (t + r->t0), rdelta = alpha * r->v0 - r->mu * tdelta;
          cost = R(0.5) * r->dm * rdelta * (R(2) * r->r0 + rdelta);
        } else if (r->state0 == 1) {
          real aq2 = alpha * r->q2, bd = r->mu * n + t;
          cost = alpha * (aq2 + r->q1) - R(0.5) * r->dm * bd * bd;
        } else cost = R(0.5) * r->dm * res * res;
        Pt o = {cost, r->dm * res * r1, r->dm * (r1 * r1 + res * (-r->mu * t2))};
        return o;
      }
    }
    { Pt o = {-r->cost0, 0, 0}; return o; }
  }
  if (r->kind == 1) {
    Pt pt = friction_point(r, r->x + alpha * r->v);
    pt.cost -= friction_point(r, r->x).cost;
    return pt;
  }
  real quad0 = R(0.5) * r->d * r->x * r->x;
  real cost0 = r->kind == 2 && r->x >= 0 ? 0 : quad0;
  if (r->kind == 2 && r->x + alpha * r->v >= 0) { Pt o = {-cost0, 0, 0}; return o; }
  real vd = r->v * r->d, h = r->v * vd, ah = alpha * h;
  Pt o = {alpha * (vd * r->x + R(0.5) * ah) + (quad0 - cost0), vd * r->x + ah, h};
  return o;
}

static Pt rows_at(const B200Model *m, const Work *k, real alpha, int zero) {
  Pt s = {0, 0, 0};
  for (int r = 0; r < k->nefc; ++r) {
    Row row = load_row(m, k, r);
    s = padd(s, zero ? eval_zero(&row) : eval_shift(&row, alpha));
  }
  return s;
}

static void linesearch(const B200Model *m, Work *k, int *overflow) {
  int nv = m->nv;
  mul_mass(m, k->M, k->search, k->Mv);
  for (int r = 0; r < k->nefc; ++r) {
    real s = 0;
    for (int i = 0; i < nv; ++i) s += k->J[r][i] * k->search[i];
    k->efc_jv[r] = s;
  }
  real impratio = (real)m->impratio_invsqrt;
  for (int r = 0; r < k->nefc; ++r) {
    if (k->efc_type[r] != 7) continue;
    int c = k->efc_id[r];
    if (r != k->con_adr[c]) continue;
    const Contact *ct = &k->con[c];
    real x = k->efc_jaref[r], v = k->efc_jv[r], d = k->efc_D[r], vd = v * d;
    real q0 = R(0.5) * x * x * d, q1 = vd * x, q2 = R(0.5) * v * vd;
    real mu = ct->friction[0] * impratio, u0 = x * mu, v0 = v * mu, uu = 0, uv = 0, vv = 0;
    for (int j = 1; j < ct->dim; ++j) {
      int t = r + j;
      real jv = k->efc_jv[t], ja = k->efc_jaref[t], dj = k->efc_D[t], djx = dj * ja;
      q0 += R(0.5) * ja * djx; q1 += jv * djx; q2 += R(0.5) * jv * dj * jv;
      real fr = ct->friction[j - 1], uj = ja * fr, vj = jv * fr;
      uu += uj * uj; uv += uj * vj; vv += vj * vj;
    }
    k->quad[r][0] = q0; k->quad[r][1] = q1; k->quad[r][2] = q2;
    k->quad[r + 1][0] = u0; k->quad[r + 1][1] = v0; k->quad[r + 1][2] = uu;
    k->quad[r + 2][0] = uv; k->quad[r + 2][1] = vv;
    real mu2 = mu * mu;
    k->quad[r + 2][2] = d / (mu2 * (R(1) + mu2));
  }
  real tol = (real)m->tolerance, lstol = (real)m->ls_tolerance;
  real scale = (real)m->meaninertia * (real)nv;
  real gtol = rmax(tol * lstol * rsqrt_(k->search_dot) * scale, R(1e-6));
  real g1 = 0, g2 = 0;
  for (int i = 0; i < nv; ++i) { g1 += k->search[i] * (k->Ma[i] - k->qfrc_smooth[i]); g2 += R(0.5) * k->search[i] * k->Mv[i]; }
  const real NoiseEps = R(8) * (real)FLT_EPSILON;
  Pt rows = rows_at(m, k, 0, 1);
  k->ls_evals += 1;
  Pt p0 = {rows.cost, g1 + rows.slope, R(2) * g2 + rows.curv};
  Pt delta = {0, p0.slope, p0.curv};
  real q1abs = rsqrt_(R(2) * rmax(rows.cost, 0) * rmax(rows.curv, 0)) + rabs(g1);
  real gacc = rmax(gtol, NoiseEps * q1abs), alpha = 0, improvement = 0;
  int converged = rabs(p0.slope) < NoiseEps * q1abs;
  real a0 = -safe_div(p0.slope, p0.curv);
  Pt init = {0, 0, 0};
  if (!converged) {
    init = padd(quadratic(g1, g2, a0), rows_at(m, k, a0, 0));
    k->ls_evals += 1;
    if (rabs(init.slope) < gacc && init.cost < 0) { converged = 1; alpha = a0; improvement = -init.cost; }
  }
  if (!converged) {
    int less = init.slope < p0.slope;
    Pt lo = less ? init : delta, hi = less ? delta : init;
    real la = less ? a0 : 0, ha = less ? 0 : a0;
    for (int it = 0; it < m->ls_iterations; ++it) {
      real ln = la - safe_div(lo.slope, lo.curv), hn = ha - safe_div(hi.slope, hi.curv), ma = R(0.5) * (la + ha);
      Pt nl = padd(quadratic(g1, g2, ln), rows_at(m, k, ln, 0));
      Pt nh = padd(quadratic(g1, g2, hn), rows_at(m, k, hn, 0));
      Pt mid = padd(quadratic(g1, g2, ma), rows_at(m, k, ma, 0));
      k->ls_evals += 3;
      int cl = rabs(nl.slope) < gacc && nl.cost < 0, ch = rabs(nh.slope) < gacc && nh.cost < 0;
      int cm = rabs(mid.slope) < gacc && mid.cost < 0;
      int any = cl || ch || cm, slo = 0, shi = 0;
      if (any) {
        Pt best = {R(1e10), 0, 0};
        real ba = 0;
        if (cl && nl.cost < best.cost) { best = nl; ba = ln; }
        if (ch && nh.cost < best.cost) { best = nh; ba = hn; }
        if (cm && mid.cost < best.cost) { best = mid; ba = ma; }
        lo = hi = best; la = ha = ba;
      } else {
        int s;
        s = in_bracket(lo, nl); if (s) { lo = nl; la = ln; } slo |= s;
        s = in_bracket(lo, mid); if (s) { lo = mid; la = ma; } slo |= s;
        s = in_bracket(lo, nh); if (s) { lo = nh; la = hn; } slo |= s;
        s = in_bracket(hi, nh) || (hi.slope < 0 && nh.slope > 0); if (s) { hi = nh; ha = hn; } shi |= s;
        s = in_bracket(hi, mid); if (s) { hi = mid; ha = ma; } shi |= s;
        s = in_bracket(hi, nl); if (s) { hi = nl; ha = ln; } shi |= s;
      }
      int done = any || (!slo && !shi) || (lo.cost < 0 && lo.slope < 0 && lo.slope > -gtol) ||
                 (hi.cost < 0 && hi.slope > 0 && hi.slope < gtol);
      if (lo.cost < 0 || hi.cost < 0) {
        int bl = lo.cost < hi.cost;
        alpha = bl ? la : ha;
        improvement = -(bl ? lo.cost : hi.cost);
      }
      if (done) { converged = 1; break; }
    }
  }
  for (int i = 0; i < nv; ++i) { k->qacc[i] += alpha * k->search[i]; k->Ma[i] += alpha * k->Mv[i]; }
  for (int r = 0; r < k->nefc; ++r) k->efc_jaref[r] += alpha * k->efc_jv[r];
  k->improvement = improvement;
  k->alpha = alpha;
  if (!converged) *overflow |= B200_OVERFLOW_LS_ITERATIONS;
}

static void newton(const B200Model *m, Work *k, const real *warmstart, int *overflow) {
  int nv = m->nv;
  int warm = !(m->disable_flags & B200_DSBL_WARMSTART);
  for (int i = 0; i < nv; ++i) k->qacc[i] = warm && k->nefc > 0 ? warmstart[i] : k->qacc_smooth[i];
  mul_mass(m, k->M, k->qacc, k->Ma);
  for (int r = 0; r < k->nefc; ++r) {
    real s = 0;
    for (int i = 0; i < nv; ++i) s += k->J[r][i] * k->qacc[i];
    k->efc_jaref[r] = s - k->efc_aref[r];
  }
  k->niter = 0; k->done = 0;
  eval_constraints(m, k);
  hessian(m, k);
  direction(m, k);
  if (m->iterations == 0) return;
  real tol = (real)m->tolerance, scale = (real)m->meaninertia * (real)nv;
  while (!k->done) {
    linesearch(m, k, overflow);
    eval_constraints(m, k);
    hessian(m, k);
    direction(m, k);
    int it = ++k->niter;
    real imp = k->improvement / scale, grad = rsqrt_(k->grad_dot) / scale, model = (R(0.5) * k->decrement) / scale;
    int done = k->alpha == 0 || (imp > 0 && imp < tol) || grad < tol || model < tol;
    if (done || it == m->iterations) {
      if (!done) *overflow |= B200_OVERFLOW_ITERATIONS;
      k->done = 1;
    }
  }
}

/* ============================================================ Euler
 * mjwarp_euler.cu:20-86, fused_euler_step.cu */
static Q4 quat_integrate(Q4 q, const real *v, real dt) {
  real len = rsqrt_(v[0] * v[0] + v[1] * v[1] + v[2] * v[2]), x = 0, y = 0, z = 0;
  if (len > 0) { x = v[0] / len; y = v[1] / len; z = v[2] / len; }
  real ang = dt * len, s, c;
  if (IS_F32) { s = (real)sinf((float)(ang * R(0.5))); c = (real)cosf((float)(ang * R(0.5))); }
  else { s = (real)sin((double)(ang * R(0.5))); c = (real)cos((double)(ang * R(0.5))); }
  Q4 b = {c, x * s, y * s, z * s};
  q = qnormalize(q);
  return qnormalize(qmul(q, b));
}

/* qpos += dt * qvel on the joint manifold (mjwarp_euler.cu:34-96) */
static void integrate_positions(const B200Model *m, real *qpos, const real *qvel, real dt) {
  for (int j = 0; j < m->njnt; ++j) {
    int kind = MI(jnt_type)[j];
    real *q = qpos + MI(jnt_qposadr)[j];
    const real *v = qvel + MI(jnt_dofadr)[j];
    if (kind == B200_JNT_FREE) { q[0] += dt * v[0]; q[1] += dt * v[1]; q[2] += dt * v[2]; q += 3; v += 3; }
    if (kind == B200_JNT_FREE || kind == B200_JNT_BALL) {
      Q4 r = quat_integrate(qload(q), v, dt);
      qstore(q, r);
    } else q[0] += dt * v[0];
  }
}

static void euler(const B200Model *m, Work *k, real *qpos, real *qvel, real *qacc_out, real *warmstart) {
  int nv = m->nv;
  real dt = (real)m->timestep, acc[MAXV];
  int damped = !(m->disable_flags & (B200_DSBL_EULERDAMP | B200_DSBL_DAMPER));
  if (damped) {
    real *Md = k->Md, *Ld = k->Ld;
    memcpy(Md, k->M, sizeof(real) * m->nM);
    for (int d = 0; d < nv; ++d) {
      int t = tree_of(m, d), a = MI(tree_dofadr)[t], n = MI(tree_dofnum)[t];
      Md[MI(tree_madr)[t] + (d - a) * n + (d - a)] += dt * MF(dof_damping)[d];
    }
    factor_mass(m, Md, Ld);
    solve_mass(m, Ld, k->Ma, acc);
  } else
    for (int d = 0; d < nv; ++d) acc[d] = k->qacc[d];
  for (int d = 0; d < nv; ++d) {
    if (qacc_out) qacc_out[d] = k->qacc[d];
    warmstart[d] = k->qacc[d];
  }
  for (int d = 0; d < nv; ++d) qvel[d] = qvel[d] + acc[d] * dt;
  integrate_positions(m, qpos, qvel, dt);
}

/* ============================================================ driver */
#define DR(name, w, width) ((d->name) ? ((real *)(d->name) + (size_t)(w) * (width)) : (real *)0)
#define DI(name, w, width) ((d->name) ? ((d->name) + (size_t)(w) * (width)) : (int *)0)

static void publish_outputs(const B200Model *m, const B200Data *d, Work *k, int w) {
  int nb = m->nbody, ng = m->ngeom, ns = m->nsite, nv = m->nv;
  real *p;
  if ((p = DR(xpos, w, nb * 3))) memcpy(p, k->xpos, sizeof(real) * nb * 3);
  if ((p = DR(xquat, w, nb * 4))) memcpy(p, k->xquat, sizeof(real) * nb * 4);
  if ((p = DR(xmat, w, nb * 9))) memcpy(p, k->xmat, sizeof(real) * nb * 9);
  if ((p = DR(geom_xpos, w, ng * 3))) memcpy(p, k->gxpos, sizeof(real) * ng * 3);
  if ((p = DR(geom_xmat, w, ng * 9))) memcpy(p, k->gxmat, sizeof(real) * ng * 9);
  if ((p = DR(site_xpos, w, ns * 3))) memcpy(p, k->sxpos, sizeof(real) * ns * 3);
  if ((p = DR(site_xmat, w, ns * 9))) memcpy(p, k->sxmat, sizeof(real) * ns * 9);
  if ((p = DR(subtree_com, w, nb * 3))) memcpy(p, k->com, sizeof(real) * nb * 3);
  if ((p = DR(qfrc_bias, w, nv))) memcpy(p, k->qfrc_bias, sizeof(real) * nv);
  if ((p = DR(qfrc_actuator, w, nv))) memcpy(p, k->qfrc_actuator, sizeof(real) * nv);
  if ((p = DR(qfrc_constraint, w, nv))) memcpy(p, k->qfrc_constraint, sizeof(real) * nv);
  if ((p = DR(qacc_smooth, w, nv))) memcpy(p, k->qacc_smooth, sizeof(real) * nv);
  if ((p = DR(qfrc_smooth, w, nv))) memcpy(p, k->qfrc_smooth, sizeof(real) * nv);
  if ((p = DR(qM, w, nv * nv)))
    for (int i = 0; i < nv; ++i)
      for (int j = 0; j < nv; ++j) p[i * nv + j] = mass_at(m, k->M, i, j);
  int nc = m->ncon_max, ne = m->nefc_max;
  if ((p = DR(con_friction, w, nc * 5))) for (int c = 0; c < k->ncon; ++c) memcpy(p + 5 * c, k->con[c].friction, sizeof(real) * 5);
  if ((p = DR(con_margin, w, nc))) for (int c = 0; c < k->ncon; ++c) p[c] = k->con[c].margin;
  if ((p = DR(con_dist, w, nc))) for (int c = 0; c < k->ncon; ++c) p[c] = k->con[c].dist;
  if ((p = DR(con_pos, w, nc * 3))) for (int c = 0; c < k->ncon; ++c) memcpy(p + 3 * c, k->con[c].pos, sizeof(real) * 3);
  if ((p = DR(con_frame, w, nc * 9))) for (int c = 0; c < k->ncon; ++c) memcpy(p + 9 * c, k->con[c].frame, sizeof(real) * 9);
  if ((p = DR(efc_force, w, ne))) for (int r = 0; r < k->nefc; ++r) p[r] = k->efc_force[r];
  if ((p = DR(efc_D, w, ne))) for (int r = 0; r < k->nefc; ++r) p[r] = k->efc_D[r];
  if ((p = DR(efc_aref, w, ne))) for (int r = 0; r < k->nefc; ++r) p[r] = k->efc_aref[r];
  if ((p = DR(efc_J, w, ne * nv))) for (int r = 0; r < k->nefc; ++r) memcpy(p + r * nv, k->J[r], sizeof(real) * nv);
  int *ip;
  if ((ip = DI(efc_type, w, ne))) for (int r = 0; r < k->nefc; ++r) ip[r] = k->efc_type[r];
  if ((ip = DI(efc_id, w, ne))) for (int r = 0; r < k->nefc; ++r) ip[r] = k->efc_id[r];
  if ((ip = DI(ncon, w, 1))) *ip = k->ncon;
  if ((ip = DI(nefc, w, 1))) *ip = k->nefc;
  if ((ip = DI(con_geom, w, nc * 2))) for (int c = 0; c < k->ncon; ++c) { ip[2 * c] = k->con[c].g1; ip[2 * c + 1] = k->con[c].g2; }
  if ((ip = DI(con_dim, w, nc))) for (int c = 0; c < k->ncon; ++c) ip[c] = k->con[c].dim;
}

/* observation slab: arm+gripper qpos/qvel (current), end-effector pose and
 * free-body poses from the last substep's kinematics, then reward and done:
 * the task body's origin above task_lift_z (the synthetic scenes' sparse
 * success predicate) */
static void publish_obs(const B200Model *m, const B200Data *d, const Work *k, int w, const real *qpos,
                        const real *qvel) {
  real *o = DR(obs, w, m->nobs);
  if (!o) return;
  for (int e = 0; e < m->nobs; ++e) o[e] = 0;
  for (int c = 0; c < 9; ++c) {
    int jq, jd;
    if (c < 7) { jq = MI(osc_qposadr)[c]; jd = MI(osc_dofadr)[c]; }
    else {
      int j = MI(actuator_trnid)[MI(osc_actuator)[c]];
      jq = MI(jnt_qposadr)[j]; jd = MI(jnt_dofadr)[j];
    }
    o[c] = qpos[jq];
    o[9 + c] = qvel[jd];
  }
  int s = m->ee_site, b = MI(site_bodyid)[s];
  for (int c = 0; c < 3; ++c) o[18 + c] = k->sxpos[s][c];
  Q4 q = qmul(qload(k->xquat[b]), qload(MF(site_quat) + 4 * s));
  o[21] = q.w; o[22] = q.x; o[23] = q.y; o[24] = q.z;
  for (int f = 0; f < m->nfree; ++f) {
    int fb = MI(free_bodyid)[f];
    for (int c = 0; c < 3; ++c) o[25 + 7 * f + c] = k->xpos[fb][c];
    for (int c = 0; c < 4; ++c) o[25 + 7 * f + 3 + c] = k->xquat[fb][c];
  }
  if (m->task_body >= 0 && m->task_body < m->nfree) {
    real success = k->xpos[MI(free_bodyid)[m->task_body]][2] > (real)m->task_lift_z ? R(1) : R(0);
    o[25 + 7 * m->nfree] = success;
    o[25 + 7 * m->nfree + 1] = success;
  }
}

/* MuJoCo mj_checkPos / mj_checkVel: a non-finite or huge (> 1e10) entry */
static int bad_state(const B200Model *m, const real *qpos, const real *qvel) {
  for (int i = 0; i < m->nq; ++i) if (!(rabs(qpos[i]) <= R(1e10))) return 1;
  for (int i = 0; i < m->nv; ++i) if (!(rabs(qvel[i]) <= R(1e10))) return 1;
  return 0;
}

/* position + velocity stage (reference Physics.step1, physics.py:185) */
static void step1(const B200Model *m, Work *k, const real *qpos, const real *qvel) {
  kinematics(m, k, qpos);
  com_pos(m, k);
  mass_matrix(m, k);
  factor_mass(m, k->M, k->L);
  collision(m, k);
  build_constraints(m, k, qpos, qvel);
  velocity_stage(m, k, qpos, qvel);
}

static int check_model(const B200Model *m) {
  return m && m->real_bytes == (int)sizeof(real) && m->nbody <= MAXB && m->nv <= MAXV && m->ngeom <= MAXG &&
         m->nsite <= 8 && m->nu <= 16 && m->nvariant >= 0 && m->variant_stride >= 0;
}

/* The model as world w of the shard sees it: the real arrays of its parameter
 * row, (world_offset + w) % nvariant (mjwarp_constraint_build.cu:18-20). */
static B200Model world_model(const B200Model *base, const B200Data *d, int w) {
  B200Model m = *base;
  if (base->nvariant > 1) {
    long long row = ((long long)d->world_offset + w) % base->nvariant;
    m.real = (const real *)base->real + (size_t)row * (size_t)base->variant_stride;
  }
  return m;
}

/* Advance worlds [w0, w1) by `substeps` substeps (reference control graph). */
int oracle_step(const B200Model *base, const B200Data *d, int w0, int w1, int substeps, int policy) {
  if (!check_model(base)) return 1;
  Work *k = (Work *)calloc(1, sizeof(Work));
  if (!k) return 2;
  int nq = base->nq, nv = base->nv, nu = base->nu;
  for (int w = w0; w < w1; ++w) {
    const B200Model mw = world_model(base, d, w), *m = &mw;
    real *qpos = DR(qpos, w, nq), *qvel = DR(qvel, w, nv), *warm = DR(qacc_warmstart, w, nv);
    int *overflow = DI(overflow, w, 1), *error = DI(error, w, 1);
    if (bad_state(m, qpos, qvel)) *overflow |= B200_STATUS_BADSTATE;
    int stepped = 0;
    for (int s = 0; s < substeps; ++s) {
      if (*overflow & B200_STATUS_BADSTATE) break; /* a bad world is not stepped (further) */
      k->overflow = 0;
      step1(m, k, qpos, qvel);
      OscState os = {DR(goal_pos, w, 3), DR(goal_rot, w, 9), DR(gripper, w, 2), DR(ctrl, w, nu), DR(action, w, 7), error};
      osc(m, k, qpos, qvel, &os, policy && s == 0);
      actuation(m, k, qpos, qvel, DR(ctrl, w, nu));
      int of = k->overflow;
      newton(m, k, warm, &of);
      *overflow |= of;
      if (d->niter) *DI(niter, w, 1) = k->niter;
      if (d->newton_total) *DI(newton_total, w, 1) += k->niter;
      if (d->ls_total) *DI(ls_total, w, 1) += k->ls_evals;
      if (d->efc_total) *DI(efc_total, w, 1) += k->nefc;
      if (d->con_total) *DI(con_total, w, 1) += k->ncon;
      if (d->newton_rows) *DI(newton_rows, w, 1) += k->niter * k->nefc;
      if (d->ls_rows) *DI(ls_rows, w, 1) += k->ls_evals * k->nefc;
      if (s < 32 && d->niter_trace) DI(niter_trace, w, 32)[s] = k->niter;
      if (s < 32 && d->ls_trace) DI(ls_trace, w, 32)[s] = k->ls_evals;
      k->ls_evals = 0;
      if (s == substeps - 1) publish_outputs(m, d, k, w);
      euler(m, k, qpos, qvel, DR(qacc, w, nv), warm);
      *DR(time, w, 1) += (real)m->timestep;
      if (d->integration_count) *DI(integration_count, w, 1) += 1;
      if (bad_state(m, qpos, qvel)) *overflow |= B200_STATUS_BADSTATE;
      ++stepped;
    }
    if (stepped > 0) publish_obs(m, d, k, w, qpos, qvel);
  }
  free(k);
  return 0;
}

/* Forward only (reference Physics.forward): no integration. */
int oracle_forward(const B200Model *base, const B200Data *d, int w0, int w1, int bootstrap) {
  if (!check_model(base)) return 1;
  Work *k = (Work *)calloc(1, sizeof(Work));
  if (!k) return 2;
  int nq = base->nq, nv = base->nv, nu = base->nu;
  for (int w = w0; w < w1; ++w) {
    const B200Model mw = world_model(base, d, w), *m = &mw;
    real *qpos = DR(qpos, w, nq), *qvel = DR(qvel, w, nv), *warm = DR(qacc_warmstart, w, nv);
    if (bad_state(m, qpos, qvel)) *DI(overflow, w, 1) |= B200_STATUS_BADSTATE;
    step1(m, k, qpos, qvel);
    if (bootstrap) {
      int site = m->ee_site;
      for (int c = 0; c < 3; ++c) DR(goal_pos, w, 3)[c] = k->sxpos[site][c];
      for (int c = 0; c < 9; ++c) DR(goal_rot, w, 9)[c] = k->sxmat[site][c];
      real *gr = DR(gripper, w, 2);
      gr[0] = gr[1] = 0;
      *DI(error, w, 1) = 0;
    }
    actuation(m, k, qpos, qvel, DR(ctrl, w, nu));
    int of = k->overflow;
    newton(m, k, warm, &of);
    *DI(overflow, w, 1) |= of;
    publish_outputs(m, d, k, w);
    publish_obs(m, d, k, w, qpos, qvel);
    real *qa = DR(qacc, w, nv);
    if (qa) memcpy(qa, k->qacc, sizeof(real) * nv);
    if (d->niter) *DI(niter, w, 1) = k->niter;
    k->ls_evals = 0;
  }
  free(k);
  return 0;
}

/* ---- leaf entry points for the golden-vector tests (one world) ---- */
int oracle_leaf_positions(const B200Model *m, const real *qpos, real *xpos, real *xquat, real *xipos, real *gxpos,
                          real *gxmat, real *com, real *cinert, real *cdof, real *M) {
  if (!check_model(m)) return 1;
  Work *k = (Work *)calloc(1, sizeof(Work));
  kinematics(m, k, qpos);
  com_pos(m, k);
  mass_matrix(m, k);
  memcpy(xpos, k->xpos, sizeof(real) * 3 * m->nbody);
  memcpy(xquat, k->xquat, sizeof(real) * 4 * m->nbody);
  memcpy(xipos, k->xipos, sizeof(real) * 3 * m->nbody);
  memcpy(gxpos, k->gxpos, sizeof(real) * 3 * m->ngeom);
  memcpy(gxmat, k->gxmat, sizeof(real) * 9 * m->ngeom);
  memcpy(com, k->com, sizeof(real) * 3 * m->nbody);
  memcpy(cinert, k->cinert, sizeof(real) * 10 * m->nbody);
  memcpy(cdof, k->cdof, sizeof(real) * 6 * m->nv);
  for (int i = 0; i < m->nv; ++i)
    for (int j = 0; j < m->nv; ++j) M[i * m->nv + j] = mass_at(m, k->M, i, j);
  free(k);
  return 0;
}

/* box/sphere/capsule vs box narrowphase on raw poses (fixtures) */
int oracle_leaf_box(int type1, const real *p1, const real *R1, const real *s1, const real *p2, const real *R2,
                    const real *s2, real margin, real *dist, real *pos, real *normal) {
  BoxOut o;
  box_init(&o, 1);
  if (type1 == B200_GEOM_SPHERE) sphere_box(&o, 0, vload(p1), s1[0], vload(p2), R2, vload(s2));
  else if (type1 == B200_GEOM_CAPSULE) capsule_box(&o, vload(p1), mcol(R1, 2), s1[0], s1[1], vload(p2), R2, vload(s2));
  else box_box(&o, vload(p1), R1, vload(s1), vload(p2), R2, vload(s2), margin);
  for (int c = 0; c < o.count; ++c) {
    dist[c] = o.dist[c];
    vstore(pos + 3 * c, o.pos[c]);
    vstore(normal + 3 * c, o.normal[c]);
  }
  return o.count;
}

/* collision + constraint rows of one world from qpos/qvel (fixtures, tests).
   Per contact: geoms[2], dim, and 28 reals (dist, pos[3], frame[9], margin,
   friction[5], solref[2], solimp[5], solreffriction[2]); per row: the dense
   Jacobian row (nv), D, aref, type, id. */
int oracle_leaf_contacts(const B200Model *m, const real *qpos, const real *qvel, int *ncon, int *geoms, int *dims,
                         real *con_reals, int *nefc, real *J, real *efc_D, real *efc_aref, int *efc_type,
                         int *efc_id) {
  if (!check_model(m)) return 1;
  Work *k = (Work *)calloc(1, sizeof(Work));
  kinematics(m, k, qpos);
  com_pos(m, k);
  collision(m, k);
  build_constraints(m, k, qpos, qvel);
  *ncon = k->ncon;
  for (int c = 0; c < k->ncon; ++c) {
    const Contact *q = &k->con[c];
    real *o = con_reals + 28 * c;
    geoms[2 * c] = q->g1; geoms[2 * c + 1] = q->g2; dims[c] = q->dim;
    o[0] = q->dist;
    memcpy(o + 1, q->pos, sizeof(real) * 3);
    memcpy(o + 4, q->frame, sizeof(real) * 9);
    o[13] = q->margin;
    memcpy(o + 14, q->friction, sizeof(real) * 5);
    memcpy(o + 19, q->solref, sizeof(real) * 2);
    memcpy(o + 21, q->solimp, sizeof(real) * 5);
    memcpy(o + 26, q->solreffriction, sizeof(real) * 2);
  }
  *nefc = k->nefc;
  for (int r = 0; r < k->nefc; ++r) {
    for (int i = 0; i < m->nv; ++i) J[r * m->nv + i] = k->J[r][i];
    efc_D[r] = k->efc_D[r]; efc_aref[r] = k->efc_aref[r]; efc_type[r] = k->efc_type[r]; efc_id[r] = k->efc_id[r];
  }
  free(k);
  return 0;
}

/* position phase of the Euler step on one world (golden-vector tests) */
int oracle_leaf_integrate(const B200Model *m, real *qpos, const real *qvel, double dt) {
  if (!check_model(m)) return 1;
  integrate_positions(m, qpos, qvel, (real)dt);
  return 0;
}

/* convex narrowphase on raw poses (golden-vector tests): geom 2 is a mesh
 * given by `vert2` (nvert2 local vertices) unless type2 is a primitive;
 * geom 1 likewise.  Returns the contact count (0 or 1). */
int oracle_leaf_convex(int type1, const real *p1, const real *R1, const real *s1, const real *vert1, int nvert1,
                       int type2, const real *p2, const real *R2, const real *s2, const real *vert2, int nvert2,
                       real margin, real tol, int iterations, int epa_iterations, real *dist, real *pos,
                       real *normal) {
  V3 origin = vload(p1);
  CShape A = {type1, v3(0, 0, 0), vload(s1), R1, vert1, nvert1, margin};
  CShape B = {type2, vsub(vload(p2), origin), vload(s2), R2, vert2, nvert2, margin};
  real full1 = 0, full2 = 0, d;
  V3 x1, x2;
  int found = 0, flags = 0; /* return: bit 0 a contact, bit 1 an EPA pool filled */
  CShape Ac = A, Bc = B;
  if (A.type == B200_GEOM_SPHERE || A.type == B200_GEOM_CAPSULE) { full1 = A.size.v[0] + R(0.5) * margin; Ac.size.v[0] = 0; Ac.margin = 0; }
  if (B.type == B200_GEOM_SPHERE || B.type == B200_GEOM_CAPSULE) { full2 = B.size.v[0] + R(0.5) * margin; Bc.size.v[0] = 0; Bc.margin = 0; }
  if (full1 + full2 > 0) {
    GjkOut r = gjk(&Ac, &Bc, tol, iterations, full1 + full2);
    if (r.separated) return 0;
    if (r.dist > tol) {
      V3 nrm = vnormalize(vsub(r.x2, r.x1));
      x1 = vadd(r.x1, vscale(nrm, full1)); x2 = vsub(r.x2, vscale(nrm, full2));
      d = r.dist - (full1 + full2); found = 1;
    }
  }
  if (!found) {
    GjkOut r = gjk(&A, &B, tol, iterations, 0);
    if (r.separated) return 0;
    if (r.dist > tol) { d = r.dist; x1 = r.x1; x2 = r.x2; }
    else {
      EpaOut e = epa(&A, &B, &r.s, tol, epa_iterations, 0);
      if (e.budget || e.horizon) flags = 2;
      if (!e.ok) { d = r.dist; x1 = r.x1; x2 = r.x2; }
      else { d = -e.depth; x1 = e.x1; x2 = e.x2; }
    }
  }
  if (!(d < 0)) return flags;
  *dist = d + margin;
  vstore(pos, vadd(vscale(vadd(x1, x2), R(0.5)), origin));
  vstore(normal, vnormalize(*dist <= margin ? vsub(x1, x2) : vsub(x2, x1)));
  return 1 | flags;
}

/* ---- Newton-piece leaves (golden-vector tests): one world's constraint rows
 * given explicitly in the reference's row layout (equality, friction loss,
 * then limit and contact rows; a contact's rows are contiguous from
 * con_adr[c], -1 for a contact without rows) and a dense mass matrix. */
typedef struct {
  int nv, nefc, ne, nf, ncon, ls_iterations;
  double impratio_invsqrt, tolerance, ls_tolerance, meaninertia;
  const real *M, *J, *D, *frictionloss, *qfrc_smooth, *search;
  const int *type, *id, *state_in, *con_dim, *con_adr;
  const real *con_friction;
  real *jaref, *qacc, *Ma, *force, *H, *alpha, *improvement;
  int *state, *ls_evals, *overflow;
} NewtonLeaf;

size_t oracle_newton_leaf_bytes(void) { return sizeof(NewtonLeaf); }

/* a model of one kinematic tree holding every dof, so that M is one block */
static int leaf_setup(const NewtonLeaf *a, B200Model *m, int *ints, Work *k) {
  int nv = a->nv;
  if (nv < 1 || nv > MAXV || a->nefc < 0 || a->nefc > MAXE || a->ncon < 0 || a->ncon > MAXC) return 1;
  memset(m, 0, sizeof(*m));
  for (int i = 0; i < nv; ++i) ints[i] = 0;
  ints[nv] = 0; ints[nv + 1] = nv; ints[nv + 2] = 0;
  m->ints = ints;
  m->off_dof_treeid = 0; m->off_tree_dofadr = nv; m->off_tree_dofnum = nv + 1; m->off_tree_madr = nv + 2;
  m->nv = nv; m->ntree = 1; m->cone = 1; m->real_bytes = (int)sizeof(real);
  m->impratio_invsqrt = a->impratio_invsqrt; m->tolerance = a->tolerance; m->ls_tolerance = a->ls_tolerance;
  m->meaninertia = a->meaninertia; m->ls_iterations = a->ls_iterations;
  k->nefc = a->nefc; k->ne = a->ne; k->nf = a->nf; k->ncon = a->ncon;
  memcpy(k->M, a->M, sizeof(real) * nv * nv);
  for (int r = 0; r < a->nefc; ++r) {
    for (int i = 0; i < nv; ++i) k->J[r][i] = a->J[(size_t)r * nv + i];
    k->efc_D[r] = a->D[r];
    k->efc_frictionloss[r] = a->frictionloss ? a->frictionloss[r] : 0;
    k->efc_type[r] = a->type[r];
    k->efc_id[r] = a->id[r];
    k->efc_jaref[r] = a->jaref[r];
    k->efc_state[r] = a->state_in ? a->state_in[r] : 0;
  }
  for (int c = 0; c < a->ncon; ++c) {
    k->con[c].dim = a->con_dim[c];
    for (int j = 0; j < 5; ++j) k->con[c].friction[j] = a->con_friction[5 * c + j];
    k->con_adr[c] = a->con_adr[c];
  }
  return 0;
}

/* row forces and states (mjwarp_constraint.cu:27-228) */
int oracle_leaf_newton_rows(const NewtonLeaf *a) {
  B200Model m;
  int ints[MAXV + 3];
  Work *k = (Work *)calloc(1, sizeof(Work));
  if (!k) return 2;
  if (leaf_setup(a, &m, ints, k)) { free(k); return 1; }
  eval_constraints(&m, k);
  for (int r = 0; r < a->nefc; ++r) { a->force[r] = k->efc_force[r]; a->state[r] = k->efc_state[r]; }
  free(k);
  return 0;
}

/* H = M + J' D J over quadratic rows + elliptic-cone curvature, from the
 * given row states (mjwarp_hessian.cu:33-212); dense nv x nv */
int oracle_leaf_newton_hessian(const NewtonLeaf *a) {
  B200Model m;
  int ints[MAXV + 3];
  Work *k = (Work *)calloc(1, sizeof(Work));
  if (!k) return 2;
  if (leaf_setup(a, &m, ints, k)) { free(k); return 1; }
  hessian(&m, k);
  memcpy(a->H, k->H, sizeof(real) * a->nv * a->nv);
  free(k);
  return 0;
}

/* one exact line search along `search` from qacc (mjwarp_linesearch.cu:80-365):
 * alpha, improvement, and qacc / Ma / jaref moved by alpha */
int oracle_leaf_newton_linesearch(const NewtonLeaf *a) {
  B200Model m;
  int ints[MAXV + 3];
  Work *k = (Work *)calloc(1, sizeof(Work));
  if (!k) return 2;
  if (leaf_setup(a, &m, ints, k)) { free(k); return 1; }
  int nv = a->nv, of = 0;
  real sd = 0;
  for (int i = 0; i < nv; ++i) {
    k->qacc[i] = a->qacc[i]; k->Ma[i] = a->Ma[i]; k->qfrc_smooth[i] = a->qfrc_smooth[i];
    k->search[i] = a->search[i]; sd += a->search[i] * a->search[i];
  }
  k->search_dot = sd;
  k->ls_evals = 0;
  linesearch(&m, k, &of);
  *a->alpha = k->alpha;
  *a->improvement = k->improvement;
  *a->ls_evals = k->ls_evals;
  *a->overflow = of;
  for (int i = 0; i < nv; ++i) { a->qacc[i] = k->qacc[i]; a->Ma[i] = k->Ma[i]; }
  for (int r = 0; r < a->nefc; ++r) a->jaref[r] = k->efc_jaref[r];
  free(k);
  return 0;
}
