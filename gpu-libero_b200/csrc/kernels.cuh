// Portions (impedance, row_params; the line-search row model Pt .. eval_shift)
// restate MuJoCo Warp's constraint and line-search formulas: Copyright 2025
// The Newton Developers, SPDX-License-Identifier: Apache-2.0 (see NOTICE).
// B200-native batched rigid-body physics step (sm_100a): device code.
// Included by inst.cu, which instantiates the kernels per precision and
// mesh support; abi.cu holds the C ABI and the launch shape.
//
// A CTA owns one or more worlds for a whole control step.  The world's state is
// loaded from HBM once, every substep of the control step runs out of shared
// memory (forward kinematics, composite-rigid-body mass matrix and factor,
// collision, constraint rows, RNE, FP64 OSC, actuation, Newton with exact line
// search, implicit-damping Euler), and state plus outputs are written back
// once.  This fuses the reference's ~40-node-per-substep CUDA graph
// (libero/libero/gpu/host/backends/cuda_fp32/runtime.py:40-56) into one launch
// per control step.  Reductions run in a fixed order, so a world's trajectory
// is bit-reproducible run to run (the reference's pooled atomics are not).
//
// Build: nvcc -gencode arch=compute_100a,code=sm_100a --fmad=true
//        --prec-div=true --prec-sqrt=true --ftz=false (the reference's
//        FP32 flags, libero/libero/gpu/cmake/MjwarpBox.cmake:15).
#pragma once
#include <cuda_runtime.h>
#include <cfloat>
#include <cstdint>
#include <cstdlib>
#include "b200phys.h"
#include "arena.cuh"
#include "math.cuh"
#include "collide.cuh"

#ifndef B200PHYS_SOURCE_ID
#define B200PHYS_SOURCE_ID "b200phys-dev"
#endif

namespace b200 {

constexpr int kSatisfied = 0, kQuadratic = 1, kLinearNeg = 2, kLinearPos = 3, kCone = 4;

// One warp owns one world: loops stride over the warp's lanes and barriers
// are warp barriers.  Worlds of a CTA meet at CTA barriers between stages.
// A world is T consecutive threads of the CTA (T = 32: one warp; T = 128:
// four warps for models whose arena leaves room for few worlds per SM).
// TID is the thread's index in its world, FOR strides a loop over the
// world's threads and SYNC() is the world's barrier (a warp barrier for
// T = 32, else the named barrier 1 + world slot).  WARP0 marks the world's
// first warp, which runs the warp-collective sections (shuffles, ballots,
// per-lane factor rows).  Every macro needs T in scope.
#define LANE ((int)(threadIdx.x & 31))
#define TID ((int)(threadIdx.x % T))
#define WARP0 (TID < 32)
#define FOR(i, n) for (int i = TID; i < (n); i += T)
#define SYNC() world_sync<T>()
template <int T> __device__ __forceinline__ void world_sync() {
  if (T == 32) __syncwarp();
  else asm volatile("bar.sync %0, %1;" ::"r"(1 + (int)(threadIdx.x / T)), "r"(T) : "memory");
}
// Barrier of G threads of a world that work apart from the rest: the whole
// world (G == T), its first warp alone (G == 32), or its other warps (named
// barrier 4 + world slot; used only by worlds of more than one warp, which
// number at most three per CTA, so the ids stay clear of the world barriers).
template <int T, int G> __device__ __forceinline__ void group_sync() {
  if (G == T) world_sync<T>();
  else if (G == 32) __syncwarp();
  else asm volatile("bar.sync %0, %1;" ::"r"(4 + (int)(threadIdx.x / T)), "r"(G) : "memory");
}

// Stage profiling (data.stage_cycles != NULL): lane 0 of each world stamps
// clock64 at stage boundaries, after a barrier.
template <int T, class R> __device__ __forceinline__ void mark(Arena<R> &A, int stage) {
  if (stage > 0 && A.iscal[10] && TID == 0) {
    const long long t = clock64();
    A.prof[stage] += t - A.prof[0];
    A.prof[0] = t;
  }
}

template <class R> __device__ __forceinline__ R warp_sum(R v) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// N sums over the world's threads in one reduction: warp shuffles, then the
// warps' partials summed in warp order; red: N * T / 32 values of scratch
template <int T, int N, class V> __device__ __forceinline__ void world_sums(V (&v)[N], V *red) {
#pragma unroll
  for (int i = 0; i < N; ++i) v[i] = warp_sum(v[i]);
  if (T == 32) return;
  SYNC();
  if (LANE == 0) {
#pragma unroll
    for (int i = 0; i < N; ++i) red[(TID >> 5) * N + i] = v[i];
  }
  SYNC();
#pragma unroll
  for (int i = 0; i < N; ++i) {
    V s = 0;
    for (int k = 0; k < T / 32; ++k) s += red[k * N + i];
    v[i] = s;
  }
}

// sum over the world's threads; red: T / 32 reals of scratch
template <int T, class R> __device__ __forceinline__ R world_sum(R v, R *red) {
  v = warp_sum(v);
  if (T == 32) return v;
  SYNC();
  if (LANE == 0) red[TID >> 5] = v;
  SYNC();
  R s = 0;
  for (int k = 0; k < T / 32; ++k) s += red[k];
  return s;
}

// M[i][j] from the per-tree dense blocks (0 across trees)
template <class R> __device__ __forceinline__ R mass_at(const Mdl<R> &M, const R *Mb, int i, int j) {
  const int t = IF(dof_treeid)[i];
  if (t != IF(dof_treeid)[j]) return R(0);
  const int a = IF(tree_dofadr)[t], n = IF(tree_dofnum)[t];
  return Mb[IF(tree_madr)[t] + (i - a) * n + (j - a)];
}

template <class R> __device__ __forceinline__ bool dof_ancestor(const Mdl<R> &M, int body, int dof) {
  return (((unsigned)IF(body_dofmask)[4 * body + (dof >> 5)]) >> (dof & 31)) & 1u;
}

// row r times a dof vector, over the row's tree segments
template <class R> __device__ __forceinline__ R jdot(const Mdl<R> &M, const Arena<R> &A, int r, const R *x) {
  const int t0 = A.row_t[2 * r], t1 = A.row_t[2 * r + 1];
  const R *row = A.J + (size_t)r * M.m.kmax_dof;
  R s = 0;
  if (t0 >= 0) {
    const int a = IF(tree_dofadr)[t0], n = IF(tree_dofnum)[t0];
    for (int i = 0; i < n; ++i) s += row[i] * x[a + i];
    row += n;
  }
  if (t1 >= 0) {
    const int a = IF(tree_dofadr)[t1], n = IF(tree_dofnum)[t1];
    for (int i = 0; i < n; ++i) s += row[i] * x[a + i];
  }
  return s;
}

// ============================================================ position stage
// forward kinematics (mjwarp_kinematics.cu:95-212 semantics): each body's
// pose relative to its parent through its joints, composed down the tree
template <class R, int T> __device__ void kinematics(const Mdl<R> &M, Arena<R> &A) {
  const B200Model &m = M.m;
  if (TID == 0) {
    A.xpos[0] = A.xpos[1] = A.xpos[2] = 0;
    A.xquat[0] = 1; A.xquat[1] = A.xquat[2] = A.xquat[3] = 0;
  }
  SYNC();
  const int *order = IF(body_order), *lstart = IF(level_start);
  if (m.nbody <= 32) {
    // one lane per body: each lane forms its body's transform relative to its
    // parent (the joints' rotations in parallel), then the tree is composed
    // by pointer jumping, ceil(log2 depth) rounds of shuffles instead of a
    // walk down every level (the same products, grouped differently)
    if (WARP0) {
      const unsigned full = 0xffffffffu;
      const int b = LANE;
      V3<R> p = v3<R>(0, 0, 0);
      Q4<R> q = {R(1), R(0), R(0), R(0)};
      int anc = 0, parent = 0;
      bool free_body = false;
      if (b > 0 && b < m.nbody) {
        const int first = IF(body_jntadr)[b], count = IF(body_jntnum)[b];
        parent = anc = IF(body_parentid)[b];
        if (count == 1 && IF(jnt_type)[first] == B200_JNT_FREE) {
          const R *qp = A.qpos + IF(jnt_qposadr)[first];
          p = v3<R>(qp[0], qp[1], qp[2]);
          q = qnormalize(Q4<R>{qp[3], qp[4], qp[5], qp[6]});
          anc = parent = 0;
          free_body = true;
          st3(A.anchor + 3 * first, p);
          st3(A.axis + 3 * first, ld3(RF(jnt_axis) + 3 * first));
        } else {
          p = ld3(RF(body_pos) + 3 * b);
          q = ldq(RF(body_quat) + 4 * b);
          for (int j = first; j < first + count; ++j) {
            const int kind = IF(jnt_type)[j], qa = IF(jnt_qposadr)[j];
            const V3<R> lpos = ld3(RF(jnt_pos) + 3 * j), lax = ld3(RF(jnt_axis) + 3 * j);
            const V3<R> anchor = qrot(lpos, q) + p, axis = qrot(lax, q);  // in the parent's frame
            if (kind == B200_JNT_BALL) {
              q = qmul(q, qnormalize(ldq(A.qpos + qa)));
              p = anchor - qrot(lpos, q);
            } else if (kind == B200_JNT_SLIDE) {
              p = p + axis * (A.qpos[qa] - RF(qpos0)[qa]);
            } else if (kind == B200_JNT_HINGE) {
              const R angle = (A.qpos[qa] - RF(qpos0)[qa]) * R(0.5);
              const R s = msin(angle), c = mcos(angle);
              q = qmul(q, Q4<R>{c, lax.x * s, lax.y * s, lax.z * s});
              p = anchor - qrot(lpos, q);
            }
            st3(A.anchor + 3 * j, anchor);
            st3(A.axis + 3 * j, axis);
          }
          q = qnormalize(q);
        }
      }
      for (int round = 0; round < 5; ++round) {
        if (!__any_sync(full, anc != 0)) break;
        const int a = anc;
        const V3<R> pa = v3<R>(__shfl_sync(full, p.x, a), __shfl_sync(full, p.y, a), __shfl_sync(full, p.z, a));
        const Q4<R> qa = {__shfl_sync(full, q.w, a), __shfl_sync(full, q.x, a), __shfl_sync(full, q.y, a),
                          __shfl_sync(full, q.z, a)};
        const int aa = __shfl_sync(full, anc, a);
        if (a != 0) {
          p = pa + qrot(p, qa);
          q = qnormalize(qmul(qa, q));
          anc = aa;
        }
      }
      // the joints' anchors and axes: the parent's world transform applied
      const V3<R> pp = v3<R>(__shfl_sync(full, p.x, parent), __shfl_sync(full, p.y, parent),
                             __shfl_sync(full, p.z, parent));
      const Q4<R> qp = {__shfl_sync(full, q.w, parent), __shfl_sync(full, q.x, parent),
                        __shfl_sync(full, q.y, parent), __shfl_sync(full, q.z, parent)};
      if (b > 0 && b < m.nbody) {
        st3(A.xpos + 3 * b, p);
        stq(A.xquat + 4 * b, q);
        if (!free_body) {
          const int first = IF(body_jntadr)[b], count = IF(body_jntnum)[b];
          for (int j = first; j < first + count; ++j) {
            st3(A.anchor + 3 * j, pp + qrot(ld3(A.anchor + 3 * j), qp));
            st3(A.axis + 3 * j, qrot(ld3(A.axis + 3 * j), qp));
          }
        }
      }
      __syncwarp();
    }
  } else if (WARP0) {  // larger trees: the world's first warp walks the levels with warp barriers
    for (int level = 1; level < m.nlevel; ++level) {
      const int a = lstart[level], n = lstart[level + 1] - a;
      for (int k = LANE; k < n; k += 32) {
        const int b = order[a + k];
        const int first = IF(body_jntadr)[b], count = IF(body_jntnum)[b], p = IF(body_parentid)[b];
        V3<R> pos;
        Q4<R> quat;
        if (count == 1 && IF(jnt_type)[first] == B200_JNT_FREE) {
          const R *q = A.qpos + IF(jnt_qposadr)[first];
          pos = v3<R>(q[0], q[1], q[2]);
          quat = qnormalize(Q4<R>{q[3], q[4], q[5], q[6]});
          st3(A.anchor + 3 * first, pos);
          st3(A.axis + 3 * first, ld3(RF(jnt_axis) + 3 * first));
        } else {
          const Q4<R> pq = ldq(A.xquat + 4 * p);
          pos = qrot(ld3(RF(body_pos) + 3 * b), pq) + ld3(A.xpos + 3 * p);
          quat = qmul(pq, ldq(RF(body_quat) + 4 * b));
          for (int j = first; j < first + count; ++j) {
            const int kind = IF(jnt_type)[j], qa = IF(jnt_qposadr)[j];
            const V3<R> lpos = ld3(RF(jnt_pos) + 3 * j), lax = ld3(RF(jnt_axis) + 3 * j);
            const V3<R> anchor = qrot(lpos, quat) + pos, axis = qrot(lax, quat);
            if (kind == B200_JNT_BALL) {
              quat = qmul(quat, qnormalize(ldq(A.qpos + qa)));
              pos = anchor - qrot(lpos, quat);
            } else if (kind == B200_JNT_SLIDE) {
              pos = pos + axis * (A.qpos[qa] - RF(qpos0)[qa]);
            } else if (kind == B200_JNT_HINGE) {
              const R angle = (A.qpos[qa] - RF(qpos0)[qa]) * R(0.5);
              const R s = msin(angle), c = mcos(angle);
              quat = qmul(quat, Q4<R>{c, lax.x * s, lax.y * s, lax.z * s});
              pos = anchor - qrot(lpos, quat);
            }
            st3(A.anchor + 3 * j, anchor);
            st3(A.axis + 3 * j, axis);
          }
          quat = qnormalize(quat);
        }
        st3(A.xpos + 3 * b, pos);
        stq(A.xquat + 4 * b, quat);
      }
      __syncwarp();
    }
  }
  SYNC();
  FOR(b, m.nbody) {
    const Q4<R> q = ldq(A.xquat + 4 * b);
    qmat(A.xmat + 9 * b, q);
    st3(A.xipos + 3 * b, ld3(A.xpos + 3 * b) + qrot(ld3(RF(body_ipos) + 3 * b), q));
    qmat(A.ximat + 9 * b, qmul(q, ldq(RF(body_iquat) + 4 * b)));
  }
  FOR(g, m.ngeom) {
    const int b = IF(geom_bodyid)[g];
    const Q4<R> q = ldq(A.xquat + 4 * b);
    st3(A.gxpos + 3 * g, ld3(A.xpos + 3 * b) + qrot(ld3(RF(geom_pos) + 3 * g), q));
    qmat(A.gxmat + 9 * g, qmul(q, ldq(RF(geom_quat) + 4 * g)));
  }
  FOR(s, m.nsite) {
    const int b = IF(site_bodyid)[s];
    const Q4<R> q = ldq(A.xquat + 4 * b);
    st3(A.sxpos + 3 * s, ld3(A.xpos + 3 * b) + qrot(ld3(RF(site_pos) + 3 * s), q));
    qmat(A.sxmat + 9 * s, qmul(q, ldq(RF(site_quat) + 4 * s)));
  }
  SYNC();
}

// subtree com, centred inertia, motion axes, CRB and the mass matrix
// (mjwarp_com_pos.cu:7-88, mjwarp_mass_matrix.cu:52-104).  Subtrees are
// contiguous body intervals, so each sum has one owner and no barrier chain.
template <class R, int T> __device__ void com_crb_mass(const Mdl<R> &M, Arena<R> &A) {
  const B200Model &m = M.m;
  const int nb = m.nbody;
  const R *mass = RF(body_mass);
  FOR(w, 3 * nb) {
    const int b = w / 3, c = w % 3;
    R s = A.xipos[3 * b + c] * mass[b];
    for (int k = b + 1; k < IF(body_subtree_end)[b]; ++k) s += A.xipos[3 * k + c] * mass[k];
    const R sm = RF(body_subtreemass)[b];
    A.com[3 * b + c] = sm != R(0) ? s / sm : s;
  }
  SYNC();
  FOR(b, nb) {
    const R *r = A.ximat + 9 * b, *in = RF(body_inertia) + 3 * b, *com = A.com + 3 * IF(body_rootid)[b];
    const R dx = A.xipos[3 * b] - com[0], dy = A.xipos[3 * b + 1] - com[1], dz = A.xipos[3 * b + 2] - com[2];
    R sc[9];
    for (int i = 0; i < 3; ++i)
      for (int j = 0; j < 3; ++j) sc[3 * i + j] = r[3 * i + j] * in[j];
    const int rows[6] = {0, 1, 2, 0, 0, 1}, cols[6] = {0, 1, 2, 1, 2, 2};
    R *o = A.cinert + 10 * b;
    const R ms = mass[b];
    for (int i = 0; i < 6; ++i) {
      const int a = 3 * rows[i], c = 3 * cols[i];
      o[i] = sc[a] * r[c] + sc[a + 1] * r[c + 1] + sc[a + 2] * r[c + 2];
    }
    o[0] += ms * (dy * dy + dz * dz); o[1] += ms * (dx * dx + dz * dz); o[2] += ms * (dx * dx + dy * dy);
    o[3] -= ms * dx * dy; o[4] -= ms * dx * dz; o[5] -= ms * dy * dz;
    o[6] = ms * dx; o[7] = ms * dy; o[8] = ms * dz; o[9] = ms;
  }
  FOR(j, m.njnt) {
    const int b = IF(jnt_bodyid)[j], kind = IF(jnt_type)[j];
    R *out = A.cdof + 6 * IF(jnt_dofadr)[j];
    const R *com = A.com + 3 * IF(body_rootid)[b];
    const R dx = com[0] - A.anchor[3 * j], dy = com[1] - A.anchor[3 * j + 1], dz = com[2] - A.anchor[3 * j + 2];
    if (kind == B200_JNT_FREE) {
      for (int a = 0; a < 3; ++a)
        for (int c = 0; c < 6; ++c) out[6 * a + c] = R(c == a + 3);
      out += 18;
    }
    if (kind == B200_JNT_FREE || kind == B200_JNT_BALL) {
      const R *r = A.xmat + 9 * b;
      for (int a = 0; a < 3; ++a) {
        const R x = r[a], y = r[3 + a], z = r[6 + a];
        R *o = out + 6 * a;
        o[0] = x; o[1] = y; o[2] = z;
        o[3] = y * dz - z * dy; o[4] = z * dx - x * dz; o[5] = x * dy - y * dx;
      }
    } else if (kind == B200_JNT_SLIDE) {
      for (int c = 0; c < 3; ++c) { out[c] = 0; out[c + 3] = A.axis[3 * j + c]; }
    } else {
      const R x = A.axis[3 * j], y = A.axis[3 * j + 1], z = A.axis[3 * j + 2];
      out[0] = x; out[1] = y; out[2] = z;
      out[3] = y * dz - z * dy; out[4] = z * dx - x * dz; out[5] = x * dy - y * dx;
    }
  }
  SYNC();
  FOR(w, 10 * nb) {
    const int b = w / 10, c = w % 10;
    R s = A.cinert[w];
    if (b > 0)
      for (int k = b + 1; k < IF(body_subtree_end)[b]; ++k) s += A.cinert[10 * k + c];
    A.crb[w] = s;
  }
  FOR(k, m.nM) A.M[k] = 0;
  SYNC();
  FOR(i, m.nv) {
    R f[6];
    inert_mul(A.crb + 10 * IF(dof_bodyid)[i], A.cdof + 6 * i, f);
    const int t = IF(dof_treeid)[i], a = IF(tree_dofadr)[t], n = IF(tree_dofnum)[t], base = IF(tree_madr)[t];
    for (int j = i; j >= 0; j = IF(dof_parentid)[j]) {
      R v = 0;
      for (int c = 0; c < 6; ++c) v += A.cdof[6 * j + c] * f[c];
      if (j == i) v = RF(dof_armature)[i] + v;
      A.M[base + (i - a) * n + (j - a)] = v;
      A.M[base + (j - a) * n + (i - a)] = v;
    }
  }
  SYNC();
}

// Block-diagonal dense factorizations.  Blocks (kinematic trees for the
// mass matrix and the implicit-damping matrix, constraint islands for the
// Newton Hessian) are dealt to the world's warps round robin; within a warp,
// lane l owns the rows q = l + 32 s (s < 4) of the concatenation of its
// blocks.  Each owned row knows its block size n, its row a inside the
// block, the block's storage base (dense n x n, row-major) and the block's
// first position in the solve vector.  A warp's blocks advance together, so
// a factorization takes as many steps as its largest block.
struct BlockRows { int n[4], a[4], base[4], start[4], rows; };
// Factor blocks are stored packed lower-triangular: entry (i, j), j <= i, of
// a block at base sits at base + i (i + 1) / 2 + j.
__device__ __forceinline__ int tri(int i, int j) { return i * (i + 1) / 2 + j; }

__device__ __forceinline__ BlockRows owned_rows(int nblocks, const int *bn, const int *bstart, const int *bbase,
                                                int lane, int wi, int nw) {
  BlockRows b;
#pragma unroll
  for (int s = 0; s < 4; ++s) { b.n[s] = 0; b.a[s] = -1; b.base[s] = 0; b.start[s] = 0; }
  int acc = 0;
  for (int k = wi; k < nblocks; k += nw) {
    const int n = bn[k];
#pragma unroll
    for (int s = 0; s < 4; ++s) {
      const int q = lane + 32 * s;
      if (q >= acc && q < acc + n) { b.n[s] = n; b.a[s] = q - acc; b.base[s] = bbase[k]; b.start[s] = bstart[k]; }
    }
    acc += n;
  }
  b.rows = acc;
  return b;
}
#define TREE_ROWS(T) owned_rows(M.m.ntree, IF(tree_dofnum), IF(tree_dofadr), IF(tree_padr), LANE, TID >> 5, (T) / 32)
#define ISLAND_ROWS(T) owned_rows(A.iscal[11], A.isl_n, A.isl_dofstart, A.isl_off, LANE, TID >> 5, (T) / 32)

// in-place lower Cholesky L L^T of a warp's blocks (right-looking)
template <class R> __device__ void chol_blocks_smem(R *H, const BlockRows &b, int maxn) {
  for (int k = 0; k < maxn; ++k) {
#pragma unroll
    for (int s = 0; s < 4; ++s)
      if (b.n[s] > k && b.a[s] == k) H[b.base[s] + tri(k, k)] = msqrt(H[b.base[s] + tri(k, k)]);
    __syncwarp();
#pragma unroll
    for (int s = 0; s < 4; ++s)
      if (b.n[s] > k && b.a[s] > k) H[b.base[s] + tri(b.a[s], k)] /= H[b.base[s] + tri(k, k)];
    __syncwarp();
#pragma unroll
    for (int s = 0; s < 4; ++s)
      if (b.n[s] > k && b.a[s] > k) {
        R *row = H + b.base[s] + tri(b.a[s], 0);
        const R l = row[k];
        for (int j = k + 1; j <= b.a[s]; ++j) row[j] -= l * H[b.base[s] + tri(j, k)];
      }
    __syncwarp();
  }
}

// Register-row variant for nv <= 32 (one row per lane): lane keeps its row of
// the block in registers; the scaled column k is broadcast through a
// double-buffered shared column, so each step costs one __syncwarp.  The
// factor is written back to H (lower triangle, diagonal = pivots) for the
// triangular solves.
template <class R, int MAXN>
__device__ void chol_blocks_reg(R *H, const BlockRows &b, int maxn, R *colbuf, int stride) {
  const int n = b.n[0], a = b.a[0];
  R row[MAXN];
#pragma unroll
  for (int j = 0; j < MAXN; ++j) row[j] = (n > 0 && j <= a && j < n) ? H[b.base[0] + tri(a, j)] : R(0);
  for (int k = 0; k < maxn; ++k) {
    R *col = colbuf + (k & 1) * stride;
    R rk = 0;
#pragma unroll
    for (int j = 0; j < MAXN; ++j)
      if (j == k) rk = row[j];
    if (n > k && a == k) {
      const R d = msqrt(rk);
      col[b.start[0] + k] = R(1) / d;  // the pivot's reciprocal, read by the rows below
#pragma unroll
      for (int j = 0; j < MAXN; ++j)
        if (j == k) row[j] = d;
    }
    __syncwarp();
    if (n > k && a > k) {
      const R l = rk * col[b.start[0] + k];
      col[b.start[0] + a] = l;
#pragma unroll
      for (int j = 0; j < MAXN; ++j)
        if (j == k) row[j] = l;
    }
    __syncwarp();
    if (n > k && a > k) {
      const R l = col[b.start[0] + a];
#pragma unroll
      for (int j = 0; j < MAXN; ++j)
        if (j > k && j <= a) row[j] -= l * col[b.start[0] + j];
    }
  }
  if (n > 0) {
#pragma unroll
    for (int j = 0; j < MAXN; ++j)
      if (j <= a && j < n) H[b.base[0] + tri(a, j)] = row[j];
  }
  __syncwarp();
}

// Factor (optional) and solve L L^T x = x of a warp's blocks when each lane
// owns at most one row (b.rows <= 32, blocks of at most MAXN): the lane's
// row of L stays in registers, so the substitutions exchange the solved
// entries by shuffles instead of shared memory and warp barriers.  Each
// pivot's reciprocal is formed once, so the serial chains multiply instead
// of divide.  xin: the lane's entry of the right-hand side; returns its
// entry of the solution.
template <class R, int MAXN>
__device__ R chol_solve_reg(R *H, const BlockRows &b, int maxn, R *colbuf, int stride, bool factor, R xin) {
  const int n = b.n[0], a = b.a[0], lane = LANE;
  const unsigned full = 0xffffffffu;
  R row[MAXN];
#pragma unroll
  for (int j = 0; j < MAXN; ++j) row[j] = (n > 0 && j <= a && j < n) ? H[b.base[0] + tri(a, j)] : R(0);
  R rinv = 0;  // 1 / the pivot of the lane's row
  if (factor) {
    for (int k = 0; k < maxn; ++k) {
      R *col = colbuf + (k & 1) * stride;
      R rk = 0;
#pragma unroll
      for (int j = 0; j < MAXN; ++j)
        if (j == k) rk = row[j];
      if (n > k && a == k) {
        const R d = msqrt(rk);
        rinv = R(1) / d;
        col[b.start[0] + k] = rinv;
#pragma unroll
        for (int j = 0; j < MAXN; ++j)
          if (j == k) row[j] = d;
      }
      __syncwarp();
      if (n > k && a > k) {
        const R l = rk * col[b.start[0] + k];
        col[b.start[0] + a] = l;
#pragma unroll
        for (int j = 0; j < MAXN; ++j)
          if (j == k) row[j] = l;
      }
      __syncwarp();
      if (n > k && a > k) {
        const R l = col[b.start[0] + a];
#pragma unroll
        for (int j = 0; j < MAXN; ++j)
          if (j > k && j <= a) row[j] -= l * col[b.start[0] + j];
      }
    }
    if (n > 0) {
#pragma unroll
      for (int j = 0; j < MAXN; ++j)
        if (j <= a && j < n) H[b.base[0] + tri(a, j)] = row[j];
    }
  }
  else if (n > 0) {
#pragma unroll
    for (int j = 0; j < MAXN; ++j)
      if (j == a) rinv = R(1) / row[j];
  }
  R x = xin;
  // forward: L y = x
#pragma unroll
  for (int k = 0; k < MAXN; ++k) {
    if (k >= maxn) break;
    if (n > k && a == k) x *= rinv;
    const R xk = __shfl_sync(full, x, (lane - a + k) & 31);
    if (n > k && a > k) x -= row[k] * xk;
  }
  // backward: L^T x = y; column entries of L come from shared memory
#pragma unroll
  for (int k = MAXN - 1; k >= 0; --k) {
    if (k >= maxn) continue;
    const R lka = (n > k && a < k) ? H[b.base[0] + tri(k, a)] : R(0);
    if (n > k && a == k) x *= rinv;
    const R xk = __shfl_sync(full, x, (lane - a + k) & 31);
    if (n > k && a < k) x -= lka * xk;
  }
  __syncwarp();
  return x;
}

// colbuf: 2 x nv reals (the register variant's double-buffered column, indexed by position)
template <class R> __device__ void chol_blocks(R *H, const BlockRows &b, int maxn, int nv, R *colbuf) {
  if (b.rows <= 32 && maxn <= 16) chol_blocks_reg<R, 16>(H, b, maxn, colbuf, nv);
  else chol_blocks_smem(H, b, maxn);
}

// solve L L^T x = x in place over a warp's blocks (x indexed by position)
template <class R> __device__ void solve_blocks(const R *H, const BlockRows &b, R *x, int maxn, int lane) {
  for (int k = 0; k < maxn; ++k) {
#pragma unroll
    for (int s = 0; s < 4; ++s)
      if (b.n[s] > k && b.a[s] == k) x[b.start[s] + b.a[s]] /= H[b.base[s] + tri(k, k)];
    __syncwarp();
#pragma unroll
    for (int s = 0; s < 4; ++s)
      if (b.n[s] > k && b.a[s] > k) x[b.start[s] + b.a[s]] -= H[b.base[s] + tri(b.a[s], k)] * x[b.start[s] + k];
    __syncwarp();
  }
  for (int k = maxn - 1; k >= 0; --k) {
#pragma unroll
    for (int s = 0; s < 4; ++s)
      if (b.n[s] > k && b.a[s] == k) x[b.start[s] + b.a[s]] /= H[b.base[s] + tri(k, k)];
    __syncwarp();
#pragma unroll
    for (int s = 0; s < 4; ++s)
      if (b.n[s] > k && b.a[s] < k) x[b.start[s] + b.a[s]] -= H[b.base[s] + tri(k, b.a[s])] * x[b.start[s] + k];
    __syncwarp();
  }
}

// L L^T x = x over the kinematic-tree blocks (positions are dofs), factoring
// first when `factor`; registers and shuffles when each lane owns at most one row
// (the world's warps [W0, W0 + NW) take the trees; by default all of them)
template <class R, int T, int W0 = 0, int NW = T / 32>
__device__ void tree_solve(const Mdl<R> &M, R *L, R *x, R *colbuf, bool factor) {
  const BlockRows b = owned_rows(M.m.ntree, IF(tree_dofnum), IF(tree_dofadr), IF(tree_padr), LANE, (TID >> 5) - W0, NW);
  const int maxn = M.m.max_tree_dofs;
  if (b.rows <= 32 && maxn <= 16) {
    const int p = b.start[0] + b.a[0];
    const R v = chol_solve_reg<R, 16>(L, b, maxn, colbuf, M.m.nv, factor, b.n[0] > 0 ? x[p] : R(0));
    if (b.n[0] > 0) x[p] = v;
    __syncwarp();
    return;
  }
  if (factor) chol_blocks_smem(L, b, maxn);
  solve_blocks(L, b, x, maxn, LANE);
}

// lower triangles of the dense tree blocks of M into packed blocks at tree_padr
// (tree_lsrc: each packed entry's index in the dense blocks, from the host)
template <class R, int T> __device__ void pack_tree_blocks(const Mdl<R> &M, const R *Mb, R *P) {
  FOR(e, M.m.nL) P[e] = Mb[IF(tree_lsrc)[e]];
}

// y = M x with the dense tree blocks (one thread per dof)
template <class R, int T> __device__ void mass_mul(const Mdl<R> &M, const R *Mb, const R *x, R *y) {
  FOR(i, M.m.nv) {
    const int t = IF(dof_treeid)[i], a = IF(tree_dofadr)[t], n = IF(tree_dofnum)[t];
    const R *row = Mb + IF(tree_madr)[t] + (i - a) * n;
    R s = 0;
    for (int j = 0; j < n; ++j) s += row[j] * x[a + j];
    y[i] = s;
  }
}

// ============================================================ collision
// CONVEX: the kernel variant for models with mesh geoms (plane-mesh and the
// GJK/EPA pairs); models without meshes run the smaller variant.  The G
// threads [G0, G0 + G) of the world run it; their pair lists start
// list_offset bytes into the stage-scoped union region.
template <class R, int T, int CONVEX, int G0, int G>
__device__ void collision(const Mdl<R> &M, Arena<R> &A, int list_offset) {
  const B200Model &m = M.m;
  const int gt = TID - G0;
  // Broadphase first, then the narrowphase over the surviving pairs grouped
  // by family, so that the threads of a warp run the same collider.  Contact
  // order is fixed by the key sort below, not by the order in which pairs are
  // processed.
  constexpr int kFam = 5;
  int *fam = (int *)((unsigned char *)A.H + list_offset), *cnt = fam + m.npair, *fill = cnt + kFam,
      *list = fill + kFam;
  const bool grouped = list_offset + (2 * m.npair + 2 * kFam) * (int)sizeof(int) <= A.ubytes;
  if (gt == 0) A.iscal[8] = A.iscal[25] = 0;
  if (grouped && gt < 2 * kFam) cnt[gt] = 0;
  group_sync<T, G>();
  if (!(m.disable_flags & (B200_DSBL_CONSTRAINT | B200_DSBL_CONTACT))) {
    if (grouped) {
      for (int p = gt; p < m.npair; p += G) {
        const int f = pair_family<R, CONVEX>(M, A, p);
        fam[p] = f;
        if (f >= 0) atomicAdd(&cnt[f], 1);
      }
      group_sync<T, G>();
      if (gt == 0) A.iscal[25] = cnt[4];  // GJK / EPA pairs, for the world's work estimate
      int off[kFam], total = 0;
      for (int f = 0; f < kFam; ++f) { off[f] = total; total += cnt[f]; }
      for (int p = gt; p < m.npair; p += G) {
        const int f = fam[p];
        if (f >= 0) list[off[f] + atomicAdd(&fill[f], 1)] = p;
      }
      group_sync<T, G>();
      // families dealt to the group's warps, convex pairs (GJK / EPA, the
      // slowest) alone on one, so that a warp runs one or two collider code
      // paths instead of all of them
      constexpr int nw = G / 32;
      constexpr int kFamWarp4[kFam] = {3, 1, 3, 2, 0}, kFamWarp3[kFam] = {1, 2, 1, 2, 0};
      const int wid = gt / 32;
      for (int f = 0; f < kFam; ++f) {
        const int owner = nw == 3 ? kFamWarp3[f] : kFamWarp4[f] % nw;
        if (owner == wid)
          for (int i = LANE; i < cnt[f]; i += 32) narrow_pair<R, CONVEX>(M, A, list[off[f] + i], f);
      }
    } else {
      for (int p = gt; p < m.npair; p += G) {
        const int f = pair_family<R, CONVEX>(M, A, p);
        if (f >= 0) narrow_pair<R, CONVEX>(M, A, p, f);
      }
    }
  }
  group_sync<T, G>();
  const int n = mmin(A.iscal[8], m.ncon_max);
  // deterministic order: rank of each contact's (pair, id) key
  for (int c = gt; c < n; c += G) {
    const int key = A.con_key[c];
    int rank = 0;
    for (int k = 0; k < n; ++k) rank += A.con_key[k] < key;
    A.con_order[rank] = c;
  }
  if (gt == 0) A.iscal[0] = n;
  group_sync<T, G>();
}

// ============================================================ constraints
// mjwarp_constraint_build.cu:24-196
// a^b with exact products for the small integer exponents solimp uses
// (MuJoCo's default power is 2); general exponents call pow
template <class R> __device__ __forceinline__ R ipow(R a, R b) {
  if (b == R(1)) return a;
  if (b == R(2)) return a * a;
  if (b == R(3)) return a * a * a;
  return mpow(a, b);
}

template <class R> struct KBI { R k, b, imp; };
template <class R> __device__ KBI<R> impedance(const B200Model &m, const R *ref, const R *imp, R position) {
  const R minval = R(1e-15), minimp = R(0.0001), maximp = R(0.9999);
  const bool refsafe = !(m.disable_flags & B200_DSBL_REFSAFE);
  const R ts = R(m.timestep);
  const R time = refsafe ? mmax(ref[0], R(2) * ts) : ref[0];
  const R lo = mclamp(imp[0], minimp, maximp), hi = mclamp(imp[1], minimp, maximp);
  const R width = mmax(minval, imp[2]), mid = mclamp(imp[3], minimp, maximp), power = mmax(R(1), imp[4]);
  KBI<R> o;
  o.k = ref[0] <= R(0) ? -ref[0] / mmax(minval, hi * hi) : R(1) / mmax(minval, hi * hi * time * time * ref[1] * ref[1]);
  o.b = ref[1] <= R(0) ? -ref[1] / mmax(minval, hi) : R(2) / mmax(minval, hi * time);
  const R x = mabs(position) / width;
  if (lo == hi || imp[2] <= minval) o.imp = R(0.5) * (lo + hi);
  else if (x <= R(0)) o.imp = lo;
  else if (x >= R(1)) o.imp = hi;
  else if (power == R(1)) o.imp = lo + x * (hi - lo);
  else if (x <= mid) o.imp = mclamp(lo + (R(1) / ipow(mid, power - R(1))) * ipow(x, power) * (hi - lo), lo, hi);
  else o.imp = mclamp(lo + (R(1) - (R(1) / ipow(R(1) - mid, power - R(1))) * ipow(R(1) - x, power)) * (hi - lo), lo, hi);
  return o;
}

template <class R>
__device__ void row_params(const B200Model &m, Arena<R> &A, int r, R pos, R imp_pos, R weight, const R *ref,
                           const R *imp, R velocity, R friction, int type, int id) {
  const KBI<R> kbi = impedance(m, ref, imp, imp_pos);
  const R k = type == 1 ? R(0) : kbi.k;
  A.efc_D[r] = R(1) / mmax(weight * (R(1) - kbi.imp) / kbi.imp, R(1e-15));
  A.efc_aref[r] = -k * kbi.imp * pos - kbi.b * velocity;
  A.efc_floss[r] = friction;
  A.efc_type[r] = type;
  A.efc_id[r] = id;
}

template <class R> __device__ __forceinline__ void set_row_trees(const Mdl<R> &M, Arena<R> &A, int r, int ta, int tb) {
  if (ta < 0) { ta = tb; tb = -1; }
  if (tb == ta) tb = -1;
  A.row_t[2 * r] = ta;
  A.row_t[2 * r + 1] = tb;
}

// Islands: kinematic trees coupled by a two-tree constraint row share one
// Newton Hessian block.  Warp 0.  Without coupling rows every tree is its own
// island and the tree layout is reused (packed blocks at tree_padr).
// Otherwise the coupled contacts join trees into components, numbered by
// their smallest tree index, so the blocks are deterministic.
template <class R> __device__ void islands(const Mdl<R> &M, Arena<R> &A, bool coupled) {
  const int nt = M.m.ntree, nv = M.m.nv, lane = LANE;
  if (!coupled) {
    for (int t = lane; t < nt; t += 32) {
      A.tree_isl[t] = t;
      A.isl_n[t] = IF(tree_dofnum)[t];
      A.isl_off[t] = IF(tree_padr)[t];
      A.isl_dofstart[t] = IF(tree_dofadr)[t];
    }
    if (lane == 0) { A.isl_dofstart[nt] = nv; A.iscal[11] = nt; A.iscal[12] = M.m.max_tree_dofs; }
    for (int d = lane; d < nv; d += 32) {
      A.isl_dof[d] = d;
      A.dof_isl[d] = IF(dof_treeid)[d];
      A.dof_loc[d] = d - IF(tree_dofadr)[IF(dof_treeid)[d]];
    }
    __syncwarp();
    return;
  }
  // lane t < nt: tree t.  Adjacency masks from the contacts that couple two
  // trees, then components by merging neighbours' masks until stable (each
  // round doubles the path length covered); a component's root is its
  // smallest tree, and islands are numbered in root order.
  const unsigned full = 0xffffffffu;
  const int ncon = A.iscal[0];
  unsigned adj = lane < nt ? 1u << lane : 0u;
  for (int base = 0; base < ncon; base += 32) {
    const int k = base + lane;
    int ta = -1, tb = -1;
    if (k < ncon) {
      const int r0 = A.con_adr[A.con_order[k]];
      if (r0 >= 0) { ta = A.row_t[2 * r0]; tb = A.row_t[2 * r0 + 1]; }
    }
    unsigned pending = __ballot_sync(full, tb >= 0);
    while (pending) {
      const int src = __ffs(pending) - 1;
      pending &= pending - 1u;
      const int a = __shfl_sync(full, ta, src), bb = __shfl_sync(full, tb, src);
      if (lane == a) adj |= 1u << bb;
      if (lane == bb) adj |= 1u << a;
    }
  }
  unsigned comp = adj;
  for (bool grew = true; grew;) {
    unsigned merged = comp;
    for (int u = 0; u < nt; ++u) {
      const unsigned mu = __shfl_sync(full, comp, u);
      if ((comp >> u) & 1u) merged |= mu;
    }
    grew = __any_sync(full, merged != comp);
    comp = merged;
  }
  const int dn = lane < nt ? IF(tree_dofnum)[lane] : 0, root = lane < nt ? __ffs(comp) - 1 : 0;
  const unsigned roots = __ballot_sync(full, lane < nt && root == lane);
  int n = 0;  // dofs of the component (meaningful at its root)
  for (int u = 0; u < nt; ++u) {
    const int v = __shfl_sync(full, dn, u);
    if ((comp >> u) & 1u) n += v;
  }
  const bool is_root = (roots >> lane) & 1u;
  int at = is_root ? n : 0, off = is_root ? n * (n + 1) / 2 : 0;
  for (int o = 1; o < 32; o <<= 1) {  // inclusive scans over the roots in tree order
    const int x = __shfl_up_sync(full, at, o), y = __shfl_up_sync(full, off, o);
    if (lane >= o) { at += x; off += y; }
  }
  const int isl = __popc(roots & ((1u << root) - 1u));
  if (lane < nt) A.tree_isl[lane] = isl;
  if (is_root) {
    A.isl_n[isl] = n;
    A.isl_dofstart[isl] = at - n;
    A.isl_off[isl] = off - n * (n + 1) / 2;
  }
  const int maxn = __reduce_max_sync(full, is_root ? n : 0);
  if (lane == 0) {
    const int nisl = __popc(roots);
    A.isl_dofstart[nisl] = nv;
    A.iscal[11] = nisl;
    A.iscal[12] = maxn;
  }
  __syncwarp();
  for (int d = lane; d < nv; d += 32) {
    const int t = IF(dof_treeid)[d], isl = A.tree_isl[t];
    int pos = d - IF(tree_dofadr)[t];
    for (int u = 0; u < t; ++u)
      if (A.tree_isl[u] == isl) pos += IF(tree_dofnum)[u];
    A.isl_dof[A.isl_dofstart[isl] + pos] = d;
    A.dof_isl[d] = isl;
    A.dof_loc[d] = pos;
  }
  __syncwarp();
}

// Per-tree segment lists (warp 0, after row allocation): a segment is one
// single-dof row or one contact's rows; each goes to the list of every tree
// it acts on, in ascending row order.  Segments are taken 32 at a time, one
// per lane (the single-dof rows, then the contacts in their sorted order,
// which is their row order); per tree present in the chunk a ballot selects
// its segments, and lane t keeps tree t's running count (first pass) or
// write position (second pass).
template <class R> __device__ void tree_segments(const Mdl<R> &M, Arena<R> &A, int nsingle, int ncon) {
  const int nt = M.m.ntree, lane = LANE, items = nsingle + ncon;
  const unsigned full = 0xffffffffu, below = (1u << lane) - 1u;
  int mine = 0;  // lane t < nt: tree t's segment count, then its write position
  for (int pass = 0; pass < 2; ++pass) {
    if (pass == 1) {
      int incl = mine;
      for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(full, incl, o);
        if (lane >= o) incl += v;
      }
      const int total = __shfl_sync(full, incl, 31);
      mine = incl - mine;
      if (lane < nt) A.tree_segadr[lane] = mine;
      if (lane == 0) A.tree_segadr[nt] = total;
    }
    for (int base = 0; base < items; base += 32) {
      const int i = base + lane;
      int t0 = -1, t1 = -1;
      unsigned code = 0, col1 = 0;
      if (i < items) {
        int r = i, len = i < nsingle ? 1 : 0;
        if (!len) {
          const int c = A.con_order[i - nsingle];
          r = A.con_adr[c];
          if (r >= 0) len = A.efc_type[r] == 6 ? 2 * (A.con_dim[c] - 1) : A.con_dim[c];
        }
        if (len) {
          t0 = A.row_t[2 * r];
          t1 = A.row_t[2 * r + 1];
          code = (unsigned)r | (unsigned)len << 16;
          col1 = (unsigned)IF(tree_dofnum)[t0] << 24;
        }
      }
      unsigned present = __reduce_or_sync(full, (t0 >= 0 ? 1u << t0 : 0u) | (t1 >= 0 ? 1u << t1 : 0u));
      while (present) {
        const int t = __ffs(present) - 1;
        present &= present - 1u;
        const unsigned m0 = __ballot_sync(full, t0 == t), m1 = __ballot_sync(full, t1 == t), mm = m0 | m1;
        if (pass == 1) {
          const int pos = __shfl_sync(full, mine, t) + __popc(mm & below);
          if ((mm >> lane) & 1u) A.tree_seg[pos] = code | ((m1 >> lane) & 1u ? col1 : 0u);
        }
        if (lane == t) mine += __popc(mm);
      }
    }
  }
  __syncwarp();
}

template <class R, int T, int G0 = 0, int G = T> __device__ void actuation(const Mdl<R> &M, Arena<R> &A);

// ACT: the world's other warps run the actuation stage while its first warp
// allocates the rows (worlds of more than one warp)
template <class R, int T, bool ACT = false> __device__ void constraints(const Mdl<R> &M, Arena<R> &A) {
  const B200Model &m = M.m;
  const int cap = m.nefc_max, kmax = m.kmax_dof;
  const bool off = m.disable_flags & B200_DSBL_CONSTRAINT;
  const bool elliptic = m.cone == 1;
  // row allocation (the world's first warp): friction rows, active limits, then contacts in
  // sorted order, each contact all-or-nothing; prefix sums by warp scans
  if (WARP0) {
    const int lane = LANE;
    const unsigned below = (1u << lane) - 1u;
    int of = 0;
    const int nf = (!off && !(m.disable_flags & B200_DSBL_FRICTIONLOSS)) ? mmin(m.nfric, cap) : 0;
    if (!off && !(m.disable_flags & B200_DSBL_FRICTIONLOSS) && m.nfric > cap) of |= B200_OVERFLOW_NEFC;
    for (int k = lane; k < nf; k += 32) {
      A.efc_type[k] = 1;
      A.efc_id[k] = IF(fric_dof)[k];
      set_row_trees(M, A, k, IF(dof_treeid)[IF(fric_dof)[k]], -1);
    }
    int nefc = nf;
    const bool limits = !off && !(m.disable_flags & B200_DSBL_LIMIT);
    for (int base = 0; base < m.nlimited; base += 32) {
      const int k = base + lane;
      bool active = false;
      int j = -1;
      if (limits && k < m.nlimited) {
        j = IF(limited_jnt)[k];
        const R *range = RF(jnt_range) + 2 * j;
        const R q = A.qpos[IF(jnt_qposadr)[j]];
        active = mmin(q - range[0], range[1] - q) - RF(jnt_margin)[j] < R(0);
      }
      const unsigned mask = __ballot_sync(0xffffffffu, active);
      const int r = nefc + __popc(mask & below);
      if (active) {
        if (r < cap) {
          A.efc_type[r] = 3;
          A.efc_id[r] = j;
          set_row_trees(M, A, r, IF(dof_treeid)[IF(jnt_dofadr)[j]], -1);
        } else of |= B200_OVERFLOW_NEFC;
      }
      nefc = mmin(nefc + __popc(mask), cap);
    }
    const int ncon = A.iscal[0];
    if (lane == 0) A.iscal[13] = nefc;  // rows [0, nefc) act on one dof each
    int end = nefc;
    bool coupled = false;
    for (int base = 0; base < ncon; base += 32) {
      const int k = base + lane;
      int count = 0, c = -1;
      if (k < ncon) {
        c = A.con_order[k];
        A.con_adr[c] = -1;
        const R *cr = A.con + (size_t)c * kCWidth;
        if (!off && !(m.disable_flags & B200_DSBL_CONTACT) && cr[kCDist] - cr[kCMargin] < R(0)) {
          const int dim = A.con_dim[c];
          count = elliptic || dim == 1 ? dim : 2 * (dim - 1);
        }
      }
      int incl = count;
      for (int o = 1; o < 32; o <<= 1) {
        const int t = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += t;
      }
      const int r0 = nefc + incl - count;
      if (count) {
        if (r0 + count <= cap) {
          A.con_adr[c] = r0;
          const int type = A.con_dim[c] == 1 ? 5 : (elliptic ? 7 : 6);
          int ta = IF(body_treeid)[IF(geom_bodyid)[A.con_g1[c]]], tb = IF(body_treeid)[IF(geom_bodyid)[A.con_g2[c]]];
          if (ta < 0) { ta = tb; tb = -1; }
          if (tb == ta) tb = -1;
          coupled |= tb >= 0;
          for (int i = 0; i < count; ++i) {
            A.efc_type[r0 + i] = type;
            A.efc_id[r0 + i] = c;
            A.row_t[2 * (r0 + i)] = ta;
            A.row_t[2 * (r0 + i) + 1] = tb;
          }
          end = mmax(end, r0 + count);
        } else of |= B200_OVERFLOW_NEFC;
      }
      nefc += __shfl_sync(0xffffffffu, incl, 31);
    }
    end = __reduce_max_sync(0xffffffffu, end);
    of = __reduce_or_sync(0xffffffffu, of);
    coupled = __any_sync(0xffffffffu, coupled);
    if (lane == 0) {
      A.iscal[1] = end;
      A.iscal[2] = nf;
      A.iscal[3] |= of;
    }
    __syncwarp();
    islands(M, A, coupled);
    tree_segments(M, A, A.iscal[13], ncon);
  } else if constexpr (ACT) {
    actuation<R, T, 32, T - 32>(M, A);
  }
  SYNC();
  const int nefc = A.iscal[1];
  // Jacobian rows over the rows' tree segments.  The single-dof rows (friction,
  // limits: rows [0, nsingle)) take one (row, slot) per thread; the contacts
  // one (contact, slot) per thread, which forms the contact point's Jacobian at
  // the slot's dof once and projects it on every row of the contact.
  const int nsingle = A.iscal[13], ncon = A.iscal[0];
  FOR(w, nsingle * kmax) {
    const int r = w / kmax, k = w % kmax, t0 = A.row_t[2 * r];
    R v = 0;
    if (t0 >= 0 && k < IF(tree_dofnum)[t0]) {
      const int d = IF(tree_dofadr)[t0] + k;
      if (A.efc_type[r] == 1) v = R(d == A.efc_id[r]);
      else {
        const int j = A.efc_id[r];
        if (d == IF(jnt_dofadr)[j]) {
          const R *range = RF(jnt_range) + 2 * j;
          const R q = A.qpos[IF(jnt_qposadr)[j]];
          v = R((q - range[0]) < (range[1] - q)) * R(2) - R(1);
        }
      }
    }
    A.J[(size_t)r * kmax + k] = v;
  }
  FOR(w, ncon * kmax) {
    const int c = w / kmax, k = w % kmax, r0 = A.con_adr[c];
    if (r0 < 0) continue;
    const int dim = A.con_dim[c], count = elliptic || dim == 1 ? dim : 2 * (dim - 1);
    const int t0 = A.row_t[2 * r0], t1 = A.row_t[2 * r0 + 1];
    const int n0 = t0 >= 0 ? IF(tree_dofnum)[t0] : 0, n1 = t1 >= 0 ? IF(tree_dofnum)[t1] : 0;
    const R *cr = A.con + (size_t)c * kCWidth;
    V3<R> l = v3<R>(0, 0, 0), a = v3<R>(0, 0, 0);
    bool hit = false;
    if (k < n0 + n1) {
      const int d = k < n0 ? IF(tree_dofadr)[t0] + k : IF(tree_dofadr)[t1] + k - n0;
      const int b1 = IF(geom_bodyid)[A.con_g1[c]], b2 = IF(geom_bodyid)[A.con_g2[c]];
      const bool in1 = dof_ancestor(M, b1, d), in2 = dof_ancestor(M, b2, d);
      hit = in1 || in2;
      if (hit) {
        const V3<R> point = ld3(cr + kCPos);
        const R *mo = A.cdof + 6 * d;
        const V3<R> ang = v3<R>(mo[0], mo[1], mo[2]), lin = v3<R>(mo[3], mo[4], mo[5]);
        if (in2) {
          l = lin + cross(ang, point - ld3(A.com + 3 * IF(body_rootid)[b2]));
          a = ang;
        }
        if (in1) {
          l = l - (lin + cross(ang, point - ld3(A.com + 3 * IF(body_rootid)[b1])));
          a = a - ang;
        }
      }
    }
    R *Jc = A.J + (size_t)r0 * kmax + k;
    for (int comp = 0; comp < count; ++comp) {
      R v = 0;
      if (hit) {
        if (elliptic) v = dot(comp < 3 ? l : a, ld3(cr + kCFrame + 3 * (comp % 3)));
        else {
          v = dot(l, ld3(cr + kCFrame));
          if (dim > 1) {
            const int dir = comp / 2 + 1;
            const R fr = cr[kCFriction + dir - 1] * (R(1) - R(2) * R(comp & 1));
            v += dot(dir < 3 ? l : a, ld3(cr + kCFrame + 3 * (dir % 3))) * fr;
          }
        }
      }
      Jc[(size_t)comp * kmax] = v;
    }
  }
  SYNC();
  // row parameters (impedance, D, aref); sum of row widths for the FLOP counters
  int ksum = 0, k2sum = 0;
  FOR(r, nefc) {
    {
      const int t0 = A.row_t[2 * r], t1 = A.row_t[2 * r + 1];
      const int k = (t0 >= 0 ? IF(tree_dofnum)[t0] : 0) + (t1 >= 0 ? IF(tree_dofnum)[t1] : 0);
      ksum += k;
      k2sum += k * k;
    }
    const int type = A.efc_type[r];
    const R jqv = jdot(M, A, r, A.qvel);
    if (type == 1) {
      const int d = A.efc_id[r];
      row_params(m, A, r, R(0), R(0), RF(dof_invweight0)[d], RF(dof_solref) + 2 * d, RF(dof_solimp) + 5 * d,
                 A.qvel[d], RF(dof_frictionloss)[d], 1, d);
    } else if (type == 3) {
      const int j = A.efc_id[r], d = IF(jnt_dofadr)[j];
      const R *range = RF(jnt_range) + 2 * j;
      const R q = A.qpos[IF(jnt_qposadr)[j]];
      const R pos = mmin(q - range[0], range[1] - q) - RF(jnt_margin)[j];
      const R sign = R((q - range[0]) < (range[1] - q)) * R(2) - R(1);
      row_params(m, A, r, pos, pos, RF(dof_invweight0)[d], RF(jnt_solref) + 2 * j, RF(jnt_solimp) + 5 * j,
                 sign * A.qvel[d], R(0), 3, j);
    } else {
      const int c = A.efc_id[r], comp = r - A.con_adr[c], dim = A.con_dim[c];
      const R *cr = A.con + (size_t)c * kCWidth;
      const int b1 = IF(geom_bodyid)[A.con_g1[c]], b2 = IF(geom_bodyid)[A.con_g2[c]];
      R weight = RF(body_invweight0)[2 * b1] + RF(body_invweight0)[2 * b2];
      const R ratio = R(m.impratio_invsqrt), position = cr[kCDist] - cr[kCMargin];
      const R *fr = cr + kCFriction;
      R scale = 1, pos_aref = position;
      if (elliptic && comp > 0) {
        scale = ratio * ratio;
        if (comp > 1) scale *= fr[0] * fr[0] / (fr[comp - 1] * fr[comp - 1]);
        pos_aref = 0;
      } else if (!elliptic && dim > 1) {
        weight = weight + fr[0] * fr[0] * weight;
        weight = weight * R(2) * fr[0] * fr[0] * ratio * ratio;
      }
      // solref / solimp are recomputed from the geom pair (mjwarp_contact.cuh:60-98 mixing)
      // rather than stored per contact
      const Material<R> mat = material(M, A.con_g1[c], A.con_g2[c]);
      row_params(m, A, r, pos_aref, position, weight, mat.solref, mat.solimp, jqv, R(0), type, c);
      if (elliptic && comp > 0) {
        A.efc_D[r] /= scale;
        const R *ref = mat.solref;
        if (mat.solreffriction[0] != R(0) || mat.solreffriction[1] != R(0)) ref = mat.solreffriction;
        A.efc_aref[r] = -impedance(m, ref, mat.solimp, position).b * jqv;
      }
    }
  }
  int ks[2] = {ksum, k2sum};
  world_sums<T>(ks, (int *)A.red);
  if (TID == 0) { A.iscal[15] = ks[0]; A.iscal[23] = ks[1]; }
  SYNC();
}

// ============================================================ velocity stage
// fused_motion.cu (cvel, cdof_dot, RNE bias), mjwarp_passive.cu, transmission
template <class R> __device__ __forceinline__ void motion_cross(const R *v, const R *u, R *o) {
  o[0] = -v[2] * u[1] + v[1] * u[2];
  o[1] = v[2] * u[0] - v[0] * u[2];
  o[2] = -v[1] * u[0] + v[0] * u[1];
  o[3] = -v[2] * u[4] + v[1] * u[5] - v[5] * u[1] + v[4] * u[2];
  o[4] = v[2] * u[3] - v[0] * u[5] + v[5] * u[0] - v[3] * u[2];
  o[5] = -v[1] * u[3] + v[0] * u[4] - v[4] * u[0] + v[3] * u[1];
}
template <class R> __device__ __forceinline__ void force_cross(const R *v, const R *f, R *o) {
  o[0] = -v[2] * f[1] + v[1] * f[2] - v[5] * f[4] + v[4] * f[5];
  o[1] = v[2] * f[0] - v[0] * f[2] + v[5] * f[3] - v[3] * f[5];
  o[2] = -v[1] * f[0] + v[0] * f[1] - v[4] * f[3] + v[3] * f[4];
  o[3] = -v[2] * f[4] + v[1] * f[5];
  o[4] = v[2] * f[3] - v[0] * f[5];
  o[5] = -v[1] * f[3] + v[0] * f[4];
}

template <class R, int T> __device__ void velocity(const Mdl<R> &M, Arena<R> &A) {
  const B200Model &m = M.m;
  if (TID < 6) {
    const int c = TID;
    A.cvel[c] = 0;
    R g = 0;
    if (c >= 3 && !(m.disable_flags & B200_DSBL_GRAVITY))
      g = -R(c == 3 ? m.gravity_x : c == 4 ? m.gravity_y : m.gravity_z);
    A.cacc[c] = g;
  }
  SYNC();
  const int *order = IF(body_order), *lstart = IF(level_start);
  if (m.nbody <= 32) {
    // one lane per body, as in the kinematics: each body's own velocity
    // increment, a pointer-jumping sum down the tree, then the bias
    // accelerations from the parents' velocities and a second sum
    if (WARP0) {
      const unsigned full = 0xffffffffu;
      const int b = LANE;
      const bool body = b > 0 && b < m.nbody;
      int parent = body ? IF(body_parentid)[b] : 0, anc = parent;
      R lv[6] = {0, 0, 0, 0, 0, 0};
      const int d0 = body ? IF(body_dofadr)[b] : 0, nd = body ? IF(body_dofnum)[b] : 0;
      for (int i = 0; i < nd; ++i)
        for (int c = 0; c < 6; ++c) lv[c] += A.cdof[6 * (d0 + i) + c] * A.qvel[d0 + i];
      for (int round = 0; round < 5; ++round) {
        if (!__any_sync(full, anc != 0)) break;
        const int a = anc;
        R add[6];
        for (int c = 0; c < 6; ++c) add[c] = __shfl_sync(full, lv[c], a);
        const int aa = __shfl_sync(full, anc, a);
        if (a != 0) {
          for (int c = 0; c < 6; ++c) lv[c] += add[c];
          anc = aa;
        }
      }
      R vel[6], la[6] = {0, 0, 0, 0, 0, 0};
      for (int c = 0; c < 6; ++c) vel[c] = __shfl_sync(full, lv[c], parent);
      if (parent == 0)
        for (int c = 0; c < 6; ++c) vel[c] = 0;
      if (body) {
        int dof = d0;
        const int j0 = IF(body_jntadr)[b], j1 = j0 + IF(body_jntnum)[b];
        for (int j = j0; j < j1; ++j) {
          const int type = IF(jnt_type)[j];
          if (type == B200_JNT_FREE) {
            for (int i = 0; i < 3; ++i) {
              for (int c = 0; c < 6; ++c) vel[c] += A.cdof[6 * (dof + i) + c] * A.qvel[dof + i];
              for (int c = 0; c < 6; ++c) A.cdof_dot[6 * (dof + i) + c] = 0;
            }
            dof += 3;
          }
          const int width = type == B200_JNT_FREE || type == B200_JNT_BALL ? 3 : 1;
          for (int i = 0; i < width; ++i) {
            R dd[6];
            motion_cross(vel, A.cdof + 6 * (dof + i), dd);
            for (int c = 0; c < 6; ++c) {
              A.cdof_dot[6 * (dof + i) + c] = dd[c];
              la[c] += dd[c] * A.qvel[dof + i];
            }
          }
          for (int i = 0; i < width; ++i)
            for (int c = 0; c < 6; ++c) vel[c] += A.cdof[6 * (dof + i) + c] * A.qvel[dof + i];
          dof += width;
        }
      }
      anc = parent;
      for (int round = 0; round < 5; ++round) {
        if (!__any_sync(full, anc != 0)) break;
        const int a = anc;
        R add[6];
        for (int c = 0; c < 6; ++c) add[c] = __shfl_sync(full, la[c], a);
        const int aa = __shfl_sync(full, anc, a);
        if (a != 0) {
          for (int c = 0; c < 6; ++c) la[c] += add[c];
          anc = aa;
        }
      }
      if (body)
        for (int c = 0; c < 6; ++c) { A.cvel[6 * b + c] = lv[c]; A.cacc[6 * b + c] = A.cacc[c] + la[c]; }
      __syncwarp();
    }
  } else if (WARP0) {  // larger trees: the world's first warp walks the levels with warp barriers
    for (int level = 1; level < m.nlevel; ++level) {
      const int a = lstart[level], n = lstart[level + 1] - a;
      for (int k = LANE; k < n; k += 32) {
        const int b = order[a + k], p = IF(body_parentid)[b];
        R vel[6], acc[6];
        for (int c = 0; c < 6; ++c) { vel[c] = A.cvel[6 * p + c]; acc[c] = A.cacc[6 * p + c]; }
        int dof = IF(body_dofadr)[b];
        const int j0 = IF(body_jntadr)[b], j1 = j0 + IF(body_jntnum)[b];
        for (int j = j0; j < j1; ++j) {
          const int type = IF(jnt_type)[j];
          if (type == B200_JNT_FREE) {
            for (int i = 0; i < 3; ++i) {
              for (int c = 0; c < 6; ++c) vel[c] += A.cdof[6 * (dof + i) + c] * A.qvel[dof + i];
              for (int c = 0; c < 6; ++c) A.cdof_dot[6 * (dof + i) + c] = 0;
            }
            dof += 3;
          }
          const int width = type == B200_JNT_FREE || type == B200_JNT_BALL ? 3 : 1;
          for (int i = 0; i < width; ++i) {
            R dd[6];
            motion_cross(vel, A.cdof + 6 * (dof + i), dd);
            for (int c = 0; c < 6; ++c) {
              A.cdof_dot[6 * (dof + i) + c] = dd[c];
              acc[c] += dd[c] * A.qvel[dof + i];
            }
          }
          for (int i = 0; i < width; ++i)
            for (int c = 0; c < 6; ++c) vel[c] += A.cdof[6 * (dof + i) + c] * A.qvel[dof + i];
          dof += width;
        }
        for (int c = 0; c < 6; ++c) { A.cvel[6 * b + c] = vel[c]; A.cacc[6 * b + c] = acc[c]; }
      }
      __syncwarp();
    }
  }
  SYNC();
  // raw body forces (into cfrc), then subtree sums
  FOR(b, m.nbody) {
    R f[6], mom[6], corr[6];
    if (b == 0) {
      for (int c = 0; c < 6; ++c) A.cfrc[c] = 0;
    } else {
      inert_mul(A.cinert + 10 * b, A.cacc + 6 * b, f);
      inert_mul(A.cinert + 10 * b, A.cvel + 6 * b, mom);
      force_cross(A.cvel + 6 * b, mom, corr);
      for (int c = 0; c < 6; ++c) A.cfrc[6 * b + c] = f[c] + corr[c];
    }
  }
  SYNC();
  // subtree composite into cacc (acceleration is no longer needed)
  FOR(w, 6 * m.nbody) {
    const int b = w / 6, c = w % 6;
    R s = A.cfrc[w];
    for (int k = b + 1; k < IF(body_subtree_end)[b]; ++k) s += A.cfrc[6 * k + c];
    A.cacc[w] = s;
  }
  SYNC();
  FOR(d, m.nv) {
    const R *f = A.cacc + 6 * IF(dof_bodyid)[d];
    R v = 0;
    for (int c = 0; c < 6; ++c) v += A.cdof[6 * d + c] * f[c];
    A.qfrc_bias[d] = v;
    const R damping = RF(dof_damping)[d];
    R force = 0;
    if (!(m.disable_flags & B200_DSBL_DAMPER) && damping != R(0)) force = -A.qvel[d] * damping;
    const int j = IF(dof_jntid)[d], kind = IF(jnt_type)[j];
    const R stiff = RF(jnt_stiffness)[j];
    if (!(m.disable_flags & B200_DSBL_SPRING) && stiff != R(0) && (kind == B200_JNT_SLIDE || kind == B200_JNT_HINGE)) {
      const int p = IF(jnt_qposadr)[j];
      force += -(A.qpos[p] - RF(qpos_spring)[p]) * stiff;
    }
    A.qfrc_passive[d] = force;
  }
  FOR(u, m.nu) {
    const int j = IF(actuator_trnid)[u];
    const R gear = RF(actuator_gear)[u];
    A.act_length[u] = gear * A.qpos[IF(jnt_qposadr)[j]];
    A.act_moment[u] = gear;
  }
  SYNC();
}

// ============================================================ OSC (FP64)
// robosuite OSC_POSE as computed by the reference (fused_control_drive.cu:35-111,
// osc_solver.cu:309-676).  Warp 0 computes; shared scratch aliases H.
namespace osc {
// FP64 OSC scratch (doubles); regions are reused once their values are dead:
// the Cholesky factor of M holds Jbar later, A and its factor hold N later.
// The 3x3 blocks keep a row stride of 6 (15 doubles each).
enum { kM = 0, kJ = 49, kMi = 91, kJbar = 91, kMJT = 140, kA = 182, kN = 182, kLA = 218, kLf = 254, kAp = 290,
       kAr = 305, kLp = 320, kLr = 335, kMisc = 350, kEnd = 397 };
}

// In-place lower Cholesky of an n x n FP64 matrix (row stride ld), one warp,
// lane i owning row i.  *bad is set when a pivot is not positive or is tiny
// relative to the matrix diagonal (near-singular: caller falls back).
static __device__ void chol_warp(double *a, int n, int ld, int lane, int *bad) {
  double dmax = 0;
  for (int i = 0; i < n; ++i) dmax = fmax(dmax, fabs(a[i * ld + i]));
  for (int k = 0; k < n; ++k) {
    const double p = a[k * ld + k];
    if (!(p > 1e-12 * dmax)) {
      if (lane == 0) *bad = 1;
    }
    const double d = sqrt(fmax(p, 1e-300)), inv = 1.0 / d;
    __syncwarp();
    if (lane == k) a[k * ld + k] = d;
    else if (lane > k && lane < n) a[lane * ld + k] *= inv;
    __syncwarp();
    if (lane > k && lane < n)
      for (int j = k + 1; j <= lane; ++j) a[lane * ld + j] -= a[lane * ld + k] * a[j * ld + k];
    __syncwarp();
  }
}

// one-sided Jacobi pseudoinverse of an n x n block (6-stride), one lane group
// of 8 lanes, lane r owning row r (osc_solver.cu:120-253 pinv_group)
static __device__ __noinline__ void pinv_group(const double *in, double *out, int n, int lane8, unsigned mask, int *ok) {
  double scale = 0;
  if (lane8 < n)
    for (int c = 0; c < n; ++c) scale = fmax(scale, fabs(in[lane8 * 6 + c]));
  for (int o = 4; o > 0; o >>= 1) scale = fmax(scale, __shfl_xor_sync(mask, scale, o, 8));
  for (int z = lane8; z < 6 * (n - 1) + n; z += 8) out[z] = 0;
  if (!(scale > 0)) { *ok = 0; return; }
  double b[6], v[6];
  for (int c = 0; c < 6; ++c) {
    b[c] = lane8 < n && c < n ? in[lane8 * 6 + c] / scale : 0.0;
    v[c] = lane8 < n && c == lane8 ? 1.0 : 0.0;
  }
  bool converged = false;
  for (int sweep = 0; sweep < 64; ++sweep) {
    int rotations = 0;
    for (int p = 0; p < n - 1; ++p)
      for (int q = p + 1; q < n; ++q) {
        double bp = 0, bq = 0, vp = 0, vq = 0;
#pragma unroll
        for (int c = 0; c < 6; ++c) {
          if (c == p) { bp = b[c]; vp = v[c]; }
          if (c == q) { bq = b[c]; vq = v[c]; }
        }
        double alpha = bp * bp, beta = bq * bq, gamma = bp * bq;
        for (int o = 4; o > 0; o >>= 1) {
          alpha += __shfl_xor_sync(mask, alpha, o, 8);
          beta += __shfl_xor_sync(mask, beta, o, 8);
          gamma += __shfl_xor_sync(mask, gamma, o, 8);
        }
        if (fabs(gamma) > DBL_EPSILON * sqrt(alpha) * sqrt(beta)) {
          const double zeta = (beta - alpha) / (2 * gamma);
          const double t = (zeta < 0 ? -1.0 : 1.0) / (fabs(zeta) + sqrt(1 + zeta * zeta));
          const double c = 1 / sqrt(1 + t * t), s = c * t;
          const double nbp = c * bp - s * bq, nbq = s * bp + c * bq, nvp = c * vp - s * vq, nvq = s * vp + c * vq;
#pragma unroll
          for (int k = 0; k < 6; ++k) {
            if (k == p) { b[k] = nbp; v[k] = nvp; }
            if (k == q) { b[k] = nbq; v[k] = nvq; }
          }
          ++rotations;
        }
      }
    if (rotations == 0) { converged = true; break; }
  }
  double norms[6], sing[6], maxn = 0;
  for (int p = 0; p < 6; ++p) {
    double s = b[p] * b[p];
    for (int o = 4; o > 0; o >>= 1) s += __shfl_xor_sync(mask, s, o, 8);
    norms[p] = s;
    sing[p] = sqrt(s);
    if (p < n) maxn = fmax(maxn, sing[p]);
  }
  double maxcorr = 0;
  for (int p = 0; p < n; ++p)
    for (int q = p + 1; q < n; ++q) {
      double g = b[p] * b[q];
      for (int o = 4; o > 0; o >>= 1) g += __shfl_xor_sync(mask, g, o, 8);
      if (sing[p] > 1e-15 * maxn && sing[q] > 1e-15 * maxn) maxcorr = fmax(maxcorr, fabs(g) / (sing[p] * sing[q]));
    }
  if (maxcorr < 2e-15) converged = true;
  // out[row][col] = sum_k V[row][k] B[col][k] / (norm_k * scale); lane owns row
  for (int c = 0; c < n; ++c) {
    double val = 0;
    for (int k = 0; k < n; ++k) {
      const double bck = __shfl_sync(mask, b[k], c, 8);
      if (sing[k] > 1e-15 * maxn) val += v[k] * bck * ((1 / norms[k]) / scale);
    }
    if (lane8 < n) out[lane8 * 6 + c] = val;
  }
  if (!converged) *ok = 0;
}

template <class R> __device__ R action_component(const Mdl<R> &M, R action, int axis) {
  const R *p = RF(osc_action_config);
  const R scale = mabs(p[18 + axis] - p[12 + axis]) / mabs(p[6 + axis] - p[axis]);
  const R a = action != action ? action : mmin(p[6 + axis], mmax(p[axis], action));
  return (a - (p[6 + axis] + p[axis]) * R(0.5)) * scale + (p[18 + axis] + p[12 + axis]) * R(0.5);
}

template <class R> __device__ void rotation_delta(R x, R y, R z, double *r) {
  const R angle = msqrt(x * x + y * y + z * z);
  const R f = angle == R(0) ? R(0) : msin(angle * R(0.5)) / angle;
  const R raw[4] = {x * f, y * f, z * f, angle == R(0) ? R(1) : mcos(angle * R(0.5))};
  // robosuite's float32 quaternion convention; every float product and sum is
  // rounded on its own (no fused multiply-add), so that the goal does not
  // depend on the compiler's contraction choices
  float q[4] = {(float)raw[3], (float)raw[0], (float)raw[1], (float)raw[2]};
  R acc = 0;
  for (int i = 0; i < 4; ++i) acc += (R)__fmul_rn(q[i], q[i]);
  const float norm = (float)acc;
  const R factor = msqrt(R(2) / (R)norm);
  for (int i = 0; i < 4; ++i) q[i] = (float)((R)q[i] * factor);
  auto sq = [&](int i) { return (R)__fmul_rn(q[i], q[i]); };
  auto sum = [&](int a, int b, int c, int d) { return (R)__fadd_rn(__fmul_rn(q[a], q[b]), __fmul_rn(q[c], q[d])); };
  auto dif = [&](int a, int b, int c, int d) { return (R)__fsub_rn(__fmul_rn(q[a], q[b]), __fmul_rn(q[c], q[d])); };
  r[0] = (double)(R(1) - sq(2) - sq(3));
  r[4] = (double)(R(1) - sq(1) - sq(3));
  r[8] = (double)(R(1) - sq(1) - sq(2));
  r[1] = (double)dif(1, 2, 3, 0);
  r[2] = (double)sum(1, 3, 2, 0);
  r[3] = (double)sum(1, 2, 3, 0);
  r[5] = (double)dif(2, 3, 1, 0);
  r[6] = (double)dif(1, 3, 2, 0);
  r[7] = (double)sum(2, 3, 1, 0);
}

// G: the threads that run it (the world's first G threads; 32 when the world's
// other warps run collision meanwhile)
template <class R, int T, int G> __device__ void osc_control(const Mdl<R> &M, Arena<R> &A, bool policy) {
  const B200Model &m = M.m;
  const int nv = m.nv, site = m.ee_site, body = IF(site_bodyid)[site];
  const int *vi = IF(osc_dofadr), *qi = IF(osc_qposadr), *ids = IF(osc_actuator);
  double *S = A.osc;
  const int lane = TID;
  // ee velocity over all dofs (non-ancestors have zero Jacobian columns)
  if (lane < 32) {  // first warp: six 4-lane groups, lanes 24..31 idle
    const int ax = lane >> 2, l4 = lane & 3;
    R v = 0;
    const V3<R> point = ld3(A.sxpos + 3 * site), com = ld3(A.com + 3 * IF(body_rootid)[body]);
    for (int d = l4; d < nv && ax < 6; d += 4) {
      if (!dof_ancestor(M, body, d)) continue;
      const R *mo = A.cdof + 6 * d;
      R jv;
      if (ax < 3) {
        const V3<R> ang = v3<R>(mo[0], mo[1], mo[2]);
        jv = mo[3 + ax] + cross(ang, point - com)[ax];
      } else jv = mo[ax - 3];
      v += jv * A.qvel[d];
    }
    v += __shfl_xor_sync(0xffffffffu, v, 2, 4);
    v += __shfl_xor_sync(0xffffffffu, v, 1, 4);
    if (l4 == 0 && ax < 6) A.ee_vel[ax] = v;
  }
  // gathers: arm mass block, 6x7 Jacobian (and its transpose)
  for (int z = lane; z < 49; z += G) S[osc::kM + z] = (double)mass_at(M, A.M, vi[z / 7], vi[z % 7]);
  for (int z = lane; z < 42; z += G) {
    const int ax = z / 7, d = vi[z % 7];
    double jv = 0;
    if (dof_ancestor(M, body, d)) {
      const R *mo = A.cdof + 6 * d;
      if (ax < 3) {
        const V3<R> ang = v3<R>(mo[0], mo[1], mo[2]);
        const V3<R> off = ld3(A.sxpos + 3 * site) - ld3(A.com + 3 * IF(body_rootid)[body]);
        jv = (double)(mo[3 + ax] + cross(ang, off)[ax]);
      } else jv = (double)mo[ax - 3];
    }
    S[osc::kJ + z] = jv;
  }
  group_sync<T, G>();
  int *err = &A.iscal[6];
  if (*err) return;  // block-uniform
  // M^-1 J^T, A = J M^-1 J^T and the task-space inverses.  A is symmetric
  // positive definite away from kinematic singularities, so its
  // pseudoinverse is its inverse: warp-parallel FP64 Cholesky factorizations
  // replace the reference's LU and one-sided Jacobi SVD (same matrices to
  // FP64 rounding).  When a pivot shows near-singularity the reference's
  // Jacobi pseudoinverse runs instead (pinv_group), rank cutoff included.
  if (WARP0) {
    int *flags = A.iscal + 16;
    double *L7 = S + osc::kMi;  // Cholesky factor of M (lower, row-major)
    for (int z = lane; z < 49; z += 32) L7[z] = S[osc::kM + z];
    if (lane < 4) flags[lane] = lane < 2 ? 0 : 1;  // [0],[1]: Cholesky failed; [2],[3]: 3x3 inverse good
    __syncwarp();
    chol_warp(L7, 7, 7, lane, &flags[0]);
    if (lane < 6) {  // column c of M^-1 J^T
      const int c = lane;
      double y[7], id[7];
#pragma unroll
      for (int i = 0; i < 7; ++i) id[i] = 1.0 / L7[i * 7 + i];
#pragma unroll
      for (int i = 0; i < 7; ++i) {
        double v = S[osc::kJ + c * 7 + i];
        for (int k = 0; k < i; ++k) v -= L7[i * 7 + k] * y[k];
        y[i] = v * id[i];
      }
#pragma unroll
      for (int i = 6; i >= 0; --i) {
        double v = y[i];
        for (int k = i + 1; k < 7; ++k) v -= L7[k * 7 + i] * y[k];
        y[i] = v * id[i];
      }
      for (int i = 0; i < 7; ++i) S[osc::kMJT + i * 6 + c] = y[i];
    }
    __syncwarp();
    for (int z = lane; z < 36; z += 32) {
      const int r = z / 6, c = z % 6;
      double v = 0;
      for (int k = 0; k < 7; ++k) v += S[osc::kJ + r * 7 + k] * S[osc::kMJT + k * 6 + c];
      S[osc::kA + z] = v;
    }
    __syncwarp();
    for (int z = lane; z < 15; z += 32) {
      const int r = z / 6, c = z % 6;
      S[osc::kAp + z] = c < 3 ? S[osc::kA + z] : 0.0;
      S[osc::kAr + z] = c < 3 ? S[osc::kA + (r + 3) * 6 + c + 3] : 0.0;
    }
    double *LA = S + osc::kLA;  // Cholesky factor of A (6x6, stride 6)
    for (int z = lane; z < 36; z += 32) LA[z] = S[osc::kA + z];
    __syncwarp();
    chol_warp(LA, 6, 6, lane, &flags[1]);
    // full inverse: lane c solves A x = e_c; 3x3 blocks by the adjugate
    if (lane < 6) {
      const int c = lane;
      double y[6], id[6];
#pragma unroll
      for (int i = 0; i < 6; ++i) id[i] = 1.0 / LA[i * 6 + i];
#pragma unroll
      for (int i = 0; i < 6; ++i) {
        double v = i == c ? 1.0 : 0.0;
        for (int k = 0; k < i; ++k) v -= LA[i * 6 + k] * y[k];
        y[i] = v * id[i];
      }
#pragma unroll
      for (int i = 5; i >= 0; --i) {
        double v = y[i];
        for (int k = i + 1; k < 6; ++k) v -= LA[k * 6 + i] * y[k];
        y[i] = v * id[i];
      }
      for (int i = 0; i < 6; ++i) S[osc::kLf + i * 6 + c] = y[i];
    } else if (lane >= 8 && lane < 26) {
      const int blk = lane < 17 ? 0 : 1, e = (lane - 8) % 9, r = e / 3, c = e % 3;
      const double *a = S + (blk ? osc::kAr : osc::kAp);
      const double a00 = a[0], a01 = a[1], a02 = a[2], a10 = a[6], a11 = a[7], a12 = a[8];
      const double a20 = a[12], a21 = a[13], a22 = a[14];
      const double c00 = a11 * a22 - a12 * a21, c01 = a12 * a20 - a10 * a22, c02 = a10 * a21 - a11 * a20;
      const double det = a00 * c00 + a01 * c01 + a02 * c02;
      double adj;  // adj[r][c] = cofactor[c][r]
      const int i0 = (c + 1) % 3, i1 = (c + 2) % 3, j0 = (r + 1) % 3, j1 = (r + 2) % 3;
      adj = a[i0 * 6 + j0] * a[i1 * 6 + j1] - a[i0 * 6 + j1] * a[i1 * 6 + j0];
      const bool good = det > 1e-12 * a00 * a11 * a22 && det > 0.0;
      if (!good) flags[2 + blk] = 0;
      double *out = S + (blk ? osc::kLr : osc::kLp);
      out[r * 6 + c] = adj / det;
    }
    __syncwarp();
    const bool fast = !flags[0] && !flags[1] && flags[2] && flags[3];
    if (flags[0]) {
      if (lane == 0) *err = 2;  // arm mass matrix not positive definite
    } else if (!fast) {
      int *ok_flags = A.iscal + 20;
      const int group = lane >> 3, l8 = lane & 7;
      const unsigned mask = 0xffu << (lane & 24);
      if (l8 == 0 && group < 3) ok_flags[group] = 1;
      __syncwarp();
      if (group == 0) pinv_group(S + osc::kA, S + osc::kLf, 6, l8, mask, &ok_flags[0]);
      else if (group == 1) pinv_group(S + osc::kAp, S + osc::kLp, 3, l8, mask, &ok_flags[1]);
      else if (group == 2) pinv_group(S + osc::kAr, S + osc::kLr, 3, l8, mask, &ok_flags[2]);
      __syncwarp();
      if (lane == 0 && !(ok_flags[0] && ok_flags[1] && ok_flags[2])) *err = 4;
    }
  }
  group_sync<T, G>();
  if (*err) return;
  for (int z = lane; z < 42; z += G) {  // Jbar = MJT Lf (7x6)
    const int r = z / 6, c = z % 6;
    double v = 0;
    for (int k = 0; k < 6; ++k) v += S[osc::kMJT + r * 6 + k] * S[osc::kLf + k * 6 + c];
    S[osc::kJbar + z] = v;
  }
  double *gp = S + osc::kMisc, *gr = gp + 3, *cur = gr + 9, *desired = cur + 9, *op = desired + 6, *opm = op + 6;
  double *pd = opm + 7;
  if (lane == 0) {
    for (int r = 0; r < 3; ++r) gp[r] = (double)A.goal_pos[r];
    for (int i = 0; i < 9; ++i) { gr[i] = (double)A.goal_rot[i]; cur[i] = (double)A.sxmat[9 * site + i]; }
    if (policy) {
      for (int r = 0; r < 3; ++r) gp[r] = (double)(R)(A.sxpos[3 * site + r] + action_component(M, A.action[r], r));
      const R x = action_component(M, A.action[3], 3), y = action_component(M, A.action[4], 4),
              z = action_component(M, A.action[5], 5);
      if (x != R(0) || y != R(0) || z != R(0)) {
        double d[9];
        rotation_delta(x, y, z, d);
        double g2[9];
        for (int r = 0; r < 3; ++r)
          for (int c = 0; c < 3; ++c) {
            double v = 0;
            for (int k = 0; k < 3; ++k) v += d[r * 3 + k] * cur[k * 3 + c];
            g2[r * 3 + c] = v;
          }
        for (int i = 0; i < 9; ++i) gr[i] = sizeof(R) == 4 ? (double)(float)g2[i] : g2[i];
      }
    }
  }
  group_sync<T, G>();
  for (int z = lane; z < 49; z += G) {  // N = I - Jbar J (7x7)
    const int r = z / 7, c = z % 7;
    double v = 0;
    for (int k = 0; k < 6; ++k) v += S[osc::kJbar + r * 6 + k] * S[osc::kJ + k * 7 + c];
    S[osc::kN + z] = (r == c ? 1.0 : 0.0) - v;
  }
  const R *gains = RF(osc_gains), *q0 = RF(osc_q0), *nul = RF(osc_null);
  if (lane < 3) {
    const int r = lane, nx = (r + 1) % 3, ls = (r + 2) % 3;
    double er = 0;
    for (int c = 0; c < 3; ++c) er += 0.5 * (cur[nx * 3 + c] * gr[ls * 3 + c] - cur[ls * 3 + c] * gr[nx * 3 + c]);
    const double ep = gp[r] - (double)A.sxpos[3 * site + r];
    desired[r] = (double)gains[r] * ep - (double)gains[r + 6] * (double)A.ee_vel[r];
    desired[r + 3] = (double)gains[r + 3] * er - (double)gains[r + 9] * (double)A.ee_vel[r + 3];
  }
  if (lane < 7)
    pd[lane] = (double)nul[0] * ((double)q0[lane] - (double)A.qpos[qi[lane]]) - (double)nul[1] * (double)A.qvel[vi[lane]];
  group_sync<T, G>();
  for (int z = lane; z < 13; z += G) {
    double v = 0;
    if (z < 6) {
      if (m.osc_uncouple) {
        const int row = z % 3, offs = z < 3 ? 0 : 3;
        const double *lam = S + (z < 3 ? osc::kLp : osc::kLr);
        for (int k = 0; k < 3; ++k) v += lam[row * 6 + k] * desired[offs + k];
      } else
        for (int k = 0; k < 6; ++k) v += S[osc::kLf + z * 6 + k] * desired[k];
      op[z] = v;
    } else {
      const int r = z - 6;
      for (int k = 0; k < 7; ++k) v += S[osc::kM + r * 7 + k] * pd[k];
      opm[r] = v;
    }
  }
  group_sync<T, G>();
  if (lane < 7) {
    const int i = lane;
    double task = 0, post = 0;
    for (int k = 0; k < 6; ++k) task += S[osc::kJ + k * 7 + i] * op[k];
    for (int k = 0; k < 7; ++k) post += S[osc::kN + k * 7 + i] * opm[k];
    const double t = task + (double)A.qfrc_bias[vi[i]] + post;
    const R *rg = RF(actuator_ctrlrange) + 2 * ids[i];
    const double lim = t != t ? t : fmin((double)rg[1], fmax((double)rg[0], t));
    A.ctrl[ids[i]] = (R)lim;
  }
  for (int i = lane; i < 3; i += G) A.goal_pos[i] = (R)gp[i];
  for (int i = lane; i < 9; i += G) A.goal_rot[i] = (R)gr[i];
  if (lane == G - 1) {
    const R a6 = A.action[6];
    const R sgn = a6 != a6 ? a6 : (a6 > R(0) ? R(1) : (a6 < R(0) ? R(-1) : R(0)));
    const R speed = RF(osc_action_config)[24];
    for (int i = 0; i < 2; ++i) {
      R v = A.gripper[i] + speed * (i == 0 ? R(-1) : R(1)) * sgn;
      v = v != v ? v : mmin(R(1), mmax(R(-1), v));
      A.gripper[i] = v;
      const R *rg = RF(actuator_ctrlrange) + 2 * ids[7 + i];
      A.ctrl[ids[7 + i]] = (rg[1] + rg[0]) * R(0.5) + (rg[1] - rg[0]) * R(0.5) * v;
    }
  }
  group_sync<T, G>();
}

// ============================================================ actuation
// The G threads [G0, G0 + G) of the world run it (whole warps).
template <class R, int T, int G0, int G> __device__ void actuation(const Mdl<R> &M, Arena<R> &A) {
  const B200Model &m = M.m;
  for (int d = TID - G0; d < m.nv; d += G) {
    R f = 0;
    for (int u = 0; u < m.nu; ++u) {
      const int j = IF(actuator_trnid)[u];
      if (IF(jnt_dofadr)[j] != d) continue;
      R c = A.ctrl[u];
      if (IF(actuator_ctrllimited)[u] && !(m.disable_flags & B200_DSBL_CLAMPCTRL)) {
        const R *rg = RF(actuator_ctrlrange) + 2 * u;
        c = mmin(mmax(rg[0], c), rg[1]);
      }
      const R *gp = RF(actuator_gainprm) + 3 * u, *bp = RF(actuator_biasprm) + 3 * u;
      const R vel = A.act_moment[u] * A.qvel[d];
      R gain = gp[0];
      if (IF(actuator_gaintype)[u] == 1) gain = gp[0] + gp[1] * A.act_length[u] + gp[2] * vel;
      R bias = 0;
      if (IF(actuator_biastype)[u] == 1) bias = bp[0] + bp[1] * A.act_length[u] + bp[2] * vel;
      R force = gain * c + bias;
      if (IF(actuator_forcelimited)[u]) {
        const R *fr = RF(actuator_forcerange) + 2 * u;
        force = mmin(mmax(fr[0], force), fr[1]);
      }
      f += A.act_moment[u] * force;
    }
    A.qfrc_actuator[d] = f;
    A.qfrc_smooth[d] = A.qfrc_passive[d] - A.qfrc_bias[d] + f;
    A.qacc_smooth[d] = A.qfrc_smooth[d];
  }
  group_sync<T, G>();
  tree_solve<R, T, G0 / 32, G / 32>(M, A.L, A.qacc_smooth, A.colbuf, false);
  group_sync<T, G>();
}

// ============================================================ Newton
// mjwarp_solver_state.cu, mjwarp_constraint.cu, mjwarp_hessian.cu,
// mjwarp_direction.cu, mjwarp_linesearch.cu
template <class R, int T> __device__ void eval_gradient(const Mdl<R> &M, Arena<R> &A) {
  const B200Model &m = M.m;
  const int nefc = A.iscal[1], nf = A.iscal[2], nv = m.nv;
  const R impratio = R(m.impratio_invsqrt);
  FOR(r, nefc) {
    const R d = A.efc_D[r], res = A.efc_jaref[r];
    R force;
    int state;
    if (r < nf) {
      const R loss = A.efc_floss[r], radius = safe_div(loss, d);
      if (res <= -radius) { force = loss; state = kLinearNeg; }
      else if (res >= radius) { force = -loss; state = kLinearPos; }
      else { force = -d * res; state = kQuadratic; }
    } else if (A.efc_type[r] == 7) {
      const int c = A.efc_id[r], head = A.con_adr[c], dim = A.con_dim[c];
      const R *fr = A.con + (size_t)c * kCWidth + kCFriction;
      const R mu = fr[0] * impratio, normal = A.efc_jaref[head], d0 = A.efc_D[head];
      R tt = 0, tscale = 0;
      for (int j = 1; j < dim; ++j) {
        const R u = A.efc_jaref[head + j] * fr[j - 1];
        tt += u * u;
        if (r == head + j) tscale = u * fr[j - 1];
      }
      const R n = normal * mu, t = tt <= R(0) ? R(0) : msqrt(tt);
      if (n >= mu * t || (t <= R(0) && n >= R(0))) { force = 0; state = kSatisfied; }
      else if (mu * n + t <= R(0) || (t <= R(0) && n < R(0))) { force = -d * res; state = kQuadratic; }
      else {
        const R dm = safe_div(d0, mu * mu * (R(1) + mu * mu));
        const R fn = -dm * (n - mu * t) * mu;
        force = r == head ? fn : -safe_div(fn, t) * tscale;
        state = kCone;
      }
    } else if (res >= R(0)) { force = 0; state = kSatisfied; }
    else { force = -d * res; state = kQuadratic; }
    A.efc_force[r] = force;
    // H depends on the states (and, for cone-state contacts, on jaref):
    // flag a refactorization when a state changes or a contact is in the cone
    if (A.efc_state[r] != state || state == kCone) A.iscal[14] = 1;
    A.efc_state[r] = state;
  }
  SYNC();
  R gd = 0;
  FOR(i, nv) {
    R tot = 0;
    const int t = IF(dof_treeid)[i], off = i - IF(tree_dofadr)[t], kmax = m.kmax_dof;
    // rows acting on the dof's tree, ascending (the same sum order as a scan of all rows)
    for (int e = A.tree_segadr[t], end = A.tree_segadr[t + 1]; e < end; ++e) {
      const unsigned sg = A.tree_seg[e];
      const int r0 = sg & 0xffffu, len = (sg >> 16) & 0xffu, col = (int)(sg >> 24) + off;
      for (int p = 0; p < len; ++p) tot += A.J[(r0 + p) * kmax + col] * A.efc_force[r0 + p];
    }
    A.qfrc_constraint[i] = tot;
    const R g = A.Ma[i] - A.qfrc_smooth[i] - tot;
    A.grad[i] = g;
    gd += g * g;
  }
  gd = world_sum<T>(gd, A.red);
  if (TID == 0) A.scal[3] = gd;
}

// H = M + J' D J over quadratic rows + elliptic-cone curvature
// (mjwarp_hessian.cu:33-212), one dense block per island (lower triangle).
// One thread per H entry (a, b) of an island forms, in this order: the mass
// entry; the D of the single-dof rows on the entry's dof (diagonal only);
// then, contact by contact in ascending row order, J_c' C J_c over the
// contacts acting on both dofs' trees.  C is diag(D) over the contact's
// quadratic rows, or the elliptic-cone curvature matrix when the contact is in
// the cone state.  Each contact term is evaluated over the contact-local dof
// pair, larger index first, so every entry's sum is deterministic.  The cone
// matrices' scalars are staged per contact in efc_quad, which the line search
// rewrites before its next use.
template <class R, int T> __device__ void hessian(const Mdl<R> &M, Arena<R> &A) {
  // unchanged constraint states and no cone-state contact: H, and its factor
  // still held in A.H, are exactly what this assembly would produce again
  if (!A.iscal[14]) return;
  const B200Model &m = M.m;
  const int nisl = A.iscal[11], nsingle = A.iscal[13], ncon = A.iscal[0], kmax = m.kmax_dof;
  const R impratio = R(m.impratio_invsqrt);
  // cone-state contacts: dm, mu^2 and mu n / t at the head row, u_p = jaref_p fr_p / t at friction row p
  FOR(c, ncon) {
    const int r0 = A.con_adr[c];
    if (r0 < 0 || A.efc_type[r0] != 7 || A.con_dim[c] <= 1 || A.efc_state[r0] != kCone) continue;
    const int dim = A.con_dim[c];
    const R *fr = A.con + (size_t)c * kCWidth + kCFriction;
    const R mu = fr[0] * impratio, mu2 = mu * mu, den = mu2 * (R(1) + mu2);
    const R dm = A.efc_D[r0] / (den != R(0) ? den : R(1e-15));
    R tt = 0;
    for (int d = 1; d < dim; ++d) {
      const R u = A.efc_jaref[r0 + d] * fr[d - 1];
      tt += u * u;
    }
    const R t = mmax(msqrt(tt), R(1e-15)), it = R(1) / t, mnt = mu * (A.efc_jaref[r0] * mu) * it;
    R *q = A.efc_quad + 3 * r0;
    q[0] = dm; q[1] = mu2; q[2] = mnt;
    for (int d = 1; d < dim; ++d) A.efc_quad[3 * (r0 + d)] = A.efc_jaref[r0 + d] * fr[d - 1] * it;
  }
  SYNC();
  int total = 0;
  for (int i = 0; i < nisl; ++i) total += A.isl_n[i] * (A.isl_n[i] + 1) / 2;
  FOR(e, total) {  // the packed island blocks are contiguous, in island order
    int isl = 0, base = 0;
    while (base + A.isl_n[isl] * (A.isl_n[isl] + 1) / 2 <= e) { base += A.isl_n[isl] * (A.isl_n[isl] + 1) / 2; ++isl; }
    const int loc = e - base;
    int a = (int)((msqrt(8.0f * loc + 1.0f) - 1.0f) * 0.5f);
    while (tri(a, 0) > loc) --a;
    while (tri(a + 1, 0) <= loc) ++a;
    const int b = loc - tri(a, 0);
    const int da = A.isl_dof[A.isl_dofstart[isl] + a], db = A.isl_dof[A.isl_dofstart[isl] + b];
    const int ta = IF(dof_treeid)[da], tb = IF(dof_treeid)[db];
    const int oa = da - IF(tree_dofadr)[ta], ob = db - IF(tree_dofadr)[tb];
    R h = mass_at(M, A.M, da, db);
    int k = A.tree_segadr[ta];
    const int kend = A.tree_segadr[ta + 1];
    // single-dof rows lead the tree's list
    R add = 0;
    for (; k < kend && (int)(A.tree_seg[k] & 0xffffu) < nsingle; ++k) {
      const int r = A.tree_seg[k] & 0xffffu;
      if (da != db || A.efc_state[r] != kQuadratic) continue;
      const int dof = A.efc_type[r] == 1 ? A.efc_id[r] : IF(jnt_dofadr)[A.efc_id[r]];
      if (dof == da) add += A.efc_D[r];
    }
    if (add != R(0)) h += add;
    for (; k < kend; ++k) {
      const unsigned sg = A.tree_seg[k];
      const int r0 = sg & 0xffffu, cnt = (sg >> 16) & 0xffu;
      const int t0 = A.row_t[2 * r0], t1 = A.row_t[2 * r0 + 1];
      if (tb != ta && tb != t0 && tb != t1) continue;
      const int ca = (int)(sg >> 24) + oa;
      const int cb = (tb == ta ? (int)(sg >> 24) : tb == t0 ? 0 : IF(tree_dofnum)[t0]) + ob;
      const int x = ca >= cb ? ca : cb, y = ca >= cb ? cb : ca;
      const int c = A.efc_id[r0], dim = A.con_dim[c];
      const R *J = A.J + (size_t)r0 * kmax;
      R v = 0;
      if (A.efc_type[r0] == 7 && dim > 1 && A.efc_state[r0] != kQuadratic) {
        const int st = A.efc_state[r0];
        if (st == kSatisfied) continue;
        const R *q = A.efc_quad + 3 * r0;
        const R dm = q[0], mu2 = q[1], mnt = q[2];
        if (dm == R(0)) continue;
        const R *fr = A.con + (size_t)c * kCWidth + kCFriction;
#pragma unroll 1
        for (int p = 0; p < cnt; ++p) {
          R cbv = 0;
#pragma unroll 1
          for (int qq = 0; qq < cnt; ++qq) {
            R w;
            if (p == 0 && qq == 0) w = mu2;
            else if (p == 0 || qq == 0) {
              const int ee = p + qq;
              w = -mu2 * A.efc_quad[3 * (r0 + ee)] * fr[ee - 1];
            } else {
              w = mnt * A.efc_quad[3 * (r0 + p)] * fr[p - 1] * A.efc_quad[3 * (r0 + qq)] * fr[qq - 1];
              if (p == qq) w += (mu2 - mnt) * fr[p - 1] * fr[p - 1];
            }
            cbv += (dm * w) * J[qq * kmax + y];
          }
          v += J[p * kmax + x] * cbv;
        }
      } else {
        bool any = false;
#pragma unroll 1
        for (int p = 0; p < cnt; ++p) {
          const bool quad = A.efc_state[r0 + p] == kQuadratic;
          any |= quad;
          v += J[p * kmax + x] * (quad ? A.efc_D[r0 + p] : R(0)) * J[p * kmax + y];
        }
        if (!any) continue;
      }
      h += v;
    }
    A.H[A.isl_off[isl] + loc] = h;
  }
  SYNC();
}

// Cholesky of every island block (islands dealt to the world's warps),
// H x = grad, search = -x (mjwarp_direction.cu:80-160)
template <class R, int T> __device__ void direction(const Mdl<R> &M, Arena<R> &A) {
  const int nv = M.m.nv;
  R *x = A.xs;
  const int lane = LANE, maxn = A.iscal[12];
  const bool refactor = A.iscal[14];
  const BlockRows b = ISLAND_ROWS(T);
  const bool reg = b.rows <= 32 && maxn <= 16;
  if (reg) {  // one row per lane: factor and solve in registers
    const int p = b.start[0] + b.a[0];
    const R xv = chol_solve_reg<R, 16>(A.H, b, maxn, A.colbuf, nv, refactor, b.n[0] > 0 ? A.grad[A.isl_dof[p]] : R(0));
    if (b.n[0] > 0) x[p] = xv;
  } else {
#pragma unroll
    for (int s = 0; s < 4; ++s)
      if (b.n[s] > 0) {
        const int p = b.start[s] + b.a[s];
        x[p] = A.grad[A.isl_dof[p]];
      }
    __syncwarp();
    if (refactor) chol_blocks_smem(A.H, b, maxn);
    solve_blocks(A.H, b, x, maxn, lane);
  }
  if (TID == 0) {
    // FLOP counter, 3x the executed block work: n^3 + 6 n^2 when a block is
    // factored and solved, 6 n^2 when its factor is reused
    int blk = 0;
    for (int i = 0; i < A.iscal[11]; ++i) blk += A.isl_n[i] * A.isl_n[i] * (refactor ? A.isl_n[i] + 6 : 6);
    A.iscal[24] += blk;
  }
  __syncwarp();
  R sq = 0, dec = 0;
#pragma unroll
  for (int s = 0; s < 4; ++s)
    if (b.n[s] > 0) {
      const int p = b.start[s] + b.a[s], d = A.isl_dof[p];
      A.search[d] = -x[p];
      sq += x[p] * x[p];
      dec += A.grad[d] * x[p];
    }
  R sd[2] = {sq, dec};
  world_sums<T>(sd, A.red);
  if (TID == 0) { A.scal[2] = sd[0]; A.scal[4] = sd[1]; }
  SYNC();
  if (TID == 0) A.iscal[14] = 0;  // H holds the factor of the current states
}

// ---- exact line search (mjwarp_linesearch.cu:80-365); row evaluations are
// spread over the world's threads
template <class R> struct Pt { R cost, slope, curv; };
template <class R> __device__ __forceinline__ Pt<R> padd(Pt<R> a, Pt<R> b) {
  return {a.cost + b.cost, a.slope + b.slope, a.curv + b.curv};
}
template <class R> __device__ __forceinline__ Pt<R> quadratic(R q1, R q2, R alpha) {
  const R aq2 = alpha * q2;
  return {alpha * aq2 + alpha * q1, R(2) * aq2 + q1, R(2) * q2};
}
template <class R> __device__ __forceinline__ bool in_bracket(Pt<R> x, Pt<R> y) {
  return (x.slope < y.slope && y.slope < R(0)) || (x.slope > y.slope && y.slope > R(0));
}
template <class R> struct LsRow {
  int kind, state0;
  R x, v, d, loss, q0, q1, q2, u0, v0, uu, uv, vv, dm, mu, cost0, t0, r0;
};
template <class R> __device__ LsRow<R> load_row(const Mdl<R> &M, const Arena<R> &A, int r, int nf) {
  LsRow<R> o;
  o.kind = 0; o.state0 = 0;
  o.x = o.v = o.d = o.loss = o.q0 = o.q1 = o.q2 = o.u0 = o.v0 = o.uu = o.uv = o.vv = o.dm = o.mu = o.cost0 = o.t0 = o.r0 = 0;
  if (r < nf) o.kind = 1;
  else if (A.efc_type[r] != 7) o.kind = 2;
  else {
    const int c = A.efc_id[r], head = A.con_adr[c];
    if (r != head) { o.kind = 4; return o; }
    o.kind = 3;
    const R *qa = A.efc_quad + 3 * r, *qb = A.efc_quad + 3 * (head + 1), *qc = A.efc_quad + 3 * (head + 2);
    o.q0 = qa[0]; o.q1 = qa[1]; o.q2 = qa[2];
    o.u0 = qb[0]; o.v0 = qb[1]; o.uu = qb[2];
    o.uv = qc[0]; o.vv = qc[1]; o.dm = qc[2];
    o.mu = A.con[(size_t)c * kCWidth + kCFriction] * R(M.m.impratio_invsqrt);
    if (o.uu <= R(0)) {
      o.state0 = o.u0 < R(0) ? 1 : 0;
      o.cost0 = o.state0 == 1 ? o.q0 : R(0);
    } else {
      o.t0 = msqrt(o.uu);
      if (o.u0 >= o.mu * o.t0) o.state0 = 0;
      else if (o.mu * o.u0 + o.t0 <= R(0)) { o.state0 = 1; o.cost0 = o.q0; }
      else { o.state0 = 4; o.r0 = o.u0 - o.mu * o.t0; o.cost0 = R(0.5) * o.dm * o.r0 * o.r0; }
    }
    return o;
  }
  o.x = A.efc_jaref[r]; o.v = A.efc_jv[r]; o.d = A.efc_D[r];
  if (o.kind == 1) o.loss = A.efc_floss[r];
  return o;
}
template <class R> __device__ Pt<R> friction_point(const LsRow<R> &r, R x) {
  const R rf = safe_div(r.loss, r.d);
  if (-rf < x && x < rf) {
    const R vd = r.v * r.d;
    return {R(0.5) * r.d * x * x, vd * x, r.v * vd};
  }
  if (x <= -rf) return {r.loss * (R(-0.5) * rf - x), -r.loss * r.v, R(0)};
  return {r.loss * (R(-0.5) * rf + x), r.loss * r.v, R(0)};
}
template <class R> __device__ Pt<R> eval_zero(const LsRow<R> &r) {
  if (r.kind == 4) return {0, 0, 0};
  if (r.kind == 3) {
    if (r.state0 == 1) return {r.q0, r.q1, R(2) * r.q2};
    if (r.state0 == 4) {
      const R ti = R(1) / r.t0, t1 = r.uv * ti, t2 = (r.vv - t1 * t1) * ti, r1 = r.v0 - r.mu * t1;
      return {r.cost0, r.dm * r.r0 * r1, r.dm * (r1 * r1 - r.mu * r.r0 * t2)};
    }
    return {0, 0, 0};
  }
  if (r.kind == 1) return friction_point(r, r.x);
  if (r.kind == 2 && r.x >= R(0)) return {0, 0, 0};
  const R vd = r.v * r.d;
  return {R(0.5) * r.d * r.x * r.x, vd * r.x, r.v * vd};
}
template <class R> __device__ Pt<R> cone_quad_shift(const LsRow<R> &r, R alpha, R n, R tsqr) {
  const R aq2 = alpha * r.q2;
  R cost = alpha * (aq2 + r.q1);
  if (r.state0 == 4) {
    const R bd = r.mu * r.u0 + r.t0;
    cost += R(0.5) * r.dm * bd * bd;
  } else if (r.state0 == 0) cost = R(0.5) * r.dm * (R(1) + r.mu * r.mu) * (n * n + mmax(tsqr, R(0)));
  return {cost, R(2) * aq2 + r.q1, R(2) * r.q2};
}
template <class R> __device__ Pt<R> eval_shift(const LsRow<R> &r, R alpha) {
  if (r.kind == 4) return {0, 0, 0};
  if (r.kind == 3) {
    const R n = r.u0 + alpha * r.v0, tsd = alpha * (R(2) * r.uv + alpha * r.vv), tsqr = r.uu + tsd;
    if (tsqr <= R(0)) {
      if (n < R(0)) return cone_quad_shift(r, alpha, n, tsqr);
    } else {
      const R t = msqrt(tsqr);
      if (n >= r.mu * t) {
      } else if (r.mu * n + t <= R(0)) return cone_quad_shift(r, alpha, n, tsqr);
      else {
        const R ti = R(1) / t, t1 = (r.uv + alpha * r.vv) * ti, t2 = (r.vv - t1 * t1) * ti;
        const R res = n - r.mu * t, r1 = r.v0 - r.mu * t1;
        R cost;
        if (r.state0 == 4) {
          const R tdelta = tsd / (t + r.t0), rdelta = alpha * r.v0 - r.mu * tdelta;
          cost = R(0.5) * r.dm * rdelta * (R(2) * r.r0 + rdelta);
        } else if (r.state0 == 1) {
          const R aq2 = alpha * r.q2, bd = r.mu * n + t;
          cost = alpha * (aq2 + r.q1) - R(0.5) * r.dm * bd * bd;
        } else cost = R(0.5) * r.dm * res * res;
        return {cost, r.dm * res * r1, r.dm * (r1 * r1 + res * (-r.mu * t2))};
      }
    }
    return {-r.cost0, 0, 0};
  }
  if (r.kind == 1) {
    Pt<R> pt = friction_point(r, r.x + alpha * r.v);
    pt.cost -= friction_point(r, r.x).cost;
    return pt;
  }
  const R quad0 = R(0.5) * r.d * r.x * r.x;
  const R cost0 = r.kind == 2 && r.x >= R(0) ? R(0) : quad0;
  if (r.kind == 2 && r.x + alpha * r.v >= R(0)) return {-cost0, 0, 0};
  const R vd = r.v * r.d, h = r.v * vd, ah = alpha * h;
  return {alpha * (vd * r.x + R(0.5) * ah) + (quad0 - cost0), vd * r.x + ah, h};
}
// (cost, slope, curvature) summed over the world's threads; every thread
// gets the same sums (same order), so the search runs identically on all
template <int T, class R> __device__ __forceinline__ Pt<R> world_pt(Pt<R> p, R *red) {
  p = {warp_sum(p.cost), warp_sum(p.slope), warp_sum(p.curv)};
  if (T == 32) return p;
  SYNC();
  if (LANE == 0) { red[3 * (TID >> 5)] = p.cost; red[3 * (TID >> 5) + 1] = p.slope; red[3 * (TID >> 5) + 2] = p.curv; }
  SYNC();
  Pt<R> s = {0, 0, 0};
  for (int k = 0; k < T / 32; ++k) s = padd(s, Pt<R>{red[3 * k], red[3 * k + 1], red[3 * k + 2]});
  return s;
}

template <class R, int T> __device__ void linesearch(const Mdl<R> &M, Arena<R> &A) {
  const B200Model &m = M.m;
  const int nv = m.nv, nefc = A.iscal[1], nf = A.iscal[2];
  mass_mul<R, T>(M, A.M, A.search, A.Mv);
  FOR(r, nefc) A.efc_jv[r] = jdot(M, A, r, A.search);
  SYNC();
  const R impratio = R(m.impratio_invsqrt);
  FOR(r, nefc) {
    if (A.efc_type[r] != 7) continue;
    const int c = A.efc_id[r];
    if (r != A.con_adr[c]) continue;
    const R *fr = A.con + (size_t)c * kCWidth + kCFriction;
    const R x = A.efc_jaref[r], v = A.efc_jv[r], d = A.efc_D[r], vd = v * d;
    R q0 = R(0.5) * x * x * d, q1 = vd * x, q2 = R(0.5) * v * vd;
    const R mu = fr[0] * impratio, u0 = x * mu, v0 = v * mu;
    R uu = 0, uv = 0, vv = 0;
    for (int j = 1; j < A.con_dim[c]; ++j) {
      const int t = r + j;
      const R jv = A.efc_jv[t], ja = A.efc_jaref[t], dj = A.efc_D[t], djx = dj * ja;
      q0 += R(0.5) * ja * djx; q1 += jv * djx; q2 += R(0.5) * jv * dj * jv;
      const R uj = ja * fr[j - 1], vj = jv * fr[j - 1];
      uu += uj * uj; uv += uj * vj; vv += vj * vj;
    }
    R *q = A.efc_quad + 3 * r;
    q[0] = q0; q[1] = q1; q[2] = q2;
    q[3] = u0; q[4] = v0; q[5] = uu;
    q[6] = uv; q[7] = vv;
    const R mu2 = mu * mu;
    q[8] = d / (mu2 * (R(1) + mu2));
  }
  SYNC();
  {  // every thread of the world runs the search on identical reduced values
    const R tol = R(m.tolerance), lstol = R(m.ls_tolerance), scale = R(m.meaninertia) * R(nv);
    const R gtol = mmax(tol * lstol * msqrt(A.scal[2]) * scale, R(1e-6));
    R g1 = 0, g2 = 0;
    FOR(i, nv) {
      g1 += A.search[i] * (A.Ma[i] - A.qfrc_smooth[i]);
      g2 += R(0.5) * A.search[i] * A.Mv[i];
    }
    Pt<R> loc = {0, 0, 0};
    FOR(r, nefc) loc = padd(loc, eval_zero(load_row(M, A, r, nf)));
    R v5[5] = {g1, g2, loc.cost, loc.slope, loc.curv};
    world_sums<T>(v5, A.red);
    g1 = v5[0];
    g2 = v5[1];
    const Pt<R> rows = {v5[2], v5[3], v5[4]};
    int evals = 1;
    const Pt<R> p0 = {rows.cost, g1 + rows.slope, R(2) * g2 + rows.curv};
    const Pt<R> delta = {0, p0.slope, p0.curv};
    const R noise = R(8) * R(FLT_EPSILON);
    const R q1abs = msqrt(R(2) * mmax(rows.cost, R(0)) * mmax(rows.curv, R(0))) + mabs(g1);
    const R gacc = mmax(gtol, noise * q1abs);
    R alpha = 0, improvement = 0;
    bool converged = mabs(p0.slope) < noise * q1abs;
    const R a0 = -safe_div(p0.slope, p0.curv);
    Pt<R> init = {0, 0, 0};
    if (!converged) {
      loc = {0, 0, 0};
      FOR(r, nefc) loc = padd(loc, eval_shift(load_row(M, A, r, nf), a0));
      init = padd(quadratic(g1, g2, a0), world_pt<T>(loc, A.red));
      ++evals;
      if (mabs(init.slope) < gacc && init.cost < R(0)) { converged = true; alpha = a0; improvement = -init.cost; }
    }
    if (!converged) {
      const bool less = init.slope < p0.slope;
      Pt<R> lo = less ? init : delta, hi = less ? delta : init;
      R la = less ? a0 : R(0), ha = less ? R(0) : a0;
      for (int it = 0; it < m.ls_iterations; ++it) {
        const R ln = la - safe_div(lo.slope, lo.curv), hn = ha - safe_div(hi.slope, hi.curv), ma = R(0.5) * (la + ha);
        Pt<R> sl = {0, 0, 0}, sh = {0, 0, 0}, sm = {0, 0, 0};
        FOR(r, nefc) {
          const LsRow<R> row = load_row(M, A, r, nf);
          sl = padd(sl, eval_shift(row, ln));
          sh = padd(sh, eval_shift(row, hn));
          sm = padd(sm, eval_shift(row, ma));
        }
        R v9[9] = {sl.cost, sl.slope, sl.curv, sh.cost, sh.slope, sh.curv, sm.cost, sm.slope, sm.curv};
        world_sums<T>(v9, A.red);
        const Pt<R> nl = padd(quadratic(g1, g2, ln), Pt<R>{v9[0], v9[1], v9[2]});
        const Pt<R> nh = padd(quadratic(g1, g2, hn), Pt<R>{v9[3], v9[4], v9[5]});
        const Pt<R> mid = padd(quadratic(g1, g2, ma), Pt<R>{v9[6], v9[7], v9[8]});
        evals += 3;
        const bool cl = mabs(nl.slope) < gacc && nl.cost < R(0), ch = mabs(nh.slope) < gacc && nh.cost < R(0);
        const bool cm = mabs(mid.slope) < gacc && mid.cost < R(0);
        const bool any = cl || ch || cm;
        bool slo = false, shi = false;
        if (any) {
          Pt<R> best = {R(1e10), 0, 0};
          R ba = 0;
          if (cl && nl.cost < best.cost) { best = nl; ba = ln; }
          if (ch && nh.cost < best.cost) { best = nh; ba = hn; }
          if (cm && mid.cost < best.cost) { best = mid; ba = ma; }
          lo = hi = best;
          la = ha = ba;
        } else {
          bool s;
          s = in_bracket(lo, nl); if (s) { lo = nl; la = ln; } slo |= s;
          s = in_bracket(lo, mid); if (s) { lo = mid; la = ma; } slo |= s;
          s = in_bracket(lo, nh); if (s) { lo = nh; la = hn; } slo |= s;
          s = in_bracket(hi, nh) || (hi.slope < R(0) && nh.slope > R(0)); if (s) { hi = nh; ha = hn; } shi |= s;
          s = in_bracket(hi, mid); if (s) { hi = mid; ha = ma; } shi |= s;
          s = in_bracket(hi, nl); if (s) { hi = nl; ha = ln; } shi |= s;
        }
        const bool done = any || (!slo && !shi) || (lo.cost < R(0) && lo.slope < R(0) && lo.slope > -gtol) ||
                          (hi.cost < R(0) && hi.slope > R(0) && hi.slope < gtol);
        if (lo.cost < R(0) || hi.cost < R(0)) {
          const bool bl = lo.cost < hi.cost;
          alpha = bl ? la : ha;
          improvement = -(bl ? lo.cost : hi.cost);
        }
        if (done) { converged = true; break; }
      }
    }
    if (TID == 0) {
      A.scal[0] = alpha;
      A.scal[1] = improvement;
      A.iscal[7] += evals;
      if (!converged) A.iscal[3] |= B200_OVERFLOW_LS_ITERATIONS;
    }
  }
  SYNC();
  const R alpha = A.scal[0];
  FOR(i, nv) {
    A.qacc[i] += alpha * A.search[i];
    A.Ma[i] += alpha * A.Mv[i];
  }
  FOR(r, nefc) A.efc_jaref[r] += alpha * A.efc_jv[r];
  SYNC();
}

// Newton solve (mjwarp_solver_state.cu, physics.py:47-70): initial
// gradient/Hessian/direction, then iterations until the world's stop rule.
template <class R, int T> __device__ void newton_init(const Mdl<R> &M, Arena<R> &A) {
  const B200Model &m = M.m;
  const int nv = m.nv, nefc = A.iscal[1];
  const bool warm = !(m.disable_flags & B200_DSBL_WARMSTART);
  FOR(i, nv) A.qacc[i] = warm && nefc > 0 ? A.warm[i] : A.qacc_smooth[i];
  SYNC();
  mass_mul<R, T>(M, A.M, A.qacc, A.Ma);
  FOR(r, nefc) A.efc_jaref[r] = jdot(M, A, r, A.qacc) - A.efc_aref[r];
  if (TID == 0) { A.iscal[4] = 0; A.iscal[5] = m.iterations == 0; A.iscal[14] = 1; }
  SYNC();
  eval_gradient<R, T>(M, A);
  hessian<R, T>(M, A);
  direction<R, T>(M, A);
  mark<T>(A, 9);
}

template <class R, int T> __device__ void newton_iteration(const Mdl<R> &M, Arena<R> &A) {
  const B200Model &m = M.m;
  const R tol = R(m.tolerance), scale = R(m.meaninertia) * R(m.nv);
  linesearch<R, T>(M, A);
  mark<T>(A, 10);
  eval_gradient<R, T>(M, A);
  mark<T>(A, 11);
  hessian<R, T>(M, A);
  mark<T>(A, 12);
  direction<R, T>(M, A);
  mark<T>(A, 13);
  if (TID == 0) {
    const int it = ++A.iscal[4];
    const R imp = A.scal[1] / scale, grad = msqrt(A.scal[3]) / scale, model = (R(0.5) * A.scal[4]) / scale;
    const bool done = A.scal[0] == R(0) || (imp > R(0) && imp < tol) || grad < tol || model < tol;
    if (done || it >= m.iterations) {
      if (!done) A.iscal[3] |= B200_OVERFLOW_ITERATIONS;
      A.iscal[5] = 1;
    }
  }
  SYNC();
}

// ============================================================ Euler
template <class R, int T> __device__ void euler(const Mdl<R> &M, Arena<R> &A) {
  const B200Model &m = M.m;
  const int nv = m.nv;
  const R dt = R(m.timestep);
  const bool damped = !(m.disable_flags & (B200_DSBL_EULERDAMP | B200_DSBL_DAMPER));
  // the mass factor is dead after the smooth solve: reuse it for M + dt*D
  R *acc = A.Mv;
  if (damped) {
    pack_tree_blocks<R, T>(M, A.M, A.H);
    SYNC();
    FOR(d, nv) {
      const int t = IF(dof_treeid)[d], l = d - IF(tree_dofadr)[t];
      A.H[IF(tree_padr)[t] + tri(l, l)] += dt * RF(dof_damping)[d];
      acc[d] = A.Ma[d];
    }
    SYNC();
    tree_solve<R, T>(M, A.H, acc, A.colbuf, true);
  } else
    FOR(d, nv) acc[d] = A.qacc[d];
  SYNC();
  FOR(d, nv) {
    A.warm[d] = A.qacc[d];
    A.qvel[d] = A.qvel[d] + acc[d] * dt;
  }
  SYNC();
  FOR(j, m.njnt) {
    const int kind = IF(jnt_type)[j];
    R *q = A.qpos + IF(jnt_qposadr)[j];
    const R *v = A.qvel + IF(jnt_dofadr)[j];
    if (kind == B200_JNT_FREE) {
      q[0] += dt * v[0]; q[1] += dt * v[1]; q[2] += dt * v[2];
      q += 3; v += 3;
    }
    if (kind == B200_JNT_FREE || kind == B200_JNT_BALL) {
      const R len = msqrt(v[0] * v[0] + v[1] * v[1] + v[2] * v[2]);
      R x = 0, y = 0, z = 0;
      if (len > R(0)) { x = v[0] / len; y = v[1] / len; z = v[2] / len; }
      const R ang = dt * len, s = msin(ang * R(0.5)), c = mcos(ang * R(0.5));
      const Q4<R> r = qnormalize(qmul(qnormalize(ldq(q)), Q4<R>{c, x * s, y * s, z * s}));
      stq(q, r);
    } else q[0] += dt * v[0];
  }
  if (TID == 0) A.scal[5] += dt;
  SYNC();
  // state check (MuJoCo mj_checkPos / mj_checkVel): non-finite or beyond 1e10
  bool bad = false;
  FOR(i, m.nq) bad |= !(mabs(A.qpos[i]) <= R(1e10));
  FOR(i, nv) bad |= !(mabs(A.qvel[i]) <= R(1e10));
  if (bad) atomicOr(&A.iscal[3], B200_STATUS_BADSTATE);
}

// ============================================================ driver
template <class R> __device__ __forceinline__ R *row_of(void *p, int w, int width) {
  return p ? (R *)p + (size_t)w * width : nullptr;
}
__device__ __forceinline__ int *irow_of(int *p, int w, int width) {
  return p ? p + (size_t)w * width : nullptr;
}

template <class R, int T> __device__ void load_world(const B200Model &m, const B200Data &d, Arena<R> &A, int w) {
  const R *src;
  src = row_of<R>(d.qpos, w, m.nq); FOR(i, m.nq) A.qpos[i] = src[i];
  src = row_of<R>(d.qvel, w, m.nv); FOR(i, m.nv) A.qvel[i] = src[i];
  src = row_of<R>(d.qacc_warmstart, w, m.nv); FOR(i, m.nv) A.warm[i] = src[i];
  src = row_of<R>(d.ctrl, w, m.nu); FOR(i, m.nu) A.ctrl[i] = src[i];
  src = row_of<R>(d.goal_pos, w, 3); FOR(i, 3) A.goal_pos[i] = src[i];
  src = row_of<R>(d.goal_rot, w, 9); FOR(i, 9) A.goal_rot[i] = src[i];
  src = row_of<R>(d.gripper, w, 2); FOR(i, 2) A.gripper[i] = src[i];
  if (d.action) { src = row_of<R>(d.action, w, 7); FOR(i, 7) A.action[i] = src[i]; }
  else FOR(i, 7) A.action[i] = 0;
  if (TID == 0) {
    A.scal[5] = row_of<R>(d.time, w, 1)[0];
    for (int k = 0; k < 32; ++k) A.iscal[k] = 0;
    A.iscal[3] = irow_of(d.overflow, w, 1)[0];
    A.iscal[6] = irow_of(d.error, w, 1)[0];
  }
  SYNC();
  // a world handed in with a bad state (MuJoCo mj_checkPos / mj_checkVel) is not stepped
  bool bad = false;
  FOR(i, m.nq) bad |= !(mabs(A.qpos[i]) <= R(1e10));
  FOR(i, m.nv) bad |= !(mabs(A.qvel[i]) <= R(1e10));
  if (bad) atomicOr(&A.iscal[3], B200_STATUS_BADSTATE);
  SYNC();
}

// obs: write the observation slab (it needs this launch's kinematics, which a
// world that did not step has not computed)
template <class R, int T>
__device__ __noinline__ void store_state(const B200Model &m, const B200Data &d, Arena<R> &A, int w, bool obs) {
  R *dst;
  dst = row_of<R>(d.qpos, w, m.nq); FOR(i, m.nq) dst[i] = A.qpos[i];
  dst = row_of<R>(d.qvel, w, m.nv); FOR(i, m.nv) dst[i] = A.qvel[i];
  dst = row_of<R>(d.qacc_warmstart, w, m.nv); FOR(i, m.nv) dst[i] = A.warm[i];
  dst = row_of<R>(d.ctrl, w, m.nu); FOR(i, m.nu) dst[i] = A.ctrl[i];
  dst = row_of<R>(d.goal_pos, w, 3); FOR(i, 3) dst[i] = A.goal_pos[i];
  dst = row_of<R>(d.goal_rot, w, 9); FOR(i, 9) dst[i] = A.goal_rot[i];
  dst = row_of<R>(d.gripper, w, 2); FOR(i, 2) dst[i] = A.gripper[i];
  if ((dst = row_of<R>(d.qacc, w, m.nv))) FOR(i, m.nv) dst[i] = A.qacc[i];
  // observation slab: arm+gripper qpos/qvel (current), end-effector pose and
  // free-body poses (last substep's kinematics, as MuJoCo publishes them)
  if (obs && (dst = row_of<R>(d.obs, w, m.nobs))) {
    const Mdl<R> M(m, model_row(m, d.world_offset, w));
    FOR(e, m.nobs) {
      R v = 0;
      if (e < 18) {
        const int k = e % 9, u = k < 7 ? -1 : IF(osc_actuator)[k];
        const int j = u < 0 ? -1 : IF(actuator_trnid)[u];
        if (e < 9) v = A.qpos[k < 7 ? IF(osc_qposadr)[k] : IF(jnt_qposadr)[j]];
        else v = A.qvel[k < 7 ? IF(osc_dofadr)[k] : IF(jnt_dofadr)[j]];
      } else if (e < 21) v = A.sxpos[3 * m.ee_site + e - 18];
      else if (e < 25) {
        const int s = m.ee_site, b = IF(site_bodyid)[s];
        const Q4<R> q = qmul(ldq(A.xquat + 4 * b), ldq(RF(site_quat) + 4 * s));
        const int c = e - 21;
        v = c == 0 ? q.w : c == 1 ? q.x : c == 2 ? q.y : q.z;
      } else if (e < 25 + 7 * m.nfree) {
        const int f = (e - 25) / 7, c = (e - 25) % 7, b = IF(free_bodyid)[f];
        v = c < 3 ? A.xpos[3 * b + c] : A.xquat[4 * b + c - 3];
      } else if (m.task_body >= 0 && m.task_body < m.nfree) {
        // reward, then done: the task body lifted above task_lift_z (sparse success)
        v = R(A.xpos[3 * IF(free_bodyid)[m.task_body] + 2] > R(m.task_lift_z));
      }
      dst[e] = v;
    }
  }
  if (TID == 0) {
    row_of<R>(d.time, w, 1)[0] = A.scal[5];
    irow_of(d.overflow, w, 1)[0] = A.iscal[3];
    irow_of(d.error, w, 1)[0] = A.iscal[6];
  }
}

// derived outputs of the last substep (pre-integration, as MuJoCo publishes)
template <class R, int T> __device__ __noinline__ void store_outputs(const B200Model &m, const B200Data &d, Arena<R> &A, int w) {
  R *dst;
  const int nb = m.nbody, ng = m.ngeom, ns = m.nsite, nv = m.nv, nc = m.ncon_max;
  if ((dst = row_of<R>(d.xpos, w, nb * 3))) FOR(i, nb * 3) dst[i] = A.xpos[i];
  if ((dst = row_of<R>(d.xquat, w, nb * 4))) FOR(i, nb * 4) dst[i] = A.xquat[i];
  if ((dst = row_of<R>(d.xmat, w, nb * 9))) FOR(i, nb * 9) dst[i] = A.xmat[i];
  if ((dst = row_of<R>(d.geom_xpos, w, ng * 3))) FOR(i, ng * 3) dst[i] = A.gxpos[i];
  if ((dst = row_of<R>(d.geom_xmat, w, ng * 9))) FOR(i, ng * 9) dst[i] = A.gxmat[i];
  if ((dst = row_of<R>(d.site_xpos, w, ns * 3))) FOR(i, ns * 3) dst[i] = A.sxpos[i];
  if ((dst = row_of<R>(d.site_xmat, w, ns * 9))) FOR(i, ns * 9) dst[i] = A.sxmat[i];
  if ((dst = row_of<R>(d.subtree_com, w, nb * 3))) FOR(i, nb * 3) dst[i] = A.com[i];
  if ((dst = row_of<R>(d.qfrc_bias, w, nv))) FOR(i, nv) dst[i] = A.qfrc_bias[i];
  if ((dst = row_of<R>(d.qfrc_actuator, w, nv))) FOR(i, nv) dst[i] = A.qfrc_actuator[i];
  if ((dst = row_of<R>(d.qfrc_constraint, w, nv))) FOR(i, nv) dst[i] = A.qfrc_constraint[i];
  if ((dst = row_of<R>(d.qacc_smooth, w, nv))) FOR(i, nv) dst[i] = A.qacc_smooth[i];
  if ((dst = row_of<R>(d.qfrc_smooth, w, nv))) FOR(i, nv) dst[i] = A.qfrc_smooth[i];
  if ((dst = row_of<R>(d.qM, w, nv * nv))) {
    const Mdl<R> M(m, model_row(m, d.world_offset, w));
    FOR(e, nv * nv) {  // the tree blocks expanded to dense dof order
      const int i = e / nv, j = e % nv, t = IF(dof_treeid)[i], a = IF(tree_dofadr)[t], n = IF(tree_dofnum)[t];
      dst[e] = IF(dof_treeid)[j] == t ? A.M[IF(tree_madr)[t] + (i - a) * n + (j - a)] : R(0);
    }
  }
  const int ncon = A.iscal[0], nefc = A.iscal[1];
  if ((dst = row_of<R>(d.con_dist, w, nc))) FOR(k, ncon) dst[k] = A.con[(size_t)A.con_order[k] * kCWidth + kCDist];
  if ((dst = row_of<R>(d.con_pos, w, nc * 3)))
    FOR(e, ncon * 3) dst[e] = A.con[(size_t)A.con_order[e / 3] * kCWidth + kCPos + e % 3];
  if ((dst = row_of<R>(d.con_frame, w, nc * 9)))
    FOR(e, ncon * 9) dst[e] = A.con[(size_t)A.con_order[e / 9] * kCWidth + kCFrame + e % 9];
  if ((dst = row_of<R>(d.con_friction, w, nc * 5)))
    FOR(e, ncon * 5) dst[e] = A.con[(size_t)A.con_order[e / 5] * kCWidth + kCFriction + e % 5];
  if ((dst = row_of<R>(d.con_margin, w, nc))) FOR(k, ncon) dst[k] = A.con[(size_t)A.con_order[k] * kCWidth + kCMargin];
  if ((dst = row_of<R>(d.efc_force, w, m.nefc_max))) FOR(r, nefc) dst[r] = A.efc_force[r];
  if ((dst = row_of<R>(d.efc_D, w, m.nefc_max))) FOR(r, nefc) dst[r] = A.efc_D[r];
  if ((dst = row_of<R>(d.efc_aref, w, m.nefc_max))) FOR(r, nefc) dst[r] = A.efc_aref[r];
  if ((dst = row_of<R>(d.efc_J, w, m.nefc_max * nv))) {
    const Mdl<R> M(m, model_row(m, d.world_offset, w));
    FOR(e, nefc * nv) {  // rows expanded to dense dof order
      const int r = e / nv, dof = e % nv, t0 = A.row_t[2 * r], t1 = A.row_t[2 * r + 1];
      const int n0 = t0 >= 0 ? IF(tree_dofnum)[t0] : 0, td = IF(dof_treeid)[dof], off = dof - IF(tree_dofadr)[td];
      const R *row = A.J + (size_t)r * m.kmax_dof;
      dst[e] = td == t0 ? row[off] : td == t1 ? row[n0 + off] : R(0);
    }
  }
  int *idst;
  if ((idst = irow_of(d.efc_type, w, m.nefc_max))) FOR(r, nefc) idst[r] = A.efc_type[r];
  if ((idst = irow_of(d.efc_id, w, m.nefc_max))) FOR(r, nefc) {
    int id = A.efc_id[r];  // contact rows: the contact's slot, published as its sorted index
    if (A.efc_type[r] >= 5)
      for (int k = 0; k < ncon; ++k)
        if (A.con_order[k] == id) { id = k; break; }
    idst[r] = id;
  }
  if ((idst = irow_of(d.con_dim, w, nc))) FOR(k, ncon) idst[k] = A.con_dim[A.con_order[k]];
  if ((idst = irow_of(d.con_geom, w, nc * 2)))
    FOR(e, ncon * 2) idst[e] = e & 1 ? A.con_g2[A.con_order[e >> 1]] : A.con_g1[A.con_order[e >> 1]];
  if (TID == 0) {
    if (d.ncon) irow_of(d.ncon, w, 1)[0] = ncon;
    if (d.nefc) irow_of(d.nefc, w, 1)[0] = nefc;
  }
}


// A CTA holds `wpc` worlds in consecutive shared-memory arenas.  The worlds
// advance through the stages of a substep together (CTA barrier after every
// stage) so that co-resident warps execute the same code region and the
// instruction caches serve them all; the Newton loop runs until every world of
// the CTA has met its stop rule, worlds already done idle.  Warps past the last
// world take part in the barriers only.
#define STAGE(call, k)       \
  do {                       \
    if (act) {               \
      call;                  \
      mark<T>(A, k);         \
    }                        \
    __syncthreads();         \
    if (act) mark<T>(A, 15); \
  } while (0)

// factor of the mass matrix, one block per kinematic tree (mjwarp_mass_factor.cu)
template <class R, int T> __device__ void mass_factor(const Mdl<R> &M, Arena<R> &A) {
  pack_tree_blocks<R, T>(M, A.M, A.L);
  SYNC();
  chol_blocks(A.L, TREE_ROWS(T), M.m.max_tree_dofs, M.m.nv, A.colbuf);
  SYNC();
}

// Position and velocity stages (reference Physics.step1, physics.py:161-186).
// RNE (velocity) runs before collision: the two touch disjoint data, and the
// control step then overlaps the FP64 OSC, which needs RNE's bias forces, with
// collision.
template <class R, int T> __device__ void position_velocity_stages(const Mdl<R> &M, Arena<R> &A, bool act) {
  STAGE((kinematics<R, T>(M, A)), 1);
  STAGE((com_crb_mass<R, T>(M, A)), 2);
  STAGE((mass_factor<R, T>(M, A)), 3);
  STAGE((velocity<R, T>(M, A)), 6);
}

// Constraint rows and actuation: the two are independent; a world of several
// warps runs actuation on its other warps while its first warp allocates the
// rows (then all its threads fill them); a one-warp world runs them in turn.
template <class R, int T> __device__ void constraints_and_actuation(const Mdl<R> &M, Arena<R> &A) {
  if constexpr (T >= 64) {
    constraints<R, T, true>(M, A);
  } else {
    constraints<R, T>(M, A);
    mark<T>(A, 5);
    actuation<R, T>(M, A);
  }
}

// Collision and the FP64 OSC.  A world of several warps runs the OSC on its
// first warp while its other warps run the broadphase and narrowphase (the
// collision lists then start after the OSC's scratch in the union region); a
// one-warp world runs them one after the other.
template <class R, int T, int CONVEX> __device__ void collide_and_control(const Mdl<R> &M, Arena<R> &A, bool policy) {
  if constexpr (T >= 64) {
    if (TID < 32) osc_control<R, T, 32>(M, A, policy);
    else collision<R, T, CONVEX, 32, T - 32>(M, A, Arena<R>::kOscDoubles * (int)sizeof(double));
    SYNC();
  } else {
    collision<R, T, CONVEX, 0, T>(M, A, 0);
    mark<T>(A, 4);
    osc_control<R, T, T>(M, A, policy);
  }
}

template <class R, int T> __device__ void newton_stages(const Mdl<R> &M, Arena<R> &A, bool act) {
  STAGE((newton_init<R, T>(M, A)), 0);
  while (__syncthreads_or(act && !A.iscal[5])) {
    if (act) mark<T>(A, 15);  // barrier wait and idle iterations of worlds already done
    if (act && !A.iscal[5]) newton_iteration<R, T>(M, A);
  }
  if (act) mark<T>(A, 15);
}

template <class R, int CONVEX, int T>
__global__ void __launch_bounds__(384, 1) control_step(const __grid_constant__ B200Model m, const __grid_constant__ B200Data d,
                                                     int substeps, int policy, int wpc, int arena) {
  static_assert(T % 32 == 0 && T / 32 <= Arena<R>::kColbufWarps, "per-warp scratch covers at most four warps");
  extern __shared__ __align__(16) unsigned char smem[];
  const int slot = threadIdx.x / T, i = blockIdx.x * wpc + slot;
  const bool in = slot < wpc && i < d.nworld;
  // the world of this slot: d.order[i] when a grouping is given (a permutation)
  int w = i;
  if (in && d.order) {
    const int o = d.order[i];
    w = o >= 0 && o < d.nworld ? o : i;
  }
  bool act = in;  // the world steps; false once its state went bad (B200_STATUS_BADSTATE)
  // the world's arena descriptor heads its shared-memory region (one copy per
  // world, read by broadcast instead of a per-thread local-memory copy)
  unsigned char *wbase = smem + (size_t)(slot < wpc ? slot : 0) * arena;
  Arena<R> &A = *reinterpret_cast<Arena<R> *>(wbase);
  if (slot < wpc && TID == 0) Arena<R>::layout(m, T, &A, wbase);
  __syncthreads();
  const Mdl<R> M(m, model_row(m, d.world_offset, w));
  if (act) {
    load_world<R, T>(m, d, A, w);
    if (TID == 0 && d.stage_cycles) {
      A.iscal[10] = 1;
      for (int k = 0; k < 16; ++k) A.prof[k] = 0;
      A.prof[0] = clock64();
    }
    SYNC();
  }
  __syncthreads();
  int stepped = 0, work = 0;  // work: kept by the world's thread 0
  for (int s = 0; s < substeps; ++s) {
    // world-uniform: the status word is read after a CTA barrier
    if (act && (A.iscal[3] & B200_STATUS_BADSTATE)) act = false;
    position_velocity_stages<R, T>(M, A, act);
    STAGE((collide_and_control<R, T, CONVEX>(M, A, policy && s == 0)), 7);
    STAGE((constraints_and_actuation<R, T>(M, A)), 8);
    newton_stages<R, T>(M, A, act);
    if (act && TID == 0) {
      const int it = A.iscal[4], nefc = A.iscal[1], evals = A.iscal[7] - A.iscal[9];
      A.iscal[9] = A.iscal[7];
      if (d.niter) irow_of(d.niter, w, 1)[0] = it;
      if (d.newton_total) irow_of(d.newton_total, w, 1)[0] += it;
      if (d.efc_total) irow_of(d.efc_total, w, 1)[0] += nefc;
      if (d.con_total) irow_of(d.con_total, w, 1)[0] += A.iscal[0];
      if (d.newton_rows) irow_of(d.newton_rows, w, 1)[0] += it * nefc;
      if (d.ls_rows) irow_of(d.ls_rows, w, 1)[0] += evals * nefc;
      if (d.efc_k) irow_of(d.efc_k, w, 1)[0] += A.iscal[15];
      if (d.efc_k2) irow_of(d.efc_k2, w, 1)[0] += A.iscal[23];
      if (d.fact_blk) irow_of(d.fact_blk, w, 1)[0] += A.iscal[24];
      A.iscal[24] = 0;
      if (s < 32 && d.niter_trace) irow_of(d.niter_trace, w, 32)[s] = it;
      if (s < 32 && d.ls_trace) irow_of(d.ls_trace, w, 32)[s] = evals;
      // a GJK / EPA pair stalls its world's collision stage about as long as
      // 1500 work units of Newton rows do: worlds with such pairs share CTAs
      work += (it + 1) * (nefc + 32) + 4 * A.iscal[0] + 1500 * A.iscal[25];
    }
    if (act && s == substeps - 1) store_outputs<R, T>(m, d, A, w);
    STAGE((euler<R, T>(M, A)), 14);
    stepped += act;
  }
  if (!in) return;
  if (TID == 0) {
    if (d.ls_total) irow_of(d.ls_total, w, 1)[0] += A.iscal[7];
    if (d.integration_count) irow_of(d.integration_count, w, 1)[0] += stepped;
    if (d.work) irow_of(d.work, w, 1)[0] = work;
  }
  store_state<R, T>(m, d, A, w, stepped > 0);
  if (TID == 0 && d.stage_cycles) {
    int *out = irow_of(d.stage_cycles, w, 16);
    for (int k = 1; k < 16; ++k) out[k] += (int)A.prof[k];
  }
}

template <class R, int CONVEX, int T>
__global__ void __launch_bounds__(384, 1) forward_step(const __grid_constant__ B200Model m, const __grid_constant__ B200Data d,
                                                     int bootstrap, const int *mask, int wpc, int arena) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int slot = threadIdx.x / T, w = blockIdx.x * wpc + slot;
  const bool act = slot < wpc && w < d.nworld && (!mask || mask[w]);
  unsigned char *wbase = smem + (size_t)(slot < wpc ? slot : 0) * arena;
  Arena<R> &A = *reinterpret_cast<Arena<R> *>(wbase);
  if (slot < wpc && TID == 0) Arena<R>::layout(m, T, &A, wbase);
  __syncthreads();
  const Mdl<R> M(m, model_row(m, d.world_offset, w));
  if (act) load_world<R, T>(m, d, A, w);
  __syncthreads();
  position_velocity_stages<R, T>(M, A, act);
  STAGE((collision<R, T, CONVEX, 0, T>(M, A, 0)), 4);
  STAGE((constraints<R, T>(M, A)), 5);
  if (act && bootstrap) {
    FOR(i, 3) A.goal_pos[i] = A.sxpos[3 * m.ee_site + i];
    FOR(i, 9) A.goal_rot[i] = A.sxmat[9 * m.ee_site + i];
    FOR(i, 2) A.gripper[i] = 0;
    if (TID == 0) A.iscal[6] = 0;
    SYNC();
  }
  STAGE((actuation<R, T>(M, A)), 8);
  newton_stages<R, T>(M, A, act);
  if (!act) return;
  if (TID == 0 && d.niter) irow_of(d.niter, w, 1)[0] = A.iscal[4];
  store_outputs<R, T>(m, d, A, w);
  store_state<R, T>(m, d, A, w, true);
}

}  // namespace b200

namespace b200 {
template <class R, int C, int T> int configure_kernels(size_t smem) {
  int rc = (int)cudaFuncSetAttribute(control_step<R, C, T>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (rc) return rc;
  return (int)cudaFuncSetAttribute(forward_step<R, C, T>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
}
template <class R, int C, int T>
void launch_step(const B200Model &m, const B200Data &d, int substeps, int policy, int wpc, int arena, int grid,
                 size_t smem, cudaStream_t s) {
  control_step<R, C, T><<<grid, T * wpc, smem, s>>>(m, d, substeps, policy, wpc, arena);
}
template <class R, int C, int T>
void launch_forward(const B200Model &m, const B200Data &d, int bootstrap, const int *mask, int wpc, int arena,
                    int grid, size_t smem, cudaStream_t s) {
  forward_step<R, C, T><<<grid, T * wpc, smem, s>>>(m, d, bootstrap, mask, wpc, arena);
}
}  // namespace b200
