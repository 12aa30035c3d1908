// Portions (sphere_box, capsule_box, box_box, clip_poly, and the box manifold
// box_manifold / clip_faces / largest_quad) restate MuJoCo Warp's contact
// geometry: Copyright 2025 The Newton Developers,
// SPDX-License-Identifier: Apache-2.0 (see NOTICE).
// Per-pair collision for one world: broadphase filters and primitive
// narrowphase.  One thread owns one candidate pair; contacts are appended to
// the world's shared-memory contact table and later ordered by
// (pair index, collision id), which makes the per-world contact list
// deterministic (the reference appends to a global pool with atomics:
// libero/libero/gpu/cuda/collision/mjwarp_broadphase.cu:110,
// mjwarp_contact.cuh:107).
//
// The decision steps are those of the reference colliders, because contact
// lists must agree exactly:
//   filters   mjwarp_broadphase.cu:21-96 (plane / bounding sphere / 6-axis OBB)
//   plane     mjwarp_plane.cu:18-60 (sphere, capsule, box)
//   box       mjwarp_box.cu:14-176 (sphere-box, capsule-box, box-box SAT+clip)
//   material  mjwarp_contact.cuh:60-98
// plus the sphere/capsule primitives, plane-mesh and the convex (GJK/EPA)
// pairs of dropped objects (see the sections below).
#pragma once
#include "arena.cuh"
#include "math.cuh"

namespace b200 {

template <class R> struct Mdl {
  const B200Model &m;
  const R *f;
  const int *i;
  // row: the world's copy of the real arrays (per-world parameter rows)
  __device__ Mdl(const B200Model &m_, int row = 0)
      : m(m_), f((const R *)m_.real + (size_t)row * (size_t)m_.variant_stride), i(m_.ints) {}
};
// The parameter row of world w of a shard: the global world index modulo the
// number of rows (mjwarp_constraint_build.cu:18-20, w % p.rows), so that a
// world's parameters do not depend on how worlds are split over GPUs.
__device__ inline int model_row(const B200Model &m, int world_offset, int w) {
  return m.nvariant > 1 ? (int)(((long long)world_offset + w) % m.nvariant) : 0;
}
#define RF(name) (M.f + M.m.off_##name)
#define IF(name) (M.i + M.m.off_##name)

template <class R> struct Material {
  int dim;
  R margin, gap, friction[5], solref[2], solreffriction[2], solimp[5];
};

template <class R> __device__ Material<R> material(const Mdl<R> &M, int g1, int g2) {
  Material<R> p;
  p.margin = RF(geom_margin)[g1] + RF(geom_margin)[g2];
  p.gap = RF(geom_gap)[g1] + RF(geom_gap)[g2];
  R m1 = RF(geom_solmix)[g1], m2 = RF(geom_solmix)[g2], mix;
  const R *f1 = RF(geom_friction) + 3 * g1, *f2 = RF(geom_friction) + 3 * g2;
  R f[3];
  const int p1 = IF(geom_priority)[g1], p2 = IF(geom_priority)[g2];
  const int c1 = IF(geom_condim)[g1], c2 = IF(geom_condim)[g2];
  if (p1 > p2) {
    mix = 1; p.dim = c1;
    for (int c = 0; c < 3; ++c) f[c] = f1[c];
  } else if (p2 > p1) {
    mix = 0; p.dim = c2;
    for (int c = 0; c < 3; ++c) f[c] = f2[c];
  } else {
    mix = m1 + m2 != R(0) ? m1 / (m1 + m2) : R(0);
    if (m1 < R(1e-15) && m2 < R(1e-15)) mix = R(0.5);
    if (m1 < R(1e-15) && m2 >= R(1e-15)) mix = 0;
    if (m1 >= R(1e-15) && m2 < R(1e-15)) mix = 1;
    p.dim = c1 > c2 ? c1 : c2;
    for (int c = 0; c < 3; ++c) f[c] = mmax(f1[c], f2[c]);
  }
  p.friction[0] = f[0]; p.friction[1] = f[0]; p.friction[2] = f[1]; p.friction[3] = f[2]; p.friction[4] = f[2];
  const R *r1 = RF(geom_solref) + 2 * g1, *r2 = RF(geom_solref) + 2 * g2;
  const R *i1 = RF(geom_solimp) + 5 * g1, *i2 = RF(geom_solimp) + 5 * g2;
  for (int c = 0; c < 2; ++c) {
    p.solref[c] = r1[0] > R(0) && r2[0] > R(0) ? mix * r1[c] + (R(1) - mix) * r2[c] : mmin(r1[c], r2[c]);
    p.solreffriction[c] = 0;
  }
  for (int c = 0; c < 5; ++c) p.solimp[c] = mix * i1[c] + (R(1) - mix) * i2[c];
  for (int c = 0; c < 5; ++c) p.friction[c] = mmax(R(1e-5), p.friction[c]);
  return p;
}

template <class R> __device__ void frame_from_normal(V3<R> a, V3<R> *f) {
  a = normalize(a);
  V3<R> b = (R(-0.5) < a.y && a.y < R(0.5)) ? v3<R>(0, 1, 0) : v3<R>(0, 0, 1);
  b = normalize(b - a * dot(a, b));
  if (msqrt(dot(a, a)) == R(0)) b = v3<R>(0, 0, 0);
  f[0] = a; f[1] = b; f[2] = cross(a, b);
}

// Append one contact if it is within margin+gap. Returns nothing; capacity
// overflow sets the world's narrowphase overflow bit.
template <class R>
__device__ void emit(const Mdl<R> &M, Arena<R> &A, const Material<R> &p, int pair, int id, int g1, int g2, R dist,
                     V3<R> pos, const V3<R> *frame) {
  if (!(dist < p.margin + p.gap)) return;
  int slot = atomicAdd(&A.iscal[8], 1);
  if (slot >= M.m.ncon_max) {
    atomicOr(&A.iscal[3], B200_OVERFLOW_NARROWPHASE);
    return;
  }
  R *c = A.con + (size_t)slot * kCWidth;
  c[kCDist] = dist;
  st3(c + kCPos, pos);
  st3(c + kCFrame, frame[0]); st3(c + kCFrame + 3, frame[1]); st3(c + kCFrame + 6, frame[2]);
  c[kCMargin] = p.margin;
  for (int k = 0; k < 5; ++k) c[kCFriction + k] = p.friction[k];
  A.con_dim[slot] = p.dim;
  A.con_g1[slot] = g1;
  A.con_g2[slot] = g2;
  A.con_key[slot] = pair * 16 + id;
}

// ---------------------------------------------------------------- filters
template <class R> __device__ bool obb_overlap(V3<R> c1, V3<R> c2, V3<R> s1, V3<R> s2, R margin, V3<R> p1, V3<R> p2,
                                               const R *R1, const R *R2) {
  V3<R> cen[2] = {rot(R1, c1) + p1, rot(R2, c2) + p2};
  V3<R> nrm[6] = {col(R1, 0), col(R1, 1), col(R1, 2), col(R2, 0), col(R2, 1), col(R2, 2)};
  V3<R> siz[2] = {s1, s2};
  for (int j = 0; j < 2; ++j)
    for (int a = 0; a < 3; ++a) {
      const V3<R> axis = nrm[3 * j + a];
      R proj[2], rad[2];
      for (int i = 0; i < 2; ++i) {
        proj[i] = dot(cen[i], axis);
        rad[i] = mabs(siz[i].x * dot(nrm[3 * i], axis)) + mabs(siz[i].y * dot(nrm[3 * i + 1], axis)) +
                 mabs(siz[i].z * dot(nrm[3 * i + 2], axis));
      }
      if (rad[0] + rad[1] + margin < mabs(proj[1] - proj[0])) return false;
    }
  return true;
}

template <class R> __device__ bool candidate(const Mdl<R> &M, const Arena<R> &A, int g1, int g2) {
  const R *aabb = RF(geom_aabb);
  const R r1 = RF(geom_rbound)[g1], r2 = RF(geom_rbound)[g2];
  const R m1 = RF(geom_margin)[g1] + RF(geom_gap)[g1], m2 = RF(geom_margin)[g2] + RF(geom_gap)[g2];
  const V3<R> p1 = ld3(A.gxpos + 3 * g1), p2 = ld3(A.gxpos + 3 * g2);
  const R *R1 = A.gxmat + 9 * g1, *R2 = A.gxmat + 9 * g2;
  if (r1 == R(0)) return dot(p2 - p1, col(R1, 2)) <= r2 + m1 + m2;
  if (r2 == R(0)) return dot(p1 - p2, col(R2, 2)) <= r1 + m1 + m2;
  const R bound = r1 + r2 + m1 + m2;
  const V3<R> d = p2 - p1;
  if (!(dot(d, d) <= bound * bound)) return false;
  return obb_overlap(ld3(aabb + 6 * g1), ld3(aabb + 6 * g2), ld3(aabb + 6 * g1 + 3), ld3(aabb + 6 * g2 + 3), m1 + m2,
                     p1, p2, R1, R2);
}

// ---------------------------------------------------------------- plane
template <class R>
__device__ void plane_pair(const Mdl<R> &M, Arena<R> &A, int pair, int g1, int g2) {
  const Material<R> p = material(M, g1, g2);
  const V3<R> o = ld3(A.gxpos + 3 * g1), c = ld3(A.gxpos + 3 * g2), n = col(A.gxmat + 9 * g1, 2);
  const R *Rg = A.gxmat + 9 * g2;
  const V3<R> size = ld3(RF(geom_size) + 3 * g2);
  const int type = IF(geom_type)[g2];
  V3<R> fr[3];
  if (type == B200_GEOM_SPHERE) {
    frame_from_normal(n, fr);
    const R d = dot(c - o, n) - size.x;
    emit(M, A, p, pair, 0, g1, g2, d, c - n * (size.x + R(0.5) * d), fr);
  } else if (type == B200_GEOM_CAPSULE) {
    const V3<R> ax = col(Rg, 2);
    const V3<R> t = ax - n * dot(n, ax);
    const R len = msqrt(dot(t, t));
    V3<R> b = len == R(0) ? t : t * (R(1) / len);
    if (len < R(0.5)) b = (R(-0.5) < n.y && n.y < R(0.5)) ? v3<R>(0, 1, 0) : v3<R>(0, 0, 1);
    fr[0] = n; fr[1] = b; fr[2] = cross(n, b);
    for (int e = 0; e < 2; ++e) {
      const V3<R> end = e == 0 ? c + ax * size.y : c - ax * size.y;
      const R d = dot(end - o, n) - size.x;
      emit(M, A, p, pair, e, g1, g2, d, end - n * (size.x + R(0.5) * d), fr);
    }
  } else if (type == B200_GEOM_BOX) {
    frame_from_normal(n, fr);
    const R cd = dot(c - o, n);
    for (int i = 0; i < 8; ++i) {
      const V3<R> corner = rot(Rg, v3<R>(i & 1 ? size.x : -size.x, i & 2 ? size.y : -size.y, i & 4 ? size.z : -size.z));
      const R d = cd + dot(n, corner);
      emit(M, A, p, pair, i, g1, g2, d, corner + c - n * (R(0.5) * d), fr);
    }
  }
}

// ---------------------------------------------------------------- box family
template <class R> struct BoxHits {
  int count;
  R dist[8];
  V3<R> pos[8], normal[8];
};

template <class R>
__device__ __noinline__ void sphere_box(BoxHits<R> &o, int id, V3<R> sphere, R radius, V3<R> center, const R *Rb, V3<R> size) {
  const V3<R> local = rotT(Rb, sphere - center);
  V3<R> clamped;
  for (int c = 0; c < 3; ++c) clamped[c] = mclamp(local[c], -size[c], size[c]);
  V3<R> dir = clamped - local;
  const R dist = msqrt(dot(dir, dir));
  dir = dist == R(0) ? dir : dir * (R(1) / dist);
  V3<R> pos, normal;
  if (dist <= R(1e-15)) {
    R closest = R(2) * (size.x + size.y + size.z);
    int face = 0;
    for (int i = 0; i < 6; ++i) {
      const R d = mabs((i % 2 ? R(1) : R(-1)) * size[i / 2] - local[i / 2]);
      if (closest > d) { closest = d; face = i; }
    }
    V3<R> nearest = v3<R>(0, 0, 0);
    nearest[face / 2] = face % 2 ? R(-1) : R(1);
    pos = local + nearest * ((radius - closest) * R(0.5));
    normal = rot(Rb, nearest);
    o.dist[id] = -closest - radius;
  } else {
    const V3<R> deepest = local + dir * radius;
    pos = (clamped + deepest) * R(0.5);
    normal = rot(Rb, dir);
    o.dist[id] = dist - radius;
  }
  o.pos[id] = center + rot(Rb, pos);
  o.normal[id] = normal;
}

template <class R>
__device__ __noinline__ void capsule_box(BoxHits<R> &o, V3<R> center, V3<R> axis, R radius, R hl, V3<R> bc, const R *Rb, V3<R> size) {
  o.count = 2;
  const V3<R> pos = rotT(Rb, center - bc);
  axis = rotT(Rb, axis);
  const V3<R> ha = axis * hl;
  const int axisdir = int(ha.x > R(0)) + 2 * int(ha.y > R(0)) + 4 * int(ha.z > R(0));
  R bestdist = R(1e32), bestseg = R(-12), bestbox = 0;
  int type = -4, face = -12, corner = -123, edge = -123;
  for (int i = -1; i <= 1; i += 2) {
    const V3<R> tip = pos + ha * R(i);
    V3<R> point = tip;
    int outside = 0, ax = -1;
    for (int j = 0; j < 3; ++j) {
      if (point[j] < -size[j]) { ++outside; ax = j; point[j] = -size[j]; }
      else if (point[j] > size[j]) { ++outside; ax = j; point[j] = size[j]; }
    }
    if (outside > 1) continue;
    const V3<R> dif = point - tip;
    const R d = dot(dif, dif);
    if (d < bestdist) { bestdist = d; bestseg = R(i); type = -2 + i; face = ax; }
  }
  for (int i = 0; i < 8; ++i)
    for (int j = 0; j < 3; ++j) {
      if (i & (1 << j)) continue;
      V3<R> point = v3<R>((i & 1 ? R(1) : R(-1)) * size.x, (i & 2 ? R(1) : R(-1)) * size.y, (i & 4 ? R(1) : R(-1)) * size.z);
      point[j] = 0;
      V3<R> dif = point - pos;
      const R u = -size[j] * dif[j], v = dot(ha, dif), ma = size[j] * size[j], mb = -size[j] * ha[j], mc = hl * hl;
      const R det = ma * mc - mb * mb;
      if (mabs(det) < R(1e-15)) continue;
      const R inv = R(1) / det;
      R x1 = (mc * u - mb * v) * inv, x2 = (ma * v - mb * u) * inv;
      int s1 = 1, s2 = 1;
      if (x1 > R(1)) { x1 = 1; s1 = 2; x2 = safe_div(v - mb, mc); }
      else if (x1 < R(-1)) { x1 = -1; s1 = 0; x2 = safe_div(v + mb, mc); }
      const bool over = x2 > R(1);
      if (over || x2 < R(-1)) {
        if (over) { x2 = 1; s2 = 2; x1 = safe_div(u - mb, ma); }
        else { x2 = -1; s2 = 0; x1 = safe_div(u + mb, ma); }
        if (x1 > R(1)) { x1 = 1; s1 = 2; } else if (x1 < R(-1)) { x1 = -1; s1 = 0; }
      }
      dif = dif - ha * x2;
      dif[j] += size[j] * x1;
      const R d = dot(dif, dif);
      const int config = s1 * 3 + s2;
      if (d < bestdist - R(1e-15)) {
        bestdist = d; bestseg = x2; bestbox = x1; corner = i + (1 << j) * (config / 6); edge = j; type = config;
      }
    }
  if (type == -4) { o.count = 0; return; }
  R second = -4;
  if (type >= 0 && type / 3 != 1) {
    int config = axisdir ^ corner;
    if (config != 0 && config != 7) {
      int mul;
      if (config == 1 || config == 2 || config == 4) mul = 1;
      else { mul = -1; config = 7 - config; }
      const int ax = config == 1 ? 0 : config == 2 ? 1 : 2, ax1 = (ax + 1) % 3, ax2 = (ax + 2) % 3;
      if (axis[ax] * axis[ax] > R(0.5)) {
        const R mm = R(2) * safe_div(size[ax], mabs(ha[ax]));
        second = mmin(R(1) - R(mul) * bestseg, mm);
      } else {
        const R mm = R(2) * mmin(safe_div(size[ax1], mabs(ha[ax1])), safe_div(size[ax2], mabs(ha[ax2])));
        second = -mmin(R(1) + R(mul) * bestseg, mm);
      }
      second *= R(mul);
    }
  } else if (type >= 0 && type / 3 == 1) {
    const int config = (axisdir ^ corner) & (7 - (1 << edge));
    if (config == 1 || config == 2 || config == 4) {
      const int ax = edge;
      int ax1 = (edge + 1) % 3, ax2 = (edge + 2) % 3;
      if (mabs(axis[ax1]) > mabs(axis[ax2])) ax1 = ax2;
      ax2 = 3 - ax - ax1;
      int mul;
      if (config & (1 << ax2)) { mul = 1; second = R(1) - bestseg; }
      else { mul = -1; second = R(1) + bestseg; }
      R e1 = R(2) * safe_div(size[ax2], mabs(ha[ax2]));
      second = mmin(e1, second);
      const R e2 = bool(axisdir & (1 << ax)) == bool(config & (1 << ax2)) ? R(1) - bestbox : R(1) + bestbox;
      e1 = size[ax] * safe_div(e2, mabs(ha[ax]));
      second = mmin(e1, second);
      second *= R(mul);
    }
  } else if (type < 0 && face != -1) {
    const int mul = type == -3 ? 1 : -1;
    second = 2;
    const V3<R> tmp = pos - ha * R(mul);
    for (int i = 0; i < 3; ++i)
      if (i != face) {
        const R inv = safe_div(R(mul), ha[i]);
        R e1 = (size[i] - tmp[i]) * inv;
        if (R(0) < e1 && e1 < second) second = e1;
        e1 = (-size[i] - tmp[i]) * inv;
        if (R(0) < e1 && e1 < second) second = e1;
      }
    second *= R(mul);
  }
  sphere_box(o, 0, rot(Rb, pos + ha * bestseg) + bc, radius, bc, Rb, size);
  if (second > R(-3)) sphere_box(o, 1, rot(Rb, pos + ha * (second + bestseg)) + bc, radius, bc, Rb, size);
  else o.dist[1] = R(1e10);
}

template <class R> __device__ __noinline__ int clip_poly(int count, V3<R> *poly, int coord, R sign, R limit) {
  R d[8];
  bool inside = true;
  for (int i = 0; i < count; ++i) {
    d[i] = sign * poly[i][coord] - limit;
    if (!(d[i] <= R(0))) inside = false;
  }
  if (inside) return count;
  V3<R> out[8];
  for (int i = 0; i < 8; ++i) out[i] = v3<R>(0, 0, 0);
  int n = 0;
  for (int i = 0; i < count; ++i) {
    const int nx = i + 1 == count ? 0 : i + 1;
    const R dp = d[i], dq = d[nx];
    if (dp <= R(0) && n < 8) out[n++] = poly[i];
    if (((dp < R(0) && dq > R(0)) || (dp > R(0) && dq < R(0))) && n < 8) {
      const R t = dp / (dp - dq);
      out[n++] = poly[i] + (poly[nx] - poly[i]) * t;
    }
  }
  for (int i = 0; i < 8; ++i) poly[i] = out[i];
  return n;
}

template <class R>
__device__ __noinline__ void box_box(BoxHits<R> &o, V3<R> p1, const R *R1, V3<R> s1, V3<R> p2, const R *R2, V3<R> s2, R margin) {
  o.count = 0;
  const V3<R> pos21 = rotT(R1, p2 - p1), pos12 = rotT(R2, p1 - p2);
  R rm[9], ab[9];
  for (int i = 0; i < 3; ++i)
    for (int j = 0; j < 3; ++j) {
      rm[3 * i + j] = dot(col(R1, i), col(R2, j));
      ab[3 * i + j] = mabs(rm[3 * i + j]);
    }
  const R septol = margin + R(1e-6) * (s1.x + s1.y + s1.z + s2.x + s2.y + s2.z);
  R best = R(-1e10);
  int code = -1;
  for (int i = 0; i < 3; ++i) {
    const R rad = ab[3 * i] * s2.x + ab[3 * i + 1] * s2.y + ab[3 * i + 2] * s2.z;
    const R sep = mabs(pos21[i]) - s1[i] - rad;
    if (sep > septol) return;
    if (sep > best) { best = sep; code = i; }
  }
  for (int j = 0; j < 3; ++j) {
    const R rad = ab[j] * s1.x + ab[3 + j] * s1.y + ab[6 + j] * s1.z;
    const R sep = mabs(pos12[j]) - s2[j] - rad;
    if (sep > septol) return;
    if (sep > best) { best = sep; code = 3 + j; }
  }
  const R face_best = best;
  const int face_code = code;
  for (int i = 0; i < 3; ++i)
    for (int j = 0; j < 3; ++j) {
      const int i1 = (i + 1) % 3, i2 = (i + 2) % 3;
      R x = -rm[3 * i2 + j], y = rm[3 * i1 + j];
      const R n2 = x * x + y * y;
      if (n2 < R(1e-7)) continue;
      const R inv = R(1) / msqrt(n2);
      x *= inv; y *= inv;
      const R rad1 = s1[i1] * mabs(x) + s1[i2] * mabs(y);
      const int j1 = (j + 1) % 3, j2 = (j + 2) % 3;
      const R a1 = x * rm[3 * i1 + j1] + y * rm[3 * i2 + j1], a2 = x * rm[3 * i1 + j2] + y * rm[3 * i2 + j2];
      const R rad2 = s2[j1] * mabs(a1) + s2[j2] * mabs(a2);
      const R sep = mabs(x * pos21[i1] + y * pos21[i2]) - rad1 - rad2;
      if (sep > septol) return;
      if (sep - R(1e-6) * mabs(sep) > best && sep > face_best) { best = sep; code = 6 + 3 * i + j; }
    }
  if (code < 0) return;
  int ei = 0, ej = 0, i1 = 0, i2 = 0;
  V3<R> axis = v3<R>(0, 0, 0);
  if (code >= 6) {
    ei = (code - 6) / 3; ej = (code - 6) % 3; i1 = (ei + 1) % 3; i2 = (ei + 2) % 3;
    axis[i1] = -rm[3 * i2 + ej];
    axis[i2] = rm[3 * i1 + ej];
    axis = normalize(axis);
    const R align = face_code < 3 ? mabs(axis[face_code]) : mabs(dot(axis, col(rm, face_code - 3)));
    if (align > R(0.99) && best < face_best + R(0.05) * mabs(face_best) + R(1e-15)) { code = face_code; best = face_best; }
  }
  if (code >= 6) {
    const int j1 = (ej + 1) % 3, j2 = (ej + 2) % 3;
    if (dot(axis, pos21) < R(0)) axis = -axis;
    const V3<R> a2 = rotT(rm, axis);
    int amb1 = -1, amb2 = -1;
    if (mabs(axis[i1]) < R(1e-5)) amb1 = i1; else if (mabs(axis[i2]) < R(1e-5)) amb1 = i2;
    if (mabs(a2[j1]) < R(1e-5)) amb2 = j1; else if (mabs(a2[j2]) < R(1e-5)) amb2 = j2;
    const V3<R> d2 = col(rm, ej);
    const R b = d2[ei], denom = R(1) - b * b;
    R best_dist = R(1e10);
    V3<R> w1 = v3<R>(0, 0, 0), w2 = v3<R>(0, 0, 0);
    for (int u1 = 0; u1 < (amb1 >= 0 ? 2 : 1); ++u1)
      for (int u2 = 0; u2 < (amb2 >= 0 ? 2 : 1); ++u2) {
        V3<R> c1 = v3<R>(0, 0, 0);
        c1[i1] = axis[i1] >= R(0) ? s1[i1] : -s1[i1];
        c1[i2] = axis[i2] >= R(0) ? s1[i2] : -s1[i2];
        if (amb1 >= 0 && u1) c1[amb1] = -c1[amb1];
        V3<R> cr = v3<R>(0, 0, 0);
        cr[j1] = a2[j1] >= R(0) ? -s2[j1] : s2[j1];
        cr[j2] = a2[j2] >= R(0) ? -s2[j2] : s2[j2];
        if (amb2 >= 0 && u2) cr[amb2] = -cr[amb2];
        const V3<R> c2 = rot(rm, cr) + pos21, e = c2 - c1;
        const R d1e = e[ei], d2e = dot(d2, e);
        R s = denom >= R(1e-15) ? (d1e - b * d2e) / denom : R(0);
        s = mclamp(s, -s1[ei], s1[ei]);
        const R t = mclamp(b * s - d2e, -s2[ej], s2[ej]);
        s = mclamp(d1e + b * t, -s1[ei], s1[ei]);
        V3<R> q1 = c1;
        q1[ei] = s;
        const V3<R> q2 = c2 + d2 * t, gap = q2 - q1;
        const R dd = dot(gap, gap);
        if (dd < best_dist) { best_dist = dd; w1 = q1; w2 = q2; }
      }
    const R dist = dot(w2 - w1, axis);
    if (dist > septol) return;
    o.count = 1;
    o.dist[0] = dist;
    o.pos[0] = rot(R1, (w1 + w2) * R(0.5)) + p1;
    o.normal[0] = rot(R1, axis);
    return;
  }
  const bool ref1 = code < 3;
  const int a = ref1 ? code : code - 3;
  const V3<R> sref = ref1 ? s1 : s2, sinc = ref1 ? s2 : s1, pref = ref1 ? p1 : p2, posoi = ref1 ? pos21 : pos12;
  const R *matref = ref1 ? R1 : R2;
  R rinc[9];
  for (int i = 0; i < 3; ++i)
    for (int j = 0; j < 3; ++j) rinc[3 * i + j] = ref1 ? rm[3 * i + j] : rm[3 * j + i];
  const R sign = posoi[a] >= R(0) ? R(1) : R(-1);
  int inc = 0;
  for (int c = 1; c < 3; ++c)
    if (mabs(rinc[3 * a + c]) > mabs(rinc[3 * a + inc])) inc = c;
  const R incsign = sign * rinc[3 * a + inc] > R(0) ? R(-1) : R(1);
  const int ax = (a + 1) % 3, ay = (a + 2) % 3, bu = (inc + 1) % 3, bv = (inc + 2) % 3;
  const int coords[3] = {ax, ay, a};
  V3<R> cx, du, dv;
  for (int r = 0; r < 3; ++r) {
    const int c = coords[r];
    cx[r] = posoi[c] + incsign * sinc[inc] * rinc[3 * c + inc];
    du[r] = sinc[bu] * rinc[3 * c + bu];
    dv[r] = sinc[bv] * rinc[3 * c + bv];
  }
  cx.z = sign * cx.z - sref[a];
  du.z *= sign;
  dv.z *= sign;
  V3<R> poly[8];
  for (int c = 0; c < 8; ++c) poly[c] = v3<R>(0, 0, 0);
  for (int c = 0; c < 4; ++c) {
    const R su = c == 0 || c == 3 ? R(1) : R(-1), sv = c < 2 ? R(1) : R(-1);
    poly[c] = cx + du * su + dv * sv;
  }
  int count = 4;
  count = clip_poly(count, poly, 0, R(1), sref[ax]);
  count = clip_poly(count, poly, 0, R(-1), sref[ax]);
  count = clip_poly(count, poly, 1, R(1), sref[ay]);
  count = clip_poly(count, poly, 1, R(-1), sref[ay]);
  int accepted = 0;
  const R dup = R(1e-10) * (sref[ax] * sref[ax] + sref[ay] * sref[ay]);
  for (int c = 0; c < count; ++c) {
    if (poly[c].z > margin) continue;
    bool dupe = false;
    for (int q = 0; q < accepted; ++q) {
      const R dx = o.pos[q].x - poly[c].x, dy = o.pos[q].y - poly[c].y;
      if (dx * dx + dy * dy < dup) { dupe = true; break; }
    }
    if (!dupe) o.pos[accepted++] = poly[c];
  }
  if (!accepted) return;
  const V3<R> normal = col(matref, a) * (ref1 ? sign : -sign);
  for (int c = 0; c < accepted; ++c) {
    const V3<R> v = o.pos[c];
    V3<R> local = v3<R>(0, 0, 0);
    local[ax] = v.x;
    local[ay] = v.y;
    local[a] = sign * (sref[a] + R(0.5) * v.z);
    o.dist[c] = v.z;
    o.pos[c] = rot(matref, local) + pref;
    o.normal[c] = normal;
  }
  o.count = accepted;
}

template <class R>
__device__ void box_pair(const Mdl<R> &M, Arena<R> &A, int pair, int g1, int g2) {
  const int t1 = IF(geom_type)[g1];
  const Material<R> p = material(M, g1, g2);
  const V3<R> p1 = ld3(A.gxpos + 3 * g1), p2 = ld3(A.gxpos + 3 * g2);
  const V3<R> s1 = ld3(RF(geom_size) + 3 * g1), s2 = ld3(RF(geom_size) + 3 * g2);
  const R *R1 = A.gxmat + 9 * g1, *R2 = A.gxmat + 9 * g2;
  BoxHits<R> o;
  o.count = 1;
  if (t1 == B200_GEOM_SPHERE) sphere_box(o, 0, p1, s1.x, p2, R2, s2);
  else if (t1 == B200_GEOM_CAPSULE) capsule_box(o, p1, col(R1, 2), s1.x, s1.y, p2, R2, s2);
  else box_box(o, p1, R1, s1, p2, R2, s2, p.margin + p.gap);
  for (int c = 0; c < o.count; ++c) {
    V3<R> fr[3];
    frame_from_normal(o.normal[c], fr);
    emit(M, A, p, pair, c, g1, g2, o.dist[c], o.pos[c], fr);
  }
}

// ---------------------------------------------------------------- sphere / capsule pairs
// MuJoCo's primitive colliders as the reference's native engine carries them
// (collision_detect_primitive.cuh: _SphereSphere :261-292, mjc_SphereCapsule
// :306-322, mjc_CapsuleCapsule :401-490 with its two-contact parallel case).
template <class R> struct PrimHits {
  int count;
  R dist[2];
  V3<R> pos[2], normal[2];
};

template <class R>
__device__ int prim_sphere_sphere(PrimHits<R> &o, R margin, V3<R> p1, const R *m1, R r1, V3<R> p2, const R *m2, R r2) {
  const V3<R> dif = p1 - p2;
  const R cd2 = dot(dif, dif), mind = margin + r1 + r2;
  if (cd2 > mind * mind) return 0;
  const int c = o.count;
  const R dist = msqrt(cd2) - r1 - r2;
  V3<R> n = p2 - p1;
  R len = msqrt(dot(n, n));
  if (len < R(1e-15)) {
    n = cross(col(m1, 2), col(m2, 2));
    len = msqrt(dot(n, n));
    n = len < R(1e-15) ? v3<R>(1, 0, 0) : n * (R(1) / len);  // mju_normalize3: +x below mjMINVAL
  } else
    n = n * (R(1) / len);
  o.dist[c] = dist;
  o.normal[c] = n;
  o.pos[c] = p1 + n * (r1 + dist * R(0.5));
  o.count = c + 1;
  return 1;
}

template <class R>
__device__ __noinline__ void prim_pair(const Mdl<R> &M, Arena<R> &A, int pair, int g1, int g2) {
  const Material<R> p = material(M, g1, g2);
  const int t1 = IF(geom_type)[g1], t2 = IF(geom_type)[g2];
  const V3<R> p1 = ld3(A.gxpos + 3 * g1), p2 = ld3(A.gxpos + 3 * g2);
  const R *m1 = A.gxmat + 9 * g1, *m2 = A.gxmat + 9 * g2;
  const R *s1 = RF(geom_size) + 3 * g1, *s2 = RF(geom_size) + 3 * g2;
  const R margin = p.margin + p.gap;
  PrimHits<R> o;
  o.count = 0;
  if (t1 == B200_GEOM_SPHERE && t2 == B200_GEOM_SPHERE) {
    prim_sphere_sphere(o, margin, p1, m1, s1[0], p2, m2, s2[0]);
  } else if (t1 == B200_GEOM_SPHERE) {
    const V3<R> axis = col(m2, 2);
    const R x = mclamp(dot(axis, p1 - p2), -s2[1], s2[1]);
    prim_sphere_sphere(o, margin, p1, m1, s1[0], p2 + axis * x, m2, s2[0]);
  } else {
    const V3<R> a1 = col(m1, 2) * s1[1], a2 = col(m2, 2) * s2[1], dif = p1 - p2;
    const R ma = dot(a1, a1), mb = -dot(a1, a2), mc = dot(a2, a2), u = -dot(a1, dif), v = dot(a2, dif);
    const R det = ma * mc - mb * mb;
    if (mabs(det) >= R(1e-15)) {
      R x1 = (mc * u - mb * v) / det, x2 = (ma * v - mb * u) / det;
      if (x1 > R(1)) { x1 = 1; x2 = (v - mb) / mc; }
      else if (x1 < R(-1)) { x1 = -1; x2 = (v + mb) / mc; }
      if (x2 > R(1)) { x2 = 1; x1 = mclamp((u - mb) / ma, R(-1), R(1)); }
      else if (x2 < R(-1)) { x2 = -1; x1 = mclamp((u + mb) / ma, R(-1), R(1)); }
      prim_sphere_sphere(o, margin, p1 + a1 * x1, m1, s1[0], p2 + a2 * x2, m2, s2[0]);
    } else {
      R x2 = mclamp((v - mb) / mc, R(-1), R(1));
      int n = prim_sphere_sphere(o, margin, p1 + a1, m1, s1[0], p2 + a2 * x2, m2, s2[0]);
      x2 = mclamp((v + mb) / mc, R(-1), R(1));
      n += prim_sphere_sphere(o, margin, p1 - a1, m1, s1[0], p2 + a2 * x2, m2, s2[0]);
      if (n < 2) {
        R x1 = mclamp((u - mb) / ma, R(-1), R(1));
        n += prim_sphere_sphere(o, margin, p1 + a1 * x1, m1, s1[0], p2 + a2, m2, s2[0]);
        if (n < 2) {
          x1 = mclamp((u + mb) / ma, R(-1), R(1));
          prim_sphere_sphere(o, margin, p1 + a1 * x1, m1, s1[0], p2 - a2, m2, s2[0]);
        }
      }
    }
  }
  for (int c = 0; c < o.count; ++c) {
    V3<R> fr[3];
    frame_from_normal(o.normal[c], fr);
    emit(M, A, p, pair, c, g1, g2, o.dist[c], o.pos[c], fr);
  }
}

// ---------------------------------------------------------------- plane - mesh
// The deepest vertex, then up to three more vertices of its most plane-facing
// incident polygon (mjwarp_plane.cu mesh manifold; restated in
// tools/validation/mjwarp_plane_reference.py mesh_manifold).
template <class R>
__device__ __noinline__ void plane_mesh(const Mdl<R> &M, Arena<R> &A, const Material<R> &p, int pair, int g1, int g2) {
  const V3<R> origin = ld3(A.gxpos + 3 * g1), n = col(A.gxmat + 9 * g1, 2), center = ld3(A.gxpos + 3 * g2);
  const R *Rg = A.gxmat + 9 * g2;
  const int mesh = IF(geom_dataid)[g2], nvert = IF(mesh_vertnum)[mesh];
  const R *vert = RF(mesh_vert) + 3 * IF(mesh_vertadr)[mesh];
  const V3<R> local = rotT(Rg, n);
  int best = 0;
  R top = -dot(ld3(vert), local);
  for (int i = 1; i < nvert; ++i) {
    const R s = -dot(ld3(vert + 3 * i), local);
    if (s > top) { top = s; best = i; }
  }
  V3<R> fr[3];
  frame_from_normal(n, fr);
  const V3<R> world = center + rot(Rg, ld3(vert + 3 * best));
  const R dist = dot(n, world - origin);
  emit(M, A, p, pair, 0, g1, g2, dist, world - n * (R(0.5) * dist), fr);
  if (IF(mesh_polynum)[mesh] <= 0 || dist > p.margin + p.gap) return;
  const int vg = IF(mesh_vertadr)[mesh] + best, madr = IF(mesh_polymapadr)[vg], mnum = IF(mesh_polymapnum)[vg];
  const int pbase = IF(mesh_polyadr)[mesh];
  int face = -1;
  R lowest = 1;
  for (int f = 0; f < mnum; ++f) {
    const int poly = pbase + IF(mesh_polymap)[madr + f];
    const R d = dot(ld3(RF(mesh_polynormal) + 3 * poly), local);
    if (d < R(1) && (face < 0 || d < lowest)) { lowest = d; face = poly; }
  }
  if (face < 0) return;
  const int *pv = IF(mesh_polyvert) + IF(mesh_polyvertadr)[face];
  const int count = IF(mesh_polyvertnum)[face];
  int a = 0;
  for (int i = 0; i < count; ++i)
    if (pv[i] == best) { a = i; break; }
  int sel[4] = {a, (a + 1) % count, (a + 2) % count, (a + 3) % count};
  if (count > 4) {
    auto area = [&](int b, int c, int d) {
      const V3<R> x = cross(ld3(vert + 3 * pv[a]) - ld3(vert + 3 * pv[c]), ld3(vert + 3 * pv[b]) - ld3(vert + 3 * pv[d]));
      return R(0.5) * msqrt(dot(x, x));
    };
    int b = sel[1], c = sel[2], d = sel[3];
    R cur = area(b, c, d);
    while (area(b, c, (d + 1) % count) > cur) {
      d = (d + 1) % count; cur = area(b, c, d);
      while (area(b, (c + 1) % count, d) > cur) { c = (c + 1) % count; cur = area(b, c, d); }
      while (area((b + 1) % count, c, d) > cur) { b = (b + 1) % count; cur = area(b, c, d); }
    }
    sel[1] = b; sel[2] = c; sel[3] = d;
  }
  const int nsel = count < 4 ? count : 4;
  for (int i = 1; i < nsel; ++i) {
    const V3<R> w = center + rot(Rg, ld3(vert + 3 * pv[sel[i]]));
    if (dot(n, w - center) > R(0)) continue;
    const R d = dot(n, w - origin);
    emit(M, A, p, pair, i, g1, g2, d, w - n * (R(0.5) * d), fr);
  }
}

// ---------------------------------------------------------------- convex pairs (GJK / EPA)
// The reference's CCD contract (mjwarp_convex_collision.cuh:46-78,
// mjwarp_convex_epa.cuh gjk_phase): supports inflated by half the pair margin
// on each shape, sphere / capsule cores first, GJK distance with a separation
// cutoff, EPA for penetration, one contact at the witness midpoint.  GJK's
// distance subalgorithm is the signed-volume method (mjwarp_convex_simplex.cuh);
// EPA is the expanding polytope method (van den Bergen 2001).  One thread
// runs one pair; the polytope lives in the thread's local memory.
template <class R> struct CShape {
  int type, nvert;
  V3<R> pos, size;
  const R *rot, *vert;
  R margin;
};

template <class R> __device__ V3<R> cs_support(const CShape<R> &s, V3<R> d) {
  if (s.type == B200_GEOM_SPHERE) return s.pos + d * (s.size.x + R(0.5) * s.margin);
  const V3<R> l = rotT(s.rot, d);
  V3<R> r;
  if (s.type == B200_GEOM_CAPSULE) {
    r = l * s.size.x;
    r.z += (l.z > R(0) ? R(1) : l.z < R(0) ? R(-1) : R(0)) * s.size.y;
  } else if (s.type == B200_GEOM_BOX) {
    r = v3<R>(l.x > R(0) ? s.size.x : -s.size.x, l.y > R(0) ? s.size.y : -s.size.y, l.z > R(0) ? s.size.z : -s.size.z);
  } else {
    int best = 0;
    R top = dot(ld3(s.vert), l);
    for (int i = 1; i < s.nvert; ++i) {
      const R v = dot(ld3(s.vert + 3 * i), l);
      if (v > top) { top = v; best = i; }
    }
    r = ld3(s.vert + 3 * best);
  }
  V3<R> p = rot(s.rot, r) + s.pos;
  if (s.margin > R(0)) p = p + d * (R(0.5) * s.margin);
  return p;
}
// A box's support point in direction d and its corner index: bit k set for
// +size on local axis k (a zero component takes the negative end), the
// labelling the box manifold reads features from
// (mjwarp_convex_geometry.cuh convex_support).
template <class R> __device__ V3<R> box_support(const CShape<R> &s, V3<R> d, int &corner) {
  const V3<R> l = rotT(s.rot, d);
  corner = int(l.x > R(0)) | int(l.y > R(0)) << 1 | int(l.z > R(0)) << 2;
  const V3<R> r = v3<R>(l.x > R(0) ? s.size.x : -s.size.x, l.y > R(0) ? s.size.y : -s.size.y,
                        l.z > R(0) ? s.size.z : -s.size.z);
  return rot(s.rot, r) + s.pos;
}

template <class R> struct SimplexCore {
  V3<R> w[4], a[4], b[4];
  R lam[4];
  int n;
};
// C: the box-box path, which also carries the support corners of a and b
template <class R, bool C = false> struct Simplex : SimplexCore<R> {};
template <class R> struct Simplex<R, true> : SimplexCore<R> { int ca[4], cb[4]; };

// Signed-volume distance sub-algorithm (Montanari, Petrinic and Barbieri,
// "Improving the GJK algorithm for faster and more reliable distance queries
// between convex objects", ACM TOG 2017), the method the reference pins
// (mjwarp_convex_simplex.cuh): barycentric weights of the simplex point
// nearest the origin.  Vertices keep the caller's order (the newest support
// point last); a face whose signed volume disagrees with the whole simplex's
// is searched recursively and the nearest candidate wins.
template <class R> struct SvWeights { R w[4]; };
template <class R> __device__ __forceinline__ bool sv_same_sign(R a, R b) {
  return (a > R(0) && b > R(0)) || (a < R(0) && b < R(0));
}
// segment (p, q); when the origin projects outside, the vertex q
template <class R> __device__ SvWeights<R> sv_segment(V3<R> p, V3<R> q) {
  const V3<R> e = q - p;
  const V3<R> o = q + e * (-dot(q, e) / dot(e, e));  // origin projected on the line
  int k = 0;
  R mu = p.x - q.x;
  if (mabs(p.y - q.y) >= mabs(mu)) { mu = p.y - q.y; k = 1; }
  if (mabs(p.z - q.z) >= mabs(mu)) { mu = p.z - q.z; k = 2; }
  const R c1 = o[k] - q[k], c2 = p[k] - o[k];
  if (sv_same_sign(mu, c1) && sv_same_sign(mu, c2)) return {{c1 / mu, c2 / mu, R(0), R(0)}};
  return {{R(0), R(1), R(0), R(0)}};
}
// origin projected on the plane of (a, b, c), trying three normal forms;
// false when the triangle is degenerate
template <class R> __device__ bool sv_plane(V3<R> a, V3<R> b, V3<R> c, V3<R> &o) {
  const V3<R> ab = b - a, ac = c - a, bc = c - b;
  V3<R> n = cross(bc, ab);
  R nv = dot(n, b), nn = dot(n, n);
  if (nn == R(0)) return false;
  if (nv != R(0) && nn > R(1e-15)) { o = n * (nv / nn); return true; }
  n = cross(ab, ac); nv = dot(n, a); nn = dot(n, n);
  if (nn == R(0)) return false;
  if (nv != R(0) && nn > R(1e-15)) { o = n * (nv / nn); return true; }
  n = cross(ac, bc); nv = dot(n, c); nn = dot(n, n);
  o = n * (nv / nn);
  return true;
}
template <class R> __device__ __forceinline__ R sv_area(V3<R> p, V3<R> u, V3<R> v, int i, int j) {
  const V3<R> a = u - p, b = v - p;
  return a[i] * b[j] - a[j] * b[i];
}
template <class R> __device__ SvWeights<R> sv_triangle(V3<R> a, V3<R> b, V3<R> c) {
  V3<R> o;
  if (!sv_plane(a, b, c, o)) return sv_segment(a, b);
  // the coordinate plane in which the triangle's projection is largest
  const V3<R> u = b - a, v = c - a;
  const R myz = u.y * v.z - u.z * v.y, mxz = u.x * v.z - u.z * v.x, mxy = u.x * v.y - u.y * v.x;
  R m;
  int i, j;
  if (mabs(myz) >= mabs(mxz) && mabs(myz) >= mabs(mxy)) { m = myz; i = 1; j = 2; }
  else if (mabs(mxz) >= mabs(mxy)) { m = mxz; i = 0; j = 2; }
  else { m = mxy; i = 0; j = 1; }
  const R s1 = sv_area(o, b, c, i, j), s2 = sv_area(o, c, a, i, j), s3 = sv_area(o, a, b, i, j);
  const bool in1 = sv_same_sign(m, s1), in2 = sv_same_sign(m, s2), in3 = sv_same_sign(m, s3);
  if (in1 && in2 && in3) return {{s1 / m, s2 / m, s3 / m, R(0)}};
  SvWeights<R> out = {{R(0), R(0), R(0), R(0)}};
  R best = R(1e30);
  if (!in1) {
    const SvWeights<R> e = sv_segment(b, c);
    const V3<R> x = b * e.w[0] + c * e.w[1];
    out = {{R(0), e.w[0], e.w[1], R(0)}};
    best = dot(x, x);
  }
  if (!in2) {
    const SvWeights<R> e = sv_segment(a, c);
    const V3<R> x = a * e.w[0] + c * e.w[1];
    const R d = dot(x, x);
    if (d < best) { out = {{e.w[0], R(0), e.w[1], R(0)}}; best = d; }
  }
  if (!in3) {
    const SvWeights<R> e = sv_segment(a, b);
    const V3<R> x = a * e.w[0] + b * e.w[1];
    if (dot(x, x) < best) out = {{e.w[0], e.w[1], R(0), R(0)}};
  }
  return out;
}
template <class R> __device__ SvWeights<R> sv_tetrahedron(V3<R> a, V3<R> b, V3<R> c, V3<R> d) {
  const R s1 = -dot(b, cross(c, d)), s2 = dot(a, cross(c, d)), s3 = -dot(a, cross(b, d)), s4 = dot(a, cross(b, c));
  const R vol = s1 + s2 + s3 + s4;
  const bool in1 = sv_same_sign(vol, s1), in2 = sv_same_sign(vol, s2), in3 = sv_same_sign(vol, s3),
             in4 = sv_same_sign(vol, s4);
  if (in1 && in2 && in3 && in4) return {{s1 / vol, s2 / vol, s3 / vol, s4 / vol}};
  SvWeights<R> out = {{R(0), R(0), R(0), R(0)}};
  R best = R(1e30);
  if (!in1) {
    const SvWeights<R> t = sv_triangle(b, c, d);
    const V3<R> x = b * t.w[0] + c * t.w[1] + d * t.w[2];
    out = {{R(0), t.w[0], t.w[1], t.w[2]}};
    best = dot(x, x);
  }
  if (!in2) {
    const SvWeights<R> t = sv_triangle(a, c, d);
    const V3<R> x = a * t.w[0] + c * t.w[1] + d * t.w[2];
    const R dd = dot(x, x);
    if (dd < best) { out = {{t.w[0], R(0), t.w[1], t.w[2]}}; best = dd; }
  }
  if (!in3) {
    const SvWeights<R> t = sv_triangle(a, b, d);
    const V3<R> x = a * t.w[0] + b * t.w[1] + d * t.w[2];
    const R dd = dot(x, x);
    if (dd < best) { out = {{t.w[0], t.w[1], R(0), t.w[2]}}; best = dd; }
  }
  if (!in4) {
    const SvWeights<R> t = sv_triangle(a, b, c);
    const V3<R> x = a * t.w[0] + b * t.w[1] + c * t.w[2];
    if (dot(x, x) < best) out = {{t.w[0], t.w[1], t.w[2], R(0)}};
  }
  return out;
}

// Reduce the simplex to the vertices with nonzero weight (order kept), the
// weights becoming the affine coordinates of the nearest point.
// C (corners): carry the box support corners (the box-box path only)
template <class R, bool C> __device__ void simplex_reduce(Simplex<R, C> &s) {
  SvWeights<R> W;
  if (s.n == 4) W = sv_tetrahedron(s.w[0], s.w[1], s.w[2], s.w[3]);
  else if (s.n == 3) W = sv_triangle(s.w[0], s.w[1], s.w[2]);
  else if (s.n == 2) W = sv_segment(s.w[0], s.w[1]);
  else W = {{R(1), R(0), R(0), R(0)}};
  Simplex<R, C> t;
  int k = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i)
    if (i < s.n && W.w[i] != R(0)) {
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (j == k) {
          t.w[j] = s.w[i]; t.a[j] = s.a[i]; t.b[j] = s.b[i]; t.lam[j] = W.w[i];
          if constexpr (C) { t.ca[j] = s.ca[i]; t.cb[j] = s.cb[i]; }
        }
      ++k;
    }
  t.n = k;
  s = t;
}

template <class R, bool C = false> struct GjkOut {
  bool separated;
  R dist;
  V3<R> x1, x2;
  Simplex<R, C> s;
};

template <class R, bool C = false>
__device__ GjkOut<R, C> gjk(const CShape<R> &A, const CShape<R> &B, R tol, int iterations, R cutoff) {
  GjkOut<R, C> o;
  o.separated = false;
  Simplex<R, C> &s = o.s;
  s.n = 0;
  V3<R> x = A.pos - B.pos;
  R norm = msqrt(dot(x, x)), prev = -1;
  for (int it = 0; it < iterations; ++it) {
    if (norm < tol || mabs(prev - norm) < R(1e-15)) break;
    const V3<R> d = x * (R(1) / norm);
    int ca = -1, cb = -1;
    V3<R> a, b;
    if constexpr (C) { a = box_support(A, -d, ca); b = box_support(B, d, cb); }
    else { a = cs_support(A, -d); b = cs_support(B, d); }
    const V3<R> w = a - b;
    if (dot(x, x - w) < R(0.5) * tol * tol) break;
    const R lower = dot(x, w);
    if (lower > R(0) && (cutoff == R(0) || lower >= cutoff * norm)) {
      o.separated = true;
      o.dist = R(1e30);
      return o;
    }
#pragma unroll
    for (int i = 0; i < 4; ++i)
      if (i == s.n) {
        s.w[i] = w; s.a[i] = a; s.b[i] = b;
        if constexpr (C) { s.ca[i] = ca; s.cb[i] = cb; }
      }
    s.n++;
    simplex_reduce<R, C>(s);
    if (s.n < 1) break;
    x = v3<R>(0, 0, 0);
#pragma unroll
    for (int i = 0; i < 4; ++i)
      if (i < s.n) x = x + s.w[i] * s.lam[i];
    prev = norm;
    norm = msqrt(dot(x, x));
    if (s.n == 4) break;
  }
  o.x1 = v3<R>(0, 0, 0); o.x2 = v3<R>(0, 0, 0);
#pragma unroll
  for (int i = 0; i < 4; ++i)
    if (i < s.n) { o.x1 = o.x1 + s.a[i] * s.lam[i]; o.x2 = o.x2 + s.b[i] * s.lam[i]; }
  if (s.n == 0) { o.x1 = A.pos; o.x2 = B.pos; }
  o.dist = s.n == 4 ? R(0) : norm;
  return o;
}

constexpr int kEpaMaxV = 48, kEpaMaxF = 96;
template <class R> struct PolytopeCore {
  V3<R> w[kEpaMaxV], a[kEpaMaxV], b[kEpaMaxV];
  int nv, nf, face[kEpaMaxF][3];
  V3<R> n[kEpaMaxF];
  R d[kEpaMaxF];
  bool alive[kEpaMaxF];
};
// C: the box-box path, which also keeps each vertex's box support corners
template <class R, bool C = false> struct Polytope : PolytopeCore<R> {};
template <class R> struct Polytope<R, true> : PolytopeCore<R> { int ca[kEpaMaxV], cb[kEpaMaxV]; };

// Drop the dead faces, keeping the live ones in their order (the best-face
// search breaks ties by the lower index, so the order is part of the result).
template <class R, bool C> __device__ void epa_compact(Polytope<R, C> &P) {
  int k = 0;
  for (int f = 0; f < P.nf; ++f) {
    if (!P.alive[f]) continue;
    if (k != f) {
      P.face[k][0] = P.face[f][0]; P.face[k][1] = P.face[f][1]; P.face[k][2] = P.face[f][2];
      P.n[k] = P.n[f]; P.d[k] = P.d[f]; P.alive[k] = true;
    }
    ++k;
  }
  P.nf = k;
}

// New face (i, j, l): its index, -1 for a degenerate triangle, -2 when the
// face pool is full even after compaction.
template <class R, bool C> __device__ int epa_add_face(Polytope<R, C> &P, int i, int j, int l) {
  if (P.nf >= kEpaMaxF) epa_compact(P);
  if (P.nf >= kEpaMaxF) return -2;
  V3<R> n = cross(P.w[j] - P.w[i], P.w[l] - P.w[i]);
  const R len = msqrt(dot(n, n));
  if (!(len > R(1e-30))) return -1;
  n = n * (R(1) / len);
  const int f = P.nf++;
  P.face[f][0] = i; P.face[f][1] = j; P.face[f][2] = l;
  P.n[f] = n; P.d[f] = dot(n, P.w[i]); P.alive[f] = true;
  return f;
}

template <class R, bool C> __device__ int epa_push(Polytope<R, C> &P, const CShape<R> &A, const CShape<R> &B, V3<R> d) {
  if (P.nv >= kEpaMaxV) return -1;
  const int v = P.nv++;
  if constexpr (C) { P.a[v] = box_support(A, d, P.ca[v]); P.b[v] = box_support(B, -d, P.cb[v]); }
  else { P.a[v] = cs_support(A, d); P.b[v] = cs_support(B, -d); }
  P.w[v] = P.a[v] - P.b[v];
  return v;
}

template <class R, bool C>
__device__ bool epa_seed(Polytope<R, C> &P, const CShape<R> &A, const CShape<R> &B, const Simplex<R, C> &s) {
  P.nf = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i)
    if (i < s.n) {
      P.w[i] = s.w[i]; P.a[i] = s.a[i]; P.b[i] = s.b[i];
      if constexpr (C) { P.ca[i] = s.ca[i]; P.cb[i] = s.cb[i]; }
    }
  P.nv = s.n;
  for (int k = 0; P.nv < 2 && k < 6; ++k) {
    V3<R> ax = v3<R>(0, 0, 0);
    ax[k / 2] = k % 2 ? R(-1) : R(1);
    const int v = epa_push<R, C>(P, A, B, ax);
    if (v == 0) continue;  // an empty simplex (coincident centres): the first vertex seeds
    const V3<R> e = P.w[v] - P.w[0];
    if (dot(e, e) < R(1e-20)) P.nv--;
  }
  if (P.nv < 2) return false;
  if (P.nv == 2) {
    const V3<R> e = P.w[1] - P.w[0];
    int m = 0;
    for (int c = 1; c < 3; ++c)
      if (mabs(e[c]) < mabs(e[m])) m = c;
    V3<R> ax = v3<R>(0, 0, 0);
    ax[m] = 1;
    const V3<R> d = normalize(cross(e, ax));
    int v = epa_push<R, C>(P, A, B, d);
    V3<R> cr = cross(P.w[v] - P.w[0], e);
    if (dot(cr, cr) < R(1e-20)) { P.nv--; v = epa_push<R, C>(P, A, B, -d); cr = cross(P.w[v] - P.w[0], e); }
    if (dot(cr, cr) < R(1e-20)) return false;
  }
  if (P.nv == 3) {
    const V3<R> n = normalize(cross(P.w[1] - P.w[0], P.w[2] - P.w[0]));
    int v = epa_push<R, C>(P, A, B, n);
    R h = dot(n, P.w[v] - P.w[0]);
    if (mabs(h) < R(1e-12) || dot(n, P.w[0]) > R(0)) {
      P.nv--;
      v = epa_push<R, C>(P, A, B, -n);
      h = dot(n, P.w[v] - P.w[0]);
    }
    if (mabs(h) < R(1e-12)) return false;
  }
  const V3<R> c = (P.w[0] + P.w[1] + P.w[2] + P.w[3]) * R(0.25);
  const int tf[4][3] = {{0, 1, 2}, {0, 3, 1}, {0, 2, 3}, {1, 3, 2}};
  for (int f = 0; f < 4; ++f) {
    int i = tf[f][0], j = tf[f][1], l = tf[f][2];
    const V3<R> n = cross(P.w[j] - P.w[i], P.w[l] - P.w[i]);
    if (dot(n, P.w[i] - c) < R(0)) { const int t = j; j = l; l = t; }
    if (epa_add_face(P, i, j, l) < 0) return false;
    if (P.d[P.nf - 1] < -R(1e-12)) return false;
  }
  return true;
}

// ok: a penetration depth was found; budget: the vertex or face pool filled
// before EPA converged (it ends with its best face, as at its iteration
// limit); horizon: the horizon edge list filled (the reference's EPA_HORIZON)
template <class R> struct EpaOut {
  bool ok, budget, horizon;
  R depth;
  V3<R> x1, x2;
};
// the support points and box corners of EPA's final face (the box manifold's input)
template <class R> struct EpaFace {
  V3<R> a[3], b[3];
  int ca[3], cb[3];
};

// C: two zero-margin boxes (polytopes), with their support corners tracked.
// EPA then stops when the support distance is within 1e-7 of the face, or
// when the new support is a corner pair the polytope already holds, which
// ends it on a face of the Minkowski difference itself
// (mjwarp_convex_epa.cuh epa_expand), and reports that face in *face.
template <class R, bool C = false>
__device__ EpaOut<R> epa(const CShape<R> &A, const CShape<R> &B, const Simplex<R, C> &s, R tol, int iterations,
                         EpaFace<R> *face = nullptr) {
  EpaOut<R> o;
  o.ok = false;
  o.budget = o.horizon = false;
  Polytope<R, C> P;
  if (!epa_seed<R, C>(P, A, B, s)) return o;
  const R eps = C ? R(1e-7) : tol;
  int best = -1;
  for (int it = 0; it <= iterations; ++it) {
    best = -1;
    for (int f = 0; f < P.nf; ++f)
      if (P.alive[f] && (best < 0 || P.d[f] < P.d[best])) best = f;
    if (best < 0) return o;
    if (it == iterations) break;
    const V3<R> n = P.n[best];
    const int v = epa_push<R, C>(P, A, B, n);
    if (v < 0) { o.budget = true; break; }
    if (dot(P.w[v], n) - P.d[best] < eps) { P.nv--; break; }
    if constexpr (C) {
      bool repeated = false;
      for (int q = 0; q < v; ++q) repeated |= P.ca[q] == P.ca[v] && P.cb[q] == P.cb[v];
      if (repeated) { P.nv--; break; }
    }
    int edges[3 * kEpaMaxF][2], ne = 0;
    for (int f = 0; f < P.nf; ++f) {
      if (!P.alive[f] || dot(P.n[f], P.w[v] - P.w[P.face[f][0]]) <= R(0)) continue;
      P.alive[f] = false;
      for (int e = 0; e < 3; ++e) {
        const int i = P.face[f][e], j = P.face[f][(e + 1) % 3];
        int dup = -1;
        for (int q = 0; q < ne; ++q)
          if (edges[q][0] == j && edges[q][1] == i) { dup = q; break; }
        if (dup >= 0) { edges[dup][0] = edges[ne - 1][0]; edges[dup][1] = edges[ne - 1][1]; --ne; }
        else if (ne < 3 * kEpaMaxF) { edges[ne][0] = i; edges[ne][1] = j; ++ne; }
        else o.horizon = true;
      }
    }
    bool full = false;
    for (int q = 0; q < ne; ++q) {
      const int f = epa_add_face(P, edges[q][0], edges[q][1], v);
      if (f < 0) { full = true; o.budget |= f == -2; break; }
    }
    if (full || o.horizon) break;
  }
  if (best < 0) return o;
  const int i = P.face[best][0], j = P.face[best][1], l = P.face[best][2];
  const V3<R> pt = P.n[best] * P.d[best];
  const V3<R> e0 = P.w[j] - P.w[i], e1 = P.w[l] - P.w[i], e2 = pt - P.w[i];
  const R d00 = dot(e0, e0), d01 = dot(e0, e1), d11 = dot(e1, e1), d20 = dot(e2, e0), d21 = dot(e2, e1);
  const R den = d00 * d11 - d01 * d01;
  const R lv = den != R(0) ? (d11 * d20 - d01 * d21) / den : R(0), lw = den != R(0) ? (d00 * d21 - d01 * d20) / den : R(0);
  const R lu = R(1) - lv - lw;
  o.x1 = P.a[i] * lu + P.a[j] * lv + P.a[l] * lw;
  o.x2 = P.b[i] * lu + P.b[j] * lv + P.b[l] * lw;
  o.depth = P.d[best];
  if constexpr (C) {
    const int fv[3] = {i, j, l};
    for (int k = 0; k < 3; ++k) {
      face->a[k] = P.a[fv[k]]; face->b[k] = P.b[fv[k]];
      face->ca[k] = P.ca[fv[k]]; face->cb[k] = P.cb[fv[k]];
    }
  }
  o.ok = true;
  return o;
}

// ---------------------------------------------------------------- box manifold
// Zero-margin box pairs reach the convex path (the reference routes box-box
// there when no box pair has a margin, cuda_fp32/physics.py:89-90) and turn
// EPA's single contact into a face manifold (mjwarp_box_manifold.cuh
// box_multicontact): the corners of EPA's final face name a feature of each
// box (a corner, an edge or a face); the features' face normals are paired
// anti-parallel within 5.1 degrees (or a face normal with an edge
// perpendicular to it within 5.1 degrees); the incident face (or edge) is
// clipped against the side planes of the reference face; the clipped points
// below the reference face are the contacts, at most four (the pair farthest
// apart for an edge, the largest-area quadrilateral for more than four).
template <class R> struct BoxManifold {
  int count;
  V3<R> one[4], two[4];
  R dist[4];
};
template <class R> struct BoxFeature {
  int dim, corner[3];
  V3<R> pt[3];
};
template <class R> struct BoxNormals {
  int count, face[3];
  V3<R> n[3];
};
constexpr float kBoxAligned = 0.99605101346969604f, kBoxPerpendicular = 0.088782943785190582f;

template <class R> __device__ BoxFeature<R> box_feature(const int *corner, const V3<R> *pt) {
  BoxFeature<R> f;
  for (int k = 0; k < 3; ++k) { f.corner[k] = corner[k]; f.pt[k] = pt[k]; }
  if (f.corner[0] != f.corner[1]) {
    f.dim = (f.corner[2] == f.corner[0] || f.corner[2] == f.corner[1]) ? 2 : 3;
  } else {
    f.corner[1] = f.corner[2];
    f.pt[1] = f.pt[2];
    f.dim = f.corner[0] != f.corner[2] ? 2 : 1;
  }
  return f;
}
template <class R> __device__ V3<R> box_axis(const CShape<R> &s, int face) {  // face 2k: +axis k, 2k+1: -axis k
  V3<R> e = v3<R>(0, 0, 0);
  e[face / 2] = face % 2 ? R(-1) : R(1);
  return rot(s.rot, e);
}
// the face whose normal is within 5.1 degrees of direction d, if any
template <class R> __device__ BoxNormals<R> box_normals_near(const CShape<R> &s, V3<R> d) {
  BoxNormals<R> o;
  o.count = 0;
  const V3<R> l = normalize(rotT(s.rot, d));
  for (int f = 0; f < 6; ++f)
    if ((f % 2 ? -l[f / 2] : l[f / 2]) > R(kBoxAligned)) {
      o.count = 1; o.face[0] = f; o.n[0] = box_axis(s, f);
      return o;
    }
  return o;
}
// the face normals a feature lies on: the axes on which all its corners agree
template <class R> __device__ BoxNormals<R> box_normals(const CShape<R> &s, const BoxFeature<R> &f, V3<R> d) {
  BoxNormals<R> o;
  o.count = 0;
  if (f.dim == 1) {
    o.count = 3;
    for (int k = 0; k < 3; ++k) {
      o.face[k] = 2 * k + ((f.corner[0] >> k) & 1 ? 0 : 1);
      o.n[k] = box_axis(s, o.face[k]);
    }
    return o;
  }
  for (int k = 0; k < 3; ++k) {
    bool all = true, none = true;
    for (int i = 0; i < f.dim; ++i) {
      const bool set = (f.corner[i] >> k) & 1;
      all &= set; none &= !set;
    }
    if (all || none) {
      o.face[o.count] = 2 * k + (all ? 0 : 1);
      o.n[o.count] = box_axis(s, o.face[o.count]);
      ++o.count;
    }
  }
  if ((f.dim == 3 && o.count == 1) || (f.dim == 2 && o.count >= 1)) return o;
  return box_normals_near(s, d);
}
// the box edges at a feature point: the edge itself for an edge, the three
// edges leaving a corner; end[k] their far ends
template <class R> __device__ BoxNormals<R> box_edges(const CShape<R> &s, const BoxFeature<R> &f, V3<R> *end) {
  BoxNormals<R> o;
  o.count = 0;
  if (f.dim == 2) {
    end[0] = f.pt[1];
    o.n[0] = normalize(f.pt[1] - f.pt[0]);
    o.count = 1;
  } else if (f.dim == 1) {
    V3<R> c;
    for (int k = 0; k < 3; ++k) c[k] = (f.corner[0] >> k) & 1 ? s.size[k] : -s.size[k];
    for (int k = 0; k < 3; ++k) {
      V3<R> q = c;
      q[k] = -q[k];
      end[k] = rot(s.rot, q) + s.pos;
      o.n[k] = normalize(end[k] - f.pt[0]);
    }
    o.count = 3;
  }
  return o;
}
// the four corners of face `face`, wound as the reference winds them
template <class R> __device__ void box_face_corners(const CShape<R> &s, int face, V3<R> *v) {
  constexpr unsigned char kWinding[6][4] = {{7, 3, 1, 5}, {2, 6, 4, 0}, {2, 3, 7, 6}, {4, 5, 1, 0}, {6, 7, 5, 4}, {3, 2, 0, 1}};
  for (int i = 0; i < 4; ++i) {
    V3<R> c;
    for (int k = 0; k < 3; ++k) c[k] = (kWinding[face][i] >> k) & 1 ? s.size[k] : -s.size[k];
    v[i] = rot(s.rot, c) + s.pos;
  }
}
template <class R> __device__ R quad_area(V3<R> a, V3<R> b, V3<R> c, V3<R> d) {
  const V3<R> n = cross(a - c, b - d);
  return R(0.5) * msqrt(dot(n, n));
}
// four of n polygon vertices spanning the largest quadrilateral, by the
// reference's rotating search (each vertex in turn as a, advancing d, then c,
// then b while the area grows)
template <class R> __device__ void largest_quad(const V3<R> *p, int n, int *q) {
  int b = 1, c = 2, d = 3;
  q[0] = 0; q[1] = b; q[2] = c; q[3] = d;
  R area = quad_area(p[0], p[b], p[c], p[d]);
  for (int a = 0; a < n; ++a) {
    for (;;) {
      R next = quad_area(p[a], p[b], p[c], p[(d + 1) % n]);
      if (next <= area) break;
      area = next; d = (d + 1) % n; q[0] = a; q[1] = b; q[2] = c; q[3] = d;
      for (;;) {
        next = quad_area(p[a], p[b], p[(c + 1) % n], p[d]);
        if (next <= area) break;
        area = next; c = (c + 1) % n; q[0] = a; q[1] = b; q[2] = c; q[3] = d;
      }
      for (;;) {
        next = quad_area(p[a], p[(b + 1) % n], p[c], p[d]);
        if (next <= area) break;
        area = next; b = (b + 1) % n; q[0] = a; q[1] = b; q[2] = c; q[3] = d;
      }
    }
    if (b == a) {
      b = (b + 1) % n;
      if (c == b) {
        c = (c + 1) % n;
        if (d == c) d = (d + 1) % n;
      }
    }
  }
}
// clip polygon `inc` (n2 points) by the side planes of face `ref` (n1 >= 3
// points, outward normal `normal`) and keep what lies below that face;
// `dir` points from the incident shape's contact points to the reference's
template <class R>
__device__ BoxManifold<R> clip_faces(const V3<R> *ref, int n1, const V3<R> *inc, int n2, V3<R> normal, V3<R> dir) {
  BoxManifold<R> o;
  o.count = 0;
  if (n1 < 3) return o;
  V3<R> side[4], buf[2][8];
  R plane[4];
  for (int i = 0; i < n1; ++i) {
    side[i] = cross(ref[(i + 1) % n1] - ref[i], (ref[i] + normal) - ref[i]);
    plane[i] = dot(side[i], ref[i]);
  }
  int count = n2, cur = 0;
  for (int i = 0; i < n2; ++i) buf[0][i] = inc[i];
  for (int e = 0; e < n1; ++e) {
    const V3<R> *in = buf[cur];
    V3<R> *out = buf[cur ^ 1];
    int m = 0;
    for (int i = 0; i < count; ++i) {
      const V3<R> p = in[i], q = in[(i + 1) % count];
      const bool inp = dot(p - ref[e], side[e]) > R(-1e-10), inq = dot(q - ref[e], side[e]) > R(-1e-10);
      if (!inp && !inq) continue;
      if (inp && inq) { if (m < 8) out[m++] = q; continue; }
      const R den = dot(side[e], q - p);
      R t = mabs(den) < R(1e-10) ? R(1e30) : (plane[e] - dot(side[e], p)) / den;
      if (t > R(-3e-7) && t < R(1) + R(3e-7)) {
        t = mmin(R(1), mmax(R(0), t));
        if (m < 8) out[m++] = p + (q - p) * t;
      }
      if (inq && m < 8) out[m++] = q;
    }
    cur ^= 1;
    count = m;
  }
  V3<R> *poly = buf[cur];
  int kept = 0;
  for (int i = 0; i < count; ++i)
    if (dot(poly[i] - ref[0], normal) <= R(0)) poly[kept++] = poly[i];
  count = kept;
  if (count < 1) return o;
  int q[4] = {0, 1, 2, 3};
  if (n2 == 2 && count > 2) {
    R best = 0;
    q[0] = 0; q[1] = 1;
    for (int i = 0; i < count; ++i)
      for (int j = i + 1; j < count; ++j) {
        const V3<R> d = poly[j] - poly[i];
        if (dot(d, d) > best) { best = dot(d, d); q[0] = i; q[1] = j; }
      }
    o.count = 2;
  } else if (count > 4) {
    largest_quad(poly, count, q);
    o.count = 4;
  } else
    o.count = count;
  for (int i = 0; i < o.count; ++i) {
    const V3<R> v = poly[q[i]];
    const R d = dot(v - ref[0], normal);
    o.one[i] = v - dir * mabs(d);
    o.two[i] = v;
    o.dist[i] = d;
  }
  return o;
}
// EPA's final face -> the box-box contact manifold (count 0: keep EPA's contact)
template <class R>
__device__ BoxManifold<R> box_manifold(const CShape<R> &A, const CShape<R> &B, const EpaOut<R> &e, const EpaFace<R> &f) {
  BoxManifold<R> none;
  none.count = 0;
  const BoxFeature<R> fa = box_feature<R>(f.ca, f.a), fb = box_feature<R>(f.cb, f.b);
  const V3<R> dir = e.x2 - e.x1;
  BoxNormals<R> na = box_normals(A, fa, -dir), nb = box_normals(B, fb, dir);
  int i = 0, j = 0;
  bool aligned = false, edge_a = false, edge_b = false;
  for (int k = 0; k < na.count && !aligned; ++k)
    for (int l = 0; l < nb.count; ++l)
      if (dot(na.n[k], nb.n[l]) < -R(kBoxAligned)) { i = k; j = l; aligned = true; break; }
  V3<R> end[3];
  if (!aligned) {
    if (fa.dim < 3 && nb.count && (fa.dim <= fb.dim || !na.count)) {
      na = box_edges(A, fa, end);
      for (int k = 0; k < nb.count && !aligned; ++k) {
        if (dot(nb.n[k], dir) <= R(1e-15)) continue;
        for (int l = 0; l < na.count; ++l)
          if (mabs(dot(na.n[l], nb.n[k])) < R(kBoxPerpendicular)) { i = l; j = k; aligned = true; break; }
      }
      if (!aligned) return none;
      edge_a = true;
    } else if (fb.dim < 3) {
      nb = box_edges(B, fb, end);
      for (int k = 0; k < na.count && !aligned; ++k) {
        if (dot(na.n[k], -dir) <= R(1e-15)) continue;
        for (int l = 0; l < nb.count; ++l)
          if (mabs(dot(nb.n[l], na.n[k])) < R(kBoxPerpendicular)) { i = l; j = k; aligned = true; break; }
      }
      if (!aligned) return none;
      edge_b = true;
    } else
      return none;
  }
  V3<R> face_a[4], face_b[4];
  int count_a = 4, count_b = 4;
  if (edge_a) { face_a[0] = fa.pt[0]; face_a[1] = end[i]; count_a = 2; }
  else box_face_corners(A, na.face[edge_b ? j : i], face_a);
  if (edge_b) { face_b[0] = fb.pt[0]; face_b[1] = end[i]; count_b = 2; }
  else box_face_corners(B, nb.face[j], face_b);
  if (edge_a) {  // B's face is the reference face; contact points swap sides
    BoxManifold<R> r = clip_faces(face_b, count_b, face_a, count_a, nb.n[j], -nb.n[j]);
    for (int k = 0; k < r.count; ++k) { const V3<R> v = r.one[k]; r.one[k] = r.two[k]; r.two[k] = v; }
    return r;
  }
  if (edge_b) return clip_faces(face_a, count_a, face_b, count_b, na.n[j], -na.n[j]);
  return clip_faces(face_a, count_a, face_b, count_b, na.n[i], nb.n[j]);
}

template <class R>
__device__ CShape<R> cs_make(const Mdl<R> &M, const Arena<R> &A, int g, V3<R> origin, R margin) {
  CShape<R> s;
  s.type = IF(geom_type)[g];
  s.pos = ld3(A.gxpos + 3 * g) - origin;
  s.size = ld3(RF(geom_size) + 3 * g);
  s.rot = A.gxmat + 9 * g;
  s.margin = margin;
  s.vert = nullptr;
  s.nvert = 0;
  if (s.type == B200_GEOM_MESH) {
    const int mesh = IF(geom_dataid)[g];
    s.vert = RF(mesh_vert) + 3 * IF(mesh_vertadr)[mesh];
    s.nvert = IF(mesh_vertnum)[mesh];
  }
  return s;
}

template <class R>
__device__ __noinline__ void convex_pair(const Mdl<R> &M, Arena<R> &A, int pair, int g1, int g2) {
  const Material<R> p = material(M, g1, g2);
  const V3<R> origin = ld3(A.gxpos + 3 * g1);
  const CShape<R> S1 = cs_make(M, A, g1, origin, p.margin), S2 = cs_make(M, A, g2, origin, p.margin);
  const R tol = R(M.m.ccd_tolerance);
  const int iters = M.m.ccd_iterations;
  R dist = 0;
  V3<R> x1 = v3<R>(0, 0, 0), x2 = v3<R>(0, 0, 0);
  bool found = false;
  R full1 = 0, full2 = 0;
  CShape<R> C1 = S1, C2 = S2;
  if (S1.type == B200_GEOM_SPHERE || S1.type == B200_GEOM_CAPSULE) { full1 = S1.size.x + R(0.5) * S1.margin; C1.size.x = 0; C1.margin = 0; }
  if (S2.type == B200_GEOM_SPHERE || S2.type == B200_GEOM_CAPSULE) { full2 = S2.size.x + R(0.5) * S2.margin; C2.size.x = 0; C2.margin = 0; }
  if (full1 + full2 > R(0)) {
    const GjkOut<R> r = gjk(C1, C2, tol, iters, p.gap + full1 + full2);
    if (r.separated) return;
    if (r.dist > tol) {
      const V3<R> nrm = normalize(r.x2 - r.x1);
      x1 = r.x1 + nrm * full1;
      x2 = r.x2 - nrm * full2;
      dist = r.dist - (full1 + full2);
      found = true;
    }
  }
  if (!found) {
    const GjkOut<R> r = gjk(S1, S2, tol, iters, p.gap);
    if (r.separated) return;
    if (r.dist > tol) { dist = r.dist; x1 = r.x1; x2 = r.x2; }
    else {
      const EpaOut<R> e = epa(S1, S2, r.s, tol, M.m.epa_iterations);
      if (e.budget) atomicOr(&A.iscal[3], B200_WARN_EPA_BUDGET);
      if (e.horizon) atomicOr(&A.iscal[3], B200_OVERFLOW_EPA_HORIZON);
      if (!e.ok) { dist = r.dist; x1 = r.x1; x2 = r.x2; }
      else { dist = -e.depth; x1 = e.x1; x2 = e.x2; }
    }
  }
  if (!(dist < p.gap)) return;
  const R distance = dist + p.margin;
  V3<R> fr[3];
  frame_from_normal(distance <= p.margin ? x1 - x2 : x2 - x1, fr);
  emit(M, A, p, pair, 0, g1, g2, distance, (x1 + x2) * R(0.5) + origin, fr);
}

// Two zero-margin boxes on the convex path: GJK and EPA with the boxes'
// support corners tracked, EPA ending on a face of the Minkowski difference,
// and that face's manifold of up to four contacts
// (mjwarp_convex_collision.cuh:63-77).  A separate function so that the
// other convex pairs carry none of its state.
template <class R>
__device__ __noinline__ void convex_box_pair(const Mdl<R> &M, Arena<R> &A, int pair, int g1, int g2) {
  const Material<R> p = material(M, g1, g2);
  const V3<R> origin = ld3(A.gxpos + 3 * g1);
  const CShape<R> S1 = cs_make(M, A, g1, origin, p.margin), S2 = cs_make(M, A, g2, origin, p.margin);
  const R tol = R(M.m.ccd_tolerance);
  const GjkOut<R, true> r = gjk<R, true>(S1, S2, tol, M.m.ccd_iterations, p.gap);
  if (r.separated) return;
  R dist = r.dist;
  V3<R> x1 = r.x1, x2 = r.x2;
  BoxManifold<R> mf;
  mf.count = 0;
  if (!(r.dist > tol)) {
    EpaFace<R> face;
    const EpaOut<R> e = epa<R, true>(S1, S2, r.s, tol, M.m.epa_iterations, &face);
    if (e.budget) atomicOr(&A.iscal[3], B200_WARN_EPA_BUDGET);
    if (e.horizon) atomicOr(&A.iscal[3], B200_OVERFLOW_EPA_HORIZON);
    if (e.ok) {
      dist = -e.depth; x1 = e.x1; x2 = e.x2;
      mf = box_manifold(S1, S2, e, face);
    }
  }
  if (!(dist < p.gap)) return;
  const R distance = dist + p.margin;
  if (mf.count < 1) { mf.count = 1; mf.one[0] = x1; mf.two[0] = x2; }
  V3<R> fr[3];
  frame_from_normal(distance <= p.margin ? mf.one[0] - mf.two[0] : mf.two[0] - mf.one[0], fr);
  for (int c = 0; c < mf.count; ++c)
    emit(M, A, p, pair, c, g1, g2, mf.count > 1 ? mf.dist[c] : distance, (mf.one[c] + mf.two[c]) * R(0.5) + origin, fr);
}

// narrowphase family of a candidate pair (-1: filtered out or unsupported):
// 0 plane-primitive, 1 box family, 2 sphere/capsule, 3 plane-mesh, 4 convex
template <class R, int CONVEX> __device__ int pair_family(const Mdl<R> &M, const Arena<R> &A, int pair) {
  const int g1 = IF(pair_geom)[2 * pair], g2 = IF(pair_geom)[2 * pair + 1];
  if (!candidate(M, A, g1, g2)) return -1;
  const int t1 = IF(geom_type)[g1], t2 = IF(geom_type)[g2];
  if (t2 == B200_GEOM_MESH) return CONVEX ? (t1 == B200_GEOM_PLANE ? 3 : 4) : -1;
  if (t1 == B200_GEOM_PLANE && t2 >= 2 && t2 <= 6) return 0;
  if (t1 == B200_GEOM_BOX && t2 == B200_GEOM_BOX && M.m.boxbox_convex) return CONVEX == 2 ? 4 : -1;
  if (t2 == B200_GEOM_BOX && (t1 == B200_GEOM_SPHERE || t1 == B200_GEOM_CAPSULE || t1 == B200_GEOM_BOX)) return 1;
  if ((t1 == B200_GEOM_SPHERE || t1 == B200_GEOM_CAPSULE) && (t2 == B200_GEOM_SPHERE || t2 == B200_GEOM_CAPSULE))
    return 2;
  return -1;
}

template <class R, int CONVEX> __device__ void narrow_pair(const Mdl<R> &M, Arena<R> &A, int pair, int family) {
  const int g1 = IF(pair_geom)[2 * pair], g2 = IF(pair_geom)[2 * pair + 1];
  if (family == 0) plane_pair(M, A, pair, g1, g2);
  else if (family == 1) box_pair(M, A, pair, g1, g2);
  else if (family == 2) prim_pair(M, A, pair, g1, g2);
  else if constexpr (CONVEX) {
    if (family == 3) plane_mesh(M, A, material(M, g1, g2), pair, g1, g2);
    else if (family == 4) {
      if constexpr (CONVEX == 2) {
        if (IF(geom_type)[g1] == B200_GEOM_BOX && IF(geom_type)[g2] == B200_GEOM_BOX &&
            RF(geom_margin)[g1] + RF(geom_margin)[g2] == R(0)) {
          convex_box_pair(M, A, pair, g1, g2);
          return;
        }
      }
      convex_pair(M, A, pair, g1, g2);
    }
  }
}

}  // namespace b200
