/* Portions restate MuJoCo Warp formulas: Copyright 2025 The Newton Developers,
 * SPDX-License-Identifier: Apache-2.0 (see NOTICE). */
/* Narrowphase families beyond plane/box (included by oracle.c; test
 * infrastructure only).
 *
 * Primitive sphere/capsule pairs follow MuJoCo's colliders that the
 * reference's native engine carries (libero/libero/gpu/cuda/collision/
 * collision_detect_primitive.cuh: _SphereSphere :261-292, mjc_SphereCapsule
 * :306-322, mjc_CapsuleCapsule :401-490, including the two-contact parallel
 * case).  Plane-mesh follows the FP32 engine's polygon manifold
 * (mjwarp_plane.cu, restated in tools/validation/mjwarp_plane_reference.py
 * mesh_manifold): the deepest vertex, then up to three more vertices of its
 * most plane-facing incident face.  Convex pairs (anything against a mesh)
 * follow the reference's CCD contract (mjwarp_convex_collision.cuh:46-78,
 * mjwarp_convex_epa.cuh gjk_phase): supports inflated by half the pair margin
 * on each shape, sphere and capsule cores shrunk to a point / segment first,
 * GJK distance with a separation cutoff, EPA for penetration, one contact at
 * the witness midpoint whose normal is x1 - x2 when the inflated shapes
 * overlap.  The GJK distance subalgorithm here searches the sub-simplices of
 * the current simplex that contain the newest support point (the minimum-norm
 * point of the best face whose affine weights are positive), and EPA is the expanding
 * polytope method of van den Bergen (2001); both give the reference's
 * geometric answer (distance, depth, normal) to the CCD tolerance.
 */

/* ------------------------------------------------------------ primitives */
typedef struct { int count; real dist[2]; V3 pos[2], normal[2]; } PrimOut;

/* MuJoCo _SphereSphere: depth along the centre line; coincident centres use
 * the cross product of the two z axes, then +x when that is shorter than
 * mjMINVAL (mju_normalize3's rule; collision_detect_primitive.cuh:276-283) */
static int prim_sphere_sphere(PrimOut *o, real margin, V3 p1, const real *m1, real r1, V3 p2, const real *m2, real r2) {
  V3 dif = vsub(p1, p2);
  real cd2 = vdot(dif, dif), mind = margin + r1 + r2;
  if (cd2 > mind * mind) return 0;
  int c = o->count;
  real dist = rsqrt_(cd2) - r1 - r2;
  V3 n = vsub(p2, p1);
  real len = rsqrt_(vdot(n, n));
  if (len < R(1e-15)) {
    n = vcross(mcol(m1, 2), mcol(m2, 2));
    len = rsqrt_(vdot(n, n));
    n = len < R(1e-15) ? v3(1, 0, 0) : vscale(n, R(1) / len);
  } else
    n = vscale(n, R(1) / len);
  o->dist[c] = dist;
  o->normal[c] = n;
  o->pos[c] = vadd(p1, vscale(n, r1 + dist * R(0.5)));
  o->count = c + 1;
  return 1;
}

static void prim_sphere_capsule(PrimOut *o, real margin, V3 p1, const real *m1, real r1, V3 p2, const real *m2,
                                real r2, real hl) {
  V3 axis = mcol(m2, 2);
  real x = rclamp(vdot(axis, vsub(p1, p2)), -hl, hl);
  prim_sphere_sphere(o, margin, p1, m1, r1, vadd(p2, vscale(axis, x)), m2, r2);
}

static void prim_capsule_capsule(PrimOut *o, real margin, V3 p1, const real *m1, const real *s1, V3 p2,
                                 const real *m2, const real *s2) {
  V3 a1 = vscale(mcol(m1, 2), s1[1]), a2 = vscale(mcol(m2, 2), s2[1]), dif = vsub(p1, p2);
  real ma = vdot(a1, a1), mb = -vdot(a1, a2), mc = vdot(a2, a2), u = -vdot(a1, dif), v = vdot(a2, dif);
  real det = ma * mc - mb * mb;
  if (rabs(det) >= R(1e-15)) {
    real x1 = (mc * u - mb * v) / det, x2 = (ma * v - mb * u) / det;
    if (x1 > 1) { x1 = 1; x2 = (v - mb) / mc; }
    else if (x1 < -1) { x1 = -1; x2 = (v + mb) / mc; }
    if (x2 > 1) { x2 = 1; x1 = rclamp((u - mb) / ma, -1, 1); }
    else if (x2 < -1) { x2 = -1; x1 = rclamp((u + mb) / ma, -1, 1); }
    prim_sphere_sphere(o, margin, vadd(p1, vscale(a1, x1)), m1, s1[0], vadd(p2, vscale(a2, x2)), m2, s2[0]);
    return;
  }
  /* parallel axes: segment ends of capsule 1, then of capsule 2 */
  real x2 = rclamp((v - mb) / mc, -1, 1);
  int n = prim_sphere_sphere(o, margin, vadd(p1, a1), m1, s1[0], vadd(p2, vscale(a2, x2)), m2, s2[0]);
  x2 = rclamp((v + mb) / mc, -1, 1);
  n += prim_sphere_sphere(o, margin, vsub(p1, a1), m1, s1[0], vadd(p2, vscale(a2, x2)), m2, s2[0]);
  if (n >= 2) return;
  real x1 = rclamp((u - mb) / ma, -1, 1);
  n += prim_sphere_sphere(o, margin, vadd(p1, vscale(a1, x1)), m1, s1[0], vadd(p2, a2), m2, s2[0]);
  if (n >= 2) return;
  x1 = rclamp((u + mb) / ma, -1, 1);
  prim_sphere_sphere(o, margin, vadd(p1, vscale(a1, x1)), m1, s1[0], vsub(p2, a2), m2, s2[0]);
}

static void prim_collide(Work *k, const B200Model *m, int g1, int g2) {
  Material p = material(m, g1, g2);
  int t1 = MI(geom_type)[g1], t2 = MI(geom_type)[g2];
  V3 p1 = vload(k->gxpos[g1]), p2 = vload(k->gxpos[g2]);
  const real *m1 = k->gxmat[g1], *m2 = k->gxmat[g2], *s1 = MF(geom_size) + 3 * g1, *s2 = MF(geom_size) + 3 * g2;
  PrimOut o;
  o.count = 0;
  real margin = p.margin + p.gap;
  if (t1 == B200_GEOM_SPHERE && t2 == B200_GEOM_SPHERE) prim_sphere_sphere(&o, margin, p1, m1, s1[0], p2, m2, s2[0]);
  else if (t1 == B200_GEOM_SPHERE && t2 == B200_GEOM_CAPSULE) prim_sphere_capsule(&o, margin, p1, m1, s1[0], p2, m2, s2[0], s2[1]);
  else prim_capsule_capsule(&o, margin, p1, m1, s1, p2, m2, s2);
  for (int c = 0; c < o.count; ++c) {
    real frame[9];
    contact_frame(o.normal[c], frame);
    publish(k, m, &p, g1, g2, o.dist[c], o.pos[c], frame);
  }
}

/* ------------------------------------------------------------ plane - mesh */
static void plane_mesh(Work *k, const B200Model *m, const Material *p, int g1, int g2, V3 n, V3 origin) {
  int mesh = MI(geom_dataid)[g2];
  V3 center = vload(k->gxpos[g2]);
  const real *Rg = k->gxmat[g2], *vert = MF(mesh_vert) + 3 * MI(mesh_vertadr)[mesh];
  int nvert = MI(mesh_vertnum)[mesh];
  V3 local = mrotT(Rg, n);
  int best = 0;
  real top = -vdot(vload(vert), local);
  for (int i = 1; i < nvert; ++i) {
    real s = -vdot(vload(vert + 3 * i), local);
    if (s > top) { top = s; best = i; }
  }
  real frame[9];
  contact_frame(n, frame);
  V3 world = vadd(center, mrot(Rg, vload(vert + 3 * best)));
  real dist = vdot(n, vsub(world, origin));
  publish(k, m, p, g1, g2, dist, vsub(world, vscale(n, R(0.5) * dist)), frame);
  if (MI(mesh_polynum)[mesh] <= 0 || dist > p->margin + p->gap) return;
  /* most plane-facing polygon among those at the deepest vertex */
  int vglobal = MI(mesh_vertadr)[mesh] + best;
  int madr = MI(mesh_polymapadr)[vglobal], mnum = MI(mesh_polymapnum)[vglobal];
  int pbase = MI(mesh_polyadr)[mesh], face = -1;
  real lowest = R(1);
  for (int f = 0; f < mnum; ++f) {
    int poly = pbase + MI(mesh_polymap)[madr + f];
    real d = vdot(vload(MF(mesh_polynormal) + 3 * poly), local);
    if (d < R(1) && (face < 0 || d < lowest)) { lowest = d; face = poly; }
  }
  if (face < 0) return;
  const int *pv = MI(mesh_polyvert) + MI(mesh_polyvertadr)[face];
  int count = MI(mesh_polyvertnum)[face], a = 0;
  for (int i = 0; i < count; ++i)
    if (pv[i] == best) { a = i; break; }
  int sel[4] = {a, (a + 1) % count, (a + 2) % count, (a + 3) % count};
  if (count > 4) { /* grow the quadrilateral of largest area (mesh_manifold) */
    #define QAREA(b, c, d) (R(0.5) * rsqrt_(vdot(vcross(vsub(vload(vert + 3 * pv[a]), vload(vert + 3 * pv[c])), \
                            vsub(vload(vert + 3 * pv[b]), vload(vert + 3 * pv[d]))), \
                            vcross(vsub(vload(vert + 3 * pv[a]), vload(vert + 3 * pv[c])), \
                            vsub(vload(vert + 3 * pv[b]), vload(vert + 3 * pv[d]))))))
    int b = sel[1], c = sel[2], d = sel[3];
    real cur = QAREA(b, c, d);
    while (QAREA(b, c, (d + 1) % count) > cur) {
      d = (d + 1) % count; cur = QAREA(b, c, d);
      while (QAREA(b, (c + 1) % count, d) > cur) { c = (c + 1) % count; cur = QAREA(b, c, d); }
      while (QAREA((b + 1) % count, c, d) > cur) { b = (b + 1) % count; cur = QAREA(b, c, d); }
    }
    sel[1] = b; sel[2] = c; sel[3] = d;
    #undef QAREA
  }
  int nsel = count < 4 ? count : 4;
  for (int i = 1; i < nsel; ++i) {
    V3 w = vadd(center, mrot(Rg, vload(vert + 3 * pv[sel[i]])));
    if (vdot(n, vsub(w, center)) > 0) continue;
    real d = vdot(n, vsub(w, origin));
    publish(k, m, p, g1, g2, d, vsub(w, vscale(n, R(0.5) * d)), frame);
  }
}

/* ------------------------------------------------------------ convex (GJK / EPA) */
typedef struct {
  int type;
  V3 pos, size;
  const real *rot, *vert;
  int nvert;
  real margin; /* inflation: half the pair margin is added along the support direction */
} CShape;

/* support point of a shape in unit direction d (mjwarp_convex_geometry.cuh:17-68
 * contract); for a box, *corner = the corner index, bit c set for +size on
 * local axis c (a zero component takes the negative end), else -1 */
static V3 cs_support_c(const CShape *s, V3 d, int *corner) {
  V3 p;
  *corner = -1;
  if (s->type == B200_GEOM_SPHERE) return vadd(s->pos, vscale(d, s->size.v[0] + R(0.5) * s->margin));
  V3 l = mrotT(s->rot, d), r;
  if (s->type == B200_GEOM_CAPSULE) {
    r = vscale(l, s->size.v[0]);
    r.v[2] += (l.v[2] > 0 ? 1 : l.v[2] < 0 ? -1 : 0) * s->size.v[1];
  } else if (s->type == B200_GEOM_BOX) {
    for (int c = 0; c < 3; ++c) r.v[c] = (l.v[c] > 0 ? 1 : -1) * s->size.v[c];
    *corner = (l.v[0] > 0) | (l.v[1] > 0) << 1 | (l.v[2] > 0) << 2;
  } else {
    int best = 0;
    real top = vdot(vload(s->vert), l);
    for (int i = 1; i < s->nvert; ++i) {
      real v = vdot(vload(s->vert + 3 * i), l);
      if (v > top) { top = v; best = i; }
    }
    r = vload(s->vert + 3 * best);
  }
  p = vadd(mrot(s->rot, r), s->pos);
  if (s->margin > 0) p = vadd(p, vscale(d, R(0.5) * s->margin));
  return p;
}
static V3 cs_support(const CShape *s, V3 d) { int c; return cs_support_c(s, d, &c); }

typedef struct { V3 w[4], a[4], b[4]; real lam[4]; int n, ca[4], cb[4]; } Simplex;

/* Signed-volume distance sub-algorithm (Montanari, Petrinic and Barbieri,
 * ACM TOG 2017), the method of the reference's
 * libero/libero/gpu/cuda/collision/mjwarp_convex_simplex.cuh:17-72: weights of
 * the simplex point nearest the origin, vertices in the caller's order (the
 * newest support point last); faces whose signed volume disagrees with the
 * whole simplex's are searched recursively, the nearest candidate winning. */
typedef struct { real w[4]; } SvW;
static int sv_same_sign(real a, real b) { return (a > 0 && b > 0) || (a < 0 && b < 0); }
static real vcomp(V3 v, int k) { return v.v[k]; }
static SvW sv_segment(V3 p, V3 q) {
  V3 e = vsub(q, p);
  V3 o = vadd(q, vscale(e, -vdot(q, e) / vdot(e, e)));
  int k = 0;
  real mu = p.v[0] - q.v[0];
  if (rabs(p.v[1] - q.v[1]) >= rabs(mu)) { mu = p.v[1] - q.v[1]; k = 1; }
  if (rabs(p.v[2] - q.v[2]) >= rabs(mu)) { mu = p.v[2] - q.v[2]; k = 2; }
  real c1 = vcomp(o, k) - vcomp(q, k), c2 = vcomp(p, k) - vcomp(o, k);
  SvW r = {{0, 1, 0, 0}};
  if (sv_same_sign(mu, c1) && sv_same_sign(mu, c2)) { r.w[0] = c1 / mu; r.w[1] = c2 / mu; }
  return r;
}
static int sv_plane(V3 a, V3 b, V3 c, V3 *o) {
  V3 ab = vsub(b, a), ac = vsub(c, a), bc = vsub(c, b);
  V3 n = vcross(bc, ab);
  real nv = vdot(n, b), nn = vdot(n, n);
  if (nn == 0) return 0;
  if (nv != 0 && nn > R(1e-15)) { *o = vscale(n, nv / nn); return 1; }
  n = vcross(ab, ac); nv = vdot(n, a); nn = vdot(n, n);
  if (nn == 0) return 0;
  if (nv != 0 && nn > R(1e-15)) { *o = vscale(n, nv / nn); return 1; }
  n = vcross(ac, bc); nv = vdot(n, c); nn = vdot(n, n);
  *o = vscale(n, nv / nn);
  return 1;
}
static real sv_area(V3 p, V3 u, V3 v, int i, int j) {
  V3 a = vsub(u, p), b = vsub(v, p);
  return vcomp(a, i) * vcomp(b, j) - vcomp(a, j) * vcomp(b, i);
}
static SvW sv_triangle(V3 a, V3 b, V3 c) {
  V3 o;
  if (!sv_plane(a, b, c, &o)) return sv_segment(a, b);
  V3 u = vsub(b, a), v = vsub(c, a);
  real myz = u.v[1] * v.v[2] - u.v[2] * v.v[1], mxz = u.v[0] * v.v[2] - u.v[2] * v.v[0], mxy = u.v[0] * v.v[1] - u.v[1] * v.v[0], m;
  int i, j;
  if (rabs(myz) >= rabs(mxz) && rabs(myz) >= rabs(mxy)) { m = myz; i = 1; j = 2; }
  else if (rabs(mxz) >= rabs(mxy)) { m = mxz; i = 0; j = 2; }
  else { m = mxy; i = 0; j = 1; }
  real s1 = sv_area(o, b, c, i, j), s2 = sv_area(o, c, a, i, j), s3 = sv_area(o, a, b, i, j);
  int in1 = sv_same_sign(m, s1), in2 = sv_same_sign(m, s2), in3 = sv_same_sign(m, s3);
  SvW out = {{0, 0, 0, 0}};
  if (in1 && in2 && in3) { out.w[0] = s1 / m; out.w[1] = s2 / m; out.w[2] = s3 / m; return out; }
  real best = R(1e30);
  if (!in1) {
    SvW e = sv_segment(b, c);
    V3 x = vadd(vscale(b, e.w[0]), vscale(c, e.w[1]));
    out.w[0] = 0; out.w[1] = e.w[0]; out.w[2] = e.w[1]; out.w[3] = 0;
    best = vdot(x, x);
  }
  if (!in2) {
    SvW e = sv_segment(a, c);
    V3 x = vadd(vscale(a, e.w[0]), vscale(c, e.w[1]));
    real d = vdot(x, x);
    if (d < best) { out.w[0] = e.w[0]; out.w[1] = 0; out.w[2] = e.w[1]; out.w[3] = 0; best = d; }
  }
  if (!in3) {
    SvW e = sv_segment(a, b);
    V3 x = vadd(vscale(a, e.w[0]), vscale(b, e.w[1]));
    if (vdot(x, x) < best) { out.w[0] = e.w[0]; out.w[1] = e.w[1]; out.w[2] = 0; out.w[3] = 0; }
  }
  return out;
}
static SvW sv_tetrahedron(V3 a, V3 b, V3 c, V3 d) {
  real s1 = -vdot(b, vcross(c, d)), s2 = vdot(a, vcross(c, d)), s3 = -vdot(a, vcross(b, d)), s4 = vdot(a, vcross(b, c));
  real vol = s1 + s2 + s3 + s4;
  int in1 = sv_same_sign(vol, s1), in2 = sv_same_sign(vol, s2), in3 = sv_same_sign(vol, s3), in4 = sv_same_sign(vol, s4);
  SvW out = {{0, 0, 0, 0}};
  if (in1 && in2 && in3 && in4) {
    out.w[0] = s1 / vol; out.w[1] = s2 / vol; out.w[2] = s3 / vol; out.w[3] = s4 / vol;
    return out;
  }
  real best = R(1e30);
  if (!in1) {
    SvW t = sv_triangle(b, c, d);
    V3 x = vadd(vadd(vscale(b, t.w[0]), vscale(c, t.w[1])), vscale(d, t.w[2]));
    out.w[0] = 0; out.w[1] = t.w[0]; out.w[2] = t.w[1]; out.w[3] = t.w[2];
    best = vdot(x, x);
  }
  if (!in2) {
    SvW t = sv_triangle(a, c, d);
    V3 x = vadd(vadd(vscale(a, t.w[0]), vscale(c, t.w[1])), vscale(d, t.w[2]));
    real dd = vdot(x, x);
    if (dd < best) { out.w[0] = t.w[0]; out.w[1] = 0; out.w[2] = t.w[1]; out.w[3] = t.w[2]; best = dd; }
  }
  if (!in3) {
    SvW t = sv_triangle(a, b, d);
    V3 x = vadd(vadd(vscale(a, t.w[0]), vscale(b, t.w[1])), vscale(d, t.w[2]));
    real dd = vdot(x, x);
    if (dd < best) { out.w[0] = t.w[0]; out.w[1] = t.w[1]; out.w[2] = 0; out.w[3] = t.w[2]; best = dd; }
  }
  if (!in4) {
    SvW t = sv_triangle(a, b, c);
    V3 x = vadd(vadd(vscale(a, t.w[0]), vscale(b, t.w[1])), vscale(c, t.w[2]));
    if (vdot(x, x) < best) { out.w[0] = t.w[0]; out.w[1] = t.w[1]; out.w[2] = t.w[2]; out.w[3] = 0; }
  }
  return out;
}

/* keep the vertices with nonzero weight (order kept); the weights become the
 * affine coordinates of the nearest point (mjwarp_convex_gjk.cuh:71-75) */
static void simplex_reduce(Simplex *s) {
  SvW W = {{1, 0, 0, 0}};
  if (s->n == 4) W = sv_tetrahedron(s->w[0], s->w[1], s->w[2], s->w[3]);
  else if (s->n == 3) W = sv_triangle(s->w[0], s->w[1], s->w[2]);
  else if (s->n == 2) W = sv_segment(s->w[0], s->w[1]);
  Simplex t;
  int k = 0;
  for (int i = 0; i < s->n; ++i)
    if (W.w[i] != 0) {
      t.w[k] = s->w[i]; t.a[k] = s->a[i]; t.b[k] = s->b[i]; t.lam[k] = W.w[i]; t.ca[k] = s->ca[i]; t.cb[k] = s->cb[i];
      ++k;
    }
  t.n = k;
  *s = t;
}

typedef struct { int separated; real dist; V3 x1, x2; Simplex s; } GjkOut;

/* distance between two convex shapes; `cutoff` > 0 ends early once the
 * distance is proven larger (reference gjk_distance cutoff semantics) */
static GjkOut gjk(const CShape *A, const CShape *B, real tol, int iterations, real cutoff) {
  GjkOut o;
  memset(&o, 0, sizeof(o));
  Simplex *s = &o.s;
  s->n = 0;
  V3 x = vsub(A->pos, B->pos);
  real norm = rsqrt_(vdot(x, x)), prev = -1;
  for (int it = 0; it < iterations; ++it) {
    if (norm < tol || rabs(prev - norm) < R(1e-15)) break;
    V3 d = vscale(x, R(1) / norm);
    int ca, cb;
    V3 a = cs_support_c(A, vneg(d), &ca), b = cs_support_c(B, d, &cb), w = vsub(a, b);
    if (vdot(x, vsub(x, w)) < R(0.5) * tol * tol) break;
    real lower = vdot(x, w);
    if (lower > 0 && (cutoff == 0 || lower >= cutoff * norm)) {
      o.separated = 1; o.dist = R(1e30);
      return o;
    }
    s->w[s->n] = w; s->a[s->n] = a; s->b[s->n] = b; s->ca[s->n] = ca; s->cb[s->n] = cb; s->n++;
    simplex_reduce(s);
    if (s->n < 1) break;
    x = v3(0, 0, 0);
    for (int i = 0; i < s->n; ++i) x = vadd(x, vscale(s->w[i], s->lam[i]));
    prev = norm;
    norm = rsqrt_(vdot(x, x));
    if (s->n == 4) break;
  }
  o.x1 = v3(0, 0, 0); o.x2 = v3(0, 0, 0);
  for (int i = 0; i < s->n; ++i) { o.x1 = vadd(o.x1, vscale(s->a[i], s->lam[i])); o.x2 = vadd(o.x2, vscale(s->b[i], s->lam[i])); }
  if (s->n == 0) { o.x1 = A->pos; o.x2 = B->pos; }
  o.dist = s->n == 4 ? 0 : norm;
  return o;
}

#define EPA_MAXV 48
#define EPA_MAXF 96
typedef struct {
  V3 w[EPA_MAXV], a[EPA_MAXV], b[EPA_MAXV];
  int ca[EPA_MAXV], cb[EPA_MAXV]; /* box support corners (-1: not a box) */
  int nv, nf, face[EPA_MAXF][3];
  V3 n[EPA_MAXF];
  real d[EPA_MAXF];
  int alive[EPA_MAXF];
} Polytope;

/* drop dead faces, keeping the live ones in order (ties in the best-face
 * search go to the lower index) */
static void epa_compact(Polytope *P) {
  int k = 0;
  for (int f = 0; f < P->nf; ++f) {
    if (!P->alive[f]) continue;
    if (k != f) {
      memcpy(P->face[k], P->face[f], sizeof(P->face[f]));
      P->n[k] = P->n[f]; P->d[k] = P->d[f]; P->alive[k] = 1;
    }
    ++k;
  }
  P->nf = k;
}

/* new face: its index, -1 when degenerate, -2 when the pool is full */
static int epa_add_face(Polytope *P, int i, int j, int l) {
  if (P->nf >= EPA_MAXF) epa_compact(P);
  if (P->nf >= EPA_MAXF) return -2;
  V3 n = vcross(vsub(P->w[j], P->w[i]), vsub(P->w[l], P->w[i]));
  real len = rsqrt_(vdot(n, n));
  if (!(len > R(1e-30))) return -1;
  n = vscale(n, R(1) / len);
  int f = P->nf++;
  P->face[f][0] = i; P->face[f][1] = j; P->face[f][2] = l;
  P->n[f] = n; P->d[f] = vdot(n, P->w[i]); P->alive[f] = 1;
  return f;
}

static int epa_push(Polytope *P, const CShape *A, const CShape *B, V3 d) {
  if (P->nv >= EPA_MAXV) return -1;
  int v = P->nv++;
  P->a[v] = cs_support_c(A, d, &P->ca[v]); P->b[v] = cs_support_c(B, vneg(d), &P->cb[v]);
  P->w[v] = vsub(P->a[v], P->b[v]);
  return v;
}

/* grow the GJK simplex to a tetrahedron that encloses the origin; 0 if the
 * shapes only touch (no volume around the origin) */
static int epa_seed(Polytope *P, const CShape *A, const CShape *B, const Simplex *s) {
  P->nv = 0; P->nf = 0;
  for (int i = 0; i < s->n; ++i) {
    P->w[i] = s->w[i]; P->a[i] = s->a[i]; P->b[i] = s->b[i]; P->ca[i] = s->ca[i]; P->cb[i] = s->cb[i];
  }
  P->nv = s->n;
  static const real axes[6][3] = {{1, 0, 0}, {-1, 0, 0}, {0, 1, 0}, {0, -1, 0}, {0, 0, 1}, {0, 0, -1}};
  for (int k = 0; P->nv < 2 && k < 6; ++k) {
    int v = epa_push(P, A, B, v3(axes[k][0], axes[k][1], axes[k][2]));
    if (v == 0) continue; /* an empty simplex (coincident centres): the first vertex seeds */
    V3 e = vsub(P->w[v], P->w[0]);
    if (vdot(e, e) < R(1e-20)) P->nv--;
  }
  if (P->nv < 2) return 0;
  if (P->nv == 2) {
    V3 e = vsub(P->w[1], P->w[0]);
    int m = 0;
    for (int c = 1; c < 3; ++c) if (rabs(e.v[c]) < rabs(e.v[m])) m = c;
    V3 ax = v3(0, 0, 0);
    ax.v[m] = 1;
    V3 d = vnormalize(vcross(e, ax));
    int v = epa_push(P, A, B, d);
    V3 cr = vcross(vsub(P->w[v], P->w[0]), e);
    if (vdot(cr, cr) < R(1e-20)) { P->nv--; v = epa_push(P, A, B, vneg(d)); cr = vcross(vsub(P->w[v], P->w[0]), e); }
    if (vdot(cr, cr) < R(1e-20)) return 0;
  }
  if (P->nv == 3) {
    V3 n = vnormalize(vcross(vsub(P->w[1], P->w[0]), vsub(P->w[2], P->w[0])));
    int v = epa_push(P, A, B, n);
    real h = vdot(n, vsub(P->w[v], P->w[0]));
    if (rabs(h) < R(1e-12) || vdot(n, P->w[0]) > 0) { /* take the other side: the origin must lie between */
      P->nv--;
      v = epa_push(P, A, B, vneg(n));
      h = vdot(n, vsub(P->w[v], P->w[0]));
    }
    if (rabs(h) < R(1e-12)) return 0;
  }
  /* orient the tetrahedron's faces outward */
  V3 c = vscale(vadd(vadd(P->w[0], P->w[1]), vadd(P->w[2], P->w[3])), R(0.25));
  static const int tf[4][3] = {{0, 1, 2}, {0, 3, 1}, {0, 2, 3}, {1, 3, 2}};
  for (int f = 0; f < 4; ++f) {
    int i = tf[f][0], j = tf[f][1], l = tf[f][2];
    V3 n = vcross(vsub(P->w[j], P->w[i]), vsub(P->w[l], P->w[i]));
    if (vdot(n, vsub(P->w[i], c)) < 0) { int t = j; j = l; l = t; }
    if (epa_add_face(P, i, j, l) < 0) return 0;
    if (P->d[P->nf - 1] < -R(1e-12)) return 0; /* origin outside the tetrahedron */
  }
  return 1;
}

/* budget: a vertex/face pool filled; horizon: the edge list did; face_*: the
 * final face's vertices (support points and box corners) */
typedef struct {
  int ok, budget, horizon;
  real depth;
  V3 x1, x2, face_a[3], face_b[3];
  int face_ca[3], face_cb[3];
} EpaOut;

/* discrete: two zero-margin boxes; EPA stops within 1e-7 or on a repeated
 * corner pair (mjwarp_convex_epa.cuh epa_expand), on a face of the Minkowski
 * difference itself */
static EpaOut epa(const CShape *A, const CShape *B, const Simplex *s, real tol, int iterations, int discrete) {
  EpaOut o;
  memset(&o, 0, sizeof(o));
  Polytope P;
  if (!epa_seed(&P, A, B, s)) return o;
  real eps = discrete ? R(1e-7) : tol;
  int best = -1;
  for (int it = 0; it <= iterations; ++it) {
    best = -1;
    for (int f = 0; f < P.nf; ++f)
      if (P.alive[f] && (best < 0 || P.d[f] < P.d[best])) best = f;
    if (best < 0) return o;
    if (it == iterations) break;
    V3 n = P.n[best];
    int v = epa_push(&P, A, B, n);
    if (v < 0) { o.budget = 1; break; }
    if (vdot(P.w[v], n) - P.d[best] < eps) { P.nv--; break; }
    if (discrete) {
      int repeated = 0;
      for (int q = 0; q < v; ++q) repeated |= P.ca[q] == P.ca[v] && P.cb[q] == P.cb[v];
      if (repeated) { P.nv--; break; }
    }
    /* remove the faces that see the new vertex; keep their horizon */
    int edges[3 * EPA_MAXF][2], ne = 0;
    for (int f = 0; f < P.nf; ++f) {
      if (!P.alive[f] || vdot(P.n[f], vsub(P.w[v], P.w[P.face[f][0]])) <= 0) continue;
      P.alive[f] = 0;
      for (int e = 0; e < 3; ++e) {
        int i = P.face[f][e], j = P.face[f][(e + 1) % 3], dup = -1;
        for (int q = 0; q < ne; ++q)
          if (edges[q][0] == j && edges[q][1] == i) { dup = q; break; }
        if (dup >= 0) { edges[dup][0] = edges[ne - 1][0]; edges[dup][1] = edges[ne - 1][1]; --ne; }
        else if (ne < 3 * EPA_MAXF) { edges[ne][0] = i; edges[ne][1] = j; ++ne; }
        else o.horizon = 1;
      }
    }
    int full = 0;
    for (int q = 0; q < ne; ++q) {
      int f = epa_add_face(&P, edges[q][0], edges[q][1], v);
      if (f < 0) { full = 1; o.budget |= f == -2; break; }
    }
    if (full || o.horizon) break;
  }
  if (best < 0) return o;
  /* witness points: barycentric coordinates of the origin's projection */
  int i = P.face[best][0], j = P.face[best][1], l = P.face[best][2];
  V3 p = vscale(P.n[best], P.d[best]);
  V3 e0 = vsub(P.w[j], P.w[i]), e1 = vsub(P.w[l], P.w[i]), e2 = vsub(p, P.w[i]);
  real d00 = vdot(e0, e0), d01 = vdot(e0, e1), d11 = vdot(e1, e1), d20 = vdot(e2, e0), d21 = vdot(e2, e1);
  real den = d00 * d11 - d01 * d01;
  real lv = den != 0 ? (d11 * d20 - d01 * d21) / den : 0, lw = den != 0 ? (d00 * d21 - d01 * d20) / den : 0;
  real lu = 1 - lv - lw;
  o.x1 = vadd(vadd(vscale(P.a[i], lu), vscale(P.a[j], lv)), vscale(P.a[l], lw));
  o.x2 = vadd(vadd(vscale(P.b[i], lu), vscale(P.b[j], lv)), vscale(P.b[l], lw));
  o.depth = P.d[best];
  int fv[3] = {i, j, l};
  for (int q = 0; q < 3; ++q) {
    o.face_a[q] = P.a[fv[q]]; o.face_b[q] = P.b[fv[q]]; o.face_ca[q] = P.ca[fv[q]]; o.face_cb[q] = P.cb[fv[q]];
  }
  o.ok = 1;
  return o;
}

/* ---- box manifold (mjwarp_box_manifold.cuh box_multicontact): EPA's final
 * face names a feature of each box by its corners; anti-parallel face normals
 * (within 5.1 degrees), or a face normal and a perpendicular edge, pick the
 * reference and incident faces; the incident polygon is clipped by the
 * reference face's side planes, and the points below that face are the
 * contacts (at most four) */
#define BOX_ALIGNED R(0.99605101346969604)
#define BOX_PERPENDICULAR R(0.088782943785190582)
typedef struct { int count; V3 one[4], two[4]; real dist[4]; } BoxManifold;
typedef struct { int dim, corner[3]; V3 pt[3]; } BoxFeature;
typedef struct { int count, face[3]; V3 n[3]; } BoxNormals;

static BoxFeature box_feature(const int *corner, const V3 *pt) {
  BoxFeature f;
  for (int q = 0; q < 3; ++q) { f.corner[q] = corner[q]; f.pt[q] = pt[q]; }
  if (f.corner[0] != f.corner[1]) f.dim = (f.corner[2] == f.corner[0] || f.corner[2] == f.corner[1]) ? 2 : 3;
  else { f.corner[1] = f.corner[2]; f.pt[1] = f.pt[2]; f.dim = f.corner[0] != f.corner[2] ? 2 : 1; }
  return f;
}
static V3 box_axis(const CShape *s, int face) {
  V3 e = v3(0, 0, 0);
  e.v[face / 2] = face % 2 ? -1 : 1;
  return mrot(s->rot, e);
}
static BoxNormals box_normals_near(const CShape *s, V3 d) {
  BoxNormals o;
  o.count = 0;
  V3 l = vnormalize(mrotT(s->rot, d));
  for (int f = 0; f < 6; ++f)
    if ((f % 2 ? -l.v[f / 2] : l.v[f / 2]) > BOX_ALIGNED) { o.count = 1; o.face[0] = f; o.n[0] = box_axis(s, f); return o; }
  return o;
}
static BoxNormals box_normals(const CShape *s, const BoxFeature *f, V3 d) {
  BoxNormals o;
  o.count = 0;
  if (f->dim == 1) {
    o.count = 3;
    for (int c = 0; c < 3; ++c) { o.face[c] = 2 * c + ((f->corner[0] >> c) & 1 ? 0 : 1); o.n[c] = box_axis(s, o.face[c]); }
    return o;
  }
  for (int c = 0; c < 3; ++c) {
    int all = 1, none = 1;
    for (int i = 0; i < f->dim; ++i) { int set = (f->corner[i] >> c) & 1; all &= set; none &= !set; }
    if (all || none) { o.face[o.count] = 2 * c + (all ? 0 : 1); o.n[o.count] = box_axis(s, o.face[o.count]); ++o.count; }
  }
  if ((f->dim == 3 && o.count == 1) || (f->dim == 2 && o.count >= 1)) return o;
  return box_normals_near(s, d);
}
static BoxNormals box_edges(const CShape *s, const BoxFeature *f, V3 *end) {
  BoxNormals o;
  o.count = 0;
  if (f->dim == 2) { end[0] = f->pt[1]; o.n[0] = vnormalize(vsub(f->pt[1], f->pt[0])); o.count = 1; }
  else if (f->dim == 1) {
    V3 c;
    for (int q = 0; q < 3; ++q) c.v[q] = (f->corner[0] >> q) & 1 ? s->size.v[q] : -s->size.v[q];
    for (int q = 0; q < 3; ++q) {
      V3 e = c;
      e.v[q] = -e.v[q];
      end[q] = vadd(mrot(s->rot, e), s->pos);
      o.n[q] = vnormalize(vsub(end[q], f->pt[0]));
    }
    o.count = 3;
  }
  return o;
}
static void box_face_corners(const CShape *s, int face, V3 *v) {
  static const unsigned char winding[6][4] = {{7, 3, 1, 5}, {2, 6, 4, 0}, {2, 3, 7, 6}, {4, 5, 1, 0}, {6, 7, 5, 4}, {3, 2, 0, 1}};
  for (int i = 0; i < 4; ++i) {
    V3 c;
    for (int q = 0; q < 3; ++q) c.v[q] = (winding[face][i] >> q) & 1 ? s->size.v[q] : -s->size.v[q];
    v[i] = vadd(mrot(s->rot, c), s->pos);
  }
}
static real quad_area(V3 a, V3 b, V3 c, V3 d) {
  V3 n = vcross(vsub(a, c), vsub(b, d));
  return R(0.5) * rsqrt_(vdot(n, n));
}
static void largest_quad(const V3 *p, int n, int *q) {
  int b = 1, c = 2, d = 3;
  q[0] = 0; q[1] = b; q[2] = c; q[3] = d;
  real area = quad_area(p[0], p[b], p[c], p[d]);
  for (int a = 0; a < n; ++a) {
    for (;;) {
      real next = quad_area(p[a], p[b], p[c], p[(d + 1) % n]);
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
      if (c == b) { c = (c + 1) % n; if (d == c) d = (d + 1) % n; }
    }
  }
}
static BoxManifold clip_faces(const V3 *ref, int n1, const V3 *inc, int n2, V3 normal, V3 dir) {
  BoxManifold o;
  o.count = 0;
  if (n1 < 3) return o;
  V3 side[4], buf[2][8];
  real plane[4];
  for (int i = 0; i < n1; ++i) {
    side[i] = vcross(vsub(ref[(i + 1) % n1], ref[i]), vsub(vadd(ref[i], normal), ref[i]));
    plane[i] = vdot(side[i], ref[i]);
  }
  int count = n2, cur = 0;
  for (int i = 0; i < n2; ++i) buf[0][i] = inc[i];
  for (int e = 0; e < n1; ++e) {
    const V3 *in = buf[cur];
    V3 *out = buf[cur ^ 1];
    int m = 0;
    for (int i = 0; i < count; ++i) {
      V3 p = in[i], q = in[(i + 1) % count];
      int inp = vdot(vsub(p, ref[e]), side[e]) > R(-1e-10), inq = vdot(vsub(q, ref[e]), side[e]) > R(-1e-10);
      if (!inp && !inq) continue;
      if (inp && inq) { if (m < 8) out[m++] = q; continue; }
      real den = vdot(side[e], vsub(q, p));
      real s = rabs(den) < R(1e-10) ? R(1e30) : (plane[e] - vdot(side[e], p)) / den;
      if (s > R(-3e-7) && s < R(1) + R(3e-7)) {
        s = s < 0 ? 0 : s > 1 ? 1 : s;
        if (m < 8) out[m++] = vadd(p, vscale(vsub(q, p), s));
      }
      if (inq && m < 8) out[m++] = q;
    }
    cur ^= 1;
    count = m;
  }
  V3 *poly = buf[cur];
  int kept = 0;
  for (int i = 0; i < count; ++i)
    if (vdot(vsub(poly[i], ref[0]), normal) <= 0) poly[kept++] = poly[i];
  count = kept;
  if (count < 1) return o;
  int q[4] = {0, 1, 2, 3};
  if (n2 == 2 && count > 2) {
    real best = 0;
    q[0] = 0; q[1] = 1;
    for (int i = 0; i < count; ++i)
      for (int j = i + 1; j < count; ++j) {
        V3 d = vsub(poly[j], poly[i]);
        if (vdot(d, d) > best) { best = vdot(d, d); q[0] = i; q[1] = j; }
      }
    o.count = 2;
  } else if (count > 4) { largest_quad(poly, count, q); o.count = 4; }
  else o.count = count;
  for (int i = 0; i < o.count; ++i) {
    V3 v = poly[q[i]];
    real d = vdot(vsub(v, ref[0]), normal);
    o.one[i] = vsub(v, vscale(dir, rabs(d)));
    o.two[i] = v;
    o.dist[i] = d;
  }
  return o;
}
static BoxManifold box_manifold(const CShape *A, const CShape *B, const EpaOut *e) {
  BoxManifold none;
  none.count = 0;
  BoxFeature fa = box_feature(e->face_ca, e->face_a), fb = box_feature(e->face_cb, e->face_b);
  V3 dir = vsub(e->x2, e->x1);
  BoxNormals na = box_normals(A, &fa, vneg(dir)), nb = box_normals(B, &fb, dir);
  int i = 0, j = 0, aligned = 0, edge_a = 0, edge_b = 0;
  for (int k = 0; k < na.count && !aligned; ++k)
    for (int l = 0; l < nb.count; ++l)
      if (vdot(na.n[k], nb.n[l]) < -BOX_ALIGNED) { i = k; j = l; aligned = 1; break; }
  V3 end[3];
  if (!aligned) {
    if (fa.dim < 3 && nb.count && (fa.dim <= fb.dim || !na.count)) {
      na = box_edges(A, &fa, end);
      for (int k = 0; k < nb.count && !aligned; ++k) {
        if (vdot(nb.n[k], dir) <= R(1e-15)) continue;
        for (int l = 0; l < na.count; ++l)
          if (rabs(vdot(na.n[l], nb.n[k])) < BOX_PERPENDICULAR) { i = l; j = k; aligned = 1; break; }
      }
      if (!aligned) return none;
      edge_a = 1;
    } else if (fb.dim < 3) {
      nb = box_edges(B, &fb, end);
      for (int k = 0; k < na.count && !aligned; ++k) {
        if (vdot(na.n[k], vneg(dir)) <= R(1e-15)) continue;
        for (int l = 0; l < nb.count; ++l)
          if (rabs(vdot(nb.n[l], na.n[k])) < BOX_PERPENDICULAR) { i = l; j = k; aligned = 1; break; }
      }
      if (!aligned) return none;
      edge_b = 1;
    } else return none;
  }
  V3 face_a[4], face_b[4];
  int count_a = 4, count_b = 4;
  if (edge_a) { face_a[0] = fa.pt[0]; face_a[1] = end[i]; count_a = 2; }
  else box_face_corners(A, na.face[edge_b ? j : i], face_a);
  if (edge_b) { face_b[0] = fb.pt[0]; face_b[1] = end[i]; count_b = 2; }
  else box_face_corners(B, nb.face[j], face_b);
  if (edge_a) {
    BoxManifold r = clip_faces(face_b, count_b, face_a, count_a, nb.n[j], vneg(nb.n[j]));
    for (int k = 0; k < r.count; ++k) { V3 v = r.one[k]; r.one[k] = r.two[k]; r.two[k] = v; }
    return r;
  }
  if (edge_b) return clip_faces(face_a, count_a, face_b, count_b, na.n[j], vneg(na.n[j]));
  return clip_faces(face_a, count_a, face_b, count_b, na.n[i], nb.n[j]);
}

static CShape cs_make(const B200Model *m, const Work *k, int g, V3 origin, real margin) {
  CShape s;
  s.type = MI(geom_type)[g];
  s.pos = vsub(vload(k->gxpos[g]), origin);
  s.size = vload(MF(geom_size) + 3 * g);
  s.rot = k->gxmat[g];
  s.margin = margin;
  s.vert = 0; s.nvert = 0;
  if (s.type == B200_GEOM_MESH) {
    int mesh = MI(geom_dataid)[g];
    s.vert = MF(mesh_vert) + 3 * MI(mesh_vertadr)[mesh];
    s.nvert = MI(mesh_vertnum)[mesh];
  }
  return s;
}

/* one convex pair (mjwarp_convex_collision.cuh:46-78 contract), computed in a
 * frame translated to geom 1 */
static void convex_collide(Work *k, const B200Model *m, int g1, int g2) {
  Material p = material(m, g1, g2);
  V3 origin = vload(k->gxpos[g1]);
  CShape A = cs_make(m, k, g1, origin, p.margin), B = cs_make(m, k, g2, origin, p.margin);
  real tol = (real)m->ccd_tolerance, cutoff = p.gap;
  int iters = m->ccd_iterations;
  real dist;
  V3 x1, x2;
  int found = 0;
  /* sphere / capsule cores first (gjk_phase): distance minus the radii */
  real full1 = 0, full2 = 0;
  CShape Ac = A, Bc = B;
  if (A.type == B200_GEOM_SPHERE || A.type == B200_GEOM_CAPSULE) { full1 = A.size.v[0] + R(0.5) * A.margin; Ac.size.v[0] = 0; Ac.margin = 0; }
  if (B.type == B200_GEOM_SPHERE || B.type == B200_GEOM_CAPSULE) { full2 = B.size.v[0] + R(0.5) * B.margin; Bc.size.v[0] = 0; Bc.margin = 0; }
  if (full1 + full2 > 0) {
    GjkOut r = gjk(&Ac, &Bc, tol, iters, cutoff + full1 + full2);
    if (r.separated) return;
    if (r.dist > tol) {
      V3 nrm = vnormalize(vsub(r.x2, r.x1));
      x1 = vadd(r.x1, vscale(nrm, full1));
      x2 = vsub(r.x2, vscale(nrm, full2));
      dist = r.dist - (full1 + full2);
      found = 1;
    }
  }
  /* two zero-margin boxes: EPA ends on a face of the Minkowski difference and
   * the contact becomes a face manifold (mjwarp_convex_collision.cuh:63-77) */
  int boxes = A.type == B200_GEOM_BOX && B.type == B200_GEOM_BOX && p.margin == 0;
  BoxManifold mf;
  mf.count = 0;
  if (!found) {
    GjkOut r = gjk(&A, &B, tol, iters, cutoff);
    if (r.separated) return;
    if (r.dist > tol) { dist = r.dist; x1 = r.x1; x2 = r.x2; }
    else {
      EpaOut e = epa(&A, &B, &r.s, tol, m->epa_iterations, boxes);
      if (e.budget) k->overflow |= B200_WARN_EPA_BUDGET;
      if (e.horizon) k->overflow |= B200_OVERFLOW_EPA_HORIZON;
      if (!e.ok) { dist = r.dist; x1 = r.x1; x2 = r.x2; }
      else {
        dist = -e.depth; x1 = e.x1; x2 = e.x2;
        if (boxes) mf = box_manifold(&A, &B, &e);
      }
    }
  }
  if (!(dist < p.gap)) return;
  real distance = dist + p.margin;
  if (mf.count < 1) { mf.count = 1; mf.one[0] = x1; mf.two[0] = x2; }
  real frame[9];
  contact_frame(distance <= p.margin ? vsub(mf.one[0], mf.two[0]) : vsub(mf.two[0], mf.one[0]), frame);
  for (int c = 0; c < mf.count; ++c)
    publish(k, m, &p, g1, g2, mf.count > 1 ? mf.dist[c] : distance,
            vadd(vscale(vadd(mf.one[c], mf.two[c]), R(0.5)), origin), frame);
}
