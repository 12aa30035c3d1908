// Contact-list checker: drives the reference's own FP32 collision leaves
// (test infrastructure only; never part of the product library).
//
// The reference's FP32 engine runs collision as four pooled launches per
// substep (libero/libero/gpu/host/backends/cuda_fp32/physics.py:95-100:
// broadphase, convex, planes, boxes).  oracle/Makefile (target ref) compiles those leaves
// unmodified from the reference checkout
//   libero/libero/gpu/cuda/collision/mjwarp_broadphase.cu  (flash_mjwarp_broadphase_launch)
//   libero/libero/gpu/cuda/collision/mjwarp_convex.cu      (flash_mjwarp_convex_collision_launch)
//   libero/libero/gpu/cuda/collision/mjwarp_plane.cu       (flash_mjwarp_plane_launch)
//   libero/libero/gpu/cuda/collision/mjwarp_box.cu         (flash_mjwarp_box_launch)
// and links them with this file into oracle/_ref/libref_contacts.so.
//
// refc_collide() takes HOST arrays: the geom model and per-world geom poses
// (the poses the B200 kernel used, read back from its geom_xpos/geom_xmat
// outputs), fills the reference's argument packs the way its host bindings do
// (host/runtime/collision/mjwarp_broadphase.py:40-75, mjwarp_plane.py,
// mjwarp_convex_collision.py:47-76), runs the leaves in the reference's order
// on one stream and copies the pooled contact list back.  Everything it
// allocates it frees before returning.
#include <cuda_runtime.h>
#include <cstdio>
#include <cstring>
#include <vector>

#include "mjwarp_broadphase.cuh"
#include "mjwarp_convex.cuh"

using flash::mjwarp::BroadphaseInputs;
using flash::mjwarp::ContactInputs;
using flash::mjwarp::ContactParameter;
using flash::mjwarp::ConvexCollisionInputs;

extern "C" {
int flash_mjwarp_broadphase_launch(const BroadphaseInputs *a, cudaStream_t stream);
int flash_mjwarp_plane_launch(const ContactInputs *a, cudaStream_t stream);
int flash_mjwarp_box_launch(const ContactInputs *a, int boxbox_enabled, cudaStream_t stream);
int flash_mjwarp_convex_collision_launch(const ConvexCollisionInputs *a, cudaStream_t stream);
size_t flash_mjwarp_broadphase_arguments_bytes();
size_t flash_mjwarp_plane_arguments_bytes();
size_t flash_mjwarp_box_arguments_bytes();
size_t flash_mjwarp_convex_collision_arguments_bytes();
}

extern "C" {
// Geom model of one scene, host pointers.  Arrays are per geom unless noted.
typedef struct RefGeomModel {
  int ngeom, npairs, nmesh, nmeshvert, nmeshpoly, nmeshpolyvert, nmeshpolymap;
  int ccd_iterations, boxbox_primitive;
  float ccd_tolerance;
  const int *geom_type, *geom_dataid, *geom_condim, *geom_priority;
  const int *pairs;  // [npairs, 2], g1 < g2: the filtered NXN pair list
  const float *aabb;  // [ngeom, 6]: center, half-size
  const float *rbound, *margin, *gap, *size /*[ngeom,3]*/, *solmix, *solref /*[ngeom,2]*/, *solimp /*[ngeom,5]*/,
      *friction /*[ngeom,3]*/;
  const int *mesh_vertadr, *mesh_vertnum, *mesh_polyadr, *mesh_polynum, *mesh_polyvertadr, *mesh_polyvertnum,
      *mesh_polyvert, *mesh_polymapadr, *mesh_polymapnum, *mesh_polymap;
  const float *mesh_vert, *mesh_polynormal;
} RefGeomModel;

// Contact pool read back from the device.  Arrays hold `capacity` entries.
typedef struct RefContacts {
  int capacity;
  int count, candidates;  // published contacts (may exceed capacity), broadphase survivors
  int *geom;    // [capacity, 2]
  int *world;   // [capacity]
  int *dim;     // [capacity]
  float *dist;  // [capacity]
  float *pos;   // [capacity, 3]
  float *frame; // [capacity, 9]
  int *overflow;  // [nworld] convex overflow bits
} RefContacts;

size_t refc_model_bytes(void) { return sizeof(RefGeomModel); }
size_t refc_contacts_bytes(void) { return sizeof(RefContacts); }
}

namespace {
struct Pool {
  std::vector<void *> ptrs;
  int rc = 0;
  template <class T> T *alloc(size_t n) {
    void *p = nullptr;
    if (rc) return nullptr;
    if (n == 0) n = 1;
    rc = (int)cudaMalloc(&p, n * sizeof(T));
    if (rc) return nullptr;
    cudaMemset(p, 0, n * sizeof(T));
    ptrs.push_back(p);
    return (T *)p;
  }
  template <class T> T *upload(const T *host, size_t n) {
    T *d = alloc<T>(n);
    if (d && host && n) rc = (int)cudaMemcpy(d, host, n * sizeof(T), cudaMemcpyHostToDevice);
    return d;
  }
  ~Pool() {
    for (void *p : ptrs) cudaFree(p);
  }
};
}  // namespace

extern "C" int refc_collide(const RefGeomModel *m, int nworld, const float *xpos, const float *xmat, RefContacts *out) {
  if (!m || !out || nworld < 1 || m->ngeom < 1 || m->npairs < 0 || out->capacity < 1) return (int)cudaErrorInvalidValue;
  const int ng = m->ngeom, np = m->npairs, cap = out->capacity;
  Pool P;
  cudaStream_t stream = 0;
  // ---- model and state
  const int *type = P.upload(m->geom_type, ng), *dataid = P.upload(m->geom_dataid, ng);
  const int *condim = P.upload(m->geom_condim, ng), *priority = P.upload(m->geom_priority, ng);
  const float *aabb = P.upload(m->aabb, (size_t)ng * 6), *rbound = P.upload(m->rbound, ng);
  const float *margin = P.upload(m->margin, ng), *gap = P.upload(m->gap, ng);
  const float *size = P.upload(m->size, (size_t)ng * 3), *solmix = P.upload(m->solmix, ng);
  const float *solref = P.upload(m->solref, (size_t)ng * 2), *solimp = P.upload(m->solimp, (size_t)ng * 5);
  const float *friction = P.upload(m->friction, (size_t)ng * 3);
  float *zeros = P.alloc<float>((size_t)ng * 5);  // adhesion, pair parameters (no explicit pairs)
  int *izeros = P.alloc<int>(ng);
  const float *dxpos = P.upload(xpos, (size_t)nworld * ng * 3), *dxmat = P.upload(xmat, (size_t)nworld * ng * 9);
  std::vector<int> ids((size_t)np * 2, -1);  // (contact pair id, sensor id): geom pairs, no sensors
  const int *pairs_in = P.upload(m->pairs, (size_t)np * 2), *pair_ids_in = P.upload(ids.data(), ids.size());
  // meshes: no vertex graph (graph address -1 selects the exhaustive support search)
  const int nmesh = m->nmesh > 0 ? m->nmesh : 1;
  std::vector<int> graphadr(nmesh, -1);
  const int *mesh_graphadr = P.upload(graphadr.data(), graphadr.size()), *mesh_graph = P.alloc<int>(1);
  const int *mesh_vertadr = P.upload(m->mesh_vertadr, m->nmesh), *mesh_vertnum = P.upload(m->mesh_vertnum, m->nmesh);
  const int *mesh_polyadr = P.upload(m->mesh_polyadr, m->nmesh), *mesh_polynum = P.upload(m->mesh_polynum, m->nmesh);
  const int *mesh_polyvertadr = P.upload(m->mesh_polyvertadr, m->nmeshpoly);
  const int *mesh_polyvertnum = P.upload(m->mesh_polyvertnum, m->nmeshpoly);
  const int *mesh_polyvert = P.upload(m->mesh_polyvert, m->nmeshpolyvert);
  const int *mesh_polymapadr = P.upload(m->mesh_polymapadr, m->nmeshvert);
  const int *mesh_polymapnum = P.upload(m->mesh_polymapnum, m->nmeshvert);
  const int *mesh_polymap = P.upload(m->mesh_polymap, m->nmeshpolymap);
  const float *mesh_vert = P.upload(m->mesh_vert, (size_t)m->nmeshvert * 3);
  const float *mesh_polynormal = P.upload(m->mesh_polynormal, (size_t)m->nmeshpoly * 3);
  // ---- broadphase pool
  const long long ncand = (long long)nworld * np;
  if (ncand > (1LL << 30)) return (int)cudaErrorInvalidValue;
  int *cand_count = P.alloc<int>(1), *cand_geom = P.alloc<int>((size_t)ncand * 2 + 2);
  int *cand_ids = P.alloc<int>((size_t)ncand * 2 + 2), *cand_world = P.alloc<int>((size_t)ncand + 1);
  // ---- contact pool
  int *count = P.alloc<int>(1), *cdim = P.alloc<int>(cap), *cgeom = P.alloc<int>((size_t)cap * 2);
  int *cworld = P.alloc<int>(cap), *ctype = P.alloc<int>(cap), *cid = P.alloc<int>(cap), *caddr = P.alloc<int>(1);
  float *cdist = P.alloc<float>(cap), *cpos = P.alloc<float>((size_t)cap * 3), *cframe = P.alloc<float>((size_t)cap * 9);
  float *cmargin = P.alloc<float>(cap), *cfric = P.alloc<float>((size_t)cap * 5), *csolref = P.alloc<float>((size_t)cap * 2);
  float *csolreff = P.alloc<float>((size_t)cap * 2), *csolimp = P.alloc<float>((size_t)cap * 5), *cadh = P.alloc<float>(cap);
  // ---- convex scratch (mjwarp_convex_collision.py:38-41, 58-66)
  // one EPA slot per broadphase candidate at most
  const int it = m->ccd_iterations, vcap = 10 + 2 * it, fcap = 6 + 5 * it, hcap = 24, naccd = (int)ncand + 1;
  int *nccd = P.alloc<int>(66), *overflow = P.alloc<int>(nworld);
  float *vertices = P.alloc<float>((size_t)naccd * vcap * 3), *projection = P.alloc<float>((size_t)naccd * fcap * 3);
  float *norm2 = P.alloc<float>((size_t)naccd * fcap);
  int *vindex = P.alloc<int>((size_t)naccd * vcap), *face = P.alloc<int>((size_t)naccd * fcap);
  int *horizon = P.alloc<int>((size_t)naccd * hcap);
  float tol = m->ccd_tolerance;
  float *dtol = P.upload(&tol, 1);
  if (P.rc) return P.rc;

  BroadphaseInputs b;
  std::memset(&b, 0, sizeof b);
  b.worlds = nworld; b.geoms = ng; b.pairs = np; b.explicit_pairs = 0; b.capacity = (int)ncand;
  b.filter = 1 | 2 | 8;  // PLANE | SPHERE | OBB (cuda_fp32/model.py:74)
  b.dataid_rows = b.aabb_rows = b.rbound_rows = b.margin_rows = b.gap_rows = 1;
  b.pair_margin_rows = b.pair_gap_rows = 1;
  b.geom_type = type; b.geom_dataid = dataid; b.pairs_in = pairs_in; b.pair_ids_in = pair_ids_in;
  b.aabb = aabb; b.rbound = rbound; b.margin = margin; b.gap = gap; b.pair_margin = zeros; b.pair_gap = zeros;
  b.xpos = dxpos; b.xmat = dxmat;
  b.count = cand_count; b.pairs_out = cand_geom; b.pair_ids_out = cand_ids; b.world_out = cand_world;

  ContactInputs c;
  std::memset(&c, 0, sizeof c);
  c.worlds = nworld; c.geoms = ng; c.explicit_pairs = 0; c.capacity = cap; c.address_columns = 0;
  auto param = [](const float *p) { return ContactParameter{p, 1}; };
  c.size = param(size); c.solmix = param(solmix); c.solref = param(solref); c.solimp = param(solimp);
  c.friction = param(friction); c.margin = param(margin); c.gap = param(gap); c.adhesion = param(zeros);
  c.pair_solref = c.pair_solreffriction = c.pair_solimp = c.pair_friction = param(zeros);
  c.pair_margin = c.pair_gap = c.pair_adhesion = param(zeros);
  c.geom_type = type; c.condim = condim; c.priority = priority; c.pair_dim = izeros; c.geom_dataid = dataid;
  c.dataid_rows = 1;
  c.mesh_vertadr = mesh_vertadr; c.mesh_vertnum = mesh_vertnum; c.mesh_graphadr = mesh_graphadr; c.mesh_graph = mesh_graph;
  c.mesh_polynum = mesh_polynum; c.mesh_polyadr = mesh_polyadr; c.mesh_polyvertadr = mesh_polyvertadr;
  c.mesh_polyvertnum = mesh_polyvertnum; c.mesh_polyvert = mesh_polyvert; c.mesh_polymapadr = mesh_polymapadr;
  c.mesh_polymapnum = mesh_polymapnum; c.mesh_polymap = mesh_polymap; c.mesh_vert = mesh_vert;
  c.mesh_polynormal = mesh_polynormal; c.xpos = dxpos; c.xmat = dxmat;
  c.candidate_count = cand_count; c.candidate_geom = cand_geom; c.candidate_ids = cand_ids; c.candidate_world = cand_world;
  c.contact_count = count; c.contact_dim = cdim; c.contact_geom = cgeom; c.contact_world = cworld; c.contact_type = ctype;
  c.contact_collisionid = cid; c.contact_address = caddr; c.contact_dist = cdist; c.contact_pos = cpos;
  c.contact_frame = cframe; c.contact_margin = cmargin; c.contact_friction = cfric; c.contact_solref = csolref;
  c.contact_solreffriction = csolreff; c.contact_solimp = csolimp; c.contact_adhesion = cadh;

  // convex families present in the pair list (mjwarp_convex_collision.py:5-22); box-box stays
  // primitive when a box-box margin exists (cuda_fp32/physics.py:89-90)
  static const int families[7][2] = {{3, 5}, {3, 7}, {5, 6}, {5, 7}, {6, 6}, {6, 7}, {7, 7}};
  std::vector<int> htype(m->geom_type, m->geom_type + ng);
  ConvexCollisionInputs v;
  std::memset(&v, 0, sizeof v);
  v.contact = c;
  v.tolerance = ContactParameter{dtol, 1};
  v.iterations = it;
  v.naccd = naccd; v.vertex_capacity = vcap; v.face_capacity = fcap; v.horizon_capacity = hcap; v.warn = 0;
  bool all_boxbox = true, any = false;
  for (int f = 0; f < 7; ++f) {
    const int t1 = families[f][0], t2 = families[f][1];
    if (t1 == 6 && t2 == 6 && m->boxbox_primitive) continue;
    bool present = false;
    for (int i = 0; i < np && !present; ++i) {
      int a = htype[m->pairs[2 * i]], bb = htype[m->pairs[2 * i + 1]];
      if (a > bb) { const int t = a; a = bb; bb = t; }
      present = a == t1 && bb == t2;
    }
    if (!present) continue;
    any = true;
    if (!(t1 == 6 && t2 == 6)) all_boxbox = false;
    v.type_pair[2 * v.active_types] = t1;
    v.type_pair[2 * v.active_types + 1] = t2;
    v.type_index[v.active_types] = t1 * (2 * 11 - t1 - 1) / 2 + t2;
    ++v.active_types;
  }
  v.epa_iterations = any && all_boxbox ? 16 : it;
  v.nccd = nccd; v.overflow = overflow; v.vertices = vertices; v.projection = projection; v.norm2 = norm2;
  v.vertex_index = vindex; v.face = face; v.horizon = horizon;

  int rc = flash_mjwarp_broadphase_launch(&b, stream);
  if (!rc) rc = flash_mjwarp_convex_collision_launch(&v, stream);
  if (!rc) rc = flash_mjwarp_plane_launch(&c, stream);
  if (!rc) rc = flash_mjwarp_box_launch(&c, m->boxbox_primitive ? 1 : 0, stream);
  if (!rc) rc = (int)cudaStreamSynchronize(stream);
  if (rc) return rc;
  int n = 0, nc = 0;
  cudaMemcpy(&n, count, sizeof n, cudaMemcpyDeviceToHost);
  cudaMemcpy(&nc, cand_count, sizeof nc, cudaMemcpyDeviceToHost);
  out->count = n;
  out->candidates = nc;
  const int k = n < cap ? n : cap;
  if (out->geom) cudaMemcpy(out->geom, cgeom, sizeof(int) * 2 * k, cudaMemcpyDeviceToHost);
  if (out->world) cudaMemcpy(out->world, cworld, sizeof(int) * k, cudaMemcpyDeviceToHost);
  if (out->dim) cudaMemcpy(out->dim, cdim, sizeof(int) * k, cudaMemcpyDeviceToHost);
  if (out->dist) cudaMemcpy(out->dist, cdist, sizeof(float) * k, cudaMemcpyDeviceToHost);
  if (out->pos) cudaMemcpy(out->pos, cpos, sizeof(float) * 3 * k, cudaMemcpyDeviceToHost);
  if (out->frame) cudaMemcpy(out->frame, cframe, sizeof(float) * 9 * k, cudaMemcpyDeviceToHost);
  if (out->overflow) cudaMemcpy(out->overflow, overflow, sizeof(int) * nworld, cudaMemcpyDeviceToHost);
  return (int)cudaGetLastError();
}

// Argument-pack sizes as the reference leaves report them, checked by the
// Python loader against this translation unit's view of the same structs.
extern "C" int refc_abi_ok(void) {
  return flash_mjwarp_broadphase_arguments_bytes() == sizeof(BroadphaseInputs) &&
         flash_mjwarp_plane_arguments_bytes() == sizeof(ContactInputs) &&
         flash_mjwarp_box_arguments_bytes() == sizeof(ContactInputs) &&
         flash_mjwarp_convex_collision_arguments_bytes() == sizeof(ConvexCollisionInputs);
}
