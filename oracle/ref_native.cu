// Contact checker for the sphere and capsule families: drives the reference's
// own native MuJoCo 2.3.7 colliders (test infrastructure only; never part of
// the product library).
//
// The reference's FP32 engine has no sphere-sphere, sphere-capsule or
// capsule-capsule leaf; its native engine carries MuJoCo 2.3.7's colliders as
// device code in libero/libero/gpu/cuda/collision/collision_detect_primitive.cuh
// (mjc_SphereSphere :297-303 over _SphereSphere :261-292, mjc_SphereCapsule
// :306-322, mjc_CapsuleCapsule :401-490), included here unmodified from the
// reference checkout.  oracle/Makefile (target ref) compiles this file the way
// the reference builds its native collision library
// (host/runtime/collision/native.py:91-95: FP64 real_t, -rdc=true, FMA on,
// IEEE division and square root, no flush-to-zero, common/vector.cuh
// pre-included) into oracle/_ref/libref_native.so.
//
// refn_collide() takes HOST arrays: the geom types and sizes, per-world geom
// poses (the poses the B200 kernel used, read back from its geom_xpos /
// geom_xmat outputs), a pair list and one margin per pair; one thread calls
// the collider of each (world, pair).  Everything it allocates it frees before
// returning.
#include <cuda_runtime.h>

#include "collision_detect_primitive.cuh"

namespace {
constexpr int kMaxHits = 2;   // these three colliders return at most two contacts
constexpr int kHitWidth = 7;  // dist, pos[3], normal[3] (the frame's first row)

__global__ void native_pairs(int nworld, int ngeom, int npairs, const int *types, const real_t *size,
                             const real_t *xpos, const real_t *xmat, const int *pairs, const real_t *margin,
                             int *count, real_t *hits) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= nworld * npairs) return;
  const int w = i / npairs, p = i % npairs, g1 = pairs[2 * p], g2 = pairs[2 * p + 1];
  mjModel m{};
  m.geom_size = const_cast<real_t *>(size);
  mjData d{const_cast<real_t *>(xpos + (size_t)w * ngeom * 3), const_cast<real_t *>(xmat + (size_t)w * ngeom * 9)};
  mjContact con[4] = {};
  const int t1 = types[g1], t2 = types[g2];
  int n = -1;  // -1: a family these colliders do not cover
  if (t1 == mjGEOM_SPHERE && t2 == mjGEOM_SPHERE) n = mjc_SphereSphere(&m, &d, con, g1, g2, margin[p]);
  else if (t1 == mjGEOM_SPHERE && t2 == mjGEOM_CAPSULE) n = mjc_SphereCapsule(&m, &d, con, g1, g2, margin[p]);
  else if (t1 == mjGEOM_CAPSULE && t2 == mjGEOM_CAPSULE) n = mjc_CapsuleCapsule(&m, &d, con, g1, g2, margin[p]);
  count[i] = n;
  for (int k = 0; k < n && k < kMaxHits; ++k) {
    real_t *h = hits + ((size_t)i * kMaxHits + k) * kHitWidth;
    h[0] = con[k].dist;
    for (int c = 0; c < 3; ++c) {
      h[1 + c] = con[k].pos[c];
      h[4 + c] = con[k].frame[c];
    }
  }
}

template <class T> cudaError_t upload(T **dst, const T *src, size_t n) {
  cudaError_t rc = cudaMalloc(dst, n * sizeof(T) + 16);
  if (rc == cudaSuccess && n) rc = cudaMemcpy(*dst, src, n * sizeof(T), cudaMemcpyHostToDevice);
  return rc;
}
}  // namespace

extern "C" {
int refn_real_bits() { return (int)(8 * sizeof(real_t)); }
int refn_max_hits() { return kMaxHits; }

// count [nworld * npairs]: contacts per (world, pair), -1 for an uncovered
// family; hits [nworld * npairs, kMaxHits, 7].  Returns a cudaError_t.
int refn_collide(int nworld, int ngeom, int npairs, const int *types, const real_t *size, const real_t *xpos,
                 const real_t *xmat, const int *pairs, const real_t *margin, int *count, real_t *hits) {
  if (nworld <= 0 || ngeom <= 0 || npairs <= 0) return (int)cudaErrorInvalidValue;
  const size_t np = (size_t)nworld * npairs;
  int *d_types = nullptr, *d_pairs = nullptr, *d_count = nullptr;
  real_t *d_size = nullptr, *d_xpos = nullptr, *d_xmat = nullptr, *d_margin = nullptr, *d_hits = nullptr;
  cudaError_t rc = upload(&d_types, types, (size_t)ngeom);
  if (rc == cudaSuccess) rc = upload(&d_size, size, (size_t)ngeom * 3);
  if (rc == cudaSuccess) rc = upload(&d_xpos, xpos, (size_t)nworld * ngeom * 3);
  if (rc == cudaSuccess) rc = upload(&d_xmat, xmat, (size_t)nworld * ngeom * 9);
  if (rc == cudaSuccess) rc = upload(&d_pairs, pairs, (size_t)npairs * 2);
  if (rc == cudaSuccess) rc = upload(&d_margin, margin, (size_t)npairs);
  if (rc == cudaSuccess) rc = cudaMalloc(&d_count, np * sizeof(int));
  if (rc == cudaSuccess) rc = cudaMalloc(&d_hits, np * kMaxHits * kHitWidth * sizeof(real_t));
  if (rc == cudaSuccess) rc = cudaMemset(d_hits, 0, np * kMaxHits * kHitWidth * sizeof(real_t));
  if (rc == cudaSuccess) {
    native_pairs<<<(unsigned)((np + 127) / 128), 128>>>(nworld, ngeom, npairs, d_types, d_size, d_xpos, d_xmat,
                                                         d_pairs, d_margin, d_count, d_hits);
    rc = cudaGetLastError();
  }
  if (rc == cudaSuccess) rc = cudaDeviceSynchronize();
  if (rc == cudaSuccess) rc = cudaMemcpy(count, d_count, np * sizeof(int), cudaMemcpyDeviceToHost);
  if (rc == cudaSuccess)
    rc = cudaMemcpy(hits, d_hits, np * kMaxHits * kHitWidth * sizeof(real_t), cudaMemcpyDeviceToHost);
  cudaFree(d_types); cudaFree(d_size); cudaFree(d_xpos); cudaFree(d_xmat);
  cudaFree(d_pairs); cudaFree(d_margin); cudaFree(d_count); cudaFree(d_hits);
  return (int)rc;
}
}
