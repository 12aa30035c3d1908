// C ABI of the B200 physics step: argument checks, launch shape, dispatch
// to the kernel instances (inst.cu).
#include <cuda_runtime.h>
#include "b200phys.h"
#include "arena.cuh"
#include "launch.h"

#ifndef B200PHYS_SOURCE_ID
#define B200PHYS_SOURCE_ID "b200phys-dev"
#endif

// ============================================================ C ABI
namespace {
constexpr int kMaxWorldsPerCta = 8;

// Largest dynamic shared memory a CTA may opt into on sm_100 (227 KB).
constexpr size_t kSm100OptinSmem = 227 * 1024;

bool model_ok(const B200Model *m) {
  return m && m->real && m->ints && (m->real_bytes == 4 || m->real_bytes == 8) && m->nv >= 1 && m->nv <= 128 &&
         m->nbody >= 2 && m->ncon_max >= 1 && m->nefc_max >= 1 && m->nefc_max <= 65535 && m->nvs >= m->nv && m->nsite > m->ee_site &&
         m->nu >= 9 && m->ntree >= 1 && m->ntree <= 32 && m->kmax_dof >= m->max_tree_dofs &&
         m->nvariant >= 0 && m->variant_stride >= 0;
}
bool data_ok(const B200Data *d) {
  return d && d->nworld >= 0 && d->qpos && d->qvel && d->qacc_warmstart && d->ctrl && d->time && d->goal_pos &&
         d->goal_rot && d->gripper && d->overflow && d->error;
}
size_t arena_for(const B200Model *m) {
  return m->real_bytes == 4 ? b200::Arena<float>::layout(*m, 32, nullptr, nullptr)
                            : b200::Arena<double>::layout(*m, 32, nullptr, nullptr);
}
// Opt-in shared memory per block of the current device, queried on every
// call (a cheap attribute read), so that each device and thread sees its own.
int max_optin_smem() {
  int dev = 0, v = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  if (cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess) return 0;
  return v;
}
// Worlds per CTA: one CTA fills the SM's shared memory.  The worlds of a CTA
// advance through the stages in lockstep, so every warp of the SM runs the
// same stage's code and the instruction caches serve them all.  Two CTAs per
// SM run different stages at a time: on scene A (one-warp worlds) that made
// instruction fetch the largest stall, and eight worlds in one CTA measured
// 79.5 ms per control step against 95.9 ms for two CTAs of four.
int worlds_per_cta(const B200Model *m, int limit) {
  const size_t arena = arena_for(m);
  if (arena == 0 || (int)arena > limit) return 0;
  const int wpc = limit / (int)arena;
  return wpc > kMaxWorldsPerCta ? kMaxWorldsPerCta : wpc;
}
// Launch shape: worlds per CTA and threads per world.  A world is one warp,
// or four warps when at most three worlds fit on an SM (large models), so
// that an SM still runs eight to twelve warps.
struct Shape {
  int wpc, T;
};
template <class R, int C> int prepare_rc(const B200Model *m, const Shape &sh) {
  const size_t smem = (size_t)sh.wpc * arena_for(m);
  return sh.T == 32 ? b200::configure_kernels<R, C, 32>(smem) : b200::configure_kernels<R, C, 128>(smem);
}
// the kernel's convex mode: 2 box-box pairs on the convex path (with or
// without meshes), 1 meshes, 0 neither
int convex_mode(const B200Model *m) { return m->boxbox_convex ? 2 : m->nmesh > 0 ? 1 : 0; }
int launch_shape(const B200Model *m, Shape *sh) {
  const int limit = max_optin_smem();
  sh->wpc = worlds_per_cta(m, limit);
  if (sh->wpc < 1) return (int)cudaErrorInvalidValue;
  const int arena = (int)arena_for(m);
  const int per_sm = ((228 * 1024) / (sh->wpc * arena + 1024)) * sh->wpc;
  sh->T = per_sm <= 3 ? 128 : 32;
  if (sh->T * sh->wpc > 384) sh->wpc = 384 / sh->T;  // the kernels' launch bound
  const int c = convex_mode(m);
  if (m->real_bytes == 4)
    return c == 2 ? prepare_rc<float, 2>(m, *sh) : c ? prepare_rc<float, 1>(m, *sh) : prepare_rc<float, 0>(m, *sh);
  return c == 2 ? prepare_rc<double, 2>(m, *sh) : c ? prepare_rc<double, 1>(m, *sh) : prepare_rc<double, 0>(m, *sh);
}
// kernel instance by precision, convex mode and threads per world
template <template <class, int, int> class F, class R, int C, class... A> void dispatch_t(bool t128, A... a) {
  t128 ? F<R, C, 128>::run(a...) : F<R, C, 32>::run(a...);
}
template <template <class, int, int> class F, class R, class... A> void dispatch_c(int c, bool t128, A... a) {
  if (c == 2) dispatch_t<F, R, 2>(t128, a...);
  else if (c == 1) dispatch_t<F, R, 1>(t128, a...);
  else dispatch_t<F, R, 0>(t128, a...);
}
template <template <class, int, int> class F, class... A> void dispatch(const B200Model *m, const Shape &sh, A... a) {
  if (m->real_bytes == 4) dispatch_c<F, float>(convex_mode(m), sh.T == 128, a...);
  else dispatch_c<F, double>(convex_mode(m), sh.T == 128, a...);
}
// Worlds sorted by their last control step's work into 256 buckets, heaviest
// first (a counting sort in one CTA; worlds within a bucket land in arrival
// order, which changes only which worlds share a CTA, never their results).
__global__ void __launch_bounds__(1024) order_worlds(const int *work, int *order, int n) {
  __shared__ int hist[256];
  __shared__ int top;
  const int t = threadIdx.x;
  if (t == 0) top = 1;
  if (t < 256) hist[t] = 0;
  __syncthreads();
  int mx = 1;
  for (int i = t; i < n; i += blockDim.x) mx = max(mx, work[i]);
  atomicMax(&top, mx);
  __syncthreads();
  const long long scale = top;
  auto bucket = [&](int i) { return 255 - (int)((long long)min(max(work[i], 0), top) * 255 / scale); };
  for (int i = t; i < n; i += blockDim.x) atomicAdd(&hist[bucket(i)], 1);
  __syncthreads();
  if (t == 0) {
    int s = 0;
    for (int k = 0; k < 256; ++k) {
      const int c = hist[k];
      hist[k] = s;
      s += c;
    }
  }
  __syncthreads();
  for (int i = t; i < n; i += blockDim.x) order[atomicAdd(&hist[bucket(i)], 1)] = i;
}

template <class R, int C, int T> struct StepLaunch {
  template <class... A> static void run(A... a) { b200::launch_step<R, C, T>(a...); }
};
template <class R, int C, int T> struct ForwardLaunch {
  template <class... A> static void run(A... a) { b200::launch_forward<R, C, T>(a...); }
};
}  // namespace

extern "C" {
const char *b200phys_source_id(void) { return B200PHYS_SOURCE_ID; }
int b200phys_arch(void) { return 100; }
size_t b200phys_model_bytes(void) { return sizeof(B200Model); }
size_t b200phys_data_bytes(void) { return sizeof(B200Data); }
size_t b200phys_world_smem_bytes(const B200Model *m) {
  if (!model_ok(m)) return 0;
  const size_t arena = arena_for(m);
  return arena <= kSm100OptinSmem ? arena : 0;
}

int b200phys_prepare(const B200Model *m) {
  if (!model_ok(m)) return (int)cudaErrorInvalidValue;
  Shape sh;
  return launch_shape(m, &sh);
}

int b200phys_step_launch(const B200Model *m, const B200Data *d, int substeps, int policy, void *stream) {
  if (!model_ok(m) || !data_ok(d) || substeps < 0) return (int)cudaErrorInvalidValue;
  if (d->nworld == 0 || substeps == 0) return 0;
  Shape sh;
  int rc;
  if ((rc = launch_shape(m, &sh))) return rc;
  const int arena = (int)arena_for(m), grid = (d->nworld + sh.wpc - 1) / sh.wpc;
  dispatch<StepLaunch>(m, sh, *m, *d, substeps, policy, sh.wpc, arena, grid, (size_t)sh.wpc * arena,
                       (cudaStream_t)stream);
  return (int)cudaGetLastError();
}

int b200phys_order_launch(const B200Model *m, const B200Data *d, void *stream) {
  if (!model_ok(m) || !data_ok(d) || !d->work || !d->order) return (int)cudaErrorInvalidValue;
  if (d->nworld == 0) return 0;
  order_worlds<<<1, 1024, 0, (cudaStream_t)stream>>>(d->work, d->order, d->nworld);
  return (int)cudaGetLastError();
}

int b200phys_forward_launch(const B200Model *m, const B200Data *d, int bootstrap, const int *mask, void *stream) {
  if (!model_ok(m) || !data_ok(d)) return (int)cudaErrorInvalidValue;
  if (d->nworld == 0) return 0;
  Shape sh;
  int rc;
  if ((rc = launch_shape(m, &sh))) return rc;
  const int arena = (int)arena_for(m), grid = (d->nworld + sh.wpc - 1) / sh.wpc;
  dispatch<ForwardLaunch>(m, sh, *m, *d, bootstrap, mask, sh.wpc, arena, grid, (size_t)sh.wpc * arena,
                          (cudaStream_t)stream);
  return (int)cudaGetLastError();
}
}
