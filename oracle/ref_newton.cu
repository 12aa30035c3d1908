// Newton-solve checker: drives the reference's own FP32 Newton leaves (test
// infrastructure only; never part of the product library).
//
// The reference's FP32 engine solves each substep's constraint problem with
// five compiled leaves (libero/libero/gpu/host/backends/cuda_fp32/physics.py
// Newton.solve: initialize, then constraint gradient + Hessian + direction,
// then while worlds are solving: line search, constraint gradient + Hessian +
// direction with the stop rule).  oracle/Makefile (target ref) compiles four
// of them unmodified from the reference checkout
//   libero/libero/gpu/cuda/newton/mjwarp_solver_state.cu  (initialize, stop)
//   libero/libero/gpu/cuda/newton/mjwarp_constraint.cu    (row forces, J'f, gradient)
//   libero/libero/gpu/cuda/newton/mjwarp_hessian.cu       (M + J'DJ + cone curvature)
//   libero/libero/gpu/cuda/newton/mjwarp_linesearch.cu    (exact line search)
// and links them with this file into oracle/_ref/libref_newton.so.  The fifth,
// the direction leaf (mjwarp_direction.cu), factors the Hessian with NVIDIA
// MathDx (cuSOLVERDx), which is not installed; this harness replaces it with
// a plain FP32 Cholesky of the Hessian's upper triangle (the triangle the
// leaf's potrf reads), one thread per world, and publishes what the leaf
// publishes: search = -H^-1 grad, |search|^2 and grad . H^-1 grad.  The stop
// rule then runs in the reference's own stop kernel.
//
// refnt_solve() takes HOST arrays in the reference's row layout (rows of a
// world contiguous, contacts pooled), builds the leaves' argument packs the
// way the reference's host plans do (host/runtime/newton/mjwarp_*.py), runs the
// solve on one stream and copies the results back, together with the first
// iteration's intermediate values for piecewise checks.  Everything it
// allocates it frees before returning.
#include <cuda_runtime.h>
#include <cstring>
#include <vector>

#include "mjwarp_constraint.cuh"
#include "mjwarp_direction.cuh"
#include "mjwarp_hessian.cuh"
#include "mjwarp_linesearch.cuh"
#include "mjwarp_solver_state.cuh"

using flash::mjwarp::ConstraintInputs;
using flash::mjwarp::DirectionInputs;
using flash::mjwarp::HessianInputs;
using flash::mjwarp::InitInputs;
using flash::mjwarp::LinesearchInputs;
using flash::mjwarp::StopInputs;

extern "C" {
std::size_t flash_mjwarp_constraint_gradient_bytes();
int flash_mjwarp_constraint_gradient(const ConstraintInputs *, const DirectionInputs *, cudaStream_t);
int flash_mjwarp_linesearch_fused(const LinesearchInputs *, cudaStream_t);
}

extern "C" {
// One batch of frozen Newton problems, host pointers.  Rows of world w are
// [w * rows, w * rows + nefc[w]); contacts are pooled over the batch.
typedef struct RefNewtonCase {
  int nworld, nv, rows, ncon, iterations, ls_iterations;
  float tolerance, ls_tolerance, meaninertia, impratio_invsqrt;
  const int *nefc, *nf;                     // [nworld]
  const float *J;                           // [nworld, rows, nv]
  const float *D, *aref, *frictionloss;     // [nworld, rows]
  const int *row_type, *row_contact;        // [nworld, rows]: MuJoCo constraint type, pooled contact or -1
  const int *con_world, *con_dim;           // [ncon]
  const int *con_address;                   // [ncon, 6]: the contact's rows (world-local), -1 past dim
  const float *con_friction;                // [ncon, 5]
  const float *con_dist, *con_margin;       // [ncon]
  const float *M;                           // [nworld, nv, nv] dense
  const float *qacc_smooth, *qacc_warmstart, *qfrc_smooth;  // [nworld, nv]
} RefNewtonCase;

// Results.  The *0 arrays hold the first iteration's values: the state at the
// initial qacc (rows' jaref and state, the Hessian, the search direction) and
// the first line search's step and improvement.
typedef struct RefNewtonOut {
  float *qacc, *qfrc_constraint;            // [nworld, nv]
  float *force;                             // [nworld, rows]
  int *state, *niter, *overflow;            // [nworld, rows], [nworld], [nworld]
  float *qacc0, *search0, *Ma0, *grad0;     // [nworld, nv]
  float *jaref0;                            // [nworld, rows]
  int *state0;                              // [nworld, rows]
  float *H0;                                // [nworld, nv, nv] (upper triangle holds the cone terms)
  float *alpha0, *improvement0;             // [nworld]
} RefNewtonOut;
}

namespace {
// The direction leaf's contract without MathDx: upper Cholesky H = U'U of the
// Hessian, search = -H^-1 grad, search_dot = |H^-1 grad|^2, decrement =
// grad . H^-1 grad (mjwarp_direction.cu publish).  One thread per world.
__global__ void harness_direction(int nworld, int nv, int pad, const bool *done, const float *hessian, const float *grad,
                                  float *factor, float *search, float *search_dot, float *decrement) {
  const int w = blockIdx.x * blockDim.x + threadIdx.x;
  if (w >= nworld || done[w]) return;
  const float *H = hessian + (size_t)w * pad * pad;
  float *U = factor + (size_t)w * pad * pad;
  for (int i = 0; i < nv; ++i) {
    float diag = H[i * pad + i];
    for (int k = 0; k < i; ++k) diag -= U[k * pad + i] * U[k * pad + i];
    const float root = sqrtf(diag > 0.f ? diag : 1.e-15f);
    U[i * pad + i] = root;
    for (int j = i + 1; j < nv; ++j) {
      float s = H[i * pad + j];
      for (int k = 0; k < i; ++k) s -= U[k * pad + i] * U[k * pad + j];
      U[i * pad + j] = s / root;
    }
  }
  float *x = search + (size_t)w * nv;  // solve U' y = g, then U x = y, in place
  const float *g = grad + (size_t)w * pad;
  for (int i = 0; i < nv; ++i) {
    float s = g[i];
    for (int k = 0; k < i; ++k) s -= U[k * pad + i] * x[k];
    x[i] = s / U[i * pad + i];
  }
  for (int i = nv - 1; i >= 0; --i) {
    float s = x[i];
    for (int k = i + 1; k < nv; ++k) s -= U[i * pad + k] * x[k];
    x[i] = s / U[i * pad + i];
  }
  float square = 0.f, dec = 0.f;
  for (int i = 0; i < nv; ++i) {
    square += x[i] * x[i];
    dec += g[i] * x[i];
    x[i] = -x[i];
  }
  search_dot[w] = square;
  decrement[w] = dec;
}

struct Device {
  std::vector<void *> owned;
  cudaError_t rc = cudaSuccess;
  template <class T> T *alloc(size_t n) {
    T *p = nullptr;
    if (rc == cudaSuccess) rc = cudaMalloc(&p, n * sizeof(T) + 16);
    if (rc == cudaSuccess) rc = cudaMemset(p, 0, n * sizeof(T) + 16);
    if (p) owned.push_back(p);
    return p;
  }
  template <class T> T *upload(const T *src, size_t n) {
    T *p = alloc<T>(n);
    if (rc == cudaSuccess && n) rc = cudaMemcpy(p, src, n * sizeof(T), cudaMemcpyHostToDevice);
    return p;
  }
  template <class T> void download(T *dst, const T *src, size_t n) {
    if (rc == cudaSuccess && dst && n) rc = cudaMemcpy(dst, src, n * sizeof(T), cudaMemcpyDeviceToHost);
  }
  void check(int code) {
    if (rc == cudaSuccess && code) rc = (cudaError_t)code;
  }
  ~Device() {
    for (void *p : owned) cudaFree(p);
  }
};

int pad_for(int nv) {  // the Hessian leaf's admitted padded sizes
  for (int p : {24, 28, 32, 48, 64})
    if (nv <= p) return p;
  return -1;
}
}  // namespace

extern "C" {
size_t refnt_case_bytes() { return sizeof(RefNewtonCase); }
size_t refnt_out_bytes() { return sizeof(RefNewtonOut); }

// The leaves' argument packs must match the reference headers this file was
// compiled against (the same headers the leaves were compiled with).
int refnt_abi_ok() {
  return flash_mjwarp_constraint_arguments_bytes() == sizeof(ConstraintInputs) &&
         flash_mjwarp_constraint_gradient_bytes() == sizeof(DirectionInputs) &&
         flash_mjwarp_hessian_arguments_bytes() == sizeof(HessianInputs) &&
         flash_mjwarp_linesearch_arguments_bytes() == sizeof(LinesearchInputs) &&
         flash_mjwarp_solver_state_init_bytes() == sizeof(InitInputs) &&
         flash_mjwarp_solver_state_stop_bytes() == sizeof(StopInputs);
}

int refnt_solve(const RefNewtonCase *c, RefNewtonOut *o) {
  if (!c || !o || c->nworld < 1 || c->nv < 1 || c->rows < 1 || c->ncon < 0) return (int)cudaErrorInvalidValue;
  const int W = c->nworld, nv = c->nv, R = c->rows, C = c->ncon, pad = pad_for(nv);
  if (pad < 0) return (int)cudaErrorInvalidValue;
  const int Cc = C > 0 ? C : 1;  // the leaves want a positive capacity
  Device dev;
  // model-shaped tables: the mass matrix as dense row-major entries, addressed
  // through a CSR of its structurally non-zero entries (kinematic tree blocks)
  const int mass_entries = nv * nv;
  std::vector<int> mass_row(nv + 1, 0), mass_col, mass_address, upper(pad * pad, -1), tri_row, tri_col;
  std::vector<char> nonzero(nv * nv, 0);
  for (int w = 0; w < W; ++w)
    for (int e = 0; e < nv * nv; ++e)
      if (c->M[(size_t)w * nv * nv + e] != 0.f) nonzero[e] = 1;
  for (int i = 0; i < nv; ++i) {
    for (int j = 0; j < nv; ++j)
      if (nonzero[i * nv + j] || i == j) {
        mass_col.push_back(j);
        mass_address.push_back(i * nv + j);
        upper[i * pad + j] = i * nv + j;
      }
    mass_row[i + 1] = (int)mass_col.size();
  }
  for (int i = 0; i < nv; ++i)
    for (int j = i; j < nv; ++j) { tri_row.push_back(i); tri_col.push_back(j); }
  std::vector<float> J((size_t)W * R * pad, 0.f);
  for (int w = 0; w < W; ++w)
    for (int r = 0; r < R; ++r)
      std::memcpy(&J[((size_t)w * R + r) * pad], c->J + ((size_t)w * R + r) * nv, sizeof(float) * nv);
  std::vector<int> ne(W, 0), count(1, C);
  std::vector<char> done(W, 0);
  const float scalars[4] = {c->impratio_invsqrt, c->tolerance, c->ls_tolerance, c->meaninertia};

  int *d_mass_row = dev.upload(mass_row.data(), mass_row.size());
  int *d_mass_col = dev.upload(mass_col.data(), mass_col.size());
  int *d_mass_address = dev.upload(mass_address.data(), mass_address.size());
  int *d_upper = dev.upload(upper.data(), upper.size());
  int *d_tri_row = dev.upload(tri_row.data(), tri_row.size());
  int *d_tri_col = dev.upload(tri_col.data(), tri_col.size());
  float *d_mass = dev.upload(c->M, (size_t)W * mass_entries);
  float *d_J = dev.upload(J.data(), J.size());
  float *d_D = dev.upload(c->D, (size_t)W * R);
  float *d_aref = dev.upload(c->aref, (size_t)W * R);
  float *d_loss = dev.upload(c->frictionloss, (size_t)W * R);
  int *d_type = dev.upload(c->row_type, (size_t)W * R);
  int *d_rcon = dev.upload(c->row_contact, (size_t)W * R);
  int *d_nefc = dev.upload(c->nefc, (size_t)W);
  int *d_nf = dev.upload(c->nf, (size_t)W);
  int *d_ne = dev.upload(ne.data(), (size_t)W);
  int *d_count = dev.upload(count.data(), 1);
  int *d_cworld = C ? dev.upload(c->con_world, (size_t)C) : dev.alloc<int>(1);
  int *d_cdim = C ? dev.upload(c->con_dim, (size_t)C) : dev.alloc<int>(1);
  int *d_caddr = C ? dev.upload(c->con_address, (size_t)C * 6) : dev.alloc<int>(6);
  float *d_cfric = C ? dev.upload(c->con_friction, (size_t)C * 5) : dev.alloc<float>(5);
  float *d_cdist = C ? dev.upload(c->con_dist, (size_t)C) : dev.alloc<float>(1);
  float *d_cmargin = C ? dev.upload(c->con_margin, (size_t)C) : dev.alloc<float>(1);
  float *d_smooth_acc = dev.upload(c->qacc_smooth, (size_t)W * nv);
  float *d_warm = dev.upload(c->qacc_warmstart, (size_t)W * nv);
  float *d_smooth = dev.upload(c->qfrc_smooth, (size_t)W * nv);
  float *d_scalars = dev.upload(scalars, 4);
  bool *d_done = dev.alloc<bool>(W);
  bool *d_exhausted = dev.alloc<bool>(W);
  bool *d_unchanged = dev.alloc<bool>(W);
  int *d_nsolving = dev.alloc<int>(1);
  float *d_qacc = dev.alloc<float>((size_t)W * nv), *d_ma = dev.alloc<float>((size_t)W * nv);
  float *d_jaref = dev.alloc<float>((size_t)W * R), *d_force = dev.alloc<float>((size_t)W * R);
  int *d_state = dev.alloc<int>((size_t)W * R), *d_niter = dev.alloc<int>(W), *d_overflow = dev.alloc<int>(W);
  float *d_qfrc = dev.alloc<float>((size_t)W * nv), *d_grad = dev.alloc<float>((size_t)W * pad);
  float *d_grad_dot = dev.alloc<float>(W), *d_decrement = dev.alloc<float>(W), *d_grad_scale = dev.alloc<float>(W);
  float *d_hessian = dev.alloc<float>((size_t)W * pad * pad), *d_factor = dev.alloc<float>((size_t)W * pad * pad);
  float *d_search = dev.alloc<float>((size_t)W * nv), *d_search_dot = dev.alloc<float>(W);
  float *d_mv = dev.alloc<float>((size_t)W * nv), *d_jv = dev.alloc<float>((size_t)W * R);
  float *d_quad = dev.alloc<float>((size_t)W * R * 3);
  float *d_alpha = dev.alloc<float>(W), *d_improvement = dev.alloc<float>(W);
  if (dev.rc != cudaSuccess) return (int)dev.rc;
  (void)done;

  InitInputs init{};
  init.worlds = W; init.nv = nv; init.pad = pad; init.rows = R; init.mass_entries = mass_entries; init.warmstart = 1;
  init.nefc = d_nefc; init.mass_row = d_mass_row; init.mass_col = d_mass_col; init.mass_address = d_mass_address;
  init.mass = d_mass; init.jacobian = d_J; init.aref = d_aref; init.warm_acceleration = d_warm;
  init.smooth_acceleration = d_smooth_acc; init.qacc = d_qacc; init.ma = d_ma; init.jaref = d_jaref;
  init.search_dot = d_search_dot; init.niter = d_niter; init.done = d_done;

  ConstraintInputs ci{};
  ci.worlds = W; ci.nv = nv; ci.pad = pad; ci.rows = R; ci.capacity = Cc; ci.impratio_count = 1;
  ci.done = d_done; ci.ne = d_ne; ci.nf = d_nf; ci.nefc = d_nefc; ci.contact_count = d_count;
  ci.contact_dimension = d_cdim; ci.contact_address = d_caddr; ci.impratio = d_scalars; ci.contact_friction = d_cfric;
  ci.row_type = d_type; ci.row_contact = d_rcon; ci.diagonal = d_D; ci.frictionloss = d_loss; ci.jaref = d_jaref;
  ci.jacobian = d_J; ci.force = d_force; ci.state = d_state; ci.qfrc_constraint = d_qfrc;

  DirectionInputs di{};
  di.worlds = W; di.nv = nv; di.pad = pad; di.ma_stride = nv; di.smooth_stride = nv; di.force_stride = nv;
  di.done = d_done; di.ma = d_ma; di.smooth = d_smooth; di.force = d_qfrc; di.hessian = d_hessian; di.grad = d_grad;
  di.grad_dot = d_grad_dot; di.decrement = d_decrement; di.grad_scale = d_grad_scale; di.search_unchanged = d_unchanged;
  di.factor = d_factor; di.search = d_search; di.search_dot = d_search_dot;

  HessianInputs hi{};
  hi.worlds = W; hi.nv = nv; hi.padded_nv = pad; hi.rows = R; hi.mass_entries = mass_entries; hi.contact_capacity = Cc;
  hi.impratio_count = 1; hi.cone_launch_groups = 1; hi.cone_contacts_per_group = Cc;  // one group: a fixed sum order
  hi.mass_upper_address = d_upper; hi.nefc = d_nefc; hi.mass = d_mass; hi.jacobian = d_J; hi.diagonal = d_D;
  hi.state = d_state; hi.jaref = d_jaref; hi.done = d_done; hi.impratio_invsqrt = d_scalars;
  hi.triangle_row = d_tri_row; hi.triangle_column = d_tri_col; hi.contact_count = d_count;
  hi.contact_world = d_cworld; hi.contact_dimension = d_cdim; hi.contact_friction = d_cfric;
  hi.contact_distance = d_cdist; hi.contact_margin = d_cmargin; hi.contact_address = d_caddr; hi.hessian = d_hessian;

  LinesearchInputs li{};
  li.worlds = W; li.nv = nv; li.pad = pad; li.rows = R; li.mass_entries = mass_entries; li.capacity = Cc;
  li.tolerance_count = li.ls_tolerance_count = li.impratio_count = li.inertia_count = 1;
  li.iterations = c->ls_iterations; li.warn_overflow = 0;
  li.done = d_done; li.ne = d_ne; li.nf = d_nf; li.nefc = d_nefc; li.contact_count = d_count;
  li.mass_row = d_mass_row; li.mass_col = d_mass_col; li.mass_address = d_mass_address; li.mass = d_mass;
  li.jacobian = d_J; li.search = d_search; li.search_dot = d_search_dot; li.smooth = d_smooth;
  li.tolerance = d_scalars + 1; li.ls_tolerance = d_scalars + 2; li.impratio = d_scalars; li.inertia = d_scalars + 3;
  li.row_type = d_type; li.row_contact = d_rcon; li.contact_dimension = d_cdim; li.contact_address = d_caddr;
  li.contact_friction = d_cfric; li.diagonal = d_D; li.frictionloss = d_loss; li.mv = d_mv; li.jv = d_jv;
  li.quad = d_quad; li.qacc = d_qacc; li.ma = d_ma; li.jaref = d_jaref; li.improvement = d_improvement;
  li.alpha = d_alpha; li.overflow = d_overflow;

  StopInputs si{};
  si.worlds = W; si.nv = nv; si.iterations = c->iterations; si.tolerance_count = si.inertia_count = 1;
  si.warn_overflow = 0; si.tolerance = d_scalars + 1; si.inertia = d_scalars + 3; si.grad_dot = d_grad_dot;
  si.decrement = d_decrement; si.improvement = d_improvement; si.alpha = d_alpha; si.niter = d_niter;
  si.overflow = d_overflow; si.nsolving = d_nsolving; si.done = d_done;

  const cudaStream_t s = 0;
  auto gradient = [&](bool stop) {
    dev.check(flash_mjwarp_constraint_gradient(&ci, &di, s));
    dev.check(flash_mjwarp_hessian_launch(&hi, 0, s));
    if (dev.rc == cudaSuccess) {
      harness_direction<<<(W + 63) / 64, 64, 0, s>>>(W, nv, pad, d_done, d_hessian, d_grad, d_factor, d_search,
                                                      d_search_dot, d_decrement);
      dev.check((int)cudaGetLastError());
    }
    if (stop) dev.check(flash_mjwarp_solver_state_stop(&si, s));
  };
  dev.check(flash_mjwarp_solver_state_fused(&init, d_grad, d_exhausted, d_nsolving, s));
  gradient(false);
  dev.check((int)cudaDeviceSynchronize());
  dev.download(o->qacc0, d_qacc, (size_t)W * nv);
  dev.download(o->Ma0, d_ma, (size_t)W * nv);
  dev.download(o->jaref0, d_jaref, (size_t)W * R);
  dev.download(o->state0, d_state, (size_t)W * R);
  dev.download(o->search0, d_search, (size_t)W * nv);
  if (o->grad0 && dev.rc == cudaSuccess) {
    std::vector<float> g((size_t)W * pad);
    dev.download(g.data(), d_grad, g.size());
    for (int w = 0; w < W; ++w) std::memcpy(o->grad0 + (size_t)w * nv, &g[(size_t)w * pad], sizeof(float) * nv);
  }
  if (o->H0 && dev.rc == cudaSuccess) {
    std::vector<float> h((size_t)W * pad * pad);
    dev.download(h.data(), d_hessian, h.size());
    for (int w = 0; w < W; ++w)
      for (int i = 0; i < nv; ++i)
        std::memcpy(o->H0 + ((size_t)w * nv + i) * nv, &h[((size_t)w * pad + i) * pad], sizeof(float) * nv);
  }
  for (int it = 0; it < c->iterations && dev.rc == cudaSuccess; ++it) {
    int solving = 0;
    dev.download(&solving, d_nsolving, 1);
    if (!solving) break;
    dev.check(flash_mjwarp_linesearch_fused(&li, s));
    if (it == 0) {
      dev.check((int)cudaDeviceSynchronize());
      dev.download(o->alpha0, d_alpha, (size_t)W);
      dev.download(o->improvement0, d_improvement, (size_t)W);
    }
    gradient(true);
    dev.check((int)cudaDeviceSynchronize());
  }
  dev.download(o->qacc, d_qacc, (size_t)W * nv);
  dev.download(o->qfrc_constraint, d_qfrc, (size_t)W * nv);
  dev.download(o->force, d_force, (size_t)W * R);
  dev.download(o->state, d_state, (size_t)W * R);
  dev.download(o->niter, d_niter, (size_t)W);
  dev.download(o->overflow, d_overflow, (size_t)W);
  return (int)dev.rc;
}
}
