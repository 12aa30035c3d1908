// Host entry points of the kernel instances (defined in inst.cu, one
// translation unit per precision and convex mode, compiled in parallel).
// Convex mode C: 0 no GJK / EPA (models without meshes); 1 GJK / EPA for
// mesh pairs; 2 also the zero-margin box-box path and its box manifold
// (models with boxbox_convex).  Mode 2 is a kernel of its own because its
// extra collider changes the code generated for the whole kernel: it costs
// mode 1 models about 3% when present.
#pragma once
#include <cuda_runtime.h>
#include <cstddef>
#include "b200phys.h"

namespace b200 {
template <class R, int C, int T> int configure_kernels(size_t smem);
template <class R, int C, int T>
void launch_step(const B200Model &m, const B200Data &d, int substeps, int policy, int wpc, int arena, int grid,
                 size_t smem, cudaStream_t s);
template <class R, int C, int T>
void launch_forward(const B200Model &m, const B200Data &d, int bootstrap, const int *mask, int wpc, int arena,
                    int grid, size_t smem, cudaStream_t s);

#define B200_INSTANCES(X, R, C) X(R, C, 32) X(R, C, 128)
#define B200_EXTERN(R, C, T)                                                                                  \
  extern template int configure_kernels<R, C, T>(size_t);                                                    \
  extern template void launch_step<R, C, T>(const B200Model &, const B200Data &, int, int, int, int, int,    \
                                            size_t, cudaStream_t);                                           \
  extern template void launch_forward<R, C, T>(const B200Model &, const B200Data &, int, const int *, int, int, \
                                               int, size_t, cudaStream_t);
B200_INSTANCES(B200_EXTERN, float, 0)
B200_INSTANCES(B200_EXTERN, float, 1)
B200_INSTANCES(B200_EXTERN, float, 2)
B200_INSTANCES(B200_EXTERN, double, 0)
B200_INSTANCES(B200_EXTERN, double, 1)
B200_INSTANCES(B200_EXTERN, double, 2)
#undef B200_EXTERN
}  // namespace b200
