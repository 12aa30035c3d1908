// Host entry points of the kernel instances (defined in inst.cu, one
// translation unit per precision and mesh support, compiled in parallel).
#pragma once
#include <cuda_runtime.h>
#include <cstddef>
#include "b200phys.h"

namespace b200 {
template <class R, bool C, int T> int configure_kernels(size_t smem);
template <class R, bool C, int T>
void launch_step(const B200Model &m, const B200Data &d, int substeps, int policy, int wpc, int arena, int grid,
                 size_t smem, cudaStream_t s);
template <class R, bool C, int T>
void launch_forward(const B200Model &m, const B200Data &d, int bootstrap, const int *mask, int wpc, int arena,
                    int grid, size_t smem, cudaStream_t s);

#define B200_INSTANCES(X, R, C) X(R, C, 32) X(R, C, 128)
#define B200_EXTERN(R, C, T)                                                                                  \
  extern template int configure_kernels<R, C, T>(size_t);                                                    \
  extern template void launch_step<R, C, T>(const B200Model &, const B200Data &, int, int, int, int, int,    \
                                            size_t, cudaStream_t);                                           \
  extern template void launch_forward<R, C, T>(const B200Model &, const B200Data &, int, const int *, int, int, \
                                               int, size_t, cudaStream_t);
B200_INSTANCES(B200_EXTERN, float, false)
B200_INSTANCES(B200_EXTERN, float, true)
B200_INSTANCES(B200_EXTERN, double, false)
B200_INSTANCES(B200_EXTERN, double, true)
#undef B200_EXTERN
}  // namespace b200
