// Kernel instances of one precision (B200_INST_REAL) and convex mode
// (B200_INST_CONVEX: 0, 1 or 2, see launch.h), for one and four warps per world.
#include "kernels.cuh"

namespace b200 {
#define B200_DEFINE(R, C, T)                                                                                  \
  template int configure_kernels<R, C, T>(size_t);                                                           \
  template void launch_step<R, C, T>(const B200Model &, const B200Data &, int, int, int, int, int, size_t,   \
                                     cudaStream_t);                                                          \
  template void launch_forward<R, C, T>(const B200Model &, const B200Data &, int, const int *, int, int, int, \
                                        size_t, cudaStream_t);
B200_DEFINE(B200_INST_REAL, B200_INST_CONVEX, 32)
B200_DEFINE(B200_INST_REAL, B200_INST_CONVEX, 128)
}  // namespace b200
