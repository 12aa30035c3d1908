/*
 * b200phys — C ABI of the B200-native batched rigid-body physics step.
 *
 * This library replaces the per-leaf native libraries that the reference's
 * FP32 engine binds with ctypes (one `flash_mjwarp_<leaf>_fp32.so` per stage,
 * bound in libero/libero/gpu/host/backends/cuda_fp32/physics.py:106-159 and
 * libero/libero/gpu/host/runtime/{dynamics,collision,newton}/mjwarp_*.py).
 * Every reference leaf exports the same four-symbol convention, e.g.
 * libero/libero/gpu/cuda/collision/mjwarp_broadphase.cu:120-133:
 *     const char* flash_<leaf>_source_id();
 *     size_t      flash_<leaf>_arguments_bytes();   // checked against ctypes
 *     int         flash_<leaf>_arch();              // checked against device
 *     int         flash_<leaf>_launch(const Args*, ..., cudaStream_t);  // cudaError_t
 * b200phys keeps that convention but exports ONE fused launch per stage
 * group: the whole 25-substep control step (step1 -> OSC -> Newton -> Euler,
 * runtime.py:40-56) runs in one kernel launch with all per-world state
 * resident in shared memory.
 *
 * Conventions (same as the reference):
 *   - all device buffers are caller-owned; launches allocate nothing;
 *   - launch functions return a cudaError_t value (0 == success) and
 *     cudaErrorInvalidValue (1) for rejected arguments;
 *   - numerical/capacity conditions are reported per world in data.overflow
 *     (bit values of B200_OVERFLOW_*, the reference's OverflowType,
 *     cuda_fp32/constants.py:70-101) and controller failures in data.error
 *     (2 = singular arm mass matrix, 4 = pseudoinverse did not converge,
 *     osc_solver.cu MassInverse / Pseudoinverse scopes); nothing traps.
 */
#ifndef B200PHYS_H
#define B200PHYS_H

#include <stddef.h>
#include "b200phys_fields.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Overflow bits (reference OverflowType, cuda_fp32/constants.py:89-101). */
#define B200_OVERFLOW_NEFC (1 << 0)
#define B200_OVERFLOW_NARROWPHASE (1 << 3)
#define B200_OVERFLOW_EPA_HORIZON (1 << 8) /* EPA horizon edge list full (fatal) */
#define B200_OVERFLOW_ITERATIONS (1 << 9)
#define B200_OVERFLOW_LS_ITERATIONS (1 << 10)
/* Non-finite or huge state (|x| > 1e10, MuJoCo's mjMAXVAL in mj_checkPos /
 * mj_checkVel): set after the substep that produced it; the world is not
 * stepped further in that launch (fatal; no reference bit has this value). */
#define B200_STATUS_BADSTATE (1 << 16)
/* EPA's vertex or face pool filled before it converged: EPA ends with the best
 * face found, as at its iteration limit (a legal exit, not fatal; the
 * reference's full face pool also ends its EPA without a status,
 * mjwarp_convex_epa.cuh:89,219). */
#define B200_WARN_EPA_BUDGET (1 << 17)

/* disable_flags bits (MuJoCo 3.x mjtDisableBit positions). */
#define B200_DSBL_CONSTRAINT (1 << 0)
#define B200_DSBL_FRICTIONLOSS (1 << 2)
#define B200_DSBL_LIMIT (1 << 3)
#define B200_DSBL_CONTACT (1 << 4)
#define B200_DSBL_SPRING (1 << 5)
#define B200_DSBL_DAMPER (1 << 6)
#define B200_DSBL_GRAVITY (1 << 7)
#define B200_DSBL_CLAMPCTRL (1 << 8)
#define B200_DSBL_WARMSTART (1 << 9)
#define B200_DSBL_REFSAFE (1 << 12)
#define B200_DSBL_EULERDAMP (1 << 15)

/* Geom types (MuJoCo mjtGeom). */
#define B200_GEOM_PLANE 0
#define B200_GEOM_SPHERE 2
#define B200_GEOM_CAPSULE 3
#define B200_GEOM_BOX 6
#define B200_GEOM_MESH 7

/* Joint types (MuJoCo mjtJoint). */
#define B200_JNT_FREE 0
#define B200_JNT_BALL 1
#define B200_JNT_SLIDE 2
#define B200_JNT_HINGE 3

/* Model descriptor: sizes, options and offsets into two packed buffers.
 * `real` holds every real array in the precision given by real_bytes
 * (4 = float, 8 = double); `ints` holds every int32 array. */
typedef struct B200Model {
  const void *real;
  const int *ints;
#define B200_X(n) int n;
  B200_MODEL_INT_SCALARS(B200_X)
#undef B200_X
#define B200_X(n) double n;
  B200_MODEL_REAL_SCALARS(B200_X)
#undef B200_X
#define B200_X(n, len) int off_##n;
  B200_MODEL_INT_ARRAYS(B200_X)
  B200_MODEL_REAL_ARRAYS(B200_X)
#undef B200_X
} B200Model;

/* World-major batch data: each pointer addresses [nworld, width] elements.
 * Output pointers may be NULL, in which case that output is not written. */
typedef struct B200Data {
  int nworld;
  int world_offset; /* global index of world 0 of this shard (diagnostics) */
#define B200_X(n, w) void *n;
  B200_DATA_REAL(B200_X)
#undef B200_X
#define B200_X(n, w) int *n;
  B200_DATA_INT(B200_X)
#undef B200_X
} B200Data;

/* ---- ABI identification (reference convention, e.g. mjwarp_broadphase.cu:120-133) ---- */
const char *b200phys_source_id(void);
int b200phys_arch(void);
size_t b200phys_model_bytes(void); /* sizeof(B200Model), checked by the host */
size_t b200phys_data_bytes(void);  /* sizeof(B200Data), checked by the host */

/* Dynamic shared memory one world needs for this model, in bytes
 * (0 if the model is rejected or one world's arena exceeds the 227 KB a
 * CTA can opt into on sm_100). */
size_t b200phys_world_smem_bytes(const B200Model *m);

/* Configure the kernels for this model (dynamic shared memory opt-in).
 * Call once per model and device before any stream capture; launches also
 * configure on demand.  Returns a cudaError_t value. */
int b200phys_prepare(const B200Model *m);

/* Advance every world by `substeps` physics substeps.
 *
 * Replaces the reference's captured 25-substep control graph
 * (cuda_fp32/runtime.py:40-56, Runtime.enqueue_substep + prepare_control_graph),
 * i.e. per substep: Physics.step1 (physics.py:161-186), FusedControlDrive
 * (fp32/fused_control_drive.cu:35-360, OSC osc_solver.cu:309-676), Newton.solve
 * (physics.py:47-70) and FusedEulerStep (fp32/fused_euler_step.cu).
 * `policy` != 0 makes the first substep a policy step: the OSC goal is moved
 * by data.action (robosuite set_goal), as runtime.py:42 passes policy_values[k==0].
 * Graph-capturable; allocates nothing. Returns a cudaError_t value. */
int b200phys_step_launch(const B200Model *m, const B200Data *d, int substeps,
                         int policy, void *stream);

/* Recompute position/velocity-dependent quantities and the Newton solve
 * without integrating (reference Runtime.forward -> Physics.forward,
 * physics.py:210: step1(factorize=False) + solve(public=True)).
 * `bootstrap` != 0 also resets the OSC goal to the current end-effector pose
 * and clears the gripper state (controller.py:124-129 Controller.bootstrap).
 * `mask` (device int32[nworld], may be NULL for all) selects the worlds. */
int b200phys_forward_launch(const B200Model *m, const B200Data *d,
                            int bootstrap, const int *mask, void *stream);

/* Regroup the worlds for the next control step: fill d->order with the worlds
 * sorted by d->work (their solver work in the last control step, written by
 * b200phys_step_launch), so that the worlds sharing a CTA, which advance
 * through the stages in lockstep, have similar work and wait less for each
 * other.  World results do not depend on the grouping.  One small kernel;
 * graph-capturable; allocates nothing.  This is the reference's world-to-CTA
 * mapping made adaptive (the reference launches one CTA per world,
 * cuda_fp32/fused_*.cu); it has no counterpart call in the reference.
 * Returns a cudaError_t value (cudaErrorInvalidValue without work or order). */
int b200phys_order_launch(const B200Model *m, const B200Data *d, void *stream);

#ifdef __cplusplus
}
#endif
#endif
