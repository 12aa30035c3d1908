/*
 * Field lists of the B200 physics C ABI (X-macros).
 *
 * One list drives three consumers that must agree byte for byte:
 *   - include/b200phys.h builds the B200Model / B200Data structs from it;
 *   - the CUDA kernels and the C oracle read model arrays through it;
 *   - the Python host parses this file to build matching ctypes structs and to
 *     pack the model arrays (gpu-libero_b200/native.py).
 *
 * Model arrays are packed into two flat buffers (one of reals, one of int32);
 * each named array is addressed by its offset into its buffer.  Names follow
 * MuJoCo's mjModel/mjData fields that the reference reads through
 * libero/libero/gpu/host/backends/cuda_fp32/layout_specs.py:37 (MODEL) and
 * :504 (DATA); entries without a MuJoCo counterpart are derived topology
 * (body levels, tree blocks, ancestor masks) or the robosuite OSC_POSE
 * configuration (libero/libero/gpu/host/backends/cuda_fp32/controller.py:46-87).
 *
 * Data fields carry a per-world width expression written in model size names;
 * the host evaluates it to allocate world-major [nworld, width] buffers.
 * Every output pointer may be NULL (not written).  Inspection outputs that a
 * step never needs (the dense constraint rows efc_J / efc_D / efc_aref /
 * efc_type / efc_id of the last substep, its dense mass matrix qM and smooth
 * force qfrc_smooth, the contacts' friction / margin / dimension, and the
 * per-substep Newton and line-search counts niter_trace / ls_trace of the
 * last control step, first 32 substeps) are allocated by the host only when
 * it asks for them.
 *
 * work / order: `work` is each world's solver work in its last control step
 * (sum over substeps of (Newton iterations + 1) x (rows + 32) + 4 contacts
 * + 1500 x GJK / EPA pairs past the broadphase);
 * `order`, when given, is the permutation that assigns worlds to the step
 * kernel's CTA slots (slot i runs world order[i]).  b200phys_order_launch
 * refills it from `work`, so that worlds of similar work share a CTA.
 *
 * boxbox_convex: box-box pairs take the convex path (GJK / EPA and the box
 * manifold) instead of the SAT box collider; set when no box-box pair has a
 * margin (the reference's has_boxbox_margin rule, cuda_fp32/model.py:187-191,
 * physics.py:89-90).  Such a model runs the kernel variant with convex support.
 *
 * nvariant / variant_stride: per-world model parameter rows.  The real
 * buffer holds max(nvariant, 1) copies of every real array, variant_stride
 * reals apart (offsets off_* are within one copy); world w of a shard reads
 * copy (world_offset + w) % nvariant, the reference's broadcast rule
 * parameter(p, w) = p.data + (w % p.rows) * width
 * (cuda/dynamics/mjwarp_constraint_build.cu:18-20).  The int arrays (the
 * topology) and the real scalars (timestep, gravity, impratio, tolerances,
 * meaninertia) are one per model.  nvariant 0 or 1 is one shared model.
 *
 * task_body / task_lift_z: the synthetic scenes' task predicate.  Success is
 * the free body free_bodyid[task_body] (its centre of mass frame origin) above
 * task_lift_z; reward = 1 and done = 1 on success, else 0 (LIBERO's sparse
 * reward, batch_env.py:463-475).  task_body < 0 disables the predicate.
 */
#ifndef B200PHYS_FIELDS_H
#define B200PHYS_FIELDS_H

/* integer scalars of the model */
#define B200_MODEL_INT_SCALARS(X) \
  X(nq) X(nv) X(nu) X(nbody) X(njnt) X(ngeom) X(nsite) X(npair) X(ntree) \
  X(nM) X(nlevel) X(nlimited) X(nfric) X(ncon_max) X(nefc_max) X(cone) \
  X(iterations) X(ls_iterations) X(disable_flags) X(ee_site) X(real_bytes) \
  X(nvs) X(kmax_dof) X(max_tree_dofs) X(osc_uncouple) X(nfree) X(nobs) \
  X(nmesh) X(nmeshvert) X(nmeshpoly) X(nmeshpolyvert) X(nmeshpolymap) \
  X(ccd_iterations) X(epa_iterations) X(nL) X(task_body) X(boxbox_convex) \
  X(nvariant) X(variant_stride)

/* real scalars of the model (stored as double, read as the kernel's real) */
#define B200_MODEL_REAL_SCALARS(X) \
  X(timestep) X(gravity_x) X(gravity_y) X(gravity_z) X(tolerance) \
  X(ls_tolerance) X(impratio_invsqrt) X(meaninertia) X(ccd_tolerance) X(task_lift_z)

/* int32 arrays: X(name, length-expression) */
#define B200_MODEL_INT_ARRAYS(X) \
  X(body_parentid, nbody) X(body_rootid, nbody) X(body_weldid, nbody) \
  X(body_jntnum, nbody) X(body_jntadr, nbody) X(body_dofnum, nbody) \
  X(body_dofadr, nbody) X(body_treeid, nbody) X(body_subtree_end, nbody) \
  X(body_order, nbody) X(level_start, nlevel + 1) X(body_dofmask, nbody * 4) \
  X(jnt_type, njnt) X(jnt_qposadr, njnt) X(jnt_dofadr, njnt) \
  X(jnt_bodyid, njnt) X(jnt_limited, njnt) \
  X(dof_bodyid, nv) X(dof_jntid, nv) X(dof_parentid, nv) X(dof_treeid, nv) \
  X(tree_dofadr, ntree) X(tree_dofnum, ntree) X(tree_madr, ntree) X(tree_padr, ntree) X(tree_lsrc, nL) \
  X(geom_type, ngeom) X(geom_bodyid, ngeom) X(geom_condim, ngeom) \
  X(geom_priority, ngeom) X(site_bodyid, nsite) X(pair_geom, npair * 2) \
  X(limited_jnt, nlimited) X(fric_dof, nfric) \
  X(actuator_trnid, nu) X(actuator_gaintype, nu) X(actuator_biastype, nu) \
  X(actuator_ctrllimited, nu) X(actuator_forcelimited, nu) \
  X(osc_qposadr, 7) X(osc_dofadr, 7) X(osc_actuator, 9) X(free_bodyid, nfree) \
  X(geom_dataid, ngeom) X(mesh_vertadr, nmesh) X(mesh_vertnum, nmesh) \
  X(mesh_polyadr, nmesh) X(mesh_polynum, nmesh) X(mesh_polyvertadr, nmeshpoly) \
  X(mesh_polyvertnum, nmeshpoly) X(mesh_polyvert, nmeshpolyvert) \
  X(mesh_polymapadr, nmeshvert) X(mesh_polymapnum, nmeshvert) X(mesh_polymap, nmeshpolymap)

/* real arrays: X(name, length-expression) */
#define B200_MODEL_REAL_ARRAYS(X) \
  X(body_pos, nbody * 3) X(body_quat, nbody * 4) X(body_ipos, nbody * 3) \
  X(body_iquat, nbody * 4) X(body_mass, nbody) X(body_subtreemass, nbody) \
  X(body_inertia, nbody * 3) X(body_invweight0, nbody * 2) \
  X(jnt_pos, njnt * 3) X(jnt_axis, njnt * 3) X(jnt_range, njnt * 2) \
  X(jnt_margin, njnt) X(jnt_solref, njnt * 2) X(jnt_solimp, njnt * 5) \
  X(jnt_stiffness, njnt) X(qpos0, nq) X(qpos_spring, nq) \
  X(dof_armature, nv) X(dof_damping, nv) X(dof_frictionloss, nv) \
  X(dof_invweight0, nv) X(dof_solref, nv * 2) X(dof_solimp, nv * 5) \
  X(geom_size, ngeom * 3) X(geom_pos, ngeom * 3) X(geom_quat, ngeom * 4) \
  X(geom_aabb, ngeom * 6) X(geom_rbound, ngeom) X(geom_friction, ngeom * 3) \
  X(geom_solmix, ngeom) X(geom_solref, ngeom * 2) X(geom_solimp, ngeom * 5) \
  X(geom_margin, ngeom) X(geom_gap, ngeom) \
  X(site_pos, nsite * 3) X(site_quat, nsite * 4) \
  X(actuator_gear, nu) X(actuator_gainprm, nu * 3) X(actuator_biasprm, nu * 3) \
  X(actuator_ctrlrange, nu * 2) X(actuator_forcerange, nu * 2) \
  X(osc_gains, 12) X(osc_q0, 7) X(osc_action_config, 25) X(osc_null, 2) \
  X(mesh_vert, nmeshvert * 3) X(mesh_polynormal, nmeshpoly * 3)

/* world-major real data: X(name, per-world width) */
#define B200_DATA_REAL(X) \
  X(qpos, nq) X(qvel, nv) X(qacc, nv) X(qacc_warmstart, nv) X(ctrl, nu) \
  X(time, 1) X(action, 7) X(goal_pos, 3) X(goal_rot, 9) X(gripper, 2) \
  X(xpos, nbody * 3) X(xquat, nbody * 4) X(xmat, nbody * 9) \
  X(geom_xpos, ngeom * 3) X(geom_xmat, ngeom * 9) X(site_xpos, nsite * 3) \
  X(site_xmat, nsite * 9) X(subtree_com, nbody * 3) X(qfrc_bias, nv) \
  X(qfrc_actuator, nv) X(qfrc_constraint, nv) X(qacc_smooth, nv) \
  X(con_dist, ncon_max) X(con_pos, ncon_max * 3) X(con_frame, ncon_max * 9) \
  X(efc_force, nefc_max) X(obs, nobs) \
  X(efc_J, nefc_max * nv) X(efc_D, nefc_max) X(efc_aref, nefc_max) \
  X(qM, nv * nv) X(qfrc_smooth, nv) X(con_friction, ncon_max * 5) X(con_margin, ncon_max)

/* world-major int32 data: X(name, per-world width) */
#define B200_DATA_INT(X) \
  X(ncon, 1) X(nefc, 1) X(con_geom, ncon_max * 2) X(overflow, 1) \
  X(error, 1) X(niter, 1) X(newton_total, 1) X(ls_total, 1) \
  X(integration_count, 1) X(efc_total, 1) X(con_total, 1) \
  X(newton_rows, 1) X(ls_rows, 1) X(efc_k, 1) X(efc_k2, 1) X(fact_blk, 1) \
  X(stage_cycles, 16) X(efc_type, nefc_max) X(efc_id, nefc_max) X(niter_trace, 32) X(ls_trace, 32) \
  X(work, 1) X(order, 1) X(con_dim, ncon_max)

#endif
