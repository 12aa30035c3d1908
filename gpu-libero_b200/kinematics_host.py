"""Float64 host kinematics used while compiling a scene (MuJoCo mj_setConst role).

Only model compilation calls this (invweights and meaninertia at qpos0); the
physics step itself runs in the CUDA kernels.  The formulas are MuJoCo's
smooth-dynamics definitions: forward kinematics (mj_kinematics), subtree
centres of mass and motion axes (mj_comPos), composite rigid bodies (mj_crb).
"""
import numpy as np

from .scene import FREE, BALL, SLIDE, HINGE, quat_mul, quat_mat, axis_quat


def _rot(q, v):
    return quat_mat(q) @ v


def forward_position(scene, qpos):
    s, I, R = scene.sizes, scene.ints, scene.reals
    nb, nv = s['nbody'], s['nv']
    xpos = np.zeros((nb, 3))
    xquat = np.tile([1.0, 0, 0, 0], (nb, 1))
    anchors, axes = {}, {}
    for b in range(1, nb):
        p = I['body_parentid'][b]
        first, count = I['body_jntadr'][b], I['body_jntnum'][b]
        if count == 1 and I['jnt_type'][first] == FREE:
            a = I['jnt_qposadr'][first]
            pos = qpos[a:a + 3].copy()
            quat = qpos[a + 3:a + 7] / np.linalg.norm(qpos[a + 3:a + 7])
            anchors[first], axes[first] = pos.copy(), R['jnt_axis'][first].copy()
        else:
            pos = _rot(xquat[p], R['body_pos'][b]) + xpos[p]
            quat = quat_mul(xquat[p], R['body_quat'][b])
            for j in range(first, first + count):
                a = I['jnt_qposadr'][j]
                anchor = _rot(quat, R['jnt_pos'][j]) + pos
                axis = _rot(quat, R['jnt_axis'][j])
                kind = I['jnt_type'][j]
                if kind == BALL:
                    quat = quat_mul(quat, qpos[a:a + 4] / np.linalg.norm(qpos[a:a + 4]))
                    pos = anchor - _rot(quat, R['jnt_pos'][j])
                elif kind == SLIDE:
                    pos = pos + axis * (qpos[a] - R['qpos0'][a])
                elif kind == HINGE:
                    quat = quat_mul(quat, axis_quat(R['jnt_axis'][j], qpos[a] - R['qpos0'][a]))
                    pos = anchor - _rot(quat, R['jnt_pos'][j])
                anchors[j], axes[j] = anchor, axis
            quat = quat / np.linalg.norm(quat)
        xpos[b], xquat[b] = pos, quat
    xipos = np.array([xpos[b] + _rot(xquat[b], R['body_ipos'][b]) for b in range(nb)])
    ximat = np.array([quat_mat(quat_mul(xquat[b], R['body_iquat'][b])) for b in range(nb)])
    mass = R['body_mass']
    com = xipos * mass[:, None]
    for b in range(nb - 1, 0, -1):
        com[I['body_parentid'][b]] += com[b]
    st = R['body_subtreemass']
    com = np.where(st[:, None] > 0, com / np.where(st > 0, st, 1)[:, None], com)
    root = I['body_rootid']
    cdof = np.zeros((nv, 6))
    for j in range(s['njnt']):
        b, d, kind = I['jnt_bodyid'][j], I['jnt_dofadr'][j], I['jnt_type'][j]
        off = com[root[b]] - anchors[j]
        if kind == FREE:
            for k in range(3):
                cdof[d + k, 3 + k] = 1.0
            d += 3
        if kind in (FREE, BALL):
            r = quat_mat(xquat[b])
            for k in range(3):
                ax = r[:, k]
                cdof[d + k] = np.r_[ax, np.cross(ax, off)]
        elif kind == SLIDE:
            cdof[d, 3:] = axes[j]
        else:
            cdof[d] = np.r_[axes[j], np.cross(axes[j], off)]
    # composite rigid body inertia about each root's subtree com
    crb = np.zeros((nb, 6, 6))
    for b in range(1, nb):
        d = xipos[b] - com[root[b]]
        rot_inertia = ximat[b] @ np.diag(R['body_inertia'][b]) @ ximat[b].T
        rot_inertia += mass[b] * (np.dot(d, d) * np.eye(3) - np.outer(d, d))
        h = mass[b] * _skew(d)
        crb[b] = np.block([[rot_inertia, h], [h.T, mass[b] * np.eye(3)]])
    for b in range(nb - 1, 0, -1):
        p = I['body_parentid'][b]
        if p > 0:
            crb[p] += crb[b]
    M = np.zeros((nv, nv))
    for i in range(nv):
        f = crb[I['dof_bodyid'][i]] @ cdof[i]
        j = i
        while j >= 0:
            M[i, j] = M[j, i] = cdof[j] @ f
            j = I['dof_parentid'][j]
        M[i, i] += R['dof_armature'][i]
    site_xpos = np.array([xpos[I['site_bodyid'][k]] + _rot(xquat[I['site_bodyid'][k]], R['site_pos'][k])
                          for k in range(s['nsite'])])
    return dict(xpos=xpos, xquat=xquat, xipos=xipos, subtree_com=com, cdof=cdof, M_dense=M,
                site_xpos=site_xpos)


def _skew(v):
    # spatial inertia coupling block for the (angular, linear) ordering:
    # momentum_angular += m (d x v_linear)
    return np.array([[0, -v[2], v[1]], [v[2], 0, -v[0]], [-v[1], v[0], 0]])


def body_jacobian(scene, state, body, point):
    """Translational / rotational Jacobians of `point` fixed to `body`."""
    I = scene.ints
    nv = scene.sizes['nv']
    jp, jr = np.zeros((3, nv)), np.zeros((3, nv))
    mask = I['body_dofmask'][4 * body:4 * body + 4].view(np.uint32)
    com = state['subtree_com'][I['body_rootid'][body]]
    for d in range(nv):
        if mask[d // 32] >> (d % 32) & 1:
            ang, lin = state['cdof'][d, :3], state['cdof'][d, 3:]
            jr[:, d] = ang
            jp[:, d] = lin + np.cross(ang, point - com)
    return jp, jr
