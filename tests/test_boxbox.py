"""Zero-margin box pairs: the convex path and its box manifold, on the CPU oracle.

When no box-box pair has a margin, the reference routes box-box pairs through
its convex leaf (cuda_fp32/model.py:187-191 has_boxbox_margin,
physics.py:89-90) and turns EPA's contact into a face manifold
(mjwarp_box_manifold.cuh box_multicontact, called at
mjwarp_convex_collision.cuh:63-77).  scene_a(box_margin=0) is such a model.
The GPU kernel is compared with the oracle and with the reference's compiled
convex leaf in tests/test_gpu_boxbox.py; here the oracle's manifold is checked
on configurations whose contacts are known in closed form.
"""
import math

import numpy as np
import pytest

from gpu_libero_b200 import native, scene as scenes


def geom_of(scene, body):
    return int(np.flatnonzero(np.asarray(scene.ints['geom_bodyid']) == scene.body_names.index(body))[0])


def qpos_of(scene, body):
    fb = list(scene.ints['free_bodyid'])
    b = scene.body_names.index(body)
    assert b in fb
    return int(scene.ints['jnt_qposadr'][np.flatnonzero(scene.ints['jnt_bodyid'] == b)[0]])


def quat_axis(axis, angle):
    axis = np.asarray(axis, float) / np.linalg.norm(axis)
    return np.r_[math.cos(angle / 2), math.sin(angle / 2) * axis]


def qmul(a, b):
    w1, x1, y1, z1 = a
    w2, x2, y2, z2 = b
    return np.array([w1 * w2 - x1 * x2 - y1 * y2 - z1 * z2, w1 * x2 + x1 * w2 + y1 * z2 - z1 * y2,
                     w1 * y2 - x1 * z2 + y1 * w2 + z1 * x2, w1 * z2 + x1 * y2 - y1 * x2 + z1 * w2])


def stacked_state(scene, n, seed):
    """box0 on the floor; box1 resting on box0 with 0.2-2 mm of penetration,
    turned about z at random (an angle away from the boxes' symmetries, so
    that one pair of faces is anti-parallel); box2 on box1 tilted by 2-20
    degrees about a horizontal axis (its lowest edge or corner in contact).
    World 0 keeps box2 level and aligned with box1 (face on face, equal
    orientation)."""
    q, v = scene.initial_state(n, seed=seed)
    v[:] = 0
    rng = np.random.default_rng(seed)
    size = np.reshape(scene.reals['geom_size'], (-1, 3))
    h0, h1, h2 = (size[geom_of(scene, 'box%d' % k)] for k in range(3))
    a0, a1, a2 = (qpos_of(scene, 'box%d' % k) for k in range(3))
    for w in range(n):
        base = np.array([0.62, 0.25, 0.0]) + rng.uniform(-0.02, 0.02, 3) * [1, 1, 0]
        # box0 0.5 mm into the floor (a contact distance of exactly zero would
        # sit on the publish threshold, where rounding decides)
        q[w, a0:a0 + 7] = np.r_[base + [0, 0, h0[2] - 0.0005], quat_axis([0, 0, 1], rng.uniform(0, math.pi))]
        turn = rng.uniform(0.15, 1.4) * rng.choice([-1, 1])
        top1 = q[w, a0 + 2] + h0[2] + h1[2] - rng.uniform(0.0002, 0.002)
        q1 = qmul(q[w, a0 + 3:a0 + 7], quat_axis([0, 0, 1], turn))
        q[w, a1:a1 + 7] = np.r_[base + [*rng.uniform(-0.008, 0.008, 2), top1], q1]
        tilt = 0.0 if w == 0 else rng.uniform(0.035, 0.35)
        axis = np.r_[rng.normal(size=2), 0.0]
        q2 = qmul(q1, quat_axis(axis, tilt)) if tilt else q1.copy()
        # lowest point of box2 after the tilt, 0.2-2 mm below box1's top face
        R2 = quat_mat(q2)
        corners = np.array([[sx, sy, sz] for sx in (-1, 1) for sy in (-1, 1) for sz in (-1, 1)]) * h2
        low = np.min(corners @ R2.T[:, 2])
        top2 = q[w, a1 + 2] + h1[2] - low - rng.uniform(0.0002, 0.002)
        q[w, a2:a2 + 7] = np.r_[q[w, a1:a1 + 2] + rng.uniform(-0.005, 0.005, 2), top2, q2]
    return q, v


def quat_mat(qu):
    w, x, y, z = qu / np.linalg.norm(qu)
    return np.array([[1 - 2 * (y * y + z * z), 2 * (x * y - z * w), 2 * (x * z + y * w)],
                     [2 * (x * y + z * w), 1 - 2 * (x * x + z * z), 2 * (y * z - x * w)],
                     [2 * (x * z - y * w), 2 * (y * z + x * w), 1 - 2 * (x * x + y * y)]])


def oracle_contacts(oracle_module, scene, q, v, precision='fp64'):
    n = q.shape[0]
    packed = native.PackedModel(scene, precision)
    host = native.alloc_numpy(packed, n)
    host['qpos'][:] = q
    host['qvel'][:] = v
    oracle_module.Oracle(precision).forward(packed.host_struct(), native.data_struct(host, n), 0, n, 1)
    return host


def pair_contacts(host, w, g1, g2):
    nc = int(host['ncon'][w, 0])
    g = host['con_geom'][w, :2 * nc].reshape(-1, 2)
    idx = [i for i in range(nc) if {int(g[i, 0]), int(g[i, 1])} == {g1, g2}]
    return (host['con_dist'][w, idx], host['con_pos'][w].reshape(-1, 3)[idx],
            host['con_frame'][w].reshape(-1, 9)[idx, :3])


def test_zero_margin_boxes_take_the_convex_path():
    a = scenes.scene_a(box_margin=0.0)
    assert a.sizes['boxbox_convex'] == 1 and a.sizes['epa_iterations'] == 16  # all convex pairs are box-box
    assert scenes.scene_a().sizes['boxbox_convex'] == 0  # any box margin: the SAT box collider
    b = scenes.scene_b(box_margin=0.0)
    assert b.sizes['boxbox_convex'] == 1 and b.sizes['epa_iterations'] == 32  # as given


@pytest.mark.parametrize('precision', ['fp64', 'fp32'])
def test_stacked_boxes_give_face_manifolds(oracle_module, precision):
    scene = scenes.scene_a(box_margin=0.0)
    n = 12
    q, v = stacked_state(scene, n, seed=4)
    host = oracle_contacts(oracle_module, scene, q, v, precision)
    g0, g1, g2 = (geom_of(scene, 'box%d' % k) for k in range(3))
    a0, a1 = qpos_of(scene, 'box0'), qpos_of(scene, 'box1')
    size = np.reshape(scene.reals['geom_size'], (-1, 3))
    tol = 1e-9 if precision == 'fp64' else 2e-5
    counts = []
    for w in range(n):
        # box1 on box0: face on face, turned, so a 3-8 sided overlap reduced to 4 points
        d, p, nrm = pair_contacts(host, w, g0, g1)
        depth = q[w, a0 + 2] + size[g0, 2] + size[g1, 2] - q[w, a1 + 2]
        assert len(d) == 4, (w, d)
        assert np.allclose(d, -depth, atol=tol), (w, d, depth)
        up = quat_mat(q[w, a0 + 3:a0 + 7])[:, 2]
        assert np.allclose(np.abs(nrm @ up), 1, atol=tol), (w, nrm)
        assert np.allclose(p @ up, (q[w, a0:a0 + 3] @ up) + size[g0, 2] - depth / 2, atol=tol)
        # box2 on box1: level and aligned in world 0 (four corners), else a
        # tilted edge (two) or corner (one), or none when the lowest corner
        # hangs beyond box1's top face
        d2, _, _ = pair_contacts(host, w, g1, g2)
        assert len(d2) <= 4 and np.all(d2 < 0), (w, d2)
        counts.append(len(d2))
    assert counts[0] == 4 and 1 in counts[1:] and 2 in counts[1:], counts
