"""Zero-margin box pairs on the GPU: the convex path and its box manifold,
against the CPU oracle and against the reference's own compiled convex leaf.

scene_a(box_margin=0) has no box margin anywhere, so box-box pairs (box on box,
finger pads on boxes) take the convex path: GJK, EPA that ends on a face of
the Minkowski difference, and the face manifold of up to four contacts
(mjwarp_box_manifold.cuh box_multicontact).  The reference's harness
(oracle/ref_contacts.cu) routes box-box pairs to its convex leaf by the same
has_boxbox_margin rule (cuda_fp32/physics.py:89-90).

States: tests/test_boxbox.py stacked_state (box1 face down on box0, turned
about the vertical; box2 on box1, tilted onto an edge or a corner; world 0
with box2 level and aligned), and a rollout of the zero-margin scene.

Checked:
- B200 kernel against the oracle, FP64 and FP32: contact lists equal (counts,
  pairs, order), distances and points within 1e-10 (FP64) / 1e-4 (FP32);
  five control steps of the zero-margin scene track the oracle;
- B200 kernel (FP32) against the reference's compiled convex leaf on the same
  poses: per pair, the same number of contacts, contact points within 2e-4 m
  and distances within 2e-4 m (the CCD tolerance band: EPA's final face and
  the clipped points are computed by two different EPA implementations),
  normals within 1e-3.  Exactly aligned boxes (world 0's level box2, box
  pairs with several anti-parallel face pairs) are compared the same way but
  reported apart: there the feature recovery depends on EPA's final triangle.
"""
import numpy as np
import pytest

torch = pytest.importorskip('torch')
pytestmark = pytest.mark.gpu

from gpu_libero_b200 import native, scene as scenes  # noqa: E402
from gpu_libero_b200.runtime import Runtime  # noqa: E402

from test_boxbox import geom_of, stacked_state  # noqa: E402


def gpu_forward(scene, q, v, precision):
    n = q.shape[0]
    rt = Runtime(scene, n, precision=precision)
    rt.set_state(np.concatenate([np.zeros((n, 1)), q, v], axis=1))
    rt.forward()
    torch.cuda.synchronize()
    out = {k: t.cpu().numpy() for k, t in rt.buffers.items()}
    rt.close()
    return out


@pytest.mark.parametrize('precision,tol', [('fp64', 1e-10), ('fp32', 1e-4)])
def test_box_manifold_matches_oracle(oracle_module, precision, tol):
    scene = scenes.scene_a(box_margin=0.0)
    n = 32
    q, v = stacked_state(scene, n, seed=9)
    gpu = gpu_forward(scene, q, v, precision)
    ref = native.alloc_numpy(native.PackedModel(scene, precision), n)
    ref['qpos'][:] = q
    ref['qvel'][:] = v
    oracle_module.Oracle(precision).forward(native.PackedModel(scene, precision).host_struct(),
                                            native.data_struct(ref, n), 0, n, 1)
    assert np.array_equal(gpu['ncon'], ref['ncon'])
    multi = 0
    for w in range(n):
        c = int(ref['ncon'][w, 0])
        assert np.array_equal(gpu['con_geom'][w, :2 * c], ref['con_geom'][w, :2 * c]), w
        for k, width in (('con_dist', 1), ('con_pos', 3), ('con_frame', 9)):
            err = np.max(np.abs(gpu[k][w, :width * c] - ref[k][w, :width * c]), initial=0.0)
            assert err <= tol * (10 if k == 'con_frame' else 1), (w, k, err)
        g = ref['con_geom'][w, :2 * c].reshape(-1, 2)
        multi += sum(1 for i in range(1, c) if tuple(g[i]) == tuple(g[i - 1]))
    assert multi >= 3 * n  # manifolds of several contacts
    assert not np.any(gpu['overflow'] & ~0x600)


@pytest.mark.parametrize('precision,tol', [('fp32', 1e-4), ('fp64', 1e-9)])
def test_zero_margin_control_steps_track_the_oracle(oracle_module, precision, tol):
    scene = scenes.scene_a(box_margin=0.0)
    n = 8
    rt = Runtime(scene, n, precision=precision)
    q, v = scene.initial_state(n, seed=5)
    rt.set_state(np.concatenate([np.zeros((n, 1)), q, v], axis=1))
    torch.cuda.synchronize()
    ref = native.alloc_numpy(rt.packed, n)
    for k, t in rt.buffers.items():
        ref[k][:] = t.cpu().numpy()
    orc = oracle_module.Oracle(precision)
    for step in range(5):
        a = scene.actions(n, step, seed=5)
        rt.enqueue_action(a)
        ref['action'][:] = a
        orc.step(rt.packed.host_struct(), native.data_struct(ref, n), 0, n, rt.substeps, 1)
    torch.cuda.synchronize()
    gpu = {k: t.cpu().numpy() for k, t in rt.buffers.items()}
    rt.close()
    assert np.max(np.abs(gpu['qpos'] - ref['qpos'])) < tol
    assert np.array_equal(gpu['ncon'], ref['ncon'])
    assert not np.any(gpu['overflow'] & ~0x600) and not np.any(gpu['error'])


@pytest.fixture(scope='module')
def ref_leaves():
    import sys
    from pathlib import Path
    sys.path.insert(0, str(Path(__file__).resolve().parents[1] / 'oracle'))
    import ref_contacts
    if not ref_contacts.available():
        pytest.skip('oracle/_ref/libref_contacts.so not built (needs the reference checkout at build time)')
    return ref_contacts.RefCollision()


def box_pairs(types, geom, world, dist, pos, normal):
    out = {}
    for i in range(len(world)):
        a, b = int(geom[i, 0]), int(geom[i, 1])
        if types[a] == 6 and types[b] == 6:
            out.setdefault((int(world[i]), a, b), []).append((float(dist[i]), pos[i].astype(float),
                                                              normal[i].astype(float)))
    return out


@pytest.mark.parametrize('seed', [9, 10])
def test_box_manifold_matches_reference_convex_leaf(ref_leaves, seed):
    from scipy.optimize import linear_sum_assignment
    scene = scenes.scene_a(box_margin=0.0)
    n = 48
    q, v = stacked_state(scene, n, seed=seed)
    out = gpu_forward(scene, q, v, 'fp32')
    types = np.asarray(scene.ints['geom_type'])
    r = ref_leaves.collide(scene, out['geom_xpos'], out['geom_xmat'])
    assert r['count'] <= r['capacity'] and not np.any(r['overflow'] & ~0x600)
    ours_w, ours_g, ours_d, ours_p, ours_n = [], [], [], [], []
    for w in range(n):
        c = int(out['ncon'][w, 0])
        ours_w += [w] * c
        ours_g.append(out['con_geom'][w, :2 * c].reshape(c, 2))
        ours_d.append(out['con_dist'][w, :c])
        ours_p.append(out['con_pos'][w, :3 * c].reshape(c, 3))
        ours_n.append(out['con_frame'][w, :9 * c].reshape(c, 9)[:, :3])
    mine = box_pairs(types, np.concatenate(ours_g), np.array(ours_w), np.concatenate(ours_d),
                     np.concatenate(ours_p), np.concatenate(ours_n))
    theirs = box_pairs(types, r['geom'], r['world'], r['dist'], r['pos'], r['frame'][:, :3])
    aligned = {(0, geom_of(scene, 'box1'), geom_of(scene, 'box2'))}
    stats = dict(pairs=0, contacts=0, dd=0.0, dp=0.0, dn=0.0)
    count_diff, aligned_report = [], []
    for key in sorted(set(mine) | set(theirs)):
        a, b = mine.get(key, []), theirs.get(key, [])
        if len(a) != len(b):
            count_diff.append((key, len(a), len(b)))
            continue
        cost = np.array([[np.linalg.norm(x[1] - y[1]) for y in b] for x in a])
        ia, ib = linear_sum_assignment(cost)
        dd = max((abs(a[i][0] - b[j][0]) for i, j in zip(ia, ib)), default=0.0)
        dp = max((float(np.max(np.abs(a[i][1] - b[j][1]))) for i, j in zip(ia, ib)), default=0.0)
        dn = max((float(np.max(np.abs(a[i][2] - b[j][2]))) for i, j in zip(ia, ib)), default=0.0)
        if key in aligned:
            aligned_report.append((key, len(a), dd, dp, dn))
            continue
        stats['pairs'] += 1
        stats['contacts'] += len(a)
        stats['dd'], stats['dp'], stats['dn'] = max(stats['dd'], dd), max(stats['dp'], dp), max(stats['dn'], dn)
    print('\n[seed %d] box pairs %s; count differences %s; aligned pairs %s (reference: %d contacts)'
          % (seed, stats, count_diff, aligned_report, r['count']))
    assert not count_diff
    assert stats['contacts'] >= 3 * n
    assert stats['dd'] <= 2e-4 and stats['dp'] <= 2e-4 and stats['dn'] <= 1e-3, stats
