"""Sphere and capsule contacts of the B200 kernel against the reference's own
native MuJoCo 2.3.7 colliders.

The reference's FP32 engine has no sphere-sphere, sphere-capsule or
capsule-capsule leaf; its native engine carries MuJoCo 2.3.7's colliders as
device code (libero/libero/gpu/cuda/collision/collision_detect_primitive.cuh:
mjc_SphereSphere, mjc_SphereCapsule, mjc_CapsuleCapsule).  oracle/Makefile
(target ref) compiles them unmodified, with real_t as double and as float,
into oracle/_ref/libref_native_{f64,f32}.so.

Both sides see the same geom poses: the B200 forward pass computes them and
writes geom_xpos / geom_xmat, and the reference colliders run on exactly those
arrays, in the same precision, with each pair's margin + gap as the margin
argument.  The reference's contacts are then filtered by the engine's publish
rule (dist < margin + gap, which every contact family shares).

Scene B holds 1 sphere-sphere, 24 sphere-capsule and 38 capsule-capsule pairs
per world, but its objects rarely touch each other in a rollout, so the states
here cluster its four capsules and two spheres, randomly posed, in a 12 cm
cube beside the arm's links (about 400 contacts of these families over 48
worlds), and add the colliders' special cases:
- world 0: two capsules with one orientation side by side (the parallel-axes
  branch with its two contacts);
- world 1: two spheres with one centre and different orientations (the normal
  from the cross product of their z axes);
- world 2: two spheres with one centre and one orientation (the fallback
  normal);
- world 3: a sphere centred at a capsule's centre (the nearest axis point is
  the sphere's centre, exactly, and the normal comes from the z axes).
A sphere centre a little way along the capsule's axis instead leaves a
residual of a few ulps against the colliders' 1e-15 threshold, on which two
compilations may branch differently; the exact case tests the branch.

Compared:
- contact counts per (world, pair) are equal;
- FP64: distances, points and normals within 1e-12 (the same formulas on the
  same doubles, up to the compilers' FMA contraction);
- FP32: distances and points within 2e-6 m, normals within 2e-5; for world
  0's parallel capsules only the distance, since in FP32 their determinant is
  rounding noise and so are the branch taken and the contact points (both
  implementations alike).

A contact whose distance lies within 1e-6 m (FP32) of its pair's cut-off sits
on the detection threshold, where two evaluations may fall on different sides;
such contacts may be present in one list only, and the test reports any it
allows.
"""
import numpy as np
import pytest

torch = pytest.importorskip('torch')
pytestmark = pytest.mark.gpu

from gpu_libero_b200 import scene as scenes  # noqa: E402

FAMILIES = {(2, 2), (2, 3), (3, 3)}
BOUNDS = {'fp64': dict(dist=1e-12, pos=1e-12, normal=1e-12, band=0.0),
          'fp32': dict(dist=2e-6, pos=2e-6, normal=2e-5, band=1e-6)}


def ref_lib(precision):
    import sys
    from pathlib import Path
    sys.path.insert(0, str(Path(__file__).resolve().parents[1] / 'oracle'))
    import ref_contacts
    if not ref_contacts.native_available():
        pytest.skip('oracle/_ref/libref_native_*.so not built (needs the reference checkout at build time)')
    return ref_contacts.RefNative(precision)


def clustered_state(scene, n, seed):
    """The scene's initial state with its capsules and spheres posed at random in
    a 12 cm cube beside the arm, plus the special cases of worlds 0-3."""
    q, v = scene.initial_state(n, seed=seed)
    rng = np.random.default_rng(seed)
    fb = list(scene.ints['free_bodyid'])
    names = [scene.body_names[x] for x in fb]

    def adr(name):
        body = fb[names.index(name)]
        return int(scene.ints['jnt_qposadr'][np.flatnonzero(scene.ints['jnt_bodyid'] == body)[0]])

    movers = ('capsule4', 'capsule5', 'capsule6', 'capsule7', 'sphere8', 'sphere9')
    center = np.array([0.45, 0.0, 0.55])
    for w in range(n):
        for name in movers:
            a = adr(name)
            quat = rng.normal(size=4)
            q[w, a:a + 3] = center + rng.uniform(-0.06, 0.06, 3)
            q[w, a + 3:a + 7] = quat / np.linalg.norm(quat)
    c4, c5, c6, s8, s9 = (adr(k) for k in ('capsule4', 'capsule5', 'capsule6', 'sphere8', 'sphere9'))
    r4, r5 = (float(np.reshape(scene.reals['geom_size'], (-1, 3))[geom_of(scene, k), 0]) for k in ('capsule4', 'capsule5'))
    q[0, c5 + 3:c5 + 7] = q[0, c4 + 3:c4 + 7]  # parallel axes, side by side, overlapping
    side = np.cross(_zaxis(q[0, c4 + 3:c4 + 7]), [0.0, 0.0, 1.0])
    side /= np.linalg.norm(side)
    q[0, c5:c5 + 3] = q[0, c4:c4 + 3] + side * (r4 + r5 - 0.004) + _zaxis(q[0, c4 + 3:c4 + 7]) * 0.01
    q[1, s9:s9 + 3] = q[1, s8:s8 + 3]  # one centre
    q[2, s9:s9 + 7] = q[2, s8:s8 + 7]  # one centre, one orientation
    q[3, s8:s8 + 3] = q[3, c6:c6 + 3]  # at the capsule's centre: its nearest axis point, exactly
    return q, v


def geom_of(scene, body_name):
    return int(np.flatnonzero(np.asarray(scene.ints['geom_bodyid']) == scene.body_names.index(body_name))[0])


def _zaxis(quat):
    w, x, y, z = quat
    return np.array([2 * (x * z + w * y), 2 * (y * z - w * x), 1 - 2 * (x * x + y * y)])


def forward_contacts(scene, precision, n, seed):
    from gpu_libero_b200.runtime import Runtime
    rt = Runtime(scene, n, precision=precision)
    q, v = clustered_state(scene, n, seed)
    rt.set_state(np.concatenate([np.zeros((n, 1)), q, v], axis=1))
    rt.forward()
    torch.cuda.synchronize()
    out = {k: rt.buffers[k].cpu().numpy() for k in ('geom_xpos', 'geom_xmat', 'ncon', 'con_geom', 'con_dist',
                                                      'con_pos', 'con_frame', 'overflow')}
    rt.close()
    return out


@pytest.mark.parametrize('precision', ['fp64', 'fp32'])
@pytest.mark.parametrize('seed', [5, 6])
def test_sphere_capsule_contacts_match_reference_native_colliders(precision, seed):
    from scipy.optimize import linear_sum_assignment
    ref = ref_lib(precision)
    scene = scenes.scene_b()
    n = 48
    out = forward_contacts(scene, precision, n, seed)
    assert not np.any(out['overflow'])
    types = np.asarray(scene.ints['geom_type'])
    pairs = np.asarray(scene.ints['pair_geom'], np.int64).reshape(-1, 2)
    fam = np.array([tuple(sorted((int(types[a]), int(types[b])))) in FAMILIES for a, b in pairs])
    pairs = pairs[fam]
    assert len(pairs) >= 60 and np.all(types[pairs[:, 0]] <= types[pairs[:, 1]])
    margin = np.asarray(scene.reals['geom_margin'], float)
    gap = np.asarray(scene.reals['geom_gap'], float)
    cut = margin[pairs[:, 0]] + margin[pairs[:, 1]] + gap[pairs[:, 0]] + gap[pairs[:, 1]]
    count, hits = ref.collide(scene, out['geom_xpos'], out['geom_xmat'], pairs, cut)
    assert np.all(count >= 0)
    b = BOUNDS[precision]
    index = {(int(a), int(c)): j for j, (a, c) in enumerate(pairs)}
    worst, where = dict(dist=0.0, pos=0.0, normal=0.0), {}
    compared = band = 0
    special = [0, 0, 0, 0]
    specials = [{geom_of(scene, a), geom_of(scene, c)} for a, c in
                (('capsule4', 'capsule5'), ('sphere8', 'sphere9'), ('sphere8', 'sphere9'), ('sphere8', 'capsule6'))]
    for w in range(n):
        nc = int(out['ncon'][w, 0])
        geom = out['con_geom'][w, :2 * nc].reshape(-1, 2)
        ours = {}
        for i in range(nc):
            key = (int(geom[i, 0]), int(geom[i, 1]))
            if key in index:
                ours.setdefault(key, []).append(i)
        for key, j in index.items():
            h = hits[w, j, :count[w, j]].astype(float)
            h = h[h[:, 0] < cut[j]]  # the publish rule
            mine = ours.get(key, [])
            d = out['con_dist'][w, mine].astype(float)
            if precision == 'fp32' and w == 0 and set(key) == specials[0]:
                # exactly parallel axes: in FP32 the determinant is rounding
                # noise, so the branch and the contact points are too; the
                # distance between the axes is not
                assert len(mine) and len(h) and abs(d.min() - h[:, 0].min()) <= b['dist']
                special[0] += 2
                continue
            p = out['con_pos'][w].reshape(-1, 3)[mine].astype(float)
            nrm = out['con_frame'][w].reshape(-1, 9)[mine, :3].astype(float)
            if len(mine) != len(h):  # only contacts on the detection threshold may differ
                longer = d if len(mine) > len(h) else h[:, 0]
                near = [x for x in longer if abs(x - cut[j]) <= b['band']]
                assert len(near) >= abs(len(mine) - len(h)) and b['band'] > 0, (w, key, d, h[:, 0])
                band += abs(len(mine) - len(h))
                continue
            if not len(h):
                continue
            cost = np.linalg.norm(p[:, None, :] - h[None, :, 1:4], axis=2)
            r, c = linear_sum_assignment(cost)
            for k, e in (('dist', np.abs(d[r] - h[c, 0])), ('pos', np.abs(p[r] - h[c, 1:4])),
                         ('normal', np.abs(nrm[r] - h[c, 4:7]))):
                if float(np.max(e)) > worst[k]:
                    worst[k], where[k] = float(np.max(e)), (w, key)
            compared += len(r)
            if w < 4 and set(key) == specials[w]:
                special[w] += len(r)
    print('\n[%s, seed %d] %d contacts compared (special worlds: %s); worst %s; %d threshold contacts in one '
          'list only' % (precision, seed, compared, special, {k: '%.1e' % v for k, v in worst.items()}, band))
    assert compared >= 300
    assert special[0] >= 2 and special[1] >= 1 and special[2] >= 1 and special[3] >= 1
    for k in worst:
        assert worst[k] <= b[k], (k, worst[k], 'world, pair', where[k])
