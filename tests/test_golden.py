"""The CPU oracle pinned against the reference's golden vectors.

Fixtures (tests/golden/, written by make_golden.py from the reference's
FP64 validation oracles and shipped box-box fixtures):
  kinematics_scene_a.npz       mjwarp_kinematics_reference.reference(c, 'composed')
  plane_contacts_scene_a.npz   mjwarp_plane_reference.reference(c) (manifolds + material mixing)
  constraint_rows_scene_a.npz  mjwarp_constraint_build_reference.build_reference(c)
  euler_position_scene_a.npz   mjwarp_euler_reference.reference(c, 'position')
  box_pairs.npz                mjwarp_box_reference.pair_math (SAT separation, segment-box distance)
  box_fixtures.json            tests/fixtures/boxbox_* and tests/cuda/precision_boxbox_test.cu cases
  gjk_tuned_direction.json     tests/data/gjk_tuned_direction.json with its SAT depth (box_separation)

Tolerances: FP64 oracle within 1e-12 absolute of the reference's FP64 values
(bit-level agreement up to summation order); FP32 oracle within 8x the
reference's propagated FP32 error radius (the reference harness's fixed8x
safety factor, mjwarp_kinematics_reference.py docstring), plus exact
agreement of every discrete result (contact sets, counts, row kinds).
"""
import numpy as np
import pytest

from golden_checks import (EPS32, PLANE, box_cases, contact_failures, load, plane_groups, unique_points,
                           witness_violation)
from gpu_libero_b200 import native, scene as scenes

PRECISIONS = ('fp64', 'fp32')


@pytest.fixture(scope='module')
def scene():
    return scenes.scene_a()


@pytest.fixture(scope='module', params=PRECISIONS)
def oracle(request, oracle_module, scene):
    orc = oracle_module.Oracle(request.param)
    return request.param, orc, native.PackedModel(scene, request.param).host_struct()


def within(got, want, err, precision, atol64=1e-12, floor32=0.0):
    """FP32: 8x the reference's error radius, plus `floor32` for the rounding
    the FP32 path carries in from upstream stages (the radius assumes exact
    FP64 inputs)."""
    got, want, err = (np.asarray(x, float) for x in (got, want, err))
    tol = atol64 if precision == 'fp64' else 8 * err + 4 * EPS32 * np.abs(want) + floor32
    return bool(np.all(np.abs(got - want) <= tol))


def test_kinematics_matches_reference(scene, oracle):
    precision, orc, ms = oracle
    g = load('kinematics_scene_a.npz')
    for w in range(len(g['qpos'])):
        got = orc.positions(ms, scene.sizes, g['qpos'][w])
        for key in ('xpos', 'xquat', 'xipos', 'geom_xpos', 'geom_xmat'):
            assert within(got[key].reshape(-1), g[key][w], g[key + '_err'][w], precision), (w, key)


def test_plane_contacts_match_reference(scene, oracle):
    precision, orc, ms = oracle
    g = load('plane_contacts_scene_a.npz')
    rows = g['rows']
    plane = scene.ints['geom_type'] == 0
    checked = 0
    for w in range(len(g['qpos'])):
        con = orc.contacts(ms, scene.sizes, g['qpos'][w], g['qvel'][w])
        mine = {}
        for i, (a, b) in enumerate(con['geom']):
            if plane[a]:
                mine.setdefault((int(a), int(b)), []).append(i)
        for pair, ref in plane_groups(rows, w).items():
            got = mine.get(pair, [])
            if precision == 'fp64':  # detection is exact in FP64 away from the threshold
                assert not any(abs(r[PLANE['dist']] - r[PLANE['margin']]) < 1e-12 for r in ref)
                emitted = [r for r in ref if r[PLANE['dist']] < r[PLANE['margin']]]
                assert len(got) == len(emitted), (w, pair)
            else:  # FP32: every certain contact present, the rest within the reference's budget band
                emitted = []
                for i in got:
                    gap = [abs(con['dist'][i] - r[PLANE['dist']]) + np.max(np.abs(con['pos'][i] - r[PLANE['pos']]))
                           for r in ref]
                    emitted.append(ref[int(np.argmin(gap))])
                ids = [int(r[3]) for r in emitted]
                assert len(set(ids)) == len(ids)
                assert {int(r[3]) for r in ref if r[PLANE['must']]} <= set(ids), (w, pair)
            for i, r in zip(got, emitted):
                tol = 1e-12 if precision == 'fp64' else r[PLANE['budget']]
                assert abs(con['dist'][i] - r[PLANE['dist']]) <= tol
                assert np.max(np.abs(con['pos'][i] - r[PLANE['pos']])) <= tol
                assert np.max(np.abs(con['frame'][i].ravel() - r[PLANE['frame']])) <= tol
                assert con['dim'][i] == r[PLANE['dim']]
                assert np.allclose(con['friction'][i], r[PLANE['friction']], rtol=1e-6)
                assert np.allclose(con['solref'][i], r[PLANE['solref']], rtol=1e-6)
                assert np.allclose(con['solimp'][i], r[PLANE['solimp']], rtol=1e-6)
                assert abs(con['margin'][i] - r[PLANE['margin']]) <= 1e-9
                checked += 1
        assert set(mine) <= set(plane_groups(rows, w)) | {p for p in mine if not mine[p]}
    assert checked >= 60


def test_constraint_rows_match_reference(scene, oracle):
    precision, orc, ms = oracle
    g = load('constraint_rows_scene_a.npz')
    rows, nv = g['rows'], scene.sizes['nv']
    kinds = {1: 'friction', 3: 'limit', 7: 'contact'}
    seen = set()
    for w in range(len(g['qpos'])):
        con = orc.contacts(ms, scene.sizes, g['qpos'][w], g['qvel'][w])
        ref = rows[rows[:, 0] == w]
        if precision == 'fp32':  # the contact set must match the FP64 reference's
            want = g['contacts'][g['contacts'][:, 0] == w]
            assert np.array_equal(con['geom'], want[:, 1:3].astype(int))
        assert con['nefc'] == len(ref)
        assert np.array_equal(con['id'], ref[:, 2].astype(int))
        seen |= {kinds[int(k)] for k in ref[:, 1]}
        J, Jerr = ref[:, 9:9 + nv], ref[:, 9 + nv:9 + 2 * nv]
        # contact Jacobians: FP32 contact points/frames/cdof enter with ~1 ulp of the lever arm
        assert within(con['J'], J, Jerr, precision, floor32=4 * EPS32 * max(1.0, np.abs(J).max()))
        assert within(con['D'], ref[:, 4], ref[:, 5], precision, atol64=1e-9 * np.abs(ref[:, 4]).max())
        assert within(con['aref'], ref[:, 6], ref[:, 7], precision, atol64=1e-9 * max(1, np.abs(ref[:, 6]).max()))
    assert seen == {'friction', 'limit', 'contact'}


def test_euler_position_phase_matches_reference(scene, oracle):
    precision, orc, ms = oracle
    g = load('euler_position_scene_a.npz')
    for w in range(len(g['qpos'])):
        got = orc.integrate(ms, g['qpos'][w], g['qvel'][w], float(g['timestep']))
        assert within(got, g['qpos_next'][w], g['qpos_next_err'][w], precision), w


def test_box_pairs_pass_reference_geometry(oracle):
    precision, orc, _ = oracle
    counts = {2: 0, 3: 0, 6: 0}
    for case in box_cases():
        dist, pos, normal = orc.box(case['kind'], case['p1'], case['R1'], case['s1'], case['p2'], case['R2'],
                                    case['s2'], 0.0)
        assert len(dist) == case['count']
        assert contact_failures(case, dist, pos, normal, case['budget']) == []
        counts[case['kind']] += int(np.sum(dist < 1e9))
    assert min(counts.values()) > 50


def run_box(orc, f, margin=0.0):
    size, pos, mat = (np.asarray(f[k], float) for k in ('size', 'pos', 'mat'))
    mat = mat.reshape(2, 3, 3)
    d, p, n = orc.box(6, pos[0], mat[0], size[0], pos[1], mat[1], size[1], margin)
    return d, p, n, size, pos, mat


def test_reference_boxbox_fixtures(oracle):
    precision, orc, _ = oracle
    fx = load('box_fixtures.json')
    tol = 1e-12 if precision == 'fp64' else 2e-7
    # captured LIBERO-10 book/table pair: four contacts, no lateral negative depth
    d, p, n, size, pos, mat = run_box(orc, fx['task5'])
    scale = float(np.max(np.abs(pos) + size))
    slack = 0.0 if precision == 'fp64' else 16 * EPS32 * scale  # FP32 rounding of metre-scale poses
    assert len(d) == fx['task5']['count']
    assert d.min() > fx['task5']['min_dist'] - slack
    assert abs(d.min() + fx['task5']['physical_overlap']) <= (1e-12 if precision == 'fp64' else 2e-7)
    assert witness_violation(d, p, n, size, pos, mat) <= (1e-12 if precision == 'fp64' else 1e-6)
    for margin in (0.01, 2.0):
        assert len(run_box(orc, fx['task5'], margin)[0]) >= 4
    for f in fx['task5_rotated']:
        d = run_box(orc, f)[0]
        assert len(d) > 0 and d.min() > (-2e-7 - slack) * f['scale'] and d.max() <= (1e-12 + slack) * f['scale']
    # edge projection: witnesses on both surfaces
    d, p, n, size, pos, mat = run_box(orc, fx['edge_projection'])
    assert len(d) >= 1 and witness_violation(d, p, n, size, pos, mat) <= (1e-10 if precision == 'fp64' else 1e-6)
    # first incident vertex belongs to the reference face, both orders
    f = fx['first_face_vertex']
    for swap in (False, True):
        g = {k: (np.asarray(f[k])[::-1] if swap else np.asarray(f[k])) for k in ('size', 'pos', 'mat')}
        d, p, n, size, pos, mat = run_box(orc, g)
        assert len(d) == f['count']
        assert witness_violation(d, p, n, size, pos, mat) <= f['tolerance'] + tol
    # face/edge SAT tie: four unique contacts at the SAT depth, three scales
    for label in ('sat_face_tie_fp32', 'sat_face_tie_fp64'):
        f = fx[label]
        for scale in (1e-3, 1.0, 1e3):
            g = dict(size=np.asarray(f['size']) * scale, pos=np.asarray(f['pos']) * scale, mat=f['mat'])
            for swap in (False, True):
                h = {k: (np.asarray(v)[::-1] if swap else np.asarray(v)) for k, v in g.items()}
                d, p, n, size, pos, mat = run_box(orc, h)
                big = max(1.0, float(np.max(np.abs(h['pos']) + h['size'])))
                assert len(unique_points(p, 16 * EPS32 * big)) == f['count']
                assert np.all(np.abs(d - f['separation'] * scale) <= 16 * EPS32 * big)
    # unit boxes: contact counts at face, edge and corner touch
    for x, y, z, count in fx['unit_boxes']['cases']:
        d, p, n = orc.box(6, [0, 0, 0], np.eye(3), [1, 1, 1], [x, y, z], np.eye(3), [1, 1, 1])
        assert len(unique_points(p, 16 * EPS32 * 3)) == count


def box_corners(size):
    return np.array([[sx * size[0], sy * size[1], sz * size[2]] for sx in (-1, 1) for sy in (-1, 1) for sz in (-1, 1)])


def test_convex_path_against_reference_box_geometry(oracle):
    """GJK/EPA on hulls built from box corners reproduces the reference's
    independent SAT separation (box pairs) and segment-box distances
    (sphere / capsule against a box hull, centres outside the box)."""
    precision, orc, _ = oracle
    tol = 1e-12 if precision == 'fp64' else 2e-5
    checked = {2: 0, 3: 0, 6: 0}
    for case in box_cases():
        kind = case['kind']
        v1 = box_corners(case['s1']) if kind == 6 else None
        got = orc.convex(7 if kind == 6 else kind, case['p1'], case['R1'], case['s1'], v1, 7, case['p2'], case['R2'],
                         case['s2'], box_corners(case['s2']))
        if kind == 6:
            want = case['separation']
        elif case['inside']:
            continue
        else:
            want = case['closest']
        if want < -max(tol, 1e-9):
            assert got is not None, case
            assert abs(got[0] - want) <= tol, (kind, got[0], want)
            assert abs(np.linalg.norm(got[2]) - 1) < 1e-5
            checked[kind] += 1
        elif want > max(tol, 1e-9):
            assert got is None
    assert min(checked.values()) >= 20


def test_recorded_boxbox_overlap_is_not_declared_separated(oracle):
    """The reference's recorded LIBERO overlap (gjk_tuned_direction.json: two
    boxes 39 µm deep that a tuned GJK direction once declared separated).
    GJK/EPA, on the boxes as primitives against hulls and as two hulls, must
    report the contact at the reference's SAT depth, within the CCD tolerance
    in FP32."""
    precision, orc, _ = oracle
    f = load('gjk_tuned_direction.json')
    p, R, s = (np.asarray(f[k], float) for k in ('pos', 'mat', 'size'))
    tol = 1e-12 if precision == 'fp64' else 2 * f['tolerance']
    kw = dict(tol=f['tolerance'], iterations=f['iterations'], epa_iterations=f['epa_iterations'])
    for kind1, v1 in ((6, None), (7, box_corners(s[0]))):
        got = orc.convex(kind1, p[0], R[0], s[0], v1, 7, p[1], R[1], s[1], box_corners(s[1]), **kw)
        assert got is not None, (precision, kind1)
        assert abs(got[0] - f['separation']) <= tol, (precision, kind1, got[0], f['separation'])
