"""The CUDA forward pass against the reference's golden vectors (tests/golden/).

Same fixtures and tolerances as test_golden.py (the CPU oracle's pins):
FP64 within 1e-10 of the reference's FP64 values, FP32 within 8x the
reference's propagated FP32 error radius; contact sets exact in FP64 and
inside the reference's must/possible band in FP32.  Constraint rows are read
from the kernel's inspection outputs (efc_J expanded to dense dof order,
efc_D, efc_aref, efc_type, efc_id of the forward's rows).
"""
import numpy as np
import pytest

torch = pytest.importorskip('torch')
pytestmark = pytest.mark.gpu

from golden_checks import EPS32, PLANE, load, plane_groups  # noqa: E402
from gpu_libero_b200 import native, scene as scenes  # noqa: E402


@pytest.fixture(scope='module')
def scene():
    return scenes.scene_a()


def forward(scene, precision, qpos, qvel=None):
    from gpu_libero_b200.runtime import Runtime
    n = len(qpos)
    rt = Runtime(scene, n, precision=precision, debug=True)
    qvel = np.zeros((n, scene.sizes['nv'])) if qvel is None else qvel
    rt.set_state(np.concatenate([np.zeros((n, 1)), qpos, qvel], axis=1))
    torch.cuda.synchronize()
    out = {k: t.cpu().numpy().astype(float) if t.is_floating_point() else t.cpu().numpy()
           for k, t in rt.buffers.items()}
    rt.close()
    return out


@pytest.mark.parametrize('precision', ['fp64', 'fp32'])
def test_cuda_kinematics_matches_reference(scene, precision):
    g = load('kinematics_scene_a.npz')
    out = forward(scene, precision, g['qpos'])
    for key in ('xpos', 'xquat', 'xmat', 'geom_xpos', 'geom_xmat', 'site_xpos', 'site_xmat'):
        want, err = g[key], g[key + '_err']
        tol = 1e-10 if precision == 'fp64' else 8 * err + 4 * EPS32 * np.abs(want)
        assert np.all(np.abs(out[key] - want) <= tol), key


@pytest.mark.parametrize('precision', ['fp64', 'fp32'])
def test_cuda_plane_contacts_match_reference(scene, precision):
    g = load('plane_contacts_scene_a.npz')
    rows = g['rows']
    out = forward(scene, precision, g['qpos'], g['qvel'])
    plane = scene.ints['geom_type'] == 0
    checked = 0
    for w in range(len(g['qpos'])):
        n = int(out['ncon'][w, 0])
        geoms = out['con_geom'][w, :2 * n].reshape(n, 2)
        dist = out['con_dist'][w, :n]
        pos = out['con_pos'][w, :3 * n].reshape(n, 3)
        frame = out['con_frame'][w, :9 * n].reshape(n, 9)
        mine = {}
        for i, (a, b) in enumerate(geoms):
            if plane[a]:
                mine.setdefault((int(a), int(b)), []).append(i)
        groups = plane_groups(rows, w)
        assert set(mine) <= set(groups)
        for pair, ref in groups.items():
            got = mine.get(pair, [])
            if precision == 'fp64':
                emitted = [r for r in ref if r[PLANE['dist']] < r[PLANE['margin']]]
                assert len(got) == len(emitted), (w, pair)
            else:
                emitted = [ref[int(np.argmin([abs(dist[i] - r[PLANE['dist']]) +
                                              np.max(np.abs(pos[i] - r[PLANE['pos']])) for r in ref]))]
                           for i in got]
                ids = [int(r[3]) for r in emitted]
                assert len(set(ids)) == len(ids)
                assert {int(r[3]) for r in ref if r[PLANE['must']]} <= set(ids), (w, pair)
            for i, r in zip(got, emitted):
                tol = 1e-10 if precision == 'fp64' else r[PLANE['budget']]
                assert abs(dist[i] - r[PLANE['dist']]) <= tol
                assert np.max(np.abs(pos[i] - r[PLANE['pos']])) <= tol
                assert np.max(np.abs(frame[i] - r[PLANE['frame']])) <= tol
                checked += 1
    assert checked >= 60


def within(got, want, err, precision, atol64, floor32=0.0):
    got, want, err = (np.asarray(x, float) for x in (got, want, err))
    tol = atol64 if precision == 'fp64' else 8 * err + 4 * EPS32 * np.abs(want) + floor32
    return bool(np.all(np.abs(got - want) <= tol))


@pytest.mark.parametrize('precision', ['fp64', 'fp32'])
def test_cuda_constraint_rows_match_reference(scene, precision):
    """Friction-loss, joint-limit and elliptic contact rows of the CUDA forward,
    row by row (kinds, ids, dense Jacobian, D, aref) against the reference's
    mjwarp_constraint_build_reference rows."""
    g = load('constraint_rows_scene_a.npz')
    rows, nv = g['rows'], scene.sizes['nv']
    out = forward(scene, precision, g['qpos'], g['qvel'])
    kinds = {1: 'friction', 3: 'limit', 7: 'contact'}
    seen = set()
    for w in range(len(g['qpos'])):
        ref = rows[rows[:, 0] == w]
        n = int(out['nefc'][w, 0])
        assert n == len(ref), w
        assert np.array_equal(out['efc_type'][w, :n], ref[:, 1].astype(int)), w
        assert np.array_equal(out['efc_id'][w, :n], ref[:, 2].astype(int)), w
        seen |= {kinds[int(k)] for k in ref[:, 1]}
        J, Jerr = ref[:, 9:9 + nv], ref[:, 9 + nv:9 + 2 * nv]
        got_J = out['efc_J'][w, :n * nv].reshape(n, nv)
        assert within(got_J, J, Jerr, precision, 1e-10, floor32=4 * EPS32 * max(1.0, np.abs(J).max())), w
        assert within(out['efc_D'][w, :n], ref[:, 4], ref[:, 5], precision, 1e-9 * np.abs(ref[:, 4]).max()), w
        assert within(out['efc_aref'][w, :n], ref[:, 6], ref[:, 7], precision,
                      1e-9 * max(1, np.abs(ref[:, 6]).max())), w
    assert seen == {'friction', 'limit', 'contact'}


@pytest.mark.parametrize('precision', ['fp64', 'fp32'])
def test_cuda_euler_position_phase(scene, oracle_module, precision):
    """One CUDA substep from the golden states: the position phase (free-joint
    quaternion exponential map, hinge/slide increments) of the new velocity
    equals the oracle's integrator, which euler_position_scene_a.npz pins to
    the reference (mjwarp_euler_reference.reference(c, 'position'))."""
    from gpu_libero_b200.runtime import Runtime
    g = load('euler_position_scene_a.npz')
    n = len(g['qpos'])
    rt = Runtime(scene, n, precision=precision)
    rt.set_state(np.concatenate([np.zeros((n, 1)), g['qpos'], g['qvel']], axis=1))
    q0 = rt.buffers['qpos'].cpu().numpy().copy()
    rt.launch_step(policy=False, substeps=1)
    torch.cuda.synchronize()
    q1, v1 = rt.buffers['qpos'].cpu().numpy(), rt.buffers['qvel'].cpu().numpy()
    orc = oracle_module.Oracle(precision)
    ms = rt.packed.host_struct()
    dt = float(scene.scalars['timestep'])
    for w in range(n):
        want = orc.integrate(ms, q0[w], v1[w], dt)
        tol = 1e-14 if precision == 'fp64' else 4 * EPS32 * np.maximum(1.0, np.abs(want))
        assert np.all(np.abs(q1[w] - want) <= tol), w
    assert float(g['timestep']) == dt
