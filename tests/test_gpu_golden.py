"""The CUDA forward pass against the reference's golden vectors (tests/golden/).

Same fixtures and tolerances as test_golden.py (the CPU oracle's pins):
FP64 within 1e-10 of the reference's FP64 values, FP32 within 8x the
reference's propagated FP32 error radius; contact sets exact in FP64 and
inside the reference's must/possible band in FP32.
"""
import numpy as np
import pytest

torch = pytest.importorskip('torch')
pytestmark = pytest.mark.gpu

from golden_checks import EPS32, PLANE, load, plane_groups  # noqa: E402
from gpu_libero_b200 import scene as scenes  # noqa: E402


@pytest.fixture(scope='module')
def scene():
    return scenes.scene_a()


def forward(scene, precision, qpos, qvel=None):
    from gpu_libero_b200.runtime import Runtime
    n = len(qpos)
    rt = Runtime(scene, n, precision=precision)
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
