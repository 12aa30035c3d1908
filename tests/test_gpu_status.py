"""Status words, the task predicate and quarantine on the GPU, world by world
against the CPU oracle, through the C ABI.

No GPU fault is involved: bad states are injected from the host into chosen
worlds' qpos / qvel, and EPA's pool is exhausted by a legal configuration (a
sphere inside a 2000-point hull with a budget of 200 expansions and a 1e-12
tolerance).  The kernel reports both through per-world status bits and
returns normally; for a bad state the host raises and quarantines the batch,
while EPA's exhausted budget is a legal exit (its best face is the result).
"""
import numpy as np
import pytest

torch = pytest.importorskip('torch')
pytestmark = pytest.mark.gpu

from gpu_libero_b200 import native, scene as scenes  # noqa: E402
from gpu_libero_b200.runtime import B200BatchEnv, Runtime  # noqa: E402

BADSTATE, EPA_BUDGET = 1 << 16, 1 << 17


def host_copy(rt):
    host = native.alloc_numpy(rt.packed, rt.n)
    for k, t in rt.buffers.items():
        host[k][:] = t.cpu().numpy()
    return host


@pytest.mark.parametrize('precision', ['fp32', 'fp64'])
def test_bad_state_worlds_match_the_oracle(oracle_module, precision):
    scene = scenes.scene_a()
    n = 6
    rt = Runtime(scene, n, precision=precision)
    q, v = scene.initial_state(n, seed=8)
    rt.set_state(np.concatenate([np.zeros((n, 1)), q, v], axis=1))
    rt.buffers['qpos'][1, 0] = float('nan')
    rt.buffers['qvel'][4, 2] = 1e11
    torch.cuda.synchronize()
    ref = host_copy(rt)
    a = scene.actions(n, 0, seed=8)
    rt.enqueue_action(a)
    ref['action'][:] = a
    oracle_module.Oracle(precision).step(rt.packed.host_struct(), native.data_struct(ref, n), 0, n, 25, 1)
    torch.cuda.synchronize()
    gpu = {k: t.cpu().numpy() for k, t in rt.buffers.items()}
    bad = (gpu['overflow'][:, 0] & BADSTATE) != 0
    assert bad.tolist() == [False, True, False, False, True, False]
    assert np.array_equal(gpu['overflow'], ref['overflow'])
    assert gpu['integration_count'][:, 0].tolist() == [25, 0, 25, 25, 0, 25]
    assert np.array_equal(gpu['integration_count'], ref['integration_count'])
    assert gpu['qvel'][4, 2] == 1e11  # not stepped
    good = [0, 2, 3, 5]
    tol = 1e-4 if precision == 'fp32' else 1e-8  # one control step: measured 1.1e-9 in FP64
    assert np.max(np.abs(gpu['qpos'][good] - ref['qpos'][good])) < tol
    with pytest.raises(RuntimeError, match='failed_worlds'):
        rt.check()


def test_public_step_quarantines_after_a_bad_state():
    env = B200BatchEnv(scenes.scene_a(), 4, seed=1)
    env.step(env.scene.actions(4, 0, seed=1))
    env.runtime.buffers['qvel'][2, 0] = float('nan')
    with pytest.raises(RuntimeError, match='failed_worlds'):
        env.step(env.scene.actions(4, 1, seed=1))
    with pytest.raises(RuntimeError, match='rebuild'):
        env.step(env.scene.actions(4, 2, seed=1))
    d = env.diagnostics()  # still reports, without raising
    assert d['failed'] and d['upstream_status'][2] & BADSTATE
    assert d['actual_integration_count'] == [50, 50, 25, 50]
    env.close()
    # the device is healthy: a fresh batch steps
    ok = B200BatchEnv(scenes.scene_a(), 4, seed=1)
    ok.step(ok.scene.actions(4, 0, seed=1))
    ok.close()


@pytest.mark.parametrize('precision', ['fp32', 'fp64'])
def test_task_predicate_matches_the_oracle(oracle_module, precision):
    scene = scenes.scene_a()
    n = 4
    rt = Runtime(scene, n, precision=precision)
    q, v = scene.initial_state(n, seed=2)
    fb = scene.ints['free_bodyid'][scene.sizes['task_body']]
    j = int(np.flatnonzero(scene.ints['jnt_bodyid'] == fb)[0])
    q[[0, 3], scene.ints['jnt_qposadr'][j] + 2] = 0.5
    rt.set_state(np.concatenate([np.zeros((n, 1)), q, v], axis=1))
    torch.cuda.synchronize()
    ref = host_copy(rt)
    a = scene.actions(n, 0, seed=2)
    rt.enqueue_action(a)
    ref['action'][:] = a
    oracle_module.Oracle(precision).step(rt.packed.host_struct(), native.data_struct(ref, n), 0, n, 25, 1)
    torch.cuda.synchronize()
    obs = rt.buffers['obs'].cpu().numpy()
    assert obs[:, -2].tolist() == [1.0, 0.0, 0.0, 1.0] and obs[:, -1].tolist() == [1.0, 0.0, 0.0, 1.0]
    assert np.array_equal(obs[:, -2:], ref['obs'][:, -2:])
    tol = 1e-4 if precision == 'fp32' else 1e-8
    assert np.max(np.abs(obs - ref['obs'])) < tol


@pytest.mark.parametrize('precision', ['fp32', 'fp64'])
def test_epa_pool_overflow_matches_the_oracle(oracle_module, precision):
    b = scenes.scene_b(hull_points=2000, epa_iterations=200, ccd_tolerance=1e-12)
    n = 4
    rt = Runtime(b, n, precision=precision)
    q, v = b.initial_state(n, seed=21)
    fb = list(b.ints['free_bodyid'])
    names = [b.body_names[x] for x in fb]
    adr = lambda body: b.ints['jnt_qposadr'][np.flatnonzero(b.ints['jnt_bodyid'] == body)[0]]  # noqa: E731
    sph, hull = fb[names.index('sphere8')], fb[names.index('hull10')]
    for w in (0, 2):
        q[w, adr(hull):adr(hull) + 7] = [0.5, 0.0, 0.3, 1, 0, 0, 0]
        q[w, adr(sph):adr(sph) + 3] = [0.503, 0.002, 0.301]
    rows = np.concatenate([np.zeros((n, 1)), q, np.zeros_like(v)], axis=1)
    rt.set_state(rows)
    torch.cuda.synchronize()
    gpu = {k: t.cpu().numpy() for k, t in rt.buffers.items()}
    ref = native.alloc_numpy(rt.packed, n)
    ref['qpos'][:] = q
    oracle_module.Oracle(precision).forward(rt.packed.host_struct(), native.data_struct(ref, n), 0, n, 1)
    # the engineered worlds exhaust the budget on both sides; elsewhere EPA may
    # converge near the budget's edge, where rounding decides the last expansion
    assert np.all(gpu['overflow'][[0, 2], 0] & EPA_BUDGET) and np.all(ref['overflow'][[0, 2], 0] & EPA_BUDGET)
    assert np.array_equal(gpu['ncon'], ref['ncon'])
    rt.check()  # a legal exit: no raise
