"""Status words, the task predicate and batch quarantine, on the CPU.

The CPU oracle carries the same status rules as the CUDA kernel (the GPU
tests compare the two world by world):
  - a world whose qpos / qvel is non-finite or beyond 1e10 (MuJoCo
    mj_checkPos / mj_checkVel) gets B200_STATUS_BADSTATE and is not stepped;
  - an EPA whose vertex or face pool fills ends with its best face and
    reports the non-fatal B200_WARN_EPA_BUDGET, like its iteration limit (the
    reference's full face pool also ends its EPA without a status,
    mjwarp_convex_epa.cuh:89,219; EPA_HORIZON stays the fatal horizon-list
    overflow of the reference's OverflowType, cuda_fp32/constants.py:89-101);
  - reward and done are the synthetic task's sparse success predicate.
Batch quarantine follows the reference env (cuda_fp32/environment.py:126-140,
batch_env.py:298-302,376-384; tests/test_gpu_batch_env.py:123): a failed
step marks the batch failed and every later call asks for a rebuild.  Those
host rules run here against a fake runtime, as the reference tests them with
injected physics.
"""
import tomllib
from pathlib import Path
from threading import RLock

import numpy as np
import pytest

from gpu_libero_b200 import native, scene as scenes

ROOT = Path(__file__).resolve().parents[1]
BADSTATE, EPA_BUDGET = 1 << 16, 1 << 17


def oracle_world_state(oracle_module, scene, n, seed=3):
    packed = native.PackedModel(scene, 'fp32')
    host = native.alloc_numpy(packed, n)
    q, v = scene.initial_state(n, seed=seed)
    host['qpos'][:] = q
    host['qvel'][:] = v
    orc = oracle_module.Oracle('fp32')
    ms, ds = packed.host_struct(), native.data_struct(host, n)
    orc.forward(ms, ds, 0, n, 1)
    return orc, packed, host, ms, ds


def test_bad_state_worlds_are_flagged_and_not_stepped(oracle_module):
    scene = scenes.scene_a()
    n = 4
    orc, packed, host, ms, ds = oracle_world_state(oracle_module, scene, n)
    host['qpos'][1, 0] = np.nan
    host['qvel'][3, 2] = 1e11
    host['action'][:] = scene.actions(n, 0, seed=3)
    before = host['qpos'].copy()
    orc.step(ms, ds, 0, n, scene.substeps, 1)
    bad = (host['overflow'][:, 0] & BADSTATE) != 0
    assert bad.tolist() == [False, True, False, True]
    assert host['integration_count'][:, 0].tolist() == [25, 0, 25, 0]
    assert np.array_equal(host['qpos'][3], before[3])  # untouched
    assert np.all(np.isfinite(host['qpos'][[0, 2]]))


def test_task_predicate_is_the_lifted_task_body(oracle_module):
    scene = scenes.scene_a()
    n = 3
    orc, packed, host, ms, ds = oracle_world_state(oracle_module, scene, n)
    fb = scene.ints['free_bodyid'][scene.sizes['task_body']]
    j = int(np.flatnonzero(scene.ints['jnt_bodyid'] == fb)[0])
    host['qpos'][0, scene.ints['jnt_qposadr'][j] + 2] = 0.5  # held in the air: falls ~1 cm in a control step
    host['action'][:] = scene.actions(n, 0, seed=3)
    orc.step(ms, ds, 0, n, scene.substeps, 1)
    assert host['obs'][:, -2].tolist() == [1.0, 0.0, 0.0]
    assert host['obs'][:, -1].tolist() == [1.0, 0.0, 0.0]
    assert scene.scalars['task_lift_z'] == pytest.approx(0.2)


def test_epa_pool_overflow_is_reported(oracle_module):
    """A sphere inside a finely tessellated hull (2000 points on a sphere):
    EPA needs more than 44 expansions to resolve the nearest facet, so with a
    budget of 200 its 48-vertex pool fills and the budget status is raised;
    32 expansions (the scenes' setting) leave 36 vertices, below the pool."""
    orc = oracle_module.Oracle('fp64')
    rng = np.random.default_rng(1)
    d = rng.normal(size=(2000, 3))
    vert = 0.05 * d / np.linalg.norm(d, axis=1, keepdims=True)
    eye = np.eye(3).ravel()
    args = (2, np.array([0.003, 0.002, 0.001]), eye, [0.01, 0, 0], None, 7, np.zeros(3), eye, [0, 0, 0], vert)
    for budget, overflow in ((32, False), (44, False), (45, True), (200, True)):
        hit = orc.convex(*args, margin=0.0, tol=1e-12, iterations=50, epa_iterations=budget)
        assert hit is not None and hit[0] < -0.05, budget
        assert orc.epa_overflow == overflow, budget


# ---------------------------------------------------------------- quarantine (host logic)
class FakeRuntime:
    """Stands in for the device runtime: step_host returns the slab and the
    (overflow, error, integration count) status rows a real step copies back."""
    substeps = 25

    def __init__(self, n, nobs):
        self.n, self.nobs = n, nobs
        self.overflow = np.zeros(n, np.int32)
        self.commit = np.full(n, 25)
        self.count = np.zeros(n, np.int64)
        self.calls = 0

    def step_host(self, actions):
        import torch
        self.calls += 1
        self.count += self.commit
        status = np.stack([self.overflow, np.zeros(self.n, np.int32), self.count.astype(np.int32)])
        return torch.zeros((self.n, self.nobs)), torch.from_numpy(status)


def fake_env(n=4):
    pytest.importorskip('torch')
    from gpu_libero_b200.runtime import B200BatchEnv
    env = object.__new__(B200BatchEnv)
    env.scene = scenes.scene_a()
    env.num_envs = n
    env._lock = RLock()
    env._closed = env._failed = False
    env._integrations = np.zeros(n, np.int64)
    env.runtime = FakeRuntime(n, env.scene.sizes['nobs'])
    return env


def test_fatal_status_quarantines_the_batch():
    env = fake_env()
    obs, rew, done, info = env.step(np.zeros((4, 7)))
    assert rew.shape == (4,) and not done.any() and not env._failed
    env.runtime.overflow[2] = BADSTATE
    with pytest.raises(RuntimeError, match='failed_worlds'):
        env.step(np.zeros((4, 7)))
    assert env._failed
    with pytest.raises(RuntimeError, match='rebuild'):
        env.step(np.zeros((4, 7)))
    assert env.runtime.calls == 2


def test_limit_bits_are_legal_exits():
    env = fake_env()
    env.runtime.overflow[:] = (1 << 9) | (1 << 10)
    env.step(np.zeros((4, 7)))
    assert not env._failed


def test_invalid_actions_do_not_quarantine():
    env = fake_env()
    for actions in (np.zeros((3, 7)), np.full((4, 7), np.nan)):
        with pytest.raises(ValueError):
            env.step(actions)
    assert not env._failed and env.runtime.calls == 0


def test_missing_substep_commit_is_detected():
    env = fake_env()
    env.runtime.commit[1] = 24
    with pytest.raises(RuntimeError, match='commit every requested physics substep'):
        env.step(np.zeros((4, 7)))
    assert env._failed


def test_package_installs_under_an_importable_name():
    """pyproject.toml maps the importable package gpu_libero_b200 onto the
    source directory, so `pip install -e .` gives `import gpu_libero_b200`."""
    cfg = tomllib.loads((ROOT / 'pyproject.toml').read_text())
    mapping = cfg['tool']['setuptools']['package-dir']
    assert cfg['tool']['setuptools']['packages'] == ['gpu_libero_b200']
    assert (ROOT / mapping['gpu_libero_b200'] / '__init__.py').is_file()
