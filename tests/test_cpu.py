"""CPU tests: C ABI surface, scene compiler, oracle behaviour, host logic."""
import ctypes as ct
import re
import xml.etree.ElementTree as ET
from pathlib import Path

import numpy as np
import pytest

from gpu_libero_b200 import native, scene as scenes, selection

ROOT = Path(__file__).resolve().parents[1]


@pytest.fixture(scope='module')
def scene():
    return scenes.scene_a()


def declared_functions():
    text = (ROOT / 'include' / 'b200phys.h').read_text()
    return sorted(set(re.findall(r'\b(b200phys_\w+)\s*\(', text)))


def test_library_exports_every_declared_symbol():
    lib = native.Library()  # also checks sizeof(B200Model/B200Data) against ctypes
    names = declared_functions()
    assert set(native.EXPORTS) == set(names)
    for name in names:
        assert hasattr(lib.lib, name), name
    assert lib.arch == 100
    assert lib.source_id.startswith('b200phys-')


def test_struct_layouts_follow_the_field_header():
    assert ct.sizeof(native.B200Data) == 8 + 8 * (len(native.LAYOUT.data_real) + len(native.LAYOUT.data_int))
    lib = native.Library()
    assert lib.lib.b200phys_model_bytes() == ct.sizeof(native.B200Model)


def test_world_smem_fits_a_b200_block(scene):
    lib = native.Library()
    for precision in ('fp32', 'fp64'):
        smem = lib.smem_bytes(native.PackedModel(scene, precision).host_struct())
        assert 0 < smem <= 227 * 1024


def test_scene_a_sizes(scene):
    s = scene.sizes
    assert (s['nq'], s['nv'], s['nu'], s['njnt']) == (30, 27, 9, 12)
    assert s['nM'] == 9 * 9 + 3 * 36 and s['ntree'] == 4
    assert set(scene.pair_families) == {(0, 3), (0, 6), (3, 6), (6, 6)}
    assert scene.supported
    # the arm never collides with itself (contype/conaffinity), as admitted by the reference
    arm = set(range(1, 11))
    g = scene.ints['geom_bodyid']
    pairs = scene.ints['pair_geom'].reshape(-1, 2)
    assert not any(g[a] in arm and g[b] in arm for a, b in pairs)
    assert np.all(scene.reals['body_invweight0'][11:] > 0)
    assert scene.scalars['meaninertia'] > 0


def test_mjcf_is_well_formed(scene):
    root = ET.fromstring(scene.mjcf())
    assert root.tag == 'mujoco'
    assert len(root.findall('.//joint')) == scene.sizes['njnt']
    assert len(root.findall('.//geom')) == scene.sizes['ngeom']
    assert len(root.findall('.//actuator/general')) == scene.sizes['nu']


def test_seeds_do_not_depend_on_shard_layout(scene):
    q_all, _ = scene.initial_state(8, seed=3)
    q_hi, _ = scene.initial_state(4, seed=3, world_offset=4)
    assert np.array_equal(q_all[4:], q_hi)
    a = scene.actions(4, 2, seed=3, world_offset=0)
    assert a.shape == (4, 7) and np.all(np.abs(a) <= 1) and set(np.unique(a[:, 6])) <= {-1.0, 1.0}
    assert np.array_equal(scene.actions(8, 2, seed=3)[5:], scene.actions(3, 2, seed=3, world_offset=5))
    assert np.array_equal(scene.actions(8, 2, seed=3)[:1], scene.actions(1, 2, seed=3))


def run_oracle(oracle_module, scene, precision, n, steps, seed):
    packed = native.PackedModel(scene, precision)
    host = native.alloc_numpy(packed, n)
    q, v = scene.initial_state(n, seed=seed)
    host['qpos'][:] = q
    host['qvel'][:] = v
    orc = oracle_module.Oracle(precision)
    ms, ds = packed.host_struct(), native.data_struct(host, n)
    orc.forward(ms, ds, 0, n, 1)
    for k in range(steps):
        host['action'][:] = scene.actions(n, k, seed=seed)
        orc.step(ms, ds, 0, n, scene.substeps, 1)
    return host


def test_oracle_is_stable_and_boxes_rest(oracle_module, scene):
    h = run_oracle(oracle_module, scene, 'fp32', 3, 20, seed=1)
    assert np.all(np.isfinite(h['qpos'])) and not np.any(h['error'])
    assert not np.any(h['overflow'] & ~0x600)
    for a in scene.ints['jnt_qposadr'][scene.ints['jnt_type'] == 0]:
        z = h['qpos'][:, a + 2]
        assert np.all(z > 0.015) and np.all(z < 0.06)
    assert np.all(h['integration_count'] == 500)
    assert np.all(h['time'][:, 0] == pytest.approx(1.0, rel=1e-5))


def test_oracle_fp32_tracks_fp64(oracle_module, scene):
    a = run_oracle(oracle_module, scene, 'fp32', 2, 4, seed=2)
    b = run_oracle(oracle_module, scene, 'fp64', 2, 4, seed=2)
    assert np.max(np.abs(a['qpos'] - b['qpos'])) < 1e-3
    assert np.array_equal(a['ncon'], b['ncon'])


def test_oracle_is_deterministic(oracle_module, scene):
    a = run_oracle(oracle_module, scene, 'fp32', 2, 3, seed=4)
    b = run_oracle(oracle_module, scene, 'fp32', 2, 3, seed=4)
    assert np.array_equal(a['qpos'], b['qpos'])


def test_resolve_engine_mirrors_reference_rules():
    assert selection.resolve_engine('auto', 'fp32') == 'cuda_fp32'
    assert selection.resolve_engine('auto', 'fp64') == 'native'
    assert selection.resolve_engine('b200', 'fp64') == 'b200'
    with pytest.raises(ValueError):
        selection.resolve_engine('warp')
    with pytest.raises(ValueError):
        selection.resolve_engine('cuda_fp32', 'fp64')
    with pytest.raises(ValueError):
        selection.resolve_engine('b200', 'fp16')


def test_product_path_fails_loudly_without_cuda(scene):
    torch = pytest.importorskip('torch')
    if torch.cuda.is_available():
        pytest.skip('a CUDA device is present')
    from gpu_libero_b200.runtime import B200BatchEnv
    with pytest.raises(RuntimeError, match='CUDA'):
        B200BatchEnv(scene, 2)


def test_oracle_pyramidal_cones_rest_and_track_fp64(oracle_module):
    pyr = scenes.scene_a(cone='pyramidal')
    assert pyr.sizes['cone'] == 0 and pyr.sizes['nefc_max'] == 9 + 9 + 4 * pyr.sizes['ncon_max']
    a = run_oracle(oracle_module, pyr, 'fp32', 2, 10, seed=6)
    b = run_oracle(oracle_module, pyr, 'fp64', 2, 10, seed=6)
    assert not np.any(a['overflow'] & ~0x600) and not np.any(a['error'])
    assert np.max(np.abs(a['qpos'] - b['qpos'])) < 1e-3
    for j in np.flatnonzero(pyr.ints['jnt_type'] == 0):
        z = a['qpos'][:, pyr.ints['jnt_qposadr'][j] + 2]
        assert np.all(z > 0.015) and np.all(z < 0.06)


@pytest.fixture(scope='module')
def scene_b():
    return scenes.scene_b()


def test_scene_b_sizes_and_families(scene_b):
    s = scene_b.sizes
    assert (s['nq'], s['nv'], s['nfree'], s['nobs']) == (93, 81, 12, 111)
    assert s['nmesh'] == 2 and s['nmeshvert'] == 64
    assert scene_b.supported
    fam = set(scene_b.pair_families)
    assert {(2, 2), (2, 3), (3, 3), (0, 7), (2, 7), (3, 7), (6, 7), (7, 7)} <= fam
    root = ET.fromstring(scene_b.mjcf())
    assert len(root.findall('.//asset/mesh')) == 2
    assert len(root.findall('.//geom')) == s['ngeom']
    # hull mass properties: centroid at the geom origin, symmetric positive inertia
    for b in scene_b.bodies:
        for g in b.geoms:
            if g.kind == scenes.MESH:
                v = g.mesh['vert']
                assert len(v) == 32 and g.mesh['volume'] > 0
                assert np.all(np.linalg.eigvalsh(g.mesh['inertia']) > 0)
                n = g.mesh['normals']
                for (a, bb, c), nn in zip(g.mesh['faces'], n):   # outward faces
                    assert np.dot(nn, v[a]) > 0


def test_oracle_scene_b_drops_and_settles(oracle_module, scene_b):
    h = run_oracle(oracle_module, scene_b, 'fp32', 2, 15, seed=3)
    assert np.all(np.isfinite(h['qpos'])) and not np.any(h['error'])
    assert not np.any(h['overflow'] & ~0x600)
    assert np.all(h['ncon'] >= 12) and np.all(h['nefc'] >= 40)
    for j in np.flatnonzero(scene_b.ints['jnt_type'] == 0):
        z = h['qpos'][:, scene_b.ints['jnt_qposadr'][j] + 2]
        assert np.all(z > 0.005) and np.all(z < 0.2)


def test_flop_count_block_sparse_reduces_to_dense():
    """With every row dense (k_r = nv) and one nv-block factored every
    iteration, the block-sparse count equals the dense-equivalent count; with
    narrower rows and reused factors it is smaller."""
    from gpu_libero_b200 import flops
    s = scenes.scene_a()
    nv, W = s.sizes['nv'], 4
    nefc, iters, ls = 50, 3, 5
    base = dict(efc_total=np.full(W, nefc), con_total=np.full(W, 10), newton_rows=np.full(W, iters * nefc),
                ls_rows=np.full(W, ls * nefc), newton_total=np.full(W, iters))
    dense_like = dict(base, efc_k=np.full(W, nefc * nv), efc_k2=np.full(W, nefc * nv * nv),
                      fact_blk=np.full(W, iters * nv * nv * (nv + 6)))
    td = s.ints['tree_dofnum']
    a = flops.substep_flops(s.sizes, td, dense_like, 1)
    b = flops.dense_substep_flops(s.sizes, td, dense_like, 1)
    assert a == pytest.approx(b, rel=1e-12)
    sparse = dict(base, efc_k=np.full(W, nefc * 7), efc_k2=np.full(W, nefc * 49),
                  fact_blk=np.full(W, 7 * 7 * (7 + 6) + 2 * 7 * 7 * 6))
    assert flops.substep_flops(s.sizes, td, sparse, 1) < 0.5 * b


def test_reference_leaf_checker_abi():
    """The checker library built from the reference's own collision leaves (when
    present) agrees with its loader and with the leaves' own argument-pack sizes."""
    import sys
    sys.path.insert(0, str(Path(__file__).resolve().parents[1] / 'oracle'))
    import ref_contacts
    if not ref_contacts.available():
        pytest.skip('oracle/_ref/libref_contacts.so not built')
    ref_contacts.RefCollision()


def test_reference_arm_prints_one_contract_line():
    """`bench.py --impl reference` (the CPU restatement of the reference step)
    prints exactly one JSON line with the bench contract's keys."""
    import json
    import subprocess
    import sys
    root = Path(__file__).resolve().parents[1]
    r = subprocess.run([sys.executable, str(root / 'bench.py'), '--impl', 'reference', '--steps', '1', '--warmup', '0'],
                       capture_output=True, text=True, timeout=600, cwd=str(root))
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [x for x in r.stdout.splitlines() if x.strip()]
    assert len(lines) == 1
    d = json.loads(lines[0])
    for k in ('metric', 'value', 'unit', 'n_gpus', 'steps', 'warmup', 'ms_per_step', 'higher_is_better', 'scaling',
              'dtype', 'config', 'cpu_baseline', 'e2e'):
        assert k in d, k
    assert d['impl'] == 'reference' and d['value'] > 0 and d['higher_is_better'] is True
    assert d['e2e']['h2d_bytes_per_step'] == 0 and d['e2e']['d2h_bytes_per_step'] == 0
    assert d['cpu_baseline']['kind'] == 'port' and d['cpu_baseline']['cores'] >= 1
