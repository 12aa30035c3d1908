"""Per-world model parameter rows, on the CPU.

The reference's leaves read every model parameter through a broadcast row:
world w reads row w % rows (cuda/dynamics/mjwarp_constraint_build.cu:18-20
``parameter(p, w)``; the collision leaves the same, mjwarp_box.cu:182).
native.PackedModel(scene, rows=...) packs lcm(rows) copies of the real arrays
and the kernel and the oracle select copy (world_offset + w) % nvariant.

Checked here: the packing (row selection, layout of the default model,
rejected inputs), scene.parameter_rows, and that the oracle stepping worlds
of a rows model gives, bit for bit, what it gives for each world under a
one-row model holding that world's row.  The GPU kernel is checked the same
way in tests/test_gpu_model_rows.py.
"""
import numpy as np
import pytest

from gpu_libero_b200 import native, scene as scenes


def test_packed_rows_select_row_w_mod_p():
    a = scenes.scene_a()
    base = native.PackedModel(a, 'fp64')
    assert base.nvariant == 1 and base.sizes['nvariant'] == 1
    assert base.variant_stride % 32 == 0 and base.reals.size == base.variant_stride
    f = np.asarray(a.reals['geom_friction'], np.float64).reshape(-1)
    m = np.asarray(a.reals['body_mass'], np.float64)
    rows = {'geom_friction': np.stack([f, 0.5 * f]),
            'body_mass': np.stack([m, 1.1 * m, 1.2 * m]).reshape(3, -1, 1)}  # [P, ...] flattens per row
    p = native.PackedModel(a, 'fp64', rows=rows)
    assert p.nvariant == 6 and p.reals.size == 6 * p.variant_stride
    for w in range(13):
        assert np.array_equal(p.row_values('geom_friction', w), rows['geom_friction'][w % 2])
        assert np.array_equal(p.row_values('body_mass', w), m * (1.0, 1.1, 1.2)[w % 3])
        # arrays without rows keep the scene's values in every copy
        assert np.array_equal(p.row_values('geom_size', w), np.asarray(a.reals['geom_size']).reshape(-1))
    st = p.host_struct()
    assert st.nvariant == 6 and st.variant_stride == p.variant_stride
    # one row of every array is the default model, value for value
    one = native.PackedModel(a, 'fp64', rows={'geom_friction': f[None]})
    assert one.nvariant == 1 and np.array_equal(one.reals, base.reals)


def test_packed_rows_reject_bad_input():
    a = scenes.scene_a()
    f = np.asarray(a.reals['geom_friction']).reshape(-1)
    with pytest.raises(ValueError, match='not a model real array'):
        native.PackedModel(a, rows={'geom_type': np.zeros((2, 14))})
    with pytest.raises(ValueError, match='expected'):
        native.PackedModel(a, rows={'geom_friction': np.zeros((2, f.size + 1))})
    with pytest.raises(ValueError, match='expected'):
        native.PackedModel(a, rows={'geom_friction': np.zeros((0, f.size))})
    with pytest.raises(ValueError, match='non-finite'):
        native.PackedModel(a, rows={'geom_friction': np.stack([f, f * np.nan])})
    with pytest.raises(ValueError, match='model copies'):  # lcm(65537, 65539) copies
        native.PackedModel(a, rows={'geom_friction': np.tile(f, (65537, 1)),
                                    'geom_margin': np.zeros((65539, a.sizes['ngeom']))})


def test_parameter_rows_from_scenes():
    seeds = [scenes.scene_a(seed=s) for s in range(3)]
    rows = scenes.parameter_rows(seeds)
    # box sizes and masses drawn per seed, with their derived arrays
    for name in ('geom_size', 'body_mass', 'body_inertia', 'geom_aabb', 'geom_rbound', 'body_invweight0'):
        assert name in rows and rows[name].shape[0] == 3
    assert 'geom_friction' not in rows and 'jnt_range' not in rows  # equal in every seed
    for k, sc in enumerate(seeds):
        assert np.array_equal(rows['geom_size'][k], np.asarray(sc.reals['geom_size']).reshape(-1))
    with pytest.raises(ValueError, match='sizes'):
        scenes.parameter_rows([scenes.scene_a(), scenes.scene_b()])
    with pytest.raises(ValueError, match='scalar'):
        scenes.parameter_rows([scenes.scene_a(), scenes.scene_a(tolerance=1e-6)])


def variant_rows(nseed=3):
    """Scene A of three seeds: box sizes, masses and inertias differ per row;
    friction and damping rows of other counts on top (lcm 12 copies)."""
    seeds = [scenes.scene_a(seed=s) for s in range(nseed)]
    rows = scenes.parameter_rows(seeds)
    f = np.asarray(seeds[0].reals['geom_friction'], np.float64).reshape(-1)
    d = np.asarray(seeds[0].reals['dof_damping'], np.float64)
    rows['geom_friction'] = np.stack([f, 0.4 * f, 0.7 * f, 1.3 * f])
    rows['dof_damping'] = np.stack([d, 3.0 * d + 0.05])
    return seeds[0], rows


def one_row(rows, world):
    """The single-row table holding what global world `world` reads."""
    return {k: v[[world % v.shape[0]]] for k, v in rows.items()}


def run_oracle(oracle_module, precision, scene, rows, q, v, world_offset, steps):
    n = q.shape[0]
    packed = native.PackedModel(scene, precision, rows=rows)
    host = native.alloc_numpy(packed, n)
    host['qpos'][:] = q
    host['qvel'][:] = v
    orc = oracle_module.Oracle(precision)
    ms, ds = packed.host_struct(), native.data_struct(host, n, world_offset)
    orc.forward(ms, ds, 0, n, 1)
    for step in range(steps):
        host['action'][:] = scene.actions(n, step, seed=11, world_offset=world_offset)
        orc.step(ms, ds, 0, n, scene.substeps, 1)
    return host


@pytest.mark.parametrize('precision', ['fp64', 'fp32'])
def test_oracle_rows_equal_one_row_models(oracle_module, precision):
    scene, rows = variant_rows()
    n, offset = 8, 5  # a shard: global worlds 5..12 read rows (5..12) % P
    q, v = scene.initial_state(n, seed=11, world_offset=offset)
    host = run_oracle(oracle_module, precision, scene, rows, q, v, offset, steps=2)
    assert not np.any(host['error']) and not np.any(host['overflow'] & ~0x600)
    for i in range(n):
        g = offset + i
        single = run_oracle(oracle_module, precision, scene, one_row(rows, g), q[i:i + 1], v[i:i + 1], g, steps=2)
        for k in ('qpos', 'qvel', 'ctrl', 'qacc_warmstart', 'ncon', 'nefc'):
            assert np.array_equal(host[k][i], single[k][0]), (i, k)
    # the rows act: global world 1 reads row 1 of every array (seed 1's boxes,
    # other friction and damping) and parts ways with the scene's own model
    rowed = run_oracle(oracle_module, precision, scene, rows, q[:1], v[:1], 1, steps=2)
    plain = run_oracle(oracle_module, precision, scene, None, q[:1], v[:1], 1, steps=2)
    assert np.max(np.abs(rowed['qpos'] - plain['qpos'])) > 1e-4
