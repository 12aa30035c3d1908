"""Per-world model parameter rows on the GPU.

A rows model (native.PackedModel(scene, rows=...)) holds lcm(rows) copies of
the real arrays; world w of a shard reads copy (world_offset + w) % nvariant,
the reference's broadcast rule (cuda/dynamics/mjwarp_constraint_build.cu:18-20).

Checked:
- every world of a rows runtime equals, bit for bit, the same world run by a
  runtime whose model is that world's one row: the kernel selects the row and
  nothing else changes;
- the rows runtime tracks the oracle stepping the same rows model (FP64 1e-9,
  FP32 1e-4 over three control steps; contact and row counts equal);
- a world-offset shard reads the rows of its global worlds.
"""
import numpy as np
import pytest

torch = pytest.importorskip('torch')
pytestmark = pytest.mark.gpu

from gpu_libero_b200 import native  # noqa: E402
from gpu_libero_b200.runtime import Runtime  # noqa: E402

from test_model_rows import one_row, variant_rows  # noqa: E402

STEPS = 3


def run_gpu(scene, rows, q, v, world_offset, precision, steps=STEPS):
    n = q.shape[0]
    rt = Runtime(scene, n, precision=precision, world_offset=world_offset, model_rows=rows)
    rt.set_state(np.concatenate([np.zeros((n, 1)), q, v], axis=1))
    for step in range(steps):
        rt.enqueue_action(scene.actions(n, step, seed=11, world_offset=world_offset))
    torch.cuda.synchronize()
    out = {k: t.cpu().numpy() for k, t in rt.buffers.items()}
    rt.close()
    return out


@pytest.mark.parametrize('precision', ['fp32', 'fp64'])
def test_rows_runtime_equals_one_row_runtimes(precision):
    scene, rows = variant_rows()
    n, offset = 24, 7
    q, v = scene.initial_state(n, seed=11, world_offset=offset)
    out = run_gpu(scene, rows, q, v, offset, precision)
    assert not np.any(out['error']) and not np.any(out['overflow'] & ~0x600)
    for i in range(n):
        g = offset + i
        single = run_gpu(scene, one_row(rows, g), q[i:i + 1], v[i:i + 1], g, precision)
        for k in ('qpos', 'qvel', 'ctrl', 'qacc_warmstart', 'ncon', 'nefc', 'niter'):
            assert np.array_equal(out[k][i], single[k][0]), (i, k)


@pytest.mark.parametrize('precision,tol', [('fp64', 1e-9), ('fp32', 1e-4)])
def test_rows_runtime_tracks_the_oracle(oracle_module, precision, tol):
    scene, rows = variant_rows()
    n, offset = 32, 3
    q, v = scene.initial_state(n, seed=11, world_offset=offset)
    rt = Runtime(scene, n, precision=precision, world_offset=offset, model_rows=rows)
    rt.set_state(np.concatenate([np.zeros((n, 1)), q, v], axis=1))
    torch.cuda.synchronize()
    ref = native.alloc_numpy(rt.packed, n)
    for k, t in rt.buffers.items():
        ref[k][:] = t.cpu().numpy()
    orc = oracle_module.Oracle(precision)
    ms, ds = rt.packed.host_struct(), native.data_struct(ref, n, offset)
    for step in range(STEPS):
        a = scene.actions(n, step, seed=11, world_offset=offset)
        rt.enqueue_action(a)
        ref['action'][:] = a
        orc.step(ms, ds, 0, n, rt.substeps, 1)
    torch.cuda.synchronize()
    gpu = {k: t.cpu().numpy() for k, t in rt.buffers.items()}
    rt.close()
    err = np.max(np.abs(gpu['qpos'] - ref['qpos']))
    print('\n[%s] rows runtime vs oracle, %d worlds x %d control steps: max |qpos| error %.3g'
          % (precision, n, STEPS, err))
    assert err < tol
    assert np.array_equal(gpu['ncon'], ref['ncon']) and np.array_equal(gpu['nefc'], ref['nefc'])
    assert not np.any(gpu['overflow'] & ~0x600) and not np.any(gpu['error'])
