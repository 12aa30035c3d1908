"""World sharding and the observation gather, as two gloo ranks on CPU.

Each rank builds its shard of scene-A worlds from the master seed by global
world index, runs the CPU oracle one control step on it (standing in for the
GPU step), and gathers its observation slab; rank 0 checks the gathered
batch against one process stepping all worlds.  The GPU path uses the same
ObservationGather over NCCL.  With per-world parameter rows, each shard reads
the rows of its global worlds ((world_offset + w) % rows), so the gathered
batch again equals the single process's.
"""
import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]
W = 3        # worlds per rank
NRANK = 2


def free_port():
    with socket.socket() as s:
        s.bind(('127.0.0.1', 0))
        return s.getsockname()[1]


def parameter_rows(scene):
    """Four rows of sliding friction and body masses: shards of 3 worlds start
    mid-cycle, so a shard that ignored its offset would read the wrong rows."""
    f = np.asarray(scene.reals['geom_friction'], np.float64).reshape(-1)
    m = np.asarray(scene.reals['body_mass'], np.float64)
    return {'geom_friction': np.stack([f * k for k in (1.0, 0.5, 0.8, 1.4)]),
            'body_mass': np.stack([m * k for k in (1.0, 1.3, 0.7, 1.1)])}


def step_worlds(scene, n, offset, seed, rows=None):
    """One control step of worlds [offset, offset + n) with the CPU oracle; returns the obs slab."""
    import __graft_entry__ as entry
    from gpu_libero_b200 import native
    packed = native.PackedModel(scene, 'fp64', rows=rows)
    host = native.alloc_numpy(packed, n)
    q, v = scene.initial_state(n, seed=seed, world_offset=offset)
    host['qpos'][:] = q
    host['qvel'][:] = v
    orc = entry.load_oracle().Oracle('fp64')
    ms, ds = packed.host_struct(), native.data_struct(host, n, offset)
    orc.forward(ms, ds, 0, n, 1)
    host['action'][:] = scene.actions(n, 0, seed=seed, world_offset=offset)
    orc.step(ms, ds, 0, n, scene.substeps, 1)
    return host['obs'].copy()


class FakeRuntime:
    def __init__(self, obs):
        self.buffers = {'obs': obs}


def rank_main(rank, port, result_dir, with_rows):
    sys.path.insert(0, str(ROOT))
    import __graft_entry__ as entry
    entry.load_package()
    import torch.distributed as dist
    from gpu_libero_b200 import scene as scenes, shard
    os.environ.update(MASTER_ADDR='127.0.0.1', MASTER_PORT=str(port))
    dist.init_process_group('gloo', rank=rank, world_size=NRANK)
    try:
        s = scenes.scene_a()
        offset = shard.shard_offset(rank, W)
        obs = torch.from_numpy(step_worlds(s, W, offset, seed=7, rows=parameter_rows(s) if with_rows else None))
        g = shard.ObservationGather(FakeRuntime(obs))
        g.launch()
        g.wait()
        np.save(Path(result_dir) / ('rank%d.npy' % rank), g.out.numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize('with_rows', [False, True])
def test_two_rank_shards_gather_to_the_single_process_batch(tmp_path, with_rows):
    from gpu_libero_b200 import scene as scenes
    port = free_port()
    ctx = mp.get_context('spawn')
    procs = [ctx.Process(target=rank_main, args=(r, port, str(tmp_path), with_rows)) for r in range(NRANK)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs)
    s = scenes.scene_a()
    whole = step_worlds(s, NRANK * W, 0, seed=7, rows=parameter_rows(s) if with_rows else None)
    if with_rows:  # the rows act: the plain model gives other observations
        assert not np.array_equal(whole, step_worlds(s, NRANK * W, 0, seed=7))
    for r in range(NRANK):
        got = np.load(tmp_path / ('rank%d.npy' % r))
        assert got.shape == whole.shape
        assert np.array_equal(got, whole)


def test_gather_rejects_a_wrong_buffer():
    from gpu_libero_b200 import shard
    import torch.distributed as dist
    if dist.is_initialized():
        pytest.skip('a process group is already initialized')
    port = free_port()
    dist.init_process_group('gloo', init_method='tcp://127.0.0.1:%d' % port, rank=0, world_size=1)
    try:
        with pytest.raises(ValueError):
            shard.all_gather_into(torch.zeros(5, 4), torch.zeros(3, 4))
        out = torch.zeros(3, 4)
        shard.all_gather_into(out, torch.ones(3, 4))
        assert torch.all(out == 1)
    finally:
        dist.destroy_process_group()
