"""Failure detection on the device without a GPU fault.

Capacity overflows are per-world status bits, as in the reference's FP32
engine (OverflowType, cuda_fp32/constants.py:89-101): the kernel clamps its
counts, sets the world's bit and carries on, and the host raises naming the
failing worlds (cuda_fp32/environment.py:126-140).  These tests make the
contact pool and the row pool too small for scene A's resting boxes, check
that the device's status words equal the CPU oracle's, that the public API
raises, and that the CUDA context stays usable afterwards.
"""
import numpy as np
import pytest

torch = pytest.importorskip('torch')
pytestmark = pytest.mark.gpu

from gpu_libero_b200 import native, scene as scenes  # noqa: E402
from gpu_libero_b200.runtime import B200BatchEnv, Runtime  # noqa: E402

NARROWPHASE, NEFC = 1 << 3, 1 << 0


def forward_status(scene, n, oracle_module):
    rt = Runtime(scene, n)
    q, v = scene.initial_state(n, seed=4)
    rt.set_state(np.concatenate([np.zeros((n, 1)), q, v], axis=1), reset=True)
    torch.cuda.synchronize()
    gpu = {k: t.cpu().numpy() for k, t in rt.buffers.items()}
    host = native.alloc_numpy(rt.packed, n)
    for k, a in gpu.items():
        host[k][:] = a
    host['overflow'][:] = 0
    oracle_module.Oracle('fp32').forward(rt.packed.host_struct(), native.data_struct(host, n), 0, n, 1)
    return rt, gpu, host


@pytest.mark.parametrize('kwargs,bit', [(dict(nconmax=4), NARROWPHASE), (dict(nconmax=32, njmax=12), NEFC)])
def test_capacity_overflow_sets_the_reference_bits(oracle_module, kwargs, bit):
    scene = scenes.scene_a(**kwargs)
    n = 8
    rt, gpu, host = forward_status(scene, n, oracle_module)
    overflow = gpu['overflow'].reshape(-1)
    assert np.all(overflow & bit), overflow
    fatal = ~(0x200 | 0x400)  # iteration and line-search limits are legal exits
    assert np.array_equal(overflow & fatal, host['overflow'].reshape(-1) & fatal)
    assert np.all(gpu['ncon'] <= scene.sizes['ncon_max']) and np.all(gpu['nefc'] <= scene.sizes['nefc_max'])
    with pytest.raises(RuntimeError) as err:
        rt.check()
    assert 'failed_worlds' in str(err.value)


def test_public_api_raises_and_the_context_survives():
    scene = scenes.scene_a(nconmax=4)
    with pytest.raises(RuntimeError) as err:
        B200BatchEnv(scene, 4, seed=2)  # reset() checks the status words
    assert "'failed_worlds': 4" in str(err.value)
    # the per-step status words that B200BatchEnv.step reads carry the bit too
    rt = Runtime(scene, 4)
    q, v = scene.initial_state(4, seed=2)
    rt.set_state(np.concatenate([np.zeros((4, 1)), q, v], axis=1))
    _, status = rt.step_host(scene.actions(4, 0, seed=2))
    assert np.all(status.numpy()[0] & NARROWPHASE)
    rt.close()
    # the device is still healthy: a well-sized engine steps normally
    ok = B200BatchEnv(scenes.scene_a(), 4, seed=2)
    obs, _, _, _ = ok.step(ok.scene.actions(4, 0, seed=2))
    assert np.all(np.isfinite(obs['robot0_joint_pos']))
    ok.close()
