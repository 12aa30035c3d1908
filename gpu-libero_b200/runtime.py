"""Host runtime of the B200 engine: device buffers, CUDA graph, env surface.

`Runtime` mirrors the reference FP32 engine's owner
(libero/libero/gpu/host/backends/cuda_fp32/runtime.py:9-92): ``enqueue_action``,
``forward``, ``prepare_control_graph``, ``count``, ``download_state``,
``close``.  `B200BatchEnv` mirrors the physics-facing part of
``CudaFP32BatchEnv`` / ``GpuBatchEnv`` (cuda_fp32/environment.py:19-333,
host/adapters/environment/batch_env.py:445-583): ``step``, ``reset``,
``set_init_state``, ``get_sim_state``, ``diagnostics``, ``work_snapshot``.

Device memory is owned by PyTorch tensors (plumbing only); every physics
computation runs in libb200phys.so.  There is no CPU fallback: without a CUDA
device or without the built library, construction raises.
"""
from contextlib import contextmanager
from threading import RLock

import numpy as np
import torch

from . import native
from .scene import Scene, scene_a

# legal exits: the Newton iteration and line-search limits, and EPA's pool
# budget (it ends with its best face, as at its iteration limit)
OVERFLOW_LIMITS = 0x200 | 0x400 | 0x20000
# inspection outputs that a step never needs: allocated only for debug runtimes
DEBUG_FIELDS = ('efc_J', 'efc_D', 'efc_aref', 'efc_type', 'efc_id', 'niter_trace', 'ls_trace', 'qM',
                'qfrc_smooth', 'con_friction', 'con_margin', 'con_dim')
# scheduling data of a runtime's CTA slots, not world state: copying world rows
# between runtimes must leave these out (`order` must stay a permutation of
# the runtime's own worlds)
SCHEDULE_FIELDS = ('order', 'work')


def failure_report(overflow, error, limit=16):
    """Fatal per-world status words (the reference raises the same pair,
    cuda_fp32/environment.py:126-140), listing at most `limit` worlds."""
    overflow, error = np.asarray(overflow).reshape(-1), np.asarray(error).reshape(-1)
    bad = np.flatnonzero((overflow & ~OVERFLOW_LIMITS) | error)
    return dict(failed_worlds=int(bad.size), b200_overflow={int(w): int(overflow[w]) for w in bad[:limit]},
                controller_error={int(w): int(error[w]) for w in bad[:limit]})


class Runtime:
    """Owned device buffers plus the control-step graph of one world shard."""

    def __init__(self, scene, num_envs, *, device='cuda:0', precision='fp32', world_offset=0, library=None,
                 debug=False, regroup=True, model_rows=None):
        if not torch.cuda.is_available():
            raise RuntimeError('the b200 physics engine requires a CUDA device')
        self.device = torch.device(device)
        self.scene = scene
        self.n = int(num_envs)
        self.world_offset = int(world_offset)
        self.lib = library or native.Library()
        # model_rows: per-world parameter rows (native.PackedModel); world
        # world_offset + i of the whole batch reads row (world_offset + i) % P
        self.packed = native.PackedModel(scene, precision, rows=model_rows)
        self.dtype = torch.float32 if self.packed.dtype == np.float32 else torch.float64
        with torch.cuda.device(self.device):
            self.model_real = torch.from_numpy(self.packed.reals).to(self.device)
            self.model_ints = torch.from_numpy(self.packed.ints).to(self.device)
            self.model = self.packed.struct(self.model_real.data_ptr(), self.model_ints.data_ptr())
            real, ints = self.packed.data_widths()
            # debug: True for every inspection output, or an iterable of their names
            wanted = set(DEBUG_FIELDS) if debug is True else set(debug or ())
            keep = lambda k: k not in DEBUG_FIELDS or k in wanted  # noqa: E731
            self.buffers = {k: torch.zeros((self.n, w), dtype=self.dtype, device=self.device)
                            for k, w in real.items() if keep(k)}
            self.buffers.update({k: torch.zeros((self.n, w), dtype=torch.int32, device=self.device)
                                 for k, w in ints.items() if keep(k)})
            self.mask = torch.ones(self.n, dtype=torch.int32, device=self.device)
            # worlds-to-CTA grouping of the step kernel: the identity, then (with
            # `regroup`) the worlds sorted by their last control step's work
            self.buffers['order'][:, 0] = torch.arange(self.n, dtype=torch.int32, device=self.device)
        self.regroup = bool(regroup)
        self.data = native.data_struct(self.buffers, self.n, self.world_offset, pointer=lambda t: t.data_ptr())
        smem = self.lib.smem_bytes(self.model)
        if smem == 0:
            raise ValueError('model rejected by libb200phys (sizes outside the admitted domain)')
        self.smem_bytes = smem
        with torch.cuda.device(self.device):
            self.lib.prepare(self.model)
        self.substeps = getattr(scene, 'substeps', 25)
        self.state_epoch = np.zeros(self.n, np.int64)
        self.reset_events = np.zeros(self.n, np.int64)
        self._graph = None
        self._graph_stream = None

    # ---- launches -----------------------------------------------------
    def _stream(self):
        return torch.cuda.current_stream(self.device).cuda_stream

    def launch_step(self, policy=True, substeps=None):
        self.lib.step(self.model, self.data, self.substeps if substeps is None else substeps, int(policy),
                      self._stream())

    def _control_step(self, stream):
        """One control step: the step kernel, then the regrouping of worlds by work."""
        self.lib.step(self.model, self.data, self.substeps, 1, stream)
        if self.regroup:
            self.lib.order(self.model, self.data, stream)

    def forward(self, bootstrap=False, mask=None):
        ptr = mask.data_ptr() if mask is not None else 0
        self.lib.forward(self.model, self.data, int(bootstrap), ptr, self._stream())

    def prepare_control_graph(self):
        """Capture one control step (all substeps in one kernel, then the
        regrouping of worlds) in a CUDA graph."""
        if self._graph is None:
            stream = torch.cuda.Stream(self.device)
            stream.wait_stream(torch.cuda.current_stream(self.device))
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.stream(stream):
                with torch.cuda.graph(graph, stream=stream):
                    self._control_step(stream.cuda_stream)
            torch.cuda.current_stream(self.device).wait_stream(stream)
            self._graph = graph
        return self

    def enqueue_action(self, actions):
        """Copy actions in and replay the control graph (runtime.py:58-77)."""
        a = self.buffers['action']
        if isinstance(actions, torch.Tensor):
            a.copy_(actions.to(a.dtype), non_blocking=True)
        else:
            a.copy_(torch.as_tensor(np.asarray(actions), dtype=a.dtype), non_blocking=True)
        if self._graph is not None:
            self._graph.replay()
        else:
            self._control_step(self._stream())

    def pinned_io(self):
        """Pinned host staging for actions (in) and the observation slab plus
        status words (out); allocated once, reused every step."""
        if getattr(self, '_pinned', None) is None:
            nobs = self.scene.sizes['nobs']
            self._pinned = dict(
                action=torch.zeros((self.n, 7), dtype=self.dtype, pin_memory=True),
                obs=torch.zeros((self.n, nobs), dtype=self.dtype, pin_memory=True),
                status=torch.zeros((3, self.n), dtype=torch.int32, pin_memory=True))
            self._status = torch.zeros((3, self.n), dtype=torch.int32, device=self.device)
        return self._pinned

    def step_host(self, actions):
        """One control step from host actions to host observations.

        H2D copy of the actions (pinned), the control graph, then one D2H copy
        of the observation slab and one of the status words (overflow, error,
        integration count); returns views of the pinned host buffers after the
        stream has drained."""
        io = self.pinned_io()
        host = io['action']
        host.numpy()[:] = actions
        self.buffers['action'].copy_(host, non_blocking=True)
        if self._graph is not None:
            self._graph.replay()
        else:
            self._control_step(self._stream())
        torch.stack([self.buffers['overflow'][:, 0], self.buffers['error'][:, 0],
                     self.buffers['integration_count'][:, 0]], out=self._status)
        io['obs'].copy_(self.buffers['obs'], non_blocking=True)
        io['status'].copy_(self._status, non_blocking=True)
        torch.cuda.current_stream(self.device).synchronize()
        return io['obs'], io['status']

    def h2d_bytes_per_step(self):
        return self.n * 7 * self.buffers['action'].element_size()

    def d2h_bytes_per_step(self):
        return self.buffers['obs'].numel() * self.buffers['obs'].element_size() + 3 * self.n * 4

    def count(self, kind, mask=None):
        """Host counters of reset/epoch events (cuda_fp32 bridges count kinds 2/3)."""
        sel = np.ones(self.n, bool) if mask is None else np.asarray(mask, bool)
        if kind in (2, 3):
            self.state_epoch[sel] += 1
        if kind == 3:
            self.reset_events[sel] += 1

    # ---- state --------------------------------------------------------
    def download_state(self):
        torch.cuda.synchronize(self.device)
        return {k: self.buffers[k].cpu().numpy() for k in ('time', 'qpos', 'qvel', 'qacc', 'qacc_warmstart', 'ctrl')}

    def set_state(self, rows, ids=None, reset=True):
        """rows: [k, 1+nq+nv] (time, qpos, qvel) for worlds `ids`."""
        nq, nv = self.scene.sizes['nq'], self.scene.sizes['nv']
        rows = np.asarray(rows, np.float64)
        ids = np.arange(self.n) if ids is None else np.asarray(ids)
        idx = torch.as_tensor(ids, device=self.device, dtype=torch.long)
        put = lambda name, v: self.buffers[name].index_copy_(0, idx, torch.as_tensor(v, dtype=self.dtype, device=self.device))  # noqa
        put('time', rows[:, :1])
        put('qpos', rows[:, 1:1 + nq])
        put('qvel', rows[:, 1 + nq:1 + nq + nv])
        if reset:
            for name in ('qacc_warmstart', 'ctrl', 'gripper', 'action'):
                self.buffers[name].index_fill_(0, idx, 0)
            for name in ('overflow', 'error'):
                self.buffers[name].index_fill_(0, idx, 0)
        mask = torch.zeros(self.n, dtype=torch.int32, device=self.device)
        mask[idx] = 1
        self.count(3 if reset else 2, mask.cpu().numpy().astype(bool))
        self.forward(bootstrap=reset, mask=mask)

    def check(self):
        torch.cuda.synchronize(self.device)
        overflow = self.buffers['overflow'].cpu().numpy().reshape(-1)
        error = self.buffers['error'].cpu().numpy().reshape(-1)
        fatal = overflow & ~OVERFLOW_LIMITS
        if np.any(fatal) or np.any(error):
            raise RuntimeError(failure_report(overflow, error))
        return overflow, error

    def close(self):
        self._graph = None
        self.buffers.clear()


class B200BatchEnv:
    """Batched environment surface of the B200 engine (physics_engine='b200')."""

    physics_engine = 'b200'

    def __init__(self, scene=None, num_envs=8, *, init_states=None, seed=0, device='cuda:0', precision='fp32',
                 physics_engine='b200', cuda_options=None, world_offset=0, model_rows=None):
        if physics_engine != 'b200':
            raise ValueError('B200BatchEnv serves physics_engine="b200"')
        if type(num_envs) is not int or num_envs < 1:
            raise ValueError('num_envs must be a positive integer')
        options = dict(cuda_options or {})
        if isinstance(scene, Scene):
            self.scene = scene
        else:
            kwargs = {k: options.pop(k) for k in ('nconmax', 'njmax', 'cone') if k in options}
            self.scene = scene_a(**kwargs) if scene in (None, 'scene_a') else scene
        if options:
            raise ValueError('unknown b200 options: ' + str(sorted(options)))
        self.num_envs = num_envs
        self.precision = precision
        self.seed_value = seed
        self.world_offset = world_offset
        self._lock = RLock()
        self.runtime = Runtime(self.scene, num_envs, device=device, precision=precision, world_offset=world_offset,
                               model_rows=model_rows)
        self.nq, self.nv = self.scene.sizes['nq'], self.scene.sizes['nv']
        self._closed = self._failed = False
        self._integrations = np.zeros(num_envs, np.int64)
        self.reset(init_states=init_states)

    # ---- failure quarantine (cuda_fp32/environment.py:126-140, batch_env.py:298-302,376-384)
    def _open(self):
        if self._closed:
            raise RuntimeError('B200 batch environment is closed')
        if self._failed:
            raise RuntimeError('B200 batch execution failed; close and rebuild required')

    @contextmanager
    def _mutation(self):
        """Any failure while device state changes quarantines the batch: its
        worlds may be partly advanced, so later calls raise until rebuilt."""
        try:
            yield
        except BaseException:
            self._failed = True
            raise

    # ---- lifecycle ----------------------------------------------------
    def _initial_rows(self, seed):
        q, v = self.scene.initial_state(self.num_envs, seed=seed, world_offset=self.world_offset)
        return np.concatenate([np.zeros((self.num_envs, 1)), q, v], axis=1)

    def reset(self, init_states=None, ids=None):
        with self._lock:
            self._open()
            rows = self._initial_rows(self.seed_value) if init_states is None else np.asarray(init_states, np.float64)
            if ids is not None and init_states is None:
                rows = rows[np.asarray(ids)]
            with self._mutation():
                self.runtime.set_state(rows, ids=ids, reset=True)
                self.runtime.check()
                self._integrations[:] = self.runtime.buffers['integration_count'][:, 0].cpu().numpy()
            return self.observations()

    def set_init_state(self, init_states, ids=None):
        """Restore [time, qpos, qvel] rows; controller history is kept (README.md:320-325)."""
        with self._lock:
            self._open()
            with self._mutation():
                self.runtime.set_state(init_states, ids=ids, reset=False)
                self.runtime.check()
            return self.observations()

    def get_sim_state(self):
        self._open()
        s = self.runtime.download_state()
        return np.concatenate([s['time'], s['qpos'], s['qvel']], axis=1)

    def step(self, actions):
        """One control step of every world: (obs, reward, done, infos).

        reward and done are the synthetic task's sparse success predicate,
        evaluated on the device.  A fatal status word, or a world that did not
        commit every substep, raises and quarantines the batch."""
        actions = np.asarray(actions)
        with self._lock:
            self._open()
            if actions.shape != (self.num_envs, 7) or not np.all(np.isfinite(actions)):
                raise ValueError('actions must be finite with shape (num_envs, 7)')
            with self._mutation():
                slab, status = self.runtime.step_host(actions)
                status = status.numpy()
                fatal = status[0] & ~OVERFLOW_LIMITS
                if np.any(fatal) or np.any(status[1]):
                    raise RuntimeError(failure_report(status[0], status[1]))
                committed = status[2].astype(np.int64) - self._integrations
                if not np.all(committed == self.runtime.substeps):
                    raise RuntimeError('B200 batch did not commit every requested physics substep')
                self._integrations += committed
            slab = slab.numpy().copy()
            nfree = self.scene.sizes['nfree']
            obs = dict(robot0_joint_pos=slab[:, :9], robot0_joint_vel=slab[:, 9:18], robot0_eef_pos=slab[:, 18:21],
                       robot0_eef_quat=slab[:, 21:25],
                       object_pose=slab[:, 25:25 + 7 * nfree].reshape(self.num_envs, nfree, 7))
            rewards = slab[:, -2].astype(np.float64)
            dones = slab[:, -1] != 0
            return obs, rewards, dones, [{} for _ in range(self.num_envs)]

    def observations(self):
        b = self.runtime.buffers
        torch.cuda.synchronize(self.runtime.device)
        return dict(qpos=b['qpos'].cpu().numpy(), qvel=b['qvel'].cpu().numpy(),
                    eef_pos=b['site_xpos'][:, 3 * self.scene.sizes['ee_site']:3 * self.scene.sizes['ee_site'] + 3]
                    .cpu().numpy())

    def diagnostics(self):
        """Status without raising (a quarantined batch still reports why)."""
        b = self.runtime.buffers
        torch.cuda.synchronize(self.runtime.device)
        overflow = b['overflow'].cpu().numpy().reshape(-1)
        error = b['error'].cpu().numpy().reshape(-1)
        return dict(physics_backend='gpu', physics_engine='b200', precision=self.precision, failed=self._failed,
                    actual_integration_count=b['integration_count'].cpu().numpy().reshape(-1).tolist(),
                    first_error=error.tolist(), substeps=self.runtime.substeps,
                    capacities=dict(nconmax=self.scene.sizes['ncon_max'], njmax=self.scene.sizes['nefc_max']),
                    upstream_status=overflow.tolist())

    def work_snapshot(self):
        b = self.runtime.buffers
        torch.cuda.synchronize(self.runtime.device)
        g = lambda k: b[k].cpu().numpy().reshape(-1).tolist()  # noqa: E731
        return dict(integration_count=g('integration_count'), state_epoch=self.runtime.state_epoch.tolist(),
                    reset_events=self.runtime.reset_events.tolist(), newton_attempts=g('newton_total'),
                    first_error=g('error'), upstream_status=g('overflow'), ncon=g('ncon'), nefc=g('nefc'),
                    newton_iterations=g('niter'), linesearch_evaluations=g('ls_total'))

    def close(self):
        with self._lock:
            if not self._closed:
                self.runtime.close()
                self._closed = True

    def __enter__(self):
        return self

    def __exit__(self, *args):
        self.close()
