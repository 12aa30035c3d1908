"""Benchmark of the B200 physics step: env control steps/s for the whole box.

One "step" is one control step (25 physics substeps, OSC policy step first)
of every world on every GPU.  The default workload is BASELINE scene B
(scene A's arm plus 12 dropped objects, 16384 worlds per GPU), the
configuration the metric is quoted on; --scene scene_a runs the smaller scene.  Worlds shard by contiguous range, one process
per GPU (torchrun), no data-path collective; each rank derives its worlds'
seeds from the master seed by global world index.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--worlds PER_GPU]
  python bench.py --impl reference ...   # the reference's CPU path (C port)

Timing: CUDA events on the launching stream around each control-step graph
replay, L2 flushed (a 256 MiB write) between timed steps, barrier +
synchronize on both sides, max over ranks.  `e2e` times the public API
(B200BatchEnv.step: pinned H2D actions, control step, D2H observations).
"""
import argparse
import json
import os
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))
import __graft_entry__ as entry  # noqa: E402

METRIC = 'env control steps/sec (whole box) at 16K worlds/GPU; physics substeps/sec'
UNIT = 'env control steps/s'
# DRAM read + write bytes per world and control step (FP32), from one ncu
# capture of control_step per scene (dram__bytes_read.sum + dram__bytes_write.sum
# of one launch divided by its worlds; per-world state is independent, so the
# traffic scales with the worlds of a launch): scene A captured at 1184 worlds,
# scene B at 444 worlds (one wave each), after 25 warm-up control steps
TRAFFIC_BYTES_PER_WORLD = {'scene_a': 1247, 'scene_b': 11377}
# control-step stages the kernel stamps with clock64 (data.stage_cycles slots 1..15);
# in worlds of several warps the FP64 OSC runs on the first warp beside collision
# on the others, and 'osc_collision' holds that overlapped stage ('collision' is
# then 0); likewise the rows' allocation beside actuation ('actuation_constraints',
# with 'constraints' 0); one-warp worlds run each pair in turn
STAGES = ('kinematics', 'com_crb', 'mass_factor', 'collision', 'constraints', 'velocity', 'osc_collision',
          'actuation_constraints',
          'newton_init', 'linesearch', 'gradient', 'hessian', 'direction', 'euler', 'barrier_wait')
WORKLOADS = {
    'scene_a': 'scene_a: Franka-like arm + gripper + plane + 3 free boxes, elliptic cones, 25 substeps/control step',
    'scene_b': 'scene_b: scene A arm + 12 dropped objects (4 boxes, 4 capsules, 2 spheres, 2 convex hulls), '
               'elliptic cones, 25 substeps/control step',
}


def parse():
    p = argparse.ArgumentParser()
    p.add_argument('--gpus', type=int, default=1)
    p.add_argument('--steps', type=int, default=30)
    p.add_argument('--warmup', type=int, default=5)
    p.add_argument('--worlds', type=int, default=16384, help='worlds per GPU')
    p.add_argument('--scene', default='scene_b', choices=('scene_a', 'scene_b'),
                   help='scene_b (16384 worlds/GPU) is the configuration the metric is quoted on')
    p.add_argument('--precision', default='fp32')
    p.add_argument('--impl', default='b200', choices=('b200', 'reference'))
    p.add_argument('--seed', type=int, default=0)
    p.add_argument('--no-cpu-baseline', action='store_true')
    p.add_argument('--no-gather', action='store_true', help='skip the per-step observation all-gather (N > 1)')
    p.add_argument('--model-rows', type=int, default=0,
                   help='per-world parameter rows: K seeded rows of body masses (x U[0.8, 1.2]) and geom sliding '
                        'frictions (x U[0.5, 1.5]); world w runs row w %% K (0: one shared model)')
    return p.parse_args()


# ---------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi clock/throttle sampling during the timed region."""
    QUERY = ('index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,'
             'clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,'
             'clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap')

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(['nvidia-smi', '-i', str(self.index), '--query-gpu=' + self.QUERY,
                                          '--format=csv,noheader,nounits', '-lms', '200'],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except (OSError, ValueError):
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, mx, reasons = [], 0.0, set()
        names = ('hw_slowdown', 'hw_thermal_slowdown', 'sw_thermal_slowdown', 'sw_power_cap')
        for line in self.lines:
            f = [x.strip() for x in line.split(',')]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = max(mx, float(f[2]))
            except ValueError:
                continue
            for name, flag in zip(names, f[5:9]):
                if flag.lower() == 'active':
                    reasons.add(name)
        if not sm:
            return None
        return dict(sm_mhz=float(np.median(sm)), sm_max_mhz=mx, reasons=sorted(reasons), samples=len(sm))


# ---------------------------------------------------------------- CPU path
def cpu_run(scene, worlds, steps, warmup, seed, threads, precision='fp64', rows=None):
    """The reference's CPU path restated (C oracle port), threads over worlds.
    FP64 by default: the reference's own CPU path is FP64 CPU MuJoCo."""
    from gpu_libero_b200 import native
    Oracle = entry.load_oracle().Oracle
    packed = native.PackedModel(scene, precision, rows=rows)
    host = native.alloc_numpy(packed, worlds)
    q, v = scene.initial_state(worlds, seed=seed)
    host['qpos'][:] = q
    host['qvel'][:] = v
    ms, ds = packed.host_struct(), native.data_struct(host, worlds)
    orc = Oracle(precision)
    orc.forward(ms, ds, 0, worlds, 1)
    times = []
    for k in range(warmup + steps):
        host['action'][:] = scene.actions(worlds, k, seed=seed)
        t0 = time.perf_counter()
        orc.step_parallel(ms, ds, worlds, scene.substeps, 1, threads)
        if k >= warmup:
            times.append(time.perf_counter() - t0)
    return float(np.sum(times))


def host_threads():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def physical_cores():
    """Physical cores of the host (hardware threads share a core), or None."""
    try:
        import psutil
        return psutil.cpu_count(logical=False)
    except ImportError:
        pass
    try:
        cores, phys, core = set(), None, None
        for line in Path('/proc/cpuinfo').read_text().splitlines():
            if line.startswith('physical id'):
                phys = line.split(':')[1].strip()
            elif line.startswith('core id'):
                core = line.split(':')[1].strip()
                cores.add((phys, core))
        return len(cores) or None
    except OSError:
        return None


CPU_NOTE = ('the reference CPU path, CPU MuJoCo 2.3.7 FP64, is not installed here, so the FP64 C restatement '
            'of the reference substep (oracle/) runs instead, one world per host thread at a time')


def cpu_baseline(scene, seed, rows=None, budget_s=12.0):
    threads = host_threads()
    worlds = 4 * threads
    probe = cpu_run(scene, worlds, 1, 0, seed, threads, rows=rows)
    steps = int(max(1, min(40, budget_s / max(probe, 1e-3))))
    secs = cpu_run(scene, worlds, steps, 0, seed, threads, rows=rows)
    return dict(value=worlds * steps / secs, unit=UNIT, cores=threads, physical_cores=physical_cores(), kind='port',
                precision='f64',
                sample='%d worlds x %d control steps (25 substeps) of %s on %d host threads; %s'
                       % (worlds, steps, scene.name, threads, CPU_NOTE))


def reference_arm(args, scene):
    rank = int(os.environ.get('RANK', '0'))
    if rank != 0:
        return
    threads = host_threads()
    worlds = 4 * threads
    secs = cpu_run(scene, worlds, args.steps, args.warmup, args.seed, threads,
                   rows=model_rows(scene, args.model_rows, args.seed))
    value = worlds * args.steps / secs
    sample = '%d worlds per control step on %d host threads (%s physical cores); %s' % (
        worlds, threads, physical_cores(), CPU_NOTE)
    line = dict(metric=METRIC, value=value, unit=UNIT, impl='reference', n_gpus=args.gpus, steps=args.steps,
                warmup=args.warmup, ms_per_step=1e3 * secs / args.steps, higher_is_better=True, scaling='weak',
                vs_baseline=None, dtype='f64', data='synthetic (seeded %s states and actions)' % scene.name,
                # the workload is the GPU arm's; each step of this arm is a bounded host sample of it
                config=dict(workload=WORKLOADS[scene.name], worlds_per_gpu=args.worlds, substeps=scene.substeps,
                            host_sample_worlds=worlds, host_threads=threads, model_rows=args.model_rows or None),
                substeps_per_sec=value * scene.substeps,
                cpu_baseline=dict(value=value, unit=UNIT, cores=threads, physical_cores=physical_cores(),
                                  kind='port', precision='f64', sample=sample),
                e2e=dict(value=value, unit=UNIT, h2d_bytes_per_step=0, d2h_bytes_per_step=0))
    print(json.dumps(line), flush=True)


def model_rows(scene, k, seed):
    """K seeded per-world parameter rows (mass and friction randomisation), or None."""
    if k <= 0:
        return None
    rng = np.random.default_rng([seed, 0x5EED])
    mass = np.asarray(scene.reals['body_mass'], np.float64)
    friction = np.asarray(scene.reals['geom_friction'], np.float64).reshape(-1, 3)
    rows_mass = mass[None] * rng.uniform(0.8, 1.2, (k, mass.size))
    rows_friction = np.repeat(friction[None], k, axis=0)
    rows_friction[:, :, 0] *= rng.uniform(0.5, 1.5, (k, friction.shape[0]))
    return {'body_mass': rows_mass, 'geom_friction': rows_friction.reshape(k, -1)}


# ---------------------------------------------------------------- GPU path
def main():
    args = parse()
    entry.load_package()
    from gpu_libero_b200 import scene as scenes
    builders = {'scene_a': scenes.scene_a, 'scene_b': scenes.scene_b}
    if args.scene not in builders:
        raise SystemExit('unknown scene ' + args.scene)
    scene = builders[args.scene]()
    if args.impl == 'reference':
        return reference_arm(args, scene)

    import torch
    import torch.distributed as dist
    from gpu_libero_b200 import flops, native
    from gpu_libero_b200.runtime import Runtime, B200BatchEnv

    world_size = int(os.environ.get('WORLD_SIZE', '1'))
    rank = int(os.environ.get('RANK', '0'))
    local = int(os.environ.get('LOCAL_RANK', '0'))
    # stdout carries exactly one JSON line: whatever the libraries print on file
    # descriptor 1 (NCCL's version banner, for one) is sent to stderr, and the
    # result is written to a duplicate of the original stdout
    sys.stdout.flush()
    result_out = os.fdopen(os.dup(1), 'w')
    os.dup2(2, 1)
    torch.cuda.set_device(local)
    dev = torch.device('cuda', local)
    if world_size > 1:
        from datetime import timedelta
        dist.init_process_group('nccl', device_id=dev, timeout=timedelta(seconds=120))
    W = args.worlds
    offset = rank * W
    rows = model_rows(scene, args.model_rows, args.seed)
    rt = Runtime(scene, W, device=dev, precision=args.precision, world_offset=offset, model_rows=rows)
    q, v = scene.initial_state(W, seed=args.seed, world_offset=offset)
    rt.set_state(np.concatenate([np.zeros((W, 1)), q, v], axis=1))
    rt.check()
    rt.prepare_control_graph()
    total = args.warmup + args.steps
    acts = torch.stack([torch.as_tensor(scene.actions(W, k, seed=args.seed, world_offset=offset), dtype=rt.dtype)
                        for k in range(total)]).to(dev)
    flush = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device=dev)  # 256 MiB > 126 MB L2
    stream = torch.cuda.current_stream(dev)
    gather = None
    if world_size > 1 and not args.no_gather:
        from gpu_libero_b200.shard import ObservationGather
        gather = ObservationGather(rt)  # every rank's obs slab to rank 0, overlapped with the next step
    for k in range(args.warmup):
        rt.buffers['action'].copy_(acts[k])
        rt._graph.replay()
        if gather:
            gather.launch()
    if gather:
        gather.wait()
    torch.cuda.synchronize(dev)
    counters0 = {k: rt.buffers[k].clone() for k in ('efc_total', 'con_total', 'newton_rows', 'ls_rows',
                                                     'newton_total', 'efc_k', 'efc_k2', 'fact_blk', 'stage_cycles')}
    events = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    clocks = ClockSampler(local)
    if world_size > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    clocks.start()
    time.sleep(0.3)
    for i in range(args.steps):
        k = args.warmup + i
        flush.fill_(float(i))
        rt.buffers['action'].copy_(acts[k])
        events[i][0].record(stream)
        rt._graph.replay()
        if gather:
            gather.launch()
        events[i][1].record(stream)
    if gather:
        gather.wait()
        events[-1][1].record(stream)  # the last gather ends inside the timed region
    torch.cuda.synchronize(dev)
    clock = clocks.stop()
    if world_size > 1:
        dist.barrier()
    step_ms = np.array([a.elapsed_time(b) for a, b in events])
    elapsed = float(step_ms.sum()) / 1e3
    t = torch.tensor([elapsed], dtype=torch.float64, device=dev)
    if world_size > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    elapsed_max = float(t.item())
    rt.check()
    # int32 device counters; the difference is taken modulo 2^32 so that a counter
    # that wraps during the interval still gives its delta
    deltas = {k: (rt.buffers[k].long() - counters0[k].long()).remainder(1 << 32).cpu().numpy()
              for k in counters0}
    # wall cycles of each stage per world and substep (lane 0 of each world stamps clock64;
    # barrier_wait is the time a world waits at CTA barriers for the other worlds of its CTA)
    stage = deltas.pop('stage_cycles').astype(np.float64).mean(0)[1:] / (args.steps * scene.substeps)
    stage_cycles = {name: round(float(c)) for name, c in zip(STAGES, stage)}
    fl = flops.substep_flops(scene.sizes, scene.ints['tree_dofnum'], deltas, scene.substeps)
    fl_dense = flops.dense_substep_flops(scene.sizes, scene.ints['tree_dofnum'], deltas, scene.substeps)
    # one control-step kernel per graph replay (the regrouping kernel after it
    # sorts 16K ints in a few microseconds)
    kernel_s = elapsed / args.steps
    sm_count = torch.cuda.get_device_properties(dev).multi_processor_count
    sm_mhz = clock['sm_mhz'] if clock else 1965.0
    fp64 = args.precision == 'fp64'
    peak = (flops.fp64_peak_tflops if fp64 else flops.fp32_peak_tflops)(sm_count, sm_mhz)
    achieved = fl / args.steps / kernel_s / 1e12
    achieved_dense = fl_dense / args.steps / kernel_s / 1e12
    real_b = rt.buffers['qpos'].element_size()
    io_real = sum(scene.sizes[k] for k in ('nq',)) * 2 + scene.sizes['nv'] * 4 + scene.sizes['nu'] * 2 + 2 * (3 + 9 + 2) + 7 + 2
    out_real = (scene.sizes['nbody'] * 16 + scene.sizes['ngeom'] * 12 + scene.sizes['nsite'] * 12 +
                scene.sizes['nbody'] * 3 + 5 * scene.sizes['nv'] + scene.sizes['nobs'])
    bytes_per_world = (io_real + out_real) * real_b
    hbm_gbs = None
    try:
        peaks = json.loads((ROOT / 'MEASURED_PEAKS.json').read_text())
        hbm_gbs, peak_src = float(peaks['hbm_gbs']), 'measured'
    except (OSError, ValueError, KeyError):
        hbm_gbs, peak_src = 6650.0, 'fallback'
    traffic = TRAFFIC_BYTES_PER_WORLD[args.scene] * W if args.precision == 'fp32' else None

    # e2e through the public API (pinned H2D actions, D2H observations)
    env = B200BatchEnv(scene, W, device=dev, precision=args.precision, seed=args.seed, world_offset=offset,
                       model_rows=rows)
    env.runtime.prepare_control_graph()
    host_actions = [scene.actions(W, k, seed=args.seed, world_offset=offset) for k in range(total)]
    for k in range(args.warmup):
        env.step(host_actions[k])
    if world_size > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(args.steps):
        env.step(host_actions[args.warmup + i])
    e1.record(stream)
    torch.cuda.synchronize(dev)
    e2e_s = e0.elapsed_time(e1) / 1e3
    t = torch.tensor([e2e_s], dtype=torch.float64, device=dev)
    if world_size > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    e2e_max = float(t.item())

    base = None
    if rank == 0 and world_size == 1 and not args.no_cpu_baseline:
        base = cpu_baseline(scene, args.seed, rows)
    if rank == 0:
        value = world_size * W * args.steps / elapsed_max
        line = dict(
            metric=METRIC, value=value, unit=UNIT, n_gpus=world_size, steps=args.steps, warmup=args.warmup,
            ms_per_step=1e3 * elapsed_max / args.steps, higher_is_better=True, scaling='weak', vs_baseline=None,
            dtype='f32' if args.precision == 'fp32' else 'f64', data='synthetic (seeded %s states and actions)' % scene.name,
            config=dict(workload=WORKLOADS[scene.name],
                        worlds_per_gpu=W, total_worlds=W * world_size, substeps=scene.substeps,
                        parallelism='world shards, one process per GPU', l2='flushed (256 MiB write) between steps',
                        model_rows=args.model_rows or None,
                        obs_gather=('NCCL all-gather of the [W, %d] observation slab every step, side stream, '
                                    '%d bytes per step' % (scene.sizes['nobs'], gather.bytes_per_launch())
                                    if gather else None)),
            substeps_per_sec=value * scene.substeps,
            e2e=dict(value=world_size * W * args.steps / e2e_max, unit=UNIT,
                     h2d_bytes_per_step=env.runtime.h2d_bytes_per_step(),
                     d2h_bytes_per_step=env.runtime.d2h_bytes_per_step()),
            roofline=dict(bound='fp64' if fp64 else 'fp32', achieved=achieved, peak=peak, unit='TFLOP/s',
                          frac=achieved / peak, traffic=traffic,
                          peak_source='nominal %s CUDA-core issue: %d SMs x %d lanes x 2 x %.0f MHz (sampled)'
                          % ('FP64' if fp64 else 'FP32', sm_count, 64 if fp64 else 128, sm_mhz),
                          flops_per_world_substep=fl / (W * args.steps * scene.substeps),
                          counting='block-sparse: k_r = dofs of the trees a row touches, Newton blocks = islands, island factor counted where executed'),
            roofline_dense=dict(achieved=achieved_dense, peak=peak, unit='TFLOP/s', frac=achieved_dense / peak,
                                flops_per_world_substep=fl_dense / (W * args.steps * scene.substeps),
                                counting='dense-equivalent: k_r = nv, one nv x nv Newton block'),
            roofline_hbm=dict(bound='hbm', achieved=bytes_per_world * W / kernel_s / 1e9, peak=hbm_gbs, unit='GB/s',
                              frac=bytes_per_world * W / kernel_s / 1e9 / hbm_gbs, peak_source=peak_src,
                              bytes_per_world=bytes_per_world, traffic=traffic),
            kernel_ms=dict(mean=float(step_ms.mean()), min=float(step_ms.min()), max=float(step_ms.max())),
            stage_cycles_per_world_substep=stage_cycles,
            cpu_baseline=base, clocks=clock,
            # per step: the control-step kernel and the world-regrouping kernel
            gpu_launches=args.steps * (2 if rt.regroup else 1))
        print(json.dumps(line), file=result_out, flush=True)
    env.close()
    rt.close()
    if world_size > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == '__main__':
    main()
