"""The B200 kernel's Newton solve against the reference's own compiled FP32 Newton leaves.

The reference's FP32 engine solves every substep's constraint problem with
its Newton leaves (libero/libero/gpu/cuda/newton/mjwarp_{solver_state,
constraint,hessian,linesearch}.cu), compiled unmodified into
oracle/_ref/libref_newton.so (`make -C oracle ref`).  Its direction leaf needs
NVIDIA MathDx (absent), so the harness (oracle/ref_newton.cu) factors the
Hessian with a plain FP32 Cholesky of its upper triangle in its place; the
loop is the reference's (cuda_fp32/physics.py Newton.solve): initialize,
constraint gradient + Hessian + direction, then line search, gradient +
Hessian + direction and the reference's stop kernel until every world stops.

Problems: scene A (nv = 27, inside the Hessian leaf's padded sizes; scene B's
nv = 81 is outside them), 64 worlds after 6 and 30 control steps, elliptic
and pyramidal cones, FP32.  The B200 forward pass (debug outputs) provides
every input of the solve: the dense rows J, D, aref and their kinds, the
contacts' friction, dimension, distance and margin, the mass matrix, the
smooth acceleration and force, and the warm start.

Checked:
1. the whole solve, reference leaves against the B200 kernel, on the same
   inputs: per-world Newton iterations equal (FP32: the two Cholesky
   factorisations round differently, so a small share of worlds may stop one
   iteration apart), qacc, row forces and qfrc_constraint within 1e-2 of
   max(1, |value|) (two FP32 Newton solves agree to eps32 times the
   Hessian's conditioning, the bound the frozen-substep parity test uses), and
   their medians within 1e-5;
2. the first iteration, reference leaves against this repository's CPU
   oracle on identical inputs (the oracle is what the B200 kernel is checked
   against everywhere else):
   - row states of the constraint projection at the initial jaref equal;
   - the Hessian (M + J'DJ with the elliptic-cone curvature) within 1e-5 of
     each world's largest entry;
   - the exact line search along the first direction: step and improvement
     within 1e-3 relative (the search stops at a slope tolerance, so the step
     is determined to that tolerance and the improvement to its square).
"""
import sys
from pathlib import Path

import numpy as np
import pytest

torch = pytest.importorskip('torch')
pytestmark = pytest.mark.gpu

from gpu_libero_b200 import scene as scenes  # noqa: E402
from gpu_libero_b200.runtime import Runtime  # noqa: E402

FRICTION_DOF, CONTACT = 1, 5  # MuJoCo constraint types (contacts: 5 frictionless, 6 pyramidal, 7 elliptic)


def ref_newton():
    sys.path.insert(0, str(Path(__file__).resolve().parents[1] / 'oracle'))
    import ref_newton as rn
    if not rn.available():
        pytest.skip('oracle/_ref/libref_newton.so not built (needs the reference checkout at build time)')
    return rn.RefNewton()


def frozen_problems(scene, n, steps, seed):
    """The B200 forward pass after `steps` control steps: its Newton inputs
    (debug outputs) and its own solve."""
    rt = Runtime(scene, n, precision='fp32', debug=True)
    q, v = scene.initial_state(n, seed=seed)
    rt.set_state(np.concatenate([np.zeros((n, 1)), q, v], axis=1))
    for k in range(steps):
        rt.enqueue_action(scene.actions(n, k, seed=seed))
    rt.forward()
    torch.cuda.synchronize()
    out = {k: t.cpu().numpy() for k, t in rt.buffers.items()}
    ms = rt.packed.host_struct()
    out['scalars'] = {k: float(getattr(ms, k)) for k in ('tolerance', 'ls_tolerance', 'meaninertia',
                                                         'impratio_invsqrt')}
    out['scalars'].update(iterations=int(ms.iterations), ls_iterations=int(ms.ls_iterations))
    rt.close()
    return out


def batch_of(scene, b):
    """The reference's row layout: rows per world, contacts pooled."""
    s = scene.sizes
    W, nv, R = b['nefc'].shape[0], s['nv'], s['nefc_max']
    nefc, ncon = b['nefc'][:, 0], b['ncon'][:, 0]
    typ, eid = b['efc_type'], b['efc_id']
    loss = np.asarray(scene.reals['dof_frictionloss'], float)
    frictionloss = np.where(typ == FRICTION_DOF, loss[np.clip(eid, 0, nv - 1)], 0.0)
    first = np.concatenate([[0], np.cumsum(ncon)])
    row_contact = np.full((W, R), -1, np.int32)
    address = np.full((int(first[-1]), 6), -1, np.int32)
    for w in range(W):
        for r in range(int(nefc[w])):
            if typ[w, r] >= CONTACT:
                c = int(first[w] + eid[w, r])
                row_contact[w, r] = c
                slot = int(np.sum(address[c] >= 0))
                if slot < 6:
                    address[c, slot] = r
    pooled = lambda k, width: np.concatenate([b[k][w, :width * int(ncon[w])].reshape(-1, width)  # noqa: E731
                                              for w in range(W)])
    batch = dict(nworld=W, nv=nv, rows=R, ncon=int(first[-1]), nefc=nefc, efc_id=eid,
                 nf=np.array([np.sum(typ[w, :nefc[w]] == FRICTION_DOF) for w in range(W)], np.int32),
                 J=b['efc_J'].reshape(W, R, nv), D=b['efc_D'], aref=b['efc_aref'], frictionloss=frictionloss,
                 row_type=typ, row_contact=row_contact, con_world=np.repeat(np.arange(W), ncon),
                 con_dim=pooled('con_dim', 1)[:, 0], con_address=address, con_friction=pooled('con_friction', 5),
                 con_dist=pooled('con_dist', 1)[:, 0], con_margin=pooled('con_margin', 1)[:, 0],
                 M=b['qM'].reshape(W, nv, nv), qacc_smooth=b['qacc_smooth'], qacc_warmstart=b['qacc_warmstart'],
                 qfrc_smooth=b['qfrc_smooth'])
    batch.update(b['scalars'])
    return batch


def oracle_case(batch, w, **extra):
    """World w of the batch in the oracle leaves' case format."""
    n = int(batch['nefc'][w])
    mine = np.flatnonzero(batch['con_world'] == w)
    first = int(mine[0]) if len(mine) else 0
    typ = batch['row_type'][w, :n]
    ids = np.where(typ >= CONTACT, batch['row_contact'][w, :n] - first, batch['efc_id'][w, :n]).astype(np.int32)
    active = batch['con_dist'][mine] - batch['con_margin'][mine] < 0
    adr = np.array([int(batch['con_address'][c, 0]) if batch['con_dim'][c] > 1 and active[k] else -1
                    for k, c in enumerate(mine)], np.int32)
    case = dict(nv=batch['nv'], ne=0, nf=int(batch['nf'][w]), type=typ, id=ids,
                D=batch['D'][w, :n], frictionloss=batch['frictionloss'][w, :n], J=batch['J'][w, :n],
                M=batch['M'][w], impratio=batch['impratio_invsqrt'], con_dim=batch['con_dim'][mine],
                con_friction=batch['con_friction'][mine].reshape(-1, 5), con_adr=adr,
                tolerance=batch['tolerance'], ls_tolerance=batch['ls_tolerance'], meaninertia=batch['meaninertia'],
                ls_iterations=batch['ls_iterations'], qfrc_smooth=batch['qfrc_smooth'][w])
    case.update(extra)
    return case


def rel(a, b):
    a, b = np.asarray(a, float), np.asarray(b, float)
    return np.abs(a - b) / np.maximum(1.0, np.abs(b))


@pytest.fixture(scope='module', params=[('elliptic', 6), ('elliptic', 30), ('pyramidal', 30)],
                ids=['elliptic-6', 'elliptic-30', 'pyramidal-30'])
def solved(request):
    cone, steps = request.param
    scene = scenes.scene_a(cone=cone)
    b = frozen_problems(scene, 64, steps, seed=11)
    batch = batch_of(scene, b)
    assert batch['ncon'] > 0 and np.all(batch['nefc'] > 0)
    return dict(tag=request.param, b=b, batch=batch, ref=ref_newton().solve(batch))


def test_newton_solve_matches_reference_leaves(solved):
    b, ref, batch = solved['b'], solved['ref'], solved['batch']
    W = len(batch['nefc'])
    same = ref['niter'] == b['niter'][:, 0]
    errs = dict(qacc=rel(b['qacc'], ref['qacc']).max(axis=1),
                qfrc_constraint=rel(b['qfrc_constraint'], ref['qfrc_constraint']).max(axis=1),
                force=np.array([rel(b['efc_force'][w, :batch['nefc'][w]], ref['force'][w, :batch['nefc'][w]]).max()
                                for w in range(W)]))
    print('\n[%s] Newton iterations equal in %d/%d worlds (reference %s, B200 %s); worst %s; median %s'
          % (solved['tag'], same.sum(), W, np.bincount(ref['niter']), np.bincount(b['niter'][:, 0]),
             {k: '%.1e' % v.max() for k, v in errs.items()}, {k: '%.1e' % np.median(v) for k, v in errs.items()}))
    assert not np.any(ref['overflow'] & ~0x600)
    assert same.mean() >= 0.9 and np.max(np.abs(ref['niter'] - b['niter'][:, 0])) <= 2
    for k, e in errs.items():
        assert e.max() <= 1e-2 and np.median(e) <= 1e-5, (k, e.max(), np.median(e))


def test_first_iteration_pieces_match_oracle(solved, oracle_module):
    ref, batch = solved['ref'], solved['batch']
    orc = oracle_module.Oracle('fp32')
    W = len(batch['nefc'])
    states = rows = 0
    worst_h = worst_alpha = worst_gain = 0.0
    for w in range(W):
        n = int(batch['nefc'][w])
        rows_out = orc.newton('rows', oracle_case(batch, w, jaref=ref['jaref0'][w, :n]))
        states += int(np.sum(rows_out['state'] == ref['state0'][w, :n]))
        rows += n
        H = orc.newton('hessian', oracle_case(batch, w, jaref=ref['jaref0'][w, :n], state=ref['state0'][w, :n]))['H']
        up = np.triu(ref['H0'][w])
        mine = up + np.triu(up, 1).T
        worst_h = max(worst_h, float(np.max(np.abs(H - mine)) / np.max(np.abs(mine))))
        ls = orc.newton('linesearch', oracle_case(batch, w, jaref=ref['jaref0'][w, :n], qacc=ref['qacc0'][w],
                                                  Ma=ref['Ma0'][w], search=ref['search0'][w]))
        a0, g0 = float(ref['alpha0'][w]), float(ref['improvement0'][w])
        worst_alpha = max(worst_alpha, abs(ls['alpha'] - a0) / max(abs(a0), 1e-30))
        worst_gain = max(worst_gain, abs(ls['improvement'] - g0) / max(abs(g0), 1e-30))
    print('\n[%s] first iteration: row states equal %d/%d; Hessian %.1e of its largest entry; line-search step '
          '%.1e and improvement %.1e relative' % (solved['tag'], states, rows, worst_h, worst_alpha, worst_gain))
    assert states == rows
    assert worst_h <= 1e-5
    assert worst_alpha <= 1e-3 and worst_gain <= 1e-3
