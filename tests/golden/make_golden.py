"""Generate the golden vectors in this folder from the reference itself.

Usage: python tests/golden/make_golden.py <reference checkout>

The expected values come from the reference's own independent FP64
validation oracles (tools/validation/mjwarp_*_reference.py) and from its
shipped box-box fixtures (tests/fixtures/boxbox_*); the inputs are scene-A
states from this package's scene compiler.  The oracle of this repository is
run here only to supply contact lists to the constraint-row oracle and to
assert, before anything is written, that it already agrees.  Tests read the
written .npz/.json files only.

Usage (one part only): python tests/golden/make_golden.py <reference checkout> newton

Reference modules used (paths inside the reference checkout):
  tools/validation/mjwarp_kinematics_reference.py   reference(c, 'composed')
  tools/validation/mjwarp_plane_reference.py        reference(c), material()
  tools/validation/mjwarp_constraint_build_reference.py  build_reference(c)
  tools/validation/mjwarp_euler_reference.py        reference(c, 'position')
  tools/validation/mjwarp_box_reference.py          pair_math(), box_separation()
  tests/fixtures/boxbox_task5.json, boxbox_edge_projection.json,
  boxbox_first_face_vertex.csv, boxbox_sat_face_tie.csv, and the unit-box
  cases of tests/cuda/precision_boxbox_test.cu:76-82.
  tests/data/gjk_tuned_direction.json (a recorded LIBERO box-box overlap).
  tools/validation/mjwarp_constraint.py   synthetic(), reference(): FP64 row
      forces and states of the Newton constraint projection (with the
      reference's ambiguity flags and error bounds)
  tools/validation/mjwarp_hessian.py      synthetic_case(), matrix_reference():
      FP64 H = M + J'DJ plus the elliptic-cone curvature (and its majorant)
  tools/validation/mjwarp_linesearch.py   synthetic(), matrix(), objective():
      the FP64 cost along the search ray; its minimiser is found here by
      golden-section search on the reference's objective
"""
import csv
import importlib
import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))


def load_reference(path):
    sys.path.insert(0, str(Path(path) / 'tools'))
    mods = {}
    for name in ('kinematics', 'plane', 'constraint_build', 'euler', 'box'):
        mods[name] = importlib.import_module('validation.mjwarp_%s_reference' % name)
    return mods


def setup():
    import __graft_entry__ as entry
    entry.load_package()
    from gpu_libero_b200 import native, scene
    s = scene.scene_a()
    oracle = entry.load_oracle()
    return s, native, oracle


def quat_mat(q):
    w, x, y, z = q / np.linalg.norm(q)
    return np.array([[w * w + x * x - y * y - z * z, 2 * (x * y - w * z), 2 * (x * z + w * y)],
                     [2 * (x * y + w * z), w * w - x * x + y * y - z * z, 2 * (y * z - w * x)],
                     [2 * (x * z - w * y), 2 * (y * z + w * x), w * w - x * x - y * y + z * z]])


# ------------------------------------------------------------------ states
def scene_states(s, count, seed):
    """Scene-A states with boxes tilted into/near the floor, some arm joints
    pushed past their limits and random velocities (limit, friction and
    contact rows all active)."""
    rng = np.random.default_rng(seed)
    q, v = s.initial_state(count, seed=seed)
    ints, reals = s.ints, s.reals
    for w in range(count):
        for j in np.flatnonzero(ints['jnt_type'] == 0):
            a = ints['jnt_qposadr'][j]
            axis = rng.normal(size=3)
            axis /= np.linalg.norm(axis)
            ang = rng.uniform(0.0, 0.15)
            dq = np.r_[np.cos(ang / 2), np.sin(ang / 2) * axis]
            q0 = q[w, a + 3:a + 7]
            qn = np.array([dq[0] * q0[0] - dq[1:] @ q0[1:], *(dq[0] * q0[1:] + q0[0] * dq[1:] + np.cross(dq[1:], q0[1:]))])
            q[w, a + 3:a + 7] = qn / np.linalg.norm(qn)
            q[w, a + 2] += rng.uniform(-0.004, 0.003)
        for j in rng.choice(ints['limited_jnt'], size=2, replace=False):
            lo, hi = reals['jnt_range'][j]
            q[w, ints['jnt_qposadr'][j]] = lo - rng.uniform(0.001, 0.01) if rng.random() < 0.5 else hi + rng.uniform(0.001, 0.01)
        v[w] = rng.normal(0.0, 0.3, v.shape[1])
    return q, v


# ------------------------------------------------------------------ kinematics
def kinematics_case(ref, s, qpos, static):
    I, Rl = s.ints, s.reals
    nb, nj, ng, ns = (s.sizes[k] for k in ('nbody', 'njnt', 'ngeom', 'nsite'))
    xquat = np.zeros((2, nb, 4))
    xquat[:, :, 0] = 1
    c = dict(nbody=nb, njnt=nj, ngeom=ng, nsite=ns, xpos=np.zeros((2, nb, 3)), xquat=xquat,
             xanchor=np.zeros((2, nj, 3)), xaxis=np.zeros((2, nj, 3)), body_jntadr=I['body_jntadr'],
             body_jntnum=I['body_jntnum'], parent=I['body_parentid'], joint_type=I['jnt_type'],
             qposadr=I['jnt_qposadr'], jnt_axis=Rl['jnt_axis'][None], jnt_pos=Rl['jnt_pos'][None],
             mocap=np.full(nb, -1), body_pos=Rl['body_pos'][None], body_quat=Rl['body_quat'][None],
             qpos0=Rl['qpos0'][None], qpos=qpos, xipos=np.zeros((2, nb, 3)), ximat=np.zeros((2, nb, 3, 3)),
             geom_xpos=np.repeat(static['geom_xpos'][None], 2, 0), geom_xmat=np.repeat(static['geom_xmat'][None], 2, 0),
             site_xpos=np.zeros((2, ns, 3)), site_xmat=np.zeros((2, ns, 3, 3)), geom_body=I['geom_bodyid'],
             site_body=I['site_bodyid'], weld=I['body_weldid'], root=I['body_rootid'],
             body_ipos=Rl['body_ipos'][None], body_iquat=Rl['body_iquat'][None], geom_pos=Rl['geom_pos'][None],
             geom_quat=Rl['geom_quat'][None], site_pos=Rl['site_pos'][None], site_quat=Rl['site_quat'][None])
    return ref.reference(c, 'composed')


def make_kinematics(mods, s, native, oracle):
    packed = native.PackedModel(s, 'fp64')
    ms = packed.host_struct()
    orc = oracle.Oracle('fp64')
    q0, _ = s.initial_state(1, seed=0)
    base = orc.positions(ms, s.sizes, q0[0])
    static = dict(geom_xpos=base['geom_xpos'], geom_xmat=base['geom_xmat'].reshape(-1, 3, 3))
    qs, _ = scene_states(s, 6, seed=101)
    keys = ('xpos', 'xquat', 'xmat', 'xipos', 'geom_xpos', 'geom_xmat', 'site_xpos', 'site_xmat')
    out = {k: [] for k in keys}
    err = {k: [] for k in keys}
    for p in range(3):
        values, errors = kinematics_case(mods['kinematics'], s, qs[2 * p:2 * p + 2], static)
        for k in keys:
            out[k].append(values[k].reshape(2, -1))
            err[k].append(np.asarray(errors[k], float).reshape(2, -1))
    data = dict(qpos=qs)
    for k in keys:
        data[k] = np.concatenate(out[k])
        data[k + '_err'] = np.concatenate(err[k])
    for w in range(6):  # the oracle must already agree before anything is written
        got = orc.positions(ms, s.sizes, qs[w])
        for k in ('xpos', 'xquat', 'xipos', 'geom_xpos', 'geom_xmat'):
            assert np.allclose(got[k].reshape(-1), data[k][w], atol=1e-12), k
    np.savez_compressed(HERE / 'kinematics_scene_a.npz', **data)
    return data


# ------------------------------------------------------------------ plane contacts
def geom_params(s):
    R = s.reals
    ng = s.sizes['ngeom']
    return dict(size=R['geom_size'][None], margin=R['geom_margin'][None], gap=R['geom_gap'][None],
                solmix=R['geom_solmix'][None], friction=R['geom_friction'][None], adhesion=np.zeros((1, ng)),
                solref=R['geom_solref'][None], solimp=R['geom_solimp'][None], priority=s.ints['geom_priority'],
                condim=s.ints['geom_condim'], geom_type=s.ints['geom_type'], ngeom=ng,
                geom_dataid=np.full((1, ng), -1), mesh_vert=np.zeros((0, 3)))


def make_plane(mods, s, native, oracle, kin):
    ref = mods['plane']
    qs, vs = scene_states(s, 8, seed=202)
    pairs = s.ints['pair_geom'].reshape(-1, 2)
    plane_pairs = [tuple(p) for p in pairs if s.ints['geom_type'][p[0]] == 0]
    packed = native.PackedModel(s, 'fp64')
    ms = packed.host_struct()
    orc = oracle.Oracle('fp64')
    rows = []
    for p in range(4):
        gx = np.zeros((2, s.sizes['ngeom'], 3))
        gm = np.zeros((2, s.sizes['ngeom'], 3, 3))
        for w in range(2):
            pos = orc.positions(ms, s.sizes, qs[2 * p + w])
            gx[w], gm[w] = pos['geom_xpos'], pos['geom_xmat'].reshape(-1, 3, 3)
        cand = np.array([(w, g1, g2) for w in range(2) for g1, g2 in plane_pairs])
        c = dict(geom_params(s), capacity=len(cand), candidate_count=[len(cand)], initial_count=[0],
                 candidate_geom=cand[:, 1:], candidate_world=cand[:, 0], candidate_ids=np.full((len(cand), 2), -1),
                 xpos=gx, xmat=gm, columns=4)
        res = ref.reference(c)
        for (w, g1, g2, cid), (row, budget, uncertain) in sorted(res['rows'].items()):
            key = (w, g1, g2, cid)
            if key not in res['possible']:
                continue
            rows.append([2 * p + w, g1, g2, cid, key in res['must'], budget, row['dist'], *row['pos'],
                         *np.asarray(row['frame']).ravel(), row['dim'], *row['friction'], *row['solref'],
                         *row['solimp'], row['includemargin']])
    rows = np.array(rows, float)
    np.savez_compressed(HERE / 'plane_contacts_scene_a.npz', qpos=qs, qvel=vs, rows=rows,
                        columns=np.array('world g1 g2 id must budget dist pos3 frame9 dim friction5 solref2 '
                                         'solimp5 includemargin'))
    # agreement of this repository's oracle before writing
    for w in range(8):
        con = orc.contacts(ms, s.sizes, qs[w], vs[w])
        mine = [(int(a), int(b)) for a, b in con['geom'] if s.ints['geom_type'][a] == 0]
        must = rows[(rows[:, 0] == w) & (rows[:, 4] == 1)]
        assert len(mine) >= len(must)
    return qs, vs


# ------------------------------------------------------------------ constraint rows
def make_rows(mods, s, native, oracle, qs, vs):
    ref_c, ref_p = mods['constraint_build'], mods['plane']
    I, Rl = s.ints, s.reals
    nv, nb, nj = s.sizes['nv'], s.sizes['nbody'], s.sizes['njnt']
    packed = native.PackedModel(s, 'fp64')
    ms = packed.host_struct()
    orc = oracle.Oracle('fp64')
    ancestor = np.zeros((nb, nv), bool)
    for b in range(nb):
        chain, x = set(), b
        while x > 0:
            chain.add(x)
            x = I['body_parentid'][x]
        for d in range(nv):
            ancestor[b, d] = I['dof_bodyid'][d] in chain
    gp = geom_params(s)
    out_rows, out_con = [], []
    for p in range(4):
        ws = (2 * p, 2 * p + 1)
        cons = [orc.contacts(ms, s.sizes, qs[w], vs[w]) for w in ws]
        kin = [orc.positions(ms, s.sizes, qs[w]) for w in ws]
        geom, world, dist, pos, frame, dim, fr, sref, simp, sfr, margin = [], [], [], [], [], [], [], [], [], [], []
        for k, con in enumerate(cons):
            for i in range(con['ncon']):
                g1, g2 = map(int, con['geom'][i])
                mat = ref_p.material(dict(gp, geom_type=I['geom_type']), 0, g1, g2, -1)
                geom.append((g1, g2)); world.append(k); dist.append(con['dist'][i]); pos.append(con['pos'][i])
                frame.append(con['frame'][i]); dim.append(mat['dim']); fr.append(mat['friction'])
                sref.append(mat['solref']); simp.append(mat['solimp']); sfr.append(mat['solreffriction'])
                margin.append(mat['margin'])
                out_con.append([ws[k], g1, g2, con['dist'][i], *con['pos'][i], *np.ravel(con['frame'][i])])
        n = len(geom)
        c = dict(disable_constraint=False, disable_friction=False, disable_limit=False, disable_contact=False,
                 disable_refsafe=False, adhesion_enabled=False, dof_friction=Rl['dof_frictionloss'][None],
                 padded_nv=nv, nv=nv, dof_weight=Rl['dof_invweight0'][None], dof_ref=Rl['dof_solref'][None],
                 dof_imp=Rl['dof_solimp'][None], qvel=vs[list(ws)], limited_joint=I['limited_jnt'],
                 joint_range=Rl['jnt_range'][None], qpos=qs[list(ws)], joint_qpos=I['jnt_qposadr'],
                 joint_margin=Rl['jnt_margin'][None], joint_dof=I['jnt_dofadr'], joint_ref=Rl['jnt_solref'][None],
                 joint_imp=Rl['jnt_solimp'][None], timestep=np.array([s.scalars['timestep']]), naconmax=n,
                 contact_count=[n], contact_type=np.ones(n, int), contact_dist=np.array(dist),
                 contact_margin=np.array(margin), contact_adhesion=np.zeros(n), contact_world=np.array(world),
                 contact_dim=np.array(dim), contact_geom=np.array(geom).reshape(n, 2), geom_body=I['geom_bodyid'],
                 body_weight=Rl['body_invweight0'][None], impratio_invsqrt=np.array([s.scalars['impratio_invsqrt']]),
                 contact_friction=np.array(fr).reshape(n, 5), contact_ref=np.array(sref).reshape(n, 2),
                 contact_imp=np.array(simp).reshape(n, 5), contact_ref_friction=np.array(sfr).reshape(n, 2),
                 cone=1, contact_pos=np.array(pos).reshape(n, 3), contact_frame=np.array(frame).reshape(n, 3, 3),
                 ancestor=ancestor, cdof=np.stack([k_['cdof'] for k_ in kin]),
                 subtree_com=np.stack([k_['com'] for k_ in kin]), root=I['body_rootid'])
        rows, counts, contacts = ref_c.build_reference(c)
        first = np.cumsum([0] + [cons[0]['ncon']])[-1]
        for k in range(2):
            for (kind, ident, comp), r in sorted(rows[k].items()):
                local = ident - (first if k == 1 and kind == 7 else 0) if kind == 7 else ident
                J, Je = r['J']
                out_rows.append([ws[k], kind, local, comp, r['D'][0], r['D'][1], r['aref'][0], r['aref'][1],
                                 r['pos'][0], *J, *Je])
    out_rows = np.array(out_rows, float)
    np.savez_compressed(HERE / 'constraint_rows_scene_a.npz', qpos=qs, qvel=vs, rows=out_rows,
                        contacts=np.array(out_con, float),
                        columns=np.array('world kind id component D D_err aref aref_err pos J[nv] J_err[nv]'))
    for w in range(8):  # agreement before writing
        con = orc.contacts(ms, s.sizes, qs[w], vs[w])
        mine = out_rows[out_rows[:, 0] == w]
        assert con['nefc'] == len(mine), (w, con['nefc'], len(mine))
        assert np.allclose(con['D'], mine[:, 4], rtol=1e-9)
        assert np.allclose(con['aref'], mine[:, 6], rtol=1e-9, atol=1e-9)
        assert np.allclose(con['J'], mine[:, 9:9 + nv], atol=1e-12)


# ------------------------------------------------------------------ Euler position phase
def make_euler(mods, s, native, oracle):
    I = s.ints
    qs, vs = scene_states(s, 6, seed=303)
    vs *= 10.0
    out, err = [], []
    for p in range(3):
        c = dict(nv=s.sizes['nv'], timestep=np.array([s.scalars['timestep']]), damping=np.zeros((1, s.sizes['nv'])),
                 dampingpoly=np.zeros((1, s.sizes['nv'], 2)), matrix=np.zeros((2, 1)), row=np.zeros(1, int),
                 nnz=np.ones(1, int), acceleration=np.zeros((2, s.sizes['nv'])), qvel=vs[2 * p:2 * p + 2],
                 qpos=qs[2 * p:2 * p + 2], joint_type=I['jnt_type'], qposadr=I['jnt_qposadr'], dofadr=I['jnt_dofadr'])
        values, errors = mods['euler'].reference(c, 'position')
        out.append(values['qpos'])
        err.append(errors['qpos'])
    data = dict(qpos=qs, qvel=vs, qpos_next=np.concatenate(out), qpos_next_err=np.concatenate(err),
                timestep=s.scalars['timestep'])
    orc = oracle.Oracle('fp64')
    ms = native.PackedModel(s, 'fp64').host_struct()
    for w in range(6):
        assert np.allclose(orc.integrate(ms, qs[w], vs[w], s.scalars['timestep']), data['qpos_next'][w], atol=1e-12)
    np.savez_compressed(HERE / 'euler_position_scene_a.npz', **data)


# ------------------------------------------------------------------ box pairs
def make_box_pairs(mods, oracle):
    ref = mods['box']
    rng = np.random.default_rng(404)
    cases = []
    orc = oracle.Oracle('fp64')
    kinds = (2, 3, 6)
    while len(cases) < 240:
        kind = kinds[len(cases) % 3]
        s1 = rng.uniform(0.02, 0.06, 3)
        s2 = rng.uniform(0.02, 0.06, 3)
        if kind == 2:
            s1[1:] = 0
        elif kind == 3:
            s1[2] = 0
        R1, R2 = quat_mat(rng.normal(size=4)), quat_mat(rng.normal(size=4))
        p1 = np.zeros(3)
        reach = (s1[0] + (s1[1] if kind == 3 else 0)) if kind != 6 else np.linalg.norm(s1)
        direction = rng.normal(size=3)
        direction /= np.linalg.norm(direction)
        p2 = direction * rng.uniform(0.5, 1.05) * (reach + np.linalg.norm(s2))
        c = dict(xpos=np.array([[p1, p2]]), xmat=np.array([[R1, R2]]), size=np.array([[s1, s2]]),
                 geom_type=np.array([kind, 6]))
        info = ref.pair_math(c, 0, 0, 1)
        dist, pos, normal = orc.box(kind, p1, R1, s1, p2, R2, s2, 0.0)
        frame = [np.vstack([n, np.zeros((2, 3))]) for n in normal]
        for i in range(len(dist)):  # the reference's own geometric checks on the oracle output
            for chk in ref.geometry_checks(info, dist[i], pos[i], frame[i], i):
                assert chk['passed'], (kind, chk['name'])
        sep = info.get('separation', np.nan)
        closest = info.get('closest', np.nan)
        inside = info.get('inside', False)
        cases.append(np.r_[kind, p1, R1.ravel(), s1, p2, R2.ravel(), s2, info['budget'], sep, closest, inside,
                           len(dist)])
    np.savez_compressed(HERE / 'box_pairs.npz', cases=np.array(cases),
                        columns=np.array('kind p1[3] R1[9] s1[3] p2[3] R2[9] s2[3] budget separation closest '
                                         'inside count'))


def make_box_fixtures(mods, path):
    F = Path(path) / 'tests' / 'fixtures'
    out = {}
    task5 = json.loads((F / 'boxbox_task5.json').read_text())
    out['task5'] = dict(size=task5['size'], pos=task5['pos'], mat=task5['mat'], count=4, min_dist=-2e-7,
                        physical_overlap=task5['physical_overlap'],
                        note='tests/test_native_box_contacts.py:147-160: four contacts, no lateral '
                             'negative depth, box-2 witness on the book')
    # rotations / swaps / scales of the captured pose (test_native_box_contacts.py:162-181)
    rng = np.random.RandomState(13)
    rotated = []
    for scale in (1e-3, 1., 1e3):
        for swap in (False, True):
            for _ in range(6):
                quat = rng.normal(size=4)
                quat /= np.linalg.norm(quat)
                m = quat_mat(quat)
                size = np.asarray(task5['size']) * scale
                pos = np.asarray(task5['pos']) @ m.T * scale
                mat = m @ np.asarray(task5['mat'])
                if swap:
                    size, pos, mat = size[::-1], pos[::-1], mat[::-1]
                rotated.append(dict(size=size.tolist(), pos=pos.tolist(), mat=mat.tolist(), scale=scale))
    out['task5_rotated'] = rotated
    edge = json.loads((F / 'boxbox_edge_projection.json').read_text())
    out['edge_projection'] = dict(size=edge['size'], pos=edge['pos'], mat=edge['mat'],
                                  note='witnesses on both box surfaces (test_native_box_contacts.py:208-216)')
    rows = [[float(x) for x in r] for r in csv.reader((F / 'boxbox_first_face_vertex.csv').open())]
    out['first_face_vertex'] = dict(size=np.reshape(rows[0], (2, 3)).tolist(), pos=np.reshape(rows[1], (2, 3)).tolist(),
                                    mat=np.reshape(rows[2], (2, 3, 3)).tolist(), count=4,
                                    tolerance=16 * float(np.finfo(np.float32).eps),
                                    note='four contacts inside both boxes (test_native_box_contacts.py:193-206)')
    flat = [float(x) for r in csv.reader((F / 'boxbox_sat_face_tie.csv').open()) for x in r]
    size = np.reshape(flat[0:6], (2, 3))
    for label, off in (('fp32', 6), ('fp64', 30)):
        pos, mat = np.reshape(flat[off:off + 6], (2, 3)), np.reshape(flat[off + 6:off + 24], (2, 3, 3))
        sep = mods['box'].box_separation(pos[0], pos[1], mat[0], mat[1], size[0], size[1])
        out['sat_face_tie_' + label] = dict(size=size.tolist(), pos=pos.tolist(), mat=mat.tolist(), count=4,
                                            separation=sep, native_tie_depth=flat[54],
                                            note='tests/cuda/precision_boxbox_test.cu:63-75: four unique '
                                                 'contacts at the face/edge SAT tie, at scales 1e-3, 1, 1e3')
    out['unit_boxes'] = dict(cases=[[0, 0, 1.9, 4], [0, 0, 2, 4], [2, 0, 2, 2], [2, 2, 2, 1], [0, 0, 2.2, 0]],
                             note='tests/cuda/precision_boxbox_test.cu:76-82: unique contact counts of two unit '
                                  'boxes, second centre at (x, y, z)')
    (HERE / 'box_fixtures.json').write_text(json.dumps(out, indent=1))


def make_gjk_direction(mods, path):
    """The reference's recorded zero-margin box-box overlap (libero_spatial task 5,
    tests/data/gjk_tuned_direction.json, used by tests/test_mjwarp_convex_gjk.py:42-52)
    whose previously tuned GJK direction wrongly claimed separation; the expected
    depth is the reference's independent SAT separation of the two boxes."""
    f = json.loads((Path(path) / 'tests' / 'data' / 'gjk_tuned_direction.json').read_text())
    a, b = np.asarray(f['position1'], float), np.asarray(f['position2'], float)
    rot, size = np.asarray(f['rotations'], float), np.asarray(f['sizes'], float)
    sep = float(mods['box'].box_separation(a, b, rot[0], rot[1], size[0], size[1]))
    assert sep < -f['tolerance']
    out = dict(pos=[a.tolist(), b.tolist()], mat=rot.tolist(), size=size.tolist(), separation=sep,
               tolerance=f['tolerance'], iterations=f['iterations'], epa_iterations=f['epa_iterations'],
               provenance=f['provenance'],
               note='penetrating boxes a tuned GJK direction once declared separated; '
                    'the convex path must report the SAT depth')
    (HERE / 'gjk_tuned_direction.json').write_text(json.dumps(out, indent=1))


# ------------------------------------------------------------------ Newton pieces
NEWTON_NV = (9, 27, 39, 57)


def world_contacts(type_row, id_row, nefc, dims, friction, address, active=None):
    """One world's contacts, renumbered 0.. in order of first use by its rows:
    (row ids remapped, dims, frictions, first-row addresses or -1)."""
    used = []
    for r in range(nefc):
        if type_row[r] == 7 and int(id_row[r]) not in used:
            used.append(int(id_row[r]))
    remap = {c: i for i, c in enumerate(used)}
    ids = np.array([remap.get(int(i), int(i)) if type_row[r] == 7 else int(i) for r, i in enumerate(id_row[:nefc])],
                   np.int32)
    dim = np.array([int(dims[c]) for c in used], np.int32)
    fr = np.array([friction[c] for c in used], np.float64).reshape(-1, 5)
    adr = np.array([int(address[c][0]) if np.all(np.asarray(address[c][:dims[c]]) >= 0) and
                    (active is None or active[c]) else -1 for c in used], np.int32)
    return ids, dim, fr, adr


def golden_section(f, hi):
    """Minimiser of a convex function of alpha on [0, hi] (after widening hi
    until f rises), to the limit of FP64."""
    lo, f_hi = 0.0, f(hi)
    while f_hi < f(0.0) and hi < 1e12:
        hi *= 2
        f_hi = f(hi)
    g = (np.sqrt(5) - 1) / 2
    a, b = lo, hi
    c, d = b - g * (b - a), a + g * (b - a)
    fc, fd = f(c), f(d)
    for _ in range(200):
        if fc < fd:
            b, d, fd = d, c, fc
            c = b - g * (b - a)
            fc = f(c)
        else:
            a, c, fc = c, d, fd
            d = a + g * (b - a)
            fd = f(d)
    return 0.5 * (a + b)


def make_newton(path):
    sys.path.insert(0, str(Path(path) / 'tools'))
    sys.path.insert(0, str(path))
    C = importlib.import_module('validation.mjwarp_constraint')
    H = importlib.import_module('validation.mjwarp_hessian')
    L = importlib.import_module('validation.mjwarp_linesearch')
    out, counts = {}, dict(rows=0, hessian=0, linesearch=0)

    def put(kind, fields):
        i = counts[kind]
        counts[kind] += 1
        for k, v in fields.items():
            out['%s%d_%s' % (kind, i, k)] = np.asarray(v)

    # row forces and states
    cases = [C.synthetic(nv) for nv in NEWTON_NV]
    cases += [C.synthetic(39, v) for v in ('world1-done', 'empty-world0', 'top-boundary', 'bottom-boundary',
                                           'zero-tangent', 'friction-boundary', 'broadcast-impratio')]
    for case in cases:
        a = case['arrays']
        force, state, ambiguous, held, bound = C.reference(a)
        nv = int(a['nv'])
        for w in range(2):
            n = int(a['nefc'][w])
            if a['done'][w] or n == 0:
                continue
            ids, dim, fr, adr = world_contacts(a['type'][w], a['id'][w], n, a['contact_dim'], a['contact_friction'],
                                               a['contact_efc_address'])
            put('rows', dict(nv=nv, ne=a['ne'][w], nf=a['nf'][w], type=a['type'][w, :n], id=ids, D=a['D'][w, :n],
                             frictionloss=a['frictionloss'][w, :n], jaref=a['jaref'][w, :n],
                             J=a['J'][w, :n, :nv], impratio=a['impratio'][w % a['impratio'].size],
                             con_dim=dim, con_friction=fr, con_adr=adr, force=force[w, :n], state=state[w, :n],
                             compare=~(ambiguous[w, :n] | held[w, :n]), bound=bound[w, :n]))
    # Hessian
    cases = [H.synthetic_case(nv) for nv in NEWTON_NV] + [H.synthetic_case(39, variant=v) for v in ('zero-friction',)]
    for case in cases:
        a, nv = case['arrays'], case['nv']
        result, magnitude, _ = H.matrix_reference(case)
        active = a['contact_distance'] - a['contact_margin'] < 0
        for w in range(2):
            n = int(a['nefc'][w])
            if a['done'][w]:
                continue
            M = np.zeros((nv, nv))
            for e, (r, c) in enumerate(zip(a['mass_row'], a['mass_column'])):
                M[r, c] = M[c, r] = a['mass'][w, e]
            mine = [c for c in range(min(int(a['contact_count'][0]), a['contact_world'].size))
                    if a['contact_world'][c] == w]
            typ = np.full(n, 3, np.int32)
            rid = np.zeros(n, np.int32)
            for k, c in enumerate(mine):
                ids = a['contact_address'][c, :a['contact_dimension'][c]]
                for r in ids[ids >= 0]:
                    if r < n:
                        typ[r], rid[r] = 7, k
            adr = np.array([int(a['contact_address'][c, 0]) if a['contact_dimension'][c] > 1 and active[c] and
                            np.all(a['contact_address'][c, :a['contact_dimension'][c]] >= 0) else -1 for c in mine],
                           np.int32)
            up = np.triu(result[w, :nv, :nv])
            mag = np.triu(magnitude[w, :nv, :nv])
            put('hessian', dict(nv=nv, type=typ, id=rid, D=a['diagonal'][w, :n], jaref=a['jaref'][w, :n],
                                J=a['jacobian'][w, :n, :nv], state=a['state'][w, :n], M=M,
                                impratio=a['impratio'][w % a['impratio'].size],
                                con_dim=np.array([a['contact_dimension'][c] for c in mine], np.int32),
                                con_friction=np.array([a['contact_friction'][c] for c in mine]).reshape(-1, 5),
                                con_adr=adr, H=up + np.triu(up, 1).T, magnitude=mag + np.triu(mag, 1).T))
    # line search
    cases = [L.synthetic(nv) for nv in NEWTON_NV]
    cases += [L.synthetic(39, v) for v in ('top-boundary', 'bottom-boundary', 'zero-tangent', 'friction-boundary',
                                           'small-search')]
    for case in cases:
        a = case['arrays']
        nv = int(a['nv'])
        mass = L.matrix(a)
        jv = np.einsum('wri,wi->wr', a['J'][:, :, :nv].astype(np.float64), a['search'].astype(np.float64))
        for w in range(2):
            n = int(a['nefc'][w])
            if a['done'][w] or not np.any(a['search'][w]):
                continue
            f = lambda alpha: L.objective(a, w, alpha, mass, jv)  # noqa: E731
            best = golden_section(f, 1.0)
            h = 1e-4 * max(best, 1e-3)
            curv = (f(best + h) - 2 * f(best) + f(best - h)) / (h * h)
            ids, dim, fr, adr = world_contacts(a['type'][w], a['id'][w], n, a['contact_dim'], a['contact_friction'],
                                               a['contact_efc_address'])
            put('linesearch', dict(nv=nv, ne=a['ne'][w], nf=a['nf'][w], type=a['type'][w, :n], id=ids,
                                   D=a['D'][w, :n], frictionloss=a['frictionloss'][w, :n], jaref=a['Jaref'][w, :n],
                                   J=a['J'][w, :n, :nv], M=mass[w], qacc=a['qacc'][w], Ma=a['Ma'][w],
                                   qfrc_smooth=a['qfrc_smooth'][w], search=a['search'][w],
                                   impratio=a['impratio_invsqrt'][w % a['impratio_invsqrt'].size],
                                   tolerance=a['tolerance'][0], ls_tolerance=a['ls_tolerance'][0],
                                   meaninertia=a['inertia'][0], ls_iterations=int(a['ls_iterations']),
                                   con_dim=dim, con_friction=fr, con_adr=adr, alpha_min=best, cost0=f(0.0),
                                   cost_min=f(best), curvature=curv))
    out.update({'count_' + k: np.array(v) for k, v in counts.items()})
    np.savez_compressed(HERE / 'newton_pieces.npz', **out)
    print('newton pieces:', counts)


def main():
    if len(sys.argv) == 3 and sys.argv[2] == 'newton':
        make_newton(sys.argv[1])
        return
    if len(sys.argv) != 2:
        raise SystemExit(__doc__)
    mods = load_reference(sys.argv[1])
    s, native, oracle = setup()
    kin = make_kinematics(mods, s, native, oracle)
    qs, vs = make_plane(mods, s, native, oracle, kin)
    make_rows(mods, s, native, oracle, qs, vs)
    make_euler(mods, s, native, oracle)
    make_box_pairs(mods, oracle)
    make_box_fixtures(mods, sys.argv[1])
    make_gjk_direction(mods, sys.argv[1])
    make_newton(sys.argv[1])
    print('golden vectors written to', HERE)


if __name__ == '__main__':
    main()
