"""Loaders and geometric checks shared by the golden-vector tests.

The fixtures in tests/golden/ hold the reference's own FP64 validation-oracle
outputs (make_golden.py says which file and function produced each); the
checks below restate the reference's contact-geometry predicates
(tools/validation/mjwarp_box_reference.py:60-81 geometry_checks) so that any
implementation's output can be held against the stored reference numbers.
"""
import json
from pathlib import Path

import numpy as np

GOLDEN = Path(__file__).resolve().parent / 'golden'
EPS32 = float(np.finfo(np.float32).eps)


def load(name):
    if name.endswith('.json'):
        return json.loads((GOLDEN / name).read_text())
    return dict(np.load(GOLDEN / name))


def box_cases():
    """Rows of box_pairs.npz as dicts."""
    out = []
    for r in load('box_pairs.npz')['cases']:
        out.append(dict(kind=int(r[0]), p1=r[1:4], R1=r[4:13].reshape(3, 3), s1=r[13:16], p2=r[16:19],
                        R2=r[19:28].reshape(3, 3), s2=r[28:31], budget=r[31], separation=r[32], closest=r[33],
                        inside=bool(r[34]), count=int(r[35])))
    return out


def signed_point_box(point, size):
    delta = np.abs(point) - size
    return np.linalg.norm(np.maximum(delta, 0)) if np.any(delta > 0) else np.max(delta)


def sat_axes(R1, R2):
    axes = [*R1.T, *R2.T]
    axes += [np.cross(a, b) for a in R1.T for b in R2.T if np.dot(np.cross(a, b), np.cross(a, b)) >= 1e-7]
    return np.array([v / np.linalg.norm(v) for v in axes])


def contact_failures(case, dist, pos, normal, budget):
    """Reference contact predicates for one narrowphase output (list of failed names)."""
    bad = []
    kind = case['kind']
    for i, (d, p, n) in enumerate(zip(dist, pos, normal)):
        if d >= 1e9:
            if not (kind == 3 and i == 1 and d == 1e10):
                bad.append('absent capsule component sentinel')
            continue
        if abs(np.linalg.norm(n) - 1) > budget:
            bad.append('unit contact normal')
        if kind in (2, 3):
            radius, axis = case['s1'][0], case['R1'][:, 2]
            half = case['s1'][1] if kind == 3 else 0.0
            centre = p - n * (radius + 0.5 * d)
            off = centre - case['p1']
            t = off @ axis
            if np.linalg.norm(off - t * axis) > budget or abs(t) > half + budget:
                bad.append('sphere centre on capsule centre line')
            local = case['R2'].T @ (centre - case['p2'])
            if abs(signed_point_box(local, case['s2']) - radius - d) > budget:
                bad.append('signed point-box distance minus radius')
            if i == 0 and not case['inside'] and abs(case['closest'] - d) > budget:
                bad.append('first contact attains the segment-box minimum')
        else:
            if abs(np.max(np.abs(sat_axes(case['R1'], case['R2']) @ n)) - 1) > budget:
                bad.append('normal is a SAT direction')
            sep = (n @ (case['p2'] - case['p1']) - np.abs(case['R1'].T @ n) @ case['s1'] -
                   np.abs(case['R2'].T @ n) @ case['s2'])
            if d < sep - budget:
                bad.append('depth bounded by supporting planes')
        for box, sgn in (((1, -1), (2, 1)) if kind == 6 else ((2, 1),)):
            w = p + sgn * 0.5 * d * n
            local = case['R%d' % box].T @ (w - case['p%d' % box])
            delta = np.abs(local) - case['s%d' % box]
            if np.max(delta) > budget or np.min(np.abs(delta)) > budget:
                bad.append('box%d surface witness' % box)
    return bad


def witness_violation(dist, pos, normal, size, pos_b, mat):
    """Largest distance of the two contact witnesses outside their boxes."""
    worst = 0.0
    for box, sgn in ((0, -1), (1, 1)):
        w = pos + sgn * 0.5 * dist[:, None] * normal
        local = (w - pos_b[box]) @ mat[box]
        worst = max(worst, float(np.max(np.abs(local) - size[box])))
    return worst


def unique_points(pos, tol):
    out = []
    for p in pos:
        if not any(np.max(np.abs(p - q)) <= tol for q in out):
            out.append(p)
    return out


def plane_groups(rows, world):
    """Golden plane rows of one world grouped by (g1, g2), id order."""
    out = {}
    for r in rows[rows[:, 0] == world]:
        out.setdefault((int(r[1]), int(r[2])), []).append(r)
    return out


PLANE = dict(must=4, budget=5, dist=6, pos=slice(7, 10), frame=slice(10, 19), dim=19, friction=slice(20, 25),
             solref=slice(25, 27), solimp=slice(27, 32), margin=32)
