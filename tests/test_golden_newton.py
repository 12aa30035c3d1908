"""The oracle's Newton pieces pinned against the reference's own FP64 restatements.

Fixture tests/golden/newton_pieces.npz, written by make_golden.py (`newton`)
from the reference's validation oracles on their own synthetic boundaries
(several dof counts, condim 3/4/6 contacts, friction-loss rows at and
around their switching radius, cone top/bottom boundaries, zero tangents):
  rows        tools/validation/mjwarp_constraint.py reference(): row forces
              and states of the constraint projection (CPU MuJoCo
              mj_constraintUpdate zones), with the reference's ambiguity
              flags near switching surfaces and its FP32 error bound
  hessian     tools/validation/mjwarp_hessian.py matrix_reference():
              H = M + J'DJ over quadratic rows plus the elliptic-cone
              curvature, with its absolute majorant
  linesearch  tools/validation/mjwarp_linesearch.py objective(): the cost
              along the search ray; the fixture holds its minimiser (golden-
              section search in FP64), the costs at 0 and at the minimiser, and
              the curvature there

Tolerances:
  rows        states equal and forces within the reference's bound (FP32);
              FP64 forces within 1e-12 of the value's scale (same formula on
              the same FP32 inputs), both where the reference marks a row
              unambiguous
  hessian     within 64 eps x the reference's majorant (eps of the precision)
  linesearch  the exact line search stops once |slope| < max(gtol, noise),
              gtol = max(tol ls_tol |search| meaninertia nv, 1e-6) and noise =
              8 FLT_EPSILON times the slope's scale (the reference's
              NoiseEps; the scale is at most 4 curvature |alpha*| on these
              rays); so |alpha - alpha*| <= 2 max(gtol, noise) / curvature
              (plus rounding); the reported improvement equals cost(0) -
              cost(alpha*) within the reference's own energy bound for its
              CUDA line search (64 eps32 (nv + rows + 32) x the cost and ray
              magnitudes, mjwarp_linesearch.py Replay.check): on these
              synthetic rows the friction rows' D are random, so the cone
              shift identity the line search's cost model uses holds only to
              that bound
The CUDA kernel's Newton solve is compared with this oracle at every
substep in the GPU parity tests (iteration and line-search counts equal).
"""
import numpy as np
import pytest

from golden_checks import load

PRECISIONS = ('fp64', 'fp32')


@pytest.fixture(scope='module')
def pieces():
    return load('newton_pieces.npz')


def cases(g, kind):
    for i in range(int(g['count_' + kind])):
        pre = '%s%d_' % (kind, i)
        yield i, {k[len(pre):]: v for k, v in g.items() if k.startswith(pre)}


@pytest.mark.parametrize('precision', PRECISIONS)
def test_row_forces_and_states(oracle_module, pieces, precision):
    orc = oracle_module.Oracle(precision)
    checked = kinds = 0
    seen = set()
    for i, c in cases(pieces, 'rows'):
        out = orc.newton('rows', c)
        cmp = c['compare'].astype(bool)
        assert np.array_equal(out['state'][cmp], c['state'][cmp]), i
        err = np.abs(out['force'] - c['force'])[cmp]
        if precision == 'fp64':
            scale = np.maximum(1.0, np.abs(c['force'][cmp]))
            assert np.all(err <= 1e-12 * scale), (i, float(np.max(err / scale, initial=0)))
        else:
            assert np.all(err <= c['bound'][cmp]), i
        checked += int(cmp.sum())
        seen |= set(int(s) for s in c['state'][cmp])
        kinds += 1
    assert kinds >= 15 and checked >= 500
    assert seen == {0, 1, 2, 3, 4}  # satisfied, quadratic, both linear friction zones, cone


@pytest.mark.parametrize('precision', PRECISIONS)
def test_hessian_with_cone_curvature(oracle_module, pieces, precision):
    orc = oracle_module.Oracle(precision)
    eps = np.finfo(np.float64 if precision == 'fp64' else np.float32).eps
    cones = 0
    for i, c in cases(pieces, 'hessian'):
        H = orc.newton('hessian', c)['H']
        assert np.all(np.abs(H - c['H']) <= 64 * eps * c['magnitude'] + 1e-300), i
        cones += int(np.sum(c['con_adr'] >= 0))
    assert cones >= 10


@pytest.mark.parametrize('precision', PRECISIONS)
def test_exact_line_search_minimises_the_reference_cost(oracle_module, pieces, precision):
    orc = oracle_module.Oracle(precision)
    eps = np.finfo(np.float64 if precision == 'fp64' else np.float32).eps
    n = 0
    for i, c in cases(pieces, 'linesearch'):
        out = orc.newton('linesearch', c)
        nv, search = int(c['nv']), np.asarray(c['search'], float)
        gtol = max(float(c['tolerance']) * float(c['ls_tolerance']) * np.linalg.norm(search) *
                   float(c['meaninertia']) * nv, 1e-6)
        curv, best = float(c['curvature']), float(c['alpha_min'])
        assert curv > 0, i
        slack = 64 * eps * (abs(best) + 1) * (1 if precision == 'fp64' else 1e3)
        noise = 8 * np.finfo(np.float32).eps * 4 * curv * abs(best)
        da = abs(out['alpha'] - best)
        assert da <= 2 * max(gtol, noise) / curv + slack, (i, out['alpha'], best)
        gain = float(c['cost0'] - c['cost_min'])
        Ma, qs, M = (np.asarray(c[k], float) for k in ('Ma', 'qfrc_smooth', 'M'))
        ray = abs(best) * float(np.abs(search) @ (np.abs(Ma) + np.abs(qs)))
        ray += 0.5 * best * best * float(np.abs(search) @ np.abs(M) @ np.abs(search))
        eps32 = np.finfo(np.float32).eps
        energy = 64 * eps32 * (nv + len(c['type']) + 32) * max(abs(float(c['cost0'])) + abs(float(c['cost_min'])) +
                                                               ray, 1e-30)
        assert abs(out['improvement'] - gain) <= energy + 0.5 * curv * (da + slack) ** 2, (i, out['improvement'], gain)
        # the accepted step moves qacc, Ma and jaref along the ray by alpha
        q0 = np.asarray(c['qacc'], float)
        assert np.all(np.abs(out['qacc'] - (q0 + out['alpha'] * search)) <=
                      4 * eps * (np.abs(q0) + abs(out['alpha']) * np.abs(search)) + 1e-300)
        n += 1
    assert n >= 15
