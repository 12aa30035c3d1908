"""Algorithmic FLOP count of the physics substep from device work counters.

Unit of work: one physics substep of one world.  One FMA = 2 FLOPs; k_r is
the number of structural nonzero dofs of constraint row r (the dofs of the at
most two kinematic trees the row touches); b runs over the Newton Hessian's
island blocks:

  F_substep = 120 nbody (FK) + 60 ngeom (frames) + 250 nbody (CoM/CRB) + 12 nM (M)
            + 2 * sum_t (n_t^3/3 + 2 n_t^2)             mass factor/solve (smooth + Euler)
            + 30 npair + 200 ncon                         broadphase + narrowphase
            + sum_r 12 k_r + 40 nefc                      constraint rows
            + 300 nbody + F_OSC                           RNE/passive, FP64 OSC (reported apart)
            + I [sum_r 2 k_r^2 + 4 k_r + 30]              Newton: block-sparse J'DJ, gradient
            + sum_iterations sum_b (b^3/3 [if factored] + 2 b^2)   Newton: island factor, solve
            + L (sum_r 2 k_r + 30 nefc) + 2 nM            line search

The island factor is counted only where the kernel factors; an iteration
whose constraint states are unchanged reuses the previous factor and is
counted with its solve alone.

Per-world device counters, accumulated over the measured interval: sum nefc,
sum ncon, sum k_r and sum k_r^2 (per substep), sum I*nefc, sum L*nefc, sum I,
and 3x the executed island work (b^3 + 6 b^2 factored, 6 b^2 reused).  The
iteration row sums use the interval's mean k_r and k_r^2 per row.

`dense_substep_flops` is the dense-equivalent count (k_r = nv, one nv x nv
factor every iteration), the formulation of the reference's dense Hessian.
"""
import numpy as np

F_OSC_FP64 = 8.0e3


def _tot(counters, k):
    return float(np.sum(np.asarray(counters[k], np.float64)))


def _n_substeps(counters, substeps):
    return len(np.asarray(counters['efc_total']).reshape(-1)) * substeps


def _fixed(sizes, tree_dofnum):
    nb, ng, nM, npair = (sizes[k] for k in ('nbody', 'ngeom', 'nM', 'npair'))
    trees = np.asarray(tree_dofnum, float)
    return (120 * nb + 60 * ng + 250 * nb + 12 * nM + 2 * np.sum(trees ** 3 / 3 + 2 * trees ** 2) +
            30 * npair + 300 * nb + 2 * nM)


def substep_flops(sizes, tree_dofnum, counters, substeps):
    """Block-sparse FP32 FLOPs (excluding the FP64 OSC) summed over all worlds
    and substeps.  counters: per-world arrays (deltas over the interval) for
    efc_total, con_total, newton_rows, ls_rows, newton_total, efc_k, efc_k2,
    fact_blk."""
    nefc = _tot(counters, 'efc_total')
    k1, k2 = _tot(counters, 'efc_k'), _tot(counters, 'efc_k2')
    mean_k = k1 / nefc if nefc else 0.0
    mean_k2 = k2 / nefc if nefc else 0.0
    rows = 12 * k1 + 40 * nefc + 200 * _tot(counters, 'con_total')
    newton = _tot(counters, 'newton_rows') * (2 * mean_k2 + 4 * mean_k + 30) + _tot(counters, 'fact_blk') / 3.0
    search = _tot(counters, 'ls_rows') * (2 * mean_k + 30)
    return _fixed(sizes, tree_dofnum) * _n_substeps(counters, substeps) + rows + newton + search


def dense_substep_flops(sizes, tree_dofnum, counters, substeps):
    """The dense-equivalent count: k_r = nv and one nv x nv factor per Newton
    iteration."""
    nv = sizes['nv']
    rows = _tot(counters, 'efc_total') * (12 * nv + 40) + _tot(counters, 'con_total') * 200
    newton = (_tot(counters, 'newton_rows') * (2 * nv * nv + 4 * nv + 30) +
              _tot(counters, 'newton_total') * (nv ** 3 / 3 + 2 * nv * nv))
    search = _tot(counters, 'ls_rows') * (2 * nv + 30)
    return _fixed(sizes, tree_dofnum) * _n_substeps(counters, substeps) + rows + newton + search


def osc_flops(worlds, substeps):
    return F_OSC_FP64 * worlds * substeps


def fp32_peak_tflops(sm_count, sm_mhz):
    """Nominal FP32 CUDA-core peak: 128 FP32 lanes per SM, 2 FLOPs per FMA."""
    return sm_count * 128 * 2 * sm_mhz * 1e6 / 1e12


def fp64_peak_tflops(sm_count, sm_mhz):
    """Nominal FP64 CUDA-core peak: 64 FP64 lanes per SM, 2 FLOPs per FMA."""
    return sm_count * 64 * 2 * sm_mhz * 1e6 / 1e12
