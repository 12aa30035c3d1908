"""Algorithmic FLOP count of the physics substep from device work counters.

Unit of work: one physics substep of one world.  The per-stage terms follow
the counting rule agreed for this path (one FMA = 2 FLOPs, dense-equivalent
constraint rows, k_r = nv, because the kernel stores dense Jacobian rows):

  F_substep = 120 nbody (FK) + 60 ngeom (frames) + 250 nbody (CoM/CRB) + 12 nM (M)
            + 2 * sum_t (n_t^3/3 + 2 n_t^2)          mass factor/solve (smooth + Euler)
            + 30 npair + sum_pairs F_narrow            broadphase + narrowphase
            + nefc (12 nv + 40)                        constraint rows
            + 300 nbody + F_OSC                        RNE/passive, FP64 OSC (reported apart)
            + I [nefc (2 nv^2 + 4 nv + 30) + nv^3/3 + 2 nv^2]   Newton iterations
            + L nefc (2 nv + 30) + 2 nM                line-search evaluations

Counters recorded per world by the kernel over a control step: substeps,
sum nefc, sum ncon, sum (iterations * nefc), sum (ls evaluations * nefc),
total iterations.  F_narrow is taken as a flat 200 FLOPs per active contact.
"""
import numpy as np

F_OSC_FP64 = 8.0e3


def substep_flops(sizes, tree_dofnum, counters, substeps):
    """FP32 FLOPs (excluding the FP64 OSC) summed over all worlds and substeps.

    counters: dict of per-world arrays (deltas over the measured interval) for
    efc_total, con_total, newton_rows, ls_rows, newton_total."""
    nb, ng, nv, nM, npair = (sizes[k] for k in ('nbody', 'ngeom', 'nv', 'nM', 'npair'))
    worlds = len(np.asarray(counters['efc_total']).reshape(-1))
    n_sub = worlds * substeps
    trees = np.asarray(tree_dofnum, float)
    fixed = (120 * nb + 60 * ng + 250 * nb + 12 * nM + 2 * np.sum(trees ** 3 / 3 + 2 * trees ** 2) +
             30 * npair + 300 * nb + 2 * nM)
    tot = lambda k: float(np.sum(np.asarray(counters[k], np.float64)))  # noqa: E731
    rows = tot('efc_total') * (12 * nv + 40) + tot('con_total') * 200
    newton = tot('newton_rows') * (2 * nv * nv + 4 * nv + 30) + tot('newton_total') * (nv ** 3 / 3 + 2 * nv * nv)
    search = tot('ls_rows') * (2 * nv + 30)
    return fixed * n_sub + rows + newton + search


def osc_flops(worlds, substeps):
    return F_OSC_FP64 * worlds * substeps


def fp32_peak_tflops(sm_count, sm_mhz):
    """Nominal FP32 CUDA-core peak: 128 FP32 lanes per SM, 2 FLOPs per FMA."""
    return sm_count * 128 * 2 * sm_mhz * 1e6 / 1e12


def fp64_peak_tflops(sm_count, sm_mhz):
    """Nominal FP64 CUDA-core peak: 64 FP64 lanes per SM, 2 FLOPs per FMA."""
    return sm_count * 64 * 2 * sm_mhz * 1e6 / 1e12
