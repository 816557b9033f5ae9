"""CPU oracle for the DF-MP2 / AO->MO path.

TEST INFRASTRUCTURE ONLY. This module restates, in numpy, the reference's
CPU algorithms so that tests can check the CUDA kernels and bench.py can time
a CPU baseline. Nothing in the product package imports it; the product path
has no CPU implementation at all.

Restated from trnsci/trntensor 0.4.0:
* ``mp2_energy_loop``  - trntensor/quantum.py:87-100 (``_cpu_mp2_energy``):
  for every ordered pair (i, j): T = B[i] @ B[j].T (einsum "ap,bp->ab"),
  denom = eps_occ[i] + eps_occ[j] - eps_vir[:,None] - eps_vir[None,:],
  E += sum(T * (2T - T.T) / denom), accumulated in the input dtype.
* ``ao_to_mo_two_step`` - the two-step form the reference's tests and
  benchmarks use (tests/test_quantum.py:73-74,
  benchmarks/bench_einsum.py:135-137): inter = einsum("mi,mnP->inP"),
  B = einsum("na,inP->iaP").
* ``ao_to_mo_fused``   - trntensor/quantum.py:188-194 (3-operand einsum),
  only for small sizes.
The arithmetic itself is BLAS (torch 2.11 CPU BLAS in the reference, numpy's
BLAS here); pinned by tests/golden fixtures made from the reference.
"""

from __future__ import annotations

import numpy as np


def mp2_pair_energy(B, eps_occ, eps_vir, i, j, dtype=None):
    """E_ij for one ordered pair, exactly the reference's loop body."""
    dt = np.dtype(dtype) if dtype is not None else B.dtype
    Bi = B[i].astype(dt, copy=False)
    Bj = B[j].astype(dt, copy=False)
    ev = eps_vir.astype(dt, copy=False)
    eo = eps_occ.astype(dt, copy=False)
    T = Bi @ Bj.T
    denom = (eo[i] + eo[j]) - ev[:, None] - ev[None, :]
    return (T * (2 * T - T.T) / denom).sum(dtype=dt)


def mp2_energy_loop(B, eps_occ, eps_vir, dtype=None, pairs=None):
    """Reference algorithm over all nocc^2 ordered pairs (or a given list).

    Returns (E, partial) with partial[i, j] = E_ij (float64 array).
    """
    dt = np.dtype(dtype) if dtype is not None else B.dtype
    nocc = B.shape[0]
    partial = np.zeros((nocc, nocc), dtype=np.float64)
    e = dt.type(0)
    it = pairs if pairs is not None else ((i, j) for i in range(nocc) for j in range(nocc))
    for i, j in it:
        eij = mp2_pair_energy(B, eps_occ, eps_vir, i, j, dt)
        partial[i, j] = eij
        e = dt.type(e + eij)
    return e, partial


def mp2_energy_fp64(B, eps_occ, eps_vir):
    """fp64 energy, vectorised over j for each i (same sum, faster)."""
    B = B.astype(np.float64)
    eo = eps_occ.astype(np.float64)
    ev = eps_vir.astype(np.float64)
    nocc, nvir, _ = B.shape
    partial = np.zeros((nocc, nocc))
    dvv = ev[:, None] + ev[None, :]
    for i in range(nocc):
        for j in range(i, nocc):
            T = B[i] @ B[j].T
            eij = (T * (2 * T - T.T) / ((eo[i] + eo[j]) - dvv)).sum()
            partial[i, j] = eij
            partial[j, i] = eij
    return partial.sum(), partial


def ao_to_mo_two_step(eri, C_occ, C_vir, dtype=None):
    """inter[i,n,P] = sum_m C_occ[m,i] eri[m,n,P]; B[i,a,P] = sum_n C_vir[n,a] inter[i,n,P]."""
    dt = np.dtype(dtype) if dtype is not None else eri.dtype
    eri = eri.astype(dt, copy=False)
    Co = C_occ.astype(dt, copy=False)
    Cv = C_vir.astype(dt, copy=False)
    nbf, _, naux = eri.shape
    inter = (Co.T @ eri.reshape(nbf, nbf * naux)).reshape(Co.shape[1], nbf, naux)
    # B[i] = Cv^T @ inter[i]  (nvir x naux)
    return np.einsum("na,inP->iaP", Cv, inter, optimize=True), inter


def ao_to_mo_fused(eri, C_occ, C_vir):
    """The reference's literal 3-operand contraction; small sizes only."""
    return np.einsum("mi,na,mnP->iaP", C_occ, C_vir, eri, optimize=False)


# ------------------------------------------------ high-precision references
# For precision="dd" (double-double) checks: the same sums in Python's
# decimal arithmetic at 60 significant digits. Every float converts to
# Decimal exactly; products, sums and quotients round at 1e-60 relative,
# far below double-double's ~1e-32. Small sizes only (pure Python loops).

def _dec(x):
    from decimal import Decimal

    return Decimal(float(x))


def mp2_energy_decimal(B, eps_occ, eps_vir, prec=60):
    """sum over ordered pairs of sum_ab T_ab (2 T_ab - T_ba) / D_ijab
    (trntensor/quantum.py:87-100) in decimal arithmetic; returns a Decimal."""
    from decimal import localcontext

    B = np.asarray(B, dtype=np.float64)
    nocc, nvir, naux = B.shape
    with localcontext() as ctx:
        ctx.prec = prec
        Bd = [[[_dec(B[i, a, p]) for p in range(naux)] for a in range(nvir)] for i in range(nocc)]
        eo = [_dec(v) for v in np.asarray(eps_occ, dtype=np.float64)]
        ev = [_dec(v) for v in np.asarray(eps_vir, dtype=np.float64)]
        total = _dec(0.0)
        for i in range(nocc):
            for j in range(nocc):
                T = [[sum(x * y for x, y in zip(Bd[i][a], Bd[j][b])) for b in range(nvir)]
                     for a in range(nvir)]
                for a in range(nvir):
                    for b in range(nvir):
                        total += T[a][b] * (2 * T[a][b] - T[b][a]) / (eo[i] + eo[j] - ev[a] - ev[b])
        return total


def matmul_decimal(A, B, prec=60):
    """A @ B (2-D) in decimal arithmetic; returns a nested list of Decimals."""
    from decimal import localcontext

    A = np.asarray(A, dtype=np.float64)
    B = np.asarray(B, dtype=np.float64)
    with localcontext() as ctx:
        ctx.prec = prec
        Ad = [[_dec(v) for v in row] for row in A]
        Bt = [[_dec(B[k, n]) for k in range(B.shape[0])] for n in range(B.shape[1])]
        return [[sum(x * y for x, y in zip(r, c)) for c in Bt] for r in Ad]
