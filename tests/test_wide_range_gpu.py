"""fp32 parity on inputs whose magnitudes span many decades along the
contraction index (the weak spot of one power-of-two scale per row or
column): MP2 rows spanning six decades along P, one-hot rows, rows with a
spike far above the rest; AO->MO eri scaled along m and C columns of mixed
magnitude. Checked against the fp64 CPU oracle (the reference's loop body,
trntensor/quantum.py:87-100, and its two-step transform) at the north-star
tolerances: |dE|/|E| <= 1e-6, max|dB| <= 1e-5 max|B|."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import trntensor_b200 as tt
from oracle import oracle
from tests.helpers import WIDE_CASES, wide_mp2_inputs
from tests.test_ozaki_format_cpu import range_estimate
from trntensor_b200.dispatch import WIDE_ROWS_MAX_EST, mp2_range_estimate

pytestmark = pytest.mark.gpu


def rel(a, b):
    return abs(float(a) - float(b)) / abs(float(b))


@pytest.mark.parametrize("shape", [(3, 96, 384), (4, 150, 512)])
@pytest.mark.parametrize("case", WIDE_CASES)
def test_wide_rows_energy(cuda_ok, shape, case):
    B, eo, ev = wide_mp2_inputs(shape, 3, *case)
    ref, _ = oracle.mp2_energy_fp64(B.numpy(), eo.numpy(), ev.numpy())
    est = mp2_range_estimate(B)
    # the device statistics are the CPU emulation's (same digits, fp64 sums)
    assert est == pytest.approx(range_estimate(B.numpy()), rel=1e-9)
    e = tt.mp2_energy(B.cuda(), eo.cuda(), ev.cuda())
    assert e.dtype == torch.float32
    assert rel(e.item(), ref) <= 1e-6, (est, e.item(), ref)
    # host-resident pinned B takes the pipelined copy path, same rule
    eh = tt.mp2_energy(B.pin_memory(), eo, ev)
    assert rel(eh.item(), ref) <= 1e-6
    p = tt.mp2_pair_energies(B.cuda(), eo.cuda(), ev.cuda()).cpu().numpy()
    assert abs(p.sum() - ref) <= 1e-6 * abs(ref)


def test_gaussian_rows_stay_on_three_digits(cuda_ok):
    from trntensor_b200.inputs import mp2_inputs

    for shape in ((8, 32, 96), (64, 448, 1536)):
        B, _, _ = mp2_inputs(*shape, seed=0)
        assert mp2_range_estimate(B) <= WIDE_ROWS_MAX_EST / 3


def test_wide_rows_at_scale(cuda_ok):
    """Six decades along P at nocc 16, nvir 700, naux 2000 (a config-2-like
    slice): the estimate decides, the energy meets 1e-6 either way."""
    B, eo, ev = wide_mp2_inputs((16, 700, 2000), 11, 6, 0, 0.0)
    ref, _ = oracle.mp2_energy_fp64(B.numpy(), eo.numpy(), ev.numpy())
    e = tt.mp2_energy(B.cuda(), eo.cuda(), ev.cuda())
    assert rel(e.item(), ref) <= 1e-6


@pytest.mark.parametrize("shape", [(128, 16, 112, 96), (300, 20, 90, 40)])
def test_wide_ao2mo(cuda_ok, shape):
    """eri scaled by logspace(-5, 0) along the contraction index m, one column
    block of C_vir 1e-4 smaller and a one-hot C_occ column."""
    from trntensor_b200.inputs import ao2mo_inputs

    nbf, nocc, nvir, naux = shape
    eri, co, cv = (t.double() for t in ao2mo_inputs(nbf, nocc, nvir, naux, seed=7))
    eri *= torch.logspace(-5, 0, nbf, dtype=torch.float64)[:, None, None]
    cv[:, ::3] *= 1e-4
    co[:, 1] = 0.0
    co[nbf // 2, 1] = 1.0
    eri, co, cv = eri.float(), co.float(), cv.float()
    ref, _ = oracle.ao_to_mo_two_step(eri.double().numpy(), co.double().numpy(),
                                      cv.double().numpy())
    got = tt.ao_to_mo_transform(eri.cuda(), co.cuda(), cv.cuda()).double().cpu().numpy()
    assert np.abs(got - ref).max() <= 1e-5 * np.abs(ref).max()
