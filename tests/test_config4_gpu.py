"""BASELINE config 4 (nocc 256, nvir 1792, naux 6144) pinned to the CPU
oracle pair by pair: 64 unordered pairs spread over the pair range (corners
and diagonal pairs included) whose fp64 energies the oracle computed from the
same row-wise seeded inputs (tests/golden/config4_pairs.json, made by
tests/golden/make_config4_pairs.py). The reference's own device tests compare
its kernel with _cpu_mp2_energy the same way (tests/test_nki_kernels.py:148-176)."""

from __future__ import annotations

import json
from pathlib import Path

import pytest
import torch

import trntensor_b200 as tt
from trntensor_b200.inputs import mp2_inputs_rowwise

pytestmark = pytest.mark.gpu

FIX = Path(__file__).resolve().parent / "golden" / "config4_pairs.json"


def test_config4_pairs_against_oracle(cuda_ok):
    fx = json.loads(FIX.read_text())
    c = fx["config"]
    B, eo, ev = mp2_inputs_rowwise(c["nocc"], c["nvir"], c["naux"], seed=c["seed"])
    for r, s in list(fx["row_sums"].items())[:4]:
        assert B[int(r)].double().sum().item() == pytest.approx(s, rel=1e-12)
    Bd = B.cuda()
    del B
    part = tt.mp2_pair_energies(Bd, eo.cuda(), ev.cuda()).cpu()
    worst = 0.0
    for i, j, e in fx["pairs"]:
        got = part[i, j].item()
        worst = max(worst, abs(got - e) / abs(e))
        # [i][j] and [j][i] receive the same terms through separate atomics
        assert part[j, i].item() == pytest.approx(got, rel=1e-12)
    assert worst <= 1e-6, worst
    # the full energy is the partials' sum
    E = tt.mp2_energy(Bd, eo.cuda(), ev.cuda())
    assert abs(E.item() - part.sum().item()) <= 1e-6 * abs(part.sum().item())
