"""The CPU oracle against golden vectors produced by the reference itself."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import oracle
from tests.helpers import AO_CASES, MP2_CASES, ao_case_inputs, mp2_case_inputs, ref_recipe_mp2


@pytest.mark.parametrize("name", MP2_CASES)
def test_mp2_loop_fp32_matches_reference(golden, name):
    B, eo, ev = (t.numpy() for t in mp2_case_inputs(golden, name))
    e, _ = oracle.mp2_energy_loop(B, eo, ev)
    ref = golden[f"{name}/e_fp32"]
    assert abs(float(e) - ref) <= 2e-6 * abs(ref)


@pytest.mark.parametrize("name", MP2_CASES)
def test_mp2_fp64_and_pairs_match_reference(golden, name):
    B, eo, ev = (t.numpy() for t in mp2_case_inputs(golden, name))
    e, part = oracle.mp2_energy_fp64(B, eo, ev)
    np.testing.assert_allclose(e, golden[f"{name}/e_fp64"], rtol=1e-12)
    np.testing.assert_allclose(part, golden[f"{name}/pair_fp64"], rtol=1e-10, atol=1e-14)
    e2, part2 = oracle.mp2_energy_loop(B, eo, ev, dtype=np.float64)
    np.testing.assert_allclose(e2, e, rtol=1e-12)
    np.testing.assert_allclose(part2, part, rtol=1e-10, atol=1e-14)


def test_manual_unrolled_kat(golden):
    """tests/test_quantum.py:11-33: the loop equals the explicit 4-index sum."""
    B, eo, ev = (t.numpy() for t in mp2_case_inputs(golden, "kat_manual"))
    e, _ = oracle.mp2_energy_loop(B, eo, ev)
    np.testing.assert_allclose(float(e), golden["kat_manual/e_unrolled"], rtol=1e-6, atol=1e-6)


def test_tutorial_value():
    """docs/tutorial_df_mp2.md:77: E_MP2 = -50.5432928801 for (5,19,72), seed 42."""
    B, eo, ev = (t.numpy() for t in ref_recipe_mp2(42, 5, 19, 72))
    e, _ = oracle.mp2_energy_loop(B, eo, ev)
    assert abs(float(e) - (-50.5432928801)) < 1e-5
    e64, _ = oracle.mp2_energy_fp64(B, eo, ev)
    assert abs(e64 - (-50.5432928801)) / 50.54 < 1e-6


def test_regenerated_inputs_match(golden):
    for name in MP2_CASES:
        B, eo, ev = mp2_case_inputs(golden, name)
        assert tuple(B.shape) == tuple(golden[f"{name}/shape"])


@pytest.mark.parametrize("name", sorted(AO_CASES))
def test_ao2mo_two_step_matches_reference(golden, name):
    vals = ao_case_inputs(golden, name)
    eri, co, cv = (v.double().numpy() for v in vals[:3])
    B, _ = oracle.ao_to_mo_two_step(eri, co, cv)
    if f"{name}/B_fp64" in golden:
        ref = golden[f"{name}/B_fp64"]
        np.testing.assert_allclose(B, ref, rtol=1e-10, atol=1e-12 * np.abs(ref).max())
        if B.size < 5000:
            np.testing.assert_allclose(oracle.ao_to_mo_fused(eri, co, cv), ref, rtol=1e-9,
                                       atol=1e-12 * np.abs(ref).max())
    else:
        idx = golden[f"{name}/B_fp64_sample_idx"]
        np.testing.assert_allclose(B.flatten()[idx], golden[f"{name}/B_fp64_sample"], rtol=1e-10,
                                   atol=1e-14)
    if f"{name}/e_fp64" in golden:
        eo, ev = (v.double().numpy() for v in vals[3:])
        e, _ = oracle.mp2_energy_fp64(B, eo, ev)
        np.testing.assert_allclose(e, golden[f"{name}/e_fp64"], rtol=1e-10)


def test_config1_inputs_are_orthonormal_and_symmetric():
    eri, co, cv = AO_CASES["config1"]()
    C = torch.cat([co, cv], 1).double()
    torch.testing.assert_close(C.T @ C, torch.eye(128, dtype=torch.float64), atol=1e-6, rtol=0)
    torch.testing.assert_close(eri, eri.transpose(0, 1))


def test_config4_fixture_reproduces():
    """Two of the 64 config-4 pair energies recomputed from regenerated rows
    (the row-wise recipe is deterministic), plus the stored row checksums."""
    import json
    from pathlib import Path

    from trntensor_b200.inputs import mp2_eps_rowwise, mp2_row

    fx = json.loads((Path(__file__).parent / "golden" / "config4_pairs.json").read_text())
    c = fx["config"]
    eo, ev = (t.numpy().astype(np.float64) for t in mp2_eps_rowwise(c["nocc"], c["nvir"], c["seed"]))
    assert len(fx["pairs"]) >= 64
    for i, j, e in (fx["pairs"][0], fx["pairs"][-1]):
        Bij = np.stack([mp2_row(i, c["nvir"], c["naux"], c["seed"]),
                        mp2_row(j, c["nvir"], c["naux"], c["seed"])]).astype(np.float64)
        got = float(oracle.mp2_pair_energy(Bij, eo[[i, j]], ev, 0, 1))
        assert got == pytest.approx(e, rel=1e-12)
        assert Bij[0].sum() == pytest.approx(fx["row_sums"][str(i)], rel=1e-12)


def test_decimal_oracle_matches_fp64_golden(golden):
    """The 60-digit decimal restatement (the precision="dd" checker) agrees
    with the reference's fp64 energies on two known-answer cases."""
    for name in ("kat_manual", "kat_public"):
        B, eo, ev = mp2_case_inputs(golden, name)
        e = float(oracle.mp2_energy_decimal(B.double().numpy(), eo.double().numpy(),
                                            ev.double().numpy()))
        assert e == pytest.approx(float(golden[f"{name}/e_fp64"]), rel=1e-13)
