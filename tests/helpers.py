"""Input regeneration for golden cases (torch's CPU generator is deterministic)."""

from __future__ import annotations

import numpy as np
import torch

from trntensor_b200.inputs import ao2mo_inputs, mp2_inputs


def checksum(t: torch.Tensor) -> np.ndarray:
    x = t.double().flatten()
    return np.array([x.sum().item(), (x * x).sum().item(), x[: min(8, x.numel())].sum().item()])


def ref_recipe_mp2(seed, nocc, nvir, naux):
    torch.manual_seed(seed)
    B = torch.randn(nocc, nvir, naux) * 0.1
    eo = -torch.sort(torch.rand(nocc))[0] - 0.5
    ev = torch.sort(torch.rand(nvir))[0] + 0.1
    return B, eo, ev


def ref_recipe_ao2mo(seed, nbf, nocc, nvir, naux, with_eps=False):
    torch.manual_seed(seed)
    eri = torch.randn(nbf, nbf, naux) * 0.1
    C_occ = torch.randn(nbf, nocc)
    C_vir = torch.randn(nbf, nvir)
    if with_eps:
        eo = -torch.sort(torch.rand(nocc))[0] - 0.5
        ev = torch.sort(torch.rand(nvir))[0] + 0.1
        return eri, C_occ, C_vir, eo, ev
    return eri, C_occ, C_vir


MP2_CASES = ["kat_manual", "kat_public", "kat_demo", "kat_medium", "ragged", "ragged_big", "config0"]


def mp2_case_inputs(golden, name):
    """Inputs of a stored MP2 golden case (stored outright)."""
    B = torch.from_numpy(golden[f"{name}/B"])
    eo = torch.from_numpy(golden[f"{name}/eps_occ"])
    ev = torch.from_numpy(golden[f"{name}/eps_vir"])
    return B, eo, ev


AO_CASES = {
    "ao_kat_small": lambda: ref_recipe_ao2mo(0, 8, 3, 5, 12),
    "ao_kat_compose": lambda: ref_recipe_ao2mo(42, 32, 5, 10, 16, with_eps=True),
    "ao_kat_k256": lambda: ref_recipe_ao2mo(50, 256, 16, 32, 32),
    "ao_kat_pad200": lambda: ref_recipe_ao2mo(51, 200, 10, 20, 24),
    "ao_kat_pipeline": lambda: ref_recipe_ao2mo(52, 256, 10, 30, 32, with_eps=True),
    "config1": lambda: ao2mo_inputs(128, 16, 112, 384, seed=0),
}


def ao_case_inputs(golden, name):
    vals = AO_CASES[name]()
    cs = np.concatenate([checksum(v) for v in vals[:3]])
    np.testing.assert_allclose(cs, golden[f"{name}/checksum"], rtol=1e-12, atol=1e-9)
    return vals


__all__ = ["mp2_inputs", "ao2mo_inputs"]


def wide_mp2_inputs(shape, seed, decades=6.0, spike=0.0, frac=0.0):
    """MP2 inputs whose B rows span ``decades`` decades along the aux index
    (B[i,a,:] *= logspace(-decades, 0, naux)[perm], a fresh permutation per
    row); a fraction ``frac`` of rows also gets one spike: ``spike`` times the
    row's largest magnitude, or (spike == 0) the row becomes one-hot 0.3."""
    nocc, nvir, naux = shape
    B, eo, ev = mp2_inputs(nocc, nvir, naux, seed=seed)
    B = B.double().numpy()
    rng = np.random.default_rng(seed + 100)
    ls = np.logspace(-decades, 0, naux)
    for i in range(nocc):
        for a in range(nvir):
            B[i, a] *= ls[rng.permutation(naux)]
    rows = rng.random((nocc, nvir)) < frac
    for i, a in zip(*np.nonzero(rows)):
        P = rng.integers(naux)
        if spike == 0:
            B[i, a] = 0.0
            B[i, a, P] = 0.3
        else:
            B[i, a, P] = spike * np.abs(B[i, a]).max()
    return torch.from_numpy(B.astype(np.float32)), eo, ev


WIDE_CASES = [(6, 0, 0.0), (6, 0, 0.05), (6, 10, 0.1), (6, 1e3, 0.1), (3, 100, 0.1),
              (0, 10, 0.1)]
