"""Generate tests/golden/golden.npz by running the reference trntensor 0.4.0.

Run in a container where the reference source is available:
    python tests/golden/make_golden.py /path/to/trntensor-reference

Every case re-runs the reference's own CPU code (trntensor.quantum
``_cpu_mp2_energy``, ``ao_to_mo_transform`` and ``trntensor.einsum``) on the
inputs of the reference's known-answer tests (tests/test_quantum.py,
tests/test_nki_kernels.py, docs/tutorial_df_mp2.md) and of the benchmark
configurations 0 and 1, in fp32 (as shipped) and on fp64-promoted inputs.
Inputs that torch's CPU generator reproduces bit-for-bit are stored as seeds
plus a checksum; small ones are stored outright.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))


def checksum(t: torch.Tensor) -> np.ndarray:
    x = t.double().flatten()
    return np.array([x.sum().item(), (x * x).sum().item(), x[: min(8, x.numel())].sum().item()])


def ref_recipe_mp2(seed, nocc, nvir, naux):
    """Input recipe of tests/test_nki_kernels.py:154-157."""
    torch.manual_seed(seed)
    B = torch.randn(nocc, nvir, naux) * 0.1
    eo = -torch.sort(torch.rand(nocc))[0] - 0.5
    ev = torch.sort(torch.rand(nvir))[0] + 0.1
    return B, eo, ev


def ref_recipe_ao2mo(seed, nbf, nocc, nvir, naux, with_eps=False):
    """Input recipe of tests/test_nki_kernels.py:184-189 / tests/test_quantum.py:66-69."""
    torch.manual_seed(seed)
    eri = torch.randn(nbf, nbf, naux) * 0.1
    C_occ = torch.randn(nbf, nocc)
    C_vir = torch.randn(nbf, nvir)
    if with_eps:
        eo = -torch.sort(torch.rand(nocc))[0] - 0.5
        ev = torch.sort(torch.rand(nvir))[0] + 0.1
        return eri, C_occ, C_vir, eo, ev
    return eri, C_occ, C_vir


def main(ref_root: str) -> None:
    sys.path.insert(0, ref_root)
    import trntensor  # the reference
    from trntensor.quantum import _cpu_mp2_energy

    from trntensor_b200.inputs import ao2mo_inputs, mp2_inputs

    assert not trntensor.HAS_NKI
    out: dict[str, np.ndarray] = {}

    def mp2_case(name, B, eo, ev, store_inputs=True, meta=None):
        e32 = _cpu_mp2_energy(B, eo, ev)
        e64 = _cpu_mp2_energy(B.double(), eo.double(), ev.double())
        nocc = B.shape[0]
        part = np.zeros((nocc, nocc))
        for i in range(nocc):
            for j in range(nocc):
                part[i, j] = _cpu_mp2_energy(
                    B[[i, j]].double(), eo[[i, j]].double(), ev.double()
                ).item()  # E over {i,j}^2 = E_ii + E_jj + 2 E_ij (i != j)
        eii = np.array([_cpu_mp2_energy(B[[i]].double(), eo[[i]].double(), ev.double()).item()
                        for i in range(nocc)])
        pair = (part - eii[:, None] - eii[None, :]) / 2.0
        np.fill_diagonal(pair, eii)
        out[f"{name}/e_fp32"] = np.array(e32.item(), dtype=np.float64)
        out[f"{name}/e_fp64"] = np.array(e64.item(), dtype=np.float64)
        out[f"{name}/pair_fp64"] = pair
        out[f"{name}/shape"] = np.array(B.shape)
        out[f"{name}/checksum"] = np.concatenate([checksum(B), checksum(eo), checksum(ev)])
        if store_inputs:
            out[f"{name}/B"] = B.numpy()
            out[f"{name}/eps_occ"] = eo.numpy()
            out[f"{name}/eps_vir"] = ev.numpy()

    # tests/test_quantum.py:11-33 (literal eps) and its unrolled 4-index value
    torch.manual_seed(0)
    B = torch.randn(2, 3, 5) * 0.1
    eo = torch.tensor([-0.5, -0.4])
    ev = torch.tensor([0.1, 0.2, 0.3])
    T = torch.einsum("iap,jbp->ijab", B, B)
    den = eo.view(-1, 1, 1, 1) + eo.view(1, -1, 1, 1) - ev.view(1, 1, -1, 1) - ev.view(1, 1, 1, -1)
    out["kat_manual/e_unrolled"] = np.array((T * (2 * T - T.transpose(-1, -2)) / den).sum().item())
    mp2_case("kat_manual", B, eo, ev)
    # tests/test_quantum.py:49-56 (arange eps)
    torch.manual_seed(1)
    B = torch.randn(3, 4, 6) * 0.1
    eo = -torch.arange(3, dtype=torch.float32) - 0.5
    ev = torch.arange(4, dtype=torch.float32) + 0.5
    mp2_case("kat_public", B, eo, ev)
    # tests/test_nki_kernels.py:148-176; docs/tutorial_df_mp2.md:77 (E = -50.5432928801)
    mp2_case("kat_demo", *ref_recipe_mp2(42, 5, 19, 72))
    mp2_case("kat_medium", *ref_recipe_mp2(43, 8, 32, 128))
    # ragged tiles: nvir not a multiple of 128, naux not a multiple of 16
    mp2_case("ragged", *ref_recipe_mp2(7, 3, 200, 37))
    mp2_case("ragged_big", *ref_recipe_mp2(8, 4, 300, 100))
    # BASELINE config 0, fp32 (drawn in fp64 then cast)
    mp2_case("config0", *mp2_inputs(8, 32, 96, seed=0))

    def ao2mo_case(name, eri, Co, Cv, store_out=True, eps=None):
        B32 = trntensor.ao_to_mo_transform(eri, Co, Cv)  # reference CPU path (fused einsum)
        inter = trntensor.einsum("mi,mnP->inP", Co, eri)
        B2 = trntensor.einsum("na,inP->iaP", Cv, inter)
        B64 = trntensor.einsum(
            "na,inP->iaP", Cv.double(), trntensor.einsum("mi,mnP->inP", Co.double(), eri.double())
        )
        out[f"{name}/shape"] = np.array([eri.shape[0], Co.shape[1], Cv.shape[1], eri.shape[2]])
        out[f"{name}/checksum"] = np.concatenate([checksum(eri), checksum(Co), checksum(Cv)])
        out[f"{name}/fused_vs_two_step_maxabs"] = np.array((B32 - B2).abs().max().item())
        if store_out:
            out[f"{name}/B_fp32"] = B32.numpy()
            out[f"{name}/B_fp64"] = B64.numpy()
        else:
            flat = B64.flatten()
            idx = np.arange(0, flat.numel(), 97)
            out[f"{name}/B_fp64_sample_idx"] = idx
            out[f"{name}/B_fp64_sample"] = flat[idx].numpy()
            out[f"{name}/B_fp64_checksum"] = checksum(B64)
        if eps is not None:
            eo, ev = eps
            out[f"{name}/e_fp32"] = np.array(_cpu_mp2_energy(B32, eo, ev).item())
            out[f"{name}/e_fp64"] = np.array(_cpu_mp2_energy(B64, eo.double(), ev.double()).item())

    ao2mo_case("ao_kat_small", *ref_recipe_ao2mo(0, 8, 3, 5, 12))
    e, co, cv, eo, ev = ref_recipe_ao2mo(42, 32, 5, 10, 16, with_eps=True)
    ao2mo_case("ao_kat_compose", e, co, cv, eps=(eo, ev))
    ao2mo_case("ao_kat_k256", *ref_recipe_ao2mo(50, 256, 16, 32, 32))
    ao2mo_case("ao_kat_pad200", *ref_recipe_ao2mo(51, 200, 10, 20, 24))
    e, co, cv, eo, ev = ref_recipe_ao2mo(52, 256, 10, 30, 32, with_eps=True)
    ao2mo_case("ao_kat_pipeline", e, co, cv, eps=(eo, ev))
    ao2mo_case("config1", *ao2mo_inputs(128, 16, 112, 384, seed=0), store_out=False)

    np.savez_compressed(HERE / "golden.npz", **out)
    print(f"wrote {len(out)} arrays to {HERE / 'golden.npz'}")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py <reference source tree>")
    main(sys.argv[1])
