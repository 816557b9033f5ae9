"""DF-MP2 primitives, drop-in for trntensor/quantum.py.

Same signatures, validation and error messages as the reference
(trntensor/quantum.py:21-84 and 103-185), plus an optional ``precision=``
keyword with ``trntensor.einsum``'s meaning (trntensor/einsum.py:108-116):
``"fast"`` computes in the input dtype (fp32-level accuracy from int8
tensor-core GEMMs on three Ozaki digits per value, accumulated exactly),
``"kahan"`` computes in fp64 and returns the input dtype, ``"dd"`` computes
in double-double (about 106 bits; CUDA-core kernels, a correctness mode) and
returns the input dtype (``mp2_energy_dd`` returns the hi and lo parts).

Unlike the reference there is no backend gate and no CPU fallback: both
functions always run the sm_100a kernels, moving host tensors to the current
CUDA device and returning results on the caller's device.
"""

from __future__ import annotations

import torch

from .dispatch import _cuda_mp2_energy, _cuda_mp2_energy_dd
from .plan import _check_precision


def _validate_mp2(B, eps_occ, eps_vir, precision):
    """Checks and messages of trntensor/quantum.py:58-64, plus ``precision``."""
    if B.dim() != 3:
        raise ValueError(f"B must be 3D (nocc, nvir, naux); got shape {tuple(B.shape)}")
    nocc, nvir, _naux = B.shape
    if eps_occ.shape != (nocc,):
        raise ValueError(f"eps_occ must have shape ({nocc},); got {tuple(eps_occ.shape)}")
    if eps_vir.shape != (nvir,):
        raise ValueError(f"eps_vir must have shape ({nvir},); got {tuple(eps_vir.shape)}")
    _check_precision(precision)


def mp2_energy(
    B: torch.Tensor,
    eps_occ: torch.Tensor,
    eps_vir: torch.Tensor,
    *,
    precision: str = "fast",
) -> torch.Tensor:
    """Second-order Møller–Plesset correlation energy, density-fitted.

        E_MP2 = Σ_{ijab} T_{ijab} (2 T_{ijab} - T_{ijba}) / Δ_{ijab}
        T_{ijab} = Σ_P B[i,a,P] B[j,b,P],  Δ_{ijab} = ε_i + ε_j - ε_a - ε_b

    One fused device pass: T is accumulated in tensor memory and reduced in
    the kernel epilogue; it never reaches HBM.

    Parameters
    ----------
    B : (nocc, nvir, naux) tensor
    eps_occ : (nocc,) tensor
    eps_vir : (nvir,) tensor
    precision : "fast" | "kahan" | "dd"

    Returns
    -------
    0-D tensor of ``B.dtype`` on ``B``'s device.
    """
    _validate_mp2(B, eps_occ, eps_vir, precision)
    nocc, nvir, _naux = B.shape
    if nocc == 0 or nvir == 0 or _naux == 0:
        return B.new_zeros(())
    if precision == "dd":
        energy, _ = _cuda_mp2_energy_dd(B, eps_occ, eps_vir)
        return energy[0].to(device=B.device, dtype=B.dtype)
    energy, _ = _cuda_mp2_energy(B, eps_occ, eps_vir, precision=precision)
    return energy.to(device=B.device, dtype=B.dtype)


def mp2_energy_dd(B: torch.Tensor, eps_occ: torch.Tensor, eps_vir: torch.Tensor) -> torch.Tensor:
    """The DF-MP2 energy in double-double as a (2,) float64 tensor [hi, lo]
    (E = hi + lo to about 2^-106 relative for well-conditioned sums), on
    ``B``'s device. Same validation as ``mp2_energy``."""
    _validate_mp2(B, eps_occ, eps_vir, "dd")
    if B.numel() == 0:
        return torch.zeros(2, dtype=torch.float64, device=B.device)
    energy, _ = _cuda_mp2_energy_dd(B, eps_occ, eps_vir)
    return energy.to(B.device)


def mp2_pair_energies(
    B: torch.Tensor,
    eps_occ: torch.Tensor,
    eps_vir: torch.Tensor,
    *,
    precision: str = "fast",
) -> torch.Tensor:
    """Per-pair energies E_ij as a (nocc, nocc) float64 tensor.

    The same (nocc, nocc) partial the reference's device kernel returns before
    its host-side sum (trntensor/nki/_kernels.py:152,205 and
    trntensor/nki/dispatch.py:283); ``.sum()`` of it is ``mp2_energy``.
    """
    _validate_mp2(B, eps_occ, eps_vir, precision)
    nocc, nvir, naux = (int(x) for x in B.shape)
    if nocc == 0 or nvir == 0 or naux == 0:
        return torch.zeros((nocc, nocc), dtype=torch.float64, device=B.device)
    if precision == "dd":
        _, partials = _cuda_mp2_energy_dd(B, eps_occ, eps_vir, return_partials=True)
        return partials[..., 0].contiguous().to(B.device)
    _, partials = _cuda_mp2_energy(B, eps_occ, eps_vir, precision=precision, return_partials=True)
    return partials.to(B.device)


def _validate_ao2mo(eri, C_occ, C_vir, precision):
    """Checks and messages of trntensor/quantum.py:138-151, plus ``precision``."""
    if eri.dim() != 3:
        raise ValueError(f"eri must be 3D (nbasis, nbasis, naux); got shape {tuple(eri.shape)}")
    nbasis_mu, nbasis_nu, _naux = eri.shape
    if nbasis_mu != nbasis_nu:
        raise ValueError(
            f"eri first two dims must match (nbasis, nbasis); got ({nbasis_mu}, {nbasis_nu})"
        )
    nbasis = nbasis_mu
    if C_occ.dim() != 2 or C_occ.shape[0] != nbasis:
        raise ValueError(f"C_occ must have shape ({nbasis}, nocc); got {tuple(C_occ.shape)}")
    if C_vir.dim() != 2 or C_vir.shape[0] != nbasis:
        raise ValueError(f"C_vir must have shape ({nbasis}, nvir); got {tuple(C_vir.shape)}")
    _check_precision(precision)


def ao_to_mo_transform(
    eri: torch.Tensor,
    C_occ: torch.Tensor,
    C_vir: torch.Tensor,
    *,
    precision: str = "fast",
) -> torch.Tensor:
    """AO→MO transform B[i,a,P] = Σ_{μν} C_occ[μ,i] C_vir[ν,a] eri[μ,ν,P].

    Two tensor-core GEMM phases ('mi,mnP->inP' then 'na,inP->iaP') with the
    (i, ν, P) intermediate in an HBM workspace, as the reference's kernel does
    (trntensor/nki/_kernels.py:209-296).
    """
    _validate_ao2mo(eri, C_occ, C_vir, precision)
    from .dispatch import _cuda_ao_to_mo_dd, _cuda_ao_to_mo_transform

    if precision == "dd":
        hi, _ = _cuda_ao_to_mo_dd(eri, C_occ, C_vir)
        return hi.to(device=eri.device, dtype=eri.dtype)
    out = _cuda_ao_to_mo_transform(eri, C_occ, C_vir, precision=precision)
    return out.to(device=eri.device, dtype=eri.dtype)


def df_mp2_energy(
    eri: torch.Tensor,
    C_occ: torch.Tensor,
    C_vir: torch.Tensor,
    eps_occ: torch.Tensor,
    eps_vir: torch.Tensor,
    *,
    precision: str = "fast",
    return_pairs: bool = False,
):
    """DF-MP2 energy from AO integrals: ``mp2_energy(ao_to_mo_transform(...))``.

    The composed workload of the reference's tests
    (trntensor tests/test_quantum.py:77-93, tests/test_nki_kernels.py:178-196):
    B stays in device memory between the two steps (the B200 counterpart of the
    reference's XLA residency). With ``return_pairs=True`` returns
    ``(E, E_ij)`` where ``E_ij`` is the (nocc, nocc) fp64 pair-energy matrix.
    """
    B = ao_to_mo_transform(
        eri.cuda() if eri.device.type == "cpu" else eri,
        C_occ, C_vir, precision=precision,
    )
    if return_pairs:
        pairs = mp2_pair_energies(B, eps_occ, eps_vir, precision=precision)
        e = pairs.sum().to(dtype=eri.dtype)
        return e.to(eri.device), pairs.to(eri.device)
    return mp2_energy(B, eps_occ, eps_vir, precision=precision).to(eri.device)
