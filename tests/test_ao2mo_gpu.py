"""AO->MO transform on the GPU against the reference's numbers.

Tolerance (north star): transformed tensors max-relative 1e-5 in fp32 and
1e-12 in fp64, where max-relative = max|B - B_ref| / max|B_ref|.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import trntensor_b200 as tt
from oracle import oracle
from tests.helpers import AO_CASES, ao_case_inputs
from trntensor_b200.inputs import ao2mo_inputs

pytestmark = pytest.mark.gpu

TOL_F32 = 1e-5
TOL_F64 = 1e-12


def max_rel(b, ref):
    b = np.asarray(b, dtype=np.float64)
    return np.abs(b - ref).max() / np.abs(ref).max()


@pytest.mark.parametrize("name", sorted(AO_CASES))
def test_fp32_and_fp64_match_reference(golden, cuda_ok, name):
    eri, co, cv = ao_case_inputs(golden, name)[:3]
    B32 = tt.ao_to_mo_transform(eri.cuda(), co.cuda(), cv.cuda())
    assert B32.dtype == torch.float32 and B32.device.type == "cuda"
    B64 = tt.ao_to_mo_transform(eri.double().cuda(), co.double().cuda(), cv.double().cuda())
    Bk = tt.ao_to_mo_transform(eri.cuda(), co.cuda(), cv.cuda(), precision="kahan")
    assert Bk.dtype == torch.float32
    if f"{name}/B_fp64" in golden:
        ref = golden[f"{name}/B_fp64"]
        assert max_rel(B32.cpu().numpy(), ref) <= TOL_F32
        assert max_rel(B64.cpu().numpy(), ref) <= TOL_F64
        assert max_rel(Bk.cpu().numpy(), ref) <= 1e-7
    else:
        idx = golden[f"{name}/B_fp64_sample_idx"]
        ref = golden[f"{name}/B_fp64_sample"]
        for B, tol in ((B32, TOL_F32), (B64, TOL_F64)):
            got = B.cpu().double().flatten().numpy()[idx]
            assert np.abs(got - ref).max() / np.abs(ref).max() <= tol


@pytest.mark.parametrize("name", ["ao_kat_compose", "ao_kat_pipeline"])
def test_pipeline_energy(golden, cuda_ok, name):
    """AO -> MO -> E on the device (tests/test_nki_kernels.py:178-196, 242-258)."""
    eri, co, cv, eo, ev = ao_case_inputs(golden, name)
    B = tt.ao_to_mo_transform(eri.cuda(), co.cuda(), cv.cuda())
    e = tt.mp2_energy(B, eo.cuda(), ev.cuda())
    ref = float(golden[f"{name}/e_fp64"])
    assert abs(e.item() - ref) / abs(ref) <= 1e-5
    B64 = tt.ao_to_mo_transform(eri.double(), co.double(), cv.double())
    e64 = tt.mp2_energy(B64, eo.double(), ev.double())
    assert abs(e64.item() - ref) / abs(ref) <= 1e-11


def test_host_round_trip(golden, cuda_ok):
    eri, co, cv = ao_case_inputs(golden, "ao_kat_small")
    B = tt.ao_to_mo_transform(eri, co, cv)
    assert B.device.type == "cpu" and B.shape == (3, 5, 12)


def test_config1_against_oracle(cuda_ok):
    eri, co, cv = ao2mo_inputs(128, 16, 112, 384, seed=0)
    ref, _ = oracle.ao_to_mo_two_step(eri.double().numpy(), co.double().numpy(),
                                      cv.double().numpy())
    B = tt.ao_to_mo_transform(eri.cuda(), co.cuda(), cv.cuda())
    assert max_rel(B.cpu().numpy(), ref) <= TOL_F32


def test_config3_p_slab(cuda_ok):
    """BASELINE config 3 (nbf 1024, nocc 128, nvir 896, naux 3072): full-size
    transform on the GPU; the transform is independent per P, so a 16-wide
    P slab is checked against the fp64 CPU oracle and against the GPU fp64
    path."""
    nbf, nocc, nvir, naux = 1024, 128, 896, 3072
    eri, co, cv = ao2mo_inputs(nbf, nocc, nvir, naux, seed=3, device="cuda")
    B = tt.ao_to_mo_transform(eri, co, cv)
    assert B.shape == (nocc, nvir, naux)
    for p0 in (0, 1500, naux - 16):
        slab = eri[:, :, p0:p0 + 16].double().cpu().numpy()
        ref, _ = oracle.ao_to_mo_two_step(slab, co.double().cpu().numpy(),
                                          cv.double().cpu().numpy())
        assert max_rel(B[:, :, p0:p0 + 16].cpu().numpy(), ref) <= TOL_F32
        B64 = tt.ao_to_mo_transform(eri[:, :, p0:p0 + 16].double(), co.double(), cv.double())
        assert max_rel(B64.cpu().numpy(), ref) <= TOL_F64


@pytest.mark.parametrize("shape", [(200, 10, 20, 24), (128, 16, 112, 384), (300, 130, 70, 50)])
def test_tensor_core_vs_cuda_core(cuda_ok, shape):
    """The int8-Ozaki tensor-core path and the plain fp32 CUDA-core path agree
    with the fp64 path (ragged tiles in every dimension)."""
    from trntensor_b200.dispatch import _cuda_ao_to_mo_transform

    nbf, nocc, nvir, naux = shape
    eri, co, cv = ao2mo_inputs(nbf, nocc, nvir, naux, seed=4) if nbf >= nocc + nvir else (
        torch.randn(nbf, nbf, naux) * 0.1, torch.randn(nbf, nocc), torch.randn(nbf, nvir))
    ref = _cuda_ao_to_mo_transform(eri.double(), co.double(), cv.double()).cpu().numpy()
    tc = _cuda_ao_to_mo_transform(eri, co, cv, kernel="tc").cpu().numpy()
    simt = _cuda_ao_to_mo_transform(eri, co, cv, kernel="simt").cpu().numpy()
    assert max_rel(tc, ref) <= TOL_F32
    assert max_rel(simt, ref) <= TOL_F32


def test_einsum_routes_ao2mo_pattern(golden, cuda_ok):
    """trntensor.einsum("mi,na,mnP->iaP") on CUDA operands runs the two-step
    transform (the reference's greedy plan would build the (m,i,n,a) outer product)."""
    eri, co, cv = ao2mo_inputs(128, 16, 112, 384, seed=0)
    ref, _ = oracle.ao_to_mo_two_step(eri.double().numpy(), co.double().numpy(),
                                      cv.double().numpy())
    import sys

    te = sys.modules["trntensor_b200.einsum"]

    calls = []
    orig = te._execute_path
    te._execute_path = lambda *a: calls.append(a) or orig(*a)  # noqa: E731
    try:
        got = tt.einsum("mi,na,mnP->iaP", co.cuda(), cv.cuda(), eri.cuda())
    finally:
        te._execute_path = orig
    assert not calls, "the generic greedy path ran instead of the AO->MO transform"
    assert max_rel(got.cpu().numpy(), ref) <= TOL_F32
    got2 = tt.einsum("xq,xyR,yb->qbR", co.cuda(), eri.cuda(), cv.cuda())
    assert max_rel(got2.cpu().numpy(), ref) <= TOL_F32


@pytest.mark.parametrize("name", ["ao_kat_compose", "ao_kat_pipeline"])
def test_df_mp2_pipeline(golden, cuda_ok, name):
    eri, co, cv, eo, ev = ao_case_inputs(golden, name)
    ref = float(golden[f"{name}/e_fp64"])
    e = tt.df_mp2_energy(eri, co, cv, eo, ev)
    assert e.device.type == "cpu" and abs(e.item() - ref) / abs(ref) <= 1e-5
    e2, pairs = tt.df_mp2_energy(eri.cuda(), co.cuda(), cv.cuda(), eo.cuda(), ev.cuda(),
                                 return_pairs=True)
    assert pairs.shape == (co.shape[1], co.shape[1])
    assert abs(pairs.sum().item() - ref) / abs(ref) <= 1e-5


@pytest.mark.parametrize("shape", [(128, 16, 112, 384), (200, 10, 20, 24), (130, 129, 129, 7),
                                   (256, 130, 100, 64)])
def test_step1_on_chip_split_matches_preslice(cuda_ok, shape, monkeypatch):
    """Step 1 with eri split in shared memory (default) and with eri pre-split
    in HBM (TRNTENSOR_B200_AO2MO_PRESLICE=1) both match fp64; naux = 7 makes
    eri's row stride unaligned, which selects the pre-split path."""
    from trntensor_b200.dispatch import _cuda_ao_to_mo_transform

    nbf, nocc, nvir, naux = shape
    g = torch.Generator().manual_seed(sum(shape))
    eri = torch.randn(nbf, nbf, naux, generator=g) * 0.1
    co = torch.randn(nbf, nocc, generator=g)
    cv = torch.randn(nbf, nvir, generator=g)
    ref = _cuda_ao_to_mo_transform(eri.double(), co.double(), cv.double()).cpu().numpy()
    a = _cuda_ao_to_mo_transform(eri, co, cv).cpu().numpy()
    monkeypatch.setenv("TRNTENSOR_B200_AO2MO_PRESLICE", "1")
    b = _cuda_ao_to_mo_transform(eri, co, cv).cpu().numpy()
    assert max_rel(a, ref) <= TOL_F32
    assert max_rel(b, ref) <= TOL_F32


@pytest.mark.parametrize("shape", [(256, 130, 100, 64), (520, 16, 40, 200), (1024, 128, 96, 160),
                                   (390, 20, 30, 36), (400, 150, 40, 48), (400, 8, 8, 4)])
def test_step1_fused_scales_match_column_pass(cuda_ok, shape, monkeypatch):
    """Step 1 computes eri's column scales inside the GEMM (a max pass over the
    next tile's strip while the current tile converts). With one CTA per tile
    (TRNTENSOR_B200_AO2MO_SPLITK=0) it uses the same scale rule as the
    separate column-max pass (TRNTENSOR_B200_AO2MO_COLMAX=1): bit-identical
    tensors. The default for nbf > 320 splits K over a CTA pair (column maxima
    exchanged between the pair, rank 1 adding its partial onto rank 0's):
    deterministic, and within the fp32 tolerance of fp64. nocc = 130 and 150
    give two row tiles per strip (the latter split-K), nbf = 520 and 390
    ragged k halves, the 1024 case more tiles than CTA pairs, the last fewer."""
    from trntensor_b200.dispatch import _cuda_ao_to_mo_transform

    nbf, nocc, nvir, naux = shape
    g = torch.Generator().manual_seed(nbf + naux)
    eri = (torch.randn(nbf, nbf, naux, generator=g) * 0.1).cuda()
    # columns of very different magnitude, so that a wrong scale would show
    eri *= torch.logspace(-3, 3, naux, device="cuda")
    co = torch.randn(nbf, nocc, generator=g).cuda()
    cv = torch.randn(nbf, nvir, generator=g).cuda()
    ref = _cuda_ao_to_mo_transform(eri.double(), co.double(), cv.double()).cpu().numpy()
    split = _cuda_ao_to_mo_transform(eri, co, cv)
    split2 = _cuda_ao_to_mo_transform(eri, co, cv)
    torch.cuda.synchronize()
    assert torch.equal(split, split2)
    assert max_rel(split.cpu().numpy(), ref) <= TOL_F32
    monkeypatch.setenv("TRNTENSOR_B200_AO2MO_SPLITK", "0")
    fused = _cuda_ao_to_mo_transform(eri, co, cv)
    monkeypatch.setenv("TRNTENSOR_B200_AO2MO_COLMAX", "1")
    sep = _cuda_ao_to_mo_transform(eri, co, cv)
    torch.cuda.synchronize()
    assert torch.equal(fused, sep)
    assert max_rel(fused.cpu().numpy(), ref) <= TOL_F32
    if nbf <= 320:
        assert torch.equal(split, fused)


@pytest.mark.parametrize("shape", [(200, 10, 20, 24), (128, 16, 112, 384), (300, 130, 70, 50),
                                   (1024, 128, 96, 160), (33, 1, 2, 3)])
def test_fp64_tensor_core_vs_cuda_core(cuda_ok, shape):
    """fp64 transform (precision="kahan"): the five-digit int8 tensor-core path
    and the CUDA-core fp64 path agree to the fp64 tolerance (ragged tiles in
    every dimension, columns of very different magnitude)."""
    from trntensor_b200.dispatch import _cuda_ao_to_mo_transform

    nbf, nocc, nvir, naux = shape
    g = torch.Generator().manual_seed(nbf * 7 + naux)
    eri = torch.randn(nbf, nbf, naux, generator=g, dtype=torch.float64)
    eri *= torch.logspace(-4, 4, naux, dtype=torch.float64)
    co = torch.randn(nbf, nocc, generator=g, dtype=torch.float64)
    cv = torch.randn(nbf, nvir, generator=g, dtype=torch.float64)
    tc = _cuda_ao_to_mo_transform(eri.cuda(), co.cuda(), cv.cuda())
    simt = _cuda_ao_to_mo_transform(eri.cuda(), co.cuda(), cv.cuda(), kernel="simt")
    assert tc.dtype == torch.float64
    assert max_rel(tc.cpu().numpy(), simt.cpu().numpy()) <= TOL_F64
    # per aux column as well: each column has its own scale
    col = (tc - simt).abs().amax(dim=(0, 1)) / simt.abs().amax(dim=(0, 1))
    assert float(col.max()) <= 1e-11


@pytest.mark.parametrize("shape,world", [((256, 16, 40, 96), 3), ((520, 24, 70, 200), 2),
                                         ((1024, 128, 96, 88), 2), ((200, 8, 8, 90), 2)])
def test_strided_p_slab_matches_contiguous(cuda_ok, shape, world):
    """Each rank's aux slab read in place from the full eri
    (tt_ao2mo_f32_slab, 3-D tensor map over the strided slab) gives the
    same tensor, bit for bit, as the transform of a contiguous copy of the
    slab; ragged slabs (not multiples of 128 columns) included. A slab whose
    first column is not 16-byte aligned (naux 90 over 2 ranks) takes the
    copy path."""
    from trntensor_b200.dispatch import _cuda_ao_to_mo_slab
    from trntensor_b200.distributed import aux_slab

    nbf, nocc, nvir, naux = shape
    g = torch.Generator().manual_seed(nbf + world)
    eri = (torch.randn(nbf, nbf, naux, generator=g) * 0.1).cuda()
    eri *= torch.logspace(-2, 2, naux, device="cuda")
    co = torch.randn(nbf, nocc, generator=g).cuda()
    cv = torch.randn(nbf, nvir, generator=g).cuda()
    ref64, _ = oracle.ao_to_mo_two_step(eri.double().cpu().numpy(), co.double().cpu().numpy(),
                                        cv.double().cpu().numpy())
    parts = []
    for r in range(world):
        p0, p1 = aux_slab(naux, r, world)
        got = _cuda_ao_to_mo_slab(eri, co, cv, p0, p1)
        want = tt.ao_to_mo_transform(eri[:, :, p0:p1].contiguous(), co, cv)
        assert torch.equal(got, want)
        parts.append(got)
    full = torch.cat(parts, dim=2).cpu().numpy()
    assert max_rel(full, ref64) <= TOL_F32


def test_one_read_split_matches_two_pass(cuda_ok, monkeypatch):
    """The one-read column split (max pass, then slices re-read from L2)
    produces the same scales and digits as the two-pass kernels, so the
    transforms agree bit for bit (ragged column blocks included)."""
    from trntensor_b200.dispatch import _cuda_ao_to_mo_transform
    eri, co, cv = ao2mo_inputs(300, 130, 70, 50, seed=5, device="cuda")
    monkeypatch.delenv("TRNTENSOR_B200_SPLIT_TWOPASS", raising=False)
    one = _cuda_ao_to_mo_transform(eri, co, cv)
    monkeypatch.setenv("TRNTENSOR_B200_SPLIT_TWOPASS", "1")
    two = _cuda_ao_to_mo_transform(eri, co, cv)
    assert torch.equal(one, two)
