"""precision="dd" (double-double) on the GPU against a 60-digit decimal
oracle (oracle.mp2_energy_decimal / matmul_decimal, the reference's sums in
Python's decimal arithmetic). The reference names the mode and raises
NotImplementedError (trntensor/einsum.py:112-116); here it runs CUDA-core
double-double kernels (csrc/dd.cu). Bar: |dE| / |E| <= 1e-20 for the
(hi, lo) energy on the reference's known-answer cases."""

from __future__ import annotations

from decimal import Decimal, localcontext

import numpy as np
import pytest
import torch

import trntensor_b200 as tt
from oracle import oracle
from tests.helpers import mp2_case_inputs

pytestmark = pytest.mark.gpu


def dd_value(t):
    hi, lo = (float(x) for x in t.cpu())
    with localcontext() as ctx:
        ctx.prec = 60
        return Decimal(hi) + Decimal(lo)


def rel_dec(x, ref):
    with localcontext() as ctx:
        ctx.prec = 60
        return float(abs(x - ref) / abs(ref))


@pytest.mark.parametrize("name", ["kat_manual", "kat_public", "kat_demo"])
@pytest.mark.parametrize("dtype", [torch.float64, torch.float32])
def test_mp2_dd_energy(golden, cuda_ok, name, dtype):
    B, eo, ev = (t.to(dtype) for t in mp2_case_inputs(golden, name))
    ref = oracle.mp2_energy_decimal(B.double().numpy(), eo.double().numpy(), ev.double().numpy())
    e2 = tt.mp2_energy_dd(B.cuda(), eo.cuda(), ev.cuda())
    assert e2.shape == (2,) and e2.dtype == torch.float64
    assert rel_dec(dd_value(e2), ref) <= 1e-20
    e = tt.mp2_energy(B.cuda(), eo.cuda(), ev.cuda(), precision="dd")
    assert e.dtype == dtype
    # rounded once to the input dtype
    assert float(e.item()) == float(torch.tensor(float(ref), dtype=torch.float64).to(dtype))
    # per-pair energies sum to the total; host inputs work too
    p = tt.mp2_pair_energies(B, eo, ev, precision="dd")
    assert abs(p.sum().item() - float(ref)) <= 1e-13 * abs(float(ref))


def test_mp2_dd_beats_fp64_on_cancellation(cuda_ok):
    """Rows whose dot products cancel to 1e-17 of their terms: fp64
    accumulation loses the result, double-double keeps it."""
    g = torch.Generator().manual_seed(3)
    B = torch.randn(2, 4, 40, generator=g, dtype=torch.float64)
    B[:, :, 20:] = -B[:, :, :20] * (1 + 1e-15)
    eo = torch.tensor([-1.0, -0.75], dtype=torch.float64)
    ev = torch.tensor([0.3, 0.5, 0.9, 1.7], dtype=torch.float64)
    ref = oracle.mp2_energy_decimal(B.numpy(), eo.numpy(), ev.numpy())
    e2 = tt.mp2_energy_dd(B.cuda(), eo.cuda(), ev.cuda())
    assert rel_dec(dd_value(e2), ref) <= 1e-20


def test_ao2mo_dd(cuda_ok):
    from trntensor_b200.dispatch import _cuda_ao_to_mo_dd

    g = torch.Generator().manual_seed(8)
    nbf, nocc, nvir, naux = 8, 3, 5, 12
    eri = torch.randn(nbf, nbf, naux, generator=g, dtype=torch.float64)
    co = torch.randn(nbf, nocc, generator=g, dtype=torch.float64)
    cv = torch.randn(nbf, nvir, generator=g, dtype=torch.float64)
    hi, lo = _cuda_ao_to_mo_dd(eri.cuda(), co.cuda(), cv.cuda())
    hi, lo = hi.cpu().numpy(), lo.cpu().numpy()
    with localcontext() as ctx:
        ctx.prec = 60
        E = [[[Decimal(float(eri[m, n, P])) for P in range(naux)] for n in range(nbf)]
             for m in range(nbf)]
        Co = [[Decimal(float(co[m, i])) for i in range(nocc)] for m in range(nbf)]
        Cv = [[Decimal(float(cv[n, a])) for a in range(nvir)] for n in range(nbf)]
        worst, big = Decimal(0), Decimal(0)
        for i in range(nocc):
            inter = [[sum(Co[m][i] * E[m][n][P] for m in range(nbf)) for P in range(naux)]
                     for n in range(nbf)]
            for a in range(nvir):
                for P in range(naux):
                    ex = sum(Cv[n][a] * inter[n][P] for n in range(nbf))
                    got = Decimal(float(hi[i, a, P])) + Decimal(float(lo[i, a, P]))
                    worst = max(worst, abs(got - ex))
                    big = max(big, abs(ex))
        assert float(worst / big) <= 1e-20
    B = tt.ao_to_mo_transform(eri, co, cv, precision="dd")
    assert B.dtype == torch.float64 and B.device.type == "cpu"
    assert np.array_equal(B.numpy(), hi)


def _exact(A, B):
    return np.array([[float(v) for v in row] for row in oracle.matmul_decimal(A, B)])


def test_einsum_dd(cuda_ok):
    g = torch.Generator().manual_seed(5)
    A = torch.randn(7, 9, generator=g, dtype=torch.float64)
    Bm = torch.randn(9, 5, generator=g, dtype=torch.float64)
    C = torch.randn(5, 4, generator=g, dtype=torch.float64)
    # cancellation: fp64 would lose these outputs entirely
    A[:, 0] = 1e16
    A[:, 1] = -1e16
    Bm[0] = Bm[1]
    ex = _exact(A.numpy(), Bm.numpy())
    got = tt.einsum("ij,jk->ik", A.cuda(), Bm.cuda(), precision="dd").cpu().numpy()
    np.testing.assert_array_equal(got, ex)  # correctly rounded here
    got_t = tt.einsum("ji,jk->ik", A.T.contiguous(), Bm, precision="dd")
    np.testing.assert_array_equal(got_t.numpy(), ex)
    # three operands through the planner's path, double-double intermediates
    ex3 = _exact(np.array(oracle.matmul_decimal(A.numpy(), Bm.numpy()), dtype=object).astype(float),
                 C.numpy())
    got3 = tt.einsum("ij,jk,kl->il", A.cuda(), Bm.cuda(), C.cuda(), precision="dd").cpu()
    np.testing.assert_allclose(got3.numpy(), ex3, rtol=1e-15, atol=1e-15 * np.abs(ex3).max())
    # batched and a reduction; fp32 in, fp32 out
    X = torch.randn(3, 4, 6, generator=g)
    Y = torch.randn(3, 6, 2, generator=g)
    r = tt.einsum("bij,bjk->bik", X.cuda(), Y.cuda(), precision="dd")
    assert r.dtype == torch.float32
    torch.testing.assert_close(r.cpu(), torch.bmm(X.double(), Y.double()).float())
    s = tt.einsum("ij->i", A.cuda(), precision="dd").cpu()
    exs = [float(sum(Decimal(float(v)) for v in row)) for row in A]
    assert s.tolist() == exs
