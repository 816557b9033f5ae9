"""Edge cases of the device path against the oracle: minimal and ragged
sizes (one past every tile edge), non-contiguous / low-precision / mixed
device inputs, empty inputs."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import trntensor_b200 as tt
from oracle import oracle
from trntensor_b200.inputs import mp2_inputs

pytestmark = pytest.mark.gpu


def rel(a, b):
    return abs(float(a) - float(b)) / max(abs(float(b)), 1e-300)


@pytest.mark.parametrize(
    "shape",
    [(1, 1, 1), (1, 5, 3), (2, 1, 7), (3, 129, 65), (2, 128, 64), (4, 257, 130), (1, 300, 1),
     (7, 33, 200)],
)
def test_mp2_shapes(cuda_ok, shape):
    B, eo, ev = mp2_inputs(*shape, seed=sum(shape))
    ref, part = oracle.mp2_energy_fp64(B.numpy(), eo.numpy(), ev.numpy())
    e = tt.mp2_energy(B.cuda(), eo.cuda(), ev.cuda())
    assert rel(e.item(), ref) <= 2e-6
    e64 = tt.mp2_energy(B.double().cuda(), eo.double().cuda(), ev.double().cuda())
    assert rel(e64.item(), ref) <= 1e-12
    p = tt.mp2_pair_energies(B.cuda(), eo.cuda(), ev.cuda()).cpu().numpy()
    np.testing.assert_allclose(p, part, rtol=1e-5, atol=1e-7 * np.abs(part).max())


def test_mp2_input_forms(cuda_ok):
    B, eo, ev = mp2_inputs(5, 140, 90, seed=3)
    ref, _ = oracle.mp2_energy_fp64(B.numpy(), eo.numpy(), ev.numpy())
    # non-contiguous view of the same values
    Bt = B.transpose(1, 2).contiguous().transpose(1, 2)
    assert not Bt.is_contiguous()
    assert rel(tt.mp2_energy(Bt.cuda(), eo.cuda(), ev.cuda()).item(), ref) <= 2e-6
    # eps on the host, B on the device; fp64 eps with fp32 B
    assert rel(tt.mp2_energy(B.cuda(), eo.double(), ev.double()).item(), ref) <= 2e-6
    # bf16 input: computed in fp32 on the bf16 values, returned as bf16
    Bb = B.bfloat16()
    refb, _ = oracle.mp2_energy_fp64(Bb.float().numpy(), eo.numpy(), ev.numpy())
    eb = tt.mp2_energy(Bb.cuda(), eo.cuda(), ev.cuda())
    assert eb.dtype == torch.bfloat16 and rel(eb.float().item(), refb) <= 1e-2
    # precision="kahan" on fp32 returns fp32 but computes in fp64
    ek = tt.mp2_energy(B.cuda(), eo.cuda(), ev.cuda(), precision="kahan")
    assert ek.dtype == torch.float32 and rel(ek.item(), ref) <= 1e-7


@pytest.mark.parametrize("shape", [(1, 1, 1, 1), (1, 1, 2, 3), (129, 2, 130, 5), (64, 63, 1, 17),
                                   (130, 129, 129, 1)])
def test_ao2mo_shapes(cuda_ok, shape):
    nbf, nocc, nvir, naux = shape
    g = torch.Generator().manual_seed(sum(shape))
    eri = torch.randn(nbf, nbf, naux, generator=g) * 0.1
    co = torch.randn(nbf, nocc, generator=g)
    cv = torch.randn(nbf, nvir, generator=g)
    ref, _ = oracle.ao_to_mo_two_step(eri.double().numpy(), co.double().numpy(),
                                      cv.double().numpy())
    for B, tol in ((tt.ao_to_mo_transform(eri.cuda(), co.cuda(), cv.cuda()), 1e-5),
                   (tt.ao_to_mo_transform(eri.double().cuda(), co.double().cuda(),
                                          cv.double().cuda()), 1e-12)):
        got = B.cpu().double().numpy()
        assert got.shape == ref.shape
        assert np.abs(got - ref).max() <= tol * np.abs(ref).max()


def test_empty_inputs(cuda_ok):
    e = tt.mp2_energy(torch.zeros(0, 4, 5, device="cuda"), torch.zeros(0, device="cuda"),
                      torch.zeros(4, device="cuda"))
    assert e.item() == 0.0 and e.device.type == "cuda"
    for shape in ((0, 4, 5), (3, 0, 5), (3, 4, 0)):
        Bz = torch.zeros(*shape, device="cuda")
        eo, ev = torch.zeros(shape[0], device="cuda"), torch.zeros(shape[1], device="cuda")
        p = tt.mp2_pair_energies(Bz, eo, ev)
        assert p.shape == (shape[0], shape[0]) and p.dtype == torch.float64 and not p.any()
        from trntensor_b200 import distributed
        assert distributed.mp2_energy(Bz, eo, ev).item() == 0.0
    B = tt.ao_to_mo_transform(torch.zeros(4, 4, 3, device="cuda"), torch.zeros(4, 0, device="cuda"),
                              torch.zeros(4, 2, device="cuda"))
    assert B.shape == (0, 2, 3)


def test_zero_rows_are_safe(cuda_ok):
    """All-zero B rows get scale 0 and contribute nothing (no NaN)."""
    B, eo, ev = mp2_inputs(3, 150, 40, seed=1)
    B[1] = 0
    B[0, 7] = 0
    ref, _ = oracle.mp2_energy_fp64(B.numpy(), eo.numpy(), ev.numpy())
    e = tt.mp2_energy(B.cuda(), eo.cuda(), ev.cuda())
    assert np.isfinite(e.item()) and rel(e.item(), ref) <= 2e-6


@pytest.mark.parametrize("bad", [float("nan"), float("inf")])
def test_nonfinite_input_propagates(cuda_ok, bad):
    """A NaN or inf in B gives a non-finite energy, as fp32 arithmetic on the
    input would (the row's Ozaki scale becomes NaN instead of the bad value
    vanishing from the row maximum)."""
    B, eo, ev = mp2_inputs(3, 150, 40, seed=2)
    B[2, 31, 5] = bad
    e = tt.mp2_energy(B.cuda(), eo.cuda(), ev.cuda())
    assert not np.isfinite(e.item())
    e64 = tt.mp2_energy(B.double().cuda(), eo.double().cuda(), ev.double().cuda())
    assert not np.isfinite(e64.item())


def test_fp64_zero_rows_and_extreme_magnitudes(cuda_ok):
    """fp64 tensor-core path: zero rows contribute nothing, and rows whose
    magnitudes differ by 1e+-20 (each row has its own power-of-two scale)
    stay at fp64 accuracy."""
    B, eo, ev = mp2_inputs(4, 150, 70, seed=5)
    B = B.double()
    B[1] = 0
    B[0, 7] = 0
    B[2, :50] *= 1e20
    B[3, 60:] *= 1e-20
    ref, _ = oracle.mp2_energy_fp64(B.numpy(), eo.double().numpy(), ev.double().numpy())
    e = tt.mp2_energy(B.cuda(), eo.double().cuda(), ev.double().cuda())
    assert np.isfinite(e.item()) and rel(e.item(), ref) <= 1e-12


def test_nonfinite_eri_propagates(cuda_ok):
    """AO->MO: an inf in eri[m, n, P] makes B[:, :, P] non-finite, the other
    aux columns stay finite and match the clean transform."""
    from trntensor_b200.inputs import ao2mo_inputs

    eri, co, cv = ao2mo_inputs(130, 5, 20, 70, seed=3)
    clean = tt.ao_to_mo_transform(eri.cuda(), co.cuda(), cv.cuda()).cpu()
    clean64 = tt.ao_to_mo_transform(eri.double().cuda(), co.double().cuda(),
                                    cv.double().cuda()).cpu()
    eri[17, 40, 9] = float("inf")
    out = tt.ao_to_mo_transform(eri.cuda(), co.cuda(), cv.cuda()).cpu()
    assert not torch.isfinite(out[:, :, 9]).all()
    keep = torch.ones(70, dtype=torch.bool)
    keep[9] = False
    assert torch.equal(out[:, :, keep], clean[:, :, keep])
    out64 = tt.ao_to_mo_transform(eri.double().cuda(), co.double().cuda(),
                                  cv.double().cuda()).cpu()
    assert not torch.isfinite(out64[:, :, 9]).all()
    assert torch.equal(out64[:, :, keep], clean64[:, :, keep])


def test_device_wait_timeout_is_reported(cuda_ok):
    """Failure detection without a GPU fault: a bounded device wait on an
    mbarrier phase that nothing completes gives up after its budget, records
    0x101 in the status word, and the context stays usable (the next energy
    is still correct). The status word raises DeviceError on the host."""
    import ctypes

    from trntensor_b200 import _lib
    from trntensor_b200.dispatch import _check_status

    lib = _lib.load()
    status = torch.full((), 7, dtype=torch.int32, device="cuda")
    cycles = torch.zeros((), dtype=torch.int64, device="cuda")
    budget = 20_000_000  # ~10 ms of SM clock
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    _lib.check(lib.tt_debug_wait_timeout(ctypes.c_void_p(status.data_ptr()), budget,
                                         ctypes.c_void_p(cycles.data_ptr()), stream),
               "tt_debug_wait_timeout")
    torch.cuda.synchronize()
    assert int(status.item()) == 0x101
    assert budget <= int(cycles.item()) < 50 * budget
    with pytest.raises(_lib.DeviceError):
        _check_status(status, "wait")
    with pytest.raises(ValueError):
        _lib.check(lib.tt_debug_wait_timeout(ctypes.c_void_p(status.data_ptr()), -1,
                                             ctypes.c_void_p(cycles.data_ptr()), stream), "x")
    B, eo, ev = mp2_inputs(3, 150, 40, seed=9)
    ref, _ = oracle.mp2_energy_fp64(B.numpy(), eo.numpy(), ev.numpy())
    e = tt.mp2_energy(B.cuda(), eo.cuda(), ev.cuda())
    assert rel(e.item(), ref) <= 2e-6
