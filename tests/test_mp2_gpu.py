"""DF-MP2 energy on the GPU against the reference's numbers (golden vectors,
the CPU oracle, and size-independent properties at the benchmark sizes).

Tolerances (north star): fp32 inputs via 3xTF32 |dE|/|E| <= 1e-6 against the
fp64 reference; fp64 path |dE|/|E| <= 1e-12.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

import trntensor_b200 as tt
from oracle import oracle
from tests.helpers import MP2_CASES, mp2_case_inputs
from trntensor_b200 import _lib
from trntensor_b200.dispatch import _cuda_mp2_energy
from trntensor_b200.inputs import mp2_inputs

pytestmark = pytest.mark.gpu

RTOL_F32 = 1e-6
RTOL_F64 = 1e-12


def rel(a, b):
    return abs(float(a) - float(b)) / abs(float(b))


@pytest.mark.parametrize("name", MP2_CASES)
def test_tc_energy_matches_reference(golden, cuda_ok, name):
    B, eo, ev = mp2_case_inputs(golden, name)
    e = tt.mp2_energy(B.cuda(), eo.cuda(), ev.cuda())
    assert e.device.type == "cuda" and e.dtype == torch.float32 and e.shape == ()
    e64, _ = _cuda_mp2_energy(B, eo, ev)
    assert rel(e64.item(), golden[f"{name}/e_fp64"]) <= RTOL_F32
    # also within the reference's own fp32 result's distance from fp64
    assert rel(e.item(), golden[f"{name}/e_fp32"]) <= 2e-6


@pytest.mark.parametrize("name", MP2_CASES)
def test_tc_pair_energies(golden, cuda_ok, name):
    B, eo, ev = mp2_case_inputs(golden, name)
    part = tt.mp2_pair_energies(B.cuda(), eo.cuda(), ev.cuda()).cpu().numpy()
    ref = golden[f"{name}/pair_fp64"]
    np.testing.assert_allclose(part, ref, rtol=1e-5, atol=1e-6 * np.abs(ref).max())
    assert rel(part.sum(), ref.sum()) <= RTOL_F32


@pytest.mark.parametrize("name", MP2_CASES)
def test_fp64_path(golden, cuda_ok, name):
    B, eo, ev = mp2_case_inputs(golden, name)
    e = tt.mp2_energy(B.double().cuda(), eo.double().cuda(), ev.double().cuda())
    assert e.dtype == torch.float64
    assert rel(e.item(), golden[f"{name}/e_fp64"]) <= RTOL_F64
    ek = tt.mp2_energy(B.cuda(), eo.cuda(), ev.cuda(), precision="kahan")
    assert ek.dtype == torch.float32
    assert rel(ek.item(), golden[f"{name}/e_fp64"]) <= 1e-7
    part = tt.mp2_pair_energies(B.double(), eo.double(), ev.double()).numpy()
    np.testing.assert_allclose(part, golden[f"{name}/pair_fp64"], rtol=1e-11, atol=1e-15)


@pytest.mark.parametrize("name", MP2_CASES)
def test_simt_cross_check(golden, cuda_ok, name):
    B, eo, ev = mp2_case_inputs(golden, name)
    e, _ = _cuda_mp2_energy(B, eo, ev, kernel="simt")
    assert rel(e.item(), golden[f"{name}/e_fp64"]) <= 1e-5


def test_host_tensors_round_trip(golden, cuda_ok):
    """Host inputs: copied to the device, result returned on the host."""
    B, eo, ev = mp2_case_inputs(golden, "kat_demo")
    e = tt.mp2_energy(B, eo, ev)
    assert e.device.type == "cpu" and e.dtype == torch.float32
    assert abs(e.item() - (-50.5432928801)) < 5e-5  # docs/tutorial_df_mp2.md:77


def test_pair_ranges_add_up(cuda_ok):
    B, eo, ev = mp2_inputs(13, 150, 70, seed=3)
    tot, _ = _cuda_mp2_energy(B, eo, ev)
    npairs = 13 * 14 // 2
    cuts = [0, 1, 17, 50, 90, npairs]
    parts = [_cuda_mp2_energy(B, eo, ev, pair_range=(a, b))[0].item() for a, b in zip(cuts, cuts[1:])]
    assert rel(sum(parts), tot.item()) <= 1e-12
    e_empty, _ = _cuda_mp2_energy(B, eo, ev, pair_range=(5, 5))
    assert e_empty.item() == 0.0


def test_capi_presplit_direct(cuda_ok):
    """tt_split_i8 + tt_mp2_energy_presplit_i8 through ctypes."""
    lib = _lib.load()
    B, eo, ev = mp2_inputs(6, 130, 48, seed=5)
    Bd, eod, evd = B.cuda(), eo.cuda(), ev.cuda()
    nocc, nvir, naux = B.shape
    pad = 64
    q = torch.empty(3, nocc * nvir, pad, dtype=torch.int8, device="cuda")
    sc = torch.empty(nocc * nvir, dtype=torch.float32, device="cuda")
    s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    p = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    assert lib.tt_split_i8(p(Bd), p(q), p(sc), nocc * nvir, naux, pad, s) == 0
    energy = torch.empty((), dtype=torch.float64, device="cuda")
    status = torch.empty((), dtype=torch.int32, device="cuda")
    st = lib.tt_mp2_energy_presplit_i8(p(q), p(sc), pad, p(eod), p(evd), nocc, nvir, 0,
                                       nocc * (nocc + 1) // 2, p(energy), None, p(status), s)
    assert st == 0
    torch.cuda.synchronize()
    assert status.item() == 0
    ref, _ = oracle.mp2_energy_fp64(B.numpy(), eo.numpy(), ev.numpy())
    assert rel(energy.item(), ref) <= RTOL_F32
    # bad arguments are rejected before launch
    assert lib.tt_mp2_energy_presplit_i8(p(q), p(sc), 40, p(eod), p(evd), nocc, nvir, 0, 1,
                                         p(energy), None, p(status), s) == 2


def test_config2_against_oracle(cuda_ok):
    """BASELINE config 2 (64, 448, 1536), full energy vs the fp64 CPU oracle."""
    B, eo, ev = mp2_inputs(64, 448, 1536, seed=0)
    e = tt.mp2_energy(B.cuda(), eo.cuda(), ev.cuda())
    e64d, _ = _cuda_mp2_energy(B.double(), eo.double(), ev.double())
    ref, _ = oracle.mp2_energy_fp64(B.numpy(), eo.numpy(), ev.numpy())
    assert rel(e64d.item(), ref) <= RTOL_F64
    e_tc, _ = _cuda_mp2_energy(B, eo, ev)
    assert rel(e_tc.item(), ref) <= RTOL_F32
    assert rel(e.item(), ref) <= 2e-6


def test_config4_sampled_pairs(cuda_ok):
    """BASELINE config 4 (256, 1792, 6144): full-size tiles, checked on pair
    ranges against the device fp64 kernel and on single pairs against the CPU
    oracle (the full fp64 CPU sum would take hours)."""
    nocc, nvir, naux = 256, 1792, 6144
    B, eo, ev = mp2_inputs(nocc, nvir, naux, seed=11, device="cuda")
    npairs = nocc * (nocc + 1) // 2
    for pb in (0, 255, npairs // 2, npairs - 40):
        rng = (pb, pb + 40)
        e_tc, part = _cuda_mp2_energy(B, eo, ev, pair_range=rng, return_partials=True)
        e_64, part64 = _cuda_mp2_energy(B.double(), eo.double(), ev.double(), pair_range=rng,
                                        return_partials=True)
        assert rel(e_tc.item(), e_64.item()) <= RTOL_F32
        torch.testing.assert_close(part, part64, rtol=2e-6, atol=0)
        assert rel(part.sum().item() * 0 + e_tc.item(), e_64.item()) <= RTOL_F32
    # single pairs against the CPU oracle (fp64)
    Bc, eoc, evc = B.cpu().numpy(), eo.cpu().numpy(), ev.cpu().numpy()
    i_idx = np.triu_indices(nocc)
    for pid in (0, 1000, npairs - 1):
        i, j = int(i_idx[0][pid]), int(i_idx[1][pid])
        ref = oracle.mp2_pair_energy(Bc, eoc, evc, i, j, np.float64)
        _, part = _cuda_mp2_energy(B, eo, ev, pair_range=(pid, pid + 1), return_partials=True)
        assert rel(part[i, j].item(), ref) <= 1e-6


@pytest.mark.parametrize("shape", [(256, 1792, 6144), (5, 300, 1000), (3, 129, 32704)])
def test_fp64_tensor_core_vs_cuda_core(cuda_ok, shape):
    """fp64 energy (precision="kahan"): the five-digit int8 tensor-core kernel
    and the CUDA-core fp64 kernel agree to 1e-12 on every pair kind (i == j,
    i < j, diagonal and off-diagonal blocks) and in the per-pair partials;
    config 4 is checked on pair ranges; naux 32704 is the longest contraction
    the int32 sums allow."""
    nocc, nvir, naux = shape
    B, eo, ev = mp2_inputs(nocc, nvir, naux, seed=21, device="cuda")
    B, eo, ev = B.double(), eo.double(), ev.double()
    npairs = nocc * (nocc + 1) // 2
    ranges = [(0, npairs)] if npairs <= 64 else [(0, 3), (255, 260), (npairs - 4, npairs)]
    for rng in ranges:
        e_tc, p_tc = _cuda_mp2_energy(B, eo, ev, pair_range=rng, return_partials=True)
        e_s, p_s = _cuda_mp2_energy(B, eo, ev, pair_range=rng, return_partials=True,
                                    kernel="simt")
        assert rel(e_tc.item(), e_s.item()) <= RTOL_F64
        torch.testing.assert_close(p_tc, p_s, rtol=1e-11, atol=1e-14 * p_s.abs().max().item())


def test_ozaki_split_is_exact_to_22_bits(cuda_ok):
    """tt_split_i8: x == s (q1 + q2/2^8 + q3/2^16) up to half a unit of the last slice."""
    lib = _lib.load()
    B, _, _ = mp2_inputs(3, 50, 100, seed=9)
    rows, cols, pad = 150, 100, 128
    Bd = B.cuda().reshape(rows, cols)
    q = torch.empty(3, rows, pad, dtype=torch.int8, device="cuda")
    s = torch.empty(rows, dtype=torch.float32, device="cuda")
    st = lib.tt_split_i8(ctypes.c_void_p(Bd.data_ptr()), ctypes.c_void_p(q.data_ptr()),
                         ctypes.c_void_p(s.data_ptr()), rows, cols, pad,
                         ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == 0
    torch.cuda.synchronize()
    qd = q.double()
    rec = s.double()[:, None] * (qd[0] + qd[1] / 256 + qd[2] / 65536)
    err = (rec[:, :cols] - Bd.double()).abs()
    assert (err <= 0.5 * s.double()[:, None] / 65536 * 1.0001).all()
    assert (q[:, :, cols:] == 0).all()
    assert (q[0].abs() <= 64).all()
    # s = 2^(e-6) with max|x| < 2^e: the largest element of each row has |q1| in [32, 64]
    top = (Bd.abs() / s[:, None]).amax(dim=1)
    assert ((top >= 32) & (top < 64)).all()
    # scales are powers of two
    m, e = torch.frexp(s)
    assert (m == 0.5).all()


def test_tf32x3_diagnostic_is_biased(cuda_ok):
    """The 3xTF32 tensor-core variant loses ~2e-8 relative per 8 aux elements
    (fp32 accumulation rounds toward zero); the int8 path does not."""
    B, eo, ev = mp2_inputs(4, 256, 2048, seed=1, device="cuda")
    e64, _ = _cuda_mp2_energy(B.double(), eo.double(), ev.double())
    e_tf, _ = _cuda_mp2_energy(B, eo, ev, kernel="tf32x3")
    e_i8, _ = _cuda_mp2_energy(B, eo, ev)
    assert rel(e_tf.item(), e64.item()) > 5e-6
    assert rel(e_i8.item(), e64.item()) < RTOL_F32


@pytest.mark.parametrize("shape", [(5, 300, 100), (4, 257, 70), (3, 128, 64), (7, 640, 200)])
def test_paired_sm_kernel(cuda_ok, shape, monkeypatch):
    """The opt-in cta_group::2 kernel (TRNTENSOR_B200_MP2_2SM=1) gives the
    same energies and pair energies as the fp64 oracle."""
    B, eo, ev = mp2_inputs(*shape, seed=sum(shape))
    ref, part = oracle.mp2_energy_fp64(B.numpy(), eo.numpy(), ev.numpy())
    monkeypatch.setenv("TRNTENSOR_B200_MP2_2SM", "1")
    e, p = _cuda_mp2_energy(B, eo, ev, return_partials=True)
    assert rel(e.item(), ref) <= RTOL_F32
    np.testing.assert_allclose(p.cpu().numpy(), part, rtol=1e-5, atol=1e-7 * np.abs(part).max())
    npairs = shape[0] * (shape[0] + 1) // 2
    e1, _ = _cuda_mp2_energy(B, eo, ev, pair_range=(1, npairs))
    e0, _ = _cuda_mp2_energy(B, eo, ev, pair_range=(0, 1))
    assert rel(e0.item() + e1.item(), ref) <= RTOL_F32


def test_host_pipelined_copy(cuda_ok):
    """Pinned host B: copy overlapped with compute in row chunks (last rows
    first); same energy as the device-resident path, also on pair ranges."""
    from trntensor_b200.dispatch import first_row_of_pair, pair_offset

    nocc = 37
    for p in range(nocc * (nocc + 1) // 2):
        i = first_row_of_pair(p, nocc)
        assert pair_offset(i, nocc) <= p < pair_offset(i + 1, nocc)
    B, eo, ev = mp2_inputs(nocc, 300, 130, seed=4)
    Bp = B.pin_memory()
    ref, _ = _cuda_mp2_energy(B.cuda(), eo, ev)
    e, _ = _cuda_mp2_energy(Bp, eo, ev)
    assert rel(e.item(), ref.item()) <= 1e-12
    e_pub = tt.mp2_energy(Bp, eo, ev)
    assert e_pub.device.type == "cpu" and rel(e_pub.item(), ref.item()) <= 1e-6
    npairs = nocc * (nocc + 1) // 2
    for rng in ((0, 100), (100, 550), (550, npairs), (5, 6)):
        a, _ = _cuda_mp2_energy(Bp, eo, ev, pair_range=rng)
        b, _ = _cuda_mp2_energy(B.cuda(), eo, ev, pair_range=rng)
        assert abs(a.item() - b.item()) <= 1e-12 * abs(ref.item())


@pytest.mark.parametrize("world", [4, 8])
def test_host_block_plan_ranks_sum_to_energy(cuda_ok, world):
    """Row-group blocks (the pair assignment of a host-resident B at 4 and 8
    ranks): the ranks' energies, each run through the pipelined host copy in
    its chunk order and, from a device copy, range by range, sum to the full
    energy."""
    from trntensor_b200.dispatch import block_assignment

    nocc = 37
    B, eo, ev = mp2_inputs(nocc, 300, 130, seed=6)
    Bp = B.pin_memory()
    ref, _ = _cuda_mp2_energy(B.cuda(), eo, ev)
    tot_host = tot_dev = 0.0
    for rank in range(world):
        blocks = block_assignment(nocc, rank, world)
        a, _ = _cuda_mp2_energy(Bp, eo, ev, blocks=blocks)
        b, _ = _cuda_mp2_energy(B.cuda(), eo, ev, blocks=blocks)
        assert abs(a.item() - b.item()) <= 1e-12 * abs(ref.item())
        tot_host += a.item()
        tot_dev += b.item()
    assert rel(tot_host, ref.item()) <= 1e-12
    assert rel(tot_dev, ref.item()) <= 1e-12
