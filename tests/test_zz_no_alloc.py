"""tt_mp2_energy_f32_noalloc: the DF-MP2 energy for callers that cannot
allocate device memory, checked against tt_mp2_energy_f32 (which takes a
caller-allocated workspace) through the C ABI.

Kept in its own file, collected last, so that a failure here never hides the
other tests of a run that stops at the first failure.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from trntensor_b200 import _lib
from trntensor_b200.inputs import mp2_inputs

pytestmark = pytest.mark.gpu

RTOL_F32 = 1e-6  # the energy tolerance of the other fp32 parity tests


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def _energy_with_workspace(lib, B, eo, ev, stream):
    nocc, nvir, naux = B.shape
    ws_bytes = int(lib.tt_mp2_workspace_bytes(nocc, nvir, naux))
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
    e = torch.empty((), dtype=torch.float64, device="cuda")
    st = torch.empty((), dtype=torch.int32, device="cuda")
    rc = lib.tt_mp2_energy_f32(_p(B), _p(eo), _p(ev), nocc, nvir, naux, 0,
                               nocc * (nocc + 1) // 2, _p(ws), ws_bytes, _p(e), None, _p(st),
                               stream)
    assert rc == 0
    torch.cuda.synchronize()
    assert st.item() == 0
    return e.item()


def test_noalloc_matches_workspace_entry_point(cuda_ok):
    lib = _lib.load()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    # two calls in a row on different problems: the second must not see the
    # first one's scratch contents
    for shape, seed in (((6, 200, 150), 21), ((5, 130, 96), 22)):
        B, eo, ev = (t.cuda() for t in mp2_inputs(*shape, seed=seed))
        ref = _energy_with_workspace(lib, B, eo, ev, stream)
        e = torch.empty((), dtype=torch.float64, device="cuda")
        st = torch.empty((), dtype=torch.int32, device="cuda")
        rc = lib.tt_mp2_energy_f32_noalloc(_p(B), _p(eo), _p(ev), *shape, _p(e), None, _p(st),
                                           stream)
        assert rc == 0, lib.tt_status_string(rc)
        torch.cuda.synchronize()
        assert st.item() == 0
        assert abs(e.item() - ref) <= RTOL_F32 * abs(ref)


def test_noalloc_leaves_device_memory_unchanged(cuda_ok):
    """After one warm-up call (which may load the kernels' code), a further
    call changes the device's free memory by nothing: no allocation routine
    runs inside it."""
    lib = _lib.load()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    B, eo, ev = (t.cuda() for t in mp2_inputs(6, 200, 150, seed=23))
    e = torch.empty((), dtype=torch.float64, device="cuda")
    st = torch.empty((), dtype=torch.int32, device="cuda")
    args = (_p(B), _p(eo), _p(ev), 6, 200, 150, _p(e), None, _p(st), stream)
    assert lib.tt_mp2_energy_f32_noalloc(*args) == 0
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    assert lib.tt_mp2_energy_f32_noalloc(*args) == 0
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0
    assert st.item() == 0


def test_noalloc_rejects_oversize(cuda_ok):
    lib = _lib.load()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    dummy = torch.zeros(4, device="cuda")
    e = torch.empty((), dtype=torch.float64, device="cuda")
    st = torch.empty((), dtype=torch.int32, device="cuda")
    # 256 x 1792 x 6144 needs ~8.5 GB of slices, far above the 64 MiB scratch
    rc = lib.tt_mp2_energy_f32_noalloc(_p(dummy), _p(dummy), _p(dummy), 256, 1792, 6144, _p(e),
                                       None, _p(st), stream)
    assert rc == _lib.TT_ERR_WORKSPACE
