"""AO->MO step 1 ring protocol: the 2 fp32 + 3 int8 slot ring
(TRNTENSOR_B200_AO2MO_RING=23) and the default 3 + 2 ring produce
bit-identical tensors, run after run. The arithmetic does not depend on the
ring depth (same digits, same k order, same epilogue and split-K order), so
any difference is a hand-off bug between producers, converters, the MMA
thread and the epilogue. Config 1 (no fused scales: nbf = 128 is two
k-chunks) and a 2-GB config-3 slab (nbf 1024, naux 512; fused scales and
split-K over CTA pairs) each run 200 times."""

from __future__ import annotations

import pytest
import torch

from trntensor_b200.dispatch import _cuda_ao_to_mo_transform
from trntensor_b200.inputs import ao2mo_inputs

pytestmark = pytest.mark.gpu

REPEATS = 200


@pytest.mark.parametrize("shape", [(128, 16, 112, 384), (1024, 128, 896, 512)])
def test_ring_depths_bitwise_identical(cuda_ok, shape, monkeypatch):
    nbf, nocc, nvir, naux = shape
    eri, co, cv = ao2mo_inputs(nbf, nocc, nvir, naux, seed=21, device="cuda")
    monkeypatch.delenv("TRNTENSOR_B200_AO2MO_RING", raising=False)
    ref = _cuda_ao_to_mo_transform(eri, co, cv)
    ref64 = _cuda_ao_to_mo_transform(eri.double(), co.double(), cv.double())
    err = ((ref.double() - ref64).abs().max() / ref64.abs().max()).item()
    assert err <= 1e-5
    del ref64
    for ring in ("32", "23"):
        monkeypatch.setenv("TRNTENSOR_B200_AO2MO_RING", ring)
        bad = 0
        for _ in range(REPEATS):
            out = _cuda_ao_to_mo_transform(eri, co, cv)
            bad += int(not torch.equal(out, ref))
        assert bad == 0, f"ring {ring}: {bad} of {REPEATS} runs differ"
