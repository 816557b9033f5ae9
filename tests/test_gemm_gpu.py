"""einsum's matmul / bmm strategies on the GPU (int8 tensor-core GEMM) against
fp64 references, for every operand layout the planner produces."""

from __future__ import annotations

import pytest
import torch

import trntensor_b200 as tt
from trntensor_b200.dispatch import _cuda_gemm

pytestmark = pytest.mark.gpu


def check(got, ref, tol=1e-5):
    err = (got.double() - ref).abs().max().item()
    scale = ref.abs().max().item()
    assert err <= tol * max(scale, 1e-30), (err, scale)


@pytest.mark.parametrize("M,N,K", [(128, 128, 64), (100, 200, 70), (1, 1, 1), (300, 257, 1000),
                                   (1792, 1792, 6144), (5, 700, 33)])
@pytest.mark.parametrize("ta,tb", [(False, False), (True, False), (False, True), (True, True)])
def test_gemm_layouts(cuda_ok, M, N, K, ta, tb):
    g = torch.Generator(device="cuda").manual_seed(M + N + K)
    A = torch.randn(K, M, device="cuda", generator=g).T if ta else torch.randn(M, K, device="cuda", generator=g)
    B = torch.randn(N, K, device="cuda", generator=g).T if tb else torch.randn(K, N, device="cuda", generator=g)
    check(_cuda_gemm(A, B), A.double() @ B.double())


def test_bmm(cuda_ok):
    g = torch.Generator(device="cuda").manual_seed(1)
    A = torch.randn(6, 130, 90, device="cuda", generator=g)
    B = torch.randn(6, 90, 200, device="cuda", generator=g)
    check(_cuda_gemm(A, B), torch.bmm(A.double(), B.double()))


def test_einsum_routes_matmul_and_bmm(cuda_ok):
    """einsum("ap,bp->ab") (the DF-MP2 pair GEMM) and "bij,bjk->bik" report
    and use the CUDA backend; results match fp64."""
    g = torch.Generator(device="cuda").manual_seed(2)
    Bi = torch.randn(448, 1536, device="cuda", generator=g) / 40
    Bj = torch.randn(448, 1536, device="cuda", generator=g) / 40
    plan = tt.plan_contraction("ap,bp->ab", Bi, Bj)
    assert plan.strategy == "matmul" and plan.backend == "cuda"
    check(tt.einsum("ap,bp->ab", Bi, Bj), Bi.double() @ Bj.double().T)
    X = torch.randn(4, 50, 60, device="cuda", generator=g)
    Y = torch.randn(4, 60, 70, device="cuda", generator=g)
    assert tt.plan_contraction("bij,bjk->bik", X, Y).backend == "cuda"
    check(tt.einsum("bij,bjk->bik", X, Y), torch.bmm(X.double(), Y.double()))
    tt.set_backend("pytorch")
    try:
        tt.clear_plan_cache()
        assert tt.plan_contraction("ap,bp->ab", Bi, Bj).backend == "pytorch"
    finally:
        tt.set_backend("auto")
        tt.clear_plan_cache()


def test_pair_loop_example_energy(cuda_ok):
    """examples/df_mp2_einsum.py's loop run through trntensor_b200.einsum on
    CUDA tensors reproduces the tutorial energy (docs/tutorial_df_mp2.md:77)."""
    from tests.helpers import ref_recipe_mp2

    B, eo, ev = (t.cuda() for t in ref_recipe_mp2(42, 5, 19, 72))
    e = 0.0
    for i in range(5):
        for j in range(5):
            T = tt.einsum("ap,bp->ab", B[i], B[j])
            d = eo[i] + eo[j] - ev.unsqueeze(1) - ev.unsqueeze(0)
            e += (T * (2 * T - T.T) / d).sum().item()
    assert abs(e - (-50.5432928801)) < 5e-5
