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


def gemm_bound(A, B):
    """The tensor-core GEMM's error bound per output element (one scale per
    row of A and per column of B): 2^-19 (M_i |B_:j|_1 + |A_i:|_1 M_j)
    + 2^-20 sqrt(K) M_i M_j with M the row / column largest magnitudes."""
    A, B = A.double(), B.double()
    K = A.shape[-1]
    Mi = A.abs().amax(-1, keepdim=True)
    Mj = B.abs().amax(-2, keepdim=True)
    return (2.0**-19 * (Mi * B.abs().sum(-2, keepdim=True) + A.abs().sum(-1, keepdim=True) * Mj)
            + 2.0**-20 * K**0.5 * Mi * Mj)


@pytest.mark.parametrize("K", [14, 906, 2760])
def test_gemm_mixed_magnitudes_elementwise(cuda_ok, K):
    """Rows of A and columns of B whose entries span six decades along K
    (a fresh permutation per row), a one-spike row and a column with one
    large entry over tiny ones: every output element stays within the stated
    per-row / per-column bound, checked elementwise against fp64."""
    g = torch.Generator().manual_seed(K)
    M, N = 40, 50
    decades = torch.logspace(-6, 0, K, dtype=torch.float64)
    A = torch.randn(M, K, generator=g, dtype=torch.float64)
    A *= torch.stack([decades[torch.randperm(K, generator=g)] for _ in range(M)])
    B = torch.randn(K, N, generator=g, dtype=torch.float64) * decades[:, None]
    A[3] = 0
    A[3, K // 2] = 7.0
    B[:, 5] *= 1e-3
    B[K // 3, 5] = 50.0
    A, B = A.float(), B.float()
    ref = A.double() @ B.double()
    got = _cuda_gemm(A.cuda(), B.cuda()).double().cpu()
    ratio = ((got - ref).abs() / gemm_bound(A, B)).max().item()
    assert ratio <= 1.0, ratio
    # transposed storage of the same operands gives the same bound
    got_t = _cuda_gemm(A.T.contiguous().cuda().T, B.T.contiguous().cuda().T).double().cpu()
    assert ((got_t - ref).abs() / gemm_bound(A, B)).max().item() <= 1.0


def test_gemm_tiny_and_nonfinite_rows(cuda_ok):
    """A row whose largest magnitude is below 1e-30 gives an exact zero output
    row; an inf in A makes that output row NaN (the row's scale is NaN); the
    other rows are unaffected."""
    g = torch.Generator().manual_seed(5)
    A = torch.randn(6, 70, generator=g)
    B = torch.randn(70, 9, generator=g)
    A[1] *= 1e-32
    A[4, 3] = float("inf")
    got = _cuda_gemm(A.cuda(), B.cuda()).cpu()
    assert torch.equal(got[1], torch.zeros(9))
    assert torch.isnan(got[4]).all()
    keep = [0, 2, 3, 5]
    ref = A[keep].double() @ B.double()
    assert ((got[keep].double() - ref).abs() / gemm_bound(A[keep], B)).max().item() <= 1.0


def test_einsum_default_is_torch_elementwise(cuda_ok):
    """The default backend ("auto") contracts CUDA fp32 operands with torch
    (cuBLAS fp32), as the reference does: elementwise fp32 rounding, inf
    stays inf."""
    A = torch.randn(30, 40, device="cuda")
    B = torch.randn(40, 20, device="cuda")
    A[2, 5] = float("inf")
    assert tt.plan_contraction("ik,kj->ij", A, B).backend == "pytorch"
    torch.testing.assert_close(tt.einsum("ik,kj->ij", A, B), A @ B, equal_nan=True)


def test_einsum_routes_matmul_and_bmm(cuda_ok):
    """With set_backend("cuda"), einsum("ap,bp->ab") (the DF-MP2 pair GEMM) and
    "bij,bjk->bik" report and use the tensor-core GEMM; results match fp64."""
    tt.set_backend("cuda")
    tt.clear_plan_cache()
    try:
        _routes()
    finally:
        tt.set_backend("auto")
        tt.clear_plan_cache()


def _routes():
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
    tt.clear_plan_cache()
    assert tt.plan_contraction("ap,bp->ab", Bi, Bj).backend == "pytorch"
    tt.set_backend("auto")
    tt.clear_plan_cache()
    assert tt.plan_contraction("ap,bp->ab", Bi, Bj).backend == "pytorch"


def test_einsum_product_orders_on_tensor_cores(cuda_ok):
    """Under set_backend("cuda") every index order of a matmul- or
    bmm-shaped contraction reaches the tensor-core GEMM with the operands
    brought into canonical form, and matches fp64 torch.einsum."""
    g = torch.Generator(device="cuda").manual_seed(4)
    A2 = torch.randn(70, 50, device="cuda", generator=g)   # (k, i)
    B2 = torch.randn(60, 70, device="cuda", generator=g)   # (l, k)
    X = torch.randn(50, 4, 60, device="cuda", generator=g)  # (i, b, j)
    Y = torch.randn(70, 60, 4, device="cuda", generator=g)  # (k, j, b)
    cases = [("ki,lk->il", A2, B2), ("ki,lk->li", A2, B2),
             ("ibj,kjb->bki", X, Y), ("ibj,kjb->ikb", X, Y)]
    tt.set_backend("cuda")
    tt.clear_plan_cache()
    try:
        import trntensor_b200.dispatch as dp

        for sub, a, b in cases:
            calls = []
            real = dp._cuda_gemm
            dp._cuda_gemm = lambda *x: calls.append(x) or real(*x)  # noqa: E731
            try:
                got = tt.einsum(sub, a, b)
            finally:
                dp._cuda_gemm = real
            ref = torch.einsum(sub, a.double(), b.double())
            assert len(calls) == 1 and got.shape == ref.shape, sub
            check(got, ref)
    finally:
        tt.set_backend("auto")
        tt.clear_plan_cache()


def test_path_steps_route_through_einsum(cuda_ok):
    """A 4-operand chain: the planner avoids outer products, and each binary
    step is planned again, so matmul-shaped steps reach the tensor-core GEMM
    under set_backend("cuda")."""
    g = torch.Generator(device="cuda").manual_seed(3)
    ops = [torch.randn(n, m, device="cuda", generator=g) for n, m in
           ((60, 70), (70, 80), (80, 90), (90, 30))]
    ref = ops[0].double() @ ops[1].double() @ ops[2].double() @ ops[3].double()
    tt.set_backend("cuda")
    tt.clear_plan_cache()
    try:
        import trntensor_b200.dispatch as dp

        calls = []
        real = dp._cuda_gemm
        dp._cuda_gemm = lambda *a: calls.append(a) or real(*a)  # noqa: E731
        try:
            got = tt.einsum("ij,jk,kl,lm->im", *ops)
        finally:
            dp._cuda_gemm = real
        assert len(calls) == 3
        check(got, ref)
    finally:
        tt.set_backend("auto")
        tt.clear_plan_cache()


def test_multi_einsum_on_gpu(cuda_ok):
    """multi_einsum with a shared host operand and CUDA operands: the shared
    operand moves to the device once and every result matches fp64."""
    g = torch.Generator().manual_seed(4)
    Bsh = torch.randn(64, 96, generator=g)
    X = torch.randn(64, 50, generator=g).cuda()
    Y = torch.randn(96, 40, generator=g).cuda()
    r1, r2 = tt.multi_einsum(("ap,ai->pi", Bsh, X), ("ap,pj->aj", Bsh, Y))
    assert r1.device.type == "cuda" and r2.device.type == "cuda"
    check(r1.cpu(), Bsh.double().T @ X.double().cpu())
    check(r2.cpu(), Bsh.double() @ Y.double().cpu())


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
