"""``einsum`` / ``multi_einsum``, drop-in for trntensor/einsum.py.

Host-side Python like the reference (trntensor/einsum.py:51-241): optional
dtype cast, planning through :mod:`trntensor_b200.plan`, cuTENSOR-style
``alpha``/``beta``/``out`` post-ops and the ``precision=`` semantics
(``"kahan"`` = contract in fp64, cast back to the input dtype; ``"dd"``
raises ``NotImplementedError``). Strategies execute with torch on the
operands' device (cuBLAS for CUDA tensors).
"""

from __future__ import annotations

import torch

from .plan import ContractionPlan, _parse_subscripts, plan_contraction

_DTYPES: dict[str, torch.dtype] = {
    "bf16": torch.bfloat16,
    "bfloat16": torch.bfloat16,
    "fp16": torch.float16,
    "float16": torch.float16,
    "f32": torch.float32,
    "float32": torch.float32,
    "f64": torch.float64,
    "float64": torch.float64,
}


def _resolve_dtype(dtype: str | torch.dtype | None) -> torch.dtype | None:
    if dtype is None or isinstance(dtype, torch.dtype):
        return dtype
    try:
        return _DTYPES[dtype.lower()]
    except KeyError:
        raise ValueError(f"unknown dtype {dtype!r}; valid strings: {sorted(_DTYPES)}") from None


def einsum(
    subscripts: str,
    *operands: torch.Tensor,
    alpha: float = 1.0,
    beta: float = 0.0,
    out: torch.Tensor | None = None,
    dtype: str | torch.dtype | None = None,
    precision: str = "fast",
) -> torch.Tensor:
    """Einstein summation with contraction planning.

    Returns ``alpha * contract(operands) + beta * out`` (``out`` optional).
    """
    target = _resolve_dtype(dtype)
    if target is not None:
        operands = tuple(op.to(target) for op in operands)
    plan = plan_contraction(subscripts, *operands, precision=precision)
    result = _execute(subscripts, operands, plan)
    if alpha != 1.0:
        result = result.mul(alpha)
    if out is not None:
        result = result.add(out, alpha=beta)
    return result


def _ao2mo_roles(subscripts: str, operands: tuple):
    """Match the 3-operand AO->MO transform "mi,na,mnP->iaP" (any letters).

    Returns (eri_index, occ_index, vir_index) into ``operands`` when the
    contraction is sum_{m,n} Cocc[m,i] Cvir[n,a] eri[m,n,P] -> out[i,a,P],
    else None.
    """
    if len(operands) != 3 or "->" not in subscripts:
        return None
    lhs, out = subscripts.split("->")
    terms = lhs.split(",")
    three = [k for k, t in enumerate(terms) if len(t) == 3]
    if len(three) != 1 or len(out) != 3 or len(set("".join(terms))) != 5:
        return None
    e = three[0]
    m, n, P = terms[e]
    occ = next((k for k, t in enumerate(terms) if k != e and len(t) == 2 and t[0] == m), None)
    vir = next((k for k, t in enumerate(terms) if k != e and len(t) == 2 and t[0] == n), None)
    if occ is None or vir is None or occ == vir:
        return None
    if out != terms[occ][1] + terms[vir][1] + P:
        return None
    return e, occ, vir


def _execute(subscripts: str, operands: tuple, plan: ContractionPlan) -> torch.Tensor:
    roles = _ao2mo_roles(subscripts, operands)
    if (
        roles is not None
        and plan.precision in ("fast", "kahan")
        and all(op.device.type == "cuda" for op in operands)
        and all(op.dtype in (torch.float32, torch.float64) for op in operands)
    ):
        # The planner's greedy order would materialise the (m,i,n,a) outer
        # product first; run the two-step tensor-core transform instead.
        from .quantum import ao_to_mo_transform

        e, occ, vir = roles
        return ao_to_mo_transform(operands[e], operands[occ], operands[vir],
                                  precision=plan.precision)
    if plan.precision == "kahan":
        dt = operands[0].dtype if operands else torch.float32
        return torch.einsum(subscripts, *(op.to(torch.float64) for op in operands)).to(dt)
    if plan.precision == "dd":
        raise NotImplementedError(
            "precision='dd' (double-double accumulation) is not available; "
            "use precision='kahan' (fp64 accumulation) as an alternative."
        )
    if plan.strategy == "matmul":
        A, B = operands
        a, b = (A.T if plan.transA else A), (B.T if plan.transB else B)
        if _tensor_core_ok(plan, a, b):
            from .dispatch import _cuda_gemm

            return _cuda_gemm(a, b)
        return torch.matmul(a, b)
    if plan.strategy == "bmm":
        if _tensor_core_ok(plan, *operands):
            from .dispatch import _cuda_gemm

            return _cuda_gemm(*operands)
        return torch.bmm(*operands)
    if plan.strategy == "path":
        return _execute_path(subscripts, operands, plan)
    return torch.einsum(subscripts, *operands)


def _tensor_core_ok(plan: ContractionPlan, *ops: torch.Tensor) -> bool:
    """matmul/bmm plans on CUDA fp32 operands run on the int8 tensor-core GEMM."""
    from .dispatch import OZAKI_MAX_K

    return (
        plan.backend == "cuda"
        and all(op.device.type == "cuda" and op.dtype == torch.float32 for op in ops)
        and ops[0].shape[-1] <= OZAKI_MAX_K
    )


def _execute_path(subscripts: str, operands: tuple, plan: ContractionPlan) -> torch.Tensor:
    """Walk ``plan.contraction_path``; each step is a binary ``einsum`` call of
    this module (as trntensor/einsum.py:151-158 does), so a matmul- or
    bmm-shaped step gets its own plan and executor."""
    lhs, out = _parse_subscripts(subscripts)
    terms = lhs.split(",")
    ops = list(operands)
    steps = plan.contraction_path
    for n, (x, y) in enumerate(steps):
        if n == len(steps) - 1:
            res_term = out
        else:
            later = set(out).union(*(set(t) for k, t in enumerate(terms) if k not in (x, y)))
            res_term = "".join(dict.fromkeys(c for c in terms[x] + terms[y] if c in later))
        res = einsum(f"{terms[x]},{terms[y]}->{res_term}", ops[x], ops[y],
                     precision=plan.precision)
        ops = [o for k, o in enumerate(ops) if k not in (x, y)] + [res]
        terms = [t for k, t in enumerate(terms) if k not in (x, y)] + [res_term]
    return ops[0]


def multi_einsum(*contractions: tuple) -> list[torch.Tensor]:
    """Run several contractions; each is ``(subscripts, *operands)``.

    Host tensors used by more than one contraction are moved to the CUDA
    device once when any operand of the batch already lives there (the B200
    counterpart of the reference's shared-operand XLA pinning,
    trntensor/einsum.py:196-241). Results come back on their inputs' device.
    """
    counts: dict[int, int] = {}
    for c in contractions:
        for op in c[1:]:
            counts[id(op)] = counts.get(id(op), 0) + 1
    cuda_dev = next(
        (op.device for c in contractions for op in c[1:] if op.device.type == "cuda"), None
    )
    moved: dict[int, torch.Tensor] = {}
    if cuda_dev is not None:
        for c in contractions:
            for op in c[1:]:
                if counts[id(op)] > 1 and op.device.type == "cpu" and id(op) not in moved:
                    moved[id(op)] = op.to(cuda_dev)
    results = []
    for c in contractions:
        ops = tuple(moved.get(id(op), op) for op in c[1:])
        res = einsum(c[0], *ops)
        if any(id(op) in moved for op in c[1:]) and all(
            op.device.type == "cpu" for op in c[1:]
        ):
            res = res.cpu()
        results.append(res)
    return results
