"""``einsum`` / ``multi_einsum``, drop-in for trntensor/einsum.py.

Host-side Python like the reference (trntensor/einsum.py:51-241): optional
dtype cast, planning through :mod:`trntensor_b200.plan`, cuTENSOR-style
``alpha``/``beta``/``out`` post-ops and the ``precision=`` semantics
(``"kahan"`` = contract in fp64, cast back to the input dtype; ``"dd"`` =
contract in double-double on the GPU, cast back to the input dtype).
Strategies execute with torch on the operands' device (cuBLAS for CUDA
tensors) unless ``set_backend("cuda")`` selects the tensor-core GEMM.
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
        dt = operands[0].dtype if operands else torch.float32
        return _einsum_dd(subscripts, operands, plan).to(device=operands[0].device, dtype=dt)
    if plan.strategy in ("matmul", "bmm"):
        # Operands are brought into the canonical ([batch,] free, k) @
        # ([batch,] k, free) form and the product into the requested output
        # order. The plan's transA/transB flags (as the reference records
        # them) only say where the contracted index sits; the reference's
        # executors (trntensor/einsum.py:129-148) stop there, which returns
        # (l, i) for 'kl,ik->il' and multiplies bmm operands as stored
        # whatever their index order. Here every matmul- or bmm-shaped
        # contraction gives torch.einsum's result.
        pair = _canonical_pair(subscripts, operands, plan)
        if pair is None:  # repeated or summed-out free indices: not a plain product
            return torch.einsum(subscripts, *operands)
        a, b, perm = pair
        if _tensor_core_ok(plan, a, b):
            from .dispatch import _cuda_gemm

            r = _cuda_gemm(a, b)
        else:
            r = torch.matmul(a, b)
        return r if perm is None else r.permute(perm).contiguous()
    if plan.strategy == "path":
        return _execute_path(subscripts, operands, plan)
    return torch.einsum(subscripts, *operands)


def _canonical_pair(subscripts: str, operands: tuple, plan: ContractionPlan):
    """(a, b, perm): a = A as ([batch,] free_a, k), b = B as ([batch,] k,
    free_b), and the permutation from the product's ([batch,] free_a,
    free_b) order to the output's (None when it is already in order); None
    when the contraction is not a plain (batched) product of distinct
    indices."""
    lhs, out = _parse_subscripts(subscripts)
    ta, tb = lhs.split(",")
    A, B = operands
    k = plan.contraction_indices[0]
    bt = plan.batch_indices[0] if plan.strategy == "bmm" else None
    if len(set(ta)) != len(ta) or len(set(tb)) != len(tb) or len(set(out)) != len(out):
        return None
    fa = [c for c in ta if c not in (k, bt)]
    fb = [c for c in tb if c not in (k, bt)]
    if len(fa) != 1 or len(fb) != 1 or fa == fb:
        return None
    fa, fb = fa[0], fb[0]
    if set(out) != {fa, fb} | ({bt} if bt is not None else set()):
        return None
    lead = [bt] if bt is not None else []
    order_a = lead + [fa, k]
    order_b = lead + [k, fb]
    a = A.permute([ta.index(c) for c in order_a])
    b = B.permute([tb.index(c) for c in order_b])
    prod = lead + [fa, fb]
    perm = [prod.index(c) for c in out]
    return a, b, (None if perm == list(range(len(prod))) else perm)


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


def _dd_reduce(hi, lo, term: str, keep: set):
    """Sum a double-double operand over its indices not in ``keep`` (a
    contraction with a ones vector, in double-double). Returns (hi, lo, term)."""
    from .dispatch import _cuda_bmm_dd

    drop = [c for c in term if c not in keep]
    if not drop:
        return hi, lo, term
    rest = [c for c in term if c in keep]
    perm = [term.index(c) for c in rest + drop]
    shp = [hi.shape[term.index(c)] for c in rest]
    k = 1
    for c in drop:
        k *= hi.shape[term.index(c)]
    r = 1
    for n in shp:
        r *= n
    h = hi.permute(perm).reshape(1, r, k)
    l_ = None if lo is None else lo.permute(perm).reshape(1, r, k)
    ones = torch.ones((1, k, 1), dtype=torch.float64, device=hi.device)
    ch, cl = _cuda_bmm_dd(h, l_, ones, None)
    return ch.reshape(shp), cl.reshape(shp), "".join(rest)


def _dd_binary(a, b, ta: str, tb: str, out: str):
    """One two-operand contraction in double-double as a batched GEMM:
    (batch, left, k) x (batch, k, right) -> permuted to ``out``."""
    from .dispatch import _cuda_bmm_dd

    (ah, al), (bh, bl) = a, b
    ah, al, ta = _dd_reduce(ah, al, ta, set(tb) | set(out))
    bh, bl, tb = _dd_reduce(bh, bl, tb, set(ta) | set(out))
    batch = [c for c in ta if c in tb and c in out]
    contr = [c for c in ta if c in tb and c not in out]
    left = [c for c in ta if c not in tb]
    right = [c for c in tb if c not in ta]
    size = {c: ah.shape[ta.index(c)] for c in ta}
    size.update({c: bh.shape[tb.index(c)] for c in tb})

    def prod(cs):
        n = 1
        for c in cs:
            n *= size[c]
        return n

    pa = [ta.index(c) for c in batch + left + contr]
    pb = [tb.index(c) for c in batch + contr + right]
    shape_a = (prod(batch), prod(left), prod(contr))
    shape_b = (prod(batch), prod(contr), prod(right))
    A = ah.permute(pa).reshape(shape_a)
    Al = None if al is None else al.permute(pa).reshape(shape_a)
    Bm = bh.permute(pb).reshape(shape_b)
    Bl = None if bl is None else bl.permute(pb).reshape(shape_b)
    ch, cl = _cuda_bmm_dd(A, Al, Bm, Bl)
    res_terms = batch + left + right
    full = [size[c] for c in res_terms]
    perm = [res_terms.index(c) for c in out]
    return ch.reshape(full).permute(perm), cl.reshape(full).permute(perm)


def _einsum_dd(subscripts: str, operands: tuple, plan: ContractionPlan) -> torch.Tensor:
    """precision="dd": the contraction in double-double on the CUDA device
    (host operands are moved there); every binary step is a double-double
    GEMM (csrc/dd.cu) and intermediates keep their lo parts. Returns the hi
    part (fp64); the caller casts to the input dtype."""
    from .dispatch import _dd_dev, _device

    lhs, out = _parse_subscripts(subscripts)
    terms = lhs.split(",")
    if any(len(set(t)) != len(t) for t in terms) or len(set(out)) != len(out):
        raise NotImplementedError("precision='dd' does not support repeated indices in a term")
    dev = next((op.device for op in operands if op.device.type == "cuda"), None) or _device()
    ops = [(_dd_dev(op, dev), None) for op in operands]
    if len(ops) == 1:
        h, l_, t = _dd_reduce(ops[0][0], None, terms[0], set(out))
        return h.permute([t.index(c) for c in out]) if out else h.reshape(())
    steps = plan.contraction_path if len(ops) > 2 else [(0, 1)]
    for n, (x, y) in enumerate(steps):
        if n == len(steps) - 1:
            res_term = out
        else:
            later = set(out).union(*(set(t) for k, t in enumerate(terms) if k not in (x, y)))
            res_term = "".join(dict.fromkeys(c for c in terms[x] + terms[y] if c in later))
        res = _dd_binary(ops[x], ops[y], terms[x], terms[y], res_term)
        ops = [o for k, o in enumerate(ops) if k not in (x, y)] + [res]
        terms = [t for k, t in enumerate(terms) if k not in (x, y)] + [res_term]
    return ops[0][0]


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
