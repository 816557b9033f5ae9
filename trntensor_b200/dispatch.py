"""Device dispatch: torch tensors in, C-ABI calls out.

This module takes the place of the reference's backend selector and its
device wrappers (trntensor/nki/dispatch.py:240-336, ``_nki_mp2_energy`` and
``_nki_ao_to_mo_transform``). Differences by design:

* the only executor is the sm_100a library (``libtrntensor_b200.so``);
  there is no CPU fallback and no FLOP threshold;
* host tensors are copied to the current CUDA device and results come back
  to the caller's device, like the reference's ``_to_xla``/``.to(orig)``;
* every buffer the kernels touch is allocated here through torch's caching
  allocator; the library itself never allocates.
"""

from __future__ import annotations

import ctypes
import math
import os

import torch

from . import _lib

HAS_NKI = False  # the Trainium NKI runtime is never used by this package

_backend = "auto"
_VALID_BACKENDS = ("auto", "cuda", "pytorch", "nki")


def set_backend(backend: str) -> None:
    """Select the executor for the generic ``einsum`` strategies.

    Mirrors trntensor/nki/dispatch.py:94-101. ``"auto"`` and ``"pytorch"``
    run matmul/bmm plans with torch on the operands' device (cuBLAS fp32 for
    CUDA tensors: elementwise fp32 rounding, like the reference's default).
    ``"cuda"`` opts CUDA fp32 operands into the int8 tensor-core GEMM
    (``tt_gemm_f32``): 2-3x cuBLAS fp32 throughput, with an error bounded
    per row and column rather than per element (see ``_cuda_gemm``).
    ``"nki"`` raises, exactly as the reference does on a host without
    neuronxcc. The two DF-MP2 primitives always run on the sm_100a library.
    """
    global _backend
    if backend not in _VALID_BACKENDS:
        raise ValueError(f"backend must be one of {_VALID_BACKENDS}; got {backend!r}")
    if backend == "nki":
        raise RuntimeError(
            "NKI backend requires neuronxcc (AWS Trainium); this build runs on NVIDIA B200"
        )
    _backend = backend


def get_backend() -> str:
    return _backend


def to_xla(tensor: torch.Tensor) -> torch.Tensor:
    """Trainium residency helper (trntensor/nki/dispatch.py:152-176).

    There is no XLA device here; raises like the reference does without NKI.
    On B200, residency is simply a CUDA tensor: use ``tensor.cuda()``.
    """
    if tensor.device.type == "xla":
        return tensor
    raise RuntimeError(
        "to_xla requires the NKI runtime. On B200 keep operands resident with tensor.cuda()."
    )


def from_xla(tensor: torch.Tensor) -> torch.Tensor:
    """Move a tensor back to CPU; no-op if already on CPU (dispatch.py:179-184)."""
    if tensor.device.type == "cpu":
        return tensor
    return tensor.to("cpu")


def _device() -> torch.device:
    if not torch.cuda.is_available():
        raise RuntimeError(
            "trntensor_b200 needs a CUDA device (NVIDIA B200, sm_100a); no CUDA device is visible "
            "and there is no CPU fallback"
        )
    return torch.device("cuda", torch.cuda.current_device())


def _stream_handle() -> int:
    return torch.cuda.current_stream().cuda_stream


def _ptr(t: torch.Tensor | None) -> ctypes.c_void_p | None:
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _to_dev(t: torch.Tensor, dev: torch.device, dtype: torch.dtype) -> torch.Tensor:
    if t.device != dev:
        t = t.to(dev, non_blocking=t.is_pinned())
    if t.dtype != dtype:
        t = t.to(dtype)
    return t.contiguous()


def _check_status(dev_status: torch.Tensor, what: str) -> None:
    if os.environ.get("TRNTENSOR_B200_ASYNC", "") in ("1", "true", "yes"):
        return
    code = int(dev_status.item())
    if code != 0:
        raise _lib.DeviceError(f"{what}: device wait ran out (status 0x{code:x})")


def mp2_compute_dtype(B: torch.Tensor, precision: str) -> torch.dtype:
    if precision == "kahan" or B.dtype == torch.float64:
        return torch.float64
    return torch.float32


def _cuda_mp2_energy(
    B: torch.Tensor,
    eps_occ: torch.Tensor,
    eps_vir: torch.Tensor,
    *,
    precision: str = "fast",
    pair_range: tuple[int, int] | None = None,
    return_partials: bool = False,
    kernel: str = "tc",
    blocks=None,
):
    """Run the DF-MP2 energy on the current CUDA device.

    Returns ``(energy_fp64_device_scalar, partials_or_None)``; both stay on the
    device. ``pair_range`` selects a half-open range of unordered pair ids
    (i <= j, row-major) for sharding. ``kernel`` picks the fp32 kernel:
    ``"tc"`` (int8 Ozaki tensor cores, the product path), ``"simt"`` (CUDA-core
    fp32 cross-check) or ``"tf32x3"`` (biased 3xTF32 diagnostic). For fp64
    (``precision="kahan"``) ``"tc"`` is the five-digit int8 Ozaki kernel and
    ``"simt"`` the CUDA-core fp64 kernel. ``blocks`` (``block_assignment``'s
    ``(ranges, chunk order)``) replaces ``pair_range`` by a set of ranges:
    a host-resident B is then copied in that chunk order, a device-resident
    one runs range by range.
    """
    if blocks is not None and not (
        B.device.type == "cpu" and B.is_pinned() and B.dtype == torch.float32
        and B.is_contiguous() and mp2_compute_dtype(B, precision) == torch.float32
        and kernel == "tc" and not return_partials
    ):
        if return_partials:
            raise ValueError("blocks and return_partials cannot be combined")
        dev = _device()
        cdt = mp2_compute_dtype(B, precision)
        Bd, eo, ev = _to_dev(B, dev, cdt), _to_dev(eps_occ, dev, cdt), _to_dev(eps_vir, dev, cdt)
        tot = None
        for rg in blocks[0]:
            e, _ = _cuda_mp2_energy(Bd, eo, ev, precision=precision, pair_range=rg,
                                    kernel=kernel)
            tot = e if tot is None else tot + e
        if tot is None:
            tot = torch.zeros((), dtype=torch.float64, device=_device())
        return tot, None
    lib = _lib.load()
    dev = _device()
    cdt = mp2_compute_dtype(B, precision)
    nocc, nvir, naux = (int(s) for s in B.shape)
    if kernel == "tc" and naux > OZAKI_MAX_K:
        kernel = "simt"  # int32 slice sums are exact only up to OZAKI_MAX_K terms
    if (
        B.device.type == "cpu" and B.is_pinned() and B.dtype == torch.float32
        and B.is_contiguous() and cdt == torch.float32 and kernel == "tc"
        and not return_partials
    ):
        npairs = int(lib.tt_mp2_num_pairs(nocc))
        pb, pe = (0, npairs) if pair_range is None else (int(pair_range[0]), int(pair_range[1]))
        return _mp2_host_pipelined(lib, dev, B, eps_occ, eps_vir, pb, pe, blocks=blocks), None
    Bd = _to_dev(B, dev, cdt)
    eo = _to_dev(eps_occ, dev, cdt)
    ev = _to_dev(eps_vir, dev, cdt)
    npairs = int(lib.tt_mp2_num_pairs(nocc))
    pb, pe = (0, npairs) if pair_range is None else (int(pair_range[0]), int(pair_range[1]))
    energy = torch.empty((), dtype=torch.float64, device=dev)
    partials = (
        torch.empty((nocc, nocc), dtype=torch.float64, device=dev) if return_partials else None
    )
    stream = ctypes.c_void_p(_stream_handle())
    if cdt == torch.float64 and kernel == "tc" and (naux + 63) // 64 * 64 <= OZAKI_F64_MAX_K:
        ws_bytes = int(lib.tt_mp2_f64_workspace_bytes(nocc, nvir, naux))
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
        dev_status = torch.empty((), dtype=torch.int32, device=dev)
        st = lib.tt_mp2_energy_f64_tc(
            _ptr(Bd), _ptr(eo), _ptr(ev), nocc, nvir, naux, pb, pe,
            _ptr(ws), ws_bytes, _ptr(energy), _ptr(partials), _ptr(dev_status), stream,
        )
        _lib.check(st, "tt_mp2_energy_f64_tc")
        _check_status(dev_status, "tt_mp2_energy_f64_tc")
        return energy, partials
    if cdt == torch.float64:
        st = lib.tt_mp2_energy_f64(
            _ptr(Bd), _ptr(eo), _ptr(ev), nocc, nvir, naux, pb, pe,
            _ptr(energy), _ptr(partials), stream,
        )
        _lib.check(st, "tt_mp2_energy_f64")
        return energy, partials
    if kernel == "simt":
        st = lib.tt_mp2_energy_simt_f32(
            _ptr(Bd), _ptr(eo), _ptr(ev), nocc, nvir, naux, pb, pe,
            _ptr(energy), _ptr(partials), stream,
        )
        _lib.check(st, "tt_mp2_energy_simt_f32")
        return energy, partials
    if kernel == "tf32x3":
        pad = (naux + 15) // 16 * 16
        hi = torch.empty((nocc, nvir, pad), dtype=torch.float32, device=dev)
        lo = torch.empty_like(hi)
        dev_status = torch.empty((), dtype=torch.int32, device=dev)
        _lib.check(lib.tt_split_tf32(_ptr(Bd), _ptr(hi), _ptr(lo), nocc * nvir, naux, pad, stream),
                   "tt_split_tf32")
        st = lib.tt_mp2_energy_tf32x3(
            _ptr(hi), _ptr(lo), pad, _ptr(eo), _ptr(ev), nocc, nvir, pb, pe,
            _ptr(energy), _ptr(partials), _ptr(dev_status), stream,
        )
        _lib.check(st, "tt_mp2_energy_tf32x3")
        _check_status(dev_status, "tt_mp2_energy_tf32x3")
        return energy, partials
    # Rows whose entries span many decades (or hold a few entries far above
    # the rest) lose accuracy in the three-digit format; their energy is
    # computed with the five-digit kernel (fp64 accuracy) instead.
    stats = torch.zeros(3, dtype=torch.float64, device=dev)
    _range_stats(lib, Bd, nocc * nvir, naux, stats, stream)
    if _needs_more_digits(stats, naux):
        return _cuda_mp2_energy(Bd, eo, ev, precision="kahan", pair_range=(pb, pe),
                                return_partials=return_partials)
    ws_bytes = int(lib.tt_mp2_workspace_bytes(nocc, nvir, naux))
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    dev_status = torch.empty((), dtype=torch.int32, device=dev)
    st = lib.tt_mp2_energy_f32(
        _ptr(Bd), _ptr(eo), _ptr(ev), nocc, nvir, naux, pb, pe,
        _ptr(ws), ws_bytes, _ptr(energy), _ptr(partials), _ptr(dev_status), stream,
    )
    _lib.check(st, "tt_mp2_energy_f32")
    _check_status(dev_status, "tt_mp2_energy_f32")
    return energy, partials


# Longest contraction the int8 Ozaki kernels sum exactly in int32
# (csrc/ozaki_digits.cuh): K * (64*128 + 128*128 + 128*64) < 2^31.
OZAKI_MAX_K = 65535
# The five-digit fp64 kernel (csrc/mp2_i8x5.cuh): K * (2*64*128 + 3*128*128) < 2^31.
OZAKI_F64_MAX_K = 32767
# The six-digit fp64 GEMM (csrc/ozaki_gemm64.cuh): K * (2*64*128 + 4*128*128) < 2^31.
OZAKI_GEMM_F64_MAX_K = 26214


def pair_offset(i: int, nocc: int) -> int:
    """Linear id of the first unordered pair (i, i) (row-major over i <= j)."""
    return i * nocc - i * (i - 1) // 2


def first_row_of_pair(p: int, nocc: int) -> int:
    """Occupied index i of the unordered pair with linear id p."""
    lo, hi = 0, nocc - 1
    while lo < hi:
        mid = (lo + hi + 1) // 2
        if pair_offset(mid, nocc) <= p:
            lo = mid
        else:
            hi = mid - 1
    return lo


def _merge(ranges: list[tuple[int, int]]) -> list[tuple[int, int]]:
    out: list[tuple[int, int]] = []
    for lo, hi in ranges:
        if hi <= lo:
            continue
        if out and out[-1][1] == lo:
            out[-1] = (out[-1][0], hi)
        else:
            out.append((lo, hi))
    return out


def _groups(nocc: int, g: int) -> list[tuple[int, int]]:
    """g contiguous row groups [lo, hi) of nearly equal size."""
    cuts = [round(k * nocc / g) for k in range(g + 1)]
    return [(cuts[k], cuts[k + 1]) for k in range(g)]


def _split(lo: int, hi: int, n: int) -> list[tuple[int, int]]:
    """[lo, hi) in n contiguous chunks (fewer when there are fewer rows)."""
    n = max(1, min(n, hi - lo))
    cuts = [lo + round(k * (hi - lo) / n) for k in range(n + 1)]
    return [(cuts[k], cuts[k + 1]) for k in range(n) if cuts[k + 1] > cuts[k]]


def block_assignment(nocc: int, rank: int, world: int, chunks: int = 16):
    """Pairs and row-copy order of ``rank`` when B is copied from the host.

    With contiguous pair ranges the first rank's pairs touch every row of B,
    so at 8 ranks rank 0 copies all of B (11.3 GB at BASELINE config 4,
    ≈400 ms at the ≈25 GB/s a GPU gets while all eight copy) while the last
    copies a sixth of it. For 4 and 8 ranks the rows are cut into row groups
    instead, and each rank takes group pairs so that it needs half of the
    rows (three quarters for two ranks at 4):

    * 8 ranks, 4 groups: ranks 0-5 take the six off-diagonal group pairs
      (Ga, Gb), a < b (all i in Ga, j in Gb); ranks 6 and 7 take the
      diagonal blocks (G0, G0) + (G1, G1) and (G2, G2) + (G3, G3);
    * 4 ranks, 2 groups: ranks 0 and 1 take (G0, G0) and (G1, G1), ranks 2
      and 3 the two halves (by i) of (G0, G1).

    Work per rank is equal to within one row group's diagonal (s² against
    s² + s pairs for groups of s rows). Returns ``(ranges, chunks)``: the
    rank's merged pair-id ranges and the row chunks [a, b) in copy order
    (interleaved between the two groups of an off-diagonal pair, last rows
    first within a diagonal block, so that pairs become runnable early), or
    None when the contiguous ranges are used (other world sizes, or fewer
    than two rows per group).
    """
    if world == 8:
        g = 4
        units = [((0, 1),), ((0, 2),), ((0, 3),), ((1, 2),), ((1, 3),), ((2, 3),),
                 ((0, 0), (1, 1)), ((2, 2), (3, 3))]
    elif world == 4:
        g = 2
        units = [((0, 0),), ((1, 1),), ((0, 1, 0),), ((0, 1, 1),)]
    else:
        return None
    if nocc < 2 * g:
        return None
    grp = _groups(nocc, g)
    pairs: list[tuple[int, int]] = []
    order: list[tuple[int, int]] = []
    for u in units[rank]:
        a, b = u[0], u[1]
        ga, gb = grp[a], grp[b]
        if len(u) == 3:  # half (by i) of an off-diagonal group pair
            ga = _split(ga[0], ga[1], 2)[u[2]]
        if a == b:
            for i in range(ga[0], ga[1]):
                pairs.append((pair_offset(i, nocc), pair_offset(i, nocc) + ga[1] - i))
            order += _split(ga[0], ga[1], max(1, chunks // len(units[rank])))[::-1]
        else:
            for i in range(ga[0], ga[1]):
                pairs.append((pair_offset(i, nocc) + gb[0] - i, pair_offset(i, nocc) + gb[1] - i))
            ca = _split(ga[0], ga[1], max(1, chunks // 2))
            cb = _split(gb[0], gb[1], max(1, chunks // 2))
            for k in range(max(len(ca), len(cb))):
                order += ca[k:k + 1] + cb[k:k + 1]
    return _merge(sorted(pairs)), order


def chunk_plan(nocc: int, ranges: list[tuple[int, int]], order: list[tuple[int, int]]):
    """Copy plan in host_copy_plan's format for the pair-id ``ranges`` when
    rows are copied in the chunk ``order``: after each chunk, the ranges of
    the pairs whose later row has just landed."""
    step_of = [-1] * nocc
    for k, (a, b) in enumerate(order):
        for r in range(a, b):
            step_of[r] = k
    runs: list[list[tuple[int, int]]] = [[] for _ in order]
    for lo, hi in ranges:
        i = first_row_of_pair(lo, nocc)
        p = lo
        while p < hi:
            end = min(hi, pair_offset(i + 1, nocc))
            si = step_of[i]
            j = i + (p - pair_offset(i, nocc))
            while p < end:  # runs of consecutive j landing in the same step
                k = max(si, step_of[j])
                q = p
                while q < end and max(si, step_of[j + (q - p)]) == k:
                    q += 1
                runs[k].append((p, q))
                j += q - p
                p = q
            i += 1
    return [(a, b, _merge(sorted(r))) for (a, b), r in zip(order, runs)]


def host_copy_plan(nocc: int, pb: int, pe: int, chunks: int = 16):
    """Copy order of a host B's rows for the pairs [pb, pe), and what to run.

    Returns ``[(a, b, ranges), ...]``: copy rows [a, b), then run the pair id
    ranges ``ranges`` (each half-open, row-major ids of i <= j), whose two
    rows are resident by then and which no earlier step ran.

    The range's pairs have i in [i0, i1] (its own rows) and j in [i, nocc).
    Own rows are copied first, last ones first: once rows [a, i1] are in, the
    pairs (i >= a, j <= i1) can run. Then the rows beyond i1 (needed only as
    j) are copied first ones first, and each chunk [a, b) runs the pairs
    (i in [i0, i1], j in [a, b)). The first pairs can thus start after one
    chunk, whatever rows the range owns. With i1 = nocc - 1 (one GPU, the last
    rank) every step is one contiguous id range; otherwise one range per own
    row i, which is still few (about nocc / world own rows).
    """
    if pe <= pb:
        return []
    i0 = first_row_of_pair(pb, nocc)
    i1 = first_row_of_pair(pe - 1, nocc)
    own = i1 - i0 + 1
    rest = nocc - 1 - i1
    n_own = max(1, round(chunks * own / (own + rest)))
    n_rest = max(1, chunks - n_own) if rest else 0
    plan = []

    def clip(lo, hi):
        return max(lo, pb), min(hi, pe)

    step = -(-own // n_own)
    b = i1 + 1
    while b > i0:
        a = max(i0, b - step)
        # rows [a, i1] resident: pairs (i in [a, b), j in [i, i1])
        plan.append((a, b, _merge([clip(pair_offset(i, nocc), pair_offset(i, nocc) + (i1 + 1 - i))
                                   for i in range(a, b)])))
        b = a
    if rest:
        step = -(-rest // n_rest)
        a = i1 + 1
        while a < nocc:
            b = min(nocc, a + step)
            plan.append((a, b, _merge([clip(pair_offset(i, nocc) + (a - i),
                                            pair_offset(i, nocc) + (b - i))
                                       for i in range(i0, i1 + 1)])))
            a = b
    return plan


def _wide_rows_estimate(stats: list[float], naux: int) -> float:
    """Relative energy error estimate of the three-digit fp32 path from
    tt_mp2_range_stats_f32's sums (see include/trntensor_b200.h)."""
    a2, a3, n = stats
    if not n > 0.0:
        return 0.0
    return 2.0 * math.sqrt(max(0.0, 2.0**-47 * a2 * a3 / naux)) / (n * n / naux)


# Above this estimate the fp32 energy is computed with the five-digit
# (fp64-accurate) kernel instead of the three-digit one; Gaussian rows stay
# well below it (1e-7 to 3e-7 at the benchmark sizes).
WIDE_ROWS_MAX_EST = 1e-6


def _range_stats(lib, X: torch.Tensor, rows: int, naux: int, stats: torch.Tensor, stream) -> None:
    _lib.check(lib.tt_mp2_range_stats_f32(_ptr(X), rows, naux, _ptr(stats), stream),
               "tt_mp2_range_stats_f32")


def mp2_range_estimate(B: torch.Tensor) -> float:
    """The wide-row error estimate of an fp32 B (nocc, nvir, naux), computed
    on the current CUDA device; the fp32 energy uses five digits above
    WIDE_ROWS_MAX_EST."""
    lib = _lib.load()
    dev = _device()
    Bd = _to_dev(B, dev, torch.float32)
    stats = torch.zeros(3, dtype=torch.float64, device=dev)
    rows = int(B.shape[0]) * int(B.shape[1])
    _range_stats(lib, Bd, rows, int(B.shape[2]), stats, ctypes.c_void_p(_stream_handle()))
    return _wide_rows_estimate(stats.tolist(), int(B.shape[2]))


def _needs_more_digits(stats: torch.Tensor, naux: int) -> bool:
    """Host read of the range statistics (one synchronisation); False when
    TRNTENSOR_B200_ASYNC asks for no host reads."""
    if os.environ.get("TRNTENSOR_B200_ASYNC", "") in ("1", "true", "yes"):
        return False
    return _wide_rows_estimate(stats.tolist(), naux) > WIDE_ROWS_MAX_EST


def _mp2_host_pipelined(lib, dev, B, eps_occ, eps_vir, pb, pe, chunks=16, blocks=None):
    """fp32 DF-MP2 energy of host-resident pinned B with the copy overlapped.

    Rows are copied on a side stream in the order of ``host_copy_plan`` (the
    pair range [pb, pe)) or, with ``blocks = (ranges, chunk order)`` from
    ``block_assignment``, of ``chunk_plan``;
    each chunk is split into int8 slices as it lands (tt_split_i8_rows) and
    the pairs it completes run on the current stream while the next chunk is
    in flight. Only the rows the pair range needs are copied. If the range
    statistics of those rows call for more digits, the energy is recomputed
    from the device copy with the five-digit kernel.
    """
    nocc, nvir, naux = (int(s) for s in B.shape)
    stream = torch.cuda.current_stream(dev)
    sp = ctypes.c_void_p(stream.cuda_stream)
    eo = _to_dev(eps_occ, dev, torch.float32)
    ev = _to_dev(eps_vir, dev, torch.float32)
    all_ranges = [(pb, pe)] if blocks is None else [r for r in blocks[0] if r[1] > r[0]]
    if not all_ranges or all_ranges[0][1] <= all_ranges[0][0]:
        return torch.zeros((), dtype=torch.float64, device=dev)
    pad = (naux + 63) // 64 * 64
    rows_total = nocc * nvir
    ws_bytes = int(lib.tt_mp2_workspace_bytes(nocc, nvir, naux))
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    qbytes = (3 * rows_total * pad + 255) // 256 * 256
    q_ptr = ws.data_ptr()
    s_ptr = ws.data_ptr() + qbytes
    plan = (host_copy_plan(nocc, pb, pe, chunks) if blocks is None
            else chunk_plan(nocc, blocks[0], blocks[1]))
    Bd = torch.empty((nocc, nvir, naux), dtype=torch.float32, device=dev)
    copied = [False] * nocc
    for a, b, _ in plan:
        copied[a:b] = [True] * (b - a)
    r = 0
    while r < nocc:  # rows no pair of the rank reads (keeps a recompute clean)
        if copied[r]:
            r += 1
            continue
        e = r
        while e < nocc and not copied[e]:
            e += 1
        Bd[r:e].zero_()
        r = e
    nlaunch = sum(len(r) for _, _, r in plan)
    energies = torch.zeros(max(1, nlaunch), dtype=torch.float64, device=dev)
    status = torch.zeros(max(1, nlaunch), dtype=torch.int32, device=dev)
    stats = torch.zeros(3, dtype=torch.float64, device=dev)
    copy_stream = torch.cuda.Stream(dev)
    copy_stream.wait_stream(stream)  # Bd / ws allocations are ordered before the copies
    k = 0
    for a, b, ranges in plan:
        with torch.cuda.stream(copy_stream):
            Bd[a:b].copy_(B[a:b], non_blocking=True)
            done = torch.cuda.Event()
            done.record(copy_stream)
        stream.wait_event(done)
        _lib.check(lib.tt_split_i8_rows(ctypes.c_void_p(Bd.data_ptr()), ctypes.c_void_p(q_ptr),
                                        ctypes.c_void_p(s_ptr), a * nvir, (b - a) * nvir,
                                        rows_total, naux, pad, sp), "tt_split_i8_rows")
        _range_stats(lib, Bd[a:b], (b - a) * nvir, naux, stats, sp)
        for lo, hi in ranges:
            st = lib.tt_mp2_energy_presplit_i8(
                ctypes.c_void_p(q_ptr), ctypes.c_void_p(s_ptr), pad, _ptr(eo), _ptr(ev), nocc,
                nvir, lo, hi, ctypes.c_void_p(energies.data_ptr() + 8 * k), None,
                ctypes.c_void_p(status.data_ptr() + 4 * k), sp)
            _lib.check(st, "tt_mp2_energy_presplit_i8")
            k += 1
    Bd.record_stream(copy_stream)
    energy = energies.sum()
    if os.environ.get("TRNTENSOR_B200_ASYNC", "") not in ("1", "true", "yes"):
        bad = status.nonzero()
        if bad.numel():
            raise _lib.DeviceError(f"tt_mp2_energy_presplit_i8: device wait ran out "
                                   f"(status 0x{int(status[bad[0, 0]].item()):x})")
    if _needs_more_digits(stats, naux):
        del ws
        energy = sum(_cuda_mp2_energy(Bd, eo, ev, precision="kahan", pair_range=rg)[0]
                     for rg in all_ranges)
    return energy


def _cuda_ao_to_mo_transform(
    eri: torch.Tensor,
    C_occ: torch.Tensor,
    C_vir: torch.Tensor,
    *,
    precision: str = "fast",
    kernel: str = "tc",
) -> torch.Tensor:
    """AO->MO transform on the current CUDA device; result stays on the device.

    ``kernel="tc"``: int8 Ozaki tensor cores (three digits for fp32, six for
    fp64); ``kernel="simt"``: plain CUDA-core cross-check in the same precision.

    fp32 inputs compute in fp32, float64 inputs or ``precision="kahan"`` in
    fp64 (trntensor/einsum.py:108-111 semantics: the caller casts back).
    """
    lib = _lib.load()
    dev = _device()
    cdt = torch.float64 if (precision == "kahan" or eri.dtype == torch.float64) else torch.float32
    nbf, _, naux = (int(s) for s in eri.shape)
    nocc, nvir = int(C_occ.shape[1]), int(C_vir.shape[1])
    if nocc * nvir * naux == 0 or nbf == 0:
        return torch.zeros((nocc, nvir, naux), dtype=cdt, device=dev)
    out = torch.empty((nocc, nvir, naux), dtype=cdt, device=dev)  # every element is written
    if kernel == "tc" and nbf > OZAKI_MAX_K:
        kernel = "simt"
    e = _to_dev(eri, dev, cdt)
    co = _to_dev(C_occ, dev, cdt)
    cv = _to_dev(C_vir, dev, cdt)
    if cdt == torch.float64 and kernel == "tc" and nbf <= OZAKI_GEMM_F64_MAX_K:
        ws_bytes = int(lib.tt_ao2mo_f64_workspace_bytes(nbf, nocc, nvir, naux))
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
        dev_status = torch.empty((), dtype=torch.int32, device=dev)
        st = lib.tt_ao2mo_f64_tc(_ptr(e), _ptr(co), _ptr(cv), nbf, nocc, nvir, naux, _ptr(ws),
                                 ws_bytes, _ptr(out), _ptr(dev_status),
                                 ctypes.c_void_p(_stream_handle()))
        _lib.check(st, "tt_ao2mo_f64_tc")
        _check_status(dev_status, "tt_ao2mo_f64_tc")
        return out
    esz = 8 if cdt == torch.float64 else 4
    ws_bytes = int(lib.tt_ao2mo_workspace_bytes(nbf, nocc, nvir, naux, esz))
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    stream = ctypes.c_void_p(_stream_handle())
    if cdt == torch.float64 or kernel == "simt":
        fn = lib.tt_ao2mo_f64 if cdt == torch.float64 else lib.tt_ao2mo_simt_f32
        st = fn(_ptr(e), _ptr(co), _ptr(cv), nbf, nocc, nvir, naux, _ptr(ws), ws_bytes,
                _ptr(out), stream)
        _lib.check(st, "tt_ao2mo")
        return out
    dev_status = torch.empty((), dtype=torch.int32, device=dev)
    st = lib.tt_ao2mo_f32(_ptr(e), _ptr(co), _ptr(cv), nbf, nocc, nvir, naux, _ptr(ws), ws_bytes,
                          _ptr(out), _ptr(dev_status), stream)
    _lib.check(st, "tt_ao2mo_f32")
    _check_status(dev_status, "tt_ao2mo_f32")
    return out


def _cuda_ao_to_mo_slab(eri: torch.Tensor, C_occ: torch.Tensor, C_vir: torch.Tensor, p0: int,
                        p1: int) -> torch.Tensor:
    """fp32 AO->MO transform of eri's aux columns [p0, p1) read in place
    (tt_ao2mo_f32_slab); eri is the full contiguous (nbf, nbf, naux) CUDA
    fp32 tensor. Falls back to a slab copy where the strided read does not
    apply (nbf <= 128, unaligned columns)."""
    lib = _lib.load()
    dev = eri.device
    nbf, _, naux = (int(s) for s in eri.shape)
    nocc, nvir, nl = int(C_occ.shape[1]), int(C_vir.shape[1]), p1 - p0
    ok = (eri.is_cuda and eri.dtype == torch.float32 and eri.is_contiguous() and nbf > 128
          and p0 % 4 == 0 and naux % 4 == 0 and nl > 0 and nocc * nvir > 0)
    if not ok:
        return _cuda_ao_to_mo_transform(eri[:, :, p0:p1], C_occ, C_vir)
    co = _to_dev(C_occ, dev, torch.float32)
    cv = _to_dev(C_vir, dev, torch.float32)
    out = torch.empty((nocc, nvir, nl), dtype=torch.float32, device=dev)
    ws_bytes = int(lib.tt_ao2mo_workspace_bytes(nbf, nocc, nvir, nl, 4))
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    status = torch.empty((), dtype=torch.int32, device=dev)
    st = lib.tt_ao2mo_f32_slab(ctypes.c_void_p(eri.data_ptr() + 4 * p0), nbf * naux, naux,
                               _ptr(co), _ptr(cv), nbf, nocc, nvir, nl, _ptr(ws), ws_bytes,
                               _ptr(out), _ptr(status), ctypes.c_void_p(_stream_handle()))
    _lib.check(st, "tt_ao2mo_f32_slab")
    _check_status(status, "tt_ao2mo_f32_slab")
    return out


def _operand_layout(X: torch.Tensor, kmajor_if_contiguous: bool):
    """(storage tensor, kmajor) for a 2-D/3-D operand without copying if possible."""
    if X.is_contiguous():
        return X, kmajor_if_contiguous
    Xt = X.transpose(-1, -2)
    if Xt.is_contiguous():
        return Xt, not kmajor_if_contiguous
    return X.contiguous(), kmajor_if_contiguous


def _cuda_gemm(A: torch.Tensor, B: torch.Tensor) -> torch.Tensor:
    """fp32 (batched) A @ B on int8 tensor cores (``set_backend("cuda")``).

    A: (M, K) or (b, M, K); B: (K, N) or (b, K, N); CUDA fp32 tensors.

    Accuracy contract: each row of A and each column of B carries one
    power-of-two scale (from its largest magnitude, M_i and M_j) and three
    int8 digits, so the error is bounded per row and column, not per element:
    |C_ij - (AB)_ij| <= 2^-19 (M_i |B_:j|_1 + |A_i:|_1 M_j)
    + 2^-20 sqrt(K) M_i M_j. For rows and columns of similar magnitudes that
    is fp32 accuracy; an entry far below its row's (column's) largest keeps
    fewer bits than fp32 would give it. A row or column with a largest
    magnitude below 1e-30 counts as zero, and one holding inf or NaN makes its
    whole output row or column NaN (fp32 would give inf in some places).
    """
    lib = _lib.load()
    dev = A.device
    batched = A.dim() == 3
    M, K = int(A.shape[-2]), int(A.shape[-1])
    N = int(B.shape[-1])
    nb = int(A.shape[0]) if batched else 1
    out = torch.empty((nb, M, N) if batched else (M, N), dtype=torch.float32, device=dev)
    if out.numel() == 0:
        return out
    if K == 0:
        return out.zero_()
    As, a_k = _operand_layout(A, True)   # (M, K) row-major is K-major
    Bs, b_k = _operand_layout(B, False)  # (K, N) row-major is N-major
    ws_bytes = int(lib.tt_gemm_workspace_bytes(M, N, K, nb, int(a_k), int(b_k)))
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    status = torch.empty((), dtype=torch.int32, device=dev)
    st = lib.tt_gemm_f32(_ptr(As), int(a_k), M * K, _ptr(Bs), int(b_k), K * N, _ptr(out), M * N,
                         M, N, K, nb, _ptr(ws), ws_bytes, _ptr(status),
                         ctypes.c_void_p(_stream_handle()))
    _lib.check(st, "tt_gemm_f32")
    _check_status(status, "tt_gemm_f32")
    return out


# ------------------------------------------------------ double-double (dd)

def _dd_dev(t: torch.Tensor, dev: torch.device) -> torch.Tensor:
    """fp64 copy on the device (exact for every float input dtype)."""
    return _to_dev(t, dev, torch.float64)


def _cuda_mp2_energy_dd(B, eps_occ, eps_vir, *, pair_range=None, return_partials=False):
    """DF-MP2 energy in double-double (precision="dd").

    Returns ``((2,) fp64 [hi, lo] device tensor, partials)`` where partials
    is a (nocc, nocc, 2) fp64 tensor of per-pair (hi, lo) or None.
    """
    lib = _lib.load()
    dev = _device()
    nocc, nvir, naux = (int(s) for s in B.shape)
    Bd, eo, ev = _dd_dev(B, dev), _dd_dev(eps_occ, dev), _dd_dev(eps_vir, dev)
    npairs = nocc * (nocc + 1) // 2
    pb, pe = (0, npairs) if pair_range is None else (int(pair_range[0]), int(pair_range[1]))
    ws_bytes = int(lib.tt_mp2_dd_workspace_bytes(nocc, nvir, naux))
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    energy = torch.empty(2, dtype=torch.float64, device=dev)
    partials = (torch.empty((nocc, nocc, 2), dtype=torch.float64, device=dev)
                if return_partials else None)
    st = lib.tt_mp2_energy_dd(_ptr(Bd), _ptr(eo), _ptr(ev), nocc, nvir, naux, pb, pe, _ptr(ws),
                              ws_bytes, _ptr(energy), _ptr(partials),
                              ctypes.c_void_p(_stream_handle()))
    _lib.check(st, "tt_mp2_energy_dd")
    return energy, partials


def _cuda_bmm_dd(A_hi, A_lo, B_hi, B_lo):
    """Batched (b, M, K) x (b, K, N) in double-double; lo parts nullable.
    All operands fp64 CUDA tensors; returns (C_hi, C_lo), each (b, M, N)."""
    lib = _lib.load()
    nb, M, K = (int(s) for s in A_hi.shape)
    N = int(B_hi.shape[-1])
    dev = A_hi.device
    C_hi = torch.empty((nb, M, N), dtype=torch.float64, device=dev)
    C_lo = torch.empty_like(C_hi)
    if C_hi.numel() == 0:
        return C_hi, C_lo
    if K == 0:
        return C_hi.zero_(), C_lo.zero_()
    A_hi, B_hi = A_hi.contiguous(), B_hi.contiguous()
    A_lo = None if A_lo is None else A_lo.contiguous()
    B_lo = None if B_lo is None else B_lo.contiguous()
    stream = ctypes.c_void_p(_stream_handle())
    for b0 in range(0, nb, 65535):
        b1 = min(nb, b0 + 65535)
        st = lib.tt_gemm_dd(
            _ptr(A_hi[b0:b1]), _ptr(None if A_lo is None else A_lo[b0:b1]), 1, M * K,
            _ptr(B_hi[b0:b1]), _ptr(None if B_lo is None else B_lo[b0:b1]), 0, K * N,
            _ptr(C_hi[b0:b1]), _ptr(C_lo[b0:b1]), M * N, M, N, K, b1 - b0, stream)
        _lib.check(st, "tt_gemm_dd")
    return C_hi, C_lo


def _cuda_ao_to_mo_dd(eri, C_occ, C_vir):
    """AO->MO transform in double-double: step 1 keeps the (i, n, P)
    intermediate as (hi, lo) and step 2 reads both. Returns (B_hi, B_lo)."""
    lib = _lib.load()
    dev = _device()
    nbf, _, naux = (int(s) for s in eri.shape)
    nocc, nvir = int(C_occ.shape[1]), int(C_vir.shape[1])
    e, co, cv = _dd_dev(eri, dev), _dd_dev(C_occ, dev), _dd_dev(C_vir, dev)
    out_hi = torch.zeros((nocc, nvir, naux), dtype=torch.float64, device=dev)
    out_lo = torch.zeros_like(out_hi)
    if out_hi.numel() == 0 or nbf == 0:
        return out_hi, out_lo
    inter_hi = torch.empty((nocc, nbf, naux), dtype=torch.float64, device=dev)
    inter_lo = torch.empty_like(inter_hi)
    stream = ctypes.c_void_p(_stream_handle())
    # step 1: inter[i, (n, P)] = sum_m C_occ[m, i] eri[m, (n, P)]
    _lib.check(lib.tt_gemm_dd(_ptr(co), None, 0, 0, _ptr(e), None, 0, 0, _ptr(inter_hi),
                              _ptr(inter_lo), nocc * nbf * naux, nocc, nbf * naux, nbf, 1,
                              stream), "tt_gemm_dd")
    # step 2: out[i] = C_vir^T inter[i] (batched over i, dd intermediate)
    _lib.check(lib.tt_gemm_dd(_ptr(cv), None, 0, 0, _ptr(inter_hi), _ptr(inter_lo), 0,
                              nbf * naux, _ptr(out_hi), _ptr(out_lo), nvir * naux, nvir, naux,
                              nbf, nocc, stream), "tt_gemm_dd")
    return out_hi, out_lo
