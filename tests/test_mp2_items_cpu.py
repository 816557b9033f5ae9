"""The fp32 MP2 kernel's work decomposition, restated on CPU.

The C ABI issues a pair range as chunked launches (``launch_chunks`` in
csrc/mp2.cu): per chunk one launch of the two-phase items (i < j, block
A < B) and one of the one-phase items (diagonal blocks A == B of every pair,
then the off-diagonal blocks of the i == j pairs). Each CTA turns its item
index into (i, j, A, B) with ``item_decode`` (csrc/mp2_i8.cuh). This test
restates both in Python, with the same integer and float64 arithmetic, and
checks that for any pair range and chunk size every (i <= j, A <= B) item of
the range is run exactly once, each in the launch kind that matches its
phase count.
"""

from __future__ import annotations

import math
import random

import pytest


def pair_offset(i, n):
    return i * n - i * (i - 1) // 2


def pair_decode(p, n):
    nn = 2.0 * n + 1.0
    ii = int((nn - math.sqrt(nn * nn - 8.0 * float(p))) * 0.5)
    ii = max(0, min(ii, n - 1))
    while ii > 0 and pair_offset(ii, n) > p:
        ii -= 1
    while ii + 1 < n and pair_offset(ii + 1, n) <= p:
        ii += 1
    return ii, ii + (p - pair_offset(ii, n))


def offdiag_decode(r, nblk):
    A = 0
    while r >= nblk - 1 - A:
        r -= nblk - 1 - A
        A += 1
    return A, A + 1 + r


def diag_pairs_before(p, n):
    lo, hi = 0, n
    while lo < hi:
        mid = (lo + hi) // 2
        if pair_offset(mid, n) >= p:
            hi = mid
        else:
            lo = mid + 1
    return lo


def item_decode(w, mode, nocc, nblk, pair_begin, pair_end, q_begin, diag_lo):
    if mode == 1:
        nodp = nblk * (nblk - 1) // 2
        i, jj = pair_decode(q_begin + w // nodp, nocc - 1)
        A, B = offdiag_decode(w % nodp, nblk)
        return i, jj + 1, A, B
    if mode == 2:
        nd = (pair_end - pair_begin) * nblk
        if w < nd:
            i, j = pair_decode(pair_begin + w // nblk, nocc)
            return i, j, w % nblk, w % nblk
        nodp = nblk * (nblk - 1) // 2
        w -= nd
        i = diag_lo + w // nodp
        A, B = offdiag_decode(w % nodp, nblk)
        return i, i, A, B
    nbp = nblk * (nblk + 1) // 2
    i, j = pair_decode(pair_begin + w // nbp, nocc)
    r, A = w % nbp, 0
    while r >= nblk - A:
        r -= nblk - A
        A += 1
    return i, j, A, A + r


def issued_items(nocc, nblk, pb, pe, per_launch, split_modes):
    """Every (i, j, A, B, mode) the launches of [pb, pe) run."""
    out = []
    nodp = nblk * (nblk - 1) // 2
    ipp = nblk * (nblk + 1) // 2
    lo = pb
    while lo < pe:
        hi = min(lo + per_launch, pe)
        if not split_modes:
            out += [item_decode(w, 0, nocc, nblk, lo, hi, 0, 0) + (0,)
                    for w in range((hi - lo) * ipp)]
        else:
            d_lo, d_hi = diag_pairs_before(lo, nocc), diag_pairs_before(hi, nocc)
            n1 = ((hi - d_hi) - (lo - d_lo)) * nodp
            out += [item_decode(w, 1, nocc, nblk, lo, hi, lo - d_lo, 0) + (1,)
                    for w in range(n1)]
            n2 = (hi - lo) * nblk + (d_hi - d_lo) * nodp
            out += [item_decode(w, 2, nocc, nblk, lo, hi, 0, d_lo) + (2,) for w in range(n2)]
        lo = hi
    return out


CASES = [(1, 1), (2, 1), (3, 2), (5, 3), (8, 14), (17, 4), (64, 4), (256, 2)]


@pytest.mark.parametrize("nocc,nblk", CASES)
@pytest.mark.parametrize("split_modes", [True, False])
def test_every_item_runs_once(nocc, nblk, split_modes):
    rng = random.Random(nocc * 100 + nblk)
    npairs = nocc * (nocc + 1) // 2
    ids = [(i, j) for i in range(nocc) for j in range(i, nocc)]
    ranges = [(0, npairs)] + [tuple(sorted(rng.sample(range(npairs + 1), 2)))
                              for _ in range(3)] if npairs > 1 else [(0, npairs)]
    for pb, pe in ranges:
        for per_launch in (1, 3, 7, max(1, npairs)):
            got = issued_items(nocc, nblk, pb, pe, per_launch, split_modes)
            want = sorted((i, j, A, B) for i, j in ids[pb:pe]
                          for A in range(nblk) for B in range(A, nblk))
            assert sorted(g[:4] for g in got) == want, (pb, pe, per_launch)
            if split_modes:
                for i, j, A, B, mode in got:  # launch kind matches the phase count
                    assert (mode == 2) == (i == j or A == B)


def test_pair_decode_at_the_abi_limits():
    """pair_decode's float64 estimate plus its correction steps invert
    pair_offset at the largest nocc the ABI accepts (65535)."""
    n = 65535
    npairs = n * (n + 1) // 2
    probe = [0, 1, n - 1, n, npairs - 2, npairs - 1]
    probe += [pair_offset(i, n) + d for i in (1, 2, 1000, 40000, n - 2, n - 1) for d in (-1, 0, 1)]
    rng = random.Random(0)
    probe += [rng.randrange(npairs) for _ in range(2000)]
    for p in probe:
        if not 0 <= p < npairs:
            continue
        i, j = pair_decode(p, n)
        assert 0 <= i <= j < n and pair_offset(i, n) + (j - i) == p
