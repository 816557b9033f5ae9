"""Multi-rank host logic on CPU with gloo (world size 2 and 4): pair and aux
partitioning, the fp64 scalar all-reduce, and a rank that fails before the
collective (the others get an error instead of hanging)."""

from __future__ import annotations

import os
import socket
import traceback

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from trntensor_b200 import distributed


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_pair_range_partition():
    for n in (1, 36, 2080, 32896, 7):
        for w in (1, 2, 3, 4, 8):
            rs = [distributed.pair_range(n, r, w) for r in range(w)]
            assert rs[0][0] == 0 and rs[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(rs, rs[1:]))
            sizes = [e - b for b, e in rs]
            assert max(sizes) - min(sizes) <= 1


def _worker(rank, world, port, mode, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        from datetime import timedelta

        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=10))
        if mode == "reduce":
            nocc = 9
            npairs = nocc * (nocc + 1) // 2
            b, e = distributed.pair_range(npairs, rank, world)
            # stand-in for the kernel: each pair id contributes (id + 1)
            local = torch.tensor(float(sum(range(b + 1, e + 1))), dtype=torch.float64)
            distributed.reduce_energy(local)
            q.put((rank, local.item(), npairs * (npairs + 1) / 2))
        elif mode == "slabs":
            naux = 10
            B = torch.arange(3 * 4 * naux, dtype=torch.float32).reshape(3, 4, naux)
            p0, p1 = distributed.aux_slab(naux, rank, world)
            full = distributed.gather_aux(B[:, :, p0:p1].contiguous(), naux)
            q.put((rank, bool(torch.equal(full, B)), True))
        elif mode == "strided":
            # each rank addresses its aux columns inside the full eri the way
            # tt_ao2mo_f32_slab's 3-D tensor map does: base + p0, strides
            # (nbf * naux, naux, 1), extents (nbf, nbf, p1 - p0)
            nbf, naux = 5, 12
            eri = torch.arange(nbf * nbf * naux, dtype=torch.float32).reshape(nbf, nbf, naux)
            p0, p1 = distributed.aux_slab(naux, rank, world)
            view = torch.as_strided(eri, (nbf, nbf, p1 - p0), (nbf * naux, naux, 1), p0)
            ok = bool(torch.equal(view, eri[:, :, p0:p1]))
            full = distributed.gather_aux(view.contiguous(), naux)
            q.put((rank, ok and bool(torch.equal(full, eri)), True))
        elif mode == "pipeline":
            # every rank copies rows in host_copy_plan order and runs the pair
            # ranges each step lists; each pair id contributes (id + 1) once
            from trntensor_b200.dispatch import host_copy_plan

            nocc = 23
            npairs = nocc * (nocc + 1) // 2
            b, e = distributed.pair_range(npairs, rank, world)
            local = torch.zeros((), dtype=torch.float64)
            for _, _, ranges in host_copy_plan(nocc, b, e, chunks=5):
                for lo, hi in ranges:
                    local += float(sum(range(lo + 1, hi + 1)))
            distributed.reduce_energy(local)
            q.put((rank, local.item(), npairs * (npairs + 1) / 2))
        elif mode == "blocks":
            # the row-group block plan: each pair id contributes (id + 1) once
            from trntensor_b200.dispatch import block_assignment, chunk_plan

            nocc = 23
            npairs = nocc * (nocc + 1) // 2
            ranges, order = block_assignment(nocc, rank, world, chunks=6)
            local = torch.zeros((), dtype=torch.float64)
            for _, _, rr in chunk_plan(nocc, ranges, order):
                for lo, hi in rr:
                    local += float(sum(range(lo + 1, hi + 1)))
            distributed.reduce_energy(local)
            q.put((rank, local.item(), npairs * (npairs + 1) / 2))
        elif mode == "fail":
            if rank == 1:
                raise RuntimeError("injected failure on rank 1 before the all-reduce")
            t = torch.ones((), dtype=torch.float64)
            try:
                dist.all_reduce(t)
                q.put((rank, "no error", "error"))
            except Exception as exc:  # the collective times out / aborts
                q.put((rank, "error", "error"))
        dist.destroy_process_group()
    except RuntimeError as exc:
        if "injected" in str(exc):
            q.put((rank, "raised", "raised"))
        else:
            q.put((rank, traceback.format_exc(), None))


def _run(world, mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = [q.get(timeout=90) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return out


@pytest.mark.parametrize("world", [2, 4])
def test_energy_all_reduce(world):
    for rank, got, want in _run(world, "reduce"):
        assert got == want, (rank, got)


@pytest.mark.parametrize("world", [2, 4])
def test_strided_slabs_and_pipelined_pairs(world):
    for rank, ok, want in _run(world, "strided"):
        assert ok is want, (rank, ok)
    for rank, got, want in _run(world, "pipeline"):
        assert got == want, (rank, got)


def test_aux_slabs_reassemble():
    for rank, ok, want in _run(2, "slabs"):
        assert ok is want, (rank, ok)


def test_failed_rank_does_not_hang_the_others():
    res = dict((r, g) for r, g, _ in _run(2, "fail"))
    assert res[1] == "raised"
    assert res[0] == "error"


def test_host_copy_plan_covers_each_ranks_pairs():
    """Host-resident B: a rank copies row chunks in host_copy_plan's order and
    runs, after each chunk, the pair ranges listed with it. Those ranges must
    partition the rank's pair range, every pair must have both rows resident
    by then, the rows copied must be exactly those host_bytes_needed counts,
    and pairs must be runnable after at most two chunks (so that the copy
    overlaps compute on every rank)."""
    from trntensor_b200.dispatch import block_assignment, host_copy_plan

    for nocc in (1, 2, 5, 17, 64, 256):
        npairs = nocc * (nocc + 1) // 2
        ids = [(i, j) for i in range(nocc) for j in range(i, nocc)]
        for world in (1, 2, 3, 8):
            for rank in range(world):
                pb, pe = distributed.pair_range(npairs, rank, world)
                plan = host_copy_plan(nocc, pb, pe)
                if pe <= pb:
                    assert plan == []
                    continue
                resident: set[int] = set()
                covered = []
                for step, (a, b, ranges) in enumerate(plan):
                    assert a < b and not resident & set(range(a, b))  # each row once
                    resident |= set(range(a, b))
                    if step == 1 and nocc >= 17:
                        assert covered or ranges, "nothing runnable after two chunks"
                    for lo, hi in ranges:
                        assert pb <= lo < hi <= pe
                        for p in range(lo, hi):
                            i, j = ids[p]
                            assert i in resident and j in resident
                        covered.extend(range(lo, hi))
                assert sorted(covered) == list(range(pb, pe))  # each pair exactly once
                rows = len(resident)
                assert resident == set(range(nocc - rows, nocc))
                if block_assignment(nocc, rank, world) is None:
                    assert rows * 7 * 3 * 4 == distributed.host_bytes_needed(nocc, 7, 3, rank,
                                                                             world)
                # launches stay few: one range per step when the rank owns the last row
                nranges = sum(len(r) for _, _, r in plan)
                assert nranges <= len(plan) * max(1, nocc // world + 2)


@pytest.mark.parametrize("world", [4, 8])
def test_block_plan_energy_all_reduce(world):
    """gloo ranks run the row-group block plan's ranges and all-reduce: every
    pair id is counted exactly once over the job."""
    for rank, got, want in _run(world, "blocks"):
        assert got == want, rank


def test_block_assignment_partition_balance_and_rows():
    """At 4 and 8 ranks the row-group blocks partition all unordered pairs,
    balance the work to within one group's diagonal, and need at most half
    (8 ranks) or three quarters (4 ranks) of the rows; chunk_plan runs every
    pair of a rank exactly once, after both of its rows have landed, and
    something is runnable after the first two chunks."""
    from trntensor_b200.dispatch import block_assignment, chunk_plan

    for nocc in (8, 9, 23, 64, 256):
        npairs = nocc * (nocc + 1) // 2
        ids = [(i, j) for i in range(nocc) for j in range(i, nocc)]
        for world in (4, 8):
            seen = []
            work = []
            for rank in range(world):
                ranges, order = block_assignment(nocc, rank, world)
                mine = [p for lo, hi in ranges for p in range(lo, hi)]
                seen += mine
                work.append(len(mine))
                rows = [r for a, b in order for r in range(a, b)]
                assert len(rows) == len(set(rows))
                limit = 0.5 if world == 8 or rank < 2 else 0.75
                assert len(rows) <= limit * nocc + 2
                assert set(rows) == {r for p in mine for r in ids[p]}
                resident: set[int] = set()
                covered = []
                for step, (a, b, rr) in enumerate(chunk_plan(nocc, ranges, order)):
                    resident |= set(range(a, b))
                    for lo, hi in rr:
                        for p in range(lo, hi):
                            assert set(ids[p]) <= resident
                        covered += range(lo, hi)
                    if step == 1 and nocc >= 64:
                        assert covered
                assert sorted(covered) == sorted(mine)
                assert distributed.host_bytes_needed(nocc, 7, 3, rank, world) == len(rows) * 84
            assert sorted(seen) == list(range(npairs))
            g = 4 if world == 8 else 2
            assert max(work) - min(work) <= 2 * (-(-nocc // g))
            if nocc == 256:
                assert max(work) / min(work) <= 1.02
    for world in (1, 2, 3):
        assert block_assignment(256, 0, world) is None
