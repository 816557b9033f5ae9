"""Multi-GPU DF-MP2 and AO->MO: one process per GPU over torch.distributed.

* ``mp2_energy``: B is replicated on every rank; the unordered occupied
  pairs (i <= j, row-major linear ids) are split into equal contiguous
  ranges (or, for a host-resident B at 4 and 8 ranks, into row-group
  blocks that halve what each rank copies), each rank runs the fused
  kernel on its pairs, and one fp64 scalar is summed across ranks (NCCL
  all-reduce on GPUs, gloo on CPU).
* ``ao_to_mo_transform``: each rank transforms its own slab of the
  auxiliary index P; there is no communication. ``aux_slab`` gives the slab.

The reference has no multi-device code; this module is B200-specific.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from .dispatch import _cuda_mp2_energy, block_assignment


def _world(group=None) -> tuple[int, int]:
    if not (dist.is_available() and dist.is_initialized()):
        return 0, 1
    return dist.get_rank(group), dist.get_world_size(group)


def pair_range(npairs: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous, balanced share [begin, end) of ``npairs`` for ``rank``."""
    base, rem = divmod(npairs, world)
    begin = rank * base + min(rank, rem)
    return begin, begin + base + (1 if rank < rem else 0)


def aux_slab(naux: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous share [p0, p1) of the auxiliary index for ``rank``."""
    return pair_range(naux, rank, world)


def host_bytes_needed(nocc: int, nvir: int, naux: int, rank: int, world: int) -> int:
    """Bytes of a host fp32 B a rank copies in ``mp2_energy``: the rows of its
    row-group blocks (``block_assignment``, 4 and 8 ranks), else rows
    first_row(pair_begin)..nocc-1 of its contiguous pair range."""
    from .dispatch import first_row_of_pair

    blocks = block_assignment(nocc, rank, world)
    if blocks is not None:
        return sum(b - a for a, b in blocks[1]) * nvir * naux * 4
    pb, pe = pair_range(nocc * (nocc + 1) // 2, rank, world)
    if pe <= pb:
        return 0
    return (nocc - first_row_of_pair(pb, nocc)) * nvir * naux * 4


def reduce_energy(local: torch.Tensor, group=None) -> torch.Tensor:
    """Sum a 0-D fp64 tensor over the group (in place) and return it."""
    _, world = _world(group)
    if world > 1:
        dist.all_reduce(local, op=dist.ReduceOp.SUM, group=group)
    return local


def mp2_energy(
    B: torch.Tensor,
    eps_occ: torch.Tensor,
    eps_vir: torch.Tensor,
    *,
    precision: str = "fast",
    group=None,
) -> torch.Tensor:
    """DF-MP2 energy with the pairs sharded over the process group.

    Every rank passes the full (replicated) inputs and gets the full energy
    back, as a 0-D tensor of ``B.dtype`` on ``B``'s device.
    """
    from .quantum import _validate_mp2

    _validate_mp2(B, eps_occ, eps_vir, precision)
    rank, world = _world(group)
    nocc = int(B.shape[0])
    if B.numel() == 0:  # same shapes on every rank: all of them return here
        return B.new_zeros(())
    npairs = nocc * (nocc + 1) // 2
    # A host-resident B is copied by every rank: at 4 and 8 ranks the pairs
    # are assigned by row-group blocks so that each rank copies about half
    # of B (block_assignment); on the device the contiguous ranges are kept.
    blocks = block_assignment(nocc, rank, world) if B.device.type == "cpu" else None
    e, _ = _cuda_mp2_energy(
        B, eps_occ, eps_vir, precision=precision, pair_range=pair_range(npairs, rank, world),
        blocks=blocks,
    )
    reduce_energy(e, group)
    return e.to(device=B.device, dtype=B.dtype)


def ao_to_mo_transform(
    eri: torch.Tensor,
    C_occ: torch.Tensor,
    C_vir: torch.Tensor,
    *,
    precision: str = "fast",
    group=None,
    sharded_input: bool = False,
) -> torch.Tensor:
    """AO->MO transform of this rank's slab of the auxiliary index.

    With ``sharded_input=False`` every rank passes the full eri and transforms
    ``eri[:, :, p0:p1]`` (its ``aux_slab``); with ``sharded_input=True`` eri is
    already the rank's contiguous slab. Returns the rank's (nocc, nvir, p1-p0)
    block of B. There is no communication.
    """
    from .dispatch import _cuda_ao_to_mo_slab
    from .quantum import ao_to_mo_transform as _single

    rank, world = _world(group)
    if sharded_input:
        return _single(eri, C_occ, C_vir, precision=precision)
    p0, p1 = aux_slab(int(eri.shape[2]), rank, world)
    if precision == "fast" and eri.is_cuda and eri.dtype == torch.float32:
        # the rank's aux columns are read in place (strided 3-D tensor map)
        from .quantum import _validate_ao2mo

        _validate_ao2mo(eri, C_occ, C_vir, precision)
        return _cuda_ao_to_mo_slab(eri, C_occ, C_vir, p0, p1)
    return _single(eri[:, :, p0:p1], C_occ, C_vir, precision=precision)


def gather_aux(local: torch.Tensor, naux: int, group=None) -> torch.Tensor:
    """Reassemble the full (nocc, nvir, naux) B from every rank's slab."""
    rank, world = _world(group)
    if world == 1:
        return local
    parts = [None] * world
    dist.all_gather_object(parts, local.cpu(), group=group)
    return torch.cat(parts, dim=2).to(local.device)
