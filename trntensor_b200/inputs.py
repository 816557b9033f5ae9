"""Seeded synthetic inputs with the shapes and value distributions of the
benchmark configurations (DF-MP2 B tensors, orbital energies, orthonormal
MO coefficients and (m,n)-symmetric 3-index integrals).

Two generators:
* ``device="cpu"`` (default): ``torch.Generator("cpu")``, values drawn in
  fp64 and then cast, so fp32 and fp64 runs see the same numbers;
* a CUDA device: drawn directly on the GPU in the requested dtype (used for
  the multi-GB benchmark configurations; different values, same
  distributions).
"""

from __future__ import annotations

import math

import torch

# BASELINE configurations: name -> sizes.
CONFIGS = {
    0: dict(kind="mp2", nocc=8, nvir=32, naux=96),
    1: dict(kind="ao2mo", nbf=128, nocc=16, nvir=112, naux=384),
    2: dict(kind="mp2", nocc=64, nvir=448, naux=1536),
    3: dict(kind="ao2mo", nbf=1024, nocc=128, nvir=896, naux=3072),
    4: dict(kind="mp2", nocc=256, nvir=1792, naux=6144),
}


def _gen(device, seed):
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def mp2_inputs(nocc, nvir, naux, seed=0, dtype=torch.float32, device="cpu"):
    """B ~ N(0,1)/sqrt(naux); eps_occ ~ U[-2.0,-0.5]; eps_vir ~ U[0.2,3.0]."""
    dev = torch.device(device)
    draw = torch.float64 if dev.type == "cpu" else dtype
    g = _gen(dev, seed)
    B = torch.randn(nocc, nvir, naux, generator=g, dtype=draw, device=dev)
    B.mul_(1.0 / math.sqrt(naux))
    eo = torch.rand(nocc, generator=g, dtype=draw, device=dev) * 1.5 - 2.0
    ev = torch.rand(nvir, generator=g, dtype=draw, device=dev) * 2.8 + 0.2
    return B.to(dtype), eo.to(dtype), ev.to(dtype)


def ao2mo_inputs(nbf, nocc, nvir, naux, seed=0, dtype=torch.float32, device="cpu"):
    """C = Q of QR(N(0,1) (nbf, nocc+nvir)); eri[m,n,P] = L[m,P] L[n,P] / naux."""
    dev = torch.device(device)
    draw = torch.float64 if dev.type == "cpu" else dtype
    g = _gen(dev, seed)
    nmo = nocc + nvir
    G = torch.randn(nbf, nmo, generator=g, dtype=draw, device=dev)
    Q, _ = torch.linalg.qr(G)
    C_occ = Q[:, :nocc].contiguous()
    C_vir = Q[:, nocc:nmo].contiguous()
    L = torch.randn(nbf, naux, generator=g, dtype=draw, device=dev)
    eri = (L.unsqueeze(1) * L.unsqueeze(0)).mul_(1.0 / naux)
    return eri.to(dtype), C_occ.to(dtype), C_vir.to(dtype)


def mp2_row(i, nvir, naux, seed=0):
    """Row i of the row-wise seeded B: N(0,1)/sqrt(naux) from numpy's
    Generator seeded with (seed, i), drawn in fp32. Any row can be made on its
    own, so a checker can rebuild just the rows of the pairs it checks."""
    import numpy as np

    x = np.random.default_rng([seed, i]).standard_normal((nvir, naux), dtype=np.float32)
    x *= np.float32(1.0 / math.sqrt(naux))
    return x


def mp2_eps_rowwise(nocc, nvir, seed=0):
    """Orbital energies of the row-wise recipe: eps_occ ~ U[-2.0,-0.5],
    eps_vir ~ U[0.2,3.0] (fp32), from a Generator seeded with (seed, 2^31)."""
    import numpy as np

    rng = np.random.default_rng([seed, 2**31])
    eo = (rng.random(nocc) * 1.5 - 2.0).astype(np.float32)
    ev = (rng.random(nvir) * 2.8 + 0.2).astype(np.float32)
    return torch.from_numpy(eo), torch.from_numpy(ev)


def mp2_inputs_rowwise(nocc, nvir, naux, seed=0, out=None, rows=None, threads=None):
    """fp32 B (nocc, nvir, naux) of the row-wise recipe plus eps, on the host.

    ``out``: a preallocated (e.g. pinned) host tensor to fill; ``rows``: fill
    only these rows (the others are left as they are). Rows are drawn on a
    thread pool (numpy releases the GIL), about 0.3 s per 11M-value row per
    thread. The multi-GB benchmark configuration uses this recipe so that the
    oracle can recompute any pair from two regenerated rows.
    """
    from concurrent.futures import ThreadPoolExecutor
    import os

    B = out if out is not None else torch.empty((nocc, nvir, naux), dtype=torch.float32)
    idx = list(range(nocc)) if rows is None else list(rows)

    def fill(i):
        B[i].copy_(torch.from_numpy(mp2_row(i, nvir, naux, seed)))

    n = threads or min(32, os.cpu_count() or 1)
    with ThreadPoolExecutor(max_workers=n) as ex:
        list(ex.map(fill, idx))
    eo, ev = mp2_eps_rowwise(nocc, nvir, seed)
    return B, eo, ev
