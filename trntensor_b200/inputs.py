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
