"""Fixture of 64 per-pair DF-MP2 energies of BASELINE config 4 (nocc 256,
nvir 1792, naux 6144), in fp64, on the row-wise seeded inputs
(``trntensor_b200.inputs.mp2_inputs_rowwise``, seed 0).

TEST INFRASTRUCTURE: each E_ij is the oracle's restatement of the
reference's loop body (oracle.mp2_pair_energy, trntensor/quantum.py:87-100)
evaluated in fp64 on the two regenerated fp32 rows i and j. The 64 unordered
pairs are drawn with a fixed seed over the whole pair range (diagonal pairs
included). Run from the repository root: ``python tests/golden/make_config4_pairs.py``
(about a minute on 8 cores).
"""

from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from oracle import oracle  # noqa: E402
from trntensor_b200.inputs import mp2_eps_rowwise, mp2_row  # noqa: E402

NOCC, NVIR, NAUX, SEED = 256, 1792, 6144, 0
OUT = Path(__file__).resolve().parent / "config4_pairs.json"


def sample_pairs(n=64):
    rng = np.random.default_rng(12345)
    pairs = set()
    # a few fixed corners of the pair range, then random unordered pairs
    for p in ((0, 0), (0, NOCC - 1), (NOCC - 1, NOCC - 1), (127, 128)):
        pairs.add(p)
    while len(pairs) < n:
        i, j = sorted(int(v) for v in rng.integers(0, NOCC, 2))
        if len(pairs) % 8 == 0:
            j = i  # some diagonal pairs
        pairs.add((i, j))
    return sorted(pairs)


def main():
    eo, ev = (t.numpy() for t in mp2_eps_rowwise(NOCC, NVIR, SEED))
    pairs = sample_pairs()
    rows = {}
    out = []
    for i, j in pairs:
        for r in (i, j):
            if r not in rows:
                rows[r] = mp2_row(r, NVIR, NAUX, SEED)
        Bij = np.stack([rows[i], rows[j]]).astype(np.float64)
        e = float(oracle.mp2_pair_energy(Bij, eo[[i, j]].astype(np.float64),
                                         ev.astype(np.float64), 0, 1))
        out.append([i, j, e])
    row_sums = {str(r): float(rows[r].astype(np.float64).sum()) for r in sorted(rows)}
    OUT.write_text(json.dumps({"config": {"nocc": NOCC, "nvir": NVIR, "naux": NAUX,
                                          "seed": SEED, "recipe": "mp2_inputs_rowwise"},
                               "pairs": out, "row_sums": row_sums}, indent=0))
    print(f"wrote {len(out)} pairs to {OUT}")


if __name__ == "__main__":
    main()
