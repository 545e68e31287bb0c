"""Seeded fault positions, drawn the way the reference's injector draws them.

pytorch/abft/injector.py:24 and :71 pick one flat output index with
``random.Random(seed).randrange(numel)`` (row-major: row = idx // N,
col = idx % N). For the multi-fault cases each further draw that reuses a
row or a column is skipped, so every fault sits in its own row and column.
"""
from __future__ import annotations

import random
from typing import List, Tuple


def seeded_fault_positions(m: int, n: int, count: int, seed: int) -> List[Tuple[int, int]]:
    if count > min(m, n):
        raise ValueError("more faults than distinct rows or columns")
    rng = random.Random(seed)
    out: List[Tuple[int, int]] = []
    rows, cols = set(), set()
    while len(out) < count:
        r, c = divmod(rng.randrange(m * n), n)
        if r in rows or c in cols:
            continue
        rows.add(r)
        cols.add(c)
        out.append((r, c))
    return out
