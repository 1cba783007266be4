"""Per-shape kernel choice, read from the committed sweep table ``dispatch_table.json``.

Replaces the reference's hand-filled tables BF16_CONFIGS / NF12_CUDA_DISPATCH / TMA_DISPATCH
(submission.py:76-127, 900-908), which its Optuna and grid sweeps filled (sweep_all.py,
sweep_cuda.py). Here ``muse_bf16_proj_b200/sweep.py`` times every candidate plan per shape on a
B200 and writes the table; rows are keyed by (N, K, M range) and name the weight format
("bf16" or "12b") and the plan. A shape no row covers takes the library's default plan
(muse_plan_default), so every shape runs on this build's kernels; nothing falls back to cuBLAS.
"""

from __future__ import annotations

import json
import os

from . import _lib

HERE = os.path.dirname(os.path.abspath(__file__))
TABLE_PATH = os.path.join(HERE, "dispatch_table.json")


class Dispatch:
    def __init__(self, path: str | None = TABLE_PATH, entries: list | None = None):
        self.entries = []
        if entries is not None:
            self.entries = list(entries)
        elif path and os.path.exists(path):
            with open(path) as f:
                self.entries = json.load(f).get("entries", [])
        self._cache: dict = {}

    def _match(self, m: int, n: int, k: int, have_12b: bool):
        for e in self.entries:
            if e["n"] == n and e["k"] == k and e["m_lo"] <= m <= e["m_hi"]:
                if e.get("weights", "bf16") == "12b" and not have_12b:
                    continue
                return e
        return None

    def plan(self, m: int, n: int, k: int, have_12b: bool = False, tiles: bool = True) -> tuple[_lib.MusePlan, str]:
        """(plan, weight format) for y[m, n] = x[m, k] W[n, k]^T; `tiles`: a packed copy of W
        exists (table rows assume it, as prepare makes one)."""
        key = (m, n, k, have_12b, tiles)
        hit = self._cache.get(key)
        if hit is None:
            e = self._match(m, n, k, have_12b)
            if e is not None:
                hit = (_lib.MusePlan.from_dict(e["plan"]), e.get("weights", "bf16"))
            else:
                hit = (_lib.plan_default(m, n, k, False, tiles=tiles), "bf16")
            self._cache[key] = hit
        return hit

    def wants_12b(self, n: int, k: int) -> bool:
        """True when some row serves this weight shape from 12-bit planes."""
        return any(e["n"] == n and e["k"] == k and e.get("weights") == "12b" for e in self.entries)

    def ms_for(self, n: int, k: int) -> list[tuple[int, int, str]]:
        return [(e["m_lo"], e["m_hi"], e.get("weights", "bf16")) for e in self.entries if e["n"] == n and e["k"] == k]
