"""Loads the golden fixtures written by tests/golden/make_golden.py (reference outputs)."""
from __future__ import annotations

import os
from dataclasses import dataclass

import numpy as np

from oracle_lib import Feature, TableDef

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
CASES = ("small_multi_table", "small_bounded", "hot_segments", "cfg1_shape")


@dataclass
class Case:
    name: str
    tables: list
    features: list
    grads: list            # per step: list of arrays (one per feature)
    lookup: dict           # shards -> list of outputs
    state: dict            # table id -> (keys, w, m, v, updates)
    steps: int


def load(name: str) -> Case:
    z = np.load(os.path.join(GOLDEN, f"{name}.npz"))
    lr = float(z["lr"])
    b = z["bounds"]
    bounds = None if np.isnan(b[0]) else (float(b[0]), float(b[1]))
    tables = [TableDef(id=int(i), dimension=int(d), learning_rate=lr, bounds=bounds,
                       init_min=-0.05, init_max=0.05, init_seed=42, rows=int(r))
              for i, d, r in zip(z["table_ids"], z["table_dims"], z["table_rows"])]
    n = int(z["feature_count"])
    feats = []
    for i in range(n):
        t, f, p = (int(x) for x in z[f"f{i}_meta"])
        feats.append(Feature(t, f, p, z[f"f{i}_keys"], z[f"f{i}_offsets"]))
    steps = int(z["steps"])
    grads = [[z[f"grad_step{s}_f{i}"] for i in range(n)] for s in range(steps)]
    lookup = {s: [z[f"lookup_s{s}_f{i}"] for i in range(n)] for s in (1, 2, 3)}
    state = {t.id: (z[f"t{t.id}_keys"], z[f"t{t.id}_w"], z[f"t{t.id}_m"], z[f"t{t.id}_v"],
                    z[f"t{t.id}_updates"]) for t in tables}
    return Case(name, tables, feats, grads, lookup, state, steps)
