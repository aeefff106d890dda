"""Helpers that read the committed golden fixtures (tests/golden/*.npz)."""

from __future__ import annotations

import json
from pathlib import Path

import numpy as np

GOLDEN = Path(__file__).resolve().parent / "golden"


def names(kind: str | None = None):
    out = []
    for p in sorted(GOLDEN.glob("*.npz")):
        if kind is None or p.stem.startswith(kind):
            out.append(p.stem)
    return out


def load(name: str):
    z = np.load(GOLDEN / f"{name}.npz")
    meta = json.loads(str(z["meta"]))
    arrs = {k: z[k] for k in z.files if k != "meta"}
    return meta, arrs
