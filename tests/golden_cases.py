"""Loader for the golden fixtures in tests/golden (made by make_golden.py)."""
import json
from pathlib import Path

import numpy as np

GOLDEN = Path(__file__).resolve().parent / "golden"


def names():
    return json.loads((GOLDEN / "index.json").read_text())


def load(name):
    z = np.load(GOLDEN / f"{name}.npz", allow_pickle=False)
    meta = json.loads(str(z["meta"]))
    return meta, z["rows"], z["o"].astype(np.float64), z["lse"]


def inputs_for(meta):
    from oracle import ref_attention as R
    if meta["kind"] == "edge":
        q, k, v, _ = R.edge_inputs(seed=meta["seed"], b=meta["b"], h=meta["h"], sq=meta["sq"], sk=meta["sk"])
    else:
        q, k, v = R.inputs(meta["b"], meta["h"], meta["sq"], meta["sk"], meta["pattern"], seed=meta["seed"])
    return q, k, v
