"""Loader for the committed golden fixtures (tests/golden/*.npz, made by make_golden.py)."""
import json
from pathlib import Path

import numpy as np
import torch

GOLDEN = Path(__file__).resolve().parent / "golden"


def cases(family: str):
    """Yields (meta dict, {array name: torch tensor}) for every case of a fixture family."""
    with np.load(GOLDEN / f"{family}.npz") as z:
        meta = json.loads(str(z["meta"]))
        for m in meta:
            prefix = m["name"] + "__"
            arrays = {k[len(prefix):]: torch.from_numpy(np.array(z[k])) for k in z.files if k.startswith(prefix)}
            yield m, arrays


def case_ids(family: str):
    return [m["name"] for m, _ in cases(family)]
