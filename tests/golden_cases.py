"""Loader for the reference-generated search fixtures in tests/golden (see make_golden.py)."""
import glob
import hashlib
import os

import numpy as np

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def names():
    return sorted(os.path.basename(p)[len("search_"):-len(".npz")]
                  for p in glob.glob(os.path.join(GOLDEN, "search_*.npz")))


def load(name):
    z = np.load(os.path.join(GOLDEN, f"search_{name}.npz"))
    return {k: z[k] for k in z.files}


def digest(a) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def children_table(parent, action, actions=225):
    n = parent.shape[0]
    ch = np.full((n, actions), -1, np.int32)
    ch[parent[1:], action[1:]] = np.arange(1, n, dtype=np.int32)
    return ch
