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


def float_names():
    """Fixtures of the reference searching with a float (fp32 ResNet) evaluator whose outputs are
    recorded per position (make_golden.py float_cases)."""
    return sorted(os.path.basename(p)[len("floatsearch_"):-len(".npz")]
                  for p in glob.glob(os.path.join(GOLDEN, "floatsearch_*.npz")))


def load_float(name):
    z = np.load(os.path.join(GOLDEN, f"floatsearch_{name}.npz"))
    return {k: z[k] for k in z.files}


class ReplayEvaluator:
    """Returns, for each position of a batch, the outputs the reference's evaluator gave for the
    same fp32 feature bytes. Accepts numpy or torch features (torch outputs for torch input)."""

    def __init__(self, g):
        self.index = {str(k): i for i, k in enumerate(g["table_keys"])}
        self.policy = g["table_policy"]
        self.value = g["table_value"]
        self.misses = 0

    def _lookup(self, f):
        f = np.ascontiguousarray(f, dtype=np.float32)
        idx = []
        for x in f:
            i = self.index.get(hashlib.sha256(x.tobytes()).hexdigest())
            if i is None:
                self.misses += 1
                i = 0
            idx.append(i)
        return self.policy[idx], self.value[idx]

    def __call__(self, f):
        return self._lookup(f)

    def evaluate_batch(self, features):
        import torch
        p, v = self._lookup(features.cpu().numpy())
        return torch.from_numpy(p).to(features.device), torch.from_numpy(v).to(features.device)
