"""Pin the C++ oracle against the reference's own search (fixtures from tests/golden/make_golden.py).

Bit-exact on every node array (visit counts, value sums, priors, virtual-loss counts, parent ids,
parent actions, the dense children table), the root policy, the final move, and the exact
sequence of feature tensors handed to the evaluator.
"""
import hashlib

import numpy as np
import pytest

from golden_cases import ReplayEvaluator, children_table, digest, float_names, load, load_float, names


def _run_oracle(pyoracle, g, trace=False):
    o = pyoracle.Oracle(int(g["capacity"]))
    h = hashlib.sha256()

    def ev(f):
        f = np.ascontiguousarray(f, np.float32)
        h.update(hashlib.sha256(f.tobytes()).digest())
        return pyoracle.synth_eval(f)

    t = o.search(g["board"], int(g["sims"]), int(g["wave"]), evaluator=ev if trace else None,
                 c_puct=float(g["c_puct"]), virtual_loss=float(g["virtual_loss"]),
                 enable_vl=bool(g["enable_vl"]))
    return t, h.hexdigest()


@pytest.mark.parametrize("name", names())
def test_oracle_matches_reference(oracle_lib, name):
    g = load(name)
    big = int(g["num_nodes"]) > 200000
    t, trace = _run_oracle(oracle_lib, g, trace=not big)
    assert t.result["status"] == 0
    assert t.result["boundary_ties"] == 0
    assert t.visits.shape[0] == int(g["num_nodes"])
    assert digest(t.visits) == str(g["sha_visits"])
    assert digest(t.value_sums) == str(g["sha_value_sums"])
    assert digest(t.priors) == str(g["sha_priors"])
    assert digest(t.virtual_loss) == str(g["sha_virtual_loss"])
    assert digest(t.parent) == str(g["sha_parent"])
    assert digest(t.action) == str(g["sha_action"])
    assert digest(children_table(t.parent, t.action)) == str(g["sha_children"])
    assert np.array_equal(t.policy, g["policy"])
    assert int(np.argmax(t.policy)) == int(g["final_move"])
    assert t.result["eval_calls"] == int(g["eval_calls"])
    assert t.result["eval_positions"] == int(g["eval_positions"])
    if not big:
        assert trace == str(g["eval_trace"])


def test_synthetic_evaluator_numpy_equals_c(oracle_lib):
    rng = np.random.default_rng(3)
    f = np.zeros((64, 19, 15, 15), np.float32)
    f[:, 0] = rng.random((64, 15, 15)) < 0.3
    f[:, 1] = rng.integers(1, 3, (64, 1, 1))
    f[:, 2].reshape(64, -1)[np.arange(64), rng.integers(0, 225, 64)] = 1
    p1, v1 = oracle_lib.synth_eval(f)
    p2, v2 = oracle_lib.c_synth_eval(f)
    assert np.array_equal(p1, p2) and np.array_equal(v1, v2)
    # legal priors are distinct multiples of 2^-24 whose sum is exact, values on a 2^-12 grid
    q = p1 * 2.0 ** 24
    assert np.array_equal(q, np.round(q))
    for row, legal in zip(q, f[:, 0].reshape(64, -1) == 0):
        vals = row[legal]
        assert len(np.unique(vals)) == len(vals)
        assert vals.sum() <= 2 ** 24
    assert np.array_equal(v1 * 4096, np.round(v1 * 4096)) and np.all(np.abs(v1) < 1)


def _const_eval(v):
    def ev(features):
        n = features.shape[0]
        return np.full((n, 225), 1.0 / 225, np.float32), np.full(n, v, np.float32)
    return ev


def test_backup_sign_convention_three_node_path(oracle_lib):
    """The reference's own anchor (python/tests/test_mcts_phases_detailed.py:578-616): after one
    simulation the path root -> child -> leaf holds leaf +v, parent -v, root +v; the policy has
    225 entries and sums to 1."""
    board = np.zeros((15, 15), np.int8)
    t = oracle_lib.Oracle(20000).search(board, 1, 1, evaluator=_const_eval(0.5))
    leaf = int(np.nonzero(t.visits[1:])[0].max()) + 1
    child = int(t.parent[leaf])
    assert t.parent[child] == 0
    assert (t.visits[0], t.visits[child], t.visits[leaf]) == (1, 1, 1)
    assert (t.value_sums[0], t.value_sums[child], t.value_sums[leaf]) == (0.5, -0.5, 0.5)
    assert t.policy.shape == (225,) and abs(t.policy.sum() - 1.0) < 1e-12


def test_torch_sum_order_is_torchs(oracle_lib):
    """The oracle's summation order of the prior normalisation (`priors.sum()`,
    wave_search.py:894-895) equals torch.sum on CPU bit for bit, at every length up to 600 and at
    sampled lengths up to 5,000 (past the 16-row cascade of the kernel), on values whose sums are
    far from exact in fp32."""
    import torch
    rng = np.random.default_rng(0)
    lengths = list(range(1, 601)) + [int(n) for n in rng.integers(601, 5001, 300)]
    for n in lengths:
        for scale in (1.0, 1e-3, 3e4):
            x = (rng.random(n) ** 3 * scale).astype(np.float32)
            assert oracle_lib.torch_sum(x) == torch.from_numpy(x).sum().numpy(), n


@pytest.mark.parametrize("name", float_names())
def test_oracle_matches_reference_with_float_evaluator(oracle_lib, name):
    """The reference searched with a float evaluator (fp32 ResNet outputs, recorded per position);
    the oracle replaying the same outputs builds the same tree bit for bit: the priors' summation
    order, and with it every prior, visit count and value sum, is the reference's."""
    g = load_float(name)
    ev = ReplayEvaluator(g)
    t = oracle_lib.Oracle(int(g["capacity"])).search(g["board"], int(g["sims"]), int(g["wave"]), evaluator=ev)
    assert ev.misses == 0
    assert t.result["status"] == 0 and t.result["boundary_ties"] == 0
    assert t.visits.shape[0] == int(g["num_nodes"])
    for k in ("visits", "value_sums", "priors", "virtual_loss", "parent", "action"):
        assert digest(getattr(t, k)) == str(g["sha_" + k]), k
    assert digest(children_table(t.parent, t.action)) == str(g["sha_children"])
    assert np.array_equal(t.policy, g["policy"])
