"""Generate the golden search fixtures from the REFERENCE implementation itself.

Runs the reference's deterministic CPU search path
    MCTS(MCTSConfig(backend='gpu', device='cpu', wave_async_expansion=False, dirichlet_epsilon=0,
                    enable_subtree_reuse=False, ...), evaluator).search(board)
(python/mcts/core/mcts.py:924, python/mcts/core/wave_search.py:555) imported from the reference
source tree, driven by the integer-exact synthetic evaluator (numpy twin in oracle/pyoracle.py).
Each case is written to tests/golden/search_<name>.npz with:
  * the root board and configuration,
  * the root policy (fp64) and root-children visit counts / value sums,
  * SHA-256 digests of the whole tree (visit counts, value sums, priors, virtual-loss counts,
    parent ids, parent actions, children table),
  * the full node arrays for small trees,
  * a digest of every feature tensor the reference passed to its evaluator, in call order.

Usage (needs the reference tree and its C++ game engines built by `make -C oracle ref`):
    python tests/golden/make_golden.py --reference <reference source tree>  (or OMQ_REFERENCE) [--only NAME ...]
This runs only in the build container; the GPU box never reads the reference.
"""
from __future__ import annotations

import argparse
import hashlib
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
FULL_ARRAYS_MAX_NODES = 6000


def digest(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def dense_board(seed: int, empties: int) -> np.ndarray:
    """A nearly full board without five in a row: colour = 1 + ((r + 2c) % 4 >= 2)."""
    r, c = np.mgrid[0:15, 0:15]
    b = (1 + ((r + 2 * c) % 4 >= 2)).astype(np.int8)
    rng = np.random.default_rng(seed)
    b.flat[rng.choice(225, empties, replace=False)] = 0
    return b


def open_four_board() -> np.ndarray:
    b = np.zeros((15, 15), np.int8)
    b[7, 3:7] = 1                      # black to move has an open four on row 7
    b[2, 2], b[3, 10], b[11, 4], b[12, 12] = 2, 2, 2, 2
    return b


def root_five_board() -> np.ndarray:
    b = np.zeros((15, 15), np.int8)
    b[7, 3:8] = 1                      # the root already contains a black five
    b[1, 1], b[2, 9], b[10, 3], b[12, 7], b[13, 13] = 2, 2, 2, 2, 2
    return b


def cases():
    from omoknuni_quantum_b200.roots import random_root
    return [
        # name, board, sims, wave, c_puct, virtual_loss, enable_vl, capacity
        ("cfg0_seed0", random_root(0), 800, 256, 1.4, 1.0, True, 200000),
        ("cfg0_seed1", random_root(1), 800, 256, 1.4, 1.0, True, 200000),
        ("ragged_seed2", random_root(2), 300, 128, 1.4, 1.0, True, 200000),
        ("wave16_seed3", random_root(3), 256, 16, 1.4, 1.0, True, 200000),
        ("dense", dense_board(7, 30), 200, 32, 1.4, 1.0, True, 200000),
        ("empty_root", np.zeros((15, 15), np.int8), 128, 64, 1.4, 1.0, True, 200000),
        ("open_four", open_four_board(), 200, 64, 1.4, 1.0, True, 200000),
        ("root_five", root_five_board(), 64, 32, 1.4, 1.0, True, 200000),
        ("novl_c25_seed4", random_root(4), 200, 64, 2.5, 1.0, False, 200000),
        ("wave1_seed6", random_root(6), 12, 1, 1.4, 1.0, True, 200000),
        ("cfg1_seed5", random_root(5), 1600, 256, 1.4, 1.0, True, 400000),
    ]


class TracingSynthEvaluator:
    """Reference-facing evaluator: numpy synthetic evaluator + a digest of each call's features."""

    def __init__(self):
        from oracle.pyoracle import synth_eval
        self._eval = synth_eval
        self.calls = 0
        self.positions = 0
        self._h = hashlib.sha256()

    def evaluate_batch(self, features):
        import torch
        f = features.cpu().numpy() if hasattr(features, "cpu") else np.asarray(features)
        f = np.ascontiguousarray(f, dtype=np.float32)
        self.calls += 1
        self.positions += f.shape[0]
        self._h.update(hashlib.sha256(f.tobytes()).digest())
        p, v = self._eval(f)
        return torch.from_numpy(p), torch.from_numpy(v)

    def trace_digest(self) -> str:
        return self._h.hexdigest()


def float_cases():
    from omoknuni_quantum_b200.roots import random_root
    return [
        # name, board, sims, wave, capacity
        ("seed30_w32", random_root(30), 160, 32, 100000),
        ("seed31_w64", random_root(31), 192, 64, 100000),
        ("dense6_w4", dense_board(10, 6), 40, 4, 100000),
        ("dense12_w16", dense_board(8, 12), 64, 16, 100000),
        ("dense40_w8", dense_board(9, 40), 96, 8, 100000),
    ]


class RecordingFloatEvaluator:
    """Reference-facing float evaluator: an fp32 ResNet 2 x 128 (the architecture of the
    reference's ResNetModel, seeded weights) evaluated one position at a time on the CPU, so that a
    position's outputs never depend on the batch it came in. Every distinct position's outputs are
    recorded under the SHA-256 of its fp32 feature bytes, so that the engine and the oracle can
    replay exactly the reference's evaluator outputs. Its priors are generic fp32 values: their
    sums are inexact, so the summation order of the prior normalisation shows."""

    def __init__(self):
        from omoknuni_quantum_b200.resnet import ResNetSpec, init_state_dict
        self.sd = init_state_dict(ResNetSpec(num_blocks=2, filters=128, fc_value_hidden=64), seed=77)
        self.table = {}
        self.calls = 0

    def evaluate_batch(self, features):
        import torch
        from omoknuni_quantum_b200.resnet import reference_forward_fp32
        f = features.cpu().numpy() if hasattr(features, "cpu") else np.asarray(features)
        f = np.ascontiguousarray(f, dtype=np.float32)
        self.calls += 1
        ps, vs = [], []
        for x in f:
            key = hashlib.sha256(x.tobytes()).hexdigest()
            if key not in self.table:
                with torch.no_grad():
                    p, v = reference_forward_fp32(self.sd, torch.from_numpy(x[None]))
                self.table[key] = (p[0].numpy().astype(np.float32), np.float32(v[0]))
            ps.append(self.table[key][0])
            vs.append(self.table[key][1])
        return torch.from_numpy(np.stack(ps)), torch.from_numpy(np.array(vs, np.float32))


def run_reference_float(board, sims, wave, cap):
    from mcts.core.mcts import MCTS
    from mcts.core.mcts_config import MCTSConfig
    from mcts.gpu.gpu_game_states import GameType
    cfg = MCTSConfig(backend="gpu", device="cpu", wave_async_expansion=False,
                     dirichlet_epsilon=0.0, enable_subtree_reuse=False, max_wave_size=wave,
                     c_puct=1.4, virtual_loss=1.0, num_simulations=sims, max_tree_nodes=cap,
                     initial_tree_nodes=cap, game_type=GameType.GOMOKU, board_size=15)
    ev = RecordingFloatEvaluator()
    m = MCTS(cfg, ev)
    policy = np.asarray(m.search(board.copy()), np.float64)
    tree, nd = m.tree, m.tree.node_data
    n = int(tree.num_nodes)
    arr = dict(
        visits=nd.visit_counts[:n].numpy().astype(np.int32),
        value_sums=nd.value_sums[:n].numpy().astype(np.float32),
        priors=nd.node_priors[:n].numpy().astype(np.float32),
        virtual_loss=nd.virtual_loss_counts[:n].numpy().astype(np.int32),
        parent=nd.parent_indices[:n].numpy().astype(np.int32),
        action=nd.parent_actions[:n].numpy().astype(np.int32),
        children=tree.children[:n].numpy().astype(np.int32),
    )
    return policy, arr, ev


def run_reference(board, sims, wave, c_puct, vl, enable_vl, cap):
    from mcts.core.mcts import MCTS
    from mcts.core.mcts_config import MCTSConfig
    from mcts.gpu.gpu_game_states import GameType
    cfg = MCTSConfig(backend="gpu", device="cpu", wave_async_expansion=False,
                     dirichlet_epsilon=0.0, enable_subtree_reuse=False, max_wave_size=wave,
                     c_puct=c_puct, virtual_loss=vl, enable_virtual_loss=enable_vl,
                     num_simulations=sims, max_tree_nodes=cap, initial_tree_nodes=cap,
                     game_type=GameType.GOMOKU, board_size=15)
    ev = TracingSynthEvaluator()
    m = MCTS(cfg, ev)
    t0 = time.time()
    policy = m.search(board.copy())
    dt = time.time() - t0
    tree = m.tree
    n = int(tree.num_nodes)
    nd = tree.node_data
    out = dict(
        visits=nd.visit_counts[:n].numpy().astype(np.int32),
        value_sums=nd.value_sums[:n].numpy().astype(np.float32),
        priors=nd.node_priors[:n].numpy().astype(np.float32),
        virtual_loss=nd.virtual_loss_counts[:n].numpy().astype(np.int32),
        parent=nd.parent_indices[:n].numpy().astype(np.int32),
        action=nd.parent_actions[:n].numpy().astype(np.int32),
        children=tree.children[:n].numpy().astype(np.int32),
    )
    return np.asarray(policy, np.float64), out, ev, dt


def reuse_cases():
    from omoknuni_quantum_b200.roots import random_root
    return [
        # name, board, sims, wave, min_visits (subtree_reuse_min_visits)
        ("seed10", random_root(10), 256, 64, 10),
        ("seed11_w32", random_root(11), 320, 32, 10),
        ("empty", np.zeros((15, 15), np.int8), 192, 64, 10),
        ("reset_seed12", random_root(12), 128, 64, 1000000),
    ]


def run_reference_reuse(board, sims, wave, min_visits, cap=200000):
    """search(board) -> update_root(argmax, new board) -> search(new board), subtree reuse on
    (tree_operations.py:53-152, csr_tree.py:1020-1229, mcts.py:1205-1260). In the reference this
    path ends in a full reset: shift_root returns a tensor, `if mapping and len(mapping) == 1`
    (tree_operations.py:120) raises, and _try_optimized_subtree_reuse falls back to
    _efficient_tree_reset (mcts.py:1250-1260). The fixtures record that observable behaviour."""
    from mcts.core.mcts import MCTS
    from mcts.core.mcts_config import MCTSConfig
    from mcts.gpu.gpu_game_states import GameType
    cfg = MCTSConfig(backend="gpu", device="cpu", wave_async_expansion=False,
                     dirichlet_epsilon=0.0, enable_subtree_reuse=True, max_wave_size=wave,
                     c_puct=1.4, virtual_loss=1.0, num_simulations=sims, max_tree_nodes=cap,
                     initial_tree_nodes=cap, game_type=GameType.GOMOKU, board_size=15,
                     subtree_reuse_min_visits=min_visits)
    ev = TracingSynthEvaluator()
    m = MCTS(cfg, ev)
    pol1 = np.asarray(m.search(board.copy()), np.float64)
    action = int(np.argmax(pol1))
    child_visits = int(m.tree.node_data.visit_counts[m.tree.children[0, action]].item())
    b2 = board.copy()
    b2.reshape(-1)[action] = 1 if int((board != 0).sum()) % 2 == 0 else 2
    m.update_root(action, b2)
    kept = int(m.tree.num_nodes)
    pol2 = np.asarray(m.search(b2.copy()), np.float64)
    tree, nd = m.tree, m.tree.node_data
    n = int(tree.num_nodes)
    arr = dict(
        visits=nd.visit_counts[:n].numpy().astype(np.int32),
        value_sums=nd.value_sums[:n].numpy().astype(np.float32),
        priors=nd.node_priors[:n].numpy().astype(np.float32),
        virtual_loss=nd.virtual_loss_counts[:n].numpy().astype(np.int32),
        parent=nd.parent_indices[:n].numpy().astype(np.int32),
        action=nd.parent_actions[:n].numpy().astype(np.int32),
        children=tree.children[:n].numpy().astype(np.int32),
    )
    return pol1, action, child_visits, kept, b2, pol2, arr, ev


def gpu_reuse_cases():
    from omoknuni_quantum_b200.roots import random_root
    return [
        # name, board, sims, wave, searches
        ("seed20", random_root(20), 256, 64, 3),
        ("seed21_w32", random_root(21), 400, 32, 3),
        ("empty", np.zeros((15, 15), np.int8), 512, 128, 3),
        ("seed22", random_root(22), 192, 64, 4),
        ("seed23_w16", random_root(23), 160, 16, 3),
    ]


def run_reference_gpu_reuse(board, sims, wave, searches, cap=200000):
    """The reference's `use_gpu_tree_reuse=True` path: search -> update_root(arg-max, new board)
    -> search ..., which goes through _gpu_friendly_tree_reuse (mcts.py:1929-2005):
    extract_subtree_gpu_optimized + rebuild_tree_from_compact (compact_subtree.py:195-313). The
    rebuild writes visit counts and value sums of the kept nodes but leaves the children table
    and the node counter reset, so the next search re-expands the root and allocates its nodes
    from id 1 again: what stays is node 0's visit count and value sum, those of the chosen child.
    The new root's game-state slot comes from a LazyStateManager (index capacity - 1) that the
    state pool does not know about; when the pool hands that slot to another node during a search
    (recorded as `aliased`), the root's state is overwritten mid-search and evaluations below it
    change. Each search's policy, tree digests and root statistics are recorded."""
    from mcts.core.mcts import MCTS
    from mcts.core.mcts_config import MCTSConfig
    from mcts.gpu.gpu_game_states import GameType
    cfg = MCTSConfig(backend="gpu", device="cpu", wave_async_expansion=False,
                     dirichlet_epsilon=0.0, enable_subtree_reuse=True, use_gpu_tree_reuse=True,
                     max_wave_size=wave, c_puct=1.4, virtual_loss=1.0, num_simulations=sims,
                     max_tree_nodes=cap, initial_tree_nodes=cap, game_type=GameType.GOMOKU,
                     board_size=15)
    m = MCTS(cfg, TracingSynthEvaluator())
    b = board.copy()
    out = []
    for i in range(searches):
        pol = np.asarray(m.search(b.copy()), np.float64)
        tree, nd = m.tree, m.tree.node_data
        n = int(tree.num_nodes)
        nts = m.node_to_state[:n].numpy()
        aliased = int(nts[0] >= 0 and bool((nts[1:] == nts[0]).any()))
        rec = dict(board=b.astype(np.int8).copy(), policy=pol, num_nodes=n, aliased=aliased,
                   root_n=int(nd.visit_counts[0]), root_w=np.float32(nd.value_sums[0]))
        for k, arr in (("visits", nd.visit_counts), ("value_sums", nd.value_sums),
                       ("priors", nd.node_priors), ("parent", nd.parent_indices),
                       ("action", nd.parent_actions)):
            rec["sha_" + k] = digest(arr[:n].numpy().astype(np.float32 if k in ("value_sums", "priors") else np.int32))
        action = int(np.argmax(pol))
        rec["action"] = action
        child = int(tree.children[0, action])
        rec["child_n"], rec["child_w"] = int(nd.visit_counts[child]), np.float32(nd.value_sums[child])
        out.append(rec)
        if i + 1 < searches:
            b2 = b.copy()
            b2.reshape(-1)[action] = 1 if int((b != 0).sum()) % 2 == 0 else 2
            m.update_root(action, b2)
            assert m.stats["tree_reuse_count"] == i + 1, "the reference's GPU reuse path did not run"
            b = b2
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("OMQ_REFERENCE"), required="OMQ_REFERENCE" not in os.environ)
    ap.add_argument("--only", nargs="*")
    args = ap.parse_args()
    sys.dont_write_bytecode = True
    sys.path.insert(0, REPO)
    sys.path.insert(0, os.path.join(REPO, "oracle", "_ref"))
    sys.path.insert(0, os.path.join(args.reference, "python"))
    import logging
    logging.disable(logging.WARNING)
    import torch
    torch.set_num_threads(os.cpu_count() or 1)

    for name, board, sims, wave, cap in float_cases():
        if args.only and name not in args.only:
            continue
        policy, arr, ev = run_reference_float(board, sims, wave, cap)
        n = arr["visits"].shape[0]
        keys = sorted(ev.table)
        # legal-prior counts of the expanded nodes: which summation paths the case exercises
        kids = np.bincount(arr["parent"][1:], minlength=n)
        rec = dict(board=board.astype(np.int8), sims=sims, wave=wave, capacity=cap, num_nodes=n,
                   policy=policy, final_move=int(np.argmax(policy)),
                   table_keys=np.array(keys), table_policy=np.stack([ev.table[k][0] for k in keys]),
                   table_value=np.array([ev.table[k][1] for k in keys], np.float32),
                   expanded_child_counts=kids[kids > 0].astype(np.int32),
                   torch_cpu_capability=str(__import__("torch").backends.cpu.get_cpu_capability()))
        for k in ("visits", "value_sums", "priors", "virtual_loss", "parent", "action", "children"):
            rec["sha_" + k] = digest(arr[k])
        if n <= FULL_ARRAYS_MAX_NODES:
            for k in ("visits", "value_sums", "priors", "parent", "action"):
                rec["full_" + k] = arr[k]
        path = os.path.join(HERE, f"floatsearch_{name}.npz")
        np.savez_compressed(path, **rec)
        print(f"float {name}: nodes={n} positions={len(keys)} move={rec['final_move']} "
              f"child counts {sorted(set(rec['expanded_child_counts'].tolist()))[:6]}... "
              f"-> {os.path.basename(path)} ({os.path.getsize(path)} B)")

    for name, board, sims, wave, searches in gpu_reuse_cases():
        if args.only and name not in args.only:
            continue
        recs = run_reference_gpu_reuse(board, sims, wave, searches)
        flat = dict(sims=sims, wave=wave, searches=searches)
        for i, r in enumerate(recs):
            for k, x in r.items():
                flat[f"s{i}_{k}"] = x
        path = os.path.join(HERE, f"gpureuse_{name}.npz")
        np.savez_compressed(path, **flat)
        print(f"gpureuse {name}: " + ", ".join(f"root N {r['root_n']} nodes {r['num_nodes']} "
                                               f"aliased {r['aliased']}" for r in recs))

    for name, board, sims, wave, minv in reuse_cases():
        if args.only and name not in args.only:
            continue
        pol1, action, child_visits, kept, b2, pol2, arr, ev = run_reference_reuse(board, sims, wave, minv)
        n = arr["visits"].shape[0]
        rec = dict(board=board.astype(np.int8), sims=sims, wave=wave, min_visits=minv,
                   policy1=pol1, action=action, child_visits=child_visits, kept=kept,
                   board2=b2.astype(np.int8), policy2=pol2, num_nodes=n,
                   eval_calls=ev.calls, eval_positions=ev.positions, eval_trace=ev.trace_digest())
        for k in ("visits", "value_sums", "priors", "virtual_loss", "parent", "action", "children"):
            rec["sha_" + k] = digest(arr[k])
        path = os.path.join(HERE, f"reuse_{name}.npz")  # reuse_<case>.npz
        np.savez_compressed(path, **rec)
        print(f"{name}: action={action} child_visits={child_visits} kept={kept} nodes={n} "
              f"evals={ev.calls}/{ev.positions} -> {os.path.basename(path)}")

    for name, board, sims, wave, c, vl, evl, cap in cases():
        if args.only and name not in args.only:
            continue
        policy, arr, ev, dt = run_reference(board, sims, wave, c, vl, evl, cap)
        n = arr["visits"].shape[0]
        # the dense children table must be the one implied by (parent, action)
        ch = np.full_like(arr["children"], -1)
        ch[arr["parent"][1:], arr["action"][1:]] = np.arange(1, n, dtype=np.int32)
        assert np.array_equal(ch, arr["children"]), name
        root_kids = np.nonzero(arr["parent"] == 0)[0]
        rec = dict(
            board=board.astype(np.int8), sims=sims, wave=wave, c_puct=np.float32(c),
            virtual_loss=np.float32(vl), enable_vl=int(evl), capacity=cap,
            num_nodes=n, policy=policy, final_move=int(np.argmax(policy)),
            root_visits=arr["visits"][0], root_value_sum=arr["value_sums"][0],
            root_children=root_kids.astype(np.int32),
            root_children_visits=arr["visits"][root_kids],
            root_children_value_sums=arr["value_sums"][root_kids],
            eval_calls=ev.calls, eval_positions=ev.positions, eval_trace=ev.trace_digest(),
            reference_seconds=dt,
        )
        for k in ("visits", "value_sums", "priors", "virtual_loss", "parent", "action", "children"):
            rec["sha_" + k] = digest(arr[k])
        if n <= FULL_ARRAYS_MAX_NODES:
            for k in ("visits", "value_sums", "priors", "virtual_loss", "parent", "action"):
                rec["full_" + k] = arr[k]
        path = os.path.join(HERE, f"search_{name}.npz")
        np.savez_compressed(path, **rec)
        print(f"{name}: nodes={n} move={rec['final_move']} evals={ev.calls}/{ev.positions} "
              f"{dt:.1f}s -> {os.path.basename(path)} ({os.path.getsize(path)} B)")


if __name__ == "__main__":
    main()
