"""Subtree reuse between searches (omq_reroot): the kept tree is the breadth-first relabelling of
the chosen child's subtree (CSRTree.shift_root, csr_tree.py:1020-1229), and search -> update_root
-> search chains on the device equal the oracle's, for Gomoku, Go (superko keys carried into the
new root) and chess; the carry mode follows the reference's use_gpu_tree_reuse path (reference
fixtures in test_reuse.py)."""
import numpy as np
import pytest
import torch



def _bfs(parent, root):
    """Old ids of root's subtree in breadth-first order, children in id (= action) order."""
    kids = {}
    for i, p in enumerate(parent):
        if p >= 0:
            kids.setdefault(int(p), []).append(i)
    order = [root]
    for o in order:
        order.extend(kids.get(o, []))
    return np.array(order)


def _play(board, action):
    b = board.copy()
    b.reshape(-1)[action] = 1 if int((board != 0).sum()) % 2 == 0 else 2
    return b


def test_oracle_keep_reroot_is_breadth_first_subtree(oracle_lib):
    from omoknuni_quantum_b200.roots import random_root
    board = random_root(31)
    o = oracle_lib.Oracle(200000)
    t = o.search(board, 400, 64)
    a = int(np.argmax(t.policy))
    c = int(np.nonzero((t.parent == 0) & (t.action == a))[0][0])
    order = _bfs(t.parent, c)
    assert o.reroot(a, keep=True) == 2
    k = o.export()
    assert k.visits.shape[0] == len(order) > 1
    for f in ("visits", "value_sums", "priors", "virtual_loss", "terminal"):
        assert np.array_equal(getattr(k, f), getattr(t, f)[order]), f
    assert k.action[0] == -1 and np.array_equal(k.action[1:], t.action[order][1:])
    new_of = {int(old): i for i, old in enumerate(order)}
    assert k.parent[0] == -1
    assert all(k.parent[i] == new_of[int(t.parent[order[i]])] for i in range(1, len(order)))
    # the next search continues on the kept tree: the root keeps its visits
    t2 = o.search(_play(board, a), 256, 64)
    assert int(t2.visits[0]) == int(t.visits[c]) + 256
    assert t2.visits.shape[0] >= len(order)


def test_oracle_reroot_fallbacks(oracle_lib):
    from omoknuni_quantum_b200.roots import random_root
    board = random_root(32)
    o = oracle_lib.Oracle(100000)
    t = o.search(board, 64, 64)
    unexplored = [a for a in range(225) if board.reshape(-1)[a] == 0 and
                  not ((t.parent == 0) & (t.action == a)).any()]
    if unexplored:                      # not a root child: fresh tree
        assert o.reroot(unexplored[0], keep=True) == 0
    leaf = [int(t.action[i]) for i in np.nonzero(t.parent == 0)[0] if not (t.parent == i).any()]
    assert leaf
    assert o.reroot(leaf[0], keep=True) == 1          # a leaf child: its statistics only
    t2 = o.search(_play(board, leaf[0]), 64, 64)
    c = int(np.nonzero((t.parent == 0) & (t.action == leaf[0]))[0][0])
    assert int(t2.visits[0]) == int(t.visits[c]) + 64
    assert o.reroot(-1) == 0


# --- device == oracle ---------------------------------------------------------------------------

def _compare(t, o):
    assert t["visits"].shape == o.visits.shape
    for k in ("parent", "action", "priors", "visits", "value_sums", "terminal"):
        assert np.array_equal(t[k], getattr(o, k)), k


@pytest.mark.gpu
@pytest.mark.parametrize("keep", [True, False])
def test_gomoku_reroot_chain_matches_oracle(oracle_lib, keep):
    """Three trees, four searches each, a different move kept per tree (arg-max, then the
    second-best child, then a leaf child, then a move that is not in the tree)."""
    from omoknuni_quantum_b200.engine import WaveEngine
    from omoknuni_quantum_b200.roots import random_root
    boards = [random_root(40 + r) for r in range(3)]
    eng = WaveEngine(3, capacity=150000, max_wave_size=64)
    orc = [oracle_lib.Oracle(150000) for _ in range(3)]
    for step in range(4):
        eng.search(torch.from_numpy(np.stack(boards)).cuda(), 320)
        acts = []
        for r in range(3):
            o = orc[r].search(boards[r], 320, 64)
            t = eng.export_tree(r)
            _compare(t, o)
            kids = np.nonzero(t["parent"] == 0)[0]
            by_n = kids[np.argsort(-t["visits"][kids], kind="stable")]
            if step == 0:
                a = int(t["action"][by_n[0]])
            elif step == 1:
                a = int(t["action"][by_n[min(1, len(by_n) - 1)]])
            elif step == 2:
                leaves = [i for i in kids if not (t["parent"] == i).any()]
                a = int(t["action"][leaves[0] if leaves else by_n[0]])
            else:
                free = [x for x in np.flatnonzero(boards[r].reshape(-1) == 0)
                        if x not in set(t["action"][kids].tolist())]
                a = int(free[0]) if free else int(t["action"][by_n[0]])
            acts.append(a)
            orc[r].reroot(a, keep=keep)
            boards[r] = _play(boards[r], a)
        eng.reroot(np.array(acts, np.int32), keep=keep)
        for r in range(3):              # the kept trees themselves, before the next search
            _compare(eng.export_tree(r), orc[r].export())


@pytest.mark.gpu
def test_go_keep_chain_matches_oracle(oracle_lib):
    """Go 9x9 with positional superko: the new root's game keys include the move just played;
    kept nodes' legality was decided with the same set of earlier positions."""
    from omoknuni_quantum_b200.engine import WaveEngine
    from omoknuni_quantum_b200.go import random_position
    n = 9
    pos = [random_position(60 + r, moves=24, board_size=n) for r in range(2)]
    eng = WaveEngine(2, board_size=n, capacity=120000, max_wave_size=64, game="go")
    orc = [oracle_lib.Oracle(120000, n) for _ in range(2)]
    for step in range(3):
        hist = np.stack([p.history_planes() for p in pos])
        meta = np.stack([p.meta() for p in pos])
        eng.search(torch.from_numpy(hist).cuda(), 384, meta=torch.from_numpy(meta),
                   keys=[p.root_keys() for p in pos])
        acts = []
        for r, p in enumerate(pos):
            o = orc[r].search_go(p.history_planes(), p.to_move, 384, 64, ko=p.ko, passes=p.passes,
                                 keys=p.root_keys())
            t = eng.export_tree(r)
            _compare(t, o)
            a = int(np.argmax(o.policy))
            acts.append(a)
            assert orc[r].reroot(a, keep=True) == 2
            p.play(a)
        eng.reroot(np.array(acts, np.int32), keep=True)


@pytest.mark.gpu
def test_chess_keep_chain_matches_oracle(oracle_lib):
    from omoknuni_quantum_b200.chess import random_position
    from omoknuni_quantum_b200.engine import WaveEngine
    pos = [random_position(70 + r) for r in range(2)]
    eng = WaveEngine(2, board_size=8, capacity=120000, max_wave_size=48, game="chess")
    orc = [oracle_lib.Oracle(120000, 8) for _ in range(2)]
    for step in range(3):
        rec = np.stack([p.root_records() for p in pos])
        eng.search(rec, 288, meta=np.array([len(p.prior) for p in pos], np.int32))
        acts = []
        for r, p in enumerate(pos):
            o = orc[r].search_chess(p.record(), 288, 48, prior=p.prior)
            t = eng.export_tree(r)
            _compare(t, o)
            a = int(np.argmax(o.policy))
            acts.append(a)
            assert orc[r].reroot(a, keep=True) == 2
            p.play(p.action_to_move(a))
        eng.reroot(np.array(acts, np.int32), keep=True)


@pytest.mark.gpu
def test_dropin_keep_subtree_and_carry(oracle_lib):
    """MCTS.update_root with keep_subtree=True / use_gpu_tree_reuse=True against the oracle, and a
    search on another engine in between dropping the pending reroot."""
    from omoknuni_quantum_b200 import MCTS, MCTSConfig, SyntheticEvaluator
    from omoknuni_quantum_b200.roots import random_root
    for kw, keep in (({"keep_subtree": True}, True), ({"use_gpu_tree_reuse": True}, False)):
        cfg = MCTSConfig(num_simulations=256, max_wave_size=64, c_puct=1.4, dirichlet_epsilon=0.0,
                         enable_subtree_reuse=True, initial_tree_nodes=100000, **kw)
        m = MCTS(cfg, SyntheticEvaluator())
        o = oracle_lib.Oracle(100000)
        b = random_root(50)
        for step in range(3):
            p = m.search(b)
            t = o.search(b, 256, 64)
            assert np.array_equal(p, t.policy), (kw, step)
            a = int(np.argmax(p))
            m.update_root(a, _play(b, a))
            o.reroot(a, keep=keep)
            b = _play(b, a)
        m.search_batch(np.stack([b, b]))          # another engine: the pending reroot is dropped
        p = m.search(b)
        assert np.array_equal(p, oracle_lib.Oracle(100000).search(b, 256, 64).policy)


@pytest.mark.gpu
@pytest.mark.parametrize("mode", ["keep", "carry"])
def test_selfplay_with_subtree_reuse_matches_oracle(oracle_lib, mode):
    """Batched self-play with reuse: every move's policy equals the oracle's search of that game
    continued on its rerooted tree (fresh again whenever the set of live games changed)."""
    from omoknuni_quantum_b200.selfplay import BatchedSelfPlay
    sp = BatchedSelfPlay(3, num_simulations=128, wave_size=32, capacity=60000, seed=5,
                         subtree_reuse=mode)
    recs = sp.play(4)
    for r in recs:
        o = oracle_lib.Oracle(60000)
        for i, ex in enumerate(r.examples):
            t = o.search(ex["state"], 128, 32)
            assert np.array_equal(ex["policy"], t.policy), (r.game_id, i)
            o.reroot(r.moves[i], keep=mode == "keep")
    assert all(not r.finished for r in recs)      # the live set stayed the same: reuse every move


def _check_bfs(t, k, c):
    order = _bfs(t.parent, c)
    assert k.visits.shape[0] == len(order)
    for f in ("visits", "value_sums", "priors", "virtual_loss", "terminal"):
        assert np.array_equal(getattr(k, f), getattr(t, f)[order]), f
    new_of = {int(old): i for i, old in enumerate(order)}
    assert all(k.parent[i] == new_of[int(t.parent[order[i]])] for i in range(1, len(order)))


def test_oracle_keep_reroot_go_and_chess(oracle_lib):
    """The keep relabelling for Go (superko keys move with the nodes) and chess (position records
    move with the nodes); a search continued on the kept tree keeps the root's visits."""
    from omoknuni_quantum_b200.chess import random_position as chess_position
    from omoknuni_quantum_b200.go import random_position as go_position
    p = go_position(61, moves=24, board_size=9)
    o = oracle_lib.Oracle(100000, 9)
    t = o.search_go(p.history_planes(), p.to_move, 384, 64, ko=p.ko, passes=p.passes, keys=p.root_keys())
    a = int(np.argmax(t.policy))
    c = int(np.nonzero((t.parent == 0) & (t.action == a))[0][0])
    assert o.reroot(a, keep=True) == 2
    _check_bfs(t, o.export(), c)
    p.play(a)
    t2 = o.search_go(p.history_planes(), p.to_move, 128, 64, ko=p.ko, passes=p.passes, keys=p.root_keys())
    assert int(t2.visits[0]) == int(t.visits[c]) + 128

    q = chess_position(71)
    o = oracle_lib.Oracle(100000, 8)
    t = o.search_chess(q.record(), 288, 48, prior=q.prior)
    a = int(np.argmax(t.policy))
    c = int(np.nonzero((t.parent == 0) & (t.action == a))[0][0])
    assert o.reroot(a, keep=True) == 2
    _check_bfs(t, o.export(), c)
    q.play(q.action_to_move(a))
    t2 = o.search_chess(q.record(), 96, 48, prior=q.prior)
    assert int(t2.visits[0]) == int(t.visits[c]) + 96
