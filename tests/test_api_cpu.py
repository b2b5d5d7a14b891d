"""Host-side API of the drop-in (no GPU needed): MCTSConfig compatibility with the reference's
field names and defaults, MCTS method semantics that do not touch the device, and the
no-fallback rule (the search itself fails loudly without CUDA)."""
import numpy as np
import pytest
import torch


def test_config_defaults_follow_reference():
    from omoknuni_quantum_b200.mcts_config import GameType, MCTSConfig
    c = MCTSConfig()
    # python/mcts/core/mcts_config.py:33-39, 53, 64, 68-69, 72-73, 79-80, 84-87, 155
    assert (c.num_simulations, c.c_puct, c.max_depth, c.max_wave_size) == (10000, 1.414, 100, 1024)
    assert (c.dirichlet_alpha, c.dirichlet_epsilon, c.virtual_loss) == (0.3, 0.25, 1.0)
    assert c.enable_virtual_loss and c.enable_subtree_reuse and c.wave_async_expansion
    assert (c.max_tree_nodes, c.initial_tree_nodes, c.tree_capacity) == (2000000, 100000, 100000)
    assert c.game_type == GameType.GOMOKU and c.board_size == 15
    assert c.use_cuda_graphs and c.block_size == 128 and c.batch_size == 256  # passthrough fields


def test_config_accepts_reference_kwargs_and_rejects_unknown():
    from omoknuni_quantum_b200.mcts_config import MCTSConfig
    c = MCTSConfig(backend="gpu", device="cpu", wave_async_expansion=False, dirichlet_epsilon=0.0,
                   enable_subtree_reuse=False, max_wave_size=256, c_puct=1.4, num_simulations=800,
                   enable_kernel_fusion=False, tree_reuse_validation_level="full", game_type="gomoku")
    assert c.enable_kernel_fusion is False and c.tree_reuse_validation_level == "full"
    assert c.to_dict()["max_wave_size"] == 256
    with pytest.raises(TypeError):
        MCTSConfig(not_a_field=1)
    with pytest.raises(ValueError):
        MCTSConfig(backend="tpu")
    assert MCTSConfig(enable_dynamic_allocation=False).tree_capacity == 2000000


def test_mcts_host_methods_and_no_cpu_fallback():
    from omoknuni_quantum_b200 import MCTS, MCTSConfig, SyntheticEvaluator
    m = MCTS(MCTSConfig(num_simulations=8, max_wave_size=4), SyntheticEvaluator())
    pol = np.zeros(225)
    pol[17] = 0.7
    pol[3] = 0.3
    assert m.select_action(None, temperature=0, policy=pol) == 17
    np.random.seed(0)
    assert m.select_action(None, temperature=1.0, policy=pol) in (3, 17)
    with pytest.raises(ValueError):
        m.update_root(225)
    m.update_root(5, np.zeros((15, 15), np.int8))
    assert m.get_root_value() == 0.0
    with pytest.raises(ValueError):
        m.search(np.zeros((9, 9), np.int8))
    # a zero-simulation config returns the uniform policy (mcts.py:1023-1031)
    m0 = MCTS(MCTSConfig(num_simulations=0), SyntheticEvaluator())
    assert np.allclose(m0.search(np.zeros((15, 15), np.int8)), 1 / 225)
    if not torch.cuda.is_available():
        with pytest.raises(RuntimeError, match="CUDA"):
            m.search(np.zeros((15, 15), np.int8))


def test_policy_from_visits():
    from omoknuni_quantum_b200.engine import WaveEngine
    v = np.zeros((2, 225), np.int32)
    v[0, [4, 9]] = [3, 1]
    p = WaveEngine.policy_from_visits(v)
    assert p.dtype == np.float64 and p[0, 4] == 0.75 and p[0, 9] == 0.25
    assert np.allclose(p[1], 1 / 225)


def test_roots_are_seeded_and_five_free():
    from omoknuni_quantum_b200.roots import has_five, random_root, random_roots
    a, b = random_root(3), random_root(3)
    assert np.array_equal(a, b) and (a == 1).sum() == 10 and (a == 2).sum() == 10
    rs = random_roots(1, 50)
    assert not any(has_five(r) for r in rs)
    five = np.zeros((15, 15), np.int8)
    five[2, 4:9] = 2
    assert has_five(five) and has_five(five.T) and has_five(np.eye(15, dtype=np.int8))
    assert has_five(np.fliplr(np.eye(15, dtype=np.int8)))


def test_mcts_go_roots_from_positions_and_move_histories():
    """MCTS(GameType.GO): 362 actions; a reference-style state (IGameState.get_move_history, pass
    = -1) is rebuilt into the same root record as the package's GoPosition; chess is refused."""
    import numpy as np
    import pytest
    from omoknuni_quantum_b200.go import GoPosition, random_position
    from omoknuni_quantum_b200.mcts import MCTS
    from omoknuni_quantum_b200.mcts_config import GameType, MCTSConfig
    m = MCTS(MCTSConfig(game_type=GameType.GO, board_size=9), "synthetic")
    assert m.action_size == 82
    g = random_position(4, moves=20, board_size=9)
    g.play(g.pass_action)
    moves = []
    replay = GoPosition(9)
    # reconstruct the move list from the position's history is not possible in general; record it
    rng = np.random.default_rng(4)
    for _ in range(20):
        cand = np.flatnonzero(replay.legal_mask()[:-1])
        a = int(cand[rng.integers(len(cand))])
        replay.play(a)
        moves.append(a)
    replay.play(replay.pass_action)
    moves.append(-1)

    class FakeGoState:
        def get_move_history(self):
            return list(moves)

    h1, m1, k1 = m._go_root(FakeGoState())
    h2, m2, k2 = m._go_root(g)
    assert np.array_equal(h1, h2) and np.array_equal(m1, m2)
    assert np.array_equal(k1, k2) and len(k1) == 20      # one superko key per non-pass move
    assert m1[2] == 1                                     # one pass made


def test_mcts_chess_roots_from_positions_fens_and_move_histories():
    import numpy as np
    from omoknuni_quantum_b200.chess import ChessPosition, random_position
    from omoknuni_quantum_b200.mcts import MCTS
    from omoknuni_quantum_b200.mcts_config import GameType, MCTSConfig
    m = MCTS(MCTSConfig(game_type=GameType.CHESS), "synthetic")
    assert m.action_size == 4672
    rng = np.random.default_rng(1)
    p, moves = ChessPosition(), []
    for _ in range(12):
        ms = p.legal_moves()
        a = ms[int(rng.integers(len(ms)))]
        p.play(a)
        moves.append(a)

    class FakeChessState:
        def get_move_history(self):
            return list(moves)

    r1, n1 = m._chess_root(FakeChessState())
    r2, n2 = m._chess_root(p)
    assert np.array_equal(r1, r2) and n1 == n2 == 12
    r3, n3 = m._chess_root(p.fen())
    assert np.array_equal(r3[0], r2[0]) and n3 == 0      # a FEN carries no earlier positions
    assert random_position(3).record()["side"] in (1, 2)


def test_reference_method_surface():
    """Every public method of the reference MCTS class (python/mcts/core/mcts.py) exists here."""
    from omoknuni_quantum_b200 import MCTS
    for name in ("search", "search_batch", "select_action", "update_root", "update_with_move",
                 "get_root_value", "get_statistics", "clear", "reset_tree", "warmup", "shutdown"):
        assert callable(getattr(MCTS, name, None)), name


def test_gomoku_state_objects_are_replayed():
    from omoknuni_quantum_b200 import MCTS, MCTSConfig, SyntheticEvaluator

    class State:                      # the IGameState surface the drop-in uses
        def get_move_history(self):
            return [112, 113, 97]

    m = MCTS(MCTSConfig(num_simulations=8), SyntheticEvaluator())
    b = m._boards(State())
    assert b.reshape(-1)[112] == 1 and b.reshape(-1)[113] == 2 and b.reshape(-1)[97] == 1
    assert int((b != 0).sum()) == 3


def test_config_presets():
    from omoknuni_quantum_b200 import create_optimized_config, create_performance_config
    c = create_performance_config(num_simulations=64)
    assert c.wave_size == 3072 and c.memory_pool_size_mb == 2048 and c.use_cuda_graphs
    assert c.num_simulations == 64
    o = create_optimized_config(num_simulations=128)
    assert o.num_simulations == 128 and o.device == "cuda"


def test_reference_models_and_evaluators_become_the_device_resnet(monkeypatch):
    """A reference ResNetModel, or a reference ResNetEvaluator holding one as ``model``, is run by
    the tensor-core ResNet with its state_dict; the board size comes from the MCTS config, and an
    evaluator under the reference's fp16 autocast (use_amp) keeps fp16."""
    from omoknuni_quantum_b200 import mcts, resnet

    made = []

    class Stub:
        def __init__(self, sd, board_size, dtype):
            made.append((sd, board_size, dtype))

    monkeypatch.setattr(resnet, "ResNetEvaluator", Stub)

    class Model:                           # the attributes of the reference ResNetModel used here
        residual_blocks = []

        def state_dict(self):
            return {"w": 1}

    class RefEvaluator:
        def __init__(self, use_amp=False):
            self.model = Model()
            self.use_amp = use_amp

        def evaluate_batch(self, x):
            raise AssertionError("the reference evaluator itself must not be called")

    assert isinstance(mcts._resolve_evaluator(Model(), 19), Stub)
    assert isinstance(mcts._resolve_evaluator(RefEvaluator(), 8), Stub)
    assert isinstance(mcts._resolve_evaluator(RefEvaluator(use_amp=True), 15), Stub)
    assert made == [({"w": 1}, 19, "bf16"), ({"w": 1}, 8, "bf16"), ({"w": 1}, 15, "fp16")]
    other = object()
    assert mcts._resolve_evaluator(other) is other
    assert mcts._resolve_evaluator("synthetic") == "synthetic"
