"""MCTS - drop-in for the reference's ``MCTS(config, evaluator, game_interface).search()``.

Same constructor, methods and return types as python/mcts/core/mcts.py (``search`` 924,
``select_action`` 1167, ``update_root`` 1205, ``get_root_value`` 1139, ``clear`` 1387,
``get_statistics`` 1429), with the whole search on the device: one ``WaveEngine`` holds the
tree(s), every wave runs as select -> evaluate leaf queue -> expand + pick -> evaluate final
queue -> backup without a host round trip (except for host-protocol evaluators, which receive the
queue's feature tensor).

Results equal the reference's deterministic CPU path (``backend='gpu', device='cpu',
wave_async_expansion=False``) for the same evaluator outputs: visit counts, tree layout and the
root policy bit for bit.

Evaluators:
  * ``SyntheticEvaluator()`` - built-in integer-exact synthetic evaluator (device kernel);
  * ``ResNetEvaluator`` of this package - tcgen05 bf16 ResNet reading the leaf queue in place;
  * a ``torch.nn.Module`` with the reference ResNetModel layout (e.g. ``single_gpu_mode=True``
    with a model, mcts.py:113-122) - its weights are folded and packed into a ResNetEvaluator;
  * any object with the reference protocol ``evaluate_batch(features) -> (policy, value)``.
"""
from __future__ import annotations

import time
from typing import Any, Dict, Optional

import numpy as np
import torch

from .engine import WaveEngine
from .mcts_config import GameType, MCTSConfig


class SyntheticEvaluator:
    """Marker for the built-in device synthetic evaluator (policy ~ softmax of N(0,1) logits
    seeded by a 64-bit hash of the feature planes, masked to legal moves; value = tanh of a
    hash-seeded N(0, 0.5) draw; integer-exact, see eval_kernels.cu)."""

    builtin = "synthetic"

    def evaluate_batch(self, features):  # pragma: no cover - device-only
        raise NotImplementedError("SyntheticEvaluator runs inside the device engine")


def _resolve_evaluator(evaluator, board_size: int = 15):
    """The evaluator the engine runs. A reference ResNetModel - passed directly, or inside a
    reference ResNetEvaluator as its ``model`` (resnet_evaluator.py:80-265, possibly TorchScript-
    compiled) - becomes this package's tensor-core ResNetEvaluator with the same weights (fp16 when
    the reference evaluator runs under its fp16 autocast, `use_amp`, else bf16); the synthetic
    evaluator runs on the device; anything else is called through evaluate_batch."""
    if isinstance(evaluator, SyntheticEvaluator) or (isinstance(evaluator, str) and evaluator == "synthetic"):
        return "synthetic"
    module = evaluator if hasattr(evaluator, "residual_blocks") else getattr(evaluator, "model", None)
    if module is not None and hasattr(module, "residual_blocks") and hasattr(module, "state_dict"):
        from . import resnet
        dtype = "fp16" if getattr(evaluator, "use_amp", False) is True else "bf16"
        return resnet.ResNetEvaluator(module.state_dict(), board_size=getattr(module, "board_size", board_size),
                                      dtype=dtype)
    return evaluator


class MCTS:
    def __init__(self, config: MCTSConfig, evaluator: Any, game_interface: Any = None,
                 single_gpu_mode: bool = False):
        self.config = config
        self.game_interface = game_interface
        self.single_gpu_mode = single_gpu_mode
        self.is_go = config.game_type == GameType.GO
        self.is_chess = config.game_type == GameType.CHESS
        if self.is_chess and config.board_size != 8:
            config.board_size = 8
        self.evaluator = evaluator
        self._eval = _resolve_evaluator(evaluator, config.board_size)
        if hasattr(evaluator, "_return_torch_tensors"):
            evaluator._return_torch_tensors = True          # mcts.py:120-121
        dev = config.device if config.device != "cpu" else "cuda"
        self.device = torch.device(dev)   # device index resolved when the first engine is made
        self._engines: Dict[int, WaveEngine] = {}
        # root-noise generator seed, drawn from numpy's global RNG (the reference draws the noise
        # itself from torch's global RNG)
        self._noise_seed = int(np.random.randint(0, 2 ** 62))
        self._last_tree = None          # (engine, index) of the last single search
        self._pending = None            # engine holding a reroot for its next search
        self._root_state = None
        self.stats = dict(total_searches=0, total_simulations=0, total_time=0.0,
                          last_search_sims_per_second=0.0, peak_sims_per_second=0.0,
                          avg_sims_per_second=0.0)

    @property
    def _graphs_on(self) -> bool:
        """MCTSConfig.use_cuda_graphs (reference default True): full-size waves replay a captured
        CUDA graph when the evaluator runs on the device queue."""
        return bool(getattr(self.config, "use_cuda_graphs", True))

    # -- engines -------------------------------------------------------------------------------
    @property
    def action_size(self) -> int:
        if self.is_chess:
            return 4672
        return self.config.board_size ** 2 + (1 if self.is_go else 0)

    def _drop_pending(self, keep_engine=None) -> None:
        """A reroot applies only to the next search on the same engine; clear it otherwise."""
        p, self._pending = self._pending, None
        if p is not None and p is not keep_engine and p._h.value:
            p.reroot(np.full(p.num_trees, -1, np.int32))

    def _engine(self, num_trees: int, go_rules: str = "chinese") -> WaveEngine:
        eng = self._engines.get(num_trees)
        if eng is not None and self.is_go and getattr(eng, "go_rules", "chinese") != go_rules:
            if self._pending is eng:          # its tree goes with it
                self._pending = None
            eng.close()
            eng = None
        if eng is None:
            if not torch.cuda.is_available():
                raise RuntimeError("MCTS search needs a CUDA device (B200); there is no CPU fallback")
            if self.device.index is None:
                self.device = torch.device("cuda", torch.cuda.current_device())
            c = self.config
            eng = WaveEngine(num_trees, board_size=c.board_size, capacity=c.tree_capacity,
                             max_wave_size=c.max_wave_size, c_puct=c.c_puct,
                             virtual_loss=c.virtual_loss, enable_virtual_loss=c.enable_virtual_loss,
                             max_depth=c.max_depth, device=self.device,
                             dirichlet_alpha=c.dirichlet_alpha, dirichlet_epsilon=c.dirichlet_epsilon,
                             noise_seed=self._noise_seed,
                             game="go" if self.is_go else "chess" if self.is_chess else "gomoku",
                             go_rules=go_rules)
            eng.go_rules = go_rules
            self._engines[num_trees] = eng
        return eng

    def _boards(self, state) -> np.ndarray:
        n = self.config.board_size
        if torch.is_tensor(state):
            if state.shape[-2:] != (n, n):
                raise ValueError(f"Invalid state shape: {tuple(state.shape)}, expected {(n, n)}")
            return state
        
        if isinstance(state, np.ndarray):
            if state.shape[-2:] != (n, n):
                raise ValueError(f"Invalid state shape: {state.shape}, expected {(n, n)}")
            return state.astype(np.int8, copy=False)
        if hasattr(state, "get_move_history"):
            # a reference IGameState (mcts.py:1520-1580 rebuilds its board from the tensor
            # planes): replay its moves on the empty board, black first
            b = np.zeros((n, n), np.int8)
            for i, m in enumerate(state.get_move_history()):
                m = int(m)
                if not 0 <= m < n * n or b.reshape(-1)[m] != 0:
                    raise ValueError(f"move {m} of the state's history is not playable")
                b.reshape(-1)[m] = 1 if i % 2 == 0 else 2
            return b
        raise TypeError("state must be a numpy/torch board [n, n] with 0 empty, 1 black, 2 white, "
                        "or a game state with get_move_history()")

    def _go_root(self, state):
        """(history int8 [8, n, n], meta int32 [3], superko keys) of a Go root: a GoPosition of this package,
        an object with the reference IGameState interface (rebuilt by replaying
        get_move_history(), pass = -1, from the empty board), or a bare board (side to move by
        stone parity as mcts.py:1509-1519, no ko, no earlier positions)."""
        from .go import GoPosition
        n = self.config.board_size
        if isinstance(state, GoPosition):
            return state.history_planes(), state.meta(), state.root_keys()
        if hasattr(state, "get_move_history"):
            g = GoPosition(n)
            for m in state.get_move_history():
                g.play(g.pass_action if int(m) < 0 else int(m))
            return g.history_planes(), g.meta(), g.root_keys()
        b = self._boards(state)
        b = b.cpu().numpy() if torch.is_tensor(b) else np.asarray(b)
        h = np.zeros((8, n, n), np.int8)
        h[0] = b
        stones = int((b != 0).sum())
        return h, np.array([1 if stones % 2 == 0 else 2, -1, 0], np.int32), np.zeros(0, np.uint64)

    def _chess_root(self, state):
        """(records POS_DTYPE [101], earlier positions) of a chess root: a ChessPosition of this
        package, a FEN string, or an object with the reference IGameState interface (rebuilt by
        replaying get_move_history() - reference move encoding - from the start position)."""
        from .chess import ChessPosition
        if isinstance(state, str):
            state = ChessPosition(state)
        elif not isinstance(state, ChessPosition) and hasattr(state, "get_move_history"):
            p = ChessPosition()
            for m in state.get_move_history():
                p.play(int(m))
            state = p
        if not isinstance(state, ChessPosition):
            raise TypeError("chess state must be a ChessPosition, a FEN string or an IGameState")
        return state.root_records(), len(state.prior)

    def _search_chess(self, states, sims: int) -> np.ndarray:
        roots = [self._chess_root(s) for s in states]
        R = len(roots)
        if sims == 0:
            return np.full((R, self.action_size), 1.0 / self.action_size)
        eng = self._engine(R)
        self._drop_pending(eng)
        t0 = time.perf_counter()
        rec = np.stack([r[0] for r in roots])
        npr = np.array([r[1] for r in roots], np.int32)
        eng.search(rec, sims, self._eval, meta=npr, graphs=self._graphs_on)
        visits = eng.root_visits().cpu().numpy()
        self._last_tree = (eng, 0)
        self._update_statistics(sims * R, time.perf_counter() - t0)
        return self._policies(visits, eng)

    def _search_go(self, states, sims: int) -> np.ndarray:
        roots = [self._go_root(s) for s in states]
        R = len(roots)
        if sims == 0:
            return np.full((R, self.action_size), 1.0 / self.action_size)
        rules = {getattr(s, "rules", "chinese") for s in states}
        if len(rules) != 1:
            raise ValueError("one search batch must use one Go rule set")
        eng = self._engine(R, rules.pop())
        self._drop_pending(eng)
        t0 = time.perf_counter()
        hist = torch.from_numpy(np.stack([r[0] for r in roots])).to(self.device)
        meta = torch.from_numpy(np.stack([r[1] for r in roots])).to(self.device)
        eng.search(hist, sims, self._eval, meta=meta, keys=[r[2] for r in roots],
                   graphs=self._graphs_on)
        visits = eng.root_visits().cpu().numpy()
        self._last_tree = (eng, 0)
        self._update_statistics(sims * R, time.perf_counter() - t0)
        return self._policies(visits, eng)

    # -- search --------------------------------------------------------------------------------
    def search(self, state: Any, num_simulations: Optional[int] = None) -> np.ndarray:
        """Policy (fp64 [actions]) = root-child visit share (mcts.py:924-979)."""
        if self.is_go or self.is_chess:
            self._root_state = state
            fn = self._search_go if self.is_go else self._search_chess
            return fn([state], int(num_simulations or self.config.num_simulations))[0]
        board = self._boards(state)
        pol = self.search_batch(board[None], num_simulations)[0]
        if torch.is_tensor(board):
            board = board.cpu().numpy()
        self._root_state = board
        return pol

    def search_batch(self, states, num_simulations: Optional[int] = None) -> np.ndarray:
        """Independent searches of several roots in lockstep on the device; policies [R, A]."""
        if self.is_go or self.is_chess:
            fn = self._search_go if self.is_go else self._search_chess
            return fn(list(states), int(num_simulations or self.config.num_simulations))
        boards = self._boards(states)
        if boards.ndim == 2:
            boards = boards[None]
        sims = int(num_simulations or self.config.num_simulations)  # as mcts.py:941
        R = boards.shape[0]
        if sims == 0:                                        # mcts.py:1023-1031
            return np.full((R, self.action_size), 1.0 / self.action_size)
        eng = self._engine(R)
        self._drop_pending(eng)
        t0 = time.perf_counter()
        if torch.is_tensor(boards):   # host tensor (pinned for an asynchronous copy) or device
            dev_boards = boards.to(self.device, torch.int8, non_blocking=True)
        else:
            dev_boards = torch.from_numpy(np.ascontiguousarray(boards)).to(self.device)
        eng.search(dev_boards, sims, self._eval, graphs=self._graphs_on)
        visits = eng.root_visits().cpu().numpy()
        dt = time.perf_counter() - t0
        self._last_tree = (eng, 0)
        self._update_statistics(sims * R, dt)
        return self._policies(visits, eng)

    def _policies(self, visits: np.ndarray, eng: WaveEngine) -> np.ndarray:
        out = WaveEngine.policy_from_visits(visits)
        # a root without children yields the uniform policy (mcts.py:1081-1087)
        return out

    # -- reference API -------------------------------------------------------------------------
    def get_root_value(self) -> float:
        if self._last_tree is None:
            return 0.0
        eng, r = self._last_tree
        n, w = eng.root_nw()[r].tolist()
        return 0.0 if n == 0 else w / n

    def select_action(self, state: Any, temperature: float = 1.0,
                      policy: Optional[np.ndarray] = None) -> int:
        """mcts.py:1167-1203."""
        if policy is None:
            policy = self.search(state)
        if temperature == 0:
            return int(np.argmax(policy)) if policy.max() > 0 else 0
        p = np.power(policy, 1.0 / temperature)
        p /= p.sum()
        return int(np.random.choice(len(policy), p=p))

    def update_root(self, action: int, new_state: Any = None) -> None:
        """mcts.py:1205-1246. With subtree reuse on, the root child reached by ``action`` seeds the
        next search (omq_reroot on the last search's tree):
          * ``keep_subtree=True`` (extension): its whole subtree is kept, renumbered breadth-first
            as CSRTree.shift_root describes (csr_tree.py:1020-1229);
          * ``use_gpu_tree_reuse=True``: the next tree is fresh but its root starts with the
            child's visit count and value sum, which is what the reference's
            _gpu_friendly_tree_reuse (mcts.py:1929-2005) leaves behind;
          * otherwise a fresh tree: the reference's default reuse path raises inside
            apply_subtree_reuse (tree_operations.py:120) and falls back to a reset
            (mcts.py:1242-1246).
        The next search must start from the position ``action`` leads to."""
        if action < 0 or action >= self.action_size:
            raise ValueError(f"Invalid action {action}. Must be in range [0, {self.action_size})")
        c = self.config
        keep = bool(c.enable_subtree_reuse and getattr(c, "keep_subtree", False))
        carry = bool(c.enable_subtree_reuse and getattr(c, "use_gpu_tree_reuse", False))
        if self._last_tree is not None:
            eng, r = self._last_tree
            acts = np.full(eng.num_trees, -1, np.int32)
            if keep or carry:
                acts[r] = int(action)
                self.stats["tree_reuse_count"] = self.stats.get("tree_reuse_count", 0) + 1
            eng.reroot(acts, keep=keep)      # -1 everywhere: clears an earlier pending reroot
            self._pending = eng if (keep or carry) else None
            if not (keep or carry):
                self._last_tree = None
        if new_state is not None:
            self._root_state = new_state if (self.is_go or self.is_chess) else self._boards(new_state)

    def update_with_move(self, move: int) -> None:
        """mcts.py update_with_move: update_root(move, None)."""
        self.update_root(move, None)

    def warmup(self, num_searches: int = 3, simulations_per_search: int = 100) -> None:
        """mcts.py warmup: a few searches of the initial position before timed use (engine
        allocation, kernel attributes, the wave graph); the tree and statistics are reset after."""
        if self.is_go:
            from .go import GoPosition
            state = GoPosition(self.config.board_size)
        elif self.is_chess:
            from .chess import ChessPosition
            state = ChessPosition()
        else:
            state = np.zeros((self.config.board_size, self.config.board_size), np.int8)
        saved = dict(self.stats)
        for _ in range(max(0, int(num_searches))):
            self.search(state, num_simulations=int(simulations_per_search))
        self.clear()
        self.stats = saved

    def clear(self) -> None:
        self._drop_pending()
        self._last_tree = None
        self._root_state = None

    def reset_tree(self) -> None:
        self.clear()

    def get_statistics(self) -> Dict[str, Any]:
        s = dict(self.stats)
        if self._last_tree is not None:
            eng, r = self._last_tree
            s["tree_nodes"] = int(eng.num_nodes()[r])
            s["tree_capacity"] = eng.capacity
        s["device_memory_bytes"] = sum(e.memory_bytes() for e in self._engines.values())
        return s

    def _update_statistics(self, sims: int, dt: float) -> None:   # mcts.py:1442-1456
        st = self.stats
        st["total_searches"] += 1
        st["total_simulations"] += sims
        st["total_time"] += dt
        rate = sims / dt if dt > 0 else 0.0
        st["last_search_sims_per_second"] = rate
        st["peak_sims_per_second"] = max(st["peak_sims_per_second"], rate)
        st["avg_sims_per_second"] = st["total_simulations"] / st["total_time"] if st["total_time"] else 0.0

    def shutdown(self) -> None:
        for e in self._engines.values():
            e.close()
        self._engines.clear()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.shutdown()
        return False
