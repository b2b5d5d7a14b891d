"""Batched self-play driver: many Gomoku games advanced move by move, all searches of a move in
one device wave loop (512 games, 800 simulations, wave 64, 30 moves).

Per move it follows the reference's ``SelfPlayGame.play_single_move``
(python/mcts/neural_networks/self_play_manager.py:218-370): search the current position, record
``(state, policy, player, move_number)``, choose the move (sampled from the policy while
``move_number < temperature_threshold``, arg-max afterwards; ``_get_temperature`` :466-470), play
it, and restart the tree from the new position (``update_root`` without subtree reuse). At the end
each example gets the game outcome from its player's perspective (:388-420), and the examples use
the reference's ``GameExample`` fields (python/mcts/neural_networks/replay_buffer.py:18-37).

The searches of all live games run as one batch of independent trees in a ``WaveEngine``, so
the leaf queue of every wave holds all games' leaves. Sampling and bookkeeping stay on the host
with one seeded generator per game, so a run is reproducible.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Callable, Dict, List, Optional

import numpy as np

from .roots import has_five


@dataclass
class GameExample:
    """Training example (replay_buffer.py:18-37)."""
    state: np.ndarray
    policy: np.ndarray
    value: float
    game_id: str = ""
    move_number: int = 0


@dataclass
class GameRecord:
    game_id: str
    moves: List[int] = field(default_factory=list)
    examples: List[dict] = field(default_factory=list)
    winner: int = 0          # +1 black (player 1) won, -1 white won, 0 draw / unfinished
    finished: bool = False

    def training_examples(self) -> List[GameExample]:
        out = []
        for ex in self.examples:
            v = self.winner if ex["player"] == 1 else -self.winner
            out.append(GameExample(state=ex["state"], policy=ex["policy"], value=float(v),
                                   game_id=self.game_id, move_number=ex["move_number"]))
        return out


def board_after(board: np.ndarray, action: int) -> np.ndarray:
    """Place the side to move's stone (black when the stone count is even)."""
    b = board.copy()
    player = 1 if int((b != 0).sum()) % 2 == 0 else 2
    flat = b.reshape(-1)
    if flat[action] != 0:
        raise ValueError(f"illegal move {action}: cell occupied")
    flat[action] = player
    return b


def game_result(board: np.ndarray) -> Optional[int]:
    """None while the game goes on; else +1 / -1 for a black / white five, 0 for a full board.
    The player who just moved is the only one who can have completed a five."""
    if has_five(board):
        stones = int((board != 0).sum())
        return 1 if stones % 2 == 1 else -1
    if not (board == 0).any():
        return 0
    return None


class BatchedSelfPlay:
    """Self-play of ``num_games`` games in lockstep.

    ``search(boards [G, n, n] int8) -> visits [G, A] int`` runs one move's searches; by default
    it is a ``WaveEngine`` search with ``evaluator`` ("synthetic", a ResNetEvaluator, or any
    evaluate_batch object). Finished games keep their final board and are not searched again.
    """

    def __init__(self, num_games: int, num_simulations: int = 800, wave_size: int = 64,
                 evaluator="synthetic", capacity: int = 200000, c_puct: float = 1.4,
                 temperature: float = 1.0, temperature_threshold: int = 30, seed: int = 0,
                 roots: Optional[np.ndarray] = None, board_size: int = 15,
                 search: Optional[Callable[[np.ndarray], np.ndarray]] = None, device=None):
        self.G = int(num_games)
        self.sims = int(num_simulations)
        self.temperature = float(temperature)
        self.temperature_threshold = int(temperature_threshold)
        self.n = board_size
        self.boards = (np.zeros((self.G, board_size, board_size), np.int8) if roots is None
                       else np.array(roots, dtype=np.int8, copy=True))
        self.rngs = [np.random.default_rng([seed, g]) for g in range(self.G)]
        self.records = [GameRecord(game_id=f"selfplay_{seed}_{g}") for g in range(self.G)]
        self.move_number = 0
        self._search = search
        if search is None:
            self._evaluator = evaluator
            self._engine_args = dict(board_size=board_size, capacity=capacity, max_wave_size=wave_size,
                                     c_puct=c_puct, device=device)
            self._engines: Dict[int, object] = {}

    # -- search ----------------------------------------------------------------------------
    def _device_search(self, boards: np.ndarray) -> np.ndarray:
        import torch
        from .engine import WaveEngine
        R = boards.shape[0]
        eng = self._engines.get(R)
        if eng is None:
            eng = WaveEngine(R, **self._engine_args)
            self._engines[R] = eng
        eng.search(torch.from_numpy(np.ascontiguousarray(boards)).to(eng.device), self.sims, self._evaluator)
        return eng.root_visits().cpu().numpy()

    def live(self) -> np.ndarray:
        return np.array([not r.finished for r in self.records])

    # -- one move of every live game ---------------------------------------------------------
    def step(self) -> int:
        """Play one move in every live game; returns the number of games that moved."""
        live = np.nonzero(self.live())[0]
        if len(live) == 0:
            return 0
        search = self._search or self._device_search
        visits = np.asarray(search(self.boards[live]))
        for i, g in enumerate(live):
            v = visits[i].astype(np.float64)
            tot = v.sum()
            policy = v / tot if tot > 0 else np.full(v.shape, 1.0 / v.size)
            board = self.boards[g]
            player = 1 if int((board != 0).sum()) % 2 == 0 else 2
            rec = self.records[g]
            rec.examples.append({"state": board.copy(), "policy": policy, "player": player,
                                 "move_number": self.move_number})
            if self.move_number < self.temperature_threshold and self.temperature > 0:
                p = policy if self.temperature == 1.0 else np.power(policy, 1.0 / self.temperature)
                p = p / p.sum()
                action = int(self.rngs[g].choice(len(p), p=p))
            else:
                action = int(np.argmax(policy))
            self.boards[g] = board_after(board, action)
            rec.moves.append(action)
            res = game_result(self.boards[g])
            if res is not None:
                rec.finished = True
                rec.winner = res
        self.move_number += 1
        return len(live)

    def play(self, max_moves: int) -> List[GameRecord]:
        for _ in range(max_moves):
            if self.step() == 0:
                break
        return self.records

    def examples(self) -> List[GameExample]:
        out: List[GameExample] = []
        for r in self.records:
            out.extend(r.training_examples())
        return out
