"""Batched self-play driver: many games advanced move by move, all searches of a move in one device
wave loop (benchmark config 2: 512 Gomoku games, 800 simulations, wave 64, 30 moves). Gomoku, Go
and chess games are supported (``game=``).

Per move it follows the reference's ``SelfPlayGame.play_single_move``
(python/mcts/neural_networks/self_play_manager.py:218-370): search the current position, record
``(state, policy, player, move_number)``, choose the move (sampled from the policy while
``move_number < temperature_threshold``, arg-max afterwards; ``_get_temperature`` :466-470), play
it, and restart the tree from the new position (``update_root`` without subtree reuse, or with
``subtree_reuse`` "carry" / "keep" as ``MCTS.update_root`` has them). At the end
each example gets the game outcome from its player's perspective (:388-420), and the examples use
the reference's ``GameExample`` fields (python/mcts/neural_networks/replay_buffer.py:18-37).

The searches of all live games run as one batch of independent trees in a ``WaveEngine``, so
the leaf queue of every wave holds all games' leaves. Two ways to choose and play the moves:
  * ``sampling="host"`` (every game type): bookkeeping on the host, one seeded numpy generator per
    game (``rng="numpy"``), or the device's counter-based draws (``rng="counter"``, temperature 0
    or 1) so that a host run replays a device run exactly;
  * ``sampling="device"`` (every game, temperature 0 or 1, the built-in engine): positions (boards,
    the chess engine's root records, or Go's history boards, side / ko / passes and position
    keys), histories and game states stay in device memory, and one kernel per move
    (``omq_selfplay_move``, ``omq_selfplay_move_chess``, ``omq_selfplay_move_go``)
    records the examples, draws and plays the moves and applies the end and resignation rules,
    so a move costs no host round trip beyond the search's status check. Tree g is game g for
    the whole run (finished games get a one-node fresh tree each move); the trees are
    independent, so results equal the host driver's, which searches only the live games.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Callable, Dict, List, Optional

import numpy as np

from .roots import has_five

_MASK64 = (1 << 64) - 1


def _mix64(x: int) -> int:
    """SplitMix64 finaliser on Python ints (the device's mix64)."""
    x &= _MASK64
    x ^= x >> 30
    x = (x * 0xBF58476D1CE4E5B9) & _MASK64
    x ^= x >> 27
    x = (x * 0x94D049BB133111EB) & _MASK64
    x ^= x >> 31
    return x


def counter_draw(seed: int, game: int, move: int) -> int:
    """The 64-bit draw of (seed, game, move) that omq_selfplay_move uses."""
    return _mix64((_mix64((_mix64(seed) + game) & _MASK64) + move) & _MASK64)


def counter_choice(visits: np.ndarray, draw: int) -> int:
    """The action omq_selfplay_move samples from a visit-count row: the first action whose
    cumulative count exceeds floor(draw / 2^64 * total) - visit-proportional sampling, i.e.
    temperature 1 on policy = visits / total; uniform over all actions when total is 0 (the
    uniform policy of an empty search)."""
    v = np.asarray(visits, np.int64)
    total = int(v.sum())
    if total == 0:
        return (draw * v.size) >> 64
    target = (draw * total) >> 64
    return int(np.searchsorted(np.cumsum(v), target, side="right"))


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
    resigned: bool = False

    def training_examples(self, use_mcts_q_values: bool = False,
                          q_value_weight: float = 0.8) -> List[GameExample]:
        """The game outcome from each example's player's perspective (self_play_manager.py:
        400-431); with ``use_mcts_q_values`` mixed as q_value_weight * root value of that move's
        search + (1 - q_value_weight) * outcome."""
        out = []
        for ex in self.examples:
            v = self.winner if ex["player"] == 1 else -self.winner
            if use_mcts_q_values:
                v = q_value_weight * ex.get("value_pred", 0.0) + (1 - q_value_weight) * v
            out.append(GameExample(state=ex["state"], policy=ex["policy"], value=float(v),
                                   game_id=self.game_id, move_number=ex["move_number"]))
        return out

    def metrics(self) -> Dict[str, object]:
        """Per-game metrics of the reference's play_game (self_play_manager.py:263-270, 433-462):
        policy entropies, sign accuracy of the root values against the outcome (|v| < 0.1 for a
        draw), game length, winner, resignation."""
        ent, acc = [], []
        for ex in self.examples:
            p = ex["policy"][ex["policy"] > 1e-10]
            ent.append(float(-(p * np.log(p)).sum()) if len(p) else 0.0)
            actual = self.winner if ex["player"] == 1 else -self.winner
            vp = ex.get("value_pred", 0.0)
            acc.append((1.0 if abs(vp) < 0.1 else 0.0) if actual == 0 else (1.0 if vp * actual > 0 else 0.0))
        return {"resigned": self.resigned, "policy_entropies": ent, "value_accuracies": acc,
                "game_length": len(self.examples), "winner": self.winner}


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


class _GomokuGame:
    """Positions are int8 boards; the side to move follows the stone count."""
    name = "gomoku"

    def __init__(self, n):
        self.n = n

    def initial(self, roots, G):
        if roots is None:
            return [np.zeros((self.n, self.n), np.int8) for _ in range(G)]
        return [np.array(r, dtype=np.int8, copy=True) for r in roots]

    def engine_input(self, positions):
        return np.stack(positions), None

    def player(self, pos):
        return 1 if int((pos != 0).sum()) % 2 == 0 else 2

    def state(self, pos):
        return pos.copy()

    def apply(self, pos, action):
        return board_after(pos, action)

    def outcome(self, pos):
        return game_result(pos)

    # device-resident games (omq_selfplay_move)
    actions = property(lambda self: self.n * self.n)
    state_bytes = property(lambda self: self.n * self.n)

    def device_roots(self, positions):
        return {"boards": np.stack(positions).astype(np.int8).reshape(len(positions), -1)}

    def device_state(self, row):
        return np.asarray(row, np.int8).reshape(self.n, self.n).copy()

    def device_position(self, roots, g, start, game_row):
        return roots["boards"][g].reshape(self.n, self.n).copy()


class _GoGame:
    """Positions are GoPosition objects; the game ends with two passes, scored by area."""
    name = "go"

    def __init__(self, n):
        self.n = n

    def initial(self, roots, G):
        from .go import GoPosition
        return [GoPosition(self.n) if roots is None else roots[g].copy() for g in range(G)]

    def engine_input(self, positions):
        return (np.stack([p.history_planes() for p in positions]),
                {"meta": np.stack([p.meta() for p in positions]),
                 "keys": [p.root_keys() for p in positions]})

    def player(self, pos):
        return pos.to_move

    def rules(self, positions):
        """The rule set of a batch (GoPosition.rules); one search batch uses one rule set."""
        rules = {getattr(p, "rules", "chinese") for p in positions}
        if len(rules) != 1:
            raise ValueError("one self-play batch must use one Go rule set")
        return rules.pop()

    def state(self, pos):
        return pos.history_planes()

    def apply(self, pos, action):
        q = pos.copy()
        q.play(int(action))
        return q

    def outcome(self, pos):
        # 4 is the Japanese rules' "no result" of a third repetition: no winner, as a draw
        r = pos.result()
        return None if r == 0 else {1: 1, 2: -1, 3: 0, 4: 0}[r]

    # device-resident games (omq_selfplay_move_go): the engine's Go roots
    actions = property(lambda self: self.n * self.n + 1)
    state_bytes = property(lambda self: 8 * self.n * self.n)

    def device_roots(self, positions):
        from . import _lib
        G, K = len(positions), _lib.GO_MAX_KEYS
        keys = np.zeros((G, K), np.uint64)
        nkeys = np.zeros(G, np.int32)
        for g, p in enumerate(positions):
            k = p.root_keys()
            keys[g, :k.size] = k
            nkeys[g] = k.size
        return {"history": np.stack([p.history_planes() for p in positions]),
                "meta": np.stack([p.meta() for p in positions]).astype(np.int32),
                "keys": keys.view(np.int64), "nkeys": nkeys}

    def device_game(self, pos):
        """Columns 5-7 of the device game record: prisoners of black and white, repetition end."""
        return [pos.prisoners[1], pos.prisoners[2], int(pos.repeated)]

    def device_state(self, row):
        return np.asarray(row, np.int8).reshape(8, self.n, self.n).copy()

    def device_position(self, roots, g, start, game_row):
        q = start.copy()
        h = roots["history"][g].reshape(8, self.n, self.n)
        q.board = h[0].copy()
        q.history = [h[k].copy() for k in range(7, -1, -1)]
        q.to_move, q.ko, q.passes = (int(x) for x in roots["meta"][g])
        q.keys = [int(k) for k in roots["keys"][g][: int(roots["nkeys"][g])].view(np.uint64)]
        q.prisoners = [0, int(game_row[5]), int(game_row[6])]
        q.repeated = bool(game_row[7])
        return q


class _ChessGame:
    """Positions are ChessPosition objects (the reference engine's rules); actions are the
    engine's 4672 AlphaZero moves of the position."""
    name = "chess"

    def __init__(self, n):
        self.n = 8

    def initial(self, roots, G):
        from .chess import ChessPosition
        return [ChessPosition() if roots is None else roots[g].copy() for g in range(G)]

    def engine_input(self, positions):
        return (np.stack([p.root_records() for p in positions]),
                {"meta": np.array([len(p.prior) for p in positions], np.int32)})

    def player(self, pos):
        return int(pos.side)

    def state(self, pos):
        return pos.record()

    def apply(self, pos, action):
        q = pos.copy()
        q.play(q.action_to_move(int(action)))
        return q

    def outcome(self, pos):
        r = pos.result()
        return None if r == 0 else {1: 1, 2: -1, 3: 0}[r]

    # device-resident games (omq_selfplay_move_chess): the engine's root records
    actions = 4672
    state_bytes = 80

    def device_roots(self, positions):
        recs = np.stack([p.root_records() for p in positions])
        return {"records": np.ascontiguousarray(recs).view(np.uint8).reshape(len(positions), -1),
                "nprior": np.array([min(len(p.prior), 100) for p in positions], np.int32)}

    def device_state(self, row):
        from .chess import POS_DTYPE
        return np.frombuffer(np.asarray(row, np.uint8).tobytes(), POS_DTYPE).reshape(()).copy()

    def device_position(self, roots, g, start, game_row):
        from .chess import POS_DTYPE, ChessPosition
        recs = np.frombuffer(np.asarray(roots["records"][g], np.uint8).tobytes(), POS_DTYPE)
        return ChessPosition.from_records(recs, int(roots["nprior"][g]))


_GAMES = {"gomoku": _GomokuGame, "go": _GoGame, "chess": _ChessGame}


class BatchedSelfPlay:
    """Self-play of ``num_games`` games in lockstep.

    ``search(inputs) -> visits [G, A] int`` runs one move's searches; by default it is a
    ``WaveEngine`` search with ``evaluator`` ("synthetic", a ResNetEvaluator, or any
    evaluate_batch object). For Gomoku ``inputs`` is the boards array [G, n, n]; for Go and chess
    it is the pair (root records, keyword arguments of ``WaveEngine.search``). Finished games keep
    their final position and are not searched again.
    """

    def __init__(self, num_games: int, num_simulations: int = 800, wave_size: int = 64,
                 evaluator="synthetic", capacity: int = 200000, c_puct: float = 1.4,
                 temperature: float = 1.0, temperature_threshold: int = 30, seed: int = 0,
                 roots=None, board_size: int = 15,
                 search: Optional[Callable] = None, device=None, game: str = "gomoku",
                 subtree_reuse: str = "none", enable_resign: bool = True,
                 resign_threshold: float = -0.98, resign_min_move: int = 10,
                 sampling: str = "host", rng: str = "numpy", max_moves: int = 512):
        if game not in _GAMES:
            raise ValueError(f"unknown game {game!r}")
        if sampling not in ("host", "device") or rng not in ("numpy", "counter"):
            raise ValueError("sampling is 'host' or 'device', rng 'numpy' or 'counter'")
        if (sampling == "device" or rng == "counter") and temperature not in (0.0, 1.0):
            raise ValueError("counter-based draws take temperature 0 or 1")
        if sampling == "device" and search is not None:
            raise ValueError("device sampling runs the games on the built-in engine")
        self.sampling, self.rng_kind, self.seed = sampling, rng, int(seed)
        if subtree_reuse not in ("none", "carry", "keep"):
            raise ValueError("subtree_reuse must be 'none', 'carry' or 'keep'")
        # between moves the played child seeds the next search of its game (omq_reroot): "keep"
        # keeps its subtree, "carry" its visit count and value sum (the reference's
        # use_gpu_tree_reuse behaviour); only while the set of live games is unchanged, so that
        # tree r still belongs to the same game
        self.subtree_reuse = subtree_reuse
        # resignation as SelfPlayGame (self_play_manager.py:350-365; SelfPlayConfig defaults)
        self.enable_resign = bool(enable_resign)
        self.resign_threshold = float(resign_threshold)
        self.resign_min_move = int(resign_min_move)
        self._last_move = None          # (live games, their moves) of the previous step
        self._live_now = None
        self._rules_now = None
        self.game = _GAMES[game](board_size)
        self.G = int(num_games)
        self.sims = int(num_simulations)
        self.temperature = float(temperature)
        self.temperature_threshold = int(temperature_threshold)
        self.n = self.game.n
        self.positions = self.game.initial(roots, self.G)
        self.rngs = [np.random.default_rng([seed, g]) for g in range(self.G)]
        self.records = [GameRecord(game_id=f"selfplay_{seed}_{g}") for g in range(self.G)]
        self.move_number = 0
        self._search = search
        if search is None:
            self._evaluator = evaluator
            self._engine_args = dict(board_size=self.n, capacity=capacity, max_wave_size=wave_size,
                                     c_puct=c_puct, device=device, game=game)
            self._engines: Dict[int, object] = {}
        self._dev = None
        if sampling == "device":
            self._init_device(int(max_moves), device)

    def close(self) -> None:
        """Free the device engines (their trees); the evaluator belongs to the caller."""
        for eng in getattr(self, "_engines", {}).values():
            eng.close()
        if hasattr(self, "_engines"):
            self._engines.clear()
        self._dev = None

    # -- device-resident games ---------------------------------------------------------------
    def _init_device(self, max_moves: int, device) -> None:
        import torch
        from .engine import WaveEngine
        args = dict(self._engine_args)
        if self.game.name == "go":
            from . import _lib
            p0 = self.positions[0]
            if any((p.rules, p.superko, p.komi) != (p0.rules, p0.superko, p0.komi) for p in self.positions):
                raise ValueError("device Go self-play needs one rule set, superko setting and komi")
            if max(len(p.keys) for p in self.positions) + max_moves > _lib.GO_MAX_KEYS:
                raise ValueError(f"device Go self-play keeps {_lib.GO_MAX_KEYS} position keys per game: "
                                 "the roots' keys plus max_moves must fit")
            args.update(go_rules=p0.rules, go_superko=p0.superko)
        eng = WaveEngine(self.G, **args)
        self._engines[("device", self.G)] = eng
        dev = eng.device
        G, A = self.G, self.game.actions
        self._start = [p.copy() for p in self.positions]
        roots = {k: torch.from_numpy(v).to(dev) for k, v in self.game.device_roots(self.positions).items()}
        self._dev = {
            "engine": eng, "roots": roots,
            "game": torch.zeros(G, 8, dtype=torch.int32, device=dev),
            "actions": torch.full((G,), -1, dtype=torch.int32, device=dev),
            "moves": torch.full((G, max_moves), -1, dtype=torch.int32, device=dev),
            "visits": torch.zeros(G, max_moves, A, dtype=torch.int32, device=dev),
            "values": torch.zeros(G, max_moves, dtype=torch.float32, device=dev),
            "states": torch.zeros(G, max_moves, self.game.state_bytes, dtype=torch.uint8, device=dev),
            "max_moves": max_moves, "synced": 0,
        }
        # games whose start position is already decided begin finished, as the host driver
        # finds them when it checks the outcome (it never searches them)
        for g, pos in enumerate(self.positions):
            res = self.game.outcome(pos)
            if res is not None:
                self.records[g].finished, self.records[g].winner = True, res
                self._dev["game"][g, 0] = 1
                self._dev["game"][g, 1] = res
            if hasattr(self.game, "device_game"):
                self._dev["game"][g, 5:8] = torch.tensor(self.game.device_game(pos), dtype=torch.int32)

    def _device_step(self) -> int:
        import ctypes
        from . import _lib
        from .engine import _stream_ptr
        d = self._dev
        if self.move_number >= d["max_moves"]:
            raise ValueError(f"max_moves ({d['max_moves']}) reached")
        live = int((d["game"][:, 0] == 0).sum().item())
        if live == 0:
            return 0
        eng, roots = d["engine"], d["roots"]
        # subtree reuse while the set of live games is unchanged, as the host driver has it
        if self.subtree_reuse != "none" and self.move_number > 0 and live == d.get("live"):
            eng.reroot(d["actions"], keep=self.subtree_reuse == "keep")
        d["live"] = live
        cfg = _lib.SelfplayStepConfig(self.move_number, d["max_moves"], self.temperature_threshold,
                                      self.temperature, int(self.enable_resign), self.resign_min_move,
                                      self.resign_threshold, self.seed & _MASK64)
        p = lambda t: ctypes.c_void_p(t.data_ptr())
        hist = (p(d["game"]), p(d["actions"]), p(d["moves"]), p(d["visits"]), p(d["values"]), p(d["states"]))
        if self.game.name == "go":
            pos0 = self._start[0]
            eng.search(roots["history"], self.sims, self._evaluator, meta=roots["meta"],
                       keys=(roots["keys"], roots["nkeys"]))
            _lib.check(eng.L.omq_selfplay_move_go(eng._h, ctypes.byref(cfg), ctypes.c_float(pos0.komi),
                                                  int(pos0.rules == "chinese"), p(roots["history"]),
                                                  p(roots["meta"]), p(roots["keys"]), p(roots["nkeys"]), *hist,
                                                  _stream_ptr()), "omq_selfplay_move_go")
        elif self.game.name == "chess":
            eng.search(roots["records"], self.sims, self._evaluator, meta=roots["nprior"])
            _lib.check(eng.L.omq_selfplay_move_chess(eng._h, ctypes.byref(cfg), p(roots["records"]),
                                                     p(roots["nprior"]), *hist, _stream_ptr()),
                       "omq_selfplay_move_chess")
        else:
            eng.search(roots["boards"].view(self.G, self.n, self.n), self.sims, self._evaluator)
            _lib.check(eng.L.omq_selfplay_move(eng._h, ctypes.byref(cfg), p(roots["boards"]), *hist, _stream_ptr()),
                       "omq_selfplay_move")
        self.move_number += 1
        return live

    def _sync_device(self) -> None:
        """Copy the device histories of the moves played since the last sync into the records
        and positions (examples as the host driver records them)."""
        d = self._dev
        if d is None or d["synced"] == self.move_number:
            return
        m0, m1 = d["synced"], self.move_number
        game = d["game"].cpu().numpy()
        if (game[:, 3] != 0).any():
            raise RuntimeError("device self-play: an illegal move was drawn")
        moves = d["moves"][:, m0:m1].cpu().numpy()
        visits = d["visits"][:, m0:m1].cpu().numpy()
        values = d["values"][:, m0:m1].cpu().numpy()
        states = d["states"][:, m0:m1].cpu().numpy()
        roots = {k: v.cpu().numpy() for k, v in d["roots"].items()}
        for g, rec in enumerate(self.records):
            for m in range(m0, min(m1, int(game[g, 4]))):
                k = m - m0
                v = visits[g, k].astype(np.float64)
                tot = v.sum()
                st = self.game.device_state(states[g, k])
                rec.examples.append({"state": st, "policy": v / tot if tot > 0 else np.full(v.shape, 1.0 / v.size),
                                     "player": self._state_player(st, g, m), "move_number": m,
                                     "value_pred": float(values[g, k])})
                rec.moves.append(int(moves[g, k]))
            self.positions[g] = self.game.device_position(roots, g, self._start[g], game[g])
            if game[g, 0] and not rec.finished:
                rec.finished, rec.winner, rec.resigned = True, int(game[g, 1]), bool(game[g, 2])
        d["synced"] = m1

    def _state_player(self, st, g: int, m: int) -> int:
        """The side to move of a recorded state (a board, a chess record, or Go history planes)."""
        if self.game.name == "chess":
            return int(st["side"])
        if self.game.name == "go":      # every move (passes included) changes the side to move
            p0 = self._start[g].to_move
            return p0 if m % 2 == 0 else 3 - p0
        return self.game.player(st)

    # -- search ----------------------------------------------------------------------------
    @property
    def boards(self) -> np.ndarray:
        """Gomoku: the games' boards [G, n, n]."""
        return np.stack(self.positions)

    def _device_search(self, inputs) -> np.ndarray:
        import torch
        from .engine import WaveEngine
        roots, kw = inputs if isinstance(inputs, tuple) else (inputs, {})
        R = roots.shape[0]
        key = (R, self._rules_now)
        eng = self._engines.get(key)
        if eng is None:
            args = dict(self._engine_args)
            if self._rules_now is not None:
                args["go_rules"] = self._rules_now      # the device engine follows the positions
            eng = WaveEngine(R, **args)
            self._engines[key] = eng
        elif (self.subtree_reuse != "none" and self._last_move is not None
              and self._last_move[0] == self._live_now):
            eng.reroot(np.asarray(self._last_move[1], np.int32), keep=self.subtree_reuse == "keep")
        if self.game.name == "gomoku":
            eng.search(torch.from_numpy(np.ascontiguousarray(roots)).to(eng.device), self.sims, self._evaluator)
        else:
            eng.search(roots, self.sims, self._evaluator, **kw)
        nw = eng.root_nw().cpu().numpy()
        values = np.where(nw[:, 0] > 0, nw[:, 1] / np.maximum(nw[:, 0], 1), 0.0)
        return eng.root_visits().cpu().numpy(), values

    def live(self) -> np.ndarray:
        self._sync_device()
        return np.array([not r.finished for r in self.records])

    # -- one move of every live game ---------------------------------------------------------
    def step(self) -> int:
        """Play one move in every live game; returns the number of games that moved."""
        if self._dev is not None:
            return self._device_step()
        live = np.nonzero(self.live())[0]
        if len(live) == 0:
            return 0
        search = self._search or self._device_search
        self._live_now = tuple(int(g) for g in live)
        self._rules_now = (self.game.rules([self.positions[g] for g in live])
                           if hasattr(self.game, "rules") else None)
        moves = []
        roots, meta = self.game.engine_input([self.positions[g] for g in live])
        res = search(roots if meta is None else (roots, meta))
        # a search returns the root visits, or (visits, root values) - the root value W / N is
        # MCTS.get_root_value(), from the side to move's perspective
        if isinstance(res, tuple):
            visits, values = np.asarray(res[0]), np.asarray(res[1], np.float64)
        else:
            visits, values = np.asarray(res), np.zeros(len(live))
        for i, g in enumerate(live):
            v = visits[i].astype(np.float64)
            tot = v.sum()
            policy = v / tot if tot > 0 else np.full(v.shape, 1.0 / v.size)
            pos = self.positions[g]
            player = self.game.player(pos)
            rec = self.records[g]
            rec.examples.append({"state": self.game.state(pos), "policy": policy, "player": player,
                                 "move_number": self.move_number,
                                 "value_pred": float(values[i])})
            if self.move_number < self.temperature_threshold and self.temperature > 0:
                if self.rng_kind == "counter":     # the device's draw (omq_selfplay_move)
                    action = counter_choice(visits[i], counter_draw(self.seed, int(g), self.move_number))
                else:
                    p = policy if self.temperature == 1.0 else np.power(policy, 1.0 / self.temperature)
                    p = p / p.sum()
                    action = int(self.rngs[g].choice(len(p), p=p))
            else:
                action = int(np.argmax(policy))
            self.positions[g] = self.game.apply(pos, action)
            rec.moves.append(action)
            moves.append(action)
            res = self.game.outcome(self.positions[g])
            if res is not None:
                rec.finished = True
                rec.winner = res
            # resignation after the move (the reference checks it even when the move ended the
            # game, and the resignation then decides the winner): the player who moved resigns
            if (self.enable_resign and self.move_number + 1 > self.resign_min_move
                    and values[i] < self.resign_threshold):
                rec.finished = True
                rec.resigned = True
                rec.winner = -1 if player == 1 else 1
        self._last_move = (self._live_now, moves)
        self.move_number += 1
        return len(live)

    def play(self, max_moves: int) -> List[GameRecord]:
        for _ in range(max_moves):
            if self.step() == 0:
                break
        self._sync_device()
        return self.records

    def examples(self) -> List[GameExample]:
        self._sync_device()
        out: List[GameExample] = []
        for r in self.records:
            out.extend(r.training_examples())
        return out
