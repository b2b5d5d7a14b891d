"""Seeded synthetic root positions for the benchmark and parity configurations.

Gomoku roots: ``stones`` stones placed uniformly at random on empty cells, colours alternating
(black first), drawn from ``numpy.random.default_rng(seed)``; boards that already contain five in
a row are rejected and redrawn with the next attempt of the same generator. The side to move
follows the reference's numpy-root rule (python/mcts/core/mcts.py:1509-1519): black (1) when the
stone count is even, white (2) otherwise.
"""
from __future__ import annotations

import numpy as np


def has_five(board: np.ndarray) -> bool:
    """True if either player has five (or more) in a row anywhere (horizontal, vertical, both
    diagonals), the win rule of python/mcts/utils/fast_terminal_check.py:233-332."""
    b = np.asarray(board)
    n = b.shape[0]
    for p in (1, 2):
        m = (b == p)
        if (m[:, 0:n - 4] & m[:, 1:n - 3] & m[:, 2:n - 2] & m[:, 3:n - 1] & m[:, 4:n]).any():
            return True
        if (m[0:n - 4] & m[1:n - 3] & m[2:n - 2] & m[3:n - 1] & m[4:n]).any():
            return True
        if (m[0:n - 4, 0:n - 4] & m[1:n - 3, 1:n - 3] & m[2:n - 2, 2:n - 2] & m[3:n - 1, 3:n - 1]
                & m[4:n, 4:n]).any():
            return True
        if (m[0:n - 4, 4:n] & m[1:n - 3, 3:n - 1] & m[2:n - 2, 2:n - 2] & m[3:n - 1, 1:n - 3]
                & m[4:n, 0:n - 4]).any():
            return True
    return False


def random_root(seed: int, stones: int = 20, board_size: int = 15) -> np.ndarray:
    """One seeded Gomoku root board, int8 [board_size, board_size] (0 empty, 1 black, 2 white)."""
    rng = np.random.default_rng(seed)
    cells = board_size * board_size
    if not 0 <= stones <= cells:
        raise ValueError(f"stones must be in [0, {cells}]")
    while True:
        b = np.zeros(cells, np.int8)
        pos = rng.choice(cells, size=stones, replace=False)
        b[pos[0::2]] = 1
        b[pos[1::2]] = 2
        b = b.reshape(board_size, board_size)
        if not has_five(b):
            return b


def random_roots(seed: int, count: int, stones: int = 20, board_size: int = 15) -> np.ndarray:
    """``count`` roots; root i uses seed ``seed * 1_000_003 + i``. int8 [count, n, n]."""
    return np.stack([random_root(seed * 1_000_003 + i, stones, board_size) for i in range(count)])
