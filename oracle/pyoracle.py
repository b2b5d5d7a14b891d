"""Parity oracle bindings - TEST INFRASTRUCTURE ONLY.

ctypes access to ``oracle/_build/liboracle.so`` (the C++ restatement of the reference's
deterministic CPU wave search, see ``oracle/oracle.h``) and a numpy twin of the integer-exact
synthetic evaluator (``oracle/synth_eval.h``), which is what the reference search is driven
with when golden fixtures are generated.

Only ``tests/``, ``bench.py`` (its CPU-baseline leg) and ``__graft_entry__.smoke()`` may import
this module, and only as the checker. The product package never imports it.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from dataclasses import dataclass

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "liboracle.so")

PLANES = 19
MASK64 = np.uint64(0xFFFFFFFFFFFFFFFF)

EXP2_TABLE = np.array([
    1048576, 1059994, 1071537, 1083205, 1095000, 1106924, 1118978, 1131163, 1143480, 1155932,
    1168519, 1181244, 1194106, 1207109, 1220254, 1233542, 1246974, 1260553, 1274279, 1288155,
    1302182, 1316362, 1330696, 1345187, 1359835, 1374642, 1389611, 1404743, 1420040, 1435503,
    1451135, 1466937, 1482910, 1499058, 1515382, 1531883, 1548564, 1565427, 1582474, 1599706,
    1617125, 1634735, 1652536, 1670531, 1688722, 1707110, 1725700, 1744491, 1763488, 1782691,
    1802103, 1821727, 1841564, 1861617, 1881889, 1902381, 1923097, 1944038, 1965207, 1986607,
    2008240, 2030108, 2052214, 2074562], dtype=np.uint64)

_SEED = np.uint64(0x243F6A8885A308D3)
_GOLDEN = np.uint64(0x9E3779B97F4A7C15)
_VALUE_SALT = np.uint64(0xD1B54A32D192ED03)


def torch_sum(x: np.ndarray) -> np.float32:
    """The oracle's restatement of torch's CPU summation order for a contiguous fp32 vector."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    return np.float32(lib().oracle_torch_sum(x.ctypes.data, int(x.size)))


def build(quiet: bool = True) -> str:
    """Compile liboracle.so (g++, no GPU needed)."""
    out = subprocess.run(["make", "-C", _HERE, "all"], capture_output=True, text=True)
    if out.returncode != 0:
        raise RuntimeError("oracle build failed:\n" + out.stdout + out.stderr)
    return _LIB_PATH


# ----------------------------------------------------------------------------------------------
# numpy twin of the synthetic evaluator
# ----------------------------------------------------------------------------------------------
def _mix64(x: np.ndarray) -> np.ndarray:
    x = x.astype(np.uint64, copy=True)
    with np.errstate(over="ignore"):
        x ^= x >> np.uint64(30)
        x *= np.uint64(0xBF58476D1CE4E5B9)
        x ^= x >> np.uint64(27)
        x *= np.uint64(0x94D049BB133111EB)
        x ^= x >> np.uint64(31)
    return x


def feature_hash(features: np.ndarray) -> np.ndarray:
    """features [B, planes, cells] -> uint64 [B] (oracle_feature_hash)."""
    f = np.asarray(features, dtype=np.float32)
    B, planes, cells = f.shape
    words = (cells + 63) // 64
    pad = np.zeros((B, planes, words * 64), dtype=np.uint64)
    pad[:, :, :cells] = (f != 0).astype(np.uint64)
    shifts = (np.uint64(1) << np.arange(64, dtype=np.uint64))
    packed = (pad.reshape(B, planes, words, 64) * shifts).sum(axis=3, dtype=np.uint64)
    h = np.full(B, _SEED, dtype=np.uint64)
    for c in range(planes):
        if c == 1:
            h = _mix64(h ^ f[:, 1, 0].astype(np.int64).astype(np.uint64))
            continue
        for j in range(words):
            h = _mix64(h ^ packed[:, c, j])
    return h


def _exp_step(r: np.ndarray) -> np.ndarray:
    m = np.uint64(0xFFFF)
    s = ((r & m).astype(np.int64) + ((r >> np.uint64(16)) & m).astype(np.int64)
         + ((r >> np.uint64(32)) & m).astype(np.int64) + ((r >> np.uint64(48)) & m).astype(np.int64)
         - 131072)
    return (s * 160) >> 16


def _exp2_fixed(t: np.ndarray) -> np.ndarray:
    return EXP2_TABLE[t & 63] << ((t >> 6) + 6).astype(np.uint64)


def synth_eval(features, actions: int | None = None):
    """features [B, planes, H, W] (numpy or torch, fp32) -> (policy [B, A] fp32, value [B] fp32)."""
    f = np.asarray(features.cpu().numpy() if hasattr(features, "cpu") else features, dtype=np.float32)
    B = f.shape[0]
    f = f.reshape(B, f.shape[1], -1)
    cells = f.shape[2]
    A = cells if actions is None else actions
    h = feature_hash(f)
    legal = np.ones((B, A), dtype=bool)
    legal[:, :cells] = f[:, 0, :] == 0
    a1 = np.arange(1, A + 1, dtype=np.uint64)
    with np.errstate(over="ignore"):
        r = _mix64(h[:, None] + _GOLDEN * a1[None, :])
    w = np.where(legal, _exp2_fixed(_exp_step(r)), np.uint64(0))
    total = w.sum(axis=1, dtype=np.uint64)
    idx = (np.cumsum(legal, axis=1) - 1).astype(np.uint64)
    safe_total = np.where(total == 0, np.uint64(1), total)
    m = (w * np.uint64(32640)) // safe_total[:, None]
    q = np.uint64(512) * m + idx
    policy = np.where(legal, q.astype(np.float32) * np.float32(1.0 / 16777216.0), np.float32(0.0))
    e = _exp2_fixed(_exp_step(_mix64(h ^ _VALUE_SALT))).astype(np.int64)
    d = np.int64(1 << 26)
    num = (e - d) * 4096
    den = e + d
    v = np.sign(num) * (np.abs(num) // den)  # truncation toward zero, as in C
    value = v.astype(np.float32) * np.float32(1.0 / 4096.0)
    return policy.astype(np.float32), value.astype(np.float32)


# ----------------------------------------------------------------------------------------------
# ctypes bindings
# ----------------------------------------------------------------------------------------------
class OracleConfig(ctypes.Structure):
    _fields_ = [("board_size", ctypes.c_int), ("num_simulations", ctypes.c_int),
                ("max_wave_size", ctypes.c_int), ("c_puct", ctypes.c_float),
                ("virtual_loss", ctypes.c_float), ("enable_virtual_loss", ctypes.c_int),
                ("max_nodes", ctypes.c_int), ("max_depth", ctypes.c_int)]


class OracleResult(ctypes.Structure):
    _fields_ = [("status", ctypes.c_int), ("num_nodes", ctypes.c_int), ("waves", ctypes.c_int),
                ("boundary_ties", ctypes.c_int), ("order_ties", ctypes.c_int),
                ("eval_calls", ctypes.c_int), ("eval_positions", ctypes.c_longlong)]


EVAL_FN = ctypes.CFUNCTYPE(None, ctypes.c_void_p, ctypes.c_int, ctypes.POINTER(ctypes.c_float),
                           ctypes.POINTER(ctypes.c_float), ctypes.POINTER(ctypes.c_float))

_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        L.oracle_tree_create.restype = ctypes.c_void_p
        L.oracle_tree_create.argtypes = [ctypes.c_int, ctypes.c_int]
        L.oracle_tree_destroy.argtypes = [ctypes.c_void_p]
        L.oracle_begin.argtypes = [ctypes.c_void_p, ctypes.POINTER(OracleConfig), ctypes.c_void_p,
                                   EVAL_FN, ctypes.c_void_p]
        L.oracle_wave.argtypes = [ctypes.c_void_p, ctypes.c_int]
        L.oracle_set_root_noise.argtypes = [ctypes.c_void_p, ctypes.c_float, ctypes.c_float, ctypes.c_void_p]
        L.oracle_search.argtypes = [ctypes.c_void_p, ctypes.POINTER(OracleConfig), ctypes.c_void_p,
                                    EVAL_FN, ctypes.c_void_p, ctypes.POINTER(OracleResult)]
        L.oracle_get_result.argtypes = [ctypes.c_void_p, ctypes.POINTER(OracleResult)]
        L.oracle_export.argtypes = [ctypes.c_void_p] + [ctypes.c_void_p] * 7
        L.oracle_root_policy.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
        L.oracle_torch_sum.restype = ctypes.c_float
        L.oracle_torch_sum.argtypes = [ctypes.c_void_p, ctypes.c_int]
        L.oracle_feature_hash.restype = ctypes.c_uint64
        L.oracle_feature_hash.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int]
        L.oracle_synth_eval.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
        L.oracle_begin_go.argtypes = [ctypes.c_void_p, ctypes.POINTER(OracleConfig), ctypes.c_void_p,
                                      ctypes.c_int, ctypes.c_int, ctypes.c_int, EVAL_FN,
                                      ctypes.c_void_p]
        L.oracle_search_go.argtypes = [ctypes.c_void_p, ctypes.POINTER(OracleConfig),
                                       ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                       EVAL_FN, ctypes.c_void_p, ctypes.POINTER(OracleResult)]
        L.oracle_actions.argtypes = [ctypes.c_void_p]
        L.oracle_reroot.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int]
        L.oracle_begin_chess.argtypes = [ctypes.c_void_p, ctypes.POINTER(OracleConfig), ctypes.c_void_p,
                                         ctypes.c_void_p, ctypes.c_int, EVAL_FN, ctypes.c_void_p]
        L.oracle_feature_hash_chess.restype = ctypes.c_uint64
        L.oracle_feature_hash_chess.argtypes = [ctypes.c_void_p]
        L.oracle_synth_eval_chess.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
        L.oracle_feature_hash_go.restype = ctypes.c_uint64
        L.oracle_feature_hash_go.argtypes = [ctypes.c_void_p, ctypes.c_int]
        L.oracle_synth_eval_go.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p,
                                           ctypes.c_void_p, ctypes.c_void_p]
        L.oracle_chess_from_fen.argtypes = [ctypes.c_char_p, ctypes.c_void_p]
        L.oracle_chess_from_fen960.argtypes = [ctypes.c_char_p, ctypes.c_void_p]
        L.oracle_chess_legal.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
        L.oracle_chess_play.argtypes = [ctypes.c_void_p, ctypes.c_int32]
        L.oracle_chess_terminal.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.POINTER(ctypes.c_int)]
        L.oracle_chess_same.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
        L.oracle_chess_action.argtypes = [ctypes.c_void_p, ctypes.c_int32]
        L.oracle_chess_move.argtypes = [ctypes.c_void_p, ctypes.c_int]
        L.oracle_chess_features.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
        L.oracle_go_key.restype = ctypes.c_uint64
        L.oracle_go_key.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int]
        L.oracle_go_legal_superko.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                              ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p]
        L.oracle_begin_go_sk.argtypes = [ctypes.c_void_p, ctypes.POINTER(OracleConfig), ctypes.c_void_p,
                                         ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p,
                                         ctypes.c_int, ctypes.c_int, EVAL_FN, ctypes.c_void_p]
        L.oracle_begin_go_rules.argtypes = [ctypes.c_void_p, ctypes.POINTER(OracleConfig), ctypes.c_void_p,
                                            ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p,
                                            ctypes.c_int, ctypes.c_int, ctypes.c_int, EVAL_FN, ctypes.c_void_p]
        L.oracle_go_play.restype = ctypes.c_int
        L.oracle_go_play.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                     ctypes.c_int, ctypes.c_void_p, ctypes.POINTER(ctypes.c_int)]
        L.oracle_go_legal.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                      ctypes.c_void_p]
        _lib = L
    return _lib


CHESS_POS = np.dtype([("sq", np.int8, 64), ("side", np.int8), ("castle", np.int8), ("ep", np.int8),
                      ("reps", np.int8), ("halfmove", np.int16), ("fullmove", np.int16),
                      ("c960", np.int8), ("rook_file", np.int8, 4), ("pad", np.int8, 3)])


def chess_from_fen(fen: str, chess960: bool = False) -> np.ndarray:
    """Oracle chess position record (chess_rules.h) from a FEN string."""
    p = np.zeros(1, CHESS_POS)
    fn = lib().oracle_chess_from_fen960 if chess960 else lib().oracle_chess_from_fen
    if fn(fen.encode(), p.ctypes.data) != 0:
        raise ValueError(f"bad FEN {fen!r}")
    return p[0]


def _pos_buf(p):
    return np.ascontiguousarray(np.array(p, dtype=CHESS_POS).reshape(1))


def chess_legal(p) -> np.ndarray:
    """Legal moves in the reference encoding (promotion << 12 | from << 6 | to), sorted."""
    b = _pos_buf(p)
    m = np.zeros(320, np.int32)
    n = lib().oracle_chess_legal(b.ctypes.data, m.ctypes.data)
    return np.sort(m[:n])


def chess_play(p, move: int) -> np.ndarray:
    b = _pos_buf(p)
    lib().oracle_chess_play(b.ctypes.data, int(move))
    return b[0]


def chess_terminal(p, reps: int = 1):
    b = _pos_buf(p)
    r = ctypes.c_int(0)
    t = lib().oracle_chess_terminal(b.ctypes.data, int(reps), ctypes.byref(r))
    return bool(t), int(r.value)


def chess_same(a, b) -> bool:
    x, y = _pos_buf(a), _pos_buf(b)
    return bool(lib().oracle_chess_same(x.ctypes.data, y.ctypes.data))


def chess_action(p, move: int) -> int:
    return int(lib().oracle_chess_action(_pos_buf(p).ctypes.data, int(move)))


def chess_move(p, action: int) -> int:
    return int(lib().oracle_chess_move(_pos_buf(p).ctypes.data, int(action)))


def go_play(board: np.ndarray, player: int, action: int, ko: int = -1):
    """Go move (go_rules.cpp): returns (new board, new ko point) or None when illegal."""
    b = np.ascontiguousarray(board, np.int8)
    n = b.shape[-1]
    out = np.zeros_like(b)
    k = ctypes.c_int(-1)
    ok = lib().oracle_go_play(b.ctypes.data, n, int(player), int(action), int(ko), out.ctypes.data,
                              ctypes.byref(k))
    return (out, k.value) if ok else None


def go_key(board: np.ndarray, ko: int = -1) -> int:
    """64-bit position key (stones + ko point) used by the superko rule."""
    b = np.ascontiguousarray(board, np.int8)
    return int(lib().oracle_go_key(b.ctypes.data, b.shape[-1], int(ko)))


def go_legal_superko(board: np.ndarray, player: int, ko: int, hist_keys) -> np.ndarray:
    b = np.ascontiguousarray(board, np.int8)
    n = b.shape[-1]
    h = np.ascontiguousarray(np.asarray(list(hist_keys), dtype=np.uint64).reshape(-1))
    if h.size == 0:
        h = np.zeros(1, np.uint64)
        nh = 0
    else:
        nh = h.size
    m = np.zeros(n * n + 1, np.uint8)
    lib().oracle_go_legal_superko(b.ctypes.data, n, int(player), int(ko), h.ctypes.data, nh, m.ctypes.data)
    return m.astype(bool)


def go_legal(board: np.ndarray, player: int, ko: int = -1) -> np.ndarray:
    """Legal-action mask [n*n + 1] (pass last) under the oracle's Go rules."""
    b = np.ascontiguousarray(board, np.int8)
    n = b.shape[-1]
    m = np.zeros(n * n + 1, np.uint8)
    lib().oracle_go_legal(b.ctypes.data, n, int(player), int(ko), m.ctypes.data)
    return m.astype(bool)


def c_synth_eval(features: np.ndarray, actions: int | None = None):
    f = np.ascontiguousarray(features, dtype=np.float32)
    B, planes = f.shape[0], f.shape[1]
    cells = int(np.prod(f.shape[2:]))
    A = cells if actions is None else actions
    pol = np.zeros((B, A), np.float32)
    val = np.zeros(B, np.float32)
    lib().oracle_synth_eval(B, planes, cells, A, f.ctypes.data, pol.ctypes.data, val.ctypes.data)
    return pol, val


def c_synth_eval_chess(features: np.ndarray):
    """Chess synthetic evaluator on 119-plane features [n, 119, 8, 8] -> (policy [n, 4672], value)."""
    f = np.ascontiguousarray(features, dtype=np.float32)
    B = f.shape[0]
    pol = np.zeros((B, 4672), np.float32)
    val = np.zeros(B, np.float32)
    lib().oracle_synth_eval_chess(B, f.ctypes.data, pol.ctypes.data, val.ctypes.data)
    return pol, val


def chess_features(hist) -> np.ndarray:
    """119 planes [119, 8, 8] from position records hist[0..7] (None where absent)."""
    bufs = [None if h is None else _pos_buf(h) for h in list(hist) + [None] * (8 - len(hist))]
    ptrs = (ctypes.c_void_p * 8)(*[None if b is None else b.ctypes.data for b in bufs])
    out = np.zeros((119, 8, 8), np.float32)
    lib().oracle_chess_features(ptrs, out.ctypes.data)
    return out


def c_synth_eval_go(features: np.ndarray):
    """Go synthetic evaluator on 17-plane features [n, 17, H, W] -> (policy [n, H*W+1], value)."""
    f = np.ascontiguousarray(features, dtype=np.float32)
    B = f.shape[0]
    cells = int(np.prod(f.shape[2:]))
    pol = np.zeros((B, cells + 1), np.float32)
    val = np.zeros(B, np.float32)
    lib().oracle_synth_eval_go(B, cells, cells + 1, f.ctypes.data, pol.ctypes.data, val.ctypes.data)
    return pol, val


@dataclass
class OracleTree:
    """Search result of the oracle: node arrays in creation order plus run statistics."""
    visits: np.ndarray
    value_sums: np.ndarray
    priors: np.ndarray
    virtual_loss: np.ndarray
    parent: np.ndarray
    action: np.ndarray
    terminal: np.ndarray
    policy: np.ndarray
    result: dict


def _go_hist(hist, n):
    h = np.asarray(hist, dtype=np.int8)
    if h.ndim == 2:
        h = np.concatenate([h[None], np.zeros((7, n, n), np.int8)])
    return np.ascontiguousarray(h.reshape(8, n, n))


class Oracle:
    """One oracle tree. ``evaluator`` is None (built-in synthetic) or a callable
    features[n,19,H,W] -> (policy[n,A], value[n])."""

    def __init__(self, max_nodes: int, board_size: int = 15):
        self._L = lib()
        self._t = self._L.oracle_tree_create(max_nodes, board_size)
        if not self._t:
            raise ValueError("oracle_tree_create failed")
        self.max_nodes = max_nodes
        self.board_size = board_size
        self.game = "gomoku"
        self._cb = None

    def __del__(self):
        try:
            if self._t:
                self._L.oracle_tree_destroy(self._t)
        except Exception:
            pass

    def _make_cb(self, evaluator):
        if evaluator is None:
            return EVAL_FN()
        H = self.board_size
        go = self.game == "go"
        A = H * H + (1 if go else 0)
        planes = 17 if go else PLANES
        if self.game == "chess":
            A, planes = 4672, 119

        def cb(_ctx, n, feat, pol, val):
            f = np.ctypeslib.as_array(feat, shape=(n, planes, H, H)).copy()
            p, v = evaluator(f)
            np.ctypeslib.as_array(pol, shape=(n, A))[:] = np.asarray(p, np.float32).reshape(n, A)
            np.ctypeslib.as_array(val, shape=(n,))[:] = np.asarray(v, np.float32).reshape(n)
        return EVAL_FN(cb)

    def config(self, sims, wave, c_puct=1.4, virtual_loss=1.0, enable_vl=True, max_depth=100):
        return OracleConfig(self.board_size, sims, wave, c_puct, virtual_loss, int(enable_vl),
                            self.max_nodes, max_depth)

    def begin_go(self, hist, to_move, cfg: OracleConfig, ko=-1, passes=0, evaluator=None,
                 superko=True, keys=(), cycle=False) -> int:
        """Go root: ``hist`` int8 [8, n, n] (hist[0] = the root position, hist[k] k plies
        earlier); a single [n, n] board means no earlier positions. With ``superko`` the moves that
        recreate a position key of ``keys`` (the game before the root) or of the path are
        refused."""
        self.game = "go"
        h = _go_hist(hist, self.board_size)
        self._cb = self._make_cb(evaluator)
        k = np.ascontiguousarray(np.asarray(list(keys), dtype=np.uint64).reshape(-1))
        self._board = (h, k)
        return self._L.oracle_begin_go_rules(self._t, ctypes.byref(cfg), h.ctypes.data, int(to_move),
                                             int(ko), int(passes), k.ctypes.data if k.size else None,
                                             int(k.size), int(bool(superko)), int(bool(cycle)),
                                             self._cb, None)

    def search_go(self, hist, to_move, sims, wave, ko=-1, passes=0, evaluator=None, superko=True,
                  keys=(), cycle=False, **kw) -> OracleTree:
        cfg = self.config(sims, wave, **kw)
        st = self.begin_go(hist, to_move, cfg, ko, passes, evaluator, superko, keys, cycle)
        done = 0
        while st == 0 and done < sims:
            w = min(wave, sims - done)
            st = self._L.oracle_wave(self._t, w)
            done += w
        return self.export()

    def begin_chess(self, root, cfg: OracleConfig, prior=(), evaluator=None) -> int:
        """Chess root: an oracle position record (``CHESS_POS``) and the game's earlier positions,
        most recent first."""
        self.game = "chess"
        r = _pos_buf(root)
        pr = np.ascontiguousarray(np.array(list(prior), dtype=CHESS_POS).reshape(-1))
        if pr.size == 0:
            pr = np.zeros(1, CHESS_POS)
            npr = 0
        else:
            npr = pr.size
        self._cb = self._make_cb(evaluator)
        self._board = (r, pr)
        return self._L.oracle_begin_chess(self._t, ctypes.byref(cfg), r.ctypes.data, pr.ctypes.data,
                                          npr, self._cb, None)

    def search_chess(self, root, sims, wave, prior=(), evaluator=None, **kw) -> OracleTree:
        cfg = self.config(sims, wave, **kw)
        st = self.begin_chess(root, cfg, prior, evaluator)
        done = 0
        while st == 0 and done < sims:
            w = min(wave, sims - done)
            st = self._L.oracle_wave(self._t, w)
            done += w
        return self.export()

    def reroot(self, action: int, keep: bool = False) -> int:
        """Between searches: the root child reached by ``action`` becomes the next search's root
        (carrying its visit count and value sum, or with ``keep`` its whole subtree). Returns the
        mode applied: 0 fresh, 1 carry, 2 kept subtree."""
        return self._L.oracle_reroot(self._t, int(action), 2 if keep else 1)

    def begin(self, board, cfg: OracleConfig, evaluator=None) -> int:
        self.game = "gomoku"
        b = np.ascontiguousarray(board, dtype=np.int8)
        self._cb = self._make_cb(evaluator)
        self._board = b
        return self._L.oracle_begin(self._t, ctypes.byref(cfg), b.ctypes.data, self._cb, None)

    def wave(self, w: int, root_noise=None, eps: float = 0.0) -> int:
        """One wave; ``root_noise`` (fp32 [actions]) replays a Dirichlet vector at the root."""
        if root_noise is not None:
            nz = np.ascontiguousarray(root_noise, np.float32)
            self._L.oracle_set_root_noise(self._t, eps, np.float32(1.0 - eps), nz.ctypes.data)
        return self._L.oracle_wave(self._t, w)

    def search(self, board, sims, wave, evaluator=None, **kw) -> OracleTree:
        self.game = "gomoku"
        cfg = self.config(sims, wave, **kw)
        b = np.ascontiguousarray(board, dtype=np.int8)
        self._cb = self._make_cb(evaluator)
        res = OracleResult()
        self._L.oracle_search(self._t, ctypes.byref(cfg), b.ctypes.data, self._cb, None,
                              ctypes.byref(res))
        return self.export()

    def export(self) -> OracleTree:
        res = OracleResult()
        self._L.oracle_get_result(self._t, ctypes.byref(res))
        n = res.num_nodes
        arr = dict(visits=np.zeros(n, np.int32), value_sums=np.zeros(n, np.float32),
                   priors=np.zeros(n, np.float32), virtual_loss=np.zeros(n, np.int32),
                   parent=np.zeros(n, np.int32), action=np.zeros(n, np.int32),
                   terminal=np.zeros(n, np.uint8))
        self._L.oracle_export(self._t, *[arr[k].ctypes.data for k in
                                         ("visits", "value_sums", "priors", "virtual_loss",
                                          "parent", "action", "terminal")])
        pol = np.zeros(self._L.oracle_actions(self._t), np.float64)
        self._L.oracle_root_policy(self._t, pol.ctypes.data)
        result = {f: getattr(res, f) for f, _ in OracleResult._fields_}
        return OracleTree(policy=pol, result=result, **arr)
