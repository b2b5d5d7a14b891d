"""Device-resident wave-MCTS engine: a set of independent trees searched in lockstep.

Python holds a handle and torch tensors for inputs/outputs; every step runs in
libomq_b200.so on the current CUDA stream. One engine = one device.

The evaluator between the select/expand/backup phases is one of
  * ``"synthetic"`` - the built-in integer-exact synthetic evaluator kernel;
  * an object with ``forward_queue(engine, queue)`` (the device ResNet evaluator of this
    package, which reads the queue in place and writes the queue's policy/value buffers);
  * any object with the reference evaluator protocol
    ``evaluate_batch(features[B,planes,H,W]) -> (policy[B,A] probabilities, value[B] or [B,1])``
    (python/mcts/core/wave_search.py:866-871, 1381-1383); features are handed over as a CUDA
    fp32 tensor, results are copied into the queue buffers.

Games: ``"gomoku"`` (A = n*n, the reference's 19 feature planes), ``"go"`` (A = n*n + 1 with
pass last, 17 history planes; roots carry 8 history boards, the side to move, the ko point and
the consecutive-pass count - see ``go_meta``) and ``"chess"`` (board 8, A = 4672 in the mover's
frame, 119 planes; roots are position records with the game's earlier positions - see
``omoknuni_quantum_b200.chess``).
"""
from __future__ import annotations

import ctypes

import numpy as np
import torch

from . import _lib

PLANES = 19
GO_PLANES = 17
GO_HISTORY = 8


def go_meta(to_move, ko=None, passes=None, num_trees=None) -> torch.Tensor:
    """int32 [R, 3] root records {side to move (1 black, 2 white), ko point (-1), passes}."""
    tm = torch.as_tensor(np.asarray(to_move, np.int32).reshape(-1))
    R = tm.numel() if num_trees is None else num_trees
    if tm.numel() == 1 and R > 1:
        tm = tm.repeat(R)
    k = torch.full((R,), -1, dtype=torch.int32) if ko is None else torch.as_tensor(np.asarray(ko, np.int32).reshape(-1))
    p = torch.zeros(R, dtype=torch.int32) if passes is None else torch.as_tensor(np.asarray(passes, np.int32).reshape(-1))
    return torch.stack([tm.to(torch.int32), k.to(torch.int32), p.to(torch.int32)], dim=1).contiguous()


def _stream_ptr(stream=None) -> ctypes.c_void_p:
    s = stream if stream is not None else torch.cuda.current_stream()
    return ctypes.c_void_p(s.cuda_stream)


class WaveEngine:
    def __init__(self, num_trees: int, board_size: int = 15, capacity: int = 200000,
                 max_wave_size: int = 256, c_puct: float = 1.4, virtual_loss: float = 1.0,
                 enable_virtual_loss: bool = True, max_depth: int = 100, device=None,
                 dirichlet_alpha: float = 0.3, dirichlet_epsilon: float = 0.0, noise_seed: int = 0,
                 game: str = "gomoku", go_superko: bool = True, go_rules: str = "chinese"):
        if not torch.cuda.is_available():
            raise RuntimeError("WaveEngine needs a CUDA device (B200); there is no CPU fallback")
        dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.device = dev
        self.L = _lib.load()
        self.num_trees = int(num_trees)
        self.board_size = int(board_size)
        self.cells = self.board_size ** 2
        if game not in _lib.GAMES:
            raise ValueError(f"unknown game {game!r} (gomoku, go, chess)")
        if go_rules not in ("chinese", "japanese", "korean"):
            raise ValueError(f"unknown Go rules {go_rules!r}")
        self.game = game
        self.is_go = game == "go"
        self.is_chess = game == "chess"
        if self.is_chess and self.board_size != 8:
            raise ValueError("chess engines have board_size 8")
        self.actions = 4672 if self.is_chess else self.cells + (1 if self.is_go else 0)
        self.planes = GO_PLANES if self.is_go else 119 if self.is_chess else PLANES
        self.capacity = int(capacity)
        self.max_wave_size = int(max_wave_size)
        cfg = _lib.EngineConfig(self.num_trees, self.board_size, self.capacity, self.max_wave_size,
                                int(max_depth), float(c_puct), float(virtual_loss),
                                int(bool(enable_virtual_loss)), dev.index or 0,
                                float(dirichlet_alpha), float(dirichlet_epsilon),
                                int(noise_seed) & 0xFFFFFFFFFFFFFFFF, _lib.GAMES[game],
                                int(bool(go_superko) and go_rules == "chinese"),
                                int(go_rules in ("japanese", "korean")))
        self.cfg = cfg
        h = ctypes.c_void_p()
        with torch.cuda.device(dev):
            _lib.check(self.L.omq_engine_create(ctypes.byref(cfg), ctypes.byref(h)), "omq_engine_create")
        self._h = h
        self.queue_capacity = self.num_trees * self.max_wave_size
        self._graphs = {}
        self._features = None
        self._visits = torch.zeros(self.num_trees, self.actions, dtype=torch.int32, device=dev)
        self._root_nw = torch.zeros(self.num_trees, 2, dtype=torch.float32, device=dev)
        self._status = torch.zeros(self.num_trees, dtype=torch.int32, device=dev)
        self._nodes = torch.zeros(self.num_trees, dtype=torch.int32, device=dev)

    # -- lifetime ------------------------------------------------------------------------------
    def close(self):
        getattr(self, "_graphs", {}).clear()     # graphs point into the engine's memory
        if getattr(self, "_h", None) and self._h.value:
            self.L.omq_engine_destroy(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def memory_bytes(self) -> int:
        b = ctypes.c_uint64()
        _lib.check(self.L.omq_engine_memory(self._h, ctypes.byref(b)), "omq_engine_memory")
        return int(b.value)

    # -- queue access --------------------------------------------------------------------------
    def queue_buffers(self, queue: int):
        """(entries int32 [cap,2], policy fp32 [cap,A], value fp32 [cap], count int32 [1]) as
        tensors aliasing the engine's device memory."""
        e, p, v, c = (ctypes.c_void_p() for _ in range(4))
        cap = ctypes.c_int32()
        _lib.check(self.L.omq_queue_buffers(self._h, queue, ctypes.byref(e), ctypes.byref(p),
                                            ctypes.byref(v), ctypes.byref(c), ctypes.byref(cap)),
                   "omq_queue_buffers")
        n = cap.value
        return (_wrap(e.value, (n, 2), torch.int32, self.device),
                _wrap(p.value, (n, self.actions), torch.float32, self.device),
                _wrap(v.value, (n,), torch.float32, self.device),
                _wrap(c.value, (1,), torch.int32, self.device))

    def queue_count(self, queue: int) -> int:
        n = ctypes.c_int32()
        _lib.check(self.L.omq_queue_count(self._h, queue, ctypes.byref(n), _stream_ptr()), "omq_queue_count")
        return int(n.value)

    def queue_features(self, queue: int) -> torch.Tensor:
        """Feature tensor of the queued positions, fp32 [count, planes, n, n] (syncs)."""
        count = self.queue_count(queue)
        if self._features is None:
            self._features = torch.empty(self.queue_capacity, self.planes, self.board_size,
                                         self.board_size, dtype=torch.float32, device=self.device)
        _lib.check(self.L.omq_queue_features(self._h, queue, ctypes.c_void_p(self._features.data_ptr()),
                                             _stream_ptr()), "omq_queue_features")
        return self._features[:count]

    def evaluate_queue(self, queue: int, evaluator) -> None:
        if isinstance(evaluator, str):
            if evaluator != "synthetic":
                raise ValueError(f"unknown built-in evaluator {evaluator!r}")
            _lib.check(self.L.omq_queue_eval_synthetic(self._h, queue, _stream_ptr()),
                       "omq_queue_eval_synthetic")
            return
        if hasattr(evaluator, "forward_queue"):
            evaluator.forward_queue(self, queue)
            return
        feats = self.queue_features(queue)
        n = feats.shape[0]
        if n == 0:
            return
        policy, value = evaluator.evaluate_batch(feats)
        _, qp, qv, _ = self.queue_buffers(queue)
        qp[:n].copy_(torch.as_tensor(np.asarray(policy) if not torch.is_tensor(policy) else policy)
                     .reshape(n, self.actions).to(self.device, torch.float32))
        qv[:n].copy_(torch.as_tensor(np.asarray(value) if not torch.is_tensor(value) else value)
                     .reshape(n).to(self.device, torch.float32))

    # -- search phases -------------------------------------------------------------------------
    def _go_keys(self, keys):
        """Per-root superko keys (a list of uint64 arrays, or None) -> device [R, 512] + counts;
        a game with more keys keeps its most recent 512. A pair of device tensors (keys, counts)
        in that layout is used as it is."""
        R = self.num_trees
        if isinstance(keys, tuple) and len(keys) == 2 and torch.is_tensor(keys[0]):
            # (int64 [R, GO_MAX_KEYS], int32 [R]) already on the device (device self-play)
            k, cnt = keys
            if tuple(k.shape) != (R, _lib.GO_MAX_KEYS) or k.dtype != torch.int64 or tuple(cnt.shape) != (R,) \
                    or cnt.dtype != torch.int32 or not k.is_contiguous() or not cnt.is_contiguous():
                raise ValueError(f"Go keys on the device must be int64 [{R}, {_lib.GO_MAX_KEYS}] and int32 [{R}]")
            return k.to(self.device), cnt.to(self.device)
        k = torch.zeros(R, _lib.GO_MAX_KEYS, dtype=torch.int64)
        cnt = torch.zeros(R, dtype=torch.int32)
        if keys is not None:
            for r, kr in enumerate(keys):
                a = np.asarray(kr, dtype=np.uint64).reshape(-1)[-_lib.GO_MAX_KEYS:]
                k[r, : a.size] = torch.from_numpy(a.view(np.int64))
                cnt[r] = a.size
        return k.to(self.device), cnt.to(self.device)

    def _go_roots(self, boards, meta):
        n, R = self.board_size, self.num_trees
        b = torch.as_tensor(boards).to(self.device, torch.int8)
        if b.dim() == 3:  # no earlier positions
            b = torch.cat([b[:, None], torch.zeros(R, GO_HISTORY - 1, n, n, dtype=torch.int8,
                                                  device=self.device)], dim=1)
        if tuple(b.shape) != (R, GO_HISTORY, n, n):
            raise ValueError(f"Go roots must be [{R}, {GO_HISTORY}, {n}, {n}] (or [{R}, {n}, {n}])")
        if meta is None:
            raise ValueError("Go roots need meta = go_meta(to_move, ko, passes)")
        m = torch.as_tensor(meta).to(self.device, torch.int32).reshape(R, 3).contiguous()
        return b.contiguous(), m

    def _chess_roots(self, records, nprior):
        """records: POS_DTYPE [R, 101] (numpy) or uint8 [R, 101*80]; nprior int32 [R]."""
        R = self.num_trees
        if isinstance(records, np.ndarray) and records.dtype.names:
            records = np.ascontiguousarray(records).view(np.uint8).reshape(R, -1)
        b = torch.as_tensor(records).to(self.device, torch.uint8).reshape(R, -1).contiguous()
        if b.shape[1] != 101 * 80:
            raise ValueError("chess roots must be 101 position records of 80 bytes per tree")
        if nprior is None:
            raise ValueError("chess roots need meta = the number of earlier positions per tree")
        m = torch.as_tensor(np.asarray(nprior, np.int32) if not torch.is_tensor(nprior) else nprior)
        m = m.to(self.device, torch.int32).reshape(R).contiguous()
        return b, m

    def begin(self, boards: torch.Tensor, meta=None, keys=None) -> None:
        if self.is_chess:
            b, m = self._chess_roots(boards, meta)
            self._boards, self._meta = b, m
            _lib.check(self.L.omq_begin_chess(self._h, ctypes.c_void_p(b.data_ptr()),
                                              ctypes.c_void_p(m.data_ptr()), _stream_ptr()), "omq_begin_chess")
            return
        if self.is_go:
            b, m = self._go_roots(boards, meta)
            k, kc = self._go_keys(keys)
            self._boards, self._meta, self._keys = b, m, (k, kc)
            _lib.check(self.L.omq_begin_go(self._h, ctypes.c_void_p(b.data_ptr()),
                                           ctypes.c_void_p(m.data_ptr()), ctypes.c_void_p(k.data_ptr()),
                                           ctypes.c_void_p(kc.data_ptr()), _stream_ptr()), "omq_begin_go")
            return
        b = boards.to(self.device, torch.int8).contiguous()
        if b.shape != (self.num_trees, self.board_size, self.board_size):
            raise ValueError(f"boards must be [{self.num_trees}, {self.board_size}, {self.board_size}]")
        self._boards = b
        _lib.check(self.L.omq_begin(self._h, ctypes.c_void_p(b.data_ptr()), _stream_ptr()), "omq_begin")

    def reroot(self, actions, keep: bool = False) -> None:
        """Between searches: make each tree's root child reached by ``actions[r]`` (-1: none) the
        next search's root; the next ``begin`` / ``search`` must start from the positions those
        moves lead to. ``keep=False`` starts a fresh tree whose root has the child's visit count
        and value sum (the reference's use_gpu_tree_reuse behaviour); ``keep=True`` keeps the
        child's whole subtree (omq_reroot, OMQ_REROOT_KEEP)."""
        a = torch.as_tensor(np.asarray(actions, np.int32) if not torch.is_tensor(actions) else actions)
        a = a.to(self.device, torch.int32).reshape(self.num_trees).contiguous()
        self._reroot_actions = a
        _lib.check(self.L.omq_reroot(self._h, ctypes.c_void_p(a.data_ptr()),
                                     _lib.REROOT_KEEP if keep else _lib.REROOT_CARRY, _stream_ptr()),
                   "omq_reroot")

    def root_expand(self, evaluator="synthetic") -> None:
        self.evaluate_queue(_lib.QUEUE_EXPAND, evaluator)
        _lib.check(self.L.omq_root_expand(self._h, _stream_ptr()), "omq_root_expand")

    def wave(self, wave_size: int, evaluator="synthetic") -> None:
        s = _stream_ptr()
        _lib.check(self.L.omq_wave_select(self._h, int(wave_size), s), "omq_wave_select")
        self.evaluate_queue(_lib.QUEUE_EXPAND, evaluator)
        _lib.check(self.L.omq_wave_expand(self._h, s), "omq_wave_expand")
        self.evaluate_queue(_lib.QUEUE_FINAL, evaluator)
        _lib.check(self.L.omq_wave_backup(self._h, s), "omq_wave_backup")

    def _wave_graph(self, w: int, evaluator):
        """CUDA graph of one wave of size w with an on-device evaluator (captured on first use;
        keyed by the evaluator and its buffer generation, so a re-created net is recaptured)."""
        key = (w, id(evaluator), getattr(evaluator, "generation", 0))
        ent = self._graphs.get(key)
        if ent is None:
            for k in [k for k in self._graphs if k[:2] == key[:2]]:
                del self._graphs[k]                # captured against an earlier net
            n0 = _lib.kernel_launches()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                self.wave(w, evaluator)
            n = _lib.kernel_launches() - n0
            _lib.add_kernel_launches(-n)          # recorded, not run
            ent = self._graphs[key] = (g, n, evaluator)
        return ent

    def search(self, boards: torch.Tensor, num_simulations: int, evaluator="synthetic",
               meta=None, keys=None, graphs: bool = False) -> None:
        """begin + forced root expansion + ceil(sims / max_wave_size) waves
        (python/mcts/core/mcts.py:1020-1063). Raises on a device status (e.g. TreeFullError).
        Go engines take history boards and ``meta`` (see ``begin``)."""
        synthetic = isinstance(evaluator, str) and evaluator == "synthetic"
        native_net = getattr(evaluator, "_net", None) if hasattr(evaluator, "forward_queue") else None
        graphed = (graphs and native_net is not None and not getattr(evaluator, "profiling", False))
        if synthetic or (native_net is not None and not graphed):
            # one native call: begin, root expansion and every wave, evaluations on the device
            # leaf queues (omq_search*, the C-ABI counterpart of MCTS._run_search)
            net = None
            if not synthetic:
                evaluator._ensure(self.queue_capacity)
                net = evaluator._net
            sims, st = int(num_simulations), _stream_ptr()
            if self.is_chess:
                b, m = self._chess_roots(boards, meta)
                self._boards, self._meta = b, m
                _lib.check(self.L.omq_search_chess(self._h, net, ctypes.c_void_p(b.data_ptr()),
                                                   ctypes.c_void_p(m.data_ptr()), sims, st), "omq_search_chess")
            elif self.is_go:
                b, m = self._go_roots(boards, meta)
                k, kc = self._go_keys(keys)
                self._boards, self._meta, self._keys = b, m, (k, kc)
                _lib.check(self.L.omq_search_go(self._h, net, ctypes.c_void_p(b.data_ptr()),
                                                ctypes.c_void_p(m.data_ptr()), ctypes.c_void_p(k.data_ptr()),
                                                ctypes.c_void_p(kc.data_ptr()), sims, st), "omq_search_go")
            else:
                b = boards.to(self.device, torch.int8).contiguous()
                if b.shape != (self.num_trees, self.board_size, self.board_size):
                    raise ValueError(f"boards must be [{self.num_trees}, {self.board_size}, {self.board_size}]")
                self._boards = b
                _lib.check(self.L.omq_search(self._h, net, ctypes.c_void_p(b.data_ptr()), sims, st), "omq_search")
            return
        self.begin(boards, meta, keys)
        self.root_expand(evaluator)
        # full-size waves replay a CUDA graph when asked (MCTSConfig.use_cuda_graphs) and the
        # evaluator runs on the device queue (no host round trip inside a wave)
        done = 0
        while done < num_simulations:
            w = min(self.max_wave_size, num_simulations - done)
            if graphed and w == self.max_wave_size:
                if hasattr(evaluator, "_ensure"):
                    evaluator._ensure(self.queue_capacity)
                g, n, _ = self._wave_graph(w, evaluator)
                g.replay()
                _lib.add_kernel_launches(n)
            else:
                self.wave(w, evaluator)
            done += w
        self.check_status()

    # -- readouts ------------------------------------------------------------------------------
    def tree_status(self):
        _lib.check(self.L.omq_tree_status(self._h, ctypes.c_void_p(self._status.data_ptr()),
                                          ctypes.c_void_p(self._nodes.data_ptr()), _stream_ptr()),
                   "omq_tree_status")
        return self._status, self._nodes

    def check_status(self) -> None:
        st, nodes = self.tree_status()
        st = st.cpu().numpy()
        bad = np.nonzero(st)[0]
        if len(bad):
            r = int(bad[0])
            code = int(st[r])
            msg = f"tree {r}: {int(nodes[r])} nodes of {self.capacity}"
            if code == _lib.OMQ_TREE_FULL:
                raise _lib.TreeFullError(code, f"Tree full: {msg}")
            raise _lib.OmqError(code, f"device status {code} in {msg}")

    def root_visits(self) -> torch.Tensor:
        """int32 [num_trees, actions]: root-child visit counts scattered by action."""
        _lib.check(self.L.omq_root_visits(self._h, ctypes.c_void_p(self._visits.data_ptr()),
                                          ctypes.c_void_p(self._root_nw.data_ptr()), _stream_ptr()),
                   "omq_root_visits")
        return self._visits

    def root_noise(self) -> torch.Tensor:
        """fp32 [num_trees, actions]: the Dirichlet noise mixed into each root's priors by the last
        wave (zeros when the noise is off)."""
        out = torch.zeros(self.num_trees, self.actions, dtype=torch.float32, device=self.device)
        _lib.check(self.L.omq_root_noise(self._h, ctypes.c_void_p(out.data_ptr()), _stream_ptr()),
                   "omq_root_noise")
        return out

    def root_nw(self) -> torch.Tensor:
        self.root_visits()
        return self._root_nw

    def num_nodes(self) -> torch.Tensor:
        return self.tree_status()[1]

    def export_tree(self, tree: int) -> dict:
        """Node arrays of one tree in creation order (numpy, host)."""
        n = int(self.num_nodes()[tree])
        d = self.device
        out = dict(visits=torch.empty(n, dtype=torch.int32, device=d),
                   value_sums=torch.empty(n, dtype=torch.float32, device=d),
                   priors=torch.empty(n, dtype=torch.float32, device=d),
                   virtual_loss=torch.empty(n, dtype=torch.int32, device=d),
                   parent=torch.empty(n, dtype=torch.int32, device=d),
                   action=torch.empty(n, dtype=torch.int32, device=d),
                   terminal=torch.empty(n, dtype=torch.uint8, device=d))
        ptr = [ctypes.c_void_p(out[k].data_ptr()) for k in
               ("visits", "value_sums", "priors", "virtual_loss", "parent", "action", "terminal")]
        _lib.check(self.L.omq_export_tree(self._h, int(tree), n, *ptr, _stream_ptr()), "omq_export_tree")
        return {k: v.cpu().numpy() for k, v in out.items()}

    @staticmethod
    def policy_from_visits(visits: np.ndarray) -> np.ndarray:
        """N_child / sum N_child in fp64 (python/mcts/core/mcts.py:1069-1137)."""
        v = np.asarray(visits)
        squeeze = v.ndim == 1
        v = np.atleast_2d(v).astype(np.float64)
        tot = v.sum(axis=1, keepdims=True)
        pol = np.where(tot > 0, v / np.where(tot > 0, tot, 1.0), 1.0 / v.shape[1])
        return pol[0] if squeeze else pol


def _wrap(ptr: int, shape, dtype, device) -> torch.Tensor:
    """A tensor view of engine-owned device memory (no copy, no ownership)."""
    n = int(np.prod(shape))
    if n == 0:
        return torch.empty(shape, dtype=dtype, device=device)
    itemsize = torch.empty((), dtype=dtype).element_size()
    t = torch.as_tensor(_DeviceBuffer(ptr, n * itemsize), device=device)
    return t.view(dtype).reshape(shape)


class _DeviceBuffer:
    """Minimal __cuda_array_interface__ exporter for a raw device pointer (uint8 bytes)."""

    def __init__(self, ptr: int, nbytes: int):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1",
                                         "data": (ptr, False), "version": 3, "strides": None}
