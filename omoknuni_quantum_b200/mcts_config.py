"""MCTSConfig - the reference's search configuration, import-compatible.

Mirrors ``MCTSConfig`` of the reference (python/mcts/core/mcts_config.py:16-285): the same field
names and defaults, so that code constructing a reference config constructs this one unchanged.
The fields the device search reads are declared explicitly below; every other reference field is
accepted, stored and returned as an attribute (``REFERENCE_FIELDS``) but does not change the
search (most of them tune reference-internal mechanisms - memory pools, stream counts, hybrid
back-ends, tactical boosts - that have no counterpart here).
"""
from __future__ import annotations

from dataclasses import dataclass, field, fields
from enum import IntEnum
from typing import Any, Dict, Optional


class GameType(IntEnum):
    """Same values as the reference's GameType (python/mcts/gpu/gpu_game_states.py:34-38)."""
    CHESS = 0
    GO = 1
    GOMOKU = 2


_DEFAULT_BOARD_SIZES = {GameType.CHESS: 8, GameType.GO: 19, GameType.GOMOKU: 15}

# Reference fields that are accepted for compatibility but not read by the device search.
REFERENCE_FIELDS: Dict[str, Any] = {
    "classical_only_mode": False,
    "enable_fast_ucb": True,
    "enable_multi_stream": True,
    "num_cuda_streams": 4,
    "stream_memory_pool_size": 256,
    "min_wave_size": 1024,
    "wave_min_size": 512,
    "wave_max_size": 1024,
    "wave_adaptive_sizing": True,
    "cpu_optimal_wave_size": 32,
    "cpu_threads_per_worker": None,
    "wave_target_sims_per_second": 100000,
    "wave_target_gpu_utilization": 0.95,
    "wave_num_pipelines": 3,
    "wave_prefetch_evaluations": True,
    "wave_memory_pool_mb": 1024,
    "enable_quantum": False,
    "memory_pool_size_mb": 4096,
    "tree_growth_factor": 2.0,
    "gc_threshold": 0.8,
    "use_gpu_tree_reuse": False,
    "tree_memory_fraction": 0.4,
    "buffer_memory_fraction": 0.3,
    "max_tree_nodes_per_worker": 800000,
    "use_tensor_cores": True,
    "enable_kernel_fusion": True,
    "gpu_memory_fraction": 0.9,
    "initial_capacity_factor": 0.5,
    "enable_memory_pooling": True,
    "enable_pinned_memory": True,
    "enable_async_evaluation": True,
    "enable_coalesced_access": True,
    "use_lazy_gpu_states": True,
    "initial_gpu_states_capacity": 10000,
    "gpu_states_growth_factor": 2.0,
    "use_parallel_mcts": False,
    "num_mcts_workers": 4,
    "worker_batch_size": 32,
    "initial_children_per_expansion": 8,
    "max_children_per_node": 50,
    "progressive_expansion_threshold": 5,
    "progressive_widening_constant": 10.0,
    "progressive_widening_exponent": 0.5,
    "initial_expansion_children": 8,
    "csr_max_actions": 225,
    "csr_use_sparse_operations": True,
    "use_blocked_csr_layout": True,
    "block_size": 128,
    "batch_size": 256,
    "inference_batch_size": 256,
    "tree_batch_size": 8,
    "gpu_batch_timeout": 0.020,
    "worker_batch_timeout": 0.050,
    "max_coordination_batch_size": 128,
    "training_batch_queue_size": 10,
    "target_sims_per_second": 100000,
    "cache_legal_moves": True,
    "cache_features": True,
    "use_zobrist_hashing": True,
    "subtree_reuse_min_visits": 10,
    "adaptive_tree_reuse": True,
    "tree_reuse_min_child_visits": 50,
    "tree_reuse_visit_ratio": 0.05,
    "tree_reuse_absolute_threshold": 200,
    "enable_efficient_tree_reuse": True,
    "tree_reuse_validation_level": 'minimal',
    "disable_tree_reuse_for_hybrid": False,
    "enable_debug_logging": False,
    "enable_state_pool_debug": False,
    "profile_gpu_kernels": False,
    "enable_tactical_boost": False,
    "tactical_boost_strength": 0.3,
    "tactical_boost_decay": 0.99,
    "gomoku_win_boost": 100.0,
    "gomoku_block_win_boost": 90.0,
    "gomoku_open_four_boost": 50.0,
    "gomoku_block_four_boost": 45.0,
    "gomoku_threat_base_boost": 40.0,
    "gomoku_threat_multiplier": 5.0,
    "gomoku_three_boost": 20.0,
    "gomoku_block_three_boost": 18.0,
    "gomoku_center_boost": 3.0,
    "gomoku_connection_boost": 2.0,
    "chess_capture_good_base": 10.0,
    "chess_capture_equal": 5.0,
    "chess_capture_bad": 2.0,
    "chess_check_boost": 8.0,
    "chess_check_capture_boost": 4.0,
    "chess_promotion_boost": 9.0,
    "chess_center_boost": 1.0,
    "chess_center_core_boost": 0.5,
    "chess_development_boost": 2.0,
    "chess_castling_boost": 6.0,
    "go_capture_boost": 15.0,
    "go_escape_boost": 12.0,
    "go_atari_boost": 10.0,
    "go_save_boost": 8.0,
    "go_territory_boost": 5.0,
    "go_connection_boost": 3.0,
    "go_eye_boost": 7.0,
    "go_corner_boost": 2.0,
    "use_cython_hybrid": False,
    "use_genuine_hybrid": False,
    "use_fixed_hybrid": True,
    "use_optimized_hybrid": False,
    "use_optimized_fixed_hybrid": False,
    "use_unified_memory": False,
    "use_cuda_streams": True,
    "enable_work_stealing": False,
    "hybrid_cpu_batch_size": 32,
    "hybrid_gpu_batch_size": 256,
    "hybrid_load_balance_interval": 100,
    "hybrid_target_gpu_utilization": 0.85,
    "hybrid_target_cpu_utilization": 0.75,
    "hybrid_pipeline_depth": 3,
    "hybrid_num_buffers": 3,
}


@dataclass
class MCTSConfig:
    # -- read by the device search (reference defaults) -----------------------------------------
    num_simulations: int = 10000
    c_puct: float = 1.414
    temperature: float = 1.0
    dirichlet_alpha: float = 0.3
    dirichlet_epsilon: float = 0.25
    max_depth: int = 100
    wave_size: Optional[int] = None
    max_wave_size: int = 1024
    wave_async_expansion: bool = True
    device: str = "cuda"
    backend: str = "gpu"
    game_type: Any = GameType.GOMOKU
    board_size: int = 15
    enable_virtual_loss: bool = True
    virtual_loss: float = 1.0
    max_tree_nodes: int = 2000000
    initial_tree_nodes: int = 100000
    enable_dynamic_allocation: bool = True
    enable_subtree_reuse: bool = True
    # B200 extension (not a reference field): with subtree reuse on, update_root keeps the chosen
    # child's whole subtree for the next search, as CSRTree.shift_root describes
    # (csr_tree.py:1020-1229) but the reference never reaches.
    keep_subtree: bool = False
    use_mixed_precision: bool = True
    use_cuda_graphs: bool = True
    # -- every other reference field ------------------------------------------------------------
    extra: Dict[str, Any] = field(default_factory=dict, repr=False)

    def __init__(self, **kwargs):
        known = {f.name for f in fields(self.__class__) if f.name != "extra"}
        for f in fields(self.__class__):
            if f.name == "extra":
                continue
            setattr(self, f.name, kwargs.pop(f.name, f.default))
        unknown = [k for k in kwargs if k not in REFERENCE_FIELDS]
        if unknown:
            raise TypeError(f"MCTSConfig got unexpected keyword argument(s) {unknown}")
        self.extra = dict(REFERENCE_FIELDS)
        self.extra.update(kwargs)
        del known
        self.__post_init__()

    def __getattr__(self, name):
        extra = self.__dict__.get("extra")
        if extra is not None and name in extra:
            return extra[name]
        raise AttributeError(name)

    def __post_init__(self):
        # mcts_config.py:262-270
        if self.backend not in ("gpu", "cpu", "hybrid"):
            raise ValueError(f"backend must be 'gpu', 'cpu', or 'hybrid', got '{self.backend}'")
        if isinstance(self.game_type, str):
            self.game_type = GameType[self.game_type.upper()]
        elif not isinstance(self.game_type, GameType):
            self.game_type = GameType(int(self.game_type))
        if self.board_size is None:
            self.board_size = _DEFAULT_BOARD_SIZES.get(self.game_type, 15)

    @property
    def tree_capacity(self) -> int:
        """Nodes per tree: the reference sizes its tree and state pool to initial_tree_nodes when
        dynamic allocation is on, else max_tree_nodes (mcts.py:627-629, 674-676)."""
        return int(self.initial_tree_nodes if self.enable_dynamic_allocation else self.max_tree_nodes)

    def to_dict(self) -> Dict[str, Any]:
        d = {f.name: getattr(self, f.name) for f in fields(self.__class__) if f.name != "extra"}
        d.update(self.extra)
        return d


def create_optimized_config(game_type=GameType.GOMOKU, num_simulations: int = 10000,
                            device: str = "cuda", enable_quantum: bool = False, **kwargs) -> MCTSConfig:
    """mcts_config.py:287-310."""
    return MCTSConfig(game_type=game_type, num_simulations=num_simulations, device=device,
                      enable_quantum=enable_quantum, **kwargs)


def create_performance_config(wave_size: int = 3072, memory_pool_mb: int = 2048, **kwargs) -> MCTSConfig:
    """mcts_config.py:315-339: the reference's performance preset (its wave_size and pool size are
    reference tuning fields; the engine's wave is max_wave_size)."""
    return MCTSConfig(wave_size=wave_size, memory_pool_size_mb=memory_pool_mb, classical_only_mode=True,
                      enable_fast_ucb=True, use_mixed_precision=True, use_cuda_graphs=True,
                      use_tensor_cores=True, **kwargs)
