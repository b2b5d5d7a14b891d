"""ctypes binding of libomq_b200.so (the C ABI declared in include/omq_b200.h).

The shared library is the only compute path: if it is missing or fails to load, every entry
point raises. There is no CPU or PyTorch fallback.
"""
from __future__ import annotations

import ctypes
import os

from .build_ext import LIB

OMQ_OK = 0
OMQ_TREE_FULL = 1
OMQ_QUEUE_OVERFLOW = 2
OMQ_TIMEOUT = 3
OMQ_BAD_ARG = 4
OMQ_CUDA_ERROR = 5
OMQ_NOT_READY = 6

QUEUE_EXPAND = 0
QUEUE_FINAL = 1


class OmqError(RuntimeError):
    """A non-OK status from the native library."""

    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status


class TreeFullError(OmqError):
    """Capacity exhausted (the reference raises RuntimeError("Tree full: ...") here)."""


class EngineConfig(ctypes.Structure):
    _fields_ = [("num_trees", ctypes.c_int32), ("board_size", ctypes.c_int32),
                ("capacity", ctypes.c_int32), ("max_wave_size", ctypes.c_int32),
                ("max_depth", ctypes.c_int32), ("c_puct", ctypes.c_float),
                ("virtual_loss", ctypes.c_float), ("enable_virtual_loss", ctypes.c_int32),
                ("device", ctypes.c_int32), ("dirichlet_alpha", ctypes.c_float),
                ("dirichlet_epsilon", ctypes.c_float), ("noise_seed", ctypes.c_uint64),
                ("game", ctypes.c_int32), ("go_superko", ctypes.c_int32), ("go_cycle", ctypes.c_int32)]


GO_MAX_KEYS = 512   # OMQ_GO_MAX_KEYS
GAME_GOMOKU = 0
GAME_GO = 1
GAME_CHESS = 2
GAMES = {"gomoku": GAME_GOMOKU, "go": GAME_GO, "chess": GAME_CHESS}
REROOT_CARRY = 1    # OMQ_REROOT_CARRY
REROOT_KEEP = 2     # OMQ_REROOT_KEEP


class ResNetConfig(ctypes.Structure):
    _fields_ = [("board_size", ctypes.c_int32), ("input_channels", ctypes.c_int32),
                ("num_blocks", ctypes.c_int32), ("filters", ctypes.c_int32),
                ("num_actions", ctypes.c_int32), ("fc_policy_hidden", ctypes.c_int32),
                ("fc_value_hidden", ctypes.c_int32), ("max_batch", ctypes.c_int32),
                ("device", ctypes.c_int32), ("dtype", ctypes.c_int32), ("trunk_per_layer", ctypes.c_int32)]


OMQ_DTYPE_BF16, OMQ_DTYPE_F16 = 0, 1


class SelfplayStepConfig(ctypes.Structure):
    _fields_ = [("move_number", ctypes.c_int32), ("max_moves", ctypes.c_int32),
                ("temperature_threshold", ctypes.c_int32), ("temperature", ctypes.c_float),
                ("enable_resign", ctypes.c_int32), ("resign_min_move", ctypes.c_int32),
                ("resign_threshold", ctypes.c_float), ("seed", ctypes.c_uint64)]


_P = ctypes.c_void_p
_I = ctypes.c_int32

# name -> argtypes (every function returns int status unless listed in _RESTYPES)
SIGNATURES = {
    "omq_status_string": [ctypes.c_int],
    "omq_last_error": [],
    "omq_engine_create": [ctypes.POINTER(EngineConfig), ctypes.POINTER(_P)],
    "omq_engine_destroy": [_P],
    "omq_engine_memory": [_P, ctypes.POINTER(ctypes.c_uint64)],
    "omq_begin": [_P, _P, _P],
    "omq_begin_go": [_P, _P, _P, _P, _P, _P],
    "omq_begin_chess": [_P, _P, _P, _P],
    "omq_root_expand": [_P, _P],
    "omq_reroot": [_P, _P, _I, _P],
    "omq_wave_select": [_P, _I, _P],
    "omq_wave_expand": [_P, _P],
    "omq_wave_backup": [_P, _P],
    "omq_queue_buffers": [_P, _I, ctypes.POINTER(_P), ctypes.POINTER(_P), ctypes.POINTER(_P),
                          ctypes.POINTER(_P), ctypes.POINTER(_I)],
    "omq_queue_count": [_P, _I, ctypes.POINTER(_I), _P],
    "omq_queue_features": [_P, _I, _P, _P],
    "omq_queue_eval_synthetic": [_P, _I, _P],
    "omq_search_synthetic": [_P, _P, _I, _P],
    "omq_search": [_P, _P, _P, _I, _P],
    "omq_search_go": [_P, _P, _P, _P, _P, _P, _I, _P],
    "omq_search_chess": [_P, _P, _P, _P, _I, _P],
    "omq_search_synthetic_go": [_P, _P, _P, _P, _P, _I, _P],
    "omq_search_synthetic_chess": [_P, _P, _P, _I, _P],
    "omq_root_visits": [_P, _P, _P, _P],
    "omq_tree_status": [_P, _P, _P, _P],
    "omq_root_noise": [_P, _P, _P],
    "omq_export_tree": [_P, _I, _I, _P, _P, _P, _P, _P, _P, _P, _P],
    "omq_resnet_create": [ctypes.POINTER(ResNetConfig), ctypes.POINTER(_P)],
    "omq_resnet_destroy": [_P],
    "omq_resnet_memory": [_P, ctypes.POINTER(ctypes.c_uint64)],
    "omq_resnet_trunk_launches": [_P, ctypes.POINTER(ctypes.c_int32)],
    "omq_resnet_param_sizes": [_P, ctypes.POINTER(ctypes.c_uint64), ctypes.POINTER(ctypes.c_uint64),
                               ctypes.POINTER(ctypes.c_uint64)],
    "omq_resnet_load": [_P, _P, _P, _P, _P],
    "omq_resnet_forward_features": [_P, _P, _I, _P, _P, _P],
    "omq_resnet_forward_packed": [_P, _P, _P, _I, _P, _P, _P],
    "omq_resnet_input_buffer": [_P, ctypes.POINTER(_P)],
    "omq_resnet_forward_queue": [_P, _P, _I, _P],
    "omq_resnet_error": [_P, ctypes.POINTER(_I), _P],
    "omq_resnet_profile": [_P, _I],
    "omq_resnet_profile_read": [_P, ctypes.POINTER(_I), _P, _P, _I],
    "omq_kernel_launches": [ctypes.POINTER(ctypes.c_uint64)],
    "omq_kernel_launches_add": [ctypes.c_int64],
    "omq_abi_struct_sizes": [ctypes.POINTER(ctypes.c_uint32), ctypes.POINTER(ctypes.c_uint32)],
    "omq_selftest_wait_timeout": [ctypes.c_uint64, _P, _P],
    "omq_selftest_prior_sum": [_P, _P, _I, _P, _P],
    "omq_selfplay_move": [_P, ctypes.POINTER(SelfplayStepConfig), _P, _P, _P, _P, _P, _P, _P, _P],
    "omq_selfplay_move_chess": [_P, ctypes.POINTER(SelfplayStepConfig), _P, _P, _P, _P, _P, _P, _P, _P, _P],
    "omq_selfplay_move_go": [_P, ctypes.POINTER(SelfplayStepConfig), ctypes.c_float, ctypes.c_int32, _P, _P, _P,
                             _P, _P, _P, _P, _P, _P, _P, _P],
    "omq_resnet_forward_noalloc": [ctypes.POINTER(ResNetConfig), _P, _P, _P, _P, _I, _P, _P, _P],
    "omq_resnet_noalloc_error": [_I, ctypes.POINTER(_I), _P],
}
_RESTYPES = {"omq_status_string": ctypes.c_char_p, "omq_last_error": ctypes.c_char_p}

_lib = None


def lib_path() -> str:
    return LIB


def load(build_if_missing: bool = True):
    """Load the native library (building it with nvcc first when it is absent)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB):
        if not build_if_missing:
            raise OSError(f"libomq_b200.so not found at {LIB}; run "
                          "`python -m omoknuni_quantum_b200.build_ext`")
        from .build_ext import build
        build()
    L = ctypes.CDLL(LIB)
    for name, args in SIGNATURES.items():
        fn = getattr(L, name)
        fn.argtypes = args
        fn.restype = _RESTYPES.get(name, ctypes.c_int)
    _lib = L
    return L


def add_kernel_launches(delta: int) -> None:
    check(load().omq_kernel_launches_add(int(delta)), "omq_kernel_launches_add")


def kernel_launches() -> int:
    """Kernels launched by libomq_b200.so in this process so far."""
    n = ctypes.c_uint64()
    check(load().omq_kernel_launches(ctypes.byref(n)), "omq_kernel_launches")
    return int(n.value)


def check(status: int, what: str = "") -> None:
    if status == OMQ_OK:
        return
    L = load()
    detail = (L.omq_last_error() or b"").decode(errors="replace")
    name = (L.omq_status_string(status) or b"").decode()
    msg = f"{what}: {name}" + (f" ({detail})" if detail else "")
    if status == OMQ_TREE_FULL:
        raise TreeFullError(status, "Tree full: " + msg)
    raise OmqError(status, msg)
