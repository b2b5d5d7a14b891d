"""B200-native wave-MCTS hot path of omoknuni_quantum.

Drop-in for the reference's ``MCTS(config, evaluator, game_interface).search()`` /
``MCTSConfig``: device-resident trees, warp-cooperative selection, prefix-scan expansion,
ordered backup, an on-device leaf queue, and a tcgen05 bf16 ResNet evaluator, all in
``libomq_b200.so`` (C ABI: include/omq_b200.h).
"""
from .mcts_config import GameType, MCTSConfig, create_optimized_config, create_performance_config  # noqa: F401

__all__ = ["MCTS", "MCTSConfig", "GameType", "SyntheticEvaluator", "ResNetEvaluator", "WaveEngine",
           "create_optimized_config", "create_performance_config"]


def __getattr__(name):  # torch-importing modules load lazily
    if name in ("MCTS", "SyntheticEvaluator"):
        from . import mcts
        return getattr(mcts, name)
    if name == "ResNetEvaluator":
        from .resnet import ResNetEvaluator
        return ResNetEvaluator
    if name == "WaveEngine":
        from .engine import WaveEngine
        return WaveEngine
    raise AttributeError(name)
