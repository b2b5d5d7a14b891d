"""Time the unmodified reference (staged by baseline/stage_reference.py under baseline/_ref) through
its own public API: MCTS(MCTSConfig, evaluator).search(board) (python/mcts/core/mcts.py:924),
with its own ResNetModel under its own ResNetEvaluator (resnet_evaluator.py:80-265).

    python baseline/run_reference.py --mode cpu|cython|gpu [--sims 1600] [--wave 256] ...

Modes (one JSON line on stdout):
  cpu     the deterministic torch WaveSearch path on the host (backend='gpu', device='cpu',
          wave_async_expansion=False; wave_search.py:555) with the fp32 ResNet on all host cores;
  cython  the CPU backend (backend='cpu': OptimizedCPUWaveSearch + the Cython tree,
          optimized_wave_search.py:27-491, cython_tree_optimized.pyx), its ResNet on the host;
          nondeterministic (its tree is lock-free multithreaded), so it is a speed figure only;
  gpu     the default CUDA path, AsyncWaveSearch (backend='gpu', device='cuda',
          wave_async_expansion=True; async_wave_search.py:414-1172) with the mcts_cuda_kernels
          extension built from mcts_kernels.cu, and its ResNet under its fp16 autocast on cuda:0.
Roots are the bench's seeded roots (omoknuni_quantum_b200.roots.random_roots(seed * 1000, n)),
weights the bench's seeded ResNet (loaded into the reference ResNetModel), so both arms search
the same positions with the same network. Whole searches are timed; `--budget` seconds bound
the number of roots searched (at least one search always completes).
"""
from __future__ import annotations

import argparse
import json
import logging
import os
import sys
import time

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
REF = os.path.join(HERE, "_ref")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--mode", choices=["cpu", "cython", "gpu"], required=True)
    ap.add_argument("--sims", type=int, default=1600)
    ap.add_argument("--wave", type=int, default=256)
    ap.add_argument("--capacity", type=int, default=400000)
    ap.add_argument("--blocks", type=int, default=10)
    ap.add_argument("--filters", type=int, default=128)
    ap.add_argument("--value-hidden", type=int, default=128)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--roots", type=int, default=256, help="roots of the seeded set to draw from")
    ap.add_argument("--first-root", type=int, default=0)
    ap.add_argument("--budget", type=float, default=20.0, help="seconds; stop after the search that passes it")
    ap.add_argument("--warmup", type=int, default=1,
                    help="untimed searches first (of one wave each on the host, full searches on the GPU)")
    ap.add_argument("--threads", type=int, default=0, help="host threads (0: all)")
    a = ap.parse_args()
    if not os.path.isdir(os.path.join(REF, "mcts")):
        print(json.dumps({"unavailable": "the reference is not staged (python baseline/stage_reference.py)"}))
        return
    sys.dont_write_bytecode = True
    sys.path.insert(0, REPO)
    sys.path.insert(0, REF)
    logging.disable(logging.WARNING)
    os.chdir(REF)  # the reference's cuda_manager looks for build_cuda_shared/ under the working directory
    import numpy as np
    import torch
    threads = a.threads or os.cpu_count() or 1
    torch.set_num_threads(threads)
    from mcts.core.evaluator import EvaluatorConfig
    from mcts.core.mcts import MCTS
    from mcts.core.mcts_config import MCTSConfig
    from mcts.gpu.gpu_game_states import GameType
    from mcts.neural_networks.resnet_evaluator import ResNetEvaluator
    from mcts.neural_networks.resnet_model import ResNetConfig, ResNetModel
    from omoknuni_quantum_b200.resnet import ResNetSpec, init_state_dict
    from omoknuni_quantum_b200.roots import random_roots

    dev = "cuda" if a.mode == "gpu" else "cpu"
    spec = ResNetSpec(num_blocks=a.blocks, filters=a.filters, fc_value_hidden=a.value_hidden)
    model = ResNetModel(ResNetConfig(num_blocks=a.blocks, num_filters=a.filters, input_channels=19,
                                     fc_value_hidden=a.value_hidden, fc_policy_hidden=256),
                        board_size=15, num_actions=225, game_type="gomoku")
    model.load_state_dict(init_state_dict(spec, seed=a.seed))
    model = model.to(dev).eval()
    ev = ResNetEvaluator(model=model, config=EvaluatorConfig(batch_size=max(64, a.wave), device=dev),
                         game_type="gomoku", device=dev)
    common = dict(num_simulations=a.sims, max_wave_size=a.wave, c_puct=1.4, virtual_loss=1.0,
                  dirichlet_epsilon=0.0, enable_subtree_reuse=False, board_size=15,
                  max_tree_nodes=a.capacity, initial_tree_nodes=a.capacity)
    if a.mode == "cpu":
        cfg = MCTSConfig(backend="gpu", device="cpu", wave_async_expansion=False, game_type=GameType.GOMOKU,
                         use_mixed_precision=False, **common)
    elif a.mode == "cython":
        cfg = MCTSConfig(backend="cpu", device="cpu", game_type=GameType.GOMOKU, use_mixed_precision=False,
                         **common)
    else:
        # wave_size set explicitly: AsyncWaveSearch compares it with an int at construction
        # (async_wave_search.py:1195), and MCTSConfig's default for it is None
        cfg = MCTSConfig(backend="gpu", device="cuda", wave_async_expansion=True, game_type=GameType.GOMOKU,
                         wave_size=a.wave, **common)
    mcts = MCTS(cfg, ev)
    roots = random_roots(a.seed * 1000, a.roots)
    kind = type(mcts.wave_search).__name__ if hasattr(mcts, "wave_search") else "?"
    async_error = None
    if a.mode == "gpu" and kind != "AsyncWaveSearch":
        # the reference fell back to its synchronous WaveSearch (mcts.py:524-534): record why
        try:
            from mcts.core.async_wave_search import AsyncWaveSearch
            AsyncWaveSearch(tree=mcts.tree, game_states=mcts.game_states, evaluator=mcts.evaluator,
                            config=cfg, device=mcts.device)
            async_error = "constructed on retry"
        except Exception as e:  # the message the reference logs and swallows
            async_error = f"{type(e).__name__}: {e}"[:300]

    def sync():
        if dev == "cuda":
            torch.cuda.synchronize()

    for i in range(a.warmup):
        mcts.search(roots[i % a.roots].copy(), num_simulations=a.sims if dev == "cuda" else a.wave)
    sync()
    done, searches, times = 0, 0, []
    t0 = time.perf_counter()
    r = a.first_root
    while True:
        t1 = time.perf_counter()
        pol = mcts.search(roots[r % a.roots].copy())
        sync()
        times.append(time.perf_counter() - t1)
        assert np.isclose(float(np.sum(pol)), 1.0, atol=1e-3)
        done += a.sims
        searches += 1
        r += 1
        if time.perf_counter() - t0 >= a.budget:
            break
    secs = time.perf_counter() - t0
    out = {"mode": a.mode, "sims_per_s": done / secs, "searches": searches, "sims": done, "seconds": secs,
           "ms_per_search": 1000.0 * secs / searches, "threads": threads if dev == "cpu" else None,
           "wave_search": kind, "first_root": a.first_root, "device": dev}
    if async_error:
        out["async_wave_search_error"] = async_error
    if dev == "cuda":
        from mcts.gpu import cuda_manager
        k = cuda_manager.detect_cuda_kernels()
        out["cuda_kernels"] = k is not None
        out["gpu"] = torch.cuda.get_device_name(0)
    print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()
