#!/usr/bin/env python
"""Benchmark of the wave-MCTS hot path: MCTS simulations/s on B200 (device-timed, whole box).

Workload (benchmark config 1, one GPU): Gomoku 15x15 single-tree searches, 1600 simulations per
root, max_wave_size 256, c_puct 1.4, virtual loss 1.0, ResNet evaluator 10 blocks x 128 filters
(value head FC 225 -> 128 -> 1), bf16 weights/activations with fp32 accumulation, seeded He-init
weights. Roots: 20 stones placed uniformly at random, colours alternating, from a seed. Each GPU
searches `--roots` independent roots in lockstep (the on-device leaf queue batches their leaves
into one ResNet call per phase); one step = one complete search of every root. Multi-GPU: one
process per GPU, roots sharded (weak scaling), weights broadcast once over NCCL, no per-wave
collective.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

Prints one JSON line (rank 0). `--impl reference` times the reference algorithm's CPU path on the
host cores (the C++ restatement in oracle/ of the reference's torch WaveSearch, with the ResNet
forward in fp32 torch on the CPU) on a bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np
import torch

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

METRIC = "MCTS simulations/sec (device-timed, whole box)"
UNIT = "simulations/s"
WORKLOAD_GO = ("config3: Go 19x19 (captures, no suicide, simple ko, positional superko, pass), 3200 sims/root, wave 512, "
               "1M-node trees, ResNet 20x256 bf16 on 17 history planes, 362 actions; 256 roots sharded "
               "across GPUs, searched in lockstep")
WORKLOAD_CHESS = ("config4: chess (the reference engine's rules), 1600 sims/root, wave 256, 500k-node "
                  "trees, ResNet 20x256 bf16 on 119 history planes, 4672 actions (8x8x73); 1024 roots "
                  "from 10-40 random plies, sharded across GPUs, searched in lockstep")
WORKLOAD = ("config1: Gomoku 15x15 single-tree searches, 1600 sims/root, wave 256, c_puct 1.4, "
            "VL 1.0, ResNet 10x128 bf16 evaluator; independent roots searched in lockstep per GPU")


def parse():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--roots", type=int, default=256, help="roots per GPU searched in lockstep")
    ap.add_argument("--sims", type=int, default=1600)
    ap.add_argument("--wave", type=int, default=256)
    ap.add_argument("--capacity", type=int, default=400000, help="tree nodes per root")
    ap.add_argument("--blocks", type=int, default=10)
    ap.add_argument("--filters", type=int, default=128)
    ap.add_argument("--value-hidden", type=int, default=128)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--cpu-seconds", type=float, default=20.0, help="CPU baseline sample budget")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-extra-configs", action="store_true",
                    help="config 1 only (by default the line also carries configs 2-4, one timed step each)")
    ap.add_argument("--workload", choices=["config1", "config2", "config3", "config4", "forward"], default="config1",
                    help="forward = ResNet leaf evaluations/s alone (--game, --batch, --blocks, --filters); "
                         "config2 = batched self-play: 512 games (sharded), 800 sims, wave 64, 20x256; "
                         "config3 = Go 19x19: 256 roots (sharded), 3200 sims, wave 512, 1M nodes, 20x256; "
                         "config4 = chess: 1024 roots (sharded), 1600 sims, wave 256, 500k nodes, 20x256")
    ap.add_argument("--game", choices=["gomoku", "go", "chess"], default="gomoku",
                    help="board shape of --workload forward")
    ap.add_argument("--batch", type=int, default=4096, help="positions per call of --workload forward")
    ap.add_argument("--dtype", choices=["bf16", "fp16"], default="bf16",
                    help="16-bit type of the ResNet (bf16: the benchmark configs' type)")
    ap.add_argument("--evaluator", choices=["resnet", "synthetic"], default="resnet",
                    help="synthetic = benchmark config 0 (tree kernels only; 800 sims, 200k nodes)")
    return ap.parse_args()


# ---------------------------------------------------------------------------------------------
# helpers
# ---------------------------------------------------------------------------------------------
def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def measured_peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return d, "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def profile_value(name: str, key: str):
    """A number recorded in a committed ncu summary under profiles/ ('key: value' line)."""
    path = os.path.join(REPO, "profiles", name)
    if not os.path.exists(path):
        return None
    with open(path) as f:
        for line in f:
            line = line.strip().lstrip("-* ")
            if line.startswith(key + ":"):
                try:
                    return float(line.split(":", 1)[1].split()[0].replace(",", ""))
                except ValueError:
                    return None
    return None


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.proc = None
        self.file = None

    def __enter__(self):
        try:
            self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=self.file, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        return False

    def summary(self):
        if self.proc is None or self.file is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.file.flush()
        with open(self.file.name) as f:
            rows = [r.strip().split(", ") for r in f if r.strip()]
        os.unlink(self.file.name)
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            if len(r) < 9:
                continue
            try:
                sm.append(float(r[1]))
                mx.append(float(r[2]))
            except ValueError:
                continue
            for n, v in zip(names, r[5:9]):
                if v.strip() == "Active":
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        busy = [s for s in sm if s > 0.5 * max(sm)] or sm
        return {"sm_mhz": statistics.median(busy), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


def config1_config(args, ws):
    """The `config` of config-1 lines: the same dict in the B200 arm and the reference arm."""
    return {"workload": WORKLOAD, "roots_per_gpu": args.roots, "global_batch": args.roots * ws,
            "sims": args.sims, "wave": args.wave, "capacity": args.capacity,
            "model": f"resnet{args.blocks}x{args.filters} (value fc {args.value_hidden})",
            "parallelism": f"dp{ws} (independent trees per GPU, weights NCCL-broadcast once)",
            "l2": "inputs larger than L2 (multi-GB activations per ResNet call)"}


def run_reference_script(args, mode, budget, timeout, extra=()):
    """baseline/run_reference.py in a child process: the unmodified reference (staged under
    baseline/_ref) through its own MCTS(config, evaluator).search, on the bench's seeded roots and
    weights. Returns its JSON result, or {"unavailable": reason}."""
    cmd = [sys.executable, os.path.join(REPO, "baseline", "run_reference.py"), "--mode", mode,
           "--sims", str(args.sims), "--wave", str(args.wave), "--capacity", str(args.capacity),
           "--blocks", str(args.blocks), "--filters", str(args.filters),
           "--value-hidden", str(args.value_hidden), "--seed", str(args.seed), "--roots", str(args.roots),
           "--budget", str(budget), *extra]
    try:
        out = subprocess.run(cmd, capture_output=True, text=True, timeout=timeout)
    except subprocess.TimeoutExpired:
        return {"unavailable": f"reference {mode} run exceeded {timeout} s"}
    for line in reversed(out.stdout.strip().splitlines()):
        if line.startswith("{"):
            return json.loads(line)
    tail = (out.stderr or out.stdout).strip().splitlines()[-1:] or ["no output"]
    return {"unavailable": f"reference {mode} run failed (rc {out.returncode}): {tail[0][:200]}"}


def make_spec(args):
    from omoknuni_quantum_b200.resnet import ResNetSpec
    if args.workload == "config4":
        return ResNetSpec(board_size=8, input_channels=119, num_blocks=args.blocks,
                          filters=args.filters, num_actions=4672, fc_policy_hidden=256,
                          fc_value_hidden=args.value_hidden)
    if args.workload == "config3":
        return ResNetSpec(board_size=19, input_channels=17, num_blocks=args.blocks,
                          filters=args.filters, num_actions=362, fc_policy_hidden=256,
                          fc_value_hidden=args.value_hidden)
    return ResNetSpec(board_size=15, input_channels=19, num_blocks=args.blocks, filters=args.filters,
                      num_actions=225, fc_policy_hidden=256, fc_value_hidden=args.value_hidden)


def apply_config4(args):
    """benchmark config 4: chess, 1600 sims per root, wave 256, 500k-node trees, ResNet 20x256 on
    119 planes with a 4672-way policy; 1024 roots (10-40 random plies) sharded across the GPUs."""
    args.sims, args.wave, args.capacity = 1600, 256, 500_000
    args.blocks, args.filters, args.value_hidden = 20, 256, 256
    if args.roots == 256:
        args.roots = 1024


def apply_config3(args):
    """benchmark config 3: Go 19x19, 3200 sims per root, wave 512, 1M-node trees, ResNet 20x256
    (value FC 361 -> 256 -> 1); 256 roots sharded across the GPUs."""
    args.sims, args.wave, args.capacity = 3200, 512, 1_000_000
    args.blocks, args.filters, args.value_hidden = 20, 256, 256


# ---------------------------------------------------------------------------------------------
# CPU arms
# ---------------------------------------------------------------------------------------------
def cpu_search_rate(args, sd, budget_s: float, game: str = "gomoku", first_root: int = 0):
    """The reference algorithm on the host as the oracle port runs it: the oracle's C++ tree
    search (restatement of the reference's torch WaveSearch) + the fp32 torch ResNet forward on
    all host cores. Whole searches of the bench's seeded roots (root first_root, first_root + 1,
    ...) until `budget_s` has passed (at least one); returns (sims/s, sims, seconds, threads,
    searches)."""
    from oracle import pyoracle
    from omoknuni_quantum_b200 import go as gomod
    from omoknuni_quantum_b200.resnet import reference_forward_fp32
    from omoknuni_quantum_b200.roots import random_roots
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    sd32 = {k: v.float() for k, v in sd.items()}

    def ev(f):
        with torch.no_grad():
            p, v = reference_forward_fp32(sd32, torch.from_numpy(f))
        return p.numpy(), v.numpy()

    gomoku_roots = random_roots(args.seed * 1000, max(args.roots, first_root + 1)) if game == "gomoku" else None
    sims_done, searches, t0 = 0, 0, time.perf_counter()
    r = first_root
    while True:
        if game == "chess":
            from omoknuni_quantum_b200 import chess as chessmod
            o = pyoracle.Oracle(args.capacity, 8)
            cfg = o.config(args.sims, args.wave)
            cp = chessmod.random_position(args.seed * 1_000_003 + r)
            st = o.begin_chess(cp.record(), cfg, prior=cp.prior, evaluator=ev)
        elif game == "go":
            o = pyoracle.Oracle(args.capacity, 19)
            cfg = o.config(args.sims, args.wave)
            g = gomod.random_position(args.seed * 1_000_003 + r, 60, 19)
            st = o.begin_go(g.history_planes(), g.to_move, cfg, ko=g.ko, passes=g.passes, evaluator=ev)
        else:
            o = pyoracle.Oracle(args.capacity)
            cfg = o.config(args.sims, args.wave)
            st = o.begin(gomoku_roots[r % len(gomoku_roots)], cfg, evaluator=ev)
        if st != 0:
            raise RuntimeError("oracle begin failed")
        done = 0
        while done < args.sims:
            w = min(args.wave, args.sims - done)
            if o.wave(w) != 0:
                raise RuntimeError("oracle wave failed")
            done += w
        sims_done += args.sims
        searches += 1
        r += 1
        if time.perf_counter() - t0 > budget_s:
            break
    dt = time.perf_counter() - t0
    return sims_done / dt, sims_done, dt, threads, searches


def run_reference_arm(args):
    """`--impl reference`: the reference's own implementation of the path on this box's host
    cores, on the B200 arm's workload and config. For config 1 that is the unmodified reference
    (baseline/_ref) searching through its own MCTS.search with its deterministic torch
    WaveSearch and its fp32 ResNet: whole searches of the bench's seeded roots within a bounded
    time (the headline, kind "reference"); beside it the oracle port (the same algorithm as a C++
    restatement) and the reference's Cython CPU backend. Configs 3-4 have no reference search
    (the reference's Go and chess wave search use placeholder rules), so the port is their
    reference arm (kind "port"). One step = 1/K of the timed sample."""
    ws, rank, _ = dist_env()
    if rank != 0:
        return
    from omoknuni_quantum_b200.resnet import init_state_dict
    game = {"config3": "go", "config4": "chess"}.get(args.workload, "gomoku")
    if game == "go":
        apply_config3(args)
    if game == "chess":
        apply_config4(args)
    sd = init_state_dict(make_spec(args), seed=args.seed)
    budget = max(2.0, args.cpu_seconds)
    ref = None
    if game == "gomoku":
        ref = run_reference_script(args, "cpu", budget, timeout=max(900, 20 * budget),
                                   extra=("--warmup", str(max(1, min(args.warmup, 1)))))
    baselines = {}
    if ref is not None and "unavailable" not in ref:
        value, secs, sims = ref["sims_per_s"], ref["seconds"], ref["sims"]
        threads, kind = ref["threads"], "reference"
        sample = (f"{ref['searches']} whole {args.sims}-simulation searches (wave {args.wave}) of the bench's seeded "
                  f"roots by the unmodified reference ({ref['wave_search']}, device cpu, its fp32 ResNetModel "
                  f"{args.blocks}x{args.filters} under its ResNetEvaluator) in {secs:.1f} s")
        rate, psims, psecs, pthreads, psearch = cpu_search_rate(args, sd, max(2.0, args.cpu_seconds / 2), game)
        baselines["oracle_port"] = {"value": rate, "unit": UNIT, "cores": pthreads, "kind": "port",
                                    "sample": f"{psearch} whole searches ({psims} simulations) in {psecs:.1f} s: "
                                              "oracle C++ tree + fp32 torch CPU ResNet"}
        cy = run_reference_script(args, "cython", max(2.0, args.cpu_seconds / 2), timeout=900)
        if "unavailable" in cy:
            baselines["reference_cython"] = cy
        else:
            baselines["reference_cython"] = {
                "value": cy["sims_per_s"], "unit": UNIT, "cores": cy["threads"], "kind": "reference",
                "nondeterministic": True,
                "sample": f"{cy['searches']} whole searches in {cy['seconds']:.1f} s by the reference's CPU backend "
                          f"({cy['wave_search']} + Cython tree), fp32 ResNet on the host"}
    else:
        if ref is not None:
            baselines["reference_torch_cpu"] = ref      # why the reference itself could not run
        value, sims, secs, threads, searches = cpu_search_rate(args, sd, budget, game)
        kind = "port"
        sample = (f"{searches} whole searches ({sims} simulations) of {args.workload} in {secs:.1f} s: oracle C++ "
                  f"tree{' with the ' + game + ' rules' if game != 'gomoku' else ''} + fp32 torch CPU ResNet "
                  f"{args.blocks}x{args.filters}")
    if game == "gomoku":
        config = config1_config(args, ws)
    else:
        config = {"workload": {"go": WORKLOAD_GO, "chess": WORKLOAD_CHESS}[game], "sims": args.sims,
                  "wave": args.wave, "model": f"resnet{args.blocks}x{args.filters}", "parallelism": "host threads"}
    line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": 1000.0 * secs / max(1, args.steps),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded roots, seeded He-init weights)", "impl": "reference",
            "config": config,
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": kind, "sample": sample},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "baselines": baselines}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------------------------
# B200 arm
# ---------------------------------------------------------------------------------------------
def run_b200(args):
    ws, rank, local = dist_env()
    if not torch.cuda.is_available():
        raise SystemExit("bench.py --impl b200 needs a CUDA device")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if ws > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=dev)
    from omoknuni_quantum_b200 import _lib, parallel
    from omoknuni_quantum_b200.engine import WaveEngine
    from omoknuni_quantum_b200.mcts import MCTS
    from omoknuni_quantum_b200.mcts_config import MCTSConfig
    from omoknuni_quantum_b200.resnet import ResNetEvaluator, init_state_dict
    from omoknuni_quantum_b200.roots import random_roots

    spec = make_spec(args)
    # weights: rank 0's seeded weights, broadcast once over NCCL (the only data collective)
    sd = parallel.broadcast_state_dict(init_state_dict(spec, seed=args.seed), dev)
    R = args.roots
    ev = ResNetEvaluator(sd, board_size=15, max_batch=R * args.wave, device=dev)
    roots = torch.from_numpy(random_roots(args.seed * 1000 + rank, R)).to(dev)
    eng = WaveEngine(R, board_size=15, capacity=args.capacity, max_wave_size=args.wave, c_puct=1.4,
                     virtual_loss=1.0, device=dev)

    def barrier():
        if ws > 1:
            import torch.distributed as dist
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        eng.search(roots, args.sims, evaluator=ev)
    barrier()
    ev.profile(1 << 14)
    launches0 = _lib.kernel_launches()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        barrier()
        start.record()
        for _ in range(args.steps):
            eng.search(roots, args.sims, evaluator=ev)
        end.record()
        barrier()
    launches = _lib.kernel_launches() - launches0
    ms = start.elapsed_time(end)
    trunk_ms, counts = ev.profile_read()
    ev.profile(0)
    ms_max = parallel.max_over_ranks(ms, dev)
    total_sims = args.sims * R * args.steps * ws
    value = total_sims / (ms_max / 1000.0)
    positions = int(parallel.sum_over_ranks(int(counts.sum()), dev)) // ws  # per-rank mean
    nodes = int(eng.num_nodes().max())

    # roofline of the dominant kernel (the tcgen05 conv): algorithmic FLOPs per launch / avg launch
    peaks, peak_kind = measured_peaks()
    conv_launches = len(trunk_ms) * ev.conv_launches_per_call
    flops = positions * ev.trunk_flops_per_position()
    avg_launch_s = float(trunk_ms.sum()) / 1000.0 / max(1, conv_launches)
    achieved = (flops / max(1, conv_launches)) / avg_launch_s / 1e12 if avg_launch_s > 0 else 0.0
    peak = float(peaks.get("bf16_tflops_sustained", peaks.get("bf16_tflops")))
    fused = ev.fused_trunk
    # DRAM bytes per position per launch from the committed ncu capture of the kernel that ran
    traffic_per_pos = (profile_value("trunk_resnet10x128.md", "dram_bytes_per_position_per_launch") if fused
                       else profile_value("conv3x3_resnet10x128.md", "dram_bytes_per_position_per_launch"))
    traffic = None
    if traffic_per_pos is not None and len(trunk_ms):
        traffic = traffic_per_pos * positions / len(trunk_ms)  # every launch covers all of a call's positions
    kernel_name = ("k_trunk_t (the whole 21-conv trunk per launch: every conv of a position in one CTA, tcgen05 "
                   "128 ch x 240 px UMMAs over one halo load per channel block, activations in an L2-resident "
                   "per-CTA scratch)" if fused else
                   "k_conv3x3_halo_t (tcgen05 implicit-GEMM 3x3 conv, 128 ch x 256 px UMMAs over one halo "
                   "load per channel block)")
    roofline = {"kernel": kernel_name,
                "bound": "tensor",
                "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
                "peak_kind": f"bf16_tflops_sustained of {peak_kind}", "traffic": traffic,
                "algorithmic_flops_per_launch": flops / max(1, conv_launches),
                "avg_launch_ms": avg_launch_s * 1e3, "launches": conv_launches}

    # end to end through the public API: host boards (pinned) in, host policies out
    e2e, mcts, m1 = None, None, None
    if not args.no_e2e:
        cfg = MCTSConfig(num_simulations=args.sims, max_wave_size=args.wave, c_puct=1.4,
                         virtual_loss=1.0, initial_tree_nodes=args.capacity, device=str(dev),
                         enable_subtree_reuse=False, dirichlet_epsilon=0.0)
        mcts = MCTS(cfg, ev)
        mcts._engines[R] = eng
        host_boards = roots.cpu().pin_memory()
        mcts.search_batch(host_boards)
        barrier()
        s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s2.record()
        for _ in range(args.steps):
            pol = mcts.search_batch(host_boards)
        e2.record()
        barrier()
        ms2 = parallel.max_over_ranks(s2.elapsed_time(e2), dev)
        assert pol.shape == (R, 225) and np.allclose(pol.sum(1), 1.0)
        e2e = {"value": total_sims / (ms2 / 1000.0), "unit": UNIT,
               "h2d_bytes_per_step": R * 225, "d2h_bytes_per_step": R * 225 * 4,
               "api": "MCTS(config, ResNetEvaluator).search_batch(pinned host boards) -> numpy policies"}

    # single-tree latency through the public API (one root per MCTS.search call, as the
    # reference's own users call it), and the reference's default CUDA search path on this GPU
    single, ref_gpu = None, None
    if rank == 0 and ws == 1 and not args.no_e2e:
        cfg1 = MCTSConfig(num_simulations=args.sims, max_wave_size=args.wave, c_puct=1.4, virtual_loss=1.0,
                          initial_tree_nodes=args.capacity, device=str(dev), enable_subtree_reuse=False,
                          dirichlet_epsilon=0.0)
        m1 = MCTS(cfg1, ev)
        host_roots = roots.cpu().numpy()
        for i in range(3):
            m1.search(host_roots[i])
        torch.cuda.synchronize()
        n1 = min(R, 32)
        s3, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s3.record()
        for i in range(n1):
            p1 = m1.search(host_roots[i])
        e3.record()
        torch.cuda.synchronize()
        assert np.isclose(p1.sum(), 1.0)
        ms1 = s3.elapsed_time(e3) / n1
        single = {"ms_per_search": ms1, "value": args.sims / (ms1 / 1000.0), "unit": UNIT, "searches": n1,
                  "api": "MCTS(config, ResNetEvaluator).search(host board), one root per call"}
        # AsyncWaveSearch sizes its own waves (at least 1024 simulations, async_wave_search.py:449-459)
        # and so allocates more nodes than the requested simulations need: 1M-node trees
        r = run_reference_script(args, "gpu", 10.0, timeout=600, extra=("--warmup", "2", "--capacity", "1000000"))
        ref_gpu = r if "unavailable" in r else {
            "ms_per_search": r["ms_per_search"], "value": r["sims_per_s"], "unit": UNIT, "searches": r["searches"],
            "wave_search": r["wave_search"], "cuda_kernels": r["cuda_kernels"],
            "api": "unmodified reference MCTS(MCTSConfig(backend='gpu', device='cuda', wave_async_expansion=True), "
                   "its ResNetEvaluator under fp16 autocast).search(board), one root per call, mcts_kernels.cu "
                   "built for sm_100"}

    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        rate, sims, secs, threads, searches = cpu_search_rate(args, sd, args.cpu_seconds)
        cpu = {"value": rate, "unit": UNIT, "cores": threads, "kind": "port",
               "sample": f"{searches} whole config-1 searches ({sims} simulations) of the bench's roots in "
                         f"{secs:.1f} s (oracle C++ tree + fp32 torch CPU ResNet 10x128)"}

    # configs 2-4 on the same GPUs: one warm-up and one timed step each, after config 1's
    # buffers are freed (their own lines come from --workload config2|3|4)
    extra = None
    if not args.no_extra_configs:
        for m in (mcts, m1):
            if m is not None:
                for e in m._engines.values():
                    if e is not eng:
                        e.close()
                m._engines.clear()
        ev.close()
        eng.close()
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
        extra = run_extra_configs(args)

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": ws, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_max / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded roots, seeded He-init weights)",
            "config": config1_config(args, ws),
            "leaf_evals_per_s": positions * ws / (ms_max / 1000.0),
            "max_tree_nodes": nodes,
            "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e, "clocks": clk.summary(),
            "gpu_launches": launches,
            "single_root_search": single, "reference_cuda_same_box": ref_gpu,
            "other_configs": extra,
        }
        print(json.dumps(line), flush=True)
    if ws > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()


def run_extra_configs(args):
    """Config 0 (20 single-tree searches) and configs 2, 3 and 4 with one warm-up and one timed
    step each (the default bench line's `other_configs`): the same code as --evaluator synthetic
    and --workload config2|config3|config4, without the e2e and CPU legs. Runs on every rank (the
    timings are maxima over ranks)."""
    import copy
    out = {}
    # config 0: one tree, 800 simulations, wave 256, the synthetic evaluator (the tree kernels
    # alone), 20 timed searches; 400k nodes, since the stated 100k overflows the reference's own
    # full expansion (about 160k nodes per search)
    a = copy.copy(args)
    a.roots, a.sims, a.wave, a.capacity, a.steps, a.warmup = 1, 800, 256, 400000, 20, 3
    line = run_b200_synthetic(a, inner=True)
    torch.cuda.synchronize()
    out["config0"] = {"value": line["value"], "unit": line["unit"], "ms_per_step": line["ms_per_step"],
                      "steps": line["steps"], "warmup": line["warmup"], "scaling": line["scaling"],
                      "config": line["config"], "clocks": line.get("clocks"),
                      "gpu_launches": line.get("gpu_launches")}
    for name, fn in (("config2", lambda a: run_b200_selfplay(a, inner=True)),
                     ("config3", lambda a: run_b200_go(a, "go", inner=True)),
                     ("config4", lambda a: run_b200_go(a, "chess", inner=True))):
        a = copy.copy(args)
        a.workload, a.steps, a.warmup, a.no_e2e, a.no_cpu_baseline = name, 1, 1, True, True
        a.roots = 256                       # the configs' own root counts are set by apply_config3/4
        line = fn(a)
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
        if line is None:
            continue
        rf = line.get("roofline") or {}
        out[name] = {"value": line["value"], "unit": line["unit"], "ms_per_step": line["ms_per_step"],
                     "steps": line["steps"], "warmup": line["warmup"], "scaling": line["scaling"],
                     "config": line["config"], "leaf_evals_per_s": line.get("leaf_evals_per_s"),
                     "roofline_frac": rf.get("frac"), "roofline_achieved_tflops": rf.get("achieved"),
                     "moves_per_s": line.get("moves_per_s"),
                     "clocks": line.get("clocks"), "gpu_launches": line.get("gpu_launches")}
    return out


def run_b200_synthetic(args, inner=False):
    """benchmark config 0 on the device: the integer-exact synthetic evaluator, so the step is the
    tree kernels alone (select, expand, backup, evaluation kernel)."""
    from omoknuni_quantum_b200 import _lib, parallel
    from omoknuni_quantum_b200.engine import WaveEngine
    from omoknuni_quantum_b200.roots import random_roots
    ws, rank, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if ws > 1:
        init_dist(dev)
    R = args.roots
    roots = torch.from_numpy(random_roots(args.seed * 1000 + rank, R)).to(dev)
    eng = WaveEngine(R, capacity=args.capacity, max_wave_size=args.wave, device=dev)
    for _ in range(args.warmup):
        eng.search(roots, args.sims)
    torch.cuda.synchronize()
    n0 = _lib.kernel_launches()
    s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        s0.record()
        for _ in range(args.steps):
            eng.search(roots, args.sims)
        s1.record()
        torch.cuda.synchronize()
    ms = parallel.max_over_ranks(s0.elapsed_time(s1), dev)
    eng.close()
    if inner or rank == 0:
        line = {
            "metric": METRIC, "value": args.sims * R * args.steps * ws / (ms / 1000.0), "unit": UNIT,
            "n_gpus": ws, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32/int32",
            "data": "synthetic (seeded roots, integer-exact synthetic evaluator)",
            "config": {"workload": f"config0: Gomoku 15x15, {args.sims} sims/root, wave {args.wave}, "
                                   "synthetic evaluator; roots searched in lockstep per GPU",
                       "roots_per_gpu": R, "capacity": args.capacity, "parallelism": f"dp{ws}"},
            "roofline": None, "cpu_baseline": None, "e2e": None, "clocks": clk.summary(),
            "gpu_launches": _lib.kernel_launches() - n0}
        if inner:
            return line
        print(json.dumps(line), flush=True)
    if ws > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


def init_dist(dev):
    """One process group per run (NCCL over NVLink between the box's GPUs)."""
    import torch.distributed as dist
    if not dist.is_initialized():
        dist.init_process_group("nccl", device_id=dev)


def run_b200_selfplay(args, inner=False):
    """benchmark config 2: 512 concurrent self-play games sharded over the ranks (total fixed),
    800 simulations per move, max_wave_size 64 (leaf batches up to games x 64), ResNet 20 x 256
    bf16; one step = one move of every game (temperature-1 sampling from the visit policy)."""
    from omoknuni_quantum_b200 import _lib, parallel
    from omoknuni_quantum_b200.resnet import ResNetEvaluator, ResNetSpec, init_state_dict
    from omoknuni_quantum_b200.selfplay import BatchedSelfPlay
    ws, rank, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if ws > 1:
        init_dist(dev)
    games_total, sims, wave = 512, 800, 64
    shard = parallel.shard_range(games_total, ws, rank)
    G = len(shard)
    spec = ResNetSpec(num_blocks=20, filters=256, fc_value_hidden=128)
    sd = parallel.broadcast_state_dict(init_state_dict(spec, seed=args.seed), dev)
    ev = ResNetEvaluator(sd, max_batch=G * wave, device=dev)
    # moves drawn and played on the device (omq_selfplay_move): no host round trip per move
    sp = BatchedSelfPlay(G, num_simulations=sims, wave_size=wave, evaluator=ev, capacity=200000,
                         temperature=1.0, temperature_threshold=30, seed=args.seed * 1000 + rank,
                         device=dev, sampling="device", max_moves=args.warmup + args.steps + 1)
    for _ in range(args.warmup):
        sp.step()
    torch.cuda.synchronize()
    ev.profile(1 << 14)
    n0 = _lib.kernel_launches()
    s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        if ws > 1:
            import torch.distributed as dist
            dist.barrier()
        s0.record()
        moved = 0
        for _ in range(args.steps):
            moved += sp.step()
        s1.record()
        torch.cuda.synchronize()
    ms = parallel.max_over_ranks(s0.elapsed_time(s1), dev)
    total_moves = parallel.sum_over_ranks(moved, dev)
    trunk_ms, counts = ev.profile_read()
    peaks, kind = measured_peaks()
    launches = len(trunk_ms) * ev.conv_launches_per_call
    flops = int(counts.sum()) * ev.trunk_flops_per_position()
    # DRAM bytes per launch from the committed capture of this kernel on 15x15 boards
    per_pos = profile_value("conv3x3_halot256_resnet20x256.md", "dram_bytes_per_position_per_launch_gomoku")
    traffic = per_pos * int(counts.sum()) / len(trunk_ms) if per_pos is not None and len(trunk_ms) else None
    avg_s = float(trunk_ms.sum()) / 1000.0 / max(1, launches)
    achieved = flops / max(1, launches) / avg_s / 1e12 if avg_s > 0 else 0.0
    peak = float(peaks.get("bf16_tflops_sustained", peaks.get("bf16_tflops")))
    line = {
            "metric": METRIC, "value": total_moves * sims / (ms / 1000.0), "unit": UNIT, "n_gpus": ws,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (empty-board self-play, seeded sampling, seeded He-init weights)",
            "config": {"workload": "config2: batched Gomoku self-play, 512 games sharded across GPUs, "
                                   "800 sims/move, wave 64, ResNet 20x256 bf16; step = one move of every game, "
                                   "drawn and played on the device",
                       "games_per_gpu": G, "global_batch": games_total, "parallelism": f"dp{ws}"},
            "leaf_evals_per_s": int(counts.sum()) * ws / (ms / 1000.0),
            "moves_per_s": total_moves / (ms / 1000.0),
            "roofline": {"kernel": "k_conv3x3_halo_t (tcgen05 conv, two 128-channel halves of 256 filters)",
                         "bound": "tensor",
                         "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
                         "peak_kind": f"bf16_tflops_sustained of {kind}", "traffic": traffic},
            "cpu_baseline": None, "e2e": None, "clocks": clk.summary(),
            "gpu_launches": _lib.kernel_launches() - n0}
    ev.close()
    sp.close()
    if inner:
        return line
    if rank == 0:
        print(json.dumps(line), flush=True)
    if ws > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


def run_b200_go(args, game="go", inner=False):
    """Configs 3 and 4 on the device: Go roots (60 random legal moves each) or chess roots (10-40
    random plies), ResNet 20x256 evaluator."""
    ws, rank, local = dist_env()
    if not torch.cuda.is_available():
        raise SystemExit("bench.py --impl b200 needs a CUDA device")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if ws > 1:
        init_dist(dev)
    from omoknuni_quantum_b200 import _lib, parallel
    from omoknuni_quantum_b200 import go as gomod
    from omoknuni_quantum_b200.engine import WaveEngine
    from omoknuni_quantum_b200.mcts import MCTS
    from omoknuni_quantum_b200.mcts_config import GameType, MCTSConfig
    from omoknuni_quantum_b200.resnet import ResNetEvaluator, init_state_dict

    from omoknuni_quantum_b200 import chess as chessmod
    chess = game == "chess"
    (apply_config4 if chess else apply_config3)(args)
    n_board, n_act = (8, 4672) if chess else (19, 362)
    spec = make_spec(args)
    sd = parallel.broadcast_state_dict(init_state_dict(spec, seed=args.seed), dev)
    total_roots = args.roots
    R = total_roots // ws + (1 if rank < total_roots % ws else 0)
    first = sum(total_roots // ws + (1 if q < total_roots % ws else 0) for q in range(rank))
    if chess:
        positions_host = [chessmod.random_position(args.seed * 1_000_003 + first + i) for i in range(R)]
        hist = torch.from_numpy(np.stack([p.root_records() for p in positions_host]).view(np.uint8)
                                .reshape(R, -1)).to(dev)
        meta = torch.tensor([len(p.prior) for p in positions_host], dtype=torch.int32, device=dev)
    else:
        positions_host = [gomod.random_position(args.seed * 1_000_003 + first + i, 60, 19) for i in range(R)]
        hist = torch.from_numpy(np.stack([g.history_planes() for g in positions_host])).to(dev)
        meta = torch.from_numpy(np.stack([g.meta() for g in positions_host])).to(dev)
    keys = None if chess else [g.root_keys() for g in positions_host]
    ev = ResNetEvaluator(sd, board_size=n_board, max_batch=R * args.wave, device=dev)
    eng = WaveEngine(R, board_size=n_board, capacity=args.capacity, max_wave_size=args.wave, c_puct=1.4,
                     virtual_loss=1.0, device=dev, game=game)

    def barrier():
        if ws > 1:
            import torch.distributed as dist
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        eng.search(hist, args.sims, evaluator=ev, meta=meta, keys=keys)
    barrier()
    ev.profile(1 << 14)
    launches0 = _lib.kernel_launches()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        barrier()
        start.record()
        for _ in range(args.steps):
            eng.search(hist, args.sims, evaluator=ev, meta=meta, keys=keys)
        end.record()
        barrier()
    launches = _lib.kernel_launches() - launches0
    ms = start.elapsed_time(end)
    trunk_ms, counts = ev.profile_read()
    ev.profile(0)
    ms_max = parallel.max_over_ranks(ms, dev)
    total_sims = int(parallel.sum_over_ranks(args.sims * R * args.steps, dev))
    value = total_sims / (ms_max / 1000.0)
    positions = int(counts.sum())
    nodes = int(eng.num_nodes().max())

    peaks, peak_kind = measured_peaks()
    conv_launches = len(trunk_ms) * ev.conv_launches_per_call
    flops = positions * ev.trunk_flops_per_position()
    avg_launch_s = float(trunk_ms.sum()) / 1000.0 / max(1, conv_launches)
    achieved = (flops / max(1, conv_launches)) / avg_launch_s / 1e12 if avg_launch_s > 0 else 0.0
    peak = float(peaks.get("bf16_tflops_sustained", peaks.get("bf16_tflops")))
    # DRAM bytes per launch: the committed ncu capture of this kernel on the same board shape
    # (profiles/conv3x3_halot256_resnet20x256.md), scaled by the positions a launch processes
    per_pos = profile_value("conv3x3_halot256_resnet20x256.md", f"dram_bytes_per_position_per_launch_{game}")
    traffic = per_pos * positions / len(trunk_ms) if per_pos is not None and len(trunk_ms) else None
    roofline = {"kernel": f"k_conv3x3_halo_t (tcgen05 implicit-GEMM 3x3 conv, two 128-channel halves of 256 "
                          f"filters, {n_board + 1}x{n_board + 1} padded pixel grid)", "bound": "tensor", "achieved": achieved, "peak": peak,
                "unit": "TFLOP/s", "frac": achieved / peak,
                "peak_kind": f"bf16_tflops_sustained of {peak_kind}", "traffic": traffic,
                "algorithmic_flops_per_launch": flops / max(1, conv_launches),
                "avg_launch_ms": avg_launch_s * 1e3, "launches": conv_launches}

    e2e = None
    if not args.no_e2e:
        cfg = MCTSConfig(game_type=GameType.CHESS if chess else GameType.GO, board_size=n_board,
                         num_simulations=args.sims,
                         max_wave_size=args.wave, c_puct=1.4, virtual_loss=1.0,
                         initial_tree_nodes=args.capacity, device=str(dev),
                         enable_subtree_reuse=False, dirichlet_epsilon=0.0)
        mcts = MCTS(cfg, ev)
        mcts._engines[R] = eng
        mcts.search_batch(positions_host)
        barrier()
        s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s2.record()
        for _ in range(args.steps):
            pol = mcts.search_batch(positions_host)
        e2.record()
        barrier()
        ms2 = parallel.max_over_ranks(s2.elapsed_time(e2), dev)
        assert pol.shape == (R, n_act) and np.allclose(pol.sum(1), 1.0)
        e2e = {"value": total_sims / (ms2 / 1000.0), "unit": UNIT,
               "h2d_bytes_per_step": R * (101 * 72 + 4) if chess else R * (8 * 361 + 12),
               "d2h_bytes_per_step": R * n_act * 4,
               "api": (f"MCTS(MCTSConfig(game_type={'CHESS' if chess else 'GO'}), ResNetEvaluator)"
                       f".search_batch({'ChessPositions' if chess else 'GoPositions'}) -> numpy policies")}

    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        rate, sims, secs, threads, searches = cpu_search_rate(args, sd, args.cpu_seconds, game)
        cpu = {"value": rate, "unit": UNIT, "cores": threads, "kind": "port",
               "sample": f"{searches} whole searches ({sims} simulations) of {args.workload} {game} in {secs:.1f} s (oracle "
                         f"C++ tree with the {game} rules + fp32 torch CPU ResNet 20x256)"}
    line = None
    if rank == 0 or inner:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": ws, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_max / args.steps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": f"synthetic (seeded {game} roots, seeded He-init weights)",
            "config": {"workload": WORKLOAD_CHESS if chess else WORKLOAD_GO, "roots_total": total_roots,
                       "roots_per_gpu": R, "sims": args.sims, "wave": args.wave, "capacity": args.capacity,
                       "model": ("resnet20x256 (119 planes, 4672 actions, value fc 256)" if chess else
                                 "resnet20x256 (17 planes, 362 actions, value fc 256)"),
                       "parallelism": f"dp{ws} (roots sharded, weights NCCL-broadcast once)",
                       "l2": "inputs larger than L2 (multi-GB activations per ResNet call)"},
            "leaf_evals_per_s": positions / (ms / 1000.0) * ws,
            "max_tree_nodes": nodes,
            "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e, "clocks": clk.summary(),
            "gpu_launches": launches,
        }
    ev.close()
    eng.close()
    if inner:
        return line
    if rank == 0:
        print(json.dumps(line), flush=True)
    if ws > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()


def run_b200_forward(args):
    """ResNet leaf evaluations/s alone: seeded random weights and features of one game's shape,
    `--batch` positions per call, one step = one forward call; also the target of the committed
    conv ncu captures. ``--game go`` is 19x19 / 17 planes / 362 actions, ``--game chess`` 8x8 /
    119 planes / 4672 actions."""
    from omoknuni_quantum_b200 import _lib
    from omoknuni_quantum_b200.resnet import ResNetEvaluator, ResNetSpec
    ws, rank, local = dist_env()
    torch.cuda.set_device(local)
    n, planes, acts = {"gomoku": (15, 19, 225), "go": (19, 17, 362), "chess": (8, 119, 4672)}[args.game]
    spec = ResNetSpec(board_size=n, input_channels=planes, num_blocks=args.blocks, filters=args.filters,
                      num_actions=acts, fc_value_hidden=args.value_hidden)
    ev = ResNetEvaluator.random(spec, seed=args.seed, max_batch=args.batch, dtype=args.dtype)
    g = torch.Generator().manual_seed(args.seed)
    x = torch.zeros(args.batch, planes, n, n)
    x[:, 0] = (torch.rand(args.batch, n, n, generator=g) < 0.2).float()
    x[:, 1] = (torch.rand(args.batch, n, n, generator=g) < 0.2).float()
    x = x.to(ev.device)
    for _ in range(args.warmup):
        ev.evaluate_batch(x)
    torch.cuda.synchronize()
    n0 = _lib.kernel_launches()
    s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        s0.record()
        for _ in range(args.steps):
            ev.evaluate_batch(x)
        s1.record()
        torch.cuda.synchronize()
    ms = s0.elapsed_time(s1)
    if ev.error() != 0:
        raise SystemExit("ResNet forward reported a device error")
    if rank == 0:
        print(json.dumps({
            "metric": "ResNet leaf evaluations/sec", "value": args.batch * args.steps / (ms / 1000.0),
            "unit": "positions/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": args.dtype, "data": "synthetic (seeded features and weights)",
            "config": {"workload": f"forward: {args.game} {n}x{n}, {planes} planes, {acts} actions",
                       "model": f"resnet{args.blocks}x{args.filters}", "batch": args.batch},
            "trunk_tflops": args.batch * args.steps * ev.trunk_flops_per_position() / (ms / 1000.0) / 1e12,
            "clocks": clk.summary(), "gpu_launches": _lib.kernel_launches() - n0}), flush=True)


def main():
    args = parse()
    if args.workload == "forward" and args.impl == "b200":
        run_b200_forward(args)
        return
    if args.workload in ("config3", "config4") and args.impl == "b200":
        run_b200_go(args, "go" if args.workload == "config3" else "chess")
        return
    if args.workload == "config2" and args.impl == "b200":
        run_b200_selfplay(args)
        return
    if args.evaluator == "synthetic" and args.impl == "b200":
        run_b200_synthetic(args)
        return
    if args.impl == "reference":
        run_reference_arm(args)
    else:
        run_b200(args)


if __name__ == "__main__":
    main()
