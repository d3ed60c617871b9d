#!/usr/bin/env python
"""Benchmark: latent-descent sample-steps/s of the EBR energy network on 30 x 30 maze boards (L = 900).

Workload (per rank, weak scaling): 128 synthetic 30 x 30 maze inputs x 5 samples = 640 latent rows, L = 900, the
4-layer / hidden 512 / 8 x 64 / SwiGLU 4x energy network in bf16 with random-init weights. One step = one segment of
16 inference microsteps (forward + first-order dE/dz each, no double backward), then the lowest-energy pick over the
5 samples. Every attention call runs the sm_100a kernels (ebr_b200.fused_attn).

Output (rank 0, one JSON line): ``value`` = sample-steps/s over all ranks with inputs resident on the device;
``e2e`` = the same through the public API with the puzzles copied from pinned host memory and the energies / picks
copied back inside the timed region; ``roofline`` = the dominant attention op's achieved TFLOP/s (algorithmic FLOPs
per call / CUDA-event duration) against the measured bf16 peak; ``cpu_baseline`` = the reference's own eager CPU path
(its models/energy.py with math attention, installed under baseline/_ref; this repository's CPU port when it is
absent) timed on a bounded sample on this host.

``--impl reference`` times only that CPU path (rank 0) on the same config and prints its own line.
``--mode sweep`` times the three attention passes alone at L in {64, 81, 100, 256, 900, 2048} and D in {64, 128} (one
line per shape), and with
``--passes qkv_rope,qkv_unfused`` the fused qkv projection against cuBLAS + the split kernel at the same shapes.
``--mode train`` times a training step (double backward, bucketed NCCL all-reduce overlapped with the backward,
AdamW) on the sudoku-like 81-token workload or, with ``--train-workload sxm100``, the multi-solution 100-token
workload with 8 candidate trajectories per input.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

import torch  # noqa: E402

METRIC = "latent-descent sample-steps/s (L=900, B=128)"
UNIT = "sample-steps/s"
INPUTS, SAMPLES, MICROSTEPS, BOARD = 128, 5, 16, 30
PASS_FLOP = {"attn_fwd": 4, "attn_bwd": 10, "attn_bwd_bwd": 24}  # x N^2 D per (b, h) slice
PASS_BYTES = {"attn_fwd": (8, 4), "attn_bwd": (16, 4), "attn_bwd_bwd": (24, 4)}  # (x N D, x N) per slice


def peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "tf_burst": d["bf16_tflops"], "tf_sustained": d["bf16_tflops_sustained"],
                "source": "measured"}  # fmt: skip
    return {"hbm_gbs": 6650.0, "tf_burst": 1590.0, "tf_sustained": 1400.0, "source": "fallback"}


def config_dict(rows: int, n_gpus: int) -> dict:
    return {
        "workload": "cfg3 maze-30x30 latent descent (inference: fwd + dE/dz per microstep)",
        "inputs_per_gpu": INPUTS,
        "samples": SAMPLES,
        "rows_per_gpu": rows,
        "seq_len": BOARD * BOARD,
        "microsteps_per_step": MICROSTEPS,
        "model": "energy net 4 layers, hidden 512, 8 heads x 64, SwiGLU 4x, RMSNorm, 2D RoPE (random init)",
        "parallelism": f"dp{n_gpus} (batch-sharded replicas, no collective)",
        "l2": "inputs larger than L2 (each activation tensor ~590 MB)",
    }


# --------------------------------------------------------------------------------------------------------- clocks


class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region (200 ms period)."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")  # fmt: skip

    def __init__(self, device_index: int) -> None:
        self.idx = device_index
        self.lines: list[str] = []
        self.proc = None

    def start(self) -> None:
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", str(self.idx)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True,
            )  # fmt: skip
            threading.Thread(target=self._pump, daemon=True).start()
        except OSError:
            self.proc = None

    def _pump(self) -> None:
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for name, val in zip(names, f[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        return {
            "sm_mhz": statistics.median(sm) if sm else None,
            "sm_max_mhz": max(mx) if mx else None,
            "reasons": sorted(reasons),
            "samples": len(sm),
        }


# --------------------------------------------------------------------------------------------------------- inputs


def maze_tokens(n: int, gen: torch.Generator) -> torch.Tensor:
    """Synthetic stand-in for Maze-Hard inputs (the dataset is not available): 30 x 30 boards, wall (1) with p = 0.5
    else open (0), one start (2) and one goal (3) cell. Path cells (4) appear only in the labels."""
    cells = BOARD * BOARD
    tok = (torch.rand(n, cells, generator=gen) < 0.5).to(torch.int32)
    idx = torch.stack([torch.randperm(cells, generator=gen)[:2] for _ in range(n)])
    tok.scatter_(1, idx[:, :1], 2)
    tok.scatter_(1, idx[:, 1:], 3)
    return tok


def build_model(device):
    """The benchmark network (4 layers, hidden 512, 8 heads x 64, SwiGLU 4x, softplus cell head, bf16) on the 30 x 30
    board, random weights from a fixed seed."""
    from ebr_b200.energy import LatentEnergyNet, NetShape

    torch.manual_seed(0)
    return LatentEnergyNet(NetShape(board=(BOARD, BOARD), vocab=5, cell_softplus=True)).to(device)


def run_segment(model, x: torch.Tensor, z: torch.Tensor):
    """One segment: 16 inference microsteps, then each input's lowest-energy sample."""
    from ebr_b200.energy import descend, lowest_energy_pick

    z, e = descend(model, z, x, MICROSTEPS)
    return z, e, lowest_energy_pick(e, SAMPLES)


# --------------------------------------------------------------------------------------------------------- reference

REF_DIR = ROOT / "baseline" / "_ref"


def reference_installed() -> bool:
    """The unmodified reference installed by ``baseline/install_reference.sh`` (git-ignored; it travels with the tree)."""
    return (REF_DIR / "models" / "energy.py").exists() and (REF_DIR / "models" / "fused_attn" / "ops.py").exists()


def import_reference(impl: str):
    """Import the installed reference's ``models.energy`` with ``EBR_FUSED_ATTN_IMPL=impl`` (``reference``: its dense
    torch path; ``triton``: its Triton kernels, an error if they do not load). Must not share a process with
    ``ebr_b200.fused_attn``: both register the ``ebr_fused::`` ops."""
    os.environ["EBR_FUSED_ATTN_IMPL"] = impl
    if str(REF_DIR) not in sys.path:
        sys.path.insert(0, str(REF_DIR))
    import models.energy as ref_energy

    return ref_energy


def reference_energy_config(ref_energy, *, board: int, vocab: int, softplus: bool, gpu_fast: bool):
    """The reference's ``EnergyConfig`` for the benchmark architecture (4 layers, hidden 512, 8 heads x 64, SwiGLU 4x,
    bf16) with the descent settings of its config/arch/ebr.yaml and config/train/maze_hard.yaml. ``gpu_fast``: its
    own fast GPU recipe (config/train/maze_hard_fast.yaml: fused Triton attention in both tiers, fused RoPE split,
    compiled dE/dz and descent wrapper, no host syncs); otherwise its eager CPU path (math attention, broadcast RoPE,
    no compilation)."""
    attn = "fused" if gpu_fast else "math"
    return ref_energy.EnergyConfig(
        seq_len=board * board, vocab_size=vocab, num_layers=4, hidden_size=512, expansion=4.0, num_heads=8,
        board_height=board, board_width=board, forward_dtype="bfloat16",
        energy_cell_activation="softplus" if softplus else "linear", attn_backend=attn, attn_nograd_backend=attn,
        cycles=MICROSTEPS, grad_cycles=7, randomize_min_cycles=MICROSTEPS, reset_cycles_low=7,
        reset_cycles_high=MICROSTEPS, halt_max_steps=16, halt_exploration_prob=0.0, step_size=250.0,
        step_size_low=200.0, step_size_high=250.0, init_std=1.0, noise_scale=0.05, noise_cosine=False,
        noise_settle_hot=0.4, microstep_ce=0.5, microstep_ce_ramp=1.0, convergence_threshold=0.75,
        convergence_temperature=0.05, convergence_window=2, explore_k=1, energy_compile=gpu_fast,
        descent_wrapper_compile=gpu_fast, rope_impl="fused" if gpu_fast else "broadcast", avoid_host_syncs=gpu_fast,
    )  # fmt: skip


def reference_network(ref_energy, device, gpu_fast: bool):
    """The reference's ``InnerNetwork`` (embeddings, energy, descent) for the maze-30x30 workload, in eval mode."""
    torch.manual_seed(0)
    cfg = reference_energy_config(ref_energy, board=BOARD, vocab=5, softplus=True, gpu_fast=gpu_fast)
    with torch.device(device):
        net = ref_energy.InnerNetwork(cfg)
    return net.eval()


def cpu_reference_sample(seconds: float = 10.0, rows: int = 2, min_steps: int = 1) -> dict:
    """The reference's CPU path timed on ``rows`` rows of the maze-30x30 workload until ``seconds`` have passed: its own
    eager modules from the installed reference (math attention, ``EBR_FUSED_ATTN_IMPL=reference``, no compilation,
    one ``EnergyDescent`` microstep per step), else this repository's CPU port (oracle attention inside the oracle's
    restatement of the network). Returns sample-steps/s and what was run."""
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    gen = torch.Generator().manual_seed(1)
    tok = maze_tokens(rows, gen)
    if reference_installed():
        ref_energy = import_reference("reference")
        net = reference_network(ref_energy, "cpu", gpu_fast=False)
        with torch.no_grad():
            x = net.input_embeddings(tok)
            z = net.fresh_states((rows, BOARD * BOARD, 512), x)
        cos_sin = net.cos_sin()
        step = lambda z_: net.level(z_, x, cos_sin)
        kind, what = "reference", "the reference's eager path (models/energy.py EnergyDescent, math attention, bf16)"
    else:
        from oracle import energy as oe
        from oracle.torch_attention import oracle_attention

        net = build_model("cpu")
        state = net.reference_state()
        spec = {"board": (BOARD, BOARD), "hidden": 512, "heads": 8, "layers": 4, "softplus": True}
        x = oe.embed(state, spec, tok, torch.bfloat16)
        z = net.fresh_states(rows)
        step = lambda z_: oe.microstep(state, spec, z_, x, noise=torch.randn_like(z_) * 0.05,
                                       attention=oracle_attention)[0]  # fmt: skip
        kind, what = "port", "the oracle's restatement of the network (numpy oracle attention, torch CPU bf16 layers)"
    steps, t0 = 0, time.perf_counter()
    with torch.no_grad():
        while steps < min_steps or time.perf_counter() - t0 < seconds:
            z = step(z)
            steps += 1
    dt = time.perf_counter() - t0
    return {
        "value": rows * steps / dt,
        "unit": UNIT,
        "cores": threads,
        "kind": kind,
        "sample": f"{rows} rows x {steps} microsteps at L=900 ({dt:.1f} s) through {what}, {threads} threads",
    }


def cpu_reference_subprocess(seconds: float) -> dict | None:
    """``cpu_reference_sample`` in a child process (the reference registers the same ``ebr_fused::`` op names as this
    package, so they cannot share one)."""
    cmd = [sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1", "--warmup", "0",
           "--cpu-seconds", str(seconds)]  # fmt: skip
    env = {**os.environ, "CUDA_VISIBLE_DEVICES": "", "RANK": "0", "WORLD_SIZE": "1"}
    try:
        res = subprocess.run(cmd, capture_output=True, text=True, env=env, timeout=max(600.0, 20 * seconds))
        line = [ln for ln in res.stdout.splitlines() if ln.startswith("{")][-1]
        return json.loads(line)["cpu_baseline"]
    except (subprocess.SubprocessError, IndexError, KeyError, json.JSONDecodeError):
        return None


def run_reference(args) -> None:
    """``--impl reference``: the reference's CPU path on the host cores (rank 0 only; other ranks exit at once).
    Each step is a bounded sample: ``--cpu-seconds`` of microsteps on 2 rows (at least one microstep)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    for _ in range(max(args.warmup, 0)):
        cpu_reference_sample(seconds=0.0, rows=2, min_steps=1)
    vals, last = [], None
    for _ in range(args.steps):
        last = cpu_reference_sample(seconds=args.cpu_seconds if args.steps == 1 else 0.0, rows=2, min_steps=1)
        vals.append(last["value"])
    value = statistics.median(vals)
    cfg = config_dict(INPUTS * SAMPLES, args.gpus)
    cfg["parallelism"] = "host CPU on rank 0 only: the figure does not grow with n_gpus"
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": value,
        "unit": UNIT,
        "n_gpus": args.gpus,
        "cpu_only": True,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": 1000.0 * 2 / value if value else None,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded maze-like boards; Maze-Hard is not available offline), random-init weights",
        "config": cfg,
        "cpu_baseline": {**last, "value": value},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_triton_descent(args) -> None:
    """``--impl triton``: the reference's own GPU path on this box, for comparison (not a contract arm): its
    ``InnerNetwork.rollout`` in eval mode with its fast recipe (fused Triton attention and RoPE split, inductor-
    compiled dE/dz and descent wrapper), one 16-microstep segment per step on the same 640 rows, CUDA events."""
    if not reference_installed():
        print(json.dumps({"impl": "triton", "unavailable": "reference not installed (baseline/install_reference.sh)"}))
        return
    ref_energy = import_reference("triton")
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    net = reference_network(ref_energy, device, gpu_fast=True)
    rows = INPUTS * SAMPLES
    gen = torch.Generator().manual_seed(1000)
    tokens = maze_tokens(INPUTS, gen).repeat_interleave(SAMPLES, dim=0).to(device)
    plan = ref_energy.SegmentPlan()
    with torch.no_grad():
        z = net.fresh_states((rows, BOARD * BOARD, 512), net.input_embeddings(tokens))
    batch = {"inputs": tokens}
    for _ in range(max(args.warmup, 1)):
        with torch.no_grad():
            z, *_ = net.rollout(z, batch, plan)
    torch.cuda.synchronize()
    sampler = ClockSampler(0)
    sampler.start()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(args.steps):
        with torch.no_grad():
            z, *_ = net.rollout(z, batch, plan)
    b.record()
    torch.cuda.synchronize()
    clocks = sampler.stop()
    ms = a.elapsed_time(b)
    print(json.dumps({
        "impl": "triton", "metric": METRIC, "value": round(rows * MICROSTEPS * args.steps / (ms / 1000.0), 3),
        "unit": UNIT, "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 3),
        "config": {**config_dict(rows, 1), "reference_recipe": "maze_hard_fast (fused Triton attention + RoPE split, "
                   "energy_compile, descent_wrapper_compile, avoid_host_syncs)"},
        "clocks": clocks,
    }), flush=True)  # fmt: skip


# --------------------------------------------------------------------------------------------------------- GPU path


def run_ours(args) -> None:
    from ebr_b200 import _native, fused_attn, runtime
    from ebr_b200.build import build

    rank, world, local = runtime.init_distributed()
    n_gpus = world
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if rank == 0:
        build()
    if world > 1:
        torch.distributed.barrier()
    model = build_model(device)
    rows = INPUTS * SAMPLES
    gen = torch.Generator().manual_seed(1000 + rank)
    tokens_host = maze_tokens(INPUTS, gen).repeat_interleave(SAMPLES, dim=0).pin_memory()
    tokens = tokens_host.to(device)
    with torch.no_grad():
        x = model.embed(tokens)
    z0 = model.fresh_states(rows)

    def barrier():
        if world > 1:
            torch.distributed.barrier()

    # warm-up
    z = z0
    for _ in range(args.warmup):
        z, e, pick = run_segment(model, x, z)
    torch.cuda.synchronize()
    _native.device_status()

    # timed region: inputs resident on the device
    sampler = ClockSampler(torch.cuda.current_device() if not os.environ.get("CUDA_VISIBLE_DEVICES") else local)
    barrier()
    torch.cuda.synchronize()
    sampler.start()
    launches0 = _native.launch_count()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with fused_attn.kernel_timer() as timer:
        start.record()
        for _ in range(args.steps):
            z, e, pick = run_segment(model, x, z)
        end.record()
        torch.cuda.synchronize()
    clocks = sampler.stop()
    launches = _native.launch_count() - launches0
    barrier()
    ms = start.elapsed_time(end)
    ms = runtime.max_over_ranks(ms)
    ops = timer.summary()
    value = n_gpus * rows * MICROSTEPS * args.steps / (ms / 1000.0)

    # end to end through the public API with host buffers
    e2e_steps = max(1, args.steps)
    energies_host = torch.empty(rows, dtype=torch.float32).pin_memory()
    picks_host = torch.empty(INPUTS, dtype=torch.int64).pin_memory()
    barrier()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    zz = z0
    for _ in range(e2e_steps):
        tok_d = tokens_host.to(device, non_blocking=True)
        with torch.no_grad():
            xx = model.embed(tok_d)
        zz, ee, pp = run_segment(model, xx, zz)
        energies_host.copy_(ee, non_blocking=True)
        picks_host.copy_(pp, non_blocking=True)
    b.record()
    torch.cuda.synchronize()
    e2e_ms = runtime.max_over_ranks(a.elapsed_time(b))
    e2e_value = n_gpus * rows * MICROSTEPS * e2e_steps / (e2e_ms / 1000.0)
    h2d = tokens_host.numel() * tokens_host.element_size()
    d2h = energies_host.numel() * 4 + picks_host.numel() * 8
    _native.device_status()

    # roofline of the dominant attention op
    pk = peaks()
    dom_name = max(ops, key=lambda n: ops[n]["ms"]) if ops else None
    roofline = None
    if dom_name:
        d = ops[dom_name]
        B_, H_, N_, D_ = d["shape"]
        flop = PASS_FLOP[dom_name] * N_ * N_ * D_ * B_ * H_
        avg_ms = d["ms"] / d["calls"]
        achieved = flop / (avg_ms / 1000.0) / 1e12
        traffic = None
        tfile = ROOT / "profiles" / "traffic.json"
        if tfile.exists():
            t = json.loads(tfile.read_text()).get(dom_name)
            if t and t.get("N") == N_ and t.get("D") == D_:
                traffic = t["bytes_per_slice"] * B_ * H_
        roofline = {
            "bound": "tensor",
            "kernel": f"{dom_name} (all launches of one call; {d['calls']} calls in the timed region)",
            "achieved": round(achieved, 2),
            "peak": pk["tf_sustained"],
            "unit": "TFLOP/s",
            "frac": round(achieved / pk["tf_sustained"], 4),
            "peak_note": f"{pk['source']} bf16 sustained (kernel timed inside a long step); burst {pk['tf_burst']}",
            "traffic": traffic,
            "flop_per_call": flop,
            "avg_ms_per_call": round(avg_ms, 4),
            "ops": {n: {"calls": v["calls"], "ms_total": round(v["ms"], 3)} for n, v in ops.items()},
        }

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_reference_subprocess(args.cpu_seconds)

    if rank == 0:
        line = {
            "metric": METRIC,
            "value": round(value, 3),
            "unit": UNIT,
            "n_gpus": n_gpus,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms / args.steps, 3),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic (seeded maze-like boards; Maze-Hard is not available offline), random-init weights",
            "config": config_dict(rows, n_gpus),
            "e2e": {"value": round(e2e_value, 3), "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
            "gpu_launches": int(launches),
            "roofline": roofline,
            "cpu_baseline": cpu,
            "clocks": clocks,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


# --------------------------------------------------------------------------------------------------------- training


TRAIN_MICROSTEPS, TRAIN_GRADED = 16, 7
SUDOKU_ROWS = 768                    # sudoku-like training (81 tokens): rows per GPU
SXM_INPUTS, SXM_K, SXM_BOARD = 32, 8, 10  # multi-solution training: inputs per GPU (256 over 8 GPUs), candidates each


def sudoku_like_tokens(n: int, gen: torch.Generator) -> torch.Tensor:
    """Synthetic stand-in for Sudoku-Extreme boards (the dataset is not available): 81 cells, 0 (blank) with
    p = 0.7, otherwise uniform in 1..9. Labels are uniform in 1..9."""
    blank = torch.rand(n, 81, generator=gen) < 0.7
    digits = torch.randint(1, 10, (n, 81), generator=gen)
    return torch.where(blank, torch.zeros_like(digits), digits).to(torch.int32), torch.randint(1, 10, (n, 81), generator=gen)


def binary_grid_tokens(n: int, gen: torch.Generator, board: int = SXM_BOARD, ones: int = SXM_BOARD):
    """Synthetic stand-in for the multi-solution boards (N-Queens 10 x 10 is not available offline): inputs are
    binary grids with exactly ``ones`` ones at uniformly random cells; labels are binary grids with one 1 per row at
    a random column (a permutation), so every label also has ``ones`` ones."""
    cells = board * board
    inputs = torch.zeros(n, cells, dtype=torch.int32)
    for i in range(n):
        inputs[i, torch.randperm(cells, generator=gen)[:ones]] = 1
    cols = torch.stack([torch.randperm(board, generator=gen) for _ in range(n)])
    labels = torch.zeros(n, board, board, dtype=torch.int64)
    labels.scatter_(2, cols.unsqueeze(-1), 1)
    return inputs, labels.view(n, cells)


def run_train(args) -> None:
    """A training step on each rank (weak scaling). Workloads:

    * ``sudoku81``: 768 rows per GPU on a 9 x 9 board (81 tokens, vocab 10), 16 microsteps per segment of which the
      last 7 carry a graph (create_graph=True: the backward runs the attention's double backward), stablemax cross
      entropy of the decoded endpoint;
    * ``sxm100``: multi-solution training on a 10 x 10 binary board (100 tokens): 32 inputs per GPU x 8 candidate
      trajectories (256 latent rows over 8 GPUs gives the workload's 256 x 8), the candidates' 16-microstep segment
      without a graph, each input's best candidate recomputed through its 7 graded microsteps (forward SXM);
      ``--heads 4`` runs it at head dim 128 (the reference's multi-solution recipe: hidden 512, 4 heads).

    Then the outer backward with the gradients all-reduced in buckets overlapped with it (NCCL; none at one GPU) and
    an AdamW step. ``value`` counts latent rows x microsteps per second over all ranks: for sxm100 every candidate's
    16 microsteps (the graded recompute of the winners is extra work, not counted)."""
    from ebr_b200 import _native, fused_attn, runtime
    from ebr_b200.build import build
    from ebr_b200.energy import LatentEnergyNet, NetShape, sxm_explore_loss, train_segment_loss

    rank, world, local = runtime.init_distributed()
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if rank == 0:
        build()
    if world > 1:
        torch.distributed.barrier()
    torch.manual_seed(0)
    gen = torch.Generator().manual_seed(2000 + rank)
    sxm = args.train_workload == "sxm100"
    if sxm:
        shape = NetShape(board=(SXM_BOARD, SXM_BOARD), vocab=2, heads=args.heads)
        tok, labels = binary_grid_tokens(SXM_INPUTS, gen)
        rows, counted_rows = SXM_INPUTS, SXM_INPUTS * SXM_K
    else:
        shape = NetShape(board=(9, 9), vocab=10, heads=args.heads)
        tok, labels = sudoku_like_tokens(SUDOKU_ROWS, gen)
        rows, counted_rows = SUDOKU_ROWS, SUDOKU_ROWS
    model = LatentEnergyNet(shape).to(device)
    runtime.broadcast_model(model)
    opt = torch.optim.AdamW(model.parameters(), lr=1e-4, fused=True)
    tok, labels = tok.to(device), labels.to(device)
    z0 = model.fresh_states(rows)
    challengers = torch.stack([model.fresh_states(rows) for _ in range(SXM_K - 1)]) if sxm else None
    params = [p for p in model.parameters() if p.requires_grad]
    buckets = runtime.GradientBuckets(params, bucket_mb=16.0)
    exposed = []  # host-side wait for the collectives after the backward (ms), per step

    def step():
        nonlocal challengers
        s0 = torch.cuda.Event(enable_timing=True)
        s0.record()
        x = model.embed(tok)
        if sxm:
            loss, _, challengers = sxm_explore_loss(model, z0, challengers, x, labels, TRAIN_MICROSTEPS - TRAIN_GRADED,
                                                    TRAIN_GRADED)  # fmt: skip
        else:
            loss = train_segment_loss(model, z0, x, labels, TRAIN_MICROSTEPS - TRAIN_GRADED, TRAIN_GRADED)
        opt.zero_grad(set_to_none=True)
        buckets.start()
        (loss / world).backward()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        buckets.finish()
        e1.record()
        opt.step()
        return loss, (s0, e0, e1)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    _native.device_status()
    if world > 1:
        torch.distributed.barrier()
    launches0 = _native.launch_count()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    marks = []
    with fused_attn.kernel_timer() as timer:
        a.record()
        for _ in range(args.steps):
            loss, ev = step()
            marks.append(ev)
        b.record()
        torch.cuda.synchronize()
    ms = runtime.max_over_ranks(a.elapsed_time(b))
    tail_ms = runtime.max_over_ranks(statistics.median(e0.elapsed_time(e1) for _, e0, e1 in marks))
    # This rank's own work per step (forward segment + backward, up to the wait for the collectives): the spread of
    # it over ranks is what the others wait for in finish().
    own_ms = statistics.median(s0.elapsed_time(e0) for s0, e0, _ in marks)
    own_max, own_min = runtime.max_over_ranks(own_ms), -runtime.max_over_ranks(-own_ms)
    ops = timer.summary()
    runtime.check_param_sync(model, rtol=1e-9)
    # The gradient all-reduce alone, for the record: one flat bucket of every gradient, CUDA events (max over ranks).
    nparam = sum(p.numel() for p in params)
    ar_ms = None
    if world > 1:
        flat = torch.zeros(nparam, device=device)
        for _ in range(3):
            torch.distributed.all_reduce(flat)
        torch.cuda.synchronize()
        c, d = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        c.record()
        for _ in range(10):
            torch.distributed.all_reduce(flat)
        d.record()
        torch.cuda.synchronize()
        ar_ms = runtime.max_over_ranks(c.elapsed_time(d) / 10)
        del flat
    value = world * counted_rows * TRAIN_MICROSTEPS * args.steps / (ms / 1000.0)
    if rank == 0:
        head_dim = 512 // args.heads
        if sxm:
            workload = (f"multi-solution SXM training, 10x10 binary board (L=100), {SXM_INPUTS} inputs x {SXM_K} "
                        f"candidates per GPU, {args.heads} heads x {head_dim}, 16 microsteps (last 7 graded, winners "
                        "recomputed with a graph), double backward, AdamW")  # fmt: skip
        else:
            workload = (f"sudoku-like training (L=81), {SUDOKU_ROWS} rows per GPU, {args.heads} heads x {head_dim}, "
                        "16 microsteps (last 7 graded), double backward, AdamW")  # fmt: skip
        line = {
            "metric": f"latent-descent training sample-steps/s ({args.train_workload})",
            "value": round(value, 3),
            "unit": "sample-steps/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms / args.steps, 3),
            "higher_is_better": True,
            "scaling": "weak",
            "dtype": "bf16",
            "data": "synthetic boards (the reference's datasets are not available offline), random-init weights",
            "config": {"workload": workload, "rows_counted_per_gpu": counted_rows, "seq_len": shape.seq_len,
                       "parallelism": f"dp{world}: gradients all-reduced in {len(buckets.buckets)} buckets overlapped "
                                      "with the outer backward"},  # fmt: skip
            "allreduce": {"params": nparam, "bytes": 4 * nparam, "buckets": len(buckets.buckets),
                          "flat_allreduce_ms": None if ar_ms is None else round(ar_ms, 3),
                          "exposed_after_backward_ms": round(tail_ms, 3),
                          "rank_compute_ms_min": round(own_min, 3), "rank_compute_ms_max": round(own_max, 3)},  # fmt: skip
            "loss": float(loss.item()),
            "gpu_launches": int(_native.launch_count() - launches0),
            "attention_ms": {n: round(v["ms"], 3) for n, v in ops.items()},
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


# --------------------------------------------------------------------------------------------------------- sweep


def median_call_ms(fn, args, budget_ms: float = 4000.0) -> float:
    """Median CUDA-event time of ``fn`` (synchronized on both sides of each call) after ``--warmup`` calls, over
    ``--steps`` calls, or fewer (at least 3) when that many would take longer than ``budget_ms``."""
    for _ in range(max(args.warmup, 1)):
        fn()
    torch.cuda.synchronize()
    ts = []
    while len(ts) < args.steps and (len(ts) < 3 or sum(ts) < budget_ms):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        ts.append(a.elapsed_time(b))
    return statistics.median(ts)


def run_sweep(args) -> None:
    """The isolated kernel sweep: each pass alone, bf16, H = 8, B = 262144 // L (per GPU), CUDA events, median of K.

    ``--impl ours``: the sm_100a kernels through ``torch.ops.ebr_fused``. ``--impl triton``: the same ops as the
    installed reference registers them (its Triton kernels, JIT-compiled for this GPU by Triton, default plans), on
    the same inputs with the same timing; the projection passes are ours only."""
    if args.impl == "triton":
        if not reference_installed():
            print(json.dumps({"impl": "triton", "unavailable": "reference not installed (baseline/install_reference.sh)"}))
            return
        import_reference("triton")
        from models.fused_attn import ops as _ref_ops  # noqa: F401  (registers ebr_fused:: with the Triton kernels)

        class _NoNative:
            @staticmethod
            def device_status() -> None:
                return None

        _native = _NoNative
    else:
        from ebr_b200 import _native
        from ebr_b200.build import build

        build()
    torch.cuda.set_device(0)
    pk = peaks()
    Ls = [int(v) for v in args.lengths.split(",")]
    for D in [int(v) for v in args.head_dims.split(",")]:
        for L in Ls:
            B, H = (args.sweep_batch or 262144 // L), 8
            g = torch.Generator(device="cuda").manual_seed(0)
            mk = lambda s: (torch.randn(B, H, L, D, device="cuda", generator=g) * s).to(torch.bfloat16)
            q, k, v, do, gq, gk, gv = mk(0.5), mk(0.5), mk(0.5), mk(1.0), mk(1.0), mk(1.0), mk(1.0)
            s = D**-0.5
            o, lse = torch.ops.ebr_fused.attn_fwd(q, k, v, s)
            dq, _, _ = torch.ops.ebr_fused.attn_bwd(q, k, v, o, lse, do, s)
            fns = {
                "attn_fwd": lambda: torch.ops.ebr_fused.attn_fwd(q, k, v, s),
                "attn_bwd": lambda: torch.ops.ebr_fused.attn_bwd(q, k, v, o, lse, do, s),
                "attn_bwd_bwd": lambda: torch.ops.ebr_fused.attn_bwd_bwd(q, k, v, o, lse, do, dq, gq, gk, gv, s),
            }
            out = {"mode": "sweep", "impl": args.impl, "L": L, "D": D, "B": B, "H": H}
            for name, fn in fns.items():
                if name not in args.passes.split(","):
                    continue
                ms = median_call_ms(fn, args)
                flop = PASS_FLOP[name] * L * L * D * B * H
                nd, nn = PASS_BYTES[name]
                byt = (nd * L * D + nn * L) * B * H
                tf, gbs = flop / ms / 1e9, byt / ms / 1e6
                out[name] = {"ms": round(ms, 4), "tflops": round(tf, 1), "tc_frac": round(tf / pk["tf_burst"], 4),
                             "gbs": round(gbs, 0), "hbm_frac": round(gbs / pk["hbm_gbs"], 4)}  # fmt: skip
            del q, k, v, do, gq, gk, gv, o, lse, dq
            torch.cuda.empty_cache()
            proj = [p for p in ("qkv_rope", "qkv_unfused", "o_proj", "o_unfused", "gate_up", "gate_up_unfused",
                                "rope_merge", "swiglu_bwd", "qkv_dx", "qkv_dx_add", "qkv_dx_unfused")
            if p in args.passes.split(",")]
            if proj and args.impl == "ours":
                out.update(sweep_qkv(args, proj, B, L, H, D, pk))
            _native.device_status()
            print(json.dumps(out), flush=True)
            torch.cuda.empty_cache()


def _no_grad_call(fn, *a):
    with torch.no_grad():
        return fn(*a)


def sweep_qkv(args, passes, B: int, L: int, H: int, D: int, pk: dict) -> dict:
    """The projections of one block at the sweep shape: qkv (x [B, L, H D], W [3 H D, H D]) as the tcgen05 GEMM with
    the RoPE split as its epilogue (``qkv_rope``) and as cuBLAS + the split kernel (``qkv_unfused``); the output
    projection from the head-major attention output (``o_proj``) and as transpose copy + cuBLAS (``o_unfused``); the
    MLP's gate / up projection with the SwiGLU activation as its epilogue (``gate_up``) and as cuBLAS + the activation
    kernel (``gate_up_unfused``); the two HBM-bound kernels of the dE/dz backward, the RoPE merge of dq / dk / dv into
    d(qkv) (``rope_merge``) and the SwiGLU backward (``swiglu_bwd``); the qkv projection's input gradient with the
    merge folded into the GEMM (``qkv_dx``; ``qkv_dx_add`` with the residual gradient joined in its epilogue, as the
    dE/dz backward runs it) and as the merge kernel + cuBLAS (``qkv_dx_unfused``)."""
    import torch.nn.functional as F

    from ebr_b200.energy import NetShape, rope_tables
    from ebr_b200.layers import _swiglu_grad, gate_up_swiglu_op, o_proj_op, qkv_rope_merge_dx_op, qkv_rope_split_op, \
        rope_merge_op, rope_split_op, swiglu_act

    side = int(round(L**0.5))
    hh, ww = (side, side) if side * side == L else (32, L // 32)
    C = H * D
    cos_t, sin_t = rope_tables(NetShape(board=(hh, ww), hidden=C, heads=H), device="cuda")
    g = torch.Generator(device="cuda").manual_seed(1)
    x = torch.randn(B, L, C, device="cuda", generator=g).to(torch.bfloat16)
    w = (torch.randn(3 * C, C, device="cuda", generator=g) * C**-0.5).to(torch.bfloat16)
    e = torch.zeros(0, device="cuda")
    o = torch.randn(B, H, L, D, device="cuda", generator=g).to(torch.bfloat16)
    wo = (torch.randn(C, C, device="cuda", generator=g) * C**-0.5).to(torch.bfloat16)
    inter = NetShape(hidden=C, heads=H).mlp_width  # the energy network's SwiGLU width (expansion 4)
    wgu = (torch.randn(2 * inter, C, device="cuda", generator=g) * C**-0.5).to(torch.bfloat16)
    need = set(passes)
    if need & {"rope_merge", "qkv_dx", "qkv_dx_add", "qkv_dx_unfused"}:
        dq3 = [torch.randn(B, H, L, D, device="cuda", generator=g).to(torch.bfloat16) for _ in range(3)]
    if "swiglu_bwd" in need:
        hgu = torch.randn(B, L, 2 * inter, device="cuda", generator=g).to(torch.bfloat16)
        gact = torch.randn(B, L, inter, device="cuda", generator=g).to(torch.bfloat16)
    fns = {
        "qkv_rope": lambda: qkv_rope_split_op(x, w, cos_t, sin_t, e, H),
        "qkv_unfused": lambda: rope_split_op(F.linear(x, w), cos_t, sin_t, e, H),
        "o_proj": lambda: o_proj_op(o, wo),
        "o_unfused": lambda: F.linear(o.transpose(1, 2).reshape(B, L, C), wo),
        "gate_up": lambda: gate_up_swiglu_op(x, wgu),
        "gate_up_unfused": lambda: swiglu_act(F.linear(x, wgu)),
        "rope_merge": lambda: rope_merge_op(*dq3, cos_t, sin_t, e),
        "qkv_dx": lambda: qkv_rope_merge_dx_op(*dq3, w, cos_t, sin_t, e),
        "qkv_dx_add": lambda: qkv_rope_merge_dx_op(*dq3, w, cos_t, sin_t, e, x),
        "qkv_dx_unfused": lambda: rope_merge_op(*dq3, cos_t, sin_t, e) @ w,
        "swiglu_bwd": lambda: _no_grad_call(_swiglu_grad, hgu, gact),  # the fused kernel (no higher-order graph)
    }
    res = {}
    for name in passes:
        ms = median_call_ms(fns[name], args)
        if name.startswith("qkv_dx"):
            flop = 2.0 * B * L * C * 3 * C
            byt = 2.0 * (3 * B * L * C + 3 * C * C + B * L * C)  # dq, dk, dv, W, dx (the fused path's bytes)
            byt += 2.0 * B * L * C if name == "qkv_dx_add" else 0.0  # the addend
        elif name.startswith("qkv"):
            flop = 2.0 * B * L * C * 3 * C
            byt = 2.0 * (B * L * C + 3 * C * C + 3 * B * L * C)  # x, W, q / k / v (the fused path's bytes)
        elif name.startswith("gate_up"):
            flop = 2.0 * B * L * C * 2 * inter
            byt = 2.0 * (B * L * C + 2 * inter * C + 3 * B * L * inter)  # x, W, h, act
        elif name == "rope_merge":
            flop, byt = 0.0, 2.0 * 6 * B * L * C  # dq, dk, dv in, d(qkv) out
        elif name == "swiglu_bwd":
            flop, byt = 0.0, 2.0 * 5 * B * L * inter  # h (gate, up) and d act in, d h out
        else:
            flop = 2.0 * B * L * C * C
            byt = 2.0 * (2 * B * L * C + C * C)  # O, W, y
        tf = flop / ms / 1e9
        res[name] = {"ms": round(ms, 4), "tflops": round(tf, 1), "tc_frac": round(tf / pk["tf_burst"], 4),
                     "gbs": round(byt / ms / 1e6, 0), "hbm_frac": round(byt / ms / 1e6 / pk["hbm_gbs"], 4)}  # fmt: skip
    del x, w, o, wo, wgu
    return res


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=4)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference", "triton"], default="ours",
                    help="reference: the reference's CPU path (the contract's reference arm); triton: the reference's "
                    "own GPU path on this box (descent or sweep mode)")
    ap.add_argument("--mode", choices=["descent", "sweep", "train"], default="descent")
    ap.add_argument("--lengths", default="64,81,100,256,900,2048")
    ap.add_argument("--head-dims", default="64,128")
    ap.add_argument("--sweep-batch", type=int, default=0,
                    help="sweep mode: batch B per shape (default 262144 // L: 268 MB per tensor at D = 64)")
    ap.add_argument("--passes", default="attn_fwd,attn_bwd,attn_bwd_bwd",
                    help="sweep: which passes to time (also qkv_rope, qkv_unfused, o_proj, o_unfused: the projections)")
    ap.add_argument("--train-workload", choices=["sudoku81", "sxm100"], default="sudoku81",
                    help="train mode: sudoku81 (L=81, 768 rows per GPU) or sxm100 (L=100, 32 inputs x 8 candidates)")
    ap.add_argument("--heads", type=int, default=8, help="train mode: attention heads (hidden 512; 4 heads = D 128)")
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3 and args.mode == "descent" and args.impl == "ours":
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    elif args.mode == "sweep":
        run_sweep(args)
    elif args.mode == "train":
        run_train(args)
    elif args.impl == "triton":
        run_triton_descent(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
