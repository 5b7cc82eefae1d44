#!/usr/bin/env python
"""Benchmark: 19x19 network positions/sec on B200 (one process per GPU).

Workload ("C4"): a 19x19 board, 20 residual blocks
of 256 filters, value_hidden 256, one history position (4 planes), batch
1024 per GPU, bf16 weights and activations with fp32 accumulation. Weights
are the reference's seeded Network(cfg, 1) with the benchmark's batch-norm
statistics; inputs are seeded synthetic positions (stones occupied with
p = 0.4, colours 50/50). One "step" is one forward pass over the batch.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl engine|reference]

For N > 1 the driver launches one rank per GPU through torch.distributed.run;
each rank runs its own batch on its own replica of the weights (broadcast
once from rank 0 over NCCL), with no per-step collective: `scaling` is weak.

Printed (rank 0, one JSON line):
  value      positions/s over all ranks, inputs resident in HBM, device time
             (CUDA events on the engine's stream, max over ranks);
  e2e        the same through the runner's C ABI (BatchRunner, 2 slots in
             flight), pinned host input copied in and logits/values copied
             out inside every pass;
  e2e_records  the same from position records (stone bytes; the planes are
             encoded on the device), one synchronous call per pass;
  roofline   the tower convolution kernel: algorithmic FLOPs per launch over
             its average CUDA-event duration, against the measured bf16 peak;
  cpu_baseline  the reference's own CPU engine (blas, one worker per core at
             batch 8) on a bounded sample, rank 0 at N = 1 only;
  selfplay   C5: playouts/s and positions
             evaluated/s of the reference's own self-play (MCTS, rules,
             InferenceHub) on this engine, 512 games per GPU, with the
             reference's CPU self-play (blas) beside it at N = 1.
`--impl reference` times the reference's CPU implementation (oracle/_ref,
OpenBLAS, all host cores) on the same config and metric instead, and adds
`ref_cuda`: the reference's own CUDA engine rebuilt for sm_100 on the same
workload, and the reference's CPU self-play.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "alphazero-go_b200"))

METRIC = "19x19 net positions/sec"
UNIT = "positions/s"
BOARD, BLOCKS, FILTERS, VALUE_HIDDEN, HISTORY = 19, 20, 256, 256, 1
BATCH = 1024
SEED = 1
WORKLOAD = "C4: 19x19 board, 20 residual blocks x 256 filters, value_hidden 256, 4 input planes, batch 1024 per GPU"

# Self-play ("C5"): the 9x9 6x64 network of C2
# (history 1, value_hidden 128, seeded as the benchmark's), PUCT MCTS with
# 200 playouts per move and c_puct 1.5, 512 concurrent games per GPU, leaves
# batched by the reference's InferenceHub into passes of up to 256, mcts
# batch 8, and the rest of configs/9x9.cfg (komi 7.5, 7 sampled opening
# moves, move cap 2n^2) with resignation off.
SP_BOARD, SP_BLOCKS, SP_FILTERS, SP_VH = 9, 6, 64, 128
SP_GAMES, SP_SIMS, SP_MCTS_BATCH, SP_CPUCT, SP_BATCH, SP_TEMP, SP_KOMI = 512, 200, 8, 1.5, 256, 7, 7.5
SP_WORKLOAD = ("C5: self-play 9x9, 6x64 network (C2), 200 playouts/move, c_puct 1.5, 512 games per GPU, "
               "inference batch 256, mcts batch 8, komi 7.5, 7 opening moves sampled, resignation off")


def conv_flops_per_position() -> float:
    """2 * F^2 * 9 * A per 3x3 tower convolution (one launch covers the batch)."""
    return 2.0 * FILTERS * FILTERS * 9 * BOARD * BOARD


def flops_per_position() -> float:
    A, F, P, V = BOARD * BOARD, FILTERS, 2 * HISTORY + 2, VALUE_HIDDEN
    return (2 * BLOCKS * conv_flops_per_position() + 2.0 * F * P * 9 * A
            + 2.0 * 3 * F * A + 2.0 * 2 * A * (A + 1) + 2.0 * A * V + 2.0 * V)


def measured_peaks() -> dict:
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return json.load(f)
    except (OSError, ValueError):
        return {}


def profiled_traffic() -> float | None:
    """DRAM bytes per conv launch from the committed ncu summary, if any."""
    path = os.path.join(ROOT, "profiles", "conv3x3_tc_pair_bf16_c4.md")
    try:
        for line in open(path):
            if line.startswith("traffic_bytes_per_launch:"):
                return float(line.split(":", 1)[1].strip())
    except OSError:
        pass
    return None


# --------------------------------------------------------------- clocks


class ClockSampler:
    """nvidia-smi sampled every 50 ms; started before the warm-up (the tool
    takes a moment to begin), kept to the samples taken inside the timed
    region [mark_start, mark_stop] (the nearest one if none falls inside)."""

    FIELDS = ("timestamp,index,pci.bus_id,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    REASONS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, bus_ids: list[str]):
        self.bus_ids = [b.lower() for b in bus_ids if b]
        self.proc = None
        self.out = None
        self.t0 = self.t1 = None

    def start(self):
        try:
            self.out = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "50"], stdout=self.out, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
            return self
        deadline = time.time() + 5.0   # until the first sample is written
        while time.time() < deadline and os.path.getsize(self.out.name) == 0:
            time.sleep(0.05)
        return self

    def mark_start(self):
        self.t0 = datetime.datetime.now()

    def mark_stop(self):
        self.t1 = datetime.datetime.now()

    def stop(self) -> dict | None:
        """Stops sampling; the summary of [mark_start, mark_stop]."""
        if self.proc is None:
            return None
        self._collect()
        return self.window(self.t0, self.t1)

    def _collect(self):
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            self.proc.wait()
        self.out.flush()
        self.out.seek(0)
        rows = [r.split(",") for r in self.out.read().splitlines() if r.strip()]
        self.out.close()
        os.unlink(self.out.name)
        self.samples = samples = []
        for r in rows:
            r = [c.strip() for c in r]
            if len(r) < 11:
                continue
            bus = r[2].lower()
            if self.bus_ids and not any(bus.endswith(b[-12:]) or b.endswith(bus[-12:]) for b in self.bus_ids):
                continue
            try:
                when = datetime.datetime.strptime(r[0], "%Y/%m/%d %H:%M:%S.%f")
                samples.append((when, float(r[3]), float(r[4]), r[7:11]))
            except ValueError:
                continue

    def window(self, t0, t1) -> dict | None:
        """Median SM clock, max clock and throttle reasons of the samples in [t0, t1]."""
        samples = getattr(self, "samples", None)
        if not samples:
            return None
        inside = samples
        if t0 and t1:
            slack = datetime.timedelta(seconds=0.1)
            inside = [x for x in samples if t0 - slack <= x[0] <= t1 + slack]
            if not inside:
                mid = t0 + (t1 - t0) / 2
                inside = [min(samples, key=lambda x: abs((x[0] - mid).total_seconds()))]
        reasons = set()
        for x in inside:
            for name, v in zip(self.REASONS, x[3]):
                if v.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(x[1] for x in inside), "sm_max_mhz": max(x[2] for x in inside),
                "reasons": sorted(reasons), "samples": len(inside)}


# ---------------------------------------------------------- distributed


class Dist:
    """One rank per GPU: RANK / LOCAL_RANK / WORLD_SIZE from the launcher.
    NCCL on the GPUs; gloo on the CPU (the multi-rank host tests)."""

    def __init__(self, gpus: int, backend: str | None = None):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.backend = backend or os.environ.get("AZB_DIST_BACKEND", "nccl")
        self.device = "cuda" if self.backend == "nccl" else "cpu"
        self.torch = None
        if self.world > 1:
            import datetime

            import torch
            import torch.distributed as dist

            timeout = datetime.timedelta(seconds=120)
            if self.device == "cuda":
                torch.cuda.set_device(self.local)
                dist.init_process_group("nccl", timeout=timeout, device_id=torch.device("cuda", self.local))
            else:
                dist.init_process_group(self.backend, timeout=timeout)
            self.torch = torch
        if gpus != self.world and self.rank == 0:
            print(f"bench: --gpus {gpus} but WORLD_SIZE {self.world}; using {self.world}", file=sys.stderr)

    def barrier(self):
        if self.torch:
            self.torch.distributed.barrier()
            if self.device == "cuda":
                self.torch.cuda.synchronize()

    def max(self, v: float) -> float:
        if not self.torch:
            return v
        t = self.torch.tensor([v], dtype=self.torch.float64, device=self.device)
        self.torch.distributed.all_reduce(t, op=self.torch.distributed.ReduceOp.MAX)
        return float(t.item())

    def sum(self, v: float) -> float:
        if not self.torch:
            return v
        t = self.torch.tensor([v], dtype=self.torch.float64, device=self.device)
        self.torch.distributed.all_reduce(t, op=self.torch.distributed.ReduceOp.SUM)
        return float(t.item())

    def broadcast(self, arr):
        """Rank 0's numpy array to every rank (once, at start: the weight replicas)."""
        if not self.torch:
            return arr
        import numpy as np

        t = self.torch.from_numpy(np.ascontiguousarray(arr)).to(self.device)
        self.torch.distributed.broadcast(t, src=0)
        return t.cpu().numpy().astype(np.float32, copy=False)

    def close(self):
        if self.torch:
            self.torch.distributed.barrier()
            self.torch.distributed.destroy_process_group()
            self.torch = None


# ----------------------------------------------------------- CPU arms


def cpu_reference_sample(steps: int, warmup: int, per_step_calls: int = 1, seconds: float = 0.0):
    """The reference's CPU engine (oracle/_ref, blas, single-threaded per
    worker as src/backend_blas.cpp:56-70 requires) on every host core.
    Returns (positions/s, workers, sample description)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O

    cfg = O.NetConfig(BOARD, HISTORY, BLOCKS, FILTERS, VALUE_HIDDEN, False)
    net = O.RefNetwork(cfg, SEED, O.KIND_BENCH)
    x = O.ref_positions(cfg, SEED, 8)
    cores = len(os.sched_getaffinity(0))
    try:
        import psutil

        avail = psutil.virtual_memory().available
        workers = max(1, min(cores, int(avail * 0.6 // (400 << 20))))   # ~300 MB of reference Workspace each
    except ImportError:
        workers = cores
    backend = "blas" if "OpenBLAS" in O.blas_description() else "naive"
    for _ in range(warmup):
        net.bench_workers(backend, workers, 8, x, max_calls=1)
    if seconds > 0:
        rate, pos = net.bench_workers(backend, workers, 8, x, seconds=seconds)
        sample = f"{workers} workers x batch 8, {pos} positions in ~{seconds:.0f} s ({backend}: {O.blas_description()})"
        return rate, workers, sample
    total_pos, total_t = 0, 0.0
    for _ in range(steps):
        t0 = time.perf_counter()
        _, pos = net.bench_workers(backend, workers, 8, x, max_calls=per_step_calls)
        total_t += time.perf_counter() - t0
        total_pos += pos
    sample = (f"{steps} steps x {workers} workers x {per_step_calls} call(s) of batch 8 = {total_pos} positions "
              f"({backend}: {O.blas_description()})")
    return total_pos / total_t, workers, sample


def cpu_batch_sample(batch: int = 16):
    """The reference's CPU engine at a large batch: one Network::infer call of
    `batch` C4 positions on one worker (its blas backend is single-threaded by
    design, src/backend_blas.cpp:56-70), after one untimed call of 1. A bounded
    stand-in for BASELINE.json's batch of 1024, which one worker would take
    minutes to evaluate; positions/s does not depend on the batch there."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O

    cfg = O.NetConfig(BOARD, HISTORY, BLOCKS, FILTERS, VALUE_HIDDEN, False)
    net = O.RefNetwork(cfg, SEED, O.KIND_BENCH)
    x = O.ref_positions(cfg, SEED, batch)
    backend = "blas" if "OpenBLAS" in O.blas_description() else "naive"
    net.infer(x[:1], backend)
    t0 = time.perf_counter()
    net.infer(x, backend)
    secs = time.perf_counter() - t0
    return {"value": batch / secs, "unit": UNIT, "cores": 1, "kind": "reference", "batch": batch,
            "sample": f"one Network::infer of {batch} positions on one worker ({backend}), {secs:.1f} s"}


def selfplay_cpu_sample(plies: int = 6):
    """The reference's self-play on its own CPU engine (blas, one worker per
    core; oracle/_ref/libazselfplay_ref.so): one game per worker, each cut at
    `plies` plies (move cap), so the sample ends in seconds."""
    sys.path.insert(0, os.path.join(ROOT, "alphazero-go_b200"))
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    import selfplay as SP   # ctypes over the library given below; it maps no engine library

    sp_desc = O.NetConfig(SP_BOARD, 1, SP_BLOCKS, SP_FILTERS, SP_VH, False)
    p, b = O.make_network(sp_desc, SEED, O.KIND_BENCH)   # the reference's seeded Network, restated
    workers = len(os.sched_getaffinity(0))
    lib = os.path.join(ROOT, "oracle", "_ref", "libazselfplay_ref.so")
    r = SP.play(sp_desc, p, b, backend="blas", workers=workers, simulations=SP_SIMS, mcts_batch=SP_MCTS_BATCH,
                c_puct=SP_CPUCT, temperature_moves=SP_TEMP, komi=SP_KOMI, max_moves=plies, seed=SEED, count=workers,
                lib_path=lib)
    return {"playouts_per_s": r["playouts_per_s"], "positions_evaluated_per_s": r["evaluations_per_s"],
            "cores": workers, "kind": "reference",
            "sample": f"{workers} games x {plies} plies on {workers} workers (blas), {r['positions']} positions in "
                      f"{r['seconds']:.1f} s"}


def refcuda_sample(steps: int = 2):
    """The reference's own CUDA engine (src/cuda, compiled unmodified for
    sm_100 by `make -C oracle refcuda`) on the same C4 workload: fp32, batch
    1024, wall clock of synchronous CudaInference::infer calls (host copies
    included, as that engine always does them), after one untimed call."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O

    if not O.refcuda_built():
        return {"unavailable": "oracle/_ref/libazrefcuda.so is not built (needs the reference tree)"}
    ok, why = O.refcuda_available()
    if not ok:
        return {"unavailable": why}
    cfg = O.NetConfig(BOARD, HISTORY, BLOCKS, FILTERS, VALUE_HIDDEN, False)
    p, b = O.make_network(cfg, SEED, O.KIND_BENCH)
    x = O.positions(cfg, SEED, BATCH)
    with O.RefCudaInference(cfg, p, b, BATCH) as net:
        secs = net.time(x, 1, steps)
    return {"value": BATCH * steps / secs, "unit": UNIT, "dtype": "f32", "batch": BATCH, "steps": steps,
            "engine": O.refcuda_description(),
            "how": "the reference's src/cuda engine (SIMT fp32) built for sm_100, CudaInference::infer, wall clock"}


def run_reference(args):
    n_gpus = int(os.environ.get("WORLD_SIZE", str(args.gpus)))
    try:
        rate, workers, sample = cpu_reference_sample(args.steps, args.warmup)
    except Exception as e:   # the reference build is missing or failed
        print(json.dumps({"impl": "reference", "unavailable": f"reference CPU engine failed: {e}"}))
        return
    line = {
        "metric": METRIC, "value": rate, "unit": UNIT, "n_gpus": n_gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": None, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": WORKLOAD.replace("batch 1024 per GPU", "batch 8 per CPU worker"),
                   "parallelism": f"{workers} CPU workers", "backend": "reference CPU (oracle/_ref)"},
        "impl": "reference",
        "cpu_baseline": {"value": rate, "unit": UNIT, "cores": workers, "kind": "reference", "sample": sample},
        "e2e": {"value": rate, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    try:
        line["cpu_batch"] = cpu_batch_sample()
    except Exception as e:
        line["cpu_batch"] = {"unavailable": f"reference CPU engine failed: {e}"}
    try:
        line["ref_cuda"] = refcuda_sample()
    except Exception as e:
        line["ref_cuda"] = {"unavailable": f"the reference's CUDA engine (oracle/_ref/libazrefcuda.so) failed: {e}"}
    if not args.no_selfplay:
        try:
            line["selfplay"] = {"workload": SP_WORKLOAD, **selfplay_cpu_sample()}
        except Exception as e:
            line["selfplay"] = {"workload": SP_WORKLOAD, "unavailable": f"reference self-play failed: {e}"}
    print(json.dumps(line))


# -------------------------------------------------------------- engine


def run_selfplay(d: "Dist", dev: int) -> dict | None:
    import azb200 as E
    import selfplay as SP

    sp_desc = E.NetDesc(SP_BOARD, 1, SP_BLOCKS, SP_FILTERS, SP_VH, 0)
    p, b = E.synth_network(sp_desc, SEED, 0)
    kw = dict(precision=E.TF32X3, simulations=SP_SIMS, mcts_batch=SP_MCTS_BATCH, c_puct=SP_CPUCT,
              temperature_moves=SP_TEMP, komi=SP_KOMI, max_moves=0, seed=SEED, generation=0,
              first=d.rank * SP_GAMES, count=SP_GAMES)
    out = {}
    # The engine's own hub (azb_hub), then the reference's InferenceHub over
    # the same engine: the same games (equal record hashes), two batchers.
    for name, play in (("engine_hub", lambda: SP.play_hub(sp_desc, p, b, devices=[dev], workers=SP_GAMES,
                                                          inference_batch=SP_BATCH, **kw)),
                       ("reference_hub", lambda: SP.play(sp_desc, p, b, backend="cuda", workers=SP_GAMES,
                                                         inference_batch=SP_BATCH, device=dev, **kw))):
        try:
            r, ok, err = play(), 1.0, ""
        except Exception as e:   # not built here, or failed: every rank still takes the same collectives
            r, ok, err = {"seconds": 0.0, "positions": 0, "evaluations": 0}, 0.0, str(e)
        secs = d.max(r["seconds"])
        pos, evals, oks = d.sum(float(r["positions"])), d.sum(float(r["evaluations"])), d.sum(ok)
        if oks < d.world:
            out[name] = {"unavailable": err if ok == 0.0 else "self-play failed on another rank"}
            continue
        out[name] = {"playouts_per_s": pos * SP_SIMS / secs, "positions_evaluated_per_s": evals / secs,
                     "positions": int(pos), "evaluations": int(evals), "seconds": secs,
                     "record_hash": r.get("record_hash")}
        if name == "engine_hub":
            out[name].update({"passes": r["passes"], "full_passes": r["full_passes"], "pass_cap": r["pass_cap"]})
    main = out.get("engine_hub", {})
    if "unavailable" in main or not main:
        main = out.get("reference_hub", {})
    if "playouts_per_s" not in main:
        return {"workload": SP_WORKLOAD, "unavailable": main.get("unavailable", "self-play failed")}
    return {"workload": SP_WORKLOAD, "playouts_per_s": main["playouts_per_s"],
            "positions_evaluated_per_s": main["positions_evaluated_per_s"], "games": SP_GAMES * d.world,
            "positions": main["positions"], "evaluations": main["evaluations"], "seconds": main["seconds"],
            "precision": "tf32x3 (the mode that meets the parity gate on this network)",
            "engine_hub": out.get("engine_hub"), "reference_hub": out.get("reference_hub"),
            "how": "the reference's playSelfPlayGame over this engine: playouts_per_s through the engine's own hub "
                   "(azb_hub); reference_hub: through the reference's InferenceHub and the bridge; one slice of "
                   "512 games per GPU, host wall clock, max over ranks"}


def runner_passes(runner, B: int, n: int) -> None:
    """n passes of B positions through the runner's C ABI, both slots kept in
    flight (each slot begins again as soon as its done() arrives)."""
    done_q, cv = [], threading.Condition()

    def done(slot, err):
        with cv:
            done_q.append((slot, err))
            cv.notify()

    inflight = started = 0
    for s in range(min(runner.slots(), n)):
        runner.begin(s, B, done)
        inflight += 1
        started += 1
    errors = []
    while inflight:
        with cv:
            while not done_q:
                cv.wait()
            slot, err = done_q.pop(0)
        inflight -= 1
        if err:
            errors.append(err)
        if started < n and not errors:
            runner.begin(slot, B, done)
            inflight += 1
            started += 1
    if errors:
        raise RuntimeError(errors[0])


def fp32_class_records(d: "Dist", E, desc, params, buffers, x, dev: int, steps: int) -> dict:
    """C4 in TF32X3 and TF32 on this rank's batch: device passes (CUDA
    events, inputs resident), the runner's C ABI with 2 slots and host copies
    (wall clock), and the tower conv's rate (events around each launch).
    Positions/s are summed over ranks from the max-over-ranks times."""
    out = {}
    for pname, prec in (("tf32x3", E.TF32X3), ("tf32", E.TF32)):
        with E.CudaInference(desc, params, buffers, BATCH, dev, prec) as net:
            net.stage(x)
            net.time(BATCH, 0, 2)
            d.barrier()
            ms, _ = net.time(BATCH, 0, steps)
            _, conv_ms = net.time(BATCH, 0, 2, conv=True)
        ms, conv_avg_ms = d.max(ms), d.max(conv_ms / (2 * 2 * BLOCKS))
        runner = E.make_cuda_runner(desc, params, buffers, BATCH, 2, dev, prec)
        for sl in range(2):
            runner.input(sl)[:] = x
        runner_passes(runner, BATCH, 2)
        d.barrier()
        t0 = time.perf_counter()
        runner_passes(runner, BATCH, steps)
        run_s = d.max(time.perf_counter() - t0)
        runner.close()
        out[pname] = {"positions_per_s": d.world * BATCH * steps / (ms / 1e3),
                      "e2e_positions_per_s": d.world * BATCH * steps / run_s,
                      "conv_tflops": conv_flops_per_position() * BATCH / (conv_avg_ms * 1e-3) / 1e12,
                      "ms_per_pass": ms / steps, "steps": steps}
    out["how"] = ("C4 at batch 1024 per GPU; positions_per_s: device passes by CUDA events (inputs resident); "
                  "e2e_positions_per_s: BatchRunner C ABI, 2 slots, host copies, wall clock; conv_tflops: events "
                  "around every tower conv (useful FLOPs: one product per MAC, whatever the mode's MMA count)")
    out["parity"] = "tf32x3: maxErr <= 1e-4 vs the reference forward (tests/test_gpu_gates.py); tf32: reported"
    return out


def run_engine(args, d: Dist):
    import numpy as np

    import azb200 as E

    dev = d.local if d.world > 1 else 0
    ok, why = E.cuda_available(dev)
    if not ok:
        raise SystemExit(f"bench: no usable GPU {dev}: {why}")
    desc = E.NetDesc(BOARD, HISTORY, BLOCKS, FILTERS, VALUE_HIDDEN, 0)
    precision = E.BF16
    if d.rank == 0:
        params, buffers = E.synth_network(desc, SEED, 0)
    else:
        np_, nb = E.arena_floats(desc)
        params, buffers = np.zeros(np_, np.float32), np.zeros(nb, np.float32)
    params, buffers = d.broadcast(params), d.broadcast(buffers)
    x = E.synth_positions(desc, SEED, BATCH, first=d.rank * BATCH)
    net = E.CudaInference(desc, params, buffers, BATCH, dev, precision)
    net.stage(x)

    # --- device-resident throughput: W untimed, then exactly K timed passes
    sampler = ClockSampler([E.pci_bus_id(dev)] if d.world == 1 else []).start() if d.rank == 0 else None
    net.time(BATCH, 0, args.warmup)
    d.barrier()
    if sampler:
        sampler.mark_start()
    ms, _ = net.time(BATCH, 0, args.steps)
    d.barrier()
    if sampler:
        sampler.mark_stop()
    ms = d.max(ms)
    value = d.world * BATCH * args.steps / (ms / 1e3)

    # --- the conv kernel alone, per launch: CUDA events around each launch.
    # The events stop programmatic dependent launch from overlapping a
    # launch's start with its predecessor's tail, so this is a lower bound
    # on the kernel's rate inside a pass (the whole-pass figure is higher).
    roof_passes = max(2, min(args.steps, 5))
    roof_t0 = datetime.datetime.now()
    r0 = time.perf_counter()
    _, conv_ms = net.time(BATCH, 0, roof_passes, conv=True)
    roof_s = time.perf_counter() - r0
    roof_t1 = datetime.datetime.now()
    clocks = sampler.stop() if sampler else None
    roof_clocks = sampler.window(roof_t0, roof_t1) if sampler else None
    conv_launches = 2 * BLOCKS * roof_passes
    conv_avg_ms = d.max(conv_ms / conv_launches)
    conv_tflops = conv_flops_per_position() * BATCH / (conv_avg_ms * 1e-3) / 1e12

    if args.only_device:
        net.close()
        if d.rank == 0:
            print(json.dumps({"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": d.world,
                              "ms_per_step": ms / args.steps, "conv_avg_ms": conv_avg_ms,
                              "conv_tflops": conv_tflops, "note": "device-only run (profiling)"}))
        d.close()
        return

    # --- end to end through the runner (the BatchRunner drop-in), 2 slots in flight
    runner = E.make_cuda_runner(desc, params, buffers, BATCH, 2, dev, precision)
    for s in range(2):
        runner.input(s)[:] = x
    runner_passes(runner, BATCH, args.warmup)
    d.barrier()
    t0 = time.perf_counter()
    runner_passes(runner, BATCH, args.steps)
    e2e_s = time.perf_counter() - t0
    d.barrier()
    e2e_s = d.max(e2e_s)
    runner.close()
    e2e = d.world * BATCH * args.steps / e2e_s

    # --- the same workload in the fp32-class modes (the reference's CUDA
    # engine computes in fp32): TF32X3 meets the 1e-4 gate, TF32 is reported
    fp32_class = fp32_class_records(d, E, desc, params, buffers, x, dev, min(args.steps, 10))

    # --- end to end from position records (the device encoder): one synchronous
    # CudaInference call per pass, records in and logits/values out every pass
    stones = np.zeros((BATCH, 1, BOARD * BOARD), np.uint8)
    to_move = np.where(x[:, 2, 0] == 1.0, 1, 2).astype(np.uint8)
    for b in range(BATCH):
        own, opp = (1, 2) if to_move[b] == 1 else (2, 1)
        stones[b, 0][x[b, 0] == 1.0] = own
        stones[b, 0][x[b, 1] == 1.0] = opp
    records = E.stones_records(stones, to_move)
    for _ in range(args.warmup):
        net.infer_stones(records)
    d.barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        net.infer_stones(records)
    rec_s = d.max(time.perf_counter() - t0)
    e2e_records = {"value": d.world * BATCH * args.steps / rec_s, "unit": UNIT,
                   "h2d_bytes_per_step": int(records.nbytes) * d.world,
                   "d2h_bytes_per_step": (BATCH * (BOARD * BOARD + 1) * 4 + BATCH * 4 + 4) * d.world,
                   "how": "CudaInference from position records (planes encoded on the device), one synchronous "
                          "call per pass, host wall clock, max over ranks"}
    net.close()

    # --- CPU baseline: the reference's CPU engine on this box's cores (rank 0, N = 1)
    cpu = None
    if d.world == 1 and not args.no_cpu_baseline:
        try:
            rate, workers, sample = cpu_reference_sample(0, 0, seconds=args.cpu_seconds)
            cpu = {"value": rate, "unit": UNIT, "cores": workers, "kind": "reference", "sample": sample}
        except Exception as e:
            cpu = {"value": None, "unit": UNIT, "cores": 0, "kind": "reference", "sample": f"unavailable: {e}"}

    # --- self-play (C5): the reference's search and hub on this engine, one
    # slice of 512 games per rank (games [rank*512, (rank+1)*512)), host
    # wall clock of the slice; playouts/s = positions x 200 / seconds
    selfplay = None
    if not args.no_selfplay:
        selfplay = run_selfplay(d, dev)
        if selfplay and d.world == 1 and not args.no_cpu_baseline:
            try:
                selfplay["cpu_baseline"] = selfplay_cpu_sample()
            except Exception as e:
                selfplay["cpu_baseline"] = {"unavailable": f"reference self-play failed: {e}"}

    if d.rank == 0:
        peaks = measured_peaks()
        peak = peaks.get("bf16_tflops_sustained")
        peak_note = "measured sustained bf16 (MEASURED_PEAKS.json)"
        if peak is None:
            peak, peak_note = 1400.0, "fallback sustained bf16"
        traffic = profiled_traffic()
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": d.world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": WORKLOAD, "global_batch": BATCH * d.world, "parallelism": f"replicas x{d.world}",
                       "precision": "bf16 weights/activations, fp32 accumulate",
                       "l2": "inputs larger than L2 (3 x 189 MB activation frames per GPU)",
                       "flop_per_position": flops_per_position()},
            "e2e": {"value": e2e, "unit": UNIT, "h2d_bytes_per_step": BATCH * 4 * BOARD * BOARD * 4 * d.world,
                    "d2h_bytes_per_step": (BATCH * (BOARD * BOARD + 1) * 4 + BATCH * 4 + 4) * d.world,
                    "how": "BatchRunner C ABI, 2 slots in flight, host wall clock, max over ranks"},
            "roofline": {"bound": "tensor", "achieved": conv_tflops, "peak": peak, "unit": "TFLOP/s",
                         "frac": conv_tflops / peak, "traffic": traffic, "peak_source": peak_note,
                         "kernel": "conv3x3_tc_pair<256,bf16>", "flop_per_launch": conv_flops_per_position() * BATCH,
                         "avg_launch_ms": conv_avg_ms, "launches": conv_launches, "timed_region_s": roof_s,
                         "sm_mhz": roof_clocks["sm_mhz"] if roof_clocks else None,
                         "how": "CUDA events around every conv launch of the passes (which stops each launch "
                                "overlapping its predecessor's tail: a lower bound on the in-pass rate)"},
            "tensor_tflops_whole_pass": flops_per_position() * BATCH * d.world * args.steps / (ms / 1e3) / 1e12,
            "gpu_launches": args.steps * (2 * BLOCKS + 5),   # stem operand + stem GEMM + tower + 3 head launches
            "clocks": clocks,
            "cpu_baseline": cpu,
            "e2e_records": e2e_records,
            "fp32_class": fp32_class,
        }
        if selfplay is not None:
            line["selfplay"] = selfplay
        print(json.dumps(line))
    d.close()


# ---------------------------------------------------------------- sweep

SWEEP = {   # BASELINE.json configs[0..3]: (board, blocks, filters, value_hidden, batch)
    "C1": (5, 4, 32, 64, 64), "C2": (9, 6, 64, 128, 256), "C3": (19, 10, 128, 256, 256), "C4": (19, 20, 256, 256, 1024),
}


def cpu_model() -> str:
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def run_profile_case(args):
    """Device-resident passes of one configuration and precision, for ncu:
    `--profile-case C2:tf32x3` runs W + K passes of C2 at its batch."""
    import azb200 as E

    name, _, pname = args.profile_case.partition(":")
    n, blocks, filters, vh, B = SWEEP[name]
    B = args.batch or B
    prec = {"tf32x3": E.TF32X3, "tf32": E.TF32, "bf16": E.BF16}[pname or "bf16"]
    desc = E.NetDesc(n, 1, blocks, filters, vh, 0)
    params, buffers = E.synth_network(desc, SEED, 0)
    with E.CudaInference(desc, params, buffers, B, 0, prec) as net:
        net.stage(E.synth_positions(desc, SEED, B))
        ms, _ = net.time(B, args.warmup, args.steps)
    print(json.dumps({"case": args.profile_case, "batch": B, "ms_per_pass": ms / args.steps,
                      "positions_per_s": B * args.steps / (ms / 1e3)}))


def run_sweep(args):
    """One JSON line per configuration C1..C4: this engine in each precision
    (device-resident passes timed by CUDA events, and the runner's C ABI with
    2 slots in flight, host wall clock), the reference's CPU engines (blas
    and naive, one single-threaded worker per core at batch 8, bounded) and
    the reference's own CUDA engine rebuilt for sm_100 at the config's batch."""
    import numpy as np

    import azb200 as E

    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O

    ok, why = E.cuda_available(0)
    if not ok:
        raise SystemExit(f"bench: no usable GPU: {why}")
    cores = len(os.sched_getaffinity(0))
    for name, (n, blocks, filters, vh, B) in SWEEP.items():
        desc = E.NetDesc(n, 1, blocks, filters, vh, 0)
        cfg = O.NetConfig(n, 1, blocks, filters, vh, False)
        params, buffers = E.synth_network(desc, SEED, 0)
        x = E.synth_positions(desc, SEED, B)
        conv_flop = 2.0 * filters * filters * 9 * n * n * B
        line = {"config": name, "board": n, "blocks": blocks, "filters": filters, "value_hidden": vh, "batch": B,
                "engine": {}, "host": {"cores": cores, "cpu": cpu_model()}}
        for pname, prec in (("tf32x3", E.TF32X3), ("tf32", E.TF32), ("bf16", E.BF16)):
            with E.CudaInference(desc, params, buffers, B, 0, prec) as net:
                net.stage(x)
                steps = 50 if B * n * n * filters < 1 << 26 else 10
                # Passes as they run (events around the timed loop only), then
                # the conv kernels alone (events around every launch).
                ms, _ = net.time(B, 5, steps)
                _, conv_ms = net.time(B, 2, steps, conv=True)
            runner = E.make_cuda_runner(desc, params, buffers, B, 2, 0, prec)
            for sl in range(2):
                runner.input(sl)[:] = x
            runner_passes(runner, B, 3)
            t0 = time.perf_counter()
            runner_passes(runner, B, steps)
            run_s = time.perf_counter() - t0
            runner.close()
            line["engine"][pname] = {"positions_per_s": B * steps / (ms / 1e3),
                                     "runner_positions_per_s": B * steps / run_s,
                                     "conv_tflops": conv_flop / (conv_ms / (steps * 2 * blocks) * 1e-3) / 1e12}
        ref = {}
        try:
            net = O.RefNetwork(cfg, SEED, O.KIND_BENCH)
            x8 = O.ref_positions(cfg, SEED, 8)
            backends = ["blas"] if "OpenBLAS" in O.blas_description() else []
            for be in backends + ["naive"]:
                if be == "naive" and name == "C4":
                    rate, pos = net.bench_workers(be, cores, 1, x8[:1], max_calls=1)   # ~10 s per call
                    sample = f"{cores} workers x 1 call of batch 1"
                else:
                    rate, pos = net.bench_workers(be, cores, 8, x8, seconds=4.0)
                    sample = f"{cores} workers x batch 8, ~4 s"
                ref[be] = {"positions_per_s": rate, "sample": sample}
        except Exception as e:
            ref["error"] = str(e)
        try:
            if O.refcuda_built() and O.refcuda_available()[0]:
                p, b = O.make_network(cfg, SEED, O.KIND_BENCH)
                xs = O.positions(cfg, SEED, B)
                with O.RefCudaInference(cfg, p, b, B) as rnet:
                    steps = 10 if name != "C4" else 2
                    secs = rnet.time(xs, 1, steps)
                ref["cuda_sm100"] = {"positions_per_s": B * steps / secs, "dtype": "f32"}
        except Exception as e:
            ref["cuda_sm100_error"] = str(e)
        line["reference"] = ref
        print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=60)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("engine", "reference"), default="engine")
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-selfplay", action="store_true", help="skip the C5 self-play figures")
    ap.add_argument("--only-device", action="store_true", help="device-resident passes only (for profilers)")
    ap.add_argument("--profile-case", default=None, help="CONFIG:PRECISION, e.g. C2:tf32x3: device passes only, for ncu")
    ap.add_argument("--batch", type=int, default=0, help="--profile-case: positions per pass (default: the config's)")
    ap.add_argument("--sweep", action="store_true",
                    help="one JSON line per configuration C1..C4: every precision, runner, and the reference's engines")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.sweep:
        run_sweep(args)
        return
    if args.profile_case:
        run_profile_case(args)
        return
    if args.impl == "reference":
        # The reference arm is CPU-only: rank 0 runs it, the other ranks exit
        # at once (no process group, so nobody waits on anybody).
        if int(os.environ.get("RANK", "0")) == 0:
            run_reference(args)
        return
    run_engine(args, Dist(args.gpus))


if __name__ == "__main__":
    main()
