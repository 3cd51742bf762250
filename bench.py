"""Benchmark of the early-exit hot path (router -> compaction -> scatter).

Default workload per GPU ("llama8b_prefill_checkpoints"): the checkpoint
sweep of a Llama-3.1-8B-architecture prefill batch of 16 x 2048 tokens =
32768 rows of H = 4096 bf16 hidden states, routers at layers 8/12/16/20/24/28
(RMSNorm eps 1e-5, router 4096 -> 128 -> 1) with biases placed so that
5/10/15/20/20/30 % of the batch exits at each checkpoint (everything by layer
28).  Each checkpoint reads its own synthetic hidden-state tensor (rows
N(0,1), the hidden states of the still-active tokens at that layer), scores
it, compacts survivors (rows, int64 positions, int32 KV slots) into a dense
buffer and writes exits, final-normed, to their original positions.  Active
counts chain on the device between checkpoints (no host sync).  One step =
the six checkpoints.  Inputs (1.1 GiB per step) exceed the 126 MB L2, so no
explicit flush is needed between steps.  The same run also measures the
8B-architecture prefill through the engine (random-init Llama-3.1-8B
architecture, bf16, batch 16 x 2048 split over the ranks): engine(input_ids)
against the model's own forward, 3 warm-up and 10 timed calls each; and the
same for a GPT-2-small-architecture model (fp16, LayerNorm, batch 8 x 512,
routers at layers 4 and 8 exiting ~20 % of the tokens at each).

Inputs: the first CAL_ROWS rows of every checkpoint's tensor and every
router's weights come from a CPU torch.Generator, so the CPU reference arm
sees bit-identical rows; the router biases are placed on those rows (both
arms compute the same biases).  The rest of the rows are drawn on the device.

Other workloads (--workload):
  qwen3_8b_decode_checkpoints  one decode step of a Qwen3-8B-architecture
      batch of 256 sequences, routers at layers 3/7/.../31 (eight
      checkpoints, H = 4096), each exiting ~10 % of the rows still active;
  kernel_fp32_4096x768  the reference's own kernel-level case, one
      checkpoint of 4096 fp32 rows of H = 768 (N(0,1) times a per-row scale
      U(0.5, 2)), RMSNorm weight N(1, 0.02), 30 % exits;
  bandwidth_sweep  one checkpoint per (N, H, f): N in 1K..1M rows (powers of
      4, split evenly over the ranks), H in {2048, 4096, 5120, 8192} bf16,
      exit fraction f in {0, 0.1, 0.5, 0.9}; HBM GB/s against the measured
      copy peak for each;
  llama8b_prefill_engine  the engine prefill measurements alone.

Multi-GPU: one process per GPU under torchrun; every rank processes its own
batch (weak scaling).  The step's exit counts are all-gathered (NCCL) inside
the timed region, overlapped with the next step on a second stream; timing
is the max over ranks.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                  [--workload NAME] [--no-engine]
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import tempfile
import threading
import time
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

THRESHOLD = 0.85
SEED = 1234
CAL_ROWS = 8192  # CPU-drawn rows per checkpoint: bias calibration and the CPU sample
WORKLOADS = {
    # exits: fraction of the whole batch per checkpoint (the last takes the rest)
    "llama8b_prefill_checkpoints": {"rows": 16 * 2048, "layers": [8, 12, 16, 20, 24, 28],
                                    "exit_fractions": [0.05, 0.10, 0.15, 0.20, 0.20, 0.30],
                                    "of": "batch"},
    # exits: fraction of the rows still active at each checkpoint
    "qwen3_8b_decode_checkpoints": {"rows": 256, "layers": [3, 7, 11, 15, 19, 23, 27, 31],
                                    "exit_fractions": [0.10] * 8, "of": "active"},
    # one router over fp32 rows scaled per row, RMSNorm weight N(1, 0.02)
    "kernel_fp32_4096x768": {"rows": 4096, "layers": [0], "exit_fractions": [0.30],
                             "of": "active", "hidden": 768, "dtype": "f32", "inputs": "k1"},
}
# workloads that are not a checkpoint sweep
SWEEP_WORKLOAD = "bandwidth_sweep"
ENGINE_WORKLOAD = "llama8b_prefill_engine"
DECODE_WORKLOAD = "qwen3_8b_decode_generate"
ATTN_WORKLOAD = "qwen3_8b_decode_attention"
SWEEP_N = [1024, 4096, 16384, 65536, 262144, 1048576]
SWEEP_H = [2048, 4096, 5120, 8192]
SWEEP_F = [0.0, 0.1, 0.5, 0.9]
DTYPE_NAMES = {"bf16": torch.bfloat16, "f32": torch.float32}
WORKLOAD = "llama8b_prefill_checkpoints"
LAYERS = WORKLOADS[WORKLOAD]["layers"]
EXIT_FRACTIONS = WORKLOADS[WORKLOAD]["exit_fractions"]
EXITS_OF = WORKLOADS[WORKLOAD]["of"]
ROWS, HIDDEN, BOTTLENECK = WORKLOADS[WORKLOAD]["rows"], 4096, 128
DTYPE = "bf16"


def configure(name: str, rows: int | None = None) -> None:
    """Select a checkpoint-sweep workload (module globals used below)."""
    wk = WORKLOADS[name]
    globals().update(WORKLOAD=name, LAYERS=wk["layers"], EXIT_FRACTIONS=wk["exit_fractions"],
                     EXITS_OF=wk["of"], ROWS=rows if rows else wk["rows"],
                     HIDDEN=wk.get("hidden", 4096), DTYPE=wk.get("dtype", "bf16"))


# DRAM bytes (read + write) of checkpoint 0's two kernels (router + mover),
# 32768 rows x 4096 bf16, from an ncu capture of those two launches in this
# benchmark's third warm-up step on the split path, caches left as the
# previous kernels left them.
NCU_TRAFFIC_CKPT0 = {"rows": 32768, "path": "tc_split",
                     "bytes": (269.6 + 58.3 + 219.1 + 209.1) * 1e6}


def e2e_step_count(requested, h2d_bytes_per_step: int) -> int:
    """Steps of the e2e region: as requested, else enough for about 8 GB of
    host-to-device copies (at least 6, at most 200), so that a small
    workload's region is not a few hundred microseconds of host jitter and
    the copies of consecutive steps reach their pipelined rate (the first
    step's load is not overlapped).  The bytes are those one step actually
    copies."""
    if requested is not None:
        return int(requested)
    return max(6, min(200, int(8e9 // max(int(h2d_bytes_per_step), 1))))


def algorithmic_bytes(n: int, exits: int, h: int, e: int) -> int:
    """Bytes a single pass must move for one checkpoint of n rows: read every
    row and write it once (survivor to the dense buffer, exit to its
    position), fp32 score + u8 decision + int32 source index per row, read
    int64 position + int32 slot per row, write position + slot per survivor."""
    return n * 2 * h * e + 21 * n + 12 * (n - exits)


def nominal_schedule(rows: int) -> tuple[list[int], list[int]]:
    """(active rows, exits) per checkpoint of the workload's exit schedule."""
    active, exits, a = [], [], rows
    for k in range(len(LAYERS)):
        if EXITS_OF == "batch":
            e = int(round(EXIT_FRACTIONS[k] * rows)) if k < len(LAYERS) - 1 else a
        else:
            e = int(round(EXIT_FRACTIONS[k] * a))
        e = min(e, a)
        active.append(a)
        exits.append(e)
        a -= e
    return active, exits


# ----------------------------------------------------------------- clocks
class ClockSampler:
    """Samples SM clock and throttle reasons through NVML while running."""

    def __init__(self, index: int, period: float = 0.02):
        self.index, self.period = index, period
        self.samples: list[tuple[int, int]] = []
        self.max_mhz = None
        self._stop = threading.Event()
        self._t = None

    def __enter__(self):
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nv = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(self.index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        except Exception as exc:  # NVML missing: clocks reported as unknown
            self._err = str(exc)
        return self

    def _run(self):
        nv = self._nv
        while not self._stop.is_set():
            try:
                mhz = nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM)
                reasons = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                self.samples.append((mhz, reasons))
            except Exception:
                pass
            time.sleep(self.period)

    def __exit__(self, *a):
        self._stop.set()
        if self._t:
            self._t.join()

    def summary(self) -> dict:
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unsampled"]}
        names = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
                 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
                 0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting"}
        seen = set()
        for _, r in self.samples:
            for bit, name in names.items():
                if r & bit:
                    seen.add(name)
        return {"sm_mhz": statistics.median(m for m, _ in self.samples),
                "sm_max_mhz": self.max_mhz, "reasons": sorted(seen), "samples": len(self.samples)}


# ----------------------------------------------------------------- setup
def dist_setup(n_gpus: int):
    from tide_b200 import dist as tdist

    return tdist.init("nccl" if int(os.environ.get("WORLD_SIZE", "1")) > 1 else None,
                      timeout_s=120.0)


def barrier(world):
    from tide_b200 import dist as tdist

    tdist.barrier(world)


def max_over_ranks(world, v: float) -> float:
    from tide_b200 import dist as tdist

    return tdist.max_over_ranks(world, v)


def norm_weight_cpu() -> torch.Tensor:
    if WORKLOADS[WORKLOAD].get("inputs") == "k1":
        from tide_b200 import workloads

        return workloads.k1(n=ROWS, h=HIDDEN)["norm_weight"]
    return torch.ones(HIDDEN)


def checkpoint_setup(k: int, rank: int, active_nominal: int, exits_nominal: int) -> dict:
    """The CPU-drawn part of checkpoint k on a rank: the first
    min(CAL_ROWS, rows) rows of its hidden-state tensor (model dtype), its
    router (down [B, H], up [1, B], fp32) and the scalar bias that makes the
    nominal share of those rows (the first active_nominal of them) exit.
    Both arms call this, so they see the same rows, weights and biases."""
    from tide_b200 import workloads

    dt = DTYPE_NAMES[DTYPE]
    cal = min(CAL_ROWS, ROWS)
    if WORKLOADS[WORKLOAD].get("inputs") == "k1":
        w = workloads.k1(n=ROWS, h=HIDDEN, b=BOTTLENECK, seed=0)  # the reference's seed-0 draw
        x, down, up = w["x"][:cal].to(dt), w["down"], w["up"]
    else:
        g = torch.Generator().manual_seed(SEED + 7919 * rank + 101 * k)
        x = torch.randn(cal, HIDDEN, generator=g).to(dt)
        down = 0.02 * torch.randn(BOTTLENECK, HIDDEN, generator=g)
        up = 0.02 * torch.randn(1, BOTTLENECK, generator=g)
    n_cal = min(cal, active_nominal)
    z = workloads.prebias_logits_torch(x[:n_cal], "rms", norm_weight_cpu(), None, 1e-5, down, up)
    frac = exits_nominal / active_nominal if active_nominal else 0.0
    bias = workloads.bias_for_exit_fraction(z, frac, THRESHOLD)
    return {"x_head": x, "down": down, "up": up, "bias": bias}


class Workload:
    """Device-resident inputs and buffers of one rank's checkpoint sweep."""

    def __init__(self, rank: int, path: int):
        from tide_b200.capi import NORM_RMS
        from tide_b200.ops import CheckpointRunner, NormSpec, prepare_router

        dev = torch.device("cuda")
        g = torch.Generator(device=dev).manual_seed(SEED + 31 * rank)
        self.path = path
        dt = DTYPE_NAMES[DTYPE]
        self.norm = NormSpec(NORM_RMS, norm_weight_cpu().to(dev), None, 1e-5)
        self.runner = CheckpointRunner(dev)
        self.x, self.routers, self.setups = [], [], []
        self.active_nominal, self.exits_nominal = nominal_schedule(ROWS)
        scaled = WORKLOADS[WORKLOAD].get("inputs") == "k1"
        for k in range(len(LAYERS)):
            s = checkpoint_setup(k, rank, self.active_nominal[k], self.exits_nominal[k])
            head = s["x_head"].to(dev)
            rest = ROWS - head.shape[0]
            if rest > 0:
                xr = torch.randn(rest, HIDDEN, generator=g, device=dev)
                if scaled:
                    xr = xr * (torch.rand(rest, 1, generator=g, device=dev) * 1.5 + 0.5)
                x = torch.cat([head, xr.to(dt)])
            else:
                x = head.contiguous()
            self.routers.append(prepare_router(s["down"].to(dev), s["up"].to(dev), s["bias"],
                                               self.norm, dt))
            self.setups.append({"down": s["down"], "up": s["up"], "bias": s["bias"]})
            self.x.append(x)
        self.positions0 = torch.arange(ROWS, device=dev, dtype=torch.int64)
        self.slots0 = torch.arange(ROWS, device=dev, dtype=torch.int32)
        self.out = torch.zeros(ROWS, HIDDEN, dtype=dt, device=dev)
        self.compact = torch.empty(ROWS, HIDDEN, dtype=dt, device=dev)
        self.pos = [torch.empty(ROWS, dtype=torch.int64, device=dev) for _ in range(2)]
        self.slots = [torch.empty(ROWS, dtype=torch.int32, device=dev) for _ in range(2)]
        self.counts = torch.zeros(len(LAYERS), 2, dtype=torch.int32, device=dev)
        self.paths = {}  # path the library chose for each checkpoint

    def checkpoint(self, k: int, xs=None, scores_out=None):
        """Checkpoint k of the sweep: positions, slots and the live row count
        come from checkpoint k-1's outputs on the device."""
        xs = xs if xs is not None else self.x
        if k == 0:
            pos_in, slot_in, cnt = self.positions0, self.slots0, None
        else:
            pos_in, slot_in, cnt = self.pos[(k - 1) % 2], self.slots[(k - 1) % 2], self.counts[k - 1, :1]
        self.runner.run(xs[k], self.routers[k], self.norm, THRESHOLD, positions=pos_in,
                        slots=slot_in, out_buffer=self.out, compact_out=self.compact,
                        positions_out=self.pos[k % 2], slots_out=self.slots[k % 2],
                        n_rows_dev=cnt, counts=self.counts[k], path=self.path,
                        scores_out=scores_out)
        self.paths[k] = self.runner.last_path

    def step(self, xs=None):
        for k in range(len(LAYERS)):
            self.checkpoint(k, xs)

    def capture(self, xs=None, per_checkpoint: bool = False, calls: int = 1):
        """CUDA graphs of the sweep: one graph for the whole step (its kernels
        overlap their neighbours' prologues through programmatic dependent
        launch, kernel to kernel), or one graph per checkpoint.  The graphs
        hold kernels only; timing events and host copies stay outside."""
        out = []
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            groups = ([[k] * calls for k in range(len(LAYERS))] if per_checkpoint
                      else [list(range(len(LAYERS)))])
            for ks in groups:
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=s):
                    for k in ks:
                        self.checkpoint(k, xs)
                out.append(g)
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        return out


# calls of one checkpoint per timing graph (the per-checkpoint roofline times)
CK_CALLS = 8


def launches_per_checkpoint(path_used: int) -> int:
    """Kernels of ours per checkpoint call: one for the fused single-pass
    kernel, two (router + stable-partition move) otherwise."""
    from tide_b200.capi import PATH_TC

    return 1 if path_used == PATH_TC else 2


PATH_NAMES = {1: "simt", 2: "tc_fused_single_pass", 3: "tc_split"}


def parity_sample(wl: "Workload", active: list[int], rows: int = 2048) -> dict:
    """Scores of the timed path against the oracle on the first `rows` rows of
    every checkpoint (untimed calls with the same arguments plus a score
    output): the largest score difference and the exit decisions that differ,
    in total and outside the score tolerance around the threshold."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import tide_oracle as O

    f32 = DTYPE == "f32"
    tol = 1e-5 if f32 else 1e-2
    odt = O.F32 if f32 else O.BF16
    norm = {"kind": "rms", "weight": wl.norm.weight.cpu().numpy(), "bias": None, "eps": 1e-5}
    res = {"rows_checked": 0, "score_tolerance": tol, "max_score_err": 0.0,
           "decision_disagreements": 0, "disagreements_outside_tolerance": 0}
    for k in range(len(LAYERS)):
        n = active[k]
        if n == 0:
            continue
        s = torch.full((wl.x[k].shape[0],), -1.0, device="cuda")  # capacity rows
        wl.checkpoint(k, scores_out=s)
        torch.cuda.synchronize()
        m = min(rows, n)
        x = wl.x[k][:m]
        xs = x.cpu().numpy() if f32 else x.view(torch.int16).cpu().numpy().view(np.uint16)
        st = wl.setups[k]
        ref = O.score_rows(xs, odt, norm, st["down"].numpy(), st["up"].numpy(), st["bias"])
        got = s[:m].cpu().numpy()
        dis = (got > THRESHOLD) != (ref > THRESHOLD)
        res["rows_checked"] += m
        res["max_score_err"] = max(res["max_score_err"], float(np.abs(got - ref).max()))
        res["decision_disagreements"] += int(dis.sum())
        res["disagreements_outside_tolerance"] += int((dis & (np.abs(ref - THRESHOLD) > tol)).sum())
    return res


def gather_timings(world: int, wl: "Workload", reps: int = 5) -> dict:
    """The output-row collective, timed on its own: every rank's output rows
    gathered to every rank (ncclAllGather over NVLink).  The path never
    needs it (each rank's rows are consumed by its own lm_head); it is the
    cost of a consumer that wants all rows in one place.  CUDA events, max
    over ranks."""
    from tide_b200 import dist as tdist

    rows_out = torch.empty((world * ROWS, HIDDEN), dtype=wl.out.dtype, device=wl.out.device)
    nbytes = wl.out.numel() * wl.out.element_size()
    tdist.all_gather_rows(world, wl.out, rows_out)
    torch.cuda.synchronize()
    barrier(world)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(reps):
        tdist.all_gather_rows(world, wl.out, rows_out)
    b.record()
    torch.cuda.synchronize()
    ms = max_over_ranks(world, a.elapsed_time(b) / reps)
    del rows_out
    return {"output_rows_all_gather": {"ms": ms, "bytes_per_rank": nbytes,
                                       "busbw_GBps": (world - 1) * nbytes / (ms / 1000.0) / 1e9}}


class CountsGather:
    """The step's collective: every rank's {survivors, exits} per checkpoint
    all-gathered (global ExitStats need them), on a second stream so that it
    overlaps the next step.  Two staging buffers: step i's counts are copied
    on the main stream, gathered on the side stream, and the copy into a
    buffer waits for the gather that last read it."""

    def __init__(self, world: int, counts: torch.Tensor):
        self.world = world
        self.side = torch.cuda.Stream()
        self.stage = [torch.empty_like(counts) for _ in range(2)]
        self.out = [torch.empty((world,) + tuple(counts.shape), dtype=counts.dtype,
                                device=counts.device) for _ in range(2)]
        self.done = [None, None]
        self.i = 0

    def after_step(self, counts: torch.Tensor) -> None:
        import torch.distributed as dist

        j = self.i % 2
        main = torch.cuda.current_stream()
        if self.done[j] is not None:
            main.wait_event(self.done[j])
        self.stage[j].copy_(counts)
        ready = torch.cuda.Event()
        ready.record(main)
        self.side.wait_event(ready)
        with torch.cuda.stream(self.side):
            dist.all_gather_into_tensor(self.out[j].view(-1), self.stage[j].view(-1))
            ev = torch.cuda.Event()
            ev.record(self.side)
        self.done[j] = ev
        self.i += 1

    def finish(self) -> None:
        torch.cuda.current_stream().wait_stream(self.side)


# ----------------------------------------------------------------- CPU leg
def host_threads() -> int:
    """Every host core for the CPU legs: torchrun sets OMP_NUM_THREADS=1 per
    rank, so the BLAS pool is raised explicitly."""
    from threadpoolctl import threadpool_limits

    n = os.cpu_count() or 1
    threadpool_limits(limits=n)
    torch.set_num_threads(n)
    return n


def cpu_sweep_inputs(sample_rows: int) -> dict:
    """The reference arm's inputs: rank 0's CPU-drawn rows, routers and
    biases of every checkpoint (checkpoint_setup), as numpy."""
    active, exits = nominal_schedule(ROWS)
    cks = []
    for k in range(len(LAYERS)):
        s = checkpoint_setup(k, 0, active[k], exits[k])
        x = s["x_head"][:sample_rows]
        xs = x.numpy() if x.dtype == torch.float32 else x.view(torch.int16).numpy().view(np.uint16)
        cks.append({"x": xs, "down": s["down"].numpy(), "up": s["up"].numpy(), "bias": s["bias"]})
    return {"checkpoints": cks, "norm_weight": norm_weight_cpu().numpy()}


def cpu_sweep_step(inp: dict) -> tuple[float, int]:
    """One step of the workload on the host by the oracle (the reference's CPU
    path, restated): every checkpoint on the sample's still-active rows, the
    survivor count chaining into the next checkpoint as on the device.
    Returns (seconds, rows routed)."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import tide_oracle as O

    odt = O.F32 if DTYPE == "f32" else O.BF16
    norm = {"kind": "rms", "weight": inp["norm_weight"], "bias": None, "eps": 1e-5}
    n = inp["checkpoints"][0]["x"].shape[0]
    out = np.zeros_like(inp["checkpoints"][0]["x"])
    routed = 0
    positions = np.arange(n, dtype=np.int64)
    slots = np.arange(n, dtype=np.int32)
    t0 = time.perf_counter()
    for ck in inp["checkpoints"]:
        if n == 0:
            break
        r = O.checkpoint(ck["x"][:n], odt, norm, ck["down"], ck["up"], ck["bias"], THRESHOLD,
                         positions=positions[:n], slots=slots[:n], out_buffer=out)
        out = r["out_buffer"]
        positions, slots = r["positions"], r["slots"]
        routed += n
        n = r["n_survivors"]
    return time.perf_counter() - t0, routed


def cpu_baseline_sample(sample_rows: int, reps: int) -> dict:
    cores = host_threads()
    inp = cpu_sweep_inputs(sample_rows)
    cpu_sweep_step(inp)
    runs = [cpu_sweep_step(inp) for _ in range(reps)]
    t, routed = min(runs, key=lambda r: r[0])
    return {"value": routed / t, "unit": "tokens/s", "cores": cores, "kind": "port",
            "sample": f"oracle on the first {sample_rows} rows of every checkpoint of "
                      f"{WORKLOAD} ({routed} rows routed per step, same rows, routers and "
                      f"biases as the device run), best of {reps}"}


# ----------------------------------------------------------------- main
def run_reference(args, world, rank):
    """--impl reference: the CPU restatement of the reference path (the
    reference is Python and cannot be built into a library), timed on the host
    cores with every thread numpy's BLAS can use; rank 0 only.  It loads
    nothing of tide_b200's native code: the rows, routers and biases come
    from the CPU generator (checkpoint_setup) and go straight to the oracle."""
    if rank != 0:
        return
    if WORKLOAD in (SWEEP_WORKLOAD, ENGINE_WORKLOAD, DECODE_WORKLOAD, ATTN_WORKLOAD):
        configure("llama8b_prefill_checkpoints")
    sample = min(2048, ROWS)
    cores = host_threads()
    inp = cpu_sweep_inputs(sample)
    for _ in range(args.warmup):
        cpu_sweep_step(inp)
    runs = [cpu_sweep_step(inp) for _ in range(args.steps)]
    t = sum(r[0] for r in runs)
    routed = sum(r[1] for r in runs)
    v = routed / t
    line = {
        "impl": "reference", "metric": "router_compact_scatter_tokens_per_s", "value": v,
        "unit": "tokens/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1000 * t / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": DTYPE, "data": "synthetic",
        "config": {"workload": WORKLOAD, "rows_per_gpu": ROWS, "hidden": HIDDEN,
                   "bottleneck": BOTTLENECK, "checkpoint_layers": LAYERS,
                   f"exit_fractions_of_{EXITS_OF}": EXIT_FRACTIONS,
                   "sample_rows_per_checkpoint": sample, "rows_routed_per_step": routed // args.steps,
                   "same_config": True,
                   "note": "the same checkpoints, routers, biases and leading rows as the device "
                           "run, on a bounded sample of each checkpoint's rows; tokens/s is rows "
                           "routed per second"},
        "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": cores, "kind": "port",
                         "sample": f"first {sample} rows of every checkpoint, chained"},
        "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def _tuned_routers(model, ids, layers, fracs, hidden, norm, seed, last_takes_rest=True):
    """Routers (down/up N(0, 0.02)) at `layers` whose output biases exit the
    scheduled share of the batch (fracs; with last_takes_rest the last one
    exits every token still active) on the model's own hidden states for
    `ids`.  norm = (kind, weight, bias, eps) of the final norm."""
    from tide_b200 import workloads
    from tide_b200.router import TokenRouter

    dev = ids.device
    kind, nw, nb, eps = norm
    hs = model(ids, output_hidden_states=True, logits_to_keep=1).hidden_states
    g = torch.Generator().manual_seed(seed)
    N = ids.numel()
    exited = torch.zeros(N, dtype=torch.bool, device=dev)
    routers = {}
    for L, f in zip(layers, fracs):
        r = TokenRouter(hidden, 128, up_bias=True)
        with torch.no_grad():
            r.down.weight.normal_(0, 0.02, generator=g)
            r.up.weight.normal_(0, 0.02, generator=g)
        h = hs[L + 1].reshape(N, -1)
        z = workloads.prebias_logits_torch(h, kind, nw, nb, eps, r.down.weight.to(dev),
                                           r.up.weight.to(dev))
        active = (~exited).nonzero()[:, 0]
        last = last_takes_rest and L == layers[-1]
        n_exit = int(active.numel()) if last else int(round(f * N))
        za = z[active]
        bias = workloads.bias_for_exit_fraction(za, n_exit / max(1, active.numel()), THRESHOLD)
        with torch.no_grad():
            r.up.bias.fill_(bias)
        exited[active[(za + bias) > workloads.logit(THRESHOLD)]] = True
        routers[L] = r
    del hs
    return routers


def _timed_calls(world: int, fn, reps: int, warmup: int) -> float:
    """Seconds for `reps` calls of fn after `warmup` untimed ones: CUDA
    events on the current stream, max over ranks."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    barrier(world)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(reps):
        fn()
    b.record()
    torch.cuda.synchronize()
    return max_over_ranks(world, a.elapsed_time(b) / 1000.0)


def _engine_measure(world, model, ids, global_tokens, routers, hidden, layers, reps, warmup,
                    keep_last: bool) -> dict:
    """engine(ids) post hoc and live (and, with keep_last, with
    logits_to_keep=1), and the model's own forward, on the same ids;
    global_tokens = tokens of one call over all ranks."""
    from tide_b200 import TIDEConfig
    from tide_b200 import dist as tdist
    from tide_b200.router import RouterCheckpoint
    from tide_b200.runtime import TIDERuntime

    tmp = Path(tempfile.mkdtemp(prefix="tide_bench_"))
    RouterCheckpoint(routers, hidden, 128).save(tmp / "router.pt")
    engine = TIDERuntime(model, tmp / "router.pt",
                         config=TIDEConfig(exit_threshold=THRESHOLD, min_layers=0))
    t_engine = _timed_calls(world, lambda: engine(ids), reps, warmup)
    stats = tdist.global_stats(world, engine.last_stats, layers)
    t_live = _timed_calls(world, lambda: engine(ids, live=True), reps, warmup)
    live_stats = tdist.global_stats(world, engine.last_stats, layers)
    t_hf = _timed_calls(world, lambda: model(ids).logits, reps, warmup)
    # the model call the post-hoc engine makes (every layer's hidden states,
    # one position's logits): the engine's time beyond it is its own
    t_hs = _timed_calls(world, lambda: model(ids, output_hidden_states=True,
                                             logits_to_keep=1).hidden_states, reps, warmup)
    tokens = global_tokens * reps
    res = {"engine_tok_s": tokens / t_engine, "engine_ms_per_call": 1000 * t_engine / reps,
           "hf_forward_tok_s": tokens / t_hf, "hf_forward_ms_per_call": 1000 * t_hf / reps,
           "hf_hidden_states_ms_per_call": 1000 * t_hs / reps,
           "engine_mode": "post-hoc (every layer runs; the reference's semantics)",
           "exit_rate": stats.exit_rate,
           "exits_per_layer": {str(k): v for k, v in sorted(stats.exits_per_layer.items())},
           "live_tok_s": tokens / t_live, "live_ms_per_call": 1000 * t_live / reps,
           "live_mode": "layers after each checkpoint on the active tokens only; exited "
                        "tokens' K/V zero-padded",
           "live_exit_rate": live_stats.exit_rate,
           "live_exits_per_layer": {str(k): v for k, v in
                                    sorted(live_stats.exits_per_layer.items())}}
    if keep_last:
        # lm_head on the last position only (what a prefill before decoding
        # needs), post hoc and live
        t_keep = _timed_calls(world, lambda: engine(ids, logits_to_keep=1), reps, warmup)
        t_live_keep = _timed_calls(world, lambda: engine(ids, live=True, logits_to_keep=1),
                                   reps, warmup)
        res.update({"last_logits_only_tok_s": tokens / t_keep,
                    "live_last_logits_only_tok_s": tokens / t_live_keep,
                    "last_logits_only_mode": "logits_to_keep=1: lm_head on each sequence's last "
                                             "position only"})
    del engine
    return res


def engine_prefill(world: int, rank: int, reps: int = 10, warmup: int = 3) -> dict:
    """8B-architecture prefill through the engine: a random-init bf16
    Llama-3.1-8B-architecture model (32 layers, H 4096, 32/8 heads, head_dim
    128, SwiGLU 14336, vocab 128256, RMSNorm eps 1e-5, RoPE theta 5e5),
    routers at layers 8..28 whose biases exit 5/10/15/20/20/30 % of the
    batch, input 16 x 2048 uniform random ids (seed 1) split by sequence
    over the ranks.  Times engine(input_ids) (3 warm-up + 10 timed, the
    reference's throughput protocol: batch * seq / time) and the model's own
    forward on the same ids."""
    from transformers import LlamaConfig, LlamaForCausalLM

    from tide_b200 import dist as tdist

    dev = torch.device("cuda")
    layers, fracs = [8, 12, 16, 20, 24, 28], [0.05, 0.10, 0.15, 0.20, 0.20, 0.30]
    B_all, S = 16, 2048
    ids_all = torch.randint(0, 128256, (B_all, S), generator=torch.Generator().manual_seed(1))
    b0, b1 = tdist.shard_range(B_all, world, rank)
    ids = ids_all[b0:b1].to(dev)
    cfg = LlamaConfig(vocab_size=128256, hidden_size=4096, intermediate_size=14336,
                      num_hidden_layers=32, num_attention_heads=32, num_key_value_heads=8,
                      head_dim=128, rms_norm_eps=1e-5, rope_theta=500000.0,
                      max_position_embeddings=8192, tie_word_embeddings=False)
    torch.manual_seed(SEED)
    prev = torch.get_default_dtype()
    torch.set_default_dtype(torch.bfloat16)
    try:
        with torch.device(dev):
            model = LlamaForCausalLM(cfg).eval()
    finally:
        torch.set_default_dtype(prev)
    res = {"model": "Llama-3.1-8B architecture, random-init bf16", "global_batch": B_all,
           "seq_len": S, "batch_per_rank": b1 - b0, "scaling": "strong", "timed_calls": reps,
           "warmup_calls": warmup, "router_layers": layers, "exit_fractions_of_batch": fracs}
    with torch.inference_mode():
        routers = _tuned_routers(model, ids, layers, fracs, 4096,
                                 ("rms", model.model.norm.weight.float(), None, 1e-5), SEED + 5)
        res.update(_engine_measure(world, model, ids, B_all * S, routers, 4096, layers, reps,
                                   warmup, keep_last=True))
    del model
    torch.cuda.empty_cache()
    return res


def gpt2_prefill(world: int, rank: int, reps: int = 10, warmup: int = 3) -> dict:
    """GPT-2-small prefill through the engine: a random-init fp16 GPT-2-small
    architecture model (12 layers, H 768, 12 heads, MLP 3072, vocab 50257,
    LayerNorm), routers at layers 4 and 8 whose biases exit about 20 % of
    the tokens at each, input 8 x 512 uniform random ids (seed 1) split by
    sequence over the ranks.  Same protocol as the 8B-architecture prefill."""
    from transformers import GPT2Config, GPT2LMHeadModel

    from tide_b200 import dist as tdist

    dev = torch.device("cuda")
    layers, fracs = [4, 8], [0.20, 0.16]  # 20 % of the tokens, then 20 % of the rest
    B_all, S = 8, 512
    ids_all = torch.randint(0, 50257, (B_all, S), generator=torch.Generator().manual_seed(1))
    b0, b1 = tdist.shard_range(B_all, world, rank)
    ids = ids_all[b0:b1].to(dev)
    cfg = GPT2Config(vocab_size=50257, n_embd=768, n_layer=12, n_head=12, n_inner=3072,
                     n_positions=1024)
    torch.manual_seed(SEED)
    with torch.device(dev):
        model = GPT2LMHeadModel(cfg).to(torch.float16).eval()
    res = {"model": "GPT-2-small architecture, random-init fp16", "global_batch": B_all,
           "seq_len": S, "batch_per_rank": b1 - b0, "scaling": "strong", "timed_calls": reps,
           "warmup_calls": warmup, "router_layers": layers, "exit_fractions_of_batch": fracs}
    with torch.inference_mode():
        ln = model.transformer.ln_f
        routers = _tuned_routers(model, ids, layers, fracs, 768,
                                 ("ln", ln.weight.float(), ln.bias.float(), ln.eps), SEED + 6,
                                 last_takes_rest=False)
        res.update(_engine_measure(world, model, ids, B_all * S, routers, 768, layers, reps,
                                   warmup, keep_last=False))
    del model
    torch.cuda.empty_cache()
    return res


def decode_checkpoints(world: int, rank: int, steps: int = 200) -> dict:
    """The decode-size regime next to the prefill one: one step of the
    qwen3_8b_decode_checkpoints workload (256 rows of H 4096 bf16 through
    eight checkpoints at layers 3..31, ~10 % of the active rows exiting at
    each, positions and KV slot ids compacted on the device), as a CUDA graph
    replayed `steps` times; rows routed per second, summed over ranks."""
    saved = {k: globals()[k] for k in ("WORKLOAD", "LAYERS", "EXIT_FRACTIONS", "EXITS_OF", "ROWS",
                                       "HIDDEN", "DTYPE")}
    try:
        configure("qwen3_8b_decode_checkpoints")
        from tide_b200.capi import PATH_AUTO

        wl = Workload(rank, PATH_AUTO)
        for _ in range(3):
            wl.step()
        torch.cuda.synchronize()
        counts = wl.counts.cpu()
        rows = int(counts.sum().item())
        g = wl.capture()[0]
        for _ in range(3):
            g.replay()
        torch.cuda.synchronize()
        barrier(world)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(steps):
            g.replay()
        b.record()
        torch.cuda.synchronize()
        t = max_over_ranks(world, a.elapsed_time(b) / 1000.0)
        wl.runner.check_errors()
        res = {"workload": WORKLOAD, "rows_per_gpu": ROWS, "checkpoint_layers": LAYERS,
               "rows_routed_per_step": rows, "exits": counts[:, 1].tolist(), "steps": steps,
               "us_per_step": 1e6 * t / steps, "rows_per_s": world * rows * steps / t,
               "paths": [PATH_NAMES.get(v, v) for v in wl.paths.values()],
               "gpu_launches_per_step": sum(launches_per_checkpoint(v) for v in wl.paths.values())}
        del g, wl
        return res
    finally:
        globals().update(saved)


def decode_generate(world: int, rank: int, steps: int = 128, batch: int = 256,
                    ctx: int = 1024) -> dict:
    """Decode at model level: a random-init bf16 Qwen3-8B-architecture
    model (36 layers, H 4096, 32/8 heads, head_dim 128, MLP 12288, vocab
    151936, QK-norm), a decode batch of 256 sequences per rank whose KV cache
    holds 1024 positions of N(0,1) keys and values, routers at layers
    3, 7, ..., 31 whose biases exit ~10 % of the rows still active at each,
    and 128 greedy tokens.  Timed four ways, each on its own copy of that
    cache: the live decoder with per-row exits (tide_b200.live.LiveDecoder:
    after a row exits its later attention and cache writes are skipped, the
    survivors' KV slot ids compacted by the checkpoint kernel; each step one
    CUDA graph replay), the same decoder launching its kernels one by one
    (no graph), the graph decoder with no exit (every checkpoint still
    runs), and the model's own greedy loop on HF's DynamicCache (every layer
    for every row, as in the reference's decode).  tokens/s = batch * steps
    / time, summed over ranks."""
    from transformers import DynamicCache, Qwen3Config, Qwen3ForCausalLM

    from tide_b200 import TIDEConfig
    from tide_b200 import dist as tdist
    from tide_b200 import workloads
    from tide_b200.live import LiveDecoder
    from tide_b200.router import RouterCheckpoint, TokenRouter
    from tide_b200.runtime import TIDERuntime
    from tide_b200.scheduler import ExitStats

    dev = torch.device("cuda")
    layers = list(range(3, 35, 4))  # 3..31: every fourth layer short of the last
    cfg = Qwen3Config(vocab_size=151936, hidden_size=4096, intermediate_size=12288,
                      num_hidden_layers=36, num_attention_heads=32, num_key_value_heads=8,
                      head_dim=128, rms_norm_eps=1e-6, rope_theta=1e6,
                      max_position_embeddings=40960, tie_word_embeddings=False)
    torch.manual_seed(SEED + 3)
    prev = torch.get_default_dtype()
    torch.set_default_dtype(torch.bfloat16)
    try:
        with torch.device(dev):
            model = Qwen3ForCausalLM(cfg).eval()
    finally:
        torch.set_default_dtype(prev)
    res = {"model": "Qwen3-8B architecture, random-init bf16", "batch_per_rank": batch,
           "kv_context": ctx, "new_tokens": steps, "router_layers": layers,
           "exit_fraction_of_active_per_checkpoint": 0.10, "scaling": "weak"}
    tok0 = torch.randint(0, cfg.vocab_size, (batch,),
                         generator=torch.Generator(device=dev).manual_seed(SEED + 7 + rank),
                         device=dev)

    def timed(fn) -> float:
        torch.cuda.synchronize()
        barrier(world)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        return max_over_ranks(world, a.elapsed_time(b) / 1000.0)

    with torch.inference_mode():
        # routers placed on one step's hidden states (the model's own decode)
        cal = DynamicCache(config=cfg)
        g = torch.Generator(device=dev).manual_seed(SEED + 11 + rank)
        for li in range(cfg.num_hidden_layers):
            cal.update(torch.randn(batch, 8, 64, 128, generator=g, device=dev).to(torch.bfloat16),
                       torch.randn(batch, 8, 64, 128, generator=g, device=dev).to(torch.bfloat16), li)
        hs = model(tok0[:, None], past_key_values=cal, use_cache=True,
                   output_hidden_states=True).hidden_states
        del cal
        gw = torch.Generator().manual_seed(SEED + 13)
        nw = model.model.norm.weight.float()
        exited = torch.zeros(batch, dtype=torch.bool, device=dev)
        routers = {}
        for L in layers:
            r = TokenRouter(4096, 128, up_bias=True)
            with torch.no_grad():
                r.down.weight.normal_(0, 0.02, generator=gw)
                r.up.weight.normal_(0, 0.02, generator=gw)
            z = workloads.prebias_logits_torch(hs[L + 1][:, -1, :], "rms", nw, None, 1e-6,
                                               r.down.weight.to(dev), r.up.weight.to(dev))
            active = (~exited).nonzero()[:, 0]
            bias = workloads.bias_for_exit_fraction(z[active], 0.10, THRESHOLD)
            with torch.no_grad():
                r.up.bias.fill_(bias)
            exited[active[(z[active] + bias) > workloads.logit(THRESHOLD)]] = True
            routers[L] = r
        del hs
        tmp = Path(tempfile.mkdtemp(prefix="tide_bench_"))
        RouterCheckpoint(routers, 4096, 128).save(tmp / "router.pt")
        engine = TIDERuntime(model, tmp / "router.pt",
                             config=TIDEConfig(exit_threshold=THRESHOLD, min_layers=0))

        def live_run(threshold: float, stats, graph: bool = True):
            engine.config.exit_threshold = threshold
            dec = LiveDecoder(engine, batch, ctx + steps + 8, graph=graph)
            dec.fill_random(ctx, torch.Generator(device=dev).manual_seed(SEED + 17 + rank))
            tok = tok0
            for _ in range(3):  # warm-up steps (the first records the step's graph)
                tok = dec.step(tok).argmax(-1)
            dec.read_stats(ExitStats())

            def loop():
                t = tok
                for _ in range(steps):
                    t = dec.step(t, stats).argmax(-1)

            t_run = timed(loop)
            dec.read_stats(stats if stats is not None else ExitStats())
            del dec
            torch.cuda.empty_cache()
            return t_run

        # the model's own loop first, on a fresh allocator (its cache grows
        # by concatenation every step)
        cache = DynamicCache(config=cfg)
        g = torch.Generator(device=dev).manual_seed(SEED + 17 + rank)
        for li in range(cfg.num_hidden_layers):
            cache.update(torch.randn(batch, 8, ctx, 128, generator=g, device=dev).to(torch.bfloat16),
                         torch.randn(batch, 8, ctx, 128, generator=g, device=dev).to(torch.bfloat16), li)
        nxt = tok0[:, None]
        for _ in range(3):
            nxt = model(nxt, past_key_values=cache, use_cache=True).logits[:, -1, :].argmax(-1, keepdim=True)

        def hf_loop():
            t = nxt
            for _ in range(steps):
                t = model(t, past_key_values=cache, use_cache=True).logits[:, -1, :].argmax(-1, keepdim=True)

        t_hf = timed(hf_loop)
        del cache
        torch.cuda.empty_cache()
        st_live = ExitStats()
        t_live = live_run(THRESHOLD, st_live)
        t_eager = live_run(THRESHOLD, None, graph=False)
        t_noexit = live_run(2.0, None)  # scores lie in [0, 1]: no row exits
        engine.config.exit_threshold = THRESHOLD
        stats = tdist.global_stats(world, st_live, layers)
    tokens = world * batch * steps
    res.update({"live_tok_s": tokens / t_live, "live_ms_per_step": 1000 * t_live / steps,
                "live_eager_tok_s": tokens / t_eager, "live_eager_ms_per_step": 1000 * t_eager / steps,
                "live_no_exit_tok_s": tokens / t_noexit, "live_no_exit_ms_per_step": 1000 * t_noexit / steps,
                "hf_greedy_tok_s": tokens / t_hf, "hf_ms_per_step": 1000 * t_hf / steps,
                "hf_cache": "DynamicCache (HF's StaticCache measured 193 ms per step here)",
                "live_exit_rate": stats.exit_rate,
                "live_exits_per_layer": {str(k): v for k, v in sorted(stats.exits_per_layer.items())}})
    del engine, model
    torch.cuda.empty_cache()
    return res


def decode_attention_bench(world: int, rank: int, steps: int, warmup: int) -> dict:
    """The live decoder's attention kernel alone (tide_decode_attention), at
    the decode workload's shapes: 256 rows, Qwen3-8B heads (32 query / 8 KV,
    head_dim 128), a 1024-position bf16 cache addressed by slot (permuted
    slots), the live row count and the length on the device; with 256, 128
    and 64 of the rows active (what the exits leave).  The cache (1.2 GB)
    is larger than L2.  Algorithmic bytes per launch: the active rows' keys
    and values (2 * 8 * 1024 * 128 * 2 bytes per row) plus their q and
    output rows.  Times: CUDA events around `steps` launches after
    `warmup`."""
    from tide_b200 import _native

    ops = _native.ops()
    dev = torch.device("cuda")
    B, hq, hkv, d, L, max_len = 256, 32, 8, 128, 1024, 1152
    g = torch.Generator(device=dev).manual_seed(SEED + 31 + rank)
    kc = torch.randn(B, hkv, max_len, d, generator=g, device=dev).to(torch.bfloat16)
    vc = torch.randn(B, hkv, max_len, d, generator=g, device=dev).to(torch.bfloat16)
    q = torch.randn(B, hq, d, generator=g, device=dev).to(torch.bfloat16)
    out = torch.empty_like(q)
    slots = torch.randperm(B, generator=torch.Generator().manual_seed(SEED)).to(torch.int32).to(dev)
    len_dev = torch.tensor([L], dtype=torch.int32, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    peak = load_peak()
    cases = []
    for live in (256, 128, 64):
        n_dev = torch.tensor([live], dtype=torch.int32, device=dev)

        def call():
            ops.decode_attention(q, kc, vc, slots, out, max_len, d ** -0.5, err, n_dev, len_dev)

        for _ in range(max(warmup, 3)):
            call()
        torch.cuda.synchronize()
        barrier(world)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(steps):
            call()
        b.record()
        torch.cuda.synchronize()
        sec = max_over_ranks(world, a.elapsed_time(b) / 1000.0 / steps)
        nbytes = live * hkv * L * d * 2 * 2 + 2 * live * hq * d * 2
        gbps = nbytes / sec / 1e9
        cases.append({"active_rows": live, "us_per_launch": sec * 1e6, "bytes": nbytes,
                      "GBps": gbps, "frac": gbps / peak})
    if int(err.item()):
        raise RuntimeError(f"decode attention raised device error bits {int(err.item())}")
    del kc, vc
    torch.cuda.empty_cache()
    return {"rows": B, "q_heads": hq, "kv_heads": hkv, "head_dim": d, "positions": L,
            "peak_GBps": peak, "cases": cases,
            "note": "cache larger than L2 (1.2 GB); one launch per timed call"}


def run_sweep(args, world, rank, local) -> None:
    """--workload bandwidth_sweep: one checkpoint per (N, H, f), N split evenly
    over the ranks; aggregate algorithmic GB/s (max device time over ranks)
    against the measured copy peak."""
    from tide_b200 import dist as tdist
    from tide_b200 import workloads
    from tide_b200.capi import NORM_RMS, PATH_AUTO
    from tide_b200.ops import CheckpointRunner, NormSpec, prepare_router

    dev = torch.device("cuda")
    peak = load_peak()
    hs = [int(h) for h in args.sweep_h.split(",")] if args.sweep_h else SWEEP_H
    ns = [int(n) for n in args.sweep_n.split(",")] if args.sweep_n else SWEEP_N
    fs = [float(f) for f in args.sweep_f.split(",")] if args.sweep_f else SWEEP_F
    runner = CheckpointRunner(dev)
    rows_out = []
    with ClockSampler(local) as clocks:
        for H in hs:
            norm = NormSpec(NORM_RMS, torch.ones(H, device=dev), None, 1e-5)
            gw = torch.Generator().manual_seed(SEED + H)
            down = (0.02 * torch.randn(BOTTLENECK, H, generator=gw)).to(dev)
            up = (0.02 * torch.randn(1, BOTTLENECK, generator=gw)).to(dev)
            for N in ns:
                r0, r1 = tdist.shard_range(N, world, rank)
                n = r1 - r0
                g = torch.Generator(device=dev).manual_seed(SEED + 17 * rank + N + H)
                x = torch.empty(n, H, dtype=torch.bfloat16, device=dev)
                for s0 in range(0, n, 65536):
                    s1 = min(n, s0 + 65536)
                    x[s0:s1] = torch.randn(s1 - s0, H, generator=g, device=dev).to(torch.bfloat16)
                z = workloads.prebias_logits_torch(x[:65536], "rms", norm.weight, None, 1e-5, down, up)
                out = torch.zeros_like(x)
                comp = torch.empty_like(x)
                pos_out = torch.empty(n, dtype=torch.int64, device=dev)
                counts = torch.zeros(2, dtype=torch.int32, device=dev)
                for f in fs:
                    bias = workloads.bias_for_exit_fraction(z, f, THRESHOLD)
                    router = prepare_router(down, up, bias, norm, torch.bfloat16)

                    def call():
                        runner.run(x, router, norm, THRESHOLD, out_buffer=out, compact_out=comp,
                                   positions_out=pos_out, counts=counts, path=PATH_AUTO)

                    for _ in range(2):
                        call()
                    torch.cuda.synchronize()
                    path = runner.last_path
                    exits = int(counts[1].item())
                    est_ms = max(0.02, 2 * n * H * 2 / 5e12 * 1e3)
                    reps = int(max(5, min(50, 100.0 / est_ms)))
                    s = torch.cuda.Stream()
                    s.wait_stream(torch.cuda.current_stream())
                    graph = torch.cuda.CUDAGraph()
                    with torch.cuda.stream(s):
                        with torch.cuda.graph(graph, stream=s):
                            call()
                    torch.cuda.current_stream().wait_stream(s)
                    graph.replay()
                    torch.cuda.synchronize()
                    barrier(world)
                    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    a.record()
                    for _ in range(reps):
                        graph.replay()
                    b.record()
                    torch.cuda.synchronize()
                    ms = max_over_ranks(world, a.elapsed_time(b) / reps)
                    alg = world * algorithmic_bytes(n, exits, H, 2)  # ranks' shares are equal +-1 row
                    gbs = alg / (ms / 1000.0) / 1e9
                    rows_out.append({"N": N, "rows_per_gpu": n, "H": H, "f": f, "exits_rank0": exits,
                                     "ms": ms, "GBps": gbs, "frac": gbs / (world * peak),
                                     "tokens_per_s": N / (ms / 1000.0), "path": PATH_NAMES.get(path, path),
                                     "reps": reps})
                    del graph
                runner.check_errors()
                del x, out, comp, pos_out
                torch.cuda.empty_cache()
    if rank == 0:
        head = [r for r in rows_out if r["H"] == 4096 and r["N"] == max(ns)
                and abs(r["f"] - 0.1) < 1e-9] or rows_out[-1:]
        v = head[0]["GBps"] if head else None
        line = {"metric": "router_compact_scatter_hbm_GBps", "value": v, "unit": "GB/s",
                "n_gpus": world, "steps": None, "warmup": 2, "ms_per_step": head[0]["ms"] if head else None,
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
                "data": "synthetic",
                "config": {"workload": SWEEP_WORKLOAD, "N_total": ns, "H": hs, "exit_fractions": fs,
                           "value_case": "H 4096, largest N, f 0.1", "peak_GBps_per_gpu": peak,
                           "l2": "one checkpoint call per graph replay; rows above ~8K x 4096 exceed L2"},
                "sweep": rows_out, "clocks": clocks.summary(),
                "gpu_launches": None}
        print(json.dumps(line), flush=True)


def load_peak() -> float:
    try:
        return float(json.loads((ROOT / "MEASURED_PEAKS.json").read_text())["hbm_gbs"])
    except Exception:
        return 6650.0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--path", default="auto", choices=["auto", "simt", "tc", "tc_split"])
    ap.add_argument("--e2e-steps", type=int, default=None,
                    help="e2e steps (default: about 2 GB of host->device copies, at least 3)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-engine", action="store_true", help="skip the engine prefill measurement")
    ap.add_argument("--workload", default=WORKLOAD,
                    choices=sorted(WORKLOADS) + [SWEEP_WORKLOAD, ENGINE_WORKLOAD, DECODE_WORKLOAD,
                                                 ATTN_WORKLOAD])
    ap.add_argument("--rows", type=int, default=None, help="rows per GPU (profiling runs)")
    ap.add_argument("--sweep-h", default=None, help="bandwidth_sweep: comma-separated H values")
    ap.add_argument("--sweep-n", default=None, help="bandwidth_sweep: comma-separated N values")
    ap.add_argument("--sweep-f", default=None, help="bandwidth_sweep: comma-separated exit fractions")
    args = ap.parse_args()
    if args.workload in WORKLOADS:
        configure(args.workload, args.rows)
    else:
        globals()["WORKLOAD"] = args.workload
    world, rank, local = dist_setup(args.gpus)
    try:
        if args.impl == "reference":
            run_reference(args, world, rank)
        elif args.workload == SWEEP_WORKLOAD:
            run_sweep(args, world, rank, local)
        elif args.workload == DECODE_WORKLOAD:
            dg = decode_generate(world, rank)
            if rank == 0:
                print(json.dumps({"metric": "decode_tokens_per_s", "value": dg["live_tok_s"],
                                  "unit": "tokens/s", "n_gpus": world, "higher_is_better": True,
                                  "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
                                  "data": "synthetic", "config": {"workload": DECODE_WORKLOAD},
                                  "decode_generate": dg}), flush=True)
        elif args.workload == ATTN_WORKLOAD:
            da = decode_attention_bench(world, rank, args.steps, args.warmup)
            if rank == 0:
                full = da["cases"][0]
                print(json.dumps({"metric": "decode_attention_GBps", "value": full["GBps"] * world,
                                  "unit": "GB/s", "n_gpus": world, "higher_is_better": True,
                                  "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
                                  "data": "synthetic", "config": {"workload": ATTN_WORKLOAD},
                                  "roofline": {"bound": "hbm", "achieved": full["GBps"],
                                               "peak": da["peak_GBps"], "unit": "GB/s",
                                               "frac": full["frac"], "traffic": None},
                                  "decode_attention": da}), flush=True)
        elif args.workload == ENGINE_WORKLOAD:
            eng = engine_prefill(world, rank)
            gpt2 = gpt2_prefill(world, rank)
            if rank == 0:
                print(json.dumps({"metric": "prefill_tokens_per_s", "value": eng["engine_tok_s"],
                                  "unit": "tokens/s", "n_gpus": world, "higher_is_better": True,
                                  "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
                                  "data": "synthetic", "config": {"workload": ENGINE_WORKLOAD},
                                  "prefill_engine": eng, "prefill_engine_gpt2": gpt2}),
                      flush=True)
        else:
            run_checkpoints(args, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


def run_checkpoints(args, world, rank, local) -> None:
    from tide_b200 import dist as tdist
    from tide_b200.capi import PATH_AUTO, PATH_SIMT, PATH_TC, PATH_TC_SPLIT

    path = {"auto": PATH_AUTO, "simt": PATH_SIMT, "tc": PATH_TC, "tc_split": PATH_TC_SPLIT}[args.path]
    wl = Workload(rank, path)
    for _ in range(max(args.warmup, 3)):
        wl.step()
    torch.cuda.synchronize()
    counts = wl.counts.cpu()
    rows_per_step = int(counts.sum().item())
    exits_per_stage = counts[:, 1].tolist()
    active = (counts[:, 0] + counts[:, 1]).tolist()
    wl.runner.check_errors()

    step_graph = wl.capture()[0]
    ck_graphs = wl.capture(per_checkpoint=True, calls=CK_CALLS)
    gather = CountsGather(world, wl.counts) if world > 1 else None
    for _ in range(2):
        step_graph.replay()
        if gather:
            gather.after_step(wl.counts)
        for g in ck_graphs:
            g.replay()
    if gather:
        gather.finish()
    torch.cuda.synchronize()

    # timed region: device-resident inputs, one graph launch per step on the
    # current stream (plus, on several ranks, the all-gather of the step's
    # exit counts on a second stream), CUDA events before the first launch
    # and after the last step's collective
    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize()
    with ClockSampler(local) as clocks:
        t_start.record()
        for _ in range(args.steps):
            step_graph.replay()
            if gather:
                gather.after_step(wl.counts)
        if gather:
            gather.finish()
        t_end.record()
        torch.cuda.synchronize()
        # per-launch device time of each checkpoint's kernels (the roofline's
        # denominator): a graph of CK_CALLS back-to-back calls of that
        # checkpoint (each launch overlaps the previous one's tail, as in the
        # step), CUDA events around every replay
        reps = max(3, min(args.steps, 50))
        ev = [[(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in LAYERS] for _ in range(reps)]
        for i in range(reps):
            for k, g in enumerate(ck_graphs):
                ev[i][k][0].record()
                g.replay()
                ev[i][k][1].record()
        torch.cuda.synchronize()
    elapsed = t_start.elapsed_time(t_end) / 1000.0
    per_ck = [sum(ev[i][k][0].elapsed_time(ev[i][k][1]) for i in range(reps)) / (reps * CK_CALLS)
              for k in range(len(LAYERS))]
    del ev
    barrier(world)
    elapsed = max_over_ranks(world, elapsed)
    value = world * rows_per_step * args.steps / elapsed
    counts_after = wl.counts.cpu()
    assert torch.equal(counts_after, counts), "graph replay changed the exit counts"
    wl.runner.check_errors()
    global_counts = (gather.out[(gather.i - 1) % 2].sum(0).cpu() if gather
                     else wl.counts.cpu().to(torch.int64))
    collectives = gather_timings(world, wl) if world > 1 else None

    e = 4 if DTYPE == "f32" else 2
    alg = [algorithmic_bytes(active[k], exits_per_stage[k], HIDDEN, e) for k in range(len(LAYERS))]
    achieved = alg[0] / (per_ck[0] / 1000.0) / 1e9  # the first (largest) checkpoint
    achieved_all = sum(alg) / (elapsed / args.steps) / 1e9
    peak = load_peak()
    path_name = PATH_NAMES.get(wl.paths[0], wl.paths[0])
    traffic = (NCU_TRAFFIC_CKPT0["bytes"] if ROWS == NCU_TRAFFIC_CKPT0["rows"]
               and path_name == NCU_TRAFFIC_CKPT0["path"] and WORKLOAD == "llama8b_prefill_checkpoints"
               else None)
    roofline = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                "frac": achieved / peak, "traffic": traffic,
                "traffic_source": "ncu capture of checkpoint 0's two kernels in this workload (warm caches)" if traffic else None,
                "peak_source": "measured" if (ROOT / "MEASURED_PEAKS.json").exists() else "fallback",
                "kernel": f"checkpoint 0 ({ROWS} rows x {HIDDEN}), every kernel of the call",
                "per_checkpoint_ms": per_ck, "per_checkpoint_reps": reps,
                "per_checkpoint_calls_per_graph": CK_CALLS,
                "achieved_all_checkpoints": achieved_all, "algorithmic_bytes_per_step": sum(alg)}

    parity = parity_sample(wl, active) if rank == 0 else None

    # e2e through the public operator with host buffers: H2D of the step's
    # hidden states from pinned memory (the rows each checkpoint routes), the
    # step graph, D2H of the output rows, of the last checkpoint's survivors
    # and of the counts
    host_x = [x[: active[k]].cpu().pin_memory() for k, x in enumerate(wl.x)]
    dev_x = [torch.empty_like(x) for x in wl.x]
    host_counts = torch.empty_like(wl.counts, device="cpu").pin_memory()
    host_out = torch.empty_like(wl.out, device="cpu").pin_memory()
    n_last = int(counts[-1, 0].item())
    host_surv = torch.empty((max(n_last, 1), HIDDEN), dtype=wl.compact.dtype).pin_memory()
    h2d = int(sum(x.numel() * x.element_size() for x in host_x))
    d2h = int(host_out.numel() * host_out.element_size() + n_last * HIDDEN * e
              + host_counts.numel() * 4)
    e2e_steps = e2e_step_count(args.e2e_steps, h2d)
    # Two input sets, each with its own step graph: step i+1's host->device
    # copies run on a copy stream while step i computes and its results go
    # back (the link is full duplex); a set is refilled only after the graph
    # that read it has finished.
    in_sets = [dev_x, [torch.empty_like(x) for x in wl.x]]
    e_graphs = [wl.capture(in_sets[0])[0], wl.capture(in_sets[1])[0]]
    s_in = torch.cuda.Stream()
    loaded = [torch.cuda.Event(), torch.cuda.Event()]
    released = [torch.cuda.Event(), torch.cuda.Event()]

    def e2e_load(i):
        b = i % 2
        with torch.cuda.stream(s_in):
            s_in.wait_event(released[b])
            for k in range(len(LAYERS)):
                in_sets[b][k][: active[k]].copy_(host_x[k], non_blocking=True)
            loaded[b].record(s_in)

    def e2e_step(i):
        b = i % 2
        cur = torch.cuda.current_stream()
        cur.wait_event(loaded[b])
        e_graphs[b].replay()
        released[b].record(cur)
        if gather:
            gather.after_step(wl.counts)
        host_out.copy_(wl.out, non_blocking=True)
        if n_last:
            host_surv[:n_last].copy_(wl.compact[:n_last], non_blocking=True)
        host_counts.copy_(wl.counts, non_blocking=True)

    for i in range(2):  # untimed: each graph's first launch uploads it to the device
        e2e_load(i)
        e2e_step(i)
    if gather:
        gather.finish()
    barrier(world)
    torch.cuda.synchronize()
    e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e_start.record()
    s_in.wait_stream(torch.cuda.current_stream())
    e2e_load(0)
    for i in range(e2e_steps):
        if i + 1 < e2e_steps:
            e2e_load(i + 1)
        e2e_step(i)
    if gather:
        gather.finish()
    torch.cuda.current_stream().wait_stream(s_in)
    e_end.record()
    torch.cuda.synchronize()
    e_el = max_over_ranks(world, e_start.elapsed_time(e_end) / 1000.0)
    e2e = {"value": world * rows_per_step * e2e_steps / e_el, "unit": "tokens/s",
           "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "steps": e2e_steps}
    del e_graphs, in_sets, step_graph, ck_graphs, host_out, dev_x

    paths_used = [PATH_NAMES.get(wl.paths[k], wl.paths[k]) for k in range(len(LAYERS))]
    n_launch = sum(launches_per_checkpoint(p) for p in wl.paths.values()) * args.steps
    engine = engine_gpt2 = decode = decode_gen = None
    if WORKLOAD == "llama8b_prefill_checkpoints" and args.rows is None:
        del wl
        torch.cuda.empty_cache()
        decode = decode_checkpoints(world, rank)
        if not args.no_engine:
            try:
                engine = engine_prefill(world, rank)
            except Exception as exc:  # reported, not fatal: the checkpoint numbers stand
                engine = {"error": f"{type(exc).__name__}: {exc}"[:400]}
            try:
                engine_gpt2 = gpt2_prefill(world, rank)
            except Exception as exc:
                engine_gpt2 = {"error": f"{type(exc).__name__}: {exc}"[:400]}
            try:
                decode_gen = decode_generate(world, rank)
            except Exception as exc:
                decode_gen = {"error": f"{type(exc).__name__}: {exc}"[:400]}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline_sample(min(2048, ROWS), 3)

    if rank == 0:
        line = {
            "metric": "router_compact_scatter_tokens_per_s", "value": value, "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": 1000 * elapsed / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": DTYPE, "data": "synthetic",
            "config": {"workload": WORKLOAD, "rows_per_gpu": ROWS, "hidden": HIDDEN,
                       "bottleneck": BOTTLENECK, "checkpoint_layers": LAYERS,
                       f"exit_fractions_of_{EXITS_OF}": EXIT_FRACTIONS,
                       "rows_routed_per_step": rows_per_step, "active_rows": active,
                       "exits": exits_per_stage,
                       "global_exits_all_ranks": global_counts[:, 1].tolist(),
                       "path": path_name, "path_per_checkpoint": paths_used,
                       "parallelism": (f"dp{world} (row shards; exit counts all-gathered every "
                                       f"step inside the timed region)" if world > 1 else "dp1"),
                       "l2": "inputs 1.1 GiB/step > 126 MB L2, no flush"},
            "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e, "parity": parity,
            "gpu_launches": n_launch, "clocks": clocks.summary(),
            "collectives_timed_separately": collectives,
            "prefill_engine": engine,
            "prefill_engine_gpt2": engine_gpt2,
            "decode_checkpoints": decode,
            "decode_generate": decode_gen,
        }
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
