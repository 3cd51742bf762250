"""Benchmark of the early-exit hot path (router -> compaction -> scatter).

Workload per GPU ("llama8b_prefill_checkpoints"): the checkpoint sweep of a
Llama-3.1-8B-architecture prefill batch of 16 x 2048 tokens = 32768 rows of
H = 4096 bf16 hidden states, routers at layers 8/12/16/20/24/28 (RMSNorm
eps 1e-5, router 4096 -> 128 -> 1) with biases placed so that 5/10/15/20/
20/30 % of the batch exits at each checkpoint (everything by layer 28).
Each checkpoint reads its own synthetic hidden-state tensor (rows N(0,1),
the hidden states of the still-active tokens at that layer), scores it,
compacts survivors (rows, int64 positions, int32 KV slots) into a dense
buffer and writes exits, final-normed, to their original positions.  Active
counts chain on the device between checkpoints (no host sync).  One step =
the six checkpoints.  Inputs (1.1 GiB per step) exceed the 126 MB L2, so no
explicit flush is needed between steps.

Third workload ("kernel_fp32_4096x768", --workload): the reference's own
kernel-level case, one checkpoint of 4096 fp32 rows of H = 768 (N(0,1) times
a per-row scale U(0.5, 2)), RMSNorm weight N(1, 0.02), 30 % exits.

Second workload ("qwen3_8b_decode_checkpoints", --workload): one decode step
of a Qwen3-8B-architecture batch of 256 sequences, routers at layers
3/7/.../31 (eight checkpoints, H = 4096), each exiting ~10 % of the rows
still active; the small-batch regime where launch and latency, not HBM,
set the time.

Multi-GPU: one process per GPU under torchrun; every rank processes its own
batch (weak scaling, no data-path collective); timing is the max over ranks.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                  [--workload llama8b_prefill_checkpoints|qwen3_8b_decode_checkpoints|
                              kernel_fp32_4096x768]
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

THRESHOLD = 0.85
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
                             "of": "active", "hidden": 768, "dtype": "f32", "inputs": "scaled"},
}
DTYPE_NAMES = {"bf16": torch.bfloat16, "f32": torch.float32}
WORKLOAD = "llama8b_prefill_checkpoints"
LAYERS = WORKLOADS[WORKLOAD]["layers"]
EXIT_FRACTIONS = WORKLOADS[WORKLOAD]["exit_fractions"]
EXITS_OF = WORKLOADS[WORKLOAD]["of"]
ROWS, HIDDEN, BOTTLENECK = WORKLOADS[WORKLOAD]["rows"], 4096, 128
DTYPE = "bf16"


# DRAM bytes (read + write) of checkpoint 0's two kernels (router + mover),
# 32768 rows x 4096 bf16, from the warm-cache ncu launch list of this
# benchmark (profiles/launches__llama8b_prefill_checkpoints.md).
NCU_TRAFFIC_CKPT0 = {"rows": 32768, "path": "tc_split", "bytes": (269.5 + 63.3 + 221.3 + 209.0) * 1e6}


def e2e_step_count(requested, h2d_bytes_nominal: int) -> int:
    """Steps of the e2e region: as requested, else enough for about 2 GB of
    host-to-device copies (at least 3, at most 200), so that a small
    workload's region is not a few hundred microseconds of host jitter.  The
    nominal bytes (rows x H x element size x checkpoints) are the same on
    every rank."""
    if requested is not None:
        return int(requested)
    return max(3, min(200, int(2e9 // max(int(h2d_bytes_nominal), 1))))


def algorithmic_bytes(n: int, exits: int, h: int, e: int) -> int:
    """Bytes a single pass must move for one checkpoint of n rows: read every
    row and write it once (survivor to the dense buffer, exit to its
    position), fp32 score + u8 decision + int32 source index per row, read
    int64 position + int32 slot per row, write position + slot per survivor."""
    return n * 2 * h * e + 21 * n + 12 * (n - exits)


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

    return tdist.init("nccl" if int(os.environ.get("WORLD_SIZE", "1")) > 1 else None)


def barrier(world):
    from tide_b200 import dist as tdist

    tdist.barrier(world)


def max_over_ranks(world, v: float) -> float:
    from tide_b200 import dist as tdist

    return tdist.max_over_ranks(world, v)


class Workload:
    """Device-resident inputs and buffers of one rank's checkpoint sweep."""

    def __init__(self, rank: int, path: int):
        from tide_b200 import workloads
        from tide_b200.ops import CheckpointRunner, NormSpec, prepare_router
        from tide_b200.capi import NORM_RMS

        dev = torch.device("cuda")
        g = torch.Generator(device=dev).manual_seed(1234 + rank)
        self.path = path
        dt = DTYPE_NAMES[DTYPE]
        scaled = WORKLOADS[WORKLOAD].get("inputs") == "scaled"
        w_norm = (1.0 + 0.02 * torch.randn(HIDDEN, generator=g, device=dev) if scaled
                  else torch.ones(HIDDEN, device=dev))
        self.norm = NormSpec(NORM_RMS, w_norm, None, 1e-5)
        self.runner = CheckpointRunner(dev)
        self.x, self.routers, self.active = [], [], []
        active = ROWS
        for k, layer in enumerate(LAYERS):
            x = torch.randn(ROWS, HIDDEN, generator=g, device=dev)
            if scaled:
                x = x * (torch.rand(ROWS, 1, generator=g, device=dev) * 1.5 + 0.5)
            x = x.to(dt)
            down = 0.02 * torch.randn(BOTTLENECK, HIDDEN, generator=g, device=dev)
            up = 0.02 * torch.randn(1, BOTTLENECK, generator=g, device=dev)
            z = workloads.prebias_logits_torch(x[:active], "rms", self.norm.weight, None, 1e-5,
                                               down, up)
            if EXITS_OF == "batch":
                exits = int(round(EXIT_FRACTIONS[k] * ROWS)) if k < len(LAYERS) - 1 else active
            else:
                exits = int(round(EXIT_FRACTIONS[k] * active))
            bias = workloads.bias_for_exit_fraction(z, exits / active, THRESHOLD)
            self.routers.append(prepare_router(down, up, bias, self.norm, dt))
            self.x.append(x)
            self.active.append(active)
            active -= exits
        self.positions0 = torch.arange(ROWS, device=dev, dtype=torch.int64)
        self.slots0 = torch.arange(ROWS, device=dev, dtype=torch.int32)
        self.count0 = torch.tensor([ROWS], dtype=torch.int32, device=dev)
        self.out = torch.zeros(ROWS, HIDDEN, dtype=dt, device=dev)
        self.compact = torch.empty(ROWS, HIDDEN, dtype=dt, device=dev)
        self.pos = [torch.empty(ROWS, dtype=torch.int64, device=dev) for _ in range(2)]
        self.slots = [torch.empty(ROWS, dtype=torch.int32, device=dev) for _ in range(2)]
        self.counts = torch.zeros(len(LAYERS), 2, dtype=torch.int32, device=dev)
        self.paths = {}  # path the library chose for each checkpoint

    def checkpoint(self, k: int, xs=None):
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
                        n_rows_dev=cnt, counts=self.counts[k], path=self.path)
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


def gather_timings(world: int, wl: "Workload", reps: int = 5) -> dict:
    """The step's two collectives, timed on their own (not part of `value`):
    the all-gather of every rank's exit counts and of every rank's output
    rows (ncclAllGather over NVLink).  CUDA events, max over ranks."""
    from tide_b200 import dist as tdist

    rows_out = torch.empty((world * ROWS, HIDDEN), dtype=wl.out.dtype, device=wl.out.device)
    res = {}
    for name, fn, nbytes in (
            ("exit_counts", lambda: tdist.all_gather_counts(world, wl.counts),
             wl.counts.numel() * 4),
            ("output_rows", lambda: tdist.all_gather_rows(world, wl.out, rows_out),
             wl.out.numel() * wl.out.element_size())):
        fn()
        torch.cuda.synchronize()
        barrier(world)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(reps):
            fn()
        b.record()
        torch.cuda.synchronize()
        ms = max_over_ranks(world, a.elapsed_time(b) / reps)
        res[name] = {"ms": ms, "bytes_per_rank": nbytes,
                     "busbw_GBps": (world - 1) * nbytes / (ms / 1000.0) / 1e9}
    del rows_out
    return res


# ----------------------------------------------------------------- CPU leg
def host_threads() -> int:
    """Every host core for the CPU legs: torchrun sets OMP_NUM_THREADS=1 per
    rank, so the BLAS pool is raised explicitly."""
    from threadpoolctl import threadpool_limits

    n = os.cpu_count() or 1
    threadpool_limits(limits=n)
    return n


def cpu_checkpoint_sample(x: np.ndarray, down: np.ndarray, up: np.ndarray, bias: float,
                          norm_weight: np.ndarray):
    """The oracle on one checkpoint's rows (the reference's CPU path,
    restated): returns seconds.  x holds bf16 bit patterns (uint16) or fp32."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import tide_oracle as O

    norm = {"kind": "rms", "weight": norm_weight, "bias": None, "eps": 1e-5}
    out = np.zeros_like(x)
    t0 = time.perf_counter()
    O.checkpoint(x, O.F32 if x.dtype == np.float32 else O.BF16, norm, down, up, bias, THRESHOLD,
                 positions=np.arange(x.shape[0], dtype=np.int64),
                 slots=np.arange(x.shape[0], dtype=np.int32), out_buffer=out)
    return time.perf_counter() - t0


def cpu_sample_inputs(wl: "Workload", rows: int):
    x = wl.x[0][:rows].contiguous()
    x = x.cpu().numpy() if x.dtype == torch.float32 else x.view(torch.int16).cpu().numpy().view(np.uint16)
    r = wl.routers[0]
    down = r.down_t.T.contiguous().cpu().numpy()
    up = r.up.cpu().numpy().reshape(1, -1)
    return x, down, up, r.up_bias, wl.norm.weight.cpu().numpy()


# ----------------------------------------------------------------- main
def run_reference(args, world, rank):
    """--impl reference: the CPU restatement of the reference path (the
    reference is Python and cannot be built into a library), timed on the host
    cores with every thread numpy's BLAS can use; rank 0 only."""
    if rank != 0:
        return
    torch.cuda.set_device(0)
    wl = Workload(rank, 0)
    rows = min(4096, ROWS)
    cores = host_threads()
    x, down, up, bias, nw = cpu_sample_inputs(wl, rows)
    for _ in range(args.warmup):
        cpu_checkpoint_sample(x, down, up, bias, nw)
    ts = [cpu_checkpoint_sample(x, down, up, bias, nw) for _ in range(args.steps)]
    t = sum(ts)
    v = rows * args.steps / t
    line = {
        "impl": "reference", "metric": "router_compact_scatter_tokens_per_s", "value": v,
        "unit": "tokens/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1000 * t / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": DTYPE, "data": "synthetic",
        "config": {"workload": WORKLOAD, "sample_rows_per_step": rows, "hidden": HIDDEN,
                   "bottleneck": BOTTLENECK,
                   "checkpoint": f"first router (layer {LAYERS[0]}), {EXIT_FRACTIONS[0]:.0%} exit"},
        "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": cores, "kind": "port",
                         "sample": f"one checkpoint ({rows} rows x {HIDDEN} {DTYPE}) per step"},
        "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


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
    ap.add_argument("--workload", default=WORKLOAD, choices=sorted(WORKLOADS))
    ap.add_argument("--rows", type=int, default=None, help="rows per GPU (profiling runs)")
    args = ap.parse_args()
    wk = WORKLOADS[args.workload]
    globals().update(WORKLOAD=args.workload, LAYERS=wk["layers"], EXIT_FRACTIONS=wk["exit_fractions"],
                     EXITS_OF=wk["of"], ROWS=args.rows if args.rows else wk["rows"],
                     HIDDEN=wk.get("hidden", 4096), DTYPE=wk.get("dtype", "bf16"))
    world, rank, local = dist_setup(args.gpus)
    if args.impl == "reference":
        run_reference(args, world, rank)
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
        return

    from tide_b200.capi import PATH_AUTO, PATH_SIMT, PATH_TC, PATH_TC_SPLIT

    path = {"auto": PATH_AUTO, "simt": PATH_SIMT, "tc": PATH_TC, "tc_split": PATH_TC_SPLIT}[args.path]
    wl = Workload(rank, path)
    for _ in range(max(args.warmup, 3)):
        wl.step()
    torch.cuda.synchronize()
    path_used = wl.runner.last_path
    counts = wl.counts.cpu()
    rows_per_step = int(counts.sum().item())
    exits_per_stage = counts[:, 1].tolist()
    active = (counts[:, 0] + counts[:, 1]).tolist()
    wl.runner.check_errors()

    step_graph = wl.capture()[0]
    ck_graphs = wl.capture(per_checkpoint=True, calls=CK_CALLS)
    for _ in range(2):
        step_graph.replay()
        for g in ck_graphs:
            g.replay()
    torch.cuda.synchronize()

    # timed region: device-resident inputs, one graph launch per step on the
    # current stream, CUDA events before the first and after the last
    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize()
    with ClockSampler(local) as clocks:
        t_start.record()
        for _ in range(args.steps):
            step_graph.replay()
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
    from tide_b200 import dist as tdist

    # every rank: global {survivors, exits} per checkpoint (host bookkeeping,
    # outside the timed region)
    global_counts = tdist.sum_counts(world, wl.counts).cpu()
    collectives = gather_timings(world, wl) if world > 1 else None

    e = 4 if DTYPE == "f32" else 2
    alg = [algorithmic_bytes(active[k], exits_per_stage[k], HIDDEN, e) for k in range(len(LAYERS))]
    achieved = alg[0] / (per_ck[0] / 1000.0) / 1e9  # the first (largest) checkpoint
    achieved_all = sum(alg) / (elapsed / args.steps) / 1e9
    peaks = {}
    try:
        peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
    except Exception:
        pass
    peak = peaks.get("hbm_gbs", 6650.0)
    path_name = PATH_NAMES.get(wl.paths[0], wl.paths[0])
    traffic = (NCU_TRAFFIC_CKPT0["bytes"] if ROWS == NCU_TRAFFIC_CKPT0["rows"]
               and path_name == NCU_TRAFFIC_CKPT0["path"] else None)
    roofline = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                "frac": achieved / peak, "traffic": traffic,
                "traffic_source": "ncu launch list (warm caches), profiles/" if traffic else None,
                "peak_source": "measured" if "hbm_gbs" in peaks else "fallback",
                "kernel": f"checkpoint 0 ({ROWS} rows x {HIDDEN}), both kernels of the call",
                "per_checkpoint_ms": per_ck, "per_checkpoint_reps": reps,
                "per_checkpoint_calls_per_graph": CK_CALLS,
                "achieved_all_checkpoints": achieved_all, "algorithmic_bytes_per_step": sum(alg)}

    # e2e through the public operator with host buffers: H2D of the step's
    # hidden states from pinned memory (the rows each checkpoint routes), the
    # step graph, D2H of the counts
    host_x = [x[: active[k]].cpu().pin_memory() for k, x in enumerate(wl.x)]
    dev_x = [torch.empty_like(x) for x in wl.x]
    host_counts = torch.empty_like(wl.counts, device="cpu").pin_memory()

    e2e_steps = e2e_step_count(args.e2e_steps, ROWS * HIDDEN * e * len(LAYERS))
    e_graph = wl.capture(dev_x)[0]
    # one untimed step: the graph's first launch uploads it to the device
    for k in range(len(LAYERS)):
        dev_x[k][: active[k]].copy_(host_x[k], non_blocking=True)
    e_graph.replay()
    host_counts.copy_(wl.counts, non_blocking=True)
    barrier(world)
    torch.cuda.synchronize()
    e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e_start.record()
    for _ in range(e2e_steps):
        for k in range(len(LAYERS)):
            dev_x[k][: active[k]].copy_(host_x[k], non_blocking=True)
        e_graph.replay()
        host_counts.copy_(wl.counts, non_blocking=True)
    e_end.record()
    torch.cuda.synchronize()
    e_el = max_over_ranks(world, e_start.elapsed_time(e_end) / 1000.0)
    e2e = {"value": world * rows_per_step * e2e_steps / e_el, "unit": "tokens/s",
           "h2d_bytes_per_step": int(sum(x.numel() * x.element_size() for x in host_x)),
           "d2h_bytes_per_step": int(host_counts.numel() * 4), "steps": e2e_steps}
    del e_graph, step_graph, ck_graphs

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        rows = min(4096, ROWS)
        cores = host_threads()
        x, down, up, bias, nw = cpu_sample_inputs(wl, rows)
        cpu_checkpoint_sample(x, down, up, bias, nw)
        t = min(cpu_checkpoint_sample(x, down, up, bias, nw) for _ in range(3))
        cpu = {"value": rows / t, "unit": "tokens/s", "cores": cores, "kind": "port",
               "sample": f"oracle, one checkpoint of {rows} rows x {HIDDEN} {DTYPE} "
                         f"(layer-{LAYERS[0]} router), best of 3"}

    n_launch = sum(launches_per_checkpoint(p) for p in wl.paths.values()) * args.steps
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
                       "path": path_name,
                       "path_per_checkpoint": [PATH_NAMES.get(wl.paths[k], wl.paths[k])
                                               for k in range(len(LAYERS))],
                       "parallelism": f"dp{world} (row shards, no collective)",
                       "l2": "inputs 1.1 GiB/step > 126 MB L2, no flush"},
            "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e,
            "gpu_launches": n_launch, "clocks": clocks.summary(),
            "collectives_timed_separately": collectives,
            "prefill_tokens_per_s": world * ROWS * args.steps / elapsed,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
