#!/usr/bin/env python
"""bench.py -- throughput of v7's fused elementwise/reduction path on B200.

Workload (the largest and the one sharded over GPUs):
C5 SwiGLU + Q8 requantisation, gate/up [16384, 12288] fp32 ~ N(0, 2) ->
int8 codes [16384, 12288] + fp32 scales [16384, 192].  The 16384 rows are
split into contiguous shards, one per GPU (rank r takes rows
[r*R/N, (r+1)*R/N)), with no collective on the timed path (rows are
independent): total work is fixed, so scaling is strong.  A step is one launch
of the fused kernel over the rank's shard.

Reported (one JSON line from rank 0):
  value      whole-job algorithmic GB/s (inputs read once + outputs written
             once) / max-over-ranks device time of K launches issued back to
             back between one start and one end event, inputs resident in HBM
  verified   every code and scale of the whole job, gathered to rank 0 over
             NCCL after timing, against the oracle on the same input bytes
             (bit-exact); a mismatch makes the run exit non-zero
  e2e        the same metric through the public API with host buffers: every
             step copies the shard's gate/up from pinned host memory and reads
             codes/scales back (pipelined in row chunks over three streams);
             e2e.link times the same copies alone, per rank and in aggregate,
             the step's floor on the host link
  roofline   the kernel's achieved GB/s against the measured HBM copy peak
  cpu_baseline  the oracle port on the host cores, whole C5 passes for about
             --cpu-seconds (N=1 only)
  kernels    the other BASELINE configs (C1-C4) and the next rows (add_inplace,
             RMSNorm->Q8, RoPE without the norm, the RoPE table build, the
             Q8-weight GEMVs), device-timed, N=1 only
``--impl reference`` times the CPU implementation instead (rank 0 only):
whole 16384-row C5 passes on the GPU arm's input bytes, all host threads.
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

METRIC = "fused-kernel HBM GB/s (% of B200 peak) and rows/s at 1/2/4/8 GPUs"
L2_BYTES = 126 * 2**20
C5_ROWS, C5_N = 16384, 12288
GROUP = 64
SEED_GATE, SEED_UP = 12, 13


def c5_bytes(rows: int, n: int = C5_N) -> int:
    """Algorithmic bytes: gate + up read once, codes + scales written once."""
    return rows * (n * 4 * 2 + n + (n // GROUP) * 4)


def measured_peaks() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def ncu_traffic() -> dict:
    """Per-launch DRAM bytes of each kernel from the committed ncu summary."""
    p = ROOT / "profiles" / "ncu_traffic.json"
    return json.loads(p.read_text()) if p.exists() else {}


# ------------------------------------------------------------------ clocks


class ClockSampler:
    """Samples SM clock and clock-event reasons through NVML while running,
    with the memory clock, board power and GPU temperature beside them.  Each
    sample carries its host time; mark_start / mark_end bracket the timed
    region, and summary() reports the samples inside it (all samples when no
    region was marked)."""

    REASONS = {"hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20, "sw_power_cap": 0x4,
               "hw_power_brake_slowdown": 0x80}

    def __init__(self, device_index: int, period_s: float = 0.001):
        self.samples: list[tuple] = []  # (t, sm MHz, reasons, memory MHz, board W, GPU C)
        self.period = period_s
        self.ok = False
        self.t0 = self.t1 = None
        try:
            import pynvml
            pynvml.nvmlInit()
            uuid = str(torch.cuda.get_device_properties(device_index).uuid)
            uuid = uuid if uuid.startswith("GPU-") else "GPU-" + uuid
            self.h = pynvml.nvmlDeviceGetHandleByUUID(uuid.encode())
            self.nvml = pynvml
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.mem_max_mhz = self._extra(lambda: pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_MEM))
            self.ok = True
        except Exception as e:  # pragma: no cover - reported in the JSON line
            self.err = repr(e)
        self._stop = threading.Event()
        self._t = None

    def sample(self, full: bool = False) -> None:
        """One reading: the SM clock and the reasons; with `full` also the
        slower readings that only explain them (memory clock, power,
        temperature)."""
        n = self.nvml
        try:
            t = time.perf_counter()
            sm = n.nvmlDeviceGetClockInfo(self.h, n.NVML_CLOCK_SM)
            reasons = n.nvmlDeviceGetCurrentClocksEventReasons(self.h)
            extra = (None, None, None)
            if full:
                extra = (self._extra(lambda: n.nvmlDeviceGetClockInfo(self.h, n.NVML_CLOCK_MEM)),
                         self._extra(lambda: n.nvmlDeviceGetPowerUsage(self.h) / 1000.0),
                         self._extra(lambda: n.nvmlDeviceGetTemperature(self.h, n.NVML_TEMPERATURE_GPU)))
            self.samples.append((t, sm, reasons) + extra)
        except Exception:
            pass

    def sample_until(self, event: "torch.cuda.Event") -> None:
        """Samples from the calling thread until `event` has completed on the
        device: called with the timed region's launches queued, so every
        reading falls inside the region however short it is."""
        if not self.ok:
            return
        k = 0
        while not event.query():
            self.sample(full=k % 10 == 0)
            k += 1

    def _run(self):
        k = 0
        while True:
            # every tenth sample with the slower readings
            self.sample(full=k % 10 == 0)
            k += 1
            if self._stop.wait(self.period):
                break

    @staticmethod
    def _extra(read):
        """A reading that only explains the clocks (memory clock, power,
        temperature): None where this driver does not give it."""
        try:
            return read()
        except Exception:
            return None

    def mark_start(self):
        self.t0 = time.perf_counter()

    def mark_end(self):
        self.t1 = time.perf_counter()

    def __enter__(self):
        if self.ok:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._t:
            self._t.join()

    def summary(self) -> dict:
        if not self.ok:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "error": getattr(self, "err", "nvml unavailable")}
        inside = [x for x in self.samples if self.t0 is None or self.t0 <= x[0] <= self.t1]
        use = inside or self.samples
        reasons = sorted({name for _, _, r, *_ in use for name, bit in self.REASONS.items() if r & bit})

        def med(i):
            v = [x[i] for x in use if x[i] is not None] or [x[i] for x in self.samples if x[i] is not None]
            return statistics.median(v) if v else None
        return {"sm_mhz": med(1), "sm_max_mhz": self.max_mhz, "reasons": reasons, "samples": len(inside),
                "samples_used": len(use), "mem_mhz": med(3), "mem_max_mhz": self.mem_max_mhz, "power_w": med(4),
                "temp_c_max": max((x[5] for x in use if x[5] is not None), default=None),
                "source": f"NVML: a background thread every {self.period * 1e3:g} ms, and back-to-back readings from the "
                          f"launching thread while the queued timed region runs (memory clock, power and temperature every "
                          f"tenth reading); samples = those inside the timed region"}


# ------------------------------------------------------------ distributed


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def shard(rows: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous row shard of rank (balanced to within one row)."""
    return rows * rank // world, rows * (rank + 1) // world


def max_over_ranks(x: float, world: int, device: str = "cuda") -> float:
    if world == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device=device)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(x: float, world: int, device: str = "cuda") -> float:
    if world == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device=device)
    torch.distributed.all_reduce(t)
    return float(t.item())


def gather_checksums(chk: torch.Tensor, world: int) -> list:
    """Per-rank output checksums to every rank (verification only, after timing)."""
    if world == 1:
        return [chk.cpu().tolist()]
    gathered = [torch.empty_like(chk) for _ in range(world)]
    torch.distributed.all_gather(gathered, chk)
    return torch.stack(gathered).cpu().tolist()


def gather_floats(vals: list, world: int, device: str = "cuda") -> list:
    """Every rank's list of floats, in rank order (NCCL all-gather, outside timed regions)."""
    t = torch.tensor(vals, dtype=torch.float64, device=device)
    if world == 1:
        return [t.cpu().tolist()]
    out = [torch.empty_like(t) for _ in range(world)]
    torch.distributed.all_gather(out, t)
    return [x.cpu().tolist() for x in out]


def barrier(world: int) -> None:
    if world > 1:
        torch.distributed.barrier()


def output_checksum(codes: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    """[sum of codes, sum of scale bit patterns] as int64: equal for equal outputs."""
    return torch.stack([codes.reshape(-1).to(torch.int64).sum(),
                        scales.contiguous().view(torch.int32).reshape(-1).to(torch.int64).sum()])


# ------------------------------------------------------------ timing helpers


def time_region(fn, steps: int, stream: torch.cuda.Stream, clk: "ClockSampler | None" = None) -> float:
    """Runs fn() `steps` times back to back on `stream` between ONE start and
    ONE end event; returns the region's ms.  No event sits between launches,
    so each launch may overlap the drain of the one ahead of it (the library's
    programmatic dependent launch), as in an engine's stream of kernels.
    With `clk`, the clocks are sampled from this thread while the queued
    region runs."""
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        # head start: keep the GPU busy (a bounded ~2 ms sleep) while the host
        # enqueues every launch, so no launch waits on the host's submission
        torch.cuda._sleep(4_000_000)
        start.record(stream)
        for _ in range(steps):
            fn()
        end.record(stream)
    if clk is not None:
        clk.sample_until(end)
    stream.synchronize()
    return start.elapsed_time(end)


def time_launches(fn, steps: int, stream: torch.cuda.Stream, flush: tuple | None = None):
    """Runs fn() `steps` times on `stream`, each launch between its own pair of
    events; returns (region_ms, per-launch ms list).  The events between
    launches keep a launch from overlapping the one ahead of it, so this gives
    single-launch times.  With `flush` = (buffer_a, buffer_b, out), both
    buffers larger than L2, buffer_a is rewritten and buffer_b read before
    every launch (outside the launch's own events): the write evicts the
    kernel's data, the read leaves L2 holding clean lines, so no write-back of
    the flush lands inside the timed launch."""
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        torch.cuda._sleep(4_000_000)
        start.record(stream)
        for a, b in ev:
            if flush is not None:
                flush[0].add_(1)
                torch.amax(flush[1], dim=0, out=flush[2])
            a.record(stream)
            fn()
            b.record(stream)
        end.record(stream)
    stream.synchronize()
    return start.elapsed_time(end), [a.elapsed_time(b) for a, b in ev]


# --------------------------------------------------------------- our arm


def run_ours(args, rank: int, world: int, local: int) -> None:
    import v7multiplikator_b200 as v7g

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    peak, peak_kind = measured_peaks()
    r0, r1 = shard(C5_ROWS, rank, world)
    rows = r1 - r0
    g = torch.empty(rows, C5_N, device=dev)
    u = torch.empty(rows, C5_N, device=dev)
    v7g.fill_normal(g, seed=SEED_GATE, mean=0.0, std=2.0, row0=r0)
    v7g.fill_normal(u, seed=SEED_UP, mean=0.0, std=2.0, row0=r0)
    codes = torch.empty(rows, C5_N, dtype=torch.int8, device=dev)
    scales = torch.empty(rows, C5_N // GROUP, device=dev)
    stream = torch.cuda.Stream(device=dev)

    def step():
        v7g.swiglu_q8_rows(codes, scales, g, u, stream=stream)

    torch.cuda.synchronize()  # inputs were written on the default stream
    with ClockSampler(local) as clk:  # running from the warm-up on; summary() keeps the timed region
        with torch.cuda.stream(stream):
            for _ in range(args.warmup):
                step()
        stream.synchronize()
        barrier(world)
        launches0 = v7g.launch_count()
        torch.cuda.synchronize()
        barrier(world)
        torch.cuda.synchronize()
        clk.mark_start()
        region_ms = time_region(step, args.steps, stream, clk)
        clk.mark_end()
        launches = v7g.launch_count() - launches0
        torch.cuda.synchronize()
        barrier(world)
    t_max = max_over_ranks(region_ms, world)
    total_bytes = c5_bytes(C5_ROWS) * args.steps
    value = total_bytes / (t_max * 1e-3) / 1e9
    rows_per_s = C5_ROWS * args.steps / (t_max * 1e-3)
    launch_ms = region_ms / args.steps  # this rank's mean launch in the back-to-back region
    achieved = c5_bytes(rows) / (launch_ms * 1e-3) / 1e9
    gpu_launches = int(sum_over_ranks(launches, world))
    # single launches (an event pair around each), outside the timed region
    _, per_launch = time_launches(step, min(args.steps, 20), stream)
    launch_ms_single = statistics.mean(per_launch)

    # verification (outside the timed region): every code and scale of the
    # whole job gathered to rank 0 over NCCL and compared with the oracle
    verified = verify_outputs(codes, scales, rank, world)
    chk_all = gather_checksums(output_checksum(codes, scales), world)

    e2e = run_e2e(args, v7g, dev, g, u, codes, scales, rows, world)

    table = None
    cpu = None
    if world == 1 and not args.no_extras:
        table = kernel_table(v7g, dev, stream, peak)
        cpu = cpu_baseline(args)
    traffic = ncu_traffic().get("swiglu_q8_c5_per_row")
    line = {
        "metric": METRIC,
        "value": round(value, 2),
        "unit": "GB/s",
        "rows_per_s": round(rows_per_s, 1),
        "pct_of_peak": round(100.0 * value / (world * peak), 2),
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(t_max / args.steps, 6),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "f32",
        "data": f"synthetic: counter-based N(0, 2) gate/up (seed {SEED_GATE}/{SEED_UP}), generated on device per row shard",
        "config": {
            "workload": "C5 SwiGLU + Q8 requantisation: gate/up [16384, 12288] fp32 -> int8 codes [16384, 12288] "
                        "+ fp32 scales [16384, 192] (one per 64-element group)",
            "rows": C5_ROWS, "n": C5_N, "rows_per_gpu": rows, "parallelism": f"row-shard x{world}, no collective",
            "bytes_per_row": c5_bytes(1), "l2": "inputs 1.61 GB > 126 MB L2: no flush needed",
            "launch_overlap": v7g.launch_overlap(),
            "timed_region": "K launches back to back between one start and one end event (no event between launches)",
        },
        "roofline": {
            "bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
            "frac": round(achieved / peak, 4),
            "peak_kind": ("measured (MEASURED_PEAKS.json hbm_gbs, a STREAM-style copy)" if peak_kind == "measured"
                          else "fallback 6650 GB/s (MEASURED_PEAKS.json absent)"),
            "traffic": round(traffic * rows) if traffic else None, "launch_ms": round(launch_ms, 5),
            "launch_ms_single": round(launch_ms_single, 5),
            "launch_ms_note": "launch_ms = this rank's timed region / K (back to back); launch_ms_single = mean of "
                              "single launches, each between its own events",
            "kernel": "k_q8_groups<true> (v7g_swiglu_q8_rows)",
        },
        "verified": verified,
        "e2e": e2e,
        "clocks": clk.summary(),
        "gpu_launches": gpu_launches,
        "checksums": chk_all,
    }
    if cpu is not None:
        line["cpu_baseline"] = cpu
    if table is not None:
        line["kernels"] = table
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()
    if verified.get("mismatches", 1) != 0:
        sys.exit(3)


def verify_outputs(codes: torch.Tensor, scales: torch.Tensor, rank: int, world: int, total_rows: int = C5_ROWS,
                   n: int = C5_N) -> dict:
    """Every code and scale of the whole job against the oracle.  The ranks'
    shards are gathered to every rank with one all-gather each (codes, scale
    bits; NCCL on the GPUs, verification only, after the timed region); rank 0
    regenerates all `total_rows` rows of gate/up on the host with the
    generator's restatement (bit-identical to the device fill), runs the
    oracle's SwiGLU -> Q8 and compares bit for bit.  The other ranks wait at a
    barrier, then learn the count by a broadcast."""
    rows = codes.shape[0]
    shard_rows = [shard(total_rows, r, world) for r in range(world)]
    max_rows = max(b - a for a, b in shard_rows)
    if world > 1:
        # equal-sized pieces for the all-gather: pad this rank's shard
        c_pad = torch.zeros(max_rows, n, dtype=torch.int8, device=codes.device)
        s_pad = torch.zeros(max_rows, n // GROUP, dtype=torch.int32, device=codes.device)
        c_pad[:rows] = codes
        s_pad[:rows] = scales.view(torch.int32)
        c_all = torch.empty(world * max_rows, n, dtype=torch.int8, device=codes.device)
        s_all = torch.empty(world * max_rows, n // GROUP, dtype=torch.int32, device=codes.device)
        torch.distributed.all_gather_into_tensor(c_all, c_pad)
        torch.distributed.all_gather_into_tensor(s_all, s_pad)
        keep = torch.cat([torch.arange(r * max_rows, r * max_rows + (b - a), device=codes.device)
                          for r, (a, b) in enumerate(shard_rows)])
        c_all, s_all = c_all[keep], s_all[keep]
    else:
        c_all, s_all = codes, scales.view(torch.int32)
    out = {"rows": total_rows, "ranks": world}
    if rank == 0:
        from oracle.pyoracle import Oracle
        t = time.perf_counter()
        orc = Oracle(nthreads=os.cpu_count() or 1)
        g = orc.fill_normal(total_rows, n, 0, SEED_GATE, 0.0, 2.0)
        u = orc.fill_normal(total_rows, n, 0, SEED_UP, 0.0, 2.0)
        want_c, want_s = orc.swiglu_q8(g, u)
        del g, u
        got_c = c_all.cpu().numpy()
        got_s = s_all.cpu().numpy()
        bad_c = int(np.count_nonzero(got_c != want_c))
        bad_s = int(np.count_nonzero(got_s != want_s.view(np.int32)))
        out.update({"codes": int(got_c.size), "scales": int(got_s.size), "code_mismatches": bad_c,
                    "scale_mismatches": bad_s, "mismatches": bad_c + bad_s,
                    "method": "all-gather of every rank's codes and scale bits; oracle/v7_oracle.c SwiGLU -> Q8 "
                              "on host-regenerated gate/up (orc_fill_normal, bit-identical to the device fill); "
                              "bit-exact comparison of every element",
                    "seconds": round(time.perf_counter() - t, 2)})
    barrier(world)
    if world > 1:
        flag = torch.tensor([out.get("mismatches", 0)], dtype=torch.int64, device=codes.device)
        torch.distributed.broadcast(flag, 0)
        out.setdefault("mismatches", int(flag.item()))
    return out


def run_e2e(args, v7g, dev, g, u, codes, scales, rows, world):
    """Public-API end to end: pinned host gate/up in, codes/scales out, every
    step.  Rows go in chunks over three streams so the host-to-device copy of
    chunk i+1 overlaps the kernel and the device-to-host copy of chunk i."""
    hg = torch.empty(rows, C5_N, dtype=torch.float32, pin_memory=True)
    hu = torch.empty(rows, C5_N, dtype=torch.float32, pin_memory=True)
    hg.copy_(g)
    hu.copy_(u)
    hc = torch.empty(rows, C5_N, dtype=torch.int8, pin_memory=True)
    hs = torch.empty(rows, C5_N // GROUP, dtype=torch.float32, pin_memory=True)
    streams = [torch.cuda.Stream(device=dev) for _ in range(3)]
    nchunks = max(1, min(16, rows // 256))
    bounds = [(rows * i // nchunks, rows * (i + 1) // nchunks) for i in range(nchunks)]

    def step():
        for i, (a, b) in enumerate(bounds):
            s = streams[i % len(streams)]
            with torch.cuda.stream(s):
                g[a:b].copy_(hg[a:b], non_blocking=True)
                u[a:b].copy_(hu[a:b], non_blocking=True)
                v7g.swiglu_q8_rows(codes[a:b], scales[a:b], g[a:b], u[a:b], stream=s)
                hc[a:b].copy_(codes[a:b], non_blocking=True)
                hs[a:b].copy_(scales[a:b], non_blocking=True)

    steps = max(3, min(args.steps, 20))
    step()
    torch.cuda.synchronize()
    barrier(world)
    t0 = time.perf_counter()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    cur = torch.cuda.current_stream(dev)
    start.record(cur)
    for _ in range(steps):
        for s in streams:
            s.wait_stream(cur)
        step()
        for s in streams:
            cur.wait_stream(s)
    end.record(cur)
    torch.cuda.synchronize()
    ms = start.elapsed_time(end)
    wall = (time.perf_counter() - t0) * 1e3
    t_max = max_over_ranks(ms, world)
    value = c5_bytes(C5_ROWS) * steps / (t_max * 1e-3) / 1e9
    # the host buffers the API filled equal the device outputs of the timed region
    same = bool(torch.equal(hc.to(dev), codes) and torch.equal(hs.to(dev).view(torch.int32), scales.view(torch.int32)))
    same = int(sum_over_ranks(0 if same else 1, world)) == 0
    per_rank_ms = gather_floats([ms / steps], world)
    link = host_link(dev, (hg, hu), (g, u), (hc, hs), (codes, scales), world)
    floor_ms = max(link["h2d_ms"], link["d2h_ms"])
    link["floor_ms_per_step"] = round(floor_ms, 4)
    link["frac"] = round(floor_ms / (t_max / steps), 4)
    return {"value": round(value, 2), "unit": "GB/s", "steps": steps,
            "h2d_bytes_per_step": int(C5_ROWS * C5_N * 8), "d2h_bytes_per_step": int(C5_ROWS * (C5_N + C5_N // GROUP * 4)),
            "ms_per_step": round(t_max / steps, 4), "wall_ms_per_step_rank0": round(wall / steps, 4),
            "ms_per_step_per_rank": [round(x[0], 4) for x in per_rank_ms],
            "outputs_match_device": same,
            "path": f"pinned host -> v7g_swiglu_q8_rows -> pinned host, {nchunks} row chunks on 3 streams",
            "link": link}


def host_link(dev, h_in, d_in, h_out, d_out, world, reps: int = 3) -> dict:
    """The host link alone: one step's input copies (pinned host -> device)
    and, separately, its output copies (device -> pinned host), each timed
    with CUDA events on one stream, max over ranks.  The slower direction is
    the floor of the end-to-end step, whose copies overlap each other and
    the kernel."""
    s = torch.cuda.Stream(device=dev)
    out = {}
    for name, src, dst in (("h2d", h_in, d_in), ("d2h", d_out, h_out)):
        nbytes = sum(t.numel() * t.element_size() for t in src)
        with torch.cuda.stream(s):
            for a, b in zip(src, dst):
                b.copy_(a, non_blocking=True)
        s.synchronize()
        barrier(world)
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record(s)
        with torch.cuda.stream(s):
            for _ in range(reps):
                for a, b in zip(src, dst):
                    b.copy_(a, non_blocking=True)
        end.record(s)
        s.synchronize()
        mine = start.elapsed_time(end) / reps
        ranks = [x[0] for x in gather_floats([mine], world)]
        ms = max(ranks)
        out[f"{name}_ms"] = round(ms, 4)
        out[f"{name}_gbs"] = round(nbytes / (ms * 1e-3) / 1e9, 2)
        # every rank's own copy rate, and the whole job's (all ranks' bytes over the slowest rank's time)
        out[f"{name}_gbs_per_rank"] = [round(nbytes / (t * 1e-3) / 1e9, 2) for t in ranks]
        out[f"{name}_gbs_aggregate"] = round(world * nbytes / (ms * 1e-3) / 1e9, 2)
    out["copies"] = "all ranks at once (after a barrier), pinned host buffers, one stream per rank"
    return out


def kernel_table(v7g, dev, stream, peak) -> dict:
    """Device-timed GB/s of the other BASELINE configs on one GPU.

    us        mean of 50 single launches, each behind an L2 flush for the
              configs whose inputs fit in L2 (C1, C2, C3 and the add,
              RMSNorm->Q8, RoPE-only and GEMV rows).  The event clock ticks
              in steps of about 2 us on this part, so the mean (the launch
              starts at a random phase of the tick) is the estimate;
              us_median is kept beside it.
    us_b2b    launches back to back, cycling over `b2b_sets` copies of the
              inputs whose total is over twice L2, so that no launch finds
              its inputs in L2: the per-launch cost in a stream of launches,
              as an inference engine issues them.  C1 (1 MB) has one set: L2
              resident, labelled as such.  Launch overlap (programmatic
              dependent launch) is on, the library's default;
              us_b2b_no_overlap repeats the figure with plain launches."""
    out = {}
    # 512 MB written + 512 MB read (each > 4x L2) before every flushed launch
    flush = (torch.zeros(128 * 2**20, device=dev), torch.zeros(1024, 128 * 1024, device=dev),
             torch.empty(128 * 1024, device=dev))
    K = 50

    def sets_for(set_bytes: int) -> int:
        return max(2, -(-2 * L2_BYTES // set_bytes) + 1)

    def b2b(fns) -> float:
        n = max(30, 3 * len(fns))
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            for f in fns:
                f()
            torch.cuda._sleep(4_000_000)  # every launch queued before the first runs
            start.record(stream)
            for i in range(n):
                fns[i % len(fns)]()
            end.record(stream)
        stream.synchronize()
        return start.elapsed_time(end) / n

    def rec(name, fns, nbytes, rows, flushed, note=""):
        fns = fns if isinstance(fns, list) else [fns]
        torch.cuda.synchronize()  # inputs were written on the default stream
        with torch.cuda.stream(stream):
            for _ in range(3):
                fns[0]()
        stream.synchronize()
        _, per = time_launches(fns[0], K, stream, flush if flushed else None)
        ms = statistics.mean(per)
        gbs = nbytes / (ms * 1e-3) / 1e9
        ms_b = b2b(fns)
        gbs_b = nbytes / (ms_b * 1e-3) / 1e9
        v7g.set_launch_overlap(False)
        try:
            ms_p = b2b(fns)
        finally:
            v7g.set_launch_overlap(True)
        out[name] = {"gbs": round(gbs, 1), "frac": round(gbs / peak, 4), "us": round(ms * 1e3, 2),
                     "us_median": round(statistics.median(per) * 1e3, 2),
                     "rows_per_s": round(rows / (ms * 1e-3), 1), "bytes": nbytes, "l2_flushed": flushed,
                     "us_b2b": round(ms_b * 1e3, 2), "gbs_b2b": round(gbs_b, 1), "frac_b2b": round(gbs_b / peak, 4),
                     "b2b_sets": len(fns), "us_b2b_no_overlap": round(ms_p * 1e3, 2)}
        if note:
            out[name]["note"] = note

    def fill(shape, seed, mean, std):
        t = torch.empty(*shape, device=dev)
        return v7g.fill_normal(t.view(-1, shape[-1]), seed=seed, mean=mean, std=std)

    def copies(n, *ts):
        return [tuple(ts)] + [tuple(t.clone() for t in ts) for _ in range(n - 1)]

    # C1 RMSNorm x[64, 2048]
    x = fill((64, 2048), 1, 0.0, 1.0)
    w = fill((1, 2048), 2, 1.0, 0.1)[0]
    o = torch.empty_like(x)
    rec("c1_rmsnorm_64x2048", lambda: v7g.rmsnorm_rows(o, x, w, 1e-6, stream=stream), 64 * 2048 * 8 + 2048 * 4, 64, True,
        "launch/latency-bound: 1 MiB of traffic; us_b2b is L2-resident")
    # C2 fused add + RMSNorm [4096, 2048]
    r = fill((4096, 2048), 3, 0.0, 1.0)
    d = fill((4096, 2048), 4, 0.0, 0.5)
    c2b = 4096 * 2048 * 16 + 2048 * 4
    sets = copies(sets_for(c2b), r, d, torch.empty_like(r))
    rec("c2_fused_add_rmsnorm_4096x2048",
        [lambda t=t: v7g.fused_add_rmsnorm_rows(t[2], t[0], t[1], w, 1e-6, stream=stream) for t in sets],
        c2b, 4096, True)
    rec("add_inplace_4096x2048", [lambda t=t: v7g.add_inplace(t[0], t[1], stream=stream) for t in sets],
        4096 * 2048 * 12, 4096, True)
    del sets
    # C3 RMSNorm + RoPE Q[8192,16,128] K[8192,8,128]
    q = fill((8192, 16 * 128), 6, 0.0, 1.0).view(8192, 16, 128)
    k = fill((8192, 8 * 128), 7, 0.0, 1.0).view(8192, 8, 128)
    wq = fill((1, 128), 8, 1.0, 0.1)[0]
    wk = fill((1, 128), 9, 1.0, 0.1)[0]
    cos, sin = v7g.rope_tables(8192, 64, 1e6, device=dev)
    c3b = 8192 * 24 * 128 * 8 + 8192 * 64 * 8
    sets = copies(sets_for(c3b), q, k, cos, sin)
    # Q + K are 100.7 MB, under the 126 MB L2: flushed
    rec("c3_rmsnorm_rope_8192x(16+8)x128",
        [lambda t=t: v7g.rmsnorm_rope_rows(t[0], t[1], wq, wk, t[2], t[3], 0, 1e-6, stream=stream) for t in sets],
        c3b + 2 * 128 * 4, 8192, True)
    # RoPE without the norm at the C3 geometry
    rec("rope_only_8192x(16+8)x128", [lambda t=t: v7g.rope_only_rows(t[0], t[1], t[2], t[3], 0, stream=stream) for t in sets],
        c3b, 8192, True)
    del q, k, sets
    # the reference's internal tables: 131072 positions x 64 pairs, cos + sin written
    tc = torch.empty(131072, 64, device=dev)
    ts = torch.empty_like(tc)
    freqs = np.ascontiguousarray(v7g.rope_freqs(64, 1e6))
    rec("rope_tables_131072x64", lambda: v7g.ops._check(v7g.lib().v7g_rope_tables(
        tc.data_ptr(), ts.data_ptr(), 0, 131072, 64, 64, freqs.ctypes.data, stream.cuda_stream)),
        131072 * 64 * 8, 131072, False, "double-precision sincos per entry: FP64-bound, not HBM-bound")
    del tc, ts
    # C4 SwiGLU [4096, 8192]
    gg = fill((4096, 8192), 10, 0.0, 2.0)
    uu = fill((4096, 8192), 11, 0.0, 2.0)
    oo = torch.empty_like(gg)
    sets = copies(2, gg, uu, oo)  # 403 MB per set: no launch finds its inputs in L2
    rec("c4_swiglu_4096x8192", [lambda t=t: v7g.swiglu(t[2], t[0], t[1], stream=stream) for t in sets],
        4096 * 8192 * 12, 4096, False)
    del gg, uu, oo, sets
    # Q8-weight GEMVs (decode, batch 1) at model shapes; weights under L2 size: flushed
    for n, d in ((2048, 8192), (4096, 12288)):
        xq, xs, gq, gs, uq, us = gemv_inputs(dev, n, d)
        y = torch.empty(1, d, device=dev)
        nb = 2 * d * (n + n // 16) + n + n // 16 + 4 * d
        sets = copies(sets_for(nb), gq, gs, uq, us)
        rec(f"swiglu_q8_gemv_{n}x{d}",
            [lambda t=t: v7g.swiglu_q8_gemv(y, xq, xs, t[0], t[1], t[2], t[3], stream=stream) for t in sets], nb, d, True)
        if n == 4096:
            # four activation rows in one call: one pass over the weights (token blocks)
            x4q, x4s = gemv_batch_acts(dev, 4, n)
            y4 = torch.empty(4, d, device=dev)
            rec(f"swiglu_q8_gemv_{n}x{d}_batch4",
                [lambda t=t: v7g.swiglu_q8_gemv(y4, x4q, x4s, t[0], t[1], t[2], t[3], stream=stream) for t in sets],
                2 * d * (n + n // 16) + 4 * (n + n // 16) + 4 * 4 * d, 4 * d, True)
        if n == 2048:
            xf = fill((1, n), 14, 0.0, 1.0)
            rec(f"swiglu_f32q8_gemv_{n}x{d}",
                [lambda t=t: v7g.swiglu_f32q8_gemv(y, xf, t[0], t[1], t[2], t[3], stream=stream) for t in sets],
                2 * d * (n + n // 16) + 4 * n + 4 * d, d, True)
        del gq, gs, uq, us, sets
    xq, xs, wq, ws, _, _ = gemv_inputs(dev, 8192, 2048, both=False)
    y = torch.empty(1, 2048, device=dev)
    nb = 2048 * (8192 + 8192 // 16) + 8192 + 8192 // 16 + 4 * 2048
    sets = copies(sets_for(nb), wq, ws)
    rec("q8_gemv_8192x2048", [lambda t=t: v7g.q8_gemv(y, xq, xs, t[0], t[1], stream=stream) for t in sets], nb, 2048, True)
    x4q, x4s = gemv_batch_acts(dev, 4, 8192)
    y4 = torch.empty(4, 2048, device=dev)
    rec("q8_gemv_8192x2048_batch4", [lambda t=t: v7g.q8_gemv(y4, x4q, x4s, t[0], t[1], stream=stream) for t in sets],
        2048 * (8192 + 8192 // 16) + 4 * (8192 + 8192 // 16) + 4 * 4 * 2048, 4 * 2048, True)
    xf = fill((1, 8192), 15, 0.0, 1.0)
    rec("q8_fused_gemv_8192x2048", [lambda t=t: v7g.q8_fused_gemv(y, xf, t[0], t[1], stream=stream) for t in sets],
        2048 * (8192 + 8192 // 16) + 4 * 8192 + 4 * 2048, 2048, True)
    del wq, ws, sets
    # RMSNorm -> Q8 at the C2 shape
    nb = 4096 * (2048 * 5 + 32 * 4) + 2048 * 4
    sets = copies(sets_for(nb), r, torch.empty(4096, 2048, dtype=torch.int8, device=dev), torch.empty(4096, 32, device=dev))
    rec("rmsnorm_quantize_4096x2048",
        [lambda t=t: v7g.rmsnorm_quantize_rows(t[1], t[2], t[0], w, 1e-6, stream=stream) for t in sets], nb, 4096, True)
    # RMSNorm at the C2 shape (4096 rows: the shared-memory row pipeline)
    nb = 4096 * 2048 * 8 + 2048 * 4
    sets = copies(sets_for(nb), r, torch.empty_like(r))
    rec("rmsnorm_4096x2048", [lambda t=t: v7g.rmsnorm_rows(t[1], t[0], w, 1e-6, stream=stream) for t in sets], nb, 4096, True)
    del sets
    # size-matched floors: torch's own copy_ of as many bytes (half read, half
    # written) as the row kernels above move, timed the same way
    for label, nbytes in (("42MB", 42_475_520), ("67MB", 67_117_056), ("134MB", 134_225_920)):
        n = nbytes // 8 // 4 * 4
        sets = copies(sets_for(8 * n), torch.zeros(n, device=dev), torch.empty(n, device=dev))
        rec(f"copy_floor_{label}", [lambda t=t: t[1].copy_(t[0]) for t in sets], 8 * n, 1, True,
            "torch copy_ of the row kernels' byte count: what a plain copy reaches at this size")
        del sets
    return out


def gemv_batch_acts(dev, batch: int, n: int):
    """Random Q8 activation rows (codes in [-127, 127], scales in [0.001, 0.02))."""
    g = torch.Generator(device=dev)
    g.manual_seed(n * 17 + batch)
    return (torch.randint(-127, 128, (batch, n), generator=g, device=dev, dtype=torch.int8),
            torch.rand(batch, n // 64, generator=g, device=dev) * 0.019 + 0.001)


def gemv_inputs(dev, n: int, d: int, both: bool = True):
    """Random Q8 activation and weights for a GEMV: codes uniform in
    [-127, 127], scales uniform in [0.001, 0.02)."""
    g = torch.Generator(device=dev)
    g.manual_seed(n * 31 + d)

    def codes(*shape):
        return torch.randint(-127, 128, shape, generator=g, device=dev, dtype=torch.int8)

    def scales(*shape):
        return torch.rand(*shape, generator=g, device=dev) * 0.019 + 0.001

    xq, xs = codes(1, n), scales(1, n // 64)
    gq, gs = codes(d, n), scales(d, n // 64)
    uq, us = (codes(d, n), scales(d, n // 64)) if both else (None, None)
    return xq, xs, gq, gs, uq, us


def c5_host_inputs(orc, rows: int = C5_ROWS):
    """C5 gate/up on the host: the generator's restatement, so these are the
    GPU arm's input bytes (rows 0 .. rows - 1)."""
    g = orc.fill_normal(rows, C5_N, 0, SEED_GATE, 0.0, 2.0)
    u = orc.fill_normal(rows, C5_N, 0, SEED_UP, 0.0, 2.0)
    return g, u


def cpu_baseline(args) -> dict:
    """The oracle port of the reference's AVX2 kernels on the host cores, on the
    GPU arm's own input bytes: whole 16384-row C5 passes into preallocated
    outputs, repeated until about --cpu-seconds of wall time (one untimed pass
    first); plus one core on 1024 rows, the way the reference runs a kernel."""
    from oracle.pyoracle import Oracle
    threads = os.cpu_count() or 1
    orc = Oracle(nthreads=threads)
    g, u = c5_host_inputs(orc)
    out = (np.empty((C5_ROWS, C5_N), np.int8), np.empty((C5_ROWS, C5_N // GROUP), np.float32))
    orc.swiglu_q8_avx2(g, u, out=out)  # untimed: first touch of the outputs
    passes = 0
    t = time.perf_counter()
    while True:
        orc.swiglu_q8_avx2(g, u, out=out)
        passes += 1
        dt = time.perf_counter() - t
        if dt >= args.cpu_seconds:
            break
    gbs = c5_bytes(C5_ROWS) * passes / dt / 1e9
    one = Oracle(nthreads=1)
    rows1 = 1024
    out1 = (out[0][:rows1], out[1][:rows1])
    one.swiglu_q8_avx2(g[:rows1], u[:rows1], out=out1)
    t = time.perf_counter()
    one.swiglu_q8_avx2(g[:rows1], u[:rows1], out=out1)
    dt1 = time.perf_counter() - t
    return {"value": round(gbs, 3), "unit": "GB/s", "rows_per_s": round(C5_ROWS * passes / dt, 1), "cores": threads,
            "kind": "port",
            "sample": f"{passes} passes over all 16384 C5 rows ({dt:.1f} s), oracle/v7_oracle.c restatement in AVX2 "
                      f"(the reference's instruction forms, bit-identical to the scalar oracle), {threads} threads, "
                      f"the GPU arm's input bytes",
            "value_1_thread": round(c5_bytes(rows1) / dt1 / 1e9, 3),
            "sample_1_thread": f"{rows1} C5 rows ({dt1:.2f} s) on one core",
            "cpu_model": cpu_model()}


def cpu_model() -> str:
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


# ------------------------------------------------------------ reference arm


def run_reference(args, rank: int, world: int) -> None:
    """The reference path's CPU implementation (the oracle port: the reference's
    NASM engine cannot be assembled here) on all host threads, on the GPU arm's
    config and input bytes: each step one whole 16384-row C5 pass into
    preallocated outputs, as the reference's loadtest times whole calls in a
    loop (tools/b_swiglu_q8_loadtest.cpp:134-137).  Rank 0 only."""
    if rank != 0:
        return
    from oracle.pyoracle import Oracle
    threads = os.cpu_count() or 1
    orc = Oracle(nthreads=threads)
    g, u = c5_host_inputs(orc)
    out = (np.empty((C5_ROWS, C5_N), np.int8), np.empty((C5_ROWS, C5_N // GROUP), np.float32))
    for _ in range(args.warmup):
        orc.swiglu_q8_avx2(g, u, out=out)
    times = []
    for _ in range(args.steps):
        t = time.perf_counter()
        orc.swiglu_q8_avx2(g, u, out=out)
        times.append(time.perf_counter() - t)
    total = sum(times)
    value = c5_bytes(C5_ROWS) * args.steps / total / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "GB/s",
        "rows_per_s": round(C5_ROWS * args.steps / total, 1), "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(total / args.steps * 1e3, 3), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": f"synthetic: counter-based N(0, 2) gate/up (seed {SEED_GATE}/{SEED_UP}), the GPU arm's input bytes "
                "(generator restated on the host)",
        "config": {"workload": "C5 SwiGLU + Q8 requantisation: gate/up [16384, 12288] fp32 -> int8 codes "
                               "[16384, 12288] + fp32 scales [16384, 192] (one per 64-element group)",
                   "rows": C5_ROWS, "n": C5_N, "rows_per_step": C5_ROWS, "parallelism": f"{threads} host threads"},
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": f"all 16384 C5 rows per step, {args.steps} steps after {args.warmup} untimed, "
                                   f"AVX2 restatement",
                         "cpu_model": cpu_model()},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "the reference engine is NASM; nasm is absent on this image, so its restatement (oracle/v7_oracle.c) "
                "is timed, in AVX2 with the reference's instruction forms (EVAL_SIGMOID, the MAXPS tree, vcvtps2dq and the "
                "saturating packs), bit-identical to the scalar restatement",
    }
    print(json.dumps(line), flush=True)


def _profile_case(name: str, rows: int, dev):
    """Inputs and launcher of one kernel at `rows` rows of its BASELINE shape."""
    import v7multiplikator_b200 as v7g

    def fill(shape, seed, mean, std):
        t = torch.empty(*shape, device=dev)
        return v7g.fill_normal(t.view(-1, shape[-1]), seed=seed, mean=mean, std=std)

    if name == "swiglu_q8":
        g, u = fill((rows, C5_N), 12, 0.0, 2.0), fill((rows, C5_N), 13, 0.0, 2.0)
        c = torch.empty(rows, C5_N, dtype=torch.int8, device=dev)
        s = torch.empty(rows, C5_N // GROUP, device=dev)
        return lambda: v7g.swiglu_q8_rows(c, s, g, u), c5_bytes(rows)
    if name == "swiglu":
        g, u = fill((rows, 8192), 10, 0.0, 2.0), fill((rows, 8192), 11, 0.0, 2.0)
        o = torch.empty_like(g)
        return lambda: v7g.swiglu(o, g, u), rows * 8192 * 12
    if name in ("rmsnorm", "fused_add_rmsnorm", "add_inplace", "rmsnorm_quantize"):
        x, d = fill((rows, 2048), 3, 0.0, 1.0), fill((rows, 2048), 4, 0.0, 0.5)
        w = fill((1, 2048), 5, 1.0, 0.1)[0]
        o = torch.empty_like(x)
        if name == "rmsnorm":
            return lambda: v7g.rmsnorm_rows(o, x, w, 1e-6), rows * 2048 * 8
        if name == "fused_add_rmsnorm":
            return lambda: v7g.fused_add_rmsnorm_rows(o, x, d, w, 1e-6), rows * 2048 * 16
        if name == "add_inplace":
            return lambda: v7g.add_inplace(x, d), rows * 2048 * 12
        c = torch.empty(rows, 2048, dtype=torch.int8, device=dev)
        s = torch.empty(rows, 32, device=dev)
        return lambda: v7g.rmsnorm_quantize_rows(c, s, x, w, 1e-6), rows * (2048 * 5 + 128)
    if name in ("rmsnorm_rope", "rope_only"):
        q, k = fill((rows, 16 * 128), 6, 0.0, 1.0).view(rows, 16, 128), fill((rows, 8 * 128), 7, 0.0, 1.0).view(rows, 8, 128)
        wq, wk = fill((1, 128), 8, 1.0, 0.1)[0], fill((1, 128), 9, 1.0, 0.1)[0]
        cos, sin = v7g.rope_tables(rows, 64, 1e6, device=dev)
        if name == "rope_only":
            return lambda: v7g.rope_only_rows(q, k, cos, sin, 0), rows * (24 * 128 * 8 + 64 * 8)
        return lambda: v7g.rmsnorm_rope_rows(q, k, wq, wk, cos, sin, 0, 1e-6), rows * (24 * 128 * 8 + 64 * 8)
    if name in ("swiglu_q8_gemv", "swiglu_f32q8_gemv", "q8_gemv", "q8_fused_gemv"):
        n = {"q8_gemv": 8192, "q8_fused_gemv": 8192, "swiglu_q8_gemv": 4096, "swiglu_f32q8_gemv": 2048}[name]  # the kernel-table shapes
        xq, xs, gq, gs, uq, us = gemv_inputs(dev, n, rows)
        y = torch.empty(1, rows, device=dev)
        if name == "q8_gemv":
            return lambda: v7g.q8_gemv(y, xq, xs, gq, gs), rows * (n + n // 16)
        if name == "q8_fused_gemv":
            xf = fill((1, n), 15, 0.0, 1.0)
            return lambda: v7g.q8_fused_gemv(y, xf, gq, gs), rows * (n + n // 16)
        if name == "swiglu_q8_gemv":
            return lambda: v7g.swiglu_q8_gemv(y, xq, xs, gq, gs, uq, us), 2 * rows * (n + n // 16)
        xf = fill((1, n), 14, 0.0, 1.0)
        return lambda: v7g.swiglu_f32q8_gemv(y, xf, gq, gs, uq, us), 2 * rows * (n + n // 16)
    if name == "rope_tables":
        tc = torch.empty(rows, 64, device=dev)
        ts = torch.empty_like(tc)
        freqs = np.ascontiguousarray(v7g.rope_freqs(64, 1e6))
        return (lambda: v7g.ops._check(v7g.lib().v7g_rope_tables(tc.data_ptr(), ts.data_ptr(), 0, rows, 64, 64,
                                                                 freqs.ctypes.data, None))), rows * 64 * 8
    raise ValueError(name)


PROFILE_CASES = ("swiglu_q8", "swiglu", "rmsnorm", "fused_add_rmsnorm", "add_inplace", "rmsnorm_quantize", "rmsnorm_rope",
                 "rope_only", "rope_tables", "swiglu_q8_gemv", "swiglu_f32q8_gemv", "q8_gemv", "q8_fused_gemv")


def run_profile(args) -> None:
    """A small, fixed case for ncu: fill, `warmup` + `steps` launches of one
    kernel, one line of device-timed GB/s (not a bench value)."""
    dev = torch.device("cuda", 0)
    fn, nbytes = _profile_case(args.profile, args.rows, dev)
    torch.cuda.synchronize()
    for _ in range(args.warmup):
        fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda._sleep(4_000_000)  # head start: every launch is queued before the first runs
    a.record()
    for _ in range(args.steps):
        fn()
    b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / args.steps
    print(json.dumps({"profile": args.profile, "rows": args.rows, "bytes_per_launch": nbytes, "us": round(ms * 1e3, 2),
                      "gbs": round(nbytes / (ms * 1e-3) / 1e9, 1)}))


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-extras", action="store_true", help="skip the per-config table and the CPU baseline")
    ap.add_argument("--cpu-seconds", type=float, default=10.0, help="CPU-baseline sample size in seconds of work")
    ap.add_argument("--profile", choices=sorted(PROFILE_CASES), help="profiling mode: launch one kernel --steps times "
                    "on a --rows-row case and exit (for ncu captures)")
    ap.add_argument("--rows", type=int, default=2048, help="rows of the --profile case")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    rank, world, local = dist_env()
    if args.profile:
        run_profile(args)
        return
    if world != args.gpus:
        if world == 1 and args.gpus > 1:
            ap.error("--gpus > 1 needs torchrun (one process per GPU)")
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    run_ours(args, rank, world, local)


if __name__ == "__main__":
    main()
