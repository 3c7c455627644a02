#!/usr/bin/env python
"""Benchmark of the cppinf hot-path kernels on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload NAME]

A step is one pass of one hot-path op over one batch of its configuration:

    qk_norm_rope    (headline) q bf16 [2048, 16, 128] + k bf16 [2048, 8, 128], per-head RMSNorm (eps 1e-6)
                    then RoPE (theta 1e6) at positions 0..2047 of this GPU's token rows
    rms_norm        x bf16 [512, 1024], w [1024]
    silu_mul        gate, up bf16 [4096, 3072]
    add_rms_norm    a, b bf16 [4096, 1024], w [1024] -> sum, y
    causal_softmax  f32 [16, 2048, 2048], scale 1/sqrt(128), lower-triangular mask
    row_argmax      logits bf16 [64, 151936] -> int64 [64]

Metric: achieved HBM GB/s = algorithmic bytes (minimum read + write) / device time. Multi-GPU (torchrun, one process
per GPU): the headline partitions one (2048 * N)-token batch into N token ranges (cppinf_b200/shard.py token_shard;
RoPE positions stay global), 2048 rows per rank (weak scaling), with no collective on the data path; time is the max
over ranks. The `sharded` object adds, for N > 1, one global batch of q/k (2048 * N and 2048 tokens), of the causal
softmax (byte-balanced row ranges) and of the argmax (row ranges) partitioned across the ranks, each timed compute
only and with the copy-back of every rank's output rows into one buffer on rank 0 (point-to-point over NCCL, i.e.
NVLink peer copies).

Timing: W eager warm-up steps, then K steps replayed from CUDA graphs of <= 1000 launches, bracketed by a barrier and
a device synchronize, CUDA events on the launch stream (a ~100 us device spin queued before the start event hides the
host's graph submission, which would otherwise sit inside a short timed region); `repeats` replays the same K steps 50 more times, each timed
alone, for the median and the spread. Consecutive steps rotate through buffer sets whose total is
more than three times the 126 MB L2, so every step reads cold data from HBM. `e2e` runs the same op through the
public API from pinned host buffers (H2D, kernel, D2H pipelined over three streams) and reports the same metric.

--impl reference times the reference's CPU implementation of the same workload on this host (the reference's own
rope.cpp compiled under oracle/_ref, and the C restatement of rms_norm whose reference needs oneDNN), with all host
threads; under torchrun only rank 0 runs it.

The line also carries `decode`: random-init Qwen3-0.6B (weights ~N(0,0.02), unit norm weights) on the device
decoder, a seeded 512-token prompt then 128 greedy tokens (1 from the prefill, 127 graph-replayed decode steps);
tok/s of the decode steps (CUDA events), the prefill time, the weight-streaming roofline, and e2e through
Qwen3Model.generate with host token ids. Across GPUs decode runs one independent replica per GPU.
"""

from __future__ import annotations

import argparse
import ctypes
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

L2_BYTES = 126 * 1024 * 1024
SPACER_CYCLES = 200_000  # ~100 us of device spin before a timed region (see time_device_steps)
FALLBACK_HBM_GBS = 6650.0
METRIC = "achieved HBM GB/s per op vs ~8 TB/s"
UNIT = "GB/s"

# Algorithmic bytes per step (minimum read + write) of each configuration.
CONFIGS = {
    "rms_norm": dict(bytes=2 * 512 * 1024 * 2 + 1024 * 2,
                     desc="RMSNorm x bf16 [512,1024] ~N(0,1), w bf16 [1024] ~N(1,0.1), eps 1e-6"),
    "qk_norm_rope": dict(bytes=2 * (2048 * 24 * 128 * 2) + 2 * 128 * 2,
                         desc="q/k per-head RMSNorm + RoPE: q bf16 [2048,16,128], k bf16 [2048,8,128] ~N(0,1), "
                              "norm weights bf16 [128] ~N(1,0.1), eps 1e-6, theta 1e6, positions 0..2047"),
    "silu_mul": dict(bytes=3 * 4096 * 3072 * 2, desc="SiLU(gate)*up: gate, up bf16 [4096,3072] ~N(0,1)"),
    "add_rms_norm": dict(bytes=4 * 4096 * 1024 * 2 + 1024 * 2,
                         desc="residual add + RMSNorm: a, b bf16 [4096,1024] ~N(0,1), w ~N(1,0.1), eps 1e-6"),
    "causal_softmax": dict(bytes=16 * (2048 * 2049 // 2) * 4 + 16 * 2048 * 2048 * 4,
                           desc="causal scaled softmax f32 [16,2048,2048] ~N(0,4), scale 1/sqrt(128)"),
    "row_argmax": dict(bytes=64 * 151936 * 2 + 64 * 8, desc="row argmax logits bf16 [64,151936] ~N(0,2)"),
    # Tensor-bound: reported in TFLOP/s against the measured dense bf16 peak as well.
    "linear_tc": dict(bytes=(512 * 1024 + 2 * 3072 * 1024 + 512 * 3072) * 2, flops=2 * 2 * 512 * 3072 * 1024,
                      desc="tensor-core prefill gate/up projection with SiLU*up: x bf16 [512,1024] ~N(0,1), "
                           "gate/up [3072,1024] ~N(0,0.02) (cppinf_linear_tc)"),
}
HEADLINE = "qk_norm_rope"


def parse_args():
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=100000)
    p.add_argument("--warmup", type=int, default=10)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--workload", choices=sorted(CONFIGS), default=HEADLINE)
    p.add_argument("--op-steps", type=int, default=2000, help="steps per secondary op measurement")
    p.add_argument("--no-ops", action="store_true", help="skip the secondary per-op measurements")
    p.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline")
    p.add_argument("--no-e2e", action="store_true", help="skip the host-buffer end-to-end measurement")
    p.add_argument("--cpu-seconds", type=float, default=8.0, help="CPU-baseline sample length")
    p.add_argument("--no-decode", action="store_true", help="skip the Qwen3-0.6B greedy-decode measurement")
    p.add_argument("--decode-runs", type=int, default=3, help="timed prefill + decode runs")
    p.add_argument("--repeats", type=int, default=50, help="further timed replays of the headline steps (spread)")
    p.add_argument("--copy-steps", type=int, default=100, help="steps of each multi-GPU copy-back measurement")
    return p.parse_args()


def read_peak_gbs() -> tuple[float, str]:
    path = REPO / "MEASURED_PEAKS.json"
    try:
        peaks = json.loads(path.read_text())
        return float(peaks["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return FALLBACK_HBM_GBS, "fallback"


def read_peak_tflops() -> tuple[float, str]:
    """Dense bf16 peak for a kernel timed alone: MEASURED_PEAKS.json bf16_tflops (burst), else the fallback."""
    try:
        return float(json.loads((REPO / "MEASURED_PEAKS.json").read_text())["bf16_tflops"]), "measured (burst)"
    except (OSError, KeyError, ValueError):
        return 1590.0, "fallback"


def read_traffic(workload: str) -> float | None:
    """DRAM bytes per launch from the committed ncu summary of the workload, if present."""
    path = REPO / "profiles" / f"{workload}.md"
    if not path.exists():
        return None
    for line in path.read_text().splitlines():
        if line.strip().startswith("traffic_bytes_per_launch"):
            try:
                return float(line.split("=")[1].split()[0].replace(",", ""))
            except (IndexError, ValueError):
                return None
    return None


# ---------------------------------------------------------------------------------------------------------------
# Process group
# ---------------------------------------------------------------------------------------------------------------


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local_rank


# ---------------------------------------------------------------------------------------------------------------
# Clock sampling (nvidia-smi, read-only)
# ---------------------------------------------------------------------------------------------------------------


class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.device_index = device_index
        self.proc = None
        self.file = None

    def _smi_index(self) -> str:
        import torch

        try:
            uuid = str(torch.cuda.get_device_properties(self.device_index).uuid)
            out = subprocess.run(["nvidia-smi", "--query-gpu=index,uuid", "--format=csv,noheader"],
                                 capture_output=True, text=True, timeout=20).stdout
            for line in out.splitlines():
                idx, u = [s.strip() for s in line.split(",")]
                if u.replace("GPU-", "") == uuid.replace("GPU-", ""):
                    return idx
        except Exception:
            pass
        return str(self.device_index)

    def start(self):
        try:
            self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "100",
                 "-i", self._smi_index()], stdout=self.file, stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except OSError:
            self.proc = None

    def stop(self) -> dict | None:
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=10)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.file.flush()
        self.file.seek(0)
        rows = [line.split(",") for line in self.file.read().splitlines() if line.count(",") >= 8]
        self.file.close()
        os.unlink(self.file.name)
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].strip().replace(".", "").isdigit()]
        max_sm = max((float(r[2]) for r in rows if r[2].strip().replace(".", "").isdigit()), default=None)
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].strip().lower() == "active"})
        busy = [s for s in sm if max_sm and s > 0.5 * max_sm] or sm
        return {"sm_mhz": statistics.median(busy) if busy else None, "sm_max_mhz": max_sm, "reasons": reasons,
                "samples": len(rows)}


# ---------------------------------------------------------------------------------------------------------------
# Device workloads
# ---------------------------------------------------------------------------------------------------------------


class Workload:
    """Buffer sets plus a launch function for one op configuration (or one rank's shard of it) on one GPU.

    Shards (cppinf_b200/shard.py): `tokens`/`position_offset` for qk_norm_rope (token rows keep their global RoPE
    positions), `rows` for causal_softmax (a range of the flattened [16 * 2048] score rows, launched per matrix piece
    at its query offset) and for row_argmax (a row count). Without a shard the whole configuration is built."""

    def __init__(self, name: str, rank: int, device, tokens: int = 2048, position_offset: int | None = None,
                 rows=None):
        import torch

        from cppinf_b200 import capi, ops
        from cppinf_b200.shard import range_bytes, softmax_pieces

        self.name = name
        self.lib = capi.load()
        self.capi = capi
        self.bytes = CONFIGS[name]["bytes"]
        self.device = device
        gen = torch.Generator(device=device).manual_seed(1000 + rank)

        def randn(shape, mean=0.0, std=1.0, dtype=torch.bfloat16):
            return (torch.randn(shape, generator=gen, device=device) * std + mean).to(dtype)

        bf16 = capi.DTYPE_BF16
        make_set = None
        if name == "rms_norm":
            w = randn(1024, 1.0, 0.1)

            def make_set():
                x, y = randn((512, 1024)), torch.empty((512, 1024), dtype=torch.bfloat16, device=device)
                return (x, y), lambda s: self.lib.cppinf_rms_norm(bf16, x.data_ptr(), 1024, w.data_ptr(),
                                                                  y.data_ptr(), 512, 1024, 1e-6, s), [y]
            set_bytes = 2 * 512 * 1024 * 2
        elif name == "qk_norm_rope":
            hq, hk, d = 16, 8, 128
            offset = rank * tokens if position_offset is None else position_offset
            qw, kw = randn(d, 1.0, 0.1), randn(d, 1.0, 0.1)
            table = ops.rope_table(1e6, d, offset + tokens, device)
            self.table = table
            self.bytes = qk_bytes(tokens)

            def make_set():
                q, k = randn((tokens, hq, d)), randn((tokens, hk, d))
                qo, ko = torch.empty_like(q), torch.empty_like(k)
                return (q, k, qo, ko), lambda s: self.lib.cppinf_qk_norm_rope(
                    bf16, q.data_ptr(), k.data_ptr(), qw.data_ptr(), kw.data_ptr(), qo.data_ptr(), ko.data_ptr(),
                    tokens, hq, hk, d, offset, 1e-6, table.data_ptr(), table.shape[0], s), [qo, ko]
            set_bytes = 2 * tokens * (hq + hk) * d * 2
        elif name == "silu_mul":
            def make_set():
                g, u = randn((4096, 3072)), randn((4096, 3072))
                o = torch.empty_like(g)
                return (g, u, o), lambda s: self.lib.cppinf_silu_mul(bf16, g.data_ptr(), u.data_ptr(), o.data_ptr(),
                                                                     g.numel(), s), [o]
            set_bytes = 3 * 4096 * 3072 * 2
        elif name == "add_rms_norm":
            w = randn(1024, 1.0, 0.1)

            def make_set():
                a, b = randn((4096, 1024)), randn((4096, 1024))
                sm, y = torch.empty_like(a), torch.empty_like(a)
                return (a, b, sm, y), lambda s: self.lib.cppinf_add_rms_norm(
                    bf16, a.data_ptr(), b.data_ptr(), w.data_ptr(), sm.data_ptr(), y.data_ptr(), 4096, 1024, 1e-6,
                    s), [sm, y]
            set_bytes = 4 * 4096 * 1024 * 2
        elif name == "causal_softmax":
            scale = 1.0 / math.sqrt(128.0)
            matrices, n = 16, 2048
            row_range = (0, matrices * n) if rows is None else rows
            pieces = softmax_pieces(row_range, n)
            nrows = row_range[1] - row_range[0]
            self.bytes = range_bytes(row_range, n, n)
            # Launches: consecutive whole matrices go to the square ops entry point in one call; a partial matrix
            # goes to the position-aware one at its query offset.
            launches = []
            for pc in pieces:
                whole = pc.query_start == 0 and pc.rows == n
                if whole and launches and launches[-1][0] == "square":
                    launches[-1][2] += 1
                elif whole:
                    launches.append(["square", None, 1])
                else:
                    launches.append(["piece", (capi.i64_array([pc.query_start]), capi.i64_array([pc.rows]),
                                               capi.i64_array([n])), pc.rows])

            def make_set():
                x = randn((nrows, n), 0.0, 2.0, torch.float32)
                y = torch.empty_like(x)

                def launch(s):
                    r0 = 0
                    for kind, arrs, count in launches:
                        rows_here = count * n if kind == "square" else count
                        xp, yp = x[r0:r0 + rows_here], y[r0:r0 + rows_here]
                        if kind == "square":
                            st = self.lib.cppinf_scaled_causal_softmax_f32(xp.data_ptr(), yp.data_ptr(), count, n,
                                                                           n, scale, s)
                        else:
                            st = self.lib.cppinf_scaled_position_causal_softmax_f32(
                                xp.data_ptr(), yp.data_ptr(), 1, 1, count, n, scale, arrs[0], arrs[1], arrs[2], s)
                        if st != 0:
                            return st
                        r0 += rows_here
                    return 0
                return (x, y), launch, [y]
            set_bytes = 2 * nrows * n * 4
        elif name == "linear_tc":
            wg, wu = randn((3072, 1024), 0.0, 0.02), randn((3072, 1024), 0.0, 0.02)

            def make_set():
                x = randn((512, 1024))
                y = torch.empty((512, 3072), dtype=torch.bfloat16, device=device)
                return (x, y), lambda s: self.lib.cppinf_linear_tc(2, x.data_ptr(), 1024, wg.data_ptr(), wu.data_ptr(),
                                                                   0, y.data_ptr(), 512, 1024, 3072, 0, s), [y]
            set_bytes = (512 * 1024 + 512 * 3072) * 2
        elif name == "row_argmax":
            nrows = 64 if rows is None else rows
            self.bytes = nrows * 151936 * 2 + nrows * 8

            def make_set():
                x = randn((nrows, 151936), 0.0, 2.0)
                o = torch.empty(nrows, dtype=torch.int64, device=device)
                return (x, o), lambda s: self.lib.cppinf_row_argmax(bf16, x.data_ptr(), nrows, 151936, 151936,
                                                                    o.data_ptr(), s), [o]
            set_bytes = nrows * 151936 * 2
        else:
            raise ValueError(name)

        n_sets = max(1, math.ceil(3 * L2_BYTES / max(set_bytes, 1)))
        self.sets = [make_set() for _ in range(n_sets)]
        self.resident_bytes = n_sets * set_bytes
        self.n_sets = n_sets

    def launch(self, i: int, stream_handle: int) -> None:
        status = self.sets[i % self.n_sets][1](stream_handle)
        if status != 0:
            self.capi.check(status, self.name)

    def outputs(self, i: int) -> list:
        return self.sets[i % self.n_sets][2]


def time_device_steps(wl: Workload, steps: int, warmup: int, stream, barrier,
                      repeats: int = 0) -> tuple[float, int, list[float]]:
    """Times exactly `steps` launches (CUDA-graph replays) on `stream`; returns (ms, launches in the timed region,
    ms of each of `repeats` further timed replays of the same steps, for the spread)."""
    import torch

    h = stream.cuda_stream
    with torch.cuda.stream(stream):
        for i in range(warmup):
            wl.launch(i, h)
    torch.cuda.synchronize()

    chunk = min(steps, 1000)

    def capture(n: int):
        g = torch.cuda.CUDAGraph()
        before = wl.capi.launch_count()
        with torch.cuda.graph(g, stream=stream):
            for i in range(n):
                wl.launch(i, stream.cuda_stream)
        return g, wl.capi.launch_count() - before

    main_graph, main_launches = capture(chunk)
    tail = steps % chunk
    tail_graph, tail_launches = capture(tail) if tail else (None, 0)
    replays = steps // chunk
    with torch.cuda.stream(stream):
        main_graph.replay()  # untimed: first replay uploads the graph
    torch.cuda.synchronize()

    def timed() -> float:
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier()
        torch.cuda.synchronize()
        with torch.cuda.stream(stream):
            # A ~100 us spin queued ahead of the start event keeps the device busy while the host submits the
            # graph, so the timed region holds the K steps and not the submission latency.
            torch.cuda._sleep(SPACER_CYCLES)
            start.record(stream)
            for _ in range(replays):
                main_graph.replay()
            if tail_graph is not None:
                tail_graph.replay()
            end.record(stream)
        torch.cuda.synchronize()
        barrier()
        return start.elapsed_time(end)

    ms = timed()
    launches = replays * main_launches + tail_launches
    spread = [timed() for _ in range(repeats)]
    del main_graph, tail_graph
    return ms, launches, spread


def time_single_launches(wl: Workload, count: int, stream) -> list[float]:
    """Latency of isolated launches: each launch alone between two events, the stream drained in between."""
    import torch

    out = []
    for i in range(count):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        with torch.cuda.stream(stream):
            e0.record(stream)
            wl.launch(i, stream.cuda_stream)
            e1.record(stream)
        torch.cuda.synchronize()
        out.append(e0.elapsed_time(e1) * 1e3)
    return out


def time_e2e(wl_name: str, rank: int, device, steps: int) -> dict:
    """Same op through the public API (cppinf_b200.ops) from pinned host buffers: per step H2D of the inputs, the
    kernel, D2H of the outputs, pipelined over three streams with double-buffered device memory."""
    import torch

    from cppinf_b200 import ops

    if wl_name != "qk_norm_rope":
        return None
    tokens, hq, hk, d = 2048, 16, 8, 128
    gen = torch.Generator().manual_seed(77 + rank)
    host_q = (torch.randn((tokens, hq, d), generator=gen)).to(torch.bfloat16).pin_memory()
    host_k = (torch.randn((tokens, hk, d), generator=gen)).to(torch.bfloat16).pin_memory()
    qw = (1 + 0.1 * torch.randn(d, generator=gen)).to(torch.bfloat16).to(device)
    kw = (1 + 0.1 * torch.randn(d, generator=gen)).to(torch.bfloat16).to(device)
    host_out = [(torch.empty_like(host_q).pin_memory(), torch.empty_like(host_k).pin_memory()) for _ in range(2)]
    dev_in = [(torch.empty_like(host_q, device=device), torch.empty_like(host_k, device=device)) for _ in range(2)]
    dev_out = [(torch.empty_like(host_q, device=device), torch.empty_like(host_k, device=device)) for _ in range(2)]
    offset = rank * tokens
    ops.rope_table(1e6, d, offset + tokens, device)
    s_h2d, s_comp, s_d2h = torch.cuda.Stream(device), torch.cuda.Stream(device), torch.cuda.Stream(device)
    ev = {k: [torch.cuda.Event() for _ in range(2)] for k in ("h2d", "comp", "d2h")}
    started = [False, False]

    def step(i: int):
        b = i % 2
        with torch.cuda.stream(s_h2d):
            if started[b]:
                s_h2d.wait_event(ev["comp"][b])
            dev_in[b][0].copy_(host_q, non_blocking=True)
            dev_in[b][1].copy_(host_k, non_blocking=True)
            ev["h2d"][b].record(s_h2d)
        with torch.cuda.stream(s_comp):
            s_comp.wait_event(ev["h2d"][b])
            if started[b]:
                s_comp.wait_event(ev["d2h"][b])
            ops.qk_norm_rope(dev_in[b][0], dev_in[b][1], qw, kw, 1e-6, offset, 1e6, out=dev_out[b])
            ev["comp"][b].record(s_comp)
        with torch.cuda.stream(s_d2h):
            s_d2h.wait_event(ev["comp"][b])
            host_out[b][0].copy_(dev_out[b][0], non_blocking=True)
            host_out[b][1].copy_(dev_out[b][1], non_blocking=True)
            ev["d2h"][b].record(s_d2h)
        started[b] = True

    for i in range(4):
        step(i)
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(s_h2d)
    for i in range(steps):
        step(i)
    s_d2h.wait_event(ev["comp"][(steps - 1) % 2])
    end.record(s_d2h)
    torch.cuda.synchronize()
    ms = start.elapsed_time(end)
    in_bytes = host_q.numel() * 2 + host_k.numel() * 2
    return {"ms": ms, "steps": steps, "h2d_bytes_per_step": in_bytes, "d2h_bytes_per_step": in_bytes}


class PeerOutputs:
    """Rank 0's global output buffers (cudaMalloc) mapped into every rank through CUDA IPC handles sent over the
    process group, opened on the rank's own device with lazy peer access, so each rank's copy engine writes its
    output rows straight into rank 0's HBM over NVLink (one cudaMemcpyAsync per output, capturable in a graph).
    Rank 0 copies its own rows locally. `path` is "nvlink peer copy" or, when a rank could not map the buffers
    (every rank learns of it), "nccl send/recv" through shard.copy_back."""

    class _Handle(ctypes.Structure):  # cudaIpcMemHandle_t (64 opaque bytes, NULs included)
        _fields_ = [("reserved", ctypes.c_ubyte * 64)]

    def __init__(self, shapes: list, rank: int, device):
        import torch
        import torch.distributed as dist

        self.rank = rank
        self.device = device
        self.shapes = shapes
        self.row_bytes = [math.prod(shape[1:]) * torch.empty((), dtype=dt).element_size() for shape, dt in shapes]
        self.nbytes = [shape[0] * rb for (shape, _), rb in zip(shapes, self.row_bytes)]
        rt = ctypes.CDLL("libcudart.so.12")
        self._rt = rt
        rt.cudaMemcpyAsync.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int, ctypes.c_void_p]
        self.ptrs, self.owned, self.dsts = [], [], None
        ok = 1
        try:
            torch.cuda.set_device(device)
            handles = None
            if rank == 0:
                handles = []
                for n in self.nbytes:
                    p = ctypes.c_void_p()
                    if rt.cudaMalloc(ctypes.byref(p), ctypes.c_size_t(n)) != 0:
                        raise RuntimeError("cudaMalloc")
                    self.owned.append(p.value)
                    h = PeerOutputs._Handle()
                    if rt.cudaIpcGetMemHandle(ctypes.byref(h), ctypes.c_void_p(p.value)) != 0:
                        raise RuntimeError("cudaIpcGetMemHandle")
                    handles.append(ctypes.string_at(ctypes.addressof(h), ctypes.sizeof(h)))
                self.ptrs = list(self.owned)
            box = [handles]
            dist.broadcast_object_list(box, src=0)
            if rank != 0:
                rt.cudaIpcOpenMemHandle.argtypes = [ctypes.POINTER(ctypes.c_void_p), PeerOutputs._Handle, ctypes.c_uint]
                for raw in box[0]:
                    h = PeerOutputs._Handle()
                    ctypes.memmove(ctypes.addressof(h), raw, ctypes.sizeof(h))
                    p = ctypes.c_void_p()
                    if rt.cudaIpcOpenMemHandle(ctypes.byref(p), h, 1) != 0:  # cudaIpcMemLazyEnablePeerAccess
                        raise RuntimeError("cudaIpcOpenMemHandle")
                    self.ptrs.append(p.value)
        except Exception:
            ok = 0
            rt.cudaGetLastError()  # a failed runtime call must not surface in a later launch check
        flag = torch.tensor([ok], dtype=torch.int32, device=device)
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)
        self.path = "nvlink peer copy" if int(flag.item()) == 1 else "nccl send/recv"
        if self.path != "nvlink peer copy":
            self.dsts = [torch.empty(shape, dtype=dt, device=device) if rank == 0 else None for shape, dt in shapes]

    def copy(self, outputs: list, ranges: list, stream) -> None:
        s, e = ranges[self.rank]
        if e <= s:
            return
        if self.dsts is not None:
            from cppinf_b200.shard import copy_back

            for out, dst in zip(outputs, self.dsts):
                copy_back(out, dst, ranges, self.rank)
            return
        for out, ptr, rb in zip(outputs, self.ptrs, self.row_bytes):
            status = self._rt.cudaMemcpyAsync(ptr + s * rb, out.data_ptr(), (e - s) * rb, 4, stream.cuda_stream)
            if status != 0:
                raise RuntimeError(f"cudaMemcpyAsync (peer copy-back) failed with {status}")

    def close(self) -> None:
        """Unmaps the peers' views, then (after every rank has) frees rank 0's buffers."""
        import torch
        import torch.distributed as dist

        torch.cuda.synchronize()
        if self.rank != 0:
            for p in self.ptrs:
                self._rt.cudaIpcCloseMemHandle(ctypes.c_void_p(p))
        dist.barrier()
        for p in self.owned:
            self._rt.cudaFree(ctypes.c_void_p(p))


def time_copy_back_steps(wl: Workload, steps: int, peer: PeerOutputs, ranges: list, stream, barrier) -> float:
    """`steps` steps of the op each followed by the copy of this rank's output rows into rank 0's buffers, timed with
    CUDA events on `stream`. Peer copies are captured with the kernels in one CUDA graph; the NCCL fallback runs
    eagerly. Returns ms on this rank: the time until its rows have landed in rank 0's HBM."""
    import torch

    def step(i):
        wl.launch(i, stream.cuda_stream)
        peer.copy(wl.outputs(i), ranges, stream)

    with torch.cuda.stream(stream):
        for i in range(3):
            step(i)
    torch.cuda.synchronize()
    g = None
    if peer.dsts is None:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            for i in range(steps):
                step(i)
        with torch.cuda.stream(stream):
            g.replay()  # untimed: uploads the graph
        torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        start.record(stream)
        if g is not None:
            g.replay()
        else:
            for i in range(steps):
                step(i)
        end.record(stream)
    torch.cuda.synchronize()
    barrier()
    del g
    return start.elapsed_time(end)


def sharded_legs(world: int, rank: int, device, stream, barrier, max_over_ranks, peak: float, steps: int,
                 copy_steps: int) -> dict:
    """Row partitioning of one global batch across the ranks (cppinf_b200/shard.py), compute only and with the
    copy-back of every shard into one buffer on rank 0:

    qk_norm_rope weak    global batch of 2048 * N tokens, 2048 per rank at their global RoPE positions
    qk_norm_rope strong  the 2048-token configuration split into N token ranges
    causal_softmax       the [16, 2048, 2048] configuration split into N byte-balanced row ranges
    row_argmax           the [64, 151936] configuration split into N row ranges

    Aggregate GB/s = the algorithmic bytes of the global batch / the max over ranks of the time; `frac` is that over
    N x the measured peak. The copy-back moves the outputs (`copy_bytes_per_step` in total; rank 0's own rows are a
    local copy) into one set of buffers in rank 0's HBM by peer copies (PeerOutputs), captured with the kernels in
    one CUDA graph per measurement."""
    import torch

    from cppinf_b200.shard import causal_row_ranges, range_bytes, row_ranges, token_shard

    legs = {}
    specs = [
        ("qk_norm_rope_weak", "qk_norm_rope", 2048 * world),
        ("qk_norm_rope_strong", "qk_norm_rope", 2048),
        ("causal_softmax_strong", "causal_softmax", None),
        ("row_argmax_strong", "row_argmax", None),
    ]
    for label, op, global_tokens in specs:
        if op == "qk_norm_rope":
            ranges = row_ranges(global_tokens, world)
            sh = token_shard(global_tokens, world, rank)
            wl = Workload(op, rank, device, tokens=sh.tokens, position_offset=sh.position_offset)
            total = qk_bytes(global_tokens)
            shapes = [((global_tokens, 16, 128), torch.bfloat16), ((global_tokens, 8, 128), torch.bfloat16)]
            desc = f"q/k RMSNorm + RoPE, {global_tokens} tokens split into {world} token ranges"
        elif op == "causal_softmax":
            ranges = causal_row_ranges(16, 2048, 2048, world)
            wl = Workload(op, rank, device, rows=ranges[rank])
            total = sum(range_bytes(r, 2048, 2048) for r in ranges)
            shapes = [((16 * 2048, 2048), torch.float32)]
            desc = f"causal softmax [16, 2048, 2048], {world} byte-balanced row ranges"
        else:
            ranges = row_ranges(64, world)
            wl = Workload(op, rank, device, rows=ranges[rank][1] - ranges[rank][0])
            total = CONFIGS[op]["bytes"]
            shapes = [((64,), torch.int64)]
            desc = f"row argmax [64, 151936], {world} row ranges"
        ms, _, _ = time_device_steps(wl, steps, 3, stream, barrier)
        ms = max_over_ranks(ms)
        gbs = total * steps / (ms * 1e-3) / 1e9
        peer = PeerOutputs(shapes, rank, device)
        copy_bytes = sum(math.prod(shape) * torch.empty((), dtype=dt).element_size() for shape, dt in shapes)
        cms = max_over_ranks(time_copy_back_steps(wl, copy_steps, peer, ranges, stream, barrier))
        cgbs = total * copy_steps / (cms * 1e-3) / 1e9
        legs[label] = {
            "workload": desc, "bytes_per_step": total,
            "compute": {"us_per_step": round(ms / steps * 1e3, 3), "gbs": round(gbs, 1),
                        "frac_of_n_peak": round(gbs / (world * peak), 4), "steps": steps},
            "with_copy_back": {"us_per_step": round(cms / copy_steps * 1e3, 3), "gbs": round(cgbs, 1),
                               "frac_of_n_peak": round(cgbs / (world * peak), 4), "steps": copy_steps,
                               "copy_bytes_per_step": copy_bytes, "path": peer.path},
        }
        peer.close()
        del wl, peer
        torch.cuda.empty_cache()
    return legs


# ---------------------------------------------------------------------------------------------------------------
# CPU paths (oracle port / reference code), used as the baseline
# ---------------------------------------------------------------------------------------------------------------


def qk_bytes(tokens: int) -> int:
    """Algorithmic bytes of the q/k RMSNorm + RoPE over `tokens` token rows (16 q + 8 k heads of 128, bf16)."""
    return 2 * tokens * 24 * 128 * 2 + 2 * 128 * 2


class CpuQkNormRope:
    """The q/k RMSNorm + RoPE configuration on the host, as the CPU baseline.

    kind "port": the C restatement (oracle/oracle.c, OpenMP over head vectors).
    kind "reference": the reference's sequence of src/nn/qwen_attention.cpp:383-390 -- ops::rms_norm per head (run
    by the restatement, because the reference's rms_norm needs oneDNN, which is not available here), then the
    reference's own nn::apply_rope from src/nn/rope.cpp (compiled in place under oracle/_ref), over token chunks on
    all host threads.
    """

    def __init__(self, kind: str):
        import numpy as np

        from oracle.oracle import Oracle, Reference, f32_to_bf16, reference_available

        self.threads = os.cpu_count() or 1
        os.environ.setdefault("OMP_NUM_THREADS", str(self.threads))
        self.oracle = Oracle()
        if kind == "reference" and not reference_available():
            kind = "port"
        self.kind = kind
        self.reference = Reference() if kind == "reference" else None
        self.pool = ThreadPoolExecutor(max_workers=self.threads) if kind == "reference" else None
        rng = np.random.default_rng(5)
        self.q = f32_to_bf16(rng.standard_normal((2048, 16, 128)).astype(np.float32))
        self.k = f32_to_bf16(rng.standard_normal((2048, 8, 128)).astype(np.float32))
        self.qw = f32_to_bf16((1 + 0.1 * rng.standard_normal(128)).astype(np.float32))
        self.kw = f32_to_bf16((1 + 0.1 * rng.standard_normal(128)).astype(np.float32))

    def step(self, tokens: int = 2048) -> None:
        q, k = self.q[:tokens], self.k[:tokens]
        if self.kind == "port":
            self.oracle.qk_norm_rope(q, k, self.qw, self.kw, 1e-6, 0, 1e6)
            return
        qn = self.oracle.rms_norm(q.reshape(-1, 128), self.qw, 1e-6).reshape(q.shape)
        kn = self.oracle.rms_norm(k.reshape(-1, 128), self.kw, 1e-6).reshape(k.shape)
        chunk = max(1, -(-tokens // self.threads))
        jobs = [self.pool.submit(self.reference.apply_rope, x[t0:t0 + chunk], t0, 1e6, 0)
                for t0 in range(0, tokens, chunk) for x in (qn, kn)]
        for j in jobs:
            j.result()

    def describe(self) -> str:
        if self.kind == "reference":
            return ("the reference's own rope.cpp (oracle/_ref) over token chunks on all threads, after the C "
                    "restatement of rms_norm (the reference's needs oneDNN, absent here)")
        return "the C restatement (oracle/oracle.c, OpenMP over head vectors)"

    def close(self) -> None:
        if self.pool is not None:
            self.pool.shutdown()


def measure_cpu(kind: str, seconds: float) -> dict:
    """Full 2048-token steps repeated for about `seconds`."""
    cpu = CpuQkNormRope(kind)
    cpu.step()  # warm-up
    n = 0
    t0 = time.perf_counter()
    while True:
        cpu.step()
        n += 1
        elapsed = time.perf_counter() - t0
        if elapsed >= seconds:
            break
    cpu.close()
    gbs = n * qk_bytes(2048) / elapsed / 1e9
    return {"value": round(gbs, 3), "unit": UNIT, "cores": cpu.threads, "cpu_model": cpu_model(), "kind": cpu.kind,
            "sample": f"{n} full 2048-token q/k steps in {elapsed:.1f} s: {cpu.describe()}"}


# ---------------------------------------------------------------------------------------------------------------
# Qwen3-0.6B greedy decode (random init), replicas only across GPUs
# ---------------------------------------------------------------------------------------------------------------

DECODE_PROMPT = 512
DECODE_NEW = 128


def decode_bytes_per_token(cfg, context: int) -> int:
    """Algorithmic HBM bytes of one decode step: every weight once (the tied embedding as the LM head; the embedding
    gather reads one row) plus the key and value rows of `context` positions in every layer."""
    weights = cfg.parameter_count() * 2
    kv = 2 * context * cfg.num_key_value_heads * cfg.head_dim * 2 * cfg.num_hidden_layers
    return weights + kv


def device_random_weights(cfg, device, seed: int = 0) -> dict:
    """~N(0, 0.02) bf16 matrices and unit norm weights, drawn on the device (seeded torch generator)."""
    import torch

    g = torch.Generator(device=device).manual_seed(seed)
    out = {}
    for name, shape in cfg.weight_shapes().items():
        if len(shape) == 1:
            out[name] = torch.ones(shape, dtype=torch.bfloat16, device=device)
        else:
            out[name] = (torch.randn(shape, generator=g, device=device) * 0.02).to(torch.bfloat16)
    return out


def measure_decode(device, runs: int) -> dict:
    """Prefill a seeded 512-token prompt, then 127 graph-replayed decode steps (128 generated tokens), `runs` times
    after one warm-up run. Device time from CUDA events on the launch stream; e2e is the wall time of the public
    Qwen3Model.generate call (host token ids in, host token ids out)."""
    import numpy as np
    import torch

    from cppinf_b200 import capi
    from cppinf_b200.qwen3 import Qwen3Config, Qwen3Model

    cfg = Qwen3Config.qwen3_0_6b()
    model = Qwen3Model(cfg, DECODE_PROMPT + DECODE_NEW, device_random_weights(cfg, device))
    prompt = np.random.default_rng(0).integers(0, cfg.vocab_size, DECODE_PROMPT).tolist()
    model.generate(prompt, DECODE_NEW)  # warm-up, captures the decode-step graph
    stream = torch.cuda.current_stream(device)
    prefill_ms, decode_ms, launches = [], [], 0
    tokens = None
    for _ in range(runs):
        model.reset()
        e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
        torch.cuda.synchronize(device)
        before = capi.launch_count()
        e0.record(stream)
        first, _ = model.forward_cached(prompt, logits=None)
        e1.record(stream)
        rest = model.decode(DECODE_NEW - 1)
        e2.record(stream)
        torch.cuda.synchronize(device)
        launches = capi.launch_count() - before
        prefill_ms.append(e0.elapsed_time(e1))
        decode_ms.append(e1.elapsed_time(e2))
        tokens = [first] + rest
    t0 = time.perf_counter()
    again = model.generate(prompt, DECODE_NEW)
    torch.cuda.synchronize(device)
    e2e_s = time.perf_counter() - t0
    # The same prefill with the prompt projections on the tensor cores (opt-in, tolerance parity).
    model.set_prefill("tensor_cores")
    tc_ms = []
    for i in range(runs + 1):
        model.reset()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize(device)
        e0.record(stream)
        tc_first, _ = model.forward_cached(prompt, logits=None)
        e1.record(stream)
        torch.cuda.synchronize(device)
        if i > 0:  # the first run is a warm-up
            tc_ms.append(e0.elapsed_time(e1))
    model.set_prefill("cuda_cores")
    step_launches = model.step_launches
    model.close()
    dec = statistics.median(decode_ms)
    return {"decode_ms": dec, "prefill_ms": statistics.median(prefill_ms), "e2e_s": e2e_s,
            "prefill_tc_ms": statistics.median(tc_ms), "prefill_tc_first_token_same": tc_first == tokens[0],
            "launches_per_run": launches, "step_launches": step_launches, "tokens": tokens,
            "deterministic": again == tokens, "cfg": cfg}


def measure_cpu_decode(seconds: float) -> dict:
    """The C restatement of the decoder (oracle/qwen3.py over oracle/oracle.c, OpenMP) on this host: a 16-token
    prompt, then greedy decode steps for about `seconds`."""
    import numpy as np

    from cppinf_b200.qwen3 import Qwen3Config, random_weights
    from oracle.qwen3 import OracleQwen3

    cfg = Qwen3Config.qwen3_0_6b()
    model = OracleQwen3(cfg, random_weights(cfg, 0), 16 + 256)
    prompt = np.random.default_rng(0).integers(0, cfg.vocab_size, 16)
    logits = model.forward_cached(prompt)
    tok = int(model.o.row_argmax(logits)[0])
    n = 0
    t0 = time.perf_counter()
    while n < 256 - 1:
        logits = model.forward_cached([tok])
        tok = int(model.o.row_argmax(logits)[0])
        n += 1
        if time.perf_counter() - t0 >= seconds:
            break
    elapsed = time.perf_counter() - t0
    return {"value": round(n / elapsed, 3), "unit": "tok/s", "cores": os.cpu_count(), "cpu_model": cpu_model(),
            "kind": "port",
            "sample": f"{n} greedy decode steps after a 16-token prompt in {elapsed:.1f} s: the C restatement of "
                      "the decoder (oracle/qwen3.py, OpenMP over output rows)"}


# ---------------------------------------------------------------------------------------------------------------
# Arms
# ---------------------------------------------------------------------------------------------------------------


def headline_config(workload: str, world: int) -> dict:
    """The `config` of both arms' JSON lines (identical keys and values for the same workload and GPU count)."""
    global_tokens = 2048 * world if workload == "qk_norm_rope" else None
    return {
        "workload": f"{workload}: {CONFIGS[workload]['desc']}",
        "global_tokens": global_tokens,
        "parallelism": (f"one {global_tokens}-token batch, token rows partitioned over {world} GPU(s) with global "
                        "RoPE positions (cppinf_b200/shard.py token_shard), no data-path collective"
                        if workload == "qk_norm_rope" else f"{world} GPU(s), one configuration per GPU"),
    }


def cpu_model() -> str:
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def run_reference(args) -> None:
    """The reference's CPU path on this host: exactly --steps timed steps after --warmup, each step a bounded token
    sample of the 2048-token configuration, sized so the whole run takes about --cpu-seconds."""
    rank, world, _ = dist_env()
    if rank != 0:
        return
    cpu = CpuQkNormRope("reference")
    t0 = time.perf_counter()
    cpu.step(256)
    per_token = (time.perf_counter() - t0) / 256
    budget = max(args.cpu_seconds, 2.0)
    tokens = int(min(2048, max(1, budget / max(args.steps, 1) / per_token)))
    for _ in range(args.warmup):
        cpu.step(tokens)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        cpu.step(tokens)
    elapsed = time.perf_counter() - t0
    cpu.close()
    value = round(args.steps * qk_bytes(tokens) / elapsed / 1e9, 3)
    sample = f"{args.steps} steps of {tokens} of the 2048 token rows in {elapsed:.1f} s: {cpu.describe()}"
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(elapsed / args.steps * 1e3, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) q/k, N(1,0.1) norm weights)",
        "config": headline_config(HEADLINE, world),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cpu.threads, "cpu_model": cpu_model(),
                         "kind": cpu.kind, "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    if not args.no_decode:
        # The reference's decoder needs oneDNN (absent here); its CPU path is timed through the C restatement.
        dec = measure_cpu_decode(max(args.cpu_seconds, 2.0))
        line["decode"] = {"metric": "random-init Qwen3-0.6B greedy decode tok/s", "value": dec["value"],
                          "unit": "tok/s", "cpu_baseline": dec,
                          "e2e": {"value": dec["value"], "unit": "tok/s", "h2d_bytes_per_step": 0,
                                  "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_ours(args) -> None:
    import torch
    import torch.distributed as dist

    rank, world, local_rank = dist_env()
    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", device_id=device, timeout=timedelta(seconds=120))

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(value: float) -> float:
        if world == 1:
            return value
        t = torch.tensor([value], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    peak, peak_kind = read_peak_gbs()
    stream = torch.cuda.Stream(device)

    if args.workload == "qk_norm_rope":
        # This rank's token rows of one (2048 * N)-token batch, at their global RoPE positions.
        from cppinf_b200.shard import token_shard

        sh = token_shard(2048 * world, world, rank)
        wl = Workload(args.workload, rank, device, tokens=sh.tokens, position_offset=sh.position_offset)
    else:
        wl = Workload(args.workload, rank, device)
    clocks = ClockSampler(local_rank)
    clocks.start()
    ms, launches, spread = time_device_steps(wl, args.steps, args.warmup, stream, barrier, repeats=args.repeats)
    clock_info = clocks.stop()
    ms_max = max_over_ranks(ms)
    spread = [max_over_ranks(x) for x in spread]
    per_step_ms = ms_max / args.steps
    value = world * wl.bytes * args.steps / (ms_max * 1e-3) / 1e9
    achieved = wl.bytes / (ms / args.steps * 1e-3) / 1e9  # this rank's kernel: bytes per launch / launch time
    resident = wl.resident_bytes
    repeats = None
    if spread:
        us = sorted(x / args.steps * 1e3 for x in spread)
        med = statistics.median(us)
        repeats = {"count": len(us), "us_per_step_median": round(med, 3), "us_per_step_min": round(us[0], 3),
                   "us_per_step_max": round(us[-1], 3), "gbs_median": round(wl.bytes / (med * 1e-6) / 1e9, 1),
                   "frac_median": round(wl.bytes / (med * 1e-6) / 1e9 / peak, 4),
                   "how": f"the same {args.steps}-step graph replayed {len(us)} more times, each timed alone"}
    del wl
    torch.cuda.empty_cache()

    e2e = None if args.no_e2e else time_e2e(args.workload, rank, device, min(args.steps, 200))
    e2e_line = None
    if e2e is not None:
        e2e_ms = max_over_ranks(e2e["ms"])
        e2e_line = {"value": round(world * CONFIGS[args.workload]["bytes"] * e2e["steps"] / (e2e_ms * 1e-3) / 1e9, 2),
                    "unit": UNIT, "h2d_bytes_per_step": e2e["h2d_bytes_per_step"],
                    "d2h_bytes_per_step": e2e["d2h_bytes_per_step"],
                    "how": "cppinf_b200.ops.qk_norm_rope from pinned host buffers; H2D, kernel and D2H on three "
                           "streams, double-buffered"}

    # One GPU: every other configuration measured on its own. Several GPUs: one global batch per configuration
    # partitioned across the ranks, with and without the copy-back to rank 0 (sharded_legs).
    per_op = {}
    if not args.no_ops and world == 1:
        for name in CONFIGS:
            if name == args.workload:
                continue
            w2 = Workload(name, rank, device)
            op_ms, _, _ = time_device_steps(w2, args.op_steps, 3, stream, barrier)
            op_ms = max_over_ranks(op_ms)
            gbs = w2.bytes / (op_ms / args.op_steps * 1e-3) / 1e9
            per_op[name] = {"gbs": round(gbs, 1), "frac": round(gbs / peak, 4), "us_per_step":
                            round(op_ms / args.op_steps * 1e3, 3), "bytes": w2.bytes,
                            "traffic": read_traffic(name)}
            if "flops" in CONFIGS[name]:
                tflops = CONFIGS[name]["flops"] / (op_ms / args.op_steps * 1e-3) / 1e12
                tpeak, tkind = read_peak_tflops()
                per_op[name].update({"bound": "tensor", "tflops": round(tflops, 1), "tflops_peak": tpeak,
                                     "tflops_frac": round(tflops / tpeak, 4), "tflops_peak_source": tkind})
            if name == "rms_norm":
                # [512, 1024] is launch-latency bound: the isolated single-launch time, beside the graph-batched one.
                single = sorted(time_single_launches(w2, 50, stream))
                per_op[name]["single_launch_us_median"] = round(statistics.median(single), 3)
                per_op[name]["single_launch_gbs"] = round(w2.bytes / (statistics.median(single) * 1e-6) / 1e9, 1)
            del w2
            torch.cuda.empty_cache()
    sharded = None
    if not args.no_ops and world > 1:
        sharded = sharded_legs(world, rank, device, stream, barrier, max_over_ranks, peak, args.op_steps,
                               args.copy_steps)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = measure_cpu("port", args.cpu_seconds)

    decode = None
    if not args.no_decode:
        barrier()
        d = measure_decode(device, max(args.decode_runs, 1))
        dec_ms = max_over_ranks(d["decode_ms"])
        steps = DECODE_NEW - 1
        tok_s = world * steps / (dec_ms * 1e-3)
        cfg = d["cfg"]
        mean_ctx = DECODE_PROMPT + steps / 2 + 1
        bpt = decode_bytes_per_token(cfg, int(mean_ctx))
        achieved_dec = bpt * steps / (d["decode_ms"] * 1e-3) / 1e9
        e2e_s = max_over_ranks(d["e2e_s"])
        decode = {
            "metric": "random-init Qwen3-0.6B greedy decode tok/s", "value": round(tok_s, 1), "unit": "tok/s",
            "ms_per_token": round(dec_ms / steps, 4), "prefill_ms": round(max_over_ranks(d["prefill_ms"]), 2),
            "prefill_tensor_cores": {
                "ms": round(max_over_ranks(d["prefill_tc_ms"]), 3),
                "first_token_same": d["prefill_tc_first_token_same"],
                "how": "Qwen3Model.set_prefill('tensor_cores'): the prompt projections and attention on tcgen05 "
                       "(tolerance parity); prefill_ms above is the default bit-exact CUDA-core path"},
            "config": {"model": "Qwen3-0.6B, random init N(0,0.02) bf16, unit norm weights, tied embeddings",
                       "prompt_tokens": DECODE_PROMPT, "generated_tokens": DECODE_NEW, "batch": 1,
                       "parallelism": f"{world} independent replica(s), one per GPU (decode does not shard)"},
            "roofline": {"bound": "hbm", "achieved": round(achieved_dec, 1), "peak": peak, "unit": UNIT,
                         "frac": round(achieved_dec / peak, 4),
                         "bytes_per_token": bpt, "note": "weights once per step + KV rows at the mean context"},
            "e2e": {"value": round(world * DECODE_NEW / e2e_s, 1), "unit": "tok/s",
                    "h2d_bytes_per_step": DECODE_PROMPT * 8, "d2h_bytes_per_step": DECODE_NEW * 8,
                    "how": "Qwen3Model.generate(prompt, 128): host token ids in, prefill + 127 decode steps, "
                           "host token ids out"},
            "gpu_launches_per_run": d["launches_per_run"], "launches_per_step": d["step_launches"],
            "deterministic": d["deterministic"], "first_tokens": d["tokens"][:8],
        }
        if rank == 0 and world == 1 and not args.no_cpu:
            decode["cpu_baseline"] = measure_cpu_decode(args.cpu_seconds)

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(per_step_ms, 6), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded on device: N(0,1) activations, N(1,0.1) norm weights)",
            "config": headline_config(args.workload, world),
            "l2": f"steps rotate through buffer sets totalling {resident / 2**20:.0f} MiB (> 3x the 126 MB L2)",
            "timing": "CUDA graphs of <=1000 launches, CUDA events on the launch stream, max over ranks",
            "repeats": repeats,
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": UNIT,
                         "frac": round(achieved / peak, 4), "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)"
                         if peak_kind == "measured" else "fallback 6650 GB/s", "frac_of_8tbs": round(achieved / 8000, 4),
                         "traffic": read_traffic(args.workload), "bytes_per_launch": CONFIGS[args.workload]["bytes"],
                         "traffic_source": "profiles/<op>.md: dram__bytes_read.sum + dram__bytes_write.sum per "
                                           "launch, mean over launches in the middle of the bench's rotation"},
            "e2e": e2e_line,
            "gpu_launches": launches,
            "clocks": clock_info,
            "ops": per_op,
            "sharded": sharded,
            "cpu_baseline": cpu,
            "decode": decode,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def main():
    args = parse_args()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
