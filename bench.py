#!/usr/bin/env python
"""GDN layer throughput on B200: chunked prefill of 2 x 4096 tokens (Qwen3-Next
geometry: 16 q/k heads, 32 v heads, head dim 128, hidden 2048) followed by the
flattened gated-RMSNorm + out_proj tail, in tokens/s.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One process per GPU (torchrun for N > 1).  With N GPUs the heads are split
evenly across ranks (head-parallel; rank r holds v-heads [r*32/N, (r+1)*32/N)
and the matching q/k heads and out_proj columns) and every rank processes 2*N
sequences of 4096 tokens, so the per-rank kernel work is that of one GPU
("weak" scaling); the rank-partial [tokens, 2048] outputs are summed inside
the timed region as a reduce-scatter that overlaps the next step: over the
copy engines (peer copies, ``gdn_b200_rank_sum``) up to 4 GPUs and by NCCL's
reduce-scatter on a communication stream at 8, the faster of the two at each
N, measured (``--reduce ce|rs|nccl|fused`` forces one).  The end-to-end
figure goes through the provider ABI, whose output is the rank-partial as in
the reference, followed by the same reduction; each rank reads back only its
row shard.  ``--config cfg4`` prints the fixed-work head-parallel line
instead (16 x 16384 prefill then a 256-sequence decode step per call).  One
JSON line is printed by rank 0.

``--impl reference`` times the CPU restatement of the reference path (the
oracle; the reference itself runs only on Ascend NPUs) on the host cores with
the same metric and workload.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "qwen38-gdn-dual-sequence-output-tail_b200")
sys.path.insert(0, PKG)

METRIC = "GDN layer tokens/sec (chunked prefill 2x4096 + output tail)"
UNIT = "tokens/s"
SEQ_LEN = 4096
SEQS_PER_GPU = 2
QK_HEADS, V_HEADS, HIDDEN = 16, 32, 2048
CHUNK_MFLOP = 11.62    # prefill core work per (chunk of 64, v-head)
# DRAM bytes (read + write) per call of the chunk core on the single-GPU
# workload, from one ncu capture (dram__bytes_read.sum + dram__bytes_write.sum
# of the prep and state kernels on this workload).
CHUNK_CORE_DRAM_BYTES = {"prep": 68519680 + 116966656, "state": 244397056 + 46440960}


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


class ClockSampler:
    """Samples the SM clock and the throttle reasons of one GPU while the timed
    region runs: NVML polled every 2 ms from a thread (the timed regions here
    are a few ms long), or nvidia-smi at its 20 ms period when NVML is absent."""

    REASONS = {"hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20,
               "hw_thermal_slowdown": 0x40, "sw_power_cap": 0x4}
    SMI_COLUMNS = {"hw_slowdown": 5, "hw_thermal_slowdown": 6, "sw_thermal_slowdown": 7,
                   "sw_power_cap": 8}
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.device_index = device_index
        self.samples = []      # (monotonic s, sm_mhz, max_mhz, reason bit mask)
        self.proc = None
        self.file = None
        self.thread = None
        self.nvml = None
        self.errors = 0
        self.t0 = 0.0
        self.stop = threading.Event()

    def _nvml_handle(self):
        import pynvml
        pynvml.nvmlInit()
        visible = os.environ.get("CUDA_VISIBLE_DEVICES", "")
        ids = [v.strip() for v in visible.split(",") if v.strip()]
        if ids and self.device_index < len(ids) and ids[self.device_index].isdigit():
            return pynvml, pynvml.nvmlDeviceGetHandleByIndex(int(ids[self.device_index]))
        return pynvml, pynvml.nvmlDeviceGetHandleByIndex(self.device_index)

    def _sample(self, nv, h, reasons, mx):
        self.samples.append((time.monotonic(), nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM),
                             mx, int(reasons(h))))

    def _poll(self, nv, h, reasons, mx):
        while not self.stop.is_set():
            try:
                self._sample(nv, h, reasons, mx)
            except Exception:
                self.errors += 1
            time.sleep(0.002)

    def __enter__(self):
        try:
            nv, h = self._nvml_handle()
            reasons = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                nv.nvmlDeviceGetCurrentClocksThrottleReasons
            mx = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
            self._sample(nv, h, reasons, mx)        # NVML answers: poll it from a thread
            self.nvml = (nv, h, reasons, mx)
            self.thread = threading.Thread(target=self._poll, args=self.nvml, daemon=True)
            self.thread.start()
        except Exception:
            self.thread = None
            self.nvml = None
            self.file = tempfile.NamedTemporaryFile(mode="w+", suffix=".csv", delete=False)
            try:
                self.proc = subprocess.Popen(
                    ["nvidia-smi", f"--id={self.device_index}", f"--query-gpu={self.QUERY}",
                     "--format=csv,noheader,nounits", "-lms", "20"],
                    stdout=self.file, stderr=subprocess.DEVNULL)
            except Exception:
                self.proc = None
            time.sleep(0.05)
        self.t0 = time.monotonic()
        return self

    def __exit__(self, *exc):
        t1 = time.monotonic()
        self.stop.set()
        if self.thread is not None:
            self.thread.join(timeout=5)
            # Samples taken inside the timed region only; if the region was
            # too short for the poller, one sample right at its end.
            inside = [x for x in self.samples if self.t0 <= x[0] <= t1]
            if not inside:
                try:
                    self._sample(*self.nvml)
                    inside = self.samples[-1:]
                except Exception:
                    self.errors += 1
            self.samples = inside
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
        if self.file is not None:
            self.file.flush()
            try:
                with open(self.file.name) as f:
                    for r in (r.split(",") for r in f.read().strip().splitlines() if r.strip()):
                        try:
                            mask = sum(self.REASONS[name] for name, col in self.SMI_COLUMNS.items()
                                       if r[col].strip().lower() == "active")
                            self.samples.append((0.0, float(r[1]), float(r[2]), mask))
                        except Exception:
                            continue
                os.unlink(self.file.name)
            except Exception:
                pass

    def summary(self):
        sm = [x[1] for x in self.samples]
        mx = max((x[2] for x in self.samples), default=0.0)
        reasons = sorted(name for name, bit in self.REASONS.items()
                         if any(x[3] & bit for x in self.samples))
        out = {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx or None,
               "reasons": reasons, "samples": len(sm),
               "source": "nvml, 2 ms" if self.thread is not None else "nvidia-smi, 20 ms"}
        if self.errors:
            out["sample_errors"] = self.errors
        return out


def workload_desc(nseq: int) -> str:
    return (f"chunked prefill {nseq}x{SEQ_LEN} tokens + flattened output tail, "
            f"Hk={QK_HEADS} Hv={V_HEADS} D=128 hidden={HIDDEN}, chunk 64")


def resolve_reduce(reduce: str, gpus: int) -> str:
    """The rank-sum method for --reduce on `gpus` GPUs.  Measured on 8 B200s
    (bench workload): the copy-engine reduce-scatter wins up to 4 GPUs
    (N = 2: 0.430 ms against 0.520 ms with NCCL's reduce-scatter), NCCL's
    reduce-scatter at 8 (0.729 against 0.796 ms)."""
    if reduce != "auto":
        return reduce
    return "ce" if gpus <= 4 else "rs"


def use_fused_reduce(world: int, reduce: str) -> bool:
    return world > 1 and reduce == "fused"


def use_ce_reduce(world: int, reduce: str) -> bool:
    return world > 1 and reduce == "ce"


def reduce_desc(world: int, reduce: str) -> str:
    if world == 1:
        return ""
    if use_fused_reduce(world, reduce):
        return " + rank sum fused into the tail GEMM (NVLink peer memory)"
    if use_ce_reduce(world, reduce):
        return (" + rank sum as a reduce-scatter over the copy engines (peer copies over "
                "NVLink, each rank receives its row shard), overlapping the next step")
    if reduce == "rs":
        return (" + nccl reduce-scatter (each rank receives its row shard), overlapping the "
                "next step on a communication stream")
    return " + nccl all-reduce, overlapping the next step on a communication stream"


def prefill_config(world: int, reduce: str) -> dict:
    """The headline workload's config, the same for both arms."""
    nseq = SEQS_PER_GPU * world
    T = nseq * SEQ_LEN
    hk, hv = QK_HEADS // world, V_HEADS // world
    qkvz_mb = (2 * T * hk * 128 + 2 * T * hv * 128) * 2 / 1e6
    return {"workload": workload_desc(nseq), "tokens_per_step": T, "sequences": nseq,
            "seq_len": SEQ_LEN,
            "parallelism": f"head-parallel tp{world}" + reduce_desc(world, reduce),
            "l2": "inputs larger than L2 (q,k,v,z = %.0f MB per step)" % qkvz_mb}


def cpu_oracle_prefill(seq_len: int, nseq: int):
    """Runs the CPU oracle (restatement of the reference's op sequence) on the
    prefill workload, with inputs from the oracle's own copy of the seeded
    generator (the product library is never loaded); returns (tokens/s,
    seconds, threads)."""
    import numpy as np
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import gdn_oracle as O
    import gdn_b200 as G          # Geometry and the input layout only: no library load
    geom = G.Geometry(QK_HEADS, V_HEADS, HIDDEN)
    cu = np.arange(nseq + 1, dtype=np.int32) * seq_len
    x = G.synthetic_layer_inputs(cu, geom, seed=1, fill=O.fill)
    st = x["state"].copy()
    t0 = time.perf_counter()
    O.layer(x["q"], x["k"], x["v"], x["a"], x["b"], x["z"], x["A_log"], x["dt_bias"],
            x["gamma"], x["w_out"], st, cu, mode=0)
    dt = time.perf_counter() - t0
    return (nseq * seq_len) / dt, dt, O.threads()


def run_reference(args):
    """The reference arm: the CPU restatement of the reference's path (the
    oracle; the reference itself runs only on Ascend NPUs) on all host threads.
    Each step is the 2x4096 prefill of one GPU's share, a bounded sample of
    the N-GPU workload; rank 0 alone runs it."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    nseq = SEQS_PER_GPU * args.gpus
    for _ in range(args.warmup):
        cpu_oracle_prefill(SEQ_LEN, SEQS_PER_GPU)
    times = []
    threads = 1
    for _ in range(args.steps):
        _, dt, threads = cpu_oracle_prefill(SEQ_LEN, SEQS_PER_GPU)
        times.append(dt)
    step = statistics.median(times)
    value = SEQS_PER_GPU * SEQ_LEN / step
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": step * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded SplitMix64/Box-Muller, benchmark distributions)",
        "config": prefill_config(args.gpus, args.reduce),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": f"{SEQS_PER_GPU}x{SEQ_LEN} tokens of the "
                                   f"{nseq}x{SEQ_LEN} workload per step (median of "
                                   f"{args.steps})"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def nbytes(*tensors) -> int:
    return sum(t.numel() * t.element_size() for t in tensors)


def flushed_timer(stream, flush):
    """Times single calls on `stream` with CUDA events, writing `flush` (larger
    than L2) before each, so every call starts with its inputs out of L2."""
    import torch

    def timed(f, iters, warm=3):
        for _ in range(warm):
            flush.zero_()
            f()
        torch.cuda.synchronize()
        total = 0.0
        for _ in range(iters):
            flush.zero_()
            s_, e_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s_.record(stream)
            f()
            e_.record(stream)
            torch.cuda.synchronize()
            total += s_.elapsed_time(e_)
        return total / iters
    return timed


def small_shape_components(dev, stream, iters):
    """The metric's other shapes on one GPU, each timed per call with L2
    flushed before the call:

    * ``prefill_2x64``: the whole layer (chunked prefill + flattened tail) over
      2 sequences of 64 tokens, the reference's admitted dual-sequence unit
      (inputs as the 2x4096 workload, zero initial state);
    * ``tail_2x64``: the dual-sequence output tail alone over 2 x 64 rows
      (o, z [128, 32, 128] ~ N(0,1), gamma 1 + N(0, 0.02), w_out [2048, 4096]
      ~ N(0, 0.02));
    * ``decode_b64``: one decode step of 64 sequences (f32 state [64, 32, 128,
      128] ~ N(0, 0.05)) plus the flattened tail over the 64 rows, and the
      decode kernel alone (the state read + write is its HBM stream).

    ``gbs`` = algorithmic bytes (every input read once, the state read and
    written, the output written) / time; ``frac`` = gbs / measured HBM copy
    bandwidth."""
    import numpy as np
    import torch
    import gdn_b200 as G
    hbm_peak, _, _ = load_peaks()
    geom = G.Geometry(QK_HEADS, V_HEADS, HIDDEN)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    timed = flushed_timer(stream, flush)
    comps = {}

    def layer_case(cu, seed, state_std):
        t = G.to_device(G.synthetic_layer_inputs(cu, geom, seed=seed, state_std=state_std), dev)
        T = int(cu[-1])
        out = torch.empty(T, HIDDEN, dtype=torch.bfloat16, device=dev)
        ws = torch.empty(G.layer_forward_workspace_bytes(cu, QK_HEADS, V_HEADS, HIDDEN),
                         dtype=torch.uint8, device=dev)
        fn = lambda: G.layer_forward(t["q"], t["k"], t["v"], t["a"], t["b"], t["z"], t["A_log"],
                                     t["dt_bias"], t["gamma"], t["w_out"], t["state"], cu,
                                     out=out, workspace=ws, stream=stream)
        alg = (nbytes(*(t[n] for n in ("q", "k", "v", "a", "b", "z", "A_log", "dt_bias",
                                       "gamma", "w_out"))) + 2 * nbytes(t["state"]) + nbytes(out))
        return t, fn, ws, alg

    # prefill 2 x 64
    cu = np.array([0, 64, 128], np.int32)
    _, fn, ws, alg = layer_case(cu, 1, 0.0)
    ms = timed(fn, iters)
    G.workspace_status(ws, stream)
    gbs = alg / (ms * 1e-3) / 1e9
    comps["prefill_2x64"] = {"us": ms * 1e3, "tokens_per_s": 128 / (ms * 1e-3),
                             "algorithmic_bytes": alg, "gbs": gbs, "frac": gbs / hbm_peak,
                             "bound": "hbm"}

    # output tail 2 x 64
    rows = 128
    x = {n: G.fill(0, i, sh, G.NORMAL, mu, sd, G.BF16) for n, i, sh, mu, sd in (
        ("o", 21, (rows, V_HEADS, 128), 0.0, 1.0), ("z", 22, (rows, V_HEADS, 128), 0.0, 1.0),
        ("gamma", 23, (128,), 1.0, 0.02), ("w", 24, (HIDDEN, V_HEADS * 128), 0.0, 0.02))}
    t = G.to_device(x, dev)
    out = torch.empty(rows, HIDDEN, dtype=torch.bfloat16, device=dev)
    ws = torch.empty(G.output_tail_workspace_bytes(rows, V_HEADS, HIDDEN), dtype=torch.uint8,
                     device=dev)
    ms = timed(lambda: G.output_tail(t["o"], t["z"], t["gamma"], t["w"], out=out, workspace=ws,
                                     stream=stream), iters)
    G.workspace_status(ws, stream)
    alg = nbytes(t["o"], t["z"], t["gamma"], t["w"], out)
    gbs = alg / (ms * 1e-3) / 1e9
    comps["tail_2x64"] = {"us": ms * 1e3, "rows_per_s": rows / (ms * 1e-3),
                          "algorithmic_bytes": alg, "gbs": gbs, "frac": gbs / hbm_peak,
                          "bound": "hbm"}

    # decode B = 64: step (decode + tail) and the decode kernel alone
    B = 64
    cu = np.arange(B + 1, dtype=np.int32)
    t, fn, ws, alg = layer_case(cu, 5, 0.05)
    ms = timed(fn, iters)
    G.workspace_status(ws, stream)
    gated = torch.empty(B, V_HEADS * 128, dtype=torch.bfloat16, device=dev)
    k_ms = timed(lambda: G.decode_step(t["q"], t["k"], t["v"], t["a"], t["b"], t["A_log"],
                                       t["dt_bias"], t["state"], z=t["z"], gamma=t["gamma"],
                                       gated_out=gated, stream=stream), iters)
    k_alg = (2 * nbytes(t["state"]) + nbytes(*(t[n] for n in ("q", "k", "v", "a", "b", "z",
                                                               "A_log", "dt_bias", "gamma")))
             + nbytes(gated))
    gbs, k_gbs = alg / (ms * 1e-3) / 1e9, k_alg / (k_ms * 1e-3) / 1e9
    comps["decode_b64"] = {"us": ms * 1e3, "tokens_per_s": B / (ms * 1e-3),
                           "algorithmic_bytes": alg, "gbs": gbs, "frac": gbs / hbm_peak,
                           "bound": "hbm", "kernel": "gdn_decode_kernel", "kernel_us": k_ms * 1e3,
                           "kernel_algorithmic_bytes": k_alg, "kernel_gbs": k_gbs,
                           "kernel_frac": k_gbs / hbm_peak}
    del flush
    return comps


CFG4_SEQS, CFG4_LEN, CFG4_DECODE = 16, 16384, 256


def run_cfg4(args):
    """The sharded workload: 16 sequences x 16384 tokens of chunked prefill,
    then one decode step of 256 sequences (f32 state ~ N(0, 0.05)), the heads
    split over N GPUs (Hv/N and Hk/N per rank, w_out columns sharded), each
    layer's rank-partial output summed by the copy-engine reduce-scatter
    (at N > 1) overlapping the next call.  Total work is fixed: "strong"
    scaling.  One JSON line at rank 0."""
    import numpy as np
    import torch
    import torch.distributed as dist
    import gdn_b200 as G
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=300))
    hk, hv = QK_HEADS // world, V_HEADS // world
    full = G.Geometry(QK_HEADS, V_HEADS, HIDDEN)
    cu_p = np.arange(CFG4_SEQS + 1, dtype=np.int32) * CFG4_LEN
    cu_d = np.arange(CFG4_DECODE + 1, dtype=np.int32)
    Tp, Td = int(cu_p[-1]), CFG4_DECODE
    shard = (rank, world) if world > 1 else None
    tp = G.to_device(G.synthetic_layer_inputs(cu_p, full, seed=41, shard=shard), dev)
    td = G.to_device(G.synthetic_layer_inputs(cu_d, full, seed=42, state_std=0.05, shard=shard), dev)
    ws_p = torch.empty(G.layer_forward_workspace_bytes(cu_p, hk, hv, HIDDEN), dtype=torch.uint8,
                       device=dev)
    ws_d = torch.empty(G.layer_forward_workspace_bytes(cu_d, hk, hv, HIDDEN), dtype=torch.uint8,
                       device=dev)
    stream = torch.cuda.Stream(device=dev)
    comm = torch.cuda.Stream(device=dev)
    torch.cuda.set_stream(stream)
    out_p = torch.empty(Tp, HIDDEN, dtype=torch.bfloat16, device=dev)
    out_d = torch.empty(Td, HIDDEN, dtype=torch.bfloat16, device=dev)
    rs = None
    if world > 1:
        def exchange(payload):
            got = [None] * world
            dist.all_gather_object(got, payload)
            return got
        rs = {n: G.RankSum(T, HIDDEN, rank, world, dev, exchange=exchange)
              for n, T in (("p", Tp), ("d", Td))}
        shards = {n: [torch.empty(T // world, HIDDEN, dtype=torch.bfloat16, device=dev)
                      for _ in range(2)] for n, T in (("p", Tp), ("d", Td))}
    epoch = [0]

    def layer(t, cu, T, out, ws, key, e):
        if rs is None:
            G.layer_forward(t["q"], t["k"], t["v"], t["a"], t["b"], t["z"], t["A_log"],
                            t["dt_bias"], t["gamma"], t["w_out"], t["state"], cu, out=out,
                            workspace=ws, stream=stream)
            return
        r = rs[key]
        r.acquire(e, stream)
        G.layer_forward(t["q"], t["k"], t["v"], t["a"], t["b"], t["z"], t["A_log"],
                        t["dt_bias"], t["gamma"], t["w_out"], t["state"], cu,
                        out=r.part(e, T), workspace=ws, stream=stream)
        r.reduce(e, T, shards[key][e & 1], stream, comm)

    def step():
        epoch[0] += 1
        layer(tp, cu_p, Tp, out_p, ws_p, "p", epoch[0])
        layer(td, cu_d, Td, out_d, ws_d, "d", epoch[0])

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    launches0 = G.kernel_launches()
    with ClockSampler(local) as clocks:
        s.record(stream)
        for _ in range(args.steps):
            step()
        stream.wait_stream(comm)
        e.record(stream)
        torch.cuda.synchronize()
    launches = G.kernel_launches() - launches0
    ms = s.elapsed_time(e) / args.steps
    G.workspace_status(ws_p, stream)
    G.workspace_status(ws_d, stream)
    if rs is not None:
        for r in rs.values():
            r.status(comm)
        v = torch.tensor([ms], device=dev)
        dist.all_reduce(v, op=dist.ReduceOp.MAX)
        ms = float(v.item())
    tokens = Tp + Td
    if rank == 0:
        line = {
            "metric": "GDN layer tokens/sec (config 4: 16x16384 prefill then a 256-sequence "
                      "decode step, head-parallel)",
            "value": tokens / (ms * 1e-3), "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded SplitMix64/Box-Muller, benchmark distributions)",
            "config": {"workload": f"chunked prefill {CFG4_SEQS}x{CFG4_LEN} tokens + tail, then "
                                   f"a decode step of {CFG4_DECODE} sequences + tail, Hk=16 "
                                   f"Hv=32 D=128 hidden=2048 over {world} GPU(s)",
                       "tokens_per_step": tokens,
                       "parallelism": f"head-parallel tp{world}" + reduce_desc(world, "ce"),
                       "l2": "inputs larger than L2"},
            "gpu_launches": launches,
            "clocks": clocks.summary(),
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.cuda.synchronize()
        dist.barrier()
        for r in rs.values():
            r.close()
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--config", choices=["cfg1", "cfg4"], default="cfg1",
                    help="cfg1 (default): the headline 2N x 4096 prefill line; cfg4: 16 x "
                         "16384 prefill then a 256-sequence decode, head-parallel (strong "
                         "scaling)")
    ap.add_argument("--component-iters", type=int, default=50,
                    help="calls timed per small-shape component (N=1 only)")
    ap.add_argument("--reduce", choices=["auto", "ce", "fused", "nccl", "rs"], default="auto",
                    help="N > 1: the rank sum as a copy-engine reduce-scatter overlapping the "
                         "next step (ce), fused into the tail GEMM over NVLink peer memory "
                         "(fused), or a bf16 NCCL all-reduce (nccl) or reduce-scatter (rs) on "
                         "a communication stream; auto (default): ce up to 4 GPUs, rs at 8")
    args = ap.parse_args()
    if args.warmup < 3:
        raise SystemExit("--warmup must be at least 3")
    args.reduce = resolve_reduce(args.reduce, args.gpus)
    if args.impl == "reference":
        run_reference(args)
        return
    if args.config == "cfg4":
        run_cfg4(args)
        return

    import numpy as np
    import torch
    import torch.distributed as dist
    import gdn_b200 as G

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=120))
    if V_HEADS % world or QK_HEADS % world:
        raise SystemExit("heads must split evenly")

    hk, hv = QK_HEADS // world, V_HEADS // world
    geom = G.Geometry(hk, hv, HIDDEN)
    nseq = SEQS_PER_GPU * world
    cu = np.arange(nseq + 1, dtype=np.int32) * SEQ_LEN
    T = int(cu[-1])
    # Seeded synthetic inputs with the benchmark distributions for this
    # rank's head shard (tensor ids offset per rank).
    x = G.synthetic_layer_inputs(cu, geom, seed=1 + 1000 * rank)
    host = {}
    for n in ("q", "k", "v", "a", "b", "z"):
        host[n] = torch.from_numpy(x[n].view(np.int16)).view(torch.bfloat16).pin_memory()
    t = G.to_device(x, dev)
    out = torch.empty(T, HIDDEN, dtype=torch.bfloat16, device=dev)
    ws = torch.empty(G.layer_forward_workspace_bytes(cu, hk, hv, HIDDEN), dtype=torch.uint8,
                     device=dev)
    # A dedicated stream: the provider ABI rejects the null stream, as the
    # reference does (qwen38_geometry_normalized_gdn_provider.cpp:2272).
    stream = torch.cuda.Stream(device=dev)
    torch.cuda.set_stream(stream)

    fused = use_fused_reduce(world, args.reduce)
    group = None
    if fused:
        # Every rank's exchange region mapped into every rank (CUDA IPC
        # handles passed through the process group).
        def exchange(payload):
            got = [None] * world
            dist.all_gather_object(got, payload)
            return got

        group = G.TailGroup(T, HIDDEN, rank, world, dev, exchange=exchange)
        o_buf = torch.empty_like(t["v"])
        ws_chunk = torch.empty(G.chunk_prefill_workspace_bytes(cu, hk, hv), dtype=torch.uint8,
                               device=dev)
        ws_ar = torch.empty(G.output_tail_allreduce_workspace_bytes(T, hv), dtype=torch.uint8,
                            device=dev)

    # NCCL reductions run on their own stream: the reduction of step i's
    # rank-partial output overlaps step i + 1, which depends only on the
    # recurrent state (two output buffers; step i + 2 reuses step i's buffer
    # once its reduction is done).
    ce = use_ce_reduce(world, args.reduce)
    rsum = None
    if ce:
        def exchange_ce(payload):
            got = [None] * world
            dist.all_gather_object(got, payload)
            return got

        rsum = G.RankSum(T, HIDDEN, rank, world, dev, exchange=exchange_ce)
        ce_shards = [torch.empty(T // world, HIDDEN, dtype=torch.bfloat16, device=dev)
                     for _ in range(2)]
    epoch = [0]

    comm = torch.cuda.Stream(device=dev) if world > 1 and not fused else None
    red_outs = [out, torch.empty_like(out)] if comm is not None else [out]
    red_shards = ([torch.empty(T // world, HIDDEN, dtype=torch.bfloat16, device=dev)
               for _ in range(2)] if args.reduce == "rs" and comm is not None else None)
    ev_red_in = [torch.cuda.Event() for _ in range(2)]
    ev_red = [torch.cuda.Event() for _ in range(2)]
    red_used = [False, False]

    def step(i=0):
        if fused:
            G.chunk_prefill(t["q"], t["k"], t["v"], t["a"], t["b"], t["A_log"], t["dt_bias"],
                            t["state"], cu, o_out=o_buf, workspace=ws_chunk, stream=stream)
            group.output_tail(o_buf, t["z"], t["gamma"], t["w_out"], workspace=ws_ar,
                              stream=stream)
            return
        if ce:
            # The layer writes its rank-partial straight into the exchange
            # buffer of this epoch; the copy engines move the rows.
            epoch[0] += 1
            e = epoch[0]
            rsum.acquire(e, stream)
            G.layer_forward(t["q"], t["k"], t["v"], t["a"], t["b"], t["z"], t["A_log"],
                            t["dt_bias"], t["gamma"], t["w_out"], t["state"], cu,
                            out=rsum.part(e, T), workspace=ws, stream=stream)
            rsum.reduce(e, T, ce_shards[e & 1], stream, comm)
            return
        b = i & 1 if comm is not None else 0
        if comm is not None and red_used[b]:
            stream.wait_event(ev_red[b])           # step i - 2's reduction has read it
        G.layer_forward(t["q"], t["k"], t["v"], t["a"], t["b"], t["z"], t["A_log"],
                        t["dt_bias"], t["gamma"], t["w_out"], t["state"], cu, out=red_outs[b],
                        workspace=ws, stream=stream)
        if comm is not None:
            ev_red_in[b].record(stream)
            with torch.cuda.stream(comm):
                comm.wait_event(ev_red_in[b])
                if red_shards is not None:
                    dist.reduce_scatter_tensor(red_shards[b], red_outs[b])
                else:
                    dist.all_reduce(red_outs[b])
                ev_red[b].record(comm)
            red_used[b] = True

    def timed(fn, iters, warm):
        for i in range(warm):
            fn(i)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(stream)
        for i in range(iters):
            fn(i)
        if comm is not None and fn is step:
            stream.wait_stream(comm)                # the last reduction is inside the region
        e.record(stream)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        ms = s.elapsed_time(e) / iters
        if world > 1:
            v = torch.tensor([ms], device=dev)
            dist.all_reduce(v, op=dist.ReduceOp.MAX)
            ms = float(v.item())
        return ms

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    G.workspace_status(ws_ar if fused else ws, stream)
    launches0 = G.kernel_launches()
    with ClockSampler(local) as clocks:
        ms = timed(step, args.steps, 0)
    launches = G.kernel_launches() - launches0
    clk = clocks.summary()
    G.workspace_status(ws_ar if fused else ws, stream)
    if rsum is not None:
        rsum.status(comm)
    value = T / (ms * 1e-3)   # T = every token of the job: ranks hold head shards of the same tokens

    # Components, timed alone with CUDA events on the launching stream:
    # the chunked core (prep + state kernels) and the output tail.
    o = torch.empty_like(t["v"])
    ws_core = torch.empty(G.chunk_prefill_workspace_bytes(cu, hk, hv), dtype=torch.uint8,
                          device=dev)
    ws_tail = torch.empty(G.output_tail_workspace_bytes(T, hv, HIDDEN), dtype=torch.uint8,
                          device=dev)
    core_ms = timed(lambda i=0: G.chunk_prefill(t["q"], t["k"], t["v"], t["a"], t["b"], t["A_log"],
                                            t["dt_bias"], t["state"], cu, o_out=o,
                                            workspace=ws_core, stream=stream), args.steps, 2)
    if fused:
        # the tail with the rank sum fused in (what the step runs)
        tail_ms = timed(lambda i=0: group.output_tail(o, t["z"], t["gamma"], t["w_out"],
                                                  workspace=ws_ar, stream=stream), args.steps, 2)
        G.workspace_status(ws_ar, stream)
    else:
        tail_ms = timed(lambda i=0: G.output_tail(o, t["z"], t["gamma"], t["w_out"], out=out,
                                              workspace=ws_tail, stream=stream), args.steps, 2)
    # The input side (x -> projections -> causal conv + SiLU -> q/k/v split,
    # conv-state update) on the same tokens, timed alone: the layer from x
    # adds it in front of the path above.
    xs = G.to_device(G.synthetic_input_side(cu, geom, seed=2 + 1000 * rank,
                                            conv_state_std=1.0), dev)
    ws_in = torch.empty(G.input_side_workspace_bytes(cu, hk, hv, HIDDEN), dtype=torch.uint8,
                        device=dev)
    in_out = (torch.empty_like(t["q"]), torch.empty_like(t["k"]), torch.empty_like(t["v"]),
              torch.empty_like(t["z"]), torch.empty_like(t["a"]), torch.empty_like(t["b"]))
    in_ms = timed(lambda i=0: G.input_side(xs["x"], xs["w_qkv"], xs["w_z"], xs["w_a"], xs["w_b"],
                                       xs["conv_w"], xs["conv_state"], cu, hk, out=in_out,
                                       workspace=ws_in, stream=stream), args.steps, 2)
    G.workspace_status(ws_in, stream)
    del xs, ws_in, in_out
    hbm_peak, tf_peak, peak_kind = load_peaks()
    chunks = nseq * (SEQ_LEN // 64)
    core_flop = CHUNK_MFLOP * 1e6 * chunks * hv
    tail_flop = 2.0 * T * (hv * 128) * HIDDEN
    core_tf = core_flop / (core_ms * 1e-3) / 1e12
    tail_tf = tail_flop / (tail_ms * 1e-3) / 1e12
    in_flop = 2.0 * T * HIDDEN * ((2 * hk + hv) * 128 + hv * 128 + 2 * hv)
    in_tf = in_flop / (in_ms * 1e-3) / 1e12
    comps = {
        "chunk_core": {"ms": core_ms, "tflops": core_tf, "frac": core_tf / tf_peak},
        "output_tail": {"ms": tail_ms, "tflops": tail_tf, "frac": tail_tf / tf_peak},
        "input_side": {"ms": in_ms, "tflops": in_tf, "frac": in_tf / tf_peak,
                       "note": "x -> q,k,v,z,a,b (projections + causal conv), not in the step"},
    }
    dom = "chunk_core" if core_ms >= tail_ms else "output_tail"
    # Measured DRAM traffic is quoted for the single-GPU workload only (the
    # per-rank shard of N GPUs has the same per-rank size, so it applies there
    # too: weak scaling keeps every rank's kernels identical).
    traffic = (sum(CHUNK_CORE_DRAM_BYTES.values()) if dom == "chunk_core" else None)
    roofline = {"bound": "tensor", "kernel": dom, "achieved": comps[dom]["tflops"],
                "peak": tf_peak, "unit": "TFLOP/s", "frac": comps[dom]["frac"],
                "peak_kind": f"{peak_kind} burst bf16", "traffic": traffic,
                "traffic_unit": "bytes per call (ncu, prep + state kernels)",
                "traffic_gbs": (traffic / (comps[dom]["ms"] * 1e-3) / 1e9) if traffic else None,
                "hbm_peak_gbs": hbm_peak}
    if world == 1:
        comps.update(small_shape_components(dev, stream, args.component_iters))

    # End to end through the provider ABI (the reference-facing plugin
    # interface), as a serving loop drives it: every step copies its inputs
    # from pinned host memory, submits the layer and copies its output back to
    # pinned host memory.  Steps are pipelined over two input/output buffer
    # sets and three streams (host->device copies, the provider's stream,
    # device->host copies), so the upload of step i+1 overlaps the compute and
    # read-back of step i; the recurrent state chains the steps in order on
    # the provider's stream.  With N GPUs each rank reads back only the rows
    # it owns (rows [r T/N, (r+1) T/N) of the reduced output), so the job
    # copies the output to the host once.
    prov = G.Provider(geom, max_tokens=T, world_size=world, rank=rank, device=local)
    r0, r1 = rank * T // world, (rank + 1) * T // world
    host_outs = [torch.empty(r1 - r0, HIDDEN, dtype=torch.bfloat16).pin_memory()
                 for _ in range(2)]
    h2d = nbytes(*host.values()) * world
    d2h = T * HIDDEN * 2
    t_in = [t, dict(t)]
    for n in host:
        t_in[1][n] = torch.empty_like(t[n])
    outs = [out, torch.empty_like(out)]
    e2e_shards = [torch.empty(T // world, HIDDEN, dtype=torch.bfloat16, device=dev)
                  for _ in range(2)]
    s_in = torch.cuda.Stream(device=dev)
    s_out = torch.cuda.Stream(device=dev)
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_comp = [torch.cuda.Event() for _ in range(2)]
    ev_out = [torch.cuda.Event() for _ in range(2)]
    pending = []

    def e2e_step(i):
        b = i & 1
        with torch.cuda.stream(s_in):
            if i >= 2:
                s_in.wait_event(ev_comp[b])     # step i - 2 is done with these inputs
            for n in host:
                t_in[b][n].copy_(host[n], non_blocking=True)
            ev_in[b].record(s_in)
        stream.wait_event(ev_in[b])
        if i >= 2:
            stream.wait_event(ev_out[b])        # step i - 2's output has been read back
        if ce:
            epoch[0] += 1
            e = epoch[0]
            rsum.acquire(e, stream)
            pending.append(prov.submit_layer(t_in[b], t["state"], rsum.part(e, T), cu,
                                             stream=stream))
            rsum.reduce(e, T, e2e_shards[b], stream, comm)
            ev_comp[b].record(comm)
            with torch.cuda.stream(s_out):
                s_out.wait_event(ev_comp[b])
                host_outs[b].copy_(e2e_shards[b], non_blocking=True)
                ev_out[b].record(s_out)
            while len(pending) > 1:
                ev = pending.pop(0)
                prov.wait(ev)
                prov.release(ev)
            return
        pending.append(prov.submit_layer(t_in[b], t["state"], outs[b], cu, stream=stream))
        if world > 1 and args.reduce == "rs":
            dist.reduce_scatter_tensor(e2e_shards[b], outs[b])
        elif world > 1:
            dist.all_reduce(outs[b])
        ev_comp[b].record(stream)
        with torch.cuda.stream(s_out):
            s_out.wait_event(ev_comp[b])
            host_outs[b].copy_(e2e_shards[b] if world > 1 and args.reduce == "rs"
                               else outs[b][r0:r1], non_blocking=True)
            ev_out[b].record(s_out)
        while len(pending) > 1:                 # keep one submission in flight
            ev = pending.pop(0)
            prov.wait(ev)
            prov.release(ev)

    def e2e_drain():
        while pending:
            ev = pending.pop(0)
            prov.wait(ev)
            prov.release(ev)
        torch.cuda.synchronize()

    for i in range(max(2, args.warmup // 2)):
        e2e_step(i)
    e2e_drain()
    if world > 1:
        dist.barrier()
    e2e_iters = max(10, args.steps // 2)
    t0 = time.perf_counter()
    for i in range(e2e_iters):
        e2e_step(i)
    e2e_drain()
    e2e_s = (time.perf_counter() - t0) / e2e_iters
    if world > 1:
        v = torch.tensor([e2e_s], device=dev)
        dist.all_reduce(v, op=dist.ReduceOp.MAX)
        e2e_s = float(v.item())
    prov.close()

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cps, csec, cthreads = cpu_oracle_prefill(SEQ_LEN, SEQS_PER_GPU)
        cpu = {"value": cps, "unit": UNIT, "cores": cthreads, "kind": "port",
               "sample": f"whole workload ({SEQS_PER_GPU}x{SEQ_LEN} tokens), one pass "
                         f"({csec:.2f} s)"}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded SplitMix64/Box-Muller, benchmark distributions)",
            "config": prefill_config(world, args.reduce),
            "roofline": roofline,
            "components": comps,
            "cpu_baseline": cpu,
            "e2e": {"value": T / e2e_s, "unit": UNIT, "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h,
                    "note": "whole-job bytes: every rank uploads its head shard's inputs, each "
                            "output row is read back once by the rank that owns it"},
            "gpu_launches": launches,
            "clocks": clk,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.cuda.synchronize()
        dist.barrier()
        if group is not None:
            group.close()
        if rsum is not None:
            rsum.close()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
