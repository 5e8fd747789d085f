#!/usr/bin/env python
"""Benchmark of the B200 Nemotron-3-Embed-1B encoder (driver contract).

python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                [--workload NAME] [--workloads all|none|a,b,...]

One "step" is one pass of the hot path over one batch of synthetic input: for
the forward workloads, one run of every engine micro-batch of the workload's
requests (NemotronExecutionPlan.run per micro-batch); for config 1, one sweep of
the standalone Q4_K matmul over 64 rotating weight copies.

Headline line (value, e2e, roofline, cpu_baseline): config 2 of the reference's
headline metric, 1 request of 15 tokens (BOS + uniform ids) through the full
16-layer random-init Q4_K_M-mix encoder. Under torchrun every rank drives its
own GPU with a full weight replica and its own request stream (request
sharding, no data-path collective; the only collectives are the timing barrier
and the max-over-ranks reduction).

`workloads` (same JSON line): every other benchmark configuration, each with
req/s (device-timed, inputs resident), e2e (through nemo_plan_run with host
buffers), the roofline of its dominant kernel and, at N=1, a CPU sample:
  config1     Q4_K dequant-matmul 15 x 2048 . (2048 x 2048)^T, f32 out, L2
              defeated by rotating 64 weight copies (151 MB)
  config2c16  16 concurrent requests x 15 tokens (one micro-batch of 16)
  config3     16 requests, lengths U[15,150]
  config4     16 requests x 1500 tokens (two engine micro-batches of 8)
  config5     1 request x 5000 tokens
  config5c16  16 requests x 5000 tokens (two engine micro-batches of 8)
  config5hp   (N = 2, 4, 8) 1 request x 5000 tokens head-parallel over all N
              GPUs from one process (the other ranks wait on a host barrier)
At N > 1 the forward workloads are one fixed set of requests split across the
ranks (every engine micro-batch's requests spread longest-first over the
ranks; "scaling": "strong"): req/s is total requests / the slowest rank's time.

--impl reference times the reference's CPU path on the host cores: the
reference is TypeScript + WGSL with no CPU forward and no JS engine here, so
its CPU path is the C++ oracle restating its CPU decode code and shader math.
"""
import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time

REPO = os.path.dirname(os.path.abspath(__file__))
PKG_DIR = os.path.join(REPO, "nemotron-3-embed-webgpu_b200")
for _p in (REPO, PKG_DIR):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import numpy as np  # noqa: E402

METRIC = "embed req/s at 15–5,000 tok (1 & 16 concurrent) on 1/2/4/8 B200; % roofline"
# The reference's published figures for the same workloads (Apple M3 Max,
# WebGPU, README.md:17-22): single-stream 15 and 5,000 tokens, 16-concurrent
# 15 tokens (native batch 16), 1,500 tokens (native batch 8) and 5,000 tokens.
PUBLISHED = {"config2": 69.68, "config5": 0.76, "config2c16": 266.02, "config4": 2.75, "config5c16": 0.72}

WORKLOADS = {
    "config1": {"desc": "Q4_K dequant-matmul X f16 [15 x 2048] . W[2048 x 2048]^T -> f32, 64 rotating weight copies",
                "kind": "qmatmul"},
    "config2": {"desc": "1 request x 15 tokens (BOS + uniform ids), single stream", "lengths": [15]},
    "config2c16": {"desc": "16 concurrent requests x 15 tokens (one engine micro-batch of 16)", "lengths": [15] * 16},
    "config3": {"desc": "16 requests, lengths U[15,150] (ragged)", "lengths": "ragged16"},
    "config4": {"desc": "16 requests x 1500 tokens (two engine micro-batches of 8)", "lengths": [1500] * 16},
    "config5": {"desc": "1 request x 5000 tokens", "lengths": [5000]},
    "config5c16": {"desc": "16 requests x 5000 tokens (two engine micro-batches of 8)", "lengths": [5000] * 16},
}
FORWARD_WORKLOADS = [k for k, v in WORKLOADS.items() if v.get("kind") != "qmatmul"]
WEIGHTS_PER_LAYER = 54_525_952
CONFIG1_BYTES = 2_359_296 + 15 * 2048 * 2 + 15 * 2048 * 4  # packed weights + X + Y
CONFIG1_COPIES = 64


def workload_lengths(name: str, seed: int) -> list:
    spec = WORKLOADS[name]["lengths"]
    if spec == "ragged16":
        return np.random.default_rng(seed).integers(15, 151, 16).tolist()
    return list(spec)


def merged_len(n: int) -> int:
    return max(1, math.ceil(n * 0.64))


def projection_flops(lengths: list, n_layers: int) -> float:
    """2 * weights * rows per layer over the valid tokens (4 layers at the
    source length, the rest at the merged length)."""
    return sum(2.0 * WEIGHTS_PER_LAYER * (4 * n + (n_layers - 4) * merged_len(n)) for n in lengths)


def kernels_per_forward(n_layers: int, fused: bool, seq: int) -> int:
    if fused:
        return 2  # run metadata + the persistent single-launch forward
    # meta, embedding, first RMSNorm; per layer QKV, attention, O, norm,
    # gate/up, down, norm (RoPE and SwiGLU live in the projection epilogues),
    # plus the compact-key gather in layers whose valid length can exceed 2048;
    # merge; pool.
    gathers = (4 if seq > 2048 else 0) + ((n_layers - 4) if merged_len(seq) > 2048 else 0)
    return 3 + 7 * n_layers + gathers + 2


# DRAM bytes (read + write) per launch of the single-launch forward, from one
# ncu capture of that kernel on this workload (dram__bytes_read.sum +
# dram__bytes_write.sum); null where no capture was taken.
NCU_TRAFFIC = {("config2", "kquant"): 530.1e6}


def measured_peaks() -> dict:
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return {"hbm_gbs": d.get("hbm_gbs"), "bf16_tflops": d.get("bf16_tflops"),
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained") or d.get("bf16_tflops"), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


class NvmlClockSampler:
    """SM clock and clock-event reasons sampled through NVML every ~1 ms by a
    background thread during the timed region (the plan's C calls release the
    GIL). Short timed regions still get samples, unlike nvidia-smi -lms."""

    REASONS = {"hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20, "sw_power_cap": 0x4,
               "hw_power_brake_slowdown": 0x80}

    def __init__(self, gpu_index: int):
        import pynvml
        self.nv = pynvml
        pynvml.nvmlInit()
        self.h = pynvml.nvmlDeviceGetHandleByIndex(gpu_index)
        self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        self.sm, self.bits = [], 0
        self.stop = False
        self.thread = None

    def _sample(self):
        nv = self.nv
        self.sm.append(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM))
        try:
            self.bits |= nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
        except Exception:
            self.bits |= nv.nvmlDeviceGetCurrentClocksThrottleReasons(self.h)

    def _loop(self):
        while not self.stop:
            self._sample()
            time.sleep(0.001)

    def __enter__(self):
        import threading
        self.stop = False
        self.thread = threading.Thread(target=self._loop, daemon=True)
        self.thread.start()
        return self

    def __exit__(self, *exc):
        self.stop = True
        self.thread.join(timeout=5)
        if not self.sm:
            self._sample()

    def summary(self) -> dict:
        reasons = sorted(k for k, v in self.REASONS.items() if self.bits & v)
        return {"sm_mhz": statistics.median(self.sm) if self.sm else None, "sm_max_mhz": self.max_mhz,
                "reasons": reasons, "samples": len(self.sm), "source": "nvml"}


class ClockSampler:
    """nvidia-smi clocks + throttle reasons during the timed region (fallback)."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = os.path.join("/tmp", f"nemo_clocks_{os.getpid()}.csv")

    def __enter__(self):
        try:
            self.out = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "200", "-i", str(self.gpu)], stdout=self.out,
                                         stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.out.close()

    def summary(self) -> dict:
        if not self.proc or not os.path.exists(self.path):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        sm, mx, reasons = [], [], set()
        names = ["active", "hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        with open(self.path) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    sm.append(float(parts[1]))
                    mx.append(float(parts[2]))
                except ValueError:
                    continue
                for name, val in zip(names[1:], parts[5:9]):
                    if val.lower().startswith("active"):
                        reasons.add(name)
        os.unlink(self.path)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def clock_sampler(gpu_index: int):
    try:
        return NvmlClockSampler(gpu_index)
    except Exception:
        return ClockSampler(gpu_index)


def physical_gpu(local_rank: int) -> int:
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        ids = [v for v in vis.split(",") if v.strip()]
        if local_rank < len(ids) and ids[local_rank].strip().isdigit():
            return int(ids[local_rank])
    return local_rank


# ----------------------------------------------------------------------------- CPU side

class CpuOracle:
    """The CPU oracle on the host cores (loaded once, reused by every sample)."""

    def __init__(self, pack_path: str, threads: int | None):
        import oracle
        self.oracle = oracle
        if threads:
            oracle.set_num_threads(threads)
        with open(pack_path, "rb") as f:
            self.model = oracle.OracleModel(f.read())

    def forward_rate(self, lengths: list, seed: int, budget_s: float, label: str) -> dict:
        """req/s of the oracle forward over `lengths` (one batch), repeated for
        about budget_s seconds (at least once)."""
        from nemo_b200 import synth
        reqs = synth.make_requests(seed, lengths, vocab=self.model.vocab)
        ids, lens, seq = synth.pad_batch(reqs)
        n, t0 = 0, time.perf_counter()
        while True:
            self.model.forward(len(lengths), seq, ids, lens)
            n += 1
            el = time.perf_counter() - t0
            if el >= budget_s or n >= 200:
                break
        return {"value": n * len(lengths) / el, "unit": "req/s", "cores": self.oracle.num_threads(), "kind": "port",
                "sample": f"{n} forward(s) of {len(lengths)} request(s) x lengths {sorted(set(lengths))} in "
                          f"{el:.1f} s (CPU oracle, f32){label}"}

    def qmatmul_rate(self, budget_s: float) -> dict:
        from nemo_b200 import synth
        x, w = synth.config1_matrix(seed=1)
        xb = x.view(np.uint16)
        n, t0 = 0, time.perf_counter()
        while True:
            w32 = self.oracle.decode_matrix(w, self.oracle.Q4_K, False, 2048, 2048)
            self.oracle.matmul_f16(xb, w32.astype(np.float16).view(np.uint16))
            n += 1
            el = time.perf_counter() - t0
            if el >= budget_s or n >= 1000:
                break
        per = el / n
        return {"value": CONFIG1_BYTES / per / 1e9, "unit": "GB/s", "matmuls_per_s": 1.0 / per,
                "cores": self.oracle.num_threads(), "kind": "port",
                "sample": f"{n} decode + matmul passes of the config-1 matrix in {el:.1f} s (CPU oracle)"}

    def close(self):
        self.model.close()


# ----------------------------------------------------------------------------- GPU side

def share_of_rank(lengths: list, world: int, rank: int, sharded: bool) -> list:
    """This rank's micro-batches: the engine's micro-batches of the request
    queue, each split across the ranks (longest-first onto the least-loaded
    rank) when sharded."""
    from nemo_b200 import dist as ndist
    from nemo_b200.engine import micro_batches
    out = []
    for mb in micro_batches(lengths):
        mb_lengths = [lengths[i] for i in mb]
        if sharded and world > 1:
            mine = [mb_lengths[i] for i in ndist.shard_requests(mb_lengths, world)[rank]]
        else:
            mine = mb_lengths
        if mine:
            out.append(mine)
    return out


class ForwardRuns:
    """Plans (cached per batch:sequence, like the engine) and resident inputs of
    one rank's micro-batches."""

    def __init__(self, torch, model, batches: list, seed: int):
        from nemo_b200 import synth
        self.torch = torch
        self.plans = {}
        self.runs = []
        for i, lengths in enumerate(batches):
            reqs = synth.make_requests(seed + 17 * i, lengths)
            ids, lens, seq = synth.pad_batch(reqs)
            key = (len(lengths), seq)
            if key not in self.plans:
                self.plans[key] = model.create_plan(len(lengths), seq)
            plan = self.plans[key]
            d_ids = torch.from_numpy(ids.astype(np.int32)).cuda()
            d_lens = torch.from_numpy(lens.astype(np.int32)).cuda()
            d_out = torch.empty((len(lengths), 2048), dtype=torch.float32, device="cuda")
            out = np.empty((len(lengths), 2048), np.float32)
            self.runs.append({"plan": plan, "ids": ids, "lens": lens, "seq": seq, "d_ids": d_ids, "d_lens": d_lens,
                              "d_out": d_out, "out": out, "n": len(lengths)})
        self.streams = {id(p): torch.cuda.ExternalStream(p.stream()) for p in self.plans.values()}

    @property
    def requests(self) -> int:
        return sum(r["n"] for r in self.runs)

    def device_steps(self, steps: int):
        """Enqueues `steps` steps (every micro-batch once per step), serialised
        across the plans' streams; returns (start, end) CUDA events."""
        torch = self.torch
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        if not self.runs:
            return None
        prev = self.streams[id(self.runs[0]["plan"])]
        start.record(prev)
        for _ in range(steps):
            for r in self.runs:
                s = self.streams[id(r["plan"])]
                if s is not prev:
                    ev = torch.cuda.Event()
                    ev.record(prev)
                    s.wait_event(ev)
                    prev = s
                r["plan"].run_device(r["d_ids"].data_ptr(), r["d_lens"].data_ptr(), r["d_out"].data_ptr())
        end.record(prev)
        return start, end

    def synchronize(self):
        for p in self.plans.values():
            p.synchronize()

    def host_steps(self, steps: int):
        for _ in range(steps):
            for r in self.runs:
                r["plan"].run_array(r["ids"], r["lens"], r["out"])

    def profile(self) -> dict:
        """Per-stage device ms of one step (sum over the micro-batches; median of 5)."""
        total = {}
        for r in self.runs:
            prof = [r["plan"].profile(r["ids"], r["lens"]) for _ in range(5)]
            for k in prof[0]:
                total[k] = total.get(k, 0.0) + statistics.median(p[k] for p in prof)
        return total

    def launches_per_step(self, n_layers: int) -> int:
        return sum(kernels_per_forward(n_layers, r["plan"].fused, r["seq"]) for r in self.runs)

    def bytes_per_step(self):
        h2d = sum(r["ids"].nbytes + (r["n"] + 1) * 4 for r in self.runs)
        d2h = sum(r["out"].nbytes + 4 for r in self.runs)
        return h2d, d2h

    def destroy(self):
        for p in self.plans.values():
            p.destroy()


def forward_workload(torch, ndist, rinfo, model, info, name: str, lengths: list, sharded: bool, args,
                     clocks=None) -> dict:
    """Measures one forward workload on this rank; collective steps are taken
    by every rank in the same order."""
    world, rank = rinfo.world, rinfo.rank
    batches = share_of_rank(lengths, world, rank, sharded)
    runs = ForwardRuns(torch, model, batches, args.seed + (0 if sharded else 1000 * rank))
    total_requests = len(lengths) if sharded else world * len(lengths)

    def barrier():
        ndist.barrier(rinfo)
        torch.cuda.synchronize()

    if runs.runs:
        runs.device_steps(args.warmup)
        runs.synchronize()
    barrier()
    ctx = clocks if clocks is not None else _Null()
    with ctx:
        ev = runs.device_steps(args.steps) if runs.runs else None
        runs.synchronize()
        barrier()
    ms = ev[0].elapsed_time(ev[1]) if ev else 0.0
    ms_max = ndist.max_over_ranks(rinfo, ms, "cuda")
    value = total_requests * args.steps / (ms_max / 1e3)

    if runs.runs:
        runs.host_steps(max(1, args.warmup))
    barrier()
    t0 = time.perf_counter()
    if runs.runs:
        runs.host_steps(args.steps)
    e2e_s = ndist.max_over_ranks(rinfo, time.perf_counter() - t0, "cuda")
    e2e = total_requests * args.steps / e2e_s
    h2d, d2h = runs.bytes_per_step() if runs.runs else (0, 0)

    roofline = None
    if runs.runs:
        prof = runs.profile()
        fused = all(r["plan"].fused for r in runs.runs)
        peaks = measured_peaks()
        my_lengths = [n for b in batches for n in b]
        if fused:
            kernel = "forward_fused (persistent single launch: weight stream + dequant + tcgen05 projections)"
            kms = prof["forward_fused"]
        else:
            kernel = "projection GEMMs (qkv, attn_output, ffn_gate_up, ffn_down)"
            kms = prof["qkv"] + prof["attention_output"] + prof["ffn_up_gate"] + prof["ffn_down"]
        if max(sum(b) for b in batches) < 64:
            work = float(info.packed_weight_bytes) * len(batches)
            achieved = work / (kms / 1e3) / 1e9
            roofline = {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                        "frac": achieved / peaks["hbm_gbs"], "peak_source": peaks["source"] + " (copy)"}
        else:
            work = projection_flops(my_lengths, info.n_layers)
            achieved = work / (kms / 1e3) / 1e12
            # timed inside back-to-back forwards of milliseconds under the 1 kW
            # cap: the sustained cuBLAS figure is the denominator
            roofline = {"bound": "tensor", "achieved": achieved, "peak": peaks["bf16_tflops_sustained"],
                        "unit": "TFLOP/s", "frac": achieved / peaks["bf16_tflops_sustained"],
                        "frac_of_burst_peak": achieved / peaks["bf16_tflops"],
                        "peak_source": peaks["source"] + " (sustained bf16 GEMM)"}
        roofline.update({"traffic": NCU_TRAFFIC.get((name, args.pack)) if fused else None, "kernel": kernel,
                         "kernel_ms_per_step": kms, "algorithmic_per_step": work, "stage_ms": prof})
    entry = {"req_s": value, "unit": "req/s", "ms_per_step": ms_max / args.steps, "steps": args.steps,
             "requests_per_step": total_requests, "desc": WORKLOADS[name]["desc"],
             "scaling": "strong" if sharded and world > 1 else "weak",
             "rank0_micro_batches": [len(b) for b in batches], "lengths": sorted(set(lengths)),
             "e2e": {"value": e2e, "unit": "req/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
             "roofline": roofline, "gpu_launches": runs.launches_per_step(info.n_layers) * args.steps,
             "vs_baseline": (value / PUBLISHED[name]) if name in PUBLISHED else None,
             "fused_single_launch": bool(runs.runs) and all(r["plan"].fused for r in runs.runs)}
    runs.destroy()
    return entry


class _Null:
    def __enter__(self):
        return self

    def __exit__(self, *exc):
        return False


def qmatmul_workload(torch, ndist, rinfo, args) -> dict:
    """Config 1 through nemo_op_qmatmul_enqueue: every step sweeps the 64
    rotating copies of the tile-slab image (151 MB, more than the 126 MB L2),
    so each matmul streams its weights from HBM. Rank-local at N > 1."""
    from nemo_b200 import synth
    from nemo_b200.runtime import check, load_library
    L = load_library()
    x, w = synth.config1_matrix(seed=1)
    n = k = 2048
    m = 15
    nbytes = L.nemo_op_qmatmul_image_bytes(0, n, k)
    images = torch.empty((CONFIG1_COPIES, nbytes), dtype=torch.uint8, device="cuda")
    d_w = torch.from_numpy(w).cuda()
    for c in range(CONFIG1_COPIES):
        check(L.nemo_op_qmatmul_image(0, d_w.data_ptr(), n, k, images[c].data_ptr()))
    d_x = torch.from_numpy(x).cuda()
    d_y = torch.empty((m, n), dtype=torch.float32, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    stream = torch.cuda.Stream()
    sp = stream.cuda_stream

    def sweep(reps):
        for _ in range(reps):
            for c in range(CONFIG1_COPIES):
                check(L.nemo_op_qmatmul_enqueue(0, images[c].data_ptr(), d_x.data_ptr(), m, n, k, d_y.data_ptr(),
                                                err.data_ptr(), sp))

    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        sweep(1)  # first calls set the kernels' attributes (not capturable)
    stream.synchronize()
    # One sweep captured as a CUDA graph (64 launches chained by programmatic
    # dependent launch): the timed region is device time, not the host's rate
    # of issuing launches through ctypes.
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        cap = torch.cuda.current_stream().cuda_stream
        for c in range(CONFIG1_COPIES):
            check(L.nemo_op_qmatmul_enqueue(0, images[c].data_ptr(), d_x.data_ptr(), m, n, k, d_y.data_ptr(),
                                            err.data_ptr(), cap))
    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            graph.replay()
    stream.synchronize()
    ndist.barrier(rinfo)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        start.record(stream)
        for _ in range(args.steps):
            graph.replay()
        end.record(stream)
    stream.synchronize()
    ms = ndist.max_over_ranks(rinfo, start.elapsed_time(end), "cuda")
    launches = args.steps * CONFIG1_COPIES
    per_s = ms / 1e3 / launches
    peaks = measured_peaks()
    achieved = CONFIG1_BYTES / per_s / 1e9
    # end to end: X from pinned host memory in, Y back to pinned host memory
    h_x = torch.from_numpy(x).pin_memory()
    h_y = torch.empty((m, n), dtype=torch.float32).pin_memory()
    calls = args.steps * 8
    with torch.cuda.stream(stream):
        t0 = time.perf_counter()
        for i in range(calls):
            d_x.copy_(h_x, non_blocking=True)
            check(L.nemo_op_qmatmul_enqueue(0, images[i % CONFIG1_COPIES].data_ptr(), d_x.data_ptr(), m, n, k,
                                            d_y.data_ptr(), err.data_ptr(), sp))
            h_y.copy_(d_y, non_blocking=True)
            stream.synchronize()
        e2e_s = time.perf_counter() - t0
    e2e_s = ndist.max_over_ranks(rinfo, e2e_s, "cuda")
    ok = int(err.item()) == 0
    del graph, images
    return {"matmuls_per_s": rinfo.world / per_s, "unit": "matmul/s", "us_per_matmul": per_s * 1e6,
            "steps": args.steps, "matmuls_per_step": CONFIG1_COPIES, "desc": WORKLOADS["config1"]["desc"],
            "scaling": "weak", "bounded_waits_ok": ok,
            "l2": "64 distinct weight images (151 MB) swept in turn: each matmul reads its weights from HBM",
            "e2e": {"value": rinfo.world * calls / e2e_s, "unit": "matmul/s", "h2d_bytes_per_step": x.nbytes,
                    "d2h_bytes_per_step": h_y.numel() * 4, "calls": calls},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": achieved / peaks["hbm_gbs"], "traffic": None,
                         "kernel": "skinny_kernel<16> (fused-dequant split-K tcgen05 projection), f32 store",
                         "algorithmic_bytes_per_matmul": CONFIG1_BYTES, "peak_source": peaks["source"] + " (copy)"},
            "gpu_launches": launches}


def head_parallel_workload(ndist, rinfo, pack: str, args, single_req_s) -> dict | None:
    """config5hp: one 5000-token request head-parallel over all N GPUs of the
    box (token-sharded projections; the QKV and attention epilogues store into
    the devices owning each head group / token row over NVLink peer memory), from
    rank 0's process through nemo_plan_run with host buffers. The other ranks
    wait on a host-only barrier meanwhile. Every rank takes the same barriers."""
    from nemo_b200 import synth
    from nemo_b200.runtime import NemotronB200Model
    world, rank = rinfo.world, rinfo.rank
    ndist.cpu_barrier(rinfo)
    entry = None
    if rank == 0:
        try:
            model = NemotronB200Model(pack, devices=list(range(world)))
        except Exception as e:  # recorded, and every rank still takes the barrier below
            model, entry = None, {"error": f"{type(e).__name__}: {e}", "n_devices": world}
    if rank == 0 and model is not None:
        try:
            reqs = synth.make_requests(args.seed, [5000])
            ids, lens, seq = synth.pad_batch(reqs)
            plan = model.create_plan(1, seq)
            assert plan.head_parallel_min and plan.head_parallel_min <= 5000
            out = np.empty((1, 2048), np.float32)
            for _ in range(args.warmup):
                plan.run_array(ids, lens, out)
            t0 = time.perf_counter()
            for _ in range(args.steps):
                plan.run_array(ids, lens, out)
            el = time.perf_counter() - t0
            value = args.steps / el
            entry = {"req_s": value, "unit": "req/s", "ms_per_step": el / args.steps * 1e3, "steps": args.steps,
                     "n_devices": world, "desc": "1 request x 5000 tokens, head-parallel over all GPUs (one process)",
                     "scaling": "strong",
                     "timing": "host wall clock around nemo_plan_run (H2D ids, D2H embedding inside every step)",
                     "single_device_req_s": single_req_s,
                     "speedup_vs_single_device": (value / single_req_s) if single_req_s else None,
                     "e2e": {"value": value, "unit": "req/s", "h2d_bytes_per_step": ids.nbytes + 4,
                             "d2h_bytes_per_step": out.nbytes}}
        except Exception as e:  # a failed run (bounded by the plan's host deadline) is recorded
            entry = {"error": f"{type(e).__name__}: {e}", "n_devices": world}
        finally:
            model.destroy()
    ndist.cpu_barrier(rinfo)
    return entry


def headline_config(name: str, args, n_layers: int, lengths: list, world: int) -> dict:
    """The `config` of the headline line (shared by both arms)."""
    seq = max(lengths)
    return {"workload": f"{name}: {WORKLOADS[name]['desc']}", "pack": args.pack, "layers": n_layers,
            "batch": len(lengths), "seq": seq, "tokens_per_step": sum(lengths),
            "l2": "no flush: every step streams all projection weights (>= 0.49 GB, > 126 MB L2)",
            "parallelism": f"request-sharded replicas x{world} (no data-path collective)"}


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from nemo_b200 import synth

    pack = synth.cached_model_pack(0, args.pack, 16)
    lengths = workload_lengths(args.workload, args.seed)
    threads = os.cpu_count()
    import oracle

    oracle.set_num_threads(threads)
    with open(pack, "rb") as f:
        data = f.read()
    model = oracle.OracleModel(data)
    # one bounded sample per step: the first request(s) of the workload's batch
    sample = lengths[:1] if max(lengths) >= 500 else lengths
    reqs = synth.make_requests(args.seed, sample, vocab=model.vocab)
    ids, lens, seq = synth.pad_batch(reqs)
    for _ in range(args.warmup):
        model.forward(len(sample), seq, ids, lens)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        model.forward(len(sample), seq, ids, lens)
    el = time.perf_counter() - t0
    value = args.steps * len(sample) / el
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "req/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": el / args.steps * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded random-init Q4_K_M-mix weights of the Nemotron-3-Embed-1B architecture, "
                    "BOS + uniform ids)",
            "config": headline_config(args.workload, args, 16, lengths, args.gpus),
            "cpu_baseline": {"value": value, "unit": "req/s", "cores": threads, "kind": "port",
                             "sample": f"{args.steps} forwards of {len(sample)} request(s); the reference is "
                                       "TypeScript + WGSL with no runnable CPU forward here, so its CPU path is "
                                       "the C++ oracle restating its decode code and shader math"},
            "e2e": {"value": value, "unit": "req/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_ours(args) -> None:
    import torch

    from nemo_b200 import dist as ndist
    from nemo_b200 import synth
    from nemo_b200.runtime import NemotronB200Model

    rinfo = ndist.rank_info()
    world, rank, local = rinfo.world, rinfo.rank, rinfo.local_rank
    torch.cuda.set_device(local)
    ndist.init("nccl", 300.0, torch.device("cuda", local))

    pack = synth.cached_model_pack(0, args.pack, 16)
    model = NemotronB200Model(pack, devices=[local])
    info = model.info()

    # --- headline: config 2 per rank (weak scaling of independent streams) ----
    lengths = workload_lengths(args.workload, args.seed + rank)
    clocks = clock_sampler(physical_gpu(local))
    head = forward_workload(torch, ndist, rinfo, model, info, args.workload, lengths, False, args, clocks=clocks)

    # --- every other workload ------------------------------------------------
    wanted = FORWARD_WORKLOADS + ["config1"] if args.workloads == "all" else (
        [] if args.workloads == "none" else args.workloads.split(","))
    workloads = {}
    for name in ["config1"] + FORWARD_WORKLOADS:
        if name not in wanted or name == args.workload:
            continue
        if name == "config1":
            workloads[name] = qmatmul_workload(torch, ndist, rinfo, args)
        else:
            workloads[name] = forward_workload(torch, ndist, rinfo, model, info, name,
                                               workload_lengths(name, args.seed), True, args)
    model.destroy()

    # --- one long request head-parallel over every GPU (N = 2, 4, 8) ---------
    if world in (2, 4, 8) and (args.workloads == "all" or "config5hp" in args.workloads.split(",")):
        single = workloads.get("config5", {}).get("req_s")
        hp = head_parallel_workload(ndist, rinfo, pack, args, single)
        if hp is not None:
            workloads["config5hp"] = hp

    # --- CPU samples (rank 0, N = 1 only) -------------------------------------
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        orc = CpuOracle(pack, None)
        cpu = orc.forward_rate(lengths, args.seed, args.cpu_budget, "")
        samples = {}  # one sample per distinct request set (config5 and config5c16 share theirs)
        for name, entry in workloads.items():
            if name == "config1":
                entry["cpu_baseline"] = orc.qmatmul_rate(3.0)
                continue
            wl = workload_lengths(name, args.seed)
            if max(wl) >= 1000:
                sample, budget, note = wl[:1], 0.0, "; 1 request of the workload, req/s extrapolated"
            elif name == "config3":
                sample, budget, note = wl[:2], 4.0, "; the first 2 requests, req/s extrapolated"
            else:
                sample, budget, note = wl, 4.0, ""
            key = tuple(sample)
            if key not in samples:
                samples[key] = orc.forward_rate(sample, args.seed, budget, note)
            entry["cpu_baseline"] = samples[key]
        orc.close()
    ndist.shutdown(rinfo)
    if rank != 0:
        return
    line = {"metric": METRIC, "value": head["req_s"], "unit": "req/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": head["ms_per_step"], "higher_is_better": True, "scaling": "weak",
            "vs_baseline": head["vs_baseline"], "dtype": "f16",
            "data": "synthetic (seeded random-init Q4_K_M-mix weights of the Nemotron-3-Embed-1B architecture, "
                    "BOS + uniform ids)",
            "config": headline_config(args.workload, args, info.n_layers, lengths, world),
            "roofline": head["roofline"],
            "cpu_baseline": cpu,
            "e2e": head["e2e"],
            "clocks": clocks.summary(),
            "gpu_launches": head["gpu_launches"],
            "workloads": workloads}
    line["roofline"]["kernel_ms_per_forward"] = line["roofline"]["kernel_ms_per_step"]
    print(json.dumps(line), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=FORWARD_WORKLOADS, default="config2")
    ap.add_argument("--workloads", default="all", help="all, none, or a comma-separated list")
    ap.add_argument("--pack", choices=["kquant", "q40"], default="kquant")
    ap.add_argument("--seed", type=int, default=20)
    ap.add_argument("--cpu-budget", type=float, default=10.0)
    ap.add_argument("--no-cpu", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
