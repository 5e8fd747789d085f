#!/usr/bin/env python
"""Benchmark of the B200 Nemotron-3-Embed-1B encoder (driver contract).

python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload NAME]

One "step" is one forward pass (NemotronExecutionPlan.run) over one
micro-batch of synthetic requests. Default workload: config 2 of the
reference's headline metric (1 request of 15 tokens, BOS + uniform ids, full
16-layer random-init Q4_K_M-mix encoder). Under torchrun each rank drives its
own GPU with a full weight replica (request sharding, no collective on the
data path; the only collectives are the timing barrier and the max-over-ranks
reduction).

  value  requests/s over all ranks, inputs resident in HBM (device timing with
         CUDA events on the plan's stream, max over ranks)
  e2e    the same metric through the public C ABI (nemo_plan_run) with host
         buffers: H2D ids/lengths and D2H embeddings inside every step
  roofline  projection GEMM stages (CUDA events per stage, nemo_plan_profile)
         against the measured HBM copy bandwidth, counting the algorithmic
         packed weight bytes per forward
  cpu_baseline  the CPU oracle (restatement of the reference's CPU decode and
         WGSL math) on the host cores, rank 0, bounded sample

--impl reference times the reference's CPU path (the oracle port: the
reference is TypeScript/WGSL and cannot run on this box) on the host cores.
"""
import argparse
import json
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
# the reference's published single-stream 15-token figure (Apple M3 Max, WebGPU).
# the reference's published figures for the same workloads
# (Apple M3 Max, WebGPU): single-stream 15 and 5,000 tokens, 16-concurrent
# 15 tokens (native batch 16) and 1,500 tokens (native batch 8).
PUBLISHED = {"config2": 69.68, "config5": 0.76, "config2c16": 266.02, "config4": 2.75}

WORKLOADS = {
    "config2": {"desc": "1 request x 15 tokens (BOS + uniform ids), single stream", "lengths": [15]},
    "config2c16": {"desc": "16 concurrent requests x 15 tokens (one engine micro-batch of 16)", "lengths": [15] * 16},
    "config3": {"desc": "16 requests, lengths U[15,150] (ragged)", "lengths": "ragged16"},
    "config4": {"desc": "8 requests x 1500 tokens (one engine micro-batch: the engine caps >=1500-token batches at 8)",
                "lengths": [1500] * 8},
    "config5": {"desc": "1 request x 5000 tokens", "lengths": [5000]},
}


def workload_lengths(name: str, seed: int) -> list:
    spec = WORKLOADS[name]["lengths"]
    if spec == "ragged16":
        return np.random.default_rng(seed).integers(15, 151, 16).tolist()
    return list(spec)


def kernels_per_forward(n_layers: int, fused: bool, seq: int) -> int:
    if fused:
        return 2  # run metadata + the persistent single-launch forward
    # meta, embedding, first RMSNorm; per layer QKV, attention, O, norm,
    # gate/up, down, norm (RoPE and SwiGLU live in the projection epilogues),
    # plus the compact-key gather in layers whose valid length can exceed 2048;
    # merge; pool.
    merged_seq = synth_merged(seq)
    gathers = (4 if seq > 2048 else 0) + ((n_layers - 4) if merged_seq > 2048 else 0)
    return 3 + 7 * n_layers + gathers + 2


# DRAM bytes (read + write) per launch of the single-launch forward, from one
# ncu capture of that kernel on this workload (dram__bytes.sum.per_second x
# gpu__time_duration.sum); null where no capture was taken.
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


def clock_sampler(gpu_index: int):
    try:
        return NvmlClockSampler(gpu_index)
    except Exception:
        return ClockSampler(gpu_index)


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


def physical_gpu(local_rank: int) -> int:
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        ids = [v for v in vis.split(",") if v.strip()]
        if local_rank < len(ids) and ids[local_rank].strip().isdigit():
            return int(ids[local_rank])
    return local_rank


def cpu_forward_rate(pack_path: str, lengths: list, seed: int, budget_s: float, threads: int | None,
                     max_requests: int | None = None) -> dict:
    """Times the CPU oracle forward on the host cores (bounded sample)."""
    import oracle
    from nemo_b200 import synth

    if threads:
        oracle.set_num_threads(threads)
    with open(pack_path, "rb") as f:
        data = f.read()
    model = oracle.OracleModel(data)
    sample = lengths if max_requests is None else lengths[:max_requests]
    reqs = synth.make_requests(seed, sample, vocab=model.vocab)
    ids, lens, seq = synth.pad_batch(reqs)
    model.forward(len(sample), seq, ids, lens)  # warm
    n, t0 = 0, time.perf_counter()
    while True:
        model.forward(len(sample), seq, ids, lens)
        n += 1
        el = time.perf_counter() - t0
        if el >= budget_s or n >= 200:
            break
    model.close()
    return {"value": n * len(sample) / el, "unit": "req/s", "cores": oracle.num_threads(), "kind": "port",
            "sample": f"{n} forwards of {len(sample)} request(s) x lengths {sorted(set(sample))} "
                      f"in {el:.1f} s (CPU oracle, f32)"}


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
            "data": "synthetic (seeded random-init Q4_K_M-mix weights, BOS + uniform ids)",
            "config": {"workload": f"{args.workload}: {WORKLOADS[args.workload]['desc']}", "pack": args.pack,
                       "sample": f"{len(sample)} request(s) per step"},
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

    def barrier():
        ndist.barrier(rinfo)
        torch.cuda.synchronize()

    def max_over_ranks(v: float) -> float:
        return ndist.max_over_ranks(rinfo, v, "cuda")

    pack = synth.cached_model_pack(0, args.pack, 16)
    lengths = workload_lengths(args.workload, args.seed + rank)
    batch = len(lengths)
    reqs = synth.make_requests(args.seed + 1000 * rank, lengths)
    ids, lens, seq = synth.pad_batch(reqs)
    model = NemotronB200Model(pack, devices=[local])
    info = model.info()
    plan = model.create_plan(batch, seq)

    # --- device-resident timing (value) -------------------------------------
    d_ids = torch.from_numpy(ids.astype(np.int32)).cuda()
    d_lens = torch.from_numpy(lens.astype(np.int32)).cuda()
    d_out = torch.empty((batch, 2048), dtype=torch.float32, device="cuda")
    stream = torch.cuda.ExternalStream(plan.stream())
    torch.cuda.synchronize()
    for _ in range(args.warmup):
        plan.run_device(d_ids.data_ptr(), d_lens.data_ptr(), d_out.data_ptr())
    plan.synchronize()
    barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with clock_sampler(physical_gpu(local)) as clocks:
        start.record(stream)
        for _ in range(args.steps):
            plan.run_device(d_ids.data_ptr(), d_lens.data_ptr(), d_out.data_ptr())
        end.record(stream)
        plan.synchronize()
        barrier()
    ms = start.elapsed_time(end)
    ms_max = max_over_ranks(ms)
    value = ndist.throughput(world, args.steps, batch, ms_max / 1e3)

    # --- end to end through the C ABI with host buffers (e2e) ----------------
    out = np.empty((batch, 2048), np.float32)
    for _ in range(max(1, args.warmup)):
        plan.run_array(ids, lens, out)
    barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        plan.run_array(ids, lens, out)
    e2e_s = max_over_ranks(time.perf_counter() - t0)
    e2e = ndist.throughput(world, args.steps, batch, e2e_s)
    h2d = ids.nbytes + (batch + 1) * 4
    d2h = out.nbytes + 4

    # --- roofline of the projection GEMMs (per-stage CUDA events) ------------
    stages = []
    for _ in range(5):
        stages.append(plan.profile(ids, lens))
    prof = {k: statistics.median(s[k] for s in stages) for k in stages[0]}
    fused = plan.fused
    if fused:
        kernel = "forward_fused (persistent single launch: weight stream + dequant + tcgen05 projections)"
        gemm_ms = prof["forward_fused"]
    else:
        kernel = "projection GEMMs (qkv, attn_output, ffn_gate_up, ffn_down)"
        gemm_ms = prof["qkv"] + prof["attention_output"] + prof["ffn_up_gate"] + prof["ffn_down"]
    peaks = measured_peaks()
    tokens = sum(lengths)
    if tokens < 64:
        bound, unit = "hbm", "GB/s"
        work = float(info.packed_weight_bytes)
        achieved = work / (gemm_ms / 1e3) / 1e9
        peak = peaks["hbm_gbs"]
    else:
        merged = sum(synth_merged(l) for l in lengths)
        flops = 2.0 * 54_525_952 * (4 * tokens + (info.n_layers - 4) * merged)
        bound, unit, work = "tensor", "TFLOP/s", flops
        achieved = flops / (gemm_ms / 1e3) / 1e12
        # The projection GEMMs are timed inside back-to-back forwards of many
        # milliseconds (a long step under the 1 kW cap), so the denominator is
        # the sustained cuBLAS figure; the burst fraction is reported beside it.
        peak = peaks["bf16_tflops_sustained"]
    roofline = {"bound": bound, "achieved": achieved, "peak": peak, "unit": unit, "frac": achieved / peak,
                "traffic": NCU_TRAFFIC.get((args.workload, args.pack)) if fused else None, "kernel": kernel,
                "kernel_ms_per_forward": gemm_ms, "algorithmic_per_forward": work,
                "peak_source": peaks["source"] + (" (sustained bf16 GEMM)" if bound == "tensor" else " (copy)"),
                "stage_ms": prof}
    if bound == "tensor":
        roofline["frac_of_burst_peak"] = achieved / peaks["bf16_tflops"]

    plan.destroy()
    model.destroy()
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_forward_rate(pack, lengths, args.seed, args.cpu_budget, None,
                               max_requests=1 if max(lengths) >= 500 else None)
    ndist.shutdown(rinfo)
    if rank != 0:
        return
    line = {"metric": METRIC, "value": value, "unit": "req/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_max / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": (value / PUBLISHED[args.workload]) if args.workload in PUBLISHED else None,
            "dtype": "f16",
            "data": "synthetic (seeded random-init Q4_K_M-mix weights of the Nemotron-3-Embed-1B architecture, "
                    "BOS + uniform ids)",
            "config": {"workload": f"{args.workload}: {WORKLOADS[args.workload]['desc']}", "pack": args.pack,
                       "layers": info.n_layers, "batch": batch, "seq": seq, "tokens_per_step": tokens,
                       "l2": "no flush: every step streams all projection weights (>= 0.49 GB, > 126 MB L2)",
                       "parallelism": f"request-sharded replicas x{world} (no data-path collective)"},
            "roofline": roofline,
            "cpu_baseline": cpu,
            "e2e": {"value": e2e, "unit": "req/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
            "clocks": clocks.summary(),
            "gpu_launches": kernels_per_forward(info.n_layers, fused, seq) * args.steps}
    print(json.dumps(line), flush=True)


def synth_merged(n: int) -> int:
    import math
    return max(1, math.ceil(n * 0.64))


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="config2")
    ap.add_argument("--pack", choices=["kquant", "q40"], default="kquant")
    ap.add_argument("--seed", type=int, default=20)
    ap.add_argument("--cpu-budget", type=float, default=12.0)
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
