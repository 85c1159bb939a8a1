#!/usr/bin/env python
"""bench.py -- benchmark of the B200 attention path (one JSON line on rank 0).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload NAME]

Headline workload (the largest case): Qwen3-8B-shaped GQA prefill,
Hq=32, Hkv=8, D=128, Sq=Sk=4096, non-causal, Q/K/V ~ N(0,1) seed 1 in bf16. A step is one
attn_flash call over one sequence (batch 1 per GPU). Under torchrun each rank runs its own
sequence -- the prefill shards by (batch x kv-head group) with no collective -- so the
scaling is weak and `value` is the whole job's TFLOP/s.

Keys of the JSON line beyond the base contract:
  roofline      dominant kernel's achieved TFLOP/s (algorithmic FLOPs / CUDA-event time per
                launch) against the measured bf16 peak in MEASURED_PEAKS.json, plus its DRAM
                traffic per launch from the committed ncu summary (profiles/traffic.json)
  cpu_baseline  the reference's own flash.c (oracle/_ref, compiled natively through the SVE
                shim) timed on this host's cores on a bounded sample of the same workload
  e2e           the same metric through the C ABI with pinned host buffers: every step copies
                Q, K, V host->device and O device->host inside the timed region; three CUDA
                streams take turns (--e2e-lanes), so one step's readback overlaps the next upload
  causal_prefill  the headline prefill with causal masking on the same buffers (useful FLOPs)
  decode        a secondary HBM-bound line: BASELINE config 3 (GQA decode, B=64, Sk=8192), per GPU
  paged_decode  the same decode through attn_flash_paged_stream (64-key pages, shuffled table)
  qkv_rope      the producer upstream of the path (attn_qkv_rope_stream: QKV split, q/k RMSNorm,
                RoPE, cache write) at the config 5 prefill shape, HBM GB/s
  long_decode  BASELINE config 5 decode (B=4, Hq=64, Hkv=8, Sk=131072) with the key axis split
                over all ranks: partial attention per rank, merged either by one NCCL all-gather
                of packed (m, l, acc) blocks and a combine, or by the peer-store merge kernel over
                NVLink; the value is the faster of the two at the rank count (both are reported)
  sharded_prefill  BASELINE config 5 prefill (B=4, Hq=64, Hkv=8, Sq=Sk=16384) as ONE problem whose
                32 (batch x kv-head group) units are split over the ranks (multigpu.sharded_prefill,
                no collective): strong scaling, `value` = the whole problem's FLOPs / max-rank time
  configs       every other BASELINE config on each GPU (config 2 at S=1024 and S=2048, config 4
                MQA prefill B=8 and decode B=128), device-timed, each with its roofline fraction
  gpu_launches  kernels the library launched inside the timed region (its own counter)
  clocks        SM clocks / throttle reasons sampled by NVML during the timed region

--impl reference times the reference's CPU implementation of the path (oracle/_ref when
present, else the oracle restatement) with all host threads on a bounded sample per step; under
torchrun only rank 0 runs it.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import sys
import threading
import time
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

METRIC = "attn TFLOP/s (prefill) and KV GB/s (decode) per GPU, % of roofline, 1/2/4/8"
L2_BYTES = 126 * 1024 * 1024

WORKLOADS = {
    # name: (Hq, Hkv, Sq, Sk, D, causal, dist, seed, dist args, description)
    "qwen3_gqa_prefill_s4096": (32, 8, 4096, 4096, 128, 0, "normal", 1, (0.0, 1.0),
                                "BASELINE config 2: Qwen3-8B-shaped GQA prefill Hq32/Hkv8 D128 Sq=Sk=4096 non-causal"),
    "qwen3_gqa_prefill_s2048": (32, 8, 2048, 2048, 128, 0, "normal", 1, (0.0, 1.0),
                                "BASELINE config 2 at Sq=Sk=2048"),
    "qwen3_gqa_prefill_s1024": (32, 8, 1024, 1024, 128, 0, "normal", 1, (0.0, 1.0),
                                "BASELINE config 2 at Sq=Sk=1024"),
    "qwen3_gqa_prefill_s4096_causal": (32, 8, 4096, 4096, 128, 1, "normal", 1, (0.0, 1.0),
                                       "BASELINE config 2 shape at S=4096 with causal masking (useful FLOPs)"),
    "mqa_prefill_b8_s2048": (8 * 16, 8, 2048, 2048, 128, 0, "uniform", 3, (-2.0, 2.0),
                             "BASELINE config 4 prefill: MQA 16/1 D128 batch 8 Sq=Sk=2048"),
    "long_prefill_b4_s16384": (4 * 64, 4 * 8, 16384, 16384, 128, 0, "normal", 4, (0.0, 0.5),
                               "BASELINE config 5 prefill: GQA 64/8 D128 batch 4 Sq=Sk=16384, N(0,0.5); "
                               "one GPU runs every kv-head group (the multi-GPU run shards them)"),
    "gqa_decode_b64_sk8192": (64 * 32, 64 * 8, 1, 8192, 128, 0, "normal", 2, (0.0, 1.0),
                              "BASELINE config 3: GQA decode B64 Hq32/Hkv8 D128 Sq=1 Sk=8192"),
    "mqa_decode_b128_sk4096": (128 * 16, 128, 1, 4096, 128, 0, "uniform", 3, (-2.0, 2.0),
                               "BASELINE config 4 decode: MQA 16/1 D128 batch 128 Sq=1 Sk=4096"),
}
DEFAULT_WORKLOAD = "qwen3_gqa_prefill_s4096"


def flops(Hq, Sq, Sk, D, causal) -> float:
    """4 * Hq * D * pairs (flash.c:1149 with attn_pairs, flash.c:874-887)."""
    if not causal:
        pairs = float(Sq) * Sk
    else:
        i = np.arange(Sq, dtype=np.float64)
        pairs = float(np.clip(Sk - Sq + i + 1, 0, Sk).sum())
    return 4.0 * Hq * D * pairs


def algo_bytes(Hq, Hkv, Sq, Sk, D) -> float:
    """Q, K, V read once in bf16 and O written once in fp32."""
    return 2.0 * Hq * Sq * D + 2.0 * 2.0 * Hkv * Sk * D + 4.0 * Hq * Sq * D


def is_decode(w) -> bool:
    return w[2] == 1


def pool_copies(w) -> tuple[int, int]:
    """(copies, bytes per copy) of the rotating input/output pool: enough Q/K/V/O sets to cover
    twice the L2, so that every timed step reads its inputs from HBM."""
    Hq, Hkv, Sq, Sk, D = w[:5]
    set_bytes = 2 * Hq * Sq * D + 2 * 2 * Hkv * Sk * D + 4 * Hq * Sq * D
    return max(1, -(-2 * L2_BYTES // set_bytes)), set_bytes


def config_dict(name: str, w, world: int) -> dict:
    """The `config` of the JSON line; both arms print the same one for the same workload."""
    Hq, Hkv, Sq, Sk, D, causal = w[:6]
    ncopy, set_bytes = pool_copies(w)
    return {"workload": name, "global_batch": world, "seq_len": Sq, "Hq": Hq, "Hkv": Hkv, "head_dim": D,
            "causal": bool(causal),
            "parallelism": f"dp{world} (one sequence per GPU, sharded by batch x kv-head group, no collective)",
            "l2": f"rotating pool of {ncopy} Q/K/V/O sets ({ncopy * set_bytes / 2**20:.0f} MiB >= 2x L2)"}


def host_inputs(w):
    import oracle

    Hq, Hkv, Sq, Sk, D, causal, dist, seed, (a, b), _ = w
    return oracle.seeded_inputs(Hq, Hkv, Sq, Sk, D, seed=seed, dist=dist, a=a, b=b)


def load_peaks() -> dict:
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained"), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


def load_traffic(workload: str):
    p = REPO / "profiles" / "traffic.json"
    if not p.exists():
        return None
    d = json.loads(p.read_text())
    e = d.get(workload)
    return None if e is None else e.get("dram_bytes_per_launch")


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """Polls SM clock and throttle reasons with NVML in a background thread."""

    REASONS = {
        "gpu_idle": 0x1, "applications_clocks_setting": 0x2, "sw_power_cap": 0x4, "hw_slowdown": 0x8,
        "sync_boost": 0x10, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40,
        "hw_power_brake_slowdown": 0x80, "display_clock_setting": 0x100,
    }

    def __init__(self, index: int):
        self.samples = []
        self.ok = False
        self.max_mhz = None
        try:
            import pynvml

            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception:  # noqa: BLE001 -- clocks are reported as unavailable
            self.ok = False
        self._stop = threading.Event()

    def _run(self):
        while not self._stop.is_set():
            try:
                mhz = self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM)
                rs = self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                pw = self.nv.nvmlDeviceGetPowerUsage(self.h) / 1000.0
                self.samples.append((time.perf_counter(), mhz, rs, pw))
            except Exception:  # noqa: BLE001
                pass
            time.sleep(0.002)

    def start(self):
        if self.ok:
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()

    def stop(self):
        if self.ok:
            self._stop.set()
            self.t.join()

    def summary(self, t0: float, t1: float) -> dict:
        if not self.ok or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0}
        inside = [s for s in self.samples if t0 <= s[0] <= t1]
        if not inside:  # region shorter than one poll: take the sample nearest its middle
            mid = 0.5 * (t0 + t1)
            inside = [min(self.samples, key=lambda s: abs(s[0] - mid))]
        mhz = sorted(s[1] for s in inside)
        bits = 0
        for s in inside:
            bits |= s[2]
        reasons = [k for k, v in self.REASONS.items() if bits & v and k != "gpu_idle"]
        pw = sorted(s[3] for s in inside)
        return {"sm_mhz": mhz[len(mhz) // 2], "sm_max_mhz": self.max_mhz, "reasons": reasons,
                "power_w_median": pw[len(pw) // 2], "samples": len(inside)}


# ------------------------------------------------------------------ CPU reference timing
def cpu_reference_sample(w, seconds: float, threads: int | None = None) -> dict:
    """Times the reference's own flash.c (oracle/_ref) -- or the oracle restatement when the
    reference build is absent -- on a bounded sample of workload w: each host thread runs
    attn_flash on its own (head, row-slice) with the workload's full key length. Non-causal
    rows are independent, so a row slice is the same computation as in the full problem."""
    import oracle

    Hq, Hkv, Sq, Sk, D, causal, *_ = w
    group = Hq // Hkv
    threads = threads or os.cpu_count() or 1
    use_ref = oracle.ref_available(128)
    kind = "reference" if use_ref else "port"
    Q, K, V = host_inputs(w)
    rows = max(1, min(Sq, 8))

    def task(t: int, nrows: int) -> float:
        h = t % Hq
        kv = h // group
        r0 = (t * 97) % max(1, Sq - nrows + 1)
        q = np.ascontiguousarray(Q.reshape(Hq, Sq, D)[h, r0:r0 + nrows])
        k = np.ascontiguousarray(K.reshape(Hkv, Sk, D)[kv])
        v = np.ascontiguousarray(V.reshape(Hkv, Sk, D)[kv])
        if use_ref:
            oracle.ref_attn_flash(q, k, v, 1, 1, nrows, Sk, D, causal, bk=128, bq=128)
        else:
            oracle.attn_blocked(q, k, v, 1, 1, nrows, Sk, D, causal, bk=128, bq=128, nthreads=1)
        return flops(1, nrows, Sk, D, causal)

    # calibrate the slice so that the timed sample takes ~`seconds`
    t0 = time.perf_counter()
    task(0, rows)
    one = max(time.perf_counter() - t0, 1e-4)
    rows = int(max(1, min(Sq, rows * seconds / one / 4)))
    with ThreadPoolExecutor(max_workers=threads) as ex:
        t0 = time.perf_counter()
        fl = sum(ex.map(lambda t: task(t, rows), range(threads * 4)))
        dt = time.perf_counter() - t0
    return {"value": fl / dt / 1e12, "unit": "TFLOP/s", "cores": threads, "kind": kind,
            "sample": f"{threads * 4} tasks of 1 head x {rows} query rows x Sk={Sk} (D={D}) on {threads} threads, "
                      f"{dt:.1f} s; non-causal rows are independent so a row slice is the full problem's work per row",
            "seconds": dt}


def cpu_attn_ref_sample(w, seconds: float, threads: int | None = None) -> dict:
    """Times the reference's fp32 reference attention (attn_ref, flash.c:262-314) compiled
    natively from the reference sources (oracle/_ref; the bit-exact restatement when that build
    is absent) on a bounded sample of workload w, one (head, row-slice) per task, all host
    threads. Its work is counted in the same unit as the kernel's (4 * D FLOPs per query-key
    pair), so the two CPU figures compare directly."""
    import oracle

    Hq, Hkv, Sq, Sk, D, causal, *_ = w
    group = Hq // Hkv
    threads = threads or os.cpu_count() or 1
    use_ref = oracle.ref_available(128)
    Q, K, V = host_inputs(w)
    rows = max(1, min(Sq, 4))

    def task(t: int, nrows: int) -> float:
        h = t % Hq
        kv = h // group
        r0 = (t * 97) % max(1, Sq - nrows + 1)
        q = np.ascontiguousarray(Q.reshape(Hq, Sq, D)[h, r0:r0 + nrows])
        k = np.ascontiguousarray(K.reshape(Hkv, Sk, D)[kv])
        v = np.ascontiguousarray(V.reshape(Hkv, Sk, D)[kv])
        idx = np.arange(nrows, dtype=np.int32)
        if use_ref:
            oracle.ref_attn_ref(q, k, v, 1, 1, nrows, Sk, D, causal, idx)
        else:
            oracle.attn_ref(q, k, v, 1, 1, nrows, Sk, D, causal, idx)
        return flops(1, nrows, Sk, D, causal)

    t0 = time.perf_counter()
    task(0, rows)
    one = max(time.perf_counter() - t0, 1e-4)
    rows = int(max(1, min(Sq, rows * seconds / one / 4)))
    with ThreadPoolExecutor(max_workers=threads) as ex:
        t0 = time.perf_counter()
        fl = sum(ex.map(lambda t: task(t, rows), range(threads * 4)))
        dt = time.perf_counter() - t0
    return {"value": fl / dt / 1e12, "unit": "TFLOP/s", "cores": threads,
            "kind": "reference" if use_ref else "port",
            "sample": f"attn_ref (flash.c:262-314, fp32, compiled natively): {threads * 4} tasks of 1 head x "
                      f"{rows} query rows x Sk={Sk} on {threads} threads, {dt:.1f} s"}


def run_reference(args, w) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import oracle

    Hq, Hkv, Sq, Sk, D, causal, *_ = w
    threads = os.cpu_count() or 1
    # size each step so that the whole run takes about a minute of CPU time
    budget = 60.0 / max(1, args.steps + args.warmup)
    for _ in range(args.warmup):
        cpu_reference_sample(w, min(budget, 2.0), threads)
    vals, secs = [], 0.0
    for _ in range(args.steps):
        r = cpu_reference_sample(w, budget, threads)
        vals.append(r["value"])
        secs += r["seconds"]
    value = float(np.mean(vals))
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * secs / max(1, args.steps),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic " + w[9],
        "config": config_dict(args.workload, w, args.gpus),
        "execution": f"{threads} host threads, rank 0 only; a bounded sample of the workload per step",
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": threads, "kind": r["kind"],
                         "sample": r["sample"]},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ GPU timing
def run_ours(args, w) -> None:
    import torch
    import torch.distributed as dist

    import transfer_station_b200 as ts

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)

    def barrier():
        if world > 1:
            t = torch.zeros(1, device=dev)
            dist.all_reduce(t)
        torch.cuda.synchronize()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    ts.load_library()
    Hq, Hkv, Sq, Sk, D, causal, *_ = w
    decode = is_decode(w)
    fl = flops(Hq, Sq, Sk, D, causal)
    by = algo_bytes(Hq, Hkv, Sq, Sk, D)
    Q, K, V = host_inputs(w)  # same seeded data on every rank; each rank owns its copy
    ncopy, set_bytes = pool_copies(w)  # rotating pool >= 2x L2: every step is L2-cold
    qs = [torch.from_numpy(Q.view(np.int16)).to(dev) for _ in range(ncopy)]
    ks = [torch.from_numpy(K.view(np.int16)).to(dev) for _ in range(ncopy)]
    vs = [torch.from_numpy(V.view(np.int16)).to(dev) for _ in range(ncopy)]
    os_ = [torch.empty(Hq * Sq * D, dtype=torch.float32, device=dev) for _ in range(ncopy)]
    scratch = torch.empty(ts.attn_flash_scratch_bytes(D, 128), dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)

    def step(i: int):
        c = i % ncopy
        rc = ts.attn_flash_stream(qs[c], ks[c], vs[c], os_[c], Hq, Hkv, Sq, Sk, D, causal, 128, scratch, 0, stream)
        if rc != ts.ATTN_OK:
            raise ts.AttnError(rc, "attn_flash_stream")

    for i in range(args.warmup):
        step(i)
    rc, code = ts.attn_flash_status(scratch, stream)
    if rc != ts.ATTN_OK:
        raise ts.AttnError(rc, f"warmup device status {code}")

    clocks = ClockSampler(local)
    clocks.start()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    barrier()
    launches0 = ts.attn_flash_kernel_launches()
    h0 = time.perf_counter()
    e0.record(stream)
    for i in range(args.steps):
        step(i)
    e1.record(stream)
    torch.cuda.synchronize()
    h1 = time.perf_counter()
    launches = ts.attn_flash_kernel_launches() - launches0
    barrier()
    clocks.stop()
    rc, code = ts.attn_flash_status(scratch, stream)
    if rc != ts.ATTN_OK:
        raise ts.AttnError(rc, f"timed-region device status {code}")
    ms_local = e0.elapsed_time(e1)
    ms = max_over_ranks(ms_local)
    ms_step = ms / args.steps
    per_launch_ms = ms_local / args.steps
    peaks = load_peaks()
    if decode:
        value = world * by * args.steps / (ms / 1e3) / 1e9
        unit = "GB/s"
        achieved = by / (per_launch_ms / 1e3) / 1e9
        roof = {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                "frac": achieved / peaks["hbm_gbs"]}
    else:
        value = world * fl * args.steps / (ms / 1e3) / 1e12
        unit = "TFLOP/s"
        achieved = fl / (per_launch_ms / 1e3) / 1e12
        roof = {"bound": "tensor", "achieved": achieved, "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                "frac": achieved / peaks["bf16_tflops"]}
    roof["traffic"] = load_traffic(args.workload)
    roof["algorithmic_per_launch"] = by if decode else fl
    roof["peak_source"] = peaks["source"] + (" burst" if not decode else " copy")
    roof["kernel"] = "ts::fa_tc_kernel (tcgen05 + TMA + TMEM)"

    def time_steps(fn, steps: int, what: str) -> float:
        """ms per step of `fn(i)` over `steps` calls after 3 warm-up calls (CUDA events on the
        launching stream, barrier and synchronize on both sides, max over ranks)."""
        for i in range(3):
            fn(i)
        barrier()
        e0.record(stream)
        for i in range(steps):
            fn(i)
        e1.record(stream)
        torch.cuda.synchronize()
        barrier()
        t = max_over_ranks(e0.elapsed_time(e1)) / steps
        rc, code = ts.attn_flash_status(scratch, stream)
        if rc != ts.ATTN_OK:
            raise ts.AttnError(rc, f"{what} device status {code}")
        return t

    def device_inputs(wl, seed: int, n: int):
        """Seeded bf16 tensor of n elements with workload wl's distribution, made on the GPU."""
        g = torch.Generator(device=dev)
        g.manual_seed(seed)
        a, b = wl[8]
        if wl[6] == "normal":
            x = torch.randn(n, device=dev, generator=g) * b + a
        else:
            x = torch.rand(n, device=dev, generator=g) * (b - a) + a
        return x.to(torch.bfloat16).view(torch.int16)

    # ---------------- the same prefill with causal masking (bottom-right), same buffers
    causal_line = None
    if not decode and not causal and not args.no_causal:
        cfl = flops(Hq, Sq, Sk, D, 1)

        def cstep(i: int):
            c = i % ncopy
            rc = ts.attn_flash_stream(qs[c], ks[c], vs[c], os_[c], Hq, Hkv, Sq, Sk, D, 1, 128, scratch, 0, stream)
            if rc != ts.ATTN_OK:
                raise ts.AttnError(rc, "attn_flash_stream (causal)")

        csteps = max(3, min(args.steps, 200))
        for i in range(3):
            cstep(i)
        barrier()
        e0.record(stream)
        for i in range(csteps):
            cstep(i)
        e1.record(stream)
        torch.cuda.synchronize()
        barrier()
        cms = max_over_ranks(e0.elapsed_time(e1)) / csteps
        rc, code = ts.attn_flash_status(scratch, stream)
        if rc != ts.ATTN_OK:
            raise ts.AttnError(rc, f"causal device status {code}")
        cach = cfl / (cms / 1e3) / 1e12
        causal_line = {"workload": args.workload + "_causal", "value": world * cach, "unit": "TFLOP/s",
                       "per_gpu_tflops": cach, "ms_per_step": cms,
                       "frac_of_measured_peak": cach / peaks["bf16_tflops"], "flops_per_step": cfl,
                       "flops": "useful (query i sees keys <= Sk - Sq + i)", "steps": csteps}

    # ---------------- e2e through the C ABI with pinned host buffers
    # E2E_LANES CUDA streams take turns, each with its own device buffers, pinned output buffer
    # and scratch block: step i's readback (device -> host) runs while step i+1's inputs go up
    # (host -> device) -- PCIe moves both directions at once -- and the kernels run in between.
    # Every step still copies its Q, K, V up and its O back inside the timed region.
    e2e_steps = max(1, min(args.steps, args.e2e_steps))
    hq = torch.from_numpy(Q.view(np.int16)).pin_memory()
    hk = torch.from_numpy(K.view(np.int16)).pin_memory()
    hv = torch.from_numpy(V.view(np.int16)).pin_memory()
    lanes = []
    n_lanes = max(1, args.e2e_lanes)
    for ln in range(n_lanes):
        if ln < ncopy:
            dq, dk, dv, do = qs[ln], ks[ln], vs[ln], os_[ln]
        else:
            dq, dk, dv = torch.empty_like(qs[0]), torch.empty_like(ks[0]), torch.empty_like(vs[0])
            do = torch.empty_like(os_[0])
        st = stream if ln == 0 else torch.cuda.Stream(dev)
        scr = scratch if ln == 0 else torch.empty_like(scratch)
        ho = torch.empty(Hq * Sq * D, dtype=torch.float32).pin_memory()
        lanes.append((dq, dk, dv, do, st, scr, ho))

    def e2e_step(i: int):
        dq, dk, dv, do, st, scr, ho = lanes[i % n_lanes]
        with torch.cuda.stream(st):
            dq.copy_(hq, non_blocking=True)
            dk.copy_(hk, non_blocking=True)
            dv.copy_(hv, non_blocking=True)
            rc = ts.attn_flash_stream(dq, dk, dv, do, Hq, Hkv, Sq, Sk, D, causal, 128, scr, 0, st)
            if rc != ts.ATTN_OK:
                raise ts.AttnError(rc, "attn_flash_stream (e2e)")
            ho.copy_(do, non_blocking=True)

    for i in range(n_lanes):
        e2e_step(i)
    barrier()
    e0.record(stream)
    for ln in lanes[1:]:
        ln[4].wait_stream(stream)
    for i in range(e2e_steps):
        e2e_step(i)
    for ln in lanes[1:]:
        stream.wait_stream(ln[4])
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1))
    e2e_val = world * (by if decode else fl) * e2e_steps / (e2e_ms / 1e3) / (1e9 if decode else 1e12)
    for ln in lanes:
        rc, code = ts.attn_flash_status(ln[5], ln[4])
        if rc != ts.ATTN_OK:
            raise ts.AttnError(rc, f"e2e device status {code}")
    del lanes

    # ---------------- secondary decode line (HBM-bound), single rank timing, max over ranks
    decode_line = None
    if not args.no_decode and not decode:
        dw = WORKLOADS["gqa_decode_b64_sk8192"]
        dHq, dHkv, dSq, dSk, dD, dc, *_ = dw
        dQ, dK, dV = host_inputs(dw)
        tq = torch.from_numpy(dQ.view(np.int16)).to(dev)
        tk = torch.from_numpy(dK.view(np.int16)).to(dev)
        tv = torch.from_numpy(dV.view(np.int16)).to(dev)
        to = torch.empty(dHq * dD, dtype=torch.float32, device=dev)
        dsteps = max(3, min(args.steps, 200))
        for _ in range(3):
            ts.attn_flash_stream(tq, tk, tv, to, dHq, dHkv, dSq, dSk, dD, dc, 128, scratch, 0, stream)
        barrier()
        e0.record(stream)
        for _ in range(dsteps):
            ts.attn_flash_stream(tq, tk, tv, to, dHq, dHkv, dSq, dSk, dD, dc, 128, scratch, 0, stream)
        e1.record(stream)
        torch.cuda.synchronize()
        barrier()
        dms = max_over_ranks(e0.elapsed_time(e1)) / dsteps
        dby = algo_bytes(dHq, dHkv, dSq, dSk, dD)
        rc, code = ts.attn_flash_status(scratch, stream)
        if rc != ts.ATTN_OK:
            raise ts.AttnError(rc, f"decode device status {code}")
        dach = dby / (dms / 1e3) / 1e9
        decode_line = {"workload": "gqa_decode_b64_sk8192", "desc": dw[9], "value": world * dach, "unit": "GB/s",
                       "per_gpu_gbs": dach, "ms_per_step": dms, "frac_of_measured_hbm": dach / peaks["hbm_gbs"],
                       "frac_of_8tbs_spec": dach / 8000.0, "bytes_per_step": dby, "steps": dsteps,
                       "l2": "K+V = 2 GiB per step > L2"}
        del tq, tk, tv, to

    # ---------------- the same decode through the paged K/V entry point (64-key pages, shuffled)
    paged_line = None
    if not args.no_decode and not decode:
        pB, pHq, pHkv, pSk, pD, pP = 64, 32, 8, 8192, 128, 64
        npages = pB * pSk // pP
        g = torch.Generator(device=dev)
        g.manual_seed(2)
        pq = torch.randn(pB * pHq * pD, device=dev, generator=g).to(torch.bfloat16).view(torch.int16)
        pk = torch.randn(npages * pHkv * pP * pD, device=dev, generator=g).to(torch.bfloat16).view(torch.int16)
        pv = torch.randn(npages * pHkv * pP * pD, device=dev, generator=g).to(torch.bfloat16).view(torch.int16)
        table = torch.randperm(npages, device=dev, generator=g).to(torch.int32)
        lens = torch.full((pB,), pSk, dtype=torch.int32, device=dev)
        po = torch.empty(pB * pHq * pD, dtype=torch.float32, device=dev)

        def paged_step():
            rc = ts.attn_flash_paged_stream(pq, pk, pv, table, lens, po, pB, pHq, pHkv, 1, pD, 0, pP, npages,
                                            pSk // pP, scratch, stream)
            if rc != ts.ATTN_OK:
                raise ts.AttnError(rc, "attn_flash_paged_stream")

        psteps = max(3, min(args.steps, 200))
        for _ in range(3):
            paged_step()
        barrier()
        e0.record(stream)
        for _ in range(psteps):
            paged_step()
        e1.record(stream)
        torch.cuda.synchronize()
        barrier()
        pms = max_over_ranks(e0.elapsed_time(e1)) / psteps
        rc, code = ts.attn_flash_status(scratch, stream)
        if rc != ts.ATTN_OK:
            raise ts.AttnError(rc, f"paged decode device status {code}")
        pby = algo_bytes(pB * pHq, pB * pHkv, 1, pSk, pD)
        pach = pby / (pms / 1e3) / 1e9
        paged_line = {"workload": "gqa_decode_b64_sk8192_paged64",
                      "desc": "BASELINE config 3 shape through attn_flash_paged_stream: 64-key pages in a "
                              "shuffled block table", "value": world * pach, "unit": "GB/s", "per_gpu_gbs": pach,
                      "ms_per_step": pms, "frac_of_measured_hbm": pach / peaks["hbm_gbs"], "steps": psteps}
        del pq, pk, pv, table, lens, po

    # ---------------- the QKV producer (attn_qkv_rope_stream) at the config 5 prefill shape
    producer_line = None
    if not args.no_producer:
        rB, rS, rHq, rHkv, rD = args.producer_batch, 16384, 64, 8, 128
        rT, rH = rB * rS, rHq + 2 * rHkv
        g = torch.Generator(device=dev)
        g.manual_seed(5)
        rqkv = torch.randn(rT * rH * rD, device=dev, generator=g).to(torch.bfloat16).view(torch.int16)
        rpos = torch.arange(rS, dtype=torch.int32, device=dev).repeat(rB)
        rqw = (1.0 + 0.1 * torch.randn(rD, device=dev, generator=g)).to(torch.bfloat16).view(torch.int16)
        rkw = (1.0 + 0.1 * torch.randn(rD, device=dev, generator=g)).to(torch.bfloat16).view(torch.int16)
        rcs = torch.empty(rS * rD, dtype=torch.float32, device=dev)
        if ts.attn_rope_table_stream(rcs, rS, rD, 1e6, stream) != ts.ATTN_OK:
            raise ts.AttnError(ts.ATTN_ERR_ARGS, "attn_rope_table_stream")
        rq = torch.empty(rT * rHq * rD, dtype=torch.int16, device=dev)
        rk = torch.empty(rB * rHkv * rS * rD, dtype=torch.int16, device=dev)
        rv = torch.empty_like(rk)

        def producer_step():
            rc = ts.attn_qkv_rope_stream(rqkv, rpos, rcs, rS, rqw, rkw, 1e-6, rB, rS, rHq, rHkv, rD, rD,
                                         ts.ATTN_ROPE_NEOX, rq, rk, rv, rS, scratch, stream)
            if rc != ts.ATTN_OK:
                raise ts.AttnError(rc, "attn_qkv_rope_stream")

        rsteps = max(3, min(args.steps, 100))
        for _ in range(3):
            producer_step()
        barrier()
        e0.record(stream)
        for _ in range(rsteps):
            producer_step()
        e1.record(stream)
        torch.cuda.synchronize()
        barrier()
        rms_ = max_over_ranks(e0.elapsed_time(e1)) / rsteps
        rc, code = ts.attn_flash_status(scratch, stream)
        if rc != ts.ATTN_OK:
            raise ts.AttnError(rc, f"producer device status {code}")
        # qkv read + Q/K/V written, plus each token's position and cos/sin table row
        rby = 2.0 * rT * rH * rD * 2 + rT * 4 + rT * rD * 4
        rach = rby / (rms_ / 1e3) / 1e9
        producer_line = {"workload": f"qwen3_qkv_rope_b{rB}_s16384",
                         "desc": f"config 5 prefill shape (B{rB}, Hq64/Hkv8, D128): fused QKV split + q/k RMSNorm + "
                                 "NeoX RoPE (theta 1e6) + contiguous cache write, attn_qkv_rope_stream",
                         "value": world * rach, "unit": "GB/s", "per_gpu_gbs": rach, "ms_per_step": rms_,
                         "frac_of_measured_hbm": rach / peaks["hbm_gbs"], "bytes_per_step": rby, "steps": rsteps,
                         "l2": f"{rby / 1e9:.2f} GB moved per step > L2"}
        del rqkv, rpos, rqw, rkw, rcs, rq, rk, rv

    # ---------------- long-context decode, key axis split over the ranks (NCCL merge)
    long_line = None
    if not args.no_decode:
        from transfer_station_b200 import multigpu

        B, lHq, lHkv, lSk, lD = 4, 64, 8, 131072, 128
        Hq5, Hkv5 = B * lHq, B * lHkv
        k0, kl = multigpu.key_shard(lSk, world, rank)
        g = torch.Generator(device=dev)
        g.manual_seed(4)
        lq = (torch.randn(Hq5 * lD, device=dev, generator=g) * 0.5).to(torch.bfloat16).view(torch.int16)
        g.manual_seed(1000 + rank)
        lk = (torch.randn(Hkv5 * kl * lD, device=dev, generator=g) * 0.5).to(torch.bfloat16).view(torch.int16)
        lv = (torch.randn(Hkv5 * kl * lD, device=dev, generator=g) * 0.5).to(torch.bfloat16).view(torch.int16)
        lo = torch.empty(Hq5 * lD, dtype=torch.float32, device=dev)
        lsteps = max(3, min(args.steps, 100))
        for _ in range(3):
            multigpu.sharded_decode(lq, lk, lv, lo, Hq5, Hkv5, 1, lSk, k0, lD, 0, scratch)
        barrier()
        e0.record(stream)
        for _ in range(lsteps):
            multigpu.sharded_decode(lq, lk, lv, lo, Hq5, Hkv5, 1, lSk, k0, lD, 0, scratch)
        e1.record(stream)
        torch.cuda.synchronize()
        barrier()
        lms = max_over_ranks(e0.elapsed_time(e1)) / lsteps
        rc, code = ts.attn_flash_status(scratch, stream)
        if rc != ts.ATTN_OK:
            raise ts.AttnError(rc, f"long decode device status {code}")
        lby = algo_bytes(Hq5, Hkv5, 1, lSk, lD)
        long_line = {"workload": "gqa_long_decode_b4_sk131072", "value": lby / (lms / 1e3) / 1e9, "unit": "GB/s",
                     "per_gpu_gbs": lby / (lms / 1e3) / 1e9 / world, "ms_per_step": lms,
                     "frac_of_measured_hbm_per_gpu": lby / (lms / 1e3) / 1e9 / world / peaks["hbm_gbs"],
                     "bytes_per_step": lby, "steps": lsteps, "scaling": "strong (key axis split over ranks)",
                     "merge": "one NCCL all-gather of packed (m, l, acc) fp32 blocks, then combine"}
        # the same decode merged by the peer-store kernel (no collective per step)
        merge = multigpu.PeerMerge(Hq5, lD, device=dev)
        pms = time_steps(lambda i: multigpu.sharded_decode_peers(lq, lk, lv, lo, Hq5, Hkv5, 1, lSk, k0, lD, 0,
                                                                 scratch, merge), lsteps, "long decode (peer merge)")
        merge.close()
        long_line["peer_merge"] = {
            "value": lby / (pms / 1e3) / 1e9, "unit": "GB/s", "per_gpu_gbs": lby / (pms / 1e3) / 1e9 / world,
            "ms_per_step": pms, "frac_of_measured_hbm_per_gpu": lby / (pms / 1e3) / 1e9 / world / peaks["hbm_gbs"],
            "merge": "attn_flash_decode_peers_stream: the partial kernel, then one kernel that stores each rank's "
                     "(m, l, acc) into every peer's exchange block over NVLink (CUDA IPC), raises flags, waits and "
                     "merges -- no collective per step"}
        # The line's value is the faster of the two merges at this rank count (both are the
        # library's public paths; every rank took both timings, max over ranks).
        long_line["ms_per_step_nccl_merge"] = lms
        long_line["ms_per_step_peer_merge"] = pms
        if world > 1 and pms < lms:
            long_line.update({"value": lby / (pms / 1e3) / 1e9, "per_gpu_gbs": lby / (pms / 1e3) / 1e9 / world,
                              "ms_per_step": pms,
                              "frac_of_measured_hbm_per_gpu": lby / (pms / 1e3) / 1e9 / world / peaks["hbm_gbs"],
                              "merge": "the peer-store merge (faster than the NCCL all-gather at this rank count): "
                                       + long_line["peer_merge"]["merge"]})
        del lq, lk, lv, lo

    # ---------------- the other BASELINE configs on each GPU (device-timed)
    config_lines = []
    if not args.no_configs:
        for name in ("qwen3_gqa_prefill_s1024", "qwen3_gqa_prefill_s2048", "mqa_prefill_b8_s2048",
                     "mqa_decode_b128_sk4096"):
            if name == args.workload:
                continue
            cw = WORKLOADS[name]
            cHq, cHkv, cSq, cSk, cD, cc = cw[:6]
            cn, _ = pool_copies(cw)
            bufs = [(device_inputs(cw, 10 * j + 1, cHq * cSq * cD), device_inputs(cw, 10 * j + 2, cHkv * cSk * cD),
                     device_inputs(cw, 10 * j + 3, cHkv * cSk * cD),
                     torch.empty(cHq * cSq * cD, dtype=torch.float32, device=dev)) for j in range(cn)]

            def cfg_step(i: int, bufs=bufs, a=(cHq, cHkv, cSq, cSk, cD, cc)):
                tq, tk, tv, to = bufs[i % len(bufs)]
                rc = ts.attn_flash_stream(tq, tk, tv, to, *a, 128, scratch, 0, stream)
                if rc != ts.ATTN_OK:
                    raise ts.AttnError(rc, f"attn_flash_stream ({name})")

            cms = time_steps(cfg_step, max(3, min(args.steps, 200)), name)
            if is_decode(cw):
                cwork, cunit, cpeak = algo_bytes(cHq, cHkv, cSq, cSk, cD) / 1e9, "GB/s", peaks["hbm_gbs"]
            else:
                cwork, cunit, cpeak = flops(cHq, cSq, cSk, cD, cc) / 1e12, "TFLOP/s", peaks["bf16_tflops"]
            per = cwork / (cms / 1e3)
            config_lines.append({"workload": name, "desc": cw[9], "value": world * per, "unit": cunit,
                                 "per_gpu": per, "ms_per_step": cms, "frac_of_measured_peak": per / cpeak,
                                 "bound": "hbm" if is_decode(cw) else "tensor",
                                 "steps": max(3, min(args.steps, 200)),
                                 "l2": f"rotating pool of {cn} sets (>= 2x L2)", "data": "synthetic, seeded on device"})
            del bufs

    # ---------------- config 5 prefill as ONE problem sharded over the ranks (strong scaling)
    sharded_line = None
    if not args.no_sharded:
        from transfer_station_b200 import multigpu

        sB, sHq, sHkv, sS, sD = 4, 64, 8, 16384, 128
        sl = multigpu.prefill_slice(sB, sHq, sHkv, sS, sS, sD, world, rank)
        # full-layout tensors; this rank fills and touches only its units' ranges
        sq = torch.empty(sB * sHq * sS * sD, dtype=torch.int16, device=dev)
        sk = torch.empty(sB * sHkv * sS * sD, dtype=torch.int16, device=dev)
        sv = torch.empty_like(sk)
        so = torch.empty(sB * sHq * sS * sD, dtype=torch.float32, device=dev)
        lw = WORKLOADS["long_prefill_b4_s16384"]
        if sl.hkv > 0:
            sq[sl.q_off:sl.q_off + sl.hq * sS * sD] = device_inputs(lw, 40 + rank, sl.hq * sS * sD)
            sk[sl.kv_off:sl.kv_off + sl.hkv * sS * sD] = device_inputs(lw, 50 + rank, sl.hkv * sS * sD)
            sv[sl.kv_off:sl.kv_off + sl.hkv * sS * sD] = device_inputs(lw, 60 + rank, sl.hkv * sS * sD)

        def sharded_step(i: int):
            multigpu.sharded_prefill(sq, sk, sv, so, sB, sHq, sHkv, sS, sS, sD, 0, scratch, stream=stream,
                                     rank=rank, world=world)

        ssteps = max(3, min(args.steps, 20))
        sms_ = time_steps(sharded_step, ssteps, "sharded prefill")
        sfl = flops(sB * sHq, sS, sS, sD, 0)
        sval = sfl / (sms_ / 1e3) / 1e12
        sharded_line = {"workload": "long_prefill_b4_s16384_sharded",
                        "desc": "BASELINE config 5 prefill (B=4, Hq=64, Hkv=8, D=128, Sq=Sk=16384) as one problem: "
                                f"its {sB * sHkv} (batch x kv-head group) units split over {world} rank(s) "
                                "(multigpu.sharded_prefill), no collective",
                        "value": sval, "unit": "TFLOP/s", "per_gpu_tflops": sval / world, "ms_per_step": sms_,
                        "frac_of_measured_peak_per_gpu": sval / world / peaks["bf16_tflops"],
                        "flops_per_step": sfl, "units_this_rank": [sl.u0, sl.u1], "steps": ssteps,
                        "scaling": "strong (fixed problem; ms_per_step is the slowest rank's)",
                        "l2": "3.4 GB of Q/K/V/O per rank > L2"}
        del sq, sk, sv, so

    # ---------------- CPU baseline (rank 0, N=1 only)
    cpu = None
    if world == 1 and rank == 0 and not args.no_cpu_baseline:
        r = cpu_reference_sample(w, args.cpu_seconds)
        cpu = {k: r[k] for k in ("value", "unit", "cores", "kind", "sample")}
        cpu["fp32_reference"] = cpu_attn_ref_sample(w, max(2.0, args.cpu_seconds / 2))

    csum = clocks.summary(h0, h1)
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": unit, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16",
            "data": f"synthetic, seeded ({w[6]}, seed {w[7]}), bf16 RNE; {w[9]}",
            "config": config_dict(args.workload, w, world),
            "roofline": roof,
            "cpu_baseline": cpu,
            "e2e": {"value": e2e_val, "unit": unit, "h2d_bytes_per_step": int(Q.nbytes + K.nbytes + V.nbytes),
                    "d2h_bytes_per_step": int(Hq * Sq * D * 4), "steps": e2e_steps,
                    "pcie_gbs": (Q.nbytes + K.nbytes + V.nbytes + Hq * Sq * D * 4) * e2e_steps / (e2e_ms / 1e3) / 1e9,
                    "bound": "PCIe: the host<->device bytes of a step (pcie_gbs, both directions overlapped) take "
                             "longer than its kernel",
                    "path": "pinned host -> cudaMemcpyAsync -> attn_flash_stream -> cudaMemcpyAsync -> pinned host",
                    "pipeline": f"{n_lanes} CUDA streams taking turns (their own device, host and scratch "
                                "buffers): a step's readback overlaps the next step's upload"},
            "gpu_launches": int(launches),
            "clocks": csum,
            "causal_prefill": causal_line,
            "decode": decode_line,
            "paged_decode": paged_line,
            "long_decode": long_line,
            "qkv_rope": producer_line,
            "sharded_prefill": sharded_line,
            "configs": config_lines,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-producer", action="store_true", help="skip the QKV producer line")
    ap.add_argument("--no-causal", action="store_true", help="skip the causal prefill line")
    ap.add_argument("--producer-batch", type=int, default=4,
                    help="sequences of 16384 tokens in the producer line (4 = the config 5 prefill shape)")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default=DEFAULT_WORKLOAD)
    ap.add_argument("--e2e-steps", type=int, default=200)
    ap.add_argument("--e2e-lanes", type=int, default=3, help="CUDA streams taking turns in the e2e line")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-decode", action="store_true")
    ap.add_argument("--no-configs", action="store_true", help="skip the other BASELINE configs' lines")
    ap.add_argument("--no-sharded", action="store_true", help="skip the sharded config 5 prefill line")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    w = WORKLOADS[args.workload]
    if args.impl == "reference":
        run_reference(args, w)
    else:
        run_ours(args, w)


if __name__ == "__main__":
    main()
