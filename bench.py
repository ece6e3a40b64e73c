#!/usr/bin/env python
"""Benchmark of the B200 attention hot path (one JSON line on stdout).

Headline (BASELINE.json metric "GQA decode attn HBM GB/s & tokens/s; prefill
attn TFLOPS"): configuration C4, batched long-context decode -- 64 sessions
per GPU with lengths uniform in [4096, 32768] (seed 3), K/V in 256-token
ColdStore-exact pages under a random physical page permutation, 32 query /
8 KV heads of dim 128.  One step = one split-KV decode of every session
(mslim_decode_split + mslim_decode_merge).  `value` is algorithmic bytes
(K+V of every session, Q and O rows, page-table entries) per second, summed
over all ranks; inputs (4.8 GB per GPU) are larger than L2, so no flush is
needed between steps.

Multi-GPU: one process per GPU (torchrun); each rank owns its own sessions
(independent objects, no data-path collective); NCCL is used only for the
barrier and the max-over-ranks step time.  --scaling strong (default) shards
the 64 sessions of the one C4 draw across the ranks by longest-processing-
time, as configuration C4 defines the multi-GPU case; the line carries every
rank's token sum and split count.  At N > 1 the weak figure (every rank
decoding its own 64 sessions) is reported beside it under "weak", and
--scaling weak makes it the headline.

The C5 leg (key "model", --no-model skips it) runs the 32-layer
Llama-3-8B-shaped decoder tensor-parallel over the same ranks (KV-head
groups, the fused NVLink reduction in the decode step) with a stated number
of decode steps, so every N of a scaling run carries the tensor-parallel
decode figures and the SHA-256 of its greedy tokens.

--impl reference times the reference's CPU hot-dense path (its C
restatement in oracle/, OpenMP across query heads like the reference's rayon
loop) on a bounded sample of the same sessions, on rank 0 only.
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

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "vk-shei_b200"))

METRIC = "GQA decode attn HBM GB/s (C4 batched split-KV decode; tokens/s and prefill TFLOPS alongside)"
QH, KVH, D, PAGE = 32, 8, 128, 256


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--scaling", choices=["weak", "strong"], default="strong")
    ap.add_argument("--sessions", type=int, default=64, help="sessions per GPU (small profiling cases)")
    ap.add_argument("--shard-of", default="",
                    help="R/N: on one GPU, time the sessions that rank R of an N-rank strong-scaling "
                         "run owns (per-rank behaviour of the multi-GPU split)")
    ap.add_argument("--no-model", action="store_true", help="skip the C5 tensor-parallel model leg")
    ap.add_argument("--no-weak", action="store_true", help="skip the weak-scaling figure at N > 1")
    ap.add_argument("--split-tokens", type=int, default=0)
    ap.add_argument("--decode-schedule", choices=["split-merge", "persistent"], default="split-merge",
                    help="mslim_cuda_set_decode_schedule for the run (same bits either way)")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--no-e2e", action="store_true", help="skip the end-to-end leg")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-prefill", action="store_true", help="skip the C2 prefill leg")
    ap.add_argument("--prefill-only", action="store_true", help="run only the C2 prefill leg (profiling)")
    ap.add_argument("--model", action="store_true",
                    help="C5: the 32-layer decoder, tensor-parallel over the torchrun ranks")
    ap.add_argument("--model-layers", type=int, default=32)
    ap.add_argument("--model-batch", type=int, default=8)
    ap.add_argument("--model-prefill", type=int, default=8192)
    ap.add_argument("--model-steps", type=int, default=256)
    ap.add_argument("--model-leg-steps", type=int, default=64,
                    help="decode steps of the C5 leg inside the default (C4) run")
    ap.add_argument("--mlp", choices=["sharded", "replicated"], default="sharded")
    ap.add_argument("--kv-mode", choices=["dense", "coldstore"], default="dense")
    ap.add_argument("--no-graph", action="store_true", help="C5 decode steps issued eagerly (no CUDA graph)")
    ap.add_argument("--decode-gemm", choices=["auto", "own", "cublas"], default="auto",
                    help="C5 decode projections: auto (= own), "
                         "own (mslim_cuda_gemv) or cublas")
    ap.add_argument("--decode-qkv", choices=["fused", "separate"], default="separate",
                    help="C5 decode with the own projections: the q|k|v projection with RoPE + K/V append in its "
                         "epilogue (fused), or the projection then the append kernel (separate)")
    ap.add_argument("--gemv", action="store_true",
                    help="the C5 decode projections: mslim_cuda_gemv against cuBLAS, per shape")
    ap.add_argument("--split-sweep", action="store_true",
                    help="time every candidate split size of the decode on equal-length batches and on the "
                         "C4 shards (one JSON line per case; the data the split policies are fitted to)")
    ap.add_argument("--layer", action="store_true",
                    help="C3: one Llama-3-8B layer, 512-token prefill + 8 decode steps, CPU path beside it")
    return ap.parse_args()


# ------------------------------------------------------------------ clocks --

_REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
            0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
            0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting"}


class ClockSampler:
    """Polls NVML (read-only) every few ms during the timed region."""

    def __init__(self, index: int):
        self.index = index
        self.samples = []
        self.reasons = 0
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None
        self._nvml = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nvml = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self._nvml = None

    def _run(self):
        p = self._nvml
        while not self._stop.is_set():
            try:
                self.samples.append(p.nvmlDeviceGetClockInfo(self._h, p.NVML_CLOCK_SM))
                self.reasons |= int(p.nvmlDeviceGetCurrentClocksEventReasons(self._h))
            except Exception:
                pass
            time.sleep(0.001)

    def start(self):
        if self._nvml:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
            # the timed regions are short (~0.1 s): return only once the thread
            # is polling, so its samples cover the region (bounded at 1 s)
            t0 = time.time()
            while len(self.samples) < 3 and time.time() - t0 < 1.0:
                time.sleep(0.001)

    def stop(self) -> dict:
        self._stop.set()
        if self._thread:
            self._thread.join()
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0}
        reasons = [name for bit, name in _REASONS.items() if self.reasons & bit and bit != 0x1]
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": reasons, "samples": len(self.samples)}


# -------------------------------------------------------------- utilities --

# Peer-to-peer copy over NVLink, per direction per GPU, measured on this pool's
# B200s (900 GB/s nominal): the denominator for bytes a kernel pulls from peers.
NVLINK_PEER_GBS = 770.0


def measured_peaks() -> dict:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return {"hbm_gbs": d.get("hbm_gbs"), "bf16_tflops": d.get("bf16_tflops"),
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained"), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


def profile_traffic(name: str):
    """dram bytes per launch from a committed ncu summary (profiles/*.json)."""
    p = os.path.join(ROOT, "profiles", name)
    if os.path.exists(p):
        with open(p) as f:
            return json.load(f)
    return None


def host_threads() -> int:
    """Every host thread this process may run on.  torchrun sets
    OMP_NUM_THREADS=1 in each rank; the CPU legs size OpenMP from the
    affinity mask instead, so the reference arm runs on the same cores at
    every N."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def lpt_shard(lengths, world: int, rank: int) -> list[int]:
    """Longest-processing-time assignment of sessions to ranks."""
    order = sorted(range(len(lengths)), key=lambda i: (-int(lengths[i]), i))
    loads = [0] * world
    owner = {}
    for i in order:
        r = min(range(world), key=lambda j: (loads[j], j))
        loads[r] += int(lengths[i])
        owner[i] = r
    return sorted(i for i in order if owner[i] == rank)


# --------------------------------------------------------------- CPU legs --

def cpu_sample_gbs(lengths, seconds: float, seed: int = 3) -> dict:
    """Times the CPU restatement of the reference hot-dense / ColdStore-exact
    decode (native_cpu_adapter.rs:253-307, :386-455) on sessions of the C4
    draw, repeating passes until `seconds` of CPU work have elapsed."""
    import numpy as np
    from oracle import oracle
    from mslim_b200 import workloads
    rng = np.random.default_rng(seed)
    threads = host_threads()
    sample = []
    for L in lengths:
        L = int(L)
        npg = (L + PAGE - 1) // PAGE
        k = workloads.normal_bf16(rng, (npg, KVH, PAGE, D))
        v = workloads.normal_bf16(rng, (npg, KVH, PAGE, D))
        q = workloads.bf16_to_f32(workloads.normal_bf16(rng, (QH * D,)))
        sample.append((L, q, k, v, np.arange(npg, dtype=np.int32)))
    done_bytes = 0
    t0 = time.perf_counter()
    passes = 0
    while True:
        for L, q, k, v, table in sample:
            oracle.paged_attention_bf16(QH, KVH, D, q, k, v, table, PAGE, L, threads)
            done_bytes += L * KVH * D * 2 * 2 + 2 * QH * D * 2
        passes += 1
        el = time.perf_counter() - t0
        if el >= seconds or passes >= 1000:
            break
    return {"value": done_bytes / el / 1e9, "unit": "GB/s", "cores": threads, "kind": "port",
            "omp_num_threads_env": os.environ.get("OMP_NUM_THREADS"),
            "sample": f"{len(sample)} C4 sessions (L={','.join(str(int(x)) for x in lengths)}) x {passes} passes, "
                      f"{el:.1f} s, oracle/mslim_oracle.c paged_attention_bf16 with {threads} OpenMP threads"}


def run_reference(args, rank: int) -> None:
    if rank != 0:
        return
    from mslim_b200 import workloads
    layout = workloads.c4_layout(seed=3)
    import numpy as np
    from oracle import oracle
    lengths = layout.lengths[:4]
    rng = np.random.default_rng(3)
    threads = host_threads()
    data = []
    for L in lengths:
        npg = (int(L) + PAGE - 1) // PAGE
        data.append((int(L), workloads.bf16_to_f32(workloads.normal_bf16(rng, (QH * D,))),
                     workloads.normal_bf16(rng, (npg, KVH, PAGE, D)), workloads.normal_bf16(rng, (npg, KVH, PAGE, D)),
                     np.arange(npg, dtype=np.int32)))
    step_bytes = sum(L * KVH * D * 4 + 2 * QH * D * 2 for L, *_ in data)

    def step():
        for L, q, k, v, t in data:
            oracle.paged_attention_bf16(QH, KVH, D, q, k, v, t, PAGE, L, threads)

    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    el = time.perf_counter() - t0
    value = step_bytes * args.steps / el / 1e9
    sample = (f"{len(data)} C4 sessions per step (L={','.join(str(L) for L, *_ in data)}), "
              f"oracle/mslim_oracle.c paged_attention_bf16, {threads} OpenMP threads")
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": el * 1e3 / args.steps,
            "higher_is_better": True, "scaling": args.scaling, "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded N(0,1) bf16)",
            "config": {"workload": "C4 batched long-context decode (bounded CPU sample)", "page_tokens": PAGE,
                       "query_heads": QH, "kv_heads": KVH, "head_dim": D},
            "cpu_baseline": {"value": value, "unit": "GB/s", "cores": threads, "kind": "port", "sample": sample,
                             "omp_num_threads_env": os.environ.get("OMP_NUM_THREADS")},
            "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------- prefill leg --

def bench_prefill(m, torch, device, args) -> dict:
    """C2: causal prefill, S = 2048, 32/8 heads,
    D = 128, through the C ABI (mslim_cuda_prefill_causal).

    One call's Q/K/V/O (40 MB) fit in the 126 MB L2, so the leg keeps six
    copies (240 MB) and rotates through them: every call reads inputs last
    touched five calls (200 MB of traffic) earlier.  The timed calls are
    captured once into a CUDA graph and replayed back to back (as consecutive
    layers' prefill would run), so host jitter (Python, the clock-sampling
    thread) cannot idle the GPU between them; after a one-second idle (the
    power limiter recovers from the HBM-bound decode legs) and three warm
    replays, three replays are timed, each between a pair of CUDA events, and
    the median is the figure.  Consecutive calls overlap launch and setup through
    programmatic dependent launch; each waits for its predecessor's memory
    before it reads an input.  The same calls issued from a plain host loop,
    and one call timed alone (which carries 4-7 us of event/launch latency on
    top of the kernel), are reported beside it."""
    S, copies = 2048, 6
    g = m.AttentionGeometry.new(QH, KVH, D)
    gen = torch.Generator(device=device)
    gen.manual_seed(1)
    q0 = torch.randn((S, QH, D), generator=gen, device=device, dtype=torch.bfloat16)
    k0 = torch.randn((S, KVH, D), generator=gen, device=device, dtype=torch.bfloat16)
    v0 = torch.randn((S, KVH, D), generator=gen, device=device, dtype=torch.bfloat16)
    sets = [(q0.clone(), k0.clone(), v0.clone(), torch.empty_like(q0)) for _ in range(copies)]
    stream = torch.cuda.current_stream()

    def call(i, st):
        q, k, v, out = sets[i % copies]
        m.prefill_causal(g, q, k, v, out, S, 0, st)

    for i in range(max(args.warmup, 3) * copies):
        call(i, stream)
    torch.cuda.synchronize()
    steps = max(12, min(args.steps, 48))
    graph = torch.cuda.CUDAGraph()
    cap = torch.cuda.Stream()
    cap.wait_stream(stream)
    launches0 = m.kernel_launches()
    with torch.cuda.graph(graph, stream=cap, capture_error_mode="thread_local"):
        for i in range(steps):
            call(i, torch.cuda.current_stream())
    captured = m.kernel_launches() - launches0  # per replay
    # a one-second idle lets the power limiter recover from the preceding
    # HBM-bound legs, then warm replays settle the clocks into this leg's
    # regime before anything is timed
    time.sleep(1.0)
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    sampler = ClockSampler(torch.cuda.current_device())
    sampler.start()
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    replays = []
    for _ in range(3):
        a.record(stream)
        graph.replay()
        b.record(stream)
        b.synchronize()
        replays.append(a.elapsed_time(b) / steps)
    ms = statistics.median(replays)
    clocks = sampler.stop()
    # the same calls from a plain host loop
    torch.cuda.synchronize()
    a.record(stream)
    for i in range(steps):
        call(i, stream)
    b.record(stream)
    b.synchronize()
    ms_loop = a.elapsed_time(b) / steps
    # one call timed alone (events around one launch)
    alone = []
    for i in range(10):
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        call(i, stream)
        e1.record(stream)
        e1.synchronize()
        alone.append(e0.elapsed_time(e1))
    del graph
    if m.device_status(torch.cuda.current_device()) != 0:
        raise SystemExit("device status reported an error during the prefill leg")
    flops = 4 * D * QH * S * (S + 1) // 2
    tflops = flops / (ms * 1e-3) / 1e12
    peaks = measured_peaks()
    kernel = "mslim_prefill_pair" if (QH // KVH) % 2 == 0 else "mslim_prefill_causal"
    traffic = profile_traffic("prefill_c2_traffic.json")
    return {"metric": "prefill attn TFLOPS (C2 causal, S 2048, 32/8 heads, D 128)", "value": tflops,
            "unit": "TFLOP/s", "ms_per_step": ms, "steps": steps,
            "timing": ("calls captured in one CUDA graph; three warm replays, then the median of "
                       "three replays each between a pair of CUDA events"),
            "ms_per_step_replays": replays,
            "ms_per_call_host_loop": ms_loop,
            "ms_single_call_events": statistics.median(alone),
            "algorithmic_flops": flops,
            "l2": (f"inputs larger than L2: {copies} rotating copies of Q/K/V/O "
                   f"({copies * 40} MB > 126 MB L2), calls back to back"),
            "roofline": {"bound": "tensor", "kernel": kernel, "achieved": tflops,
                         "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                         "frac": tflops / peaks["bf16_tflops"] if peaks["bf16_tflops"] else None,
                         "peak_source": ("measured (MEASURED_PEAKS.json bf16_tflops, burst)"
                                         if peaks["source"] == "measured" else "fallback 1590 TFLOP/s"),
                         "frac_of_sustained": (tflops / peaks["bf16_tflops_sustained"]
                                               if peaks.get("bf16_tflops_sustained") else None),
                         "traffic": traffic["dram_bytes_per_launch"] if traffic else None,
                         "traffic_source": ("profiles/prefill_c2_traffic.json (one ncu capture of this C2 call), "
                                            "not measured in this run" if traffic else None)},
            "gpu_launches": captured, "clocks": clocks}


GEMV_SHAPES = [("tp1_qkv", 6144, 4096), ("tp1_o", 4096, 4096), ("tp1_gate_up", 28672, 4096),
               ("tp1_down", 4096, 14336), ("tp1_lm_head", 128256, 4096), ("tp8_qkv", 768, 4096),
               ("tp8_o", 4096, 512), ("tp8_gate_up", 3584, 4096), ("tp8_down", 4096, 1792),
               ("tp8_lm_head", 16032, 4096)]


def bench_gemv(m, torch, device, args) -> dict:
    """The C5 decode step's projections (batch 8 rows; TP 1 and per-rank TP 8
    shapes) through mslim_cuda_gemv (the tcgen05 weight stream) and through
    cuBLAS (torch.matmul), each as 40 calls captured in one CUDA graph, best
    of five replays between CUDA events; the gate|up shapes also with SwiGLU
    (mslim_cuda_gemv_swiglu, or either projection then mslim_cuda_swiglu_rows).  Weight copies rotate so that every
    call streams its weights from HBM (> 400 MB of weights per replay)."""
    from mslim_b200 import attention as att
    torch.backends.cuda.matmul.allow_bf16_reduced_precision_reduction = False
    rows, reps = args.model_batch, 40
    out = []
    for name, n, k in GEMV_SHAPES:
        wbytes = n * k * 2
        copies = max(1, min(16, (400 << 20) // wbytes + 1))
        gen = torch.Generator(device=device)
        gen.manual_seed(11)
        ws = [torch.randn((n, k), generator=gen, device=device, dtype=torch.bfloat16) * 0.02 for _ in range(copies)]
        x = torch.randn((rows, k), generator=gen, device=device, dtype=torch.bfloat16)
        y = torch.empty((rows, n), device=device, dtype=torch.bfloat16)
        res = {"shape": name, "n": n, "k": k, "rows": rows, "weight_bytes": wbytes}
        act = torch.empty((rows, n // 2), device=device, dtype=torch.bfloat16)
        # gate|up shapes: also SwiGLU, fused into the projection (interleaved
        # weights) or as a second launch after either projection
        kinds = ("own", "cublas") + (("fused_swiglu", "own_then_swiglu", "cublas_then_swiglu")
                                     if "gate_up" in name else ())
        for kind in kinds:
            def call(i, st):
                w = ws[i % copies]
                if kind == "own":
                    att.gemv(x, w, y, rows, n, k, stream=st)
                elif kind == "cublas":
                    torch.matmul(x, w.t(), out=y)
                elif kind == "fused_swiglu":
                    att.gemv_swiglu(x, w, act, rows, n // 2, k, stream=st)
                else:
                    if kind == "own_then_swiglu":
                        att.gemv(x, w, y, rows, n, k, stream=st)
                    else:
                        torch.matmul(x, w.t(), out=y)
                    att.swiglu_rows(y, act, rows * (n // 2) // 64, 64, stream=st)
            stream = torch.cuda.current_stream()
            for i in range(6):
                call(i, stream)
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            cap = torch.cuda.Stream()
            cap.wait_stream(stream)
            with torch.cuda.graph(graph, stream=cap, capture_error_mode="thread_local"):
                for i in range(reps):
                    call(i, torch.cuda.current_stream())
            graph.replay()
            torch.cuda.synchronize()
            a = torch.cuda.Event(enable_timing=True)
            b = torch.cuda.Event(enable_timing=True)
            best = float("inf")
            for _ in range(5):
                a.record(stream)
                graph.replay()
                b.record(stream)
                b.synchronize()
                best = min(best, a.elapsed_time(b) / reps)
            del graph
            res[f"{kind}_us"] = best * 1e3
            res[f"{kind}_gbs"] = wbytes / (best * 1e-3) / 1e9
        out.append(res)
        del ws
        torch.cuda.empty_cache()
    if m.device_status(torch.cuda.current_device()) != 0:
        raise SystemExit("device status reported an error during the GEMV leg")
    return {"metric": "decode projection time (C5 shapes, batch rows)", "unit": "us", "shapes": out,
            "peak_hbm_gbs": measured_peaks()["hbm_gbs"]}


def bench_layer(m, torch, device, args) -> dict:
    """C3: one Llama-3-8B-shaped layer, 512-token
    prefill then 8 forced decode steps, dense KV and ColdStore-exact KV, device
    time by CUDA events; the CPU decoder (oracle forward_token, one layer) is
    timed beside it on a bounded sample of the same tokens."""
    import hashlib

    import numpy as np
    from mslim_b200 import layer as lay
    sys.path.insert(0, ROOT)
    from oracle import oracle as orc

    P, steps, seed = 512, 8, 2
    spec = lay.LayerSpec()
    weights = lay.random_layer_weights(spec, seed)
    ids = np.random.default_rng(seed).integers(0, 128256, size=P + steps)
    emb = lay.embedding_rows(ids, spec.hidden, seed)
    x = torch.from_numpy(emb.view(np.int16)).to(device).view(torch.bfloat16)
    out = {}
    for mode in ("dense", "coldstore"):
        times = []
        for rep in range(max(args.warmup, 3) + 5):
            L = lay.DeviceLayer(spec, weights, P + steps, kv_mode=mode, page_tokens=256, page_seed=seed)
            torch.cuda.synchronize()
            e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
            e0.record()
            y, *_ = L.prefill(x[:P])
            e1.record()
            ys = [L.decode(x[P + i:P + i + 1])[0] for i in range(steps)]
            e2.record()
            torch.cuda.synchronize()
            if rep >= max(args.warmup, 3):
                times.append((e0.elapsed_time(e1), e1.elapsed_time(e2)))
            last = torch.cat([y] + ys).view(torch.int16).cpu().numpy()
            del L
        pf = statistics.median(t[0] for t in times)
        dc = statistics.median(t[1] for t in times)
        out[mode] = {"prefill_ms": pf, "prefill_tokens_per_s": P / (pf * 1e-3),
                     "decode_ms_per_step": dc / steps, "decode_tokens_per_s": steps / (dc * 1e-3),
                     "outputs_sha256": hashlib.sha256(last.tobytes()).hexdigest()}
    # the CPU decoder on the first tokens of the same prompt (all host threads)
    lo = orc.LayerOracle(weights, spec.hidden, spec.intermediate, spec.query_heads, spec.kv_heads,
                         spec.head_dim, spec.eps, spec.theta, P + steps)
    xf = orc.bf16_to_f32(emb).reshape(emb.shape)
    t0 = time.time()
    n = 0
    while n < P and (n < 8 or time.time() - t0 < args.cpu_seconds):
        lo.forward(xf[n])
        n += 1
    cpu_s = time.time() - t0
    return {
        "metric": "C3 one-layer tokens/s (Llama-3-8B layer, 512-token prefill + 8 decode steps)",
        "value": out["dense"]["prefill_tokens_per_s"], "unit": "tokens/s", "n_gpus": 1,
        "dtype": "bf16", "data": "synthetic (seed 2: N(0,0.02) projections, norms 1, N(0,1) embedding rows)",
        "config": {"workload": "C3", "prefill": P, "decode_steps": steps},
        "dense": out["dense"], "coldstore": out["coldstore"],
        "dense_equals_coldstore": out["dense"]["outputs_sha256"] == out["coldstore"]["outputs_sha256"],
        "cpu_baseline": {"value": n / cpu_s, "unit": "tokens/s", "cores": orc.max_threads(), "kind": "port",
                         "sample": f"the first {n} prompt tokens through oracle forward_token (one layer), "
                                   f"{cpu_s:.1f} s"},
    }


SPLIT_CANDIDATES = (256, 512, 768, 1024, 1536, 2048, 2688, 3072)
# equal-length batches: ((query heads, KV heads, head_dim), sessions, tokens, name)
SPLIT_SWEEP_SHAPES = [
    ((32, 8, 128), 8, 8257, "C5 tp1"), ((16, 4, 128), 8, 8257, "C5 tp2"), ((4, 1, 128), 8, 8257, "C5 tp8"),
    ((32, 8, 128), 4, 4096, "b4 4k"), ((32, 8, 128), 16, 2048, "b16 2k"), ((32, 8, 128), 1, 131072, "b1 128k"),
    ((32, 8, 64), 4, 4096, "d64 b4 4k"), ((32, 8, 256), 2, 16384, "d256 b2 16k"),
    ((64, 2, 128), 3, 5000, "g32 b3 5k"), ((32, 8, 128), 32, 16384, "b32 16k"),
    ((32, 8, 128), 8, 32768, "b8 32k"), ((32, 8, 128), 2, 65536, "b2 64k"),
    ((16, 4, 128), 4, 4096, "tp2 b4 4k"), ((32, 8, 128), 64, 1024, "b64 1k"), ((8, 2, 128), 8, 16384, "tp4 b8 16k"),
]
SPLIT_SWEEP_SHARDS = [(1, 0), (2, 0), (2, 1), (4, 0), (4, 3), (8, 0), (8, 3), (8, 7)]


def _graph_us(torch, call, reps: int) -> float:
    """Median of three graph replays of `reps` calls, microseconds per call."""
    for _ in range(3):
        call()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.graph(graph, stream=side):
        for _ in range(reps):
            call()
    torch.cuda.current_stream().wait_stream(side)
    graph.replay()
    torch.cuda.synchronize()
    times = []
    for _ in range(3):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        graph.replay()
        b.record()
        torch.cuda.synchronize()
        times.append(a.elapsed_time(b) * 1e3 / reps)
    del graph
    return sorted(times)[1]


def bench_split_sweep(m, torch, device, args) -> None:
    """Every candidate split size of the split-KV decode, timed on one GPU:
    equal-length batches (dense caches, several rotating copies so the K/V
    streamed per graph replay exceeds L2) with the pick of the policy without
    host lengths, then the C4 shards of 1, 2, 4 and 8 GPUs (ColdStore pages)
    with the pick of mslim_cuda_decode_split_tokens_for_lengths.  One JSON
    line per case, microseconds per decode call."""
    import numpy as np
    from mslim_b200 import workloads
    for (qh, kvh, d), n_seq, L, name in SPLIT_SWEEP_SHAPES:
        g = m.AttentionGeometry.new(qh, kvh, d)
        cap = L + 3
        per = n_seq * cap * kvh * d * 4
        copies = max(1, -(-(512 << 20) // per))
        ks = [torch.randn((n_seq, cap, kvh, d), device=device, dtype=torch.bfloat16) for _ in range(copies)]
        vs = [torch.randn((n_seq, cap, kvh, d), device=device, dtype=torch.bfloat16) for _ in range(copies)]
        q = torch.randn((n_seq, qh, d), device=device, dtype=torch.bfloat16)
        seq = torch.full((n_seq,), L, dtype=torch.int32, device=device)
        ws = torch.zeros(m.decode_workspace_bytes(g, n_seq, cap, 256), dtype=torch.uint8, device=device)
        o = torch.empty((n_seq, qh, d), device=device, dtype=torch.bfloat16)
        us = {}
        for st in SPLIT_CANDIDATES:
            if st > max(256, (cap + 63) // 64 * 64) and st != SPLIT_CANDIDATES[-1]:
                continue   # one split per session, the same CTAs as the longest candidate

            def calls(st=st):
                for i in range(copies):
                    m.decode_dense(g, q, ks[i], vs[i], seq, n_seq, cap, ws, o, st)
            us[st] = _graph_us(torch, calls, max(4, 40 // copies)) / copies
        pick = m.decode_split_tokens(g, n_seq, cap)
        print(json.dumps({"case": name, "geometry": [qh, kvh, d], "sessions": n_seq, "tokens": L,
                          "max_tokens": cap, "us": {str(k): round(v, 2) for k, v in us.items()},
                          "policy": "mslim_cuda_decode_split_tokens", "pick": pick,
                          "fastest": min(us, key=us.get)}), flush=True)
        del ks, vs
        torch.cuda.empty_cache()
    layout = workloads.c4_layout(seed=3)
    lengths_all = layout.lengths[:64]
    for world, rank in SPLIT_SWEEP_SHARDS:
        lengths = lengths_all[lpt_shard(lengths_all, world, rank)].astype(np.int32)
        c4 = C4Pages(np, torch, device, m, lengths, seed=3 + rank)
        pick = c4.split_tokens
        c4.ws = torch.zeros(m.decode_workspace_bytes(c4.g, c4.n_seq, c4.max_pages * PAGE, 256),
                            dtype=torch.uint8, device=device)
        us = {}

        def c4_step():
            c4.stream = torch.cuda.current_stream()   # the capturing stream inside the graph
            c4.step()
        for st in SPLIT_CANDIDATES:
            c4.split_tokens = st
            us[st] = _graph_us(torch, c4_step, 40 if world >= 4 else 20)
        print(json.dumps({"case": f"C4 shard {rank}/{world}", "geometry": [QH, KVH, D], "sessions": c4.n_seq,
                          "tokens": c4.tokens, "us": {str(k): round(v, 2) for k, v in us.items()},
                          "policy": "mslim_cuda_decode_split_tokens_for_lengths", "pick": pick,
                          "fastest": min(us, key=us.get)}), flush=True)
        c4.close()
        del c4
        torch.cuda.empty_cache()
    if m.device_status(torch.cuda.current_device()) != 0:
        raise SystemExit("device status reported an error during the split sweep")


def bench_model(m, torch, device, args, rank, world, dist) -> dict | None:
    """C5: a Llama-3-8B-shaped decoder with random
    weights, batch 8, 8192-token prefill then 256 greedy decode steps,
    tensor-parallel over the WORLD_SIZE ranks by KV-head group (NCCL
    all-reduce of the row-parallel o-projection, and of the MLP down
    projection when the MLP is sharded).  Strong scaling: the model and the
    batch are fixed, the ranks split them.  Device time by CUDA events,
    barrier + synchronize around each timed region, max over ranks."""
    import hashlib

    import numpy as np
    from mslim_b200 import model as mdl

    B, S, steps = args.model_batch, args.model_prefill, args.model_steps
    spec = mdl.ModelSpec(layers=args.model_layers)
    L = spec.layer
    t0 = time.time()
    # decode projections: the own tcgen05 GEMV at every TP degree, its gate|up
    # projection with SwiGLU fused into the epilogue (measured faster per step
    # than cuBLAS at TP 1 and 2, and per shape at TP 8; `--gemv` times each shape)
    gemm = args.decode_gemm if args.decode_gemm != "auto" else "own"
    M = mdl.DeviceModel(spec, B, S + steps + 4, seed=5, tp_rank=rank, tp_world=world, mlp=args.mlp,
                        kv_mode=args.kv_mode, decode_gemm=gemm, fuse_qkv=args.decode_qkv == "fused")
    build_s = time.time() - t0
    ids = torch.from_numpy(np.random.default_rng(5).integers(0, spec.vocab, size=(B, S))).to(device)

    def sync():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x: float) -> float:
        if dist is None:
            return x
        v = torch.tensor([x], dtype=torch.float64, device=device)
        dist.all_reduce(v, op=dist.ReduceOp.MAX)
        return float(v.item())

    # warm-up: a short prompt and a few steps through the same kernels
    tok, _ = M.prefill(ids[:, :min(S, 256)])
    for _ in range(max(args.warmup, 3)):
        tok, _ = M.decode_step(tok)
    graphed = not args.no_graph
    if graphed:
        M.capture_decode()
        for _ in range(2):
            tok, _ = M.decode_step_graphed(tok)
    sync()
    sampler = ClockSampler(torch.cuda.current_device())
    sampler.start()
    e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
    e0.record()
    tok, _ = M.prefill(ids)
    e1.record()
    out = [tok.clone()]
    step = M.decode_step_graphed if graphed else M.decode_step
    for _ in range(steps):
        tok, _ = step(tok)
        out.append(tok.clone())
    e2.record()
    sync()
    clocks = sampler.stop()
    prefill_ms = max_over_ranks(e0.elapsed_time(e1))
    decode_ms = max_over_ranks(e1.elapsed_time(e2))
    tokens = torch.stack(out, 1).cpu().numpy().astype(np.int32)   # [B][steps + 1]
    # one more decode step, issued eagerly with CUDA events around every op.
    # A bounded spin kernel queued first keeps the GPU busy while the host
    # enqueues the whole step, so each op's events bracket its device time and
    # not the host's launch latency (ops run back to back, without the
    # programmatic-dependent-launch overlap of the graph).
    M.profile = mdl.SectionTimer(torch)
    torch.cuda._sleep(int(0.05 * 1.965e9))
    M.decode_step(tok)
    sync()
    step_split = M.profile.totals_ms()
    step_ops = M.profile.per_op()
    M.profile = None
    M.close()
    if m.device_status(torch.cuda.current_device()) != 0:
        raise SystemExit("device status reported an error during the model leg")
    if rank != 0:
        return None
    peaks = measured_peaks()
    kernels = []
    for e in step_ops:
        if e["ms"] <= 0.0 or e["bytes"] <= 0:
            continue
        gbs = e["bytes"] / (e["ms"] * 1e-3) / 1e9
        peak = peaks["hbm_gbs"] if e["link"] == "hbm" else NVLINK_PEER_GBS
        kernels.append({"op": e["op"], "kernel": e["kernel"], "launches": e["launches"],
                        "us_per_launch": 1e3 * e["ms"] / e["launches"], "bytes_per_launch": e["bytes"] // e["launches"],
                        "share_of_step": e["ms"] / sum(x["ms"] for x in step_ops),
                        "bound": e["link"], "achieved_gbs": gbs, "peak_gbs": peak, "frac": gbs / peak})
    kvh, qh = L.kv_heads // world, L.query_heads // world
    inter = L.intermediate if args.mlp == "replicated" else L.intermediate // world
    params_layer = L.hidden * (qh + 2 * kvh) * L.head_dim + L.hidden * qh * L.head_dim + 3 * L.hidden * inter
    ctx = S + steps / 2.0
    return {
        "metric": "C5 decode tokens/s (32-layer Llama-3-8B-shaped decoder, batch 8, prefill 8192, 256 greedy "
                  "steps, KV-head tensor parallel)",
        "value": B * steps / (decode_ms * 1e-3), "unit": "tokens/s", "n_gpus": world, "steps": steps,
        "higher_is_better": True, "scaling": "strong", "dtype": "bf16",
        "data": "synthetic (random-init weights: projections and tied embedding N(0,0.02), norms 1; "
                "prompt ids uniform [0,128256), seed 5)",
        "config": {"workload": "C5", "layers": spec.layers, "batch": B, "prefill": S, "decode_steps": steps,
                   "parallelism": f"tp{world} by KV-head group, MLP {args.mlp}", "kv": args.kv_mode,
                   "allreduce_per_layer": 1 if args.mlp == "replicated" else 2,
                   "decode_issue": "one CUDA graph per step" if graphed else "eager",
                   "decode_projections": "mslim_cuda_gemv" if gemm == "own" else "cuBLAS",
                   "decode_qkv": args.decode_qkv if gemm == "own" else "separate"},
        "prefill_ms": prefill_ms, "prefill_tokens_per_s": B * S / (prefill_ms * 1e-3),
        "decode_ms_per_step": decode_ms / steps,
        "decode_step_split_ms": step_split,
        "decode_step_kernels": kernels,
        "decode_step_split_note": "one extra step of rank 0 issued eagerly behind a bounded spin kernel, CUDA "
                                  "events around every op (device time of each op run alone, no launch gaps, "
                                  "no programmatic-dependent-launch overlap); the timed steps replay a graph. "
                                  "decode_step_kernels: per op its algorithmic bytes (weights, K/V, activations "
                                  "in and out) / its device time, against hbm_gbs of MEASURED_PEAKS.json, or "
                                  f"for NVLink the {NVLINK_PEER_GBS:.0f} GB/s per-direction peer copy measured "
                                  "on this pool",
        "per_rank_roofline": {
            "decode_weight_bytes_per_step": 2 * (params_layer * spec.layers + spec.vocab * L.hidden),
            "decode_weight_gbs": 2 * (params_layer * spec.layers + spec.vocab * L.hidden)
            / (step_split.get("gemm", 0.0) * 1e-3) / 1e9 if step_split.get("gemm") else None,
            "decode_attention_bytes_per_step": int(B * ctx * kvh * L.head_dim * 4 * spec.layers),
            "decode_attention_gbs": B * ctx * kvh * L.head_dim * 4 * spec.layers
            / (step_split.get("attention", 0.0) * 1e-3) / 1e9 if step_split.get("attention") else None,
            "hbm_peak_gbs": peaks["hbm_gbs"],
        },
        "tokens_sha256": hashlib.sha256(tokens.tobytes()).hexdigest(),
        "first_tokens": tokens[:, :8].tolist(),
        "model_build_s": build_s, "clocks": clocks,
    }


# --------------------------------------------------------------- GPU leg --

def main():
    args = parse()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank)
        return
    import numpy as np
    import torch
    import mslim_b200 as m
    from mslim_b200 import workloads

    torch.cuda.set_device(local)
    device = f"cuda:{local}"
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device(device))
    m.load()
    m.set_decode_schedule(m.DECODE_PERSISTENT if args.decode_schedule == "persistent" else m.DECODE_SPLIT_MERGE)
    if args.layer:
        print(json.dumps(bench_layer(m, torch, device, args)), flush=True)
        return
    if args.gemv:
        print(json.dumps(bench_gemv(m, torch, device, args)), flush=True)
        return
    if args.split_sweep:
        bench_split_sweep(m, torch, device, args)
        return
    if args.model:
        line = bench_model(m, torch, device, args, rank, world, dist)
        if line is not None:
            print(json.dumps(line), flush=True)
        if dist is not None:
            dist.barrier()
            dist.destroy_process_group()
        return
    if args.prefill_only:
        print(json.dumps({"prefill": bench_prefill(m, torch, device, args)}), flush=True)
        return

    layout = workloads.c4_layout(seed=3)
    all_sessions = list(range(min(args.sessions, len(layout.lengths))))
    shard_world, shard_rank = world, rank
    if args.shard_of:
        shard_rank, shard_world = (int(x) for x in args.shard_of.split("/"))
    strong = args.scaling == "strong" and shard_world > 1
    if strong:
        mine = lpt_shard(layout.lengths[all_sessions], shard_world, shard_rank)
    else:
        mine = all_sessions
    c4 = C4Pages(np, torch, device, m, layout.lengths[mine].astype(np.int32), seed=3 + rank,
                 split_tokens=args.split_tokens)

    def barrier():
        if dist is not None:
            dist.barrier()

    def max_over_ranks(x: float) -> float:
        if dist is None:
            return x
        t = torch.tensor([x], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def sum_over_ranks(*xs):
        if dist is None:
            return [float(x) for x in xs]
        t = torch.tensor(list(xs), device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        return [float(x) for x in t.tolist()]

    def per_rank(*xs):
        """[world][len(xs)] of every rank's values (rank order)."""
        t = torch.tensor([list(xs)], device=device, dtype=torch.float64)
        if dist is None:
            return t.tolist()
        every = torch.empty((world, len(xs)), device=device, dtype=torch.float64)
        dist.all_gather_into_tensor(every, t)
        return every.tolist()

    # ---- device-timed region (CUDA events on the launching stream) ----
    timed = c4.time_steps(args.steps, max(args.warmup, 3), local, barrier)
    elapsed_ms = max_over_ranks(timed["elapsed_ms"])
    total_bytes, total_seq, total_tokens = sum_over_ranks(c4.step_bytes, c4.n_seq, c4.tokens)
    total_seq = int(total_seq)
    ms_per_step = elapsed_ms / args.steps
    value = total_bytes / (ms_per_step * 1e-3) / 1e9
    ranks = per_rank(c4.tokens, c4.n_seq, c4.split_tokens, c4.ctas, timed["elapsed_ms"] / args.steps)
    status = m.device_status(local)

    # ---- end-to-end leg: the C-ABI calls a decode step makes, host buffers ----
    e2e = None
    if not args.no_e2e:
        e = c4.time_e2e(args.steps, barrier)
        e_ms = max_over_ranks(e["ms"])
        e_bytes, = sum_over_ranks(e["bytes"])
        e2e = {"value": e_bytes / (e_ms / args.steps * 1e-3) / 1e9, "unit": "GB/s",
               "h2d_bytes_per_step": e["h2d"] * world, "d2h_bytes_per_step": e["d2h"] * world,
               "ms_per_step": e_ms / args.steps,
               "path": "pinned host q/k/v -> mslim_cuda_rope_append_decode_paged -> mslim_cuda_decode_paged "
                       "-> host output; the step's copies and launches replayed as one CUDA graph, the "
                       "host waits for every step's result"}
        if m.device_status(local) != 0:
            raise SystemExit("device status reported an error during the e2e leg")
    timed_launches_per_step = timed["launches"] / args.steps
    c4_local = {"step_bytes": c4.step_bytes, "launch_ms": timed["launch_ms"], "n_seq": c4.n_seq,
                "lengths": c4.lengths}
    c4.close()
    del c4
    torch.cuda.empty_cache()

    # ---- weak scaling beside the strong headline (N > 1): every rank its own 64 sessions ----
    weak = None
    if strong and world > 1 and not args.no_weak:
        w4 = C4Pages(np, torch, device, m, layout.lengths[all_sessions].astype(np.int32), seed=3 + rank,
                     split_tokens=args.split_tokens)
        wt = w4.time_steps(args.steps, max(args.warmup, 3), local, barrier)
        w_ms = max_over_ranks(wt["elapsed_ms"]) / args.steps
        w_bytes, w_seq = sum_over_ranks(w4.step_bytes, w4.n_seq)
        weak = {"value": w_bytes / (w_ms * 1e-3) / 1e9, "unit": "GB/s", "ms_per_step": w_ms,
                "global_sessions": int(w_seq), "sessions_per_gpu": w4.n_seq,
                "note": "every rank decodes its own copy of the 64 C4 sessions (weak scaling)"}
        w4.close()
        del w4
        torch.cuda.empty_cache()

    prefill = None
    if rank == 0 and not args.no_prefill:
        prefill = bench_prefill(m, torch, device, args)
        torch.cuda.empty_cache()

    # ---- C5 leg: the tensor-parallel decoder over the same ranks ----
    model = None
    if not args.no_model:
        margs = argparse.Namespace(**vars(args))
        margs.model_steps = args.model_leg_steps
        barrier()
        model = bench_model(m, torch, device, margs, rank, world, dist)
        torch.cuda.empty_cache()

    if rank != 0:
        if dist is not None:
            dist.barrier()
            dist.destroy_process_group()
        return

    peaks = measured_peaks()
    step_bytes = c4_local["step_bytes"]
    achieved = step_bytes / (c4_local["launch_ms"] * 1e-3) / 1e9
    traffic = profile_traffic("decode_c4_traffic.json")
    roofline = {"bound": "hbm", "kernel": ("mslim_decode_persist (split-KV with the merge in-kernel)"
                                           if timed_launches_per_step == 1 else
                                           "mslim_decode_split + mslim_decode_merge_row"),
                "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                "frac": achieved / peaks["hbm_gbs"] if peaks["hbm_gbs"] else None,
                "peak_source": f"{peaks['source']} (MEASURED_PEAKS.json hbm_gbs)" if peaks["source"] == "measured"
                else "fallback 6650 GB/s",
                "traffic": (int(traffic["traffic_over_algorithmic"] * step_bytes) if traffic else None),
                "traffic_source": ("scaled from profiles/decode_c4_traffic.json, not measured in this run: one "
                                   "ncu capture of 8 C4 sessions gave DRAM bytes / algorithmic bytes = "
                                   f"{traffic['traffic_over_algorithmic']:.4f}, applied to this launch's "
                                   "algorithmic bytes" if traffic else None),
                "algorithmic_bytes_per_launch": step_bytes,
                "achieved_note": "rank 0's algorithmic bytes / its per-step time (the graph replay of the K steps "
                                 "between CUDA events, divided by K): every kernel of a step"}
    cpu = None
    if not args.no_cpu and world == 1:
        cpu = cpu_sample_gbs(c4_local["lengths"][:4], args.cpu_seconds)
    rank_tokens = [r[0] for r in ranks]
    mean_tokens = sum(rank_tokens) / len(rank_tokens)
    line = {"metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
            "scaling": "strong" if (strong or world == 1) and args.scaling == "strong" else "weak",
            "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded N(0,1) bf16 K/V/Q; no dataset)",
            "config": {"workload": "C4 batched long-context decode: 64 sessions with L ~ U[4096,32768] (seed 3), "
                                   "256-token ColdStore-exact pages in a random physical permutation, "
                                   "QH 32 / KVH 8 / D 128, one query per session",
                       "sessions_per_gpu": c4_local["n_seq"], "global_sessions": total_seq, "page_tokens": PAGE,
                       "split_tokens": [int(r[2]) for r in ranks],
                       "split_tokens_source": ("--split-tokens" if args.split_tokens else
                                               "mslim_cuda_decode_split_tokens_for_lengths on each rank's "
                                               "host-side session lengths"),
                       "l2": "no flush: inputs larger than L2 (%.2f GB per GPU per step)" % (step_bytes / 1e9),
                       "issue": "the K timed steps captured as one CUDA graph and replayed once",
                       "decode_schedule": ("persistent" if m.get_decode_schedule() == m.DECODE_PERSISTENT
                                           else "split + merge"),
                       "parallelism": (f"sessions LPT-sharded over {world} GPUs (strong: one 64-session C4 draw)"
                                       if strong else
                                       f"session-sharded x{world} ({args.scaling})"),
                       **({"shard_of": args.shard_of} if args.shard_of else {})},
            "tokens_per_s": total_seq / (ms_per_step * 1e-3),
            "eager_ms_per_step": timed["eager_ms"],
            "per_rank": {"tokens": rank_tokens, "sessions": [int(r[1]) for r in ranks],
                         "split_tokens": [int(r[2]) for r in ranks], "split_ctas": [int(r[3]) for r in ranks],
                         "ms_per_step": [r[4] for r in ranks],
                         "token_imbalance_max_over_mean": max(rank_tokens) / mean_tokens if mean_tokens else None},
            "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e, "prefill": prefill,
            "weak": weak, "model": model,
            "gpu_launches": timed["launches"],
            "gpu_launches_note": "the library's kernel launches recorded into the timed graph "
                                 "(mslim_cuda_kernel_launches before and after its capture)",
            "clocks": timed["clocks"], "device_status": status}
    print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


class C4Pages:
    """One rank's C4 sessions in 256-token ColdStore-exact pages (random
    physical permutation) with the decode's query, output and workspace."""

    def __init__(self, np, torch, device, m, lengths, seed: int, split_tokens: int = 0):
        self.np, self.torch, self.device, self.m = np, torch, device, m
        self.lengths = lengths
        self.n_seq = n_seq = len(lengths)
        # pages for L + 1 tokens: the e2e leg appends the step's new token at L
        pages = (lengths + 1 + PAGE - 1) // PAGE
        self.n_pages = n_pages = int(pages.sum())
        rng = np.random.default_rng(seed)
        perm = rng.permutation(n_pages).astype(np.int32)
        self.max_pages = max_pages = int(pages.max())
        table = np.zeros((n_seq, max_pages), np.int32)
        cur = 0
        for s in range(n_seq):
            table[s, :pages[s]] = perm[cur:cur + pages[s]]
            cur += pages[s]
        gen = torch.Generator(device=device)
        gen.manual_seed(seed)
        self.k_pool = torch.randn((n_pages, KVH, PAGE, D), generator=gen, device=device, dtype=torch.bfloat16)
        self.v_pool = torch.randn((n_pages, KVH, PAGE, D), generator=gen, device=device, dtype=torch.bfloat16)
        self.q = torch.randn((n_seq, QH, D), generator=gen, device=device, dtype=torch.bfloat16)
        self.out = torch.empty((n_seq, QH, D), device=device, dtype=torch.bfloat16)
        self.table_d = torch.from_numpy(table).to(device)
        self.seq_d = torch.from_numpy(lengths).to(device)
        self.g = m.AttentionGeometry.new(QH, KVH, D)
        max_tokens = max_pages * PAGE
        # the split size for this rank's sessions from their host-side lengths
        # (fewest waves of split CTAs), as a serving host that tracks its
        # sessions' lengths would choose it
        self.split_tokens = split_tokens or m.decode_split_tokens_for_lengths(self.g, lengths)
        self.ws = torch.zeros(m.decode_workspace_bytes(self.g, n_seq, max_tokens, self.split_tokens),
                              dtype=torch.uint8, device=device)
        self.ctas = int(sum(-(-int(L) // self.split_tokens) for L in lengths)) * KVH
        self.tokens = int(lengths.astype(np.int64).sum())
        self.step_bytes = self.tokens * KVH * D * 4 + n_seq * QH * D * 4 + int(((lengths + PAGE - 1) // PAGE).sum()) * 4
        self.stream = torch.cuda.current_stream()

    def step(self):
        self.m.decode_paged(self.g, self.q, self.k_pool, self.v_pool, self.n_pages, PAGE, self.table_d,
                            self.max_pages, self.seq_d, self.n_seq, self.ws, self.out, self.split_tokens,
                            self.stream)

    def time_steps(self, steps: int, warmup: int, local: int, barrier) -> dict:
        """The K timed decode steps are captured once as a CUDA graph (the way a
        serving loop issues its decode steps) and replayed once between two
        CUDA events; the same K steps issued one by one from the host are
        timed beside it (`eager_ms`)."""
        torch = self.torch
        for _ in range(warmup):
            self.step()
        torch.cuda.synchronize()
        if self.m.device_status(local) != 0:
            raise SystemExit("device status reported a bounded wait timeout during warm-up")
        graph = torch.cuda.CUDAGraph()
        cap = torch.cuda.Stream()
        cap.wait_stream(self.stream)
        main_stream = self.stream
        self.stream = cap
        launches0 = self.m.kernel_launches()
        with torch.cuda.graph(graph, stream=cap, capture_error_mode="thread_local"):
            for _ in range(steps):
                self.step()
        captured = self.m.kernel_launches() - launches0  # the library's kernels in the timed graph
        self.stream = main_stream
        torch.cuda.synchronize()
        graph.replay()  # one untimed replay: the graph's first launch uploads it
        torch.cuda.synchronize()
        sampler = ClockSampler(local)
        barrier()
        torch.cuda.synchronize()
        sampler.start()
        t_start = torch.cuda.Event(enable_timing=True)
        t_end = torch.cuda.Event(enable_timing=True)
        t_start.record(self.stream)
        graph.replay()
        t_end.record(self.stream)
        torch.cuda.synchronize()
        barrier()
        clocks = sampler.stop()
        elapsed = t_start.elapsed_time(t_end)
        del graph
        # the same steps issued one by one
        torch.cuda.synchronize()
        t_start.record(self.stream)
        for _ in range(steps):
            self.step()
        t_end.record(self.stream)
        torch.cuda.synchronize()
        return {"elapsed_ms": elapsed, "launch_ms": elapsed / steps, "eager_ms": t_start.elapsed_time(t_end) / steps,
                "clocks": clocks, "launches": captured}

    def time_e2e(self, steps: int, barrier) -> dict:
        """Per step: the new token's q, k and v of every session from one
        pinned host buffer -> RoPE + paged append -> split-KV decode -> the
        output back in pinned host memory, captured once as a CUDA graph and
        replayed; the host waits for every step's result."""
        torch, np, m = self.torch, self.np, self.m
        n_seq, lengths, stream = self.n_seq, self.lengths, self.stream
        rope_cfg = m.RopeKernelConfig(theta=500000.0)
        nq_el, nkv_el = n_seq * QH * D, 2 * n_seq * KVH * D
        in_host = torch.empty(nq_el + nkv_el, dtype=torch.bfloat16).pin_memory()
        in_host[:nq_el].copy_(torch.randn(nq_el, generator=torch.Generator().manual_seed(5)).to(torch.bfloat16))
        in_host[nq_el:].copy_(torch.randn(nkv_el, generator=torch.Generator().manual_seed(6)).to(torch.bfloat16))
        out_host = torch.empty((n_seq, QH, D), dtype=torch.bfloat16).pin_memory()
        in_dev = torch.empty(nq_el + nkv_el, device=self.device, dtype=torch.bfloat16)
        q_in = in_dev[:nq_el].view(n_seq, QH, D)
        kv_in = in_dev[nq_el:].view(2, n_seq, KVH, D)
        q_rot = torch.empty_like(self.q)
        pos_d = torch.from_numpy(lengths).to(self.device)          # new token at position L
        seq1_d = torch.from_numpy(lengths + 1).to(self.device)     # then attend over L + 1

        def calls(st):
            in_dev.copy_(in_host, non_blocking=True)
            m.rope_append_decode_paged(self.g, q_in, q_rot, kv_in[0], kv_in[1], pos_d, n_seq, rope_cfg,
                                       self.k_pool, self.v_pool, self.n_pages, PAGE, self.table_d,
                                       self.max_pages, st)
            m.decode_paged(self.g, q_rot, self.k_pool, self.v_pool, self.n_pages, PAGE, self.table_d,
                           self.max_pages, seq1_d, n_seq, self.ws, self.out, self.split_tokens, st)
            out_host.copy_(self.out, non_blocking=True)

        calls(stream)
        stream.synchronize()
        graph = torch.cuda.CUDAGraph()
        cap = torch.cuda.Stream()
        cap.wait_stream(stream)
        # thread-local capture: other threads of the process (the process
        # group's) may touch CUDA while this thread captures
        with torch.cuda.graph(graph, stream=cap, capture_error_mode="thread_local"):
            calls(torch.cuda.current_stream())
        torch.cuda.synchronize()

        def e2e_step():
            graph.replay()
            stream.synchronize()

        for _ in range(3):
            e2e_step()
        e_bytes = int((lengths + 1).astype(np.int64).sum()) * KVH * D * 4 + n_seq * QH * D * 4 + int(
            ((lengths + 1 + PAGE - 1) // PAGE).sum()) * 4
        barrier()
        torch.cuda.synchronize()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(steps):
            e2e_step()
        b.record(stream)
        torch.cuda.synchronize()
        ms = a.elapsed_time(b)
        del graph
        return {"ms": ms, "bytes": e_bytes, "h2d": int(in_host.numel() * 2), "d2h": int(out_host.numel() * 2)}

    def close(self):
        for name in ("k_pool", "v_pool", "q", "out", "ws", "table_d", "seq_d"):
            setattr(self, name, None)


if __name__ == "__main__":
    main()
