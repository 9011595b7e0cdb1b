"""Benchmark of the Satori decode hot path on B200 (one JSON line on rank 0).

Default workload (the configuration its MatVec metric is quoted on):
one step = one GGUF Q8_0 4096x4096 MatVec plus one Q4_0 11008x4096 MatVec in the decode
(ExecuteBatch) order, over seeded N(0, 0.02^2) weights and an N(0,1) input.  The step rotates
through enough distinct weight copies that the timed working set (several times the 126 MB L2)
streams from HBM on every launch.  value = payload GB/s (weights incl. scales).

--gpus N (torchrun): weak scaling; every rank processes its own independent matrices (no
data-path collective; the path shards by object); value = all ranks' bytes / max-over-ranks time.

Other workloads (for the profiles and the design tables): --workload attention | ternary | decode7b |
decode1p5b.  --impl reference times the reference's CPU path (the C restatement of
ExecuteBatchFloat, all host threads) on the same config and metric.
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

import numpy as np  # noqa: E402

GB = 1e9


def _peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as fh:
            p = json.load(fh)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


# ------------------------------------------------------------------ clocks sampler
class ClockSampler:
    """nvidia-smi sampling during the timed region (SM clock median, throttle reasons)."""

    def __init__(self, index: int):
        self.index = index
        self.samples = []
        self._proc = None

    def __enter__(self):
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self._proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={q}", "--format=csv,noheader,nounits",
                                           "-i", str(self.index), "-lms", "100"],
                                          stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
            time.sleep(0.3)
        except Exception:
            self._proc = None
        return self

    def _read(self):
        for line in self._proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                self.samples.append(parts)

    def __exit__(self, *exc):
        if self._proc:
            time.sleep(0.15)
            self._proc.terminate()
            try:
                self._proc.wait(timeout=5)
            except Exception:
                self._proc.kill()

    def summary(self):
        def num(s):
            try:
                return float(s)
            except ValueError:
                return None
        sm = [v for v in (num(s[1]) for s in self.samples) if v is not None]
        mx = [v for v in (num(s[2]) for s in self.samples) if v is not None]
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for s in self.samples:
            for n, v in zip(names, s[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(self.samples)}


# ------------------------------------------------------------------ distributed plumbing
def dist_init():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    return rank, world, local


def dist_max(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def dist_barrier(world: int):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


# ------------------------------------------------------------------ device helpers
def device_quantized(ctx, rows, cols, fmt, seed, sigma=0.02):
    """Seeded N(0, sigma^2) weights generated and quantized on the device (this library's quantizer)."""
    import torch

    from satori_b200 import _lib
    g = torch.Generator(device="cuda").manual_seed(seed)
    w = torch.randn(rows * cols, generator=g, device="cuda", dtype=torch.float32) * sigma
    bb = 34 if fmt == 0 else 18
    out = torch.empty(rows * (cols // 32) * bb, dtype=torch.uint8, device="cuda")
    torch.cuda.synchronize()  # the quantizer runs on the library's stream, not torch's
    _lib.check(_lib.lib().satori_quantize_q_device(ctx.handle, w.data_ptr(), rows, cols, fmt, out.data_ptr()),
               "quantize")
    ctx.synchronize()
    del w
    return out


def events_time(fn, stream, steps: int) -> float:
    """Device time (ms) of `steps` calls of fn() bracketed by CUDA events on `stream`."""
    import torch
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):  # CUDAGraph.replay() launches on the current stream
        start.record(stream)
        for _ in range(steps):
            fn()
        end.record(stream)
    torch.cuda.synchronize()
    return start.elapsed_time(end)


# ------------------------------------------------------------------ MatVec workload
MATVEC_SHAPES = [(0, 4096, 4096), (1, 11008, 4096)]
MATVEC_METRIC = "MatVec payload GB/s (GGUF Q8_0 4096x4096 + Q4_0 11008x4096, decode ExecuteBatch order)"
MATVEC_WORKLOAD = "configs[1]: GGUF Q8_0 4096x4096 and Q4_0 11008x4096 MatVec"
# dram__bytes_read.sum + dram__bytes_write.sum per launch, averaged over the two kernels, from one ncu
# capture of this workload (Q8_0 17,875,712 + Q4_0 25,412,352 bytes; profiles/gemv_rows_matvec_bench.md).
MATVEC_NCU_TRAFFIC = (17875712 + 25412352) / 2


def bench_matvec(args, rank, world, local):
    import torch

    import satori_b200 as sat
    from satori_b200 import _lib
    ctx = sat.Context(local)
    step_bytes = sum(r * (c // 32) * (34 if f == 0 else 18) for f, r, c in MATVEC_SHAPES)
    copies = max(1, int(args.copies))
    mats = []
    for c in range(copies):
        for fmt, rows, cols in MATVEC_SHAPES:
            dev = device_quantized(ctx, rows, cols, fmt, seed=1000 * rank + 10 * c + fmt)
            mats.append(sat.CudaQuantizedMatrix.from_device(ctx, dev.data_ptr(), dev.numel(), rows, cols, fmt))
            del dev
    gen = torch.Generator(device="cuda").manual_seed(77)
    x = torch.randn(4096, generator=gen, device="cuda", dtype=torch.float32)
    y = torch.empty(11008, device="cuda", dtype=torch.float32)
    torch.cuda.synchronize()
    stream = torch.cuda.Stream()
    ctx.set_stream(stream.cuda_stream)

    def one_step(i):
        for k in range(2):
            mats[2 * (i % copies) + k].execute_device(x.data_ptr(), y.data_ptr(), 1, _lib.ORDER_BATCH)

    # Warm-up outside capture, then capture the rotation (copies steps) into one CUDA graph.
    with torch.cuda.stream(stream):
        for i in range(args.warmup):
            one_step(i)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for i in range(copies):
            one_step(i)
    torch.cuda.synchronize()
    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()
    replays = max(1, args.steps // copies)
    steps = replays * copies
    dist_barrier(world)
    with ClockSampler(local) as clocks:
        ms = events_time(graph.replay, stream, replays)
    ms = dist_max(ms, world)
    launches = steps * 2
    value = step_bytes * steps * world / (ms / 1e3) / GB
    achieved = step_bytes * steps / (ms / 1e3) / GB   # per GPU: the kernel's algorithmic bytes / device time

    # e2e through the public C ABI with host buffers: H2D x, MatVec, D2H y per call (pinned staging).
    ctx.set_stream(None)
    xh = np.random.default_rng(5).standard_normal(4096).astype(np.float32)
    for m in mats:
        m.execute_batch(xh, 1)
    e2e_steps = max(4, min(steps, 200))
    dist_barrier(world)
    t0 = time.perf_counter()
    for i in range(e2e_steps):
        for k in range(2):
            mats[2 * (i % copies) + k].execute_batch(xh, 1)
    e2e_s = dist_max(time.perf_counter() - t0, world)
    e2e_value = step_bytes * e2e_steps * world / e2e_s / GB
    peak, peak_kind = _peaks()
    result = {
        "metric": MATVEC_METRIC,
        "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": steps, "warmup": args.warmup,
        "ms_per_step": round(ms / steps, 5), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "q8_0/q4_0 weights, f32 activations and accumulation",
        "data": "synthetic: seeded N(0,0.02^2) weights quantized on the device, N(0,1) input",
        "config": {"workload": MATVEC_WORKLOAD,
                   "order": "ExecuteBatch (decode) FP32 order, bit-exact to the reference",
                   "weight_copies_rotated": copies, "working_set_MB": round(step_bytes * copies / 1e6, 1),
                   "l2_policy": "inputs larger than L2: rotating distinct weight copies",
                   "parallelism": f"replicas x{world} (independent matrices per rank)"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                     "traffic": MATVEC_NCU_TRAFFIC, "traffic_source": "profiles/gemv_rows_matvec_bench.md",
                     "algorithmic_bytes_per_launch": step_bytes / 2},
        "e2e": {"value": round(e2e_value, 2), "unit": "GB/s", "h2d_bytes_per_step": 2 * 4096 * 4,
                "d2h_bytes_per_step": (4096 + 11008) * 4},
        "gpu_launches": launches,
        "clocks": clocks.summary(),
    }
    for m in mats:
        m.dispose()
    return result


def cpu_baseline_matvec(budget_s: float = 10.0):
    """The C restatement of ExecuteBatchFloat + Dot (AVX2+FMA) on all host threads, bounded sample."""
    from oracle import oracle
    threads = os.cpu_count() or 1
    rng = np.random.default_rng(3)
    data = []
    for fmt, rows, cols in MATVEC_SHAPES:
        w = rng.standard_normal(rows * cols, dtype=np.float32) * np.float32(0.02)
        data.append((oracle.q_quantize(w, rows, cols, fmt), rows, cols, fmt))
    x = rng.standard_normal(4096).astype(np.float32)
    step_bytes = sum(p.size for p, *_ in data)
    for p, r, c, f in data:
        oracle.q_matvec(p, r, c, f, x, order="batch", threads=threads)
    n, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < budget_s:
        for p, r, c, f in data:
            oracle.q_matvec(p, r, c, f, x, order="batch", threads=threads)
        n += 1
    dt = time.perf_counter() - t0
    return {"value": round(step_bytes * n / dt / GB, 3), "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"{n} steps (Q8_0 4096x4096 + Q4_0 11008x4096, ExecuteBatchFloat order) in {dt:.1f}s"}


# ------------------------------------------------------------------ attention workload
def bench_attention(args, rank, world, local):
    import torch

    import satori_b200 as sat
    from satori_b200 import _lib
    ctx = sat.Context(local)
    qh, kvh, hd = 28, 4, 128
    T = int(args.tokens)
    kv_bytes = 2 * T * kvh * hd * 4
    layers = max(2, int(np.ceil(4 * 126e6 / kv_bytes)))
    gen = torch.Generator(device="cuda").manual_seed(9)
    kc = torch.randn(layers, T * kvh * hd, generator=gen, device="cuda")
    vc = torch.randn(layers, T * kvh * hd, generator=gen, device="cuda")
    q = torch.randn(qh * hd, generator=gen, device="cuda")
    out = torch.empty(qh * hd, device="cuda")
    torch.cuda.synchronize()
    stream = torch.cuda.Stream()
    ctx.set_stream(stream.cuda_stream)
    L = _lib.lib()

    def call(i):
        _lib.check(L.satori_grouped_attention_device(ctx.handle, q.data_ptr(), kc[i % layers].data_ptr(),
                                                     vc[i % layers].data_ptr(), qh, kvh, hd, T, out.data_ptr()))

    with torch.cuda.stream(stream):
        for i in range(args.warmup):
            call(i)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for i in range(layers):
            call(i)
    graph.replay()
    torch.cuda.synchronize()
    replays = max(1, args.steps // layers)
    dist_barrier(world)
    with ClockSampler(local) as clocks:
        ms = events_time(graph.replay, stream, replays)
    ms = dist_max(ms, world)
    steps = replays * layers
    per = ms / steps
    peak, peak_kind = _peaks()
    achieved = kv_bytes / (per / 1e3) / GB
    return {
        "metric": f"decode attention K+V GB/s (28q/4kv x 128, T={T})",
        "value": round(kv_bytes * steps * world / (ms / 1e3) / GB, 2), "unit": "GB/s",
        "n_gpus": world, "steps": steps, "warmup": args.warmup, "ms_per_step": round(per, 5),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic N(0,1) q/k/v",
        "config": {"workload": f"configs[2]: GQA 28/4 x 128, T={T}", "layers_rotated": layers},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "peak_kind": peak_kind, "traffic": None,
                     "algorithmic_bytes_per_launch": kv_bytes},
        "gpu_launches": steps * 2, "clocks": clocks.summary(),
    }


# ------------------------------------------------------------------ Ternary2 workload
def bench_ternary(args, rank, world, local):
    import torch

    import satori_b200 as sat
    from satori_b200 import _lib
    from satori_b200.core import ternary2_byte_length
    ctx = sat.Context(local)
    n, bs = int(args.n), int(args.block)
    nbytes = ternary2_byte_length(n, n, bs)
    copies = max(4, int(np.ceil(4 * 126e6 / nbytes)))
    base = []
    rng = np.random.default_rng(1)
    w = rng.standard_normal(n * n).astype(np.float32)
    for c in range(4):
        base.append(sat.Ternary2Matrix.quantize(np.roll(w, c * 7919), n, n, bs, ctx=ctx).device)
    mats = list(base)
    while len(mats) < copies:
        src = base[len(mats) % 4]
        mats.append(sat.CudaQuantizedMatrix.from_device(ctx, src.device_payload, nbytes, n, n, bs))
    x = torch.randn(n, device="cuda")
    y = torch.empty(n, device="cuda")
    torch.cuda.synchronize()
    stream = torch.cuda.Stream()
    ctx.set_stream(stream.cuda_stream)
    order = _lib.ORDER_EXECUTE if args.order == "execute" else _lib.ORDER_SCALAR
    with torch.cuda.stream(stream):
        for m in mats[:args.warmup]:
            m.execute_device(x.data_ptr(), y.data_ptr(), 1, order)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for m in mats:
            m.execute_device(x.data_ptr(), y.data_ptr(), 1, order)
    graph.replay()
    torch.cuda.synchronize()
    replays = max(1, args.steps // copies)
    dist_barrier(world)
    with ClockSampler(local) as clocks:
        ms = events_time(graph.replay, stream, replays)
    ms = dist_max(ms, world)
    steps = replays * copies
    per = ms / steps
    peak, peak_kind = _peaks()
    achieved = nbytes / (per / 1e3) / GB
    return {"metric": f"Ternary2 MatVec payload GB/s ({n}x{n}, block {bs}, {args.order} order)",
            "value": round(nbytes * steps * world / (ms / 1e3) / GB, 2), "unit": "GB/s", "n_gpus": world,
            "steps": steps, "warmup": args.warmup, "ms_per_step": round(per, 5), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "ternary2 weights, f32", "data": "synthetic N(0,1)",
            "config": {"workload": f"configs[0]: Ternary2 {n}^2 bs{bs}", "copies": copies},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_kind": peak_kind, "traffic": None,
                         "algorithmic_bytes_per_launch": nbytes},
            "gpu_launches": steps, "clocks": clocks.summary()}


# ------------------------------------------------------------------ decode workloads
def device_model(ctx, spec, seed):
    import torch
    tensors = {}
    for i, (name, (rows, cols)) in enumerate(spec.matrix_shapes().items()):
        tensors[name] = device_quantized(ctx, rows, cols, spec.format_of(name), seed + i)
    g = torch.Generator(device="cuda").manual_seed(seed)
    for name, n in spec.vector_shapes().items():
        if name.endswith("norm.weight"):
            tensors[name] = 1.0 + 0.1 * torch.randn(n, generator=g, device="cuda")
        else:
            tensors[name] = 0.02 * torch.randn(n, generator=g, device="cuda")
    return tensors


def bench_decode(args, rank, world, local, spec):
    import torch

    import satori_b200 as sat
    ctx = sat.Context(local)
    context = args.prompt + args.decode + 8
    tensors = device_model(ctx, spec, seed=31)
    torch.cuda.synchronize()
    if world == 1:
        sess = sat.CudaDenseSession(spec, tensors, context, ctx=ctx)
    else:
        sess = sat.CudaDenseSession(spec, tensors, context, ctx=ctx, rank=rank, world=world,
                                    nccl_id=sat.broadcast_nccl_id())
    del tensors
    torch.cuda.empty_cache()
    prompt = np.random.default_rng(4).integers(0, spec.vocab, args.prompt).astype(np.int32)
    last = sess.prefill(prompt)
    ext = torch.cuda.ExternalStream(ctx.stream)
    torch.cuda.synchronize()
    dist_barrier(world)
    with ClockSampler(local) as clocks:
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(ext)
        t0 = time.perf_counter()
        toks = sess.generate(int(last), args.decode)
        wall = time.perf_counter() - t0
        end.record(ext)
        torch.cuda.synchronize()
    ms = dist_max(start.elapsed_time(end), world)
    tps = args.decode / (ms / 1e3)
    wbytes = spec.weight_bytes(include_embedding_table=False) + spec.hidden // 32 * 34
    kv_avg = 2 * spec.layers * spec.kv_width * 4 * (args.prompt + args.decode / 2)
    # Per GPU: a 1/world row share of every matrix and the KV heads of this rank's query heads.
    achieved = (wbytes + kv_avg) / world / (ms / 1e3 / args.decode) / GB
    peak, peak_kind = _peaks()
    return {"metric": f"decode tokens/s ({spec.name})", "value": round(tps, 2), "unit": "tokens/s",
            "n_gpus": world, "steps": args.decode, "warmup": args.prompt, "ms_per_step": round(ms / args.decode, 4),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "quantized weights, f32 activations", "data": "synthetic seeded weights, random prompt",
            "config": {"workload": spec.name, "prompt": args.prompt, "decode": args.decode,
                       "parallelism": "single GPU" if world == 1 else
                       f"tp{world}: row-sharded projections, query-head-sharded attention, all-gathers",
                       "exchange": None if world == 1 else os.environ.get("SATORI_EXCHANGE", "p2p")},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_kind": peak_kind, "traffic": None,
                         "algorithmic_bytes_per_launch": wbytes + kv_avg},
            "e2e": {"value": round(args.decode / wall, 2), "unit": "tokens/s", "h2d_bytes_per_step": 4,
                    "d2h_bytes_per_step": 4},
            "first_tokens": [int(t) for t in toks[:8]], "clocks": clocks.summary()}


# ------------------------------------------------------------------ reference arm
def reference_arm(args, rank, world):
    if rank != 0:
        return None
    base = cpu_baseline_matvec(budget_s=max(3.0, min(20.0, 0.05 * args.steps)))
    return {"metric": MATVEC_METRIC, "value": base["value"], "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "impl": "reference", "dtype": "q8_0/q4_0 weights, f32", "data": "synthetic seeded",
            "config": {"workload": MATVEC_WORKLOAD,
                       "implementation": "C restatement of QuantizedMatVec.ExecuteBatchFloat/Dot (AVX2+FMA), all "
                                         "host threads (the C# reference cannot be built in this image)"},
            "cpu_baseline": base, "e2e": {"value": base["value"], "unit": "GB/s", "h2d_bytes_per_step": 0,
                                          "d2h_bytes_per_step": 0}}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=600)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="satori", choices=["satori", "reference"])
    ap.add_argument("--workload", default="matvec",
                    choices=["matvec", "attention", "ternary", "decode7b", "decode1p5b"])
    ap.add_argument("--copies", type=int, default=12)
    ap.add_argument("--tokens", type=int, default=32768)
    ap.add_argument("--n", type=int, default=4096)
    ap.add_argument("--block", type=int, default=128)
    ap.add_argument("--order", default="execute", choices=["execute", "scalar"])
    ap.add_argument("--prompt", type=int, default=2048)
    ap.add_argument("--decode", type=int, default=256)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    if args.impl == "reference":
        rank = int(os.environ.get("RANK", "0"))
        world = int(os.environ.get("WORLD_SIZE", "1"))
        res = reference_arm(args, rank, world)
        if res is not None:
            print(json.dumps(res), flush=True)
        return
    rank, world, local = dist_init()
    import satori_b200 as sat
    if args.workload == "matvec":
        res = bench_matvec(args, rank, world, local)
        if rank == 0 and world == 1 and not args.no_cpu_baseline:
            res["cpu_baseline"] = cpu_baseline_matvec()
    elif args.workload == "attention":
        res = bench_attention(args, rank, world, local)
    elif args.workload == "ternary":
        res = bench_ternary(args, rank, world, local)
    elif args.workload == "decode7b":
        res = bench_decode(args, rank, world, local, sat.qwen2_7b())
    else:
        res = bench_decode(args, rank, world, local, sat.qwen2_1_5b())
    if rank == 0 and res is not None:
        print(json.dumps(res), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
