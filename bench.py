"""Benchmark of the Satori decode hot path on B200 (one JSON line on rank 0).

Default workload -- BASELINE.json's decode metric, configs[4]: greedy decode of the Qwen2-style 7B
shape (hidden 3584, 28 layers, 28/4 heads x 128, FFN 18944, vocab 152064; Q4_0 projections, Q8_0
embedding and lm_head, seeded N(0, 0.02^2) weights quantized on the device).  A 2048-token random
prompt is cached once; one step = 256 greedy tokens decoded from that context (the session is
rewound to position 2048 before every step, so every step decodes the same positions).
value = tokens/s of the whole job.

--gpus N (torchrun, one process per GPU): the same model row-sharded over N GPUs (every projection
split by rows, attention by query heads, vectors all-gathered over NVLink inside the step graph):
strong scaling, value = tokens / max-over-ranks device time.

Before timing, at every N, a short parity check runs the session on the same 7B tensors for 4 prompt
tokens + 4 greedy tokens and compares every step's logits (1e-4 relative + 5e-5 absolute) and greedy
token (identical) with the CPU oracle's DenseSession restatement; the line carries the result.

At N = 1 the line also carries `kernels` (each hot kernel alone, >= 5 repeats of >= 0.5 s regions,
min / median / spread): configs[1] MatVec, configs[2] attention at T = 512 / 4096 / 32768 and
configs[0] Ternary2 4096^2 at block 64 / 128 / 256; and `cpu_baseline`: the oracle's decode step on
the host cores at the same context, all threads and one thread, with `cpu_baseline.kernels` holding
the oracle's configs[0] / [1] / [2] kernels on one thread and on all threads.

--impl reference times the reference's CPU path (the oracle's C restatement of DenseSession.Append,
all host threads; the C# reference cannot run in this image) on the same metric and config.
Other workloads, for profiling one kernel: --workload matvec | attention | ternary | decode1p5b.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import platform
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402

GB = 1e9
LOGIT_REL, LOGIT_ABS = 1e-4, 5e-5      # stated tolerance on logits after a full decode step (as the tests)


def _peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as fh:
            p = json.load(fh)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def _cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as fh:
            for line in fh:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return platform.processor() or "unknown"


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


def events_time(fn, stream, calls: int) -> float:
    """Device time (ms) of `calls` calls of fn() bracketed by CUDA events on `stream`."""
    import torch
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):  # CUDAGraph.replay() launches on the current stream
        start.record(stream)
        for _ in range(calls):
            fn()
        end.record(stream)
    torch.cuda.synchronize()
    return start.elapsed_time(end)


def repeat_regions(replay, stream, units_per_replay: int, min_region_s: float = 0.5, repeats: int = 5):
    """ms per unit over `repeats` timed regions of >= min_region_s each (replays of one CUDA graph)."""
    ms1 = max(events_time(replay, stream, 1), 1e-3)
    n = max(1, int(math.ceil(min_region_s * 1e3 / ms1)))
    return [events_time(replay, stream, n) / (n * units_per_replay) for _ in range(repeats)]


def stats_record(bytes_per_unit: float, ms_list, peak: float, peak_kind: str, extra=None):
    """GB/s record from per-unit times: best (min time), median and spread, with the roofline fraction."""
    best, med = min(ms_list), statistics.median(ms_list)
    rec = {"value": round(bytes_per_unit / (best / 1e3) / GB, 1),
           "median": round(bytes_per_unit / (med / 1e3) / GB, 1), "unit": "GB/s",
           "spread": round((max(ms_list) - best) / best, 4), "repeats": len(ms_list),
           "us_per_unit_min": round(best * 1e3, 3), "algorithmic_bytes_per_unit": bytes_per_unit,
           "frac": round(bytes_per_unit / (best / 1e3) / GB / peak, 4), "peak": peak, "peak_kind": peak_kind}
    if extra:
        rec.update(extra)
    return rec


# ------------------------------------------------------------------ kernel measurements (N = 1)
MATVEC_SHAPES = [(0, 4096, 4096), (1, 11008, 4096)]


def kernel_matvec(ctx, stream, copies=12, **kw):
    """one Q8_0 4096x4096 + one Q4_0 11008x4096 MatVec (decode order) per unit, rotating
    `copies` distinct weight copies (working set > 4x L2)."""
    import torch

    import satori_b200 as sat
    from satori_b200 import _lib
    mats = []
    for c in range(copies):
        for fmt, rows, cols in MATVEC_SHAPES:
            dev = device_quantized(ctx, rows, cols, fmt, seed=10 * c + fmt)
            mats.append(sat.CudaQuantizedMatrix.from_device(ctx, dev.data_ptr(), dev.numel(), rows, cols, fmt))
            del dev
    x = torch.randn(4096, generator=torch.Generator(device="cuda").manual_seed(77), device="cuda")
    y = torch.empty(11008, device="cuda")
    torch.cuda.synchronize()
    ctx.set_stream(stream.cuda_stream)
    with torch.cuda.stream(stream):
        for m in mats:
            m.execute_device(x.data_ptr(), y.data_ptr(), 1, _lib.ORDER_BATCH)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for m in mats:
            m.execute_device(x.data_ptr(), y.data_ptr(), 1, _lib.ORDER_BATCH)
    torch.cuda.synchronize()
    ms = repeat_regions(graph.replay, stream, copies, **kw)
    ctx.set_stream(None)
    step_bytes = sum(r * (c // 32) * (34 if f == 0 else 18) for f, r, c in MATVEC_SHAPES)
    del graph
    for m in mats:
        m.dispose()
    return step_bytes, ms


DECODE_SHAPES = [("lm_head", 0, 152064, 3584), ("gate_up", 1, 37888, 3584), ("down", 1, 3584, 18944),
                 ("qkv", 1, 4608, 3584)]


def kernel_matvec_shape(ctx, stream, fmt, rows, cols, **kw):
    """One 7B decode projection alone (decode order, one position), rotating enough weight copies that
    the working set exceeds L2 four times over."""
    import torch

    import satori_b200 as sat
    from satori_b200 import _lib
    nbytes = rows * (cols // 32) * (34 if fmt == 0 else 18)
    copies = max(1, int(math.ceil(4 * 126e6 / nbytes)))
    base = device_quantized(ctx, rows, cols, fmt, seed=rows + fmt)
    mats = [sat.CudaQuantizedMatrix.from_device(ctx, base.data_ptr(), base.numel(), rows, cols, fmt)]
    for c in range(1, copies):
        mats.append(sat.CudaQuantizedMatrix.from_device(ctx, base.data_ptr(), base.numel(), rows, cols, fmt))
    del base
    x = torch.randn(cols, generator=torch.Generator(device="cuda").manual_seed(9), device="cuda")
    y = torch.empty(rows, device="cuda")
    torch.cuda.synchronize()
    ctx.set_stream(stream.cuda_stream)
    with torch.cuda.stream(stream):
        mats[0].execute_device(x.data_ptr(), y.data_ptr(), 1, _lib.ORDER_BATCH)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for m in mats:
            m.execute_device(x.data_ptr(), y.data_ptr(), 1, _lib.ORDER_BATCH)
    torch.cuda.synchronize()
    ms = repeat_regions(graph.replay, stream, copies, **kw)
    ctx.set_stream(None)
    del graph
    for m in mats:
        m.dispose()
    return nbytes, ms, copies


def kernel_attention(ctx, stream, T, **kw):
    """GQA 28/4 x 128 over T cached tokens (stream + merge launches), rotating layers."""
    import torch

    from satori_b200 import _lib
    qh, kvh, hd = 28, 4, 128
    kv_bytes = 2 * T * kvh * hd * 4
    layers = max(2, int(np.ceil(4 * 126e6 / kv_bytes)))
    gen = torch.Generator(device="cuda").manual_seed(9)
    kc = torch.randn(layers, T * kvh * hd, generator=gen, device="cuda")
    vc = torch.randn(layers, T * kvh * hd, generator=gen, device="cuda")
    q = torch.randn(qh * hd, generator=gen, device="cuda")
    out = torch.empty(qh * hd, device="cuda")
    torch.cuda.synchronize()
    ctx.set_stream(stream.cuda_stream)
    L = _lib.lib()

    def call(i):
        _lib.check(L.satori_grouped_attention_device(ctx.handle, q.data_ptr(), kc[i].data_ptr(), vc[i].data_ptr(),
                                                     qh, kvh, hd, T, out.data_ptr()))

    with torch.cuda.stream(stream):
        call(0)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for i in range(layers):
            call(i)
    torch.cuda.synchronize()
    ms = repeat_regions(graph.replay, stream, layers, **kw)
    ctx.set_stream(None)
    del graph, kc, vc
    return kv_bytes, ms, layers


def kernel_ternary(ctx, stream, n, bs, order="execute", **kw):
    """Ternary2 n x n MatVec, block bs, N(0,1) weights, rotating copies (> 4x L2)."""
    import torch

    import satori_b200 as sat
    from satori_b200 import _lib
    from satori_b200.core import ternary2_byte_length
    nbytes = ternary2_byte_length(n, n, bs)
    copies = max(4, int(np.ceil(4 * 126e6 / nbytes)))
    rng = np.random.default_rng(1)
    w = rng.standard_normal(n * n).astype(np.float32)
    base = [sat.Ternary2Matrix.quantize(np.roll(w, c * 7919), n, n, bs, ctx=ctx).device for c in range(4)]
    mats = list(base)
    while len(mats) < copies:
        src = base[len(mats) % 4]
        mats.append(sat.CudaQuantizedMatrix.from_device(ctx, src.device_payload, nbytes, n, n, bs))
    x = torch.randn(n, device="cuda")
    y = torch.empty(n, device="cuda")
    torch.cuda.synchronize()
    ctx.set_stream(stream.cuda_stream)
    o = _lib.ORDER_EXECUTE if order == "execute" else _lib.ORDER_SCALAR
    with torch.cuda.stream(stream):
        mats[0].execute_device(x.data_ptr(), y.data_ptr(), 1, o)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for m in mats:
            m.execute_device(x.data_ptr(), y.data_ptr(), 1, o)
    torch.cuda.synchronize()
    ms = repeat_regions(graph.replay, stream, copies, **kw)
    ctx.set_stream(None)
    del graph
    for m in mats:
        m.dispose()
    return nbytes, ms, copies


PREFILL_SHAPES = [("qkv", 1, 4608, 3584), ("o", 1, 3584, 3584), ("gate_up", 1, 37888, 3584),
                  ("down", 1, 3584, 18944), ("lm_head", 0, 152064, 3584)]


def _tensor_peak():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["bf16_tflops"]), "measured"
    except (OSError, KeyError, ValueError):
        return 1590.0, "fallback"


def kernel_prefill_gemm(ctx, stream, name, fmt, rows, cols, positions=128, min_region_s=0.5, repeats=5):
    """One 7B projection of a 128-position prefill chunk on the tensor cores (SATORI_ORDER_TENSOR: the
    activation split, the tcgen05 GEMM and, for split-K shapes, the ordered reduction)."""
    import torch

    import satori_b200 as sat
    from satori_b200 import _lib
    dev = device_quantized(ctx, rows, cols, fmt, seed=5 + rows)
    m = sat.CudaQuantizedMatrix.from_device(ctx, dev.data_ptr(), dev.numel(), rows, cols, fmt)
    del dev
    x = torch.randn(positions * cols, generator=torch.Generator(device="cuda").manual_seed(3), device="cuda")
    y = torch.empty(positions * rows, device="cuda")
    torch.cuda.synchronize()
    ctx.set_stream(stream.cuda_stream)
    with torch.cuda.stream(stream):      # grows the scratch before capture
        m.execute_device(x.data_ptr(), y.data_ptr(), positions, _lib.ORDER_TENSOR)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        m.execute_device(x.data_ptr(), y.data_ptr(), positions, _lib.ORDER_TENSOR)
    torch.cuda.synchronize()
    ms = repeat_regions(graph.replay, stream, 1, min_region_s=min_region_s, repeats=repeats)
    ctx.set_stream(None)
    del graph
    m.dispose()
    best, med = min(ms), statistics.median(ms)
    flops = 2.0 * rows * cols * positions
    mmas = 6 if fmt == 0 else 5          # bf16 part products per weight/activation pair
    peak, kind = _tensor_peak()
    pipe = flops * mmas / (best / 1e3) / 1e12
    return {"shape": f"{name} {rows}x{cols} {'Q8_0' if fmt == 0 else 'Q4_0'}, {positions} positions",
            "us_min": round(best * 1e3, 2), "us_median": round(med * 1e3, 2),
            "spread": round((max(ms) - best) / best, 4), "repeats": len(ms),
            "logical_tflops": round(flops / (best / 1e3) / 1e12, 1),
            "tensor_pipe_tflops": round(pipe, 1), "mma_parts_per_product": mmas,
            "peak_tflops": peak, "peak_kind": kind, "frac": round(pipe / peak, 4),
            "weight_gbs": round(rows * (cols // 32) * (34 if fmt == 0 else 18) / (best / 1e3) / GB, 1)}


def prefill_record(sess, spec, P, stream_ctx, repeats=3):
    """satori_session_forward_tensor on a P-token prompt from position 0 (reset before each run): the
    tensor-core prefill of the first P - 1 tokens plus the last token's decode step, device time."""
    import torch
    prompt = np.random.default_rng(4).integers(0, spec.vocab, P).astype(np.int32)
    ext = torch.cuda.ExternalStream(stream_ctx.stream)
    sess.reset()
    sess.forward(prompt, tensor_cores=True)      # allocates the chunk buffers
    times = []
    for _ in range(repeats):
        sess.reset()
        torch.cuda.synchronize()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(ext)
        t0 = time.perf_counter()
        sess.forward(prompt, tensor_cores=True)
        wall = time.perf_counter() - t0
        end.record(ext)
        torch.cuda.synchronize()
        times.append((start.elapsed_time(end), wall))
    best = min(t[0] for t in times)
    best_wall = min(t[1] for t in times)
    return {"prompt_tokens": P, "chunk_positions": 128, "ms_min": round(best, 2),
            "tokens_per_s": round(P / (best / 1e3), 1), "e2e_tokens_per_s": round(P / best_wall, 1),
            "repeats": repeats,
            "api": "satori_session_forward_tensor (host tokens in, host logits out)",
            "order": "projections on tcgen05, FP32 accumulation of exact bf16 part products (not bit-exact); "
                     "the rest as the decode step"}


def kernel_matvec_kquant(ctx, stream, fmt, rows, cols, **kw):
    """GGUF Q4_K / Q6_K MatVec in the decode (ExecuteBatch) order: random blocks with finite fp16 scales
    (timing only: the block term's cost does not depend on the values), rotating copies > 4x L2."""
    import torch

    import satori_b200 as sat
    from satori_b200 import _lib
    bb = 144 if fmt == _lib.Q4_K else 210
    nblk = rows * (cols // 256)
    rng = np.random.default_rng(fmt)
    host = rng.integers(0, 256, size=(nblk, bb), dtype=np.uint8)
    sc = (rng.standard_normal((nblk, 2)) * 0.01).astype(np.float16).view(np.uint16)
    if fmt == _lib.Q4_K:
        host[:, 0], host[:, 1], host[:, 2], host[:, 3] = sc[:, 0] & 0xFF, sc[:, 0] >> 8, sc[:, 1] & 0xFF, sc[:, 1] >> 8
    else:
        host[:, 208], host[:, 209] = sc[:, 0] & 0xFF, sc[:, 0] >> 8
    nbytes = host.size
    copies = max(1, int(math.ceil(4 * 126e6 / nbytes)))
    first = sat.CudaQuantizedMatrix(ctx, host.reshape(-1), rows, cols, fmt)
    mats = [first] + [sat.CudaQuantizedMatrix.from_device(ctx, first.device_payload, nbytes, rows, cols, fmt)
                      for _ in range(copies - 1)]
    x = torch.randn(cols, generator=torch.Generator(device="cuda").manual_seed(3), device="cuda")
    y = torch.empty(rows, device="cuda")
    torch.cuda.synchronize()
    ctx.set_stream(stream.cuda_stream)
    with torch.cuda.stream(stream):
        mats[0].execute_device(x.data_ptr(), y.data_ptr(), 1, _lib.ORDER_BATCH)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for m in mats:
            m.execute_device(x.data_ptr(), y.data_ptr(), 1, _lib.ORDER_BATCH)
    torch.cuda.synchronize()
    ms = repeat_regions(graph.replay, stream, copies, **kw)
    ctx.set_stream(None)
    del graph
    for m in mats:
        m.dispose()
    return nbytes, ms, copies


def kernel_bitplane(ctx, stream, n, bs, **kw):
    """STB1 bitplane n x n MatVec (TernaryBitplaneAvx2Kernel order) from the same N(0,1) Ternary2 matrix as
    configs[0], rotating copies > 4x L2."""
    import torch

    import satori_b200 as sat
    from satori_b200 import _lib
    from satori_b200.core import ternary2_byte_length
    nbytes = ternary2_byte_length(n, n, bs)
    copies = max(4, int(np.ceil(4 * 126e6 / nbytes)))
    w = np.random.default_rng(1).standard_normal(n * n).astype(np.float32)
    tb = sat.TernaryBitplaneMatrix.from_ternary2(sat.Ternary2Matrix.quantize(w, n, n, bs, ctx=ctx))
    fmt = {64: _lib.TB_64, 128: _lib.TB_128, 256: _lib.TB_256}[bs]
    mats = [tb.device] + [sat.CudaQuantizedMatrix.from_device(ctx, tb.device.device_payload, nbytes, n, n, fmt)
                          for _ in range(copies - 1)]
    x = torch.randn(n, device="cuda")
    y = torch.empty(n, device="cuda")
    torch.cuda.synchronize()
    ctx.set_stream(stream.cuda_stream)
    with torch.cuda.stream(stream):
        mats[0].execute_device(x.data_ptr(), y.data_ptr(), 1, _lib.ORDER_EXECUTE)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for m in mats:
            m.execute_device(x.data_ptr(), y.data_ptr(), 1, _lib.ORDER_EXECUTE)
    torch.cuda.synchronize()
    ms = repeat_regions(graph.replay, stream, copies, **kw)
    ctx.set_stream(None)
    del graph
    for m in mats[1:]:
        m.dispose()
    return nbytes, ms, copies


def kernels_record(ctx, min_region_s=0.5, repeats=5):
    import torch
    peak, kind = _peaks()
    stream = torch.cuda.Stream()
    kw = dict(min_region_s=min_region_s, repeats=repeats)
    out = {}
    b, ms = kernel_matvec(ctx, stream, **kw)
    out["matvec_q8_0_4096x4096+q4_0_11008x4096"] = stats_record(
        b, ms, peak, kind, {"workload": "configs[1]", "launches_per_unit": 2,
                            "order": "ExecuteBatch (decode), bit-exact"})
    for name, fmt, rows, cols in DECODE_SHAPES:
        b, ms, copies = kernel_matvec_shape(ctx, stream, fmt, rows, cols, **kw)
        out[f"matvec_7b_{name}_{'q8_0' if fmt == 0 else 'q4_0'}_{rows}x{cols}"] = stats_record(
            b, ms, peak, kind, {"workload": "configs[4] decode projection", "copies": copies,
                                "order": "ExecuteBatch (decode), bit-exact"})
    for T in (512, 4096, 32768):
        b, ms, layers = kernel_attention(ctx, stream, T, **kw)
        out[f"attention_T{T}"] = stats_record(b, ms, peak, kind, {"workload": f"configs[2] 28/4 x 128, T={T}",
                                                                  "layers_rotated": layers})
    for bs in (64, 128, 256):
        b, ms, copies = kernel_ternary(ctx, stream, 4096, bs, **kw)
        out[f"ternary2_4096x4096_bs{bs}"] = stats_record(b, ms, peak, kind,
                                                         {"workload": f"configs[0] bs{bs}", "copies": copies,
                                                          "order": "Ternary2Avx2Kernel, bit-exact"})
    from satori_b200 import _lib
    for fmt, label in ((_lib.Q4_K, "q4_k"), (_lib.Q6_K, "q6_k")):
        b, ms, copies = kernel_matvec_kquant(ctx, stream, fmt, 4096, 4096, **kw)
        out[f"matvec_{label}_4096x4096"] = stats_record(
            b, ms, peak, kind, {"workload": "GGUF K-quant, configs[1] Q8_0 shape", "copies": copies,
                                "order": "ExecuteBatch with Q8_K activations (decode), bit-exact"})
    b, ms, copies = kernel_bitplane(ctx, stream, 4096, 128, **kw)
    out["bitplane_stb1_4096x4096_bs128"] = stats_record(
        b, ms, peak, kind, {"workload": "configs[0] shape, STB1 layout", "copies": copies,
                            "order": "TernaryBitplaneAvx2Kernel, bit-exact"})
    for name, fmt, rows, cols in PREFILL_SHAPES:
        out[f"prefill_gemm_{name}"] = kernel_prefill_gemm(ctx, stream, name, fmt, rows, cols, **kw)
    return out


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


def decode_parity(sess, spec, tensors, rank, n_prompt=4, n_gen=4):
    """Every rank steps the session; rank 0 replays the same tokens through the oracle and compares."""
    prompt = [int(t) for t in np.random.default_rng(11).integers(0, spec.vocab, n_prompt)]
    feed, logits, greedy = [], [], []
    tok = None
    for i in range(n_prompt + n_gen):
        t = prompt[i] if i < n_prompt else tok
        lg, tok = sess.append(t)
        feed.append(t)
        logits.append(lg)
        greedy.append(tok)
    sess.reset()
    if rank != 0:
        return None, None
    from oracle.oracle import OracleSession
    host = {k: v.cpu().numpy() for k, v in tensors.items()}
    ref = OracleSession(spec, host, n_prompt + n_gen + 1)
    threads = os.cpu_count() or 1
    worst, tokens_ok, logits_ok = 0.0, True, True
    for i, t in enumerate(feed):
        lr, ar = ref.append(t, threads=threads)
        err = np.abs(logits[i].astype(np.float64) - lr)
        bound = LOGIT_REL * np.abs(lr) + LOGIT_ABS
        worst = max(worst, float(np.max(err / bound)))
        logits_ok &= bool(np.all(err <= bound))
        tokens_ok &= ar == greedy[i]
    ref.close()
    rec = {"ok": bool(tokens_ok and logits_ok), "steps": len(feed), "greedy_tokens_identical": bool(tokens_ok),
           "logits_within_tol": bool(logits_ok), "tolerance": f"{LOGIT_REL} rel + {LOGIT_ABS} abs",
           "worst_err_over_bound": round(worst, 4), "against": "oracle DenseSession restatement (CPU)"}
    return rec, host


def cpu_decode_rate(spec, host, context, threads, min_s, min_tokens, max_tokens, cache_seed=5):
    """The oracle's DenseSession.Append at position `context` (synthetic cache rows), host cores."""
    from oracle.oracle import OracleSession
    ref = OracleSession(spec, host, context + max_tokens + 1)
    ref.fill_cache(context, cache_seed)
    ref.append(1, threads=threads)                 # warm-up (page-in)
    n, t0 = 0, time.perf_counter()
    while n < max_tokens and (n < min_tokens or time.perf_counter() - t0 < min_s):
        ref.append(1 + n, threads=threads)
        n += 1
    dt = time.perf_counter() - t0
    ref.close()
    return n / dt, n, dt


def host_random_model(spec, seed):
    """Payloads cut from one seeded 16 MiB random pattern, with finite fp16 scales written into every
    block (timing only: decode cost does not depend on the values), and the model's float vectors;
    built on the host without the GPU."""
    rng = np.random.default_rng(seed)
    pattern = np.frombuffer(rng.bytes(1 << 24), dtype=np.uint8)
    host = {}
    for i, (name, (rows, cols)) in enumerate(spec.matrix_shapes().items()):
        fmt = spec.format_of(name)
        bb = 34 if fmt == 0 else 18
        nblk = rows * (cols // 32)
        flat = np.empty(nblk * bb, dtype=np.uint8)
        src = np.roll(pattern, 4099 * i)
        for off in range(0, flat.size, src.size):
            flat[off:off + src.size] = src[:flat.size - off]
        buf = flat.reshape(nblk, bb)
        scale = np.float16(0.02 / (127.0 if fmt == 0 else 8.0))
        buf[:, 0:2] = np.frombuffer(scale.tobytes(), dtype=np.uint8)
        host[name] = flat
    for name, n in spec.vector_shapes().items():
        host[name] = ((1.0 if name.endswith("norm.weight") else 0.0) +
                      0.02 * rng.standard_normal(n)).astype(np.float32)
    return host


def cpu_baseline_decode(spec, host, context):
    all_threads = os.cpu_count() or 1
    v_all, n_all, dt_all = cpu_decode_rate(spec, host, context, all_threads, min_s=8.0, min_tokens=3,
                                           max_tokens=64)
    v_one, n_one, dt_one = cpu_decode_rate(spec, host, context, 1, min_s=5.0, min_tokens=1, max_tokens=8)
    return {"value": round(v_all, 4), "unit": "tokens/s", "cores": all_threads, "kind": "port",
            "sample": f"{n_all} decode steps at context {context} in {dt_all:.1f}s (oracle DenseSession.Append "
                      f"restatement, AVX2/FMA, OpenMP row split, synthetic cache rows)",
            "single_thread": {"value": round(v_one, 4), "unit": "tokens/s", "cores": 1,
                              "sample": f"{n_one} decode steps in {dt_one:.1f}s"},
            "cpu_model": _cpu_model()}


def _cpu_rate(call, nbytes, min_s):
    """GB/s of one host call repeated for at least `min_s` seconds, after one untimed call."""
    call()
    n, t0 = 0, time.perf_counter()
    while n < 1 or time.perf_counter() - t0 < min_s:
        call()
        n += 1
    dt = time.perf_counter() - t0
    return nbytes / (dt / n) / GB, n, dt


def cpu_kernel_baselines(min_s=0.5):
    """The oracle's restatements of the kernel-level configs on the host cores, on one thread and on all
    threads, beside the GPU kernel records: configs[0] Ternary2Avx2Kernel at 4096^2 (bs 64 / 128 / 256),
    configs[1] ExecuteBatchFloat over Q8_0 4096^2 + Q4_0 11008x4096, configs[2] GroupedAttention (FP64) at
    28/4 heads x 128, T = 4096.  Seeded host inputs with the GPU records' shapes and distributions."""
    from oracle import oracle as O
    rng = np.random.default_rng(21)
    all_threads = os.cpu_count() or 1
    out = {}

    def record(name, call, nbytes, workload):
        v1, n1, d1 = _cpu_rate(lambda: call(1), nbytes, min_s)
        va, na, da = _cpu_rate(lambda: call(all_threads), nbytes, min_s)
        out[name] = {"value_1_thread": round(v1, 3), "value_all_threads": round(va, 3), "unit": "GB/s",
                     "cores": all_threads, "algorithmic_bytes_per_unit": int(nbytes), "workload": workload,
                     "sample": f"{n1} calls in {d1:.2f}s on 1 thread, {na} calls in {da:.2f}s on {all_threads}"}

    n = 4096
    w = rng.standard_normal(n * n).astype(np.float32)
    x = rng.standard_normal(n).astype(np.float32)
    for bs in (64, 128, 256):
        p = O.t2_quantize(w, n, n, bs)
        record(f"ternary2_4096x4096_bs{bs}", lambda t, p=p, bs=bs: O.t2_matvec(p, n, n, bs, x, "avx2", threads=t),
               p.size, f"configs[0] bs{bs}, Ternary2Avx2Kernel order")
    del w
    p8 = O.q_quantize((0.02 * rng.standard_normal(n * n)).astype(np.float32), n, n, 0)
    p4 = O.q_quantize((0.02 * rng.standard_normal(11008 * n)).astype(np.float32), 11008, n, 1)
    record("matvec_q8_0_4096x4096+q4_0_11008x4096",
           lambda t: (O.q_matvec(p8, n, n, 0, x, "batch", threads=t), O.q_matvec(p4, 11008, n, 1, x, "batch", threads=t)),
           p8.size + p4.size, "configs[1], ExecuteBatchFloat order")
    del p8, p4
    T, qh, kvh, hd = 4096, 28, 4, 128
    q = rng.standard_normal(qh * hd).astype(np.float32)
    keys = rng.standard_normal(T * kvh * hd).astype(np.float32)
    values = rng.standard_normal(T * kvh * hd).astype(np.float32)
    record(f"attention_T{T}", lambda t: O.grouped_attention(q, keys, values, qh, kvh, hd, T, threads=t),
           2 * T * kvh * hd * 4, "configs[2] 28/4 x 128, GroupedAttention (FP64)")
    return out


def _embedding_table_bytes(spec, world):
    """Bytes of token_embd.weight inside a session's weight bytes that a step does not stream (a step
    reads one row): the whole table, unless it is also the single-GPU output matrix."""
    if spec.tied_embeddings and world == 1:
        return 0
    return spec.vocab * (spec.hidden // 32) * 34


def bench_decode(args, rank, world, local, spec, with_kernels: bool):
    import torch

    import satori_b200 as sat
    ctx = sat.Context(local)
    P, D = args.prompt, args.decode
    context = P + D + 8
    tensors = device_model(ctx, spec, seed=31)
    torch.cuda.synchronize()
    if world == 1:
        sess = sat.CudaDenseSession(spec, tensors, context, ctx=ctx)
    else:
        sess = sat.CudaDenseSession(spec, tensors, context, ctx=ctx, rank=rank, world=world,
                                    nccl_id=sat.broadcast_nccl_id())
    info = sess.info()
    parity, host = decode_parity(sess, spec, tensors, rank)
    del tensors
    torch.cuda.empty_cache()
    dist_barrier(world)

    prompt = np.random.default_rng(4).integers(0, spec.vocab, P).astype(np.int32)
    last = sess.prefill(prompt)
    for _ in range(args.warmup):
        sess.rewind(P)
        ref_tokens = sess.generate(int(last), D)
    ext = torch.cuda.ExternalStream(ctx.stream)
    torch.cuda.synchronize()
    dist_barrier(world)
    stable = True
    with ClockSampler(local) as clocks:
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(ext)
        t0 = time.perf_counter()
        for _ in range(args.steps):
            sess.rewind(P)
            toks = sess.generate(int(last), D)
            stable &= bool(np.array_equal(toks, ref_tokens))
        wall = time.perf_counter() - t0
        end.record(ext)
        torch.cuda.synchronize()
    ms = dist_max(start.elapsed_time(end), world)
    wall = dist_max(wall, world)
    tokens = args.steps * D
    tps = tokens / (ms / 1e3)
    # Per GPU and token: this rank's weight rows, one embedding row, and the cached K/V it reads.
    kv_avg = info["kv_bytes_per_position"] * (P + D / 2)
    bytes_per_token = (info["weight_bytes"] - _embedding_table_bytes(spec, world) + spec.hidden // 32 * 34
                       + kv_avg)
    achieved = bytes_per_token / (ms / 1e3 / tokens) / GB
    peak, peak_kind = _peaks()
    res = {
        "metric": f"decode tokens/s ({spec.name}, {P}-token context, {D} greedy tokens per step)",
        "value": round(tps, 2), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 3), "ms_per_token": round(ms / tokens, 4),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "q4_0/q8_0 weights, f32 activations and accumulation",
        "data": "synthetic: seeded N(0,0.02^2) weights quantized on the device, seeded random prompt",
        "config": {"workload": f"configs[{4 if spec.name.startswith('qwen2-7b') else 3}]: {spec.name}",
                   "context": P, "decode_tokens_per_step": D,
                   "l2_policy": "inputs larger than L2: every token streams all weights (GBs) from HBM",
                   "parallelism": "single GPU" if world == 1 else
                   f"tp{world}: row-sharded projections, query-head-sharded attention, in-graph all-gathers",
                   "exchange": None if world == 1 else os.environ.get("SATORI_EXCHANGE", "p2p")},
        "parity": parity,
        "deterministic_steps": stable,
        "roofline": {"bound": "hbm", "unit_of_work": "one decode token (every launch of the step, this GPU)",
                     "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "peak_kind": peak_kind, "traffic": None,
                     "algorithmic_bytes_per_token": int(bytes_per_token)},
        "e2e": {"value": round(tokens / wall, 2), "unit": "tokens/s", "h2d_bytes_per_step": 8,
                "d2h_bytes_per_step": 4 * D + 28,
                "api": "satori_session_rewind + satori_session_generate (host token in, host tokens out)"},
        "gpu_launches": info["kernels_per_step"] * tokens,
        "launches_per_token": info["kernels_per_step"],
        "first_tokens": [int(t) for t in ref_tokens[:8]],
        "clocks": clocks.summary(),
    }
    if world == 1 and not args.no_prefill:
        res["prefill"] = prefill_record(sess, spec, P, ctx)
    sess.dispose()
    if with_kernels and rank == 0 and world == 1:
        res["kernels"] = kernels_record(ctx, min_region_s=args.region, repeats=args.repeats)
    if rank == 0 and world == 1 and host is not None and not args.no_cpu_baseline:
        res["cpu_baseline"] = cpu_baseline_decode(spec, host, P)
        try:   # the kernel-level CPU figures are context for the kernel records; never fatal to the line
            res["cpu_baseline"]["kernels"] = cpu_kernel_baselines()
        except Exception as e:
            res["cpu_baseline"]["kernels"] = {"error": f"{type(e).__name__}: {e}"[:300]}
    return res


def bench_matvec_sharded(args, rank, world, local):
    """The row-sharded large MatVec (Q4_0 11008x4096, decode order) over N GPUs: every rank computes its
    contiguous row block and NCCL all-gathers y (satori_matrix_sharded_execute_device).  Each timed call
    follows an untimed read of a 256 MB buffer (L2 refilled with clean lines: a rank's slice alone would
    fit in L2);
    device time of the calls only, max over ranks; value = the whole matrix's payload bytes per call time."""
    import torch

    import satori_b200 as sat
    from satori_b200 import _lib
    ctx = sat.Context(local)
    rows, cols, fmt = 11008, 4096, 1
    dev = device_quantized(ctx, rows, cols, fmt, seed=123)          # the same bytes on every rank
    nccl_id = sat.broadcast_nccl_id() if world > 1 else None
    m = sat.CudaShardedMatrix(ctx, dev, sat.QuantizedMatrixShape(rows, cols, fmt), rank, world, nccl_id)
    del dev
    x = torch.randn(cols, generator=torch.Generator(device="cuda").manual_seed(7), device="cuda")
    y = torch.empty(rows, device="cuda")
    flush = torch.ones(256 << 20, dtype=torch.uint8, device="cuda")
    ext = torch.cuda.ExternalStream(ctx.stream)
    for _ in range(args.warmup):
        m.execute_device(x.data_ptr(), y.data_ptr(), _lib.ORDER_BATCH)
    torch.cuda.synchronize()
    dist_barrier(world)
    total = 0.0
    with ClockSampler(local) as clocks:
        for _ in range(args.steps):
            with torch.cuda.stream(ext):
                flush.sum(dtype=torch.int64)
            torch.cuda.synchronize()
            dist_barrier(world)           # every rank enters the timed call together (no flush skew inside)
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            start.record(ext)
            m.execute_device(x.data_ptr(), y.data_ptr(), _lib.ORDER_BATCH)
            end.record(ext)
            torch.cuda.synchronize()
            total += start.elapsed_time(end)
    ms = dist_max(total / args.steps, world)
    nbytes = rows * (cols // 32) * 18
    m.dispose()
    peak, kind = _peaks()
    gbs = nbytes / (ms / 1e3) / GB
    return {"metric": "row-sharded MatVec payload GB/s (Q4_0 11008x4096 + all-gather of y)",
            "value": round(gbs, 1), "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "q4_0 weights, f32 activations", "data": "synthetic: seeded N(0,0.02^2) weights",
            "config": {"workload": "configs[1] Q4_0 11008x4096, rows sharded over the GPUs",
                       "l2_policy": "256 MB buffer read before every timed call",
                       "parallelism": f"row shards x{world} + NCCL all-gather"},
            "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(gbs / peak, 4), "peak_kind": kind, "traffic": None},
            "gpu_launches": 2 * args.steps, "clocks": clocks.summary()}


def bench_prefill(args, local):
    """The 7B tensor-core prefill alone (profiling): a --prompt-token satori_session_forward_tensor."""
    import torch

    import satori_b200 as sat
    ctx = sat.Context(local)
    spec = sat.qwen2_7b()
    tensors = device_model(ctx, spec, seed=31)
    torch.cuda.synchronize()
    sess = sat.CudaDenseSession(spec, tensors, args.prompt + 8, ctx=ctx)
    del tensors
    torch.cuda.empty_cache()
    rec = prefill_record(sess, spec, args.prompt, ctx, repeats=args.repeats)
    sess.dispose()
    return {"metric": f"prefill tokens/s ({spec.name}, {args.prompt}-token prompt, tensor cores)",
            "value": rec["tokens_per_s"], "unit": "tokens/s", "n_gpus": 1, "higher_is_better": True, "prefill": rec}


# ------------------------------------------------------------------ single-kernel workloads (profiling)
def bench_kernel(args, local):
    import torch

    import satori_b200 as sat
    ctx = sat.Context(local)
    stream = torch.cuda.Stream()
    peak, kind = _peaks()
    kw = dict(min_region_s=args.region, repeats=args.repeats)
    if args.workload == "matvec":
        b, ms = kernel_matvec(ctx, stream, **kw)
        name, launches = "configs[1] MatVec Q8_0 4096^2 + Q4_0 11008x4096", 2
    elif args.workload == "attention":
        b, ms, _ = kernel_attention(ctx, stream, args.tokens, **kw)
        name, launches = f"configs[2] attention T={args.tokens}", 2
    elif args.workload == "prefill_gemm":
        rec = kernel_prefill_gemm(ctx, stream, "gate_up", 1, 37888, 3584, **kw)
        return {"metric": "prefill GEMM tensor-pipe TFLOP/s (7B gate/up, 128 positions)",
                "value": rec["tensor_pipe_tflops"], "unit": "TFLOP/s", "n_gpus": 1, "higher_is_better": True,
                "kernel": rec, "gpu_launches_per_unit": 2}
    else:
        b, ms, _ = kernel_ternary(ctx, stream, args.n, args.block, args.order, **kw)
        name, launches = f"configs[0] Ternary2 {args.n}^2 bs{args.block}", 1
    rec = stats_record(b, ms, peak, kind)
    return {"metric": f"{name} payload GB/s", "value": rec["value"], "unit": "GB/s", "n_gpus": 1,
            "higher_is_better": True, "kernel": rec, "gpu_launches_per_unit": launches}


# ------------------------------------------------------------------ reference arm
def reference_arm(args, rank, world, spec):
    if rank != 0:
        return None
    P = args.prompt
    host = host_random_model(spec, seed=3)
    threads = os.cpu_count() or 1
    from oracle.oracle import OracleSession
    ref = OracleSession(spec, host, P + args.warmup + args.steps + 2)
    ref.fill_cache(P, 5)
    for i in range(args.warmup):
        ref.append(1 + i, threads=threads)
    t0 = time.perf_counter()
    for i in range(args.steps):
        ref.append(100 + i, threads=threads)
    dt = time.perf_counter() - t0
    ref.close()
    tps = args.steps / dt
    v_one, n_one, dt_one = cpu_decode_rate(spec, host, P, 1, min_s=5.0, min_tokens=1, max_tokens=4)
    base = {"value": round(tps, 4), "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"{args.steps} decode steps at context {P} in {dt:.1f}s (one step = one token; synthetic "
                      f"cache rows; seeded random payloads)",
            "single_thread": {"value": round(v_one, 4), "unit": "tokens/s", "cores": 1,
                              "sample": f"{n_one} decode steps in {dt_one:.1f}s"},
            "cpu_model": _cpu_model()}
    return {"metric": f"decode tokens/s ({spec.name}, {P}-token context, {args.decode} greedy tokens per step)",
            "value": round(tps, 4), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "impl": "reference", "dtype": "q4_0/q8_0 weights, f32", "data": "synthetic seeded",
            "config": {"workload": f"configs[{4 if spec.name.startswith('qwen2-7b') else 3}]: {spec.name}",
                       "context": P,
                       "implementation": "C restatement of DenseSession.Append / DenseForward.Step (AVX2+FMA "
                                         "ExecuteBatchFloat, FP64 attention), all host threads (the C# reference "
                                         "cannot be built in this image)"},
            "cpu_baseline": base,
            "e2e": {"value": round(tps, 4), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="satori", choices=["satori", "reference"])
    ap.add_argument("--workload", default="decode7b",
                    choices=["decode7b", "decode1p5b", "prefill7b", "matvec_sharded", "matvec", "attention", "ternary",
                             "prefill_gemm"])
    ap.add_argument("--tokens", type=int, default=32768)
    ap.add_argument("--n", type=int, default=4096)
    ap.add_argument("--block", type=int, default=128)
    ap.add_argument("--order", default="execute", choices=["execute", "scalar"])
    ap.add_argument("--prompt", type=int, default=2048)
    ap.add_argument("--decode", type=int, default=256)
    ap.add_argument("--region", type=float, default=0.5, help="seconds per timed region (kernel workloads)")
    ap.add_argument("--repeats", type=int, default=5)
    ap.add_argument("--no-kernels", action="store_true", help="skip the per-kernel records of the decode line")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-prefill", action="store_true", help="skip the tensor-core prefill record")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    args.steps = max(1, args.steps)
    import satori_b200 as sat
    if args.impl == "reference":
        rank = int(os.environ.get("RANK", "0"))
        world = int(os.environ.get("WORLD_SIZE", "1"))
        spec = sat.qwen2_1_5b() if args.workload == "decode1p5b" else sat.qwen2_7b()
        res = reference_arm(args, rank, world, spec)
        if res is not None:
            print(json.dumps(res), flush=True)
        return
    rank, world, local = dist_init()
    if args.workload in ("decode7b", "decode1p5b"):
        spec = sat.qwen2_7b() if args.workload == "decode7b" else sat.qwen2_1_5b()
        res = bench_decode(args, rank, world, local, spec, with_kernels=not args.no_kernels)
    elif args.workload == "prefill7b":
        res = bench_prefill(args, local) if rank == 0 else None
    elif args.workload == "matvec_sharded":
        res = bench_matvec_sharded(args, rank, world, local)
    else:
        res = bench_kernel(args, local) if rank == 0 else None
    if rank == 0 and res is not None:
        print(json.dumps(res), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
