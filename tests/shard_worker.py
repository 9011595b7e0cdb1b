"""One rank of a sharded decode session, run as a spawned child process by the sharded-session tests.

Each rank owns one GPU (device = rank), builds the same seeded synthetic model, creates its share of
the session through satori_session_create_sharded and records, for a teacher-forced token sequence,
every step's full logits and greedy token, then a device-side greedy generation after a reset.
"""
from __future__ import annotations

import os

import numpy as np


def run_rank(rank: int, world: int, nccl_id: bytes, spec_kwargs: dict, seed: int, context: int, tokens: list,
             gen_first: int, gen_count: int, out_path: str) -> None:
    import satori_b200 as sat
    from model_util import synthetic_tensors

    spec = sat.tiny(**spec_kwargs)
    tensors = synthetic_tensors(spec, seed)
    ctx = sat.Context(rank)
    s = sat.CudaDenseSession(spec, tensors, context, ctx=ctx, rank=rank, world=world, nccl_id=nccl_id)
    logits, greedy = [], []
    for t in tokens:
        lg, ag = s.append(int(t))
        logits.append(lg)
        greedy.append(ag)
    s.reset()
    gen = s.generate(gen_first, gen_count)
    s.dispose()
    tmp = out_path + ".part"
    with open(tmp, "wb") as f:
        np.savez(f, logits=np.stack(logits), greedy=np.array(greedy, np.int32), gen=gen)
    os.replace(tmp, out_path)


def run_silent_peer(rank: int, world: int, nccl_id: bytes, spec_kwargs: dict, seed: int, done, out_path: str) -> None:
    """Rank 0 steps alone while the other ranks stay idle between steps: rank 0's exchange wait must
    expire with a timeout status (and latch it), and no rank may have a kernel left in flight."""
    import time

    import satori_b200 as sat
    from model_util import synthetic_tensors

    spec = sat.tiny(**spec_kwargs)
    s = sat.CudaDenseSession(spec, synthetic_tensors(spec, seed), 16, ctx=sat.Context(rank), rank=rank, world=world,
                             nccl_id=nccl_id)
    result = {}
    if rank == 0:
        t0 = time.perf_counter()
        try:
            s.append(1)
            result["first"] = "ok"
        except sat.SatoriError as e:
            result["first"] = e.status
        result["first_s"] = time.perf_counter() - t0
        try:
            s.append(2)
            result["second"] = "ok"
        except sat.SatoriError as e:
            result["second"] = e.status
        done.set()
    else:
        done.wait(120)
    s.dispose()
    with open(out_path, "w") as f:
        f.write(repr(result))


def sharded_matvec_cases():
    """(rows, cols, format, order name, seed): an even Q4_0 split (the large GEMV shape), a Q8_0 split that
    leaves a padded last slice, and Ternary2 in the AVX2 order."""
    return [(11008, 4096, 1, "batch", 1), (1003, 1024, 0, "batch", 2), (1003, 1024, 0, "execute", 3),
            (4096, 4096, 64, "execute", 4)]


def case_inputs(rows: int, cols: int, fmt: int, seed: int):
    """The same seeded payload and input on every rank (and in the parent that checks them)."""
    rng = np.random.default_rng(seed)
    if fmt >= 64:
        from oracle import oracle
        w = rng.standard_normal(rows * cols).astype(np.float32)
        payload = oracle.t2_quantize(w, rows, cols, fmt)
    else:
        bb = 34 if fmt == 0 else 18
        payload = rng.integers(0, 256, size=rows * (cols // 32) * bb, dtype=np.uint8)
        scales = (rng.standard_normal(rows * (cols // 32)) * 0.05).astype(np.float16).view(np.uint16)
        p2 = payload.reshape(-1, bb)
        p2[:, 0] = scales & 0xFF
        p2[:, 1] = scales >> 8
    x = rng.standard_normal(cols).astype(np.float32)
    return payload, x


def run_sharded_matvec(rank: int, world: int, nccl_ids: list, out_path: str) -> None:
    """Every case through CudaShardedMatrix on this rank (one NCCL id per case: an id serves one
    communicator); saves the full gathered outputs."""
    import satori_b200 as sat
    from satori_b200 import _lib

    ctx = sat.Context(rank)
    outs = {}
    for i, (rows, cols, fmt, order, seed) in enumerate(sharded_matvec_cases()):
        payload, x = case_inputs(rows, cols, fmt, seed)

        class Shape:
            pass
        shape = Shape()
        shape.rows, shape.columns, shape.format = rows, cols, fmt
        m = sat.CudaShardedMatrix(ctx, payload, shape, rank, world, nccl_ids[i])
        o = _lib.ORDER_BATCH if order == "batch" else _lib.ORDER_EXECUTE
        outs[f"y{i}"] = m.execute(x, o)
        outs[f"r{i}"] = np.array([m.row_begin, m.row_end], np.int32)
        m.dispose()
    tmp = out_path + ".part"
    with open(tmp, "wb") as f:
        np.savez(f, **outs)
    os.replace(tmp, out_path)
