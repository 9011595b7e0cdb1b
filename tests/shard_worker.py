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
