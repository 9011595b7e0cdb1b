"""Sharded decode session (one process per GPU, NCCL all-gathers) vs the oracle's DenseSession.

Projections are sharded by rows, so every logit is produced by the same per-row FP32 chain as on
one GPU; attention is sharded by query heads.  Every rank must hold the same full logits (bitwise:
they are all-gathered), within the single-GPU tolerance of the oracle, with identical greedy tokens.
The shapes cover an even head split, a split that cuts a GQA group (two ranks compute one KV head),
and an uneven query-head split (padded context exchange).  Backends: P2P with one exchange kernel per
all-gather, P2P with the exchanges carried by the producing row-MatVec launches where the shape allows
(hidden 256 takes that path for every projection), and NCCL.
"""
import multiprocessing as mp
import os

import numpy as np
import pytest

from golden_util import bits_equal
from model_util import synthetic_tensors

pytestmark = pytest.mark.gpu

LOGIT_REL, LOGIT_ABS = 1e-4, 1e-5
CHILD_TIMEOUT_S = 300


def _gpu_count() -> int:
    import torch
    return torch.cuda.device_count()


@pytest.fixture(scope="module")
def sat():
    from satori_b200 import build
    build.build()
    import satori_b200
    return satori_b200


def _spawn(target, argsets, env):
    """Starts one spawned child per rank with `env` added to the environment; returns their exit codes."""
    mpc = mp.get_context("spawn")
    saved = {k: os.environ.get(k) for k in env}
    os.environ.update(env)
    try:
        procs = [mpc.Process(target=target, args=a) for a in argsets]
        for p in procs:
            p.start()
    finally:
        for k, v in saved.items():
            if v is None:
                os.environ.pop(k, None)
            else:
                os.environ[k] = v
    for p in procs:
        p.join(CHILD_TIMEOUT_S)
    for p in procs:
        if p.is_alive():
            p.kill()
            p.join()
    return [p.exitcode for p in procs]


def _run_world(sat, world, spec_kwargs, seed, context, tokens, gen_first, gen_count, tmp_path, backend):
    import shard_worker
    nccl_id = sat.nccl_unique_id()
    outs = [str(tmp_path / ("rank%d.npz" % r)) for r in range(world)]
    codes = _spawn(shard_worker.run_rank,
                   [(r, world, nccl_id, spec_kwargs, seed, context, tokens, gen_first, gen_count, outs[r])
                    for r in range(world)],
                   {"NCCL_NVLS_ENABLE": "0", "SATORI_EXCHANGE": backend.split("-")[0],
                    "SATORI_EXCHANGE_CARRY": "1" if backend.endswith("-carry") else "0"})
    assert codes == [0] * world
    return [np.load(o) for o in outs]


CASES = [
    # (world, tiny() overrides): even split; a split inside a GQA group; an uneven query-head split
    (2, dict(layers=2, hidden=256, ffn=512, q_heads=4, kv_heads=2, head_dim=64, vocab=1000)),
    (2, dict(layers=2, hidden=384, ffn=768, q_heads=6, kv_heads=3, head_dim=64, vocab=1000, proj_format=1)),
    (2, dict(layers=3, hidden=192, ffn=384, q_heads=3, kv_heads=1, head_dim=64, vocab=1002, has_bias=False)),
    (4, dict(layers=2, hidden=384, ffn=768, q_heads=6, kv_heads=2, head_dim=64, vocab=1000)),
    # the 7B shape's head pattern (28 query / 4 KV heads) split over 4 and 8 ranks: 7 or 3.5 query heads per
    # rank, so at 8 ranks every KV head is cached by the two ranks that share its group
    (4, dict(layers=2, hidden=896, ffn=1024, q_heads=28, kv_heads=4, head_dim=32, vocab=1000, proj_format=1)),
    (8, dict(layers=2, hidden=896, ffn=1024, q_heads=28, kv_heads=4, head_dim=32, vocab=1000, proj_format=1)),
    (8, dict(layers=2, hidden=512, ffn=1024, q_heads=8, kv_heads=8, head_dim=64, vocab=1024)),
]


@pytest.mark.parametrize("backend", ["p2p-carry", "p2p-kernel", "nccl"])
@pytest.mark.parametrize("world,kw", CASES)
def test_sharded_session_matches_oracle(sat, oracle_lib, tmp_path, world, kw, backend):
    if _gpu_count() < world:
        pytest.skip("needs %d GPUs" % world)
    from oracle.oracle import OracleSession
    spec = sat.tiny(**kw)
    tokens = [int(t) for t in np.random.default_rng(world + kw["q_heads"]).integers(0, spec.vocab, 20)]
    res = _run_world(sat, world, kw, seed=17, context=48, tokens=tokens, gen_first=tokens[0], gen_count=12,
                     tmp_path=tmp_path, backend=backend)
    for r in range(1, world):
        assert np.array_equal(res[r]["logits"].view(np.uint32), res[0]["logits"].view(np.uint32))
        assert np.array_equal(res[r]["gen"], res[0]["gen"])
    ref = OracleSession(spec, synthetic_tensors(spec, 17), 48)
    for i, t in enumerate(tokens):
        lr, ar = ref.append(t, threads=8)
        lg = res[0]["logits"][i]
        err = np.abs(lg.astype(np.float64) - lr)
        assert np.all(err <= LOGIT_REL * np.abs(lr) + LOGIT_ABS), (i, float(err.max()))
        assert int(res[0]["greedy"][i]) == ar, i
    ref = OracleSession(spec, synthetic_tensors(spec, 17), 48)
    t, expect = tokens[0], []
    for _ in range(12):
        _, t = ref.append(t, threads=8)
        expect.append(t)
    assert list(res[0]["gen"]) == expect


def test_silent_peer_times_out_and_latches(sat, tmp_path):
    """Failure detection without a GPU fault: rank 1 never steps, so rank 0's first exchange finds no
    signal; its bounded wait expires (0.5 s here), the step reports a timeout, and the session refuses
    later steps.  Rank 1 has no kernel in flight and both ranks dispose normally."""
    if _gpu_count() < 2:
        pytest.skip("needs 2 GPUs")
    import ast

    import shard_worker
    nccl_id = sat.nccl_unique_id()
    done = mp.get_context("spawn").Event()
    outs = [str(tmp_path / ("silent%d.txt" % r)) for r in range(2)]
    codes = _spawn(shard_worker.run_silent_peer, [(r, 2, nccl_id, {}, 5, done, outs[r]) for r in range(2)],
                   {"NCCL_NVLS_ENABLE": "0", "SATORI_EXCHANGE": "p2p", "SATORI_PEER_TIMEOUT_MS": "500"})
    assert codes == [0, 0]
    r0 = ast.literal_eval(open(outs[0]).read())
    assert r0["first"] == sat._lib.ERR_TIMEOUT and r0["second"] == sat._lib.ERR_TIMEOUT
    assert 0.4 < r0["first_s"] < 30


@pytest.mark.parametrize("world", [2, 4, 8])
def test_sharded_matvec_equals_single_gpu_reference(sat, oracle_lib, tmp_path, world):
    """The row-sharded large MatVec (satori_matrix_create_sharded): rank r holds rows [r*S, (r+1)*S) and
    every rank ends with the full output after the NCCL all-gather; every value equals the oracle's
    single-GPU result bit for bit (each row keeps the reference's operation order), including the padded
    last slice of an uneven split."""
    if _gpu_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import shard_worker
    ids = [sat.nccl_unique_id() for _ in shard_worker.sharded_matvec_cases()]
    outs = [str(tmp_path / ("mv%d.npz" % r)) for r in range(world)]
    codes = _spawn(shard_worker.run_sharded_matvec, [(r, world, ids, outs[r]) for r in range(world)],
                   {"NCCL_NVLS_ENABLE": "0"})
    assert codes == [0] * world
    res = [np.load(o) for o in outs]
    for i, (rows, cols, fmt, order, seed) in enumerate(shard_worker.sharded_matvec_cases()):
        payload, x = shard_worker.case_inputs(rows, cols, fmt, seed)
        if fmt >= 64:
            ref = oracle_lib.t2_matvec(payload, rows, cols, fmt, x, "avx2", threads=8)
        else:
            ref = oracle_lib.q_matvec(payload, rows, cols, fmt, x, order="batch" if order == "batch" else "avx2",
                                      threads=8)
        slice_ = -(-rows // world)
        for r in range(world):
            y = res[r][f"y{i}"]
            assert list(res[r][f"r{i}"]) == [r * slice_, min(rows, (r + 1) * slice_)]
            assert bits_equal(y, np.asarray(ref, np.float32)), (i, r)
