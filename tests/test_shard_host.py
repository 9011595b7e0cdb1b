"""Host side of the sharded decode session (no GPU): the row/head split every rank computes, the
shapes it rejects, and the NCCL id hand-off over a world-2 gloo group."""
import multiprocessing as mp
import socket

import numpy as np
import pytest


@pytest.fixture(scope="module")
def sat():
    from satori_b200 import build
    build.build()
    import satori_b200
    return satori_b200


@pytest.mark.parametrize("world", [1, 2, 4, 8])
@pytest.mark.parametrize("which", ["qwen2_1_5b", "qwen2_7b"])
def test_shards_tile_every_dimension(sat, world, which):
    spec = getattr(sat, which)()
    parts = [sat.shard_ranges(spec, r, world) for r in range(world)]
    for dim, n in (("hidden", spec.hidden), ("ffn", spec.ffn), ("vocab", spec.vocab), ("q_heads", spec.q_heads)):
        cover = np.zeros(n, np.int32)
        for p in parts:
            a, b = p[dim]
            assert 0 <= a < b <= n
            cover[a:b] += 1
        assert np.all(cover == 1), dim          # disjoint and complete
    group = spec.q_heads // spec.kv_heads
    for p in parts:
        qa, qb = p["q_heads"]
        ka, kb = p["kv_heads"]
        assert set(range(ka, kb)) == {h // group for h in range(qa, qb)}   # exactly the KV heads read here


def test_uneven_query_heads_split_by_floor(sat):
    spec = sat.tiny(hidden=192, ffn=384, q_heads=3, kv_heads=1, head_dim=64, vocab=1002)
    assert [sat.shard_ranges(spec, r, 2)["q_heads"] for r in range(2)] == [(0, 1), (1, 3)]
    assert [sat.shard_ranges(spec, r, 2)["kv_heads"] for r in range(2)] == [(0, 1), (0, 1)]


def test_shapes_that_do_not_shard_are_rejected(sat):
    with pytest.raises(sat.NotSupportedError):
        sat.shard_ranges(sat.tiny(vocab=1001), 0, 2)           # vocab rows
    with pytest.raises(sat.NotSupportedError):
        sat.shard_ranges(sat.tiny(q_heads=4, kv_heads=2), 0, 8)  # fewer query heads than ranks


def test_sharded_create_checks_arguments_before_touching_a_device(sat):
    import ctypes as C
    lib = sat._lib.lib()
    h = C.c_void_p()
    assert lib.satori_session_create_sharded(None, None, 8, 0, 2, None, C.byref(h)) == sat._lib.ERR_ARGUMENT


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gloo_rank(rank, world, port, q):
    import torch.distributed as dist

    import satori_b200 as sat
    dist.init_process_group("gloo", init_method="tcp://127.0.0.1:%d" % port, rank=rank, world_size=world)
    try:
        q.put((rank, sat.broadcast_nccl_id()))
    finally:
        dist.destroy_process_group()


def test_nccl_id_reaches_every_rank_over_gloo(sat):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gloo_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(60)
    assert [p.exitcode for p in procs] == [0, 0]
    assert len(got[0]) == 128 and got[0] == got[1]


# ---------------------------------------------------------------- row-sharded MatVec (satori_matrix_create_sharded)
@pytest.mark.parametrize("rows,world", [(11008, 8), (11008, 3), (1003, 4), (1003, 8), (5, 5), (1, 1)])
def test_sharded_matrix_rows_tile_the_matrix(sat, rows, world):
    cover = np.zeros(rows, np.int32)
    s = -(-rows // world)
    for r in range(world):
        a, b = sat.sharded_matrix_rows(rows, r, world)
        assert a == r * s and 0 <= a < b <= rows
        cover[a:b] += 1
    assert np.all(cover == 1)


def test_sharded_matrix_rejects_ranks_without_rows(sat):
    with pytest.raises(sat.NotSupportedError):
        sat.sharded_matrix_rows(5, 0, 4)          # S = 2: rank 3 would start at row 6
    with pytest.raises(sat.ArgumentError):
        sat.sharded_matrix_rows(8, 2, 2)


def test_sharded_matrix_create_checks_arguments_before_touching_a_device(sat):
    import ctypes as C
    lib = sat._lib.lib()
    h = C.c_void_p()
    assert lib.satori_matrix_create_sharded(None, None, 0, 8, 32, 0, 0, 0, 2, None, C.byref(h)) == sat._lib.ERR_ARGUMENT


def _gloo_sharded_matvec(rank, world, port, q):
    """One rank of a row-sharded Q4_0 MatVec on the CPU: its row block through the oracle's ExecuteBatch
    restatement, then a gloo all-gather of the padded slices (the collective the GPU path runs over NCCL)."""
    import torch
    import torch.distributed as dist

    import satori_b200 as sat
    from oracle import oracle
    dist.init_process_group("gloo", init_method="tcp://127.0.0.1:%d" % port, rank=rank, world_size=world)
    try:
        rows, cols = 1003, 256
        rng = np.random.default_rng(7)
        payload = oracle.q_quantize((rng.standard_normal(rows * cols) * 0.02).astype(np.float32), rows, cols, 1)
        x = rng.standard_normal(cols).astype(np.float32)
        a, b = sat.sharded_matrix_rows(rows, rank, world)
        s = -(-rows // world)
        mine = oracle.q_matvec(payload[a * (cols // 32) * 18:b * (cols // 32) * 18], b - a, cols, 1, x, order="batch")
        slot = torch.zeros(s, dtype=torch.float32)
        slot[:b - a] = torch.from_numpy(np.asarray(mine, np.float32))
        parts = [torch.zeros(s, dtype=torch.float32) for _ in range(world)]
        dist.all_gather(parts, slot)
        y = torch.cat(parts)[:rows].numpy()
        full = np.asarray(oracle.q_matvec(payload, rows, cols, 1, x, order="batch"), np.float32)
        q.put((rank, bool(np.array_equal(y.view(np.uint32), full.view(np.uint32)))))
    finally:
        dist.destroy_process_group()


def test_sharded_matvec_rows_and_gather_over_gloo(sat, oracle_lib):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gloo_sharded_matvec, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(60)
    assert got == {0: True, 1: True}
