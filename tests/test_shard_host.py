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
