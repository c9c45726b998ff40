"""Sharding host logic: balanced ranges, and the all-gather of uneven row shards across
two gloo ranks on CPU (the multi-GPU path's only collective)."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from enigma.shard import shard_range, shard_sizes


@pytest.mark.parametrize("n,world", [(0, 1), (7, 2), (262144, 8), (5, 8), (256, 3)])
def test_shard_range_covers_once(n, world):
    spans = [shard_range(n, world, r) for r in range(world)]
    assert spans[0][0] == 0 and spans[-1][1] == n
    assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
    sizes = shard_sizes(n, world)
    assert max(sizes) - min(sizes) <= 1 and sum(sizes) == n


def test_shard_range_rejects_bad_rank():
    with pytest.raises(ValueError):
        shard_range(10, 2, 2)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _gather_worker(rank, world, port, rows, q):
    import torch.distributed as dist
    from enigma.shard import gather_rows, shard_range
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world)
    try:
        lo, hi = shard_range(rows, world, rank)
        full = torch.arange(rows * 3, dtype=torch.float32).reshape(rows, 3)
        got = gather_rows(full[lo:hi].clone(), rows)
        q.put((rank, bool(torch.equal(got, full))))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("rows", [7, 8])
def test_gather_rows_two_gloo_ranks(rows):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gather_worker, args=(r, 2, port, rows, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert results == {0: True, 1: True}


def _fail_worker(rank, world, port, q):
    """Rank 1 leaves before the collective; rank 0 must get an error, not hang."""
    import datetime
    import torch.distributed as dist
    from enigma.shard import gather_rows
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        os._exit(0)
    try:
        gather_rows(torch.zeros(1, 2), 2)
        q.put("no error")
    except Exception as e:  # noqa: BLE001 - any failure of the collective is the point
        q.put(type(e).__name__)


def test_gather_rows_peer_exit_is_reported():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_fail_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert out != "no error"


def _decode_cfg_worker(rank, world, port, q):
    import torch.distributed as dist
    from enigma.decode_layer import DecodeConfig
    from enigma.shard import decode_shard_config
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world)
    try:
        q.put((rank, decode_shard_config(DecodeConfig(batch=7)).batch))
    finally:
        dist.destroy_process_group()


def test_decode_shard_config_two_ranks():
    """Sequences of a decode batch split across gloo ranks: 7 -> 4 + 3, nothing else changes."""
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_decode_cfg_worker, args=(r, world, port, q)) for r in range(world)]
    for p in ps:
        p.start()
    got = dict(q.get(timeout=120) for _ in range(world))
    for p in ps:
        p.join(timeout=60)
    assert got == {0: 4, 1: 3}
