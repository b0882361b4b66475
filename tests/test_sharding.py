"""Batch-row sharding host logic on 2 CPU ranks (gloo): row split and the final gather."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from dwarf_v2_b200.sharding import gather_rows, rows_for_rank


def test_rows_for_rank_partition():
    parts = [rows_for_rank(256, r, 8) for r in range(8)]
    assert [p.start for p in parts] == list(range(0, 256, 32)) and parts[-1].stop == 256
    with pytest.raises(ValueError):
        rows_for_rank(256, 0, 3)
    with pytest.raises(ValueError):
        rows_for_rank(256, 4, 4)


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        full = torch.arange(8 * 5, dtype=torch.float32).reshape(8, 5)
        mine = full[rows_for_rank(8, rank, world)]
        got = gather_rows(mine * 1.0)
        q.put((rank, bool(torch.equal(got, full))))
    finally:
        dist.destroy_process_group()


def test_gather_rows_two_gloo_ranks():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert results == {0: True, 1: True}
