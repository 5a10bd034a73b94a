"""The multi-GPU bench's host plumbing on CPU: two gloo ranks (the bench's own
dist_setup, all_max, all_sum, barrier) and the per-rank config 5 prompts.

bench.py runs one independent sequence (or batch) per GPU and meets the other
ranks only on the host: the timed region's max over ranks and the box-total
token counts. These checks need no GPU.
"""

import os
import socket
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, ws, port, q):
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(ws), LOCAL_RANK=str(rank),
                      MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    sys.path.insert(0, ROOT)
    import bench
    import torch.distributed as dist

    try:
        got_ws, got_rank, local = bench.dist_setup()
        times = bench.all_max([1.0 + rank, 10.0 - rank], got_ws)
        toks = bench.all_sum([127.0, 64.0 * (rank + 1)], got_ws)
        bench.barrier(got_ws)
        prompts = bench.c5_prompts(got_rank)
        q.put((rank, got_ws, got_rank, local, times, toks, [len(p) for p in prompts[:4]], int(prompts[0][0])))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def test_two_gloo_ranks():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = {}
    for _ in procs:
        r = q.get(timeout=120)
        out[r[0]] = r
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r in (0, 1):
        _, ws, rank, local, times, toks, lens, first = out[r]
        assert (ws, rank, local) == (2, r, r)
        assert times == [2.0, 10.0]            # max over ranks of each timed quantity
        assert toks == [254.0, 64.0 + 128.0]   # box totals
    # each rank's config 5 prompts are its own, seeded (lengths on the workload's range)
    assert out[0][6] != out[1][6] or out[0][7] != out[1][7]
    for r in (0, 1):
        assert all(16 <= n <= 512 for n in out[r][6])


def test_single_rank_is_local():
    sys.path.insert(0, ROOT)
    import bench

    assert bench.all_max([3.0, 1.0], 1) == [3.0, 1.0]
    assert bench.all_sum([3.0, 1.0], 1) == [3.0, 1.0]
    bench.barrier(1)
    assert bench.c5_prompts(0)[0].tolist() == bench.c5_prompts(0)[0].tolist()


if __name__ == "__main__":
    pytest.main([__file__, "-q"])
