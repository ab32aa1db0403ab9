"""CPU: the token-row slicing of bench.py's tensor-parallel block (the slices whose
reductions overlap the next GEMM slice) and the sequence-parallel row layout, checked
with two gloo ranks: reduce-scatter emulated per slice, then all-gathered back, must
reproduce the all-reduced tensor."""
import os
import sys

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

sys.path.insert(0, os.path.join(os.path.dirname(__file__), ".."))
import bench  # noqa: E402


@pytest.mark.parametrize("M,chunks,world", [(4608, 2, 2), (4608, 2, 8), (32760, 4, 8), (32760, 4, 4), (4096, 3, 2),
                                           (64, 4, 2)])
def test_slice_bounds_cover_rows_and_divide(M, chunks, world):
    b = bench.slice_bounds(M, chunks, world)
    assert b[0][0] == 0 and b[-1][1] == M
    assert all(b[i][1] == b[i + 1][0] for i in range(len(b) - 1))
    assert all((r1 - r0) % world == 0 and r1 > r0 for r0, r1 in b)
    assert all((r1 - r0) % (32 * world) == 0 for r0, r1 in b[:-1])
    assert len(b) <= chunks


def test_slice_bounds_rejects_indivisible_rows():
    with pytest.raises(ValueError):
        bench.slice_bounds(4610, 2, 4)


def _worker(rank, world, port, M, N, chunks, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    g = torch.Generator().manual_seed(100 + rank)
    part = torch.randn(M, N, generator=g)               # this rank's partial sums
    full = part.clone()
    dist.all_reduce(full)                                # the reference: one all-reduce
    shard = torch.empty(M // world, N)
    gathered = torch.empty(M, N)
    for r0, r1 in bench.slice_bounds(M, chunks, world):
        s = part[r0:r1].clone()
        dist.all_reduce(s)                               # reduce-scatter of the slice ...
        k = (r1 - r0) // world
        shard[r0 // world:r1 // world] = s[rank * k:(rank + 1) * k]   # ... keeps rank's rows
        outs = [torch.empty(k, N) for _ in range(world)]
        dist.all_gather(outs, shard[r0 // world:r1 // world].contiguous())
        gathered[r0:r1] = torch.cat(outs)
    q.put((rank, bool(torch.allclose(gathered, full))))
    dist.destroy_process_group()


def test_sequence_parallel_layout_round_trips_gloo():
    world, M, N = 2, 4608, 8
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29600 + os.getpid() % 200
    ps = [ctx.Process(target=_worker, args=(r, world, port, M, N, 2, q)) for r in range(world)]
    for p in ps:
        p.start()
    res = [q.get(timeout=120) for _ in ps]
    for p in ps:
        p.join(timeout=60)
    assert all(ok for _, ok in res), res
