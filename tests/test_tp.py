"""CPU: Megatron sharding of packed weights (qlinear.tp) and the row-parallel all-reduce,
run as two gloo ranks.  The per-rank partial products are computed with the oracle; the
all-reduced sum must equal the unsharded result (column shards must concatenate to it)."""
import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle as O
from helpers import rand_bf16


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from qlinear import tp

    rng = np.random.default_rng(0)
    N, K, M, gs, bits = 64, 512, 5, 64, 4
    w = rand_bf16((N, K), 0.02, rng)
    x = O.to_f32(rand_bf16((M, K), 1.0, rng))
    wq, s, b = O.quantize(w, gs, bits)
    T = lambda a: torch.from_numpy(a.view(np.int32) if a.dtype == np.uint32 else a.view(np.int16))
    # row-parallel: K split on group boundaries, partial sums all-reduced
    rq, rs, rb, k0, k1 = tp.row_shard(T(wq), T(s), T(b), gs, bits, rank, world)
    d = O.to_f32(O.dequantize(rq.numpy().view(np.uint32), rs.numpy().view(np.uint16),
                              rb.numpy().view(np.uint16), gs, bits, out_dtype=O.F32))
    part = torch.from_numpy((x[:, k0:k1].astype(np.float64) @ d.T.astype(np.float64)))
    dist.all_reduce(part)
    full = x.astype(np.float64) @ O.to_f32(O.dequantize(wq, s, b, gs, bits, out_dtype=O.F32)).T
    # column-parallel: rows split, shards gathered
    cq, cs, cb, _ = tp.column_shard(T(wq), T(s), T(b), None, rank, world)
    dc = O.to_f32(O.dequantize(cq.numpy().view(np.uint32), cs.numpy().view(np.uint16),
                               cb.numpy().view(np.uint16), gs, bits, out_dtype=O.F32))
    yc = torch.from_numpy(x.astype(np.float64) @ dc.T.astype(np.float64))
    parts = [torch.empty_like(yc) for _ in range(world)]
    dist.all_gather(parts, yc)
    q.put((rank, float(np.abs(part.numpy() - full).max()), float(np.abs(torch.cat(parts, 1).numpy() - full).max())))
    dist.destroy_process_group()


def test_tp_row_and_column_parallel_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + os.getpid() % 1000
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(30)
        assert p.exitcode == 0
    for _, row_err, col_err in res:
        assert row_err < 1e-9 and col_err < 1e-9


def test_row_shard_rejects_unaligned_split():
    from qlinear import tp

    wq = torch.zeros(4, 3840 * 4 // 32, dtype=torch.int32)
    s = torch.zeros(4, 3840 // 64, dtype=torch.bfloat16)
    with pytest.raises(ValueError):  # Z-Image to_out K=3840 at TP=8 is 7.5 groups per rank
        tp.row_shard(wq, s, s, 64, 4, 0, 8)
