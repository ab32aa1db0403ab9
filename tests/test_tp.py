"""CPU: Megatron tensor parallelism of packed Q4/Q8 linears (qlinear.tp), run as gloo ranks.

* the sharding helpers against the unsharded products (oracle arithmetic);
* qlinear.tp.TPBlock -- the product's sharded block, the same code bench.py times on the
  GPUs -- driven with CPU tensors and the oracle as the per-linear matmul, against
  qlinear.tp.reference_forward (the unsharded chain) in both reduction modes;
* the token-row slicing of the overlapped reductions;
* qlinear.tp.Comm: a rank that never joins a collective ends the other rank's bounded wait
  with CommError (the group is aborted) instead of a hang.
The reference is single-device (gen-core/src/runtime.rs:56-58); the sharded call is
LinearBase::forward's quantized_matmul + bias (src/adapters.rs:300-322)."""
import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle as O
from helpers import rand_bf16


def _T(a):
    return torch.from_numpy(np.ascontiguousarray(a.view(np.int32) if a.dtype == np.uint32 else a.view(np.int16)))


def _bf(t):
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def oracle_matmul(x, lin, out, max_ctas):
    """qlinear.tp's per-linear matmul hook on CPU tensors: the oracle's exact-mode
    quantized_matmul with the reference's rounding points (bias after rounding, GELU op by op)."""
    act = {None: O.ACT_NONE, "gelu_tanh": O.ACT_GELU_TANH}[lin.act]
    y = O.quantized_matmul(_bf(x), lin.wq.numpy().view(np.uint32), _bf(lin.scales), _bf(lin.biases),
                           lin.group_size, lin.bits, bias=None if lin.bias is None else _bf(lin.bias), act=act)
    out.copy_(torch.from_numpy(y.view(np.int16)).view(torch.bfloat16))


FLUX_SPEC = [("qkv", None, "col", "x"), ("out", None, "row", "attn"), ("up", "gelu_tanh", "col", "out"),
             ("down", None, "row", "up")]
WAN_SPEC = [("q", None, "col", "x"), ("v", None, "col", "x"), ("o", None, "row", "v"), ("cq", None, "col", "o"),
            ("co", None, "row", "cq"), ("up", "gelu_tanh", "col", "co"), ("down", None, "row", "up")]


def _weights(spec, hidden, mlp, gs, bits, seed):
    rng = np.random.default_rng(seed)
    shapes = {"qkv": (3 * hidden, hidden), "out": (hidden, hidden), "up": (mlp, hidden), "down": (hidden, mlp),
              "q": (hidden, hidden), "v": (hidden, hidden), "o": (hidden, hidden), "cq": (hidden, hidden),
              "co": (hidden, hidden)}
    W = {}
    for name, *_ in spec:
        N, K = shapes[name]
        wq, s, b = O.quantize(rand_bf16((N, K), 0.02, rng), gs, bits)
        W[name] = (_T(wq), _T(s).view(torch.bfloat16), _T(b).view(torch.bfloat16),
                   _T(rand_bf16((N,), 0.02, rng)).view(torch.bfloat16))
    x = _T(rand_bf16((128, hidden), 1.0, rng)).view(torch.bfloat16)
    attn = _T(rand_bf16((128, hidden), 1.0, rng)).view(torch.bfloat16)
    return W, x, {"attn": attn}


def _block_worker(rank, world, port, specname, mode, bits, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from qlinear import tp

    spec = FLUX_SPEC if specname == "flux" else WAN_SPEC
    W, x, ext = _weights(spec, 256, 512, 64, bits, 7)
    comm = tp.Comm(None, timeout_s=60)
    blk = tp.TPBlock(spec, W, 64, bits, x.shape[0], comm=comm, chunks=2, mode=mode,
                     device=torch.device("cpu"), matmul=oracle_matmul)
    blk.forward(x, ext)
    got = blk.gather_output()
    ref = tp.reference_forward(spec, W, 64, bits, x, ext, matmul=oracle_matmul)["out"]
    q.put((rank, tp.parity(got, ref, world), blk.bounds, blk.launches))
    comm.close()


def _spawn(target, world, args):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + (os.getpid() * 7 + hash(args) % 500) % 2000
    ps = [ctx.Process(target=target, args=(r, world, port) + args + (q,)) for r in range(world)]
    for p in ps:
        p.start()
    res = [q.get(timeout=180) for _ in ps]
    for p in ps:
        p.join(60)
        assert p.exitcode == 0
    return sorted(res, key=lambda r: r[0])


@pytest.mark.parametrize("specname,mode,bits", [("flux", "allreduce", 8), ("wan", "seqpar", 4),
                                                ("wan", "allreduce", 4)])
def test_tp_block_matches_unsharded_gloo(specname, mode, bits):
    for rank, par, bounds, launches in _spawn(_block_worker, 2, (specname, mode, bits)):
        assert par["ok"], (rank, par)
        assert par["rel_l2"] < 1e-2
        assert bounds == [(0, 64), (64, 128)]


def _shard_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from qlinear import tp

    rng = np.random.default_rng(0)
    N, K, M, gs, bits = 64, 512, 5, 64, 4
    w = rand_bf16((N, K), 0.02, rng)
    x = O.to_f32(rand_bf16((M, K), 1.0, rng))
    wq, s, b = O.quantize(w, gs, bits)
    # row-parallel: K split on group boundaries, partial sums all-reduced
    rq, rs, rb, k0, k1 = tp.row_shard(_T(wq), _T(s), _T(b), gs, bits, rank, world)
    d = O.to_f32(O.dequantize(rq.numpy().view(np.uint32), rs.numpy().view(np.uint16),
                              rb.numpy().view(np.uint16), gs, bits, out_dtype=O.F32))
    part = torch.from_numpy((x[:, k0:k1].astype(np.float64) @ d.T.astype(np.float64)))
    dist.all_reduce(part)
    full = x.astype(np.float64) @ O.to_f32(O.dequantize(wq, s, b, gs, bits, out_dtype=O.F32)).T
    # column-parallel: rows split, shards gathered
    cq, cs, cb, _ = tp.column_shard(_T(wq), _T(s), _T(b), None, rank, world)
    dc = O.to_f32(O.dequantize(cq.numpy().view(np.uint32), cs.numpy().view(np.uint16),
                               cb.numpy().view(np.uint16), gs, bits, out_dtype=O.F32))
    yc = torch.from_numpy(x.astype(np.float64) @ dc.T.astype(np.float64))
    parts = [torch.empty_like(yc) for _ in range(world)]
    dist.all_gather(parts, yc)
    q.put((rank, float(np.abs(part.numpy() - full).max()), float(np.abs(torch.cat(parts, 1).numpy() - full).max())))
    dist.destroy_process_group()


def test_tp_row_and_column_parallel_gloo():
    for _, row_err, col_err in _spawn(_shard_worker, 2, ()):
        assert row_err < 1e-9 and col_err < 1e-9


def _timeout_worker(rank, world, port, how, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    from qlinear import tp

    comm = tp.Comm(None, timeout_s=1.0)
    if rank == 1:  # this rank never joins the collective: it idles, or its process exits
        q.put((rank, "idle"))
        if how == "idle":
            import time
            time.sleep(4)
        return
    t = torch.ones(4)
    comm.all_reduce(t)
    try:
        comm.wait()
        q.put((rank, "completed"))
    except tp.CommError as e:
        q.put((rank, "CommError" if comm.aborted else f"not aborted: {e}"))


@pytest.mark.parametrize("how", ["idle", "exit"])
def test_comm_wait_times_out_and_aborts_gloo(how):
    res = dict(_spawn(_timeout_worker, 2, (how,)))
    assert res[0] == "CommError", res
    assert res[1] == "idle"


@pytest.mark.parametrize("M,chunks,world", [(4608, 2, 2), (4608, 2, 8), (32760, 4, 8), (32760, 4, 4), (4096, 3, 2),
                                           (64, 4, 2)])
def test_slice_bounds_cover_rows_and_divide(M, chunks, world):
    from qlinear import tp

    b = tp.slice_bounds(M, chunks, world)
    assert b[0][0] == 0 and b[-1][1] == M
    assert all(b[i][1] == b[i + 1][0] for i in range(len(b) - 1))
    assert all((r1 - r0) % world == 0 and r1 > r0 for r0, r1 in b)
    assert all((r1 - r0) % (32 * world) == 0 for r0, r1 in b[:-1])
    assert len(b) <= chunks


def test_slice_bounds_rejects_indivisible_rows():
    from qlinear import tp

    with pytest.raises(ValueError):
        tp.slice_bounds(4610, 2, 4)


def test_row_shard_rejects_unaligned_split():
    from qlinear import tp

    wq = torch.zeros(4, 3840 * 4 // 32, dtype=torch.int32)
    s = torch.zeros(4, 3840 // 64, dtype=torch.bfloat16)
    with pytest.raises(ValueError):  # Z-Image to_out K=3840 at TP=8 is 7.5 groups per rank
        tp.row_shard(wq, s, s, 64, 4, 0, 8)


def test_tp_linear_bias_on_rank0_only():
    from qlinear import tp

    wq = torch.zeros(8, 128 * 4 // 32, dtype=torch.int32)
    s = torch.zeros(8, 2, dtype=torch.bfloat16)
    bias = torch.ones(8, dtype=torch.bfloat16)
    l0 = tp.TPLinear(wq, s, s, bias, 64, 4, "row", 0, 2)
    l1 = tp.TPLinear(wq, s, s, bias, 64, 4, "row", 1, 2)
    lc = tp.TPLinear(wq, s, s, bias, 64, 4, "col", 1, 2)
    assert l0.bias is not None and l1.bias is None and (l0.k0, l0.k1, l1.k0, l1.k1) == (0, 64, 64, 128)
    assert lc.N == 4 and lc.bias.shape == (4,)
