"""GPU: qlinear.tp's TPBlock on the CUDA GEMM.

* one process: the block with no communicator equals the unsharded chain
  (reference_forward) bit for bit -- the same kernels in the same order;
* two or more GPUs (skipped otherwise): NCCL ranks run the sharded FLUX-shaped block
  (column / row parallel, M-sliced all-reduce) and the sequence-parallel Wan-shaped block,
  and the gathered output must meet qlinear.tp.parity's bound against the unsharded chain
  computed on each rank.  The reference is single-device; the sharded call is
  LinearBase::forward's quantized_matmul + bias (src/adapters.rs:300-322)."""
import os

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

FLUX_SPEC = [("qkv", None, "col", "x"), ("out", None, "row", "attn"), ("up", "gelu_tanh", "col", "out"),
             ("down", None, "row", "up")]
WAN_SPEC = [("q", None, "col", "x"), ("v", None, "col", "x"), ("o", None, "row", "v"), ("cq", None, "col", "o"),
            ("co", None, "row", "cq"), ("up", "gelu_tanh", "col", "co"), ("down", None, "row", "up")]


def _weights(dev, spec, hidden, mlp, bits, seed):
    import qlinear
    g = torch.Generator(device=dev).manual_seed(seed)
    shapes = {"qkv": (3 * hidden, hidden), "out": (hidden, hidden), "up": (mlp, hidden), "down": (hidden, mlp),
              "q": (hidden, hidden), "v": (hidden, hidden), "o": (hidden, hidden), "cq": (hidden, hidden),
              "co": (hidden, hidden)}
    W = {}
    for name, *_ in spec:
        N, K = shapes[name]
        w = (torch.randn(N, K, device=dev, generator=g) * 0.02).to(torch.bfloat16)
        b = (torch.randn(N, device=dev, generator=g) * 0.02).to(torch.bfloat16)
        W[name] = (*qlinear.quantize(w, 64, bits), b)
    x = torch.randn(1024, hidden, device=dev, generator=g).to(torch.bfloat16)
    attn = torch.randn(1024, hidden, device=dev, generator=g).to(torch.bfloat16)
    return W, x, {"attn": attn}


@pytest.mark.parametrize("specname,bits", [("flux", 8), ("wan", 4)])
def test_tp_block_single_gpu_is_the_unsharded_chain(dev, specname, bits):
    from qlinear import tp
    spec = FLUX_SPEC if specname == "flux" else WAN_SPEC
    W, x, ext = _weights(dev, spec, 1024, 2048, bits, 3)
    blk = tp.TPBlock(spec, W, 64, bits, x.shape[0], comm=None, device=dev)
    got = blk.forward(x, ext).clone()
    ref = tp.reference_forward(spec, W, 64, bits, x, ext)["out"]
    torch.cuda.synchronize()
    assert torch.equal(got, ref)
    par = tp.parity(got, ref, 1)
    assert par["ok"] and par["bitwise_equal"]


@pytest.mark.parametrize("specname,bits", [("flux", 8), ("wan", 4)])
def test_tp_block_graph_replay_is_the_eager_forward(dev, specname, bits):
    """TPBlock.capture: a CUDA-graph replay gives the eager forward's output bit for bit,
    and a replay after the bound input changed follows the new input."""
    from qlinear import tp
    spec = FLUX_SPEC if specname == "flux" else WAN_SPEC
    W, x, ext = _weights(dev, spec, 1024, 2048, bits, 3)
    blk = tp.TPBlock(spec, W, 64, bits, x.shape[0], comm=None, device=dev)
    want = blk.forward(x, ext).clone()
    xb = x.clone()
    gr = blk.capture(xb, ext)
    assert torch.equal(gr.replay(), want)
    x2 = torch.randn_like(x)
    want2 = blk.forward(x2, ext).clone()
    xb.copy_(x2)
    got2 = gr.replay().clone()
    torch.cuda.synchronize()
    assert torch.equal(got2, want2)


def _rank(rank, world, port, specname, mode, q, graph=False):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    from qlinear import tp
    comm = tp.Comm.init("nccl", device=dev, timeout_s=60)
    spec = FLUX_SPEC if specname == "flux" else WAN_SPEC
    W, x, ext = _weights(dev, spec, 1024, 2048, 8 if specname == "flux" else 4, 5)
    blk = tp.TPBlock(spec, W, 64, 8 if specname == "flux" else 4, x.shape[0], comm=comm, chunks=2, mode=mode,
                     device=dev)
    if graph:
        xb = x.clone()
        gr = blk.capture(xb, ext)
        xb.zero_()
        gr.replay()
        xb.copy_(x)  # the replay that counts reads the refilled input
        gr.replay()
    else:
        blk.forward(x, ext)
    got = blk.gather_output()
    if graph:
        gr.reset()  # before the communicator's teardown
    ref = tp.reference_forward(spec, W, 64, 8 if specname == "flux" else 4, x, ext)["out"]
    torch.cuda.synchronize()
    q.put((rank, tp.parity(got, ref, world)))
    comm.close()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("specname,mode,graph", [("flux", "allreduce", False), ("wan", "seqpar", False),
                                                  ("flux", "allreduce", True), ("wan", "seqpar", True)])
def test_tp_block_two_gpus_matches_unsharded(specname, mode, graph):
    """NCCL ranks, eager and as a captured CUDA graph (collectives inside the graph)."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29700 + (os.getpid() * 4 + 2 * graph + (mode == "seqpar")) % 200
    ps = [ctx.Process(target=_rank, args=(r, 2, port, specname, mode, q, graph)) for r in range(2)]
    for p in ps:
        p.start()
    res = [q.get(timeout=300) for _ in ps]
    for p in ps:
        p.join(60)
        assert p.exitcode == 0
    for rank, par in res:
        assert par["ok"], (rank, par)
