"""Megatron-style tensor parallelism on packed Q4/Q8 weights.

The reference is single-device (gen-core/src/runtime.rs:56-59): every quantized linear
is one ``quantized_matmul`` call followed by its bias add (src/adapters.rs:300-322).
This module shards those calls over the GPUs of one node, one process per GPU:

* Column-parallel linears (QKV, MLP up, Wan's q/k/v/cross-q/FFN-up) split W's output
  rows.  Each packed row is self-contained, so a rank keeps rows ``[r*N/P, (r+1)*N/P)``
  of wq, scales, biases and the dense bias; its output shard needs no communication.
* Row-parallel linears (attention out, MLP down) split K on group boundaries: a rank
  keeps words ``[K0*bits/32, K1*bits/32)`` and groups ``[K0/gs, K1/gs)`` of every row
  and produces a partial ``[M, N]`` sum that a collective completes.  The dense bias is
  added once: rank 0's GEMM adds it to its (rounded) partial, the others add none.

``TPBlock`` runs a chain of such linears with their real data dependencies: a linear
that reads a row-parallel output waits for that output's reduction.  Communication
overlaps computation in token-row slices: a row-parallel linear runs slice by slice, the
reduction of slice i runs on a second stream while the GEMM of slice i+1 runs, and the
consumer starts its slice i as soon as slice i is reduced.  Two reduction modes:
``"allreduce"`` (one all-reduce per slice) and ``"seqpar"`` (sequence parallel: a
reduce-scatter over the token rows, then an all-gather for the consumer -- the same bytes
in two shorter collectives).

``Comm`` is the communicator handle: the process group, an initialisation timeout, a
bounded host-side wait on outstanding collectives (the equivalent of polling
``ncclCommGetAsyncError``) and ``abort``.  Every collective is issued asynchronously and
tracked; ``Comm.wait`` raises ``CommError`` after aborting the group when a collective
fails or does not finish in time, so a dead or missing peer ends the step with an error
instead of a hang.
"""
from __future__ import annotations

import datetime
import os
import time
from typing import Callable, Dict, List, Optional, Sequence, Tuple

import torch
import torch.distributed as dist


# ----------------------------------------------------------------------------- sharding

def column_shard(wq: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor,
                 bias: Optional[torch.Tensor], rank: int, world: int):
    """Rows ``[rank*N/world, (rank+1)*N/world)`` of a packed linear (and of its dense bias)."""
    N = scales.shape[0]
    if N % world:
        raise ValueError(f"column-parallel split needs N % world == 0 (N={N}, world={world})")
    n0, n1 = rank * N // world, (rank + 1) * N // world
    return (wq[n0:n1].contiguous(), scales[n0:n1].contiguous(), biases[n0:n1].contiguous(),
            None if bias is None else bias[n0:n1].contiguous())


def row_bounds(G: int, group_size: int, rank: int, world: int) -> Tuple[int, int]:
    """K range ``[k0, k1)`` of rank's row-parallel slice (whole groups)."""
    if G % world:
        raise ValueError(f"row-parallel split must fall on group boundaries "
                         f"(K={G * group_size}, gs={group_size}, world={world})")
    g0, g1 = rank * G // world, (rank + 1) * G // world
    return g0 * group_size, g1 * group_size


def row_shard(wq: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor, group_size: int, bits: int,
              rank: int, world: int) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor, int, int]:
    """Split K into `world` group-aligned slices; returns (wq, scales, biases, k0, k1)."""
    G = scales.shape[1]
    k0, k1 = row_bounds(G, group_size, rank, world)
    g0, g1 = k0 // group_size, k1 // group_size
    w0, w1 = k0 * bits // 32, k1 * bits // 32
    return (wq[:, w0:w1].contiguous(), scales[:, g0:g1].contiguous(), biases[:, g0:g1].contiguous(), k0, k1)


def slice_bounds(M: int, chunks: int, world: int) -> List[Tuple[int, int]]:
    """Token-row slices ``[(r0, r1), ...]`` for the overlapped reductions: about `chunks`
    slices, each a multiple of 32 * world rows except possibly the last, and every slice a
    multiple of `world` rows (a reduce-scatter gives each rank (r1 - r0) / world rows)."""
    if M % world:
        raise ValueError("M must be a multiple of the GPU count")
    unit = 32 * world
    step = (M + chunks - 1) // chunks
    step = (step + unit - 1) // unit * unit
    return [(r0, min(M, r0 + step)) for r0 in range(0, M, step)]


# ----------------------------------------------------------------------------- communicator

class CommError(RuntimeError):
    """A collective failed or did not complete within the communicator's timeout; the
    process group has been aborted."""


class Comm:
    """Communicator handle over a torch.distributed process group (NCCL on GPUs, gloo on
    CPU).  Collectives are issued with ``async_op=True`` and tracked until ``wait``."""

    def __init__(self, group=None, timeout_s: float = 60.0):
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.timeout_s = float(timeout_s)
        self._pending: List = []
        self.aborted = False

    @classmethod
    def init(cls, backend: str = "nccl", device: Optional[torch.device] = None, timeout_s: float = 60.0,
             init_timeout_s: Optional[float] = None) -> "Comm":
        """Initialise the default process group from the torchrun environment (RANK,
        WORLD_SIZE, MASTER_ADDR, MASTER_PORT).  `init_timeout_s` bounds the rendezvous and
        every collective inside the backend (NCCL's watchdog aborts a communicator whose
        collective exceeds it); `timeout_s` bounds ``Comm.wait`` on the host."""
        if backend == "nccl":
            # the watchdog tears the communicator down on an asynchronous NCCL error
            # (ncclCommGetAsyncError) instead of leaving later collectives to hang
            os.environ.setdefault("TORCH_NCCL_ASYNC_ERROR_HANDLING", "3")
        kw = {"timeout": datetime.timedelta(seconds=init_timeout_s or timeout_s)}
        if device is not None and backend == "nccl":
            kw["device_id"] = device
        dist.init_process_group(backend, **kw)
        return cls(None, timeout_s)

    # collectives (on the current stream; the caller picks the stream)
    def _track(self, work, t: Optional[torch.Tensor] = None):
        if work is not None:
            self._pending.append(work)
            if t is not None and t.is_cuda:
                # orders the current CUDA stream after the collective; the host does not block
                work.wait()
        return work

    def all_reduce(self, t: torch.Tensor):
        return self._track(dist.all_reduce(t, group=self.group, async_op=True), t)

    def reduce_scatter(self, out: torch.Tensor, inp: torch.Tensor):
        if not inp.is_cuda:
            # gloo has no reduce-scatter of a flat tensor: all-reduce a copy, keep this rank's rows
            full = inp.contiguous().clone()
            self._track(dist.all_reduce(full, group=self.group, async_op=True), full)
            self.wait()
            k = out.shape[0]
            out.copy_(full[self.rank * k:(self.rank + 1) * k])
            return None
        return self._track(dist.reduce_scatter_tensor(out, inp, group=self.group, async_op=True), out)

    def all_gather(self, out: torch.Tensor, inp: torch.Tensor):
        return self._track(dist.all_gather_into_tensor(out, inp, group=self.group, async_op=True), out)

    def broadcast(self, t: torch.Tensor, src: int = 0):
        return self._track(dist.broadcast(t, src, group=self.group, async_op=True), t)

    def poll(self) -> bool:
        """True when every tracked collective has completed (drops the completed ones).  A
        collective that completed with an error raises it here."""
        still = []
        for w in self._pending:
            if w.is_completed():
                w.wait()  # returns at once; raises the collective's error, if any
            else:
                still.append(w)
        self._pending = still
        return not still

    def wait(self, timeout_s: Optional[float] = None) -> None:
        """Bounded wait for the tracked collectives.  On timeout or failure the group is
        aborted and CommError raised."""
        limit = self.timeout_s if timeout_s is None else float(timeout_s)
        t0 = time.monotonic()
        try:
            while not self.poll():
                if time.monotonic() - t0 > limit:
                    self.abort()
                    raise CommError(f"rank {self.rank}: {len(self._pending)} collective(s) did not complete "
                                    f"within {limit:.1f} s; process group aborted")
                time.sleep(0.0005)
        except CommError:
            raise
        except Exception as e:  # a collective raised (peer gone, transport error)
            self.abort()
            raise CommError(f"rank {self.rank}: collective failed: {e}") from e

    def barrier(self) -> None:
        self._track(dist.barrier(group=self.group, async_op=True))
        self.wait()

    def abort(self) -> None:
        """Abort the process group (pending collectives end with an error) and forget them."""
        if self.aborted:
            return
        self.aborted = True
        self._pending = []
        abort = getattr(dist.distributed_c10d, "_abort_process_group", None)
        try:
            if abort is not None:
                abort(self.group) if self.group is not None else abort()
            else:
                dist.destroy_process_group(self.group)
        except Exception:
            pass

    def close(self) -> None:
        if not self.aborted and dist.is_initialized():
            dist.destroy_process_group(self.group)


# ----------------------------------------------------------------------------- sharded linears and block

def default_matmul(x, lin, out, max_ctas):
    """One quantized linear through the C ABI (tcgen05 GEMM), writing `out`."""
    import qlinear

    return qlinear.quantized_matmul(x, lin.wq, lin.scales, lin.biases, True, lin.group_size, lin.bits,
                                    bias=lin.bias, act=lin.act, kernel=qlinear.KERNEL_GEMM, out=out,
                                    max_ctas=max_ctas)


class TPLinear:
    """One packed linear, sharded for `rank` of `world` ("col": output rows; "row": K)."""

    def __init__(self, wq, scales, biases, bias, group_size: int, bits: int, style: str, rank: int, world: int,
                 act: Optional[str] = None):
        if style not in ("col", "row"):
            raise ValueError(f"style must be 'col' or 'row', not {style!r}")
        self.group_size, self.bits, self.style, self.act = group_size, bits, style, act
        self.K_full = scales.shape[1] * group_size
        self.N_full = scales.shape[0]
        self.k0, self.k1 = 0, self.K_full
        if world > 1 and style == "col":
            wq, scales, biases, bias = column_shard(wq, scales, biases, bias, rank, world)
        elif world > 1 and style == "row":
            wq, scales, biases, self.k0, self.k1 = row_shard(wq, scales, biases, group_size, bits, rank, world)
            if rank != 0:
                bias = None  # added once: the reduction sums rank 0's biased partial
        self.wq, self.scales, self.biases, self.bias = wq, scales, biases, bias
        self.N = scales.shape[0]
        self.K = self.k1 - self.k0


class TPBlock:
    """A chain of quantized linears (one DiT block), Megatron-sharded over `comm`'s ranks.

    spec: ``[(name, act, style, src), ...]`` in execution order; `src` is ``"x"`` (the block
    input), the name of an external input passed to ``forward`` (full width; a row-parallel
    linear reads its K slice) or the name of an earlier linear.  weights: ``name ->
    (wq, scales, biases, bias)`` unsharded (identical on every rank).  comm: a ``Comm`` or
    None (one process, unsharded).  The GEMMs leave `comm_sms` SMs to the collectives (0:
    the GEMMs take every SM and NCCL's kernels share them -- measured fastest on the FLUX
    and Wan blocks at 4 and 8 GPUs).
    `matmul(x, lin, out, max_ctas)` runs one linear (default: the C ABI's GEMM; tests
    substitute a CPU implementation)."""

    def __init__(self, spec: Sequence[Tuple[str, Optional[str], str, str]], weights: Dict[str, tuple],
                 group_size: int, bits: int, M: int, comm: Optional[Comm] = None, chunks: int = 2,
                 mode: str = "allreduce", comm_sms: int = 0, dtype=torch.bfloat16,
                 device: Optional[torch.device] = None,
                 matmul: Callable = default_matmul):
        if mode not in ("allreduce", "seqpar"):
            raise ValueError(f"mode must be 'allreduce' or 'seqpar', not {mode!r}")
        self.spec = list(spec)
        self.comm = comm
        self.world = comm.world if comm is not None else 1
        self.rank = comm.rank if comm is not None else 0
        self.M, self.mode, self.matmul = M, mode, matmul
        self.dev = device if device is not None else weights[self.spec[0][0]][0].device
        self.cuda = self.dev.type == "cuda"
        W = self.world
        self.lin = {name: TPLinear(*weights[name], group_size, bits, style, self.rank, W, act=act)
                    for name, act, style, _ in self.spec}
        self.src = {name: src for name, _, _, src in self.spec}
        self.row = W > 1
        self.reduced = {n for n, l in self.lin.items() if self.row and l.style == "row"}
        consumers = set(self.src.values())
        self.bounds = slice_bounds(M, chunks, W) if self.row else [(0, M)]
        self.out = {n: torch.empty(M, l.N, device=self.dev, dtype=dtype) for n, l in self.lin.items()}
        self.shard, self.full = {}, {}
        for n in self.reduced:
            if mode == "seqpar":
                self.shard[n] = torch.empty(M // W, self.lin[n].N, device=self.dev, dtype=dtype)
                if n in consumers:
                    self.full[n] = torch.empty(M, self.lin[n].N, device=self.dev, dtype=dtype)
        self.max_ctas = 0
        if self.row and self.cuda:
            self.max_ctas = torch.cuda.get_device_properties(self.dev).multi_processor_count - comm_sms
        self.main = torch.cuda.current_stream(self.dev) if self.cuda else None
        self.comm_stream = torch.cuda.Stream(self.dev) if (self.row and self.cuda) else None
        self._ext_cache: Dict[Tuple[str, int], torch.Tensor] = {}
        self.flops = sum(2.0 * M * l.N_full * l.K_full for l in self.lin.values())
        self.launches = sum(1 if (not self.row or (l.style == "col" and self.src[n] not in self.reduced))
                            else len(self.bounds) for n, l in self.lin.items())

    def _external(self, name: str, t: torch.Tensor, lin: TPLinear) -> torch.Tensor:
        """A full-width external input narrowed to lin's K slice (cached per tensor)."""
        if lin.k0 == 0 and lin.k1 == t.shape[1]:
            return t
        key = (name, t.data_ptr())
        if key not in self._ext_cache:
            self._ext_cache[key] = t[:, lin.k0:lin.k1].contiguous()
        return self._ext_cache[key]

    def result_rows(self) -> Tuple[torch.Tensor, int]:
        """(tensor, rows) holding this rank's part of the block output: the full output in
        "allreduce" mode; in "seqpar" mode M/W rows, slice by slice: for every slice
        ``(r0, r1)`` of ``self.bounds`` (k = (r1 - r0) / W rows per rank), rows
        ``r0 + rank*k .. r0 + (rank+1)*k`` of the output (see ``own_rows``)."""
        last = self.spec[-1][0]
        return (self.shard[last], self.M // self.world) if last in self.shard else (self.out[last], self.M)

    def forward(self, x: torch.Tensor, inputs: Optional[Dict[str, torch.Tensor]] = None, evs=None,
                cevs=None, ev_names=None) -> torch.Tensor:
        """Runs the block on this rank; returns ``result_rows()[0]``.  `evs` / `cevs`, if
        lists, receive ``(name, start_event, end_event)`` for every GEMM launch (main
        stream; only the linears in `ev_names` when given) / every slice's collectives
        (communication stream)."""
        inputs = inputs or {}
        W = self.world
        if self.cuda:
            self.main = torch.cuda.current_stream(self.dev)  # the caller's stream (a capture stream too)
        ready = {}  # name -> per-slice events: rows r0:r1 of the (reduced) output are usable
        for name, _, _, src in self.spec:
            l = self.lin[name]
            y = self.out[name]
            from_red = src in self.reduced
            if src == "x":
                inp = x
            elif src in self.lin:
                inp = self.full[src] if src in self.full else self.out[src]
            else:
                inp = self._external(src, inputs[src], l)
            sliced = self.row and (l.style == "row" or from_red)
            for c, (r0, r1) in enumerate(self.bounds if sliced else [(0, self.M)]):
                if from_red and self.cuda:
                    self.main.wait_event(ready[src][c])  # rows r0:r1 of the input are reduced
                rec = evs is not None and self.cuda and (ev_names is None or name in ev_names)
                if rec:
                    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    e0.record()
                self.matmul(inp[r0:r1], l, y[r0:r1], self.max_ctas)
                if rec:
                    e1.record()
                    evs.append((name, e0, e1))
                if name in self.reduced:
                    ready.setdefault(name, []).append(self._reduce(name, y, r0, r1, cevs))
        if self.comm_stream is not None:
            self.main.wait_stream(self.comm_stream)  # the block output's last slice is reduced
        return self.result_rows()[0]

    def capture(self, x: torch.Tensor, inputs: Optional[Dict[str, torch.Tensor]] = None) -> "BlockGraph":
        """``forward(x, inputs)`` captured into a CUDA graph: the GEMM launches, the
        collectives (NCCL records them into the graph) and the stream joins between them.
        A replay issues the whole block with one host call, so a short sharded step is not
        bound by the host issuing dozens of launches.  x and the inputs are bound at capture:
        fill those tensors, then replay.  Every rank must capture (and replay) the same
        block in the same order, as with the eager forward.  The graph holds NCCL work of
        the communicator: ``reset()`` every BlockGraph before ``Comm.close()``, whose
        teardown otherwise waits on it."""
        if not self.cuda:
            raise ValueError("capture needs CUDA tensors")
        side = torch.cuda.Stream(self.dev)
        side.wait_stream(torch.cuda.current_stream(self.dev))
        with torch.cuda.stream(side):
            self.forward(x, inputs)  # warm-up on the capture's stream (communicators, caches)
        torch.cuda.current_stream(self.dev).wait_stream(side)
        torch.cuda.synchronize(self.dev)
        pending = len(self.comm._pending) if self.comm is not None else 0
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=side):
            out = self.forward(x, inputs)
        if self.comm is not None:
            del self.comm._pending[pending:]  # capture-time handles: the replays carry no host work
        self.main = torch.cuda.current_stream(self.dev)
        return BlockGraph(g, out)

    def _reduce(self, name, y, r0, r1, cevs=None):
        W = self.world
        ev = None
        if self.cuda:
            self.comm_stream.wait_stream(self.main)
            ctx = torch.cuda.stream(self.comm_stream)
        else:
            import contextlib
            ctx = contextlib.nullcontext()
        with ctx:
            if cevs is not None and self.cuda:
                c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                c0.record(self.comm_stream)
            if self.mode == "seqpar":
                part = self.shard[name][r0 // W:r1 // W]
                self.comm.reduce_scatter(part, y[r0:r1])
                if name in self.full:
                    self.comm.all_gather(self.full[name][r0:r1], part)
            else:
                self.comm.all_reduce(y[r0:r1])
            if cevs is not None and self.cuda:
                c1.record(self.comm_stream)
                cevs.append((name, c0, c1))
            if self.cuda:
                ev = torch.cuda.Event()
                ev.record(self.comm_stream)
        if not self.cuda:
            self.comm.wait()
        return ev

    def own_rows(self) -> torch.Tensor:
        """Output row indices held by this rank in "seqpar" mode (``result_rows`` order)."""
        W, idx = self.world, []
        for r0, r1 in self.bounds:
            k = (r1 - r0) // W
            idx.append(torch.arange(r0 + self.rank * k, r0 + (self.rank + 1) * k))
        return torch.cat(idx)

    def gather_output(self) -> torch.Tensor:
        """The whole block output ``[M, N]`` on every rank (all-gathers the seqpar shards
        slice by slice)."""
        t, rows = self.result_rows()
        if rows == self.M:
            return t
        W = self.world
        full = torch.empty(self.M, t.shape[1], dtype=t.dtype, device=t.device)
        for r0, r1 in self.bounds:
            self.comm.all_gather(full[r0:r1], t[r0 // W:r1 // W].contiguous())
        self.comm.wait()
        return full


class BlockGraph:
    """A ``TPBlock.forward`` captured by ``TPBlock.capture``: ``replay()`` runs it on the
    current stream and returns the block's output tensor (the same tensor every time)."""

    def __init__(self, graph, out: torch.Tensor):
        self.graph, self.out = graph, out

    def replay(self) -> torch.Tensor:
        self.graph.replay()
        return self.out

    def reset(self) -> None:
        """Synchronises and frees the graph (call before closing the communicator)."""
        if self.graph is not None:
            torch.cuda.synchronize(self.out.device)
            self.graph.reset()
            self.graph = None


def reference_forward(spec, weights, group_size: int, bits: int, x: torch.Tensor,
                      inputs: Optional[Dict[str, torch.Tensor]] = None, matmul: Callable = default_matmul,
                      outputs: Sequence[str] = ()) -> Dict[str, torch.Tensor]:
    """The same chain unsharded, one linear per call (the reference's single-device
    forward, src/adapters.rs:300-322).  Returns the last linear's output under "out" plus
    the linears named in `outputs`."""
    inputs = inputs or {}
    res: Dict[str, torch.Tensor] = {}
    for name, act, style, src in spec:
        lin = TPLinear(*weights[name], group_size, bits, style, 0, 1, act=act)
        inp = x if src == "x" else (res[src] if src in res else inputs[src])
        y = torch.empty(inp.shape[0], lin.N, dtype=x.dtype, device=x.device)
        matmul(inp, lin, y, 0)
        res[name] = y
    out = {n: res[n] for n in outputs}
    out["out"] = res[spec[-1][0]]
    return out


# Tolerance of the tensor-parallel block against the unsharded one.  Both use the same
# kernels and fp32 accumulation; what differs is where bf16 rounding happens: each rank's
# partial sum is rounded to bf16 before the collective adds the partials (in the
# collective's order), where the unsharded GEMM rounds the full sum once.  That adds up to
# about (world + 1) / 2 bf16 half-ulps per row-parallel output, and the chain carries it
# through the later linears.  Element-wise bound: 4 * world ulp_bf16(|ref|) plus 1/128
# of the output scale; relative L2 <= 1e-2 (the single-GPU matmul tolerance is 2 ulp +
# 2e-3 of the scale and 4e-3 relative L2).
def parity(got: torch.Tensor, ref: torch.Tensor, world: int) -> dict:
    g, r = got.double(), ref.double()
    err = (g - r).abs()
    scale = float(r.abs().max()) if r.numel() else 0.0
    ulp = torch.exp2(torch.floor(torch.log2(r.abs().clamp_min(1e-30))) - 7)
    bound = 4 * max(world, 1) * ulp + scale / 128
    denom = float(torch.linalg.vector_norm(r))
    rel = float(torch.linalg.vector_norm(g - r)) / denom if denom > 0 else 0.0
    bad = int((err > bound).sum())
    ok = bad == 0 and rel <= 1e-2 and bool(torch.isfinite(g).all())
    return {"max_abs": float(err.max()) if err.numel() else 0.0, "rel_l2": rel, "scale": scale,
            "out_of_bound": bad, "bitwise_equal": bool(torch.equal(got, ref)), "ok": ok,
            "tolerance": "|d| <= 4*world ulp_bf16(|ref|) + max|ref|/128 element-wise, rel L2 <= 1e-2"}
