"""GPU: ql_quantized_matmul_noalloc, the entry point for callers that cannot allocate
device memory (allocator hooks, real-time loops, runtimes whose memory is all reserved).

It must give the same result as ql_quantized_matmul with a caller-allocated workspace,
on two calls in a row (the shared fixed scratch keeps the previous call's contents),
and refuse a LoRA workspace larger than its fixed 8 MiB array.  This file is collected
last on purpose; it passes alone in a fresh process as well as after the other tests."""
import ctypes as C

import numpy as np
import pytest
import torch

import oracle as O
import qlinear
from helpers import assert_bf16_close, np2t, rand_bf16, t2np
from qlinear import _lib

pytestmark = pytest.mark.gpu


def _call(fn, x, wq, s, b, N, K, gs, bits, A, B, scale, bias, kernel, ws=None):
    M = x.shape[0]
    y = torch.empty(M, N, device=x.device, dtype=torch.bfloat16)
    ep = _lib.Epilogue()
    ep.bias = bias.data_ptr()
    ep.lora_a, ep.lora_b, ep.lora_rank, ep.lora_scale = A.data_ptr(), B.data_ptr(), A.shape[1], scale
    ep.kernel = kernel
    if ws is not None:
        ep.workspace, ep.workspace_bytes = ws.data_ptr(), ws.numel()
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = fn(C.c_void_p(x.data_ptr()), _lib.QL_BF16, M, K, C.c_void_p(wq.data_ptr()), C.c_void_p(s.data_ptr()),
            C.c_void_p(b.data_ptr()), _lib.QL_BF16, N, gs, bits, 1, C.byref(ep), C.c_void_p(y.data_ptr()),
            _lib.QL_BF16, stream)
    return rc, y


@pytest.mark.parametrize("kernel,M", [(qlinear.KERNEL_GEMM, 270), (qlinear.KERNEL_GEMV, 6)])
def test_noalloc_matches_workspace_entry_point(kernel, M):
    dev = torch.device("cuda:0")
    L = _lib.lib()
    N, K, gs, bits, rank = 256, 384, 64, 4, 32
    for call in range(2):  # two calls in a row, different inputs
        rng = np.random.default_rng(1000 * call + M)
        w = rand_bf16((N, K), 0.02, rng)
        wq, s, b = (np2t(a, dev) for a in O.quantize(w, gs, bits))
        x = np2t(rand_bf16((M, K), 1.0, rng), dev)
        A = np2t(rand_bf16((K, rank), 1.0 / np.sqrt(rank), rng), dev)
        B = np2t(rand_bf16((rank, N), 0.01, rng), dev)
        bias = np2t(rand_bf16((N,), 0.1, rng), dev)
        ws = torch.empty(qlinear.workspace_size(M, N, K, rank), dtype=torch.uint8, device=dev)
        rc0, y0 = _call(L.ql_quantized_matmul, x, wq, s, b, N, K, gs, bits, A, B, 0.5, bias, kernel, ws)
        rc1, y1 = _call(L.ql_quantized_matmul_noalloc, x, wq, s, b, N, K, gs, bits, A, B, 0.5, bias, kernel)
        torch.cuda.synchronize()
        assert rc0 == 0 and rc1 == 0, L.ql_last_error()
        assert_bf16_close(O.to_f32(t2np(y1)), O.to_f32(t2np(y0)), what=f"noalloc call {call}")
    assert qlinear.device_error() == 0


def test_noalloc_rejects_oversized_workspace():
    dev = torch.device("cuda:0")
    L = _lib.lib()
    M, N, K, rank = 70000, 128, 128, 64  # 70000 * 64 * 2 bytes > 8 MiB
    x = torch.zeros(M, K, device=dev, dtype=torch.bfloat16)
    wq = torch.zeros(N, K // 8, device=dev, dtype=torch.int32)
    s = torch.zeros(N, K // 64, device=dev, dtype=torch.bfloat16)
    A = torch.zeros(K, rank, device=dev, dtype=torch.bfloat16)
    B = torch.zeros(rank, N, device=dev, dtype=torch.bfloat16)
    rc, _ = _call(L.ql_quantized_matmul_noalloc, x, wq, s, s, N, K, 64, 4, A, B, 1.0, s[:, 0].contiguous(),
                  qlinear.KERNEL_GEMM)
    assert rc == _lib.QL_EUNSUPPORTED
    assert b"exceeds" in L.ql_last_error()
