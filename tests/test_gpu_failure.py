"""GPU: the failure path of the bounded waits, without a GPU fault.

Every pipelined kernel bounds its mbarrier waits (%globaltimer); when one runs out the
kernel records a timeout code in the device error word, all roles drain, TMEM is freed
and the kernel returns, leaving the context usable.  Here the test hook makes the tcgen05
GEMM's TMA producer issue nothing (a flag nothing in production sets) with the wait limit
shortened to 50 ms: the launch must end by itself, ql_device_error must report a timeout,
and the next, normal call must run correctly on the same context.  The reference's
failure model is the cooperative cancel flag (gen-core/src/runtime.rs:239-258)."""
import time

import numpy as np
import pytest
import torch

import oracle as O
import qlinear
from helpers import assert_bf16_close, np2t, rand_bf16, t2np
from qlinear import _lib

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("kernel", [qlinear.KERNEL_GEMM, qlinear.KERNEL_GEMM_PAIR])
def test_gemm_wait_runs_out_and_reports(dev, kernel):
    rng = np.random.default_rng(3)
    M, N, K, gs, bits = 300, 256, 512, 64, 4
    w = rand_bf16((N, K), 0.02, rng)
    x = rand_bf16((M, K), 1.0, rng)
    wq, s, b = O.quantize(w, gs, bits)
    xt, wqt, st, bt = np2t(x, dev), np2t(wq, dev), np2t(s, dev), np2t(b, dev)
    assert qlinear.device_error() == 0
    try:
        _lib.debug_inject(_lib.INJECT_GEMM_PRODUCER_SILENT, 50_000_000)
        t0 = time.monotonic()
        qlinear.quantized_matmul(xt, wqt, st, bt, True, gs, bits, kernel=kernel)
        err = qlinear.device_error()  # synchronises
        dt = time.monotonic() - t0
    finally:
        _lib.debug_inject(0, 0)
    assert err & (_lib.DEV_ERR_TIMEOUT_FULL | _lib.DEV_ERR_TIMEOUT_EMPTY | _lib.DEV_ERR_TIMEOUT_ACC), err
    assert dt < 10.0, f"the aborted launch took {dt:.1f} s"
    assert qlinear.device_error() == 0  # cleared by the read above
    # the context is intact: the same call now runs normally
    y = qlinear.quantized_matmul(xt, wqt, st, bt, True, gs, bits, kernel=kernel)
    torch.cuda.synchronize()
    assert qlinear.device_error() == 0
    assert_bf16_close(O.to_f32(t2np(y)), O.to_f32(O.quantized_matmul(x, wq, s, b, gs, bits)), what="after abort")


def test_wait_limit_restored(dev):
    """The hook's defaults: a short limit does not fire on healthy launches."""
    rng = np.random.default_rng(4)
    M, N, K, gs, bits = 512, 512, 1024, 64, 8
    w = rand_bf16((N, K), 0.02, rng)
    x = rand_bf16((M, K), 1.0, rng)
    wq, s, b = O.quantize(w, gs, bits)
    try:
        _lib.debug_inject(0, 50_000_000)
        y = qlinear.quantized_matmul(np2t(x, dev), np2t(wq, dev), np2t(s, dev), np2t(b, dev), True, gs, bits)
        torch.cuda.synchronize()
        assert qlinear.device_error() == 0
    finally:
        _lib.debug_inject(0, 0)
    assert_bf16_close(O.to_f32(t2np(y)), O.to_f32(O.quantized_matmul(x, wq, s, b, gs, bits)), what="short limit")
