"""GPU parity under adversarial activations: every GEMV kernel (tcgen05 e4m3-piece GEMV,
TMA-fed and register-fed mma.sync GEMVs, the automatic choice) and the GEMM against the
oracle, within the stated tolerance (tests/helpers.py).

The tcgen05 GEMV splits each bf16 activation into two e4m3 pieces under one power-of-two
scale per (token, group); these cases put that split under stress with the value ranges
real DiT / LLM activations carry: one large outlier per group (massive-activation
channels), groups mixing 1e-3 and 1e2, all-zero groups and tokens, the smallest normal
and the subnormal bf16 range, and very large magnitudes.  The reference feeds bf16 x
exactly into an fp32-accumulating quantized_matmul (src/adapters.rs:301-317)."""
import numpy as np
import pytest
import torch

import oracle as O
import qlinear
from helpers import assert_bf16_close, np2t, rand_bf16, t2np

pytestmark = pytest.mark.gpu
GEMV, GEMV_TC, GEMV_TMA, GEMV_REGS, GEMM = (qlinear.KERNEL_GEMV, qlinear.KERNEL_GEMV_TC, qlinear.KERNEL_GEMV_TMA,
                                            qlinear.KERNEL_GEMV_REGS, qlinear.KERNEL_GEMM)


def adversarial_x(kind, M, K, gs, rng):
    x = rng.standard_normal((M, K)).astype(np.float32)
    G = K // gs
    if kind == "outlier":        # one element of +-2^10 per group, the rest ~N(0, 1)
        pos = rng.integers(0, gs, size=(M, G))
        sign = np.where(rng.random((M, G)) < 0.5, -1.0, 1.0)
        for m in range(M):
            x[m, np.arange(G) * gs + pos[m]] = sign[m] * 1024.0
    elif kind == "outlier_2e13":  # beyond the two-piece split's exact range
        pos = rng.integers(0, gs, size=(M, G))
        for m in range(M):
            x[m, np.arange(G) * gs + pos[m]] = 8192.0
    elif kind == "mixed":        # 1e-3 and 1e2 magnitudes interleaved inside every group
        x *= np.where(np.arange(K) % 2 == 0, 1e-3, 1e2).astype(np.float32)
    elif kind == "zero_groups":  # every third group all zero, and the last token all zero
        for g in range(0, G, 3):
            x[:, g * gs:(g + 1) * gs] = 0
        x[-1] = 0
    elif kind == "tiny":         # around the smallest normal bf16 (2^-126)
        x *= 2.0 ** -122
    elif kind == "subnormal":    # bf16 subnormals only
        x = (rng.integers(1, 128, size=(M, K)) * np.where(rng.random((M, K)) < 0.5, -1, 1)).astype(np.float32)
        x *= 2.0 ** -133
    elif kind == "huge":         # large magnitudes (2^100), far from overflow of the sums
        x *= 2.0 ** 100
    elif kind == "channel":      # a few massive channels shared by every token (LLM style)
        ch = rng.choice(K, size=max(1, K // 256), replace=False)
        x[:, ch] *= 300.0
    return O.to_bf16(x)


KINDS = ["outlier", "outlier_2e13", "mixed", "zero_groups", "tiny", "subnormal", "huge", "channel"]


def _case(dev, kind, M, N, K, gs, bits, seed):
    rng = np.random.default_rng(seed)
    w = rand_bf16((N, K), 0.02, rng)
    x = adversarial_x(kind, M, K, gs, rng)
    wq, s, b = O.quantize(w, gs, bits)
    return x, wq, s, b, np2t(x, dev), np2t(wq, dev), np2t(s, dev), np2t(b, dev)


@pytest.mark.parametrize("kind", KINDS)
@pytest.mark.parametrize("kernel", [GEMV_TC, GEMV, GEMV_TMA, GEMV_REGS])
@pytest.mark.parametrize("M", [1, 4, 8])
@pytest.mark.parametrize("bits", [4, 8])
def test_gemv_adversarial_activations(dev, kind, kernel, M, bits):
    N, K, gs = 256, 1024, 64
    x, wq, s, b, xt, wqt, st, bt = _case(dev, kind, M, N, K, gs, bits, 31 * M + bits + KINDS.index(kind))
    y = qlinear.quantized_matmul(xt, wqt, st, bt, True, gs, bits, kernel=kernel)
    torch.cuda.synchronize()
    assert qlinear.device_error() == 0
    ref = O.to_f32(O.quantized_matmul(x, wq, s, b, gs, bits))
    got = O.to_f32(t2np(y))
    assert np.isfinite(got).all()
    # Subnormal activations give outputs of a few bf16 subnormal steps (2^-133 apart), where
    # an fp32 accumulation of subnormal products (the reference's, and the kernels') keeps
    # only ~10 bits per product: the element-wise bound stands, the relative-L2 bound is
    # loosened to 1e-2.
    assert_bf16_close(got, ref, rl2=1e-2 if kind == "subnormal" else 4e-3, what=f"{kind} kernel={kernel} M={M} Q{bits}")


@pytest.mark.parametrize("kind", ["outlier", "mixed", "tiny", "channel"])
def test_gemm_adversarial_activations(dev, kind):
    M, N, K, gs, bits = 300, 256, 1024, 64, 8
    x, wq, s, b, xt, wqt, st, bt = _case(dev, kind, M, N, K, gs, bits, 5 + KINDS.index(kind))
    y = qlinear.quantized_matmul(xt, wqt, st, bt, True, gs, bits, kernel=GEMM)
    torch.cuda.synchronize()
    assert qlinear.device_error() == 0
    assert_bf16_close(O.to_f32(t2np(y)), O.to_f32(O.quantized_matmul(x, wq, s, b, gs, bits)), what=f"gemm {kind}")


@pytest.mark.parametrize("kind", ["normal", "outlier", "channel"])
@pytest.mark.parametrize("M", [1, 8])
def test_lm_head_gemv_adversarial(dev, kind, M):
    """The Llama-3.2-3B lm_head shape (N=128256, K=3072, Q4 g64) through the automatic choice
    (the tcgen05 GEMV at this width), every output checked against the oracle."""
    N, K, gs, bits = 128256, 3072, 64, 4
    rng = np.random.default_rng(77 + M)
    g = torch.Generator(device=dev).manual_seed(9)
    w = (torch.randn(N, K, device=dev, generator=g) * 0.02).to(torch.bfloat16)
    wqt, st, bt = qlinear.quantize(w, gs, bits)
    x = adversarial_x(kind if kind != "normal" else "none", M, K, gs, rng)
    y = qlinear.quantized_matmul(np2t(x, dev), wqt, st, bt, True, gs, bits)
    torch.cuda.synchronize()
    assert qlinear.device_error() == 0
    ref = O.quantized_matmul_fast(x, t2np(wqt), t2np(st), t2np(bt), gs, bits)
    assert_bf16_close(O.to_f32(t2np(y)), O.to_f32(ref), what=f"lm_head {kind} M={M}")


def test_full_size_gemm_every_row_against_oracle(dev):
    """configs[0] at full size (M=4096, 3072x3072 Q4 g64): every output row of the tcgen05
    GEMM against the oracle's multithreaded mode (fp32 accumulation)."""
    M, N, K, gs, bits = 4096, 3072, 3072, 64, 4
    g = torch.Generator(device=dev).manual_seed(0)
    w = (torch.randn(N, K, device=dev, generator=g) * 0.02).to(torch.bfloat16)
    x = torch.randn(M, K, device=dev, generator=g).to(torch.bfloat16)
    wq, s, b = qlinear.quantize(w, gs, bits)
    y = qlinear.quantized_matmul(x, wq, s, b, True, gs, bits, kernel=GEMM)
    torch.cuda.synchronize()
    assert qlinear.device_error() == 0
    ref = O.quantized_matmul_fast(t2np(x), t2np(wq), t2np(s), t2np(b), gs, bits)
    assert_bf16_close(O.to_f32(t2np(y)), O.to_f32(ref), what="cfg1 every row")
