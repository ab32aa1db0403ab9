"""GPU parity: quantized_matmul (GEMV, tcgen05 GEMM, generic) and its fused epilogues
against the oracle, within the stated bf16 tolerance (tests/helpers.py
assert_bf16_close: 2 bf16 ulps + 2e-3 of the output scale element-wise, relative L2
<= 4e-3; activation epilogues, which the reference rounds op by op in bf16, get 4 ulps)."""
import numpy as np
import pytest
import torch

import oracle as O
import qlinear
from helpers import assert_bf16_close, np2t, rand_bf16, t2np

pytestmark = pytest.mark.gpu
GEMV, GEMM, GENERIC = qlinear.KERNEL_GEMV, qlinear.KERNEL_GEMM, qlinear.KERNEL_GENERIC
GEMV_TC = qlinear.KERNEL_GEMV_TC
GEMV_TMA, GEMV_REGS = qlinear.KERNEL_GEMV_TMA, qlinear.KERNEL_GEMV_REGS
GEMM2 = qlinear.KERNEL_GEMM_PAIR


def make_case(dev, M, N, K, gs, bits, seed, wstd=0.02):
    rng = np.random.default_rng(seed)
    w = rand_bf16((N, K), wstd, rng)
    x = rand_bf16((M, K), 1.0, rng)
    wq, s, b = O.quantize(w, gs, bits)
    return rng, x, wq, s, b, np2t(x, dev), np2t(wq, dev), np2t(s, dev), np2t(b, dev)


@pytest.mark.parametrize("bits", [8, 4])
def test_fixture_qmm_f32(golden, dev, bits):
    """f32 activations and scales (generic kernel) vs the MLX golden qmm
    (reference gate allclose 1e-2/1e-2, tests/quant_parity.rs:59-64)."""
    p = f"q{bits}_"
    y = qlinear.quantized_matmul(np2t(golden["x"], dev), np2t(golden[p + "wq"], dev),
                                 np2t(golden[p + "scales"], dev), np2t(golden[p + "biases"], dev), True, 64, bits)
    np.testing.assert_allclose(t2np(y), golden[p + "qmm"], rtol=1e-4, atol=1e-3)


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("gs", [32, 64, 128])
@pytest.mark.parametrize("M", [1, 2, 3, 8])
@pytest.mark.parametrize("K", [384, 1024, 2560])
@pytest.mark.parametrize("kernel", [GEMV, GEMV_TMA, GEMV_REGS])
def test_gemv_parity(dev, bits, gs, M, K, kernel):
    """The automatic GEMV choice and each mma.sync GEMV pinned: the register-fed one (any
    K) and the TMA-fed one (K a multiple of 8 groups; 2560 has a partial last stage)."""
    if kernel == GEMV_TMA and (K // gs) % 8:
        pytest.skip("the TMA GEMV needs K to be a whole number of 8-group batches")
    N = 200
    _, x, wq, s, b, xt, wqt, st, bt = make_case(dev, M, N, K, gs, bits, 100 * M + gs + bits)
    y = qlinear.quantized_matmul(xt, wqt, st, bt, True, gs, bits, kernel=kernel)
    assert_bf16_close(O.to_f32(t2np(y)), O.to_f32(O.quantized_matmul(x, wq, s, b, gs, bits)), what="gemv")


@pytest.mark.parametrize("kernel", [GEMM, GEMM2])
@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("gs", [32, 64, 128])
@pytest.mark.parametrize("M,N,K", [(9, 128, 64), (256, 128, 256), (300, 200, 448), (513, 384, 128), (40, 136, 96)])
def test_gemm_parity(dev, bits, gs, M, N, K, kernel):
    if K % gs:
        pytest.skip("K must be a multiple of the group size")
    _, x, wq, s, b, xt, wqt, st, bt = make_case(dev, M, N, K, gs, bits, M + N + K + gs + bits)
    y = qlinear.quantized_matmul(xt, wqt, st, bt, True, gs, bits, kernel=kernel)
    torch.cuda.synchronize()
    assert qlinear.device_error() == 0
    assert_bf16_close(O.to_f32(t2np(y)), O.to_f32(O.quantized_matmul(x, wq, s, b, gs, bits)), what="gemm")


@pytest.mark.parametrize("kernel", [GEMV, GEMM, GEMM2, GENERIC])
@pytest.mark.parametrize("act", [None, "gelu_tanh", "gelu"])
def test_bias_act_epilogue(dev, kernel, act):
    M = 4 if kernel == GEMV else 260
    N, K, gs, bits = 192, 256, 64, 8
    rng, x, wq, s, b, xt, wqt, st, bt = make_case(dev, M, N, K, gs, bits, 5)
    bias = rand_bf16((N,), 0.5, rng)
    y = qlinear.quantized_matmul(xt, wqt, st, bt, True, gs, bits, bias=np2t(bias, dev), act=act, kernel=kernel)
    code = {None: O.ACT_NONE, "gelu_tanh": O.ACT_GELU_TANH, "gelu": O.ACT_GELU_ERF}[act]
    ref = O.quantized_matmul(x, wq, s, b, gs, bits, bias=bias, act=code)
    assert_bf16_close(O.to_f32(t2np(y)), O.to_f32(ref), ulps=4 if act else 2, what=f"bias+{act}")


@pytest.mark.parametrize("kernel", [GEMV, GEMM, GEMM2, GENERIC])
@pytest.mark.parametrize("bits", [4, 8])
def test_swiglu_epilogue(dev, kernel, bits):
    M = 5 if kernel == GEMV else 300
    N, K, gs = 160, 320, 64
    rng, x, wq, s, b, xt, wqt, st, bt = make_case(dev, M, N, K, gs, bits, 9)
    w3 = rand_bf16((N, K), 0.02, rng)
    wq3, s3, b3 = O.quantize(w3, gs, bits)
    y = qlinear.quantized_matmul(xt, wqt, st, bt, True, gs, bits, act="swiglu",
                                 up=(np2t(wq3, dev), np2t(s3, dev), np2t(b3, dev)), kernel=kernel)
    h1 = O.quantized_matmul(x, wq, s, b, gs, bits)
    h3 = O.quantized_matmul(x, wq3, s3, b3, gs, bits)
    assert_bf16_close(O.to_f32(t2np(y)), O.to_f32(O.swiglu(h1, h3)), ulps=4, what="swiglu")


@pytest.mark.parametrize("kernel", [GEMV, GEMM, GEMM2, GENERIC])
@pytest.mark.parametrize("rank", [8, 12, 32, 96])
def test_lora_epilogue(dev, kernel, rank):
    """LoRA residual scale*(x.A).B fused into the accumulator (src/adapters.rs:260-270).  The
    reference rounds the base output and the residual to bf16 separately before summing them;
    where the two cancel, that leaves up to one bf16 ulp of the operands' magnitude, so the
    stated bound is 4 ulps of the result plus 1/128 of the output scale."""
    M = 7 if kernel == GEMV else 270
    N, K, gs, bits = 256, 384, 64, 4
    rng, x, wq, s, b, xt, wqt, st, bt = make_case(dev, M, N, K, gs, bits, rank)
    A = rand_bf16((K, rank), 1.0 / np.sqrt(rank), rng)
    B = rand_bf16((rank, N), 0.01, rng)
    bias = rand_bf16((N,), 0.1, rng)
    y = qlinear.quantized_matmul(xt, wqt, st, bt, True, gs, bits, bias=np2t(bias, dev),
                                 lora=(np2t(A, dev), np2t(B, dev), 0.75), kernel=kernel)
    ref = O.quantized_matmul(x, wq, s, b, gs, bits, bias=bias, lora_a=A, lora_b=B, lora_scale=0.75)
    assert_bf16_close(O.to_f32(t2np(y)), O.to_f32(ref), ulps=4, atol_frac=2 ** -7, what=f"lora r{rank}")


@pytest.mark.parametrize("M,K,rank", [(9600, 192, 8), (9600, 448, 40), (300, 192, 12), (300, 448, 12),
                                       (300, 448, 40), (2304, 3840, 32)])
def test_lora_prepass_splits(dev, M, K, rank):
    """The LoRA pre-pass T = s.(x.A) in each of its forms: one CTA per row tile (many tiles,
    or K under four chunks) and a 2-CTA cluster splitting the chunks with a DSMEM reduction
    (odd chunk counts split unevenly), TMA-fed (rank % 8 == 0) and cp.async-fed, 32 or 64
    columns computed; checked through the GEMM's output against the oracle."""
    N, gs, bits = 256, 64, 4
    rng, x, wq, s, b, xt, wqt, st, bt = make_case(dev, M, N, K, gs, bits, 1000 + rank + K)
    A = rand_bf16((K, rank), 1.0 / np.sqrt(rank), rng)
    B = rand_bf16((rank, N), 0.01, rng)
    y = qlinear.quantized_matmul(xt, wqt, st, bt, True, gs, bits, lora=(np2t(A, dev), np2t(B, dev), 0.5),
                                 kernel=GEMM)
    torch.cuda.synchronize()
    assert qlinear.device_error() == 0
    ref = O.quantized_matmul(x, wq, s, b, gs, bits, lora_a=A, lora_b=B, lora_scale=0.5)
    assert_bf16_close(O.to_f32(t2np(y)), O.to_f32(ref), ulps=4, atol_frac=2 ** -7, what=f"lora M{M} K{K} r{rank}")


def test_kernels_agree_with_each_other(dev):
    """GEMM, GEMV (M<=8 slices) and the generic kernel on the same operands."""
    M, N, K, gs, bits = 8, 512, 1024, 64, 4
    _, x, wq, s, b, xt, wqt, st, bt = make_case(dev, M, N, K, gs, bits, 3)
    ys = [t2np(qlinear.quantized_matmul(xt, wqt, st, bt, True, gs, bits, kernel=k)) for k in (GEMV, GEMM, GENERIC)]
    for y in ys[1:]:
        assert_bf16_close(O.to_f32(y), O.to_f32(ys[0]), what="cross-kernel")


@pytest.mark.parametrize("bits,N,K,act", [(8, 12288, 3072, "gelu_tanh"), (4, 3072, 3072, None),
                                          (4, 5120, 13824, None)])
def test_full_size_gemm_properties(dev, bits, N, K, act):
    """BASELINE shapes at full size (FLUX MLP-up Q8, cfg1 Q4, Wan FFN-down Q4), M=4608:
    (1) rows sampled across the whole output match the oracle; (2) the GEMM equals
    dequantize -> fp32 matmul (a size-independent identity)."""
    M, gs = 4608, 64
    g = torch.Generator(device=dev).manual_seed(1)
    w = (torch.randn(N, K, device=dev, generator=g) * 0.02).to(torch.bfloat16)
    x = torch.randn(M, K, device=dev, generator=g).to(torch.bfloat16)
    bias = (torch.randn(N, device=dev, generator=g) * 0.02).to(torch.bfloat16)
    wq, s, b = qlinear.quantize(w, gs, bits)
    y = qlinear.quantized_matmul(x, wq, s, b, True, gs, bits, bias=bias, act=act, kernel=GEMM)
    torch.cuda.synchronize()
    assert qlinear.device_error() == 0
    rows = [0, 1, 255, 256, 2047, 4095, 4352, 4607]
    code = O.ACT_GELU_TANH if act else O.ACT_NONE
    ref = O.quantized_matmul(t2np(x[rows]), t2np(wq), t2np(s), t2np(b), gs, bits, bias=t2np(bias), act=code)
    assert_bf16_close(O.to_f32(t2np(y[rows])), O.to_f32(ref), ulps=4 if act else 2, what="sampled rows")
    if act is None:
        d = qlinear.dequantize(wq, s, b, gs, bits).float()
        ref_all = ((x.float() @ d.t()).to(torch.bfloat16).float() + bias.float()).to(torch.bfloat16).float()
        err = (y.float() - ref_all).abs()
        assert err.max() <= ref_all.abs().max() * 2 ** -6
        assert (err.norm() / ref_all.norm()) <= 4e-3


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("epi", ["bias_gelu", "swiglu", "lora"])
def test_gemv_tma_epilogues(dev, bits, epi):
    """Fused epilogues on the TMA-fed GEMV (K a multiple of 8 groups).  This kernel uses the
    weights exactly (no bf16 rounding of the dequantized value) while the oracle, like MLX,
    rounds them to bf16 first; with GELU / SwiGLU (rounded op by op in the reference)
    relative L2 is allowed 6e-3."""
    M, N, K, gs = 5, 176, 2048, 64
    rng, x, wq, s, b, xt, wqt, st, bt = make_case(dev, M, N, K, gs, bits, 17)
    bias = rand_bf16((N,), 0.2, rng)
    if epi == "bias_gelu":
        y = qlinear.quantized_matmul(xt, wqt, st, bt, True, gs, bits, bias=np2t(bias, dev), act="gelu_tanh",
                                     kernel=GEMV_TMA)
        ref = O.quantized_matmul(x, wq, s, b, gs, bits, bias=bias, act=O.ACT_GELU_TANH)
        tol = dict(ulps=4, rl2=6e-3)
    elif epi == "swiglu":
        w3 = rand_bf16((N, K), 0.02, rng)
        wq3, s3, b3 = O.quantize(w3, gs, bits)
        y = qlinear.quantized_matmul(xt, wqt, st, bt, True, gs, bits, act="swiglu",
                                     up=(np2t(wq3, dev), np2t(s3, dev), np2t(b3, dev)), kernel=GEMV_TMA)
        ref = O.swiglu(O.quantized_matmul(x, wq, s, b, gs, bits), O.quantized_matmul(x, wq3, s3, b3, gs, bits))
        tol = dict(ulps=4, rl2=6e-3)
    else:
        A = rand_bf16((K, 32), 1.0 / np.sqrt(32), rng)
        B = rand_bf16((32, N), 0.01, rng)
        y = qlinear.quantized_matmul(xt, wqt, st, bt, True, gs, bits, bias=np2t(bias, dev),
                                     lora=(np2t(A, dev), np2t(B, dev), 0.5), kernel=GEMV_TMA)
        ref = O.quantized_matmul(x, wq, s, b, gs, bits, bias=bias, lora_a=A, lora_b=B, lora_scale=0.5)
        tol = dict(ulps=4, atol_frac=2 ** -7)
    torch.cuda.synchronize()
    assert qlinear.device_error() == 0
    assert_bf16_close(O.to_f32(t2np(y)), O.to_f32(ref), what=f"gemv-tma {epi}", **tol)


@pytest.mark.parametrize("bits,gs,M,N,K,epi", [
    (4, 64, 1, 19300, 1024, None),         # more tiles than SMs, ragged last tile
    (8, 128, 3, 300, 4096, None),          # Q8, 2 groups per stage, K split over a cluster
    (4, 128, 8, 128, 8192, "bias_gelu"),   # one tile: the widest K split
    (8, 64, 2, 500, 3072, "swiglu"),
    (4, 64, 1, 3072, 3072, "bias"),        # decode-sized projection
    (4, 64, 6, 1000, 512, "gelu_erf"),     # one stage per row tile
])
def test_gemv_tc_shapes(dev, bits, gs, M, N, K, epi):
    """The tcgen05 GEMV (M <= 8, group size 64/128, K a whole number of 256-byte row
    stages): tile counts above the SM count, K split across a cluster, every epilogue.
    Like the mma.sync GEMV it uses the weights exactly while the oracle rounds them to bf16
    first, so activation epilogues get relative L2 6e-3."""
    rng, x, wq, s, b, xt, wqt, st, bt = make_case(dev, M, N, K, gs, bits, 31 + M + bits)
    tol = {}
    if epi == "swiglu":
        w3 = rand_bf16((N, K), 0.02, rng)
        wq3, s3, b3 = O.quantize(w3, gs, bits)
        bias3 = rand_bf16((N,), 0.2, rng)
        y = qlinear.quantized_matmul(xt, wqt, st, bt, True, gs, bits, act="swiglu",
                                     up=(np2t(wq3, dev), np2t(s3, dev), np2t(b3, dev), np2t(bias3, dev)),
                                     kernel=GEMV_TC)
        ref = O.swiglu(O.quantized_matmul(x, wq, s, b, gs, bits),
                       O.quantized_matmul(x, wq3, s3, b3, gs, bits, bias=bias3))
        tol = dict(ulps=4, rl2=6e-3)
    else:
        bias = rand_bf16((N,), 0.2, rng) if epi else None
        act = {None: None, "bias": None, "bias_gelu": "gelu_tanh", "gelu_erf": "gelu"}[epi]
        oact = {None: O.ACT_NONE, "gelu_tanh": O.ACT_GELU_TANH, "gelu": O.ACT_GELU_ERF}[act]
        y = qlinear.quantized_matmul(xt, wqt, st, bt, True, gs, bits, bias=None if bias is None else np2t(bias, dev),
                                     act=act, kernel=GEMV_TC)
        ref = O.quantized_matmul(x, wq, s, b, gs, bits, bias=bias, act=oact)
        if act:
            tol = dict(ulps=4, rl2=6e-3)
    torch.cuda.synchronize()
    assert qlinear.device_error() == 0
    assert_bf16_close(O.to_f32(t2np(y)), O.to_f32(ref), what=f"gemv-tc {bits} {gs} {M}x{N}x{K} {epi}", **tol)


def test_gemv_tc_rejects_what_it_cannot_run(dev):
    """Forcing the tcgen05 GEMV on a shape it does not take is an error, not a silent
    fallback (Q4 with group size 32, K not a whole number of stages, M > 8)."""
    for (M, K, gs, bits) in [(1, 1024, 32, 4), (1, 384, 64, 4), (9, 1024, 64, 4)]:
        _, x, wq, s, b, xt, wqt, st, bt = make_case(dev, M, 128, K, gs, bits, 5)
        with pytest.raises(qlinear.QlError):
            qlinear.quantized_matmul(xt, wqt, st, bt, True, gs, bits, kernel=GEMV_TC)


@pytest.mark.parametrize("bits,K", [(8, 32768), (4, 65536)])
def test_gemv_long_k_falls_back(dev, bits, K):
    """An M * K whose activations fit no GEMV's shared memory: the tcgen05 GEMV refuses it
    when forced, and the automatic choice (M = 8 would pick a GEMV) streams x through the
    GEMM instead of failing (the reference takes any K)."""
    M, N, gs = 8, 256, 64
    _, x, wq, s, b, xt, wqt, st, bt = make_case(dev, M, N, K, gs, bits, 3 + bits)
    with pytest.raises(qlinear.QlError):
        qlinear.quantized_matmul(xt, wqt, st, bt, True, gs, bits, kernel=GEMV_TC)
    y = qlinear.quantized_matmul(xt, wqt, st, bt, True, gs, bits)
    torch.cuda.synchronize()
    assert qlinear.device_error() == 0
    assert_bf16_close(O.to_f32(t2np(y)), O.to_f32(O.quantized_matmul(x, wq, s, b, gs, bits)), what="gemv-long-k")


@pytest.mark.parametrize("bits,gs", [(4, 64), (4, 128), (8, 32), (8, 64), (8, 128)])
@pytest.mark.parametrize("M", [1, 3, 8])
@pytest.mark.parametrize("K", [1024, 2048])
def test_gemv_tc_parity(dev, bits, gs, M, K):
    """The tcgen05 GEMV forced on small shapes (the automatic choice sends these to the
    mma.sync kernel): every group size and bit width it takes, M = 1..8."""
    N = 200
    _, x, wq, s, b, xt, wqt, st, bt = make_case(dev, M, N, K, gs, bits, 7 * M + gs + bits)
    y = qlinear.quantized_matmul(xt, wqt, st, bt, True, gs, bits, kernel=GEMV_TC)
    torch.cuda.synchronize()
    assert qlinear.device_error() == 0
    assert_bf16_close(O.to_f32(t2np(y)), O.to_f32(O.quantized_matmul(x, wq, s, b, gs, bits)), what="gemv-tc")


@pytest.mark.parametrize("kernel,M", [(GEMV, 1), (GEMV_TMA, 5), (GEMV_REGS, 2), (GEMV_TC, 3), (GEMM, 300),
                                      (GEMM2, 300), (GENERIC, 7)])
@pytest.mark.parametrize("gate_mode", ["none", "row", "period"])
def test_gated_residual_epilogue(dev, kernel, M, gate_mode):
    """y = residual + gate * (x W^T + bias) fused in the epilogue, each op rounded to bf16
    as the reference's eager ops (src/nn.rs:166-176); gate per column, or per batch of
    `period` token rows."""
    N, K, gs, bits = 256, 1024, 64, 4
    rng, x, wq, s, b, xt, wqt, st, bt = make_case(dev, M, N, K, gs, bits, 41 + M)
    bias = rand_bf16((N,), 0.2, rng)
    res = rand_bf16((M, N), 1.0, rng)
    gate, period = None, 0
    if gate_mode == "row":
        gate = rand_bf16((N,), 1.0, rng)
    elif gate_mode == "period":
        period = 2
        gate = rand_bf16(((M + period - 1) // period, N), 1.0, rng)
    y = qlinear.quantized_matmul(xt, wqt, st, bt, True, gs, bits, bias=np2t(bias, dev), kernel=kernel,
                                 residual=np2t(res, dev), gate=None if gate is None else np2t(gate, dev),
                                 gate_period=period)
    torch.cuda.synchronize()
    assert qlinear.device_error() == 0
    lin = O.quantized_matmul(x, wq, s, b, gs, bits, bias=bias)
    ref = O.gated(res, gate, lin, period)
    # the linear's own tolerance, carried through the gate (|gate| ~ 1) and the residual add
    assert_bf16_close(O.to_f32(t2np(y)), O.to_f32(ref), ulps=4, what=f"gated {gate_mode}")


@pytest.mark.parametrize("kernel,M", [(qlinear.KERNEL_AUTO, 3), (GEMM, 300), (GENERIC, 9)])
@pytest.mark.parametrize("bits", [4, 8])
def test_lokr_delta(dev, kernel, M, bits):
    """LoKr residual ``scale * x . delta^T`` (dense delta, src/adapters.rs:263-266) fused
    into the dequantized weights, against the reference's separate rounding of base and
    residual (4 ulps + 1/128 of the output scale, as for LoRA); M <= 8 on AUTO runs the
    GEMM (the GEMV kernels do not take a delta)."""
    N, K, gs = 256, 1024, 64
    rng, x, wq, s, b, xt, wqt, st, bt = make_case(dev, M, N, K, gs, bits, 61 + M + bits)
    bias = rand_bf16((N,), 0.2, rng)
    delta = rand_bf16((N, K), 0.01, rng)
    scale = 0.75
    y = qlinear.quantized_matmul(xt, wqt, st, bt, True, gs, bits, bias=np2t(bias, dev),
                                 lokr=(np2t(delta, dev), scale), kernel=kernel)
    torch.cuda.synchronize()
    assert qlinear.device_error() == 0
    ref = O.add_bf16(O.quantized_matmul(x, wq, s, b, gs, bits, bias=bias), O.lokr_residual(x, delta, scale))
    assert_bf16_close(O.to_f32(t2np(y)), O.to_f32(ref), ulps=4, atol_frac=2 ** -7, what="lokr")


def test_lokr_with_lora_and_gate_through_adaptable_linear(dev):
    """AdaptableLinear with one LoRA and one LoKr adapter runs fused (one call), with the
    gated residual on top, against the reference's op-by-op composition."""
    M, N, K, gs, bits = 260, 384, 512, 64, 4
    rng, x, wq, s, b, xt, wqt, st, bt = make_case(dev, M, N, K, gs, bits, 77)
    A = rand_bf16((K, 16), 1.0 / 4, rng)
    B = rand_bf16((16, N), 0.01, rng)
    delta = rand_bf16((N, K), 0.01, rng)
    lin = qlinear.AdaptableLinear.from_quantized_parts(wqt, st, bt, None, gs, bits)
    lin.push(qlinear.Lora(np2t(A, dev), np2t(B, dev), 0.5))
    lin.push(qlinear.Lokr(np2t(delta, dev), 2.0))
    y = lin.forward(xt)
    torch.cuda.synchronize()
    assert qlinear.device_error() == 0
    base = O.quantized_matmul(x, wq, s, b, gs, bits, lora_a=A, lora_b=B, lora_scale=0.5)
    ref = O.add_bf16(base, O.lokr_residual(x, delta, 2.0))
    assert_bf16_close(O.to_f32(t2np(y)), O.to_f32(ref), ulps=4, atol_frac=2 ** -7, what="lora+lokr")


def test_adaptable_linear_f32_lora_factors_promote_to_f32(dev):
    """f32 LoRA factors (the reference goldens' dtype) on a quantized base with bf16 x:
    the reference's output is the bf16 base plus an f32 residual, promoted to f32
    (src/adapters.rs:240-258), so the stack runs unfused: the base on libqlinear, the
    residual in f32."""
    M, N, K, gs, bits = 40, 256, 512, 64, 4
    rng, x, wq, s, b, xt, wqt, st, bt = make_case(dev, M, N, K, gs, bits, 91)
    A = (rng.standard_normal((K, 8)) / np.sqrt(8)).astype(np.float32)
    B = (rng.standard_normal((8, N)) * 0.01).astype(np.float32)
    lin = qlinear.AdaptableLinear.from_quantized_parts(wqt, st, bt, None, gs, bits)
    lin.push(qlinear.Lora(torch.from_numpy(A).to(dev), torch.from_numpy(B).to(dev), 0.5))
    y = lin.forward(xt)
    torch.cuda.synchronize()
    assert y.dtype == torch.float32 and qlinear.device_error() == 0
    base = O.to_f32(O.quantized_matmul(x, wq, s, b, gs, bits)).astype(np.float64)
    res = (O.to_f32(x).astype(np.float64) @ A @ B) * 0.5
    got = y.cpu().numpy().astype(np.float64)
    assert np.abs(got - (base + res)).max() <= 2 ** -7 * np.abs(base).max() + 1e-4


@pytest.mark.parametrize("bits", [8, 4])
def test_output_dtype_promotes_like_mlx(golden, dev, bits):
    """bf16 activations against the fixture's f32 scales: mlx's quantized_matmul returns
    promote(bf16, f32) = f32 (the generic kernel serves the mixed case)."""
    p = f"q{bits}_"
    xb = O.to_bf16(golden["x"].astype(np.float32))
    y = qlinear.quantized_matmul(np2t(xb, dev), np2t(golden[p + "wq"], dev), np2t(golden[p + "scales"], dev),
                                 np2t(golden[p + "biases"], dev), True, 64, bits)
    assert y.dtype == torch.float32
    w = O.dequantize(golden[p + "wq"], golden[p + "scales"], golden[p + "biases"], 64, bits).astype(np.float64)
    ref = O.to_f32(xb).astype(np.float64) @ w.T
    np.testing.assert_allclose(t2np(y), ref, rtol=1e-4, atol=1e-3)


@pytest.mark.parametrize("bits", [8, 4])
def test_adaptable_linear_quantize_matches_bf16_reference(golden, dev, bits):
    """AdaptableLinear.quantize quantizes the bf16-cast weight (tests/quant_parity.rs:68-96):
    its forward on the fixture's f32 x matches the oracle's quantize(bf16(w)) + qmm within
    the reference's (1e-3, 1e-4)."""
    lin = qlinear.AdaptableLinear.dense(torch.from_numpy(golden["w"]).to(dev))
    assert not lin.is_quantized()
    lin.quantize(bits)
    assert lin.is_quantized()
    out = lin(torch.from_numpy(golden["x"]).to(dev))
    assert out.dtype == torch.float32
    wq, s, b = O.quantize(O.to_bf16(golden["w"]), 64, bits)
    ref = O.to_f32(O.quantized_matmul(golden["x"], wq, s, b, 64, bits))
    np.testing.assert_allclose(out.cpu().numpy(), ref, rtol=1e-3, atol=1e-4)


def test_quantized_forward_approximates_dense(golden, dev):
    """Peak-relative error against the dense forward: Q8 < 2 %, Q4 < 12 %
    (tests/quant_parity.rs:98-127)."""
    w = torch.from_numpy(golden["w"]).to(dev)
    x = torch.from_numpy(golden["x"]).to(dev)
    dense = qlinear.AdaptableLinear.dense(w)(x)
    peak = dense.abs().max().item()
    for bits, max_rel in [(8, 0.02), (4, 0.12)]:
        q = qlinear.AdaptableLinear.dense(w)
        q.quantize(bits)
        assert (q(x) - dense).abs().max().item() / peak < max_rel


def test_q8_forward_close_to_dense_across_shapes(dev):
    """Q8 forward vs the f32 dense forward over the transformer's linear shapes at M = 4,
    f32 and bf16 activations, bias 0.1: mean relative error < 5 %
    (mlx-gen-qwen-image/tests/q8_smoke.rs:15-60)."""
    g = torch.Generator(device=dev).manual_seed(0)
    worst = 0.0
    for out, inn in [(3072, 64), (3072, 128), (3072, 3072), (3072, 3584), (64, 3072)]:
        w = torch.randn(out, inn, device=dev, generator=g).to(torch.bfloat16)
        b = torch.full((out,), 0.1, device=dev).to(torch.bfloat16)
        x32 = torch.randn(1, 4, inn, device=dev, generator=g)
        lin = qlinear.AdaptableLinear.dense(w, b)
        d32 = lin(x32)
        lin.quantize(8)
        q32, q16 = lin(x32), lin(x32.to(torch.bfloat16))
        assert q32.shape == q16.shape == (1, 4, out)
        for q in (q32, q16):
            worst = max(worst, ((q.float() - d32).abs().sum() / d32.abs().sum()).item())
    torch.cuda.synchronize()
    assert qlinear.device_error() == 0
    assert worst < 0.05, worst


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_one_process_drives_two_gpus():
    """Kernel attributes are per device: the same entry points called on cuda:0 and then
    cuda:1 from one process (GEMM, GEMM with LoRA, GEMV) give the same results."""
    outs = []
    for d in (0, 1):
        dev = torch.device(f"cuda:{d}")
        with torch.cuda.device(dev):
            rng, x, wq, s, b, xt, wqt, st, bt = make_case(dev, 300, 256, 512, 64, 4, 7)
            A = rand_bf16((512, 16), 0.25, rng)
            B = rand_bf16((16, 256), 0.01, rng)
            y1 = qlinear.quantized_matmul(xt, wqt, st, bt, True, 64, 4)
            y2 = qlinear.quantized_matmul(xt, wqt, st, bt, True, 64, 4, lora=(np2t(A, dev), np2t(B, dev), 0.5))
            y3 = qlinear.quantized_matmul(xt[:2].contiguous(), wqt, st, bt, True, 64, 4)
            torch.cuda.synchronize(dev)
            outs.append([t2np(y) for y in (y1, y2, y3)])
    for a, b in zip(*outs):
        assert np.array_equal(a, b)
