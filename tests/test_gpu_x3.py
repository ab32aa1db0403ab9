"""GPU parity: f32 and f16 activations on the tcgen05 GEMM (the three-pass bf16 split:
x = xhi + xlo, w = whi + wlo, y = whi.xhi + whi.xlo + wlo.xhi accumulated in fp32) against
the oracle, which accumulates in fp64 the dequantized weights in the computation dtype
promote(x, scales) (src/adapters.rs:252, src/nn.rs:295: f32 activations with bf16 scales;
mlx casts quantized_matmul's operands to that dtype).

Stated tolerance for this path: each product keeps about 16 significant bits, so
|y - y_ref| <= 2^-13 * sum_k |w_k x_k| (+ the output dtype's rounding: 1 ulp of |y_ref| for
f16 outputs, 4 ulp after GELU) element-wise, and relative L2 <= 1e-4 (f32) / 2e-3 (f16)."""
import numpy as np
import pytest
import torch

import oracle as O
import qlinear
from helpers import np2t, rand_bf16, t2np

pytestmark = pytest.mark.gpu


def _ulp16(a):
    return np.exp2(np.floor(np.log2(np.maximum(np.abs(a), 2.0 ** -14))) - 10)


def _check(got, ref, absw_absx, out, act):
    got, ref = got.astype(np.float64), ref.astype(np.float64)
    bound = 2.0 ** -13 * absw_absx
    if out == "f16":
        bound = bound + (4.0 if act else 1.0) * _ulp16(ref)
    elif act:
        bound = bound + 2.0 ** -20 * np.abs(ref)
    err = np.abs(got - ref)
    bad = err > bound + 1e-30
    assert not bad.any(), f"{bad.sum()} elements out of bound; worst excess {(err - bound).max():.3e}"
    rel = np.linalg.norm(got - ref) / max(np.linalg.norm(ref), 1e-30)
    assert rel <= (1e-4 if out == "f32" else 2e-3), rel


@pytest.mark.parametrize("xdt,sdt", [("f32", "bf16"), ("f16", "bf16"), ("f16", "f16"), ("f32", "f16")])
@pytest.mark.parametrize("bits,gs", [(4, 64), (8, 64), (4, 128), (8, 32)])
@pytest.mark.parametrize("M,N,K", [(300, 256, 448), (513, 384, 1024)])
def test_x3_gemm_matches_oracle(dev, xdt, sdt, bits, gs, M, N, K):
    if K % gs:
        pytest.skip("K must be a multiple of the group size")
    rng = np.random.default_rng(M + N + K + bits + gs)
    w = rand_bf16((N, K), 0.02, rng)
    wq, s, b = O.quantize(w, gs, bits, sb_dtype=O.F16 if sdt == "f16" else O.BF16)
    xf = (rng.standard_normal((M, K))).astype(np.float32)
    x = xf if xdt == "f32" else xf.astype(np.float16)
    out = "f32" if (xdt == "f32" or sdt != xdt) else "f16"
    y = qlinear.quantized_matmul(torch.from_numpy(x).to(dev), np2t(wq, dev), np2t(s, dev), np2t(b, dev),
                                 True, gs, bits, kernel=qlinear.KERNEL_GEMM)
    torch.cuda.synchronize()
    assert qlinear.device_error() == 0
    assert y.dtype == (torch.float32 if out == "f32" else torch.float16)
    ref = O.quantized_matmul(x.astype(np.float32) if out == "f32" else x, wq, s, b, gs, bits,
                             out_dtype=O.F32 if out == "f32" else O.F16)
    wd = O.to_f32(O.dequantize(wq, s, b, gs, bits, out_dtype=O.F32)).astype(np.float64)
    _check(t2np(y), ref, np.abs(x.astype(np.float64)) @ np.abs(wd).T, out, False)


@pytest.mark.parametrize("act", [None, "gelu_tanh", "gelu"])
def test_x3_bias_act(dev, act):
    rng = np.random.default_rng(5)
    M, N, K, gs, bits = 260, 192, 512, 64, 4
    w = rand_bf16((N, K), 0.02, rng)
    wq, s, b = O.quantize(w, gs, bits)
    x = rng.standard_normal((M, K)).astype(np.float32)
    bias = (rng.standard_normal(N) * 0.02).astype(np.float32)
    y = qlinear.quantized_matmul(torch.from_numpy(x).to(dev), np2t(wq, dev), np2t(s, dev), np2t(b, dev), True, gs, bits,
                                 bias=torch.from_numpy(bias).to(dev), act=act)
    torch.cuda.synchronize()
    code = {None: O.ACT_NONE, "gelu_tanh": O.ACT_GELU_TANH, "gelu": O.ACT_GELU_ERF}[act]
    ref = O.quantized_matmul(x, wq, s, b, gs, bits, bias=bias, act=code, out_dtype=O.F32)
    wd = O.to_f32(O.dequantize(wq, s, b, gs, bits, out_dtype=O.F32)).astype(np.float64)
    _check(t2np(y), ref, np.abs(x.astype(np.float64)) @ np.abs(wd).T + np.abs(bias), "f32", act is not None)


def test_x3_matches_cuda_core_kernel_at_size(dev):
    """FLUX.2-like f32 activations at a DiT size: the tensor-core split path against the
    fp32 CUDA-core kernel (a second, independent implementation), every element."""
    g = torch.Generator(device=dev).manual_seed(2)
    M, N, K = 2048, 3072, 3072
    w = (torch.randn(N, K, device=dev, generator=g) * 0.02).to(torch.bfloat16)
    x = torch.randn(M, K, device=dev, generator=g)
    wq, s, b = qlinear.quantize(w, 64, 8)
    y = qlinear.quantized_matmul(x, wq, s, b, True, 64, 8, kernel=qlinear.KERNEL_GEMM)
    y2 = qlinear.quantized_matmul(x, wq, s, b, True, 64, 8, kernel=qlinear.KERNEL_GENERIC)
    torch.cuda.synchronize()
    assert qlinear.device_error() == 0
    wd = qlinear.dequantize(wq, s, b, 64, 8, out_dtype=torch.float32)
    absb = x.abs() @ wd.abs().t()
    assert ((y - y2).abs() <= 2.0 ** -13 * absb + 1e-6).all()
    assert float((y - y2).norm() / y2.norm()) < 1e-4
