"""numpy/ctypes front end of the CPU oracle (oracle/qref.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, ``__graft_entry__.smoke()`` and the
CPU-baseline legs of ``bench.py``.  The product library never imports it.

bf16 arrays are carried as ``np.uint16`` bit patterns; f32 as ``np.float32``;
f16 as ``np.float16``.  Every function mirrors one entry point of qref.c, which
cites the reference file:line it restates.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

F32, BF16, F16 = 0, 1, 2
ACT_NONE, ACT_GELU_TANH, ACT_GELU_ERF = 0, 1, 2

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_ref", "libqref.so")
_lib = None


def build() -> str:
    """Compile qref.c with oracle/Makefile (a no-op when up to date)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = C.CDLL(_LIB_PATH)
        i64, vp, i32 = C.c_int64, C.c_void_p, C.c_int
        L.qref_quantize.argtypes = [vp, i32, i64, i64, i32, i32, vp, vp, vp, i32]
        L.qref_dequantize.argtypes = [vp, vp, vp, i32, i64, i64, i32, i32, vp, i64, vp, i32]
        L.qref_qmm.argtypes = [vp, i32, i64, i64, vp, vp, vp, i32, i64, i32, i32, vp, i32,
                               vp, vp, i64, C.c_float, vp, i32]
        L.qref_qmm_fast.argtypes = [vp, i32, i64, i64, vp, vp, vp, i32, i64, i32, i32, vp, vp,
                                    i32, i32]
        L.qref_swiglu.argtypes = [vp, vp, i64, i32, vp]
        L.qref_f32_to_bf16.argtypes = [vp, vp, i64]
        for f in (L.qref_quantize, L.qref_dequantize, L.qref_qmm, L.qref_qmm_fast):
            f.restype = i32
        _lib = L
    return _lib


def _p(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def dtype_code(a: np.ndarray) -> int:
    if a.dtype == np.float32:
        return F32
    if a.dtype == np.uint16:
        return BF16
    if a.dtype == np.float16:
        return F16
    raise TypeError(f"unsupported dtype {a.dtype}")


def np_dtype(code: int):
    return {F32: np.float32, BF16: np.uint16, F16: np.float16}[code]


def to_bf16(a: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 bits, round to nearest even."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    out = np.empty(a.shape, np.uint16)
    lib().qref_f32_to_bf16(_p(a), _p(out), a.size)
    return out


def bf16_to_f32(a: np.ndarray) -> np.ndarray:
    return (a.astype(np.uint32) << 16).view(np.float32)


def to_f32(a: np.ndarray) -> np.ndarray:
    return bf16_to_f32(a) if a.dtype == np.uint16 else a.astype(np.float32)


def quantize(w: np.ndarray, group_size: int = 64, bits: int = 4, sb_dtype: int | None = None):
    """(wq u32 [N, K*bits/32], scales [N, K/gs], biases [N, K/gs]); scales in w's dtype."""
    w = np.ascontiguousarray(w)
    N, K = w.shape
    sd = dtype_code(w) if sb_dtype is None else sb_dtype
    wq = np.empty((N, K * bits // 32), np.uint32)
    s = np.empty((N, K // group_size), np_dtype(sd))
    b = np.empty_like(s)
    rc = lib().qref_quantize(_p(w), dtype_code(w), N, K, group_size, bits, _p(wq), _p(s), _p(b), sd)
    if rc:
        raise ValueError(f"qref_quantize rc={rc}")
    return wq, s, b


def dequantize(wq, scales, biases, group_size=64, bits=4, ids=None, out_dtype=None):
    """mlx affine dequantize (src/nn.rs:55): fma(code, scale, bias) rounded once to
    out_dtype (default: the scales' dtype).  With ids: the quantized embedding gather
    (src/nn.rs:42-59), rows ids of the dequantized table in the scales' dtype, then cast
    to out_dtype."""
    if ids is not None and out_dtype is not None and out_dtype != dtype_code(scales):
        rows = dequantize(wq, scales, biases, group_size, bits, ids=ids)
        f = to_f32(rows)
        return {F32: lambda: f, BF16: lambda: to_bf16(f), F16: lambda: f.astype(np.float16)}[out_dtype]()
    wq = np.ascontiguousarray(wq, np.uint32)
    N, G = scales.shape
    K = G * group_size
    od = dtype_code(scales) if out_dtype is None else out_dtype
    rows = N
    idp = None
    if ids is not None:
        ids = np.ascontiguousarray(ids, np.int64).reshape(-1)
        rows = ids.size
        idp = ids
    out = np.empty((rows, K), np_dtype(od))
    rc = lib().qref_dequantize(_p(wq), _p(np.ascontiguousarray(scales)), _p(np.ascontiguousarray(biases)),
                               dtype_code(scales), N, K, group_size, bits, _p(idp), rows, _p(out), od)
    if rc:
        raise ValueError(f"qref_dequantize rc={rc}")
    return out


def quantized_matmul(x, wq, scales, biases, group_size=64, bits=4, bias=None, act=ACT_NONE,
                     lora_a=None, lora_b=None, lora_scale=1.0, out_dtype=None):
    """Exact-mode y = x . dequant(W)^T with the reference's rounding points (see qref.c)."""
    x = np.ascontiguousarray(x)
    M, K = x.shape
    N = scales.shape[0]
    od = dtype_code(x) if out_dtype is None else out_dtype
    y = np.empty((M, N), np_dtype(od))
    rank = 0 if lora_a is None else lora_a.shape[1]
    rc = lib().qref_qmm(_p(x), dtype_code(x), M, K, _p(np.ascontiguousarray(wq, np.uint32)),
                        _p(np.ascontiguousarray(scales)), _p(np.ascontiguousarray(biases)),
                        dtype_code(scales), N, group_size, bits,
                        _p(None if bias is None else np.ascontiguousarray(bias)), act,
                        _p(None if lora_a is None else np.ascontiguousarray(lora_a)),
                        _p(None if lora_b is None else np.ascontiguousarray(lora_b)),
                        rank, float(lora_scale), _p(y), od)
    if rc:
        raise ValueError(f"qref_qmm rc={rc}")
    return y


def quantized_matmul_fast(x, wq, scales, biases, group_size=64, bits=4, bias=None, threads=None):
    """The timed CPU baseline (fp32 accumulation, pthreads)."""
    x = np.ascontiguousarray(x)
    M, K = x.shape
    N = scales.shape[0]
    od = dtype_code(x)
    y = np.empty((M, N), np_dtype(od))
    nt = threads or os.cpu_count() or 1
    rc = lib().qref_qmm_fast(_p(x), od, M, K, _p(np.ascontiguousarray(wq, np.uint32)),
                             _p(np.ascontiguousarray(scales)), _p(np.ascontiguousarray(biases)),
                             dtype_code(scales), N, group_size, bits,
                             _p(None if bias is None else np.ascontiguousarray(bias)), _p(y), od, nt)
    if rc:
        raise ValueError(f"qref_qmm_fast rc={rc}")
    return y


def swiglu(a, b):
    a = np.ascontiguousarray(a)
    b = np.ascontiguousarray(b)
    out = np.empty_like(a)
    lib().qref_swiglu(_p(a), _p(b), a.size, dtype_code(a), _p(out))
    return out


def gated(res, gate, y, period=0):
    """``res + gate * y`` with each op rounded to bf16, as the reference's eager
    ``add(x, multiply(gate, y))`` on bf16 arrays (src/nn.rs:166-176).  All bf16 bits;
    gate is [N] or [rows, N] with row m // period (period 0: row 0 for every m)."""
    y32 = bf16_to_f32(np.ascontiguousarray(y))
    M, N = y32.shape
    if gate is not None:
        g = bf16_to_f32(np.ascontiguousarray(gate)).reshape(-1, N)
        rows = (np.arange(M) // period) if period > 0 else np.zeros(M, np.int64)
        y32 = bf16_to_f32(to_bf16(g[rows] * y32))
    return to_bf16(bf16_to_f32(np.ascontiguousarray(res)) + y32)


def lokr_residual(x, delta, scale):
    """``scale * x . delta^T`` as the reference computes it for bf16 x: delta cast to x's
    dtype, the matmul rounded to bf16, then the scalar product rounded
    (src/adapters.rs:263-266).  bf16 bits in and out."""
    xm = bf16_to_f32(np.ascontiguousarray(x)).astype(np.float64)
    dm = bf16_to_f32(np.ascontiguousarray(delta)).astype(np.float64)
    r = bf16_to_f32(to_bf16((xm @ dm.T).astype(np.float32)))
    s = bf16_to_f32(to_bf16(np.float32([scale])))[0]
    return to_bf16(r * s)


def add_bf16(a, b):
    """Elementwise bf16 add, rounded (the residual sum of AdaptableLinear::forward)."""
    return to_bf16(bf16_to_f32(np.ascontiguousarray(a)) + bf16_to_f32(np.ascontiguousarray(b)))


def layernorm_modulate(x, scale=None, shift=None, eps=1e-6, period=0, f32_out=False):
    """``(1 + scale) * layer_norm(x) + shift`` with the reference's rounding points:
    mlx fast::layer_norm (fp32 statistics, output rounded to bf16), then nn::modulate
    (src/nn.rs:262-287): with one_matches_scale every op rounded to bf16 (FLUX.1), else
    f32 arithmetic and an f32 result (FLUX.2).  x, scale, shift bf16 bits.  The mean and
    variance are taken in float64 (the reference's exact fp32 reduction order is not
    published): rounding ties of the bf16 normalised value may differ."""
    xf = bf16_to_f32(np.ascontiguousarray(x)).astype(np.float64)
    M, D = xf.shape
    mean = xf.mean(axis=1, keepdims=True)
    var = ((xf - mean) ** 2).mean(axis=1, keepdims=True)
    n = bf16_to_f32(to_bf16(((xf - mean) / np.sqrt(var + eps)).astype(np.float32)))
    rows = (np.arange(M) // period) if period > 0 else np.zeros(M, np.int64)
    r = n
    if scale is not None:
        s = bf16_to_f32(np.ascontiguousarray(scale)).reshape(-1, D)[rows]
        if f32_out:
            r = (r * (s + np.float32(1.0))).astype(np.float32)
        else:
            r = bf16_to_f32(to_bf16(r * bf16_to_f32(to_bf16(s + np.float32(1.0)))))
    if shift is not None:
        h = bf16_to_f32(np.ascontiguousarray(shift)).reshape(-1, D)[rows]
        r = (r + h).astype(np.float32)
    return r.astype(np.float32) if f32_out else to_bf16(r)



def _round_to(a64, bf16: bool):
    """Round float64 values to the factors' dtype (bf16 or f32), returned as f32."""
    a32 = np.asarray(a64, dtype=np.float64).astype(np.float32)
    return bf16_to_f32(to_bf16(a32)) if bf16 else a32


def _factor(f, bf16: bool):
    """A full factor, or an (a, b) low-rank pair multiplied in the factors' dtype."""
    if isinstance(f, tuple):
        a, b = f
        return _round_to(np.asarray(a, np.float64) @ np.asarray(b, np.float64), bf16)
    return np.asarray(f, np.float32)


def lokr_delta(scale, base_shape, f1, f2, factors_bf16=True):
    """``scale * kron(f1, f2)`` with the reference's rounding points
    (src/adapters.rs:71-101): low-rank products and the Kronecker product in the factors'
    dtype, the scale applied in f32 (a one-element f32 array), one cast to bf16.  Factor
    values are f32 arrays (bf16-representable when factors_bf16); returns bf16 bits."""
    a = _factor(f1, factors_bf16)
    b = _factor(f2, factors_bf16)
    k = _round_to(np.kron(a.astype(np.float64), b.astype(np.float64)), factors_bf16)
    return to_bf16((k * np.float32(scale)).astype(np.float32).reshape(base_shape))


def loha_delta(scale, base_shape, w1, w2, factors_bf16=True):
    """``scale * ((w1_a @ w1_b) * (w2_a @ w2_b))`` (src/adapters.rs:138-158); w1, w2 are
    (a, b) pairs; rounding as lokr_delta.  Returns bf16 bits."""
    m1 = _factor(w1, factors_bf16)
    m2 = _factor(w2, factors_bf16)
    h = _round_to(m1.astype(np.float64) * m2.astype(np.float64), factors_bf16)
    return to_bf16((h * np.float32(scale)).astype(np.float32).reshape(base_shape))
