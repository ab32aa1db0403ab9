"""Tensor-level operators of the quantized-linear path, mirroring mlx-rs's
``ops::{quantize, dequantize, quantized_matmul}`` as the reference calls them
(src/quant.rs:140, src/nn.rs:51-56, src/adapters.rs:309-317).

torch is used only for device memory and the current stream; every arithmetic
operation runs in libqlinear's CUDA kernels through the C ABI.
"""
from __future__ import annotations

import ctypes as C
from typing import Optional, Sequence

import torch

from . import _lib
from ._lib import (ACT_GELU_ERF, ACT_GELU_TANH, ACT_NONE, ACT_SWIGLU, KERNEL_AUTO, Epilogue,
                   check, lib)

_DT = {torch.float32: _lib.QL_F32, torch.bfloat16: _lib.QL_BF16, torch.float16: _lib.QL_F16}
_ACTS = {None: ACT_NONE, "none": ACT_NONE, "gelu_tanh": ACT_GELU_TANH, "gelu": ACT_GELU_ERF,
         "gelu_erf": ACT_GELU_ERF, "swiglu": ACT_SWIGLU}


def dtype_code(t: torch.Tensor) -> int:
    try:
        return _DT[t.dtype]
    except KeyError:
        raise TypeError(f"unsupported dtype {t.dtype}; expected float32, bfloat16 or float16") from None


def _ptr(t: Optional[torch.Tensor]):
    return None if t is None else C.c_void_p(t.data_ptr())


def _stream(device: torch.device):
    return C.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _need_cuda(*ts: Optional[torch.Tensor]) -> None:
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("libqlinear operates on CUDA tensors only")


def quantize(w: torch.Tensor, group_size: int = 64, bits: int = 4):
    """Group-wise affine quantization of a 2-D weight [N, K] along K.

    Returns ``(wq, scales, biases)``: uint32-packed codes ``[N, K*bits/32]`` (as int32
    storage, bit-identical) and per-group scales/biases ``[N, K/group_size]`` in w's dtype,
    as ``mlx_rs::ops::quantize`` does (src/quant.rs:140)."""
    _need_cuda(w)
    if w.dim() != 2:
        raise ValueError("quantize expects a 2-D weight [out, in]")
    w = w.contiguous()
    N, K = w.shape
    wq = torch.empty((N, K * bits // 32), dtype=torch.int32, device=w.device)
    scales = torch.empty((N, max(K // group_size, 1)), dtype=w.dtype, device=w.device)
    biases = torch.empty_like(scales)
    check(lib().ql_quantize(_ptr(w), dtype_code(w), N, K, group_size, bits, _ptr(wq), _ptr(scales),
                            _ptr(biases), dtype_code(scales), _stream(w.device)))
    return wq, scales, biases


def dequantize(wq: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor, group_size: int = 64,
               bits: int = 4, out_dtype: Optional[torch.dtype] = None) -> torch.Tensor:
    """``w = code * scale + bias`` (one rounding), ``[N, K]`` in the scales' dtype by default."""
    _need_cuda(wq, scales, biases)
    N, G = scales.shape
    K = G * group_size
    out = torch.empty((N, K), dtype=out_dtype or scales.dtype, device=wq.device)
    check(lib().ql_dequantize(_ptr(wq.contiguous()), _ptr(scales.contiguous()), _ptr(biases.contiguous()),
                              dtype_code(scales), N, K, group_size, bits, _ptr(out), dtype_code(out),
                              _stream(wq.device)))
    return out


def dequantize_rows(ids: torch.Tensor, wq: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor,
                    group_size: int = 64, bits: int = 4,
                    out_dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """Quantized embedding gather: rows ``ids`` (any shape) dequantized -> ``[*ids.shape, K]``."""
    _need_cuda(ids, wq, scales, biases)
    N, G = scales.shape
    K = G * group_size
    flat = ids.reshape(-1).to(torch.int64).contiguous()
    out = torch.empty((flat.numel(), K), dtype=out_dtype, device=wq.device)
    check(lib().ql_dequantize_rows(_ptr(flat), flat.numel(), _ptr(wq.contiguous()), _ptr(scales.contiguous()),
                                   _ptr(biases.contiguous()), dtype_code(scales), N, K, group_size, bits,
                                   _ptr(out), dtype_code(out), _stream(wq.device)))
    return out.reshape(*ids.shape, K)


def layernorm_modulate(x: torch.Tensor, scale: Optional[torch.Tensor] = None, shift: Optional[torch.Tensor] = None,
                       eps: float = 1e-6, period: int = 0, out_dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    """``(1 + scale) * layer_norm(x) + shift`` in one pass (the DiT adaLN prologue:
    ``fast::layer_norm`` then ``nn::modulate``, mlx-gen-flux/src/transformer.rs:891-913).
    x bf16 ``[..., D]``; scale / shift ``[D]`` or ``[rows, D]`` with row ``m // period``.
    out_dtype bf16: FLUX.1 rounding (every op in bf16); float32: FLUX.2 (a strong f32 1)."""
    _need_cuda(x, scale, shift)
    D = x.shape[-1]
    x2 = x.reshape(-1, D).to(torch.bfloat16).contiguous()
    y = torch.empty(x2.shape, dtype=out_dtype, device=x.device)
    sc = None if scale is None else scale.to(torch.bfloat16).reshape(-1, D).contiguous()
    sh = None if shift is None else shift.to(torch.bfloat16).reshape(-1, D).contiguous()
    check(lib().ql_layernorm_modulate(_ptr(x2), x2.shape[0], D, float(eps), _ptr(sc), _ptr(sh), int(period),
                                      _ptr(y), dtype_code(y), _stream(x.device)))
    return y.reshape(x.shape)


def workspace_size(M: int, N: int, K: int, lora_rank: int = 0) -> int:
    ep = Epilogue()
    if lora_rank:
        ep.lora_a = C.c_void_p(1)
        ep.lora_rank = lora_rank
    return int(lib().ql_matmul_workspace_size(M, N, K, C.byref(ep)))


def quantized_matmul(x: torch.Tensor, wq: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor,
                     transpose: bool = True, group_size: int = 64, bits: int = 4, *,
                     bias: Optional[torch.Tensor] = None, act: Optional[str] = None,
                     up: Optional[Sequence[Optional[torch.Tensor]]] = None,
                     lora: Optional[tuple] = None, workspace: Optional[torch.Tensor] = None,
                     kernel: int = KERNEL_AUTO, out: Optional[torch.Tensor] = None,
                     max_ctas: int = 0, residual: Optional[torch.Tensor] = None,
                     gate: Optional[torch.Tensor] = None, gate_period: int = 0,
                     lokr: Optional[tuple] = None) -> torch.Tensor:
    """``y = x . dequant(W)^T`` (+ fused epilogue), like ``mlx_rs::ops::quantized_matmul``
    with ``transpose=true`` followed by the ops the reference runs after it.

    x: ``[..., K]``.  bias: ``[N]`` (added after rounding the matmul, as
    src/adapters.rs:318-320 does).  act: None, "gelu_tanh", "gelu" or "swiglu" (then
    ``up = (wq3, scales3, biases3[, bias3])`` is the second projection and the result is
    ``silu(x W^T) * (x W3^T)``).  lora: ``(A [K, r], B [r, N], scale)`` adds
    ``scale * (x.A).B``.  lokr: ``(delta [N, K], scale)`` adds ``scale * x.delta^T``
    (src/adapters.rs:263-266), fused into the dequantized weights.  residual / gate: the gated residual ``residual + gate * y``
    (src/nn.rs:166-176), gate ``[N]`` or ``[M / gate_period, N]``.  Output dtype =
    promote(x, scales), as mlx's; bias, residual and gate are taken in that dtype."""
    _need_cuda(x, wq, scales, biases, bias)
    if not transpose:
        raise NotImplementedError("only transpose=True is supported (the reference's only form)")
    K = x.shape[-1]
    N = scales.shape[0]
    lead = x.shape[:-1]
    x2 = x.reshape(-1, K).contiguous()
    M = x2.shape[0]
    # mlx's quantized_matmul returns promote(x, scales): bf16 x with f32 scales gives f32
    ydt = torch.promote_types(x.dtype, scales.dtype)
    y = out if out is not None else torch.empty((*lead, N), dtype=ydt, device=x.device)
    ep = Epilogue()
    keep = []  # tensors whose memory the call reads
    if bias is not None:
        bias = bias.to(y.dtype).contiguous()
        keep.append(bias)
        ep.bias = bias.data_ptr()
    ep.act = _ACTS[act]
    if ep.act == ACT_SWIGLU:
        if up is None:
            raise ValueError("act='swiglu' needs up=(wq, scales, biases[, bias])")
        uq, us, ub = up[0].contiguous(), up[1].contiguous(), up[2].contiguous()
        keep += [uq, us, ub]
        ep.wq_up, ep.scales_up, ep.biases_up = uq.data_ptr(), us.data_ptr(), ub.data_ptr()
        if len(up) > 3 and up[3] is not None:
            ubias = up[3].to(y.dtype).contiguous()
            keep.append(ubias)
            ep.bias_up = ubias.data_ptr()
    if lora is not None:
        a, b, s = lora
        a = a.to(x.dtype).contiguous()
        b = b.to(x.dtype).contiguous()
        keep += [a, b]
        ep.lora_a, ep.lora_b = a.data_ptr(), b.data_ptr()
        ep.lora_rank = a.shape[1]
        ep.lora_scale = float(s)
        need = int(lib().ql_matmul_workspace_size(M, N, K, C.byref(ep)))
        if workspace is None or workspace.numel() * workspace.element_size() < need:
            workspace = torch.empty(need, dtype=torch.uint8, device=x.device)
        keep.append(workspace)
        ep.workspace = workspace.data_ptr()
        ep.workspace_bytes = workspace.numel() * workspace.element_size()
    if lokr is not None:
        delta, lscale = lokr
        delta = delta.to(x.dtype).contiguous()
        if tuple(delta.shape) != (N, K):
            raise ValueError(f"LoKr delta must be [{N}, {K}], got {tuple(delta.shape)}")
        keep.append(delta)
        ep.lokr_delta = delta.data_ptr()
        ep.lokr_scale = float(lscale)
    if residual is not None:
        residual = residual.to(y.dtype).reshape(-1, N).contiguous()
        keep.append(residual)
        ep.residual = residual.data_ptr()
        if gate is not None:
            gate = gate.to(y.dtype).reshape(-1, N).contiguous()
            keep.append(gate)
            ep.gate = gate.data_ptr()
            ep.gate_period = int(gate_period)
    elif gate is not None:
        raise ValueError("a gate needs a residual")
    ep.kernel = kernel
    ep.max_ctas = max_ctas
    if x2.dtype in (torch.float32, torch.float16) and lora is None:
        # f32 / f16 activations: the workspace that lets them run on the tensor cores
        need = int(lib().ql_matmul_workspace_size_x(M, N, K, C.byref(ep), dtype_code(x2)))
        if need:
            if workspace is None or workspace.numel() * workspace.element_size() < need:
                workspace = torch.empty(need, dtype=torch.uint8, device=x.device)
            keep.append(workspace)
            ep.workspace = workspace.data_ptr()
            ep.workspace_bytes = workspace.numel() * workspace.element_size()
    check(lib().ql_quantized_matmul(_ptr(x2), dtype_code(x2), M, K, _ptr(wq.contiguous()),
                                    _ptr(scales.contiguous()), _ptr(biases.contiguous()),
                                    dtype_code(scales), N, group_size, bits, 1, C.byref(ep), _ptr(y),
                                    dtype_code(y), _stream(x.device)))
    return y
