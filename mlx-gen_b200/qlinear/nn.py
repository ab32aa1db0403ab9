"""Module-level API of the quantized-linear path, mirroring the reference's
``AdaptableLinear`` / ``LinearBase`` / ``Adapter`` (src/adapters.rs:231-550),
mlx-rs's ``nn::QuantizedLinear`` (constructed at src/adapters.rs:375-384,
533-537) and ``TokenEmbedding`` (src/nn.rs:29-105).

Same names, argument meaning and error behaviour as the reference: quantizing
casts the dense weight and bias to bf16 first (PARITY-BF16,
src/adapters.rs:510-528); the quantized forward feeds activations as-is and adds
the bias after the matmul (src/adapters.rs:300-322); adapters are summed on top
of the base (src/adapters.rs:543-549); merging into a quantized base is an
error (src/adapters.rs:414-426).  The quantized arithmetic runs in libqlinear;
the dense arm (not on the quantized path) uses torch matmuls.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional, Union

import torch

from . import ops
from ._lib import KERNEL_AUTO

DEFAULT_GROUP_SIZE = 64  # src/quant.rs:32


@dataclass
class Linear:
    """Dense ``nn::Linear``: weight ``[out, in]``, optional bias ``[out]``."""

    weight: torch.Tensor
    bias: Optional[torch.Tensor] = None

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        # fused addmm: one rounding of x.W^T + b (src/adapters.rs:286-298), in the promoted
        # dtype of x, W and b (bf16 x against f32 weights computes in f32, as mlx does)
        dt = torch.promote_types(x.dtype, self.weight.dtype)
        if self.bias is not None:
            dt = torch.promote_types(dt, self.bias.dtype)
        w, x = self.weight.to(dt), x.to(dt)
        if self.bias is None:
            return x @ w.t()
        return torch.addmm(self.bias.to(dt), x.reshape(-1, x.shape[-1]), w.t()).reshape(
            *x.shape[:-1], w.shape[0])


@dataclass
class QuantizedLinear:
    """mlx-rs ``nn::QuantizedLinear``: packed ``weight`` (u32 codes), ``scales``,
    ``biases`` (per group), optional dense ``bias``, ``group_size``, ``bits``."""

    weight: torch.Tensor
    scales: torch.Tensor
    biases: torch.Tensor
    bias: Optional[torch.Tensor]
    group_size: int
    bits: int

    @staticmethod
    def try_from_linear(linear: Linear, group_size: int = DEFAULT_GROUP_SIZE,
                        bits: int = 4) -> "QuantizedLinear":
        wq, s, b = ops.quantize(linear.weight, group_size, bits)
        return QuantizedLinear(wq, s, b, linear.bias, group_size, bits)

    @property
    def shape(self):
        """Logical ``[out, in]`` recovered from the scales grid (src/adapters.rs:491-502)."""
        return [self.scales.shape[0], self.scales.shape[1] * self.group_size]

    def forward(self, x: torch.Tensor, *, act: Optional[str] = None, lora=None,
                kernel: int = KERNEL_AUTO, residual: Optional[torch.Tensor] = None,
                gate: Optional[torch.Tensor] = None, gate_period: int = 0, lokr=None) -> torch.Tensor:
        """``residual``/``gate`` fuse the DiT blocks' gated residual ``residual + gate * y``
        (the reference's ``nn::gated``, src/nn.rs:166-176) into the epilogue."""
        return ops.quantized_matmul(x, self.weight, self.scales, self.biases, True, self.group_size,
                                    self.bits, bias=self.bias, act=act, lora=lora, kernel=kernel,
                                    residual=residual, gate=gate, gate_period=gate_period, lokr=lokr)


@dataclass
class Lora:
    """``residual = scale * (x.A).B`` with ``A [in, r]``, ``B [r, out]``
    (src/adapters.rs:231-233; alpha/rank already folded, src/adapters/loader.rs:597)."""

    a: torch.Tensor
    b: torch.Tensor
    scale: float

    def residual(self, x: torch.Tensor) -> torch.Tensor:
        # factors keep their loaded dtype: bf16 x with f32 factors runs (and returns) f32
        # (src/adapters.rs:240-258); the scale is a scalar of the residual's dtype
        dt = torch.promote_types(torch.promote_types(x.dtype, self.a.dtype), self.b.dtype)
        r = (x.to(dt) @ self.a.to(dt)) @ self.b.to(dt)
        return r * torch.tensor(self.scale, dtype=r.dtype, device=r.device)


@dataclass
class Lokr:
    """``residual = scale * x.delta^T`` with ``delta [out, in]`` cast to x's dtype
    (src/adapters.rs:234-235, 263-266)."""

    delta: torch.Tensor
    scale: float

    def residual(self, x: torch.Tensor) -> torch.Tensor:
        r = x @ self.delta.to(x.dtype).t()
        return r * torch.tensor(self.scale, dtype=r.dtype, device=r.device)


Adapter = Union[Lora, Lokr]


class AdaptableLinear:
    """A dense-or-quantized base plus a stack of adapters: ``base(x) + sum residual(x)``."""

    def __init__(self, base: Union[Linear, QuantizedLinear]):
        self.base = base
        self.adapters: List[Adapter] = []

    # ---- constructors (src/adapters.rs:338-385)
    @staticmethod
    def dense(weight: torch.Tensor, bias: Optional[torch.Tensor] = None) -> "AdaptableLinear":
        return AdaptableLinear(Linear(weight, bias))

    @staticmethod
    def from_linear(linear: Linear) -> "AdaptableLinear":
        return AdaptableLinear(linear)

    @staticmethod
    def from_quantized(q: QuantizedLinear) -> "AdaptableLinear":
        return AdaptableLinear(q)

    @staticmethod
    def from_quantized_parts(weight, scales, biases, bias, group_size: int, bits: int) -> "AdaptableLinear":
        return AdaptableLinear(QuantizedLinear(weight, scales, biases, bias, group_size, bits))

    # ---- adapter stack
    def push(self, adapter: Adapter) -> None:
        self.adapters.append(adapter)

    def set_adapters(self, adapters: List[Adapter]) -> None:
        self.adapters = list(adapters)

    def merge_dense_delta(self, delta: torch.Tensor) -> None:
        if isinstance(self.base, QuantizedLinear):
            raise ValueError("merge_dense_delta: base is quantized; a LoRA must be merged before quantization")
        self.base.weight = self.base.weight + delta.to(self.base.weight.dtype)

    # ---- introspection
    def is_quantized(self) -> bool:
        return isinstance(self.base, QuantizedLinear)

    def quantized_params(self):
        if not isinstance(self.base, QuantizedLinear):
            return None
        q = self.base
        return q.weight, q.scales, q.biases, q.bias, q.group_size, q.bits

    def dense_weight(self):
        if isinstance(self.base, QuantizedLinear):
            return None
        return self.base.weight, self.base.bias

    def base_shape(self):
        if isinstance(self.base, QuantizedLinear):
            return self.base.shape
        return list(self.base.weight.shape)

    # ---- quantize in place (src/adapters.rs:508-541)
    def quantize(self, bits: int, group_size: Optional[int] = None) -> None:
        if isinstance(self.base, QuantizedLinear):
            return
        w = self.base.weight.to(torch.bfloat16)  # PARITY-BF16
        b = None if self.base.bias is None else self.base.bias.to(torch.bfloat16)
        self.base = QuantizedLinear.try_from_linear(Linear(w, b), group_size or DEFAULT_GROUP_SIZE, bits)

    # ---- forward (src/adapters.rs:543-549)
    def forward(self, x: torch.Tensor) -> torch.Tensor:
        """``base(x) + sum residual(x)``.  A quantized base with bf16 activations and at
        most one LoRA (bf16 factors) plus at most one LoKr adapter runs as ONE fused kernel
        (the LoRA residual accumulates into the same fp32 tile, the LoKr delta is added to
        the dequantized weights); any other stack adds the residuals separately, with the
        reference's dtype promotion (f32 factors make the output f32)."""
        loras = [a for a in self.adapters if isinstance(a, Lora)]
        lokrs = [a for a in self.adapters if isinstance(a, Lokr)]
        # f32 LoRA factors promote the reference's output to f32: that stack is not fused
        if (isinstance(self.base, QuantizedLinear) and x.dtype == torch.bfloat16
                and self.base.scales.dtype == torch.bfloat16 and self.adapters
                and len(loras) <= 1 and len(lokrs) <= 1
                and all(l.a.dtype == torch.bfloat16 and l.b.dtype == torch.bfloat16 for l in loras)):
            lo = (loras[0].a, loras[0].b, loras[0].scale) if loras else None
            lk = (lokrs[0].delta, lokrs[0].scale) if lokrs else None
            return self.base.forward(x, lora=lo, lokr=lk)
        out = self.base.forward(x)
        for ad in self.adapters:
            out = out + ad.residual(x)
        return out

    __call__ = forward


class TokenEmbedding:
    """Dense or quantized token table; ``forward(ids) -> [*ids, hidden]`` in f32
    (src/nn.rs:29-59)."""

    def __init__(self, dense: Optional[torch.Tensor] = None, *, wq=None, scales=None, biases=None,
                 group_size: int = DEFAULT_GROUP_SIZE, bits: int = 4):
        self.dense = dense
        self.wq, self.scales, self.biases = wq, scales, biases
        self.group_size, self.bits = group_size, bits

    @staticmethod
    def from_quantized_parts(wq, scales, biases, group_size: int, bits: int) -> "TokenEmbedding":
        return TokenEmbedding(None, wq=wq, scales=scales, biases=biases, group_size=group_size, bits=bits)

    def is_quantized(self) -> bool:
        return self.wq is not None

    def quantize(self, bits: int, cast_to_bf16: bool) -> None:
        """Quantize in place at group size 64 (src/nn.rs:88-104)."""
        if self.wq is not None:
            return
        w = self.dense.to(torch.bfloat16) if cast_to_bf16 else self.dense
        self.wq, self.scales, self.biases = ops.quantize(w, 64, bits)
        self.group_size, self.bits, self.dense = 64, bits, None

    def forward(self, ids: torch.Tensor) -> torch.Tensor:
        if self.wq is None:
            return self.dense[ids].to(torch.float32)
        return ops.dequantize_rows(ids, self.wq, self.scales, self.biases, self.group_size, self.bits,
                                   out_dtype=torch.float32)

    __call__ = forward
