"""Packed-weight helpers, mirroring the reference's src/quant.rs.

``packed_bits`` (src/quant.rs:38-41), ``lin`` (:49-71), ``embedding`` (:75-90) and
``quantize_map`` (:125-149), operating on a ``{name: tensor}`` map (what a
safetensors file holds).  Packed tensors keep the reference's on-disk format:
``{base}.weight`` u32 codes (stored as int32 bit patterns), ``{base}.scales`` and
``{base}.biases`` per group.
"""
from __future__ import annotations

from typing import Callable, Dict

import torch

from . import ops
from .nn import DEFAULT_GROUP_SIZE, AdaptableLinear, TokenEmbedding


class PackedShapeError(ValueError):
    """A packed triple whose shapes do not describe a Q4 or Q8 affine-quantized matrix."""


def packed_bits(wq: torch.Tensor, scales: torch.Tensor, group_size: int) -> int:
    """``bits = wq.cols * 32 / (scales.cols * group_size)``, as src/quant.rs:38-41 infers it,
    but with the shapes checked first: the reference indexes ``shape()[1]`` unchecked and
    divides by a possibly zero ``in_dim``, so a 1-D or zero-width ``scales`` panics there
    (and a non-integral or unsupported width would silently pick a wrong bit count).  Here
    every malformed triple raises ``PackedShapeError``."""
    if group_size not in (32, 64, 128):
        raise PackedShapeError(f"group_size must be 32, 64 or 128 (got {group_size})")
    if wq.dim() != 2 or scales.dim() != 2:
        raise PackedShapeError(f"packed weight and scales must be 2-D (got {tuple(wq.shape)} and "
                               f"{tuple(scales.shape)})")
    if wq.shape[0] != scales.shape[0]:
        raise PackedShapeError(f"packed weight has {wq.shape[0]} rows, scales {scales.shape[0]}")
    in_dim = scales.shape[1] * group_size
    if in_dim == 0 or wq.shape[1] == 0:
        raise PackedShapeError(f"zero-width packed weight or scales ({tuple(wq.shape)}, {tuple(scales.shape)})")
    if (wq.shape[1] * 32) % in_dim:
        raise PackedShapeError(f"{wq.shape[1]} packed words per row do not hold a whole number of bits per "
                               f"code over {in_dim} inputs")
    bits = wq.shape[1] * 32 // in_dim
    if bits not in (4, 8):
        raise PackedShapeError(f"inferred {bits} bits per code; only 4 and 8 are supported")
    return bits


def _require(w: Dict[str, torch.Tensor], key: str) -> torch.Tensor:
    if key not in w:
        raise KeyError(f"missing tensor: {key}")
    return w[key]


def lin(w: Dict[str, torch.Tensor], base: str, bias: bool, group_size: int = DEFAULT_GROUP_SIZE) -> AdaptableLinear:
    """Packed when ``{base}.scales`` exists (bits inferred), dense otherwise."""
    b = _require(w, f"{base}.bias") if bias else None
    scales = w.get(f"{base}.scales")
    if scales is not None:
        wq = _require(w, f"{base}.weight")
        return AdaptableLinear.from_quantized_parts(wq, scales, _require(w, f"{base}.biases"), b, group_size,
                                                    packed_bits(wq, scales, group_size))
    return AdaptableLinear.dense(_require(w, f"{base}.weight"), b)


def embedding(w: Dict[str, torch.Tensor], base: str, group_size: int = DEFAULT_GROUP_SIZE) -> TokenEmbedding:
    scales = w.get(f"{base}.scales")
    if scales is not None:
        wq = _require(w, f"{base}.weight")
        return TokenEmbedding.from_quantized_parts(wq, scales, _require(w, f"{base}.biases"), group_size,
                                                   packed_bits(wq, scales, group_size))
    return TokenEmbedding(_require(w, f"{base}.weight"))


def quantize_map(m: Dict[str, torch.Tensor], bits: int, group_size: int,
                 is_target: Callable[[str], bool]) -> Dict[str, torch.Tensor]:
    """Pack every target 2-D ``{base}.weight`` with ``in % gs == 0 and in >= gs`` (bf16 cast
    first, as src/quant.rs:131-140 does); pass everything else through."""
    out: Dict[str, torch.Tensor] = {}
    for k, v in m.items():
        base = k[: -len(".weight")] if k.endswith(".weight") else None
        ok = (base is not None and is_target(base) and v.dim() == 2 and v.shape[1] % group_size == 0
              and v.shape[1] >= group_size)
        if ok:
            wq, s, b = ops.quantize(v.to(torch.bfloat16), group_size, bits)
            out[f"{base}.weight"], out[f"{base}.scales"], out[f"{base}.biases"] = wq, s, b
        else:
            out[k] = v
    return out
