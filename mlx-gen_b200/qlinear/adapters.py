"""Load-time reconstruction of the dense adapter deltas that the fused LoKr epilogue
consumes (``ql_epilogue.lokr_delta``), mirroring src/adapters.rs:25-158:
``reconstruct_lokr_delta`` (:34-59), ``reconstruct_lokr_delta_scaled`` (:71-101),
``match_trailing_rank`` (:105-112), the LyCORIS tucker rebuild (:117-127) and
``reconstruct_loha_delta`` (:138-158, whose delta the reference installs as a LoKr
residual, src/adapters/loader.rs:397-464).

These run once per adapter file, not per step, so they are torch ops on whatever device
the factors live on.  The rounding points follow the reference's MLX ops: factor
products in the factors' dtype, ``kron`` (or the Hadamard product) in that dtype, the
scale applied as a one-element f32 array (so bf16 factors promote to f32 there), then
one cast to ``out_dtype`` (bf16 on the residual path, src/adapters/loader.rs:176).
"""
from __future__ import annotations

from typing import Optional, Sequence

import torch


def _scale_array(scale: float, like: torch.Tensor) -> torch.Tensor:
    # crate::array::scalar(v) is a shape-[1] f32 array: multiplying by it promotes bf16/f16
    # operands to f32 (an array, not a weak Python scalar).
    return torch.tensor([scale], dtype=torch.float32, device=like.device)


def _match_trailing_rank(a: torch.Tensor, ndim: int) -> torch.Tensor:
    """Append length-1 dims to ``a`` until it has ``ndim`` (LyCORIS ``make_kron``'s
    unsqueeze loop, src/adapters.rs:105-112); a no-op at or above ``ndim``."""
    if a.dim() >= ndim:
        return a
    return a.reshape(*a.shape, *([1] * (ndim - a.dim())))


def _rebuild_tucker(t2: torch.Tensor, wa: torch.Tensor, wb: torch.Tensor) -> torch.Tensor:
    """``einsum("ijhw,ip,jr->prhw")`` (src/adapters.rs:117-127): only the 4-D conv form."""
    if t2.dim() != 4:
        raise ValueError(f"LoKr tucker: expected a 4-D lokr_t2 [in,out,kH,kW], got shape {tuple(t2.shape)}")
    return torch.einsum("ijhw,ip,jr->prhw", t2, wa, wb)


def reconstruct_lokr_delta_scaled(scale: float, base_shape: Sequence[int], w1: Optional[torch.Tensor] = None,
                                  w1_a: Optional[torch.Tensor] = None, w1_b: Optional[torch.Tensor] = None,
                                  w2: Optional[torch.Tensor] = None, w2_t2: Optional[torch.Tensor] = None,
                                  w2_a: Optional[torch.Tensor] = None, w2_b: Optional[torch.Tensor] = None,
                                  out_dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    """``ΔW = scale · kron(factor1, factor2)`` reshaped to ``base_shape`` and cast to
    ``out_dtype`` (src/adapters.rs:71-101).  factor1 is ``w1`` or ``w1_a @ w1_b``;
    factor2 is ``w2``, the tucker rebuild of ``w2_t2, w2_a, w2_b``, or ``w2_a @ w2_b``."""
    if w1 is not None:
        f1 = w1
    elif w1_a is not None and w1_b is not None:
        f1 = w1_a @ w1_b
    else:
        raise ValueError("LoKr: w1 missing (need full w1 or w1_a@w1_b)")
    if w2 is not None:
        f2 = w2
    elif w2_t2 is not None and w2_a is not None and w2_b is not None:
        f2 = _rebuild_tucker(w2_t2, w2_a, w2_b)
    elif w2_a is not None and w2_b is not None:
        f2 = w2_a @ w2_b
    else:
        raise ValueError("LoKr: w2 missing (need full w2, tucker t2+w2_a+w2_b, or w2_a@w2_b)")
    f1 = _match_trailing_rank(f1, f2.dim())
    delta = torch.kron(f1.contiguous(), f2.contiguous()) * _scale_array(scale, f1)
    return delta.reshape(tuple(base_shape)).to(out_dtype)


def reconstruct_lokr_delta(alpha: float, rank: float, base_shape: Sequence[int], w1=None, w1_a=None, w1_b=None,
                           w2=None, w2_a=None, w2_b=None, out_dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    """The SceneWorks/peft LoKr form (src/adapters.rs:34-59): scale ``alpha / rank`` taken
    in f32, no tucker factor."""
    scale = float(torch.tensor(alpha, dtype=torch.float32) / torch.tensor(rank, dtype=torch.float32))
    return reconstruct_lokr_delta_scaled(scale, base_shape, w1, w1_a, w1_b, w2, None, w2_a, w2_b, out_dtype)


def _loha_rebuild_tucker(t: torch.Tensor, w_b: torch.Tensor, w_a: torch.Tensor) -> torch.Tensor:
    """``einsum("ijhw,jr,ip->prhw", t, w_b, w_a)`` (src/adapters.rs:162-171)."""
    if t.dim() != 4:
        raise ValueError(f"LoHa tucker: expected a 4-D hada_t [dim,dim,kH,kW], got shape {tuple(t.shape)}")
    return torch.einsum("ijhw,jr,ip->prhw", t, w_b, w_a)


def reconstruct_loha_delta(scale: float, base_shape: Sequence[int], w1_a: torch.Tensor, w1_b: torch.Tensor,
                           w2_a: torch.Tensor, w2_b: torch.Tensor, t1: Optional[torch.Tensor] = None,
                           t2: Optional[torch.Tensor] = None, out_dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    """``ΔW = scale · ((w1_a @ w1_b) ⊙ (w2_a @ w2_b))`` (tucker rebuilds when both ``t1``
    and ``t2`` are given), reshaped and cast (src/adapters.rs:138-158)."""
    if t1 is not None and t2 is not None:
        m1, m2 = _loha_rebuild_tucker(t1, w1_b, w1_a), _loha_rebuild_tucker(t2, w2_b, w2_a)
    else:
        m1, m2 = w1_a @ w1_b, w2_a @ w2_b
    delta = (m1 * m2) * _scale_array(scale, m1)
    return delta.reshape(tuple(base_shape)).to(out_dtype)
