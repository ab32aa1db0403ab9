"""Megatron-style tensor parallelism on packed Q4/Q8 weights.

The reference is single-device (gen-core/src/runtime.rs:56-59); this module is new.
Column-parallel linears (QKV, MLP up) split W's output rows: each packed row is
self-contained, so a rank keeps rows [r*N/P, (r+1)*N/P) of wq, scales and biases
and its output shard needs no communication.  Row-parallel linears (attention
out, MLP down) split K on group boundaries: a rank keeps words
[K0*bits/32, K1*bits/32) and groups [K0/gs, K1/gs) of every row, produces a
partial [M, N] sum, and one all-reduce (NCCL over NVLink) completes it; the
dense bias is added once, after the reduction.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch


def column_shard(wq: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor,
                 bias: Optional[torch.Tensor], rank: int, world: int):
    N = scales.shape[0]
    if N % world:
        raise ValueError(f"column-parallel split needs N % world == 0 (N={N}, world={world})")
    n0, n1 = rank * N // world, (rank + 1) * N // world
    return (wq[n0:n1].contiguous(), scales[n0:n1].contiguous(), biases[n0:n1].contiguous(),
            None if bias is None else bias[n0:n1].contiguous())


def row_shard(wq: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor, group_size: int, bits: int,
              rank: int, world: int) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor, int, int]:
    """Split K into `world` group-aligned slices; returns (wq, scales, biases, k0, k1)."""
    G = scales.shape[1]
    K = G * group_size
    if G % world:
        raise ValueError(f"row-parallel split must fall on group boundaries (K={K}, gs={group_size}, world={world})")
    g0, g1 = rank * G // world, (rank + 1) * G // world
    k0, k1 = g0 * group_size, g1 * group_size
    w0, w1 = k0 * bits // 32, k1 * bits // 32
    return (wq[:, w0:w1].contiguous(), scales[:, g0:g1].contiguous(), biases[:, g0:g1].contiguous(), k0, k1)
