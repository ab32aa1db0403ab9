"""Shared test helpers: bf16 <-> numpy conversion and the stated tolerances."""
import numpy as np
import torch

import oracle as O


def t2np(t: torch.Tensor) -> np.ndarray:
    """torch tensor (any device) -> numpy; bf16 as uint16 bits, int32 codes as uint32."""
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    if t.dtype == torch.int32:
        return t.numpy().view(np.uint32)
    return t.numpy()


def np2t(a: np.ndarray, device) -> torch.Tensor:
    """numpy -> torch on device; uint16 is read as bf16 bits, uint32 as int32 codes."""
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint16:
        return torch.from_numpy(a.view(np.int16).copy()).view(torch.bfloat16).to(device)
    if a.dtype == np.uint32:
        return torch.from_numpy(a.view(np.int32).copy()).to(device)
    return torch.from_numpy(a.copy()).to(device)


def f32(a: np.ndarray) -> np.ndarray:
    return O.to_f32(a)


def rand_bf16(shape, std, rng) -> np.ndarray:
    return O.to_bf16((rng.standard_normal(shape) * std).astype(np.float32))


# Stated matmul tolerance (bf16 output, fp32 accumulation on both sides; the oracle
# accumulates in fp64):  |y - y_ref| <= ULPS * ulp_bf16(|y_ref|) + ATOL_FRAC * max|y_ref|
# element-wise, and relative L2 error <= RL2.
def assert_bf16_close(got: np.ndarray, ref: np.ndarray, ulps: float = 2.0, atol_frac: float = 2e-3,
                      rl2: float = 4e-3, what: str = ""):
    got = got.astype(np.float64)
    ref = ref.astype(np.float64)
    assert got.shape == ref.shape, (got.shape, ref.shape)
    scale = np.abs(ref).max() if ref.size else 0.0
    ulp = np.exp2(np.floor(np.log2(np.maximum(np.abs(ref), 1e-30))) - 7)
    err = np.abs(got - ref)
    bound = ulps * ulp + atol_frac * scale
    bad = err > bound
    assert not bad.any(), (f"{what}: {bad.sum()} / {bad.size} elements out of tolerance; "
                           f"worst err {err.max():.3e} (scale {scale:.3e})")
    denom = np.linalg.norm(ref)
    if denom > 0:
        r = np.linalg.norm(got - ref) / denom
        assert r <= rl2, f"{what}: relative L2 {r:.3e} > {rl2}"
