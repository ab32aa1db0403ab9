"""GPU parity: the fused adaLN prologue ``(1 + scale) * layer_norm(x) + shift``
(ql_layernorm_modulate) against the oracle's restatement of mlx fast::layer_norm +
nn::modulate (src/nn.rs:262-287).  The normalised value is rounded to bf16 before the
modulate ops, so a statistics difference in the last fp32 bit can move it by one bf16
ulp: tolerance 2 bf16 ulps element-wise, relative L2 1e-3."""
import numpy as np
import pytest
import torch

import oracle as O
import qlinear
from helpers import np2t, rand_bf16, t2np

pytestmark = pytest.mark.gpu


def _case(M, D, seed):
    rng = np.random.default_rng(seed)
    # per-token offsets and spreads, so the normalisation does real work
    x32 = rng.standard_normal((M, D)) * rng.uniform(0.2, 5.0, (M, 1)) + rng.uniform(-3, 3, (M, 1))
    x = O.to_bf16(x32.astype(np.float32))
    return rng, x


@pytest.mark.parametrize("mode", ["bf16", "f32", "norm_only", "shift_only"])
@pytest.mark.parametrize("period", [0, 150])
def test_layernorm_modulate(dev, mode, period):
    M, D = 300, 3072
    rng, x = _case(M, D, 7 + period)
    rows = 1 if period == 0 else (M + period - 1) // period
    scale = rand_bf16((rows, D), 0.5, rng) if mode in ("bf16", "f32") else None
    shift = rand_bf16((rows, D), 0.5, rng) if mode != "norm_only" else None
    out_dtype = torch.float32 if mode == "f32" else torch.bfloat16
    y = qlinear.layernorm_modulate(np2t(x, dev), None if scale is None else np2t(scale, dev),
                                   None if shift is None else np2t(shift, dev), eps=1e-6, period=period,
                                   out_dtype=out_dtype)
    torch.cuda.synchronize()
    ref = O.layernorm_modulate(x, scale, shift, 1e-6, period, f32_out=(mode == "f32"))
    got = y.cpu().numpy() if mode == "f32" else O.to_f32(t2np(y))
    want = ref if mode == "f32" else O.to_f32(ref)
    # a one-ulp change of the bf16 normalised value n propagates through (1 + scale) and
    # survives the + shift even when the sum cancels: bound by the terms' magnitude
    n = O.to_f32(O.layernorm_modulate(x, None, None, 1e-6, period))
    rws = (np.arange(M) // period) if period else np.zeros(M, np.int64)
    mag = np.abs(n) * (np.abs(1 + O.to_f32(scale).reshape(-1, D)[rws]) if scale is not None else 1.0)
    mag = np.maximum(mag, np.abs(want))
    ulp = 2.0 ** (np.floor(np.log2(np.maximum(mag, 1e-30))) - 7)
    assert np.all(np.abs(got - want) <= 2 * ulp + 1e-6), f"max err {np.abs(got - want).max()}"
    assert np.linalg.norm(got - want) <= 1e-3 * np.linalg.norm(want)


def test_layernorm_modulate_rejects_bad_shapes(dev):
    x = torch.zeros(4, 12, device=dev, dtype=torch.bfloat16)  # D not a multiple of 8
    with pytest.raises(qlinear.QlError):
        qlinear.layernorm_modulate(x)
