"""Load-time adapter delta reconstruction (qlinear.adapters), the input of the fused LoKr
epilogue: LoKr ``scale * kron(w1, w2)`` and LoHa ``scale * (w1_a w1_b) * (w2_a w2_b)``
(src/adapters.rs:25-158), against the oracle's restatement and the reference's own 2x2
known-answer case (src/adapters.rs:695-714).  CPU only."""
import numpy as np
import pytest
import torch

import oracle as O
from qlinear import adapters as A
from helpers import np2t, rand_bf16, t2np


def _bits(t):
    return t2np(t.to(torch.bfloat16))


def test_lokr_known_answer_2x2():
    """reconstruct_lokr_delta(alpha 8, rank 4, [2,2], w1 [[.5],[.6]], w2 [[.7,.8]]) in bf16:
    2 * kron(w1, w2) with the f32 products rounded once."""
    w1 = torch.tensor([[0.5], [0.6]], dtype=torch.float32)
    w2 = torch.tensor([[0.7, 0.8]], dtype=torch.float32)
    d = A.reconstruct_lokr_delta(8.0, 4.0, [2, 2], w1=w1, w2=w2)
    assert d.dtype == torch.bfloat16 and tuple(d.shape) == (2, 2)
    want = O.to_bf16((np.kron(np.float32([[0.5], [0.6]]), np.float32([[0.7, 0.8]])) * np.float32(2.0))
                     .astype(np.float32))
    np.testing.assert_array_equal(_bits(d), want)


@pytest.mark.parametrize("form", ["full", "w1_lowrank", "both_lowrank"])
def test_lokr_matches_oracle(form):
    """bf16 factors in the three linear forms the loaders emit; a [N, K] = [96, 160]
    delta from [8, 10] x [12, 16] factors (rank 4 products)."""
    rng = np.random.default_rng(3)
    a1, b1 = rand_bf16((8, 4), 0.5, rng), rand_bf16((4, 10), 0.5, rng)
    a2, b2 = rand_bf16((12, 4), 0.5, rng), rand_bf16((4, 16), 0.5, rng)
    w1, w2 = rand_bf16((8, 10), 0.5, rng), rand_bf16((12, 16), 0.5, rng)
    t = lambda a: np2t(a, "cpu")
    f = O.bf16_to_f32
    if form == "full":
        d = A.reconstruct_lokr_delta(16.0, 4.0, [96, 160], w1=t(w1), w2=t(w2))
        ref = O.lokr_delta(4.0, (96, 160), f(w1), f(w2))
    elif form == "w1_lowrank":
        d = A.reconstruct_lokr_delta(16.0, 4.0, [96, 160], w1_a=t(a1), w1_b=t(b1), w2=t(w2))
        ref = O.lokr_delta(4.0, (96, 160), (f(a1), f(b1)), f(w2))
    else:
        d = A.reconstruct_lokr_delta(16.0, 4.0, [96, 160], w1_a=t(a1), w1_b=t(b1), w2_a=t(a2), w2_b=t(b2))
        ref = O.lokr_delta(4.0, (96, 160), (f(a1), f(b1)), (f(a2), f(b2)))
    got = _bits(d)
    if form == "full":
        np.testing.assert_array_equal(got, ref)
    else:
        # rank-4 products: the f32 accumulation order may move a rounding by one bf16 ulp
        diff = np.abs(got.astype(np.int32) - ref.astype(np.int32))
        assert diff.max() <= 1 and (diff > 0).mean() < 0.01


def test_lokr_scale_is_f32_and_promotes_bf16_factors():
    """The scale multiplies as an f32 array: a bf16 kron times 1/3 is rounded once to bf16
    from f32, not through a bf16 scale."""
    w1 = torch.tensor([[1.0]], dtype=torch.bfloat16)
    w2 = torch.tensor([[3.0, 5.0]], dtype=torch.bfloat16)
    d = A.reconstruct_lokr_delta_scaled(1.0 / 3.0, [1, 2], w1=w1, w2=w2, out_dtype=torch.float32)
    np.testing.assert_array_equal(d.numpy(), (np.float32([3.0, 5.0]) * np.float32(1.0 / 3.0)).reshape(1, 2))


def test_lokr_trailing_rank_and_tucker():
    """A 2-D w1 against a 4-D conv w2 gets trailing unit dims (make_kron); the tucker
    rebuild is einsum('ijhw,ip,jr->prhw'); a 3-D t2 is refused."""
    g = torch.Generator().manual_seed(0)
    w1 = torch.randn(2, 3, generator=g)
    t2 = torch.randn(4, 5, 3, 3, generator=g)
    wa, wb = torch.randn(4, 6, generator=g), torch.randn(5, 7, generator=g)
    d = A.reconstruct_lokr_delta_scaled(0.5, [12, 21, 3, 3], w1=w1, w2_t2=t2, w2_a=wa, w2_b=wb,
                                        out_dtype=torch.float32)
    f2 = torch.einsum("ijhw,ip,jr->prhw", t2, wa, wb)
    np.testing.assert_allclose(d.numpy(), (torch.kron(w1[:, :, None, None].contiguous(), f2.contiguous()) * 0.5).numpy(), rtol=1e-6)
    with pytest.raises(ValueError, match="4-D"):
        A.reconstruct_lokr_delta_scaled(1.0, [1], w1=w1, w2_t2=t2[0], w2_a=wa, w2_b=wb)
    with pytest.raises(ValueError, match="w1 missing"):
        A.reconstruct_lokr_delta_scaled(1.0, [1], w2=w1)
    with pytest.raises(ValueError, match="w2 missing"):
        A.reconstruct_lokr_delta_scaled(1.0, [1], w1=w1, w2_a=wa)


def test_loha_matches_oracle():
    rng = np.random.default_rng(5)
    a1, b1 = rand_bf16((64, 8), 0.3, rng), rand_bf16((8, 96), 0.3, rng)
    a2, b2 = rand_bf16((64, 8), 0.3, rng), rand_bf16((8, 96), 0.3, rng)
    t = lambda a: np2t(a, "cpu")
    f = O.bf16_to_f32
    d = A.reconstruct_loha_delta(0.25, [64, 96], t(a1), t(b1), t(a2), t(b2))
    ref = O.loha_delta(0.25, (64, 96), (f(a1), f(b1)), (f(a2), f(b2)))
    diff = np.abs(_bits(d).astype(np.int32) - ref.astype(np.int32))
    assert diff.max() <= 1 and (diff > 0).mean() < 0.01


def test_adapter_residual_dtypes_follow_the_reference():
    """Adapter::residual (src/adapters.rs:240-270): LoRA factors keep their dtype, so bf16 x
    with f32 factors gives an f32 residual and an f32 output; bf16 factors stay bf16 with
    the scale rounded to bf16; a LoKr delta is cast to x's dtype."""
    from qlinear import AdaptableLinear, Lokr, Lora
    g = torch.Generator().manual_seed(1)
    x = torch.randn(3, 16, generator=g).to(torch.bfloat16)
    a32, b32 = torch.randn(16, 4, generator=g), torch.randn(4, 8, generator=g) * 0.1
    r = Lora(a32, b32, 0.5).residual(x)
    assert r.dtype == torch.float32
    torch.testing.assert_close(r, ((x.float() @ a32) @ b32) * 0.5, rtol=0, atol=0)
    a16, b16 = a32.to(torch.bfloat16), b32.to(torch.bfloat16)
    r16 = Lora(a16, b16, 0.3).residual(x)
    assert r16.dtype == torch.bfloat16
    assert torch.equal(r16, ((x @ a16) @ b16) * torch.tensor(0.3, dtype=torch.bfloat16))
    w = (torch.randn(8, 16, generator=g) * 0.1).to(torch.bfloat16)
    lin = AdaptableLinear.dense(w)
    lin.push(Lora(a32, b32, 0.5))
    y = lin(x)
    assert y.dtype == torch.float32
    torch.testing.assert_close(y, (x @ w.t()).float() + r, rtol=0, atol=0)
    delta = torch.randn(8, 16, generator=g)
    rk = Lokr(delta, 2.0).residual(x)
    assert rk.dtype == torch.bfloat16
    assert torch.equal(rk, (x @ delta.to(torch.bfloat16).t()) * 2.0)


def _dense_case():
    """The reference's deterministic 64x64 case (src/adapters.rs:840-870)."""
    i = torch.arange(64 * 64, dtype=torch.float32)
    w = (torch.sin(i * 0.013) * 0.05).reshape(64, 64).to(torch.bfloat16)
    bias = (torch.cos(torch.arange(64, dtype=torch.float32) * 0.7) * 0.1).to(torch.bfloat16)
    x = (torch.sin(torch.arange(4 * 64, dtype=torch.float32) * 0.031) * 0.5).reshape(4, 64)
    return w, bias, x


def test_biased_dense_forward_is_fused_addmm():
    """bf16 activations: bit-exact to addmm(bias, x, W^T) and not the double-rounded
    matmul + add; f32 activations: addmm == matmul + add bit for bit."""
    from qlinear import AdaptableLinear
    w, bias, x = _dense_case()
    xb = x.to(torch.bfloat16)
    got = AdaptableLinear.dense(w, bias)(xb)
    assert torch.equal(got, torch.addmm(bias, xb, w.t()))
    assert not torch.equal(got, xb @ w.t() + bias)
    got32 = AdaptableLinear.dense(w, bias)(x)
    assert got32.dtype == torch.float32
    assert torch.equal(got32, x @ w.float().t() + bias.float())


def test_scale_zero_lokr_is_a_bit_exact_noop_and_stacks_sum():
    from qlinear import AdaptableLinear, Lokr, Lora
    w = torch.tensor([[0.1, 0.2], [0.3, 0.4]])
    x = torch.tensor([[1.0, 2.0]])
    lin = AdaptableLinear.dense(w)
    base = lin(x)
    delta = A.reconstruct_lokr_delta(8.0, 4.0, [2, 2], w1=torch.tensor([[0.5], [0.6]]),
                                     w2=torch.tensor([[0.7, 0.8]]))
    lin.push(Lokr(delta, 0.0))
    assert torch.equal(lin(x), base)
    # mixed LoRA + LoKr: the residuals are summed over one base application
    a, b = torch.tensor([[0.5], [-0.25]]), torch.tensor([[1.0, 2.0]])
    lin.set_adapters([Lora(a, b, 0.5), Lokr(delta, 1.0)])
    want = base + ((x @ a) @ b) * 0.5 + x @ delta.float().t()
    assert torch.equal(lin(x), want)


def test_merge_into_a_quantized_base_is_refused():
    """src/adapters.rs:414-426: a LoRA must be merged before quantization."""
    from qlinear import AdaptableLinear
    q = AdaptableLinear.from_quantized_parts(torch.zeros(4, 8, dtype=torch.int32), torch.ones(4, 1),
                                             torch.zeros(4, 1), None, 64, 4)
    with pytest.raises(ValueError, match="quantized"):
        q.merge_dense_delta(torch.zeros(4, 64))
    d = AdaptableLinear.dense(torch.zeros(2, 2))
    d.merge_dense_delta(torch.ones(2, 2))
    assert torch.equal(d.dense_weight()[0], torch.ones(2, 2))
