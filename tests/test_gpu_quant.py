"""GPU parity: quantize / dequantize / dequantize_rows through the C ABI against the
oracle, bit-exact (the reference's tests/quant_parity.rs:29-57 checked byte-level)."""
import numpy as np
import pytest
import torch

import oracle as O
import qlinear
from helpers import np2t, rand_bf16, t2np

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("bits", [8, 4])
def test_fixture_quantize_dequantize_bit_exact(golden, dev, bits):
    w = np2t(golden["w"], dev)
    wq, s, b = qlinear.quantize(w, 64, bits)
    p = f"q{bits}_"
    assert np.array_equal(t2np(wq), golden[p + "wq"])
    assert np.array_equal(t2np(s), golden[p + "scales"])
    assert np.array_equal(t2np(b), golden[p + "biases"])
    d = qlinear.dequantize(wq, s, b, 64, bits)
    assert np.array_equal(t2np(d), golden[p + "deq"])


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("gs", [32, 64, 128])
@pytest.mark.parametrize("shape", [(1, 128), (37, 384), (256, 1024)])
def test_quantize_bf16_bit_exact(dev, bits, gs, shape):
    rng = np.random.default_rng(hash((bits, gs, shape)) % 2**32)
    w = rand_bf16(shape, 0.02, rng)
    wq, s, b = qlinear.quantize(np2t(w, dev), gs, bits)
    rq, rs, rb = O.quantize(w, gs, bits)
    assert np.array_equal(t2np(wq), rq)
    assert np.array_equal(t2np(s), rs)
    assert np.array_equal(t2np(b), rb)
    for od, odt in ((O.BF16, torch.bfloat16), (O.F32, torch.float32), (O.F16, torch.float16)):
        d = qlinear.dequantize(wq, s, b, gs, bits, out_dtype=odt)
        assert np.array_equal(t2np(d).view(np.uint16 if odt != torch.float32 else np.float32),
                              O.dequantize(rq, rs, rb, gs, bits, out_dtype=od).view(
                                  np.uint16 if odt != torch.float32 else np.float32))


@pytest.mark.parametrize("bits", [4, 8])
def test_quantize_edge_values(dev, bits):
    """Constant / zero / one-sided / huge / tiny groups, f32 and f16 inputs."""
    rng = np.random.default_rng(7)
    w = (rng.standard_normal((8, 256)) * 0.02).astype(np.float32)
    w[0] = 0.0
    w[1] = 0.75
    w[2] = -2.5
    w[3] = np.abs(w[3]) + 1.0
    w[4] *= 1e4
    w[5] *= 1e-30
    w[6, ::2] = 0.0
    w[7, :64] = np.linspace(-1, 1, 64)
    for arr in (w, w.astype(np.float16)):
        wq, s, b = qlinear.quantize(np2t(arr, dev), 64, bits)
        rq, rs, rb = O.quantize(arr, 64, bits)
        assert np.array_equal(t2np(wq), rq)
        assert np.array_equal(t2np(s).view(np.uint8), rs.view(np.uint8))
        assert np.array_equal(t2np(b).view(np.uint8), rb.view(np.uint8))


@pytest.mark.parametrize("bits", [4, 8])
def test_dequantize_rows_gather(dev, bits):
    """Quantized embedding gather (src/nn.rs:42-59): f32 rows, ids of any shape; values
    are dequantized in the scales' dtype (bf16) and then widened, as the reference's
    dequantize + cast, so every f32 output is bf16-representable."""
    rng = np.random.default_rng(11)
    w = rand_bf16((500, 256), 0.02, rng)
    wq, s, b = qlinear.quantize(np2t(w, dev), 64, bits)
    ids = rng.integers(0, 500, size=(3, 7))
    got = qlinear.dequantize_rows(torch.from_numpy(ids).to(dev), wq, s, b, 64, bits)
    ref = O.dequantize(t2np(wq), t2np(s), t2np(b), 64, bits, ids=ids, out_dtype=O.F32)
    assert got.shape == (3, 7, 256)
    assert np.array_equal(t2np(got).reshape(-1, 256), ref)
    assert np.array_equal(O.bf16_to_f32(O.to_bf16(ref)), ref)
    emb = qlinear.TokenEmbedding(np2t(w, dev))
    emb.quantize(bits, cast_to_bf16=True)
    assert np.array_equal(t2np(emb(torch.from_numpy(ids).to(dev))).reshape(-1, 256), ref)


def test_dequantize_rows_bad_id_sets_error(dev):
    w = torch.randn(16, 128, device=dev, dtype=torch.bfloat16)
    wq, s, b = qlinear.quantize(w, 64, 4)
    qlinear.device_error(clear=True)
    out = qlinear.dequantize_rows(torch.tensor([0, 99], device=dev), wq, s, b, 64, 4)
    assert qlinear.device_error(clear=True) != 0
    assert torch.all(out[1] == 0)


def test_quantize_full_size_roundtrip(dev):
    """Full Wan2.2 FFN shape [13824, 5120]: the dequant error stays within one step, and
    re-quantizing the dequantized weights moves no value by more than one (new) step
    (size-independent properties); sampled rows are bit-exact against the oracle."""
    g = torch.Generator(device=dev).manual_seed(0)
    w = (torch.randn(13824, 5120, device=dev, generator=g) * 0.02).to(torch.bfloat16)
    for bits in (4, 8):
        wq, s, b = qlinear.quantize(w, 64, bits)
        d = qlinear.dequantize(wq, s, b, 64, bits)
        step = s.float().abs().repeat_interleave(64, dim=1)
        # one step, plus the bf16 rounding of the stored scale (codes use the fp32 scale) times
        # the largest code, plus the bf16 rounding of the output
        slack = 1.001 + (2 ** bits) * 2 ** -8
        assert torch.all((d.float() - w.float()).abs() <= step * slack + w.float().abs() * 2 ** -7)
        wq2, s2, b2 = qlinear.quantize(d, 64, bits)
        d2 = qlinear.dequantize(wq2, s2, b2, 64, bits)
        step2 = s2.float().abs().repeat_interleave(64, dim=1)
        assert torch.all((d2.float() - d.float()).abs() <= step2 * slack + d.float().abs() * 2 ** -7)
        # sampled rows bit-exact against the oracle at full K
        rows = [0, 4095, 13823]
        rq, rs, rb = O.quantize(t2np(w[rows]), 64, bits)
        assert np.array_equal(t2np(wq[rows]), rq) and np.array_equal(t2np(s[rows]), rs)
