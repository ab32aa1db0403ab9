"""CPU: the oracle (oracle/qref.c) against the reference's golden fixture.

The fixture is the reference's tests/fixtures/quant_q4q8.safetensors (MLX 0.31,
tools/dump_quant.py), copied unchanged into tests/golden/quant_q4q8.npz.  The
assertions mirror tests/quant_parity.rs:29-66 but tighter: codes, scales, biases
and dequant are checked bit-exactly.
"""
import numpy as np
import pytest

import oracle as O
from helpers import rand_bf16


@pytest.mark.parametrize("bits", [8, 4])
def test_quantize_bit_exact_vs_fixture(golden, bits):
    wq, s, b = O.quantize(golden["w"], 64, bits)
    p = f"q{bits}_"
    assert np.array_equal(wq, golden[p + "wq"])
    assert np.array_equal(s, golden[p + "scales"])
    assert np.array_equal(b, golden[p + "biases"])


@pytest.mark.parametrize("bits", [8, 4])
def test_dequantize_bit_exact_vs_fixture(golden, bits):
    p = f"q{bits}_"
    d = O.dequantize(golden[p + "wq"], golden[p + "scales"], golden[p + "biases"], 64, bits)
    assert np.array_equal(d, golden[p + "deq"])


@pytest.mark.parametrize("bits", [8, 4])
def test_qmm_vs_fixture(golden, bits):
    p = f"q{bits}_"
    y = O.quantized_matmul(golden["x"], golden[p + "wq"], golden[p + "scales"], golden[p + "biases"], 64, bits)
    # reference gate: allclose(rtol=1e-2, atol=1e-2) (tests/quant_parity.rs:59-64); the oracle is far inside it
    np.testing.assert_allclose(y, golden[p + "qmm"], rtol=1e-5, atol=1e-4)
    yf = O.quantized_matmul_fast(golden["x"], golden[p + "wq"], golden[p + "scales"], golden[p + "biases"], 64, bits)
    np.testing.assert_allclose(yf, golden[p + "qmm"], rtol=1e-5, atol=1e-4)


def test_fixture_discriminates_naive_affine(golden):
    """A naive scale=(max-min)/n, bias=min quantizer must NOT match (the fixture pins the
    zero-point-exact variant)."""
    w = golden["w"].reshape(128, 4, 64)
    mn, mx = w.min(-1), w.max(-1)
    assert not np.allclose((mx - mn) / 15, golden["q4_scales"])


@pytest.mark.parametrize("bits,gs", [(4, 32), (4, 64), (4, 128), (8, 32), (8, 64), (8, 128)])
def test_oracle_bf16_properties(bits, gs):
    """bf16 input: codes in range, dequant error within one step (+ bf16 rounding)."""
    rng = np.random.default_rng(bits * 1000 + gs)
    w = rand_bf16((64, 512), 0.02, rng)
    wq, s, b = O.quantize(w, gs, bits)
    assert s.dtype == np.uint16 and b.dtype == np.uint16
    d = O.to_f32(O.dequantize(wq, s, b, gs, bits))
    wf = O.to_f32(w)
    step = np.abs(O.to_f32(s)).repeat(gs, axis=1)
    # the zero-point shift (bias = edge) can push the far end of a group to one full step
    assert (np.abs(d - wf) <= step * 1.001 + np.abs(wf) * 2 ** -7 + 1e-6).all()


def test_oracle_degenerate_groups():
    """Constant, zero and one-sided groups exercise the eps and q0 == 0 branches."""
    w = np.zeros((4, 64), np.float32)
    w[1] = 0.5                       # constant positive
    w[2] = -3.0                      # constant negative
    w[3] = np.linspace(0.1, 0.9, 64)  # all positive, q0 != 0
    for bits in (4, 8):
        wq, s, b = O.quantize(w, 64, bits)
        d = O.dequantize(wq, s, b, 64, bits)
        np.testing.assert_allclose(d, w, atol=np.abs(s).max() * 1.001 + 1e-6)


def test_oracle_epilogue_helpers_follow_the_reference_rounding():
    """gated / lokr_residual / layernorm_modulate restate the reference's op sequences
    (each op rounded to bf16): checked here against a step-by-step float32 evaluation."""
    rng = np.random.default_rng(11)
    bf = lambda a: O.to_bf16(np.asarray(a, np.float32))
    f = O.bf16_to_f32
    M, N, K = 6, 40, 64
    res, gate, y = bf(rng.standard_normal((M, N))), bf(rng.standard_normal((2, N))), bf(rng.standard_normal((M, N)))
    out = O.gated(res, gate, y, period=3)
    rows = np.arange(M) // 3
    want = bf(f(res) + f(bf(f(gate)[rows] * f(y))))
    assert np.array_equal(out, want)
    assert np.array_equal(O.gated(res, None, y), bf(f(res) + f(y)))
    x, d = bf(rng.standard_normal((M, K))), bf(rng.standard_normal((N, K)) * 0.1)
    r = O.lokr_residual(x, d, 0.3)
    want = bf(f(bf(f(x).astype(np.float64) @ f(d).astype(np.float64).T)) * f(bf([0.3]))[0])
    assert np.array_equal(r, want)
    xs = bf(rng.standard_normal((M, 64)) * 3 + 1)
    sc, sh = bf(rng.standard_normal(64) * 0.2), bf(rng.standard_normal(64) * 0.2)
    n = O.layernorm_modulate(xs)
    xf = f(xs).astype(np.float64)
    z = (xf - xf.mean(1, keepdims=True)) / np.sqrt(xf.var(1, keepdims=True) + 1e-6)
    assert np.array_equal(n, bf(z))
    m = O.layernorm_modulate(xs, sc, sh)
    assert np.array_equal(m, bf(f(bf(f(n) * f(bf(f(sc) + 1.0)))) + f(sh)))
    m32 = O.layernorm_modulate(xs, sc, sh, f32_out=True)
    assert np.allclose(m32, f(n) * (f(sc) + 1.0) + f(sh), rtol=0, atol=1e-6)
