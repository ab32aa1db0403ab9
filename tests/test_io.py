"""Packed safetensors I/O (qlinear.io), the reference's on-disk format: ``{base}.weight``
U32 codes + ``.scales`` / ``.biases`` (src/quant.rs:92-149, src/weights.rs:13-120).

CPU tests round-trip oracle-packed tensors through files; the GPU test runs the converter
(on-device quantize) and checks it against the oracle bit for bit."""
import os

import numpy as np
import pytest
import torch
from safetensors import safe_open
from safetensors.torch import save_file

import oracle as O
import qlinear
from qlinear import io as qio
from qlinear import quant
from helpers import rand_bf16


def _packed_triple(N=48, K=256, gs=64, bits=4, seed=0):
    rng = np.random.default_rng(seed)
    w = rand_bf16((N, K), 0.02, rng)
    wq, s, b = O.quantize(w, gs, bits)
    t = lambda a: torch.from_numpy(a.view(np.int32) if a.dtype == np.uint32 else a.view(np.int16)).clone()
    return w, {"weight": t(wq), "scales": t(s).view(torch.bfloat16), "biases": t(b).view(torch.bfloat16)}


def test_save_load_round_trip_keeps_u32_on_disk(tmp_path):
    _, tr = _packed_triple()
    m = {f"blk.lin.{k}": v for k, v in tr.items()}
    m["blk.norm.weight"] = torch.ones(8, dtype=torch.bfloat16)
    p = str(tmp_path / "packed.safetensors")
    qio.save_map(p, m, {"note": "x"})
    with safe_open(p, framework="pt") as f:
        assert f.get_slice("blk.lin.weight").get_dtype() == "U32"   # the reference's code dtype
        assert f.get_slice("blk.lin.scales").get_dtype() == "BF16"
        assert f.get_slice("blk.norm.weight").get_dtype() == "BF16"  # dense tensors pass through
        assert f.metadata()["note"] == "x"
    w = qio.Weights.from_file(p)
    for k, v in m.items():
        assert w[k].dtype == v.dtype and torch.equal(w[k], v)
    assert qio.packed_bases(w.tensors) == {"blk.lin.weight"}
    # bits inferred from the shapes (src/quant.rs:38-41), as quant.lin does
    assert quant.packed_bits(w["blk.lin.weight"], w["blk.lin.scales"], 64) == 4


def test_from_dir_merges_shards_and_rejects_duplicates(tmp_path):
    _, tr = _packed_triple(bits=8)
    d = tmp_path / "shards"
    d.mkdir()
    save_file({"a.weight": torch.zeros(2, 2)}, str(d / "model-00001.safetensors"))
    qio.save_map(str(d / "model-00002.safetensors"), {f"b.{k}": v for k, v in tr.items()})
    w = qio.Weights.from_dir(str(d))
    assert set(w.keys()) == {"a.weight", "b.weight", "b.scales", "b.biases"}
    assert quant.packed_bits(w["b.weight"], w["b.scales"], 64) == 8
    save_file({"a.weight": torch.ones(2, 2)}, str(d / "model-00003.safetensors"))
    with pytest.raises(ValueError, match="duplicate tensor key"):
        qio.Weights.from_dir(str(d))
    with pytest.raises(FileNotFoundError):
        qio.Weights.from_dir(str(tmp_path))


@pytest.mark.gpu
def test_convert_matches_oracle_and_loads(tmp_path, dev):
    """The converter packs target 2-D weights (bf16 cast first) byte-identically to the
    oracle, skips non-targets / 1-D / non-divisible weights, and the file loads through
    quant.lin into a working QuantizedLinear."""
    rng = np.random.default_rng(3)
    w32 = (rng.standard_normal((96, 320)) * 0.02).astype(np.float32)   # 320 = 5 groups of 64
    src = {"layers.0.proj.weight": torch.from_numpy(w32), "layers.0.proj.bias": torch.zeros(96),
           "layers.0.norm.weight": torch.ones(320), "head.weight": torch.from_numpy(w32[:, :100].copy()),
           "skip.weight": torch.from_numpy(w32.copy())}
    sp, dp = str(tmp_path / "dense.safetensors"), str(tmp_path / "packed.safetensors")
    save_file(src, sp)
    qio.convert(sp, dp, bits=4, group_size=64, is_target=lambda b: not b.startswith("skip"), device=str(dev))
    w = qio.Weights.from_file(dp, device=str(dev))
    assert qio.packed_bases(w.tensors) == {"layers.0.proj.weight"}
    wbf = O.to_bf16(w32)
    wq, s, b = O.quantize(wbf, 64, 4)
    assert np.array_equal(w["layers.0.proj.weight"].cpu().numpy().view(np.uint32), wq)
    assert np.array_equal(w["layers.0.proj.scales"].cpu().view(torch.int16).numpy().view(np.uint16), s)
    assert np.array_equal(w["layers.0.proj.biases"].cpu().view(torch.int16).numpy().view(np.uint16), b)
    assert w["head.weight"].dtype == torch.float32 and w["skip.weight"].dtype == torch.float32
    lin = quant.lin(w.tensors, "layers.0.proj", bias=True)
    x = torch.randn(3, 320, device=dev).to(torch.bfloat16)
    y = lin.forward(x)
    assert y.shape == (3, 96) and torch.isfinite(y.float()).all()
