"""Packed safetensors I/O and the offline pre-quantization converter, mirroring the
reference's weight loading (src/weights.rs:13-120) and converter plumbing
(src/quant.rs:92-149: ``load_dir_map``, ``save_map``, ``quantize_map``).

On disk a packed linear is the reference's triple ``{base}.weight`` (U32 codes),
``{base}.scales`` and ``{base}.biases`` (bf16), so snapshots written by the reference load
unchanged and files written here load in the reference.  In memory the codes are int32
tensors holding the same bits (torch's kernels and the C ABI take them as 32-bit words).

    python -m qlinear.io convert SRC DST [--bits 4] [--group-size 64] [--target REGEX]

quantizes every target 2-D ``*.weight`` of the safetensors file or directory SRC on the
GPU (``ql_quantize``) and writes one packed file DST.
"""
from __future__ import annotations

import argparse
import os
import re
from typing import Callable, Dict, Iterable, Optional

import torch
from safetensors import safe_open
from safetensors.torch import save_file

from .nn import DEFAULT_GROUP_SIZE


def _to_memory(t: torch.Tensor) -> torch.Tensor:
    """U32 codes -> int32 with the same bits (what the kernels take)."""
    return t.view(torch.int32) if t.dtype == torch.uint32 else t


def _to_disk(key: str, t: torch.Tensor, packed: set) -> torch.Tensor:
    t = t.detach().contiguous().cpu()
    if key in packed and t.dtype == torch.int32:
        return t.view(torch.uint32)  # the reference's on-disk dtype for codes
    return t


class Weights:
    """Named tensors (dotted keys) plus the file's string metadata (src/weights.rs:13-17)."""

    def __init__(self, tensors: Optional[Dict[str, torch.Tensor]] = None,
                 metadata: Optional[Dict[str, str]] = None):
        self.tensors: Dict[str, torch.Tensor] = dict(tensors or {})
        self.metadata: Dict[str, str] = dict(metadata or {})

    @staticmethod
    def from_file(path: str, device: str | torch.device = "cpu") -> "Weights":
        tensors = {}
        with safe_open(path, framework="pt", device=str(device)) as f:
            meta = f.metadata() or {}
            for k in f.keys():
                tensors[k] = _to_memory(f.get_tensor(k))
        return Weights(tensors, meta)

    @staticmethod
    def from_dir(path: str, device: str | torch.device = "cpu") -> "Weights":
        """Merge every ``*.safetensors`` under ``path`` (sorted); shards must be disjoint
        (a repeated key is an error, as src/weights.rs:50-62 makes it)."""
        files = sorted(os.path.join(path, f) for f in os.listdir(path) if f.endswith(".safetensors"))
        if not files:
            raise FileNotFoundError(f"no .safetensors files in {path}")
        out = Weights()
        for fp in files:
            w = Weights.from_file(fp, device)
            for k, v in w.tensors.items():
                if k in out.tensors:
                    raise ValueError(f"duplicate tensor key `{k}` across shards in {path} (non-disjoint shard set)")
                out.tensors[k] = v
            out.metadata.update(w.metadata)
        return out

    @staticmethod
    def load(path: str, device: str | torch.device = "cpu") -> "Weights":
        return Weights.from_dir(path, device) if os.path.isdir(path) else Weights.from_file(path, device)

    def get(self, key: str) -> Optional[torch.Tensor]:
        return self.tensors.get(key)

    def keys(self) -> Iterable[str]:
        return self.tensors.keys()

    def __contains__(self, key: str) -> bool:
        return key in self.tensors

    def __getitem__(self, key: str) -> torch.Tensor:
        if key not in self.tensors:
            raise KeyError(f"missing tensor: {key}")
        return self.tensors[key]


def packed_bases(m: Dict[str, torch.Tensor]) -> set:
    """Keys ``{base}.weight`` that hold packed codes (a ``{base}.scales`` exists)."""
    return {k for k in m if k.endswith(".weight") and f"{k[:-len('.weight')]}.scales" in m}


def load_dir_map(path: str, device: str | torch.device = "cpu") -> Dict[str, torch.Tensor]:
    """Every tensor of a file or (sharded) directory as a key -> tensor map."""
    return dict(Weights.load(path, device).tensors)


def save_map(path: str, m: Dict[str, torch.Tensor], metadata: Optional[Dict[str, str]] = None) -> None:
    """Write one safetensors file; packed codes are stored as U32 (src/quant.rs:104-117)."""
    packed = packed_bases(m)
    parent = os.path.dirname(os.path.abspath(path))
    os.makedirs(parent, exist_ok=True)
    save_file({k: _to_disk(k, v, packed) for k, v in m.items()}, path, metadata=metadata)


def convert(src: str, dst: str, bits: int = 4, group_size: int = DEFAULT_GROUP_SIZE,
            is_target: Callable[[str], bool] = lambda base: True,
            device: str | torch.device = "cuda") -> Dict[str, torch.Tensor]:
    """Load SRC, pack every target linear on the GPU (``quant.quantize_map``) and save DST."""
    from .quant import quantize_map

    w = Weights.load(src, device)
    out = quantize_map(w.tensors, bits, group_size, is_target)
    meta = dict(w.metadata)
    meta.update({"quantization_bits": str(bits), "quantization_group_size": str(group_size)})
    save_map(dst, out, meta)
    return out


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="python -m qlinear.io", description=__doc__.split("\n\n")[0])
    sub = ap.add_subparsers(dest="cmd", required=True)
    c = sub.add_parser("convert", help="pack the linears of a safetensors file or directory")
    c.add_argument("src")
    c.add_argument("dst")
    c.add_argument("--bits", type=int, default=4, choices=(4, 8))
    c.add_argument("--group-size", type=int, default=DEFAULT_GROUP_SIZE, choices=(32, 64, 128))
    c.add_argument("--target", default=None, help="regex on the key minus '.weight' (default: every 2-D weight)")
    a = ap.parse_args(argv)
    rx = re.compile(a.target) if a.target else None
    out = convert(a.src, a.dst, a.bits, a.group_size, (lambda b: bool(rx.search(b))) if rx else (lambda b: True))
    n = len(packed_bases(out))
    print(f"wrote {a.dst}: {len(out)} tensors, {n} packed linears (Q{a.bits}, group {a.group_size})")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
