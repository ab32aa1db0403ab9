"""Regenerate tests/golden/quant_q4q8.npz from the reference's committed fixture.

The reference (SceneWorks/mlx-gen) pins its quant path with
``tests/fixtures/quant_q4q8.safetensors``, produced by ``tools/dump_quant.py`` from
MLX 0.31 (mx.random.seed(0); w f32 [128,256] ~N(0,1); x f32 [4,256] ~N(0,1);
for bits in (8, 4) at group_size 64: wq, scales, biases, deq, qmm) and checked by
``tests/quant_parity.rs:29-66``.  This script copies those tensors, unchanged, into
a numpy archive so the GPU box (which has no reference checkout) can read them.

Usage:  python tests/golden/make_golden.py [path/to/reference]
"""
import os
import sys

import numpy as np
from safetensors.numpy import load_file


def main() -> None:
    ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("QL_REFERENCE")
    if not ref:
        sys.exit("usage: python tests/golden/make_golden.py path/to/reference (or set QL_REFERENCE)")
    src = os.path.join(ref, "tests", "fixtures", "quant_q4q8.safetensors")
    t = load_file(src)
    out = os.path.join(os.path.dirname(os.path.abspath(__file__)), "quant_q4q8.npz")
    np.savez_compressed(out, **{k.replace(".", "_"): v for k, v in t.items()})
    for k in sorted(t):
        print(f"{k}: {t[k].dtype} {t[k].shape}")
    print("wrote", out)


if __name__ == "__main__":
    main()
