"""CPU: the C-ABI library loads, exports every symbol include/qlinear.h declares, and
the ctypes mirror of ql_epilogue has the C layout.  No compute call (no GPU here)."""
import ctypes as C
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "qlinear.h")


def declared():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"^[a-z_ ]+\**\s*\**(ql_\w+)\(", src, flags=re.M)))


def test_header_declarations_match_binding():
    from qlinear import _lib

    assert declared() == sorted(_lib.EXPORTS)


def test_library_exports_every_declared_symbol():
    from qlinear import _lib

    L = _lib.lib()
    for name in declared():
        assert hasattr(L, name), f"libqlinear.so does not export {name}"
    assert L.ql_version() >= 100
    assert L.ql_last_error() == b""


def test_epilogue_layout_matches_c(tmp_path):
    from qlinear._lib import Epilogue

    prog = tmp_path / "layout.c"
    fields = [f[0] for f in Epilogue._fields_]
    body = "\n".join(f'printf("%zu ", offsetof(ql_epilogue, {f}));' for f in fields)
    prog.write_text(f'#include <stddef.h>\n#include <stdio.h>\n#include "{HEADER}"\n'
                    f'int main(void){{ {body} printf("%zu\\n", sizeof(ql_epilogue)); return 0; }}\n')
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-o", str(exe), str(prog)], check=True)
    out = [int(v) for v in subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split()]
    py = [getattr(Epilogue, f).offset for f in fields] + [C.sizeof(Epilogue)]
    assert out == py


def test_validation_errors_need_no_gpu():
    """Argument checks run on the host before any CUDA call."""
    from qlinear import _lib

    L = _lib.lib()
    dummy = C.c_void_p(0x1000)
    rc = L.ql_quantize(dummy, 1, 16, 100, 64, 4, dummy, dummy, dummy, 1, None)  # K % gs != 0
    assert rc == _lib.QL_EINVAL_SHAPE and b"multiple of group_size" in L.ql_last_error()
    rc = L.ql_quantize(dummy, 1, 16, 128, 64, 3, dummy, dummy, dummy, 1, None)  # bits
    assert rc == _lib.QL_EUNSUPPORTED
    rc = L.ql_quantize(dummy, 1, 16, 128, 48, 4, dummy, dummy, dummy, 1, None)  # group size
    assert rc == _lib.QL_EUNSUPPORTED
    rc = L.ql_quantize(None, 1, 16, 128, 64, 4, dummy, dummy, dummy, 1, None)
    assert rc == _lib.QL_EINVAL_ARG
    rc = L.ql_quantize(C.c_void_p(0x1004), 1, 16, 128, 64, 4, dummy, dummy, dummy, 1, None)
    assert rc == _lib.QL_EINVAL_ARG and b"aligned" in L.ql_last_error()
    ep = _lib.Epilogue()
    rc = L.ql_quantized_matmul(dummy, 1, 4, 128, dummy, dummy, dummy, 1, 64, 64, 4, 0, C.byref(ep), dummy, 1, None)
    assert rc == _lib.QL_EUNSUPPORTED  # transpose=false
    ep.act = _lib.ACT_SWIGLU
    rc = L.ql_quantized_matmul(dummy, 1, 4, 128, dummy, dummy, dummy, 1, 64, 64, 4, 1, C.byref(ep), dummy, 1, None)
    assert rc == _lib.QL_EINVAL_ARG  # swiglu without the up projection
    ep = _lib.Epilogue()
    ep.kernel = _lib.KERNEL_GEMM
    rc = L.ql_quantized_matmul(dummy, 0, 4, 128, dummy, dummy, dummy, 0, 64, 64, 4, 1, C.byref(ep), dummy, 0, None)
    assert rc == _lib.QL_EUNSUPPORTED  # tcgen05 kernel needs bf16
    ep = _lib.Epilogue()
    ep.lora_a = 0x1000
    ep.lora_b = 0x1000
    ep.lora_rank = 32
    assert L.ql_matmul_workspace_size(100, 64, 128, C.byref(ep)) == 100 * 64 * 2
    rc = L.ql_quantized_matmul(dummy, 1, 100, 128, dummy, dummy, dummy, 1, 64, 64, 4, 1, C.byref(ep), dummy, 1, None)
    assert rc == _lib.QL_EINVAL_ARG and b"workspace" in L.ql_last_error()
    # M == 0 is a no-op
    assert L.ql_quantized_matmul(dummy, 1, 0, 128, dummy, dummy, dummy, 1, 64, 64, 4, 1, None, dummy, 1, None) == 0
    # gated residual: a gate needs a residual, the period is >= 0
    ep = _lib.Epilogue()
    ep.gate = 0x1000
    rc = L.ql_quantized_matmul(dummy, 1, 4, 128, dummy, dummy, dummy, 1, 64, 64, 4, 1, C.byref(ep), dummy, 1, None)
    assert rc == _lib.QL_EINVAL_ARG and b"residual" in L.ql_last_error()
    ep.residual = 0x1000
    ep.gate_period = -1
    rc = L.ql_quantized_matmul(dummy, 1, 4, 128, dummy, dummy, dummy, 1, 64, 64, 4, 1, C.byref(ep), dummy, 1, None)
    assert rc == _lib.QL_EINVAL_ARG
    # LoKr: not with SwiGLU, not on a GEMV kernel, 16-byte aligned
    ep = _lib.Epilogue()
    ep.lokr_delta = 0x1000
    ep.act = _lib.ACT_SWIGLU
    ep.wq_up = ep.scales_up = ep.biases_up = 0x1000
    rc = L.ql_quantized_matmul(dummy, 1, 4, 128, dummy, dummy, dummy, 1, 64, 64, 4, 1, C.byref(ep), dummy, 1, None)
    assert rc == _lib.QL_EUNSUPPORTED
    ep = _lib.Epilogue()
    ep.lokr_delta = 0x1000
    ep.kernel = _lib.KERNEL_GEMV
    rc = L.ql_quantized_matmul(dummy, 1, 4, 128, dummy, dummy, dummy, 1, 64, 64, 4, 1, C.byref(ep), dummy, 1, None)
    assert rc == _lib.QL_EUNSUPPORTED and b"LoKr" in L.ql_last_error()
    ep.kernel = _lib.KERNEL_AUTO
    ep.lokr_delta = 0x1004
    rc = L.ql_quantized_matmul(dummy, 1, 4, 128, dummy, dummy, dummy, 1, 64, 64, 4, 1, C.byref(ep), dummy, 1, None)
    assert rc == _lib.QL_EINVAL_ARG
    # explicit kernels that cannot take the shape fail instead of falling back
    ep = _lib.Epilogue()
    ep.kernel = _lib.KERNEL_GEMV_TMA
    rc = L.ql_quantized_matmul(dummy, 1, 4, 384, dummy, dummy, dummy, 1, 64, 64, 4, 1, C.byref(ep), dummy, 1, None)
    assert rc == _lib.QL_EUNSUPPORTED
    ep.kernel = 8
    rc = L.ql_quantized_matmul(dummy, 1, 4, 128, dummy, dummy, dummy, 1, 64, 64, 4, 1, C.byref(ep), dummy, 1, None)
    assert rc == _lib.QL_EINVAL_ARG and b"unknown kernel" in L.ql_last_error()
    # layer norm + modulate: D a multiple of 8, bf16 or f32 output, aligned pointers
    rc = L.ql_layernorm_modulate(dummy, 4, 12, 1e-6, None, None, 0, dummy, 1, None)
    assert rc == _lib.QL_EINVAL_SHAPE
    rc = L.ql_layernorm_modulate(dummy, 4, 64, 1e-6, None, None, 0, dummy, 2, None)
    assert rc == _lib.QL_EUNSUPPORTED
    rc = L.ql_layernorm_modulate(dummy, 4, 64, 1e-6, None, None, -1, dummy, 1, None)
    assert rc == _lib.QL_EINVAL_ARG
    assert L.ql_layernorm_modulate(dummy, 0, 64, 1e-6, None, None, 0, dummy, 1, None) == 0


def test_packed_bits_and_lin_dense():
    import torch
    from qlinear import lin, packed_bits

    wq = torch.zeros(8, 128 * 4 // 32, dtype=torch.int32)
    s = torch.zeros(8, 2, dtype=torch.bfloat16)
    assert packed_bits(wq, s, 64) == 4
    assert packed_bits(torch.zeros(8, 32, dtype=torch.int32), s, 64) == 8
    m = {"a.weight": torch.randn(8, 128)}
    al = lin(m, "a", False)
    assert not al.is_quantized() and al.base_shape() == [8, 128]
    with pytest.raises(KeyError):
        lin(m, "a", True)  # missing bias
    q = lin({"a.weight": wq, "a.scales": s, "a.biases": s}, "a", False, 64)
    assert q.is_quantized() and q.quantized_params()[5] == 4 and q.base_shape() == [8, 128]
    with pytest.raises(ValueError):
        q.merge_dense_delta(torch.zeros(8, 128))


@pytest.mark.parametrize("wq_shape,s_shape,gs", [
    ((8, 32), (8,), 64),         # 1-D scales (the reference indexes shape()[1] unchecked)
    ((8, 32), (8, 0), 64),       # zero-width scales (the reference divides by zero)
    ((8, 0), (8, 4), 64),        # zero-width codes
    ((8, 12), (8, 4), 64),       # 6 bits per code
    ((8, 16), (8, 4), 64),       # 2 bits per code
    ((8, 33), (8, 4), 64),       # not a whole number of bits
    ((4, 32), (8, 4), 64),       # row counts differ
    ((8, 32), (8, 4), 48),       # unsupported group size
    ((8,), (8, 4), 64),          # 1-D codes
])
def test_packed_bits_rejects_malformed_shapes(wq_shape, s_shape, gs):
    """Malformed packed triples raise a typed error instead of the reference's panic / a
    wrong bit count (CODE_REVIEW finding F-011 against src/quant.rs:38-41)."""
    import torch
    from qlinear import PackedShapeError, packed_bits

    with pytest.raises(PackedShapeError):
        packed_bits(torch.zeros(wq_shape, dtype=torch.int32), torch.zeros(s_shape, dtype=torch.bfloat16), gs)
    with pytest.raises(ValueError):  # it is a ValueError too
        packed_bits(torch.zeros(wq_shape, dtype=torch.int32), torch.zeros(s_shape, dtype=torch.bfloat16), gs)
