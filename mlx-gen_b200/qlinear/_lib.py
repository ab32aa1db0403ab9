"""ctypes binding of libqlinear.so (the C ABI declared in include/qlinear.h).

This is the Python counterpart of the Rust FFI crate a reference-side
maintainer would add (`qlinear-sys`): raw `extern "C"` signatures, no
logic.  Loading fails loudly when the library has not been built -- there is
no CPU or PyTorch fallback behind it.
"""
from __future__ import annotations

import ctypes as C
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
# QL_LIB_PATH overrides the library location (e.g. an instrumented developer build).
LIB_PATH = os.environ.get("QL_LIB_PATH") or os.path.join(_HERE, "libqlinear.so")

QL_F32, QL_BF16, QL_F16 = 0, 1, 2
QL_OK, QL_EINVAL_SHAPE, QL_EUNSUPPORTED, QL_ECUDA, QL_EINVAL_ARG, QL_ETIMEOUT = range(6)
ACT_NONE, ACT_GELU_TANH, ACT_GELU_ERF, ACT_SWIGLU = range(4)
(KERNEL_AUTO, KERNEL_GENERIC, KERNEL_GEMV, KERNEL_GEMM, KERNEL_GEMM_PAIR, KERNEL_GEMV_TC, KERNEL_GEMV_TMA,
 KERNEL_GEMV_REGS) = range(8)

STATUS_NAMES = {
    QL_OK: "QL_OK",
    QL_EINVAL_SHAPE: "QL_EINVAL_SHAPE",
    QL_EUNSUPPORTED: "QL_EUNSUPPORTED",
    QL_ECUDA: "QL_ECUDA",
    QL_EINVAL_ARG: "QL_EINVAL_ARG",
    QL_ETIMEOUT: "QL_ETIMEOUT",
}

# Every symbol include/qlinear.h declares (tests check the library exports them).
EXPORTS = (
    "ql_version",
    "ql_last_error",
    "ql_device_error",
    "ql_quantize",
    "ql_dequantize",
    "ql_dequantize_rows",
    "ql_layernorm_modulate",
    "ql_quantized_matmul",
    "ql_matmul_workspace_size",
    "ql_quantized_matmul_noalloc",
    "ql_debug_inject",
    "ql_matmul_workspace_size_x",
)


class QlError(RuntimeError):
    """A libqlinear call returned a non-zero ql_status."""

    def __init__(self, status: int, message: str):
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {message}")
        self.status = status


class Epilogue(C.Structure):
    """Mirror of `ql_epilogue`."""

    _fields_ = [
        ("bias", C.c_void_p),
        ("act", C.c_int),
        ("wq_up", C.c_void_p),
        ("scales_up", C.c_void_p),
        ("biases_up", C.c_void_p),
        ("bias_up", C.c_void_p),
        ("lora_a", C.c_void_p),
        ("lora_b", C.c_void_p),
        ("lora_rank", C.c_int64),
        ("lora_scale", C.c_float),
        ("workspace", C.c_void_p),
        ("workspace_bytes", C.c_size_t),
        ("kernel", C.c_int),
        ("max_ctas", C.c_int),
        ("residual", C.c_void_p),
        ("gate", C.c_void_p),
        ("gate_period", C.c_int64),
        ("lokr_delta", C.c_void_p),
        ("lokr_scale", C.c_float),
    ]


_lib = None


def lib():
    """Load libqlinear.so once; raise if it is missing (build it with __graft_entry__.build())."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"libqlinear.so not found at {LIB_PATH}; build it first "
                "(python -c 'import __graft_entry__ as g; g.build()')")
        L = C.CDLL(LIB_PATH)
        vp, i64, i32 = C.c_void_p, C.c_int64, C.c_int
        L.ql_version.restype = i32
        L.ql_last_error.restype = C.c_char_p
        L.ql_device_error.argtypes = [i32]
        L.ql_debug_inject.argtypes = [C.c_uint, C.c_ulonglong]
        L.ql_debug_inject.restype = i32
        L.ql_device_error.restype = i32
        L.ql_quantize.argtypes = [vp, i32, i64, i64, i32, i32, vp, vp, vp, i32, vp]
        L.ql_dequantize.argtypes = [vp, vp, vp, i32, i64, i64, i32, i32, vp, i32, vp]
        L.ql_dequantize_rows.argtypes = [vp, i64, vp, vp, vp, i32, i64, i64, i32, i32, vp, i32, vp]
        L.ql_layernorm_modulate.argtypes = [vp, i64, i64, C.c_float, vp, vp, i64, vp, i32, vp]
        L.ql_quantized_matmul.argtypes = [vp, i32, i64, i64, vp, vp, vp, i32, i64, i32, i32, i32,
                                          C.POINTER(Epilogue), vp, i32, vp]
        L.ql_quantized_matmul_noalloc.argtypes = L.ql_quantized_matmul.argtypes
        L.ql_matmul_workspace_size.argtypes = [i64, i64, i64, C.POINTER(Epilogue)]
        L.ql_matmul_workspace_size.restype = C.c_size_t
        L.ql_matmul_workspace_size_x.argtypes = [i64, i64, i64, C.POINTER(Epilogue), i32]
        L.ql_matmul_workspace_size_x.restype = C.c_size_t
        for f in ("ql_quantize", "ql_dequantize", "ql_dequantize_rows", "ql_layernorm_modulate", "ql_quantized_matmul",
                  "ql_quantized_matmul_noalloc"):
            getattr(L, f).restype = i32
        _lib = L
    return _lib


def check(status: int) -> None:
    if status != QL_OK:
        msg = lib().ql_last_error().decode(errors="replace")
        raise QlError(status, msg)


DEV_ERR_TIMEOUT_FULL, DEV_ERR_TIMEOUT_EMPTY, DEV_ERR_TIMEOUT_ACC, DEV_ERR_BAD_INDEX = 1, 2, 4, 8
INJECT_GEMM_PRODUCER_SILENT = 1


def debug_inject(flags: int = 0, wait_limit_ns: int = 0) -> None:
    """Test hook (ql_debug_inject): shortens every kernel's bounded wait to `wait_limit_ns`
    (0 = the 2 s default) and sets injection flags (INJECT_GEMM_PRODUCER_SILENT: the tcgen05
    GEMM's TMA producer issues nothing, so its consumers' waits run out)."""
    check(lib().ql_debug_inject(int(flags), int(wait_limit_ns)))


def device_error(clear: bool = True) -> int:
    """Device-side error word (bounded-wait timeouts, bad gather ids); 0 = none."""
    return lib().ql_device_error(1 if clear else 0)
