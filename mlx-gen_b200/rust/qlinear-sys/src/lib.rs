//! Raw bindings of the C ABI in `include/qlinear.h` -- one `extern "C"` item per entry
//! point, the `ql_epilogue` struct with the same field order, and the enum values as
//! constants.  No logic: the safe layer is the `qlinear` crate beside this one.
//!
//! What each entry point replaces in the reference (mlx-gen):
//! - `ql_quantize`: `mlx_rs::ops::quantize` via `QuantizedLinear::try_from_linear`
//!   (src/quant.rs:140, src/adapters.rs:533-537, src/nn.rs:91-93).
//! - `ql_dequantize`: `mlx_rs::ops::dequantize` (src/nn.rs:55).
//! - `ql_dequantize_rows`: the quantized `TokenEmbedding` gather (src/nn.rs:42-59).
//! - `ql_quantized_matmul`: `quantized_matmul(x, wq, scales, biases, true, gs, bits)` plus
//!   bias in `LinearBase::forward` (src/adapters.rs:300-322) and the adapter residuals of
//!   `AdaptableLinear::forward` (src/adapters.rs:543-549).
//! - `ql_layernorm_modulate`: `fast::layer_norm` + `nn::modulate`
//!   (mlx-gen-flux/src/transformer.rs:891-913, src/nn.rs:262-287).
#![allow(non_camel_case_types)]

use std::os::raw::{c_char, c_int, c_uint, c_ulonglong, c_void};

pub type ql_dtype = c_int;
pub const QL_F32: ql_dtype = 0;
pub const QL_BF16: ql_dtype = 1;
pub const QL_F16: ql_dtype = 2;

pub type ql_status = c_int;
pub const QL_OK: ql_status = 0;
pub const QL_EINVAL_SHAPE: ql_status = 1;
pub const QL_EUNSUPPORTED: ql_status = 2;
pub const QL_ECUDA: ql_status = 3;
pub const QL_EINVAL_ARG: ql_status = 4;
pub const QL_ETIMEOUT: ql_status = 5;

pub type ql_act = c_int;
pub const QL_ACT_NONE: ql_act = 0;
pub const QL_ACT_GELU_TANH: ql_act = 1;
pub const QL_ACT_GELU_ERF: ql_act = 2;
pub const QL_ACT_SWIGLU: ql_act = 3;

pub type ql_kernel = c_int;
pub const QL_KERNEL_AUTO: ql_kernel = 0;
pub const QL_KERNEL_GENERIC: ql_kernel = 1;
pub const QL_KERNEL_GEMV: ql_kernel = 2;
pub const QL_KERNEL_GEMM: ql_kernel = 3;
pub const QL_KERNEL_GEMM_PAIR: ql_kernel = 4;
pub const QL_KERNEL_GEMV_TC: ql_kernel = 5;
pub const QL_KERNEL_GEMV_TMA: ql_kernel = 6;
pub const QL_KERNEL_GEMV_REGS: ql_kernel = 7;

/// Mirror of `ql_epilogue`: the ops fused into one `ql_quantized_matmul` call.  All
/// pointers are device pointers; NULL turns the corresponding op off.
#[repr(C)]
#[derive(Debug, Clone, Copy)]
pub struct ql_epilogue {
    pub bias: *const c_void,
    pub act: c_int,
    pub wq_up: *const u32,
    pub scales_up: *const c_void,
    pub biases_up: *const c_void,
    pub bias_up: *const c_void,
    pub lora_a: *const c_void,
    pub lora_b: *const c_void,
    pub lora_rank: i64,
    pub lora_scale: f32,
    pub workspace: *mut c_void,
    pub workspace_bytes: usize,
    pub kernel: c_int,
    pub max_ctas: c_int,
    pub residual: *const c_void,
    pub gate: *const c_void,
    pub gate_period: i64,
    pub lokr_delta: *const c_void,
    pub lokr_scale: f32,
}

impl Default for ql_epilogue {
    fn default() -> Self {
        use std::ptr::{null, null_mut};
        ql_epilogue {
            bias: null(),
            act: QL_ACT_NONE,
            wq_up: null(),
            scales_up: null(),
            biases_up: null(),
            bias_up: null(),
            lora_a: null(),
            lora_b: null(),
            lora_rank: 0,
            lora_scale: 0.0,
            workspace: null_mut(),
            workspace_bytes: 0,
            kernel: QL_KERNEL_AUTO,
            max_ctas: 0,
            residual: null(),
            gate: null(),
            gate_period: 0,
            lokr_delta: null(),
            lokr_scale: 0.0,
        }
    }
}

extern "C" {
    pub fn ql_version() -> c_int;
    pub fn ql_last_error() -> *const c_char;
    pub fn ql_device_error(clear: c_int) -> c_int;
    pub fn ql_debug_inject(flags: c_uint, wait_limit_ns: c_ulonglong) -> c_int;
    pub fn ql_quantize(w: *const c_void, w_dtype: c_int, n: i64, k: i64, group_size: c_int, bits: c_int,
                       wq: *mut u32, scales: *mut c_void, biases: *mut c_void, sb_dtype: c_int,
                       stream: *mut c_void) -> c_int;
    pub fn ql_dequantize(wq: *const u32, scales: *const c_void, biases: *const c_void, sb_dtype: c_int,
                         n: i64, k: i64, group_size: c_int, bits: c_int, out: *mut c_void, out_dtype: c_int,
                         stream: *mut c_void) -> c_int;
    pub fn ql_dequantize_rows(ids: *const i64, r: i64, wq: *const u32, scales: *const c_void,
                              biases: *const c_void, sb_dtype: c_int, n: i64, k: i64, group_size: c_int,
                              bits: c_int, out: *mut c_void, out_dtype: c_int, stream: *mut c_void) -> c_int;
    pub fn ql_layernorm_modulate(x: *const c_void, m: i64, d: i64, eps: f32, scale: *const c_void,
                                 shift: *const c_void, period: i64, y: *mut c_void, y_dtype: c_int,
                                 stream: *mut c_void) -> c_int;
    pub fn ql_quantized_matmul(x: *const c_void, x_dtype: c_int, m: i64, k: i64, wq: *const u32,
                               scales: *const c_void, biases: *const c_void, sb_dtype: c_int, n: i64,
                               group_size: c_int, bits: c_int, transpose: c_int, ep: *const ql_epilogue,
                               y: *mut c_void, y_dtype: c_int, stream: *mut c_void) -> c_int;
    pub fn ql_matmul_workspace_size(m: i64, n: i64, k: i64, ep: *const ql_epilogue) -> usize;
    pub fn ql_matmul_workspace_size_x(m: i64, n: i64, k: i64, ep: *const ql_epilogue, x_dtype: c_int) -> usize;
    pub fn ql_quantized_matmul_noalloc(x: *const c_void, x_dtype: c_int, m: i64, k: i64, wq: *const u32,
                                       scales: *const c_void, biases: *const c_void, sb_dtype: c_int, n: i64,
                                       group_size: c_int, bits: c_int, transpose: c_int,
                                       ep: *const ql_epilogue, y: *mut c_void, y_dtype: c_int,
                                       stream: *mut c_void) -> c_int;
}
