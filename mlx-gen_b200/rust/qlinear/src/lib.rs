//! Safe layer over `qlinear-sys` with the shapes of the reference's quantized arm.
//!
//! Device memory stays with the caller (any CUDA allocator: the host runtime's own, or a
//! crate such as cudarc); this layer takes device pointers wrapped in [`DevicePtr`],
//! checks the host-side arguments the reference would reject, and turns a non-zero
//! `ql_status` into [`Error::Msg`] carrying `ql_last_error()`, the convention of the
//! reference's `Error::Msg` (src/error.rs:9-36).
//!
//! A provider crate's quantized linear (src/adapters.rs:300-322) becomes:
//! ```ignore
//! let w = QuantizedWeights { wq, scales, biases, sb_dtype: Dtype::Bf16, n, k, group_size: 64, bits: 8 };
//! let mut ep = Epilogue::default();
//! ep.bias(bias).act(Act::GeluTanh);
//! w.matmul(x, Dtype::Bf16, m, &ep, y, Dtype::Bf16, stream)?;
//! ```
use qlinear_sys as sys;
use std::ffi::CStr;
use std::os::raw::c_void;

#[derive(Debug, Clone, PartialEq, Eq)]
pub enum Error {
    /// A libqlinear call failed: the status and `ql_last_error()`.
    Msg { status: i32, message: String },
    /// A bounded device wait ran out; the word is `ql_device_error`'s.
    DeviceTimeout { word: i32 },
}

impl std::fmt::Display for Error {
    fn fmt(&self, f: &mut std::fmt::Formatter<'_>) -> std::fmt::Result {
        match self {
            Error::Msg { status, message } => write!(f, "libqlinear status {status}: {message}"),
            Error::DeviceTimeout { word } => write!(f, "libqlinear device wait ran out (error word {word:#x})"),
        }
    }
}

impl std::error::Error for Error {}

pub type Result<T> = std::result::Result<T, Error>;

fn check(status: i32) -> Result<()> {
    if status == sys::QL_OK {
        return Ok(());
    }
    let message = unsafe {
        let p = sys::ql_last_error();
        if p.is_null() { String::new() } else { CStr::from_ptr(p).to_string_lossy().into_owned() }
    };
    if status == sys::QL_ETIMEOUT {
        let word = unsafe { sys::ql_device_error(1) };
        return Err(Error::DeviceTimeout { word });
    }
    Err(Error::Msg { status, message })
}

#[derive(Debug, Clone, Copy, PartialEq, Eq)]
pub enum Dtype {
    F32,
    Bf16,
    F16,
}

impl Dtype {
    fn raw(self) -> i32 {
        match self {
            Dtype::F32 => sys::QL_F32,
            Dtype::Bf16 => sys::QL_BF16,
            Dtype::F16 => sys::QL_F16,
        }
    }
}

#[derive(Debug, Clone, Copy, PartialEq, Eq)]
pub enum Act {
    None,
    GeluTanh,
    GeluErf,
    SwiGlu,
}

/// A device pointer owned by the caller.
#[derive(Debug, Clone, Copy)]
pub struct DevicePtr(pub *mut c_void);

/// A CUDA stream handle (`cudaStream_t`); null is the legacy default stream.
#[derive(Debug, Clone, Copy)]
pub struct Stream(pub *mut c_void);

/// The packed parts of one `QuantizedLinear` (src/adapters.rs:367-385): `wq [n, k*bits/32]`
/// u32, `scales` / `biases [n, k/group_size]` in `sb_dtype`.
#[derive(Debug, Clone, Copy)]
pub struct QuantizedWeights {
    pub wq: DevicePtr,
    pub scales: DevicePtr,
    pub biases: DevicePtr,
    pub sb_dtype: Dtype,
    pub n: i64,
    pub k: i64,
    pub group_size: i32,
    pub bits: i32,
}

/// `packed_bits` with typed errors (src/quant.rs:38-41 infers bits from the shapes and
/// divides by the scales' width without checking it).
pub fn packed_bits(wq_cols: i64, scales_cols: i64, group_size: i64) -> Result<i32> {
    let bad = |m: &str| Err(Error::Msg { status: sys::QL_EINVAL_SHAPE, message: m.to_string() });
    if wq_cols <= 0 || scales_cols <= 0 || group_size <= 0 {
        return bad("packed_bits: empty packed weight or scales");
    }
    let k = scales_cols * group_size;
    if (wq_cols * 32) % k != 0 {
        return bad("packed_bits: packed width is not a whole number of bits per element");
    }
    match wq_cols * 32 / k {
        b @ (4 | 8) => Ok(b as i32),
        _ => bad("packed_bits: derived bits not in {4, 8}"),
    }
}

impl QuantizedWeights {
    /// `QuantizedLinear::try_from_linear` on a dense `[n, k]` weight (src/adapters.rs:533-537):
    /// fills this struct's buffers, which the caller sized.
    pub fn quantize_from(&self, w: DevicePtr, w_dtype: Dtype, stream: Stream) -> Result<()> {
        check(unsafe {
            sys::ql_quantize(w.0, w_dtype.raw(), self.n, self.k, self.group_size, self.bits, self.wq.0 as *mut u32,
                             self.scales.0, self.biases.0, self.sb_dtype.raw(), stream.0)
        })
    }

    /// `dequantize(wq, scales, biases, group_size, bits)` into `out [n, k]`.
    pub fn dequantize(&self, out: DevicePtr, out_dtype: Dtype, stream: Stream) -> Result<()> {
        check(unsafe {
            sys::ql_dequantize(self.wq.0 as *const u32, self.scales.0, self.biases.0, self.sb_dtype.raw(), self.n,
                               self.k, self.group_size, self.bits, out.0, out_dtype.raw(), stream.0)
        })
    }

    /// The quantized `TokenEmbedding` lookup (src/nn.rs:42-59): rows `ids [r]` (i64, device).
    pub fn gather_rows(&self, ids: DevicePtr, r: i64, out: DevicePtr, out_dtype: Dtype, stream: Stream) -> Result<()> {
        check(unsafe {
            sys::ql_dequantize_rows(ids.0 as *const i64, r, self.wq.0 as *const u32, self.scales.0, self.biases.0,
                                    self.sb_dtype.raw(), self.n, self.k, self.group_size, self.bits, out.0,
                                    out_dtype.raw(), stream.0)
        })
    }

    /// `y [m, n] = x [m, k] . W^T` plus the epilogue, as `LinearBase::forward` /
    /// `AdaptableLinear::forward` compute it (src/adapters.rs:300-322, :543-549).
    #[allow(clippy::too_many_arguments)]
    pub fn matmul(&self, x: DevicePtr, x_dtype: Dtype, m: i64, ep: &Epilogue, y: DevicePtr, y_dtype: Dtype,
                  stream: Stream) -> Result<()> {
        check(unsafe {
            sys::ql_quantized_matmul(x.0, x_dtype.raw(), m, self.k, self.wq.0 as *const u32, self.scales.0,
                                     self.biases.0, self.sb_dtype.raw(), self.n, self.group_size, self.bits, 1,
                                     &ep.raw, y.0, y_dtype.raw(), stream.0)
        })
    }

    /// Device workspace bytes `matmul` needs with this epilogue and activation dtype.
    pub fn workspace_bytes(&self, m: i64, ep: &Epilogue, x_dtype: Dtype) -> usize {
        unsafe { sys::ql_matmul_workspace_size_x(m, self.n, self.k, &ep.raw, x_dtype.raw()) }
    }
}

/// Builder over `ql_epilogue`.
#[derive(Debug, Clone, Copy, Default)]
pub struct Epilogue {
    pub raw: sys::ql_epilogue,
}

impl Epilogue {
    pub fn bias(&mut self, b: DevicePtr) -> &mut Self {
        self.raw.bias = b.0;
        self
    }
    pub fn act(&mut self, a: Act) -> &mut Self {
        self.raw.act = match a {
            Act::None => sys::QL_ACT_NONE,
            Act::GeluTanh => sys::QL_ACT_GELU_TANH,
            Act::GeluErf => sys::QL_ACT_GELU_ERF,
            Act::SwiGlu => sys::QL_ACT_SWIGLU,
        };
        self
    }
    /// The up projection of a fused SwiGLU (`silu(x W^T) * (x W_up^T)`).
    pub fn swiglu_up(&mut self, up: &QuantizedWeights, bias_up: Option<DevicePtr>) -> &mut Self {
        self.raw.act = sys::QL_ACT_SWIGLU;
        self.raw.wq_up = up.wq.0 as *const u32;
        self.raw.scales_up = up.scales.0;
        self.raw.biases_up = up.biases.0;
        self.raw.bias_up = bias_up.map_or(std::ptr::null(), |p| p.0);
        self
    }
    /// One LoRA adapter `scale . (x a) b` (src/adapters.rs:231-261); `workspace` of
    /// `QuantizedWeights::workspace_bytes` bytes.
    pub fn lora(&mut self, a: DevicePtr, b: DevicePtr, rank: i64, scale: f32, workspace: DevicePtr,
                workspace_bytes: usize) -> &mut Self {
        self.raw.lora_a = a.0;
        self.raw.lora_b = b.0;
        self.raw.lora_rank = rank;
        self.raw.lora_scale = scale;
        self.raw.workspace = workspace.0;
        self.raw.workspace_bytes = workspace_bytes;
        self
    }
    /// One LoKr adapter `scale . x delta^T` with the reconstructed dense delta (src/adapters.rs:263-266).
    pub fn lokr(&mut self, delta: DevicePtr, scale: f32) -> &mut Self {
        self.raw.lokr_delta = delta.0;
        self.raw.lokr_scale = scale;
        self
    }
    /// `nn::gated(residual, gate, linear(..))`: y = residual + gate . y, one gate row per
    /// `period` tokens.
    pub fn gated(&mut self, residual: DevicePtr, gate: DevicePtr, period: i64) -> &mut Self {
        self.raw.residual = residual.0;
        self.raw.gate = gate.0;
        self.raw.gate_period = period;
        self
    }
}

/// `fast::layer_norm` + `nn::modulate` of the DiT blocks in one pass
/// (mlx-gen-flux/src/transformer.rs:891-913, src/nn.rs:262-287).
#[allow(clippy::too_many_arguments)]
pub fn layernorm_modulate(x: DevicePtr, m: i64, d: i64, eps: f32, scale: Option<DevicePtr>,
                          shift: Option<DevicePtr>, period: i64, y: DevicePtr, y_dtype: Dtype,
                          stream: Stream) -> Result<()> {
    let p = |o: Option<DevicePtr>| o.map_or(std::ptr::null(), |v| v.0 as *const c_void);
    check(unsafe { sys::ql_layernorm_modulate(x.0, m, d, eps, p(scale), p(shift), period, y.0, y_dtype.raw(), stream.0) })
}

/// Reads and clears the device error word (bounded-wait timeouts, bad gather ids).
pub fn device_error() -> i32 {
    unsafe { sys::ql_device_error(1) }
}

#[cfg(test)]
mod tests {
    use super::*;

    #[test]
    fn packed_bits_typed() {
        assert_eq!(packed_bits(384, 48, 64).unwrap(), 4);
        assert_eq!(packed_bits(768, 48, 64).unwrap(), 8);
        assert!(packed_bits(0, 48, 64).is_err());
        assert!(packed_bits(384, 0, 64).is_err());
        assert!(packed_bits(96, 48, 64).is_err());
    }
}
