/*
 * qlinear.h -- C ABI of libqlinear, the B200 (sm_100a) group-wise affine Q4/Q8
 * quantized-linear library.
 *
 * This ABI is the drop-in boundary for the reference's quantized-linear path.
 * The reference (SceneWorks/mlx-gen, Rust on MLX) reaches the arithmetic
 * through mlx-rs; each entry point below names the call it replaces.
 *
 * Conventions
 *   - Every pointer argument is caller-owned DEVICE memory (except ql_last_error's
 *     result).  The library allocates nothing on any call path.
 *   - Row-major, contiguous.  W is [N, K] (out, in), x is [M, K], y is [M, N].
 *   - Packing (byte-identical to MLX affine quantization): wq is uint32
 *     [N, K*bits/32]; element k of a row is code (wq[k/(32/bits)] >> (bits*(k%(32/bits))))
 *     & (2^bits-1); scales / biases are [N, K/group_size]; w = code*scale + bias.
 *   - `stream` is a cudaStream_t (NULL = legacy default stream).  Calls are
 *     asynchronous, hold no global mutable state and may run concurrently on
 *     different streams -- except ql_quantized_matmul_noalloc, whose LoRA calls share
 *     one fixed device array (see its declaration).
 *   - Return value is a ql_status.  On failure, ql_last_error() returns a
 *     thread-local message.  No call aborts or exits.
 */
#ifndef QLINEAR_H
#define QLINEAR_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
    QL_F32 = 0,
    QL_BF16 = 1,
    QL_F16 = 2,
} ql_dtype;

typedef enum {
    QL_OK = 0,
    QL_EINVAL_SHAPE = 1,  /* K % group_size, sizes <= 0, mismatched shapes      */
    QL_EUNSUPPORTED = 2,  /* bits not in {4,8}, group_size not in {32,64,128},
                             dtype combination without a kernel                 */
    QL_ECUDA = 3,         /* a CUDA runtime / driver call failed                */
    QL_EINVAL_ARG = 4,    /* NULL pointer, misaligned pointer, small workspace  */
    QL_ETIMEOUT = 5,      /* a kernel's bounded wait ran out (see ql_device_error) */
} ql_status;

typedef enum {
    QL_ACT_NONE = 0,
    QL_ACT_GELU_TANH = 1, /* 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3)))     */
    QL_ACT_GELU_ERF = 2,  /* 0.5 x (1 + erf(x / sqrt 2))                         */
    QL_ACT_SWIGLU = 3,    /* silu(x W^T) * (x W_up^T); needs the *_up weights    */
} ql_act;

typedef enum {
    QL_KERNEL_AUTO = 0,    /* GEMV for M <= 8, tcgen05 GEMM otherwise (bf16)    */
    QL_KERNEL_GENERIC = 1, /* CUDA-core fp32 kernel; any dtype                   */
    QL_KERNEL_GEMV = 2,    /* M <= 8, bf16 x and bf16 scales                     */
    QL_KERNEL_GEMM = 3,    /* tcgen05 / TMEM GEMM, one CTA per MMA (cta_group::1) */
    QL_KERNEL_GEMM_PAIR = 4, /* the same GEMM on CTA pairs (cta_group::2); slower today */
    QL_KERNEL_GEMV_TC = 5, /* the tcgen05 GEMV alone (M <= 8, no LoRA, group 64/128 or Q8/32;
                              QL_EUNSUPPORTED otherwise); QL_KERNEL_GEMV picks it for wide N */
    QL_KERNEL_GEMV_TMA = 6, /* the TMA-fed mma.sync GEMV alone (M <= 8, K a whole number of
                               8-group batches)                                          */
    QL_KERNEL_GEMV_REGS = 7, /* the register-fed GEMV alone (M <= 8)                     */
} ql_kernel;

/* Fused epilogue and options of ql_quantized_matmul.  Zero-initialise, then set
 * what is needed.  Replaces the ops the reference runs after quantized_matmul:
 * the bias add (src/adapters.rs:318-320), the LoRA residual sum
 * (src/adapters.rs:260-270,545-547), GELU (src/nn.rs:321-355) and SwiGLU
 * (mlx-gen-z-image/src/feed_forward.rs:34-38). */
typedef struct {
    const void *bias;          /* [N] in y's dtype, or NULL                           */
    int act;                   /* ql_act                                               */
    /* SwiGLU second projection (w3 / "up"), same shapes and dtypes as the main one. */
    const uint32_t *wq_up;
    const void *scales_up;
    const void *biases_up;
    const void *bias_up;       /* [N] or NULL                                          */
    /* LoRA residual: y += lora_scale * (x . A) . B with A [K, rank], B [rank, N] in
     * x's dtype, any rank in [1, 4096].  Needs `workspace` of ql_matmul_workspace_size(). */
    const void *lora_a;
    const void *lora_b;
    int64_t lora_rank;
    float lora_scale;
    void *workspace;
    size_t workspace_bytes;
    int kernel;                /* ql_kernel (QL_KERNEL_AUTO unless testing a path)     */
    int max_ctas;              /* GEMM: cap on resident CTAs (0 = one per SM); leaves
                                  SMs free for a collective running alongside          */
    /* Gated residual (the DiT blocks' `x + gate * linear(x)`, src/nn.rs:166-176):
       y = residual + gate * f(x W^T + bias), each op rounded to y's dtype.  NULL residual:
       off.  gate [rows, N] with row m / gate_period (gate_period 0: one row for all M);
       NULL gate: y = residual + f(...).  Both in y's dtype; residual may alias y.      */
    const void *residual;      /* [M, N]                                               */
    const void *gate;          /* [M / gate_period, N] or [N]                          */
    int64_t gate_period;       /* token rows per gate row (0: one gate row)            */
    /* LoKr residual (src/adapters.rs:263-266): y += lokr_scale * x . delta^T, delta a dense
       [N, K] matrix in x's dtype (the reconstructed Kronecker product).  The tensor-core
       path adds lokr_scale * delta to each dequantized weight (no extra MMA); it needs
       the 1-CTA GEMM without SwiGLU (QL_KERNEL_AUTO picks it for any M).  NULL: off.  */
    const void *lokr_delta;
    float lokr_scale;
} ql_epilogue;

/* Library version (major*10000 + minor*100 + patch). */
int ql_version(void);

/* Thread-local message describing the last failure on this thread ("" if none). */
const char *ql_last_error(void);

/* Reads (and with clear != 0 resets) the device-side error word that kernels set
 * when a bounded wait runs out.  Synchronises the current device.  0 = no error. */
int ql_device_error(int clear);

/* Test hook for the failure path (no counterpart in the reference, whose failure model is
 * a cooperative cancel flag, gen-core/src/runtime.rs:239-258).  Every pipelined kernel's
 * waits are bounded: when one runs out the kernel records a DEV_ERR timeout code in the
 * device error word (read with ql_device_error), every role drains, TMEM is freed and the
 * kernel returns; the context stays usable.  wait_limit_ns replaces the 2 s limit on the
 * current device (0 restores it); flags bit 0 makes the tcgen05 GEMM's TMA producer issue
 * nothing, so its consumers' waits run out.  Synchronises the current device.  Not for
 * production use: set flags back to 0 afterwards. */
int ql_debug_inject(unsigned flags, unsigned long long wait_limit_ns);

/* Replaces mlx_rs::ops::quantize(w, group_size, bits) -> (wq, scales, biases)
 * (called at src/quant.rs:140, src/adapters.rs:533-537 via
 * QuantizedLinear::try_from_linear, src/nn.rs:91-93).  w [N, K] in w_dtype;
 * scales/biases written in sb_dtype (the reference stores them in w's dtype). */
int ql_quantize(const void *w, int w_dtype, int64_t N, int64_t K, int group_size, int bits,
                uint32_t *wq, void *scales, void *biases, int sb_dtype, void *stream);

/* Replaces mlx_rs::ops::dequantize(wq, scales, biases, group_size, bits)
 * (src/nn.rs:55, tests/quant_parity.rs:53).  out [N, K] in out_dtype;
 * w = fma(code, scale, bias) in fp32, rounded once. */
int ql_dequantize(const uint32_t *wq, const void *scales, const void *biases, int sb_dtype,
                  int64_t N, int64_t K, int group_size, int bits, void *out, int out_dtype,
                  void *stream);

/* Replaces the quantized TokenEmbedding gather: take_axis(wq|scales|biases, ids)
 * followed by dequantize and a cast (src/nn.rs:42-59).  ids [R] int64 into the
 * N rows; out [R, K] in out_dtype.  Each value is fma(code, scale, bias) in fp32
 * rounded to sb_dtype (dequantize's output dtype), then converted to out_dtype.  An id
 * outside [0, N) yields a zero row and sets the device error word. */
int ql_dequantize_rows(const int64_t *ids, int64_t R, const uint32_t *wq, const void *scales,
                       const void *biases, int sb_dtype, int64_t N, int64_t K, int group_size,
                       int bits, void *out, int out_dtype, void *stream);

/* The DiT blocks' adaLN prologue in one pass: y = (1 + scale) * layer_norm(x) + shift.
   Replaces mlx_rs::fast::layer_norm(x, None, None, eps) followed by nn::modulate
   (mlx-gen-flux/src/transformer.rs:891-913, src/nn.rs:262-287).  x bf16 [M, D], D a
   multiple of 8; scale / shift bf16 [M / period, D] (period 0: one row for all M) or NULL
   (plain layer norm).  y_dtype QL_BF16: each modulate op rounded to bf16 (FLUX.1, the 1
   in scale's dtype); QL_F32: computed and stored in f32 (FLUX.2, a strong f32 1). */
int ql_layernorm_modulate(const void *x, int64_t M, int64_t D, float eps, const void *scale, const void *shift,
                          int64_t period, void *y, int y_dtype, void *stream);

/* Replaces mlx_rs::ops::quantized_matmul(x, wq, scales, biases, transpose=true,
 * group_size, bits) as called by LinearBase::forward (src/adapters.rs:309-317),
 * plus the ops fused through `ep` (may be NULL).  y [M, N] in y_dtype.
 * transpose must be 1 (the only form the reference uses). */
int ql_quantized_matmul(const void *x, int x_dtype, int64_t M, int64_t K, const uint32_t *wq,
                        const void *scales, const void *biases, int sb_dtype, int64_t N,
                        int group_size, int bits, int transpose, const ql_epilogue *ep,
                        void *y, int y_dtype, void *stream);

/* Bytes of device workspace ql_quantized_matmul needs for this shape and
 * epilogue (0 when none; the LoRA residual needs M * round_up(rank, 64) * 2). */
size_t ql_matmul_workspace_size(int64_t M, int64_t N, int64_t K, const ql_epilogue *ep);

/* Workspace for ql_quantized_matmul when x is x_dtype: the LoRA need above, or -- for f32 /
 * f16 activations -- the two bf16 pieces of x ([M, 2 * round_up(K, 64)] bf16) that the
 * tensor-core path for those dtypes stages.  Given that workspace, an f32 / f16 x with bf16
 * or f16 scales, f32 / f16 y, a plain or GELU linear (no SwiGLU, LoRA, LoKr or gated
 * residual) runs on the tcgen05 GEMM in three bf16 passes (x and each dequantized weight
 * split into two bf16 pieces: about 16 significant bits per product, fp32 accumulation --
 * the activations of FLUX.2 / Qwen image streams / LTX text encoders, src/adapters.rs:252,
 * src/nn.rs:295); without it those calls run on the CUDA-core kernel. */
size_t ql_matmul_workspace_size_x(int64_t M, int64_t N, int64_t K, const ql_epilogue *ep, int x_dtype);

/* Same as ql_quantized_matmul, for callers that cannot allocate device memory
 * (allocator hooks, real-time loops that must not enter the driver's allocator,
 * runtimes whose memory is fully reserved).  No counterpart in the reference.
 * The LoRA workspace comes from a fixed 8 MiB device array inside the library
 * (ep->workspace is ignored); a request above that (M * round_up(rank, 64) * 2
 * bytes) returns QL_EUNSUPPORTED.  The first call on a device (LoRA or not) looks up the array
 * with that device current -- make it before any stream capture.  Calls share the
 * array: calls that overlap on the GPU race.  Allocates nothing. */
int ql_quantized_matmul_noalloc(const void *x, int x_dtype, int64_t M, int64_t K,
                                const uint32_t *wq, const void *scales, const void *biases,
                                int sb_dtype, int64_t N, int group_size, int bits, int transpose,
                                const ql_epilogue *ep, void *y, int y_dtype, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* QLINEAR_H */
