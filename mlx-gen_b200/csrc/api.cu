// api.cu -- the extern "C" entry points of libqlinear (declared in include/qlinear.h).
//
// Validation happens here, on the host, before any launch: shapes, group size,
// bit width, dtype combination, pointer alignment, workspace size.  A failed
// check returns a status and leaves a thread-local message; nothing aborts.
// Dispatch: bf16 activations and scales go to the tensor-core kernels (GEMV for
// M <= 8, tcgen05 GEMM otherwise); other dtypes go to the CUDA-core kernel.
#include <stdarg.h>
#include <stdio.h>

#include "ql_common.cuh"

namespace ql {

static thread_local char g_err[512] = "";

void set_error(const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
}

int fail(int status, const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
    return status;
}

int launch_quantize(const void *, int, int64_t, int64_t, int, int, uint32_t *, void *, void *, int,
                    cudaStream_t);
int launch_dequantize(const int64_t *, int64_t, int64_t, int64_t, int, int, const uint32_t *,
                      const void *, const void *, int, void *, int, bool, cudaStream_t);
int launch_qgemv(const void *, int64_t, int64_t, const uint32_t *, const void *, const void *,
                 const uint32_t *, const void *, const void *, int64_t, int, int, const void *,
                 const void *, int, const void *, const void *, int64_t, void *, const Gated &, int, cudaStream_t);
bool qgemv_tc_supported(int64_t, int64_t, int, int, const void *, bool);
int launch_qgemv_tc(const void *, int64_t, int64_t, const uint32_t *, const void *, const void *, const uint32_t *,
                    const void *, const void *, int64_t, int, int, const void *, const void *, int, void *,
                    const Gated &, cudaStream_t);
int launch_qgemm_sm100(const void *, int64_t, int64_t, const uint32_t *, const void *, const void *,
                       const uint32_t *, const void *, const void *, int64_t, int, int, const void *,
                       const void *, int, const void *, const void *, int64_t, void *, int, int, const Gated &,
                       const void *, float, cudaStream_t);
int launch_qmm_generic(const void *, int, int64_t, int64_t, const uint32_t *, const void *,
                       const void *, const uint32_t *, const void *, const void *, int, int64_t, int,
                       int, const void *, const void *, int, const void *, const void *, int64_t,
                       float, void *, int, const Gated &, const void *, float, cudaStream_t);
size_t qgemm_x3_workspace(int64_t M, int64_t K);
int launch_qgemm_x3(const void *, int, int64_t, int64_t, const uint32_t *, const void *, const void *, int, int64_t,
                    int, int, const void *, int, void *, int, void *, int, cudaStream_t);
int launch_lora_t(const void *, int64_t, int64_t, const void *, int64_t, float, void *, cudaStream_t);
int launch_ln_modulate(const void *, int64_t, int64_t, float, const void *, const void *, int64_t, void *, int,
                       cudaStream_t);

static bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
static bool valid_dtype(int dt) { return dt == QL_F32 || dt == QL_BF16 || dt == QL_F16; }

static int check_quant_params(int64_t N, int64_t K, int gs, int bits) {
    if (bits != 4 && bits != 8) return fail(QL_EUNSUPPORTED, "bits must be 4 or 8 (got %d)", bits);
    if (gs != 32 && gs != 64 && gs != 128)
        return fail(QL_EUNSUPPORTED, "group_size must be 32, 64 or 128 (got %d)", gs);
    if (N <= 0 || K <= 0) return fail(QL_EINVAL_SHAPE, "N and K must be positive (N=%lld K=%lld)",
                                      (long long)N, (long long)K);
    if (K % gs) return fail(QL_EINVAL_SHAPE, "K=%lld is not a multiple of group_size=%d", (long long)K, gs);
    if (N > INT32_MAX || K > INT32_MAX) return fail(QL_EINVAL_SHAPE, "N or K exceeds 2^31-1");
    return QL_OK;
}

static size_t lora_ws_bytes(int64_t M, int64_t rank) {
    return rank > 0 ? (size_t)M * (size_t)((rank + 63) / 64 * 64) * 2 : 0;
}

}  // namespace ql

using namespace ql;

extern "C" {

int ql_version(void) { return 100; }

const char *ql_last_error(void) { return g_err; }

int ql_device_error(int clear) {
    if (cudaDeviceSynchronize() != cudaSuccess) {
        fail(QL_ECUDA, "cudaDeviceSynchronize failed");
        return -1;
    }
    unsigned v = 0;
    if (cudaMemcpyFromSymbol(&v, g_dev_error, sizeof(v)) != cudaSuccess) return -1;
    if (clear) {
        unsigned z = 0;
        cudaMemcpyToSymbol(g_dev_error, &z, sizeof(z));
    }
    return (int)v;
}

int ql_debug_inject(unsigned flags, unsigned long long wait_limit_ns) {
    g_err[0] = 0;
    const unsigned long long lim = wait_limit_ns ? wait_limit_ns : kWaitLimitNs;
    QL_CUDA_TRY(cudaDeviceSynchronize());
    QL_CUDA_TRY(cudaMemcpyToSymbol(g_wait_limit_ns, &lim, sizeof(lim)));
    QL_CUDA_TRY(cudaMemcpyToSymbol(g_debug_inject, &flags, sizeof(flags)));
    return QL_OK;
}

int ql_quantize(const void *w, int w_dtype, int64_t N, int64_t K, int group_size, int bits,
                uint32_t *wq, void *scales, void *biases, int sb_dtype, void *stream) {
    g_err[0] = 0;
    if (int rc = check_quant_params(N, K, group_size, bits)) return rc;
    if (!w || !wq || !scales || !biases) return fail(QL_EINVAL_ARG, "ql_quantize: NULL pointer");
    if (!valid_dtype(w_dtype) || !valid_dtype(sb_dtype)) return fail(QL_EUNSUPPORTED, "unknown dtype");
    if (!aligned16(w) || !aligned16(wq))
        return fail(QL_EINVAL_ARG, "ql_quantize: w and wq must be 16-byte aligned");
    return launch_quantize(w, w_dtype, N, K, group_size, bits, wq, scales, biases, sb_dtype,
                           (cudaStream_t)stream);
}

int ql_dequantize(const uint32_t *wq, const void *scales, const void *biases, int sb_dtype,
                  int64_t N, int64_t K, int group_size, int bits, void *out, int out_dtype,
                  void *stream) {
    g_err[0] = 0;
    if (int rc = check_quant_params(N, K, group_size, bits)) return rc;
    if (!wq || !scales || !biases || !out) return fail(QL_EINVAL_ARG, "ql_dequantize: NULL pointer");
    if (!valid_dtype(sb_dtype) || !valid_dtype(out_dtype)) return fail(QL_EUNSUPPORTED, "unknown dtype");
    if (!aligned16(wq) || !aligned16(out))
        return fail(QL_EINVAL_ARG, "ql_dequantize: wq and out must be 16-byte aligned");
    return launch_dequantize(nullptr, N, N, K, group_size, bits, wq, scales, biases, sb_dtype, out,
                             out_dtype, false, (cudaStream_t)stream);
}

int ql_layernorm_modulate(const void *x, int64_t M, int64_t D, float eps, const void *scale, const void *shift,
                          int64_t period, void *y, int y_dtype, void *stream) {
    g_err[0] = 0;
    if (M < 0 || D <= 0 || D % 8) return fail(QL_EINVAL_SHAPE, "ql_layernorm_modulate: D must be a positive multiple of 8");
    if (M == 0) return QL_OK;
    if (!x || !y) return fail(QL_EINVAL_ARG, "ql_layernorm_modulate: NULL pointer");
    if (y_dtype != QL_BF16 && y_dtype != QL_F32) return fail(QL_EUNSUPPORTED, "y must be bf16 or f32");
    if (period < 0) return fail(QL_EINVAL_ARG, "period must be >= 0");
    if (!aligned16(x) || !aligned16(y)) return fail(QL_EINVAL_ARG, "x and y must be 16-byte aligned");
    return launch_ln_modulate(x, M, D, eps, scale, shift, period, y, y_dtype, (cudaStream_t)stream);
}

int ql_dequantize_rows(const int64_t *ids, int64_t R, const uint32_t *wq, const void *scales,
                       const void *biases, int sb_dtype, int64_t N, int64_t K, int group_size,
                       int bits, void *out, int out_dtype, void *stream) {
    g_err[0] = 0;
    if (int rc = check_quant_params(N, K, group_size, bits)) return rc;
    if (R < 0) return fail(QL_EINVAL_SHAPE, "R must be >= 0");
    if (R == 0) return QL_OK;
    if (!ids || !wq || !scales || !biases || !out)
        return fail(QL_EINVAL_ARG, "ql_dequantize_rows: NULL pointer");
    if (!valid_dtype(sb_dtype) || !valid_dtype(out_dtype)) return fail(QL_EUNSUPPORTED, "unknown dtype");
    if (!aligned16(wq) || !aligned16(out))
        return fail(QL_EINVAL_ARG, "ql_dequantize_rows: wq and out must be 16-byte aligned");
    return launch_dequantize(ids, R, N, K, group_size, bits, wq, scales, biases, sb_dtype, out,
                             out_dtype, true, (cudaStream_t)stream);
}

size_t ql_matmul_workspace_size_x(int64_t M, int64_t N, int64_t K, const ql_epilogue *ep, int x_dtype) {
    size_t w = ql_matmul_workspace_size(M, N, K, ep);
    if ((x_dtype == QL_F32 || x_dtype == QL_F16) && M > 0 && K > 0) {
        const size_t x3 = qgemm_x3_workspace(M, K);
        if (x3 > w) w = x3;
    }
    return w;
}

size_t ql_matmul_workspace_size(int64_t M, int64_t N, int64_t K, const ql_epilogue *ep) {
    (void)N;
    (void)K;
    if (!ep || !ep->lora_a || ep->lora_rank <= 0) return 0;
    return lora_ws_bytes(M, ep->lora_rank);
}

int ql_quantized_matmul(const void *x, int x_dtype, int64_t M, int64_t K, const uint32_t *wq,
                        const void *scales, const void *biases, int sb_dtype, int64_t N,
                        int group_size, int bits, int transpose, const ql_epilogue *ep, void *y,
                        int y_dtype, void *stream) {
    g_err[0] = 0;
    cudaStream_t st = (cudaStream_t)stream;
    ql_epilogue e{};
    if (ep) e = *ep;
    if (!transpose) return fail(QL_EUNSUPPORTED, "only transpose=true (y = x . W^T) is supported");
    if (int rc = check_quant_params(N, K, group_size, bits)) return rc;
    if (M < 0 || M > INT32_MAX) return fail(QL_EINVAL_SHAPE, "bad M=%lld", (long long)M);
    if (M == 0) return QL_OK;
    if (!x || !wq || !scales || !biases || !y) return fail(QL_EINVAL_ARG, "ql_quantized_matmul: NULL pointer");
    if (!valid_dtype(x_dtype) || !valid_dtype(sb_dtype) || !valid_dtype(y_dtype))
        return fail(QL_EUNSUPPORTED, "unknown dtype");
    if (!aligned16(x) || !aligned16(wq) || !aligned16(y))
        return fail(QL_EINVAL_ARG, "x, wq and y must be 16-byte aligned");
    if (e.act < QL_ACT_NONE || e.act > QL_ACT_SWIGLU) return fail(QL_EINVAL_ARG, "unknown activation %d", e.act);
    const bool swiglu = e.act == QL_ACT_SWIGLU;
    if (swiglu && (!e.wq_up || !e.scales_up || !e.biases_up))
        return fail(QL_EINVAL_ARG, "SwiGLU needs wq_up, scales_up and biases_up");
    if (swiglu && !aligned16(e.wq_up)) return fail(QL_EINVAL_ARG, "wq_up must be 16-byte aligned");
    const bool lora = e.lora_a != nullptr && e.lora_rank > 0;
    if (lora && !e.lora_b) return fail(QL_EINVAL_ARG, "LoRA needs both lora_a and lora_b");
    if (lora && swiglu)
        return fail(QL_EUNSUPPORTED, "a LoRA residual cannot be fused with SwiGLU; run the projections separately");
    if (lora && e.lora_rank > 4096) return fail(QL_EUNSUPPORTED, "LoRA rank > 4096");

    const bool tc_dtypes = x_dtype == QL_BF16 && sb_dtype == QL_BF16 && y_dtype == QL_BF16;
    if (e.gate && !e.residual) return fail(QL_EINVAL_ARG, "a gate needs a residual");
    if (e.gate_period < 0) return fail(QL_EINVAL_ARG, "gate_period must be >= 0");
    const Gated gd{e.residual, e.gate, e.gate_period};
    int kernel = e.kernel;
    const bool lokr = e.lokr_delta != nullptr;
    if (lokr && swiglu) return fail(QL_EUNSUPPORTED, "a LoKr delta cannot be fused with SwiGLU");
    if (lokr && !aligned16(e.lokr_delta)) return fail(QL_EINVAL_ARG, "lokr_delta must be 16-byte aligned");
    // f32 / f16 activations on the tensor cores (three-pass bf16 split) when the caller gave
    // the workspace for the split activations (ql_matmul_workspace_size_x); the CUDA-core
    // generic kernel otherwise
    const bool x3_shape = (x_dtype == QL_F32 || x_dtype == QL_F16) && sb_dtype != QL_F32 &&
                          (y_dtype == QL_F32 || y_dtype == QL_F16) && !swiglu && !lora && !gd.res && !lokr &&
                          (e.act == QL_ACT_NONE || e.act == QL_ACT_GELU_TANH || e.act == QL_ACT_GELU_ERF);
    if (x3_shape && ((e.kernel == QL_KERNEL_AUTO && M > 8) || e.kernel == QL_KERNEL_GEMM) && e.workspace &&
        e.workspace_bytes >= qgemm_x3_workspace(M, K)) {
        if (!aligned16(e.workspace)) return fail(QL_EINVAL_ARG, "workspace must be 16-byte aligned");
        return launch_qgemm_x3(x, x_dtype, M, K, wq, scales, biases, sb_dtype, N, group_size, bits, e.bias, e.act, y,
                               y_dtype, e.workspace, e.max_ctas, st);
    }
    if (e.kernel == QL_KERNEL_GEMM && !tc_dtypes)
        return fail(QL_EUNSUPPORTED, "the tensor-core GEMM with f32 / f16 activations needs a plain or GELU linear "
                                     "with bf16 or f16 scales and the workspace of ql_matmul_workspace_size_x");
    if (kernel == QL_KERNEL_AUTO)
        kernel = !tc_dtypes ? QL_KERNEL_GENERIC : ((M <= 8 && !lokr) ? QL_KERNEL_GEMV : QL_KERNEL_GEMM);
    if (lokr && kernel != QL_KERNEL_GEMM && kernel != QL_KERNEL_GENERIC)
        return fail(QL_EUNSUPPORTED, "a LoKr delta runs on the 1-CTA GEMM or the generic kernel");
    if (kernel != QL_KERNEL_GENERIC && !tc_dtypes)
        return fail(QL_EUNSUPPORTED, "tensor-core kernels need bf16 x, scales and y");
    if ((kernel == QL_KERNEL_GEMV || kernel == QL_KERNEL_GEMV_TC || kernel == QL_KERNEL_GEMV_TMA ||
         kernel == QL_KERNEL_GEMV_REGS) && M > 8)
        return fail(QL_EUNSUPPORTED, "GEMV kernel needs M <= 8");
    if (kernel < QL_KERNEL_AUTO || kernel > QL_KERNEL_GEMV_REGS) return fail(QL_EINVAL_ARG, "unknown kernel %d", kernel);
    if (kernel == QL_KERNEL_GEMV_TC) {
        if (lora || !qgemv_tc_supported(M, K, group_size, bits, x, false) ||
            !aligned16(scales) || !aligned16(biases) || (swiglu && (!aligned16(e.scales_up) || !aligned16(e.biases_up))))
            return fail(QL_EUNSUPPORTED, "tcgen05 GEMV: unsupported shape, group size or LoRA");
        return launch_qgemv_tc(x, M, K, wq, scales, biases, e.wq_up, e.scales_up, e.biases_up, N, group_size, bits,
                               e.bias, e.bias_up, e.act, y, gd, st);
    }

    if (kernel == QL_KERNEL_GENERIC)
        return launch_qmm_generic(x, x_dtype, M, K, wq, scales, biases, e.wq_up, e.scales_up, e.biases_up,
                                  sb_dtype, N, group_size, bits, e.bias, e.bias_up, e.act,
                                  lora ? e.lora_a : nullptr, e.lora_b, lora ? e.lora_rank : 0,
                                  e.lora_scale, y, y_dtype, gd, e.lokr_delta, e.lokr_scale, st);

    const void *lora_t = nullptr;
    if (lora) {
        const size_t need = lora_ws_bytes(M, e.lora_rank);
        if (!e.workspace || e.workspace_bytes < need)
            return fail(QL_EINVAL_ARG, "LoRA needs a workspace of %zu bytes (got %zu)", need, e.workspace_bytes);
        if (!aligned16(e.workspace)) return fail(QL_EINVAL_ARG, "workspace must be 16-byte aligned");
        if (int rc = launch_lora_t(x, M, K, e.lora_a, e.lora_rank, e.lora_scale, e.workspace, st)) return rc;
        lora_t = e.workspace;
    }
    if (kernel == QL_KERNEL_GEMV || kernel == QL_KERNEL_GEMV_TMA || kernel == QL_KERNEL_GEMV_REGS) {
        const int rc = launch_qgemv(x, M, K, wq, scales, biases, e.wq_up, e.scales_up, e.biases_up, N, group_size,
                                    bits, e.bias, e.bias_up, e.act, lora_t, e.lora_b, lora ? e.lora_rank : 0, y, gd,
                                    kernel == QL_KERNEL_GEMV_TMA ? 1 : kernel == QL_KERNEL_GEMV_REGS ? 2 : 0, st);
        // The GEMVs stage all of x in shared memory and refuse (before launching anything)
        // an M * K that does not fit; the automatic choice then streams x through the GEMM.
        if (rc != QL_EUNSUPPORTED || e.kernel != QL_KERNEL_AUTO) return rc;
    }
    return launch_qgemm_sm100(x, M, K, wq, scales, biases, e.wq_up, e.scales_up, e.biases_up, N, group_size,
                              bits, e.bias, e.bias_up, e.act, lora_t, e.lora_b, lora ? e.lora_rank : 0, y,
                              kernel == QL_KERNEL_GEMM_PAIR ? 2 : 1, e.max_ctas, gd, e.lokr_delta, e.lokr_scale, st);
}

}  // extern "C"

