/*
 * qref.c -- CPU restatement of the group-wise affine Q4/Q8 quantized-linear path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity oracle and the timed CPU
 * baseline.  Only tests/, __graft_entry__.smoke() and bench.py (its cpu_baseline
 * leg and its `--impl reference` arm) may load it.  The product path
 * (libqlinear.so) never links or calls it.
 *
 * What it restates.  The reference (SceneWorks/mlx-gen) reaches this arithmetic
 * through the third-party MLX 0.31.2 library (pmetal-mlx-rs 0.25.8 /
 * pmetal-mlx-sys 0.2.4, Cargo.toml:11-16,38,43), which is not vendored and
 * cannot be built here.  The semantics below follow the reference's call sites:
 *   - quantize:          src/quant.rs:140, src/adapters.rs:533-537, tools/dump_quant.py:27
 *   - dequantize:        src/nn.rs:51-56, tools/dump_quant.py:28
 *   - quantized_matmul:  src/adapters.rs:309-320 (transpose=true, bias added as a
 *                        separate op after the matmul), tools/dump_quant.py:29
 *   - LoRA residual:     src/adapters.rs:260-270 (scale * (x.A).B)
 *   - gelu_tanh:         src/nn.rs:321-329 (every constant cast to x's dtype)
 *   - gelu (erf):        src/nn.rs:344-355
 *   - swiglu:            mlx-gen-z-image/src/feed_forward.rs:34-38,61-70
 * and are pinned bit-exactly (codes, scales, biases, dequant) against the
 * reference's committed golden fixture tests/fixtures/quant_q4q8.safetensors
 * (checked by tests/quant_parity.rs:29-66 in the reference; re-checked by
 * tests/test_oracle.py here).
 *
 * Choices the fixture does not pin (documented, deliberate):
 *   - rounding of codes is round-half-to-even (rintf);
 *   - the per-element code uses a true division (w - bias) / scale;
 *   - for a bf16/f16 input the statistics, scale and bias are computed in fp32
 *     from the (exactly upcast) input; codes use the fp32 scale/bias; scale and
 *     bias are rounded to the storage dtype only when stored.  This follows the
 *     structure of MLX's published affine quantization (its CPU `quantize` and the
 *     Metal `affine_quantize` kernel accumulate the group min/max and derive scale
 *     and bias in float, quantize each element with those float values, and cast
 *     scale/bias to the output dtype at the store); it is not pinned by a golden
 *     vector of the reference for bf16 input.
 *   - quantized_matmul dequantizes in the computation dtype promote(x, scales)
 *     (mlx casts the operands to the result dtype): bf16 x with bf16 scales rounds
 *     each weight to bf16, f32 or mixed-dtype activations keep the fp32 value.
 *
 * dtype codes: 0 = f32, 1 = bf16, 2 = f16  (same numbering as include/qlinear.h).
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define QREF_F32 0
#define QREF_BF16 1
#define QREF_F16 2

/* ---------------------------------------------------------------- dtypes */

static inline float bf16_to_f32(uint16_t h) {
    uint32_t u = (uint32_t)h << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

/* round-to-nearest-even float -> bf16 (NaN kept quiet) */
static inline uint16_t f32_to_bf16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

static inline float rnd_bf16(float f) { return bf16_to_f32(f32_to_bf16(f)); }

static inline float load_el(const void *p, int dt, int64_t i) {
    switch (dt) {
    case QREF_F32: return ((const float *)p)[i];
    case QREF_BF16: return bf16_to_f32(((const uint16_t *)p)[i]);
    default: return (float)((const _Float16 *)p)[i];
    }
}

static inline void store_el(void *p, int dt, int64_t i, float v) {
    switch (dt) {
    case QREF_F32: ((float *)p)[i] = v; break;
    case QREF_BF16: ((uint16_t *)p)[i] = f32_to_bf16(v); break;
    default: ((_Float16 *)p)[i] = (_Float16)v; break;
    }
}

/* value rounded to the storage precision of dtype dt */
static inline float round_to(int dt, float v) {
    switch (dt) {
    case QREF_F32: return v;
    case QREF_BF16: return rnd_bf16(v);
    default: return (float)(_Float16)v;
    }
}

/* ---------------------------------------------------------------- quantize */

/* One (row, group): MLX affine quantization, restated.  Returns the codes in
 * q[0..gs) and the fp32 scale / bias.  Order of operations is the one that
 * reproduces the fixture bit-exactly. */
static void quant_group(const float *w, int gs, int bits, uint32_t *q, float *scale_out,
                        float *bias_out) {
    float wmin = w[0], wmax = w[0];
    for (int i = 1; i < gs; ++i) {
        wmin = fminf(wmin, w[i]);
        wmax = fmaxf(wmax, w[i]);
    }
    const float n_bins = (float)((1 << bits) - 1);
    const float eps = 1e-7f;
    float s = fmaxf((wmax - wmin) / n_bins, eps);
    const int neg_side = fabsf(wmin) > fabsf(wmax);
    s = neg_side ? s : -s;
    const float edge = neg_side ? wmin : wmax;
    const float q0 = rintf(edge / s);
    float b = 0.0f;
    if (q0 != 0.0f) {
        s = edge / q0;
        b = edge;
    }
    for (int i = 0; i < gs; ++i) {
        float c = rintf((w[i] - b) / s);
        c = fminf(fmaxf(c, 0.0f), n_bins);
        q[i] = (uint32_t)c;
    }
    *scale_out = s;
    *bias_out = b;
}

int qref_quantize(const void *w, int w_dtype, int64_t N, int64_t K, int gs, int bits,
                  uint32_t *wq, void *scales, void *biases, int sb_dtype) {
    if (bits != 4 && bits != 8) return 2;
    if (gs != 32 && gs != 64 && gs != 128) return 2;
    if (K % gs) return 1;
    const int epw = 32 / bits;
    const int64_t G = K / gs;
    float buf[128];
    uint32_t q[128];
    for (int64_t n = 0; n < N; ++n) {
        for (int64_t g = 0; g < G; ++g) {
            for (int i = 0; i < gs; ++i) buf[i] = load_el(w, w_dtype, n * K + g * gs + i);
            float s, b;
            quant_group(buf, gs, bits, q, &s, &b);
            store_el(scales, sb_dtype, n * G + g, s);
            store_el(biases, sb_dtype, n * G + g, b);
            for (int i = 0; i < gs; i += epw) {
                uint32_t word = 0;
                for (int j = 0; j < epw; ++j) word |= q[i + j] << (bits * j);
                wq[(n * K + g * gs + i) / epw] = word;
            }
        }
    }
    return 0;
}

/* ---------------------------------------------------------------- dequantize */

static inline uint32_t code_at(const uint32_t *row_words, int bits, int64_t k) {
    const int epw = 32 / bits;
    return (row_words[k / epw] >> (bits * (k % epw))) & ((1u << bits) - 1u);
}

/* w = fma(q, scale, bias) in fp32, one rounding to out_dtype.  ids (optional)
 * selects the packed rows (quantized embedding gather, src/nn.rs:51-56). */
int qref_dequantize(const uint32_t *wq, const void *scales, const void *biases, int sb_dtype,
                    int64_t N, int64_t K, int gs, int bits, const int64_t *ids, int64_t R,
                    void *out, int out_dtype) {
    if (bits != 4 && bits != 8) return 2;
    if (K % gs) return 1;
    const int64_t G = K / gs, W = K * bits / 32;
    const int64_t rows = ids ? R : N;
    for (int64_t r = 0; r < rows; ++r) {
        const int64_t n = ids ? ids[r] : r;
        if (n < 0 || n >= N) return 1;
        for (int64_t k = 0; k < K; ++k) {
            float s = load_el(scales, sb_dtype, n * G + k / gs);
            float b = load_el(biases, sb_dtype, n * G + k / gs);
            float v = fmaf((float)code_at(wq + n * W, bits, k), s, b);
            store_el(out, out_dtype, r * K + k, v);
        }
    }
    return 0;
}

/* ---------------------------------------------------------------- epilogue math */

#define QREF_ACT_NONE 0
#define QREF_ACT_GELU_TANH 1
#define QREF_ACT_GELU_ERF 2

/* reference gelu_tanh in dtype dt: every op rounds to dt (src/nn.rs:321-329) */
static float gelu_tanh_ref(float x, int dt) {
    const float c = (float)sqrt(2.0 / 3.14159265358979323846);
    const float k1 = round_to(dt, 0.044715f), kc = round_to(dt, c);
    const float half = round_to(dt, 0.5f), one = round_to(dt, 1.0f);
    float x3 = round_to(dt, x * x * x);
    float inner = round_to(dt, round_to(dt, x + round_to(dt, x3 * k1)) * kc);
    float gate = round_to(dt, round_to(dt, tanhf(inner)) + one);
    return round_to(dt, round_to(dt, x * half) * gate);
}

/* reference exact gelu in dtype dt: x * (1 + erf(x / sqrt2)) / 2 (src/nn.rs:344-355) */
static float gelu_erf_ref(float x, int dt) {
    const float r2 = round_to(dt, (float)sqrt(2.0));
    float inner = round_to(dt, erff(round_to(dt, x / r2)));
    float gate = round_to(dt, round_to(dt, 1.0f) + inner);
    return round_to(dt, round_to(dt, x * gate) / round_to(dt, 2.0f));
}

/* reference silu(a) * b in dtype dt (mlx-gen-z-image/src/feed_forward.rs:61-70) */
static float swiglu_ref(float a, float b, int dt) {
    float sig = round_to(dt, 1.0f / (1.0f + expf(-a)));
    return round_to(dt, round_to(dt, a * sig) * b);
}

/* ---------------------------------------------------------------- quantized_matmul */

/* Exact-mode quantized_matmul with the reference's rounding points:
 *   y0  = round_out( sum_k x[m,k] * deq[n,k] )   (double accumulation, deq rounded to
 *                                                  the scales' dtype as MLX's kernels do)
 *   y1  = round_out( y0 + bias[n] )              (separate op, src/adapters.rs:318-320)
 *   lora: t = round_out(x.A) ; r = round_out(t.B) ; r = round_out(r * scale);
 *         y2 = round_out(y1 + r)                  (src/adapters.rs:260-270, 545-547)
 *   act: applied to y (after bias) with the reference's op-by-op rounding.
 * For swiglu, the caller passes two weight sets via qref_qmm twice and combines
 * with qref_swiglu.  out dtype = x dtype (bf16 activations -> bf16 outputs). */
int qref_qmm(const void *x, int x_dtype, int64_t M, int64_t K, const uint32_t *wq,
             const void *scales, const void *biases, int sb_dtype, int64_t N, int gs, int bits,
             const void *bias, int act, const void *lora_a, const void *lora_b, int64_t rank,
             float lora_scale, void *y, int y_dtype) {
    if (bits != 4 && bits != 8) return 2;
    if (K % gs) return 1;
    const int64_t G = K / gs, W = K * bits / 32;
    float *deq = (float *)malloc(sizeof(float) * (size_t)K);
    double *xd = (double *)malloc(sizeof(double) * (size_t)(M * K));
    float *t = NULL;
    if (!deq || !xd) { free(deq); free(xd); return 3; }
    for (int64_t i = 0; i < M * K; ++i) xd[i] = load_el(x, x_dtype, i);
    if (lora_a && rank > 0) {
        t = (float *)malloc(sizeof(float) * (size_t)(M * rank));
        for (int64_t m = 0; m < M; ++m)
            for (int64_t r = 0; r < rank; ++r) {
                double acc = 0;
                for (int64_t k = 0; k < K; ++k) acc += xd[m * K + k] * load_el(lora_a, y_dtype, k * rank + r);
                t[m * rank + r] = round_to(y_dtype, (float)acc);
            }
    }
    for (int64_t n = 0; n < N; ++n) {
        for (int64_t k = 0; k < K; ++k) {
            float s = load_el(scales, sb_dtype, n * G + k / gs);
            float b = load_el(biases, sb_dtype, n * G + k / gs);
            /* the dequantized weight in the computation dtype, promote(x, scales) = the
               output dtype (mlx casts the operands of quantized_matmul to it): bf16 x with bf16
               scales rounds w to bf16; f32 or mixed-dtype activations keep the fp32 value */
            deq[k] = round_to(y_dtype, fmaf((float)code_at(wq + n * W, bits, k), s, b));
        }
        for (int64_t m = 0; m < M; ++m) {
            double acc = 0;
            const double *xr = xd + m * K;
            for (int64_t k = 0; k < K; ++k) acc += xr[k] * (double)deq[k];
            float v = round_to(y_dtype, (float)acc);
            if (bias) v = round_to(y_dtype, v + load_el(bias, y_dtype, n));
            if (t) {
                double r = 0;
                for (int64_t j = 0; j < rank; ++j) r += (double)t[m * rank + j] * load_el(lora_b, y_dtype, j * N + n);
                float rv = round_to(y_dtype, (float)r);
                rv = round_to(y_dtype, rv * round_to(y_dtype, lora_scale));
                v = round_to(y_dtype, v + rv);
            }
            if (act == QREF_ACT_GELU_TANH) v = gelu_tanh_ref(v, y_dtype);
            else if (act == QREF_ACT_GELU_ERF) v = gelu_erf_ref(v, y_dtype);
            store_el(y, y_dtype, m * N + n, v);
        }
    }
    free(t);
    free(deq);
    free(xd);
    return 0;
}

/* out[i] = swiglu(a[i], b[i]) with reference rounding, all in dtype dt */
void qref_swiglu(const void *a, const void *b, int64_t n, int dt, void *out) {
    for (int64_t i = 0; i < n; ++i) store_el(out, dt, i, swiglu_ref(load_el(a, dt, i), load_el(b, dt, i), dt));
}

/* ---------------------------------------------------------------- fast mode (CPU baseline) */

/* The timed CPU baseline: same math as qref_qmm without LoRA/act, fp32 accumulation.
 * Each worker owns a contiguous range of output columns n; per column it dequantizes
 * one row of W (rounded to the scales' dtype) and dots it with every row of x,
 * four rows at a time.  Threads are plain pthreads (no OpenMP runtime here). */
typedef struct {
    const float *xf;
    int64_t M, K, N, n0, n1;
    const uint32_t *wq;
    const void *scales, *biases, *bias;
    int sb_dtype, gs, bits, y_dtype;
    void *y;
} fast_job;

static void *fast_worker(void *arg) {
    const fast_job *j = (const fast_job *)arg;
    const int64_t K = j->K, M = j->M, N = j->N, G = K / j->gs, W = K * j->bits / 32;
    float *deq = (float *)malloc(sizeof(float) * (size_t)K);
    if (!deq) return NULL;
    for (int64_t n = j->n0; n < j->n1; ++n) {
        const uint32_t *row = j->wq + n * W;
        for (int64_t g = 0; g < G; ++g) {
            const float s = load_el(j->scales, j->sb_dtype, n * G + g);
            const float b = load_el(j->biases, j->sb_dtype, n * G + g);
            for (int i = 0; i < j->gs; ++i) {
                const int64_t k = g * j->gs + i;
                deq[k] = round_to(j->sb_dtype, fmaf((float)code_at(row, j->bits, k), s, b));
            }
        }
        int64_t m = 0;
        for (; m + 4 <= M; m += 4) {
            const float *x0 = j->xf + m * K, *x1 = x0 + K, *x2 = x1 + K, *x3 = x2 + K;
            float a0 = 0, a1 = 0, a2 = 0, a3 = 0;
            for (int64_t k = 0; k < K; ++k) {
                const float d = deq[k];
                a0 += x0[k] * d; a1 += x1[k] * d; a2 += x2[k] * d; a3 += x3[k] * d;
            }
            float acc[4] = {a0, a1, a2, a3};
            for (int q = 0; q < 4; ++q) {
                float v = round_to(j->y_dtype, acc[q]);
                if (j->bias) v = round_to(j->y_dtype, v + load_el(j->bias, j->y_dtype, n));
                store_el(j->y, j->y_dtype, (m + q) * N + n, v);
            }
        }
        for (; m < M; ++m) {
            float a = 0;
            const float *xr = j->xf + m * K;
            for (int64_t k = 0; k < K; ++k) a += xr[k] * deq[k];
            float v = round_to(j->y_dtype, a);
            if (j->bias) v = round_to(j->y_dtype, v + load_el(j->bias, j->y_dtype, n));
            store_el(j->y, j->y_dtype, m * N + n, v);
        }
    }
    free(deq);
    return NULL;
}

int qref_qmm_fast(const void *x, int x_dtype, int64_t M, int64_t K, const uint32_t *wq,
                  const void *scales, const void *biases, int sb_dtype, int64_t N, int gs,
                  int bits, const void *bias, void *y, int y_dtype, int nthreads) {
    if (bits != 4 && bits != 8) return 2;
    if (K % gs) return 1;
    if (nthreads < 1) nthreads = 1;
    if (nthreads > 256) nthreads = 256;
    float *xf = (float *)malloc(sizeof(float) * (size_t)(M * K));
    if (!xf) return 3;
    for (int64_t i = 0; i < M * K; ++i) xf[i] = load_el(x, x_dtype, i);
    pthread_t th[256];
    fast_job jobs[256];
    const int64_t per = (N + nthreads - 1) / nthreads;
    int started = 0;
    for (int t = 0; t < nthreads; ++t) {
        fast_job jb = {xf, M, K, N, t * per, (t + 1) * per < N ? (t + 1) * per : N, wq,
                       scales, biases, bias, sb_dtype, gs, bits, y_dtype, y};
        jobs[t] = jb;
        if (jobs[t].n0 >= jobs[t].n1) break;
        if (pthread_create(&th[t], NULL, fast_worker, &jobs[t]) != 0) { fast_worker(&jobs[t]); continue; }
        started = t + 1;
    }
    for (int t = 0; t < started; ++t) pthread_join(th[t], NULL);
    free(xf);
    return 0;
}

/* fp32 -> bf16 / bf16 -> fp32 helpers for the Python side */
void qref_f32_to_bf16(const float *in, uint16_t *out, int64_t n) {
    for (int64_t i = 0; i < n; ++i) out[i] = f32_to_bf16(in[i]);
}
