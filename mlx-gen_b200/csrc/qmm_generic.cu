// qmm_generic.cu -- CUDA-core quantized matmul for any dtype combination, and
// the LoRA pre-pass used by the tensor-core kernels.
//
// The generic kernel serves the f32 / f16 activation paths (the reference runs
// FLUX.2's and Qwen's f32 image streams through the same quantized_matmul,
// src/adapters.rs:301-308) and is a GPU-side cross-check of the fast kernels.
// It dequantizes W tiles into shared memory with the same rounding as
// ql_dequantize (fma in fp32, rounded to the scales' dtype, as MLX's kernels
// hold dequantized weights in that dtype) and accumulates in fp32.
#include "ql_common.cuh"

namespace ql {

namespace generic {

constexpr int TM = 32, TN = 32, TK = 32;  // 256 threads, 2x2 outputs each

__device__ __forceinline__ float round_to(int dt, float v) {
    if (dt == QL_F32) return v;
    if (dt == QL_BF16) return round_bf16(v);
    return __half2float(__float2half_rn(v));
}

struct Params {
    const void *x;
    int xdt;
    int M, N, K, gs, G, bits;
    const uint32_t *wq[2];
    const void *scales[2], *biases[2];
    int sdt;
    const void *bias[2];
    const void *lora_a, *lora_b;  // x's dtype
    int rank;
    float lora_scale;
    int act;
    void *y;
    int ydt;
};

__device__ __forceinline__ float act_f(float v, int act) {
    if (act == QL_ACT_GELU_TANH) return 0.5f * v * (1.0f + tanhf(0.7978845608028654f * (v + 0.044715f * v * v * v)));
    if (act == QL_ACT_GELU_ERF) return 0.5f * v * (1.0f + erff(v * 0.7071067811865476f));
    return v;
}

__global__ void __launch_bounds__(256) qmm_generic_kernel(const Params p) {
    __shared__ float xs[TM][TK + 1];
    __shared__ float ws[2][TN][TK + 1];
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    const int m0 = blockIdx.y * TM, n0 = blockIdx.x * TN;
    const int npass = p.act == QL_ACT_SWIGLU ? 2 : 1;
    const int epw = 32 / p.bits;
    const int64_t wpr = (int64_t)p.K / epw;
    float acc[2][2][2] = {};
    for (int k0 = 0; k0 < p.K; k0 += TK) {
        for (int i = threadIdx.x; i < TM * TK; i += 256) {
            const int r = i / TK, kk = i % TK;
            const int m = m0 + r, k = k0 + kk;
            xs[r][kk] = (m < p.M && k < p.K) ? load_as_f32(p.x, p.xdt, (int64_t)m * p.K + k) : 0.f;
        }
        for (int ps = 0; ps < npass; ++ps)
            for (int i = threadIdx.x; i < TN * TK; i += 256) {
                const int r = i / TK, kk = i % TK;
                const int n = n0 + r, k = k0 + kk;
                float v = 0.f;
                if (n < p.N && k < p.K) {
                    const uint32_t w = p.wq[ps][(int64_t)n * wpr + k / epw];
                    const uint32_t code = (w >> (p.bits * (k % epw))) & ((1u << p.bits) - 1u);
                    const int64_t g = (int64_t)n * p.G + k / p.gs;
                    v = round_to(p.sdt, fmaf((float)code, load_as_f32(p.scales[ps], p.sdt, g),
                                             load_as_f32(p.biases[ps], p.sdt, g)));
                }
                ws[ps][r][kk] = v;
            }
        __syncthreads();
        for (int kk = 0; kk < TK; ++kk)
            for (int ps = 0; ps < npass; ++ps)
#pragma unroll
                for (int a = 0; a < 2; ++a)
#pragma unroll
                    for (int b = 0; b < 2; ++b)
                        acc[ps][a][b] += xs[ty * 2 + a][kk] * ws[ps][tx * 2 + b][kk];
        __syncthreads();
    }
    for (int a = 0; a < 2; ++a)
        for (int b = 0; b < 2; ++b) {
            const int m = m0 + ty * 2 + a, n = n0 + tx * 2 + b;
            if (m >= p.M || n >= p.N) continue;
            float lora = 0.f;
            if (p.lora_a) {
                for (int j = 0; j < p.rank; ++j) {
                    float t = 0.f;
                    for (int k = 0; k < p.K; ++k)
                        t += load_as_f32(p.x, p.xdt, (int64_t)m * p.K + k) *
                             load_as_f32(p.lora_a, p.xdt, (int64_t)k * p.rank + j);
                    lora += t * load_as_f32(p.lora_b, p.xdt, (int64_t)j * p.N + n);
                }
                lora *= p.lora_scale;
            }
            float v = round_to(p.ydt, acc[0][a][b] + lora);
            if (p.bias[0]) v = round_to(p.ydt, v + load_as_f32(p.bias[0], p.ydt, n));
            if (p.act == QL_ACT_SWIGLU) {
                float u = round_to(p.ydt, acc[1][a][b]);
                if (p.bias[1]) u = round_to(p.ydt, u + load_as_f32(p.bias[1], p.ydt, n));
                v = v / (1.0f + expf(-v)) * u;
            } else {
                v = act_f(v, p.act);
            }
            store_from_f32(p.y, p.ydt, (int64_t)m * p.N + n, v);
        }
}

// T[m, j] = bf16(scale * sum_k x[m,k] A[k,j]) for j < rank, 0 for rank <= j < rpad.
// One CTA per 32 rows of x; x and A chunks are staged through shared memory.
__global__ void __launch_bounds__(256) lora_t_kernel(const __nv_bfloat16 *__restrict__ x, int M, int K,
                                                     const __nv_bfloat16 *__restrict__ A, int rank, int rpad,
                                                     float scale, __nv_bfloat16 *__restrict__ T) {
    constexpr int R = 32, KC = 64;
    __shared__ float xs[R][KC + 1];
    __shared__ float as[KC][64 + 1];
    const int m0 = blockIdx.x * R;
    for (int jb = 0; jb < rpad; jb += 64) {
        // each thread: row r = tid / 8, columns jb + (tid % 8) + 8*c, c < 8
        const int r = threadIdx.x >> 3, cj = threadIdx.x & 7;
        float acc[8] = {};
        for (int k0 = 0; k0 < K; k0 += KC) {
            for (int i = threadIdx.x; i < R * KC; i += 256) {
                const int rr = i / KC, kk = i % KC, m = m0 + rr, k = k0 + kk;
                xs[rr][kk] = (m < M && k < K) ? __bfloat162float(x[(int64_t)m * K + k]) : 0.f;
            }
            for (int i = threadIdx.x; i < KC * 64; i += 256) {
                const int kk = i / 64, jj = i % 64, k = k0 + kk, j = jb + jj;
                as[kk][jj] = (k < K && j < rank) ? __bfloat162float(A[(int64_t)k * rank + j]) : 0.f;
            }
            __syncthreads();
            for (int kk = 0; kk < KC; ++kk) {
                const float xv = xs[r][kk];
#pragma unroll
                for (int c = 0; c < 8; ++c) acc[c] += xv * as[kk][cj + 8 * c];
            }
            __syncthreads();
        }
        const int m = m0 + r;
        if (m < M)
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                const int j = jb + cj + 8 * c;
                T[(int64_t)m * rpad + j] = __float2bfloat16_rn(j < rank ? scale * acc[c] : 0.f);
            }
    }
}

}  // namespace generic

int launch_qmm_generic(const void *x, int xdt, int64_t M, int64_t K, const uint32_t *wq,
                       const void *scales, const void *biases, const uint32_t *wq2,
                       const void *scales2, const void *biases2, int sdt, int64_t N, int gs,
                       int bits, const void *bias, const void *bias2, int act, const void *lora_a,
                       const void *lora_b, int64_t rank, float lora_scale, void *y, int ydt,
                       cudaStream_t st) {
    generic::Params p{};
    p.x = x;
    p.xdt = xdt;
    p.M = (int)M;
    p.N = (int)N;
    p.K = (int)K;
    p.gs = gs;
    p.G = (int)(K / gs);
    p.bits = bits;
    p.wq[0] = wq;
    p.wq[1] = wq2;
    p.scales[0] = scales;
    p.scales[1] = scales2;
    p.biases[0] = biases;
    p.biases[1] = biases2;
    p.sdt = sdt;
    p.bias[0] = bias;
    p.bias[1] = bias2;
    p.lora_a = lora_a;
    p.lora_b = lora_b;
    p.rank = (int)rank;
    p.lora_scale = lora_scale;
    p.act = act;
    p.y = y;
    p.ydt = ydt;
    dim3 grid((unsigned)((N + generic::TN - 1) / generic::TN), (unsigned)((M + generic::TM - 1) / generic::TM));
    generic::qmm_generic_kernel<<<grid, 256, 0, st>>>(p);
    QL_CUDA_TRY(cudaGetLastError());
    return QL_OK;
}

int launch_lora_t(const void *x, int64_t M, int64_t K, const void *A, int64_t rank, float scale,
                  void *T, cudaStream_t st) {
    const int rpad = (int)((rank + 63) / 64 * 64);
    const int grid = (int)((M + 31) / 32);
    generic::lora_t_kernel<<<grid, 256, 0, st>>>((const __nv_bfloat16 *)x, (int)M, (int)K,
                                                  (const __nv_bfloat16 *)A, (int)rank, rpad, scale,
                                                  (__nv_bfloat16 *)T);
    QL_CUDA_TRY(cudaGetLastError());
    return QL_OK;
}

}  // namespace ql
