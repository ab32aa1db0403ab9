// modulate.cu -- the adaLN prologue of the DiT linears in one pass:
//     y = (1 + scale) * layer_norm(x) + shift
// as FLUX's blocks compute it before their QKV / MLP linears
// (mlx-gen-flux/src/transformer.rs:891-913 -> mlx_rs::fast::layer_norm(x, None, None, eps)
// and src/nn.rs:262-287 `modulate`).  HBM-bound: one read of x, one write of y.
//
// Rounding follows the reference's op sequence on bf16 arrays: the normalisation is
// computed in fp32 (mean, then the variance of x - mean) and rounded to bf16; with a bf16
// output (FLUX.1: the literal 1 cast to scale's dtype) 1 + scale, the product and the sum
// are each rounded to bf16; with an f32 output (FLUX.2: a strong f32 1) they are f32.
// scale / shift: [rows, D] with row m / period (period 0: one row for every m), or NULL
// (plain layer norm).
#include "ql_common.cuh"

namespace ql {
namespace modulate_k {

constexpr int THREADS = 256;

__device__ __forceinline__ float block_sum(float v, float *red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();  // red is reused between calls
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float t = 0.f;
#pragma unroll
    for (int w = 0; w < THREADS / 32; ++w) t += red[w];
    return t;
}

// the same over a block of any whole number of warps (red holds 32 floats)
__device__ __forceinline__ float block_sum_n(float v, float *red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float t = 0.f;
    for (int w = 0; w < nw; ++w) t += red[w];
    return t;
}

// one CTA per row; rows of a few KB stay in L1 between the passes
template <bool F32_OUT>
__global__ void __launch_bounds__(THREADS) ln_modulate_kernel(const __nv_bfloat16 *__restrict__ x, int D, float eps,
                                                              const __nv_bfloat16 *__restrict__ scale,
                                                              const __nv_bfloat16 *__restrict__ shift, int64_t period,
                                                              void *__restrict__ y) {
    __shared__ float red[THREADS / 32];
    const int64_t m = blockIdx.x;
    const __nv_bfloat16 *xr = x + m * D;
    const int D2 = D / 2;  // D is even; bf16 pairs
    const __nv_bfloat162 *x2 = reinterpret_cast<const __nv_bfloat162 *>(xr);
    float s = 0.f;
    for (int i = threadIdx.x; i < D2; i += THREADS) {
        const float2 v = __bfloat1622float2(x2[i]);
        s += v.x + v.y;
    }
    const float mean = block_sum(s, red) / (float)D;
    float q = 0.f;
    for (int i = threadIdx.x; i < D2; i += THREADS) {
        const float2 v = __bfloat1622float2(x2[i]);
        const float a = v.x - mean, b = v.y - mean;
        q += a * a + b * b;
    }
    const float var = block_sum(q, red) / (float)D;
    const float inv = 1.0f / sqrtf(var + eps);
    const int64_t gr = period > 0 ? m / period : 0;
    const __nv_bfloat16 *sc = scale ? scale + gr * D : nullptr;
    const __nv_bfloat16 *sh = shift ? shift + gr * D : nullptr;
    for (int i = threadIdx.x; i < D2; i += THREADS) {
        const float2 v = __bfloat1622float2(x2[i]);
        float n[2] = {round_bf16((v.x - mean) * inv), round_bf16((v.y - mean) * inv)};
        float o[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int k = 2 * i + h;
            float r = n[h];
            if (sc) {
                const float s1 = __bfloat162float(sc[k]) + 1.0f;
                r = F32_OUT ? r * s1 : round_bf16(r * round_bf16(s1));
                if (!F32_OUT) r = round_bf16(r);
            }
            if (sh) r = r + __bfloat162float(sh[k]);
            o[h] = r;
        }
        if (F32_OUT)
            reinterpret_cast<float2 *>(y)[m * D2 + i] = make_float2(o[0], o[1]);
        else
            reinterpret_cast<uint32_t *>(y)[m * D2 + i] = pack_bf16x2(o[0], o[1]);
    }
}

// The same computation with the row held in registers: each thread loads its MAXC 16-byte
// chunks of x (and of scale / shift) once, so x is read from HBM exactly once and the two
// statistics passes and the output pass run on registers.  The block is sized to the row
// (ceil(D / 8 / MAXC) threads rounded up to a warp, D a multiple of 8, D <= 8 * 1024 *
// MAXC), so that short rows (FLUX's 3072: 96 threads) leave room for many rows in flight
// on each SM -- one 256-thread block per row held too few bytes in flight per SM to
// cover HBM latency.
constexpr int MAXC = 4;
template <bool F32_OUT>
__global__ void __launch_bounds__(1024) ln_modulate_reg_kernel(const __nv_bfloat16 *__restrict__ x, int D, float eps,
                                                                  const __nv_bfloat16 *__restrict__ scale,
                                                                  const __nv_bfloat16 *__restrict__ shift,
                                                                  int64_t period, void *__restrict__ y) {
    __shared__ float red[32];
    const int64_t m = blockIdx.x;
    const int nch = D / 8, nt = blockDim.x;
    uint4 xv[MAXC];
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < MAXC; ++j) {
        const int c = threadIdx.x + j * nt;
        xv[j] = c < nch ? __ldg(reinterpret_cast<const uint4 *>(x + m * D) + c) : make_uint4(0, 0, 0, 0);
        const uint32_t w[4] = {xv[j].x, xv[j].y, xv[j].z, xv[j].w};
#pragma unroll
        for (int i = 0; i < 4; ++i) s += bf16lo(w[i]) + bf16hi(w[i]);
    }
    const float mean = block_sum_n(s, red) / (float)D;
    float q = 0.f;
#pragma unroll
    for (int j = 0; j < MAXC; ++j) {
        if (threadIdx.x + j * nt >= nch) continue;
        const uint32_t w[4] = {xv[j].x, xv[j].y, xv[j].z, xv[j].w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float a = bf16lo(w[i]) - mean, b = bf16hi(w[i]) - mean;
            q += a * a + b * b;
        }
    }
    const float var = block_sum_n(q, red) / (float)D;
    const float inv = 1.0f / sqrtf(var + eps);
    const int64_t gr = period > 0 ? m / period : 0;
#pragma unroll
    for (int j = 0; j < MAXC; ++j) {
        const int c = threadIdx.x + j * nt;
        if (c >= nch) continue;
        const uint32_t w[4] = {xv[j].x, xv[j].y, xv[j].z, xv[j].w};
        uint4 scv = make_uint4(0, 0, 0, 0), shv = scv;
        if (scale) scv = __ldg(reinterpret_cast<const uint4 *>(scale + gr * D) + c);
        if (shift) shv = __ldg(reinterpret_cast<const uint4 *>(shift + gr * D) + c);
        const uint32_t sw[4] = {scv.x, scv.y, scv.z, scv.w}, hw[4] = {shv.x, shv.y, shv.z, shv.w};
        float o[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float v = (i & 1) ? bf16hi(w[i >> 1]) : bf16lo(w[i >> 1]);
            float r = round_bf16((v - mean) * inv);
            if (scale) {
                const float s1 = ((i & 1) ? bf16hi(sw[i >> 1]) : bf16lo(sw[i >> 1])) + 1.0f;
                r = F32_OUT ? r * s1 : round_bf16(r * round_bf16(s1));
            }
            if (shift) r = r + ((i & 1) ? bf16hi(hw[i >> 1]) : bf16lo(hw[i >> 1]));
            o[i] = r;
        }
        if (F32_OUT) {
            float4 *yp = reinterpret_cast<float4 *>(reinterpret_cast<float *>(y) + m * D) + 2 * c;
            yp[0] = make_float4(o[0], o[1], o[2], o[3]);
            yp[1] = make_float4(o[4], o[5], o[6], o[7]);
        } else {
            reinterpret_cast<uint4 *>(reinterpret_cast<__nv_bfloat16 *>(y) + m * D)[c] =
                make_uint4(pack_bf16x2(o[0], o[1]), pack_bf16x2(o[2], o[3]), pack_bf16x2(o[4], o[5]),
                           pack_bf16x2(o[6], o[7]));
        }
    }
}

}  // namespace modulate_k

int launch_ln_modulate(const void *x, int64_t M, int64_t D, float eps, const void *scale, const void *shift,
                       int64_t period, void *y, int y_dtype, cudaStream_t st) {
    if (M <= 0) return QL_OK;
    const dim3 grid((unsigned)M);
    const bool al = ((reinterpret_cast<uintptr_t>(scale) | reinterpret_cast<uintptr_t>(shift)) & 15) == 0;
    if (D <= 8 * 1024 * modulate_k::MAXC && al) {
        const int nt = (int)((((D / 8 + modulate_k::MAXC - 1) / modulate_k::MAXC) + 31) / 32 * 32);
        if (y_dtype == QL_F32)
            modulate_k::ln_modulate_reg_kernel<true><<<grid, nt, 0, st>>>(
                (const __nv_bfloat16 *)x, (int)D, eps, (const __nv_bfloat16 *)scale, (const __nv_bfloat16 *)shift,
                period, y);
        else
            modulate_k::ln_modulate_reg_kernel<false><<<grid, nt, 0, st>>>(
                (const __nv_bfloat16 *)x, (int)D, eps, (const __nv_bfloat16 *)scale, (const __nv_bfloat16 *)shift,
                period, y);
        QL_CUDA_TRY(cudaGetLastError());
        return QL_OK;
    }
    if (y_dtype == QL_F32)
        modulate_k::ln_modulate_kernel<true><<<grid, modulate_k::THREADS, 0, st>>>(
            (const __nv_bfloat16 *)x, (int)D, eps, (const __nv_bfloat16 *)scale, (const __nv_bfloat16 *)shift, period, y);
    else
        modulate_k::ln_modulate_kernel<false><<<grid, modulate_k::THREADS, 0, st>>>(
            (const __nv_bfloat16 *)x, (int)D, eps, (const __nv_bfloat16 *)scale, (const __nv_bfloat16 *)shift, period, y);
    QL_CUDA_TRY(cudaGetLastError());
    return QL_OK;
}

}  // namespace ql
