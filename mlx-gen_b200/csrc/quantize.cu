// quantize.cu -- group-wise affine quantize / dequantize kernels.
//
// Both kernels are HBM-bound streaming kernels: one thread per packed uint32
// word (8 Q4 codes or 4 Q8 codes), so a warp reads/writes contiguous 128-byte
// segments.  A group of `gs` elements is covered by gs*bits/32 consecutive
// lanes; the group's min/max is a shuffle-xor reduction among them.
//
// Arithmetic follows MLX affine quantization as the reference calls it
// (src/quant.rs:140, src/adapters.rs:533-537; restated and pinned against the
// reference fixture in oracle/qref.c quant_group()).  Every division is an
// IEEE round-to-nearest division and no multiply-add is contracted, so the
// codes, scales and biases are bit-identical to the oracle.
#include "ql_common.cuh"

namespace ql {

template <int BITS>
struct WordIO {
    static constexpr int EPW = 32 / BITS;  // elements per packed word
};

// Load EPW consecutive elements of row-major input starting at element index e.
template <int EPW>
__device__ __forceinline__ void load_elems(const void *w, int dt, int64_t e, float (&v)[EPW]) {
    if (dt == QL_F32) {
        const float4 *p = reinterpret_cast<const float4 *>(reinterpret_cast<const float *>(w) + e);
#pragma unroll
        for (int i = 0; i < EPW / 4; ++i) {
            float4 f = __ldg(p + i);
            v[4 * i + 0] = f.x; v[4 * i + 1] = f.y; v[4 * i + 2] = f.z; v[4 * i + 3] = f.w;
        }
    } else {
        // 16-bit inputs: EPW*2 bytes = 16 (Q4) or 8 (Q8)
        const uint16_t *p = reinterpret_cast<const uint16_t *>(w) + e;
        uint32_t raw[EPW / 2];
        if constexpr (EPW == 8) {
            uint4 r = __ldg(reinterpret_cast<const uint4 *>(p));
            raw[0] = r.x; raw[1] = r.y; raw[2] = r.z; raw[3] = r.w;
        } else {
            uint2 r = __ldg(reinterpret_cast<const uint2 *>(p));
            raw[0] = r.x; raw[1] = r.y;
        }
#pragma unroll
        for (int i = 0; i < EPW / 2; ++i) {
            if (dt == QL_BF16) {
                v[2 * i] = bf16lo(raw[i]);
                v[2 * i + 1] = bf16hi(raw[i]);
            } else {
                __half2 h = *reinterpret_cast<__half2 *>(&raw[i]);
                float2 f = __half22float2(h);
                v[2 * i] = f.x;
                v[2 * i + 1] = f.y;
            }
        }
    }
}

template <int BITS>
__global__ void __launch_bounds__(256) quantize_kernel(const void *__restrict__ w, int w_dtype,
                                                       int64_t total_words, int gs,
                                                       uint32_t *__restrict__ wq,
                                                       void *__restrict__ scales,
                                                       void *__restrict__ biases, int sb_dtype) {
    constexpr int EPW = 32 / BITS;
    const int tpg = gs / EPW;  // lanes per group: power of two in [4, 32]
    const float n_bins = (float)((1 << BITS) - 1);
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    // total_words is a multiple of tpg, and tpg divides 32, so every lane of a
    // group runs the same number of iterations (the shuffles stay converged).
    for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
         t - (threadIdx.x & 31) < total_words; t += stride) {
        const bool live = t < total_words;
        float v[EPW];
        if (live) load_elems<EPW>(w, w_dtype, t * EPW, v);
        else {
#pragma unroll
            for (int i = 0; i < EPW; ++i) v[i] = 0.f;
        }
        float mn = v[0], mx = v[0];
#pragma unroll
        for (int i = 1; i < EPW; ++i) {
            mn = fminf(mn, v[i]);
            mx = fmaxf(mx, v[i]);
        }
        for (int o = 1; o < tpg; o <<= 1) {
            mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        }
        if (!live) continue;
        float s = fmaxf(__fdiv_rn(__fsub_rn(mx, mn), n_bins), 1e-7f);
        const bool neg_side = fabsf(mn) > fabsf(mx);
        s = neg_side ? s : -s;
        const float edge = neg_side ? mn : mx;
        const float q0 = rintf(__fdiv_rn(edge, s));
        float b = 0.0f;
        if (q0 != 0.0f) {
            s = __fdiv_rn(edge, q0);
            b = edge;
        }
        uint32_t word = 0;
#pragma unroll
        for (int i = 0; i < EPW; ++i) {
            float c = rintf(__fdiv_rn(__fsub_rn(v[i], b), s));
            c = fminf(fmaxf(c, 0.0f), n_bins);
            word |= (uint32_t)c << (BITS * i);
        }
        wq[t] = word;
        if ((t % tpg) == 0) {
            const int64_t g = t / tpg;
            store_from_f32(scales, sb_dtype, g, s);
            store_from_f32(biases, sb_dtype, g, b);
        }
    }
}

// One thread per packed word of the output rows.  ids == nullptr: row r reads
// packed row r; otherwise packed row ids[r] (quantized embedding gather).  round_sb: the
// value is first rounded to the scales' dtype (mlx's dequantize output) and then converted
// to out_dtype, as the reference's gather + dequantize + cast does.
template <int BITS>
__global__ void __launch_bounds__(256) dequantize_kernel(
    const int64_t *__restrict__ ids, int64_t rows, int64_t N, int64_t words_per_row, int gs,
    const uint32_t *__restrict__ wq, const void *__restrict__ scales,
    const void *__restrict__ biases, int sb_dtype, void *__restrict__ out, int out_dtype, bool round_sb) {
    constexpr int EPW = 32 / BITS;
    const int64_t total = rows * words_per_row;
    const int64_t G = words_per_row * EPW / gs;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total; t += stride) {
        const int64_t r = t / words_per_row, wi = t - r * words_per_row;
        int64_t n = r;
        bool ok = true;
        if (ids) {
            n = __ldg(ids + r);
            if (n < 0 || n >= N) {
                ok = false;
                if (wi == 0) raise_dev_error(DEV_ERR_BAD_INDEX);
            }
        }
        float o[EPW];
        if (ok) {
            const uint32_t word = __ldg(wq + n * words_per_row + wi);
            const int64_t g = n * G + (wi * EPW) / gs;
            const float s = load_as_f32(scales, sb_dtype, g);
            const float b = load_as_f32(biases, sb_dtype, g);
#pragma unroll
            for (int i = 0; i < EPW; ++i) {
                o[i] = fmaf((float)((word >> (BITS * i)) & ((1u << BITS) - 1u)), s, b);
                if (round_sb) o[i] = round_to(sb_dtype, o[i]);
            }
        } else {
#pragma unroll
            for (int i = 0; i < EPW; ++i) o[i] = 0.f;
        }
        const int64_t e = t * EPW;  // == r*K + wi*EPW
        if (out_dtype == QL_F32) {
            float4 *p = reinterpret_cast<float4 *>(reinterpret_cast<float *>(out) + e);
#pragma unroll
            for (int i = 0; i < EPW / 4; ++i)
                p[i] = make_float4(o[4 * i], o[4 * i + 1], o[4 * i + 2], o[4 * i + 3]);
        } else {
            uint32_t packed[EPW / 2];
#pragma unroll
            for (int i = 0; i < EPW / 2; ++i) {
                if (out_dtype == QL_BF16) {
                    packed[i] = pack_bf16x2(o[2 * i], o[2 * i + 1]);
                } else {
                    __half2 h = __floats2half2_rn(o[2 * i], o[2 * i + 1]);
                    packed[i] = *reinterpret_cast<uint32_t *>(&h);
                }
            }
            uint16_t *p = reinterpret_cast<uint16_t *>(out) + e;
            if constexpr (EPW == 8)
                *reinterpret_cast<uint4 *>(p) = make_uint4(packed[0], packed[1], packed[2], packed[3]);
            else
                *reinterpret_cast<uint2 *>(p) = make_uint2(packed[0], packed[1]);
        }
    }
}

static int grid_for(int64_t work, int block) {
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    int64_t blocks = (work + block - 1) / block;
    const int64_t cap = (int64_t)sms * 16;  // 16 x 256 threads resident per SM
    if (blocks > cap) blocks = cap;
    return (int)(blocks < 1 ? 1 : blocks);
}

int launch_quantize(const void *w, int w_dtype, int64_t N, int64_t K, int gs, int bits,
                    uint32_t *wq, void *scales, void *biases, int sb_dtype, cudaStream_t st) {
    const int64_t words = N * K * bits / 32;
    const int grid = grid_for(words, 256);
    if (bits == 4)
        quantize_kernel<4><<<grid, 256, 0, st>>>(w, w_dtype, words, gs, wq, scales, biases, sb_dtype);
    else
        quantize_kernel<8><<<grid, 256, 0, st>>>(w, w_dtype, words, gs, wq, scales, biases, sb_dtype);
    QL_CUDA_TRY(cudaGetLastError());
    return QL_OK;
}

int launch_dequantize(const int64_t *ids, int64_t rows, int64_t N, int64_t K, int gs, int bits,
                      const uint32_t *wq, const void *scales, const void *biases, int sb_dtype,
                      void *out, int out_dtype, bool round_sb, cudaStream_t st) {
    const int64_t wpr = K * bits / 32;
    const int grid = grid_for(rows * wpr, 256);
    if (bits == 4)
        dequantize_kernel<4><<<grid, 256, 0, st>>>(ids, rows, N, wpr, gs, wq, scales, biases,
                                                    sb_dtype, out, out_dtype, round_sb);
    else
        dequantize_kernel<8><<<grid, 256, 0, st>>>(ids, rows, N, wpr, gs, wq, scales, biases,
                                                    sb_dtype, out, out_dtype, round_sb);
    QL_CUDA_TRY(cudaGetLastError());
    return QL_OK;
}

}  // namespace ql
