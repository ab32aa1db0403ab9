// quantize.cu -- group-wise affine quantize / dequantize kernels.
//
// Both kernels are HBM-bound streaming kernels.  quantize: one thread per packed
// uint32 word (8 Q4 codes or 4 Q8 codes), so a warp reads/writes contiguous 128-byte
// segments; a group of `gs` elements is covered by gs*bits/32 consecutive lanes and
// its min/max is a shuffle-xor reduction among them.  dequantize: one thread per
// 16 bytes of packed codes (one group's scale and bias), 16-byte stores.
//
// Arithmetic follows MLX affine quantization as the reference calls it
// (src/quant.rs:140, src/adapters.rs:533-537; restated and pinned against the
// reference fixture in oracle/qref.c quant_group()).  Every division is an
// IEEE round-to-nearest division (or provably equal to one, see the code loop) and
// no multiply-add is contracted, so the codes, scales and biases are bit-identical
// to the oracle.
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
    // Each thread packs 2 consecutive words (16 / 8 elements); a group spans
    // tpg = gs / (2 * EPW) consecutive lanes (a power of two in [2, 16]).
    constexpr int EPW = 32 / BITS;
    const int tpg = gs / (2 * EPW);
    const float n_bins = (float)((1 << BITS) - 1);
    const int64_t pairs = total_words / 2;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    // pairs is a multiple of tpg, and tpg divides 32, so every lane of a group runs
    // the same number of iterations (the shuffles stay converged).
    for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t - (threadIdx.x & 31) < pairs; t += stride) {
        const bool live = t < pairs;
        float v[2][EPW];
        if (live) {
            load_elems<EPW>(w, w_dtype, 2 * t * EPW, v[0]);
            load_elems<EPW>(w, w_dtype, (2 * t + 1) * EPW, v[1]);
        } else {
#pragma unroll
            for (int i = 0; i < EPW; ++i) v[0][i] = v[1][i] = 0.f;
        }
        float mn = v[0][0], mx = v[0][0];
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
            for (int i = 0; i < EPW; ++i) {
                mn = fminf(mn, v[h][i]);
                mx = fmaxf(mx, v[h][i]);
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
        // code = clamp(rint((v - b) / s)) with the IEEE quotient.  The quotient is first
        // taken as a product with the rounded reciprocal, within 2 ulps (relative 2^-22) of
        // the exact one: below -1 or above 300 the clamp decides the code either way, and
        // inside [-1, 300] the product is within 2^-13 of the quotient, so rint agrees
        // unless the product lies within 2^-10 of a rounding boundary (x.5); only then (or
        // for a NaN) is the exact division done.  The codes are the exact ones.
        //
        // rint without the slow rounding / conversion instructions: adding 1.5 * 2^23 rounds
        // qf to an integer (round-to-nearest-even, exact for |qf| < 2^22) held in the low
        // mantissa bits, so the sum's bit pattern minus that of 1.5 * 2^23 is rint(qf) as an
        // integer.  The boundary test uses d = qf - rint(qf) (exact): qf lies within 2^-10 of
        // x.5 exactly when |d| > 0.5 - 2^-10.
        const float rs = __frcp_rn(s);
        constexpr float kMagic = 12582912.0f;  // 1.5 * 2^23
        uint32_t word[2] = {0u, 0u};
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
            for (int i = 0; i < EPW; ++i) {
                const float a = __fsub_rn(v[h][i], b);
                float qf = __fmul_rn(a, rs);
                float t = __fadd_rn(qf, kMagic);
                const float d = __fsub_rn(qf, __fsub_rn(t, kMagic));
                const bool in_range = qf >= -1.0f && qf <= 300.0f;
                if ((in_range && fabsf(d) > 0.5f - 0x1p-10f) || qf != qf) {
                    qf = __fdiv_rn(a, s);
                    t = __fadd_rn(qf, kMagic);
                }
                // qf < 0 (and NaN) gives code 0, as the clamp of rint(qf) does; for qf >= 0 the
                // sum is a positive float whose bits grow with qf
                const int c =
                    qf >= 0.0f ? min((int)(__float_as_uint(t) - __float_as_uint(kMagic)), (1 << BITS) - 1) : 0;
                word[h] |= (uint32_t)c << (BITS * i);
            }
        reinterpret_cast<uint2 *>(wq)[t] = make_uint2(word[0], word[1]);
        if ((t % tpg) == 0) {
            const int64_t g = t / tpg;
            store_from_f32(scales, sb_dtype, g, s);
            store_from_f32(biases, sb_dtype, g, b);
        }
    }
}

// ids == nullptr: row r reads
// packed row r; otherwise packed row ids[r] (quantized embedding gather).  round_sb: the
// value is first rounded to the scales' dtype (mlx's dequantize output) and then converted
// to out_dtype, as the reference's gather + dequantize + cast does.
template <int BITS>
__global__ void __launch_bounds__(256) dequantize_kernel(
    const int64_t *__restrict__ ids, int64_t rows, int64_t N, int64_t words_per_row, int gs,
    const uint32_t *__restrict__ wq, const void *__restrict__ scales,
    const void *__restrict__ biases, int sb_dtype, void *__restrict__ out, int out_dtype, bool round_sb) {
    // Each thread handles 4 consecutive packed words (16 bytes: 32 Q4 / 16 Q8 codes, always
    // inside one group since a row holds a multiple of 32 codes and gs >= 32).
    constexpr int EPW = 32 / BITS;
    constexpr int E4 = 4 * EPW;
    const int64_t qpr = words_per_row / 4;  // 16-byte quads per row
    const int64_t total = rows * qpr;
    const int64_t G = words_per_row * EPW / gs;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total; t += stride) {
        const int64_t r = t / qpr, qi = t - r * qpr;
        int64_t n = r;
        bool ok = true;
        if (ids) {
            n = __ldg(ids + r);
            if (n < 0 || n >= N) {
                ok = false;
                if (qi == 0) raise_dev_error(DEV_ERR_BAD_INDEX);
            }
        }
        uint32_t words[4] = {0u, 0u, 0u, 0u};
        float s = 0.f, b = 0.f;
        if (ok) {
            const uint4 wv = __ldg(reinterpret_cast<const uint4 *>(wq + n * words_per_row) + qi);
            words[0] = wv.x, words[1] = wv.y, words[2] = wv.z, words[3] = wv.w;
            const int64_t g = n * G + (qi * E4) / gs;
            s = load_as_f32(scales, sb_dtype, g);
            b = load_as_f32(biases, sb_dtype, g);
        }
        // element k of the quad: code (words[k / EPW] >> (BITS * (k % EPW))) & mask
        auto val = [&](int k) -> float {
            if (!ok) return 0.f;
            float v = fmaf((float)((words[k / EPW] >> (BITS * (k % EPW))) & ((1u << BITS) - 1u)), s, b);
            return round_sb ? round_to(sb_dtype, v) : v;
        };
        const int64_t e = t * E4;  // == r*K + qi*E4
        if (out_dtype == QL_F32) {
            float4 *p = reinterpret_cast<float4 *>(reinterpret_cast<float *>(out) + e);
#pragma unroll
            for (int i = 0; i < E4 / 4; ++i) p[i] = make_float4(val(4 * i), val(4 * i + 1), val(4 * i + 2), val(4 * i + 3));
        } else {
            uint4 *p = reinterpret_cast<uint4 *>(reinterpret_cast<uint16_t *>(out) + e);
#pragma unroll
            for (int i = 0; i < E4 / 8; ++i) {
                uint32_t pk[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const float lo = val(8 * i + 2 * j), hi = val(8 * i + 2 * j + 1);
                    if (out_dtype == QL_BF16) {
                        pk[j] = pack_bf16x2(lo, hi);
                    } else {
                        __half2 h = __floats2half2_rn(lo, hi);
                        pk[j] = *reinterpret_cast<uint32_t *>(&h);
                    }
                }
                p[i] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
            }
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
    const int64_t words = N * K * bits / 32;  // even: K is a multiple of 32
    const int grid = grid_for(words / 2, 256);
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
    const int grid = grid_for(rows * wpr / 4, 256);
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
