// qgemv.cu -- small-M (M <= 8) quantized matmul for LLM decode.
//
// y[M, N] = x[M, K] . dequant(W)[N, K]^T, bf16 activations and scales, fp32
// accumulation.  This is the M <= 8 arm of quantized_matmul (the reference's
// decode-time and adaLN/timestep callers, e.g. mlx-gen-z-image/src/transformer_block.rs:122).
//
// The kernel is HBM-bound: every packed byte of W is read once, with 16-byte
// coalesced loads (four lanes cover 64 contiguous bytes of a row).  The
// dequantized weights go straight from registers into legacy warp-level MMAs
// (m16n8k16, bf16 -> fp32): with at most 8 tokens the tensor-core work is tiny
// and register-resident operands avoid any shared-memory staging; the
// roofline that matters is HBM bandwidth, not MMA throughput.
//
// Decomposition: a CTA of 8 warps owns one strip of 16 weight rows; its warps
// split K in chunks of 128 (each lane covers 32 consecutive codes of two rows,
// g and g+8).  Partial 16x8 tiles are summed through shared memory and the
// fused epilogue (bias, LoRA, GELU / SwiGLU) writes y.
//
// Dequantized weights are exact bf16 roundings of fma(code, scale, bias) --
// the same values ql_dequantize produces -- so GEMV, GEMM and dequant+matmul
// agree on the operand.
#include <stdlib.h>

#include "ql_common.cuh"

namespace ql {
namespace gemv {

constexpr int WARPS = 8;
constexpr int CHUNK = 128;  // K per warp step (4 lanes x 32 codes)

struct Params {
    const __nv_bfloat16 *x;  // [M, K]
    int M, N, K, gs, G;
    const uint32_t *wq, *wq2;
    const uint16_t *scales, *biases, *scales2, *biases2;
    const __nv_bfloat16 *bias, *bias2;
    const __nv_bfloat16 *lora_t;  // [M, rpad] = s.(x.A), or null
    const __nv_bfloat16 *lora_b;  // [rank, N]
    int rank, rpad;
    int act;
    __nv_bfloat16 *y;
    Gated gd;
};

__device__ __forceinline__ void mma16816(float d[4], const uint32_t a[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
        "{%8, %9}, {%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint4 ldg16(const void *p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

// Accumulate one chunk (this lane's 32 codes of rows g and g+8) into d.
template <int BITS>
__device__ __forceinline__ void chunk_mma(float d[4], const uint32_t *wg_words, const uint32_t *wh_words,
                                          uint32_t sg, uint32_t bg, uint32_t sh, uint32_t bh,
                                          const uint4 xv[4]) {
    if constexpr (BITS == 4) {
        // 4 words per row; word i holds codes 8i..8i+7.  Pairs (j, j+4) come out of
        // a word with one shift+mask; x is permuted the same way.
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            uint32_t pg[4], ph[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                pg[j] = hfma2_bf16(hsub2_bf16(((wg_words[i] >> (4 * j)) & 0x000f000fu) | 0x43004300u, 0x43004300u),
                                   sg, bg);
                ph[j] = hfma2_bf16(hsub2_bf16(((wh_words[i] >> (4 * j)) & 0x000f000fu) | 0x43004300u, 0x43004300u),
                                   sh, bh);
            }
            const uint4 X = xv[i];  // x codes 8i..8i+7 as (0,1) (2,3) (4,5) (6,7)
            const uint32_t x04 = prmt(X.x, X.z, 0x5410u), x15 = prmt(X.x, X.z, 0x7632u);
            const uint32_t x26 = prmt(X.y, X.w, 0x5410u), x37 = prmt(X.y, X.w, 0x7632u);
            const uint32_t a0[4] = {pg[0], ph[0], pg[1], ph[1]};
            mma16816(d, a0, x04, x15);
            const uint32_t a1[4] = {pg[2], ph[2], pg[3], ph[3]};
            mma16816(d, a1, x26, x37);
        }
    } else {
        // 8 words per row; word i holds codes 4i..4i+3 (natural pairs).
        const float fsg = bf16lo(sg), fbg = bf16lo(bg), fsh = bf16lo(sh), fbh = bf16lo(bh);
#pragma unroll
        for (int i = 0; i < 4; ++i) {  // two words (8 codes) per step
            uint32_t pg[4], ph[4];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const uint32_t wg = wg_words[2 * i + h], wh = wh_words[2 * i + h];
                pg[2 * h] = pack_bf16x2(fmaf(q8_code_f32(wg, 0), fsg, fbg), fmaf(q8_code_f32(wg, 1), fsg, fbg));
                pg[2 * h + 1] = pack_bf16x2(fmaf(q8_code_f32(wg, 2), fsg, fbg), fmaf(q8_code_f32(wg, 3), fsg, fbg));
                ph[2 * h] = pack_bf16x2(fmaf(q8_code_f32(wh, 0), fsh, fbh), fmaf(q8_code_f32(wh, 1), fsh, fbh));
                ph[2 * h + 1] = pack_bf16x2(fmaf(q8_code_f32(wh, 2), fsh, fbh), fmaf(q8_code_f32(wh, 3), fsh, fbh));
            }
            const uint4 X = xv[i];  // x codes 8i..8i+7
            const uint32_t a0[4] = {pg[0], ph[0], pg[1], ph[1]};
            mma16816(d, a0, X.x, X.y);
            const uint32_t a1[4] = {pg[2], ph[2], pg[3], ph[3]};
            mma16816(d, a1, X.z, X.w);
        }
    }
}

__device__ __forceinline__ void prefetch_l2(const void *p, uint32_t bytes) {
    bytes &= ~15u;  // a hint: rounding down keeps it inside the allocation
    if (bytes)
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// Smem layout of x: token g at g * XSTRIDE elements; inside a 128-wide chunk the
// order is (word i, lane c, element e) so that the four lanes of a row read 64
// contiguous bytes and the 32-element pad makes two token rows of a quarter-warp
// fall in different banks.
__device__ __forceinline__ int xs_index(int k) {
    const int ch = k >> 7, r = k & 127, c = r >> 5, i = (r >> 3) & 3, e = r & 7;
    return (ch << 7) + (i << 5) + (c << 3) + e;
}

template <int BITS, bool SWIGLU>
__global__ void __launch_bounds__(WARPS * 32, 2) qgemv_kernel(const Params p) {
    constexpr int NW = BITS;             // packed words per lane per row per chunk (32 codes)
    constexpr int NPASS = SWIGLU ? 2 : 1;
    constexpr int U = SWIGLU ? 2 : 4;    // chunks whose loads are in flight together
    constexpr int PF = 2;                // strips prefetched into L2 ahead of use
    extern __shared__ __align__(16) uint16_t xs[];
    __shared__ float red[NPASS][WARPS][16][8];

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, c = lane & 3;
    const int nstrips = (p.N + 15) / 16;
    const int64_t wpr = (int64_t)p.K * BITS / 32;  // words per row
    const int nchunks = (p.K + CHUNK - 1) / CHUNK;
    const int xstride = nchunks * CHUNK + 32;  // whole chunks: the permuted layout fills 128 slots

    // Weights do not depend on the previous kernel: start pulling this CTA's first
    // strips into L2 before waiting on it (programmatic dependent launch).
    auto prefetch_strip = [&](int st) {
        const int r0 = st * 16, rows = min(16, p.N - r0);
        for (int ps = 0; ps < NPASS; ++ps) {
            const uint32_t *W = ps ? p.wq2 : p.wq;
            const uint16_t *S = ps ? p.scales2 : p.scales;
            const uint16_t *B = ps ? p.biases2 : p.biases;
            prefetch_l2(W + (int64_t)r0 * wpr, (uint32_t)(rows * wpr * 4));
            prefetch_l2(S + (int64_t)r0 * p.G, (uint32_t)(rows * p.G * 2));
            prefetch_l2(B + (int64_t)r0 * p.G, (uint32_t)(rows * p.G * 2));
        }
    };
    if (threadIdx.x < PF) {
        const int st = blockIdx.x + threadIdx.x * gridDim.x;
        if (st < nstrips) prefetch_strip(st);
    }
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");

    // x -> shared memory (permuted, see xs_index)
    for (int e = threadIdx.x * 8; e < p.M * p.K; e += WARPS * 32 * 8) {
        const int m = e / p.K, k = e - m * p.K;
        *reinterpret_cast<uint4 *>(xs + m * xstride + xs_index(k)) =
            __ldg(reinterpret_cast<const uint4 *>(p.x + e));
    }
    __syncthreads();

    for (int st = blockIdx.x; st < nstrips; st += gridDim.x) {
        if (threadIdx.x == 0 && st + PF * (int)gridDim.x < nstrips) prefetch_strip(st + PF * gridDim.x);
        const int n0 = st * 16;
        const int rg = min(n0 + g, p.N - 1), rh = min(n0 + g + 8, p.N - 1);  // clamped (stores masked)
        float d[NPASS][4] = {};
        for (int cb = warp; cb < nchunks; cb += WARPS * U) {
            // ---- issue every load of U chunks first
            uint32_t wgw[U][NPASS][NW], whw[U][NPASS][NW], sbv[U][NPASS][4];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int ch = cb + u * WARPS;
                const bool kval = ch < nchunks && ch * CHUNK + 32 * c < p.K;
                const int k = kval ? ch * CHUNK + 32 * c : 0;
                const int grp = k / p.gs;
#pragma unroll
                for (int ps = 0; ps < NPASS; ++ps) {
                    const uint32_t *W = ps ? p.wq2 : p.wq;
                    const uint16_t *S = ps ? p.scales2 : p.scales;
                    const uint16_t *B = ps ? p.biases2 : p.biases;
                    const uint32_t *pgp = W + rg * wpr + (int64_t)k * BITS / 32;
                    const uint32_t *php = W + rh * wpr + (int64_t)k * BITS / 32;
#pragma unroll
                    for (int v = 0; v < NW / 4; ++v) {
                        uint4 a = make_uint4(0, 0, 0, 0), b = a;
                        if (kval) {
                            a = ldg16(pgp + 4 * v);
                            b = ldg16(php + 4 * v);
                        }
                        wgw[u][ps][4 * v] = a.x; wgw[u][ps][4 * v + 1] = a.y;
                        wgw[u][ps][4 * v + 2] = a.z; wgw[u][ps][4 * v + 3] = a.w;
                        whw[u][ps][4 * v] = b.x; whw[u][ps][4 * v + 1] = b.y;
                        whw[u][ps][4 * v + 2] = b.z; whw[u][ps][4 * v + 3] = b.w;
                    }
                    sbv[u][ps][0] = __ldg(S + (int64_t)rg * p.G + grp);
                    sbv[u][ps][1] = __ldg(B + (int64_t)rg * p.G + grp);
                    sbv[u][ps][2] = __ldg(S + (int64_t)rh * p.G + grp);
                    sbv[u][ps][3] = __ldg(B + (int64_t)rh * p.G + grp);
                }
            }
            // ---- then dequantize + MMA
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int ch = cb + u * WARPS;
                const bool kval = ch < nchunks && ch * CHUNK + 32 * c < p.K;
                uint4 xv[4];
                if (g < p.M && kval) {
                    const uint4 *xp = reinterpret_cast<const uint4 *>(xs + g * xstride + ch * CHUNK + c * 8);
#pragma unroll
                    for (int i = 0; i < 4; ++i) xv[i] = xp[i * 4];  // word i: +32 elements
                } else {
#pragma unroll
                    for (int i = 0; i < 4; ++i) xv[i] = make_uint4(0, 0, 0, 0);
                }
#pragma unroll
                for (int ps = 0; ps < NPASS; ++ps)
                    chunk_mma<BITS>(d[ps], wgw[u][ps], whw[u][ps], sbv[u][ps][0] * 0x10001u,
                                    sbv[u][ps][1] * 0x10001u, sbv[u][ps][2] * 0x10001u,
                                    sbv[u][ps][3] * 0x10001u, xv);
            }
        }
        // D fragment: d[0],d[1] = (row g, tokens 2c, 2c+1); d[2],d[3] = (row g+8, tokens 2c, 2c+1)
#pragma unroll
        for (int ps = 0; ps < NPASS; ++ps) {
            red[ps][warp][g][2 * c] = d[ps][0];
            red[ps][warp][g][2 * c + 1] = d[ps][1];
            red[ps][warp][g + 8][2 * c] = d[ps][2];
            red[ps][warp][g + 8][2 * c + 1] = d[ps][3];
        }
        __syncthreads();
        if (threadIdx.x < 128) {
            const int r = threadIdx.x >> 3, m = threadIdx.x & 7;
            const int n = n0 + r;
            if (n < p.N && m < p.M) {
                float acc = 0.f, acc2 = 0.f;
#pragma unroll
                for (int w = 0; w < WARPS; ++w) {
                    acc += red[0][w][r][m];
                    if (SWIGLU) acc2 += red[NPASS - 1][w][r][m];
                }
                if (p.lora_t) {
                    const __nv_bfloat16 *t = p.lora_t + (int64_t)m * p.rpad;
                    for (int j = 0; j < p.rank; ++j)
                        acc += __bfloat162float(t[j]) * __bfloat162float(p.lora_b[(int64_t)j * p.N + n]);
                }
                float v = round_bf16(acc);
                if (p.bias) v = round_bf16(v + __bfloat162float(p.bias[n]));
                if (SWIGLU) {
                    float u = round_bf16(acc2);
                    if (p.bias2) u = round_bf16(u + __bfloat162float(p.bias2[n]));
                    v = v / (1.0f + __expf(-v)) * u;
                } else if (p.act == QL_ACT_GELU_TANH) {
                    float t;
                    const float inner = 0.7978845608028654f * (v + 0.044715f * v * v * v);
                    asm("tanh.approx.f32 %0, %1;" : "=f"(t) : "f"(inner));
                    v = 0.5f * v * (1.0f + t);
                } else if (p.act == QL_ACT_GELU_ERF) {
                    v = 0.5f * v * (1.0f + erff(v * 0.7071067811865476f));
                }
                p.y[(int64_t)m * p.N + n] = __float2bfloat16_rn(apply_gated(v, p.gd, m, n, p.N));
            }
        }
        __syncthreads();
    }
}

}  // namespace gemv

bool qgemv_tma_supported(int64_t M, int64_t K, int gs);
int launch_qgemv_tma(const void *x, int64_t M, int64_t K, const uint32_t *wq, const void *scales,
                     const void *biases, const uint32_t *wq2, const void *scales2, const void *biases2,
                     int64_t N, int gs, int bits, const void *bias, const void *bias2, int act,
                     const void *lora_t, const void *lora_b, int64_t rank, void *y, const Gated &gd, cudaStream_t st);

bool qgemv_tc_supported(int64_t M, int64_t K, int gs, int bits, const void *x, bool lora);
int launch_qgemv_tc(const void *x, int64_t M, int64_t K, const uint32_t *wq, const void *scales, const void *biases,
                    const uint32_t *wq2, const void *scales2, const void *biases2, int64_t N, int gs, int bits,
                    const void *bias, const void *bias2, int act, void *y, const Gated &gd, cudaStream_t st);

static bool all_aligned16(std::initializer_list<const void *> ps) {
    for (const void *p : ps)
        if (p && reinterpret_cast<uintptr_t>(p) % 16) return false;
    return true;
}

int launch_qgemv(const void *x, int64_t M, int64_t K, const uint32_t *wq, const void *scales,
                 const void *biases, const uint32_t *wq2, const void *scales2, const void *biases2,
                 int64_t N, int gs, int bits, const void *bias, const void *bias2, int act,
                 const void *lora_t, const void *lora_b, int64_t rank, void *y, const Gated &gd, int which,
                 cudaStream_t st) {
    // which: 0 = automatic (below), 1 = the TMA-fed mma.sync kernel only, 2 = the
    // register-fed kernel only.  Automatic: the tcgen05 kernel (qgemv_tc.cu) when the shape
    // allows it and pays, else the TMA-fed kernel (qgemv_tma.cu), else the one below.
    if (which == 1) {
        if (!qgemv_tma_supported(M, K, gs))
            return fail(QL_EUNSUPPORTED, "TMA GEMV: K must be a whole number of 8-group batches");
        return launch_qgemv_tma(x, M, K, wq, scales, biases, wq2, scales2, biases2, N, gs, bits, bias, bias2, act,
                                lora_t, lora_b, rank, y, gd, st);
    }
    static const bool env_regs = getenv("QL_GEMV_REGS") != nullptr;  // profiling switches
    const bool force_regs = env_regs || which == 2;
    static const bool force_mma = getenv("QL_GEMV_MMA") != nullptr;
    // The tcgen05 kernel wins once its row tiles (128 rows, 64 with SwiGLU) fill the GPU;
    // below that its fixed start-up (TMEM, activation conversion, pipeline fill) dominates
    // at every M (Llama-3.2-3B decode step, per step: M = 6 1.85 ms on it against 1.56 on
    // the register-fed kernel, M = 8 1.93 against 1.75 on the TMA-fed kernel).
    static PerDeviceInt sm_count;
    const int cur_dev = current_device();
    int n_sms = sm_count.get(cur_dev);
    if (!n_sms) {
        if (cudaDeviceGetAttribute(&n_sms, cudaDevAttrMultiProcessorCount, cur_dev) != cudaSuccess || n_sms <= 0)
            n_sms = 148;
        sm_count.put(cur_dev, n_sms);
    }
    static const bool force_tc = getenv("QL_GEMV_TC") != nullptr;
    const int64_t tiles = (N + (act == QL_ACT_SWIGLU ? 63 : 127)) / (act == QL_ACT_SWIGLU ? 64 : 128);
    if (!force_regs && !force_mma && (force_tc || tiles >= n_sms) &&
        qgemv_tc_supported(M, K, gs, bits, x, lora_t != nullptr) && all_aligned16({scales, biases, scales2, biases2}))
        return launch_qgemv_tc(x, M, K, wq, scales, biases, wq2, scales2, biases2, N, gs, bits, bias, bias2, act, y,
                               gd, st);
    // Narrow projections at M = 1 and every shape at M = 2..6 run best on the register-fed
    // kernel below (no TMA / barrier set-up; measured on the Llama-3.2-3B decode step);
    // wider ones at M = 1, 7, 8 on the TMA-fed one.
    const bool regs_pick = (M >= 2 && M <= 6) || (act != QL_ACT_SWIGLU && N <= 4096);
    if (!force_regs && !regs_pick && qgemv_tma_supported(M, K, gs)) {
        const int rc = launch_qgemv_tma(x, M, K, wq, scales, biases, wq2, scales2, biases2, N, gs, bits, bias, bias2,
                                        act, lora_t, lora_b, rank, y, gd, st);
        if (rc != QL_EUNSUPPORTED) return rc;  // refused before launching: x does not fit its staging
    }
    using namespace gemv;
    Params p{};
    p.gd = gd;
    p.x = (const __nv_bfloat16 *)x;
    p.M = (int)M;
    p.N = (int)N;
    p.K = (int)K;
    p.gs = gs;
    p.G = (int)(K / gs);
    p.wq = wq;
    p.wq2 = wq2;
    p.scales = (const uint16_t *)scales;
    p.biases = (const uint16_t *)biases;
    p.scales2 = (const uint16_t *)scales2;
    p.biases2 = (const uint16_t *)biases2;
    p.bias = (const __nv_bfloat16 *)bias;
    p.bias2 = (const __nv_bfloat16 *)bias2;
    p.lora_t = (const __nv_bfloat16 *)lora_t;
    p.lora_b = (const __nv_bfloat16 *)lora_b;
    p.rank = (int)rank;
    p.rpad = (int)(rank > 0 ? (rank + 63) / 64 * 64 : 0);
    p.act = act;
    p.y = (__nv_bfloat16 *)y;
    int dev = 0, sms = 148;
    QL_CUDA_TRY(cudaGetDevice(&dev));
    QL_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    const int nstrips = (int)((N + 15) / 16);
    const size_t smem = (size_t)M * (size_t)((K + CHUNK - 1) / CHUNK * CHUNK + 32) * 2;
    if (smem > 200 * 1024) {
        // the tcgen05 kernel splits K over a cluster and may still take this x
        if (!force_regs && qgemv_tc_supported(M, K, gs, bits, x, lora_t != nullptr) &&
            all_aligned16({scales, biases, scales2, biases2}))
            return launch_qgemv_tc(x, M, K, wq, scales, biases, wq2, scales2, biases2, N, gs, bits, bias, bias2, act,
                                   y, gd, st);
        return fail(QL_EUNSUPPORTED, "GEMV: M*K too large for the x staging buffer");
    }
    const int per_sm = smem <= 48 * 1024 ? 2 : 1;
    const int grid = nstrips < per_sm * sms ? nstrips : per_sm * sms;
    const bool sw = act == QL_ACT_SWIGLU;
    void (*kfn)(const Params) = bits == 4 ? (sw ? qgemv_kernel<4, true> : qgemv_kernel<4, false>)
                                          : (sw ? qgemv_kernel<8, true> : qgemv_kernel<8, false>);
    if (smem > 48 * 1024)
        QL_CUDA_TRY(cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    // Programmatic dependent launch: the kernel may start (and prefetch its weights)
    // while the previous kernel on the stream finishes; it waits for that kernel's
    // results (griddepcontrol.wait) before touching x.
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(WARPS * 32);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    QL_CUDA_TRY(cudaLaunchKernelEx(&cfg, kfn, p));
    QL_CUDA_TRY(cudaGetLastError());
    return QL_OK;
}

}  // namespace ql
