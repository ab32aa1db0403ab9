// qgemv_tma.cu -- small-M (M <= 8) quantized matmul, TMA-fed (the default GEMV).
//
// y[M, N] = x[M, K] . dequant(W)[N, K]^T, bf16 activations and scales.  The path the
// reference takes for decode-time and timestep linears (quantized_matmul with few rows,
// src/adapters.rs:309-317) is HBM-bound, so this kernel is built to keep HBM busy
// with as few instructions per weight byte as possible:
//
//   * A producer warp streams each 16-row strip of packed W (plus its scales and
//     biases) through a ring of shared-memory stages with TMA, 1024 codes of K per
//     stage, in boxes of 16 rows x 128 bytes with the 128-byte swizzle so that the
//     eight rows a consumer instruction touches land in different banks.  Weights do not depend on the previous kernel, so the
//     producer starts before griddepcontrol.wait (programmatic dependent launch) and
//     the stream of one launch overlaps the tail of the previous one.
//   * Consumers never apply scale and bias per element.  Codes become exact bf16
//     values 128 + q with one shift and one lop3 per pair, feed mma.sync m16n8k16
//     (tokens padded to 8) and accumulate per group; each finished group is folded
//     in as  y += s * D + (b - 128 s) * sum_k x_k  with the per-group sums of x
//     precomputed once per CTA.  Q8 codes are split into nibbles (q = 16 h + l)
//     accumulated separately.  Mathematically this is sum_k x_k (q_k s + b): the
//     weights are used exactly, without the bf16 rounding of the dequantized value.
//   * The 8 consumer warps split each stage's K (128 codes each); per-strip partial
//     tiles are summed through shared memory and the fused epilogue (bias, LoRA, GELU,
//     SwiGLU) writes y.
// Used when K is a multiple of 8 groups (TMA row pitch of the scales); other shapes use
// the register-fed kernel in qgemv.cu.
#include "ql_common.cuh"

namespace ql {
namespace gemv2 {

constexpr int CWARPS = 8;            // consumer warps
constexpr int NTHREADS = (CWARPS + 1) * 32;
constexpr int KS = 1024;             // codes of K per stage
constexpr int RUNS = KS / 32;        // 32-code runs per stage

struct Params {
    int M, N, K, gs, G, nks;         // nks: stages per strip
    int act;
    const __nv_bfloat16 *x;
    const __nv_bfloat16 *bias, *bias2;
    const __nv_bfloat16 *lora_t, *lora_b;
    int rank, rpad;
    __nv_bfloat16 *y;
    Gated gd;
};

template <int BITS, bool SWIGLU>
struct Cfg {
    static constexpr int NPASS = SWIGLU ? 2 : 1;
    static constexpr int RUNW = BITS;                       // words per 32-code run
    static constexpr int W_BYTES = 16 * KS * BITS / 8;      // one pass, one stage
    static constexpr int STAGES = BITS == 4 ? (SWIGLU ? 4 : 6) : (SWIGLU ? 3 : 4);
};

__device__ __forceinline__ void mma16816(float d[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
        "{%8, %9}, {%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// bf16x2 (128 + code_lo, 128 + code_hi) from the nibbles at bit 4j and 16 + 4j
__device__ __forceinline__ uint32_t nib2(uint32_t w, int j) {
    return ((w >> (4 * j)) & 0x000f000fu) | 0x43004300u;
}

template <int BITS, bool SWIGLU, int GS>
__global__ void __launch_bounds__(NTHREADS, 2)
    qgemv_tma_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_s,
                     const __grid_constant__ CUtensorMap tm_b, const __grid_constant__ CUtensorMap tm_w2,
                     const __grid_constant__ CUtensorMap tm_s2, const __grid_constant__ CUtensorMap tm_b2,
                     const Params p) {
    using C = Cfg<BITS, SWIGLU>;
    constexpr int NPASS = C::NPASS, STAGES = C::STAGES;
    constexpr int GPS = KS / GS;                            // groups per stage
    constexpr int SB_BYTES = 16 * GPS * 2;                  // scales (or biases) per stage
    constexpr int PASS_BYTES = (C::W_BYTES + 2 * SB_BYTES + 1023) / 1024 * 1024;  // swizzled boxes: 1 KB aligned
    constexpr int STAGE_BYTES = NPASS * PASS_BYTES;
    constexpr int WBOXES = KS * BITS / 8 / 128;             // 128-byte-wide boxes per stage
    const int nstrips = (p.N + 15) / 16;
    const int nruns = p.nks * RUNS;                          // runs of x staged (zero past K)
    const int xstride = nruns * 64 + ((nruns & 1) ? 0 : 64);  // bytes per token in smem

    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *stages = smem;                                           // STAGES * STAGE_BYTES
    uint8_t *xs = stages + STAGES * STAGE_BYTES;                      // M * xstride
    float *xsum = reinterpret_cast<float *>(xs + p.M * xstride);      // [8][G]
    float *red = xsum + 8 * p.G;                                      // [2][NPASS][8][16][8]
    uint64_t *bars = reinterpret_cast<uint64_t *>(red + 2 * NPASS * CWARPS * 128);
    uint64_t *full = bars, *empty = bars + STAGES;
    volatile int *abort_flag = reinterpret_cast<volatile int *>(bars + 2 * STAGES);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], CWARPS);
        }
        *abort_flag = 0;
        mbar_fence_init();
    }
    __syncthreads();
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

    if (warp == CWARPS) {
        // ---------------------------------------------------------------- TMA producer
        // Weights, scales and biases do not depend on the previous kernel: stream them
        // before griddepcontrol.wait.
        if (lane == 0) {
            uint32_t it = 0;
            for (int st = blockIdx.x; st < nstrips && !*abort_flag; st += gridDim.x) {
                for (int kc = 0; kc < p.nks; ++kc, ++it) {
                    const int s = it % STAGES;
                    if (!mbar_wait(&empty[s], ((it / STAGES) & 1) ^ 1, abort_flag, DEV_ERR_TIMEOUT_EMPTY)) break;
                    uint8_t *sp = stages + s * STAGE_BYTES;
                    mbar_arrive_expect_tx(&full[s], NPASS * (C::W_BYTES + 2 * SB_BYTES));
#pragma unroll
                    for (int ps = 0; ps < NPASS; ++ps) {
                        uint8_t *pp = sp + ps * PASS_BYTES;
#pragma unroll
                        for (int bx = 0; bx < WBOXES; ++bx)
                            tma_load_2d(pp + bx * 2048, ps ? &tm_w2 : &tm_w, &full[s], (kc * KS * BITS / 8 + bx * 128) / 4,
                                        st * 16);
                        tma_load_2d(pp + C::W_BYTES, ps ? &tm_s2 : &tm_s, &full[s], kc * GPS, st * 16);
                        tma_load_2d(pp + C::W_BYTES + SB_BYTES, ps ? &tm_b2 : &tm_b, &full[s], kc * GPS, st * 16);
                    }
                }
            }
        }
        return;  // the producer takes no part in the consumers' named barriers
    }

    // -------------------------------------------------------------------- consumers
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int tid = threadIdx.x;  // consumer thread, 0 .. CWARPS * 32 - 1
    // x -> smem, permuted so that lane c of a warp reads its four bf16 pairs of a run in
    // one 16-byte load: Q4 pairs (0,4) (1,5) (2,6) (3,7), Q8 pairs (0,2) (1,3) (4,6) (5,7)
    // of the lane's 8 consecutive codes.
    for (int u = tid; u < p.M * nruns * 4; u += CWARPS * 32) {
        const int m = u / (nruns * 4), rc = u - m * nruns * 4;   // rc = run * 4 + c
        const int k = rc * 8;
        uint4 v = make_uint4(0, 0, 0, 0);
        if (k < p.K) v = __ldg(reinterpret_cast<const uint4 *>(p.x + (int64_t)m * p.K + k));
        uint4 o;
        if (BITS == 4) {
            o.x = prmt(v.x, v.z, 0x5410u);  // (0,4)
            o.y = prmt(v.x, v.z, 0x7632u);  // (1,5)
            o.z = prmt(v.y, v.w, 0x5410u);  // (2,6)
            o.w = prmt(v.y, v.w, 0x7632u);  // (3,7)
        } else {
            o.x = prmt(v.x, v.y, 0x5410u);  // (0,2)
            o.y = prmt(v.x, v.y, 0x7632u);  // (1,3)
            o.z = prmt(v.z, v.w, 0x5410u);  // (4,6)
            o.w = prmt(v.z, v.w, 0x7632u);  // (5,7)
        }
        *reinterpret_cast<uint4 *>(xs + m * xstride + rc * 16) = o;
    }
    named_bar_sync(1, CWARPS * 32);
    // per-group sums of x (fp32) from the staged copy (any order of the group's values),
    // zero for padded tokens
    for (int u = tid; u < 8 * p.G; u += CWARPS * 32) {
        const int m = u / p.G, gi = u - m * p.G;
        float acc = 0.f;
        if (m < p.M) {
            const uint4 *xp = reinterpret_cast<const uint4 *>(xs + m * xstride) + gi * (GS / 8);
#pragma unroll 4
            for (int e = 0; e < GS / 8; ++e) {
                const uint4 v = xp[e];
                acc += (bf16lo(v.x) + bf16hi(v.x)) + (bf16lo(v.y) + bf16hi(v.y)) + (bf16lo(v.z) + bf16hi(v.z)) +
                       (bf16lo(v.w) + bf16hi(v.w));
            }
        }
        xsum[u] = acc;
    }
    named_bar_sync(1, CWARPS * 32);

    const int g = lane >> 2, c = lane & 3;
    const float cfold = BITS == 4 ? 128.f : 2176.f;  // offset folded back per group
    const int lw = warp;                             // consumer warp
    constexpr int runs_per_group = GS / 32;
    uint32_t it = 0, strip_iter = 0;
    for (int st = blockIdx.x; st < nstrips; st += gridDim.x) {
        float acc[NPASS][4] = {};
        bool ok = true;
        for (int kc = 0; kc < p.nks; ++kc, ++it) {
            const int s = it % STAGES;
            if (!mbar_wait(&full[s], (it / STAGES) & 1, abort_flag, DEV_ERR_TIMEOUT_FULL)) {
                ok = false;
                break;
            }
            const uint8_t *sp = stages + s * STAGE_BYTES;
            // ---- load phase: everything this warp needs from the stage goes to registers,
            //      then the stage is released so the producer can refill it at once
            constexpr int NG = 128 / GS;                 // groups covered by this warp's 4 runs
            constexpr int NWW = BITS == 4 ? 1 : 2;       // words per lane per row per run
            uint32_t wgv[NPASS][4][NWW], whv[NPASS][4][NWW];
            uint16_t sgv[NPASS][NG], shv[NPASS][NG], bgv[NPASS][NG], bhv[NPASS][NG];
            uint4 X[4];
#pragma unroll
            for (int rr = 0; rr < 4; ++rr) {
                const int r = lw * 4 + rr;  // run within the stage
                X[rr] = make_uint4(0, 0, 0, 0);  // tokens past M are zero
                if (g < p.M) X[rr] = *reinterpret_cast<const uint4 *>(xs + g * xstride + ((kc * RUNS + r) * 4 + c) * 16);
#pragma unroll
                for (int ps = 0; ps < NPASS; ++ps) {
                    const uint8_t *wp = sp + ps * PASS_BYTES;
                    if constexpr (BITS == 4) {
                        // box r/8 holds runs [8b, 8b+8) as 16 rows x 128 B; 16-byte chunk j of
                        // row g sits at chunk j ^ (g % 8) (TMA 128-byte swizzle)
                        const uint8_t *bp = wp + (r >> 3) * 2048 + g * 128 + (((r & 7) ^ g) << 4) + 4 * c;
                        wgv[ps][rr][0] = *reinterpret_cast<const uint32_t *>(bp);
                        whv[ps][rr][0] = *reinterpret_cast<const uint32_t *>(bp + 8 * 128);
                    } else {
                        // box r/4 holds runs [4b, 4b+4) (32 B each), swizzled as above
                        const uint8_t *bp = wp + (r >> 2) * 2048 + g * 128 +
                                            ((((2 * (r & 3)) + (c >> 1)) ^ g) << 4) + 8 * (c & 1);
                        const uint2 a = *reinterpret_cast<const uint2 *>(bp);
                        const uint2 bb = *reinterpret_cast<const uint2 *>(bp + 8 * 128);
                        wgv[ps][rr][0] = a.x;
                        wgv[ps][rr][NWW - 1] = a.y;
                        whv[ps][rr][0] = bb.x;
                        whv[ps][rr][NWW - 1] = bb.y;
                    }
                }
            }
#pragma unroll
            for (int ps = 0; ps < NPASS; ++ps) {
                const uint16_t *sc = reinterpret_cast<const uint16_t *>(sp + ps * PASS_BYTES + C::W_BYTES);
                const uint16_t *bi = sc + SB_BYTES / 2;
#pragma unroll
                for (int q = 0; q < NG; ++q) {
                    const int gl = lw * NG + q;  // group within the stage
                    sgv[ps][q] = sc[g * GPS + gl];
                    shv[ps][q] = sc[(g + 8) * GPS + gl];
                    bgv[ps][q] = bi[g * GPS + gl];
                    bhv[ps][q] = bi[(g + 8) * GPS + gl];
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
            // ---- compute phase.  Every MMA of the stage first (independent accumulators:
            //      per group, per plane -- Q4 halves a/b, Q8 low/high nibbles -- and, for
            //      one group per warp, per run parity), runs of different groups interleaved;
            //      then one fold per group.
            constexpr int RP = NG == 1 ? 2 : 1;
            constexpr int ORD[4] = {0, NG == 2 ? 2 : 1, NG == 2 ? 1 : 2, 3};
#pragma unroll
            for (int ps = 0; ps < NPASS; ++ps) {
                float ac[NG][2][RP][4];
#pragma unroll
                for (int q = 0; q < NG; ++q)
#pragma unroll
                    for (int m = 0; m < 2; ++m)
#pragma unroll
                        for (int t = 0; t < RP; ++t)
#pragma unroll
                            for (int i = 0; i < 4; ++i) ac[q][m][t][i] = 0.f;
#pragma unroll
                for (int oi = 0; oi < 4; ++oi) {
                    const int rr = ORD[oi];
                    const int q = rr / runs_per_group, t = rr % RP;
                    const uint32_t *wg = wgv[ps][rr], *wh = whv[ps][rr];
                    if constexpr (BITS == 4) {
                        mma16816(ac[q][0][t], nib2(wg[0], 0), nib2(wh[0], 0), nib2(wg[0], 1), nib2(wh[0], 1), X[rr].x, X[rr].y);
                        mma16816(ac[q][1][t], nib2(wg[0], 2), nib2(wh[0], 2), nib2(wg[0], 3), nib2(wh[0], 3), X[rr].z, X[rr].w);
                    } else {
                        // low nibbles: (l0,l2) at shift 0, (l1,l3) at shift 8; high: 4, 12
                        mma16816(ac[q][0][t], nib2(wg[0], 0), nib2(wh[0], 0), nib2(wg[0], 2), nib2(wh[0], 2), X[rr].x, X[rr].y);
                        mma16816(ac[q][1][t], nib2(wg[0], 1), nib2(wh[0], 1), nib2(wg[0], 3), nib2(wh[0], 3), X[rr].x, X[rr].y);
                        mma16816(ac[q][0][t], nib2(wg[NWW - 1], 0), nib2(wh[NWW - 1], 0), nib2(wg[NWW - 1], 2),
                                 nib2(wh[NWW - 1], 2), X[rr].z, X[rr].w);
                        mma16816(ac[q][1][t], nib2(wg[NWW - 1], 1), nib2(wh[NWW - 1], 1), nib2(wg[NWW - 1], 3),
                                 nib2(wh[NWW - 1], 3), X[rr].z, X[rr].w);
                    }
                }
#pragma unroll
                for (int q = 0; q < NG; ++q) {
                    // fold the group: y += s D + (b - cfold s) X
                    const int gg = kc * GPS + lw * NG + q;  // global group
                    const float sg = bf16lo((uint32_t)sgv[ps][q]);
                    const float sh = bf16lo((uint32_t)shv[ps][q]);
                    const float bg = bf16lo((uint32_t)bgv[ps][q]) - cfold * sg;
                    const float bh = bf16lo((uint32_t)bhv[ps][q]) - cfold * sh;
                    const float x0 = gg < p.G ? xsum[(2 * c) * p.G + gg] : 0.f;
                    const float x1 = gg < p.G ? xsum[(2 * c + 1) * p.G + gg] : 0.f;
                    float d[4];
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        float lo = ac[q][0][0][i], hi = ac[q][1][0][i];
                        if (RP == 2) {
                            lo += ac[q][0][RP - 1][i];
                            hi += ac[q][1][RP - 1][i];
                        }
                        d[i] = BITS == 8 ? fmaf(16.f, hi, lo) : lo + hi;
                    }
                    acc[ps][0] += fmaf(sg, d[0], bg * x0);
                    acc[ps][1] += fmaf(sg, d[1], bg * x1);
                    acc[ps][2] += fmaf(sh, d[2], bh * x0);
                    acc[ps][3] += fmaf(sh, d[3], bh * x1);
                }
            }
        }
        // partial tiles of the 8 warps -> one 16 x 8 tile -> epilogue.  The buffer
        // alternates per strip: the epilogue of strip i reads buffer i%2 while the
        // other warps go on; the barrier of strip i+1 orders it before its reuse.
        float *rb = red + (strip_iter & 1) * NPASS * CWARPS * 128;
        ++strip_iter;
#pragma unroll
        for (int ps = 0; ps < NPASS; ++ps) {
            float *rp = rb + (ps * CWARPS + warp) * 128;
            rp[g * 8 + 2 * c] = acc[ps][0];
            rp[g * 8 + 2 * c + 1] = acc[ps][1];
            rp[(g + 8) * 8 + 2 * c] = acc[ps][2];
            rp[(g + 8) * 8 + 2 * c + 1] = acc[ps][3];
        }
        named_bar_sync(1, CWARPS * 32);  // every warp reaches it, aborted or not
        if (!ok || *abort_flag) break;
        if (tid < 128) {
            const int r = tid >> 3, m = tid & 7, n = st * 16 + r;
            if (n < p.N && m < p.M) {
                float a = 0.f, a2 = 0.f;
#pragma unroll
                for (int w = 0; w < CWARPS; ++w) {
                    a += rb[w * 128 + r * 8 + m];
                    if (SWIGLU) a2 += rb[(CWARPS + w) * 128 + r * 8 + m];
                }
                if (p.lora_t) {
                    const __nv_bfloat16 *t = p.lora_t + (int64_t)m * p.rpad;
                    for (int j = 0; j < p.rank; ++j)
                        a += __bfloat162float(t[j]) * __bfloat162float(p.lora_b[(int64_t)j * p.N + n]);
                }
                float v = round_bf16(a);
                if (p.bias) v = round_bf16(v + __bfloat162float(p.bias[n]));
                if (SWIGLU) {
                    float uu = round_bf16(a2);
                    if (p.bias2) uu = round_bf16(uu + __bfloat162float(p.bias2[n]));
                    v = v / (1.0f + __expf(-v)) * uu;
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
    }
}

static int make_map(CUtensorMap *map, CUtensorMapDataType dt, const void *base, int rank, const uint64_t *dims,
                    const uint64_t *strides_bytes, const uint32_t *box,
                    CUtensorMapSwizzle sw = CU_TENSOR_MAP_SWIZZLE_NONE) {
    gemm::PFN_encodeTiled enc = gemm::get_encode();
    if (!enc) return fail(QL_ECUDA, "cuTensorMapEncodeTiled unavailable");
    cuuint64_t d[3], st[2];
    cuuint32_t b[3], e[3] = {1, 1, 1};
    for (int i = 0; i < rank; ++i) {
        d[i] = dims[i];
        b[i] = box[i];
    }
    for (int i = 0; i + 1 < rank; ++i) st[i] = strides_bytes[i];
    CUresult r = enc(map, dt, (cuuint32_t)rank, const_cast<void *>(base), d, st, b, e, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(QL_ECUDA, "cuTensorMapEncodeTiled (gemv) failed (%d)", (int)r);
    return QL_OK;
}

template <int BITS, bool SWIGLU, int GS>
static int launch_t(const CUtensorMap *maps, const Params &p, cudaStream_t st) {
    using C = Cfg<BITS, SWIGLU>;
    auto kfn = qgemv_tma_kernel<BITS, SWIGLU, GS>;
    const int GPS = KS / p.gs;
    const size_t stage_bytes = (size_t)C::NPASS * ((C::W_BYTES + 2 * 16 * GPS * 2 + 1023) / 1024 * 1024);
    const int nruns = p.nks * RUNS;
    const size_t xstride = (size_t)nruns * 64 + ((nruns & 1) ? 0 : 64);
    const size_t smem = 1024 + C::STAGES * stage_bytes + (size_t)p.M * xstride + 8 * (size_t)p.G * 4 +
                        2 * (size_t)C::NPASS * CWARPS * 128 * 4 + 2 * C::STAGES * 8 + 16;
    if (smem > 227 * 1024) return fail(QL_EUNSUPPORTED, "GEMV: K too large for the staged kernel");
    QL_CUDA_TRY(cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    int dev = 0, sms = 148;
    QL_CUDA_TRY(cudaGetDevice(&dev));
    QL_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    const int nstrips = (p.N + 15) / 16;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(nstrips < 2 * sms ? nstrips : 2 * sms));
    cfg.blockDim = dim3(NTHREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    QL_CUDA_TRY(cudaLaunchKernelEx(&cfg, kfn, maps[0], maps[1], maps[2], maps[3], maps[4], maps[5], p));
    return QL_OK;
}

}  // namespace gemv2

// True when the staged kernel handles this shape (scales' row pitch must be a multiple of
// 16 bytes for TMA, i.e. K a multiple of 8 groups).
bool qgemv_tma_supported(int64_t M, int64_t K, int gs) { return M >= 1 && M <= 8 && (K / gs) % 8 == 0; }

int launch_qgemv_tma(const void *x, int64_t M, int64_t K, const uint32_t *wq, const void *scales,
                     const void *biases, const uint32_t *wq2, const void *scales2, const void *biases2,
                     int64_t N, int gs, int bits, const void *bias, const void *bias2, int act,
                     const void *lora_t, const void *lora_b, int64_t rank, void *y, const Gated &gd, cudaStream_t st) {
    using namespace gemv2;
    const bool sw = act == QL_ACT_SWIGLU;
    Params p{};
    p.gd = gd;
    p.M = (int)M;
    p.N = (int)N;
    p.K = (int)K;
    p.gs = gs;
    p.G = (int)(K / gs);
    p.nks = (int)((K + KS - 1) / KS);
    p.act = act;
    p.x = (const __nv_bfloat16 *)x;
    p.bias = (const __nv_bfloat16 *)bias;
    p.bias2 = (const __nv_bfloat16 *)bias2;
    p.lora_t = (const __nv_bfloat16 *)lora_t;
    p.lora_b = (const __nv_bfloat16 *)lora_b;
    p.rank = (int)rank;
    p.rpad = (int)(rank > 0 ? (rank + 63) / 64 * 64 : 0);
    p.y = (__nv_bfloat16 *)y;

    CUtensorMap maps[6];
    for (int ps = 0; ps < (sw ? 2 : 1); ++ps) {
        const uint32_t *w = ps ? wq2 : wq;
        const void *s = ps ? scales2 : scales, *b = ps ? biases2 : biases;
        // W as words x rows; boxes of 128 B x 16 rows with the 128-byte swizzle
        const uint64_t wd[2] = {(uint64_t)K * bits / 32, (uint64_t)N};
        const uint64_t ws[1] = {(uint64_t)K * bits / 8};
        const uint32_t wb[2] = {32, 16};
        if (int rc = make_map(&maps[3 * ps], CU_TENSOR_MAP_DATA_TYPE_UINT32, w, 2, wd, ws, wb,
                              CU_TENSOR_MAP_SWIZZLE_128B))
            return rc;
        const uint64_t sd[2] = {(uint64_t)p.G, (uint64_t)N};
        const uint64_t ss[1] = {(uint64_t)p.G * 2};
        const uint32_t sbx[2] = {(uint32_t)(KS / gs), 16};
        if (int rc = make_map(&maps[3 * ps + 1], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, s, 2, sd, ss, sbx)) return rc;
        if (int rc = make_map(&maps[3 * ps + 2], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, b, 2, sd, ss, sbx)) return rc;
    }
    if (!sw)
        for (int i = 0; i < 3; ++i) maps[3 + i] = maps[i];
#define QL_GEMV_GS(GS_)                                                                          \
    if (gs == GS_) {                                                                             \
        if (bits == 4) return sw ? launch_t<4, true, GS_>(maps, p, st) : launch_t<4, false, GS_>(maps, p, st); \
        return sw ? launch_t<8, true, GS_>(maps, p, st) : launch_t<8, false, GS_>(maps, p, st);   \
    }
    QL_GEMV_GS(32)
    QL_GEMV_GS(64)
    QL_GEMV_GS(128)
#undef QL_GEMV_GS
    return fail(QL_EUNSUPPORTED, "group size %d", gs);
}

}  // namespace ql
