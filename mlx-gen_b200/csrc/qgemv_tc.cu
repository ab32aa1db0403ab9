// qgemv_tc.cu -- small-M (M <= 8) quantized matmul on tcgen05 tensor cores, fp8 operands.
//
// The decode-time quantized_matmul (few activation rows, src/adapters.rs:309-317) streams
// every packed weight once; its speed is set by the work per code between HBM and the
// accumulator.  A tcgen05.mma with M = 128 costs about the same for any N up to 128, so
// for a handful of tokens the cost per weight code is what matters, and kind::f8f6f4
// (K = 32 per instruction) halves it against kind::f16.  The packed codes reach the MMA
// almost untouched:
//
//   * A nibble q in a byte, read as e4m3, is exactly q * 2^-9 (0x00-0x07 are the
//     subnormals m * 2^-9, 0x08-0x0f the binade [2^-6, 2^-5) with step 2^-9).  So a Q4
//     word w gives two A words with one mask each: w & 0x0f0f0f0f (codes 0,2,4,6) and
//     (w >> 4) & 0x0f0f0f0f (codes 1,3,5,7).  The K order inside each 8 codes becomes
//     0,2,4,6,1,3,5,7, and the activations are laid out in the same order.  Q8 words
//     give a low-nibble and a high-nibble plane the same way (K order c0..c3 low, c0..c3
//     high) and the activations of the high plane carry a factor 16.
//   * The activations (bf16, 8 significant bits) are split exactly into two e4m3 pieces
//     per element with a power-of-two scale per token and quantization group:
//         x * 2^k = hi + lo * 2^-5,  hi = e4m3(x 2^k),  lo = e4m3((x 2^k - hi) 2^5)
//     which reproduces every element down to 2^-10 of its group's largest magnitude.
//     The 8 tokens' hi pieces are MMA rows 0-7 and the lo pieces rows 8-15 (N = 16).
//     Each CTA converts the activations of its K range once, into shared memory, and
//     keeps them there for every row tile it processes.
//   * Every quantization group accumulates into its own 16-column TMEM range; fold warps
//     read it and apply the group's affine map once per row and token:
//         y += s * 2^(9-k) * (D_hi + D_lo / 32) + b * sum_k x_k
//   * A producer warp streams stages of 128 rows x 256 packed bytes, and the scales /
//     biases in batches of 8 groups, with TMA.  The weight stream starts before
//     griddepcontrol.wait, so under programmatic dependent launch it overlaps the end of
//     the previous kernel.
//   * Few output tiles (N small): the K range is split over the CTAs of a cluster and the
//     partial sums are pushed into the leader CTA's shared memory (DSMEM), which runs the
//     epilogue.  No global workspace, no atomics.
//   * SwiGLU: a tile holds 64 gate rows (TMEM lanes 0-63) and the same 64 up rows (lanes
//     64-127); the fold warps pair them through shared memory.
//   * tcgen05.commit stalls the issuing thread until the tensor pipe drains, so the MMAs
//     are issued by three warps in turn, one commit per unit of 128 K elements (256 for
//     Q8 with group size 128), and that one commit tells both the dequant warps (A slot
//     free) and the fold warps (accumulators ready).
// Every mbarrier wait is bounded (ql_common.cuh).  bf16 x / scales / output, group sizes
// 64 and 128 (and 32 for Q8), no LoRA; other cases go to the mma.sync kernels
// (qgemv_tma.cu, qgemv.cu).
#include "ql_common.cuh"

namespace ql {
namespace gemv3 {

constexpr int ROWS = 128;     // weight rows per tile (MMA M)
constexpr int STAGES = 3;     // weight stages of 128 rows x 256 bytes
constexpr int CPS = 4;        // chunks per stage: 64 packed bytes of a row = 128 K elements
constexpr int SBR = 4;        // scale/bias ring (batches of 8 groups)
constexpr int AR = 8;         // A ring: 8 chunks of 32 TMEM columns (columns 0-255)
#ifndef QL_GEMV_NISSUE
#define QL_GEMV_NISSUE 3
#endif
constexpr int NISSUE = QL_GEMV_NISSUE;  // MMA issuer warps (1-3)
constexpr int NTHREADS = 512; // warps: 0 TMA, 1-3 MMA, 4-7 dequant, 8-15 fold (2 sets)
constexpr int NCONV = NTHREADS - 64;  // warps 2-15 convert the activations at the start
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t D_COL = 256;
constexpr int W_BYTES = ROWS * 256;
constexpr int SB_SLOT = 2 * ROWS * 16;
constexpr int MAX_SPLIT = 8;
constexpr int BX_STAGE = 4 * 2048;  // activation bytes per stage: 4 blocks of 128 K x 16 rows

constexpr int SMEM_SB = STAGES * W_BYTES;
constexpr int SMEM_XCH = SMEM_SB + SBR * SB_SLOT;  // SwiGLU exchange [64][8] f32
constexpr int SMEM_ACC = SMEM_XCH + 64 * 8 * 4;    // fold set 1 partial sums [128][8] f32
constexpr int SMEM_BAR = SMEM_ACC + ROWS * 8 * 4;
constexpr int NBAR = 2 * STAGES + 3 * AR + 2 * SBR + 6;
constexpr int SMEM_BX = (SMEM_BAR + NBAR * 8 + 16 + 1023) / 1024 * 1024;
// then: B (activation pieces) [stages of the slice][8 KB], red [(split-1)][128][8] f32,
// ginfo [groups of the slice][8] float2, kscale [groups of the slice][8] f32

struct Params {
    int M, N, K, G;
    int ntiles, rows_out;    // output rows per tile: 128, or 64 for SwiGLU
    int split, sps;          // CTAs per cluster sharing one tile's K range; stages per CTA
    int act;
    const __nv_bfloat16 *x, *bias, *bias2;
    __nv_bfloat16 *y;
    Gated gd;
};

__device__ __forceinline__ void st_cluster_v4(uint32_t addr, float a, float b, float c, float d) {
    asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(a), "f"(b), "f"(c), "f"(d)
                 : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem desc]^T, kind::f8f6f4 (e4m3 in, fp32 accumulate).
__device__ __forceinline__ void tc_mma_ts_f8(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                             uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Instruction descriptor, kind::f8f6f4: e4m3 A and B, fp32 accumulator, both K-major.
__host__ __device__ constexpr uint32_t idesc_e4m3(int M, int N) {
    return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// two floats -> two e4m3 bytes (a in the low byte), round to nearest, saturating
__device__ __forceinline__ uint32_t e4m3x2(float a, float b) {
    uint16_t r;
    asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(b), "f"(a));
    return r;
}
__device__ __forceinline__ void e4m3x2_to_f32(uint32_t v, float &a, float &b) {
    uint32_t h;
    asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h) : "h"((uint16_t)v));
    a = __half2float(__ushort_as_half((unsigned short)(h & 0xffffu)));
    b = __half2float(__ushort_as_half((unsigned short)(h >> 16)));
}

// 16 scaled activations -> 16 hi bytes and 16 lo bytes (x = hi + lo / 32)
__device__ __forceinline__ void split_pieces(const float v[16], uint4 &hi, uint4 &lo) {
    uint32_t h[8], l[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        h[i] = e4m3x2(v[2 * i], v[2 * i + 1]);
        float a, b;
        e4m3x2_to_f32(h[i], a, b);
        l[i] = e4m3x2((v[2 * i] - a) * 32.f, (v[2 * i + 1] - b) * 32.f);
    }
    hi = make_uint4(h[0] | h[1] << 16, h[2] | h[3] << 16, h[4] | h[5] << 16, h[6] | h[7] << 16);
    lo = make_uint4(l[0] | l[1] << 16, l[2] | l[3] << 16, l[4] | l[5] << 16, l[6] | l[7] << 16);
}

template <int BITS, bool SWIGLU, int GS>
__global__ void __launch_bounds__(NTHREADS, 1)
    qgemv_tc_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_w2,
                    const __grid_constant__ CUtensorMap tm_s, const __grid_constant__ CUtensorMap tm_s2,
                    const __grid_constant__ CUtensorMap tm_b, const __grid_constant__ CUtensorMap tm_b2,
                    const Params p) {
    constexpr int CODES_STAGE = 256 * 8 / BITS;   // codes of a row per stage
    constexpr int GPS = CODES_STAGE / GS;         // groups per stage: 2 .. 16
    constexpr int PLANES = BITS == 4 ? 1 : 2;
    constexpr int KPG = GS * PLANES / 32;         // MMA k-steps per group: 1 .. 8
    constexpr int KTOP = BITS == 4 ? 6 : 2;       // x * 2^k < 128 (Q8: 16 x 2^k < 128)
    // A unit is what one issuer handles with one commit: one chunk (128 K elements), or two
    // when a group is longer (Q8, group size 128).  Each unit slot owns 32 * UCH A columns
    // and 16 * GPUN accumulator columns.
    constexpr int UCH = KPG > 4 ? KPG / 4 : 1;    // chunks per unit
    constexpr int KPU = 4 * UCH;                  // k-steps per unit
    constexpr int GPUN = KPU / KPG;               // groups per unit: 1 or 2
    constexpr int AU = AR / UCH;                  // unit slots
    constexpr int UPS = CPS / UCH;                // units per stage
    static_assert(GPUN == 1 || GPUN == 2, "group size");
    static_assert(AU * GPUN * 16 <= 256, "accumulator columns");
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *sb_ring = smem + SMEM_SB;
    float *xch = reinterpret_cast<float *>(smem + SMEM_XCH);
    float *accx = reinterpret_cast<float *>(smem + SMEM_ACC);
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + SMEM_BAR);
    uint64_t *full = bars, *empty = bars + STAGES;
    // per unit slot: A written (dequant -> MMA), MMAs done (-> dequant and fold), D read (fold -> MMA)
    uint64_t *afull = bars + 2 * STAGES, *udone = afull + AR, *dfree = udone + AR;
    uint64_t *sbfull = dfree + AR, *sbempty = sbfull + SBR;
    uint64_t *redfull = sbempty + SBR, *redfree = redfull + 1;
    uint64_t *xchfull = redfree + 1, *xchfree = redfree + 2;  // SwiGLU up rows -> gate rows
    uint64_t *accfull = redfree + 3, *accfree = redfree + 4;  // fold set 1 -> fold set 0, per tile
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + NBAR);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(bars + NBAR) + 1;
    uint8_t *bx = smem + SMEM_BX;                                               // activation pieces
    float *red = reinterpret_cast<float *>(bx + p.sps * BX_STAGE);              // [(split-1)][128][8]
    float2 *ginfo = reinterpret_cast<float2 *>(red + (p.split - 1) * ROWS * 8); // [groups][8] (s-scale, sum x)
    float *kscale = reinterpret_cast<float *>(ginfo + p.sps * GPS * 8);         // [groups][8] 2^k

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int rank = p.split > 1 ? (int)cluster_ctarank() : 0;
    const int cluster = blockIdx.x / p.split, nclusters = gridDim.x / p.split;
    const int nstages = p.K / CODES_STAGE;
    const int st0 = rank * p.sps;
    const int st1 = min(nstages, st0 + p.sps);
    const int nst = st1 > st0 ? st1 - st0 : 0;
    const int ngroups = nst * GPS;
    const int nbatch = ngroups / 8;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 4);  // 4 dequant warps
        }
        for (int a = 0; a < AR; ++a) {
            mbar_init(&afull[a], 4);
            mbar_init(&udone[a], 1);
            mbar_init(&dfree[a], 4);
        }
        for (int b = 0; b < SBR; ++b) {
            mbar_init(&sbfull[b], 1);
            mbar_init(&sbempty[b], 2 * ROWS);  // both fold sets
        }
        mbar_init(redfull, p.split > 1 ? (p.split - 1) * ROWS : 1);
        mbar_init(redfree, ROWS);
        mbar_init(xchfull, 64);
        mbar_init(xchfree, 64);
        mbar_init(accfull, ROWS);
        mbar_init(accfree, ROWS);
        *abort_flag = 0;
        mbar_fence_init();
    }
    __syncthreads();
    if (p.split > 1) cluster_sync_all();  // peers' barriers are initialised before any remote arrive
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    // the TMEM allocation happens off the producer's path: the weight stream starts now and
    // the TMEM users pick the address up at the barrier below
    if (warp == 1) {
        tmem_alloc(tmem_slot, TMEM_COLS);
        tc_fence_before();
    }

    if (warp >= 2) {
        // ---------------------------------------------- activations -> e4m3 pieces in smem
        asm volatile("griddepcontrol.wait;" ::: "memory");
        const int tid = threadIdx.x - 64;
        // pass 1: per (group, token) the power-of-two scale and the exact sum
        for (int i = tid; i < ngroups * 8; i += NCONV) {
            const int g = i >> 3, t = i & 7;
            float amax = 0.f, sum = 0.f;
            if (t < p.M) {
                const uint4 *xp = reinterpret_cast<const uint4 *>(p.x + (int64_t)t * p.K +
                                                                  (int64_t)(st0 * GPS + g) * GS);
#pragma unroll 4
                for (int e = 0; e < GS / 8; ++e) {
                    const uint4 v = xp[e];
                    const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const float a = bf16lo(w4[j]), b = bf16hi(w4[j]);
                        sum += a + b;
                        amax = fmaxf(amax, fmaxf(fabsf(a), fabsf(b)));
                    }
                }
            }
            const int ea = (int)((__float_as_uint(amax) >> 23) & 0xff) - 127;
            // 2^k and 2^(9-k) must both be normal floats: k in [-118, 127] (a subnormal
            // group max gives ea = -127 and the largest scale, 2^127)
            const int k = max(-118, min(127, KTOP - ea));
            kscale[i] = __int_as_float((k + 127) << 23);
            ginfo[i] = make_float2(__int_as_float((9 - k + 127) << 23), sum);
        }
        named_bar_sync(2, NCONV);
        // pass 2: per (128-K block, token row, 16-element piece): hi row t, lo row 8 + t,
        // 128-byte swizzled K-major rows as the MMA's B operand reads them
        const int npieces = nst * 4 * 8 * 8;
        for (int i = tid; i < npieces; i += NCONV) {
            const int j = i & 7, t = (i >> 3) & 7, blk = i >> 6;
            uint4 hi = make_uint4(0, 0, 0, 0), lo = hi;
            if (t < p.M) {
                float v[16];
                if (BITS == 4) {
                    // 16 K elements = 16 codes, K order 0,2,4,6,1,3,5,7 within each 8
                    const int c0 = blk * 128 + j * 16;  // code offset in the slice
                    const float sc = kscale[(c0 / GS) * 8 + t];
                    const uint4 *xp = reinterpret_cast<const uint4 *>(p.x + (int64_t)t * p.K +
                                                                      (int64_t)st0 * CODES_STAGE + c0);
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const uint4 u = xp[h];
                        const uint32_t w4[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
                        for (int q = 0; q < 4; ++q) {
                            v[8 * h + q] = bf16lo(w4[q]) * sc;      // even codes
                            v[8 * h + 4 + q] = bf16hi(w4[q]) * sc;  // odd codes
                        }
                    }
                } else {
                    // 16 K elements = 8 codes: c0..c3 low plane, c0..c3 high plane (x16)
                    const int c0 = blk * 64 + j * 8;
                    const float sc = kscale[(c0 / GS) * 8 + t];
                    const uint4 u = *reinterpret_cast<const uint4 *>(p.x + (int64_t)t * p.K +
                                                                     (int64_t)st0 * CODES_STAGE + c0);
                    const float xs[8] = {bf16lo(u.x), bf16hi(u.x), bf16lo(u.y), bf16hi(u.y),
                                         bf16lo(u.z), bf16hi(u.z), bf16lo(u.w), bf16hi(u.w)};
#pragma unroll
                    for (int h = 0; h < 2; ++h)
#pragma unroll
                        for (int q = 0; q < 4; ++q) {
                            v[8 * h + q] = xs[4 * h + q] * sc;
                            v[8 * h + 4 + q] = (xs[4 * h + q] * sc) * 16.f;  // sc may be 2^127
                        }
                }
                split_pieces(v, hi, lo);
            }
            uint8_t *bb = bx + blk * 2048 + t * 128 + ((j ^ (t & 7)) << 4);
            *reinterpret_cast<uint4 *>(bb) = hi;
            *reinterpret_cast<uint4 *>(bb + 1024) = lo;
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // visible to tcgen05.mma
    }
    if (warp >= 1) named_bar_sync(1, NTHREADS - 32);  // warps 1-15: pieces, group info and TMEM ready
    tc_fence_after();
    const uint32_t tmem = warp >= 1 ? *tmem_slot : 0u;

    if (warp == 0) {
        // ---------------------------------------------------------------- TMA producer
        if (lane == 0) {
            uint32_t it = 0, sbc = 0;
            bool ok = true;
            for (int tile = cluster; tile < p.ntiles && ok; tile += nclusters) {
                const int r0 = tile * p.rows_out;
                for (int st = st0; st < st1; ++st, ++it) {
                    for (int g8 = st * GPS; g8 < (st + 1) * GPS; g8 += 8) {
                        if (g8 % 8) continue;  // GPS < 8: the batch started in an earlier stage
                        const int b = sbc % SBR;
                        if (!mbar_wait(&sbempty[b], ((sbc / SBR) & 1) ^ 1, abort_flag,
                                                  DEV_ERR_TIMEOUT_EMPTY)) {
                            ok = false;
                            break;
                        }
                        uint8_t *sp = sb_ring + b * SB_SLOT;
                        mbar_arrive_expect_tx(&sbfull[b], SB_SLOT);
                        tma_load_2d(sp, &tm_s, &sbfull[b], g8, r0);
                        tma_load_2d(sp + ROWS * 16, &tm_b, &sbfull[b], g8, r0);
                        if (SWIGLU) {
                            tma_load_2d(sp + 64 * 16, &tm_s2, &sbfull[b], g8, r0);
                            tma_load_2d(sp + ROWS * 16 + 64 * 16, &tm_b2, &sbfull[b], g8, r0);
                        }
                        ++sbc;
                    }
                    if (!ok) break;
                    const int s = it % STAGES;
                    if (!mbar_wait(&empty[s], ((it / STAGES) & 1) ^ 1, abort_flag, DEV_ERR_TIMEOUT_EMPTY)) {
                        ok = false;
                        break;
                    }
                    uint8_t *sp = smem + s * W_BYTES;
                    mbar_arrive_expect_tx(&full[s], W_BYTES);
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        tma_load_2d(sp + h * (ROWS * 128), &tm_w, &full[s], st * 64 + h * 32, r0);
                        if (SWIGLU)
                            tma_load_2d(sp + h * (ROWS * 128) + 64 * 128, &tm_w2, &full[s], st * 64 + h * 32, r0);
                    }
                }
            }
        }
    } else if (warp <= NISSUE) {
        // ------------------------------------------------ MMA issuers (warps 1-3, round robin)
        // A commit stalls its thread until the tensor pipe drains, so units alternate
        // between issuer warps: one warp's commit overlaps the others' MMAs.
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_e4m3(ROWS, 16);
            const uint32_t bxs = smem_u32(bx);
            const int upt = nst * UPS;  // units per tile
            uint32_t u = 0;
            bool ok = true;
            for (int tile = cluster; tile < p.ntiles && ok; tile += nclusters) {
#pragma unroll 1
                for (int uu = 0; uu < upt; ++uu, ++u) {
                    if ((int)(u % NISSUE) != warp - 1) continue;
                    const int us = u % AU;
                    const uint32_t ph = (u / AU) & 1;
                    if (!mbar_wait(&afull[us], ph, abort_flag, DEV_ERR_TIMEOUT_FULL) ||
                        !mbar_wait(&dfree[us], ph ^ 1, abort_flag, DEV_ERR_TIMEOUT_ACC)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t dbase = tmem + D_COL + us * GPUN * 16, abase = tmem + us * 32 * UCH;
#pragma unroll
                    for (int ks = 0; ks < KPU; ++ks) {
                        const int c = uu * UCH + ks / 4;  // chunk of the slice = 128-K block of B
                        const uint64_t bdesc = umma_desc_k_sw128(bxs + c * 2048) + 2 * (ks % 4);
                        tc_mma_ts_f8(dbase + (ks / KPG) * 16, abase + ks * 8, bdesc, idesc, (ks % KPG) ? 1u : 0u);
                    }
                    tc_commit(&udone[us]);
                }
            }
        }
    } else if (warp >= 4 && warp < 8) {
        // ---------------------------------------------------------------- dequant warps
        const int q = warp & 3, row = q * 32 + lane;
        const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16);
        uint32_t it = 0, u = 0;
        bool ok = true;
        for (int tile = cluster; tile < p.ntiles && ok; tile += nclusters) {
            for (int st = st0; st < st1 && ok; ++st, ++it) {
                const int s = it % STAGES;
                if (!mbar_wait(&full[s], (it / STAGES) & 1, abort_flag,
                                                           DEV_ERR_TIMEOUT_FULL)) {
                    ok = false;
                    break;
                }
                const uint8_t *wrow = smem + s * W_BYTES + row * 128;
                // the loads of unit j + 1 are issued while unit j's TMEM store is in flight
                uint4 wv[4 * UCH];
                auto load_unit = [&](int j) {
#pragma unroll
                    for (int ch = 0; ch < UCH; ++ch) {
                        const int c = j * UCH + ch;  // chunk of the stage: 64 bytes of the row
                        const int h = c >> 1, j0 = (c & 1) * 4;
#pragma unroll
                        for (int i = 0; i < 4; ++i)
                            wv[4 * ch + i] =
                                *reinterpret_cast<const uint4 *>(wrow + h * (ROWS * 128) + (((j0 + i) ^ (row & 7)) << 4));
                    }
                };
                load_unit(0);
#pragma unroll
                for (int j = 0; j < UPS; ++j, ++u) {
                    const int us = u % AU;
                    if (!mbar_wait(&udone[us], ((u / AU) & 1) ^ 1, abort_flag,
                                                               DEV_ERR_TIMEOUT_EMPTY)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
#pragma unroll
                    for (int ch = 0; ch < UCH; ++ch) {
                        uint32_t r[32];
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            const uint4 w = wv[4 * ch + i];
                            const uint32_t w4[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                            for (int e = 0; e < 4; ++e) {
                                r[8 * i + 2 * e] = w4[e] & 0x0f0f0f0fu;
                                r[8 * i + 2 * e + 1] = (w4[e] >> 4) & 0x0f0f0f0fu;
                            }
                        }
                        tmem_st32(taddr + us * 32 * UCH + ch * 32, r);
                    }
                    if (j + 1 < UPS) {
                        load_unit(j + 1);
                    } else {
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&empty[s]);  // the stage's weights are all in registers
                    }
                    tmem_st_wait();
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&afull[us]);
                }
            }
        }
    } else if (warp >= 8) {
        // ------------------------------------------------- fold warps: two sets, units alternate
        const int fset = (warp - 8) >> 2;
        const int q = warp & 3, row = q * 32 + lane;
        const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + D_COL;
        const int upt = nst * UPS, upb = 8 / GPUN;  // units per tile, per batch of 8 groups
        uint32_t u = 0, sbc = 0, tc = 0;
        bool ok = true;
        for (int tile = cluster; tile < p.ntiles && ok; tile += nclusters, ++tc) {
            float acc[8];
#pragma unroll
            for (int t = 0; t < 8; ++t) acc[t] = 0.f;
#pragma unroll 1
            for (int ub = 0; ub < upt && ok; ub += upb, ++sbc) {
                const int b = sbc % SBR;
                if (!mbar_wait(&sbfull[b], (sbc / SBR) & 1, abort_flag,
                                                           DEV_ERR_TIMEOUT_FULL)) {
                    ok = false;
                    break;
                }
                const uint8_t *sp = sb_ring + b * SB_SLOT;
#pragma unroll 1
                for (int uu = ub + fset; uu < ub + upb; uu += 2) {
                    const uint32_t uc = u + (uu - ub);  // unit counter of this unit
                    const int us = uc % AU;
                    if (!mbar_wait(&udone[us], (uc / AU) & 1, abort_flag,
                                                               DEV_ERR_TIMEOUT_ACC)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    uint32_t v[16 * GPUN];
                    if (GPUN == 2)
                        tmem_ld32(taddr + us * 32, v);
                    else
                        tmem_ld16(taddr + us * 16, v);
                    tmem_ld_wait();
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&dfree[us]);
#pragma unroll
                    for (int gi = 0; gi < GPUN; ++gi) {
                        const int g = uu * GPUN + gi, j8 = g & 7;
                        const float sc = __uint_as_float(
                            (uint32_t)*reinterpret_cast<const uint16_t *>(sp + row * 16 + j8 * 2) << 16);
                        const float bi = __uint_as_float(
                            (uint32_t)*reinterpret_cast<const uint16_t *>(sp + ROWS * 16 + row * 16 + j8 * 2) << 16);
                        const float2 *gp = ginfo + g * 8;
#pragma unroll
                        for (int t = 0; t < 8; ++t)
                            if (t < p.M) {
                                const float2 g2 = gp[t];
                                const float dot =
                                    fmaf(__uint_as_float(v[16 * gi + 8 + t]), 0.03125f, __uint_as_float(v[16 * gi + t]));
                                acc[t] = fmaf(sc * g2.x, dot, fmaf(bi, g2.y, acc[t]));
                            }
                    }
                }
                u += upb;
                mbar_arrive(&sbempty[b]);
            }
            if (!ok) break;
            // set 1 hands its partial sums to set 0, which finishes the tile
            if (fset == 1) {
                if (!mbar_wait(accfree, (tc & 1) ^ 1, abort_flag, DEV_ERR_TIMEOUT_ACC)) break;
                float4 *ap = reinterpret_cast<float4 *>(accx + row * 8);
                ap[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
                ap[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
                mbar_arrive(accfull);
                continue;
            }
            if (!mbar_wait(accfull, tc & 1, abort_flag, DEV_ERR_TIMEOUT_ACC)) break;
            {
                const float4 *ap = reinterpret_cast<const float4 *>(accx + row * 8);
                const float4 a0 = ap[0], a1 = ap[1];
                acc[0] += a0.x;
                acc[1] += a0.y;
                acc[2] += a0.z;
                acc[3] += a0.w;
                acc[4] += a1.x;
                acc[5] += a1.y;
                acc[6] += a1.z;
                acc[7] += a1.w;
                mbar_arrive(accfree);
            }
            if (!ok) break;
            if (p.split > 1) {
                if (rank != 0) {
                    // push the partial sums into the leader's buffer for this rank
                    if (!mbar_wait<true>(redfree, (tc & 1) ^ 1, abort_flag, DEV_ERR_TIMEOUT_ACC)) {
                        ok = false;
                        break;
                    }
                    const uint32_t dst = mapa_shared(smem_u32(red + ((rank - 1) * ROWS + row) * 8), 0);
                    st_cluster_v4(dst, acc[0], acc[1], acc[2], acc[3]);
                    st_cluster_v4(dst + 16, acc[4], acc[5], acc[6], acc[7]);
                    mbar_arrive_cluster(mapa_shared(smem_u32(redfull), 0));
                    continue;
                }
                if (!mbar_wait<true>(redfull, tc & 1, abort_flag, DEV_ERR_TIMEOUT_ACC)) {
                    ok = false;
                    break;
                }
                for (int r = 0; r < p.split - 1; ++r) {
                    const float4 *rp = reinterpret_cast<const float4 *>(red + (r * ROWS + row) * 8);
                    const float4 u0 = rp[0], u1 = rp[1];
                    acc[0] += u0.x;
                    acc[1] += u0.y;
                    acc[2] += u0.z;
                    acc[3] += u0.w;
                    acc[4] += u1.x;
                    acc[5] += u1.y;
                    acc[6] += u1.z;
                    acc[7] += u1.w;
                }
                for (int r = 1; r < p.split; ++r) mbar_arrive_cluster(mapa_shared(smem_u32(redfree), (uint32_t)r));
            }
            // epilogue: round the matmul, add the bias (second rounding), activation, store
            const int n = SWIGLU ? tile * 64 + (row & 63) : tile * ROWS + row;
            const __nv_bfloat16 *bp = (SWIGLU && row >= 64) ? p.bias2 : p.bias;
            const float bias = (bp && n < p.N) ? __bfloat162float(bp[n]) : 0.f;
            float v8[8];
#pragma unroll
            for (int t = 0; t < 8; ++t) {
                float v = round_bf16(acc[t]);
                if (bp) v = round_bf16(v + bias);
                v8[t] = v;
            }
            if (SWIGLU) {
                // up rows hand their values to the gate rows (bounded mbarrier waits, so an
                // aborted warp cannot strand the others)
                if (row >= 64) {
                    if (!mbar_wait(xchfree, (tc & 1) ^ 1, abort_flag, DEV_ERR_TIMEOUT_ACC)) break;
#pragma unroll
                    for (int t = 0; t < 8; ++t) xch[(row - 64) * 8 + t] = v8[t];
                    mbar_arrive(xchfull);
                } else {
                    if (!mbar_wait(xchfull, tc & 1, abort_flag, DEV_ERR_TIMEOUT_ACC)) break;
                    if (n < p.N)
#pragma unroll
                        for (int t = 0; t < 8; ++t)
                            if (t < p.M) {
                                const float g = v8[t];
                                p.y[(int64_t)t * p.N + n] = __float2bfloat16_rn(
                                    apply_gated(g / (1.0f + __expf(-g)) * xch[row * 8 + t], p.gd, t, n, p.N));
                            }
                    mbar_arrive(xchfree);
                }
            } else if (n < p.N) {
#pragma unroll
                for (int t = 0; t < 8; ++t)
                    if (t < p.M) {
                        float v = v8[t];
                        if (p.act == QL_ACT_GELU_TANH) {
                            float th;
                            const float inner = 0.7978845608028654f * (v + 0.044715f * v * v * v);
                            asm("tanh.approx.f32 %0, %1;" : "=f"(th) : "f"(inner));
                            v = 0.5f * v * (1.0f + th);
                        } else if (p.act == QL_ACT_GELU_ERF) {
                            v = 0.5f * v * (1.0f + erff(v * 0.7071067811865476f));
                        }
                        p.y[(int64_t)t * p.N + n] = __float2bfloat16_rn(apply_gated(v, p.gd, t, n, p.N));
                    }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (p.split > 1) cluster_sync_all();  // no CTA leaves while a peer may still write to it
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, TMEM_COLS);
    }
}

// ------------------------------------------------------------------ host side

static int make_map(CUtensorMap *map, CUtensorMapDataType dt, const void *base, const uint64_t *dims,
                    uint64_t stride_bytes, const uint32_t *box, CUtensorMapSwizzle sw) {
    gemm::PFN_encodeTiled enc = gemm::get_encode();
    if (!enc) return fail(QL_ECUDA, "cuTensorMapEncodeTiled unavailable");
    cuuint64_t d[2] = {dims[0], dims[1]}, st[1] = {stride_bytes};
    cuuint32_t b[2] = {box[0], box[1]}, e[2] = {1, 1};
    CUresult r = enc(map, dt, 2, const_cast<void *>(base), d, st, b, e, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(QL_ECUDA, "cuTensorMapEncodeTiled (gemv tc) failed (%d)", (int)r);
    return QL_OK;
}

static size_t smem_bytes(int split, int sps, int gps) {
    const size_t groups = (size_t)sps * gps;
    return 1024 + SMEM_BX + (size_t)sps * BX_STAGE + (size_t)(split - 1) * ROWS * 8 * 4 + groups * 8 * 8 +
           groups * 8 * 4;
}

static int stages_per_cta(int nstages, int unit, int split) {
    int sp = (nstages + split - 1) / split;
    return (sp + unit - 1) / unit * unit;
}

// Split of the K range over a cluster: fewest (waves x stages per CTA), ties to the smaller split.
static bool plan(int bits, int gs, int64_t K, int ntiles, int sms, int *split, int *sps) {
    const int GPS = 256 * 8 / bits / gs;
    const int nstages = (int)(K / (256 * 8 / bits));
    const int unit = GPS >= 8 ? 1 : 8 / GPS;  // slices start on a batch of 8 groups
    int64_t best = -1;
    for (int s = 1; s <= MAX_SPLIT; ++s) {
        const int sp = stages_per_cta(nstages, unit, s);
        if (s > 1 && (int64_t)(s - 1) * sp >= nstages) continue;  // a CTA would get no K
        if (smem_bytes(s, sp, GPS) > 227 * 1024) continue;
        const int resident = sms / s;
        const int64_t waves = (ntiles + resident - 1) / resident;
        const int64_t cost = waves * (sp + 2) + sp / 4;  // + pipeline fill / epilogue per tile, + conversion
        if (best < 0 || cost < best) {
            best = cost;
            *split = s;
            *sps = sp;
        }
    }
    return best >= 0;
}

template <int BITS, bool SWIGLU, int GS>
static int launch_t(const CUtensorMap *maps, const Params &p, size_t smem, int sms, cudaStream_t st) {
    auto kfn = qgemv_tc_kernel<BITS, SWIGLU, GS>;
    QL_CUDA_TRY(cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    const int nclusters = std::min(p.ntiles, std::max(1, sms / p.split));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(nclusters * p.split));
    cfg.blockDim = dim3(NTHREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    static const bool no_pdl = getenv("QL_GEMV_NOPDL") != nullptr;  // tuning switch
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = no_pdl ? 0 : 1;
    int na = 1;
    if (p.split > 1) {
        attr[1].id = cudaLaunchAttributeClusterDimension;
        attr[1].val.clusterDim.x = (unsigned)p.split;
        attr[1].val.clusterDim.y = 1;
        attr[1].val.clusterDim.z = 1;
        na = 2;
    }
    cfg.attrs = attr;
    cfg.numAttrs = na;
    QL_CUDA_TRY(cudaLaunchKernelEx(&cfg, kfn, maps[0], maps[1], maps[2], maps[3], maps[4], maps[5], p));
    return QL_OK;
}

}  // namespace gemv3

// Shapes the tcgen05 GEMV takes: M <= 8, K a whole number of stages (256 bytes of each
// packed row) and of 8-group batches, 16-byte aligned operands, no LoRA.
bool qgemv_tc_supported(int64_t M, int64_t K, int gs, int bits, const void *x, bool lora) {
    if (lora || M < 1 || M > 8 || (bits != 4 && bits != 8)) return false;
    if (gs != 64 && gs != 128 && !(gs == 32 && bits == 8)) return false;  // Q4 / 32: too many accumulator columns
    if (reinterpret_cast<uintptr_t>(x) % 16) return false;
    const int64_t per_stage = 256 * 8 / bits;
    if (K % per_stage != 0 || (K / gs) % 8 != 0 || K > (1 << 20)) return false;
    // the activations of a CTA's K range live in shared memory: some split must fit
    int split = 0, sps = 0;
    return gemv3::plan(bits, gs, K, 1, 148, &split, &sps);
}

int launch_qgemv_tc(const void *x, int64_t M, int64_t K, const uint32_t *wq, const void *scales, const void *biases,
                    const uint32_t *wq2, const void *scales2, const void *biases2, int64_t N, int gs, int bits,
                    const void *bias, const void *bias2, int act, void *y, const Gated &gd, cudaStream_t st) {
    using namespace gemv3;
    const bool sw = act == QL_ACT_SWIGLU;
    Params p{};
    p.gd = gd;
    p.M = (int)M;
    p.N = (int)N;
    p.K = (int)K;
    p.G = (int)(K / gs);
    p.rows_out = sw ? 64 : ROWS;
    p.ntiles = (int)((N + p.rows_out - 1) / p.rows_out);
    p.act = act;
    p.x = (const __nv_bfloat16 *)x;
    p.bias = (const __nv_bfloat16 *)bias;
    p.bias2 = (const __nv_bfloat16 *)bias2;
    p.y = (__nv_bfloat16 *)y;
    int dev = 0, sms = 148;
    QL_CUDA_TRY(cudaGetDevice(&dev));
    QL_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    const int GPS = 256 * 8 / bits / gs, unit = GPS >= 8 ? 1 : 8 / GPS;
    if (!plan(bits, gs, K, p.ntiles, sms, &p.split, &p.sps)) return fail(QL_EUNSUPPORTED, "GEMV (tcgen05): K too large");
    static const int force_split = getenv("QL_GEMV_SPLIT") ? atoi(getenv("QL_GEMV_SPLIT")) : 0;  // tuning switch
    if (force_split > 0 && force_split <= MAX_SPLIT) {
        const int nst = (int)(K / (256 * 8 / bits)), sp = stages_per_cta(nst, unit, force_split);
        if ((force_split == 1 || (int64_t)(force_split - 1) * sp < nst) && smem_bytes(force_split, sp, GPS) <= 227 * 1024) {
            p.split = force_split;
            p.sps = sp;
        }
    }
    const size_t smem = smem_bytes(p.split, p.sps, GPS);

    CUtensorMap maps[6];
    const uint32_t rows_box = sw ? 64 : ROWS;
    for (int ps = 0; ps < (sw ? 2 : 1); ++ps) {
        const uint32_t *w = ps ? wq2 : wq;
        const void *s = ps ? scales2 : scales, *b = ps ? biases2 : biases;
        const uint64_t wd[2] = {(uint64_t)K * bits / 32, (uint64_t)N};
        const uint32_t wb[2] = {32, rows_box};
        if (int rc = make_map(&maps[ps], CU_TENSOR_MAP_DATA_TYPE_UINT32, w, wd, (uint64_t)K * bits / 8, wb,
                              CU_TENSOR_MAP_SWIZZLE_128B))
            return rc;
        const uint64_t sd[2] = {(uint64_t)p.G, (uint64_t)N};
        const uint32_t sbx[2] = {8, rows_box};
        if (int rc = make_map(&maps[2 + ps], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, s, sd, (uint64_t)p.G * 2, sbx,
                              CU_TENSOR_MAP_SWIZZLE_NONE))
            return rc;
        if (int rc = make_map(&maps[4 + ps], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, b, sd, (uint64_t)p.G * 2, sbx,
                              CU_TENSOR_MAP_SWIZZLE_NONE))
            return rc;
    }
    if (!sw) {
        maps[1] = maps[0];
        maps[3] = maps[2];
        maps[5] = maps[4];
    }
#define QL_GEMV_TC(B_, GS_)                                                                          \
    if (bits == B_ && gs == GS_)                                                                     \
        return sw ? launch_t<B_, true, GS_>(maps, p, smem, sms, st) : launch_t<B_, false, GS_>(maps, p, smem, sms, st);
    QL_GEMV_TC(4, 64)
    QL_GEMV_TC(4, 128)
    QL_GEMV_TC(8, 32)
    QL_GEMV_TC(8, 64)
    QL_GEMV_TC(8, 128)
#undef QL_GEMV_TC
    return fail(QL_EUNSUPPORTED, "group size %d", gs);
}

}  // namespace ql
