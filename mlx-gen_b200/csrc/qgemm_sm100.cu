// qgemm_sm100.cu -- large-M quantized GEMM on tcgen05 tensor cores (sm_100a).
//
// Computes y[M, N] = x[M, K] . dequant(W)[N, K]^T (+ LoRA residual) with a
// fused bias / GELU / SwiGLU epilogue.  This replaces MLX's quantized_matmul as
// called by LinearBase::forward (src/adapters.rs:309-320) for bf16 activations.
//
// Design (B200-first, not a translation of any reference kernel):
//   * The MMA is transposed: D^T = W_tile . x_tile^T.  The 128 weight rows of a
//     tile are the MMA's M side and live in TENSOR MEMORY as the A operand; the
//     256 tokens of the tile are the N side and stream through shared memory.
//     Dequantized weights therefore never round-trip through shared memory:
//     packed words arrive by TMA, dequant warps turn them into bf16 in
//     registers and write them straight into TMEM with tcgen05.st.  Shared
//     memory bandwidth is spent only on the x tiles the MMA reads.
//   * Warp roles in a 512-thread CTA (one CTA per SM, persistent over tiles):
//       warp 0      TMA producer (x tile + packed W tile per k-step)
//       warp 1      TMEM allocator and single-thread tcgen05.mma issuer
//       warps 4-7   epilogue (TMEM -> registers -> bias/act -> global)
//       warps 8-15  two dequant warpgroups, alternating k-steps
//   * Pipelines: STAGES-deep smem ring (x + packed W) and a 4-slot TMEM ring of
//     dequantized A tiles, each guarded by full/empty mbarriers.  The fp32
//     accumulator (128 lanes x 256 columns) occupies TMEM columns [0, 256).
//   * LoRA: the residual s.(x.A).B is folded into the same accumulator as extra
//     k-steps: T = s.(x.A) (a small pre-pass, [M, r_pad] bf16) is the smem
//     operand and B^T (rows of B for this tile) is written to TMEM as A.
//   * SwiGLU: a tile holds 64 rows of W1 (gate) in TMEM lanes 0-63 and the same
//     64 rows of W3 (up) in lanes 64-127; the epilogue pairs them through smem.
//   * Every mbarrier wait is bounded (ql_common.cuh mbar_wait); on timeout the
//     kernel records an error, every role drains, and TMEM is freed.
#include <stdio.h>
#include <stdlib.h>

#include "ql_common.cuh"

namespace ql {

namespace gemm {

#define expr (expr)

constexpr int BT = 256;        // tokens per tile (MMA N)
constexpr int BW = 128;        // weight rows per CTA per tile (MMA M per CTA)
constexpr int BK = 64;         // K per pipeline step (one 128-byte swizzle row of bf16)
constexpr int AST = 4;         // TMEM A ring depth (32 columns each)
constexpr int KR = 8;          // k-step completion ring (>= STAGES and AST)
constexpr int SBR = 8;         // scale/bias ring depth (k-steps staged ahead by warp 2)
constexpr int NTHREADS = 512;
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t ACC_COL = 0;
constexpr uint32_t A_COL = 256;
constexpr uint32_t STG_COL = 384;   // bf16 staging of the finished tile (128 columns)

// CG = CTAs per MMA: 1 (cta_group::1, 128 x 256 tile per CTA) or 2 (a CTA pair runs
// cta_group::2 MMAs on a 256 x 256 tile; each CTA holds 128 weight rows in its TMEM and
// stages 128 of the 256 tokens in its smem, which halves the x traffic per SM).
// LOKR: a dense bf16 LoKr delta tile (128 rows x 64 K, 128-byte swizzled) travels with
// each packed-W stage; three stages leave room for it.
template <int BITS, int CG, bool LOKR = false>
struct Cfg {
    static constexpr int STAGES = LOKR ? 3 : (CG == 1 ? 5 : (BITS == 4 ? 8 : 7));  // smem ring depth
    static constexpr int XROWS = BT / CG;                          // tokens staged per CTA
    static constexpr int X_STAGE_BYTES = XROWS * BK * 2;           // 32 KB / 16 KB
    static constexpr int W_ROW_BYTES = BK * BITS / 8;              // 32 (Q4) / 64 (Q8)
    static constexpr int W_STAGE_BYTES = BW * W_ROW_BYTES;         // 4 KB / 8 KB
    static constexpr int W_BOX_WORDS = BK * BITS / 32;             // 8 / 16
    static constexpr int SMEM_X = 0;
    static constexpr int SMEM_W = SMEM_X + STAGES * X_STAGE_BYTES;
    static constexpr int D_STAGE_BYTES = LOKR ? BW * BK * 2 : 0;   // 16 KB
    static constexpr int SMEM_D = SMEM_W + STAGES * W_STAGE_BYTES;    // LoKr delta tiles (1 KB aligned)
    static constexpr int SMEM_XCH = SMEM_D + STAGES * D_STAGE_BYTES;  // swiglu exchange
    static constexpr int XCH_BYTES = 64 * 33 * 4;
    static constexpr int SMEM_SB = SMEM_XCH + XCH_BYTES;             // scale/bias ring
    static constexpr int SB_SLOT_BYTES = BW * 8;                      // {s0 b0, s1 b1} per row
    static constexpr int SMEM_BAR = SMEM_SB + SBR * SB_SLOT_BYTES;
    static constexpr int NBAR = 3 * STAGES + AST + KR + 2 + 2 * SBR;
    static_assert(KR >= STAGES && KR >= AST, "k-step ring");
    static constexpr int SMEM_MISC = SMEM_BAR + NBAR * 8;
    static constexpr int SMEM_TOTAL = SMEM_MISC + 16 + 1024;  // + alignment slack
};

struct Params {
    int M, N, K;            // N: output columns (for SwiGLU, rows of W1 == rows of W3)
    int gs, G;              // group size, groups per row
    int ktw;                // k-steps over W (ceil(K / BK))
    int ktl;                // LoRA k-steps (ceil(rank_pad / BK)), 0 if none
    int act;
    int num_w_tiles, num_t_tiles;
    const __nv_bfloat16 *scales, *biases;
    const __nv_bfloat16 *scales2, *biases2;  // SwiGLU up projection
    const __nv_bfloat16 *bias, *bias2;
    const __nv_bfloat16 *lora_b;             // [rank, N]
    int lora_rank;
    __nv_bfloat16 *y;
};

__device__ __forceinline__ float gelu_tanh_f(float x) {
    const float k0 = 0.7978845608028654f, k1 = 0.044715f;
    float t;
    const float inner = k0 * (x + k1 * x * x * x);
    asm("tanh.approx.f32 %0, %1;" : "=f"(t) : "f"(inner));
    return 0.5f * x * (1.0f + t);
}

__device__ __forceinline__ float gelu_erf_f(float x) {
    return 0.5f * x * (1.0f + erff(x * 0.7071067811865476f));
}

__device__ __forceinline__ float silu_f(float x) { return x / (1.0f + __expf(-x)); }

// The kernel body.  GATED compiles the gated-residual epilogue in; it is a separate
// __global__ entry point with its own parameter (qgemm_gated_kernel), so the plain
// kernel's code and parameter block are exactly those of a kernel without it (a larger
// Params block measurably slowed the plain kernel).
// LOKR: the dequant warps add lokr_scale * dW (a dense bf16 [N, K] delta staged by TMA with
// the packed weights) to each dequantized weight, so a LoKr adapter costs no extra MMA.
// X3: the split path for f32 / f16 activations.  x arrives as two bf16 pieces (x = hi +
// lo, [M, 2 * Kp] with Kp = ktw * BK, lo at column Kp) and each dequantized weight w (fp32,
// one rounding as the reference's dequantize) as two bf16 pieces (w = whi + wlo); the
// k-steps run three times over K -- whi.hi, whi.lo, wlo.hi -- into the one fp32
// accumulator, and the epilogue writes f32 or f16.  See launch_qgemm_x3.
constexpr int QL_EPI_OUT_F32 = 0x200;  // Params::act flags of the X3 path
constexpr int QL_EPI_OUT_F16 = 0x400;
constexpr int QL_EPI_SB_F16 = 0x800;

template <int BITS, bool SWIGLU, int CG, bool GATED, bool LOKR = false, bool X3 = false>
__device__ __forceinline__ void qgemm_body(const CUtensorMap &tm_x, const CUtensorMap &tm_w, const CUtensorMap &tm_w2,
                                           const CUtensorMap &tm_t, const Params &p, const Gated &gd,
                                           const CUtensorMap *tm_d = nullptr, uint32_t lokr_scale2 = 0) {
    using C = Cfg<BITS, CG, LOKR>;
    constexpr int STAGES = C::STAGES;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                ~uintptr_t(1023));
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + C::SMEM_BAR);
    uint64_t *xfull = bars;                 // x halves landed (used in the leader CTA)
    uint64_t *wfull = bars + STAGES;        // packed W landed (local)
    uint64_t *empty = bars + 2 * STAGES;    // packed W of the stage read by the local dequant warps
    uint64_t *afull = bars + 3 * STAGES;    // TMEM A slot written (leader: both CTAs' warps)
    // MMAs of k-step i complete (one commit per step: a commit stalls the issuing thread
    // until the tensor pipe drains).  It frees the x stage (producer, step i + STAGES) and
    // the TMEM A slot (dequant, step i + AST).
    uint64_t *kdone = afull + AST;
    uint64_t *accfull = kdone + KR;         // accumulator complete
    uint64_t *accempty = accfull + 1;       // accumulator drained (leader: both CTAs' warps)
    uint64_t *sbfull = accempty + 1;        // scale/bias slot written (warp 2, 32 lanes)
    uint64_t *sbempty = sbfull + SBR;       // scale/bias slot read (4 dequant warps)
    uint2 *sb_ring = reinterpret_cast<uint2 *>(smem + C::SMEM_SB);
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + C::SMEM_MISC);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + C::SMEM_MISC + 4);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = CG == 2 ? cluster_ctarank() : 0;
    const int cid = (int)blockIdx.x / CG, ncl = (int)gridDim.x / CG;
    const int num_tiles = p.num_w_tiles * p.num_t_tiles;
    const int KT = X3 ? 3 * p.ktw : p.ktw + p.ktl;
    // shared::cluster addresses in the leader CTA (rank 0) / of the peer's abort flag
    auto leader = [&](const void *local) -> uint32_t {
        return CG == 2 ? mapa_shared(smem_u32(local), 0) : smem_u32(local);
    };
    const uint32_t peer_abort = CG == 2 ? mapa_shared(smem_u32((const void *)abort_flag), rank ^ 1) : 0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&xfull[s], 1);
            mbar_init(&wfull[s], 1);
            mbar_init(&empty[s], 4);  // 4 local dequant warps
        }
        for (int j = 0; j < AST; ++j) mbar_init(&afull[j], 4 * CG);
        for (int j = 0; j < KR; ++j) mbar_init(&kdone[j], 1);
        mbar_init(accfull, 1);
        mbar_init(accempty, 4 * CG);
        for (int j = 0; j < SBR; ++j) {
            mbar_init(&sbfull[j], 32);
            mbar_init(&sbempty[j], 4);
        }
        *abort_flag = 0;
        mbar_fence_init();
        prefetch_tmap(&tm_x);
        prefetch_tmap(&tm_w);
        if (SWIGLU) prefetch_tmap(&tm_w2);
        if (p.ktl) prefetch_tmap(&tm_t);
    }
    if (warp == 1) {
        if (CG == 2) tmem_alloc_pair(tmem_slot, TMEM_COLS);
        else tmem_alloc(tmem_slot, TMEM_COLS);
    }
    tc_fence_before();
    if (CG == 2) cluster_sync_all();  // peer barriers initialised before any remote arrive
    else __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ---------------------------------------------------------------- TMA producer
        // (a test can make it issue nothing, so that its consumers' bounded waits run out)
        if (lane == 0 && !(*reinterpret_cast<volatile unsigned *>(&g_debug_inject) & 1u)) {
            uint32_t it = 0;
            for (int tile = cid; tile < num_tiles && !*abort_flag; tile += ncl) {
                const int wt = tile % p.num_w_tiles, tt = tile / p.num_w_tiles;
                const int xrow = tt * BT + (int)rank * C::XROWS;
                for (int kk = 0; kk < KT; ++kk, ++it) {
                    // X3: segment seg of the three passes over K, k-step kt inside it
                    const int seg = X3 ? kk / p.ktw : 0, kt = X3 ? kk - seg * p.ktw : kk;
                    const int s = it % STAGES;
                    if (!mbar_wait<CG == 2>(&empty[s], ((it / STAGES) & 1) ^ 1, abort_flag, DEV_ERR_TIMEOUT_EMPTY,
                                   peer_abort))
                        break;
                    if (it >= (uint32_t)STAGES) {  // the MMAs that read this x stage are done
                        const uint32_t i = it - STAGES;
                        if (!mbar_wait<CG == 2>(&kdone[i % KR], (i / KR) & 1, abort_flag, DEV_ERR_TIMEOUT_EMPTY,
                                                           peer_abort))
                            break;
                    }
                    uint8_t *xs = smem + C::SMEM_X + s * C::X_STAGE_BYTES;
                    uint8_t *ws = smem + C::SMEM_W + s * C::W_STAGE_BYTES;
                    const bool wstep = X3 || kt < p.ktw;
                    // x half (or LoRA T half): counted on the leader's xfull[s]
                    if (rank == 0) mbar_arrive_expect_tx(&xfull[s], CG * C::X_STAGE_BYTES);
                    const CUtensorMap *xm = wstep ? &tm_x : &tm_t;
                    const int xk = X3 ? (seg == 1 ? p.ktw * BK : 0) + kt * BK : (wstep ? kt * BK : (kt - p.ktw) * BK);
                    if (CG == 2) tma_load_2d_pair(xs, xm, leader(&xfull[s]), xk, xrow);
                    else tma_load_2d(xs, xm, &xfull[s], xk, xrow);
                    // packed W rows of this CTA: counted on the local wfull[s]
                    if (wstep) {
                        mbar_arrive_expect_tx(&wfull[s], C::W_STAGE_BYTES + C::D_STAGE_BYTES);
                        if constexpr (LOKR)
                            tma_load_2d(smem + C::SMEM_D + s * C::D_STAGE_BYTES, tm_d, &wfull[s], kt * BK,
                                        (wt * CG + (int)rank) * BW);
                        if (SWIGLU) {
                            const int r0 = (wt * CG + (int)rank) * 64;
                            tma_load_2d(ws, &tm_w, &wfull[s], kt * C::W_BOX_WORDS, r0);
                            tma_load_2d(ws + 64 * C::W_ROW_BYTES, &tm_w2, &wfull[s], kt * C::W_BOX_WORDS, r0);
                        } else {
                            tma_load_2d(ws, &tm_w, &wfull[s], kt * C::W_BOX_WORDS, (wt * CG + (int)rank) * BW);
                        }
                    } else {
                        mbar_arrive(&wfull[s]);  // nothing to load; keep the phase moving
                    }
                }
            }
        }
    } else if (warp == 1) {
        // ---------------------------------------------------------------- MMA issuer (leader CTA)
        if (lane == 0 && rank == 0) {
            constexpr uint32_t idesc = umma_idesc_bf16(BW * CG, BT);
            uint32_t it = 0, tcount = 0;
            for (int tile = cid; tile < num_tiles && !*abort_flag; tile += ncl, ++tcount) {
                if (!mbar_wait<CG == 2>(accempty, (tcount & 1) ^ 1, abort_flag, DEV_ERR_TIMEOUT_ACC, peer_abort)) break;
                tc_fence_after();
                bool ok = true;
                for (int kt = 0; kt < KT; ++kt, ++it) {
                    const int s = it % STAGES, j = it % AST;
                    if (!mbar_wait<CG == 2>(&xfull[s], (it / STAGES) & 1, abort_flag, DEV_ERR_TIMEOUT_FULL, peer_abort) ||
                        !mbar_wait<CG == 2>(&afull[j], (it / AST) & 1, abort_flag, DEV_ERR_TIMEOUT_FULL, peer_abort)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint64_t bdesc = umma_desc_k_sw128(smem_u32(smem + C::SMEM_X + s * C::X_STAGE_BYTES));
#pragma unroll
                    for (int kk = 0; kk < BK / 16; ++kk) {
                        if (CG == 2)
                            tc_mma_ts_pair(tmem + ACC_COL, tmem + A_COL + j * 32 + kk * 8, bdesc + 2 * kk, idesc,
                                           (kt | kk) != 0);
                        else
                            tc_mma_ts(tmem + ACC_COL, tmem + A_COL + j * 32 + kk * 8, bdesc + 2 * kk, idesc,
                                      (kt | kk) != 0);
                    }
                    if (CG == 2) {  // signal both CTAs of the pair
                        tc_commit_pair(smem_u32(&kdone[it % KR]));
                        tc_commit_pair(mapa_shared(smem_u32(&kdone[it % KR]), 1));
                    } else {
                        tc_commit(&kdone[it % KR]);
                    }
                }
                if (!ok) break;
                if (CG == 2) {
                    tc_commit_pair(smem_u32(accfull));
                    tc_commit_pair(mapa_shared(smem_u32(accfull), 1));
                } else {
                    tc_commit(accfull);
                }
            }
        }
    } else if (warp >= 4 && warp < 8) {
        // ---------------------------------------------------------------- epilogue
        // Phase 1 drains the fp32 accumulator as fast as possible: each 32-column
        // chunk is rounded (+ bias, rounded again: the reference's two roundings) and
        // packed to bf16 pairs into the free TMEM columns [STG_COL, STG_COL + 128),
        // then the accumulator is released so the MMA can start the next tile.
        // Phase 2 reads the staged bf16 values back, applies the activation and
        // writes y with warp-coalesced stores (32 lanes = 32 consecutive columns).
        const int q = warp & 3;
        const int row = q * 32 + lane;  // TMEM lane == weight row within this CTA's half
        const uint32_t lane_base = tmem + ((uint32_t)(q * 32) << 16);
        const uint32_t accempty_leader = leader(accempty);
        float *xch = reinterpret_cast<float *>(smem + C::SMEM_XCH);
        uint32_t tcount = 0;
        for (int tile = cid; tile < num_tiles && !*abort_flag; tile += ncl, ++tcount) {
            const int wt = tile % p.num_w_tiles, tt = tile / p.num_w_tiles;
            int n;
            const __nv_bfloat16 *bp;
            if (SWIGLU) {
                n = (wt * CG + (int)rank) * 64 + (row & 63);
                bp = row < 64 ? p.bias : p.bias2;
            } else {
                n = (wt * CG + (int)rank) * BW + row;
                bp = p.bias;
            }
            const bool has_bias = bp != nullptr;
            const uint32_t bias2 = (has_bias && n < p.N) ? 0x10001u * reinterpret_cast<const uint16_t *>(bp)[n] : 0u;
            if (!mbar_wait<CG == 2>(accfull, tcount & 1, abort_flag, DEV_ERR_TIMEOUT_ACC, peer_abort)) break;
            tc_fence_after();
            if constexpr (X3) {
                // f32 / f16 output straight from the accumulator (long-K tiles: the drain is a
                // small part of the tile); the reference's rounding points in the output dtype
                const bool f32o = (p.act & QL_EPI_OUT_F32) != 0;
                const int act = p.act & 0xff;
                float bias_f = 0.f;
                if (has_bias && n < p.N)
                    bias_f = f32o ? reinterpret_cast<const float *>(bp)[n]
                                  : __half2float(reinterpret_cast<const __half *>(bp)[n]);
                const int m0 = tt * BT;
#pragma unroll 1
                for (int c = 0; c < BT / 32; ++c) {
                    uint32_t v[32];
                    tmem_ld32(lane_base + ACC_COL + c * 32, v);
                    tmem_ld_wait();
                    if (n < p.N) {
#pragma unroll
                        for (int i = 0; i < 32; ++i) {
                            const int m = m0 + c * 32 + i;
                            float a = __uint_as_float(v[i]);
                            if (!f32o) a = __half2float(__float2half_rn(a));
                            if (has_bias) a = f32o ? a + bias_f : __half2float(__float2half_rn(a + bias_f));
                            if (act == QL_ACT_GELU_TANH) a = 0.5f * a * (1.0f + tanhf(0.7978845608028654f * (a + 0.044715f * a * a * a)));
                            else if (act == QL_ACT_GELU_ERF) a = gelu_erf_f(a);
                            if (m < p.M) {
                                if (f32o) reinterpret_cast<float *>(p.y)[(int64_t)m * p.N + n] = a;
                                else reinterpret_cast<__half *>(p.y)[(int64_t)m * p.N + n] = __float2half_rn(a);
                            }
                        }
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(accempty);
                continue;
            }
#pragma unroll 1
            for (int c = 0; c < BT / 32; ++c) {
                uint32_t v[32], pk[16];
                tmem_ld32(lane_base + ACC_COL + c * 32, v);
                tmem_ld_wait();
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    pk[i] = pack_bf16x2(__uint_as_float(v[2 * i]), __uint_as_float(v[2 * i + 1]));
                    if (has_bias) pk[i] = hfma2_bf16(pk[i], 0x3f803f80u, bias2);
                }
                tmem_st16(lane_base + STG_COL + c * 16, pk);
            }
            tmem_st_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {  // accumulator free for the next tile
                if (CG == 2 && rank != 0) mbar_arrive_cluster(accempty_leader);
                else mbar_arrive(accempty);
            }

            const int m0 = tt * BT;
#pragma unroll 1
            for (int c = 0; c < BT / 32; ++c) {
                uint32_t pk[16];
                tmem_ld16(lane_base + STG_COL + c * 16, pk);
                tmem_ld_wait();
                if (SWIGLU) {
                    if (row >= 64) {
#pragma unroll
                        for (int i = 0; i < 16; ++i) {
                            xch[(row - 64) * 33 + 2 * i] = bf16lo(pk[i]);
                            xch[(row - 64) * 33 + 2 * i + 1] = bf16hi(pk[i]);
                        }
                    }
                    named_bar_sync(1, 128);
                    if (row < 64 && n < p.N) {
                        if constexpr (!GATED) {
#pragma unroll
                            for (int i = 0; i < 32; ++i) {
                                const int m = m0 + c * 32 + i;
                                const float g = (i & 1) ? bf16hi(pk[i >> 1]) : bf16lo(pk[i >> 1]);
                                const float u = xch[row * 33 + i];
                                if (m < p.M) p.y[(int64_t)m * p.N + n] = __float2bfloat16_rn(silu_f(g) * u);
                            }
                        } else {
#pragma unroll
                            for (int i = 0; i < 32; ++i) {
                                const int m = m0 + c * 32 + i;
                                const float g = (i & 1) ? bf16hi(pk[i >> 1]) : bf16lo(pk[i >> 1]);
                                const float u = xch[row * 33 + i];
                                if (m < p.M)
                                    p.y[(int64_t)m * p.N + n] =
                                        __float2bfloat16_rn(apply_gated(silu_f(g) * u, gd, m, n, p.N));
                            }
                        }
                    }
                    named_bar_sync(1, 128);
                } else if (!GATED && n < p.N && p.act == QL_ACT_NONE && m0 + c * 32 + 32 <= p.M) {
                    // plain linear, 32 tokens in range: the staged halves are the output bits
                    // (short-K tiles are bound by this loop's instruction count)
                    uint16_t *yp = reinterpret_cast<uint16_t *>(p.y) + (int64_t)(m0 + c * 32) * p.N + n;
#pragma unroll
                    for (int i = 0; i < 32; ++i)
                        yp[(int64_t)i * p.N] = (uint16_t)((i & 1) ? (pk[i >> 1] >> 16) : pk[i >> 1]);
                } else if (!GATED && n < p.N && p.act == QL_ACT_GELU_TANH && m0 + c * 32 + 32 <= p.M) {
                    __nv_bfloat16 *yp = p.y + (int64_t)(m0 + c * 32) * p.N + n;
#pragma unroll
                    for (int i = 0; i < 32; ++i)
                        yp[(int64_t)i * p.N] =
                            __float2bfloat16_rn(gelu_tanh_f((i & 1) ? bf16hi(pk[i >> 1]) : bf16lo(pk[i >> 1])));
                } else if (!GATED && n < p.N) {
#pragma unroll
                    for (int i = 0; i < 32; ++i) {
                        const int m = m0 + c * 32 + i;
                        float v = (i & 1) ? bf16hi(pk[i >> 1]) : bf16lo(pk[i >> 1]);
                        if (p.act == QL_ACT_GELU_TANH) v = gelu_tanh_f(v);
                        else if (p.act == QL_ACT_GELU_ERF) v = gelu_erf_f(v);
                        if (m < p.M) p.y[(int64_t)m * p.N + n] = __float2bfloat16_rn(v);
                    }
                } else if (GATED && n < p.N) {  // gated residual
#pragma unroll
                    for (int i = 0; i < 32; ++i) {
                        const int m = m0 + c * 32 + i;
                        float v = (i & 1) ? bf16hi(pk[i >> 1]) : bf16lo(pk[i >> 1]);
                        if (p.act == QL_ACT_GELU_TANH) v = gelu_tanh_f(v);
                        else if (p.act == QL_ACT_GELU_ERF) v = gelu_erf_f(v);
                        if (m < p.M) p.y[(int64_t)m * p.N + n] = __float2bfloat16_rn(apply_gated(v, gd, m, n, p.N));
                    }
                }
            }
        }
    } else if (warp == 2) {
        // ---------------------------------------------------------------- scale/bias producer
        // For every k-step of this CTA (flattened over its tiles, in the dequant warps'
        // order) the warp writes a shared-memory ring slot holding, per weight row,
        // {s(group of k0) | b << 16, s(group of k0 + 32) | b << 16}.  Lane l serves rows l,
        // l + 32, l + 64, l + 96.  Scales and biases are read from global memory in chunks
        // of 8 groups per row (one 16-byte load each when the rows allow it), and the next
        // chunk's loads are in flight while the current chunk's slots are written, so
        // their latency stays in this warp.
        const int my_tiles = cid < num_tiles ? (num_tiles - 1 - cid) / ncl + 1 : 0;
        const bool vec = (p.G % 8) == 0 && ((reinterpret_cast<uintptr_t>(p.scales) | reinterpret_cast<uintptr_t>(p.biases)) & 15) == 0 &&
                         (!SWIGLU || ((reinterpret_cast<uintptr_t>(p.scales2) | reinterpret_cast<uintptr_t>(p.biases2)) & 15) == 0);
        const int nchunk = (p.G + 7) / 8;  // chunks of 8 groups per tile
        // chunk registers: per row r4, 8 scales (4 words) then 8 biases (4 words)
        auto load_chunk = [&](int lt, int c, uint32_t (&o)[4][8]) {
            const int wt = (cid + lt * ncl) % p.num_w_tiles;
#pragma unroll
            for (int r4 = 0; r4 < 4; ++r4) {
                const int row = r4 * 32 + lane;
                const uint16_t *sc, *bi;
                int n;
                if (SWIGLU) {
                    sc = reinterpret_cast<const uint16_t *>(row < 64 ? p.scales : p.scales2);
                    bi = reinterpret_cast<const uint16_t *>(row < 64 ? p.biases : p.biases2);
                    n = (wt * CG + (int)rank) * 64 + (row & 63);
                } else {
                    sc = reinterpret_cast<const uint16_t *>(p.scales);
                    bi = reinterpret_cast<const uint16_t *>(p.biases);
                    n = (wt * CG + (int)rank) * BW + row;
                }
#pragma unroll
                for (int i = 0; i < 8; ++i) o[r4][i] = 0;
                if (n >= p.N || lt >= my_tiles) continue;
                const int64_t base = (int64_t)n * p.G + c * 8;
                if (vec) {
                    const uint4 sv = __ldg(reinterpret_cast<const uint4 *>(sc + base));
                    const uint4 bv = __ldg(reinterpret_cast<const uint4 *>(bi + base));
                    o[r4][0] = sv.x, o[r4][1] = sv.y, o[r4][2] = sv.z, o[r4][3] = sv.w;
                    o[r4][4] = bv.x, o[r4][5] = bv.y, o[r4][6] = bv.z, o[r4][7] = bv.w;
                } else {
#pragma unroll
                    for (int g = 0; g < 8; ++g) {
                        if (c * 8 + g < p.G) {
                            o[r4][g >> 1] |= (uint32_t)__ldg(sc + base + g) << (16 * (g & 1));
                            o[r4][4 + (g >> 1)] |= (uint32_t)__ldg(bi + base + g) << (16 * (g & 1));
                        }
                    }
                }
            }
        };
        // 16-bit entry g (0..7) of a 4-word register group
        auto pick = [](const uint32_t *w4, int g) -> uint32_t {
            const uint32_t lo = (g & 2) ? w4[1] : w4[0], hi = (g & 2) ? w4[3] : w4[2];
            const uint32_t wsel = (g & 4) ? hi : lo;
            return (g & 1) ? (wsel >> 16) : (wsel & 0xffffu);
        };
        uint32_t cur[4][8], nxt[4][8];
        uint32_t it = 0;
        bool ok = true;
        if (nchunk > 0) load_chunk(0, 0, nxt);
        constexpr int NSEG = X3 ? 3 : 1;  // X3: the scales of every pass over K
        for (int lt = 0; lt < my_tiles && ok; ++lt) {
            for (int cs = 0; cs < NSEG * nchunk && ok; ++cs) {
                const int c = cs % nchunk;
#pragma unroll
                for (int r4 = 0; r4 < 4; ++r4)
#pragma unroll
                    for (int i = 0; i < 8; ++i) cur[r4][i] = nxt[r4][i];
                // prefetch the next chunk (of this tile and pass, the next pass, or the next tile)
                if (c + 1 < nchunk) load_chunk(lt, c + 1, nxt);
                else if (cs + 1 < NSEG * nchunk) load_chunk(lt, 0, nxt);
                else load_chunk(lt + 1, 0, nxt);
                // k-steps whose first group lies in chunk c
                const int kt0 = (c * 8 * p.gs + BK - 1) / BK;
                const int kt1 = min(p.ktw, ((c + 1) * 8 * p.gs + BK - 1) / BK);
                for (int kt = kt0; kt < kt1; ++kt, ++it) {
                    const int slot = it % SBR;
                    if (!mbar_wait<false>(&sbempty[slot], ((it / SBR) & 1) ^ 1, abort_flag, DEV_ERR_TIMEOUT_EMPTY)) {
                        ok = false;
                        break;
                    }
                    const int g0 = kt * BK / p.gs - c * 8, g1 = (kt * BK + 32) / p.gs - c * 8;
#pragma unroll
                    for (int r4 = 0; r4 < 4; ++r4) {
                        // g1 may fall in the next chunk only when gs = 32 and the step straddles
                        // chunks, which cannot happen (8 groups of 32 = 4 whole k-steps)
                        const uint32_t s0 = pick(cur[r4], g0), b0 = pick(cur[r4] + 4, g0);
                        const uint32_t s1 = pick(cur[r4], g1 & 7), b1 = pick(cur[r4] + 4, g1 & 7);
                        sb_ring[slot * BW + r4 * 32 + lane] = make_uint2(s0 | (b0 << 16), s1 | (b1 << 16));
                    }
                    mbar_arrive(&sbfull[slot]);  // each lane after its own stores (count 32)
                }
            }
            // LoRA k-steps of this tile: no scales (the dequant warps do not read the slot)
            for (int kt = p.ktw; kt < (X3 ? p.ktw : KT) && ok; ++kt, ++it) {
                const int slot = it % SBR;
                if (!mbar_wait<false>(&sbempty[slot], ((it / SBR) & 1) ^ 1, abort_flag, DEV_ERR_TIMEOUT_EMPTY)) {
                    ok = false;
                    break;
                }
                mbar_arrive(&sbfull[slot]);
            }
        }
    } else if (warp >= 8) {
        // ---------------------------------------------------------------- dequant warpgroups
        // Warpgroup wg handles this CTA's k-steps it = wg, wg + 2, ... (flattened over
        // tiles); the scales / biases of each step come from warp 2's ring.
        const int wg = (warp - 8) >> 2, q = warp & 3;
        const int row = q * 32 + lane;
        const uint32_t taddr_lane = tmem + ((uint32_t)(q * 32) << 16) + A_COL;
        const int my_tiles = cid < num_tiles ? (num_tiles - 1 - cid) / ncl + 1 : 0;
        const uint32_t total = (uint32_t)my_tiles * (uint32_t)KT;

        // weight row (global) of this thread for tile `tile` (LoRA steps)
        auto row_n = [&](int tile) -> int {
            const int wt = tile % p.num_w_tiles;
            return SWIGLU ? (wt * CG + (int)rank) * 64 + (row & 63) : (wt * CG + (int)rank) * BW + row;
        };
        for (uint32_t it = (uint32_t)wg; it < total; it += 2) {
            const int slot = it % SBR;
            if (!mbar_wait<false>(&sbfull[slot], (it / SBR) & 1, abort_flag, DEV_ERR_TIMEOUT_FULL)) break;
            const uint2 sbv = sb_ring[slot * BW + row];
            __syncwarp();
            if (lane == 0) mbar_arrive(&sbempty[slot]);
            const uint32_t sb[4] = {sbv.x & 0xffffu, sbv.x >> 16, sbv.y & 0xffffu, sbv.y >> 16};
            const int lt = (int)(it / (uint32_t)KT), kt = (int)(it - (uint32_t)lt * KT);
            const int s = it % STAGES, j = it % AST;
            if (!mbar_wait<CG == 2>(&wfull[s], (it / STAGES) & 1, abort_flag, DEV_ERR_TIMEOUT_FULL, peer_abort) ||
                (it >= (uint32_t)AST &&  // the MMAs of step it - AST released this A slot
                 !mbar_wait<CG == 2>(&kdone[(it - AST) % KR], ((it - AST) / KR) & 1, abort_flag,
                                                                 DEV_ERR_TIMEOUT_EMPTY, peer_abort)))
                break;
            uint32_t r[32];
            if constexpr (X3) {
                // w = fma(code, s, b) in fp32 (the reference's dequantize), then the bf16 piece
                // of this pass: whi = bf16(w) for passes 0 and 1, wlo = bf16(w - whi) for pass 2
                const bool lo_pass = kt >= 2 * p.ktw;
                const bool sb16 = (p.act & QL_EPI_SB_F16) != 0;
                auto sbf = [&](uint32_t v) { return sb16 ? __half2float(__ushort_as_half((unsigned short)v)) : bf16lo(v); };
                const float fs0 = sbf(sb[0]), fb0 = sbf(sb[1]), fs1 = sbf(sb[2]), fb1 = sbf(sb[3]);
                const uint4 *wrow = reinterpret_cast<const uint4 *>(smem + C::SMEM_W + s * C::W_STAGE_BYTES +
                                                                    row * C::W_ROW_BYTES);
                uint32_t wv[BITS * 2];  // the step's 64 codes: 8 (Q4) / 16 (Q8) words
                if constexpr (BITS == 4) {
                    const int sw = (row >> 2) & 1;
                    const uint4 a = wrow[sw], b = wrow[sw ^ 1];
                    wv[0] = a.x, wv[1] = a.y, wv[2] = a.z, wv[3] = a.w, wv[4] = b.x, wv[5] = b.y, wv[6] = b.z, wv[7] = b.w;
                } else {
#pragma unroll
                    for (int h = 0; h < 4; ++h) {
                        const uint4 a = wrow[h ^ ((row >> 1) & 3)];
                        wv[4 * h] = a.x, wv[4 * h + 1] = a.y, wv[4 * h + 2] = a.z, wv[4 * h + 3] = a.w;
                    }
                }
                // an f16 computation dtype (f16 x and scales) rounds w to f16 first, as the
                // reference's f16 quantized_matmul does; f16 has 11 bits, so whi + wlo hold it exactly
                const bool w16 = (p.act & QL_EPI_OUT_F16) != 0;
                auto piece = [&](int k) -> float {
                    constexpr int EPW = 32 / BITS;
                    const uint32_t code = (wv[k / EPW] >> (BITS * (k % EPW))) & ((1u << BITS) - 1u);
                    float w = fmaf(__uint_as_float(0x4B000000u | code) - 8388608.0f, k < 32 ? fs0 : fs1,
                                   k < 32 ? fb0 : fb1);
                    if (w16) w = __half2float(__float2half_rn(w));
                    const float hi = round_bf16(w);
                    return lo_pass ? w - hi : hi;
                };
#pragma unroll
                for (int m = 0; m < 32; ++m) r[m] = pack_bf16x2(piece(2 * m), piece(2 * m + 1));
            } else if (kt < p.ktw) {
                const uint32_t s0 = sb[0] * 0x10001u, b0 = sb[1] * 0x10001u;  // bf16x2 broadcast
                const uint32_t s1 = sb[2] * 0x10001u, b1 = sb[3] * 0x10001u;
                // The packed rows arrive 32-byte (Q4) / 64-byte (Q8) swizzled: 16-byte chunk h of
                // row r sits at chunk h ^ ((r >> 2) & 1) (Q4) / h ^ ((r >> 1) & 3) (Q8), so the
                // eight rows a quarter-warp reads hit eight different bank groups.
                const uint4 *wrow = reinterpret_cast<const uint4 *>(smem + C::SMEM_W + s * C::W_STAGE_BYTES +
                                                                    row * C::W_ROW_BYTES);
                if constexpr (BITS == 4) {
                    const int sw = (row >> 2) & 1;
                    uint4 a = wrow[sw];
                    uint4 b = wrow[sw ^ 1];
                    const uint32_t wv[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        uint32_t qp[4];
                        q4_word_to_bf16_pairs(wv[i], qp);
                        const uint32_t ss = i < 4 ? s0 : s1, bb = i < 4 ? b0 : b1;
#pragma unroll
                        for (int t = 0; t < 4; ++t) r[4 * i + t] = hfma2_bf16(qp[t], ss, bb);
                    }
                } else {
                    // A code byte c placed in bits 8-15 of 0x47000000 reads as the float
                    // 32768 + c (one prmt).  s * (32768 + c) is exact in fp32 (8 x 16
                    // significant bits), so fma(s, 32768 + c, b - 32768 s) is the fp32
                    // rounding of s c + b whenever b - 32768 s is exact -- the same value
                    // as fma(c, s, b) -- and within an fp32 ulp of 32768 s otherwise.  Two codes
                    // per fma.rn.f32x2.
                    const float fs0 = bf16lo(s0), fs1 = bf16lo(s1);
                    const float fb0 = fmaf(-32768.f, fs0, bf16lo(b0)), fb1 = fmaf(-32768.f, fs1, bf16lo(b1));
#pragma unroll
                    for (int h = 0; h < 4; ++h) {
                        uint4 a = wrow[h ^ ((row >> 1) & 3)];
                        const uint32_t wv[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            const int wi = 4 * h + i;  // word index: codes 4wi..4wi+3
                            const float ss = wi < 8 ? fs0 : fs1, bb = wi < 8 ? fb0 : fb1;
                            uint32_t lo0, hi0, lo1, hi1;
                            asm("{\n\t.reg .b64 a, b, c, d;\n\t"
                                "mov.b64 a, {%4, %5};\n\tmov.b64 b, {%8, %8};\n\tmov.b64 c, {%9, %9};\n\t"
                                "fma.rn.f32x2 d, a, b, c;\n\tmov.b64 {%0, %1}, d;\n\t"
                                "mov.b64 a, {%6, %7};\n\tfma.rn.f32x2 d, a, b, c;\n\tmov.b64 {%2, %3}, d;\n\t}"
                                : "=r"(lo0), "=r"(hi0), "=r"(lo1), "=r"(hi1)
                                : "r"(prmt(wv[i], 0x47000000u, 0x7604u)), "r"(prmt(wv[i], 0x47000000u, 0x7614u)),
                                  "r"(prmt(wv[i], 0x47000000u, 0x7624u)), "r"(prmt(wv[i], 0x47000000u, 0x7634u)),
                                  "r"(__float_as_uint(ss)), "r"(__float_as_uint(bb)));
                            r[2 * wi] = pack_bf16x2(__uint_as_float(lo0), __uint_as_float(hi0));
                            r[2 * wi + 1] = pack_bf16x2(__uint_as_float(lo1), __uint_as_float(hi1));
                        }
                    }
                }
            } else {
                // LoRA step: A = B^T rows for this tile, columns [64l, 64l + 64) of rank.
                const int n = row_n(cid + lt * ncl);
                const bool row_ok = n < p.N;
                const int l0 = (kt - p.ktw) * BK;
#pragma unroll
                for (int c = 0; c < 32; ++c) {
                    const int j0 = l0 + 2 * c;
                    uint32_t lo = 0, hi = 0;
                    if (row_ok && j0 < p.lora_rank)
                        lo = reinterpret_cast<const uint16_t *>(p.lora_b)[(int64_t)j0 * p.N + n];
                    if (row_ok && j0 + 1 < p.lora_rank)
                        hi = reinterpret_cast<const uint16_t *>(p.lora_b)[(int64_t)(j0 + 1) * p.N + n];
                    r[c] = lo | (hi << 16);
                }
            }
            if constexpr (LOKR) {
                if (kt < p.ktw) {  // w += scale * dW, one bf16 fma per pair (row's 128 B, swizzled)
                    const uint8_t *drow = smem + C::SMEM_D + s * C::D_STAGE_BYTES + row * 128;
#pragma unroll
                    for (int c = 0; c < 8; ++c) {
                        const uint4 dv = *reinterpret_cast<const uint4 *>(drow + ((c ^ (row & 7)) << 4));
                        r[4 * c + 0] = hfma2_bf16(dv.x, lokr_scale2, r[4 * c + 0]);
                        r[4 * c + 1] = hfma2_bf16(dv.y, lokr_scale2, r[4 * c + 1]);
                        r[4 * c + 2] = hfma2_bf16(dv.z, lokr_scale2, r[4 * c + 2]);
                        r[4 * c + 3] = hfma2_bf16(dv.w, lokr_scale2, r[4 * c + 3]);
                    }
                }
            }
            tmem_st32(taddr_lane + j * 32, r);
            tmem_st_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                if (CG == 2 && rank != 0) mbar_arrive_cluster(leader(&afull[j]));
                else mbar_arrive(&afull[j]);
                mbar_arrive(&empty[s]);
            }
        }
    }

    tc_fence_before();
    // no CTA of a pair may exit while its peer can still signal its barriers
    if (CG == 2) cluster_sync_all();
    else __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        if (CG == 2) tmem_dealloc_pair(tmem, TMEM_COLS);
        else tmem_dealloc(tmem, TMEM_COLS);
    }
}

template <int BITS, bool SWIGLU, int CG>
__global__ void __launch_bounds__(NTHREADS, 1)
    qgemm_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w,
                 const __grid_constant__ CUtensorMap tm_w2, const __grid_constant__ CUtensorMap tm_t,
                 const Params p) {
    qgemm_body<BITS, SWIGLU, CG, false>(tm_x, tm_w, tm_w2, tm_t, p, Gated{});
}

// f32 / f16 activations through the three-pass bf16 split (1-CTA tiles, plain or GELU).
template <int BITS>
__global__ void __launch_bounds__(NTHREADS, 1)
    qgemm_x3_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w,
                    const Params p) {
    qgemm_body<BITS, false, 1, false, false, true>(tm_x, tm_w, tm_w, tm_x, p, Gated{});
}

// Plain or gated linear plus a LoKr delta (1-CTA tiles, no SwiGLU).
struct LokrArgs {
    uint32_t scale2;  // lokr_scale as a bf16 pair
    Gated gd;
};
template <int BITS, bool GATED>
__global__ void __launch_bounds__(NTHREADS, 1)
    qgemm_lokr_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w,
                      const __grid_constant__ CUtensorMap tm_w2, const __grid_constant__ CUtensorMap tm_t,
                      const Params p, const __grid_constant__ CUtensorMap tm_d, const LokrArgs la) {
    qgemm_body<BITS, false, 1, GATED, true>(tm_x, tm_w, tm_w2, tm_t, p, la.gd, &tm_d, la.scale2);
}

template <int BITS, bool SWIGLU, int CG>
__global__ void __launch_bounds__(NTHREADS, 1)
    qgemm_gated_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w,
                       const __grid_constant__ CUtensorMap tm_w2, const __grid_constant__ CUtensorMap tm_t,
                       const Params p, const Gated gd) {
    qgemm_body<BITS, SWIGLU, CG, true>(tm_x, tm_w, tm_w2, tm_t, p, gd);
}

// ------------------------------------------------------------------ host side

typedef CUresult (*PFN_encodeTiled)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                    const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                    const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                    CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// The driver entry point, resolved once (a function-local static: thread-safe
// initialisation; a failed lookup is retried on the next call).
static PFN_encodeTiled get_encode() {
    static std::atomic<PFN_encodeTiled> fn{nullptr};
    PFN_encodeTiled f = fn.load(std::memory_order_acquire);
    if (!f) {
        void *ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess) {
            f = reinterpret_cast<PFN_encodeTiled>(ptr);
            fn.store(f, std::memory_order_release);
        }
    }
    return f;
}

static int make_map_2d(CUtensorMap *map, CUtensorMapDataType dt, int elem_bytes, const void *base,
                       uint64_t inner, uint64_t outer, uint64_t row_stride_bytes, uint32_t box_inner,
                       uint32_t box_outer, CUtensorMapSwizzle sw) {
    PFN_encodeTiled enc = get_encode();
    if (!enc) return fail(QL_ECUDA, "cuTensorMapEncodeTiled unavailable");
    cuuint64_t dims[2] = {inner, outer};
    cuuint64_t strides[1] = {row_stride_bytes};
    cuuint32_t box[2] = {box_inner, box_outer};
    cuuint32_t estr[2] = {1, 1};
    (void)elem_bytes;
    CUresult r = enc(map, dt, 2, const_cast<void *>(base), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(QL_ECUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return QL_OK;
}

template <int BITS, bool SWIGLU, int CG, bool GATED>
static int launch_t(const CUtensorMap &mx, const CUtensorMap &mw, const CUtensorMap &mw2,
                    const CUtensorMap &mt, const Params &p, const Gated &gd, int max_ctas, cudaStream_t st) {
    using C = Cfg<BITS, CG>;
    auto kfn = GATED ? (const void *)qgemm_gated_kernel<BITS, SWIGLU, CG> : (const void *)qgemm_kernel<BITS, SWIGLU, CG>;
    static PerDeviceFlag configured;  // per template instance and device
    int dev = 0, sms = 148;
    QL_CUDA_TRY(cudaGetDevice(&dev));
    if (!configured.test(dev)) {
        QL_CUDA_TRY(cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_TOTAL));
        if (CG == 2) QL_CUDA_TRY(cudaFuncSetAttribute(kfn, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
        configured.set(dev);
    }
    QL_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    const int tiles = p.num_w_tiles * p.num_t_tiles;
    cudaLaunchConfig_t cfg = {};
    cfg.blockDim = dim3(NTHREADS);
    cfg.dynamicSmemBytes = C::SMEM_TOTAL;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = CG;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = CG == 2 ? 1 : 0;  // a plain launch for the 1-CTA kernel
    // persistent grid: as many clusters as can be resident at once (pairs need two free
    // SMs of one GPC), never more than there are tiles
    static PerDeviceInt resident;
    int max_clusters = resident.get(dev);
    if (!max_clusters) {
        cfg.gridDim = dim3((unsigned)((sms / CG) * CG));
        int mc = 0;
        if (CG == 1 || cudaOccupancyMaxActiveClusters(&mc, kfn, &cfg) != cudaSuccess || mc <= 0) mc = sms / CG;
        max_clusters = mc;
        resident.put(dev, mc);
        if (getenv("QL_DEBUG")) fprintf(stderr, "qgemm CG=%d: %d resident clusters, smem %d\n", CG, mc, C::SMEM_TOTAL);
    }
    int clusters = tiles < max_clusters ? tiles : max_clusters;
    if (max_ctas > 0 && clusters > max_ctas / CG) clusters = max_ctas / CG > 0 ? max_ctas / CG : 1;
    cfg.gridDim = dim3((unsigned)(clusters * CG));
    if constexpr (GATED)
        QL_CUDA_TRY(cudaLaunchKernelEx(&cfg, qgemm_gated_kernel<BITS, SWIGLU, CG>, mx, mw, mw2, mt, p, gd));
    else
        QL_CUDA_TRY(cudaLaunchKernelEx(&cfg, qgemm_kernel<BITS, SWIGLU, CG>, mx, mw, mw2, mt, p));
    return QL_OK;
}

template <int BITS, bool GATED>
static int launch_lokr(const CUtensorMap &mx, const CUtensorMap &mw, const CUtensorMap &mt, const Params &p,
                       const CUtensorMap &md, const LokrArgs &la, int max_ctas, cudaStream_t st) {
    using C = Cfg<BITS, 1, true>;
    auto kfn = qgemm_lokr_kernel<BITS, GATED>;
    static PerDeviceFlag configured;
    int dev = 0, sms = 148;
    QL_CUDA_TRY(cudaGetDevice(&dev));
    if (!configured.test(dev)) {
        QL_CUDA_TRY(cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_TOTAL));
        configured.set(dev);
    }
    QL_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    const int tiles = p.num_w_tiles * p.num_t_tiles;
    int ctas = tiles < sms ? tiles : sms;
    if (max_ctas > 0 && ctas > max_ctas) ctas = max_ctas;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)ctas);
    cfg.blockDim = dim3(NTHREADS);
    cfg.dynamicSmemBytes = C::SMEM_TOTAL;
    cfg.stream = st;
    QL_CUDA_TRY(cudaLaunchKernelEx(&cfg, kfn, mx, mw, mw, mt, p, md, la));
    return QL_OK;
}

}  // namespace gemm


// x [M,K] bf16, W packed [N,K] (+ W3 for SwiGLU), scales/biases bf16.
// lora_t: [M, r_pad] bf16 (r_pad = round_up(rank, 64)) already holding s.(x.A), or null.
// a float as a pair of bf16 (round to nearest even), host side
static uint32_t pack_scale_bf16x2(float v) {
    uint32_t u;
    memcpy(&u, &v, 4);
    const uint32_t r = (u + 0x7fffu + ((u >> 16) & 1u)) >> 16;
    return r | (r << 16);
}

template <int BITS, bool SWIGLU, int CG>
static int launch_g(const CUtensorMap &mx, const CUtensorMap &mw, const CUtensorMap &mw2, const CUtensorMap &mt,
                    const gemm::Params &p, const Gated &gd, int max_ctas, cudaStream_t st) {
    return gd.res ? gemm::launch_t<BITS, SWIGLU, CG, true>(mx, mw, mw2, mt, p, gd, max_ctas, st)
                  : gemm::launch_t<BITS, SWIGLU, CG, false>(mx, mw, mw2, mt, p, gd, max_ctas, st);
}

int launch_qgemm_sm100(const void *x, int64_t M, int64_t K, const uint32_t *wq, const void *scales,
                       const void *biases, const uint32_t *wq2, const void *scales2,
                       const void *biases2, int64_t N, int gs, int bits, const void *bias,
                       const void *bias2, int act, const void *lora_t, const void *lora_b,
                       int64_t rank, void *y, int cg, int max_ctas, const Gated &gd, const void *lokr_delta,
                       float lokr_scale, cudaStream_t st) {
    using namespace gemm;
    const bool swiglu = act == QL_ACT_SWIGLU;
    const int wrows = (swiglu ? 64 : BW) * cg;  // output columns per tile
    Params p{};
    p.M = (int)M;
    p.N = (int)N;
    p.K = (int)K;
    p.gs = gs;
    p.G = (int)(K / gs);
    p.ktw = (int)((K + BK - 1) / BK);
    const int64_t rpad = rank > 0 ? (rank + BK - 1) / BK * BK : 0;
    p.ktl = (int)(rpad / BK);
    p.act = act;
    p.num_w_tiles = (int)((N + wrows - 1) / wrows);
    p.num_t_tiles = (int)((M + BT - 1) / BT);
    p.scales = (const __nv_bfloat16 *)scales;
    p.biases = (const __nv_bfloat16 *)biases;
    p.scales2 = (const __nv_bfloat16 *)scales2;
    p.biases2 = (const __nv_bfloat16 *)biases2;
    p.bias = (const __nv_bfloat16 *)bias;
    p.bias2 = (const __nv_bfloat16 *)bias2;
    p.lora_b = (const __nv_bfloat16 *)lora_b;
    p.lora_rank = (int)rank;
    p.y = (__nv_bfloat16 *)y;

    CUtensorMap mx, mw, mw2, mt;
    const uint32_t xbox = (uint32_t)(BT / cg);
    int rc = make_map_2d(&mx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, x, (uint64_t)K, (uint64_t)M,
                         (uint64_t)K * 2, BK, xbox, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    const uint64_t words = (uint64_t)K * bits / 32;
    const uint32_t box_words = (uint32_t)(BK * bits / 32);
    const uint32_t box_rows = swiglu ? 64 : BW;
    // rows of 32 B (Q4) / 64 B (Q8) per k-step, swizzled so that the dequant warps' reads
    // are free of bank conflicts
    const CUtensorMapSwizzle wsw = bits == 4 ? CU_TENSOR_MAP_SWIZZLE_32B : CU_TENSOR_MAP_SWIZZLE_64B;
    rc = make_map_2d(&mw, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, wq, words, (uint64_t)N, words * 4, box_words,
                     box_rows, wsw);
    if (rc) return rc;
    mw2 = mw;
    if (swiglu) {
        rc = make_map_2d(&mw2, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, wq2, words, (uint64_t)N, words * 4,
                         box_words, box_rows, wsw);
        if (rc) return rc;
    }
    mt = mx;
    if (rpad) {
        rc = make_map_2d(&mt, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, lora_t, (uint64_t)rpad, (uint64_t)M,
                         (uint64_t)rpad * 2, BK, xbox, CU_TENSOR_MAP_SWIZZLE_128B);
        if (rc) return rc;
    }
    if (lokr_delta) {  // LoKr delta fused into the dequant (1-CTA tiles, no SwiGLU)
        if (swiglu || cg != 1) return fail(QL_EUNSUPPORTED, "a fused LoKr delta needs the 1-CTA GEMM without SwiGLU");
        CUtensorMap md;
        rc = make_map_2d(&md, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, lokr_delta, (uint64_t)K, (uint64_t)N,
                         (uint64_t)K * 2, BK, BW, CU_TENSOR_MAP_SWIZZLE_128B);
        if (rc) return rc;
        LokrArgs la{pack_scale_bf16x2(lokr_scale), gd};
        if (bits == 4)
            return gd.res ? launch_lokr<4, true>(mx, mw, mt, p, md, la, max_ctas, st)
                          : launch_lokr<4, false>(mx, mw, mt, p, md, la, max_ctas, st);
        return gd.res ? launch_lokr<8, true>(mx, mw, mt, p, md, la, max_ctas, st)
                      : launch_lokr<8, false>(mx, mw, mt, p, md, la, max_ctas, st);
    }
    if (cg == 2) {
        if (bits == 4)
            return swiglu ? launch_g<4, true, 2>(mx, mw, mw2, mt, p, gd, max_ctas, st) : launch_g<4, false, 2>(mx, mw, mw2, mt, p, gd, max_ctas, st);
        return swiglu ? launch_g<8, true, 2>(mx, mw, mw2, mt, p, gd, max_ctas, st) : launch_g<8, false, 2>(mx, mw, mw2, mt, p, gd, max_ctas, st);
    }
    if (bits == 4)
        return swiglu ? launch_g<4, true, 1>(mx, mw, mw2, mt, p, gd, max_ctas, st) : launch_g<4, false, 1>(mx, mw, mw2, mt, p, gd, max_ctas, st);
    return swiglu ? launch_g<8, true, 1>(mx, mw, mw2, mt, p, gd, max_ctas, st) : launch_g<8, false, 1>(mx, mw, mw2, mt, p, gd, max_ctas, st);
}

}  // namespace ql

namespace ql {
namespace gemm {

// x (f32 or f16) [M, K] -> the two bf16 pieces [M, 2 * Kp]: hi = bf16(x) at column k, lo =
// bf16(x - hi) at column Kp + k; columns K..Kp-1 of both halves are zero.
__global__ void split_x_kernel(const void *__restrict__ x, int x_dtype, int64_t M, int64_t K, int64_t Kp,
                               __nv_bfloat16 *__restrict__ xs) {
    const int64_t total = M * Kp;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t m = i / Kp, k = i - m * Kp;
        const float v = k < K ? load_as_f32(x, x_dtype, m * K + k) : 0.f;
        const __nv_bfloat16 hi = __float2bfloat16_rn(v);
        xs[m * 2 * Kp + k] = hi;
        xs[m * 2 * Kp + Kp + k] = __float2bfloat16_rn(v - __bfloat162float(hi));
    }
}

}  // namespace gemm

size_t qgemm_x3_workspace(int64_t M, int64_t K) {
    const int64_t Kp = (K + gemm::BK - 1) / gemm::BK * gemm::BK;
    return (size_t)M * (size_t)Kp * 2 * 2;
}

// y [M, N] (f32 or f16) = x [M, K] (f32 or f16) . dequant(W)^T (+ bias, GELU) on tcgen05
// tensor cores: x and each dequantized weight are split into two bf16 pieces and three
// bf16 passes (whi.xhi + whi.xlo + wlo.xhi) accumulate in fp32.  Each piece pair keeps 16
// significant bits, so a product is exact to about 2^-16 of |w x| (the dropped wlo.xlo term
// and the pieces' roundings) and the sum carries the fp32 accumulation error on top.
int launch_qgemm_x3(const void *x, int x_dtype, int64_t M, int64_t K, const uint32_t *wq, const void *scales,
                    const void *biases, int sb_dtype, int64_t N, int gs, int bits, const void *bias, int act,
                    void *y, int y_dtype, void *workspace, int max_ctas, cudaStream_t st) {
    using namespace gemm;
    const int64_t Kp = (K + BK - 1) / BK * BK;
    __nv_bfloat16 *xs = static_cast<__nv_bfloat16 *>(workspace);
    {
        int dev = 0, sms = 148;
        QL_CUDA_TRY(cudaGetDevice(&dev));
        QL_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
        const int64_t total = M * Kp;
        int64_t blocks = (total + 255) / 256;
        if (blocks > (int64_t)sms * 8) blocks = (int64_t)sms * 8;
        split_x_kernel<<<(unsigned)blocks, 256, 0, st>>>(x, x_dtype, M, K, Kp, xs);
        QL_CUDA_TRY(cudaGetLastError());
    }
    Params p{};
    p.M = (int)M;
    p.N = (int)N;
    p.K = (int)K;
    p.gs = gs;
    p.G = (int)(K / gs);
    p.ktw = (int)(Kp / BK);
    p.ktl = 0;
    p.act = act | (y_dtype == QL_F32 ? QL_EPI_OUT_F32 : QL_EPI_OUT_F16) | (sb_dtype == QL_F16 ? QL_EPI_SB_F16 : 0);
    p.num_w_tiles = (int)((N + BW - 1) / BW);
    p.num_t_tiles = (int)((M + BT - 1) / BT);
    p.scales = (const __nv_bfloat16 *)scales;
    p.biases = (const __nv_bfloat16 *)biases;
    p.bias = (const __nv_bfloat16 *)bias;
    p.y = (__nv_bfloat16 *)y;
    CUtensorMap mx, mw;
    int rc = make_map_2d(&mx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, xs, (uint64_t)(2 * Kp), (uint64_t)M,
                         (uint64_t)(2 * Kp) * 2, BK, BT, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    const uint64_t words = (uint64_t)K * bits / 32;
    rc = make_map_2d(&mw, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, wq, words, (uint64_t)N, words * 4,
                     (uint32_t)(BK * bits / 32), BW, bits == 4 ? CU_TENSOR_MAP_SWIZZLE_32B : CU_TENSOR_MAP_SWIZZLE_64B);
    if (rc) return rc;
    auto kfn = bits == 4 ? qgemm_x3_kernel<4> : qgemm_x3_kernel<8>;
    const int smem_bytes = bits == 4 ? Cfg<4, 1>::SMEM_TOTAL : Cfg<8, 1>::SMEM_TOTAL;
    static PerDeviceFlag configured4, configured8;
    PerDeviceFlag &configured = bits == 4 ? configured4 : configured8;
    int dev = 0, sms = 148;
    QL_CUDA_TRY(cudaGetDevice(&dev));
    if (!configured.test(dev)) {
        QL_CUDA_TRY(cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes));
        configured.set(dev);
    }
    QL_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    const int tiles = p.num_w_tiles * p.num_t_tiles;
    int ctas = tiles < sms ? tiles : sms;
    if (max_ctas > 0 && ctas > max_ctas) ctas = max_ctas;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)ctas);
    cfg.blockDim = dim3(NTHREADS);
    cfg.dynamicSmemBytes = smem_bytes;
    cfg.stream = st;
    QL_CUDA_TRY(cudaLaunchKernelEx(&cfg, kfn, mx, mw, p));
    return QL_OK;
}

}  // namespace ql
