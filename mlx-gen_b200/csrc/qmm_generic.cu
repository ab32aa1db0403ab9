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
    Gated gd;  // residual and gate in y's dtype
    const void *lokr_delta;  // [N, K] in x's dtype, or null
    float lokr_scale;
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
                    v = round_to(p.ydt, fmaf((float)code, load_as_f32(p.scales[ps], p.sdt, g),
                                             load_as_f32(p.biases[ps], p.sdt, g)));
                    if (p.lokr_delta && ps == 0)  // LoKr: w + scale * delta, in fp32
                        v = fmaf(p.lokr_scale, load_as_f32(p.lokr_delta, p.xdt, (int64_t)n * p.K + k), v);
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
            if (p.gd.res) {  // gated residual, each op rounded to y's dtype
                v = round_to(p.ydt, v);
                if (p.gd.gate) {
                    const int64_t gr = p.gd.period > 0 ? m / p.gd.period : 0;
                    v = round_to(p.ydt, load_as_f32(p.gd.gate, p.ydt, gr * p.N + n) * v);
                }
                v = load_as_f32(p.gd.res, p.ydt, (int64_t)m * p.N + n) + v;
            }
            store_from_f32(p.y, p.ydt, (int64_t)m * p.N + n, v);
        }
}

// LoRA pre-pass on tensor cores: T[M, rpad] = bf16(scale * (x . A)), columns >= rank zero.
// x [M, K] bf16 (read once, the cost of this pass), A [K, rank] bf16 (small, L2-resident).
// CTA tile 32 rows x 64 columns of T; K in chunks of 64 through an 8-deep ring of 128-byte
// rows with a 16-byte-unit XOR swizzle (conflict-free ldmatrix); mma.sync.m16n8k16 bf16
// with fp32 accumulation.  Eight warps: warps w and w + 4 own the same 16 x 32 piece of
// the tile and take the first / second half of each chunk's K, so that each warp's chain
// of dependent MMAs per chunk is half as long; their partials meet in shared memory at the
// end.  KS = 2: the CTAs of a 2-CTA cluster take the two halves of the chunk range and the
// second pushes its partial tile into the first's shared memory (distributed shared
// memory), which doubles the CTAs (and the warps per SM) when the row tiles alone do not
// fill the GPU.
namespace lt {
constexpr int BM = 32, BN = 64, BKC = 64, ST = 8, NT = 256;
constexpr int SMEM = ST * (BM + BKC) * 128 + 1024;

__device__ __forceinline__ void cp_async16(void *dst, const void *src, int src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(src_bytes)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t r[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t r[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}
__device__ __forceinline__ void mma_bf16(float c[4], const uint32_t a[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// byte offset of 16-byte unit c of 128-byte row r
__device__ __forceinline__ int swz(int r, int c) { return r * 128 + ((c ^ (r & 7)) << 4); }

// TMA: thread 0 loads each chunk with two tensor-map boxes (x: 64 K x 32 rows, A: 64
// columns x 64 K, both 128-byte swizzled, which is the layout swz() reads); otherwise
// every thread issues 16-byte cp.async copies (A's rank not a multiple of 8).
// NH = 16-column halves per warp: 2 computes all 64 columns of the tile, 1 only the first
// 32 (rank <= 32) and writes zeros to the rest.
template <bool TMA, int NH, int KS>
__global__ void __launch_bounds__(NT) lora_t_mma_kernel(const __grid_constant__ CUtensorMap tm_x,
                                                         const __grid_constant__ CUtensorMap tm_a,
                                                         const __nv_bfloat16 *__restrict__ x, int M, int K,
                                                         const __nv_bfloat16 *__restrict__ A, int rank, int rpad,
                                                         float scale, __nv_bfloat16 *__restrict__ T, int vec_a) {
    extern __shared__ uint8_t lt_smem_raw[];
    __shared__ uint64_t full[ST];
    __shared__ int abort_flag;
    uint8_t *base = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(lt_smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t(*sx)[BM * 128] = reinterpret_cast<uint8_t(*)[BM * 128]>(base);
    uint8_t(*sa)[BKC * 128] = reinterpret_cast<uint8_t(*)[BKC * 128]>(base + ST * BM * 128);
    const int kr = KS > 1 ? (int)cluster_ctarank() : 0;  // this CTA's part of K
    const int mt = blockIdx.x / KS;
    const int m0 = mt * BM, n0 = blockIdx.y * BN;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int tp = warp & 3, kh = warp >> 2;  // piece of the tile, half of each chunk's K
    const int wm = tp & 1, wn = tp >> 1;      // rows 16 wm .. +16, columns 16 NH wn .. + 16 NH
    const int nk_all = (K + BKC - 1) / BKC;
    const int c0 = kr * nk_all / KS, nk = (kr + 1) * nk_all / KS - c0;  // this CTA's chunks

    // CTAs start at different K chunks so that they do not all read the same lines of A
    // at once (144 CTAs on one L2 line serialise); each CTA still sums its chunks in order
    const int kstart = nk > 0 ? (int)((mt * 5u) % (unsigned)nk) : 0;
    if (TMA) {
        if (tid == 0) {
            for (int i = 0; i < ST; ++i) mbar_init(&full[i], 1);
            abort_flag = 0;
            mbar_fence_init();
        }
        __syncthreads();
    }
    auto load = [&](int kc, int s) {
        int kq = kc + kstart;
        if (kq >= nk) kq -= nk;
        const int k0 = (c0 + kq) * BKC;
        if constexpr (TMA) {
            if (tid == 0) {
                mbar_arrive_expect_tx(&full[s], (BM + BKC) * 128);
                tma_load_2d(sx[s], &tm_x, &full[s], k0, m0);
                tma_load_2d(sa[s], &tm_a, &full[s], n0, k0);
            }
        } else {
            for (int i = tid; i < BM * 8; i += NT) {
                const int r = i >> 3, c = i & 7, m = m0 + r, k = k0 + c * 8;
                const bool ok = m < M && k < K;  // K is a multiple of 8
                cp_async16(sx[s] + swz(r, c), ok ? (const void *)(x + (int64_t)m * K + k) : (const void *)x,
                           ok ? 16 : 0);
            }
            for (int i = tid; i < BKC * 8; i += NT) {
                const int r = i >> 3, c = i & 7, k = k0 + r, n = n0 + c * 8;
                if (vec_a) {
                    const bool ok = k < K && n < rank;  // rank is a multiple of 8 here
                    cp_async16(sa[s] + swz(r, c), ok ? (const void *)(A + (int64_t)k * rank + n) : (const void *)A,
                               ok ? 16 : 0);
                } else {
                    uint16_t v[8];
#pragma unroll
                    for (int e = 0; e < 8; ++e)
                        v[e] = (k < K && n + e < rank) ? reinterpret_cast<const uint16_t *>(A)[(int64_t)k * rank + n + e]
                                                       : 0;
                    *reinterpret_cast<uint4 *>(sa[s] + swz(r, c)) =
                        make_uint4(v[0] | (uint32_t)v[1] << 16, v[2] | (uint32_t)v[3] << 16,
                                   v[4] | (uint32_t)v[5] << 16, v[6] | (uint32_t)v[7] << 16);
                }
            }
        }
    };

    float acc[2 * NH][4] = {};
#pragma unroll
    for (int s = 0; s < ST - 1; ++s) {
        if (s < nk) load(s, s);
        cp_async_commit();
    }
    for (int kc = 0; kc < nk; ++kc) {
        if (TMA)  // a timed-out wait only records the error: every thread keeps to the same barriers
            mbar_wait(&full[kc % ST], (kc / ST) & 1, &abort_flag, DEV_ERR_TIMEOUT_FULL);
        else
            cp_async_wait<ST - 2>();
        __syncthreads();  // chunk kc landed for every thread; stage (kc - 1) % ST is free
        if (kc + ST - 1 < nk) load(kc + ST - 1, (kc + ST - 1) % ST);
        cp_async_commit();
        const int s = kc % ST;
        const uint32_t xb = smem_u32(sx[s]), ab = smem_u32(sa[s]);
#pragma unroll
        for (int k2 = 0; k2 < BKC / 32; ++k2) {
            const int kk = 2 * kh + k2;
            uint32_t af[4];
            ldsm_x4(xb + swz(16 * wm + (lane & 15), 2 * kk + (lane >> 4)), af);
#pragma unroll
            for (int h = 0; h < NH; ++h) {
                uint32_t bf[4];
                ldsm_x4_t(ab + swz(16 * kk + (lane & 15), 2 * NH * wn + 2 * h + (lane >> 4)), bf);
                mma_bf16(acc[2 * h], af, bf[0], bf[1]);
                mma_bf16(acc[2 * h + 1], af, bf[2], bf[3]);
            }
        }
    }
    cp_async_wait<0>();
    __syncthreads();  // every chunk consumed: the ring's memory is reused below

    // partials: [tp][lane][8 NH floats]; the upper half of the warps hands its K half to the
    // lower half, then (KS = 2) the second CTA of the cluster hands its tile to the first
    constexpr int RED = 4 * 32 * 8 * NH;  // floats
    float *red = reinterpret_cast<float *>(base);
    float *peer = red + RED;
    float *mine = red + (tp * 32 + lane) * 8 * NH;
    if (kh == 1) {
#pragma unroll
        for (int j = 0; j < 2 * NH; ++j)
            *reinterpret_cast<float4 *>(mine + 4 * j) = make_float4(acc[j][0], acc[j][1], acc[j][2], acc[j][3]);
    }
    __syncthreads();
    if (kh == 0) {
#pragma unroll
        for (int j = 0; j < 2 * NH; ++j) {
            const float4 v = *reinterpret_cast<const float4 *>(mine + 4 * j);
            acc[j][0] += v.x, acc[j][1] += v.y, acc[j][2] += v.z, acc[j][3] += v.w;
        }
    }
    if constexpr (KS > 1) {
        cluster_sync_all();  // both CTAs are past their ring and their first reduction
        if (kr == 1 && kh == 0) {
            const uint32_t dst = mapa_shared(smem_u32(peer + (tp * 32 + lane) * 8 * NH), 0);
#pragma unroll
            for (int j = 0; j < 2 * NH; ++j)
                asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(dst + 16 * j), "f"(acc[j][0]),
                             "f"(acc[j][1]), "f"(acc[j][2]), "f"(acc[j][3])
                             : "memory");
        }
        cluster_sync_all();  // the second CTA's partial is in the first's shared memory
        if (kr == 1) return;
        if (kh == 0) {
            const float *pp = peer + (tp * 32 + lane) * 8 * NH;
#pragma unroll
            for (int j = 0; j < 2 * NH; ++j) {
                const float4 v = *reinterpret_cast<const float4 *>(pp + 4 * j);
                acc[j][0] += v.x, acc[j][1] += v.y, acc[j][2] += v.z, acc[j][3] += v.w;
            }
        }
    }
    if (kh != 0) return;
    const int g = lane >> 2, t = lane & 3;
#pragma unroll
    for (int j = 0; j < 2 * NH; ++j) {
        const int n = n0 + 16 * NH * wn + 8 * j + 2 * t;
#pragma unroll
        for (int hr = 0; hr < 2; ++hr) {
            const int m = m0 + 16 * wm + g + 8 * hr;
            if (m < M) {
                const float v0 = n < rank ? scale * acc[j][2 * hr] : 0.f;
                const float v1 = n + 1 < rank ? scale * acc[j][2 * hr + 1] : 0.f;
                *reinterpret_cast<uint32_t *>(T + (int64_t)m * rpad + n) = pack_bf16x2(v0, v1);
                if (NH == 1) *reinterpret_cast<uint32_t *>(T + (int64_t)m * rpad + n + 32) = 0u;
            }
        }
    }
}
}  // namespace lt

}  // namespace generic

int launch_qmm_generic(const void *x, int xdt, int64_t M, int64_t K, const uint32_t *wq,
                       const void *scales, const void *biases, const uint32_t *wq2,
                       const void *scales2, const void *biases2, int sdt, int64_t N, int gs,
                       int bits, const void *bias, const void *bias2, int act, const void *lora_a,
                       const void *lora_b, int64_t rank, float lora_scale, void *y, int ydt,
                       const Gated &gd, const void *lokr_delta, float lokr_scale, cudaStream_t st) {
    generic::Params p{};
    p.gd = gd;
    p.lokr_delta = lokr_delta;
    p.lokr_scale = lokr_scale;
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
    using namespace generic::lt;
    const int vec_a = rank % 8 == 0 && reinterpret_cast<uintptr_t>(A) % 16 == 0;
    static PerDeviceInt sm_count;
    const int cur_dev = current_device();
    int sms = sm_count.get(cur_dev);
    if (!sms) {
        if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, cur_dev) != cudaSuccess || sms <= 0) sms = 148;
        QL_CUDA_TRY(cudaFuncSetAttribute(lora_t_mma_kernel<true, 1, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM));
        QL_CUDA_TRY(cudaFuncSetAttribute(lora_t_mma_kernel<true, 2, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM));
        QL_CUDA_TRY(cudaFuncSetAttribute(lora_t_mma_kernel<false, 1, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM));
        QL_CUDA_TRY(cudaFuncSetAttribute(lora_t_mma_kernel<false, 2, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM));
        QL_CUDA_TRY(cudaFuncSetAttribute(lora_t_mma_kernel<true, 1, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM));
        QL_CUDA_TRY(cudaFuncSetAttribute(lora_t_mma_kernel<true, 2, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM));
        QL_CUDA_TRY(cudaFuncSetAttribute(lora_t_mma_kernel<false, 1, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM));
        QL_CUDA_TRY(cudaFuncSetAttribute(lora_t_mma_kernel<false, 2, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM));
        sm_count.put(cur_dev, sms);
    }
    CUtensorMap mx{}, ma{};
    if (vec_a) {
        if (int rc = gemm::make_map_2d(&mx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, x, (uint64_t)K, (uint64_t)M,
                                       (uint64_t)K * 2, BKC, BM, CU_TENSOR_MAP_SWIZZLE_128B))
            return rc;
        if (int rc = gemm::make_map_2d(&ma, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, A, (uint64_t)rank, (uint64_t)K,
                                       (uint64_t)rank * 2, BN, BKC, CU_TENSOR_MAP_SWIZZLE_128B))
            return rc;
    }
    // two CTAs per row tile (K halves, cluster reduction) while the row tiles alone leave
    // SMs without a second CTA; each CTA keeps at least two chunks
    const int64_t tiles = ((M + BM - 1) / BM) * (rpad / BN);
    const int ks = (tiles < 2 * (int64_t)sms && (K + BKC - 1) / BKC >= 4) ? 2 : 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)((M + BM - 1) / BM * ks), (unsigned)(rpad / BN));
    cfg.blockDim = dim3(NT);
    cfg.dynamicSmemBytes = SMEM;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)ks;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const bool nh1 = rank <= 32;
    void (*kfn)(CUtensorMap, CUtensorMap, const __nv_bfloat16 *, int, int, const __nv_bfloat16 *, int, int, float,
                __nv_bfloat16 *, int);
    if (vec_a)
        kfn = ks == 2 ? (nh1 ? lora_t_mma_kernel<true, 1, 2> : lora_t_mma_kernel<true, 2, 2>)
                      : (nh1 ? lora_t_mma_kernel<true, 1, 1> : lora_t_mma_kernel<true, 2, 1>);
    else
        kfn = ks == 2 ? (nh1 ? lora_t_mma_kernel<false, 1, 2> : lora_t_mma_kernel<false, 2, 2>)
                      : (nh1 ? lora_t_mma_kernel<false, 1, 1> : lora_t_mma_kernel<false, 2, 1>);
    QL_CUDA_TRY(cudaLaunchKernelEx(&cfg, kfn, mx, ma, (const __nv_bfloat16 *)x, (int)M, (int)K,
                                   (const __nv_bfloat16 *)A, (int)rank, rpad, scale, (__nv_bfloat16 *)T, vec_a));
    QL_CUDA_TRY(cudaGetLastError());
    return QL_OK;
}

}  // namespace ql
