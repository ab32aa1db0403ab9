// ql_common.cuh -- shared helpers of libqlinear (sm_100a only).
//
// Error plumbing, dtype conversion, and thin inline-PTX wrappers for the
// Blackwell primitives the kernels use: mbarriers with bounded waits, TMA
// (cp.async.bulk.tensor), and the tcgen05 family (TMEM alloc, MMA, commit,
// ld/st).  Everything here is written from the PTX ISA; no library code.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>

#include "../../include/qlinear.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "libqlinear is built for sm_100a only"
#endif

namespace ql {

// Host-side set-up done once per device (kernel attributes belong to a device's context;
// calls may come from several threads and devices, and repeating the set-up is harmless).
constexpr int kMaxDevices = 64;
struct PerDeviceFlag {
    std::atomic<uint64_t> mask{0};
    bool test(int dev) const {  // devices past the mask are set up on every call
        return dev < kMaxDevices && ((mask.load(std::memory_order_acquire) >> dev) & 1u);
    }
    void set(int dev) {
        if (dev < kMaxDevices) mask.fetch_or(1ull << dev, std::memory_order_release);
    }
};
struct PerDeviceInt {  // 0 = not yet known
    std::atomic<int> v[kMaxDevices];
    int get(int dev) const { return dev < kMaxDevices ? v[dev].load(std::memory_order_relaxed) : 0; }
    void put(int dev, int x) {
        if (dev < kMaxDevices) v[dev].store(x, std::memory_order_relaxed);
    }
};
inline int current_device() {
    int d = 0;
    return cudaGetDevice(&d) == cudaSuccess ? d : 0;
}

// ------------------------------------------------------------------ host errors

void set_error(const char *fmt, ...);
int fail(int status, const char *fmt, ...);

#define QL_CUDA_TRY(expr)                                                                  \
    do {                                                                                   \
        cudaError_t _e = (expr);                                                           \
        if (_e != cudaSuccess)                                                             \
            return ::ql::fail(QL_ECUDA, "%s failed: %s (%s:%d)", #expr, cudaGetErrorString(_e), \
                              __FILE__, __LINE__);                                         \
    } while (0)

// ------------------------------------------------------------------ device error word

// Device-side error word.  Kernels OR a code in when a bounded wait runs out or
// an index is out of range; the host reads it with ql_device_error().
enum : unsigned {
    DEV_ERR_TIMEOUT_FULL = 1u << 0,
    DEV_ERR_TIMEOUT_EMPTY = 1u << 1,
    DEV_ERR_TIMEOUT_ACC = 1u << 2,
    DEV_ERR_BAD_INDEX = 1u << 3,
};
// Defined here: libqlinear is built as a single translation unit (libqlinear.cu).
__device__ unsigned g_dev_error = 0;

__device__ __forceinline__ void raise_dev_error(unsigned code) { atomicOr(&g_dev_error, code); }

// ------------------------------------------------------------------ dtypes

__device__ __forceinline__ float load_as_f32(const void *p, int dt, int64_t i) {
    if (dt == QL_F32) return __ldg(reinterpret_cast<const float *>(p) + i);
    if (dt == QL_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16 *>(p)[i]);
    return __half2float(reinterpret_cast<const __half *>(p)[i]);
}

__device__ __forceinline__ void store_from_f32(void *p, int dt, int64_t i, float v) {
    if (dt == QL_F32) reinterpret_cast<float *>(p)[i] = v;
    else if (dt == QL_BF16) reinterpret_cast<__nv_bfloat16 *>(p)[i] = __float2bfloat16_rn(v);
    else reinterpret_cast<__half *>(p)[i] = __float2half_rn(v);
}

__device__ __forceinline__ float round_bf16(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
    uint32_t r;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}

// v rounded to the precision of dtype dt (QL_F32 / QL_BF16 / QL_F16), returned as f32
__device__ __forceinline__ float round_to(int dt, float v) {
    if (dt == QL_F32) return v;
    if (dt == QL_BF16) return round_bf16(v);
    return __half2float(__float2half_rn(v));
}

__device__ __forceinline__ float bf16lo(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float bf16hi(uint32_t v) { return __uint_as_float(v & 0xffff0000u); }

// d = a * b + c on bf16x2, one rounding per lane (fma.rn.bf16x2).
__device__ __forceinline__ uint32_t hfma2_bf16(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// d = a - b on bf16x2 (exact for the small integers used below).
__device__ __forceinline__ uint32_t hsub2_bf16(uint32_t a, uint32_t b) {
    uint32_t d;
    // a - b = a * 1.0 + (-b)
    asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(0x3f803f80u), "r"(b ^ 0x80008000u));
    return d;
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}

// Q4 word (8 codes, code i in bits [4i, 4i+4)) -> four bf16x2 registers holding
// codes (0,1), (2,3), (4,5), (6,7) as exact bf16 integers (low half = even code).
__device__ __forceinline__ void q4_word_to_bf16_pairs(uint32_t w, uint32_t out[4]) {
    const uint32_t v = w & 0x0f0f0f0fu;          // bytes: c0 c2 c4 c6
    const uint32_t u = (w >> 4) & 0x0f0f0f0fu;   // bytes: c1 c3 c5 c7
    const uint32_t t0 = prmt(v, u, 0x5140u);     // bytes: c0 c1 c2 c3
    const uint32_t t1 = prmt(v, u, 0x7362u);     // bytes: c4 c5 c6 c7
    // 0x43 in the high byte of each half -> bf16 value 128 + code; subtract 128.
    const uint32_t k = 0x43434343u;
    out[0] = hsub2_bf16(prmt(t0, k, 0x4140u), 0x43004300u);  // c0 | 43 | c1 | 43
    out[1] = hsub2_bf16(prmt(t0, k, 0x4342u), 0x43004300u);
    out[2] = hsub2_bf16(prmt(t1, k, 0x4140u), 0x43004300u);
    out[3] = hsub2_bf16(prmt(t1, k, 0x4342u), 0x43004300u);
}

// Exact float value of byte `sel` of a Q8 word (0..255).
__device__ __forceinline__ float q8_code_f32(uint32_t w, int byte) {
    // bytes [code, 0, 0, 0x4B] -> float 2^23 + code, minus 2^23 exactly.
    const uint32_t f = prmt(w, 0x4b000000u, 0x7540u + (uint32_t)byte);
    return __uint_as_float(f) - 8388608.0f;
}

// Gated residual epilogue, y = residual + gate * f(x W^T + bias), each op rounded to bf16
// as the reference's eager `add(x, multiply(gate, y))` does (src/nn.rs:166-176).
// res: [M, N] (NULL: no residual), gate: [M / period, N] (NULL: no gate; period 0: one
// gate row for every token row), both bf16.
struct Gated {
    const void *res;
    const void *gate;
    int64_t period;
};

// v: the linear's final value (after bias and activation, not yet rounded); returns the
// value to round to bf16 and store.
__device__ __forceinline__ float apply_gated(float v, const Gated &g, int64_t m, int64_t n, int64_t N) {
    if (!g.res) return v;
    float y = round_bf16(v);
    if (g.gate) {
        const int64_t gr = g.period > 0 ? m / g.period : 0;
        y = round_bf16(__bfloat162float(reinterpret_cast<const __nv_bfloat16 *>(g.gate)[gr * N + n]) * y);
    }
    return __bfloat162float(reinterpret_cast<const __nv_bfloat16 *>(g.res)[m * N + n]) + y;
}

// ------------------------------------------------------------------ mbarrier

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_fence_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

template <bool CLUSTER = false>
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    if (CLUSTER)  // arrivals may come from the paired CTA: acquire at cluster scope
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(ok)
            : "r"(smem_u32(bar)), "r"(parity)
            : "memory");
    else
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(ok)
            : "r"(smem_u32(bar)), "r"(parity)
            : "memory");
    return ok != 0;
}

// Bounded wait.  Every wait in the pipelined kernels goes through here: once
// kWaitLimitNs of wall time (%globaltimer) has passed without the phase
// completing -- far beyond any legal wait -- the kernel records `code` in the
// device error word, sets *abort and returns false, so every role can drain and
// exit instead of hanging the GPU.  Waits also give up as soon as another role
// has aborted.
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s
// The limit in force (kWaitLimitNs unless a test shortened it through ql_debug_inject), and
// the test hook's injection flags (bit 0: the tcgen05 GEMM's TMA producer issues nothing).
__device__ unsigned long long g_wait_limit_ns = kWaitLimitNs;
__device__ unsigned g_debug_inject = 0;

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}


template <bool CLUSTER = false>
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, volatile int *abort,
                                          unsigned code, uint32_t peer_abort = 0) {
    if (mbar_try_wait<CLUSTER>(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t i = 1;; ++i) {
        if (mbar_try_wait<CLUSTER>(bar, parity)) return true;
        if ((i & 63u) == 0) {
            if (*abort) return false;
            if (globaltimer_ns() - t0 > *reinterpret_cast<volatile unsigned long long *>(&g_wait_limit_ns)) {
                raise_dev_error(code);
                *abort = 1;
                // peer_abort: shared::cluster address of the paired CTA's abort flag
                if (peer_abort) asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(peer_abort), "r"(1) : "memory");
                return false;
            }
        }
    }
}

// ------------------------------------------------------------------ TMA

__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, uint64_t *bar, int c0,
                                            int c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, "
        "%4}], [%2];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
        : "memory");
}

__device__ __forceinline__ void tma_load_3d(void *dst, const CUtensorMap *map, uint64_t *bar, int c0, int c1,
                                            int c2) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, "
        "%4, %5}], [%2];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
        : "memory");
}

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap *map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}


// ------------------------------------------------------------------ clusters (CTA pairs)

__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// shared::cluster address of the same variable in CTA `rank` of this cluster
__device__ __forceinline__ uint32_t mapa_shared(uint32_t smem_addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr), "r"(rank));
    return r;
}

// arrive on an mbarrier given by its shared::cluster address (local or in the peer CTA)
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

// TMA 2-D load into this CTA's smem whose completion is counted on an mbarrier that may
// live in the pair's leader CTA (cta_group::2 form; no multicast).
__device__ __forceinline__ void tma_load_2d_pair(void *dst, const CUtensorMap *map, uint32_t bar_cluster_addr,
                                                 int c0, int c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, "
        "%4}], [%2];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster_addr), "r"(c0), "r"(c1)
        : "memory");
}

__device__ __forceinline__ void tmem_alloc_pair(uint32_t *dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
                 "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// Pair MMA (issued by the leader CTA only): D[256 x N] (+)= A[256 x 16] . B[N x 16]^T with
// A rows split across the two CTAs' TMEM and B rows split across their smem.
__device__ __forceinline__ void tc_mma_ts_pair(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                               uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrive (once) on the mbarrier at a shared::cluster address when all prior pair MMAs
// issued by this thread complete.
__device__ __forceinline__ void tc_commit_pair(uint32_t bar_cluster_addr) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     bar_cluster_addr)
                 : "memory");
}

// ------------------------------------------------------------------ tcgen05

__device__ __forceinline__ void tmem_alloc(uint32_t *dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(dst_smem)),
                 "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[tmem] * B[smem desc]^T, kind::f16 (bf16 in, fp32 accumulate).
__device__ __forceinline__ void tc_mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                          uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrive on `bar` when every tcgen05.mma issued so far by this thread completes.
__device__ __forceinline__ void tc_commit(uint64_t *bar) {
    asm volatile(
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
            smem_u32(bar))
        : "memory");
}

#define QL_REG32(r)                                                                         \
    "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), \
        "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),   \
        "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), \
        "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), \
        "r"(r[29]), "r"(r[30]), "r"(r[31])
#define QL_OUT32(r)                                                                            \
    "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),        \
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), \
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),           \
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),           \
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])

// Each thread of the warp writes 32 consecutive 32-bit columns of its own lane.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t r[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
        "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, "
        "%28, %29, %30, %31, %32};" ::"r"(taddr),
        QL_REG32(r)
        : "memory");
}

__device__ __forceinline__ void tmem_st_wait() {
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Each thread of the warp reads 32 consecutive 32-bit columns of its own lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t r[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
        "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, "
        "%28, %29, %30, %31}, [%32];"
        : QL_OUT32(r)
        : "r"(taddr)
        : "memory");
}

#define QL_REG16(r)                                                                         \
    "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), \
        "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),   \
        "r"(r[15])
#define QL_OUT16(r)                                                                            \
    "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),        \
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), \
        "=r"(r[14]), "=r"(r[15])

// 16-column variants of the above.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t r[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
        "%11, %12, %13, %14, %15, %16};" ::"r"(taddr),
        QL_REG16(r)
        : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t r[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
        "%11, %12, %13, %14, %15}, [%16];"
        : QL_OUT16(r)
        : "r"(taddr)
        : "memory");
}

__device__ __forceinline__ void tmem_ld_wait() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Named barrier over `nthreads` threads (a multiple of 32).
__device__ __forceinline__ void named_bar_sync(uint32_t id, uint32_t nthreads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// UMMA shared-memory descriptor for a K-major operand stored in 128-byte
// swizzled rows (the layout TMA writes with CU_TENSOR_MAP_SWIZZLE_128B):
// 8-row atoms of 1024 bytes, so the stride between atoms (SBO) is 1024 B.
__device__ __forceinline__ uint64_t umma_desc_k_sw128(uint32_t smem_addr) {
    uint64_t d = 0;
    d |= (uint64_t)((smem_addr & 0x3ffffu) >> 4);  // start address, bits [0,14)
    d |= (uint64_t)1 << 16;                         // LBO (unused for swizzled K-major)
    d |= (uint64_t)(1024 >> 4) << 32;               // SBO, bits [32,46)
    d |= (uint64_t)1 << 46;                         // descriptor version (sm_100)
    d |= (uint64_t)2 << 61;                         // layout: SWIZZLE_128B
    return d;
}

// Instruction descriptor, kind::f16: bf16 A and B, fp32 accumulator, both K-major.
__host__ __device__ constexpr uint32_t umma_idesc_bf16(int M, int N) {
    return (1u << 4)                       // D format f32
           | (1u << 7)                     // A format bf16
           | (1u << 10)                    // B format bf16
           | ((uint32_t)(N >> 3) << 17)    // N / 8
           | ((uint32_t)(M >> 4) << 24);   // M / 16
}

}  // namespace ql
