// noalloc.cu -- ql_quantized_matmul_noalloc: the matmul entry point for callers that
// cannot allocate device memory.
//
// Some callers cannot call cudaMalloc at all: code running inside a host-side
// allocator hook, a real-time loop that must not block on the driver's allocator,
// or a runtime whose memory is fully reserved by its own pool.  The only scratch the
// matmul path needs is the LoRA workspace T = scale * (x . A) (M x round_up(rank, 64)
// bf16).  This entry point takes that workspace from a fixed file-scope device array
// instead of from the caller, and allocates nothing.
//
// Limits and behaviour:
//   * The array holds kNoAllocScratchBytes (8 MiB): M * round_up(rank, 64) * 2 bytes
//     must fit (e.g. M = 32768 tokens at rank <= 128).  Larger requests are rejected
//     with QL_EUNSUPPORTED and a message; nothing runs.
//   * Every GPU that loads the library holds the 8 MiB until the process exits.
//   * The first call on a device (with or without a LoRA residual) looks up the
//     array's device address (cudaGetSymbolAddress) with that device current; make
//     that first call before any stream capture.
//   * All calls on a device share the one array.  The LoRA pre-pass overwrites every
//     byte it later reads, so no clearing is needed between calls, but two calls whose
//     kernels overlap on the GPU (different streams, no ordering) race on it.
#include <mutex>

#include "ql_common.cuh"

namespace ql {

constexpr size_t kNoAllocScratchBytes = 8u << 20;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// Device address of g_noalloc_scratch on the current device (looked up once per device).
static int noalloc_scratch(void **out) {
    static void *addr[kMaxDevices] = {};
    static std::mutex mu;
    int dev = 0;
    QL_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kMaxDevices) return fail(QL_EUNSUPPORTED, "device ordinal %d out of range", dev);
    std::lock_guard<std::mutex> lock(mu);
    if (!addr[dev]) {
        void *p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess)
            return fail(QL_ECUDA, "cudaGetSymbolAddress(noalloc scratch) failed: %s", cudaGetErrorString(e));
        addr[dev] = p;
    }
    *out = addr[dev];
    return QL_OK;
}

}  // namespace ql

extern "C" int ql_quantized_matmul_noalloc(const void *x, int x_dtype, int64_t M, int64_t K,
                                           const uint32_t *wq, const void *scales, const void *biases,
                                           int sb_dtype, int64_t N, int group_size, int bits,
                                           int transpose, const ql_epilogue *ep, void *y, int y_dtype,
                                           void *stream) {
    using namespace ql;
    ql_epilogue e{};
    if (ep) e = *ep;
    const size_t need = ql_matmul_workspace_size(M, N, K, &e);
    if (need > kNoAllocScratchBytes)
        return fail(QL_EUNSUPPORTED,
                    "ql_quantized_matmul_noalloc: LoRA workspace of %zu bytes exceeds the fixed %zu-byte "
                    "scratch (M * round_up(rank, 64) * 2)",
                    need, kNoAllocScratchBytes);
    // The lookup runs on every call (cached per device), so the first call on a device
    // does it whatever its epilogue: a warm-up call without LoRA before stream capture
    // is enough.
    void *scratch = nullptr;
    if (int rc = noalloc_scratch(&scratch)) return rc;
    if (need > 0) {
        e.workspace = scratch;
        e.workspace_bytes = kNoAllocScratchBytes;
    }
    return ql_quantized_matmul(x, x_dtype, M, K, wq, scales, biases, sb_dtype, N, group_size, bits,
                               transpose, &e, y, y_dtype, stream);
}
