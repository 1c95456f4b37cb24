// bee_b200_reduce_global_noalloc: the global reduce without any allocation.
//
// Who needs this: code that must not allocate device memory at the moment it
// reduces — error handling or diagnostics that run after an out-of-memory
// failure, a host runtime that has handed every byte of device memory to its
// own allocator and does not let libraries take more, or a latency-critical
// loop that cannot risk the stream-ordered pool growing (which calls into the
// driver).  bee_b200_reduce_global takes its per-block scratch from that pool
// on every call; this variant uses a fixed array compiled into the library
// instead, and the caller still supplies the input and the output.
//
// The array is a file-scope __device__ variable, so every GPU on which the
// library is loaded holds it (kScratchBytes) from module load until the
// process exits.  Host code cannot use the variable's name as a device
// address, so the first call on each device looks the address up with
// cudaGetSymbolAddress (with that device current) and caches it; make that
// first call before any stream capture.  All calls share the one array and it
// keeps whatever the last call left there: the ticket word that must start at
// zero is cleared on the stream before every launch, and calls whose kernels
// overlap on the GPU (different streams at once) race on the array — issue
// them on one stream, or use bee_b200_reduce_global.
#include <mutex>

#include "reduce.cuh"

namespace bee_b200 {

namespace {

// Ticket header (256 bytes) plus per-CTA partials: 64 KiB holds 8160 partials
// of 8 bytes; the kernel launches at most eight CTAs per SM (1184 on a B200).
constexpr size_t kScratchBytes = 64 * 1024;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_addr[kMaxDevices] = {nullptr};

// Device address of g_noalloc_scratch on the current device (set-up once per device).
int scratch_address(void** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return fail(static_cast<int>(e), "reduce_global_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
    if (dev < 0 || dev >= kMaxDevices) return fail(cudaErrorInvalidDevice, "reduce_global_noalloc: device %d out of range", dev);
    std::lock_guard<std::mutex> lock(g_mu);
    if (!g_addr[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || !p)
            return fail(e != cudaSuccess ? static_cast<int>(e) : cudaErrorInvalidSymbol,
                        "reduce_global_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
        g_addr[dev] = p;
    }
    *out = g_addr[dev];
    return 0;
}

template <int OP, typename T>
int run_noalloc(const void* src, void* dst, size_t n, cudaStream_t st) {
    const unsigned grid = global_grid<T>(n, sm_count());
    const size_t bytes = sizeof(GlobalScratch) + static_cast<size_t>(grid) * sizeof(T);
    if (bytes > kScratchBytes)
        return fail(cudaErrorInvalidValue,
                    "reduce_global_noalloc: %u block partials need %zu bytes of scratch, the fixed scratch holds %zu",
                    grid, bytes, kScratchBytes);
    void* scratch = nullptr;
    if (int rc = scratch_address(&scratch)) return rc;
    cudaError_t e = cudaMemsetAsync(scratch, 0, sizeof(GlobalScratch), st);
    if (e != cudaSuccess) return fail(static_cast<int>(e), "reduce_global_noalloc: clearing the ticket: %s", cudaGetErrorString(e));
    reduce_global_kernel<ElemRed<OP, T>><<<grid, kGlobalThreads, 0, st>>>(static_cast<const T*>(src), static_cast<T*>(dst), n,
                                                                 static_cast<GlobalScratch*>(scratch));
    return launch_status("reduce_global_noalloc");
}

template <typename T>
int dispatch_noalloc(int op, const void* src, void* dst, size_t n, cudaStream_t st) {
    switch (op) {
    case RED_SUM: if constexpr (!std::is_same_v<T, uint8_t>) return run_noalloc<RED_SUM, T>(src, dst, n, st); break;
    case RED_PROD: if constexpr (!std::is_same_v<T, uint8_t>) return run_noalloc<RED_PROD, T>(src, dst, n, st); break;
    case RED_MIN: return run_noalloc<RED_MIN, T>(src, dst, n, st);
    case RED_MAX: return run_noalloc<RED_MAX, T>(src, dst, n, st);
    default: return fail(cudaErrorInvalidValue, "reduce_global_noalloc: unknown op code %d", op);
    }
    return fail(cudaErrorInvalidValue, "reduce_global_noalloc: op %d does not support U8", op);
}

}  // namespace
}  // namespace bee_b200

using namespace bee_b200;

extern "C" int bee_b200_reduce_global_noalloc(int op, int dt, const void* src, void* dst, size_t n,
                                              bee_b200_stream_t stream) {
    if (n == 0) return fail(cudaErrorInvalidValue, "reduce_global_noalloc: empty input");
    if (!src || !dst) return fail(cudaErrorInvalidValue, "reduce_global_noalloc: null pointer");
    cudaStream_t st = as_stream(stream);
    switch (dt) {
    case DT_U8: return dispatch_noalloc<uint8_t>(op, src, dst, n, st);
    case DT_I32: return dispatch_noalloc<int32_t>(op, src, dst, n, st);
    case DT_I64: return dispatch_noalloc<int64_t>(op, src, dst, n, st);
    case DT_F32: return dispatch_noalloc<float>(op, src, dst, n, st);
    case DT_F64: return dispatch_noalloc<double>(op, src, dst, n, st);
    default: return fail(cudaErrorInvalidValue, "reduce_global_noalloc: unsupported dtype %d", dt);
    }
}
