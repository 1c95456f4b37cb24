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
// The array is a file-scope __device__ variable: every GPU on which this
// library's module is loaded holds it (kScratchBytes) until the process exits.
// Host code cannot use the variable's name as a device address, so the entry
// point looks the address up with cudaGetSymbolAddress (with the device
// current) on every call; that lookup is a host-side table read once the module
// is loaded, and repeating it means a device reset, which reloads the module
// and may move the array, never leaves a stale address behind.
//
// Warm-up: CUDA loads modules and kernels lazily (on first use) by default, and
// loading can itself need device memory.  The first call on each device (and
// the first after a device reset) therefore does the set-up: it loads the
// module, takes the array's address and loads every kernel this entry point can
// launch (all ops and dtypes).  Make one call per device at start-up, while
// memory is still available and before any stream capture; after that no call
// loads anything.  All calls share the one array and it keeps whatever the last
// call left there: the ticket word that must start at zero is cleared on the
// stream before every launch, and calls whose kernels overlap on the GPU
// (different streams at once) race on the array — issue them on one stream, or
// use bee_b200_reduce_global.
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
void* g_loaded_at[kMaxDevices] = {nullptr};  // array address seen when this device's kernels were loaded

template <int OP, typename T> int load_kernel() {
    cudaFuncAttributes attr;
    const cudaError_t e = cudaFuncGetAttributes(&attr, reduce_global_kernel<ElemRed<OP, T>>);
    return e == cudaSuccess ? 0 : fail(static_cast<int>(e), "reduce_global_noalloc: loading a kernel: %s", cudaGetErrorString(e));
}

template <typename T> int load_kernels_of() {
    int rc = load_kernel<RED_MIN, T>();
    if (!rc) rc = load_kernel<RED_MAX, T>();
    if constexpr (!std::is_same_v<T, uint8_t>) {
        if (!rc) rc = load_kernel<RED_SUM, T>();
        if (!rc) rc = load_kernel<RED_PROD, T>();
    }
    return rc;
}

// Device address of g_noalloc_scratch on the current device.  The first call
// on a device (or the first after a reset moved the array) also loads every
// kernel this entry point launches, so later calls load nothing.
int scratch_address(void** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return fail(static_cast<int>(e), "reduce_global_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
    if (dev < 0 || dev >= kMaxDevices) return fail(cudaErrorInvalidDevice, "reduce_global_noalloc: device %d out of range", dev);
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p)
        return fail(e != cudaSuccess ? static_cast<int>(e) : cudaErrorInvalidSymbol,
                    "reduce_global_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
    std::lock_guard<std::mutex> lock(g_mu);
    if (g_loaded_at[dev] != p) {
        int rc = load_kernels_of<uint8_t>();
        if (!rc) rc = load_kernels_of<int32_t>();
        if (!rc) rc = load_kernels_of<int64_t>();
        if (!rc) rc = load_kernels_of<float>();
        if (!rc) rc = load_kernels_of<double>();
        if (rc) return rc;
        g_loaded_at[dev] = p;
    }
    *out = p;
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
