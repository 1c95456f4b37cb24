// Status reporting, device memory and stream entry points of the C ABI.
//
// Mirrors bee::cuda's runtime wrappers (Bee/CUDA/Api.cpp:117-192): allocation
// is stream-ordered from the current device's default pool, copies are
// cudaMemcpyAsync on the caller's stream.  Unlike the reference nothing here
// synchronises implicitly; bee_b200_stream_synchronize is the explicit fence.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "common.cuh"

namespace bee_b200 {

namespace {
thread_local char g_msg[512] = "";
}

int fail(int code, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_msg, sizeof(g_msg), fmt, ap);
    va_end(ap);
    return code;
}

int ok() {
    g_msg[0] = '\0';
    return 0;
}

int api_fail(cudaError_t e, const char* fmt, ...) {
    cudaGetLastError();  // a failed runtime call must not be reported again by the next launch check
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_msg, sizeof(g_msg), fmt, ap);
    va_end(ap);
    return static_cast<int>(e);
}

int launch_status(const char* what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(static_cast<int>(e), "%s: launch failed: %s", what, cudaGetErrorString(e));
    return ok();
}

int sm_count() {
    static std::atomic<int> cached[kMaxDevices];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 148;
    int n = cached[dev].load(std::memory_order_relaxed);
    if (n == 0) {
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) return 148;
        cached[dev].store(n, std::memory_order_relaxed);
    }
    return n;
}

cudaError_t pool_malloc(void** ptr, size_t bytes, cudaStream_t st) {
    static std::mutex mu;
    static cudaMemPool_t pools[64] = {nullptr};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    cudaMemPool_t pool;
    {
        std::lock_guard<std::mutex> lock(mu);
        if (!pools[dev]) {
            cudaMemPool_t p = nullptr;
            e = cudaDeviceGetDefaultMemPool(&p, dev);
            if (e != cudaSuccess) return e;
            uint64_t keep = ~uint64_t{0};
            e = cudaMemPoolSetAttribute(p, cudaMemPoolAttrReleaseThreshold, &keep);
            if (e != cudaSuccess) return e;
            pools[dev] = p;
        }
        pool = pools[dev];
    }
    return cudaMallocFromPoolAsync(ptr, bytes, pool, st);
}

// SM clock of the SM this runs on, measured against the global nanosecond
// timer over `ns` nanoseconds (one thread; bounded by the timer and by an
// iteration cap).  Launched on a side stream while other work runs, it reads
// the clock under load without querying NVML.
__global__ void clock_probe_kernel(unsigned long long ns, float* out_mhz) {
    unsigned long long t0, t1, c0, c1;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
    c0 = clock64();
    t1 = t0;
    for (unsigned int i = 0; i < (1u << 26) && t1 - t0 < ns; ++i) asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t1));
    c1 = clock64();
    *out_mhz = t1 > t0 ? static_cast<float>(static_cast<double>(c1 - c0) * 1e3 / static_cast<double>(t1 - t0)) : 0.f;
}

}  // namespace bee_b200

using namespace bee_b200;

extern "C" {

const char* bee_b200_last_error(void) { return g_msg; }

const char* bee_b200_status_string(int status) { return cudaGetErrorString(static_cast<cudaError_t>(status)); }

int bee_b200_version(void) { return 100; }

int bee_b200_allocate(void** out_ptr, size_t nbytes, size_t alignment, bee_b200_stream_t stream) {
    if (!out_ptr) return fail(cudaErrorInvalidValue, "allocate: out_ptr is null");
    *out_ptr = nullptr;
    if (alignment > 256 || (alignment & (alignment - 1)) != 0)
        return fail(cudaErrorInvalidValue, "allocate: alignment %zu unsupported (power of two <= 256)", alignment);
    if (nbytes == 0) return ok();
    cudaError_t e = pool_malloc(out_ptr, nbytes, as_stream(stream));
    if (e != cudaSuccess) return api_fail(e, "allocate(%zu): %s", nbytes, cudaGetErrorString(e));
    return ok();
}

int bee_b200_deallocate(void* ptr, bee_b200_stream_t stream) {
    if (!ptr) return ok();
    cudaError_t e = cudaFreeAsync(ptr, as_stream(stream));
    if (e != cudaSuccess) return api_fail(e, "deallocate: %s", cudaGetErrorString(e));
    return ok();
}

static int copy(void* dst, const void* src, size_t nbytes, cudaMemcpyKind kind, bee_b200_stream_t stream,
                const char* what) {
    if (nbytes == 0) return ok();
    if (!dst || !src) return fail(cudaErrorInvalidValue, "%s: null pointer", what);
    cudaError_t e = cudaMemcpyAsync(dst, src, nbytes, kind, as_stream(stream));
    if (e != cudaSuccess) return api_fail(e, "%s(%zu): %s", what, nbytes, cudaGetErrorString(e));
    return ok();
}

int bee_b200_memcpy_h2d(void* dst, const void* src, size_t nbytes, bee_b200_stream_t stream) {
    return copy(dst, src, nbytes, cudaMemcpyHostToDevice, stream, "memcpy_h2d");
}

int bee_b200_memcpy_d2h(void* dst, const void* src, size_t nbytes, bee_b200_stream_t stream) {
    return copy(dst, src, nbytes, cudaMemcpyDeviceToHost, stream, "memcpy_d2h");
}

int bee_b200_memcpy_d2d(void* dst, const void* src, size_t nbytes, bee_b200_stream_t stream) {
    return copy(dst, src, nbytes, cudaMemcpyDeviceToDevice, stream, "memcpy_d2d");
}

int bee_b200_memset(void* ptr, int value, size_t nbytes, bee_b200_stream_t stream) {
    if (nbytes == 0) return ok();
    if (!ptr) return fail(cudaErrorInvalidValue, "memset: null pointer");
    cudaError_t e = cudaMemsetAsync(ptr, value & 0xff, nbytes, as_stream(stream));
    if (e != cudaSuccess) return api_fail(e, "memset(%zu): %s", nbytes, cudaGetErrorString(e));
    return ok();
}


int bee_b200_ipc_alloc(void** out_ptr, size_t nbytes) {
    if (!out_ptr) return fail(cudaErrorInvalidValue, "ipc_alloc: out_ptr is null");
    *out_ptr = nullptr;
    if (nbytes == 0) return fail(cudaErrorInvalidValue, "ipc_alloc: zero bytes");
    cudaError_t e = cudaMalloc(out_ptr, nbytes);
    if (e != cudaSuccess) return api_fail(e, "ipc_alloc(%zu): %s", nbytes, cudaGetErrorString(e));
    return ok();
}

int bee_b200_ipc_free(void* ptr) {
    if (!ptr) return ok();
    cudaError_t e = cudaFree(ptr);
    if (e != cudaSuccess) return api_fail(e, "ipc_free: %s", cudaGetErrorString(e));
    return ok();
}

int bee_b200_ipc_handle(const void* ptr, void* handle_out) {
    if (!ptr || !handle_out) return fail(cudaErrorInvalidValue, "ipc_handle: null pointer");
    cudaIpcMemHandle_t h;
    cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void*>(ptr));
    if (e != cudaSuccess) return api_fail(e, "ipc_handle: %s", cudaGetErrorString(e));
    static_assert(sizeof(h) == 64, "cudaIpcMemHandle_t is 64 bytes");
    memcpy(handle_out, &h, sizeof(h));
    return ok();
}

int bee_b200_ipc_open(const void* handle, void** out_ptr) {
    if (!handle || !out_ptr) return fail(cudaErrorInvalidValue, "ipc_open: null pointer");
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    cudaError_t e = cudaIpcOpenMemHandle(out_ptr, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return api_fail(e, "ipc_open: %s", cudaGetErrorString(e));
    return ok();
}

int bee_b200_ipc_close(void* ptr) {
    if (!ptr) return ok();
    cudaError_t e = cudaIpcCloseMemHandle(ptr);
    if (e != cudaSuccess) return api_fail(e, "ipc_close: %s", cudaGetErrorString(e));
    return ok();
}

int bee_b200_set_device(int device) {
    cudaError_t e = cudaSetDevice(device);
    if (e != cudaSuccess) return api_fail(e, "set_device(%d): %s", device, cudaGetErrorString(e));
    return ok();
}

int bee_b200_get_device(int* device) {
    if (!device) return fail(cudaErrorInvalidValue, "get_device: null pointer");
    cudaError_t e = cudaGetDevice(device);
    if (e != cudaSuccess) return api_fail(e, "get_device: %s", cudaGetErrorString(e));
    return ok();
}

int bee_b200_device_count(int* count) {
    if (!count) return fail(cudaErrorInvalidValue, "device_count: null pointer");
    cudaError_t e = cudaGetDeviceCount(count);
    if (e != cudaSuccess) return api_fail(e, "device_count: %s", cudaGetErrorString(e));
    return ok();
}

int bee_b200_clock_probe(unsigned long long ns, float* out_mhz, bee_b200_stream_t stream) {
    if (!out_mhz) return fail(cudaErrorInvalidValue, "clock_probe: null pointer");
    if (ns == 0 || ns > 10000000ull) return fail(cudaErrorInvalidValue, "clock_probe: duration must be in (0, 10 ms]");
    clock_probe_kernel<<<1, 1, 0, as_stream(stream)>>>(ns, out_mhz);
    return launch_status("clock_probe");
}

int bee_b200_stream_synchronize(bee_b200_stream_t stream) {
    cudaError_t e = cudaStreamSynchronize(as_stream(stream));
    if (e != cudaSuccess) return api_fail(e, "stream_synchronize: %s", cudaGetErrorString(e));
    return ok();
}

}  // extern "C"
