// Global and per-axis reductions (HBM-bound).
//
// Replaces K7/K8 of the reference (Bee/CUDA/Ops/Reduce.cu:129-183).  The
// reference's axis reduce gives one thread a whole row, so for a row reduce
// neighbouring threads read addresses a row apart; here a row is owned by a
// CTA (long rows) or a warp (short rows) that streams it with coalesced
// 16-byte loads and combines with warp shuffles.  The global reduce is one
// launch: every CTA reduces a grid-stride slice into a partial, and the last
// CTA to finish (atomic ticket) folds the partials in index order, so float
// results do not depend on scheduling.
//
// Accumulation semantics follow the reference's OpReduce* functors
// (Bee/Tensor/Cpu/ReduceCpu.hpp:177-290): accumulate in the element type
// (integer sums and products wrap), min/max by comparison, identities
// 0 / 1 / numeric max / numeric lowest.
#include <mutex>
#include <vector>

#include "reduce.cuh"

namespace bee_b200 {

// ---------------------------------------------------------------- axis

// One 256-thread CTA per row of length `axis` (inner == 1), launched one CTA
// per row so that the rows in flight on the GPU form a contiguous window of
// memory (better DRAM locality than a grid-stride over rows).
template <int OP, typename T>
__global__ void __launch_bounds__(256) reduce_rows_cta_kernel(const T* __restrict__ src, T* __restrict__ dst,
                                                              size_t rows, size_t axis) {
    __shared__ T smem[32];
    for (size_t r = blockIdx.x; r < rows; r += gridDim.x) {
        T v = strided_reduce<OP, T, 8>(src + r * axis, 0, axis, threadIdx.x, blockDim.x);
        v = block_reduce<OP>(v, smem);
        if (threadIdx.x == 0) dst[r] = v;
    }
}

// One warp per row (short rows, inner == 1).
template <int OP, typename T>
__global__ void __launch_bounds__(256) reduce_rows_warp_kernel(const T* __restrict__ src, T* __restrict__ dst,
                                                               size_t rows, size_t axis) {
    const size_t warps = static_cast<size_t>(gridDim.x) * (blockDim.x >> 5);
    const int lane = threadIdx.x & 31;
    for (size_t r = static_cast<size_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); r < rows; r += warps) {
        T v = strided_reduce<OP>(src + r * axis, 0, axis, lane, 32);
        v = warp_reduce<OP>(v);
        if (lane == 0) dst[r] = v;
    }
}

// [outer, axis, inner] with inner > 1: one thread per output, neighbouring
// threads read neighbouring inner elements (coalesced), walking the axis.
template <int OP, typename T>
__global__ void __launch_bounds__(256) reduce_inner_kernel(const T* __restrict__ src, T* __restrict__ dst,
                                                           size_t outer, size_t axis, size_t inner) {
    const size_t total = outer * inner;
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    for (size_t idx = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; idx < total; idx += stride) {
        const size_t o = idx / inner, i = idx - o * inner;
        const T* p = src + o * axis * inner + i;
        T acc = Red<OP, T>::identity();
        for (size_t k = 0; k < axis; ++k) acc = Red<OP, T>::apply(acc, p[k * inner]);
        dst[idx] = acc;
    }
}

// Scratch of the global reduce: one 16 KiB block (ticket + up to 2016
// partials of 8 bytes) per (device, stream), taken from the stream-ordered
// pool on a stream's first reduce, ticket zeroed once, and kept for the life
// of the process; the kernel re-arms the ticket itself, so later calls on the
// stream are a single launch.  Streams are keyed by cudaStreamGetId, which is
// never reused, so a destroyed stream's block is never handed to another
// stream.  During stream capture (and past 256 streams on one device) the call
// instead allocates, zeroes and frees a block around the launch, stream-ordered.
constexpr size_t kStreamScratchBytes = 16 * 1024;

struct StreamScratch {
    unsigned long long id;
    void* ptr;
};

static int stream_scratch(cudaStream_t st, void** out) {
    static std::mutex mu;
    static std::vector<StreamScratch> table[64];
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(st, &cap) != cudaSuccess || cap != cudaStreamCaptureStatusNone) return 1;
    unsigned long long id = 0;
    int dev = 0;
    if (cudaStreamGetId(st, &id) != cudaSuccess || cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 1;
    std::lock_guard<std::mutex> lock(mu);
    for (const StreamScratch& e : table[dev])
        if (e.id == id) {
            *out = e.ptr;
            return 0;
        }
    if (table[dev].size() >= 256) return 1;
    void* p = nullptr;
    if (pool_malloc(&p, kStreamScratchBytes, st) != cudaSuccess) return 1;
    if (cudaMemsetAsync(p, 0, sizeof(GlobalScratch), st) != cudaSuccess) {
        cudaFreeAsync(p, st);
        return 1;
    }
    table[dev].push_back({id, p});
    *out = p;
    return 0;
}

template <int OP, typename T>
static int run_global(const void* src, void* dst, size_t n, cudaStream_t st) {
    const unsigned grid = global_grid<T>(n, sm_count());
    const size_t bytes = sizeof(GlobalScratch) + static_cast<size_t>(grid) * sizeof(T);
    void* scratch = nullptr;
    if (bytes <= kStreamScratchBytes && stream_scratch(st, &scratch) == 0) {
        cudaGetLastError();  // a failed probe above must not be reported as a launch error
        reduce_global_kernel<OP, T><<<grid, kGlobalThreads, 0, st>>>(static_cast<const T*>(src), static_cast<T*>(dst),
                                                                     n, static_cast<GlobalScratch*>(scratch));
        return launch_status("reduce_global");
    }
    cudaGetLastError();
    cudaError_t e = pool_malloc(&scratch, bytes, st);
    if (e != cudaSuccess) return fail(static_cast<int>(e), "reduce_global: scratch allocation: %s", cudaGetErrorString(e));
    e = cudaMemsetAsync(scratch, 0, sizeof(GlobalScratch), st);
    if (e == cudaSuccess) {
        reduce_global_kernel<OP, T><<<grid, kGlobalThreads, 0, st>>>(static_cast<const T*>(src), static_cast<T*>(dst),
                                                                     n, static_cast<GlobalScratch*>(scratch));
        e = cudaGetLastError();
    }
    cudaError_t e2 = cudaFreeAsync(scratch, st);
    if (e != cudaSuccess) return fail(static_cast<int>(e), "reduce_global: %s", cudaGetErrorString(e));
    if (e2 != cudaSuccess) return fail(static_cast<int>(e2), "reduce_global: scratch release: %s", cudaGetErrorString(e2));
    return ok();
}

template <int OP, typename T>
static int run_axis(const void* src, void* dst, size_t outer, size_t axis, size_t inner, cudaStream_t st) {
    const T* s = static_cast<const T*>(src);
    T* d = static_cast<T*>(dst);
    const size_t cap = static_cast<size_t>(sm_count()) * 16;
    if (inner == 1) {
        if (axis >= 2048) {
            const size_t grid = outer < (size_t(1) << 30) ? outer : (size_t(1) << 30);
            reduce_rows_cta_kernel<OP, T><<<static_cast<unsigned>(grid), 256, 0, st>>>(s, d, outer, axis);
        } else {
            size_t grid = (outer + 7) / 8;
            if (grid > cap) grid = cap;
            reduce_rows_warp_kernel<OP, T><<<static_cast<unsigned>(grid), 256, 0, st>>>(s, d, outer, axis);
        }
    } else {
        size_t grid = (outer * inner + 255) / 256;
        if (grid > cap) grid = cap;
        reduce_inner_kernel<OP, T><<<static_cast<unsigned>(grid), 256, 0, st>>>(s, d, outer, axis, inner);
    }
    return launch_status("reduce_axis");
}

template <typename T>
static int dispatch_global(int op, const void* src, void* dst, size_t n, cudaStream_t st) {
    switch (op) {
    case RED_SUM: if constexpr (!std::is_same_v<T, uint8_t>) return run_global<RED_SUM, T>(src, dst, n, st); break;
    case RED_PROD: if constexpr (!std::is_same_v<T, uint8_t>) return run_global<RED_PROD, T>(src, dst, n, st); break;
    case RED_MIN: return run_global<RED_MIN, T>(src, dst, n, st);
    case RED_MAX: return run_global<RED_MAX, T>(src, dst, n, st);
    default: return fail(cudaErrorInvalidValue, "reduce_global: unknown op code %d", op);
    }
    return fail(cudaErrorInvalidValue, "reduce_global: op %d does not support U8", op);
}

template <typename T>
static int dispatch_axis(int op, const void* src, void* dst, size_t outer, size_t axis, size_t inner, cudaStream_t st) {
    switch (op) {
    case RED_SUM: if constexpr (!std::is_same_v<T, uint8_t>) return run_axis<RED_SUM, T>(src, dst, outer, axis, inner, st); break;
    case RED_PROD: if constexpr (!std::is_same_v<T, uint8_t>) return run_axis<RED_PROD, T>(src, dst, outer, axis, inner, st); break;
    case RED_MIN: return run_axis<RED_MIN, T>(src, dst, outer, axis, inner, st);
    case RED_MAX: return run_axis<RED_MAX, T>(src, dst, outer, axis, inner, st);
    default: return fail(cudaErrorInvalidValue, "reduce_axis: unknown op code %d", op);
    }
    return fail(cudaErrorInvalidValue, "reduce_axis: op %d does not support U8", op);
}

}  // namespace bee_b200

using namespace bee_b200;

extern "C" {

int bee_b200_reduce_global(int op, int dt, const void* src, void* dst, size_t n, bee_b200_stream_t stream) {
    if (n == 0) return fail(cudaErrorInvalidValue, "reduce_global: empty input");
    if (!src || !dst) return fail(cudaErrorInvalidValue, "reduce_global: null pointer");
    cudaStream_t st = as_stream(stream);
    switch (dt) {
    case DT_U8: return dispatch_global<uint8_t>(op, src, dst, n, st);
    case DT_I32: return dispatch_global<int32_t>(op, src, dst, n, st);
    case DT_I64: return dispatch_global<int64_t>(op, src, dst, n, st);
    case DT_F32: return dispatch_global<float>(op, src, dst, n, st);
    case DT_F64: return dispatch_global<double>(op, src, dst, n, st);
    default: return fail(cudaErrorInvalidValue, "reduce_global: unsupported dtype %d", dt);
    }
}

int bee_b200_reduce_axis(int op, int dt, const void* src, void* dst, size_t outer, size_t axis, size_t inner,
                         bee_b200_stream_t stream) {
    if (outer == 0 || axis == 0 || inner == 0) return fail(cudaErrorInvalidValue, "reduce_axis: empty extent");
    if (!src || !dst) return fail(cudaErrorInvalidValue, "reduce_axis: null pointer");
    cudaStream_t st = as_stream(stream);
    switch (dt) {
    case DT_U8: return dispatch_axis<uint8_t>(op, src, dst, outer, axis, inner, st);
    case DT_I32: return dispatch_axis<int32_t>(op, src, dst, outer, axis, inner, st);
    case DT_I64: return dispatch_axis<int64_t>(op, src, dst, outer, axis, inner, st);
    case DT_F32: return dispatch_axis<float>(op, src, dst, outer, axis, inner, st);
    case DT_F64: return dispatch_axis<double>(op, src, dst, outer, axis, inner, st);
    default: return fail(cudaErrorInvalidValue, "reduce_axis: unsupported dtype %d", dt);
    }
}

}  // extern "C"
