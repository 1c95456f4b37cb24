// Device-side building blocks of the reductions: accumulation functors with
// the reference's semantics, warp/block reduce, vectorised strided reduce and
// the one-launch global reduce kernel (per-CTA partials folded by the last CTA).
#pragma once

#include <cfloat>
#include <climits>

#include "common.cuh"

namespace bee_b200 {

template <typename T> struct Lim;
template <> struct Lim<uint8_t> { static __device__ uint8_t lo() { return 0; } static __device__ uint8_t hi() { return 255; } };
template <> struct Lim<int32_t> { static __device__ int32_t lo() { return INT_MIN; } static __device__ int32_t hi() { return INT_MAX; } };
template <> struct Lim<int64_t> { static __device__ int64_t lo() { return LLONG_MIN; } static __device__ int64_t hi() { return LLONG_MAX; } };
template <> struct Lim<float> { static __device__ float lo() { return -FLT_MAX; } static __device__ float hi() { return FLT_MAX; } };
template <> struct Lim<double> { static __device__ double lo() { return -DBL_MAX; } static __device__ double hi() { return DBL_MAX; } };

// Integer sum/prod go through the unsigned type so that wrap-around is
// defined behaviour (two's complement, identical bits to the reference).
template <typename T> struct Wrap { using U = T; };
template <> struct Wrap<int32_t> { using U = uint32_t; };
template <> struct Wrap<int64_t> { using U = uint64_t; };

template <int OP, typename T> struct Red {
    static __device__ __forceinline__ T identity() {
        if constexpr (OP == RED_SUM) return T(0);
        else if constexpr (OP == RED_PROD) return T(1);
        else if constexpr (OP == RED_MIN) return Lim<T>::hi();
        else return Lim<T>::lo();
    }
    static __device__ __forceinline__ T apply(T a, T b) {
        using U = typename Wrap<T>::U;
        if constexpr (OP == RED_SUM) return static_cast<T>(static_cast<U>(a) + static_cast<U>(b));
        else if constexpr (OP == RED_PROD) return static_cast<T>(static_cast<U>(a) * static_cast<U>(b));
        else if constexpr (OP == RED_MIN) return b < a ? b : a;
        else return b > a ? b : a;
    }
};

// Reduction policies: input element In, accumulator Acc, output Out.
//   ElemRed<OP, T>: the reference's reduce semantics, accumulating in T.
//   MeanInt<T>: integer mean (Bee/Tensor/Cpu/ReduceCpu.hpp:431-466, 551-610):
//     the exact integer sum in int64 (two's complement, no overflow while
//     |sum| < 2^63), then double(sum) / double(count).  The reference
//     accumulates in double, which is exact while every partial sum stays
//     below 2^53 in magnitude; in that range both give the same bits.
template <int OP, typename T> struct ElemRed {
    using In = T;
    using Acc = T;
    using Out = T;
    static __device__ __forceinline__ Acc identity() { return Red<OP, T>::identity(); }
    static __device__ __forceinline__ Acc add(Acc a, In x) { return Red<OP, T>::apply(a, x); }
    static __device__ __forceinline__ Acc combine(Acc a, Acc b) { return Red<OP, T>::apply(a, b); }
    static __device__ __forceinline__ Out finish(Acc a, size_t) { return a; }
};

template <typename T> struct MeanInt {
    using In = T;
    using Acc = long long;
    using Out = double;
    static __device__ __forceinline__ Acc identity() { return 0; }
    static __device__ __forceinline__ Acc combine(Acc a, Acc b) {
        return static_cast<Acc>(static_cast<unsigned long long>(a) + static_cast<unsigned long long>(b));
    }
    static __device__ __forceinline__ Acc add(Acc a, In x) { return combine(a, static_cast<Acc>(x)); }
    static __device__ __forceinline__ Out finish(Acc a, size_t n) {
        return static_cast<double>(a) / static_cast<double>(n);
    }
};

template <typename P> __device__ __forceinline__ typename P::Acc warp_reduce(typename P::Acc v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = P::combine(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Block-wide reduce; the result is valid in every thread.  `smem` holds
// blockDim.x / 32 entries.
template <typename P> __device__ __forceinline__ typename P::Acc block_reduce(typename P::Acc v, typename P::Acc* smem) {
    using Acc = typename P::Acc;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    v = warp_reduce<P>(v);
    __syncthreads();
    if (lane == 0) smem[warp] = v;
    __syncthreads();
    Acc r = P::identity();
    for (int w = 0; w < nwarps; ++w) r = P::combine(r, smem[w]);
    return r;
}

template <typename T> union V16 {
    uint4 v;
    T s[16 / sizeof(T)];
};

// Folds a 16-byte vector of In into `acc` lane by lane (fixed order).
template <typename P> __device__ __forceinline__ typename P::Acc fold(typename P::Acc acc, uint4 raw) {
    using In = typename P::In;
    V16<In> x;
    x.v = raw;
#pragma unroll
    for (int k = 0; k < int(16 / sizeof(In)); ++k) acc = P::add(acc, x.s[k]);
    return acc;
}

// Reduces src[lo, hi) cooperatively by `nthr` threads (index `tid`); the
// 16-byte vector path is used when src+lo is 16-byte aligned.
template <typename P, int U = 4>
__device__ __forceinline__ typename P::Acc strided_reduce(const typename P::In* __restrict__ src, size_t lo, size_t hi,
                                                          size_t tid, size_t nthr) {
    using In = typename P::In;
    constexpr size_t E = 16 / sizeof(In);
    typename P::Acc acc = P::identity();
    const In* base = src + lo;
    const size_t len = hi - lo;
    size_t head = 0;
    if ((reinterpret_cast<uintptr_t>(base) & 15u) == 0) {
        const size_t nvec = len / E;
        const uint4* v = reinterpret_cast<const uint4*>(base);
        size_t i = tid;
        for (; i + (U - 1) * nthr < nvec; i += U * nthr) {
            uint4 r[U];
#pragma unroll
            for (int u = 0; u < U; ++u) r[u] = ld_stream_u4(v + i + u * nthr);
#pragma unroll
            for (int u = 0; u < U; ++u) acc = fold<P>(acc, r[u]);
        }
        for (; i < nvec; i += nthr) acc = fold<P>(acc, ld_stream_u4(v + i));
        head = nvec * E;
    }
    for (size_t j = head + tid; j < len; j += nthr) acc = P::add(acc, base[j]);
    return acc;
}

// ---------------------------------------------------------------- global

struct GlobalScratch {
    unsigned int ticket;  // number of CTAs that have published their partial
    unsigned int pad[63];
    // followed by gridDim.x partials of sizeof(Acc), 256-byte aligned
};

// Global reduce, one launch.  The input is cut into units of 256 threads x 8
// vectors of 16 bytes (32 KiB); CTA b folds units b, b + G, b + 2G, ... (so
// the units in flight across the GPU form a contiguous window of memory, and
// each thread has 8 independent 16-byte loads outstanding), reduces its
// partial through shared memory, and the last CTA to take a ticket folds the
// G partials in index order.  The assignment of elements to threads and the
// folding order depend only on n and G, so float results are reproducible.
constexpr int kGlobalThreads = 256;
constexpr int kGlobalUnroll = 8;

// Grid of the global reduce for n elements of T: at most 8 CTAs per SM, never
// more CTAs than 32 KiB units.
template <typename T> inline unsigned global_grid(size_t n, int sms) {
    const size_t unit = static_cast<size_t>(kGlobalThreads) * kGlobalUnroll * (16 / sizeof(T));
    const size_t need = (n + unit - 1) / unit;
    const size_t cap = static_cast<size_t>(sms) * 8;
    return static_cast<unsigned>(need < 1 ? 1 : (need < cap ? need : cap));
}

template <typename P>
__global__ void __launch_bounds__(kGlobalThreads) reduce_global_kernel(const typename P::In* __restrict__ src,
                                                                       typename P::Out* __restrict__ dst, size_t n,
                                                                       GlobalScratch* scratch) {
    using In = typename P::In;
    using Acc = typename P::Acc;
    constexpr size_t E = 16 / sizeof(In);
    constexpr size_t UNIT = static_cast<size_t>(kGlobalThreads) * kGlobalUnroll;  // vectors per unit
    __shared__ Acc smem[32];
    __shared__ bool last;
    Acc* partials = reinterpret_cast<Acc*>(scratch + 1);
    const unsigned tid = threadIdx.x;
    Acc acc = P::identity();
    pdl_wait();
    if ((reinterpret_cast<uintptr_t>(src) & 15u) == 0) {
        const uint4* v = reinterpret_cast<const uint4*>(src);
        const size_t nvec = n / E;
        for (size_t base = static_cast<size_t>(blockIdx.x) * UNIT; base < nvec; base += static_cast<size_t>(gridDim.x) * UNIT) {
            if (base + UNIT <= nvec) {
                uint4 r[kGlobalUnroll];
#pragma unroll
                for (int k = 0; k < kGlobalUnroll; ++k) r[k] = ld_stream_u4(v + base + k * kGlobalThreads + tid);
#pragma unroll
                for (int k = 0; k < kGlobalUnroll; ++k) acc = fold<P>(acc, r[k]);
            } else {
                for (int k = 0; k < kGlobalUnroll; ++k) {
                    const size_t idx = base + k * kGlobalThreads + tid;
                    if (idx < nvec) acc = fold<P>(acc, ld_stream_u4(v + idx));
                }
            }
        }
        if (blockIdx.x == 0)
            for (size_t j = nvec * E + tid; j < n; j += kGlobalThreads) acc = P::add(acc, src[j]);
    } else {
        const size_t stride = static_cast<size_t>(gridDim.x) * kGlobalThreads;
        for (size_t j = static_cast<size_t>(blockIdx.x) * kGlobalThreads + tid; j < n; j += stride)
            acc = P::add(acc, src[j]);
    }
    pdl_trigger();
    acc = block_reduce<P>(acc, smem);
    if (tid == 0) {
        partials[blockIdx.x] = acc;
        __threadfence();
        unsigned int t = atomicAdd(&scratch->ticket, 1u);
        last = (t == gridDim.x - 1);
    }
    __syncthreads();
    if (!last) return;
    __threadfence();
    // Last CTA: fold the partials in index order (thread-strided, then the
    // block reduce), then re-arm the ticket for the next call.
    Acc r = P::identity();
    for (unsigned i = tid; i < gridDim.x; i += kGlobalThreads)
        r = P::combine(r, *reinterpret_cast<volatile Acc*>(partials + i));
    r = block_reduce<P>(r, smem);
    if (tid == 0) {
        *dst = P::finish(r, n);
        scratch->ticket = 0;
    }
}

}  // namespace bee_b200
