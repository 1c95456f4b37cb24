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
#include "sm100.cuh"

namespace bee_b200 {

// ---------------------------------------------------------------- axis

// One 256-thread CTA per row of length `axis` (inner == 1), launched one CTA
// per row so that the rows in flight on the GPU form a contiguous window of
// memory (better DRAM locality than a grid-stride over rows).
template <typename P>
__global__ void __launch_bounds__(256) reduce_rows_cta_kernel(const typename P::In* __restrict__ src,
                                                              typename P::Out* __restrict__ dst, size_t rows,
                                                              size_t axis) {
    __shared__ typename P::Acc smem[32];
    pdl_wait();
    pdl_trigger();  // counts once every CTA (all waves) has started
    for (size_t r = blockIdx.x; r < rows; r += gridDim.x) {
        typename P::Acc v = strided_reduce<P, 8>(src + r * axis, 0, axis, threadIdx.x, blockDim.x);
        v = block_reduce<P>(v, smem);
        if (threadIdx.x == 0) dst[r] = P::finish(v, axis);
    }
}

// One warp per row (short rows, inner == 1).
template <typename P>
__global__ void __launch_bounds__(256) reduce_rows_warp_kernel(const typename P::In* __restrict__ src,
                                                               typename P::Out* __restrict__ dst, size_t rows,
                                                               size_t axis) {
    const size_t warps = static_cast<size_t>(gridDim.x) * (blockDim.x >> 5);
    const int lane = threadIdx.x & 31;
    pdl_wait();
    for (size_t r = static_cast<size_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); r < rows; r += warps) {
        typename P::Acc v = strided_reduce<P>(src + r * axis, 0, axis, lane, 32);
        v = warp_reduce<P>(v);
        if (lane == 0) dst[r] = P::finish(v, axis);
    }
    pdl_trigger();
}

// Cross-CTA combine of a split reduction: `count` CTAs publish partials of one
// output group; the last to take the group's ticket folds them in index order
// and re-arms the ticket.
struct SplitScratch {
    unsigned int* tickets;  // one per output group, zero on entry
    void* partials;         // Acc[count][group width]
};

// Few long rows (inner == 1): S CTAs per row, each folding an interleaved
// share of the row's 32 KiB units, partials combined by the row's last CTA in
// index order (deterministic for a given S).
template <typename P>
__global__ void __launch_bounds__(256) reduce_rows_split_kernel(const typename P::In* __restrict__ src,
                                                                typename P::Out* __restrict__ dst, size_t rows,
                                                                size_t axis, unsigned S, SplitScratch sc) {
    using Acc = typename P::Acc;
    using In = typename P::In;
    constexpr size_t E = 16 / sizeof(In);
    constexpr size_t UNIT = 256 * 8;  // vectors per unit
    __shared__ Acc smem[32];
    __shared__ bool last;
    Acc* partials = static_cast<Acc*>(sc.partials);
    for (size_t b = blockIdx.x; b < rows * S; b += gridDim.x) {
        const size_t row = b / S;
        const unsigned part = static_cast<unsigned>(b % S);
        const In* base = src + row * axis;
        Acc acc = P::identity();
        if ((reinterpret_cast<uintptr_t>(base) & 15u) == 0) {
            const uint4* v = reinterpret_cast<const uint4*>(base);
            const size_t nvec = axis / E;
            for (size_t u = static_cast<size_t>(part) * UNIT; u < nvec; u += static_cast<size_t>(S) * UNIT) {
                uint4 r[8];
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    const size_t idx = u + k * 256 + threadIdx.x;
                    r[k] = idx < nvec ? ld_stream_u4(v + idx) : make_uint4(0, 0, 0, 0);
                }
#pragma unroll
                for (int k = 0; k < 8; ++k)
                    if (u + k * 256 + threadIdx.x < nvec) acc = fold<P>(acc, r[k]);
            }
            if (part == 0)
                for (size_t j = nvec * E + threadIdx.x; j < axis; j += 256) acc = P::add(acc, base[j]);
        } else {
            for (size_t j = static_cast<size_t>(part) * 256 + threadIdx.x; j < axis; j += static_cast<size_t>(S) * 256)
                acc = P::add(acc, base[j]);
        }
        acc = block_reduce<P>(acc, smem);
        if (threadIdx.x == 0) {
            partials[row * S + part] = acc;
            __threadfence();
            last = atomicAdd(&sc.tickets[row], 1u) == S - 1;
        }
        __syncthreads();
        if (last) {
            __threadfence();
            Acc r = P::identity();
            for (unsigned i = threadIdx.x; i < S; i += 256)
                r = P::combine(r, *reinterpret_cast<volatile Acc*>(partials + row * S + i));
            r = block_reduce<P>(r, smem);
            if (threadIdx.x == 0) {
                dst[row] = P::finish(r, axis);
                sc.tickets[row] = 0;
            }
        }
        __syncthreads();
    }
}

// [outer, axis, inner] with inner > 1 (reduce over a non-innermost dim).  A
// work item is (o, column tile, axis segment): the 32 lanes of a warp cover a
// tile of 32 x E contiguous columns (E = 16 / sizeof(In) when inner allows
// 16-byte vectors, else 1), so every row access is one coalesced 512-byte (or
// 32-element) segment; the 8 warps take rows k = k0 + w, k0 + w + 8, ... of
// the segment, four rows in flight each; warp partials are combined in warp
// order through shared memory.  With G > 1 segments, tile partials go to
// scratch and the segment that arrives last folds them in segment order.
template <typename P, int E>
__global__ void __launch_bounds__(256) reduce_cols_kernel(const typename P::In* __restrict__ src,
                                                          typename P::Out* __restrict__ dst, size_t outer, size_t axis,
                                                          size_t inner, size_t ctiles, unsigned G, size_t seg,
                                                          SplitScratch sc) {
    using Acc = typename P::Acc;
    using In = typename P::In;
    constexpr int TW = 32 * E;  // columns per tile
    __shared__ Acc red[8][TW];
    __shared__ bool last;
    Acc* partials = static_cast<Acc*>(sc.partials);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const size_t items = outer * ctiles * G;
    for (size_t w = blockIdx.x; w < items; w += gridDim.x) {
        const unsigned g = static_cast<unsigned>(w % G);
        const size_t rest = w / G;
        const size_t ct = rest % ctiles, o = rest / ctiles;
        const size_t col0 = ct * TW;
        const size_t col = col0 + static_cast<size_t>(lane) * E;
        const size_t k0 = static_cast<size_t>(g) * seg;
        const size_t k1 = k0 + seg < axis ? k0 + seg : axis;
        Acc acc[E];
#pragma unroll
        for (int j = 0; j < E; ++j) acc[j] = P::identity();
        const In* base = src + o * axis * inner + col;
        if constexpr (E > 1) {
            if (col < inner) {  // inner % E == 0: the whole vector is in range
                size_t k = k0 + warp;
                for (; k + 24 < k1; k += 32) {
                    uint4 r[4];
#pragma unroll
                    for (int u = 0; u < 4; ++u) r[u] = ld_stream_u4(reinterpret_cast<const uint4*>(base + (k + 8 * u) * inner));
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        V16<In> x;
                        x.v = r[u];
#pragma unroll
                        for (int j = 0; j < E; ++j) acc[j] = P::add(acc[j], x.s[j]);
                    }
                }
                for (; k < k1; k += 8) {
                    V16<In> x;
                    x.v = ld_stream_u4(reinterpret_cast<const uint4*>(base + k * inner));
#pragma unroll
                    for (int j = 0; j < E; ++j) acc[j] = P::add(acc[j], x.s[j]);
                }
            }
        } else {
            if (col < inner) {
                size_t k = k0 + warp;
                for (; k + 24 < k1; k += 32) {
                    In r[4];
#pragma unroll
                    for (int u = 0; u < 4; ++u) r[u] = base[(k + 8 * u) * inner];
#pragma unroll
                    for (int u = 0; u < 4; ++u) acc[0] = P::add(acc[0], r[u]);
                }
                for (; k < k1; k += 8) acc[0] = P::add(acc[0], base[k * inner]);
            }
        }
#pragma unroll
        for (int j = 0; j < E; ++j) red[warp][lane * E + j] = acc[j];
        __syncthreads();
        for (int c = threadIdx.x; c < TW; c += 256) {
            Acc r = red[0][c];
#pragma unroll
            for (int v = 1; v < 8; ++v) r = P::combine(r, red[v][c]);
            if (col0 + c < inner) {
                if (G == 1) dst[o * inner + col0 + c] = P::finish(r, axis);
                else partials[(static_cast<size_t>(g) * outer + o) * inner + col0 + c] = r;
            }
        }
        if (G > 1) {
            __threadfence();
            __syncthreads();
            if (threadIdx.x == 0) last = atomicAdd(&sc.tickets[o * ctiles + ct], 1u) == G - 1;
            __syncthreads();
            if (last) {
                __threadfence();
                for (int c = threadIdx.x; c < TW; c += 256) {
                    if (col0 + c >= inner) continue;
                    Acc r = P::identity();
                    for (unsigned gg = 0; gg < G; ++gg)
                        r = P::combine(r, *reinterpret_cast<volatile Acc*>(partials + (static_cast<size_t>(gg) * outer + o) * inner + col0 + c));
                    dst[o * inner + col0 + c] = P::finish(r, axis);
                }
                if (threadIdx.x == 0) sc.tickets[o * ctiles + ct] = 0;
            }
        }
        __syncthreads();
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

template <typename P>
static int run_global(const void* src, void* dst, size_t n, cudaStream_t st) {
    using In = typename P::In;
    using Out = typename P::Out;
    const unsigned grid = global_grid<In>(n, sm_count());
    const size_t bytes = sizeof(GlobalScratch) + static_cast<size_t>(grid) * sizeof(typename P::Acc);
    void* scratch = nullptr;
    if (bytes <= kStreamScratchBytes && stream_scratch(st, &scratch) == 0) {
        cudaGetLastError();  // a failed probe above must not be reported as a launch error
        launch_pdl(reduce_global_kernel<P>, grid, kGlobalThreads, 0, st, static_cast<const In*>(src), static_cast<Out*>(dst),
                   n, static_cast<GlobalScratch*>(scratch));
        return launch_status("reduce_global");
    }
    cudaGetLastError();
    cudaError_t e = pool_malloc(&scratch, bytes, st);
    if (e != cudaSuccess) return fail(static_cast<int>(e), "reduce_global: scratch allocation: %s", cudaGetErrorString(e));
    e = cudaMemsetAsync(scratch, 0, sizeof(GlobalScratch), st);
    if (e == cudaSuccess) {
        reduce_global_kernel<P><<<grid, kGlobalThreads, 0, st>>>(static_cast<const In*>(src), static_cast<Out*>(dst), n,
                                                                 static_cast<GlobalScratch*>(scratch));
        e = cudaGetLastError();
    }
    cudaError_t e2 = cudaFreeAsync(scratch, st);
    if (e != cudaSuccess) return fail(static_cast<int>(e), "reduce_global: %s", cudaGetErrorString(e));
    if (e2 != cudaSuccess) return fail(static_cast<int>(e2), "reduce_global: scratch release: %s", cudaGetErrorString(e2));
    return ok();
}

// Stream-ordered scratch for a split reduction: `groups` tickets (zeroed) and
// `partial_bytes` of partials, released on the stream after the launch.
template <typename Launch>
static int with_split_scratch(size_t groups, size_t partial_bytes, cudaStream_t st, const char* what, Launch&& launch) {
    const size_t tbytes = (groups * sizeof(unsigned int) + 255) / 256 * 256;
    void* mem = nullptr;
    cudaError_t e = pool_malloc(&mem, tbytes + partial_bytes, st);
    if (e != cudaSuccess) return fail(static_cast<int>(e), "%s: scratch allocation: %s", what, cudaGetErrorString(e));
    e = cudaMemsetAsync(mem, 0, tbytes, st);
    if (e == cudaSuccess) {
        SplitScratch sc{static_cast<unsigned int*>(mem), static_cast<uint8_t*>(mem) + tbytes};
        launch(sc);
        e = cudaGetLastError();
    }
    cudaError_t e2 = cudaFreeAsync(mem, st);
    if (e != cudaSuccess) return fail(static_cast<int>(e), "%s: %s", what, cudaGetErrorString(e));
    if (e2 != cudaSuccess) return fail(static_cast<int>(e2), "%s: scratch release: %s", what, cudaGetErrorString(e2));
    return ok();
}

template <typename P>
static int run_axis(const void* src, void* dst, size_t outer, size_t axis, size_t inner, cudaStream_t st) {
    using In = typename P::In;
    using Out = typename P::Out;
    using Acc = typename P::Acc;
    const In* s = static_cast<const In*>(src);
    Out* d = static_cast<Out*>(dst);
    const size_t sms = static_cast<size_t>(sm_count());
    const size_t cap = sms * 16;
    const size_t target = sms * 8;  // resident 256-thread CTAs
    if (inner == 1) {
        if (outer == 1) return run_global<P>(src, dst, axis, st);
        if (outer < sms && axis >= (size_t(1) << 16)) {
            // few long rows: split every row over S CTAs
            size_t S = (target + outer - 1) / outer;
            const size_t max_s = (axis + 256 * 8 * 4 - 1) / (256 * 8 * 4);  // at least four 32 KiB-ish units each
            if (S > max_s) S = max_s;
            if (S > 1) {
                return with_split_scratch(outer, outer * S * sizeof(Acc), st, "reduce_axis", [&](SplitScratch sc) {
                    const size_t grid = outer * S < target ? outer * S : target;
                    reduce_rows_split_kernel<P><<<static_cast<unsigned>(grid), 256, 0, st>>>(
                        s, d, outer, axis, static_cast<unsigned>(S), sc);
                });
            }
        }
        if (axis >= 2048) {
            const size_t grid = outer < (size_t(1) << 30) ? outer : (size_t(1) << 30);
            launch_pdl(reduce_rows_cta_kernel<P>, static_cast<unsigned>(grid), 256, 0, st, s, d, outer, axis);
        } else {
            size_t grid = (outer + 7) / 8;
            if (grid > cap) grid = cap;
            launch_pdl(reduce_rows_warp_kernel<P>, static_cast<unsigned>(grid), 256, 0, st, s, d, outer, axis);
        }
        return launch_status("reduce_axis");
    }
    constexpr int EV = 16 / sizeof(In);
    const bool vec = inner % EV == 0 && aligned16(src);
    const size_t tw = vec ? 32 * EV : 32;
    const size_t ctiles = (inner + tw - 1) / tw;
    const size_t tiles = outer * ctiles;
    // as many segments as keep every work item resident at once, about four
    // CTAs per SM (one more item than the GPU holds would run alone in a second
    // wave at a fraction of the bandwidth); on [8192, 8192] fp32 four per SM ran
    // 0.0459 ms against 0.0466 ms at eight (more, shorter segments) and 0.0537 ms
    // at two
    size_t G = target / 2 / tiles;
    const size_t max_g = (axis + 63) / 64;  // segments of at least 64 rows (8 per warp)
    if (G > max_g) G = max_g;
    if (G < 1) G = 1;
    const size_t seg = (axis + G - 1) / G;
    G = (axis + seg - 1) / seg;
    auto launch = [&](SplitScratch sc) {
        const size_t items = tiles * G;
        const size_t grid = items < cap ? items : cap;
        if (vec)
            reduce_cols_kernel<P, EV><<<static_cast<unsigned>(grid), 256, 0, st>>>(
                s, d, outer, axis, inner, ctiles, static_cast<unsigned>(G), seg, sc);
        else
            reduce_cols_kernel<P, 1><<<static_cast<unsigned>(grid), 256, 0, st>>>(
                s, d, outer, axis, inner, ctiles, static_cast<unsigned>(G), seg, sc);
    };
    if (G == 1) {
        launch(SplitScratch{nullptr, nullptr});
        return launch_status("reduce_axis");
    }
    return with_split_scratch(tiles, G * outer * inner * sizeof(Acc), st, "reduce_axis", launch);
}

// ---------------------------------------------------------------- reduce across GPUs

// Status word of the cross-GPU reduce (a peer that never delivered its partial
// within the wait limit): read and cleared by bee_b200_device_status.
__device__ int g_allranks_status = 0;

int allranks_status_take(int* code) {
    int zero = 0;
    cudaError_t e = cudaMemcpyFromSymbol(code, g_allranks_status, sizeof(int));
    if (e == cudaSuccess) e = cudaMemcpyToSymbol(g_allranks_status, &zero, sizeof(int));
    return static_cast<int>(e);
}

constexpr int kMaxRanks = 8;
struct PeerSlots {
    unsigned long long* slot[kMaxRanks];  // rank r's receive array (world words), mapped in this process
};

// Relaxed system-scope accesses: the tag and the value travel in one 64-bit
// word, so a reader that sees the tag has the value; no fence is needed.
__device__ __forceinline__ void st_relaxed_sys(unsigned long long* p, unsigned long long v) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_relaxed_sys(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// The global reduce of reduce_global_kernel, then, in the last CTA, the
// exchange with the other GPUs of the job: thread 0 stores (tag, partial) as
// one 64-bit word into slot `rank` of bank tag & 1 of every rank's receive
// array (two banks of `world` words; peer stores
// over NVLink), waits until its own array holds this call's tag in every slot
// (bounded by wait_ns: on expiry it records the status and writes its local
// partial), and folds the world partials in rank order, so every rank writes
// the same bits.  32-bit element types only (the value and the tag share one
// word, so a reader never sees a torn update).
template <typename P>
__global__ void __launch_bounds__(kGlobalThreads) reduce_allranks_kernel(const typename P::In* __restrict__ src,
                                                                         typename P::Out* __restrict__ dst, size_t n,
                                                                         GlobalScratch* scratch, PeerSlots peers,
                                                                         int world, int rank, unsigned int tag,
                                                                         unsigned long long wait_ns) {
    using In = typename P::In;
    using Acc = typename P::Acc;
    static_assert(sizeof(Acc) == 4, "32-bit partials");
    constexpr size_t E = 16 / sizeof(In);
    constexpr size_t UNIT = static_cast<size_t>(kGlobalThreads) * kGlobalUnroll;
    __shared__ Acc smem[32];
    __shared__ bool last;
    Acc* partials = reinterpret_cast<Acc*>(scratch + 1);
    const unsigned tid = threadIdx.x;
    Acc acc = P::identity();
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
    acc = block_reduce<P>(acc, smem);
    if (tid == 0) {
        partials[blockIdx.x] = acc;
        __threadfence();
        last = atomicAdd(&scratch->ticket, 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (!last) return;
    __threadfence();
    Acc r = P::identity();
    for (unsigned i = tid; i < gridDim.x; i += kGlobalThreads)
        r = P::combine(r, *reinterpret_cast<volatile Acc*>(partials + i));
    r = block_reduce<P>(r, smem);
    if (tid == 0) {
        scratch->ticket = 0;
        uint32_t bits;
        memcpy(&bits, &r, 4);
        const unsigned long long word = (static_cast<unsigned long long>(tag) << 32) | bits;
        // two banks by tag parity: a rank that finished this call may already store the next
        // call's word while a slower rank still reads this one
        const int bank = static_cast<int>(tag & 1u) * world;
        for (int p = 0; p < world; ++p) st_relaxed_sys(peers.slot[p] + bank + rank, word);
        Acc total = P::identity();
        const unsigned long long* mine = peers.slot[rank] + bank;
        const unsigned long long t0 = sm100::globaltimer_ns();
        bool ok = true;
        for (int s = 0; s < world && ok; ++s) {
            unsigned long long w = ld_relaxed_sys(mine + s);
            for (uint32_t i = 0; static_cast<unsigned int>(w >> 32) != tag; ++i) {
                if ((i & 63u) == 63u && sm100::globaltimer_ns() - t0 > wait_ns) {
                    atomicCAS(&g_allranks_status, 0, 40 + s);
                    ok = false;
                    break;
                }
                __nanosleep(64);  // poll gently: the wait is normally a few microseconds
                w = ld_relaxed_sys(mine + s);
            }
            if (ok) {
                const uint32_t vb = static_cast<uint32_t>(w);
                Acc v;
                memcpy(&v, &vb, 4);
                total = P::combine(total, v);
            }
        }
        *dst = ok ? P::finish(total, n) : P::finish(r, n);
    }
}

template <typename P>
static int run_allranks(const void* src, void* dst, size_t n, const PeerSlots& peers, int world, int rank,
                        unsigned int tag, unsigned long long wait_ns, cudaStream_t st) {
    using In = typename P::In;
    using Out = typename P::Out;
    const unsigned grid = global_grid<In>(n, sm_count());
    const size_t bytes = sizeof(GlobalScratch) + static_cast<size_t>(grid) * sizeof(typename P::Acc);
    void* scratch = nullptr;
    if (bytes > kStreamScratchBytes || stream_scratch(st, &scratch) != 0)
        return fail(cudaErrorInvalidValue, "reduce_global_allranks: no per-stream scratch (stream capture?)");
    cudaGetLastError();
    reduce_allranks_kernel<P><<<grid, kGlobalThreads, 0, st>>>(static_cast<const In*>(src), static_cast<Out*>(dst), n,
                                                               static_cast<GlobalScratch*>(scratch), peers, world,
                                                               rank, tag, wait_ns);
    return launch_status("reduce_global_allranks");
}

template <typename T>
static int dispatch_global(int op, const void* src, void* dst, size_t n, cudaStream_t st) {
    switch (op) {
    case RED_SUM: if constexpr (!std::is_same_v<T, uint8_t>) return run_global<ElemRed<RED_SUM, T>>(src, dst, n, st); break;
    case RED_PROD: if constexpr (!std::is_same_v<T, uint8_t>) return run_global<ElemRed<RED_PROD, T>>(src, dst, n, st); break;
    case RED_MIN: return run_global<ElemRed<RED_MIN, T>>(src, dst, n, st);
    case RED_MAX: return run_global<ElemRed<RED_MAX, T>>(src, dst, n, st);
    default: return fail(cudaErrorInvalidValue, "reduce_global: unknown op code %d", op);
    }
    return fail(cudaErrorInvalidValue, "reduce_global: op %d does not support U8", op);
}

template <typename T>
static int dispatch_axis(int op, const void* src, void* dst, size_t outer, size_t axis, size_t inner, cudaStream_t st) {
    switch (op) {
    case RED_SUM: if constexpr (!std::is_same_v<T, uint8_t>) return run_axis<ElemRed<RED_SUM, T>>(src, dst, outer, axis, inner, st); break;
    case RED_PROD: if constexpr (!std::is_same_v<T, uint8_t>) return run_axis<ElemRed<RED_PROD, T>>(src, dst, outer, axis, inner, st); break;
    case RED_MIN: return run_axis<ElemRed<RED_MIN, T>>(src, dst, outer, axis, inner, st);
    case RED_MAX: return run_axis<ElemRed<RED_MAX, T>>(src, dst, outer, axis, inner, st);
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

int bee_b200_reduce_mean_int(int dt, const void* src, double* dst, size_t outer, size_t axis, size_t inner,
                             bee_b200_stream_t stream) {
    if (outer == 0 || axis == 0 || inner == 0) return fail(cudaErrorInvalidValue, "reduce_mean_int: empty extent");
    if (!src || !dst) return fail(cudaErrorInvalidValue, "reduce_mean_int: null pointer");
    cudaStream_t st = as_stream(stream);
    switch (dt) {
    case DT_I32: return run_axis<MeanInt<int32_t>>(src, dst, outer, axis, inner, st);
    case DT_I64: return run_axis<MeanInt<int64_t>>(src, dst, outer, axis, inner, st);
    default: return fail(cudaErrorInvalidValue, "reduce_mean_int: dtype %d is not I32 or I64", dt);
    }
}

int bee_b200_reduce_global_allranks(int op, int dt, const void* src, size_t n, void* dst, void* const* recv_slots,
                                    int world, int rank, unsigned int tag, unsigned long long wait_ns,
                                    bee_b200_stream_t stream) {
    if (n == 0) return fail(cudaErrorInvalidValue, "reduce_global_allranks: empty input");
    if (!src || !dst || !recv_slots) return fail(cudaErrorInvalidValue, "reduce_global_allranks: null pointer");
    if (world < 1 || world > kMaxRanks || rank < 0 || rank >= world)
        return fail(cudaErrorInvalidValue, "reduce_global_allranks: rank %d / world %d out of range (world <= %d)", rank,
                    world, kMaxRanks);
    if (tag == 0) return fail(cudaErrorInvalidValue, "reduce_global_allranks: tag 0 is reserved (fresh slots read 0)");
    PeerSlots peers{};
    for (int r = 0; r < world; ++r) {
        if (!recv_slots[r] || (reinterpret_cast<uintptr_t>(recv_slots[r]) & 7u) != 0)
            return fail(cudaErrorInvalidValue, "reduce_global_allranks: receive array %d missing or misaligned", r);
        peers.slot[r] = static_cast<unsigned long long*>(recv_slots[r]);
    }
    cudaStream_t st = as_stream(stream);
    switch (dt) {
    case DT_I32:
        switch (op) {
        case RED_SUM: return run_allranks<ElemRed<RED_SUM, int32_t>>(src, dst, n, peers, world, rank, tag, wait_ns, st);
        case RED_MIN: return run_allranks<ElemRed<RED_MIN, int32_t>>(src, dst, n, peers, world, rank, tag, wait_ns, st);
        case RED_MAX: return run_allranks<ElemRed<RED_MAX, int32_t>>(src, dst, n, peers, world, rank, tag, wait_ns, st);
        case RED_PROD: return run_allranks<ElemRed<RED_PROD, int32_t>>(src, dst, n, peers, world, rank, tag, wait_ns, st);
        default: break;
        }
        break;
    case DT_F32:
        switch (op) {
        case RED_SUM: return run_allranks<ElemRed<RED_SUM, float>>(src, dst, n, peers, world, rank, tag, wait_ns, st);
        case RED_MIN: return run_allranks<ElemRed<RED_MIN, float>>(src, dst, n, peers, world, rank, tag, wait_ns, st);
        case RED_MAX: return run_allranks<ElemRed<RED_MAX, float>>(src, dst, n, peers, world, rank, tag, wait_ns, st);
        case RED_PROD: return run_allranks<ElemRed<RED_PROD, float>>(src, dst, n, peers, world, rank, tag, wait_ns, st);
        default: break;
        }
        break;
    default:
        return fail(cudaErrorInvalidValue, "reduce_global_allranks: dtype %d unsupported (I32 or F32)", dt);
    }
    return fail(cudaErrorInvalidValue, "reduce_global_allranks: unknown op code %d", op);
}

}  // extern "C"
