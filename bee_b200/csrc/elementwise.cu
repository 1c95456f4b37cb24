// Elementwise binary / unary / cast / scale kernels (HBM-bound).
//
// Replaces the reference's K4/K5/K6/K9 kernels (Bee/CUDA/Ops/ElementWise.cu:94-226,
// Bee/CUDA/Ops/Cast.cu:29-45, Bee/CUDA/Ops/Reduce.cu:188-193).  Design for B200:
// every thread moves 16-byte vectors, UNROLL independent vectors are loaded
// before any is used (enough bytes in flight to cover HBM latency with
// 148 SMs x 2048 threads), loads/stores are streaming (evict-first), and the
// grid is a multiple of the SM count with a grid-stride loop.  The scalar tail
// (n not a multiple of the vector width) is handled by block 0 in the same
// launch, so one op is one kernel.
#include <cmath>

#include "common.cuh"

namespace bee_b200 {

// bf16 / f16 storage tags: raw bits, arithmetic in fp32, RNE on store.
struct bf16_t {
    uint16_t bits;
};
struct f16_t {
    uint16_t bits;
};

template <typename S> struct Compute { using T = S; };
template <> struct Compute<uint8_t> { using T = int; };
template <> struct Compute<bf16_t> { using T = float; };
template <> struct Compute<f16_t> { using T = float; };

template <typename S> __device__ __forceinline__ typename Compute<S>::T to_c(S s) {
    return static_cast<typename Compute<S>::T>(s);
}
template <> __device__ __forceinline__ float to_c<bf16_t>(bf16_t s) {
    return __uint_as_float(static_cast<uint32_t>(s.bits) << 16);
}
template <> __device__ __forceinline__ float to_c<f16_t>(f16_t s) { return __half2float(__ushort_as_half(s.bits)); }
template <typename S> __device__ __forceinline__ S from_c(typename Compute<S>::T c) { return static_cast<S>(c); }
template <> __device__ __forceinline__ bf16_t from_c<bf16_t>(float c) {
    __nv_bfloat16 h = __float2bfloat16_rn(c);
    return bf16_t{*reinterpret_cast<uint16_t*>(&h)};
}
template <> __device__ __forceinline__ f16_t from_c<f16_t>(float c) { return f16_t{__half_as_ushort(__float2half_rn(c))}; }

template <int OP, typename C> __device__ __forceinline__ C bin(C a, C b) {
    if constexpr (OP == OP_ADD) return a + b;
    else if constexpr (OP == OP_SUB) return a - b;
    else if constexpr (OP == OP_MUL) return a * b;
    else return a / b;
}

template <int OP, typename C> __device__ __forceinline__ C una(C a) {
    if constexpr (OP == OP_NEG) return -a;
    else if constexpr (OP == OP_ABS) return a < C(0) ? -a : a;
    else if constexpr (OP == OP_SQRT) return sqrt(a);
    else if constexpr (OP == OP_EXP) return exp(a);
    else return log(a);
}

template <typename S> union Pack16 {
    uint4 v;
    S s[16 / sizeof(S)];
};

template <typename S, int OP> __device__ __forceinline__ uint4 vec_bin(uint4 x, uint4 y) {
    Pack16<S> a, b, o;
    a.v = x;
    b.v = y;
#pragma unroll
    for (int k = 0; k < int(16 / sizeof(S)); ++k) o.s[k] = from_c<S>(bin<OP>(to_c(a.s[k]), to_c(b.s[k])));
    return o.v;
}

template <typename S, int OP> __device__ __forceinline__ uint4 vec_una(uint4 x) {
    Pack16<S> a, o;
    a.v = x;
#pragma unroll
    for (int k = 0; k < int(16 / sizeof(S)); ++k) o.s[k] = from_c<S>(una<OP>(to_c(a.s[k])));
    return o.v;
}

constexpr int kThreads = 256;
constexpr int kUnroll = 4;

template <typename S, int OP>
__global__ void __launch_bounds__(kThreads) binary_kernel(const S* __restrict__ a, const S* __restrict__ b,
                                                          S* __restrict__ out, size_t n) {
    constexpr size_t E = 16 / sizeof(S);
    const size_t nvec = n / E;
    const uint4* va = reinterpret_cast<const uint4*>(a);
    const uint4* vb = reinterpret_cast<const uint4*>(b);
    uint4* vo = reinterpret_cast<uint4*>(out);
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    pdl_wait();
    for (; i + (kUnroll - 1) * stride < nvec; i += kUnroll * stride) {
        uint4 x[kUnroll], y[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            x[u] = ld_stream_u4(va + i + u * stride);
            y[u] = ld_stream_u4(vb + i + u * stride);
        }
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) st_stream_u4(vo + i + u * stride, vec_bin<S, OP>(x[u], y[u]));
    }
    pdl_trigger();
    for (; i < nvec; i += stride) st_stream_u4(vo + i, vec_bin<S, OP>(ld_stream_u4(va + i), ld_stream_u4(vb + i)));
    if (blockIdx.x == 0)
        for (size_t j = nvec * E + threadIdx.x; j < n; j += blockDim.x) out[j] = from_c<S>(bin<OP>(to_c(a[j]), to_c(b[j])));
}

// Fallback for buffers that are not 16-byte aligned: one element per thread.
template <typename S, int OP>
__global__ void __launch_bounds__(kThreads) binary_scalar_kernel(const S* __restrict__ a, const S* __restrict__ b,
                                                                 S* __restrict__ out, size_t n) {
    pdl_wait();
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride)
        out[i] = from_c<S>(bin<OP>(to_c(a[i]), to_c(b[i])));
}

// Broadcasting / strided binary op: out (contiguous, viewed [rows, L]) =
// a op b where each operand is a strided view of out's shape (stride 0 on
// broadcast dims).  Work item = one 16-byte chunk of an output row; an operand
// whose innermost stride is 1 is read in 16-byte vectors when aligned, one with
// innermost stride 0 is read once per chunk, any other stride element by element.
constexpr int kMaxBcastDims = 8;
struct BcastDims {
    int nd;                                // outer dims (all but the innermost)
    long long shape[kMaxBcastDims];
    long long sa[kMaxBcastDims], sb[kMaxBcastDims];
};

template <typename S>
__device__ __forceinline__ void load_chunk(const S* p, long long inner, bool vec, int cnt, Pack16<S>& v) {
    constexpr int E = 16 / sizeof(S);
    if (inner == 1 && vec && cnt == E) {
        v.v = __ldcs(reinterpret_cast<const uint4*>(p));
    } else if (inner == 0) {
        const S x = p[0];
#pragma unroll
        for (int k = 0; k < E; ++k) v.s[k] = x;
    } else {
#pragma unroll
        for (int k = 0; k < E; ++k) v.s[k] = k < cnt ? p[k * inner] : p[0];
    }
}

template <typename S, int OP>
__device__ __forceinline__ void strided_chunk(const S* __restrict__ a, const S* __restrict__ b, S* __restrict__ o,
                                              long long c, long long L, long long ia, long long ib, int a_vec,
                                              int b_vec, int o_vec) {
    constexpr int E = 16 / sizeof(S);
    const int cnt = static_cast<int>(L - c < E ? L - c : E);
    Pack16<S> va, vb, vo;
    load_chunk<S>(a + c * ia, ia, a_vec, cnt, va);
    load_chunk<S>(b + c * ib, ib, b_vec, cnt, vb);
#pragma unroll
    for (int k = 0; k < E; ++k) vo.s[k] = from_c<S>(bin<OP>(to_c(va.s[k]), to_c(vb.s[k])));
    if (o_vec && cnt == E) {
        __stcs(reinterpret_cast<uint4*>(o + c), vo.v);
    } else {
#pragma unroll
        for (int k = 0; k < E; ++k)
            if (k < cnt) o[c + k] = vo.s[k];
    }
}

// ROW_MODE (rows of at least 4 KiB): one CTA per output row at a time, the two
// operand row offsets computed once per row, UNROLL chunks per thread with
// their loads issued first.  Otherwise a work item is one chunk of a row.
template <typename S, int OP, bool ROW_MODE>
__global__ void __launch_bounds__(kThreads) binary_strided_kernel(const S* __restrict__ a, const S* __restrict__ b,
                                                                  S* __restrict__ out, long long rows, long long L,
                                                                  BcastDims d, long long ia, long long ib, int a_vec,
                                                                  int b_vec, int o_vec) {
    constexpr int E = 16 / sizeof(S);
    const long long per_row = (L + E - 1) / E;
    pdl_wait();
    if constexpr (ROW_MODE) {
        for (long long row = blockIdx.x; row < rows; row += gridDim.x) {
            if (row + gridDim.x >= rows) pdl_trigger();  // this CTA's last row
            long long r = row, oa = 0, ob = 0;
            for (int k = d.nd - 1; k >= 0; --k) {
                const long long x = r % d.shape[k];
                r /= d.shape[k];
                oa += x * d.sa[k];
                ob += x * d.sb[k];
            }
            const S* ar = a + oa;
            const S* br = b + ob;
            S* orow = out + row * L;
            long long j = threadIdx.x;
            for (; j + (kUnroll - 1) * kThreads < per_row; j += kUnroll * kThreads) {
                Pack16<S> va[kUnroll], vb[kUnroll];
#pragma unroll
                for (int u = 0; u < kUnroll; ++u) {
                    const long long c = (j + u * kThreads) * E;
                    load_chunk<S>(ar + c * ia, ia, a_vec, E, va[u]);
                    load_chunk<S>(br + c * ib, ib, b_vec, E, vb[u]);
                }
#pragma unroll
                for (int u = 0; u < kUnroll; ++u) {
                    Pack16<S> vo;
#pragma unroll
                    for (int k = 0; k < E; ++k) vo.s[k] = from_c<S>(bin<OP>(to_c(va[u].s[k]), to_c(vb[u].s[k])));
                    const long long c = (j + u * kThreads) * E;
                    if (o_vec) {
                        __stcs(reinterpret_cast<uint4*>(orow + c), vo.v);
                    } else {
#pragma unroll
                        for (int k = 0; k < E; ++k) orow[c + k] = vo.s[k];
                    }
                }
            }
            for (; j < per_row; j += kThreads) strided_chunk<S, OP>(ar, br, orow, j * E, L, ia, ib, a_vec, b_vec, o_vec);
        }
    } else {
        const long long items = rows * per_row;
        const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
        for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < items; i += stride) {
            long long r = i / per_row;
            const long long c = (i - r * per_row) * E;
            const long long orow = r;
            long long oa = 0, ob = 0;
            for (int k = d.nd - 1; k >= 0; --k) {
                const long long x = r % d.shape[k];
                r /= d.shape[k];
                oa += x * d.sa[k];
                ob += x * d.sb[k];
            }
            strided_chunk<S, OP>(a + oa, b + ob, out + orow * L, c, L, ia, ib, a_vec, b_vec, o_vec);
        }
    }
}

template <typename S, int OP>
__global__ void __launch_bounds__(kThreads) unary_kernel(const S* __restrict__ a, S* __restrict__ out, size_t n,
                                                         int vectorised) {
    pdl_wait();
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (!vectorised) {
        for (; i < n; i += stride) out[i] = from_c<S>(una<OP>(to_c(a[i])));
        return;
    }
    constexpr size_t E = 16 / sizeof(S);
    const size_t nvec = n / E;
    const uint4* va = reinterpret_cast<const uint4*>(a);
    uint4* vo = reinterpret_cast<uint4*>(out);
    for (; i + (kUnroll - 1) * stride < nvec; i += kUnroll * stride) {
        uint4 x[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) x[u] = ld_stream_u4(va + i + u * stride);
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) st_stream_u4(vo + i + u * stride, vec_una<S, OP>(x[u]));
    }
    for (; i < nvec; i += stride) st_stream_u4(vo + i, vec_una<S, OP>(ld_stream_u4(va + i)));
    if (blockIdx.x == 0)
        for (size_t j = nvec * E + threadIdx.x; j < n; j += blockDim.x) out[j] = from_c<S>(una<OP>(to_c(a[j])));
}

// fp32 -> bf16, round to nearest even: 32 bytes in, 16 bytes out per vector step.
__global__ void __launch_bounds__(kThreads) cast_f32_bf16_kernel(const float* __restrict__ src,
                                                                  uint16_t* __restrict__ dst, size_t n) {
    const size_t nvec = n / 8;
    const float4* vs = reinterpret_cast<const float4*>(src);
    uint4* vd = reinterpret_cast<uint4*>(dst);
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    pdl_wait();
    for (; i + (kUnroll - 1) * stride < nvec; i += kUnroll * stride) {
        float4 x[kUnroll][2];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            x[u][0] = ld_stream(vs + 2 * (i + u * stride));
            x[u][1] = ld_stream(vs + 2 * (i + u * stride) + 1);
        }
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            uint4 o;
            o.x = pack_bf16x2(x[u][0].x, x[u][0].y);
            o.y = pack_bf16x2(x[u][0].z, x[u][0].w);
            o.z = pack_bf16x2(x[u][1].x, x[u][1].y);
            o.w = pack_bf16x2(x[u][1].z, x[u][1].w);
            st_stream_u4(vd + i + u * stride, o);
        }
    }
    pdl_trigger();
    for (; i < nvec; i += stride) {
        float4 p = ld_stream(vs + 2 * i), q = ld_stream(vs + 2 * i + 1);
        uint4 o;
        o.x = pack_bf16x2(p.x, p.y);
        o.y = pack_bf16x2(p.z, p.w);
        o.z = pack_bf16x2(q.x, q.y);
        o.w = pack_bf16x2(q.z, q.w);
        st_stream_u4(vd + i, o);
    }
    if (blockIdx.x == 0)
        for (size_t j = nvec * 8 + threadIdx.x; j < n; j += blockDim.x) {
            __nv_bfloat16 h = __float2bfloat16_rn(src[j]);
            dst[j] = *reinterpret_cast<uint16_t*>(&h);
        }
}

// bf16 -> fp32 (exact): 16 bytes in, 32 bytes out per vector step.
__global__ void __launch_bounds__(kThreads) cast_bf16_f32_kernel(const uint16_t* __restrict__ src,
                                                                  float* __restrict__ dst, size_t n) {
    pdl_wait();
    const size_t nvec = n / 8;
    const uint4* vs = reinterpret_cast<const uint4*>(src);
    float4* vd = reinterpret_cast<float4*>(dst);
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < nvec; i += stride) {
        uint4 w = ld_stream_u4(vs + i);
        st_stream(vd + 2 * i, make_float4(bf16_lo(w.x), bf16_hi(w.x), bf16_lo(w.y), bf16_hi(w.y)));
        st_stream(vd + 2 * i + 1, make_float4(bf16_lo(w.z), bf16_hi(w.z), bf16_lo(w.w), bf16_hi(w.w)));
    }
    if (blockIdx.x == 0)
        for (size_t j = nvec * 8 + threadIdx.x; j < n; j += blockDim.x)
            dst[j] = __uint_as_float(static_cast<uint32_t>(src[j]) << 16);
}

// Generic element-by-element cast (static_cast semantics, ->Bool is x != 0).
template <typename Si, typename So>
__global__ void __launch_bounds__(kThreads) cast_kernel(const Si* __restrict__ src, So* __restrict__ dst, size_t n) {
    pdl_wait();
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) {
        auto c = to_c(src[i]);
        if constexpr (std::is_same_v<So, bool>) dst[i] = (c != decltype(c)(0));
        else if constexpr (std::is_same_v<So, bf16_t>) dst[i] = from_c<bf16_t>(static_cast<float>(c));
        else if constexpr (std::is_same_v<So, f16_t> && std::is_same_v<Si, double>)
            dst[i] = f16_t{__half_as_ushort(__double2half(c))};  // one rounding from double
        else if constexpr (std::is_same_v<So, f16_t>) dst[i] = from_c<f16_t>(static_cast<float>(c));
        else dst[i] = static_cast<So>(c);
    }
}

template <typename T>
__global__ void __launch_bounds__(kThreads) scale_kernel(T* __restrict__ buf, T factor, size_t n) {
    pdl_wait();
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) buf[i] *= factor;
}

// Grid for a grid-stride kernel over `work` items: never more than 8 resident
// 256-thread CTAs per SM (2048 threads, full occupancy), never more CTAs than
// items need.
static unsigned grid_for(size_t work) {
    size_t cap = static_cast<size_t>(sm_count()) * 8;
    size_t need = (work + kThreads - 1) / kThreads;
    if (need == 0) need = 1;
    return static_cast<unsigned>(need < cap ? need : cap);
}

template <typename S, int OP>
static void launch_binary(const void* a, const void* b, void* out, size_t n, cudaStream_t st) {
    const S* pa = static_cast<const S*>(a);
    const S* pb = static_cast<const S*>(b);
    S* po = static_cast<S*>(out);
    if (aligned16(a) && aligned16(b) && aligned16(out))
        launch_pdl(binary_kernel<S, OP>, grid_for((n * sizeof(S) / 16 + kUnroll - 1) / kUnroll), kThreads, 0, st, pa, pb,
                   po, n);
    else
        launch_pdl(binary_scalar_kernel<S, OP>, grid_for(n), kThreads, 0, st, pa, pb, po, n);
}

template <typename S>
static int dispatch_binary_op(int op, const void* a, const void* b, void* out, size_t n, cudaStream_t st) {
    switch (op) {
    case OP_ADD: launch_binary<S, OP_ADD>(a, b, out, n, st); break;
    case OP_SUB: launch_binary<S, OP_SUB>(a, b, out, n, st); break;
    case OP_MUL: launch_binary<S, OP_MUL>(a, b, out, n, st); break;
    case OP_DIV: launch_binary<S, OP_DIV>(a, b, out, n, st); break;
    default: return fail(cudaErrorInvalidValue, "ew_binary: unknown op code %d", op);
    }
    return launch_status("ew_binary");
}

struct StridedOperands {
    int nd;  // simplified dims, innermost last
    long long shape[kMaxBcastDims], sa[kMaxBcastDims], sb[kMaxBcastDims];
};

template <typename S, int OP>
static void launch_binary_strided(const void* a, const void* b, void* out, const StridedOperands& v, cudaStream_t st) {
    constexpr int E = 16 / sizeof(S);
    const long long L = v.shape[v.nd - 1];
    long long rows = 1;
    BcastDims d{};
    d.nd = v.nd - 1;
    for (int k = 0; k < v.nd - 1; ++k) {
        d.shape[k] = v.shape[k];
        d.sa[k] = v.sa[k];
        d.sb[k] = v.sb[k];
        rows *= v.shape[k];
    }
    const long long ia = v.sa[v.nd - 1], ib = v.sb[v.nd - 1];
    bool a_vec = aligned16(a), b_vec = aligned16(b);
    for (int k = 0; k < v.nd - 1; ++k) {
        a_vec = a_vec && (v.sa[k] * static_cast<long long>(sizeof(S))) % 16 == 0;
        b_vec = b_vec && (v.sb[k] * static_cast<long long>(sizeof(S))) % 16 == 0;
    }
    const int o_vec = aligned16(out) && (L * static_cast<long long>(sizeof(S))) % 16 == 0;
    const long long per_row = (L + E - 1) / E;
    if (per_row >= 256) {
        const long long cap = static_cast<long long>(sm_count()) * 8;
        launch_pdl(binary_strided_kernel<S, OP, true>, static_cast<unsigned>(rows < cap ? rows : cap), kThreads, 0, st,
                   static_cast<const S*>(a), static_cast<const S*>(b), static_cast<S*>(out), rows, L, d, ia, ib,
                   a_vec ? 1 : 0, b_vec ? 1 : 0, o_vec);
    } else {
        launch_pdl(binary_strided_kernel<S, OP, false>, grid_for(static_cast<size_t>(rows * per_row)), kThreads, 0, st,
                   static_cast<const S*>(a), static_cast<const S*>(b), static_cast<S*>(out), rows, L, d, ia, ib,
                   a_vec ? 1 : 0, b_vec ? 1 : 0, o_vec);
    }
}

template <typename S>
static int dispatch_binary_strided(int op, const void* a, const void* b, void* out, const StridedOperands& v,
                                   cudaStream_t st) {
    switch (op) {
    case OP_ADD: launch_binary_strided<S, OP_ADD>(a, b, out, v, st); break;
    case OP_SUB: launch_binary_strided<S, OP_SUB>(a, b, out, v, st); break;
    case OP_MUL: launch_binary_strided<S, OP_MUL>(a, b, out, v, st); break;
    case OP_DIV: launch_binary_strided<S, OP_DIV>(a, b, out, v, st); break;
    default: return fail(cudaErrorInvalidValue, "ew_binary_strided: unknown op code %d", op);
    }
    return launch_status("ew_binary_strided");
}

template <typename S, int OP>
static void launch_unary(const void* a, void* out, size_t n, cudaStream_t st) {
    int vec = aligned16(a) && aligned16(out);
    size_t work = vec ? (n * sizeof(S) / 16 + kUnroll - 1) / kUnroll : n;
    launch_pdl(unary_kernel<S, OP>, grid_for(work), kThreads, 0, st, static_cast<const S*>(a), static_cast<S*>(out), n, vec);
}

template <typename S>
static int dispatch_unary_op(int op, bool fp, const void* a, void* out, size_t n, cudaStream_t st) {
    switch (op) {
    case OP_NEG: launch_unary<S, OP_NEG>(a, out, n, st); break;
    case OP_ABS: launch_unary<S, OP_ABS>(a, out, n, st); break;
    case OP_SQRT:
    case OP_EXP:
    case OP_LOG:
        if (!fp) return fail(cudaErrorInvalidValue, "ew_unary: op %d needs a floating dtype", op);
        if constexpr (std::is_floating_point_v<typename Compute<S>::T>) {
            if (op == OP_SQRT) launch_unary<S, OP_SQRT>(a, out, n, st);
            else if (op == OP_EXP) launch_unary<S, OP_EXP>(a, out, n, st);
            else launch_unary<S, OP_LOG>(a, out, n, st);
        }
        break;
    default: return fail(cudaErrorInvalidValue, "ew_unary: unknown op code %d", op);
    }
    return launch_status("ew_unary");
}

template <typename Si>
static int cast_from(int dst_dt, const void* src, void* dst, size_t n, cudaStream_t st) {
    const Si* s = static_cast<const Si*>(src);
    unsigned g = grid_for(n);
    switch (dst_dt) {
    case DT_BOOL: launch_pdl(cast_kernel<Si, bool>, g, kThreads, 0, st, s, static_cast<bool*>(dst), n); break;
    case DT_U8: launch_pdl(cast_kernel<Si, uint8_t>, g, kThreads, 0, st, s, static_cast<uint8_t*>(dst), n); break;
    case DT_I32: launch_pdl(cast_kernel<Si, int32_t>, g, kThreads, 0, st, s, static_cast<int32_t*>(dst), n); break;
    case DT_I64: launch_pdl(cast_kernel<Si, int64_t>, g, kThreads, 0, st, s, static_cast<int64_t*>(dst), n); break;
    case DT_F32: launch_pdl(cast_kernel<Si, float>, g, kThreads, 0, st, s, static_cast<float*>(dst), n); break;
    case DT_F64: launch_pdl(cast_kernel<Si, double>, g, kThreads, 0, st, s, static_cast<double*>(dst), n); break;
    case DT_BF16: launch_pdl(cast_kernel<Si, bf16_t>, g, kThreads, 0, st, s, static_cast<bf16_t*>(dst), n); break;
    case DT_F16: launch_pdl(cast_kernel<Si, f16_t>, g, kThreads, 0, st, s, static_cast<f16_t*>(dst), n); break;
    default: return fail(cudaErrorInvalidValue, "ew_cast: unsupported destination dtype %d", dst_dt);
    }
    return launch_status("ew_cast");
}

}  // namespace bee_b200

using namespace bee_b200;

extern "C" {

int bee_b200_ew_binary(int op, int dt, const void* a, const void* b, void* out, size_t n, bee_b200_stream_t stream) {
    if (n == 0) return ok();
    if (!a || !b || !out) return fail(cudaErrorInvalidValue, "ew_binary: null pointer");
    cudaStream_t st = as_stream(stream);
    switch (dt) {
    case DT_U8: return dispatch_binary_op<uint8_t>(op, a, b, out, n, st);
    case DT_I32: return dispatch_binary_op<int32_t>(op, a, b, out, n, st);
    case DT_I64: return dispatch_binary_op<int64_t>(op, a, b, out, n, st);
    case DT_F32: return dispatch_binary_op<float>(op, a, b, out, n, st);
    case DT_F64: return dispatch_binary_op<double>(op, a, b, out, n, st);
    case DT_BF16: return dispatch_binary_op<bf16_t>(op, a, b, out, n, st);
    case DT_F16: return dispatch_binary_op<f16_t>(op, a, b, out, n, st);
    default: return fail(cudaErrorInvalidValue, "ew_binary: unsupported dtype %d", dt);
    }
}

int bee_b200_ew_binary_strided(int op, int dt, int ndim, const int64_t* shape, const void* a, const int64_t* a_strides,
                               const void* b, const int64_t* b_strides, void* out, bee_b200_stream_t stream) {
    if (ndim < 0 || ndim > kMaxBcastDims)
        return fail(cudaErrorInvalidValue, "ew_binary_strided: ndim %d outside [0, %d]", ndim, kMaxBcastDims);
    if (ndim > 0 && (!shape || !a_strides || !b_strides))
        return fail(cudaErrorInvalidValue, "ew_binary_strided: null shape or strides");
    long long n = 1;
    for (int k = 0; k < ndim; ++k) {
        if (shape[k] < 0) return fail(cudaErrorInvalidValue, "ew_binary_strided: negative extent in dim %d", k);
        n *= shape[k];
        if (n > (1LL << 46)) return fail(cudaErrorInvalidValue, "ew_binary_strided: too many elements");
    }
    if (n == 0) return ok();
    if (!a || !b || !out) return fail(cudaErrorInvalidValue, "ew_binary_strided: null pointer");
    // simplify: drop extent-1 dims, merge neighbours contiguous with each other in both operands
    StridedOperands v{};
    for (int k = 0; k < ndim; ++k) {
        if (shape[k] == 1) continue;
        if (v.nd > 0 && v.sa[v.nd - 1] == a_strides[k] * shape[k] && v.sb[v.nd - 1] == b_strides[k] * shape[k]) {
            v.shape[v.nd - 1] *= shape[k];
            v.sa[v.nd - 1] = a_strides[k];
            v.sb[v.nd - 1] = b_strides[k];
        } else {
            v.shape[v.nd] = shape[k];
            v.sa[v.nd] = a_strides[k];
            v.sb[v.nd] = b_strides[k];
            ++v.nd;
        }
    }
    if (v.nd == 0) {
        v.nd = 1;
        v.shape[0] = 1;
        v.sa[0] = v.sb[0] = 1;
    }
    if (v.nd == 1 && v.sa[0] == 1 && v.sb[0] == 1) return bee_b200_ew_binary(op, dt, a, b, out, static_cast<size_t>(n), stream);
    cudaStream_t st = as_stream(stream);
    switch (dt) {
    case DT_U8: return dispatch_binary_strided<uint8_t>(op, a, b, out, v, st);
    case DT_I32: return dispatch_binary_strided<int32_t>(op, a, b, out, v, st);
    case DT_I64: return dispatch_binary_strided<int64_t>(op, a, b, out, v, st);
    case DT_F32: return dispatch_binary_strided<float>(op, a, b, out, v, st);
    case DT_F64: return dispatch_binary_strided<double>(op, a, b, out, v, st);
    case DT_BF16: return dispatch_binary_strided<bf16_t>(op, a, b, out, v, st);
    case DT_F16: return dispatch_binary_strided<f16_t>(op, a, b, out, v, st);
    default: return fail(cudaErrorInvalidValue, "ew_binary_strided: unsupported dtype %d", dt);
    }
}

int bee_b200_ew_unary(int op, int dt, const void* src, void* dst, size_t n, bee_b200_stream_t stream) {
    if (n == 0) return ok();
    if (!src || !dst) return fail(cudaErrorInvalidValue, "ew_unary: null pointer");
    cudaStream_t st = as_stream(stream);
    switch (dt) {
    case DT_I32: return dispatch_unary_op<int32_t>(op, false, src, dst, n, st);
    case DT_I64: return dispatch_unary_op<int64_t>(op, false, src, dst, n, st);
    case DT_F32: return dispatch_unary_op<float>(op, true, src, dst, n, st);
    case DT_F64: return dispatch_unary_op<double>(op, true, src, dst, n, st);
    case DT_BF16: return dispatch_unary_op<bf16_t>(op, true, src, dst, n, st);
    case DT_F16: return dispatch_unary_op<f16_t>(op, true, src, dst, n, st);
    default: return fail(cudaErrorInvalidValue, "ew_unary: unsupported dtype %d", dt);
    }
}

int bee_b200_ew_cast(int src_dt, const void* src, int dst_dt, void* dst, size_t n, bee_b200_stream_t stream) {
    if (n == 0) return ok();
    if (!src || !dst) return fail(cudaErrorInvalidValue, "ew_cast: null pointer");
    cudaStream_t st = as_stream(stream);
    if (src_dt == DT_F32 && dst_dt == DT_BF16 && aligned16(src) && aligned16(dst)) {
        launch_pdl(cast_f32_bf16_kernel, grid_for((n / 8 + kUnroll - 1) / kUnroll), kThreads, 0, st,
                   static_cast<const float*>(src), static_cast<uint16_t*>(dst), n);
        return launch_status("ew_cast");
    }
    if (src_dt == DT_BF16 && dst_dt == DT_F32 && aligned16(src) && aligned16(dst)) {
        launch_pdl(cast_bf16_f32_kernel, grid_for(n / 8), kThreads, 0, st, static_cast<const uint16_t*>(src),
                   static_cast<float*>(dst), n);
        return launch_status("ew_cast");
    }
    switch (src_dt) {
    case DT_BOOL: return cast_from<bool>(dst_dt, src, dst, n, st);
    case DT_U8: return cast_from<uint8_t>(dst_dt, src, dst, n, st);
    case DT_I32: return cast_from<int32_t>(dst_dt, src, dst, n, st);
    case DT_I64: return cast_from<int64_t>(dst_dt, src, dst, n, st);
    case DT_F32: return cast_from<float>(dst_dt, src, dst, n, st);
    case DT_F64: return cast_from<double>(dst_dt, src, dst, n, st);
    case DT_BF16: return cast_from<bf16_t>(dst_dt, src, dst, n, st);
    case DT_F16: return cast_from<f16_t>(dst_dt, src, dst, n, st);
    default: return fail(cudaErrorInvalidValue, "ew_cast: unsupported source dtype %d", src_dt);
    }
}

int bee_b200_scale_fp(int dt, void* buf, double factor, size_t n, bee_b200_stream_t stream) {
    if (n == 0) return ok();
    if (!buf) return fail(cudaErrorInvalidValue, "scale_fp: null pointer");
    cudaStream_t st = as_stream(stream);
    if (dt == DT_F32) launch_pdl(scale_kernel<float>, grid_for(n), kThreads, 0, st, static_cast<float*>(buf), float(factor), n);
    else if (dt == DT_F64) launch_pdl(scale_kernel<double>, grid_for(n), kThreads, 0, st, static_cast<double*>(buf), factor, n);
    else return fail(cudaErrorInvalidValue, "scale_fp: dtype %d is not F32/F64", dt);
    return launch_status("scale_fp");
}

}  // extern "C"
