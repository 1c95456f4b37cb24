// Layout kernels: 2-D transpose and strided-view materialisation.
//
// bee_b200_transpose_2d replaces ops_transpose_2d (Bee/CUDA/Ops/OpsBridge.hpp:37-38,
// Bee/CUDA/Ops/Transpose.cu:110-145): dst[i, j] = src[j, i] for a contiguous
// [rows, cols] src.  bee_b200_strided_copy is the device path for
// Tensor::contiguous() of an arbitrary view, which the reference serves with a
// 2-D transpose fast path and otherwise a device -> host -> device round trip
// (Bee/Tensor/Core/Tensor.cpp:468-508).
//
// Both are pure data movement (HBM-bound: every byte read once, written once)
// and move elements by their size only, so every dtype of one size shares a
// kernel.  Three kernels:
//   * transpose_tile_kernel: dst[b][p][q] = src[b*sb + q*ld + p] through a
//     16 KiB shared-memory tile, 16-byte global loads and stores on both
//     sides when the rows allow it (batched: a transposed view of the two
//     innermost dims, such as K^T of [heads, seq, d]);
//   * rows_copy_kernel: views whose innermost dim is contiguous (slices such
//     as the halves of a RoPE head) — 16-byte vectors along each row;
//   * gather_kernel: any other view, one element at a time.
// A view's dims are first simplified: size-1 dims dropped, neighbours merged
// where the outer stride equals inner stride x inner extent.
#include <algorithm>
#include <cstring>

#include "common.cuh"

namespace bee_b200 {

namespace {

constexpr int kMaxDims = 8;

template <int ES> struct Word;
template <> struct Word<1> { using T = uint8_t; };
template <> struct Word<2> { using T = uint16_t; };
template <> struct Word<4> { using T = uint32_t; };
template <> struct Word<8> { using T = unsigned long long; };

// Tile shape per element size: 16 KiB of data, TQ source rows of TP elements.
// Both sides move 1024 16-byte vectors per tile, four per thread, all loads of a
// thread issued before its shared-memory writes.  A warp instruction covers 4
// rows x 8 vectors (128 contiguous bytes per row) on both sides, which with a
// one-element row pad keeps the scalar shared-memory accesses at most 2-way
// conflicted (4-way for 1-byte elements).
template <int ES> struct TileShape;
template <> struct TileShape<1> { static constexpr int TP = 128, TQ = 128, PAD = 4; };
template <> struct TileShape<2> { static constexpr int TP = 64, TQ = 128, PAD = 2; };
template <> struct TileShape<4> { static constexpr int TP = 64, TQ = 64, PAD = 1; };
template <> struct TileShape<8> { static constexpr int TP = 32, TQ = 64, PAD = 1; };

template <int ES>
__global__ void __launch_bounds__(256) transpose_tile_kernel(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst,
                                                             long long batch, long long P, long long Q, long long ld,
                                                             long long sb, int src_vec, int dst_vec) {
    using T = typename Word<ES>::T;
    using Sh = TileShape<ES>;
    constexpr int TP = Sh::TP, TQ = Sh::TQ, PITCH = TP + Sh::PAD;
    constexpr int VEC = 16 / ES;
    constexpr int VPRL = TP / VEC, VPRS = TQ / VEC;  // vectors per source row / per destination row
    constexpr int SEGL = VPRL / 8, SEGS = VPRS / 8;  // 8-vector segments per row
    constexpr int ITERS = (TQ * VPRL) / 256;         // = (TP * VPRS) / 256 = 4
    static_assert(TQ * VPRL == 1024 && TP * VPRS == 1024, "16 KiB tiles");
    __shared__ T tile[TQ][PITCH];  // [q][p]
    const T* s = reinterpret_cast<const T*>(src);
    T* d = reinterpret_cast<T*>(dst);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const long long tp = (P + TP - 1) / TP, tq = (Q + TQ - 1) / TQ;
    const long long tiles = batch * tp * tq;
    // the 16-byte loads of tile t (registers), issued a tile ahead so that they
    // overlap the shared-memory transpose and the stores of the previous tile
    auto load = [&](long long t, uint4 (&w)[ITERS]) {
        const long long b = t / (tp * tq);
        const long long rem = t - b * tp * tq;
        const long long q0 = (rem / tp) * TQ, p0 = (rem % tp) * TP;
        const T* sbase = s + b * sb;
#pragma unroll
        for (int it = 0; it < ITERS; ++it) {
            const int slot = it * 8 + warp;  // 4 rows x 8 vectors
            const int qq = (slot / SEGL) * 4 + (lane >> 3), pv = (slot % SEGL) * 8 + (lane & 7);
            const long long q = q0 + qq, p = p0 + pv * VEC;
            if (q < Q && src_vec && p + VEC <= P) w[it] = __ldcs(reinterpret_cast<const uint4*>(sbase + q * ld + p));
        }
    };
    uint4 w[ITERS];
    pdl_wait();  // nothing global is touched before the previous kernel on the stream has completed
    if (static_cast<long long>(blockIdx.x) < tiles) load(blockIdx.x, w);
    for (long long t = blockIdx.x; t < tiles; t += gridDim.x) {
        if (t + gridDim.x >= tiles) pdl_trigger();  // this CTA's last tile
        const long long b = t / (tp * tq);
        const long long rem = t - b * tp * tq;
        const long long q0 = (rem / tp) * TQ, p0 = (rem % tp) * TP;
        const T* sbase = s + b * sb;
#pragma unroll
        for (int it = 0; it < ITERS; ++it) {
            const int slot = it * 8 + warp;
            const int qq = (slot / SEGL) * 4 + (lane >> 3), pv = (slot % SEGL) * 8 + (lane & 7);
            const long long q = q0 + qq, p = p0 + pv * VEC;
            if (q >= Q) continue;
            if (src_vec && p + VEC <= P) {
                T e[VEC];
                memcpy(e, &w[it], 16);
#pragma unroll
                for (int j = 0; j < VEC; ++j) tile[qq][pv * VEC + j] = e[j];
            } else {
                const T* g = sbase + q * ld + p;
                for (int j = 0; j < VEC && p + j < P; ++j) tile[qq][pv * VEC + j] = g[j];
            }
        }
        __syncthreads();
        if (t + gridDim.x < tiles) load(t + gridDim.x, w);  // w is free again: its values are in the tile
        T* dbase = d + b * P * Q;
#pragma unroll
        for (int it = 0; it < ITERS; ++it) {
            const int slot = it * 8 + warp;
            const int pp = (slot / SEGS) * 4 + (lane >> 3), qv = (slot % SEGS) * 8 + (lane & 7);
            const long long p = p0 + pp, q = q0 + qv * VEC;
            if (p >= P) continue;
            T* g = dbase + p * Q + q;
            if (dst_vec && q + VEC <= Q) {
                T e[VEC];
#pragma unroll
                for (int j = 0; j < VEC; ++j) e[j] = tile[qv * VEC + j][pp];
                uint4 o;
                memcpy(&o, e, 16);
                __stcs(reinterpret_cast<uint4*>(g), o);
            } else {
                for (int j = 0; j < VEC && q + j < Q; ++j) g[j] = tile[qv * VEC + j][pp];
            }
        }
        __syncthreads();
    }
}

// Full 16-bit tiles (64 p x 128 q, both sides 16-byte vectorisable): a thread
// reads the same 8-element vector of two adjacent source rows, pairs their
// elements into 32-bit words with a byte permute and stores the words p-major,
// so a 16-byte output vector is four 32-bit shared loads.  Row p keeps word
// q / 2 in column (q / 2 + 4 * (p / 32)) % 64 of a 65-word pitch: with that
// rotation the 32 lanes of a store hit 32 different banks.  Half the shared-memory instructions per
// element of the generic kernel, which moves 16-bit elements one at a time.
__global__ void __launch_bounds__(256) transpose_b16_pairs_kernel(const uint16_t* __restrict__ src,
                                                                  uint16_t* __restrict__ dst, long long batch,
                                                                  long long P, long long Q, long long ld, long long sb) {
    constexpr int TP = 64, TQ = 128, PITCHW = TQ / 2 + 1;
    __shared__ uint32_t tile[TP][PITCHW];  // [p][q / 2]: word = (src[q][p], src[q + 1][p])
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const long long tp = P / TP, tq = Q / TQ;
    const long long tiles = batch * tp * tq;
    // load item i (0, 1) of this thread: rows 2r, 2r + 1 of the tile, vector pv
    auto coords = [&](int i, int& r, int& pv) {
        const int slot = i * 8 + warp;  // 16 slots of 4 row pairs x 8 vectors
        r = slot * 4 + (lane >> 3);
        pv = lane & 7;
    };
    auto load = [&](long long t, uint4 (&w)[2][2]) {
        const long long b = t / (tp * tq), rem = t - b * tp * tq;
        const long long q0 = (rem / tp) * TQ, p0 = (rem % tp) * TP;
        const uint16_t* base = src + b * sb + q0 * ld + p0;
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            int r, pv;
            coords(i, r, pv);
            w[i][0] = __ldcs(reinterpret_cast<const uint4*>(base + (2 * r) * ld + pv * 8));
            w[i][1] = __ldcs(reinterpret_cast<const uint4*>(base + (2 * r + 1) * ld + pv * 8));
        }
    };
    uint4 w[2][2];
    pdl_wait();  // nothing global is touched before the previous kernel on the stream has completed
    if (static_cast<long long>(blockIdx.x) < tiles) load(blockIdx.x, w);
    for (long long t = blockIdx.x; t < tiles; t += gridDim.x) {
        if (t + gridDim.x >= tiles) pdl_trigger();  // this CTA's last tile
        const long long b = t / (tp * tq), rem = t - b * tp * tq;
        const long long q0 = (rem / tp) * TQ, p0 = (rem % tp) * TP;
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            int r, pv;
            coords(i, r, pv);
            const uint32_t a[4] = {w[i][0].x, w[i][0].y, w[i][0].z, w[i][0].w};
            const uint32_t c[4] = {w[i][1].x, w[i][1].y, w[i][1].z, w[i][1].w};
            const int col = (r + 4 * (pv >> 2)) & 63;  // rows pv * 8 .. + 7 all lie in one half (p / 32 = pv / 4)
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                tile[pv * 8 + 2 * k][col] = __byte_perm(a[k], c[k], 0x5410);      // low halves: element 2k
                tile[pv * 8 + 2 * k + 1][col] = __byte_perm(a[k], c[k], 0x7632);  // high halves: element 2k + 1
            }
        }
        __syncthreads();
        if (t + gridDim.x < tiles) load(t + gridDim.x, w);  // w is free again: its values are in the tile
        uint16_t* dbase = dst + b * P * Q + p0 * Q + q0;
#pragma unroll
        for (int it = 0; it < 4; ++it) {
            const int slot = it * 8 + warp;  // 32 slots of 2 rows x 16 vectors
            const int pp = slot * 2 + (lane >> 4), qv = lane & 15;
            const int c0 = (qv * 4 + 4 * (pp >> 5)) & 63;  // four contiguous words (the rotation is by 4)
            uint4 o;
            o.x = tile[pp][c0 + 0];
            o.y = tile[pp][c0 + 1];
            o.z = tile[pp][c0 + 2];
            o.w = tile[pp][c0 + 3];
            __stcs(reinterpret_cast<uint4*>(dbase + pp * Q + qv * 8), o);
        }
        __syncthreads();
    }
}

struct ViewDims {
    int nd;                       // outer dims (all but the innermost)
    long long shape[kMaxDims];    // outer extents
    long long stride[kMaxDims];   // outer strides, elements
};

// Source offset (elements) of outer row `r` of the view.
__device__ __forceinline__ long long row_offset(long long r, const ViewDims& v) {
    long long off = 0;
    for (int i = v.nd - 1; i >= 0; --i) {
        const long long x = r % v.shape[i];
        r /= v.shape[i];
        off += x * v.stride[i];
    }
    return off;
}

// dst [rows, L] contiguous; row r of the view starts at src + row_offset(r); its
// L elements are contiguous.  Long rows (ROW_MODE): one CTA per row at a time,
// the row offset computed once, four 16-byte vectors in flight per thread.
// Short rows: work item = one 16-byte vector of a row.
template <int ES, bool ROW_MODE>
__global__ void __launch_bounds__(256) rows_copy_kernel(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst,
                                                        long long rows, long long L, ViewDims v, int vec_ok) {
    pdl_wait();
    using T = typename Word<ES>::T;
    constexpr int VEC = 16 / ES;
    const T* s = reinterpret_cast<const T*>(src);
    T* d = reinterpret_cast<T*>(dst);
    const long long per_row = (L + VEC - 1) / VEC;
    if constexpr (ROW_MODE) {
        for (long long r = blockIdx.x; r < rows; r += gridDim.x) {
            const T* g = s + row_offset(r, v);
            T* o = d + r * L;
            long long c = threadIdx.x;
            if (vec_ok) {
                const long long full = L / VEC;
                for (; c + 3 * 256 < full; c += 4 * 256) {
                    uint4 x[4];
#pragma unroll
                    for (int u = 0; u < 4; ++u) x[u] = __ldcs(reinterpret_cast<const uint4*>(g + (c + u * 256) * VEC));
#pragma unroll
                    for (int u = 0; u < 4; ++u) __stcs(reinterpret_cast<uint4*>(o + (c + u * 256) * VEC), x[u]);
                }
                for (; c < full; c += 256)
                    __stcs(reinterpret_cast<uint4*>(o + c * VEC), __ldcs(reinterpret_cast<const uint4*>(g + c * VEC)));
                for (long long e = full * VEC + threadIdx.x; e < L; e += 256) o[e] = g[e];
            } else {
                for (long long e = threadIdx.x; e < L; e += 256) o[e] = g[e];
            }
        }
    } else {
        const long long items = rows * per_row;
        const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
        for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < items; i += stride) {
            const long long r = i / per_row, c = (i - r * per_row) * VEC;
            const T* g = s + row_offset(r, v) + c;
            T* o = d + r * L + c;
            if (vec_ok && c + VEC <= L) {
                __stcs(reinterpret_cast<uint4*>(o), __ldcs(reinterpret_cast<const uint4*>(g)));
            } else {
                for (int j = 0; j < VEC && c + j < L; ++j) o[j] = g[j];
            }
        }
    }
}

// Any view: one element per work item; the innermost dim has stride `inner_stride`.
template <int ES>
__global__ void __launch_bounds__(256) gather_kernel(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst,
                                                     long long n, long long L, long long inner_stride, ViewDims v) {
    pdl_wait();
    using T = typename Word<ES>::T;
    const T* s = reinterpret_cast<const T*>(src);
    T* d = reinterpret_cast<T*>(dst);
    const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
    for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) {
        const long long r = i / L, c = i - r * L;
        d[i] = s[row_offset(r, v) + c * inner_stride];
    }
}

int elem_size(int dt) {
    switch (dt) {
    case DT_BOOL: case DT_U8: case DT_I8: return 1;
    case DT_F16: case DT_BF16: return 2;
    case DT_I32: case DT_F32: return 4;
    case DT_I64: case DT_F64: return 8;
    default: return 0;
    }
}

unsigned persistent_grid(long long work, int per_sm) {
    const long long cap = static_cast<long long>(sm_count()) * per_sm;
    return static_cast<unsigned>(std::max(1LL, std::min(work, cap)));
}

template <int ES>
int launch_transpose(const void* src, void* dst, long long batch, long long P, long long Q, long long ld, long long sb,
                     cudaStream_t st) {
    const int src_vec = aligned16(src) && (ld * ES) % 16 == 0 && (sb * ES) % 16 == 0;
    const int dst_vec = aligned16(dst) && (Q * ES) % 16 == 0;
    using Sh = TileShape<ES>;
    const long long tiles = batch * ((P + Sh::TP - 1) / Sh::TP) * ((Q + Sh::TQ - 1) / Sh::TQ);
    if constexpr (ES == 2) {
        if (src_vec && dst_vec && P % Sh::TP == 0 && Q % Sh::TQ == 0) {
            launch_pdl(transpose_b16_pairs_kernel, persistent_grid(tiles, 8), 256, 0, st, static_cast<const uint16_t*>(src),
                       static_cast<uint16_t*>(dst), batch, P, Q, ld, sb);
            return launch_status("transpose");
        }
    }
    launch_pdl(transpose_tile_kernel<ES>, persistent_grid(tiles, 8), 256, 0, st, static_cast<const uint8_t*>(src),
               static_cast<uint8_t*>(dst), batch, P, Q, ld, sb, src_vec, dst_vec);
    return launch_status("transpose");
}

int transpose_by_size(int es, const void* src, void* dst, long long batch, long long P, long long Q, long long ld,
                      long long sb, cudaStream_t st) {
    switch (es) {
    case 1: return launch_transpose<1>(src, dst, batch, P, Q, ld, sb, st);
    case 2: return launch_transpose<2>(src, dst, batch, P, Q, ld, sb, st);
    case 4: return launch_transpose<4>(src, dst, batch, P, Q, ld, sb, st);
    default: return launch_transpose<8>(src, dst, batch, P, Q, ld, sb, st);
    }
}

template <int ES>
int launch_rows(const void* src, void* dst, long long rows, long long L, const ViewDims& v, cudaStream_t st) {
    bool vec_ok = aligned16(src) && aligned16(dst) && (L * ES) % 16 == 0;
    for (int i = 0; i < v.nd; ++i) vec_ok = vec_ok && (v.stride[i] * ES) % 16 == 0;
    const long long per_row = (L + 16 / ES - 1) / (16 / ES);
    if (per_row >= 256) {  // rows of 4 KiB or more: a CTA per row
        launch_pdl(rows_copy_kernel<ES, true>, persistent_grid(rows, 8), 256, 0, st, static_cast<const uint8_t*>(src),
                   static_cast<uint8_t*>(dst), rows, L, v, vec_ok ? 1 : 0);
    } else {
        launch_pdl(rows_copy_kernel<ES, false>, persistent_grid((rows * per_row + 255) / 256, 8), 256, 0, st,
                   static_cast<const uint8_t*>(src), static_cast<uint8_t*>(dst), rows, L, v, vec_ok ? 1 : 0);
    }
    return launch_status("strided_copy(rows)");
}

template <int ES>
int launch_gather(const void* src, void* dst, long long n, long long L, long long inner_stride, const ViewDims& v,
                  cudaStream_t st) {
    launch_pdl(gather_kernel<ES>, persistent_grid((n + 255) / 256, 8), 256, 0, st, static_cast<const uint8_t*>(src),
               static_cast<uint8_t*>(dst), n, L, inner_stride, v);
    return launch_status("strided_copy(gather)");
}

}  // namespace
}  // namespace bee_b200

using namespace bee_b200;

extern "C" {

int bee_b200_transpose_2d(int dt, const void* src, void* dst, size_t rows, size_t cols, bee_b200_stream_t stream) {
    const int es = elem_size(dt);
    if (es == 0) return fail(cudaErrorInvalidValue, "transpose_2d: unsupported dtype %d", dt);
    if (rows == 0 || cols == 0) return ok();
    if (!src || !dst) return fail(cudaErrorInvalidValue, "transpose_2d: null pointer");
    if (rows > (1ull << 40) || cols > (1ull << 40)) return fail(cudaErrorInvalidValue, "transpose_2d: extent too large");
    // dst [cols, rows]: dst[p][q] = src[q * cols + p]
    return transpose_by_size(es, src, dst, 1, static_cast<long long>(cols), static_cast<long long>(rows),
                             static_cast<long long>(cols), 0, as_stream(stream));
}

int bee_b200_strided_copy(int dt, const void* src, int ndim, const int64_t* shape, const int64_t* strides, void* dst,
                          bee_b200_stream_t stream) {
    const int es = elem_size(dt);
    if (es == 0) return fail(cudaErrorInvalidValue, "strided_copy: unsupported dtype %d", dt);
    if (ndim < 0 || ndim > kMaxDims) return fail(cudaErrorInvalidValue, "strided_copy: ndim %d outside [0, %d]", ndim, kMaxDims);
    if (ndim > 0 && (!shape || !strides)) return fail(cudaErrorInvalidValue, "strided_copy: null shape or strides");
    long long n = 1;
    for (int i = 0; i < ndim; ++i) {
        if (shape[i] < 0) return fail(cudaErrorInvalidValue, "strided_copy: negative extent in dim %d", i);
        n *= shape[i];
        if (n > (1LL << 46)) return fail(cudaErrorInvalidValue, "strided_copy: too many elements");
    }
    if (n == 0) return ok();
    if (!src || !dst) return fail(cudaErrorInvalidValue, "strided_copy: null pointer");
    cudaStream_t st = as_stream(stream);

    // simplify: drop size-1 dims, merge neighbours that are contiguous with each other
    long long sh[kMaxDims], sd[kMaxDims];
    int nd = 0;
    for (int i = 0; i < ndim; ++i) {
        if (shape[i] == 1) continue;
        if (nd > 0 && sd[nd - 1] == strides[i] * shape[i]) {
            sh[nd - 1] *= shape[i];
            sd[nd - 1] = strides[i];
        } else {
            sh[nd] = shape[i];
            sd[nd] = strides[i];
            ++nd;
        }
    }
    if (nd == 0) {  // a single element
        sh[0] = 1;
        sd[0] = 1;
        nd = 1;
    }
    if (nd == 1 && sd[0] == 1) {
        cudaError_t e = cudaMemcpyAsync(dst, src, static_cast<size_t>(n) * es, cudaMemcpyDeviceToDevice, st);
        if (e != cudaSuccess) return fail(static_cast<int>(e), "strided_copy: %s", cudaGetErrorString(e));
        return ok();
    }
    // a transposed pair of innermost dims: [.., Q-dim stride 1 .., P-dim] -> batched tiles
    if (nd >= 2 && sd[nd - 2] == 1 && sd[nd - 1] != 1 && (nd == 2 || nd == 3)) {
        const long long P = sh[nd - 2], Q = sh[nd - 1];
        const long long ld = sd[nd - 1];
        const long long batch = nd == 3 ? sh[0] : 1;
        const long long sb = nd == 3 ? sd[0] : 0;
        // dst[b][p][q] = src[b*sb + q*ld + p] with dst [batch][P][Q]; the tile
        // kernel names the dst rows p and the dst columns q.
        return transpose_by_size(es, src, dst, batch, P, Q, ld, sb, st);
    }
    ViewDims v{};
    v.nd = nd - 1;
    for (int i = 0; i < nd - 1; ++i) {
        v.shape[i] = sh[i];
        v.stride[i] = sd[i];
    }
    const long long L = sh[nd - 1], rows = n / L;
    if (sd[nd - 1] == 1) {
        switch (es) {
        case 1: return launch_rows<1>(src, dst, rows, L, v, st);
        case 2: return launch_rows<2>(src, dst, rows, L, v, st);
        case 4: return launch_rows<4>(src, dst, rows, L, v, st);
        default: return launch_rows<8>(src, dst, rows, L, v, st);
        }
    }
    switch (es) {
    case 1: return launch_gather<1>(src, dst, n, L, sd[nd - 1], v, st);
    case 2: return launch_gather<2>(src, dst, n, L, sd[nd - 1], v, st);
    case 4: return launch_gather<4>(src, dst, n, L, sd[nd - 1], v, st);
    default: return launch_gather<8>(src, dst, n, L, sd[nd - 1], v, st);
    }
}

}  // extern "C"
