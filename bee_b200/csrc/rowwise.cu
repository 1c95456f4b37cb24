// Row-wise operators: softmax, RMSNorm, RoPE and the fused RMSNorm+RoPE.
//
// None of these exist in the reference (its CPU oracle composes them from
// public ops: max/sub/exp/sum/div for softmax, mul/mean/add/sqrt/div/mul for
// RMSNorm, slice views with mul/sub/add for RoPE).  B200 design: one CTA owns
// one row at a time and keeps it in registers, so every byte is read from HBM
// once and written once (the single-pass minimum); loads are 16 bytes (fp32)
// or 8/16 bytes (bf16) and streaming; the reductions are warp shuffles plus
// one shared-memory exchange; the grid is a multiple of the SM count and
// strides over rows.
#include <cmath>

#include "common.cuh"

namespace bee_b200 {

constexpr float kLog2e = 1.4426950408889634f;

// ---------------------------------------------------------------- element IO

// A "quad" is 4 consecutive elements: fp32 -> one 16-byte load, bf16 -> 8 bytes.
template <typename T> struct Quad;
template <> struct Quad<float> {
    static __device__ __forceinline__ void load(const float* p, float v[4]) {
        float4 q = __ldcs(reinterpret_cast<const float4*>(p));
        v[0] = q.x; v[1] = q.y; v[2] = q.z; v[3] = q.w;
    }
    static __device__ __forceinline__ void store(float* p, const float v[4]) {
        __stcs(reinterpret_cast<float4*>(p), make_float4(v[0], v[1], v[2], v[3]));
    }
    static __device__ __forceinline__ float get(const float* p, size_t i) { return p[i]; }
    static __device__ __forceinline__ void put(float* p, size_t i, float v) { p[i] = v; }
};
template <> struct Quad<uint16_t> {  // bf16 bits
    static __device__ __forceinline__ void load(const uint16_t* p, float v[4]) {
        uint2 q = __ldcs(reinterpret_cast<const uint2*>(p));
        v[0] = bf16_lo(q.x); v[1] = bf16_hi(q.x); v[2] = bf16_lo(q.y); v[3] = bf16_hi(q.y);
    }
    static __device__ __forceinline__ void store(uint16_t* p, const float v[4]) {
        __stcs(reinterpret_cast<uint2*>(p), make_uint2(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3])));
    }
    static __device__ __forceinline__ float get(const uint16_t* p, size_t i) {
        return __uint_as_float(static_cast<uint32_t>(p[i]) << 16);
    }
    static __device__ __forceinline__ void put(uint16_t* p, size_t i, float v) {
        __nv_bfloat16 h = __float2bfloat16_rn(v);
        p[i] = *reinterpret_cast<uint16_t*>(&h);
    }
};

// Loads the row slots owned by this thread: slot s covers elements
// [(s*THREADS + tid)*4, +4).  `vec` selects quad loads (row start aligned and
// cols % 4 == 0) versus element loads; missing elements get `fill`.
template <typename T, int THREADS, int NQ>
__device__ __forceinline__ void load_row(const T* row, size_t cols, bool vec, float fill, float v[NQ][4]) {
#pragma unroll
    for (int s = 0; s < NQ; ++s) {
        const size_t e = (static_cast<size_t>(s) * THREADS + threadIdx.x) * 4;
        if (vec && e + 4 <= cols) {
            Quad<T>::load(row + e, v[s]);
        } else {
#pragma unroll
            for (int k = 0; k < 4; ++k) v[s][k] = (e + k < cols) ? Quad<T>::get(row, e + k) : fill;
        }
    }
}

template <typename T, int THREADS, int NQ>
__device__ __forceinline__ void store_row(T* row, size_t cols, bool vec, const float v[NQ][4]) {
#pragma unroll
    for (int s = 0; s < NQ; ++s) {
        const size_t e = (static_cast<size_t>(s) * THREADS + threadIdx.x) * 4;
        if (vec && e + 4 <= cols) {
            Quad<T>::store(row + e, v[s]);
        } else {
#pragma unroll
            for (int k = 0; k < 4; ++k)
                if (e + k < cols) Quad<T>::put(row, e + k, v[s][k]);
        }
    }
}

template <int THREADS> __device__ __forceinline__ float block_max(float v, float* red) {
    v = warp_max(v);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float r = red[0];
#pragma unroll
    for (int w = 1; w < THREADS / 32; ++w) r = fmaxf(r, red[w]);
    return r;
}

template <int THREADS> __device__ __forceinline__ float block_sum(float v, float* red) {
    v = warp_sum(v);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float r = 0.f;
#pragma unroll
    for (int w = 0; w < THREADS / 32; ++w) r += red[w];
    return r;
}

// Block-wide sum with one barrier: the warp partials of consecutive calls go to
// alternating halves of `red` ([2][THREADS / 32], `parity` flips per call), so a
// call's writes never meet the previous call's reads (every thread has passed
// the previous call's barrier after reading, before the next write).
template <int THREADS> __device__ __forceinline__ float block_sum_1bar(float v, float (*red)[THREADS / 32], int parity) {
    v = warp_sum(v);
    if ((threadIdx.x & 31) == 0) red[parity][threadIdx.x >> 5] = v;
    __syncthreads();
    float r = 0.f;
#pragma unroll
    for (int w = 0; w < THREADS / 32; ++w) r += red[parity][w];
    return r;
}

// ---------------------------------------------------------------- softmax

template <typename Ti, typename To, int THREADS, int NQ>
__global__ void __launch_bounds__(THREADS) softmax_rows_kernel(const Ti* __restrict__ src, To* __restrict__ dst,
                                                               size_t rows, size_t cols, int vec) {
    __shared__ float red[THREADS / 32];
    pdl_wait();
    for (size_t r = blockIdx.x; r < rows; r += gridDim.x) {
        if (r + gridDim.x >= rows) pdl_trigger();  // this CTA's last row
        float v[NQ][4];
        load_row<Ti, THREADS, NQ>(src + r * cols, cols, vec, -INFINITY, v);
        float m = -INFINITY;
#pragma unroll
        for (int s = 0; s < NQ; ++s)
#pragma unroll
            for (int k = 0; k < 4; ++k) m = fmaxf(m, v[s][k]);
        m = block_max<THREADS>(m, red);
        const float ms = m * kLog2e;
        float sum = 0.f;
#pragma unroll
        for (int s = 0; s < NQ; ++s)
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                // exp(x - m) = 2^(x*log2e - m*log2e); padding (-inf) gives 0.
                v[s][k] = exp2f(fmaf(v[s][k], kLog2e, -ms));
                sum += v[s][k];
            }
        sum = block_sum<THREADS>(sum, red);
        const float inv = 1.0f / sum;
#pragma unroll
        for (int s = 0; s < NQ; ++s)
#pragma unroll
            for (int k = 0; k < 4; ++k) v[s][k] *= inv;
        store_row<To, THREADS, NQ>(dst + r * cols, cols, vec, v);
    }
}

// Rows longer than the register-resident limit: online max/sum in one read,
// normalise in a second read (3 passes of traffic instead of 2).
template <typename Ti, typename To>
__global__ void __launch_bounds__(1024) softmax_rows_long_kernel(const Ti* __restrict__ src, To* __restrict__ dst,
                                                                 size_t rows, size_t cols) {
    __shared__ float red_m[32], red_s[32];
    for (size_t r = blockIdx.x; r < rows; r += gridDim.x) {
        const Ti* row = src + r * cols;
        float m = -INFINITY, s = 0.f;
        for (size_t j = threadIdx.x; j < cols; j += blockDim.x) {
            const float x = Quad<Ti>::get(row, j);
            const float nm = fmaxf(m, x);
            s = s * exp2f((m - nm) * kLog2e) + exp2f((x - nm) * kLog2e);
            m = nm;
        }
        // combine (m, s) pairs across the warp, then across warps
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float om = __shfl_xor_sync(0xffffffffu, m, o), os = __shfl_xor_sync(0xffffffffu, s, o);
            const float nm = fmaxf(m, om);
            s = (nm == -INFINITY) ? 0.f : s * exp2f((m - nm) * kLog2e) + os * exp2f((om - nm) * kLog2e);
            m = nm;
        }
        __syncthreads();
        if ((threadIdx.x & 31) == 0) {
            red_m[threadIdx.x >> 5] = m;
            red_s[threadIdx.x >> 5] = s;
        }
        __syncthreads();
        float M = -INFINITY;
        for (int w = 0; w < int(blockDim.x >> 5); ++w) M = fmaxf(M, red_m[w]);
        float S = 0.f;
        for (int w = 0; w < int(blockDim.x >> 5); ++w)
            S += (red_m[w] == -INFINITY) ? 0.f : red_s[w] * exp2f((red_m[w] - M) * kLog2e);
        const float inv = 1.0f / S;
        for (size_t j = threadIdx.x; j < cols; j += blockDim.x)
            Quad<To>::put(dst + r * cols, j, exp2f((Quad<Ti>::get(row, j) - M) * kLog2e) * inv);
    }
}

// ---------------------------------------------------------------- RMSNorm (+RoPE)

struct RopeArgs {
    int enabled;
    size_t seq;
    size_t head_dim;
    size_t pos_offset;
    double log_theta;
};

// One CTA per row.  NORM: scale by 1/sqrt(mean(x^2)+eps) * w.  ROPE: rotate
// each head's halves; the partner element of a head lives in another thread,
// so the row passes through shared memory (fp32) between the two steps.
// Angles: turns_i = p * f_i / (2 pi) is formed in double, its integer part
// dropped in double, and the remaining fraction (|r| <= 1/2 turn) goes to
// sincospif in fp32, so the angle keeps ~1e-7 rad accuracy at p = 2047
// without a double-precision sin/cos per element.
template <typename T, int THREADS, int NQ, bool NORM, bool ROPE>
__global__ void __launch_bounds__(THREADS) norm_rope_kernel(const T* __restrict__ x, const T* __restrict__ w,
                                                            T* __restrict__ y, size_t rows, size_t cols, float eps,
                                                            RopeArgs rope, int vec) {
    extern __shared__ float smem[];  // ROPE: cols floats of row + head_dim/2 float2 of (cos, sin)
    __shared__ float red[THREADS / 32];
    __shared__ double turns_per_pos[128];  // f_i / (2 pi)
    const uint32_t hd = static_cast<uint32_t>(rope.head_dim);
    const uint32_t half = hd / 2;
    if (ROPE) {
        for (uint32_t i = threadIdx.x; i < half; i += THREADS)
            turns_per_pos[i] = exp(-(2.0 * static_cast<double>(i) / static_cast<double>(hd)) * rope.log_theta) *
                               0.15915494309189533577;  // 1 / (2 pi)
    }
    float wv[NQ][4];
    if (NORM) load_row<T, THREADS, NQ>(w, cols, vec, 0.f, wv);
    float* rowbuf = smem;
    float2* cs = reinterpret_cast<float2*>(smem + cols);
    const uint32_t ucols = static_cast<uint32_t>(cols);
    for (size_t r = blockIdx.x; r < rows; r += gridDim.x) {
        float v[NQ][4];
        load_row<T, THREADS, NQ>(x + r * cols, cols, vec, 0.f, v);
        if (NORM) {
            float ss = 0.f;
#pragma unroll
            for (int s = 0; s < NQ; ++s)
#pragma unroll
                for (int k = 0; k < 4; ++k) ss = fmaf(v[s][k], v[s][k], ss);
            ss = block_sum<THREADS>(ss, red);
            const float inv = 1.0f / sqrtf(ss / static_cast<float>(cols) + eps);
#pragma unroll
            for (int s = 0; s < NQ; ++s)
#pragma unroll
                for (int k = 0; k < 4; ++k) v[s][k] = v[s][k] * inv * wv[s][k];
        }
        if (ROPE) {
            const double p = static_cast<double>(r % rope.seq + rope.pos_offset);
            __syncthreads();  // previous row's readers of rowbuf / cs are done
            for (uint32_t i = threadIdx.x; i < half; i += THREADS) {
                const double t = p * turns_per_pos[i];
                const float frac = static_cast<float>(t - rint(t));  // in [-1/2, 1/2] turns
                float sn, c;
                sincospif(2.0f * frac, &sn, &c);
                cs[i] = make_float2(c, sn);
            }
#pragma unroll
            for (int s = 0; s < NQ; ++s) {
                const uint32_t e = (static_cast<uint32_t>(s) * THREADS + threadIdx.x) * 4;
#pragma unroll
                for (int k = 0; k < 4; ++k)
                    if (e + k < ucols) rowbuf[e + k] = v[s][k];
            }
            __syncthreads();
#pragma unroll
            for (int s = 0; s < NQ; ++s) {
                const uint32_t e = (static_cast<uint32_t>(s) * THREADS + threadIdx.x) * 4;
                uint32_t d = e % hd;  // one 32-bit modulo per quad
#pragma unroll
                for (int k = 0; k < 4; ++k, ++d) {
                    if (d >= hd) d -= hd;
                    const uint32_t idx = e + k;
                    if (idx >= ucols) continue;
                    if (d < half) {
                        const float2 t = cs[d];
                        v[s][k] = v[s][k] * t.x - rowbuf[idx + half] * t.y;
                    } else {
                        const float2 t = cs[d - half];
                        v[s][k] = v[s][k] * t.x + rowbuf[idx - half] * t.y;
                    }
                }
            }
        }
        store_row<T, THREADS, NQ>(y + r * cols, cols, vec, v);
    }
}

// Pipelined RMSNorm / RoPE for rows whose length is a whole number of 16-byte
// chunks (and head_dim a multiple of two chunks when rotating): every thread
// streams its share of upcoming rows into a shared-memory ring with cp.async
// (S rows per CTA in flight, no spin-waits: cp.async.wait_group), so HBM keeps
// streaming while earlier rows are reduced, rotated and written back with
// 16-byte stores.  The rotate-half partner chunk is read from the same ring
// slot, so no extra exchange pass is needed.
__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gmem_src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst))),
                 "l"(gmem_src)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N> __device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

template <typename T> struct Chunk;
template <> struct Chunk<float> {
    static constexpr int E = 4;
    static __device__ __forceinline__ void unpack(uint4 q, float v[4]) {
        v[0] = __uint_as_float(q.x); v[1] = __uint_as_float(q.y); v[2] = __uint_as_float(q.z); v[3] = __uint_as_float(q.w);
    }
    static __device__ __forceinline__ uint4 pack(const float v[4]) {
        return make_uint4(__float_as_uint(v[0]), __float_as_uint(v[1]), __float_as_uint(v[2]), __float_as_uint(v[3]));
    }
};
template <> struct Chunk<uint16_t> {
    static constexpr int E = 8;
    static __device__ __forceinline__ void unpack(uint4 q, float v[8]) {
        v[0] = bf16_lo(q.x); v[1] = bf16_hi(q.x); v[2] = bf16_lo(q.y); v[3] = bf16_hi(q.y);
        v[4] = bf16_lo(q.z); v[5] = bf16_hi(q.z); v[6] = bf16_lo(q.w); v[7] = bf16_hi(q.w);
    }
    static __device__ __forceinline__ uint4 pack(const float v[8]) {
        return make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]), pack_bf16x2(v[4], v[5]), pack_bf16x2(v[6], v[7]));
    }
};

// Work assignment: a "unit" is one 16-byte chunk (RMSNorm only) or, with RoPE,
// a rotate-half pair of chunks — chunk c of the first half of a head and chunk
// c + half/E of its second half — so a thread holds both partners.  Thread t
// owns units t + k*THREADS (k < NP) of every row and copies exactly those
// chunks into its own part of the ring, so row data needs no block barrier:
// cp.async.wait_group makes the thread's own copies visible to itself.  The
// only barriers per row are the two of the sum-of-squares reduction (RMSNorm)
// or one publishing the cos/sin table (RoPE alone).  Weights and per-unit
// offsets stay in registers for the whole kernel; 1/rms is folded into the
// row's cos/sin values, leaving about three FP instructions per element.
// A thread keeps its share of the row and the matching weights unpacked in
// registers between the sum-of-squares pass and the output pass, so each element
// is unpacked once per row and each weight once per kernel.  Every configuration
// the dispatcher launches gives a thread at most 32 elements, which fits in 128
// registers at 512 threads per SM; on 4096-column rows, where the kernel is bound
// by instruction issue, this ran 6-9% faster in bf16 than reloading the row from
// the ring and re-expanding packed weights at 1024 threads per SM.
template <typename T, int NP, bool ROPE>
constexpr int pipe_share() {
    return NP * (ROPE ? 2 : 1) * (16 / static_cast<int>(sizeof(T)));
}

template <typename T, int THREADS, int NP, int S, bool NORM, bool ROPE>
__global__ void __launch_bounds__(THREADS, 512 / THREADS) norm_rope_pipe_kernel(const T* __restrict__ x, const T* __restrict__ w,
                                                                 T* __restrict__ y, size_t rows, uint32_t cols,
                                                                 float eps, RopeArgs rope) {
    using CK = Chunk<T>;
    constexpr int E = CK::E;
    constexpr int CPU = ROPE ? 2 : 1;  // chunks per unit
    extern __shared__ __align__(16) uint8_t pipe_smem[];
    __shared__ float red[2][THREADS / 32];
    __shared__ double turns_per_pos[128];
    const uint32_t chunks = cols / E;
    const uint32_t units = chunks / CPU;
    const uint32_t row_bytes = cols * static_cast<uint32_t>(sizeof(T));
    uint8_t* ring = pipe_smem;
    // cos / sin tables of the current and previous row: [2][half] floats each
    float* cos_t = reinterpret_cast<float*>(pipe_smem + S * row_bytes);
    float* sin_t = cos_t + rope.head_dim;
    const uint32_t hd = static_cast<uint32_t>(rope.head_dim);
    const uint32_t half = hd / 2;
    const uint32_t tid = threadIdx.x;
    // angle per position of each frequency: kernel arguments only, so it is
    // computed before the wait for the previous kernel on the stream
    if (ROPE)
        for (uint32_t i = tid; i < half; i += THREADS)
            turns_per_pos[i] = exp(-(2.0 * static_cast<double>(i) / static_cast<double>(hd)) * rope.log_theta) *
                               0.15915494309189533577;  // 1 / (2 pi)
    pdl_wait();

    // Per-unit constants: chunk indices, table offset, weights.
    uint32_t cidx[NP][CPU];
    uint32_t toff[NP];
    bool live[NP];
    static_assert(pipe_share<T, NP, ROPE>() <= 32, "a thread's share of the row must fit in registers");
    float wv[NP][CPU][E];  // weights, unpacked once
#pragma unroll
    for (int u = 0; u < NP; ++u) {
        const uint32_t unit = tid + u * THREADS;
        live[u] = unit < units;
        if (ROPE) {
            const uint32_t pairs_per_head = half / E;
            const uint32_t h = live[u] ? unit / pairs_per_head : 0, j = live[u] ? unit % pairs_per_head : 0;
            cidx[u][0] = h * (hd / E) + j;
            cidx[u][CPU - 1] = cidx[u][0] + pairs_per_head;
            toff[u] = j * E;
        } else {
            cidx[u][0] = live[u] ? unit : 0;
            toff[u] = 0;
        }
#pragma unroll
        for (int q = 0; q < CPU; ++q) {
            CK::unpack((NORM && live[u]) ? reinterpret_cast<const uint4*>(w)[cidx[u][q]] : make_uint4(0, 0, 0, 0), wv[u][q]);
        }
    }
    if (ROPE) __syncthreads();  // turns_per_pos is read by other threads below

    // Row order.  RMSNorm alone: CTA b takes rows b, b + G, ... .  With RoPE the
    // rows are visited in position-major order — item i is position p = i / B
    // of batch entry m = i % B, i.e. row m * seq + p (B = rows / seq) — and
    // CTA b takes the contiguous items [b * chunk, (b + 1) * chunk), so its
    // rows share a position for B items at a time and the cos/sin table is
    // rebuilt only when the position changes.
    const size_t G = gridDim.x;
    const size_t B = rows / rope.seq;
    const size_t chunk = (rows + G - 1) / G;
    const size_t i_begin = ROPE ? blockIdx.x * chunk : blockIdx.x;
    const size_t i_end = ROPE ? (i_begin + chunk < rows ? i_begin + chunk : rows) : rows;
    const size_t i_step = ROPE ? 1 : G;
    auto row_of = [&](size_t i) -> size_t { return ROPE ? (i % B) * rope.seq + i / B : i; };
    auto pos_of = [&](size_t i) -> size_t { return ROPE ? i / B : 0; };

    size_t i_issue = i_begin;
    int slot_issue = 0;
    auto issue = [&]() {
        if (i_issue < i_end) {
            const uint4* src = reinterpret_cast<const uint4*>(x + row_of(i_issue) * cols);
            uint4* dst = reinterpret_cast<uint4*>(ring + slot_issue * row_bytes);
#pragma unroll
            for (int u = 0; u < NP; ++u)
#pragma unroll
                for (int q = 0; q < CPU; ++q)
                    if (live[u]) cp_async16(dst + cidx[u][q], src + cidx[u][q]);
        }
        cp_async_commit();  // one group per row slot, empty past the end, so wait counts stay uniform
        i_issue += i_step;
        slot_issue = slot_issue + 1 == S ? 0 : slot_issue + 1;
    };
#pragma unroll
    for (int j = 0; j < S - 1; ++j) issue();

    int slot = 0;
    uint32_t parity = 1;
    size_t cur_pos = ~size_t(0);
    int red_parity = 0;
    for (size_t i = i_begin; i < i_end; i += i_step, slot = slot + 1 == S ? 0 : slot + 1) {
        if (i + i_step >= i_end) pdl_trigger();  // this CTA's last row
        issue();
        cp_async_wait<S - 1>();  // this thread's copies of this row have landed
        const size_t r = row_of(i);
        const uint4* row = reinterpret_cast<const uint4*>(ring + slot * row_bytes);
        bool new_table = false;
        if (ROPE) {
            const size_t pos = pos_of(i);
            if (pos != cur_pos) {
                cur_pos = pos;
                parity ^= 1u;
                new_table = true;
                const double p = static_cast<double>(pos + rope.pos_offset);
                float* cw = cos_t + parity * half;
                float* sw = sin_t + parity * half;
                for (uint32_t k = tid; k < half; k += THREADS) {
                    const double t = p * turns_per_pos[k];
                    const float frac = static_cast<float>(t - rint(t));
                    float sn, c;
                    sincospif(2.0f * frac, &sn, &c);
                    cw[k] = c;
                    sw[k] = sn;
                }
            }
        }
        const float* cosj = cos_t + parity * half;
        const float* sinj = sin_t + parity * half;
        // the thread's elements of this row, unpacked once for both passes
        float xv[NP][CPU][E];
#pragma unroll
        for (int u = 0; u < NP; ++u)
#pragma unroll
            for (int q = 0; q < CPU; ++q) CK::unpack(live[u] ? row[cidx[u][q]] : make_uint4(0, 0, 0, 0), xv[u][q]);
        auto elem = [&](int u, int q, float (&t)[E]) {
#pragma unroll
            for (int k = 0; k < E; ++k) t[k] = xv[u][q][k];
        };
        auto weight = [&](int u, int q, float (&t)[E]) {
#pragma unroll
            for (int k = 0; k < E; ++k) t[k] = wv[u][q][k];
        };
        float ss = 0.f;
        if (NORM) {
#pragma unroll
            for (int u = 0; u < NP; ++u)
#pragma unroll
                for (int q = 0; q < CPU; ++q)
                    if (live[u]) {
                        float t[E];
                        elem(u, q, t);
#pragma unroll
                        for (int k = 0; k < E; ++k) ss = fmaf(t[k], t[k], ss);
                    }
        }
        float inv = 1.0f;
        if (NORM) {
            ss = block_sum_1bar<THREADS>(ss, red, red_parity);  // also publishes a rebuilt cos / sin table
            red_parity ^= 1;
            inv = rsqrtf(ss / static_cast<float>(cols) + eps);
        } else if (new_table) {
            __syncthreads();  // publish the rebuilt cos / sin table (uniform: every thread sees the same position)
        }
        uint4* dst = reinterpret_cast<uint4*>(y + r * cols);
#pragma unroll
        for (int u = 0; u < NP; ++u) {
            if (!live[u]) continue;
            if (ROPE) {
                float a[E], b[E];
                elem(u, 0, a);
                elem(u, 1, b);
                if (NORM) {
                    float wa[E], wb[E];
                    weight(u, 0, wa);
                    weight(u, 1, wb);
#pragma unroll
                    for (int k = 0; k < E; ++k) {
                        a[k] *= wa[k];
                        b[k] *= wb[k];
                    }
                }
#pragma unroll
                for (int k = 0; k < E; k += 4) {
                    const float4 c4 = *reinterpret_cast<const float4*>(cosj + toff[u] + k);
                    const float4 s4 = *reinterpret_cast<const float4*>(sinj + toff[u] + k);
                    const float cv[4] = {c4.x * inv, c4.y * inv, c4.z * inv, c4.w * inv};
                    const float sv[4] = {s4.x * inv, s4.y * inv, s4.z * inv, s4.w * inv};
#pragma unroll
                    for (int m = 0; m < 4; ++m) {
                        const float a0 = a[k + m], b0 = b[k + m];
                        a[k + m] = fmaf(a0, cv[m], -b0 * sv[m]);
                        b[k + m] = fmaf(b0, cv[m], a0 * sv[m]);
                    }
                }
                __stcs(dst + cidx[u][0], CK::pack(a));
                __stcs(dst + cidx[u][1], CK::pack(b));
            } else {
                float a[E], wa[E];
                elem(u, 0, a);
                weight(u, 0, wa);
#pragma unroll
                for (int k = 0; k < E; ++k) a[k] = a[k] * inv * wa[k];
                __stcs(dst + cidx[u][0], CK::pack(a));
            }
        }
        // No barrier here: ring slots are private per thread, and a table
        // buffer is rewritten only after the barrier that published the other.
    }
    cp_async_wait<0>();
}

// ---------------------------------------------------------------- launchers

static unsigned row_grid(size_t rows, int ctas_per_sm) {
    size_t cap = static_cast<size_t>(sm_count()) * ctas_per_sm;
    return static_cast<unsigned>(rows < cap ? rows : cap);
}

template <typename Ti, typename To>
static int launch_softmax(const void* src, void* dst, size_t rows, size_t cols, cudaStream_t st) {
    const Ti* s = static_cast<const Ti*>(src);
    To* d = static_cast<To*>(dst);
    const int vec = (cols % 4 == 0) && aligned16(src) && aligned16(dst) ? 1 : 0;
    // Register-resident variants: up to 32 fp32 values per thread.
    if (cols <= 256 * 4)
        launch_pdl(softmax_rows_kernel<Ti, To, 256, 1>, row_grid(rows, 8), 256, 0, st, s, d, rows, cols, vec);
    else if (cols <= 256 * 4 * 4)
        launch_pdl(softmax_rows_kernel<Ti, To, 256, 4>, row_grid(rows, 8), 256, 0, st, s, d, rows, cols, vec);
    else if (cols <= 256 * 4 * 8)
        launch_pdl(softmax_rows_kernel<Ti, To, 256, 8>, row_grid(rows, 8), 256, 0, st, s, d, rows, cols, vec);
    else if (cols <= 1024 * 4 * 8)
        launch_pdl(softmax_rows_kernel<Ti, To, 1024, 8>, row_grid(rows, 2), 1024, 0, st, s, d, rows, cols, vec);
    else softmax_rows_long_kernel<Ti, To><<<row_grid(rows, 2), 1024, 0, st>>>(s, d, rows, cols);
    return launch_status("softmax_rows");
}

template <typename T, int THREADS, int NP, int S, bool NORM, bool ROPE>
static int launch_pipe(const T* px, const T* pw, T* py, size_t rows, size_t cols, float eps, RopeArgs rope,
                       cudaStream_t st) {
    const size_t row_bytes = cols * sizeof(T);
    const size_t smem = S * row_bytes + (ROPE ? 2 * rope.head_dim * sizeof(float) : 0);
    auto k = norm_rope_pipe_kernel<T, THREADS, NP, S, NORM, ROPE>;
    if (smem + 2048 > 48 * 1024) {  // dynamic + static shared memory above the default 48 KiB
        cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return fail(static_cast<int>(e), "rms_norm/rope: shared memory attribute: %s", cudaGetErrorString(e));
    }
    int per_sm = static_cast<int>((220 * 1024) / (smem + 1024 + 1024));
    const int by_threads = 2048 / THREADS;
    per_sm = per_sm < 1 ? 1 : (per_sm > by_threads ? by_threads : per_sm);
    launch_pdl(k, row_grid(rows, per_sm), THREADS, smem, st, px, pw, py, rows, static_cast<uint32_t>(cols), eps, rope);
    return launch_status(NORM ? (ROPE ? "rms_norm_rope" : "rms_norm_rows") : "rope");
}

// Picks threads-per-CTA and units-per-thread for the pipelined kernel (at most
// four 16-byte chunks per thread, so values and weights stay in registers);
// returns -1 when the row is too long for it.
template <typename T, int S, bool NORM, bool ROPE>
static int dispatch_pipe(const T* px, const T* pw, T* py, size_t rows, size_t cols, float eps, RopeArgs rope,
                         cudaStream_t st) {
    constexpr size_t E = 16 / sizeof(T);
    const size_t chunks = cols / E;
    const size_t units = chunks / (ROPE ? 2 : 1);
    if constexpr (ROPE) {
        if (units <= 128) return launch_pipe<T, 128, 1, S, NORM, ROPE>(px, pw, py, rows, cols, eps, rope, st);
        if (units <= 256) return launch_pipe<T, 128, 2, S, NORM, ROPE>(px, pw, py, rows, cols, eps, rope, st);
        if (units <= 512) return launch_pipe<T, 256, 2, S, NORM, ROPE>(px, pw, py, rows, cols, eps, rope, st);
    } else {
        if (units <= 128) return launch_pipe<T, 128, 1, S, NORM, ROPE>(px, pw, py, rows, cols, eps, rope, st);
        if (units <= 256) return launch_pipe<T, 128, 2, S, NORM, ROPE>(px, pw, py, rows, cols, eps, rope, st);
        if (units <= 512) return launch_pipe<T, 128, 4, S, NORM, ROPE>(px, pw, py, rows, cols, eps, rope, st);
        if (units <= 1024) return launch_pipe<T, 256, 4, S, NORM, ROPE>(px, pw, py, rows, cols, eps, rope, st);
    }
    return -1;
}

template <typename T, bool NORM, bool ROPE>
static int launch_norm_rope(const void* x, const void* w, void* y, size_t rows, size_t cols, float eps, RopeArgs rope,
                            cudaStream_t st) {
    const T* px = static_cast<const T*>(x);
    const T* pw = static_cast<const T*>(w);
    T* py = static_cast<T*>(y);
    constexpr size_t E = 16 / sizeof(T);
    const size_t row_bytes = cols * sizeof(T);
    const bool pipe_ok = cols % E == 0 && aligned16(x) && aligned16(y) && (!NORM || aligned16(w)) &&
                         (!ROPE || rope.head_dim % (2 * E) == 0) && row_bytes <= 16 * 1024;
    if (pipe_ok) {
        const int rc = dispatch_pipe<T, 3, NORM, ROPE>(px, pw, py, rows, cols, eps, rope, st);
        if (rc != -1) return rc;
    }
    const int vec = (cols % 4 == 0) && aligned16(x) && aligned16(y) && (!NORM || aligned16(w)) ? 1 : 0;
    const size_t smem = ROPE ? cols * sizeof(float) + (rope.head_dim / 2) * sizeof(float2) : 0;
    if (smem > 200 * 1024) return fail(cudaErrorInvalidValue, "rope: row of %zu elements exceeds shared memory", cols);
#define BEE_NR_LAUNCH(THREADS, NQ, CTAS)                                                                              \
    do {                                                                                                              \
        auto k = norm_rope_kernel<T, THREADS, NQ, NORM, ROPE>;                                                       \
        if (smem + 2048 > 48 * 1024) cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));  \
        k<<<row_grid(rows, CTAS), THREADS, smem, st>>>(px, pw, py, rows, cols, eps, rope, vec);                       \
    } while (0)
    if (cols <= 128 * 4 * 2) BEE_NR_LAUNCH(128, 2, 12);
    else if (cols <= 256 * 4 * 4) BEE_NR_LAUNCH(256, 4, 8);
    else if (cols <= 512 * 4 * 4) BEE_NR_LAUNCH(512, 4, 4);
    else if (cols <= 1024 * 4 * 8) BEE_NR_LAUNCH(1024, 8, 2);
    else return fail(cudaErrorInvalidValue, "rms_norm/rope: row of %zu elements exceeds 32768", cols);
#undef BEE_NR_LAUNCH
    return launch_status(NORM ? (ROPE ? "rms_norm_rope" : "rms_norm_rows") : "rope");
}

static int check_rope(size_t rows, size_t seq, size_t heads, size_t head_dim, double theta, const char* what) {
    if (seq == 0 || heads == 0 || head_dim == 0) return fail(cudaErrorInvalidValue, "%s: empty extent", what);
    if (head_dim % 2 != 0 || head_dim > 256)
        return fail(cudaErrorInvalidValue, "%s: head_dim %zu must be even and <= 256", what, head_dim);
    if (rows % seq != 0) return fail(cudaErrorInvalidValue, "%s: rows %zu not a multiple of seq %zu", what, rows, seq);
    if (!(theta > 0.0)) return fail(cudaErrorInvalidValue, "%s: theta must be positive", what);
    return 0;
}

}  // namespace bee_b200

using namespace bee_b200;

extern "C" {

int bee_b200_softmax_rows_to(int src_dt, const void* src, int dst_dt, void* dst, size_t rows, size_t cols,
                             bee_b200_stream_t stream) {
    if (rows == 0) return ok();
    if (cols == 0) return fail(cudaErrorInvalidValue, "softmax_rows: zero columns");
    if (!src || !dst) return fail(cudaErrorInvalidValue, "softmax_rows: null pointer");
    cudaStream_t st = as_stream(stream);
    if (src_dt == DT_F32 && dst_dt == DT_F32) return launch_softmax<float, float>(src, dst, rows, cols, st);
    if (src_dt == DT_BF16 && dst_dt == DT_BF16) return launch_softmax<uint16_t, uint16_t>(src, dst, rows, cols, st);
    if (src_dt == DT_F32 && dst_dt == DT_BF16) return launch_softmax<float, uint16_t>(src, dst, rows, cols, st);
    if (src_dt == DT_BF16 && dst_dt == DT_F32) return launch_softmax<uint16_t, float>(src, dst, rows, cols, st);
    return fail(cudaErrorInvalidValue, "softmax_rows: unsupported dtypes %d -> %d", src_dt, dst_dt);
}

int bee_b200_softmax_rows(int dt, const void* src, void* dst, size_t rows, size_t cols, bee_b200_stream_t stream) {
    return bee_b200_softmax_rows_to(dt, src, dt, dst, rows, cols, stream);
}

int bee_b200_rms_norm_rows(int dt, const void* x, const void* w, void* y, size_t rows, size_t cols, float eps,
                           bee_b200_stream_t stream) {
    if (rows == 0) return ok();
    if (cols == 0) return fail(cudaErrorInvalidValue, "rms_norm_rows: zero columns");
    if (!x || !w || !y) return fail(cudaErrorInvalidValue, "rms_norm_rows: null pointer");
    if (!(eps >= 0.f)) return fail(cudaErrorInvalidValue, "rms_norm_rows: eps must be >= 0");
    cudaStream_t st = as_stream(stream);
    RopeArgs none{0, 1, 2, 0, 0.0};
    if (dt == DT_F32) return launch_norm_rope<float, true, false>(x, w, y, rows, cols, eps, none, st);
    if (dt == DT_BF16) return launch_norm_rope<uint16_t, true, false>(x, w, y, rows, cols, eps, none, st);
    return fail(cudaErrorInvalidValue, "rms_norm_rows: unsupported dtype %d", dt);
}

int bee_b200_rope(int dt, const void* x, void* y, size_t rows, size_t seq, size_t heads, size_t head_dim, double theta,
                  size_t pos_offset, bee_b200_stream_t stream) {
    if (rows == 0) return ok();
    if (int rc = check_rope(rows, seq, heads, head_dim, theta, "rope")) return rc;
    if (!x || !y) return fail(cudaErrorInvalidValue, "rope: null pointer");
    cudaStream_t st = as_stream(stream);
    RopeArgs ra{1, seq, head_dim, pos_offset, log(theta)};
    const size_t cols = heads * head_dim;
    if (dt == DT_F32) return launch_norm_rope<float, false, true>(x, x, y, rows, cols, 0.f, ra, st);
    if (dt == DT_BF16) return launch_norm_rope<uint16_t, false, true>(x, x, y, rows, cols, 0.f, ra, st);
    return fail(cudaErrorInvalidValue, "rope: unsupported dtype %d", dt);
}

int bee_b200_rms_norm_rope(int dt, const void* x, const void* w, void* y, size_t rows, size_t seq, size_t heads,
                           size_t head_dim, float eps, double theta, size_t pos_offset, bee_b200_stream_t stream) {
    if (rows == 0) return ok();
    if (int rc = check_rope(rows, seq, heads, head_dim, theta, "rms_norm_rope")) return rc;
    if (!x || !w || !y) return fail(cudaErrorInvalidValue, "rms_norm_rope: null pointer");
    if (!(eps >= 0.f)) return fail(cudaErrorInvalidValue, "rms_norm_rope: eps must be >= 0");
    cudaStream_t st = as_stream(stream);
    RopeArgs ra{1, seq, head_dim, pos_offset, log(theta)};
    const size_t cols = heads * head_dim;
    if (dt == DT_F32) return launch_norm_rope<float, true, true>(x, w, y, rows, cols, eps, ra, st);
    if (dt == DT_BF16) return launch_norm_rope<uint16_t, true, true>(x, w, y, rows, cols, eps, ra, st);
    return fail(cudaErrorInvalidValue, "rms_norm_rope: unsupported dtype %d", dt);
}

}  // extern "C"
