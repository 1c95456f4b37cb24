// Dense GEMM: C = alpha * A . op(B), batched.
//
// Replaces the reference's matmul kernels K1-K3 (Bee/CUDA/Ops/Matmul.cu:29-122,
// Bee/CUDA/Ops/MatmulCutlass.cu:49-105, Bee/CUDA/Ops/MatmulTmaWmma.cu:77-211),
// none of which has an sm_100 path.
//
// bf16 path (the hot one): a persistent, warp-specialised tcgen05 kernel.
//   * warp 0 — TMA producer: 128x64 A tiles and 64xBN B tiles, 128-byte
//     swizzle, into a STAGES-deep shared-memory ring guarded by mbarriers
//     (no cluster multicast anywhere: the code is safe on any number of GPUs);
//   * warp 1 — MMA issuer: tcgen05.mma.cta_group::1.kind::f16 (M=128, N=BN,
//     K=16), fp32 accumulators in TMEM, double-buffered (2 x BN columns) so the
//     epilogue of tile i overlaps the main loop of tile i+1; tcgen05.commit
//     releases ring slots and hands finished accumulators over;
//   * warps 2-5 — epilogue: tcgen05.ld 32 columns at a time, scale by alpha,
//     convert (bf16 RNE or fp32) and store.
//   Tiles are visited in a grouped raster (16 M-blocks per group) so the ~148
//   tiles in flight share A and B panels in L2.  Every mbarrier wait is
//   bounded: a wait that gives up records a code in the device status word,
//   raises a CTA-wide abort flag, and the CTA drains and frees TMEM.
//
// Other dtypes (F32 for the parity config, F64, I32, I64) and bf16 shapes the
// TMA path cannot express (row strides not a multiple of 16 bytes) use a
// shared-memory tiled SIMT kernel with boundary checks.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"
#include "sm100.cuh"

namespace bee_b200 {

using namespace sm100;

// Device status word: code of the first bounded wait that gave up (0 = none).
__device__ int g_gemm_status = 0;

constexpr int kMaxPeers = 8;

struct GemmParams {
    int M, N, K;
    int m_tiles, n_tiles, tiles_per_batch, total_tiles;
    int num_kb;
    long long ldc;             // elements
    long long batch_stride_c;  // elements
    float alpha;
    void* C;
    int c_vec;                 // C, ldc and batch_stride_c allow 16-byte stores
    int in_f16;                // A and B are f16 (else bf16); sets the MMA's operand format
    int out_f16;               // 16-bit C is f16 (else bf16)
    // split-K scatter mode: fp32 256x256 partial tiles go to the receive buffer of
    // tile owner (tile % world), slot `rank`, over NVLink peer stores
    float* peer_recv[kMaxPeers];
    int world, rank, owned;  // owned = tiles per owner = ceil(total_tiles / world)
};

// 1-SM tiles: 128xBN.  BN = 128 streams K in 128-wide stages (every TMA box
// 16 KiB, 3 stages); BN = 256 keeps 64-wide stages so that 4 stages fit.
template <int BN> struct TileCfg {
    static constexpr int BM = 128;
    static constexpr int BK = (BN == 128) ? 128 : 64;
    static constexpr int K_HALF = BM * 64 * 2;  // one 128-row x 64-K swizzled block (16 KiB)
    static constexpr int A_BYTES = BM * BK * 2;
    static constexpr int B_BYTES = BN * BK * 2;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int STAGES = (BN == 256) ? 4 : 3;
    static constexpr int SMEM = STAGES * STAGE_BYTES + 1024;
    static constexpr uint32_t TMEM_COLS = 2 * BN;
    static constexpr int THREADS = 192;
};

constexpr int kGroupM = 16;

__device__ __forceinline__ void grouped_tile(int t, int m_tiles, int n_tiles, int& mb, int& nb) {
    const int per_group = kGroupM * n_tiles;
    const int group = t / per_group;
    const int first_m = group * kGroupM;
    const int gsize = min(m_tiles - first_m, kGroupM);
    const int r = t - group * per_group;
    mb = first_m + r % gsize;
    nb = r / gsize;
}

// K order of a persistent CTA's i-th tile: forward for even i, backward for odd
// i.  The CTAs move through their tiles together, so the tiles of one wave
// start on the K blocks the previous wave (which shares their A panels under
// the grouped raster) read last, while those are still in L2.  The MMA side
// accumulates in iteration order whatever the coordinate.
__device__ __forceinline__ int k_block(int kb, int i, int num_kb) { return (i & 1) ? num_kb - 1 - kb : kb; }

__device__ __forceinline__ void tile_coords(int tile, const GemmParams& p, int& b, int& mb, int& nb) {
    b = tile / p.tiles_per_batch;
    grouped_tile(tile - b * p.tiles_per_batch, p.m_tiles, p.n_tiles, mb, nb);
}

// Stores one thread's 32 consecutive accumulator columns (row `row_off`,
// columns col0..col0+31) scaled by alpha, as fp32 or bf16 (RNE), with 16-byte
// stores when the whole chunk is in range and rows are 16-byte aligned.
template <bool OUT_F32>
__device__ __forceinline__ void store_chunk32(const GemmParams& p, const uint32_t (&r)[32], bool row_ok,
                                              long long row_off, int col0) {
    if (!row_ok || col0 >= p.N) return;
    if constexpr (OUT_F32) {
        float* dst = static_cast<float*>(p.C) + row_off + col0;
        if (col0 + 32 <= p.N && p.c_vec) {
#pragma unroll
            for (int v = 0; v < 8; ++v)
                reinterpret_cast<float4*>(dst)[v] =
                    make_float4(__uint_as_float(r[4 * v]) * p.alpha, __uint_as_float(r[4 * v + 1]) * p.alpha,
                                __uint_as_float(r[4 * v + 2]) * p.alpha, __uint_as_float(r[4 * v + 3]) * p.alpha);
        } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
                if (col0 + j < p.N) dst[j] = __uint_as_float(r[j]) * p.alpha;
        }
    } else {
        uint16_t* dst = static_cast<uint16_t*>(p.C) + row_off + col0;
        // 16-bit output: bf16 or f16, both round-to-nearest-even (uniform branch per chunk)
        auto pack = [&](int j) {
            const float lo = __uint_as_float(r[j]) * p.alpha, hi = __uint_as_float(r[j + 1]) * p.alpha;
            return p.out_f16 ? pack_f16x2(lo, hi) : pack_bf16x2(lo, hi);
        };
        if (col0 + 32 <= p.N && p.c_vec) {
#pragma unroll
            for (int v = 0; v < 4; ++v)
                reinterpret_cast<uint4*>(dst)[v] = make_uint4(pack(8 * v), pack(8 * v + 2), pack(8 * v + 4), pack(8 * v + 6));
        } else {
#pragma unroll
            for (int j = 0; j < 32; j += 2) {
                const uint32_t w = pack(j);
                if (col0 + j < p.N) dst[j] = static_cast<uint16_t>(w & 0xffffu);
                if (col0 + j + 1 < p.N) dst[j + 1] = static_cast<uint16_t>(w >> 16);
            }
        }
    }
}

template <int BN, bool B_KMAJOR, bool OUT_F32>
__global__ void __launch_bounds__(192, 1) gemm_bf16_tcgen05_kernel(const __grid_constant__ CUtensorMap tmA,
                                                                   const __grid_constant__ CUtensorMap tmB,
                                                                   const GemmParams p) {
    using Cfg = TileCfg<BN>;
    constexpr int STAGES = Cfg::STAGES;
    extern __shared__ uint8_t smem_raw[];
    __shared__ __align__(8) uint64_t full_bar[STAGES];
    __shared__ __align__(8) uint64_t empty_bar[STAGES];
    __shared__ __align__(8) uint64_t tfull_bar[2];
    __shared__ __align__(8) uint64_t tempty_bar[2];
    __shared__ __align__(8) uint64_t done_bar;
    __shared__ uint32_t tmem_base_sh;
    __shared__ int abort_sh;

    // 128-byte swizzled tiles need 1024-byte alignment
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    volatile int* abort_flag = &abort_sh;
    int* status = &g_gemm_status;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&empty_bar[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&tfull_bar[a], 1);
            mbar_init(&tempty_bar[a], 128);
        }
        mbar_init(&done_bar, 1);
        abort_sh = 0;
        fence_mbar_init();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch(&tmA);
        tma_prefetch(&tmB);
    }
    if (warp == 1) tmem_alloc<Cfg::TMEM_COLS>(&tmem_base_sh);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = tmem_base_sh;
    // the launch may overlap the previous kernel's tail: no global access before it has completed
    pdl_wait();
    pdl_trigger();

    if (warp == 0) {
        // ------------------------------------------------ TMA producer
        int stage = 0;
        uint32_t phase = 0;
        long long issued = 0;
        for (int tile = blockIdx.x; tile < p.total_tiles; tile += gridDim.x) {
            if (__any_sync(0xffffffffu, *abort_flag != 0)) break;
            int b, mb, nb;
            tile_coords(tile, p, b, mb, nb);
            for (int kb = 0; kb < p.num_kb; ++kb) {
                bool ok = true;
                if (lane == 0) ok = mbar_wait(&empty_bar[stage], phase ^ 1u, abort_flag, status, 1);
                ok = __shfl_sync(0xffffffffu, ok, 0);
                if (!ok) break;
                if (lane == 0) {
                    uint8_t* sa = smem + stage * Cfg::STAGE_BYTES;
                    uint8_t* sb = sa + Cfg::A_BYTES;
                    mbar_arrive_expect_tx(&full_bar[stage], Cfg::STAGE_BYTES);
                    const int k0 = k_block(kb, tile / static_cast<int>(gridDim.x), p.num_kb) * Cfg::BK;
#pragma unroll
                    for (int h = 0; h < Cfg::BK / 64; ++h)
                        tma_load_3d(sa + h * Cfg::K_HALF, &tmA, &full_bar[stage], k0 + h * 64, mb * Cfg::BM, b);
                    if constexpr (B_KMAJOR) {
#pragma unroll
                        for (int h = 0; h < Cfg::BK / 64; ++h)
                            tma_load_3d(sb + h * (BN * 64 * 2), &tmB, &full_bar[stage], k0 + h * 64, nb * BN, b);
                    } else {
#pragma unroll
                        for (int j = 0; j < BN / 64; ++j)
                            tma_load_3d(sb + j * (64 * Cfg::BK * 2), &tmB, &full_bar[stage], nb * BN + j * 64, k0, b);
                    }
                }
                __syncwarp();
                ++issued;
                if (++stage == STAGES) {
                    stage = 0;
                    phase ^= 1u;
                }
            }
        }
        // Drain: the last (up to) STAGES loads must have landed before the CTA
        // may exit (normally the MMA warp has already consumed them).
        if (lane == 0) {
            const long long first = issued > STAGES ? issued - STAGES : 0;
            for (long long it = first; it < issued; ++it)
                mbar_wait(&full_bar[it % STAGES], static_cast<uint32_t>((it / STAGES) & 1), abort_flag, status, 2,
                          200000000ull);
        }
        __syncwarp();
    } else if (warp == 1) {
        // ------------------------------------------------ MMA issuer
        const uint32_t idesc = idesc_f16_f32(128, BN, !B_KMAJOR, p.in_f16 != 0);
        int stage = 0;
        uint32_t phase = 0;
        int local = 0;
        bool issued_any = false;
        for (int tile = blockIdx.x; tile < p.total_tiles; tile += gridDim.x, ++local) {
            if (__any_sync(0xffffffffu, *abort_flag != 0)) break;
            const int acc = local & 1;
            const uint32_t acc_phase = static_cast<uint32_t>((local >> 1) & 1);
            bool ok = true;
            if (lane == 0) ok = mbar_wait(&tempty_bar[acc], acc_phase ^ 1u, abort_flag, status, 3);
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) break;
            tc_fence_after();
            const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
            for (int kb = 0; kb < p.num_kb; ++kb) {
                if (lane == 0) ok = mbar_wait(&full_bar[stage], phase, abort_flag, status, 4);
                ok = __shfl_sync(0xffffffffu, ok, 0);
                if (!ok) break;
                tc_fence_after();
                if (lane == 0) {
                    const uint32_t a_base = smem_u32(smem + stage * Cfg::STAGE_BYTES);
                    const uint32_t b_base = a_base + Cfg::A_BYTES;
#pragma unroll
                    for (int k = 0; k < Cfg::BK / 16; ++k) {
                        // K-major tiles: 64-wide K blocks, 32 bytes per 16-K step inside a block
                        const uint32_t a_off = (k / 4) * Cfg::K_HALF + (k % 4) * 32;
                        const uint32_t b_off = (k / 4) * (BN * 64 * 2) + (k % 4) * 32;
                        const uint64_t adesc = sdesc_sw128(a_base + a_off, 16, 1024);
                        const uint64_t bdesc = B_KMAJOR ? sdesc_sw128(b_base + b_off, 16, 1024)
                                                        : sdesc_sw128(b_base + k * 16 * 128, 64 * Cfg::BK * 2, 1024);
                        mma_f16_ss(d_tmem, adesc, bdesc, idesc, (kb | k) != 0 ? 1u : 0u);
                    }
                    mma_commit(&empty_bar[stage]);
                    issued_any = true;
                }
                __syncwarp();
                if (++stage == STAGES) {
                    stage = 0;
                    phase ^= 1u;
                }
            }
            if (!ok) break;
            if (lane == 0) mma_commit(&tfull_bar[acc]);
            __syncwarp();
        }
        // every MMA this thread issued must be complete before TMEM is freed
        if (lane == 0 && issued_any) {
            mma_commit(&done_bar);
            mbar_wait(&done_bar, 0, abort_flag, status, 5, 200000000ull);
        }
        __syncwarp();
    } else {
        // ------------------------------------------------ epilogue (warps 2-5)
        const int q = warp & 3;  // TMEM lane quarter this warp may access
        int local = 0;
        for (int tile = blockIdx.x; tile < p.total_tiles; tile += gridDim.x, ++local) {
            if (__any_sync(0xffffffffu, *abort_flag != 0)) break;
            int b, mb, nb;
            tile_coords(tile, p, b, mb, nb);
            const int acc = local & 1;
            const uint32_t acc_phase = static_cast<uint32_t>((local >> 1) & 1);
            bool ok = mbar_wait(&tfull_bar[acc], acc_phase, abort_flag, status, 6);
            if (!__all_sync(0xffffffffu, ok)) break;
            tc_fence_after();
            const int row = mb * Cfg::BM + q * 32 + lane;
            const bool row_ok = row < p.M;
            const long long row_off = static_cast<long long>(b) * p.batch_stride_c + static_cast<long long>(row) * p.ldc;
#pragma unroll 1
            for (int c = 0; c < BN / 32; ++c) {
                uint32_t r[32];
                tmem_ld_32x32b_x32(tmem_base + static_cast<uint32_t>(acc * BN + c * 32) +
                                       (static_cast<uint32_t>(q * 32) << 16),
                                   r);
                tmem_ld_wait();
                store_chunk32<OUT_F32>(p, r, row_ok, row_off, nb * BN + c * 32);
            }
            tc_fence_before();
            mbar_arrive(&tempty_bar[acc]);
        }
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc<Cfg::TMEM_COLS>(tmem_base);
}

// ---------------------------------------------------------------- 2-SM variant
// Two CTAs of a (2,1,1) cluster compute one 256x256 output tile with
// tcgen05.mma.cta_group::2 (M=256, N=256, K=16): each CTA TMA-loads its own
// 128 rows of A and its own 128 columns of B (no multicast), so per SM the
// operand traffic per MMA is 2/3 of the 1-SM 128x256 tile.  Both CTAs' loads
// complete on the leader CTA's (rank 0) full barrier, armed by the leader for
// both halves; only the leader issues MMAs; each commit multicasts its arrive
// to both CTAs (ring slots free, accumulator ready); both CTAs' epilogues read
// their own 128 TMEM lanes and arrive remotely on the leader's
// accumulator-empty barrier.  All waits are bounded as in the 1-SM kernel.
// BK = 128 per stage: every TMA box is 16 KiB (A: two 128x64 K-halves; B:
// two 64-wide column chunks of 128 K-rows, or two 128x64 K-halves when B is
// K-major) — fewer, larger boxes deliver more L2->SMEM bandwidth than 8 KiB ones.
struct Pair2Cfg {
    static constexpr int BM = 256, BN = 256, BK = 128;
    static constexpr int A_HALF = 128 * 64 * 2;   // one 128-row x 64-K swizzled half (16 KiB)
    static constexpr int A_BYTES = 128 * BK * 2;  // this CTA's 128 rows
    static constexpr int B_BYTES = 128 * BK * 2;  // this CTA's 128 columns
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int STAGES = 3;
    static constexpr int SMEM = STAGES * STAGE_BYTES + 1024;
    static constexpr uint32_t TMEM_COLS = 512;
};

template <bool B_KMAJOR, bool OUT_F32, bool SCATTER = false>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(192, 1)
    gemm_bf16_tcgen05_2sm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                                 const GemmParams p) {
    using Cfg = Pair2Cfg;
    constexpr int STAGES = Cfg::STAGES;
    extern __shared__ uint8_t smem_raw[];
    __shared__ __align__(8) uint64_t full_bar[STAGES];
    __shared__ __align__(8) uint64_t empty_bar[STAGES];
    __shared__ __align__(8) uint64_t tfull_bar[2];
    __shared__ __align__(8) uint64_t tempty_bar[2];
    __shared__ __align__(8) uint64_t done_bar;
    __shared__ uint32_t tmem_base_sh;
    __shared__ int abort_sh;

    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    volatile int* abort_flag = &abort_sh;
    int* status = &g_gemm_status;
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();  // 0 = leader
    const bool leader = rank == 0;
    const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&empty_bar[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&tfull_bar[a], 1);
            mbar_init(&tempty_bar[a], 8);  // 4 epilogue warps in each CTA of the pair
        }
        mbar_init(&done_bar, 1);
        abort_sh = 0;
        fence_mbar_init();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch(&tmA);
        tma_prefetch(&tmB);
    }
    if (warp == 1) tmem_alloc_pair<Cfg::TMEM_COLS>(&tmem_base_sh);
    tc_fence_before();
    __syncthreads();
    cluster_sync();  // both CTAs' barriers and TMEM exist before any cross-CTA traffic
    tc_fence_after();
    const uint32_t tmem_base = tmem_base_sh;

    if (warp == 0) {
        // ------------------------------------------------ TMA producer (both CTAs)
        int stage = 0;
        uint32_t phase = 0;
        long long issued = 0;
        for (int tile = pair; tile < p.total_tiles; tile += npairs) {
            if (__any_sync(0xffffffffu, *abort_flag != 0)) break;
            int b, mb, nb;
            tile_coords(tile, p, b, mb, nb);
            for (int kb = 0; kb < p.num_kb; ++kb) {
                bool ok = true;
                if (lane == 0) ok = mbar_wait(&empty_bar[stage], phase ^ 1u, abort_flag, status, 11);
                ok = __shfl_sync(0xffffffffu, ok, 0);
                if (!ok) break;
                if (lane == 0) {
                    uint8_t* sa = smem + stage * Cfg::STAGE_BYTES;
                    uint8_t* sb = sa + Cfg::A_BYTES;
                    const uint32_t full_leader = mapa_shared(smem_u32(&full_bar[stage]), 0);
                    if (leader) mbar_arrive_expect_tx(&full_bar[stage], 2 * Cfg::STAGE_BYTES);
                    const int m0 = mb * Cfg::BM + static_cast<int>(rank) * 128;
                    const int n0 = nb * Cfg::BN + static_cast<int>(rank) * 128;
                    const int k0 = k_block(kb, tile / npairs, p.num_kb) * Cfg::BK;
                    tma_load_3d_pair(sa, &tmA, full_leader, k0, m0, b);
                    tma_load_3d_pair(sa + Cfg::A_HALF, &tmA, full_leader, k0 + 64, m0, b);
                    if constexpr (B_KMAJOR) {
                        tma_load_3d_pair(sb, &tmB, full_leader, k0, n0, b);
                        tma_load_3d_pair(sb + Cfg::A_HALF, &tmB, full_leader, k0 + 64, n0, b);
                    } else {
                        tma_load_3d_pair(sb, &tmB, full_leader, n0, k0, b);
                        tma_load_3d_pair(sb + 64 * Cfg::BK * 2, &tmB, full_leader, n0 + 64, k0, b);
                    }
                }
                __syncwarp();
                ++issued;
                if (++stage == STAGES) {
                    stage = 0;
                    phase ^= 1u;
                }
            }
        }
        // Drain: the leader's full barriers count both CTAs' loads, so the
        // leader waits for the last (up to) STAGES of them before the final
        // cluster barrier lets either CTA exit.
        if (lane == 0 && leader) {
            const long long first = issued > STAGES ? issued - STAGES : 0;
            for (long long it = first; it < issued; ++it)
                mbar_wait(&full_bar[it % STAGES], static_cast<uint32_t>((it / STAGES) & 1), abort_flag, status, 12,
                          200000000ull);
        }
        __syncwarp();
    } else if (warp == 1) {
        // ------------------------------------------------ MMA issuer (leader CTA only)
        if (leader) {
            const uint32_t idesc = idesc_f16_f32(256, 256, !B_KMAJOR, p.in_f16 != 0);
            int stage = 0;
            uint32_t phase = 0;
            int local = 0;
            bool issued_any = false;
            for (int tile = pair; tile < p.total_tiles; tile += npairs, ++local) {
                if (__any_sync(0xffffffffu, *abort_flag != 0)) break;
                const int acc = local & 1;
                const uint32_t acc_phase = static_cast<uint32_t>((local >> 1) & 1);
                bool ok = true;
                if (lane == 0) ok = mbar_wait_cluster(&tempty_bar[acc], acc_phase ^ 1u, abort_flag, status, 13);
                ok = __shfl_sync(0xffffffffu, ok, 0);
                if (!ok) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * Cfg::BN);
                for (int kb = 0; kb < p.num_kb; ++kb) {
                    if (lane == 0) ok = mbar_wait(&full_bar[stage], phase, abort_flag, status, 14);
                    ok = __shfl_sync(0xffffffffu, ok, 0);
                    if (!ok) break;
                    tc_fence_after();
                    if (lane == 0) {
                        const uint32_t a_base = smem_u32(smem + stage * Cfg::STAGE_BYTES);
                        const uint32_t b_base = a_base + Cfg::A_BYTES;
#pragma unroll
                        for (int k = 0; k < Cfg::BK / 16; ++k) {
                            // K-major tiles: 64-wide K halves of 16 KiB, 32 bytes per 16-K step inside a half
                            const uint32_t kmaj = (k / 4) * Cfg::A_HALF + (k % 4) * 32;
                            const uint64_t adesc = sdesc_sw128(a_base + kmaj, 16, 1024);
                            const uint64_t bdesc = B_KMAJOR ? sdesc_sw128(b_base + kmaj, 16, 1024)
                                                            : sdesc_sw128(b_base + k * 16 * 128, 64 * Cfg::BK * 2, 1024);
                            mma_f16_ss_pair(d_tmem, adesc, bdesc, idesc, (kb | k) != 0 ? 1u : 0u);
                        }
                        mma_commit_pair(&empty_bar[stage], 0x3);
                        issued_any = true;
                    }
                    __syncwarp();
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (!ok) break;
                if (lane == 0) mma_commit_pair(&tfull_bar[acc], 0x3);
                __syncwarp();
            }
            if (lane == 0 && issued_any) {
                mma_commit_pair(&done_bar, 0x1);
                mbar_wait(&done_bar, 0, abort_flag, status, 15, 200000000ull);
            }
            __syncwarp();
        }
    } else {
        // ------------------------------------------------ epilogue (warps 2-5, both CTAs)
        const int q = warp & 3;
        const uint32_t tempty_leader0 = mapa_shared(smem_u32(&tempty_bar[0]), 0);
        const uint32_t tempty_leader1 = mapa_shared(smem_u32(&tempty_bar[1]), 0);
        int local = 0;
        for (int tile = pair; tile < p.total_tiles; tile += npairs, ++local) {
            if (__any_sync(0xffffffffu, *abort_flag != 0)) break;
            int b, mb, nb;
            tile_coords(tile, p, b, mb, nb);
            const int acc = local & 1;
            const uint32_t acc_phase = static_cast<uint32_t>((local >> 1) & 1);
            bool ok = mbar_wait(&tfull_bar[acc], acc_phase, abort_flag, status, 16);
            if (!__all_sync(0xffffffffu, ok)) break;
            tc_fence_after();
            const int row = mb * Cfg::BM + static_cast<int>(rank) * 128 + q * 32 + lane;
            const bool row_ok = row < p.M;
            const long long row_off = static_cast<long long>(b) * p.batch_stride_c + static_cast<long long>(row) * p.ldc;
#pragma unroll 1
            for (int c = 0; c < Cfg::BN / 32; ++c) {
                uint32_t r[32];
                tmem_ld_32x32b_x32(tmem_base + static_cast<uint32_t>(acc * Cfg::BN + c * 32) +
                                       (static_cast<uint32_t>(q * 32) << 16),
                                   r);
                tmem_ld_wait();
                if constexpr (SCATTER) {
                    // fp32 partial straight into the owner's slot for this rank (peer stores over
                    // NVLink).  Slot layout: float4 (row r, columns 4g..4g+3) at index g * 256 + r,
                    // so the 32 lanes (32 consecutive rows) of each store cover 512 contiguous bytes.
                    float4* dst = reinterpret_cast<float4*>(
                                      p.peer_recv[tile % p.world] +
                                      (static_cast<size_t>(p.rank) * p.owned + tile / p.world) * (Cfg::BM * Cfg::BN)) +
                                  static_cast<int>(rank) * 128 + q * 32 + lane;
#pragma unroll
                    for (int v = 0; v < 8; ++v)
                        dst[(c * 8 + v) * 256] = make_float4(__uint_as_float(r[4 * v]), __uint_as_float(r[4 * v + 1]),
                                                             __uint_as_float(r[4 * v + 2]), __uint_as_float(r[4 * v + 3]));
                } else {
                    store_chunk32<OUT_F32>(p, r, row_ok, row_off, nb * Cfg::BN + c * 32);
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(acc ? tempty_leader1 : tempty_leader0);
        }
        // peer stores must be visible to the other GPUs before anything later in the stream
        if constexpr (SCATTER) __threadfence_system();
    }

    tc_fence_before();
    __syncthreads();
    cluster_sync();  // no CTA leaves while its peer may still touch its barriers or shared memory
    tc_fence_after();
    if (warp == 1) tmem_dealloc_pair<Cfg::TMEM_COLS>(tmem_base);
}

// ---------------------------------------------------------------- split-K reduce
// Tiles are numbered in the GEMM's grouped raster order (grouped_tile).
// Rank `rank` owns tiles t = rank + i * world.  Its receive buffer holds, per
// source rank s, the fp32 partial of every owned tile: slot (s, i) at
// (s * owned + i) * 65536 floats, float4 (row r, columns 4g..4g+3) at g * 256 + r.
// One CTA reduces a 32-row band of one tile: it sums the world slots in fixed
// order (slot 0, 1, ...) with coalesced reads, transposes the band through
// shared memory and writes bf16 rows, 512 contiguous bytes per warp store, into
// every rank's C (local and peer stores over NVLink).
struct SplitKReduceParams {
    int M, N, m_tiles, n_tiles, total_tiles, world, rank, owned;
    long long ldc;
    uint16_t* c_peer[kMaxPeers];
};

__global__ void __launch_bounds__(256) splitk_reduce_kernel(const float* __restrict__ recv, const SplitKReduceParams p) {
    constexpr int BAND = 32, PITCH = 256 + 4;  // pitch: float4 stores of 8 consecutive rows hit distinct banks
    __shared__ __align__(16) float band[BAND * PITCH];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int units = p.owned * (256 / BAND);
    for (int u = blockIdx.x; u < units; u += gridDim.x) {
        const int i = u / (256 / BAND), r0 = (u % (256 / BAND)) * BAND;
        const int tile = p.rank + i * p.world;
        if (tile >= p.total_tiles) break;  // owned tiles are visited in increasing order
        int mb, nb;
        grouped_tile(tile, p.m_tiles, p.n_tiles, mb, nb);  // the GEMM's tile order
        // sum: thread (warp w, lane l) handles column groups g = k * 8 + w of row r0 + l
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const int g = k * 8 + warp;
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int s = 0; s < p.world; ++s) {
                const float4* src = reinterpret_cast<const float4*>(recv + (static_cast<size_t>(s) * p.owned + i) * 65536);
                const float4 v = __ldcs(src + g * 256 + r0 + lane);
                acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
            }
            *reinterpret_cast<float4*>(&band[lane * PITCH + g * 4]) = acc;
        }
        __syncthreads();
        // write: 32 rows x 32 chunks of 8 columns; a warp covers one row
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int f = k * 256 + tid;
            const int rr = f >> 5, c8 = f & 31;
            const int row = mb * 256 + r0 + rr, col = nb * 256 + c8 * 8;
            if (row < p.M && col < p.N) {
                const float4 a = *reinterpret_cast<const float4*>(&band[rr * PITCH + c8 * 8]);
                const float4 b = *reinterpret_cast<const float4*>(&band[rr * PITCH + c8 * 8 + 4]);
                const uint4 o = make_uint4(pack_bf16x2(a.x, a.y), pack_bf16x2(a.z, a.w), pack_bf16x2(b.x, b.y),
                                           pack_bf16x2(b.z, b.w));
                const size_t off = static_cast<size_t>(row) * p.ldc + col;
                if (col + 8 <= p.N) {
                    for (int r = 0; r < p.world; ++r) *reinterpret_cast<uint4*>(p.c_peer[r] + off) = o;
                } else {
                    const uint16_t* h = reinterpret_cast<const uint16_t*>(&o);
                    for (int r = 0; r < p.world; ++r)
                        for (int e = 0; e < 8 && col + e < p.N; ++e) p.c_peer[r][off + e] = h[e];
                }
            }
        }
        __syncthreads();
    }
    __threadfence_system();  // peer stores visible to the other GPUs before later stream work
}

// ---------------------------------------------------------------- SIMT GEMM

template <typename T> struct Acc { using type = T; };
template <> struct Acc<uint16_t> { using type = float; };  // bf16 bits
template <> struct Acc<__half> { using type = float; };

template <typename T> __device__ __forceinline__ typename Acc<T>::type ld_as_acc(const T* p) { return *p; }
template <> __device__ __forceinline__ float ld_as_acc<uint16_t>(const uint16_t* p) {
    return __uint_as_float(static_cast<uint32_t>(*p) << 16);
}
template <> __device__ __forceinline__ float ld_as_acc<__half>(const __half* p) { return __half2float(*p); }

template <typename T, typename TO> __device__ __forceinline__ void st_from_acc(TO* p, typename Acc<T>::type v, float alpha) {
    if constexpr (std::is_same_v<TO, uint16_t>) {
        __nv_bfloat16 h = __float2bfloat16_rn(static_cast<float>(v) * alpha);
        *p = *reinterpret_cast<uint16_t*>(&h);
    } else if constexpr (std::is_same_v<TO, __half>) {
        *p = __float2half_rn(static_cast<float>(v) * alpha);
    } else if constexpr (std::is_floating_point_v<TO>) {
        *p = static_cast<TO>(v * static_cast<typename Acc<T>::type>(alpha));
    } else {
        *p = static_cast<TO>(v);
    }
}

template <typename T> __device__ __forceinline__ typename Acc<T>::type fma_acc(typename Acc<T>::type a, typename Acc<T>::type b,
                                                                              typename Acc<T>::type c) {
    using A = typename Acc<T>::type;
    if constexpr (std::is_same_v<A, int32_t>)
        return static_cast<int32_t>(static_cast<uint32_t>(c) + static_cast<uint32_t>(a) * static_cast<uint32_t>(b));
    else if constexpr (std::is_same_v<A, int64_t>)
        return static_cast<int64_t>(static_cast<uint64_t>(c) + static_cast<uint64_t>(a) * static_cast<uint64_t>(b));
    else
        return fma(a, b, c);
}

// 64x64 output tile per 256-thread CTA, 4x4 outputs per thread (strided by 16
// so shared-memory reads are broadcasts / conflict-free), BK = 16.
template <typename T, typename TO>
__global__ void __launch_bounds__(256) gemm_simt_kernel(const T* __restrict__ A, const T* __restrict__ B,
                                                        TO* __restrict__ C, int M, int N, int K, long long lda,
                                                        long long ldb, long long ldc, long long sA, long long sB,
                                                        long long sC, int b_trans, float alpha) {
    using AT = typename Acc<T>::type;
    constexpr int BM = 64, BN = 64, BK = 16;
    __shared__ AT As[BK][BM + 1];
    __shared__ AT Bs[BK][BN + 1];
    const int bz = blockIdx.z;
    A += bz * sA;
    B += bz * sB;
    C += bz * sC;
    const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    AT acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = AT(0);
    for (int k0 = 0; k0 < K; k0 += BK) {
#pragma unroll
        for (int l = 0; l < 4; ++l) {
            const int idx = threadIdx.x + l * 256;
            const int r = idx / BK, k = idx % BK;  // A: row r, col k
            const int gm = m0 + r, gk = k0 + k;
            As[k][r] = (gm < M && gk < K) ? ld_as_acc(A + static_cast<long long>(gm) * lda + gk) : AT(0);
            if (!b_trans) {
                const int kk = idx / BN, n = idx % BN;  // B [K, N]
                const int gk2 = k0 + kk, gn = n0 + n;
                Bs[kk][n] = (gk2 < K && gn < N) ? ld_as_acc(B + static_cast<long long>(gk2) * ldb + gn) : AT(0);
            } else {
                const int n = idx / BK, kk = idx % BK;  // B stored [N, K]
                const int gk2 = k0 + kk, gn = n0 + n;
                Bs[kk][n] = (gk2 < K && gn < N) ? ld_as_acc(B + static_cast<long long>(gn) * ldb + gk2) : AT(0);
            }
        }
        __syncthreads();
#pragma unroll
        for (int k = 0; k < BK; ++k) {
            AT a[4], bv[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) a[i] = As[k][ty + 16 * i];
#pragma unroll
            for (int j = 0; j < 4; ++j) bv[j] = Bs[k][tx + 16 * j];
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fma_acc<T>(a[i], bv[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int gm = m0 + ty + 16 * i, gn = n0 + tx + 16 * j;
            if (gm < M && gn < N) st_from_acc<T, TO>(C + static_cast<long long>(gm) * ldc + gn, acc[i][j], alpha);
        }
}

// ---------------------------------------------------------------- host side

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

// 3-D tensor map of 16-bit elements (bf16, or f16 when `f16`) {inner, outer,
// batch} with 128-byte swizzle.
static int make_map(CUtensorMap* map, const void* ptr, uint64_t inner, uint64_t outer, uint64_t batch,
                    uint64_t row_stride, uint64_t batch_stride, uint32_t box_inner, uint32_t box_outer,
                    bool f16 = false) {
    auto enc = encode_fn();
    if (!enc) return fail(cudaErrorNotSupported, "bmm: cuTensorMapEncodeTiled unavailable");
    cuuint64_t dims[3] = {inner, outer, batch};
    cuuint64_t strides[2] = {row_stride * 2, batch_stride * 2};
    cuuint32_t box[3] = {box_inner, box_outer, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = enc(map, f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3,
                     const_cast<void*>(ptr), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(cudaErrorInvalidValue, "bmm: tensor map encoding failed (CUresult %d)", int(r));
    return 0;
}

template <int BN, bool B_KMAJOR, bool OUT_F32>
static int launch_tc(const CUtensorMap& ta, const CUtensorMap& tb, const GemmParams& p, cudaStream_t st) {
    using Cfg = TileCfg<BN>;
    auto kern = gemm_bf16_tcgen05_kernel<BN, B_KMAJOR, OUT_F32>;
    static SmemLimit smem_limit;
    if (int rc = smem_limit.ensure(kern, Cfg::SMEM, "bmm")) return rc;
    const int grid = p.total_tiles < sm_count() ? p.total_tiles : sm_count();
    launch_pdl(kern, grid, Cfg::THREADS, Cfg::SMEM, st, ta, tb, p);
    return launch_status("bmm(tcgen05)");
}

template <bool B_KMAJOR, bool OUT_F32>
static int dispatch_tc_bn(int bn, const CUtensorMap& ta, const CUtensorMap& tb, const GemmParams& p, cudaStream_t st) {
    return bn == 256 ? launch_tc<256, B_KMAJOR, OUT_F32>(ta, tb, p, st) : launch_tc<128, B_KMAJOR, OUT_F32>(ta, tb, p, st);
}

template <bool B_KMAJOR, bool OUT_F32>
static int launch_tc_pair(const CUtensorMap& ta, const CUtensorMap& tb, const GemmParams& p, cudaStream_t st) {
    auto kern = gemm_bf16_tcgen05_2sm_kernel<B_KMAJOR, OUT_F32>;
    static SmemLimit smem_limit;
    if (int rc = smem_limit.ensure(kern, Pair2Cfg::SMEM, "bmm")) return rc;
    const int pairs = sm_count() / 2;
    const int grid = 2 * (p.total_tiles < pairs ? p.total_tiles : pairs);
    kern<<<grid, 192, Pair2Cfg::SMEM, st>>>(ta, tb, p);
    return launch_status("bmm(tcgen05 2-SM)");
}

// Element strides of a batched product: A[b][m][k] at A + b*sa + m*lda + k,
// B[b][k][n] at B + b*sb + k*ldb + n (B^T: B[b][n][k] at B + b*sb + n*ldb + k),
// C[b][m][n] at C + b*sc + m*ldc + n.
struct BmmStrides {
    long long lda, ldb, ldc, sa, sb, sc;
};

static BmmStrides contiguous_strides(size_t M, size_t K, size_t N, int b_trans) {
    return BmmStrides{static_cast<long long>(K), static_cast<long long>(b_trans ? K : N), static_cast<long long>(N),
                      static_cast<long long>(M * K), static_cast<long long>(K * N), static_cast<long long>(M * N)};
}

// bf16 x bf16 -> (bf16 | fp32), or f16 x f16 -> (f16 | fp32) when dt_in is
// F16, on the tensor cores.  Returns 0, an error, or -1 when the shape or the
// strides cannot be expressed with TMA (the caller falls back to the SIMT kernel).
// M > 128 and N > 128 use 256x256 tiles on CTA pairs (cta_group::2); smaller
// problems use 128xBN tiles on single CTAs.  small_tiles: 128x128 tiles on single
// CTAs whatever the shape (more tiles for outputs that would not fill the GPU).
static int bmm_bf16_tc(int dt_out, const void* A, const void* B, void* C, size_t batch, size_t M, size_t K, size_t N,
                       int b_trans, float alpha, const BmmStrides& sd, cudaStream_t st, bool small_tiles = false,
                       int dt_in = DT_BF16) {
    const bool f16 = dt_in == DT_F16;
    // TMA: 16-byte aligned bases, row and batch strides multiples of 16 bytes (8 bf16), positive
    auto ok16 = [](long long v) { return v > 0 && v % 8 == 0 && v < (1ll << 36); };
    if (!ok16(sd.lda) || !ok16(sd.ldb) || !aligned16(A) || !aligned16(B)) return -1;
    if (batch > 1 && (!ok16(sd.sa) || !ok16(sd.sb))) return -1;
    if (M > (1u << 31) || N > (1u << 31) || K > (1u << 31) || batch > 65535) return -1;
    const uint64_t sa = batch > 1 ? static_cast<uint64_t>(sd.sa) : static_cast<uint64_t>(sd.lda) * M;
    const uint64_t sb = batch > 1 ? static_cast<uint64_t>(sd.sb) : static_cast<uint64_t>(sd.ldb) * (b_trans ? N : K);
    const int bn = N > 128 && !small_tiles ? 256 : 128;
    const bool pair = N > 128 && M > 128 && !small_tiles;
    CUtensorMap ta, tb;
    if (make_map(&ta, A, K, M, batch, static_cast<uint64_t>(sd.lda), sa, 64, 128, f16)) return -1;
    if (b_trans) {
        if (make_map(&tb, B, K, N, batch, static_cast<uint64_t>(sd.ldb), sb, 64,
                     pair ? 128u : static_cast<uint32_t>(bn), f16))
            return -1;
    } else {
        const uint32_t kbox = pair ? Pair2Cfg::BK : (bn == 256 ? TileCfg<256>::BK : TileCfg<128>::BK);
        if (make_map(&tb, B, N, K, batch, static_cast<uint64_t>(sd.ldb), sb, 64, kbox, f16)) return -1;
    }
    GemmParams p{};
    p.M = static_cast<int>(M);
    p.N = static_cast<int>(N);
    p.K = static_cast<int>(K);
    p.m_tiles = static_cast<int>(pair ? (M + 255) / 256 : (M + 127) / 128);
    p.n_tiles = static_cast<int>((N + bn - 1) / bn);
    p.tiles_per_batch = p.m_tiles * p.n_tiles;
    const long long total = static_cast<long long>(p.tiles_per_batch) * static_cast<long long>(batch);
    if (total > (1ll << 31) - 1) return -1;
    p.total_tiles = static_cast<int>(total);
    const size_t bk = pair ? Pair2Cfg::BK : (bn == 256 ? TileCfg<256>::BK : TileCfg<128>::BK);
    p.num_kb = static_cast<int>((K + bk - 1) / bk);
    p.ldc = sd.ldc;
    p.batch_stride_c = sd.sc;
    p.alpha = alpha;
    p.C = C;
    p.in_f16 = f16 ? 1 : 0;
    p.out_f16 = dt_out == DT_F16 ? 1 : 0;
    const bool f32 = dt_out == DT_F32;
    const long long vq = f32 ? 4 : 8;  // elements per 16 bytes
    p.c_vec = aligned16(C) && sd.ldc % vq == 0 && sd.sc % vq == 0 ? 1 : 0;
    if (pair) {
        if (b_trans) return f32 ? launch_tc_pair<true, true>(ta, tb, p, st) : launch_tc_pair<true, false>(ta, tb, p, st);
        return f32 ? launch_tc_pair<false, true>(ta, tb, p, st) : launch_tc_pair<false, false>(ta, tb, p, st);
    }
    if (b_trans) return f32 ? dispatch_tc_bn<true, true>(bn, ta, tb, p, st) : dispatch_tc_bn<true, false>(bn, ta, tb, p, st);
    return f32 ? dispatch_tc_bn<false, true>(bn, ta, tb, p, st) : dispatch_tc_bn<false, false>(bn, ta, tb, p, st);
}

template <typename T, typename TO>
static int launch_simt(const void* A, const void* B, void* C, size_t batch, size_t M, size_t K, size_t N, int b_trans,
                       float alpha, const BmmStrides& sd, cudaStream_t st) {
    if (M > (1u << 30) || N > (1u << 30) || K > (1u << 30) || batch > 65535)
        return fail(cudaErrorInvalidValue, "matmul: extent too large for the SIMT path");
    dim3 grid(static_cast<unsigned>((N + 63) / 64), static_cast<unsigned>((M + 63) / 64), static_cast<unsigned>(batch));
    if (grid.y > 65535) return fail(cudaErrorInvalidValue, "matmul: M too large for the SIMT path");
    gemm_simt_kernel<T, TO><<<grid, 256, 0, st>>>(static_cast<const T*>(A), static_cast<const T*>(B), static_cast<TO*>(C),
                                                  static_cast<int>(M), static_cast<int>(N), static_cast<int>(K), sd.lda,
                                                  sd.ldb, sd.ldc, sd.sa, sd.sb, sd.sc, b_trans, alpha);
    return launch_status("matmul(simt)");
}

// ---------------------------------------------------------------- fp32 matmul on the bf16 tensor cores
//
// Exact-enough fp32 products from bf16 MMAs.  Every fp32 value x is split into
// three bf16 pieces, hi = bf16(x), mid = bf16(x - hi), lo = bf16(x - hi - mid)
// (each subtraction is exact in fp32), so x = hi + mid + lo to within 2^-27 |x|.
// Of the nine piece products of a*b the six largest, hh, hm, mh, hl, lh and mm,
// are kept (the dropped ones are below 2^-26 |a||b|); bf16 products are exact
// and the tensor core accumulates them in fp32, so the result carries the error
// of an fp32 accumulation, like the scalar fp32 kernel.  The six products
// are laid out along K: the split writes A' [S][M][g*K] and B' [S][g*K][N]
// (g = 6 / S products per batch, piece of A / B per product below), one
// batched bf16 GEMM with fp32 output computes the S partial products, and for
// S > 1 a last kernel adds the partials.  Outputs too small to fill the GPU
// with 256x256 tiles use 128x128 tiles and, if that still leaves SMs idle,
// S > 1.  Rows of A or columns of B holding a value that is not finite or is
// too large for bf16 (|x| >= 3e38) are marked by the split; their outputs are
// recomputed by plain fp32 dot products at the end, so infinities and NaNs
// propagate as in an fp32 product.

constexpr int kSplitProducts = 6;
// piece of A and of B in product p (0 = hi, 1 = mid, 2 = lo): hh hm mh hl lh mm
__host__ __device__ constexpr int piece_a(int p) { return p == 2 || p == 5 ? 1 : (p == 4 ? 2 : 0); }
__host__ __device__ constexpr int piece_b(int p) { return p == 1 || p == 5 ? 1 : (p == 3 ? 2 : 0); }

__device__ __forceinline__ uint16_t bf16_rn_bits(float x) {
    return __bfloat16_as_ushort(__float2bfloat16_rn(x));
}

// One operand of the split: src [rows, cols] fp32 -> dst pieces.  For A
// element (r, c) of product p = s*g + q goes to dst[s][r][q*cols + c]
// and a bad value marks flags[1 + r]; for B element (r, c) goes to
// dst[s][q*rows + r][c] and marks flags[1 + M + c].
struct SplitOperand {
    const float* src;
    size_t rows, cols;
    uint16_t* dst;
};

// Both operands in one launch, 8 consecutive elements of a row per thread
// (cols % 8 == 0): the first A.rows * A.cols / 8 work items split A, the rest B.
__global__ void __launch_bounds__(256) split3_bf16_kernel(const SplitOperand opA, const SplitOperand opB, int g,
                                                         size_t M, int* __restrict__ flags) {
    const size_t groups_a = opA.rows * (opA.cols / 8);
    const size_t groups = groups_a + opB.rows * (opB.cols / 8);
    pdl_wait();
    for (size_t gi0 = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; gi0 < groups;
         gi0 += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const bool is_a = gi0 < groups_a;
        const float* src = is_a ? opA.src : opB.src;
        uint16_t* dst = is_a ? opA.dst : opB.dst;
        const size_t gi = is_a ? gi0 : gi0 - groups_a;
        const size_t rows = is_a ? opA.rows : opB.rows, cols = is_a ? opA.cols : opB.cols;
        const size_t slab = rows * cols * static_cast<size_t>(g);  // elements per batch of dst
        const size_t r = gi / (cols / 8), c = (gi % (cols / 8)) * 8;
        const float4 v0 = reinterpret_cast<const float4*>(src + r * cols + c)[0];
        const float4 v1 = reinterpret_cast<const float4*>(src + r * cols + c)[1];
        const float x[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
        uint32_t piece[3][4];
        bool bad = false;
#pragma unroll
        for (int e = 0; e < 8; e += 2) {
            uint16_t h[2], m[2], l[2];
#pragma unroll
            for (int u = 0; u < 2; ++u) {
                const float xv = x[e + u];
                if (!(fabsf(xv) < 3.0e38f)) {  // inf, NaN, or beyond bf16's range
                    bad = true;
                    h[u] = m[u] = l[u] = 0;
                    continue;
                }
                h[u] = bf16_rn_bits(xv);
                const float r1 = xv - __uint_as_float(static_cast<uint32_t>(h[u]) << 16);
                m[u] = bf16_rn_bits(r1);
                const float r2 = r1 - __uint_as_float(static_cast<uint32_t>(m[u]) << 16);
                l[u] = bf16_rn_bits(r2);
            }
            piece[0][e / 2] = static_cast<uint32_t>(h[0]) | (static_cast<uint32_t>(h[1]) << 16);
            piece[1][e / 2] = static_cast<uint32_t>(m[0]) | (static_cast<uint32_t>(m[1]) << 16);
            piece[2][e / 2] = static_cast<uint32_t>(l[0]) | (static_cast<uint32_t>(l[1]) << 16);
        }
        if (bad) {
            flags[0] = 1;
            if (is_a) {
                flags[1 + r] = 1;
            } else {
#pragma unroll
                for (int e = 0; e < 8; ++e)
                    if (!(fabsf(x[e]) < 3.0e38f)) flags[1 + M + c + e] = 1;
            }
        }
#pragma unroll
        for (int p = 0; p < kSplitProducts; ++p) {
            const int s = p / g, q = p % g;
            const int pa = piece_a(p), pb = piece_b(p);  // constants once p is unrolled
            const size_t off = is_a ? s * slab + r * (cols * g) + q * cols + c : s * slab + (q * rows + r) * cols + c;
            const uint4 w = is_a ? make_uint4(piece[pa][0], piece[pa][1], piece[pa][2], piece[pa][3])
                                 : make_uint4(piece[pb][0], piece[pb][1], piece[pb][2], piece[pb][3]);
            *reinterpret_cast<uint4*>(dst + off) = w;
        }
    }
}

// Plain fp32 dot product of row r of A and column c of B in k order.
__device__ __forceinline__ float dot_f32(const float* __restrict__ A, const float* __restrict__ B, size_t r, size_t c,
                                         size_t K, size_t N) {
    float acc = 0.f;
    for (size_t k = 0; k < K; ++k) acc = fmaf(A[r * K + k], B[k * N + c], acc);
    return acc;
}

// C[i] = sum of the S partials, the later (smaller) products first (M*N % 4 ==
// 0); outputs in a marked row or column are replaced by plain fp32 dot products.
__global__ void __launch_bounds__(256) sum_partials_kernel(const float* __restrict__ part, float* __restrict__ C, int S,
                                                          const float* __restrict__ A, const float* __restrict__ B,
                                                          size_t M, size_t K, size_t N, const int* __restrict__ flags) {
    const size_t n = M * N;
    pdl_wait();
    const bool any_bad = flags[0] != 0;
    for (size_t i = (blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x) * 4; i < n;
         i += static_cast<size_t>(gridDim.x) * blockDim.x * 4) {
        float4 acc = *reinterpret_cast<const float4*>(part + static_cast<size_t>(S - 1) * n + i);
        for (int s = S - 2; s >= 0; --s) {
            const float4 v = *reinterpret_cast<const float4*>(part + static_cast<size_t>(s) * n + i);
            acc.x += v.x;
            acc.y += v.y;
            acc.z += v.z;
            acc.w += v.w;
        }
        if (any_bad) {
            float* a4 = &acc.x;
            for (int e = 0; e < 4; ++e) {
                const size_t r = (i + e) / N, c = (i + e) % N;
                if (flags[1 + r] || flags[1 + M + c]) a4[e] = dot_f32(A, B, r, c, K, N);
            }
        }
        *reinterpret_cast<float4*>(C + i) = acc;
    }
}

// Outputs whose row of A or column of B was marked (single-batch case): plain
// fp32 dot products.  Returns at once when nothing was marked (flags[0] == 0).
__global__ void __launch_bounds__(256) split_fixup_kernel(const float* __restrict__ A, const float* __restrict__ B,
                                                         float* __restrict__ C, size_t M, size_t K, size_t N,
                                                         const int* __restrict__ flags) {
    pdl_wait();
    if (flags[0] == 0) return;
    for (size_t r = blockIdx.x; r < M; r += gridDim.x) {
        const bool row_bad = flags[1 + r] != 0;
        for (size_t c = threadIdx.x; c < N; c += blockDim.x)
            if (row_bad || flags[1 + M + c] != 0) C[r * N + c] = dot_f32(A, B, r, c, K, N);
    }
}

// Tiling of the split products for an M x N output: 256x256 pair tiles and one
// batch (S = 1) when those tiles fill the GPU; otherwise 128x128 single-CTA
// tiles, one batch if they fill it, else the S (1, 2, 3 or 6) with the fewest
// tile waves times products per batch (ties to the smaller S, which writes
// fewer partials).
struct SplitPlan {
    int S;
    bool small_tiles;
};
static SplitPlan split_plan(size_t M, size_t N) {
    const size_t pair_tiles = ((M + 255) / 256) * ((N + 255) / 256);
    const size_t sms = static_cast<size_t>(sm_count() > 0 ? sm_count() : 148);
    if (M > 128 && N > 128 && pair_tiles >= sms / 2) return {1, false};
    const size_t tiles = ((M + 127) / 128) * ((N + 127) / 128);
    if (tiles >= sms) return {1, true};
    int best = 1;
    size_t best_cost = ~size_t(0);
    for (int S : {1, 2, 3, 6}) {
        const size_t cost = ((tiles * S + sms - 1) / sms) * static_cast<size_t>(kSplitProducts / S);
        if (cost < best_cost) {
            best_cost = cost;
            best = S;
        }
    }
    return {best, true};
}

// C = A . B for contiguous row-major fp32 A [M, K], B [K, N], C [M, N] through
// the split above.  Returns -1 (nothing launched, nothing allocated) when the
// shape does not suit it; the caller then runs the scalar kernel.
static int matmul_f32_split(const float* A, const float* B, float* C, size_t M, size_t K, size_t N, cudaStream_t st) {
    if (K % 8 != 0 || N % 8 != 0 || K < 64 || !aligned16(A) || !aligned16(B) || !aligned16(C)) return -1;
    // ~25 us of fixed cost (scratch, split, partial sum, fix-up launches): below 2^28
    // multiply-adds the scalar kernel finishes first
    if (static_cast<double>(M) * static_cast<double>(N) * static_cast<double>(K) < 268435456.0) return -1;
    if (M > (1u << 30) || N > (1u << 30) || K * kSplitProducts > (1u << 30)) return -1;
    const SplitPlan plan = split_plan(M, N);
    const int S = plan.S;
    const int g = kSplitProducts / S;
    auto up = [](size_t b) { return (b + 255) & ~size_t(255); };
    const size_t a_bytes = up(static_cast<size_t>(kSplitProducts) * M * K * 2);
    const size_t b_bytes = up(static_cast<size_t>(kSplitProducts) * K * N * 2);
    const size_t p_bytes = S > 1 ? up(static_cast<size_t>(S) * M * N * 4) : 0;
    const size_t f_bytes = up((1 + M + N) * sizeof(int));
    void* mem = nullptr;
    cudaError_t e = pool_malloc(&mem, a_bytes + b_bytes + p_bytes + f_bytes, st);
    if (e != cudaSuccess) return api_fail(e, "matmul(f32 split): scratch of %zu bytes: %s",
                                          a_bytes + b_bytes + p_bytes + f_bytes, cudaGetErrorString(e));
    uint8_t* base = static_cast<uint8_t*>(mem);
    uint16_t* a3 = reinterpret_cast<uint16_t*>(base);
    uint16_t* b3 = reinterpret_cast<uint16_t*>(base + a_bytes);
    float* part = S > 1 ? reinterpret_cast<float*>(base + a_bytes + b_bytes) : C;
    int* flags = reinterpret_cast<int*>(base + a_bytes + b_bytes + p_bytes);
    int rc = 0;
    e = cudaMemsetAsync(flags, 0, (1 + M + N) * sizeof(int), st);
    if (e != cudaSuccess) rc = api_fail(e, "matmul(f32 split): %s", cudaGetErrorString(e));
    const int sms = sm_count() > 0 ? sm_count() : 148;
    auto grid_for = [&](size_t work) {
        const size_t blocks = (work + 255) / 256;
        return static_cast<unsigned>(blocks < static_cast<size_t>(sms) * 8 ? (blocks ? blocks : 1) : static_cast<size_t>(sms) * 8);
    };
    if (rc == 0) {
        const SplitOperand opA{A, M, K, a3}, opB{B, K, N, b3};
        launch_pdl(split3_bf16_kernel, grid_for(M * (K / 8) + K * (N / 8)), 256, 0, st, opA, opB, g, M, flags);
        rc = launch_status("matmul(f32 split)");
    }
    if (rc == 0) {
        const long long gk = static_cast<long long>(g) * static_cast<long long>(K);
        BmmStrides sd{gk, static_cast<long long>(N), static_cast<long long>(N), static_cast<long long>(M) * gk,
                      gk * static_cast<long long>(N), static_cast<long long>(M * N)};
        rc = bmm_bf16_tc(DT_F32, a3, b3, part, static_cast<size_t>(S), M, static_cast<size_t>(gk), N, 0, 1.0f, sd, st,
                         plan.small_tiles);
        if (rc == -1) rc = fail(cudaErrorNotSupported, "matmul(f32 split): tensor-core path rejected the split operands");
    }
    if (rc == 0 && S > 1) {
        launch_pdl(sum_partials_kernel, grid_for(M * N / 4), 256, 0, st, part, C, S, A, B, M, K, N, flags);
        rc = launch_status("matmul(f32 split sum)");
    }
    if (rc == 0 && S == 1) {
        split_fixup_kernel<<<static_cast<unsigned>(M < static_cast<size_t>(sms) * 4 ? M : static_cast<size_t>(sms) * 4), 256, 0,
                             st>>>(A, B, C, M, K, N, flags);
        rc = launch_status("matmul(f32 split fixup)");
    }
    cudaError_t e2 = cudaFreeAsync(mem, st);
    if (rc == 0 && e2 != cudaSuccess) rc = api_fail(e2, "matmul(f32 split): %s", cudaGetErrorString(e2));
    return rc;
}

}  // namespace bee_b200

using namespace bee_b200;

// Sum of the S K-chunk partials of a split product, in chunk order (so the result
// does not depend on timing), times alpha, rounded to the output type (n % 4 == 0).
__global__ void __launch_bounds__(256) sum_ksplit_kernel(const float* __restrict__ part, void* __restrict__ C, int S,
                                                         size_t n, float alpha, int out_dt) {
    pdl_wait();
    for (size_t i = (blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x) * 4; i < n;
         i += static_cast<size_t>(gridDim.x) * blockDim.x * 4) {
        float4 acc = *reinterpret_cast<const float4*>(part + i);
        for (int s = 1; s < S; ++s) {
            const float4 v = *reinterpret_cast<const float4*>(part + static_cast<size_t>(s) * n + i);
            acc.x += v.x;
            acc.y += v.y;
            acc.z += v.z;
            acc.w += v.w;
        }
        acc.x *= alpha;
        acc.y *= alpha;
        acc.z *= alpha;
        acc.w *= alpha;
        if (out_dt == DT_F32) {
            *reinterpret_cast<float4*>(static_cast<float*>(C) + i) = acc;
        } else {
            const bool h = out_dt == DT_F16;
            uint2 o;
            o.x = h ? pack_f16x2(acc.x, acc.y) : pack_bf16x2(acc.x, acc.y);
            o.y = h ? pack_f16x2(acc.z, acc.w) : pack_bf16x2(acc.z, acc.w);
            *reinterpret_cast<uint2*>(static_cast<uint16_t*>(C) + i) = o;
        }
    }
}

// One 16-bit product whose output tiles would leave most SMs idle (small M or
// N, long K): K is cut into S chunks that run as the S entries of a batched
// product on 128 x 128 tiles (each chunk a view of A and B at an offset, fp32
// partials in pool scratch), then summed in chunk order.  Returns -1 when the
// shape does not qualify or the chunk views cannot be described by TMA.
static int bmm_ksplit(int dt_in, int dt_out, const void* A, const void* B, void* C, size_t M, size_t K, size_t N,
                      int b_trans, float alpha, const BmmStrides& sd, cudaStream_t st) {
    const size_t sms = static_cast<size_t>(sm_count());
    const size_t tiles = ((M + 127) / 128) * ((N + 127) / 128);
    if (sd.ldc != static_cast<long long>(N) || (M * N) % 4 != 0 || !aligned16(C)) return -1;
    if (K % 128 != 0 || K < 2048 || tiles * 2 > sms) return -1;
    // S divides the 128-wide K stages, fills at most the GPU, keeps chunks >= 1024 long
    const size_t kb = K / 128;
    size_t S = 1;
    for (size_t cand = 2; cand <= 8; ++cand)
        if (kb % cand == 0 && tiles * cand <= sms && K / cand >= 1024) S = cand;
    if (S < 2) return -1;
    const size_t Kc = K / S;
    void* mem = nullptr;
    cudaError_t e = pool_malloc(&mem, S * M * N * sizeof(float), st);
    if (e != cudaSuccess) return api_fail(e, "bmm (K split): scratch of %zu bytes: %s", S * M * N * sizeof(float),
                                          cudaGetErrorString(e));
    float* part = static_cast<float*>(mem);
    const BmmStrides ps{sd.lda, sd.ldb, static_cast<long long>(N), static_cast<long long>(Kc),
                        b_trans ? static_cast<long long>(Kc) : static_cast<long long>(Kc) * sd.ldb,
                        static_cast<long long>(M * N)};
    int rc = bmm_bf16_tc(DT_F32, A, B, part, S, M, Kc, N, b_trans, 1.0f, ps, st, true, dt_in);
    if (rc == 0) {
        const size_t work = (M * N / 4 + 255) / 256, cap = sms * 8;
        launch_pdl(sum_ksplit_kernel, static_cast<unsigned>(work < cap ? work : cap), 256, 0, st, part, C,
                   static_cast<int>(S), M * N, alpha, dt_out);
        rc = launch_status("bmm (K split sum)");
    }
    cudaError_t e2 = cudaFreeAsync(mem, st);
    if (rc == 0 && e2 != cudaSuccess) rc = api_fail(e2, "bmm (K split): %s", cudaGetErrorString(e2));
    return rc;
}

static int bmm_impl(int dt_in, int dt_out, const void* A, const void* B, void* C, size_t batch, size_t M, size_t K,
                    size_t N, int b_trans, float alpha, const BmmStrides& sd, cudaStream_t st) {
    if (dt_in == DT_BF16) {
        if (dt_out != DT_BF16 && dt_out != DT_F32)
            return fail(cudaErrorInvalidValue, "bmm: bf16 input needs a BF16 or F32 output, got %d", dt_out);
        int rc = K == 0 || batch != 1 ? -1 : bmm_ksplit(dt_in, dt_out, A, B, C, M, K, N, b_trans, alpha, sd, st);
        if (rc != -1) return rc;
        rc = K == 0 ? -1 : bmm_bf16_tc(dt_out, A, B, C, batch, M, K, N, b_trans, alpha, sd, st);
        if (rc != -1) return rc;
        return dt_out == DT_F32 ? launch_simt<uint16_t, float>(A, B, C, batch, M, K, N, b_trans, alpha, sd, st)
                                : launch_simt<uint16_t, uint16_t>(A, B, C, batch, M, K, N, b_trans, alpha, sd, st);
    }
    if (dt_in == DT_F16) {
        if (dt_out != DT_F16 && dt_out != DT_F32)
            return fail(cudaErrorInvalidValue, "bmm: f16 input needs an F16 or F32 output, got %d", dt_out);
        int rc = K == 0 || batch != 1 ? -1 : bmm_ksplit(dt_in, dt_out, A, B, C, M, K, N, b_trans, alpha, sd, st);
        if (rc != -1) return rc;
        rc = K == 0 ? -1 : bmm_bf16_tc(dt_out, A, B, C, batch, M, K, N, b_trans, alpha, sd, st, false, DT_F16);
        if (rc != -1) return rc;
        return dt_out == DT_F32 ? launch_simt<__half, float>(A, B, C, batch, M, K, N, b_trans, alpha, sd, st)
                                : launch_simt<__half, __half>(A, B, C, batch, M, K, N, b_trans, alpha, sd, st);
    }
    if (dt_out != dt_in) return fail(cudaErrorInvalidValue, "bmm: output dtype must equal input dtype for %d", dt_in);
    switch (dt_in) {
    case DT_F32: return launch_simt<float, float>(A, B, C, batch, M, K, N, b_trans, alpha, sd, st);
    case DT_F64: return launch_simt<double, double>(A, B, C, batch, M, K, N, b_trans, alpha, sd, st);
    case DT_I32: return launch_simt<int32_t, int32_t>(A, B, C, batch, M, K, N, b_trans, alpha, sd, st);
    case DT_I64: return launch_simt<int64_t, int64_t>(A, B, C, batch, M, K, N, b_trans, alpha, sd, st);
    default: return fail(cudaErrorInvalidValue, "bmm: unsupported dtype %d", dt_in);
    }
}

extern "C" {

int bee_b200_bmm(int dt_in, int dt_out, const void* A, const void* B, void* C, size_t batch, size_t M, size_t K,
                 size_t N, int b_trans, float alpha, bee_b200_stream_t stream) {
    if (batch == 0 || M == 0 || N == 0) return ok();
    if (!A || !B || !C) return fail(cudaErrorInvalidValue, "bmm: null pointer");
    cudaStream_t st = as_stream(stream);
    if ((dt_in == DT_BF16 || dt_in == DT_F16) && K == 0 && (dt_out == dt_in || dt_out == DT_F32)) {
        cudaError_t e = cudaMemsetAsync(C, 0, batch * M * N * (dt_out == DT_F32 ? 4 : 2), st);
        return e == cudaSuccess ? ok() : fail(static_cast<int>(e), "bmm: %s", cudaGetErrorString(e));
    }
    return bmm_impl(dt_in, dt_out, A, B, C, batch, M, K, N, b_trans, alpha, contiguous_strides(M, K, N, b_trans), st);
}

int bee_b200_bmm_strided(int dt_in, int dt_out, const void* A, int64_t lda, int64_t stride_a, const void* B,
                         int64_t ldb, int64_t stride_b, void* C, int64_t ldc, int64_t stride_c, size_t batch, size_t M,
                         size_t K, size_t N, int b_trans, float alpha, bee_b200_stream_t stream) {
    if (batch == 0 || M == 0 || N == 0) return ok();
    if (!A || !B || !C) return fail(cudaErrorInvalidValue, "bmm_strided: null pointer");
    if (M > (1u << 30) || N > (1u << 30) || K > (1u << 30) || batch > 65535)
        return fail(cudaErrorInvalidValue, "bmm_strided: extent too large");
    if (lda < static_cast<int64_t>(K) || ldb < static_cast<int64_t>(b_trans ? K : N) || ldc < static_cast<int64_t>(N))
        return fail(cudaErrorInvalidValue, "bmm_strided: leading dimension shorter than a row");
    if (stride_a < 0 || stride_b < 0 || stride_c < 0)
        return fail(cudaErrorInvalidValue, "bmm_strided: negative batch stride");
    if (batch > 1 && stride_c < static_cast<int64_t>((M - 1) * ldc + N))
        return fail(cudaErrorInvalidValue, "bmm_strided: output batches overlap");
    BmmStrides sd{lda, ldb, ldc, stride_a, stride_b, stride_c};
    if (batch > 1 && stride_b == 0 && stride_a == static_cast<int64_t>(M) * lda && stride_c == static_cast<int64_t>(M) * ldc) {
        // one B for every batch, A and C batches stacked row after row: one product of batch * M rows
        M *= batch;
        batch = 1;
        sd.sa = static_cast<long long>(M) * lda;
        sd.sc = static_cast<long long>(M) * ldc;
    }
    // K == 0: C = 0 (row by row through the product path would read nothing); use the SIMT kernel
    return bmm_impl(dt_in, dt_out, A, B, C, batch, M, K, N, b_trans, alpha, sd, as_stream(stream));
}

int bee_b200_matmul(int dt, const void* A, const void* B, void* C, size_t M, size_t K, size_t N,
                    bee_b200_stream_t stream) {
    if (dt == DT_F32 && M != 0 && N != 0 && A && B && C) {
        const int rc = matmul_f32_split(static_cast<const float*>(A), static_cast<const float*>(B), static_cast<float*>(C),
                                        M, K, N, as_stream(stream));
        if (rc != -1) return rc == 0 ? ok() : rc;
    }
    return bee_b200_bmm(dt, dt, A, B, C, 1, M, K, N, 0, 1.0f, stream);
}

int bee_b200_device_status(int* out_code) {
    if (!out_code) return fail(cudaErrorInvalidValue, "device_status: null pointer");
    int zero = 0, attn = 0, coll = 0;
    cudaError_t e = cudaMemcpyFromSymbol(out_code, g_gemm_status, sizeof(int));
    if (e == cudaSuccess) e = cudaMemcpyToSymbol(g_gemm_status, &zero, sizeof(int));
    if (e == cudaSuccess) e = static_cast<cudaError_t>(attention_status_take(&attn));
    if (e == cudaSuccess) e = static_cast<cudaError_t>(allranks_status_take(&coll));
    if (e != cudaSuccess) return fail(static_cast<int>(e), "device_status: %s", cudaGetErrorString(e));
    if (*out_code == 0) *out_code = attn;
    if (*out_code == 0) *out_code = coll;
    return ok();
}


size_t bee_b200_splitk_recv_bytes(size_t M, size_t N, int world) {
    if (world < 1) return 0;
    const size_t tiles = ((M + 255) / 256) * ((N + 255) / 256);
    const size_t owned = (tiles + world - 1) / world;
    return static_cast<size_t>(world) * owned * 256 * 256 * sizeof(float);
}

int bee_b200_gemm_splitk_scatter(const void* A, size_t lda, const void* B, size_t M, size_t K, size_t N,
                                 void* const* recv_peers, int world, int rank, bee_b200_stream_t stream) {
    if (M == 0 || N == 0) return ok();
    if (!A || !B || !recv_peers) return fail(cudaErrorInvalidValue, "splitk_scatter: null pointer");
    if (world < 1 || world > kMaxPeers || rank < 0 || rank >= world)
        return fail(cudaErrorInvalidValue, "splitk_scatter: rank %d / world %d out of range (world <= %d)", rank, world,
                    kMaxPeers);
    for (int r = 0; r < world; ++r)
        if (!recv_peers[r] || !aligned16(recv_peers[r]))
            return fail(cudaErrorInvalidValue, "splitk_scatter: receive buffer %d missing or misaligned", r);
    if (K == 0 || K % 8 != 0 || N % 8 != 0 || lda % 8 != 0 || lda < K || !aligned16(A) || !aligned16(B))
        return fail(cudaErrorInvalidValue, "splitk_scatter: needs K, N, lda multiples of 8 and 16-byte aligned A, B");
    if (M > (1u << 30) || N > (1u << 30) || K > (1u << 30))
        return fail(cudaErrorInvalidValue, "splitk_scatter: extent too large");
    CUtensorMap ta, tb;
    if (int rc = make_map(&ta, A, K, M, 1, lda, lda * M, 64, 128)) return rc;
    if (int rc = make_map(&tb, B, N, K, 1, N, K * N, 64, Pair2Cfg::BK)) return rc;
    GemmParams p{};
    p.M = static_cast<int>(M);
    p.N = static_cast<int>(N);
    p.K = static_cast<int>(K);
    p.m_tiles = static_cast<int>((M + 255) / 256);
    p.n_tiles = static_cast<int>((N + 255) / 256);
    p.tiles_per_batch = p.m_tiles * p.n_tiles;
    p.total_tiles = p.tiles_per_batch;
    p.num_kb = static_cast<int>((K + Pair2Cfg::BK - 1) / Pair2Cfg::BK);
    p.ldc = static_cast<long long>(N);
    p.batch_stride_c = 0;
    p.alpha = 1.0f;
    p.C = nullptr;
    p.world = world;
    p.rank = rank;
    p.owned = (p.total_tiles + world - 1) / world;
    for (int r = 0; r < world; ++r) p.peer_recv[r] = static_cast<float*>(recv_peers[r]);
    auto kern = gemm_bf16_tcgen05_2sm_kernel<false, true, true>;
    static SmemLimit smem_limit;
    if (int rc = smem_limit.ensure(kern, Pair2Cfg::SMEM, "splitk_scatter")) return rc;
    const int pairs = sm_count() / 2;
    const int grid = 2 * (p.total_tiles < pairs ? p.total_tiles : pairs);
    kern<<<grid, 192, Pair2Cfg::SMEM, as_stream(stream)>>>(ta, tb, p);
    return launch_status("splitk_scatter");
}

int bee_b200_gemm_splitk_reduce(const void* recv_local, void* const* c_peers, size_t M, size_t N, int world, int rank,
                                bee_b200_stream_t stream) {
    if (M == 0 || N == 0) return ok();
    if (!recv_local || !c_peers) return fail(cudaErrorInvalidValue, "splitk_reduce: null pointer");
    if (world < 1 || world > kMaxPeers || rank < 0 || rank >= world)
        return fail(cudaErrorInvalidValue, "splitk_reduce: rank %d / world %d out of range", rank, world);
    if (N % 8 != 0) return fail(cudaErrorInvalidValue, "splitk_reduce: N must be a multiple of 8");
    SplitKReduceParams p{};
    p.M = static_cast<int>(M);
    p.N = static_cast<int>(N);
    p.m_tiles = static_cast<int>((M + 255) / 256);
    p.n_tiles = static_cast<int>((N + 255) / 256);
    p.total_tiles = p.m_tiles * p.n_tiles;
    p.world = world;
    p.rank = rank;
    p.owned = (p.total_tiles + world - 1) / world;
    p.ldc = static_cast<long long>(N);
    for (int r = 0; r < world; ++r) {
        if (!c_peers[r] || !aligned16(c_peers[r])) return fail(cudaErrorInvalidValue, "splitk_reduce: C %d missing or misaligned", r);
        p.c_peer[r] = static_cast<uint16_t*>(c_peers[r]);
    }
    size_t grid = static_cast<size_t>(p.owned) * 8;  // 32-row bands
    const size_t cap = static_cast<size_t>(sm_count()) * 6;
    if (grid > cap) grid = cap;
    splitk_reduce_kernel<<<static_cast<unsigned>(grid), 256, 0, as_stream(stream)>>>(static_cast<const float*>(recv_local), p);
    return launch_status("splitk_reduce");
}

}  // extern "C"
