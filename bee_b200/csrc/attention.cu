// Fused attention forward: O = softmax(Q K^T * scale) V, per head, bf16 in/out,
// fp32 scores and softmax, fp32 accumulation.
//
// The reference has no attention (its user composes per-head matmul, scale,
// softmax and matmul, each round-tripping through memory).  Here one CTA owns
// two 128-query tiles (A and B) of one head and streams the keys/values past
// them in blocks of 128, so S and P never leave the SM:
//   * warp 0 — TMA: Q_A, Q_B and K_0 once, then a two-stage ring whose stage
//     j & 1 holds V_j and K_{j+1} (one 64x128 box shape serves all three; K is
//     read as the K-major operand of Q.K^T, V as the MN-major operand of P.V);
//   * warp 1 — MMA, ping-pong between the tiles: O_A += P_A(j).V_j,
//     S_A(j+1) = Q_A.K_{j+1}^T, O_B += P_B(j).V_j, S_B(j+1) = Q_B.K_{j+1}^T,
//     so the tensor core works on one tile while the other tile's softmax runs.
//     This one thread paces the kernel: each mbarrier wait or tcgen05.commit it
//     executes costs ~100 cycles even when nothing is pending, so per block it
//     does one wait for the ring stage, one per tile for P, one commit per tile
//     for S and one to release the stage, with descriptors precomputed and the
//     ring slot a compile-time constant (blocks are unrolled in pairs);
//     warps 2-3 idle; this warpgroup gives most of its registers to the next two
//     (setmaxnreg);
//   * warps 4-7 / 8-11 — softmax of tile A / B, one thread per query row: the
//     thread reads its 128 scores from TMEM, keeps a running max m (log2 units)
//     and sum l, and writes P = 2^(s*c - m) as bf16 back into TMEM over the
//     first 64 columns of its own scores (three quarters of the exponentials
//     on the MUFU, one quarter on the FMA pipe); P.V then reads P straight from TMEM
//     (tcgen05.mma with the A operand in tensor memory).  The running max is
//     only raised when a block's max exceeds it by more than 8 (a factor 2^8):
//     until then P <= 256, which bf16 and fp32 hold exactly enough, and O / l
//     is unchanged; when it is raised the thread rescales its row of O in TMEM
//     (the previous P.V is complete by then: the MMA that produced the current
//     scores was issued after it).  At the end each thread divides its O row
//     by l into shared memory, and two TMA stores per tile write O.
// TMEM (512 columns): S_A 0-127, S_B 128-255, O_A 256-383, O_B 384-511.
// Every wait is bounded; a wait that gives up records a code in the status
// word read by bee_b200_device_status and the CTA abandons its work.
#include <cuda.h>
#include <type_traits>
#include <cudaTypedefs.h>

#include "common.cuh"
#include "sm100.cuh"

namespace bee_b200 {

using namespace sm100;

__device__ int g_attn_status = 0;

namespace {

constexpr int kBlock = 128;                       // queries per tile, keys per step
constexpr int kHead = 128;                        // head dim
constexpr int kHalf = 128 * 64 * 2;               // one 128-row x 64-col bf16 swizzled block
constexpr int kTile = 2 * kHalf;                  // 128 x 128 bf16
constexpr int kSmem = 2 * kTile /*Q_A, Q_B*/ + 2 * kTile /*K*/ + 2 * kTile /*V*/ + 1024;
constexpr float kRescaleThreshold = 8.0f;         // log2 units

__device__ __forceinline__ void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
        "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
        "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
        "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
        "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// 2^x for a packed pair on the FMA pipe, beside the MUFU ex2: Cody-Waite split
// x = n + f with n = floor(x) (x + 1.5 * 2^23 rounded toward -inf leaves n in the
// low mantissa bits) and f in [0, 1); 2^f by a cubic fitted here for minimum
// relative error on [0, 1] (7.5e-5 at most, against 2^-9 for the bf16 rounding of
// P that follows); n added to the exponent field.  x is clamped at -126 so the
// exponent field never goes negative (2^-126 and below read as ~0 in bf16 P and
// in the fp32 row sum).
__device__ __forceinline__ void ex2_fma_x2(uint64_t x2, float& e0, float& e1) {
    float x0, x1;
    unpack_f32x2(x2, x0, x1);
    const uint64_t xc = pack_f32x2(fmaxf(x0, -126.0f), fmaxf(x1, -126.0f));
    const uint64_t magic = pack_f32x2(12582912.0f, 12582912.0f);
    uint64_t t, n, f;
    asm("add.rm.f32x2 %0, %1, %2;" : "=l"(t) : "l"(xc), "l"(magic));
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(n) : "l"(t), "l"(magic));
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(f) : "l"(xc), "l"(n));
    uint64_t q = fma_f32x2(f, pack_f32x2(0.07802427560091019f, 0.07802427560091019f),
                           pack_f32x2(0.22606725990772247f, 0.22606725990772247f));
    q = fma_f32x2(q, f, pack_f32x2(0.6958336234092712f, 0.6958336234092712f));
    q = fma_f32x2(q, f, pack_f32x2(0.9999251961708069f, 0.9999251961708069f));
    float q0, q1, t0, t1;
    unpack_f32x2(q, q0, q1);
    unpack_f32x2(t, t0, t1);
    e0 = __uint_as_float(__float_as_uint(q0) + (__float_as_uint(t0) << 23));
    e1 = __uint_as_float(__float_as_uint(q1) + (__float_as_uint(t1) << 23));
}

// Which pairs of a row's 64 take ex2_fma_x2 instead of the MUFU: bit (i % 16) of
// the mask for pair i.
constexpr uint32_t kEx2FmaMask = 0x2222u;

// Three-input maximum (one instruction on sm_100).
__device__ __forceinline__ float max3(float a, float b, float c) {
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}

// Maximum of 128 values as a tree of three-input maxima (depth 5 rather than a
// chain of 127 dependent two-input maxima).
__device__ __forceinline__ float row_max128(const uint32_t (&s)[128]) {
    float t[43];
#pragma unroll
    for (int i = 0; i < 42; ++i)
        t[i] = max3(__uint_as_float(s[3 * i]), __uint_as_float(s[3 * i + 1]), __uint_as_float(s[3 * i + 2]));
    t[42] = fmaxf(__uint_as_float(s[126]), __uint_as_float(s[127]));
    float u[15];
#pragma unroll
    for (int i = 0; i < 14; ++i) u[i] = max3(t[3 * i], t[3 * i + 1], t[3 * i + 2]);
    u[14] = t[42];
    float v[5];
#pragma unroll
    for (int i = 0; i < 5; ++i) v[i] = max3(u[3 * i], u[3 * i + 1], u[3 * i + 2]);
    return fmaxf(max3(v[0], v[1], v[2]), fmaxf(v[3], v[4]));
}

// ---------------------------------------------------------------- MMA issuer
// The issuing thread paces the kernel: each mbarrier wait or tcgen05.commit on
// it costs ~100 cycles even when nothing is pending, so everything below keeps
// them to one wait for the ring stage, one per tile for P, one commit per tile
// for S and one to release the stage, with the shared-memory descriptors built
// once and the ring slot a compile-time constant.
struct MmaRing {
    uint32_t tmem;
    uint64_t dq[2], dk[2], dv[2];  // descriptors of Q_A / Q_B, K slots, V slots
    uint64_t *op_full, *op_empty, *s_full, *p_full, *o_done;
    volatile int* abort;
    int* status;
    int nkv;
};

constexpr uint32_t kIdescS = idesc_bf16_f32(128, 128, false);  // B = K rows, K-major
constexpr uint32_t kIdescO = idesc_bf16_f32(128, 128, true);   // B = V, MN-major

// S_t = Q_t . K^T (K in ring slot KS) into TMEM columns t * 128, then signal the
// tile's softmax.  Within a tile only the descriptors' start-address field
// (address >> 4, low 14 bits; every address here is below 2^18, so it never
// carries out) moves, by a compile-time amount per K step.
template <int T, int KS>
__device__ __forceinline__ void issue_s(const MmaRing& r) {
    // opaque copies: otherwise the compiler hoists every (base + step) of the
    // unrolled loop out of it and runs out of registers
    uint64_t qd = r.dq[T], kd = r.dk[KS];
    asm volatile("" : "+l"(qd), "+l"(kd));
#pragma unroll
    for (int k = 0; k < kHead / 16; ++k) {
        const uint64_t step = static_cast<uint64_t>(((k / 4) * kHalf + (k % 4) * 32) >> 4);
        mma_f16_ss(r.tmem + static_cast<uint32_t>(T * 128), qd + step, kd + step, kIdescS, k != 0 ? 1u : 0u);
    }
    mma_commit(&r.s_full[T]);
}

// O_t += P_t . V (V in ring slot VS); P_t sits in TMEM columns t * 128 .. + 63 as bf16 pairs.
template <int T, int VS>
__device__ __forceinline__ void issue_o(const MmaRing& r, bool acc) {
    uint64_t vd = r.dv[VS];
    asm volatile("" : "+l"(vd));
#pragma unroll
    for (int k = 0; k < kBlock / 16; ++k)
        mma_f16_ts(r.tmem + 256u + static_cast<uint32_t>(T * 128), r.tmem + static_cast<uint32_t>(T * 128 + k * 8),
                   vd + static_cast<uint64_t>((k * 16 * 128) >> 4), kIdescO, (acc || k != 0) ? 1u : 0u);
}

// Block j of the keys, ring stage ST = j & 1 holding V_j and K_{j+1}.
template <int NT, int ST>
__device__ __forceinline__ bool mma_block(const MmaRing& r, int j) {
    if (!mbar_wait(&r.op_full[ST], static_cast<uint32_t>((j >> 1) & 1), r.abort, r.status, 27)) return false;
    const bool next = j + 1 < r.nkv;
    if (!mbar_wait(&r.p_full[0], static_cast<uint32_t>(j & 1), r.abort, r.status, 26)) return false;
    tc_fence_after();
    issue_o<0, ST>(r, j != 0);
    if (next)
        issue_s<0, ST>(r);
    else
        mma_commit(&r.o_done[0]);  // tile A's epilogue may start while B finishes
    if (NT == 2) {
        if (!mbar_wait(&r.p_full[1], static_cast<uint32_t>(j & 1), r.abort, r.status, 26)) return false;
        tc_fence_after();
        issue_o<1, ST>(r, j != 0);
        if (next)
            issue_s<1, ST>(r);
        else
            mma_commit(&r.o_done[1]);
    }
    mma_commit(&r.op_empty[ST]);
    return true;
}

template <int NT>
__device__ __forceinline__ bool mma_all(const MmaRing& r, bool ok) {
    if (!ok || r.nkv == 0) return ok;
    tc_fence_after();
    issue_s<0, 1>(r);  // K_0 sits in the K slot of stage 1
    if (NT == 2) issue_s<1, 1>(r);
    mma_commit(&r.op_empty[1]);
    for (int j = 0; ok && j < r.nkv; j += 2) {
        ok = mma_block<NT, 0>(r, j);
        if (ok && j + 1 < r.nkv) ok = mma_block<NT, 1>(r, j + 1);
    }
    return ok;
}

struct AttnParams {
    int seq;          // queries == keys per head (multiple of 128)
    int nkv;          // seq / 128
    float scale_log2; // scale * log2(e)
};

constexpr int kThreads = 384;  // warpgroup 0: TMA warp, MMA warp, 2 idle; warpgroups 1-2: softmax
// Register split.  The launch gives every thread 168 registers (three warps per
// SM sub-partition, 16384 registers each); warpgroup 0 drops to 56 and the two
// softmax warpgroups take what it frees, so the total stays what was launched.
constexpr int kRegsLaunch = 168, kRegsControl = 56, kRegsSoftmax = 224;
static_assert(kRegsControl * 128 + kRegsSoftmax * 256 <= kRegsLaunch * kThreads,
              "setmaxnreg split exceeds the registers the block was launched with");
static_assert(kRegsLaunch * kThreads <= 65536 && kRegsLaunch * 3 * 32 <= 16384, "launch register budget");

__global__ void __launch_bounds__(kThreads, 1) attention_fwd_kernel(const __grid_constant__ CUtensorMap tmQ,
                                                                         const __grid_constant__ CUtensorMap tmK,
                                                                         const __grid_constant__ CUtensorMap tmV,
                                                                         const __grid_constant__ CUtensorMap tmO,
                                                                         const AttnParams p) {
    extern __shared__ uint8_t smem_raw[];
    __shared__ __align__(8) uint64_t q_full;
    __shared__ __align__(8) uint64_t op_full[2], op_empty[2];  // ring stage: V_j and K_{j+1}
    __shared__ __align__(8) uint64_t s_full[2], p_full[2];  // [tile]
    __shared__ __align__(8) uint64_t done_bar;
    __shared__ __align__(8) uint64_t o_done[2];   // [tile]: its last P.V has completed
    __shared__ __align__(8) uint64_t o_ready[2];  // [tile]: its 4 warps have staged O
    __shared__ uint32_t tmem_base_sh;
    __shared__ int abort_sh;

    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sQ = smem;            // [2] tiles A, B
    uint8_t* sK = sQ + 2 * kTile;  // [2] ring
    uint8_t* sV = sK + 2 * kTile;  // [2] ring
    volatile int* abort_flag = &abort_sh;
    int* status = &g_attn_status;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int pair = blockIdx.x, head = blockIdx.y;
    const int nkv = p.nkv;
    const int q0 = pair * 2 * kBlock;
    const int ntiles = q0 + kBlock < p.seq ? 2 : 1;  // the last pair of an odd tile count has only tile A

    if (threadIdx.x == 0) {
        mbar_init(&q_full, 1);
        for (int i = 0; i < 2; ++i) {
            mbar_init(&op_full[i], 1);
            mbar_init(&op_empty[i], 1);
            mbar_init(&s_full[i], 1);
            mbar_init(&p_full[i], 4);  // one arrive per softmax warp of the tile
        }
        mbar_init(&done_bar, 1);
        mbar_init(&o_done[0], 1);
        mbar_init(&o_done[1], 1);
        mbar_init(&o_ready[0], 4);
        mbar_init(&o_ready[1], 4);
        abort_sh = 0;
        fence_mbar_init();
        // thread 0 is also the TMA thread: Q_A, Q_B and K_0 (into the K slot of
        // stage 1) start loading on q_full now, under the TMEM allocation and the
        // first block barrier
        mbar_arrive_expect_tx(&q_full, static_cast<uint32_t>((ntiles + (nkv > 0 ? 1 : 0)) * kTile));
        for (int t = 0; t < ntiles; ++t) {
            tma_load_3d(sQ + t * kTile, &tmQ, &q_full, 0, q0 + t * kBlock, head);
            tma_load_3d(sQ + t * kTile + kHalf, &tmQ, &q_full, 64, q0 + t * kBlock, head);
        }
        if (nkv > 0) {
            tma_load_3d(sK + kTile, &tmK, &q_full, 0, 0, head);
            tma_load_3d(sK + kTile + kHalf, &tmK, &q_full, 64, 0, head);
        }
        tma_prefetch(&tmV);
        tma_prefetch(&tmO);
    }
    if (warp == 1) tmem_alloc<512>(&tmem_base_sh);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_base_sh;

    if (warp < 4) {
        // warpgroup 0 needs few registers: hand them to the softmax warpgroups
        asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;\n" ::"n"(kRegsControl) : "memory");
        if (warp == 0) {
            // ------------------------------------------------ TMA producer
            if (lane == 0) {
                // (Q_A, Q_B and K_0 were issued with the barrier initialisation)
                // stage s = j & 1 takes V_j and K_{j+1}; stage 1 is first released
                // by the MMA that read K_0, so its waits run one phase behind stage 0's
                int filled = 0;
                for (int j = 0; j < nkv; ++j) {
                    const int s = j & 1;
                    const uint32_t par = static_cast<uint32_t>((j >> 1) & 1) ^ (s == 0 ? 1u : 0u);
                    if (!mbar_wait(&op_empty[s], par, abort_flag, status, 21)) break;
                    const bool knext = j + 1 < nkv;
                    mbar_arrive_expect_tx(&op_full[s], static_cast<uint32_t>((knext ? 2 : 1) * kTile));
                    tma_load_3d(sV + s * kTile, &tmV, &op_full[s], 0, j * kBlock, head);
                    tma_load_3d(sV + s * kTile + kHalf, &tmV, &op_full[s], 64, j * kBlock, head);
                    if (knext) {
                        tma_load_3d(sK + s * kTile, &tmK, &op_full[s], 0, (j + 1) * kBlock, head);
                        tma_load_3d(sK + s * kTile + kHalf, &tmK, &op_full[s], 64, (j + 1) * kBlock, head);
                    }
                    filled = j + 1;
                }
                // the last loads must have landed before the CTA may exit
                // (normally the MMA warp consumed them already)
                mbar_wait(&q_full, 0, abort_flag, status, 33, 200000000ull);
                for (int j = filled > 2 ? filled - 2 : 0; j < filled; ++j)
                    mbar_wait(&op_full[j & 1], static_cast<uint32_t>((j >> 1) & 1), abort_flag, status, 34, 200000000ull);
            }
            __syncwarp();
        } else if (warp == 1) {
            // ------------------------------------------------ MMA issuer
            if (lane == 0) {
                // Shared-memory descriptors of the operand slots, built once: a thread
                // that rebuilt both descriptors per MMA took about as long to issue a
                // 128x128x16 product as the tensor core takes to retire it.
                const uint64_t dq0 = sdesc_sw128(smem_u32(sQ), 16, 1024), dq1 = sdesc_sw128(smem_u32(sQ + kTile), 16, 1024);
                const uint64_t dk0 = sdesc_sw128(smem_u32(sK), 16, 1024), dk1 = sdesc_sw128(smem_u32(sK + kTile), 16, 1024);
                const uint64_t dv0 = sdesc_sw128(smem_u32(sV), kHalf, 1024), dv1 = sdesc_sw128(smem_u32(sV + kTile), kHalf, 1024);
                MmaRing r{tmem, {dq0, dq1}, {dk0, dk1}, {dv0, dv1}, op_full, op_empty, s_full, p_full, o_done, abort_flag, status, nkv};
                bool ok = mbar_wait(&q_full, 0, abort_flag, status, 23);
                const bool issued = ok && nkv > 0;
                if (ntiles == 2)
                    mma_all<2>(r, ok);
                else
                    mma_all<1>(r, ok);
                if (issued) {
                    mma_commit(&done_bar);
                    mbar_wait(&done_bar, 0, abort_flag, status, 28, 200000000ull);
                }
            }
            __syncwarp();
        }
    } else {
        asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;\n" ::"n"(kRegsSoftmax) : "memory");
        // ------------------------------------------------ softmax / epilogue (warps 4-11)
        const int t = (warp - 4) >> 2;          // tile A (warps 4-7) or B (warps 8-11)
        const int q = warp & 3;                 // TMEM lane quarter
        const int row = q * 32 + lane;          // query row within the tile
        const uint32_t lane_addr = static_cast<uint32_t>(q * 32) << 16;
        const uint32_t s_col = tmem + static_cast<uint32_t>(t * 128) + lane_addr;
        const uint32_t o_col = tmem + 256u + static_cast<uint32_t>(t * 128) + lane_addr;
        const float c = p.scale_log2;
        float m = -INFINITY, l = 0.f;
        bool ok = t < ntiles;
        for (int j = 0; ok && j < nkv; ++j) {
            ok = mbar_wait(&s_full[t], static_cast<uint32_t>(j & 1), abort_flag, status, 29);
            if (!__all_sync(0xffffffffu, ok)) {
                ok = false;
                break;
            }
            tc_fence_after();
            // all four 32-column loads in flight before one wait
            uint32_t sc[128];
            tmem_ld_32x32b_x32(s_col + 0u, *reinterpret_cast<uint32_t(*)[32]>(&sc[0]));
            tmem_ld_32x32b_x32(s_col + 32u, *reinterpret_cast<uint32_t(*)[32]>(&sc[32]));
            tmem_ld_32x32b_x32(s_col + 64u, *reinterpret_cast<uint32_t(*)[32]>(&sc[64]));
            tmem_ld_32x32b_x32(s_col + 96u, *reinterpret_cast<uint32_t(*)[32]>(&sc[96]));
            tmem_ld_wait();
            // the loaded registers are defined only after the wait: route them
            // through it so no use is scheduled ahead of it
#pragma unroll
            for (int i = 0; i < 128; ++i) asm volatile("" : "+r"(sc[i]));
            float mx = row_max128(sc) * c;  // scale > 0: the max of the scaled scores
            if (j == 0) {
                m = mx;
            } else if (__any_sync(0xffffffffu, mx > m + kRescaleThreshold)) {
                // raise the running max of the rows that need it; O_t (after the
                // previous P.V, complete before these scores were produced) and l
                const float m_new = mx > m + kRescaleThreshold ? mx : m;
                const float alpha = ex2(m - m_new);
#pragma unroll 1
                for (int cc = 0; cc < 4; ++cc) {
                    uint32_t r[32];
                    tmem_ld_32x32b_x32(o_col + static_cast<uint32_t>(cc * 32), r);
                    tmem_ld_wait();
#pragma unroll
                    for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * alpha);
                    tmem_st_32x32b_x32(o_col + static_cast<uint32_t>(cc * 32), r);
                }
                l *= alpha;
                m = m_new;
            }
            // P = 2^(s*c - m) as bf16 pairs over the first 64 score columns; the
            // arguments and the row sum in packed pairs, the sum in four
            // independent accumulators
            const uint64_t c2 = pack_f32x2(c, c), nm2 = pack_f32x2(-m, -m);
            uint64_t acc[4] = {0ull, 0ull, 0ull, 0ull};
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                uint32_t w[32];
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    const int k = h * 64 + 2 * i;
                    const uint64_t x2 = fma_f32x2(pack_f32x2(__uint_as_float(sc[k]), __uint_as_float(sc[k + 1])), c2, nm2);
                    float e0, e1;
                    if ((kEx2FmaMask >> (i % 16)) & 1u) {
                        ex2_fma_x2(x2, e0, e1);
                    } else {
                        float x0, x1;
                        unpack_f32x2(x2, x0, x1);
                        e0 = ex2(x0);
                        e1 = ex2(x1);
                    }
                    acc[i & 3] = add_f32x2(acc[i & 3], pack_f32x2(e0, e1));
                    w[i] = pack_bf16x2(e0, e1);
                }
                tmem_st_32x32b_x32(s_col + static_cast<uint32_t>(h * 32), w);
            }
            tmem_st_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&p_full[t]);
            float a0, a1, a2, a3, a4, a5, a6, a7;
            unpack_f32x2(acc[0], a0, a1);
            unpack_f32x2(acc[1], a2, a3);
            unpack_f32x2(acc[2], a4, a5);
            unpack_f32x2(acc[3], a6, a7);
            l += ((a0 + a1) + (a2 + a3)) + ((a4 + a5) + (a6 + a7));
        }
        // epilogue: O / l -> bf16, staged in shared memory (the K slots are free
        // once the tile's last P.V has completed: every MMA that reads K was
        // issued before it, and the tensor core retires them in order) in the
        // 128-byte-swizzled layout of the
        // tensor map, then written by two TMA stores per tile: 16-byte stores
        // from registers, one row per thread, took ~4000 cycles per CTA
        if (ok && nkv > 0) {
            ok = mbar_wait(&o_done[t], 0, abort_flag, status, 32);
            if (__all_sync(0xffffffffu, ok)) {
                tc_fence_after();
                const float inv = 1.0f / l;
                uint8_t* so = sK + t * kTile;  // [2 halves of 64 columns][128 rows][128 bytes]
#pragma unroll 1
                for (int cc = 0; cc < 4; ++cc) {
                    uint32_t r[32];
                    tmem_ld_32x32b_x32(o_col + static_cast<uint32_t>(cc * 32), r);
                    tmem_ld_wait();
                    uint8_t* half_row = so + (cc >> 1) * kHalf + row * 128;
#pragma unroll
                    for (int v = 0; v < 4; ++v) {
                        uint4 o;
                        o.x = pack_bf16x2(__uint_as_float(r[8 * v + 0]) * inv, __uint_as_float(r[8 * v + 1]) * inv);
                        o.y = pack_bf16x2(__uint_as_float(r[8 * v + 2]) * inv, __uint_as_float(r[8 * v + 3]) * inv);
                        o.z = pack_bf16x2(__uint_as_float(r[8 * v + 4]) * inv, __uint_as_float(r[8 * v + 5]) * inv);
                        o.w = pack_bf16x2(__uint_as_float(r[8 * v + 6]) * inv, __uint_as_float(r[8 * v + 7]) * inv);
                        const int chunk = (cc & 1) * 4 + v;  // 16-byte chunk within the 128-byte row
                        *reinterpret_cast<uint4*>(half_row + ((chunk ^ (row & 7)) << 4)) = o;
                    }
                }
                fence_async_smem();
                __syncwarp();
                if (lane == 0) mbar_arrive(&o_ready[t]);
                if (q == 0 && lane == 0) {
                    if (mbar_wait(&o_ready[t], 0, abort_flag, status, 36)) {
                        tma_store_3d(&tmO, so, 0, q0 + t * kBlock, head);
                        tma_store_3d(&tmO, so + kHalf, 64, q0 + t * kBlock, head);
                        tma_store_commit();
                        tma_store_wait_read();
                    }
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc<512>(tmem);
}

PFN_cuTensorMapEncodeTiled_v12000 encode() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            return static_cast<PFN_cuTensorMapEncodeTiled_v12000>(nullptr);
        return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    }();
    return fn;
}

// [heads, seq, 128] bf16 viewed as {128, seq, heads}, 64x128 boxes, 128-byte swizzle.
int make_qkv_map(CUtensorMap* map, const void* ptr, size_t heads, size_t seq) {
    auto enc = encode();
    if (!enc) return fail(cudaErrorNotSupported, "attention: cuTensorMapEncodeTiled unavailable");
    cuuint64_t dims[3] = {static_cast<cuuint64_t>(kHead), static_cast<cuuint64_t>(seq), static_cast<cuuint64_t>(heads)};
    cuuint64_t strides[2] = {kHead * 2, static_cast<cuuint64_t>(seq) * kHead * 2};
    cuuint32_t box[3] = {64, kBlock, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(ptr), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(cudaErrorInvalidValue, "attention: tensor map encoding failed (CUresult %d)", int(r));
    return 0;
}

}  // namespace

int attention_status_take(int* code) {
    int zero = 0;
    cudaError_t e = cudaMemcpyFromSymbol(code, g_attn_status, sizeof(int));
    if (e == cudaSuccess) e = cudaMemcpyToSymbol(g_attn_status, &zero, sizeof(int));
    return static_cast<int>(e);
}

}  // namespace bee_b200

using namespace bee_b200;

extern "C" int bee_b200_attention(int dt, const void* q, const void* k, const void* v, void* o, size_t heads,
                                  size_t seq, size_t head_dim, float scale, bee_b200_stream_t stream) {
    if (heads == 0 || seq == 0) return ok();
    if (!q || !k || !v || !o) return fail(cudaErrorInvalidValue, "attention: null pointer");
    if (dt != DT_BF16) return fail(cudaErrorInvalidValue, "attention: dtype %d unsupported (BF16 only)", dt);
    if (head_dim != static_cast<size_t>(kHead))
        return fail(cudaErrorInvalidValue, "attention: head_dim %zu unsupported (128 only)", head_dim);
    if (seq % kBlock != 0 || seq > (1u << 30) || heads > 65535)
        return fail(cudaErrorInvalidValue, "attention: seq %zu must be a multiple of %d", seq, kBlock);
    if (!(scale > 0.0f) || !(scale < 3.0e38f))
        return fail(cudaErrorInvalidValue, "attention: scale must be positive and finite");
    if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(o))
        return fail(cudaErrorInvalidValue, "attention: buffers must be 16-byte aligned");
    CUtensorMap tq, tk, tv, to;
    if (int rc = make_qkv_map(&tq, q, heads, seq)) return rc;
    if (int rc = make_qkv_map(&tk, k, heads, seq)) return rc;
    if (int rc = make_qkv_map(&tv, v, heads, seq)) return rc;
    if (int rc = make_qkv_map(&to, o, heads, seq)) return rc;
    AttnParams p;
    p.seq = static_cast<int>(seq);
    p.nkv = static_cast<int>(seq / kBlock);
    p.scale_log2 = scale * 1.4426950408889634f;
    // setmaxnreg.inc waits until the registers it asks for are free, so the
    // split is only safe when the kernel launches with exactly kRegsLaunch
    static std::atomic<int> launch_regs{0};
    int regs = launch_regs.load(std::memory_order_acquire);
    if (regs == 0) {
        cudaFuncAttributes fa;
        cudaError_t e = cudaFuncGetAttributes(&fa, attention_fwd_kernel);
        if (e != cudaSuccess) return api_fail(e, "attention: kernel attributes: %s", cudaGetErrorString(e));
        regs = fa.numRegs;
        launch_regs.store(regs, std::memory_order_release);
    }
    if (regs != kRegsLaunch)
        return fail(cudaErrorLaunchOutOfResources, "attention: kernel built with %d registers per thread, the register "
                    "split assumes %d", regs, kRegsLaunch);
    static SmemLimit smem_limit;
    if (int rc = smem_limit.ensure(attention_fwd_kernel, kSmem, "attention")) return rc;
    dim3 grid(static_cast<unsigned>((seq / kBlock + 1) / 2), static_cast<unsigned>(heads));
    attention_fwd_kernel<<<grid, kThreads, kSmem, as_stream(stream)>>>(tq, tk, tv, to, p);
    return launch_status("attention");
}
