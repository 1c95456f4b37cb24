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
//
// Scheduling.  A unit is one head's pair of query tiles.  By default one CTA
// runs one unit (attention_fwd_kernel on a (pair, head) grid).  When the units
// outnumber the SMs and the last wave would leave most of them idle (a cost
// model on the host), attention_shares_kernel runs one persistent CTA per SM
// over an equal contiguous share of the (unit, key block) sequence instead; a
// unit cut between two CTAs is computed as two pieces whose unnormalised O and
// (m, l) go to scratch, and the piece that takes the unit's ticket second
// merges them (no CTA ever waits for another).
// Every wait is bounded; a wait that gives up records a code in the status
// word read by bee_b200_device_status and the CTA abandons its work.
#include <cuda.h>
#include <cmath>
#include <mutex>
#include <type_traits>
#include <vector>
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
// scratch of one cut unit: two pieces x two tiles of fp32 O (128 x 128), then (m, l) per row
constexpr size_t kSlotPartBytes = 2 * 2 * 128 * 128 * sizeof(float);
constexpr size_t kSlotBytes = kSlotPartBytes + 2 * 2 * 128 * 2 * sizeof(float);

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
    int seq;            // queries == keys per head (multiple of 128)
    int nkv;            // seq / 128
    int npairs;         // query-tile pairs per head
    float scale_log2;   // scale * log2(e)
    long long blocks;   // units * nkv: the (unit, key block) sequence the CTAs share
    float4* part;       // partial O of cut units: [slot][piece][tile][32 chunks of 4][128 rows]
    float2* part_ml;    // their (m, l): [slot][piece][tile][128 rows]
    unsigned* tickets;  // [slot], zero between launches
};

// A CTA's piece of one unit (a head's pair of query tiles): key blocks
// j0 .. j0 + len - 1.  A unit cut between two CTAs has a piece 0 (keys from
// block 0, the end of the earlier CTA's range) and a piece 1 (keys to the last
// block, the start of the later CTA's range); slot = the later CTA's index.
struct Segment {
    int head, q0, ntiles, j0, len;
    bool cut;
    int piece, slot;
};

__device__ __forceinline__ Segment segment_at(long long g, long long g_end, const AttnParams& p) {
    Segment s;
    const long long u = g / p.nkv;
    s.j0 = static_cast<int>(g - u * p.nkv);
    const long long rest = g_end - g;
    s.len = static_cast<int>(rest < static_cast<long long>(p.nkv - s.j0) ? rest : static_cast<long long>(p.nkv - s.j0));
    s.head = static_cast<int>(u / p.npairs);
    s.q0 = static_cast<int>(u - static_cast<long long>(s.head) * p.npairs) * 2 * kBlock;
    s.ntiles = s.q0 + kBlock < p.seq ? 2 : 1;  // the last pair of an odd tile count has only tile A
    s.cut = s.len != p.nkv;
    s.piece = s.j0 == 0 ? 0 : 1;
    s.slot = static_cast<int>(blockIdx.x) + (s.piece == 0 ? 1 : 0);
    return s;
}

__device__ __forceinline__ void named_bar_sync(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

__device__ __forceinline__ void mbar_inval(uint64_t* bar) {
    asm volatile("mbarrier.inval.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}

constexpr int kThreads = 384;  // warpgroup 0: TMA warp, MMA warp, 2 idle; warpgroups 1-2: softmax
// Register split.  The launch gives every thread 168 registers (three warps per
// SM sub-partition, 16384 registers each); warpgroup 0 drops to 56 and the two
// softmax warpgroups take what it frees, so the total stays what was launched.
constexpr int kRegsLaunch = 168, kRegsControl = 56, kRegsSoftmax = 224;
static_assert(kRegsControl * 128 + kRegsSoftmax * 256 <= kRegsLaunch * kThreads,
              "setmaxnreg split exceeds the registers the block was launched with");
static_assert(kRegsLaunch * kThreads <= 65536 && kRegsLaunch * 3 * 32 <= 16384, "launch register budget");
constexpr int kBarSegment = 1;  // named barrier of all 384 threads between segments
constexpr int kBarSoftmax = 2;  // named barrier of the 256 softmax threads (cut-unit tickets)

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
        // first block barrier, once the previous kernel on the stream has completed
        // (the launch may overlap its tail)
        pdl_wait();
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
    pdl_wait();     // every thread, before its first global access (O)
    pdl_trigger();  // the next kernel may launch once every CTA, second wave included, has started

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

// One persistent CTA per SM (1-D grid) runs its share of the (unit, key block)
// sequence as segments: the same per-block pipeline as attention_fwd_kernel,
// with the barriers re-created between segments and the pieces of a unit cut
// between two CTAs merged by whichever finishes second.
__global__ void __launch_bounds__(kThreads, 1) attention_shares_kernel(const __grid_constant__ CUtensorMap tmQ,
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
    __shared__ int merge_sh;  // this CTA's piece of a cut unit arrived second: it merges
    // [0]: start of the current segment in the (unit, key block) sequence, [1]: end of
    // this CTA's share.  Kept in shared memory, not registers: the softmax loop runs at
    // the register limit.
    __shared__ long long seg_sh[2];

    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sQ = smem;            // [2] tiles A, B
    uint8_t* sK = sQ + 2 * kTile;  // [2] ring
    uint8_t* sV = sK + 2 * kTile;  // [2] ring
    volatile int* abort_flag = &abort_sh;
    int* status = &g_attn_status;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    // barrier set of one segment (re-created for each: every phase starts at 0)
    auto init_barriers = [&](bool again) {
        if (again) {
            uint64_t* all[14] = {&q_full,   &op_full[0], &op_full[1], &op_empty[0], &op_empty[1],
                                 &s_full[0], &s_full[1],  &p_full[0],  &p_full[1],   &done_bar,
                                 &o_done[0], &o_done[1],  &o_ready[0], &o_ready[1]};
            for (uint64_t* b : all) mbar_inval(b);
        }
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
        fence_mbar_init();
    };
    // Q_A, Q_B and K_{j0} (into the K slot of stage 1) of a segment, on q_full
    auto first_loads = [&](const Segment& s) {
        mbar_arrive_expect_tx(&q_full, static_cast<uint32_t>((s.ntiles + 1) * kTile));
        for (int t = 0; t < s.ntiles; ++t) {
            tma_load_3d(sQ + t * kTile, &tmQ, &q_full, 0, s.q0 + t * kBlock, s.head);
            tma_load_3d(sQ + t * kTile + kHalf, &tmQ, &q_full, 64, s.q0 + t * kBlock, s.head);
        }
        tma_load_3d(sK + kTile, &tmK, &q_full, 0, s.j0 * kBlock, s.head);
        tma_load_3d(sK + kTile + kHalf, &tmK, &q_full, 64, s.j0 * kBlock, s.head);
    };
    // Between segments: every role has finished (loads landed, MMAs retired, TMEM
    // reads waited, O stores have read shared memory); thread 0 moves the cursor,
    // re-creates the barriers and starts the next segment's first loads.  Every
    // thread passes both barriers once per segment, abandoned or not, and reads the
    // cursor only between them and the next segment's end.
    auto next_segment = [&](int len) {
        tc_fence_before();
        named_bar_sync(kBarSegment, kThreads);
        if (threadIdx.x == 0) {
            const long long g = seg_sh[0] + len;
            seg_sh[0] = g;
            if (g < seg_sh[1] && *abort_flag == 0) {
                init_barriers(true);
                first_loads(segment_at(g, seg_sh[1], p));
            }
        }
        named_bar_sync(kBarSegment, kThreads);
        tc_fence_after();
    };

    if (threadIdx.x == 0) {
        abort_sh = 0;
        init_barriers(false);
        // thread 0 is also the TMA thread: the first segment's loads start now,
        // under the TMEM allocation and the first block barrier
        // this CTA's contiguous share of the (unit, key block) sequence
        const long long g_begin = p.blocks * blockIdx.x / gridDim.x;
        const long long g_end = p.blocks * (blockIdx.x + 1) / gridDim.x;
        seg_sh[0] = g_begin;
        seg_sh[1] = g_end;
        if (g_begin < g_end) first_loads(segment_at(g_begin, g_end, p));
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
        while (seg_sh[0] < seg_sh[1]) {
            const Segment sg = segment_at(seg_sh[0], seg_sh[1], p);
            const bool live = __all_sync(0xffffffffu, *abort_flag == 0);  // one value per warp
            if (warp == 0 && live) {
                // ------------------------------------------------ TMA producer
                if (lane == 0) {
                    // stage s = j & 1 takes V_j and K_{j+1}; stage 1 is first released
                    // by the MMA that read K_{j0}, so its waits run one phase behind stage 0's
                    int filled = 0;
                    for (int j = 0; j < sg.len; ++j) {
                        const int s = j & 1;
                        const uint32_t par = static_cast<uint32_t>((j >> 1) & 1) ^ (s == 0 ? 1u : 0u);
                        if (!mbar_wait(&op_empty[s], par, abort_flag, status, 21)) break;
                        const bool knext = j + 1 < sg.len;
                        const int kb = sg.j0 + j;
                        mbar_arrive_expect_tx(&op_full[s], static_cast<uint32_t>((knext ? 2 : 1) * kTile));
                        tma_load_3d(sV + s * kTile, &tmV, &op_full[s], 0, kb * kBlock, sg.head);
                        tma_load_3d(sV + s * kTile + kHalf, &tmV, &op_full[s], 64, kb * kBlock, sg.head);
                        if (knext) {
                            tma_load_3d(sK + s * kTile, &tmK, &op_full[s], 0, (kb + 1) * kBlock, sg.head);
                            tma_load_3d(sK + s * kTile + kHalf, &tmK, &op_full[s], 64, (kb + 1) * kBlock, sg.head);
                        }
                        filled = j + 1;
                    }
                    // the segment's loads must have landed before its barriers are
                    // re-created or the CTA exits (normally the MMA warp consumed them already)
                    mbar_wait(&q_full, 0, abort_flag, status, 33, 200000000ull);
                    for (int j = filled > 2 ? filled - 2 : 0; j < filled; ++j)
                        mbar_wait(&op_full[j & 1], static_cast<uint32_t>((j >> 1) & 1), abort_flag, status, 34,
                                  200000000ull);
                }
                __syncwarp();
            } else if (warp == 1 && live) {
                // ------------------------------------------------ MMA issuer
                if (lane == 0) {
                    // Shared-memory descriptors of the operand slots, built once: a thread
                    // that rebuilt both descriptors per MMA took about as long to issue a
                    // 128x128x16 product as the tensor core takes to retire it.
                    const uint64_t dq0 = sdesc_sw128(smem_u32(sQ), 16, 1024), dq1 = sdesc_sw128(smem_u32(sQ + kTile), 16, 1024);
                    const uint64_t dk0 = sdesc_sw128(smem_u32(sK), 16, 1024), dk1 = sdesc_sw128(smem_u32(sK + kTile), 16, 1024);
                    const uint64_t dv0 = sdesc_sw128(smem_u32(sV), kHalf, 1024), dv1 = sdesc_sw128(smem_u32(sV + kTile), kHalf, 1024);
                    MmaRing r{tmem, {dq0, dq1}, {dk0, dk1}, {dv0, dv1}, op_full, op_empty, s_full, p_full, o_done,
                              abort_flag, status, sg.len};
                    bool ok = mbar_wait(&q_full, 0, abort_flag, status, 23);
                    const bool issued = ok && sg.len > 0;
                    if (sg.ntiles == 2)
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
            next_segment(sg.len);
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
        while (seg_sh[0] < seg_sh[1]) {
            // only the segment's length and tile count stay live through the block
            // loop (the rest is read again after it): it runs at the register limit
            int len, ntiles;
            {
                const Segment s0 = segment_at(seg_sh[0], seg_sh[1], p);
                len = s0.len;
                ntiles = s0.ntiles;
            }
            float m = -INFINITY, l = 0.f;
            bool ok = __all_sync(0xffffffffu, *abort_flag == 0) && t < ntiles;  // one value per warp
            for (int j = 0; ok && j < len; ++j) {
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
            const Segment sg = segment_at(seg_sh[0], seg_sh[1], p);
            if (ok) {
                ok = mbar_wait(&o_done[t], 0, abort_flag, status, 32);
                ok = __all_sync(0xffffffffu, ok);
            }
            // Epilogue: O / l -> bf16, staged in shared memory (the K slots are free
            // once the tile's last P.V has completed: every MMA that reads K was
            // issued before it, and the tensor core retires them in order) in the
            // 128-byte-swizzled layout of the tensor map, then written by two TMA
            // stores per tile: 16-byte stores from registers, one row per thread,
            // took ~4000 cycles per CTA.  value(cc, v, r, x) fills x with columns
            // 32 cc + 8 v .. + 7 of this row's output, r holding its O columns
            // 32 cc .. + 31 from TMEM.
            auto store_tile = [&](auto value) {
                uint8_t* so = sK + t * kTile;  // [2 halves of 64 columns][128 rows][128 bytes]
#pragma unroll 1
                for (int cc = 0; cc < 4; ++cc) {
                    uint32_t r[32];
                    tmem_ld_32x32b_x32(o_col + static_cast<uint32_t>(cc * 32), r);
                    tmem_ld_wait();
                    uint8_t* half_row = so + (cc >> 1) * kHalf + row * 128;
#pragma unroll
                    for (int v = 0; v < 4; ++v) {
                        float x[8];
                        value(cc, v, r, x);
                        uint4 o;
                        o.x = pack_bf16x2(x[0], x[1]);
                        o.y = pack_bf16x2(x[2], x[3]);
                        o.z = pack_bf16x2(x[4], x[5]);
                        o.w = pack_bf16x2(x[6], x[7]);
                        const int chunk = (cc & 1) * 4 + v;  // 16-byte chunk within the 128-byte row
                        *reinterpret_cast<uint4*>(half_row + ((chunk ^ (row & 7)) << 4)) = o;
                    }
                }
                fence_async_smem();
                __syncwarp();
                if (lane == 0) mbar_arrive(&o_ready[t]);
                if (q == 0 && lane == 0) {
                    if (mbar_wait(&o_ready[t], 0, abort_flag, status, 36)) {
                        tma_store_3d(&tmO, so, 0, sg.q0 + t * kBlock, sg.head);
                        tma_store_3d(&tmO, so + kHalf, 64, sg.q0 + t * kBlock, sg.head);
                        tma_store_commit();
                        tma_store_wait_read();
                    }
                }
            };
            if (!sg.cut) {
                if (ok) {
                    tc_fence_after();
                    const float inv = 1.0f / l;
                    store_tile([&](int, int v, const uint32_t (&r)[32], float (&x)[8]) {
#pragma unroll
                        for (int i = 0; i < 8; ++i) x[i] = __uint_as_float(r[8 * v + i]) * inv;
                    });
                }
            } else {
                // A piece of a cut unit: both pieces write their unnormalised O and
                // (m, l); the one that takes the slot's ticket second merges them and
                // re-arms the ticket.  The merge is symmetric in the two pieces
                // (separate roundings, no fused multiply-add), so the result does not
                // depend on which piece arrives second.  Chunk-major rows: a warp's
                // access is 512 contiguous bytes.
                const size_t mine = (static_cast<size_t>(sg.slot) * 2 + sg.piece) * 2 + t;
                const size_t other = (static_cast<size_t>(sg.slot) * 2 + (1 - sg.piece)) * 2 + t;
                if (ok) {
                    tc_fence_after();
                    float4* dst = p.part + mine * 32 * 128 + row;
#pragma unroll 1
                    for (int cc = 0; cc < 4; ++cc) {
                        uint32_t r[32];
                        tmem_ld_32x32b_x32(o_col + static_cast<uint32_t>(cc * 32), r);
                        tmem_ld_wait();
#pragma unroll
                        for (int v = 0; v < 8; ++v)
                            __stcg(dst + (cc * 8 + v) * 128,
                                   make_float4(__uint_as_float(r[4 * v]), __uint_as_float(r[4 * v + 1]),
                                               __uint_as_float(r[4 * v + 2]), __uint_as_float(r[4 * v + 3])));
                    }
                    __stcg(p.part_ml + mine * 128 + row, make_float2(m, l));
                }
                __threadfence();
                named_bar_sync(kBarSoftmax, 256);
                if (threadIdx.x == 128) merge_sh = atomicAdd(&p.tickets[sg.slot], 1u) == 1u ? 1 : 0;
                named_bar_sync(kBarSoftmax, 256);
                const bool merge = merge_sh != 0;
                if (merge && ok) {
                    __threadfence();
                    const float2 ml2 = __ldcg(p.part_ml + other * 128 + row);
                    const float mm = fmaxf(m, ml2.x);
                    const float a_me = ex2(m - mm), a_ot = ex2(ml2.x - mm);
                    const float inv = 1.0f / __fadd_rn(__fmul_rn(l, a_me), __fmul_rn(ml2.y, a_ot));
                    const float4* src = p.part + other * 32 * 128 + row;
                    store_tile([&](int cc, int v, const uint32_t (&r)[32], float (&x)[8]) {
                        const float4 o0 = __ldcg(src + (cc * 8 + 2 * v) * 128);
                        const float4 o1 = __ldcg(src + (cc * 8 + 2 * v + 1) * 128);
                        const float ot[8] = {o0.x, o0.y, o0.z, o0.w, o1.x, o1.y, o1.z, o1.w};
#pragma unroll
                        for (int i = 0; i < 8; ++i)
                            x[i] = __fmul_rn(__fadd_rn(__fmul_rn(__uint_as_float(r[8 * v + i]), a_me), __fmul_rn(ot[i], a_ot)), inv);
                    });
                }
                if (merge && threadIdx.x == 128) p.tickets[sg.slot] = 0u;
            }
            next_segment(sg.len);
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

// Tickets of the cut units: one zeroed block of kMaxSlots per (device, stream),
// taken from the stream-ordered pool on the stream's first call and kept for
// the life of the process (the merging CTA re-arms each ticket it takes, so
// later calls need no memset).  Streams are keyed by cudaStreamGetId, which is
// never reused.  Returns 1 during stream capture or past 256 streams on a
// device: the call then runs one unit per CTA, with no cut units.
constexpr int kMaxSlots = 1024;

struct TicketBlock {
    unsigned long long id;
    unsigned* ptr;
};

int stream_tickets(cudaStream_t st, unsigned** out) {
    static std::mutex mu;
    static std::vector<TicketBlock> table[64];
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(st, &cap) != cudaSuccess || cap != cudaStreamCaptureStatusNone) return 1;
    unsigned long long id = 0;
    int dev = 0;
    if (cudaStreamGetId(st, &id) != cudaSuccess || cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 1;
    std::lock_guard<std::mutex> lock(mu);
    for (const TicketBlock& e : table[dev])
        if (e.id == id) {
            *out = e.ptr;
            return 0;
        }
    if (table[dev].size() >= 256) return 1;
    void* ptr = nullptr;
    if (pool_malloc(&ptr, kMaxSlots * sizeof(unsigned), st) != cudaSuccess) return 1;
    if (cudaMemsetAsync(ptr, 0, kMaxSlots * sizeof(unsigned), st) != cudaSuccess) {
        cudaFreeAsync(ptr, st);
        return 1;
    }
    table[dev].push_back({id, static_cast<unsigned*>(ptr)});
    *out = static_cast<unsigned*>(ptr);
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
    // setmaxnreg.inc waits until the registers it asks for are free, so the
    // split is only safe when the kernel launches with exactly kRegsLaunch
    static std::atomic<int> launch_regs{0};
    int regs = launch_regs.load(std::memory_order_acquire);
    if (regs == 0) {
        cudaFuncAttributes fa, fb;
        cudaError_t e = cudaFuncGetAttributes(&fa, attention_fwd_kernel);
        if (e == cudaSuccess) e = cudaFuncGetAttributes(&fb, attention_shares_kernel);
        if (e != cudaSuccess) return api_fail(e, "attention: kernel attributes: %s", cudaGetErrorString(e));
        regs = fa.numRegs == fb.numRegs ? fa.numRegs : -1;
        launch_regs.store(regs, std::memory_order_release);
    }
    if (regs != kRegsLaunch)
        return fail(cudaErrorLaunchOutOfResources, "attention: kernels built with %d registers per thread (-1: the two "
                    "differ), the register split assumes %d", regs, kRegsLaunch);
    static SmemLimit smem_units, smem_shares;
    if (int rc = smem_units.ensure(attention_fwd_kernel, kSmem, "attention")) return rc;
    if (int rc = smem_shares.ensure(attention_shares_kernel, kSmem, "attention")) return rc;
    // Units (a head's pair of query tiles) and the CTAs that run them.  By default
    // one CTA per unit.  With more units than SMs and a last wave that would leave
    // most SMs idle, one persistent CTA per SM instead takes an equal contiguous
    // share of the (unit, key block) sequence; a unit cut between two CTAs is
    // merged by whichever finishes second.  Every segment a CTA runs costs about
    // kSegmentCost key blocks of pipeline fill and drain (measured: two whole units
    // per CTA take as long as two waves of fresh CTAs) and a cut unit about
    // kMergeCost more, so the shares are used only where that model gains 10%:
    // 160 units of 16 blocks on 148 SMs, 16% faster; 256 units, 17% slower.
    const size_t npairs = (seq / kBlock + 1) / 2;
    const size_t units = heads * npairs;
    if (units > (1u << 30)) return fail(cudaErrorInvalidValue, "attention: %zu units of work exceed the grid", units);
    const size_t sms = static_cast<size_t>(sm_count());
    const cudaStream_t st = as_stream(stream);
    size_t ctas = units;
    void* part = nullptr;
    unsigned* tickets = nullptr;
    if (units > sms && units % sms != 0) {
        constexpr double kSegmentCost = 3.5, kMergeCost = 5.0;  // in key blocks
        const double nkv = static_cast<double>(seq / kBlock);
        const double waves = static_cast<double>((units + sms - 1) / sms);
        const double share = static_cast<double>(units) * nkv / static_cast<double>(sms);
        const double segments = std::ceil(share / nkv) + 1.0;  // most a share can touch
        const double t_units = waves * (nkv + kSegmentCost);
        const double t_shares = share + segments * kSegmentCost + kMergeCost;
        if (t_shares < 0.9 * t_units && sms <= static_cast<size_t>(kMaxSlots)) {
            if (stream_tickets(st, &tickets) == 0 && pool_malloc(&part, sms * kSlotBytes, st) == cudaSuccess) {
                ctas = sms;
            } else {
                cudaGetLastError();  // keep one unit per CTA
                part = nullptr;
                tickets = nullptr;
            }
        }
    }
    AttnParams p;
    p.seq = static_cast<int>(seq);
    p.nkv = static_cast<int>(seq / kBlock);
    p.npairs = static_cast<int>(npairs);
    p.scale_log2 = scale * 1.4426950408889634f;
    p.blocks = static_cast<long long>(units) * p.nkv;
    p.part = static_cast<float4*>(part);
    p.part_ml = part ? reinterpret_cast<float2*>(static_cast<uint8_t*>(part) + ctas * kSlotPartBytes) : nullptr;
    p.tickets = tickets;
    if (part)
        attention_shares_kernel<<<static_cast<unsigned>(ctas), kThreads, kSmem, st>>>(tq, tk, tv, to, p);
    else
        launch_pdl(attention_fwd_kernel, dim3(static_cast<unsigned>(npairs), static_cast<unsigned>(heads)), kThreads, kSmem,
                   st, tq, tk, tv, to, p);
    int rc = launch_status("attention");
    if (part) {
        cudaError_t e = cudaFreeAsync(part, st);
        if (rc == 0 && e != cudaSuccess) rc = api_fail(e, "attention: scratch release: %s", cudaGetErrorString(e));
    }
    return rc;
}
