// Shared device helpers and host-side status plumbing for the bee_b200 kernels.
//
// Conventions mirror the reference's int-returning kernel bridge
// (Bee/CUDA/Ops/OpsBridge.hpp:22-43): every entry point returns a plain int,
// 0 on success, otherwise a cudaError_t value.  Argument problems detected on
// the host return cudaErrorInvalidValue (1) and leave a readable message in a
// thread-local buffer (bee_b200_last_error()).
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <atomic>
#include <cstddef>
#include <cstdint>

#include "bee_b200.h"

namespace bee_b200 {

// dtype codes: identical to bee::DType (Bee/Tensor/Core/DType.hpp:17-32).
enum DT : int {
    DT_BOOL = 0, DT_U8 = 1, DT_I32 = 2, DT_I64 = 3, DT_F32 = 4, DT_F64 = 5,
    DT_I8 = 6, DT_F16 = 7, DT_BF16 = 8,
};

// op codes: identical to bee::cuda::BinaryOp / UnaryOp / ReduceOp
// (Bee/CUDA/Api.hpp:77-100).
enum BinOp : int { OP_ADD = 0, OP_SUB = 1, OP_MUL = 2, OP_DIV = 3 };
enum UnOp : int { OP_NEG = 0, OP_ABS = 1, OP_SQRT = 2, OP_EXP = 3, OP_LOG = 4 };
enum RedOp : int { RED_SUM = 0, RED_MIN = 1, RED_MAX = 2, RED_PROD = 3 };

// Records a message for bee_b200_last_error() and returns `code`.
int fail(int code, const char* fmt, ...);
// fail() for a failed CUDA runtime call: also clears the runtime's last error,
// so that the next launch check does not report it again.
int api_fail(cudaError_t e, const char* fmt, ...);
// Clears the thread-local message; returns 0.
int ok();
// Converts the pending launch error (if any) into a status.
int launch_status(const char* what);

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Programmatic dependent launch.  A kernel launched by launch_pdl may start
// (its CTAs scheduled, its prologue run) while the previous kernel on the
// stream finishes; it must call pdl_wait() before its first global-memory
// access, which returns once that kernel has completed and its writes are
// visible (for a normal launch, or after a copy or a kernel that never calls
// pdl_trigger, it returns at once).  pdl_trigger() lets the next such kernel
// start launching; a CTA that exits without it counts as having called it.
// Measured on back-to-back [8192, 8192] fp32 adds: 2.3 us less per launch.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <typename... KArgs, typename... Args>
inline void launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);  // errors reach launch_status via cudaGetLastError
}

// Raises a kernel's dynamic shared-memory limit once per device
// (cudaFuncSetAttribute applies to the current device); safe to call from any
// host thread.  Keep one instance per kernel as a function-local static.
constexpr int kMaxDevices = 64;
struct SmemLimit {
    std::atomic<int> raised[kMaxDevices];
    template <typename Kernel>
    int ensure(Kernel kernel, int bytes, const char* what) {
        int dev = 0;
        if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
            return fail(cudaErrorInvalidDevice, "%s: no usable current device", what);
        if (raised[dev].load(std::memory_order_acquire) >= bytes) return 0;
        cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
        if (e != cudaSuccess) return api_fail(e, "%s: shared memory attribute: %s", what, cudaGetErrorString(e));
        raised[dev].store(bytes, std::memory_order_release);
        return 0;
    }
};

// Number of SMs of the current device (cached per device ordinal).
int sm_count();

// Stream-ordered allocation from the current device's default memory pool,
// whose release threshold is raised to the maximum on first use (as the
// reference's MemoryPool::get_default does, Bee/CUDA/Mem/MemoryPool.hpp:33-49)
// so freed blocks stay reserved and later allocations are sub-allocations.
cudaError_t pool_malloc(void** ptr, size_t bytes, cudaStream_t st);

// Reads and clears the status word of the fused attention kernel (cudaError_t).
int attention_status_take(int* code);
// Reads and clears the status word of the cross-GPU reduce (a peer that never arrived).
int allranks_status_take(int* code);

inline cudaStream_t as_stream(bee_b200_stream_t s) { return reinterpret_cast<cudaStream_t>(s); }

// ---------------------------------------------------------------- device side

template <typename T>
__device__ __forceinline__ T warp_sum(T v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Streaming (evict-first) 128-bit global load / store: each input byte of the
// memory-bound kernels is touched exactly once, so keep it out of L1 and mark
// it first-to-evict in L2.
__device__ __forceinline__ float4 ld_stream(const float4* p) { return __ldcs(p); }
__device__ __forceinline__ void st_stream(float4* p, float4 v) { __stcs(p, v); }
__device__ __forceinline__ uint4 ld_stream_u4(const uint4* p) { return __ldcs(p); }
__device__ __forceinline__ void st_stream_u4(uint4* p, uint4 v) { __stcs(p, v); }

__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }
// Packs two floats into a bf16x2 word with round-to-nearest-even (cvt.rn.bf16x2.f32).
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
    __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
}

// Packs two floats into an f16x2 word with round-to-nearest-even (cvt.rn.f16x2.f32).
__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
}

// Packed fp32 pairs (sm_100 .f32x2): one instruction computes both lanes of a
// 64-bit register pair.
__device__ __forceinline__ uint64_t pack_f32x2(float lo, float hi) {
    uint64_t d;
    asm("mov.b64 %0, {%1, %2};" : "=l"(d) : "f"(lo), "f"(hi));
    return d;
}
__device__ __forceinline__ void unpack_f32x2(uint64_t v, float& lo, float& hi) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t fma_f32x2(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
__device__ __forceinline__ uint64_t mul_f32x2(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ uint64_t add_f32x2(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("add.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
// A bf16x2 word as an fp32 pair (exact).
__device__ __forceinline__ uint64_t bf16x2_to_f32x2(uint32_t w) { return pack_f32x2(bf16_lo(w), bf16_hi(w)); }
// An fp32 pair rounded to a bf16x2 word (nearest even).
__device__ __forceinline__ uint32_t f32x2_to_bf16x2(uint64_t v) {
    float lo, hi;
    unpack_f32x2(v, lo, hi);
    return pack_bf16x2(lo, hi);
}

}  // namespace bee_b200
