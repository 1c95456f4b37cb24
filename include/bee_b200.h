/*
 * bee_b200 — C ABI of the B200 (sm_100a) backend for the Bee::Tensor compute path.
 *
 * Every function takes plain device pointers, element counts and a CUDA stream
 * (passed as an opaque pointer; NULL means the legacy default stream) and
 * returns an int status: 0 on success, otherwise a cudaError_t value.  Bad
 * arguments (unknown dtype/op code, sizes that do not fit, misaligned
 * pointers where a kernel needs 16-byte alignment) return 1
 * (cudaErrorInvalidValue) and store a message readable through
 * bee_b200_last_error() on the calling thread.  All compute calls are
 * asynchronous on the given stream; a caller that wants the reference's
 * synchronous semantics synchronises the stream afterwards (the C++ bridge in
 * bee_b200/host does exactly that).  Most kernels launch with programmatic
 * stream serialisation: they may start while the previous kernel on the stream
 * finishes but touch no memory until it has completed, and they let the next
 * such launch start early; a caller's own kernel launched with that attribute
 * right after one of them must wait (griddepcontrol.wait) before reading its
 * outputs.  Ordinary launches, copies and events see plain stream order.
 *
 * Integer codes are the reference's:
 *   dtype   = bee::DType            (Bee/Tensor/Core/DType.hpp:17-32)
 *             Bool 0, U8 1, I32 2, I64 3, F32 4, F64 5, I8 6, F16 7, BF16 8
 *   binary  = bee::cuda::BinaryOp   (Bee/CUDA/Api.hpp:77-83)   Add 0, Sub 1, Mul 2, Div 3
 *   unary   = bee::cuda::UnaryOp    (Bee/CUDA/Api.hpp:85-92)   Neg 0, Abs 1, Sqrt 2, Exp 3, Log 4
 *   reduce  = bee::cuda::ReduceOp   (Bee/CUDA/Api.hpp:94-100)  Sum 0, Min 1, Max 2, Prod 3
 *
 * Each declaration names the reference interface it replaces (file:line).
 */
#ifndef BEE_B200_H
#define BEE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define BEE_B200_API __attribute__((visibility("default")))
#else
#define BEE_B200_API
#endif

typedef void* bee_b200_stream_t; /* a cudaStream_t */

/* ----------------------------------------------------------------- status */

/* Message describing the last failure on this thread ("" after a success). */
BEE_B200_API const char* bee_b200_last_error(void);
/* cudaGetErrorString() for a status returned by this library. */
BEE_B200_API const char* bee_b200_status_string(int status);
/* Library ABI version: major*10000 + minor*100 + patch. */
BEE_B200_API int bee_b200_version(void);

/* ------------------------------------------------------ memory and streams
 * Replace bee::tensor::cuda::allocate / deallocate / memcpy_h2d / memcpy_d2h /
 * memcpy_d2d / memset / synchronize (Bee/Tensor/Cuda/Backend.hpp:20-46,84),
 * which forward to Bee/CUDA/Api.cpp:117-192.  Allocation is stream-ordered
 * from the device's default memory pool, like the reference's
 * cudaMallocFromPoolAsync (Bee/CUDA/Mem/MemoryPool.hpp:55-70); `alignment`
 * above 256 is rejected (pool allocations are 256-byte aligned). */
BEE_B200_API int bee_b200_allocate(void** out_ptr, size_t nbytes, size_t alignment, bee_b200_stream_t stream);
BEE_B200_API int bee_b200_deallocate(void* ptr, bee_b200_stream_t stream);
BEE_B200_API int bee_b200_memcpy_h2d(void* dst, const void* src, size_t nbytes, bee_b200_stream_t stream);
BEE_B200_API int bee_b200_memcpy_d2h(void* dst, const void* src, size_t nbytes, bee_b200_stream_t stream);
BEE_B200_API int bee_b200_memcpy_d2d(void* dst, const void* src, size_t nbytes, bee_b200_stream_t stream);
BEE_B200_API int bee_b200_memset(void* ptr, int value, size_t nbytes, bee_b200_stream_t stream);
BEE_B200_API int bee_b200_stream_synchronize(bee_b200_stream_t stream);

/* Device selection.  Every entry point works on the calling thread's current
 * device (the reference's Device has no index, Bee/Base/Memory/Device.hpp:10);
 * the stream passed to a call must belong to that device.  These wrap
 * cudaSetDevice / cudaGetDevice / cudaGetDeviceCount for callers that do not
 * link the CUDA runtime themselves (one process per GPU: set it once). */
/* Measures the SM clock (MHz) of the SM it lands on over `ns` nanoseconds
 * (<= 10 ms) with one thread, clock64 against the global timer, writing the
 * result to out_mhz (device memory).  Run on a side stream during a timed
 * region, it samples the clock under load without an NVML query. */
BEE_B200_API int bee_b200_clock_probe(unsigned long long ns, float* out_mhz, bee_b200_stream_t stream);
BEE_B200_API int bee_b200_set_device(int device);
BEE_B200_API int bee_b200_get_device(int* device);
BEE_B200_API int bee_b200_device_count(int* count);

/* ------------------------------------------------------------- elementwise */

/* out[i] = a[i] (op) b[i] over n contiguous elements of dtype dt.
 * dt in {U8, I32, I64, F32, F64, F16, BF16}; F16 and BF16 compute in fp32 and
 * round to nearest even.  Replaces ops_binary (Bee/CUDA/Ops/OpsBridge.hpp:27) behind
 * tensor::cuda::ew_binary (Bee/Tensor/Cuda/Backend.hpp:51). */
BEE_B200_API int bee_b200_ew_binary(int op, int dt, const void* a, const void* b, void* out, size_t n,
                       bee_b200_stream_t stream);
/* New: the CUDA side of broadcasting binary ops, which the reference rejects
 * on CUDA (Bee/Tensor/Ops/ElementWise.cpp:110-111) and runs on the CPU with
 * numpy-style broadcasting (Bee/Tensor/Ops/Broadcast.cpp).  out is a
 * contiguous tensor of `shape` (ndim <= 8); a and b are strided views of that
 * shape (strides in elements; 0 on a broadcast dim), so the caller's broadcast
 * (or any non-contiguous operand) needs no materialisation.  Same ops, dtypes
 * and arithmetic as bee_b200_ew_binary. */
BEE_B200_API int bee_b200_ew_binary_strided(int op, int dt, int ndim, const int64_t* shape, const void* a,
                                            const int64_t* a_strides, const void* b, const int64_t* b_strides,
                                            void* out, bee_b200_stream_t stream);


/* dst[i] = op(src[i]).  Neg/Abs: I32, I64, F32, F64, F16, BF16; Sqrt/Exp/Log:
 * F32, F64, F16, BF16.  Replaces ops_unary (Bee/CUDA/Ops/OpsBridge.hpp:28) behind
 * tensor::cuda::ew_unary (Bee/Tensor/Cuda/Backend.hpp:54). */
BEE_B200_API int bee_b200_ew_unary(int op, int dt, const void* src, void* dst, size_t n, bee_b200_stream_t stream);

/* dst[i] = cast(src[i]) between Bool, U8, I32, I64, F32, F64, F16 and BF16.
 * ->BF16 and ->F16 round to nearest even (F64->F16 in one rounding; NaN stays
 * NaN; beyond F16's range is +-inf); ->Bool is (x != 0);
 * float->int truncates toward zero like static_cast.  Replaces ops_cast
 * (Bee/CUDA/Ops/OpsBridge.hpp:29) behind tensor::cuda::ew_cast
 * (Bee/Tensor/Cuda/Backend.hpp:57), which has no BF16 or F16 case
 * (Bee/CUDA/Ops/Cast.cu:96-104). */
BEE_B200_API int bee_b200_ew_cast(int src_dt, const void* src, int dst_dt, void* dst, size_t n,
                     bee_b200_stream_t stream);

/* buf[i] *= factor for dt in {F32, F64} (mean = sum then scale).  Replaces
 * ops_scale_fp (Bee/CUDA/Ops/OpsBridge.hpp:35). */
BEE_B200_API int bee_b200_scale_fp(int dt, void* buf, double factor, size_t n, bee_b200_stream_t stream);

/* ------------------------------------------------------------------ reduce */

/* *dst = reduce(src[0..n)).  Sum/Prod: I32, I64, F32, F64; Min/Max also U8.
 * Integer sums wrap like the reference's T-typed accumulation
 * (Bee/Tensor/Cpu/ReduceCpu.hpp:190-193) and are bit-exact under any order.
 * Float results are deterministic (fixed reduction tree).  n == 0 is an
 * error, as in Bee/CUDA/Api.cpp:237-238.  Scratch for the per-block partials
 * comes from the stream-ordered pool, as in the reference
 * (Bee/CUDA/Ops/Reduce.cu:196-224), but is allocated once per (device, stream)
 * (16 KiB, kept until exit) so later calls are one kernel launch; during
 * stream capture it is allocated and freed around the launch.  Replaces
 * ops_reduce_global (Bee/CUDA/Ops/OpsBridge.hpp:31) behind
 * tensor::cuda::reduce_global (Bee/Tensor/Cuda/Backend.hpp:60). */
BEE_B200_API int bee_b200_reduce_global(int op, int dt, const void* src, void* dst, size_t n,
                           bee_b200_stream_t stream);

/* bee_b200_reduce_global without any allocation — no counterpart in the
 * reference (its global reduce always allocates, Bee/CUDA/Ops/Reduce.cu:208).
 * For callers that must not allocate device memory during the call: error
 * handling or diagnostics after an out-of-memory failure, a host runtime that
 * owns all device memory through its own allocator, or a latency-critical loop
 * that cannot let the stream-ordered pool grow.  Per-block scratch lives in a
 * fixed 64 KiB array compiled into the library, which every GPU that loads the
 * library's module holds until the process exits; a call whose partials would
 * not fit (more than 8160 blocks of 8-byte partials) is rejected with
 * cudaErrorInvalidValue and a message.  Warm-up is required: CUDA loads modules
 * and kernels lazily, and loading can need device memory, so the first call on
 * each device (and the first after a device reset) loads the module, looks up
 * the array's address and loads every kernel this entry point launches, all ops
 * and dtypes.  Make one call per device at start-up, while memory is available
 * and before any stream capture; later calls load and allocate nothing (the
 * address is looked up again on every call, a host-side read, so a reset never
 * leaves it stale).  All calls share the array: calls whose kernels overlap on
 * the GPU (different streams at once) race, so keep them on one stream.
 * Same arguments, dtypes, ops and results as bee_b200_reduce_global. */
BEE_B200_API int bee_b200_reduce_global_noalloc(int op, int dt, const void* src, void* dst, size_t n,
                                                bee_b200_stream_t stream);

/* New: the global reduce across the GPUs of one box in one launch (the only
 * exchange step of the row-sharded sweep).  Each rank reduces its shard; the
 * kernel's last block stores (tag, partial) as one 64-bit word into slot `rank`
 * of every rank's receive array (peer stores over NVLink), waits until its own
 * array holds `tag` in all `world` slots, and folds the partials in rank order,
 * so every rank's dst gets the same bits.  recv_slots[r]: rank r's receive
 * array (2 * world 8-byte words, two banks used by tag parity; CUDA IPC memory
 * opened in this process, zeroed once); tag: nonzero, consecutive calls
 * consecutive values (e.g. a call counter), the same on every rank.  The wait
 * is bounded by wait_ns: a peer that does not deliver in time leaves dst = the
 * local partial and a nonzero code for bee_b200_device_status.  I32 and F32,
 * every reduce op; world <= 8; all ranks call with the same op, dtype and tag. */
BEE_B200_API int bee_b200_reduce_global_allranks(int op, int dt, const void* src, size_t n, void* dst,
                                                 void* const* recv_slots, int world, int rank, unsigned int tag,
                                                 unsigned long long wait_ns, bee_b200_stream_t stream);

/* [outer, axis, inner] -> [outer, inner] (same dtype set as reduce_global;
 * F32 sums accumulate in fp32).  Replaces ops_reduce_axis
 * (Bee/CUDA/Ops/OpsBridge.hpp:32) behind tensor::cuda::reduce_axis
 * (Bee/Tensor/Cuda/Backend.hpp:63); inner == 1 is the row reduce. */
BEE_B200_API int bee_b200_reduce_axis(int op, int dt, const void* src, void* dst, size_t outer, size_t axis,
                         size_t inner, bee_b200_stream_t stream);

/* New: integer mean on the device, which the reference's CUDA path rejects
 * (Bee/Tensor/Ops/Reduce.cpp:155-160) and its CPU path computes by double
 * accumulation (Bee/Tensor/Cpu/ReduceCpu.hpp:431-466, 551-610).  Mean over the
 * `axis` dim of a contiguous [outer, axis, inner] I32 or I64 tensor into F64
 * dst [outer, inner] (outer = inner = 1: the global mean).  The sum is exact
 * (int64), then double(sum) / axis: the reference's result whenever its double
 * accumulation is exact (partial sums below 2^53 in magnitude). */
BEE_B200_API int bee_b200_reduce_mean_int(int dt, const void* src, double* dst, size_t outer, size_t axis, size_t inner,
                                          bee_b200_stream_t stream);

/* ----------------------------------------------------- row-wise operators
 * New operators (the reference has none; its CPU oracle composes them from
 * public ops: max/sub/exp/sum/div for softmax, mul/mean/add/sqrt/div/mul for
 * RMSNorm, slice views with mul/sub/add for RoPE). */

/* Numerically stable softmax over each row of a [rows, cols] matrix:
 * y = exp(x - max(x)) / sum(exp(x - max(x))).  dt in {F32, BF16}; math in
 * fp32.  dst may alias src. */
BEE_B200_API int bee_b200_softmax_rows(int dt, const void* src, void* dst, size_t rows, size_t cols,
                          bee_b200_stream_t stream);

/* Softmax with a different output dtype (F32 or BF16 each side), e.g. fp32
 * attention scores -> bf16 probabilities in one pass; math in fp32. */
BEE_B200_API int bee_b200_softmax_rows_to(int src_dt, const void* src, int dst_dt, void* dst, size_t rows,
                                          size_t cols, bee_b200_stream_t stream);

/* y = x / sqrt(mean(x^2) + eps) * w over each row of [rows, cols]; w has
 * cols elements.  dt in {F32, BF16}; math in fp32. */
BEE_B200_API int bee_b200_rms_norm_rows(int dt, const void* x, const void* w, void* y, size_t rows, size_t cols,
                           float eps, bee_b200_stream_t stream);

/* Rotate-half RoPE on x viewed as [rows, heads, head_dim], rows = batch*seq,
 * position of row r = r % seq + pos_offset, inv_freq_i = theta^(-2i/head_dim):
 *   y[i]      = x[i] cos(p f_i) - x[i+h/2] sin(p f_i)
 *   y[i+h/2]  = x[i+h/2] cos(p f_i) + x[i] sin(p f_i),  i < head_dim/2.
 * dt in {F32, BF16}; head_dim even and at most 256; rows a multiple of seq. */
BEE_B200_API int bee_b200_rope(int dt, const void* x, void* y, size_t rows, size_t seq, size_t heads,
                  size_t head_dim, double theta, size_t pos_offset, bee_b200_stream_t stream);

/* RMSNorm followed by RoPE in one pass (row = one token of heads*head_dim). */
BEE_B200_API int bee_b200_rms_norm_rope(int dt, const void* x, const void* w, void* y, size_t rows, size_t seq,
                           size_t heads, size_t head_dim, float eps, double theta, size_t pos_offset,
                           bee_b200_stream_t stream);

/* ------------------------------------------------------------------ matmul */

/* C[M,N] = A[M,K] . B[K,N], row-major contiguous, same dtype.
 * BF16 / F16: tcgen05 tensor cores with fp32 accumulation and a bf16 / f16
 * (RNE) result (F16 outputs beyond its range are +-inf; small outputs with a
 * long K are cut along K as in bee_b200_bmm);
 * F32 from 2^28 multiply-adds up (K and N multiples of 8, 16-byte aligned
 * buffers): every value split into three bf16 pieces, six piece products on
 * the same tensor cores with fp32 accumulation (fp32-level error; rows and
 * columns holding inf, NaN or |x| >= 3e38 recomputed in plain fp32), with
 * 12*(M*K + K*N) + 4*(1 + M + N) bytes of scratch from the stream-ordered
 * pool, plus 4*S*M*N for S > 1 batches of partial products (S <= 6; S = 1
 * when the output tiles fill the GPU);
 * smaller F32, and F64 / I32 / I64: tiled SIMT kernel
 * accumulating in the element type (I32/I64 wrap).  Replaces ops_matmul
 * (Bee/CUDA/Ops/OpsBridge.hpp:38) behind tensor::cuda::matmul
 * (Bee/Tensor/Cuda/Backend.hpp:70). */
BEE_B200_API int bee_b200_matmul(int dt, const void* A, const void* B, void* C, size_t M, size_t K, size_t N,
                                 bee_b200_stream_t stream);

/* Batched C[b] = alpha * A[b] . op(B[b]) over `batch` contiguous matrices:
 * A [batch, M, K]; B [batch, K, N], or [batch, N, K] when b_trans != 0 (so
 * Q.K^T reads K as stored); C [batch, M, N].  dt_in BF16 with dt_out BF16 or
 * F32, and dt_in F16 with dt_out F16 or F32, run on the tensor cores (TMA needs K % 8 == 0, N % 8 == 0 unless
 * b_trans, 16-byte aligned A and B; other shapes use the SIMT kernel); other
 * dtypes need dt_out == dt_in.  A single 16-bit product (batch 1, and for
 * bmm_strided ldc == N) whose 128x128 output tiles number at most half the
 * SMs, with K a multiple of 128 and at least 2048, is cut along K into S <= 8
 * chunks computed side by side: 4*S*M*N bytes of fp32 partials from the
 * stream-ordered pool, summed in chunk order (results do not depend on
 * timing).  New: the reference matmul is 2-D only
 * (Bee/Tensor/Ops/Matmul.cpp:63-64). */
BEE_B200_API int bee_b200_bmm(int dt_in, int dt_out, const void* A, const void* B, void* C, size_t batch, size_t M,
                              size_t K, size_t N, int b_trans, float alpha, bee_b200_stream_t stream);

/* bee_b200_bmm over strided views (the bmm_strided of the boundary): element
 * strides, A[b][m][k] at A + b*stride_a + m*lda + k; B[b][k][n] at
 * B + b*stride_b + k*ldb + n (b_trans: B[b][n][k] at B + b*stride_b + n*ldb + k);
 * C[b][m][n] at C + b*stride_c + m*ldc + n.  Leading dimensions at least a row;
 * batch strides >= 0 (0 repeats an operand for every batch), output batches
 * must not overlap.  bf16 and f16 inputs take the tensor cores when lda, ldb and the
 * input batch strides are positive multiples of 8 elements and A, B are 16-byte
 * aligned, else the SIMT kernel (same results up to accumulation order).
 * New: the reference's matmul is 2-D and contiguous only. */
BEE_B200_API int bee_b200_bmm_strided(int dt_in, int dt_out, const void* A, int64_t lda, int64_t stride_a, const void* B,
                                      int64_t ldb, int64_t stride_b, void* C, int64_t ldc, int64_t stride_c,
                                      size_t batch, size_t M, size_t K, size_t N, int b_trans, float alpha,
                                      bee_b200_stream_t stream);

/* Fused attention forward, per head: O = softmax(Q.K^T * scale) . V with
 * fp32 scores, softmax and accumulation; Q, K, V, O are [heads, seq, head_dim]
 * bf16, contiguous, 16-byte aligned.  One pass: scores and probabilities stay
 * in tensor memory.  head_dim must be 128, seq a multiple of 128 and scale
 * positive (other shapes: compose bee_b200_bmm, bee_b200_softmax_rows_to and
 * bee_b200_bmm).  With more units (a head's pair of query tiles) than SMs and a
 * last wave that would leave most SMs idle, one persistent CTA per SM runs an
 * equal share of the work instead; the call then takes about 260 KiB per SM of
 * scratch from the stream-ordered pool (released on the stream after the
 * launch) and keeps a 4 KiB block of tickets per stream for the life of the
 * process (during stream capture it keeps one CTA per unit).  The result does
 * not depend on timing.  New: the reference has no attention. */
BEE_B200_API int bee_b200_attention(int dt, const void* q, const void* k, const void* v, void* o, size_t heads,
                                    size_t seq, size_t head_dim, float scale, bee_b200_stream_t stream);

/* ------------------------------------------------- layout
 * Replaces ops_transpose_2d (Bee/CUDA/Ops/OpsBridge.hpp:37-38): dst[i, j] =
 * src[j, i] for a contiguous [rows, cols] src (dst is [cols, rows]).  Every
 * dtype code (moved by element size); size 0 succeeds without work. */
BEE_B200_API int bee_b200_transpose_2d(int dt, const void* src, void* dst, size_t rows, size_t cols,
                                       bee_b200_stream_t stream);

/* New: the device path of Tensor::contiguous() for any view, which the
 * reference serves with a device -> host -> device round trip except for the
 * 2-D transpose (Bee/Tensor/Core/Tensor.cpp:468-508).  `src` points at the
 * view's first element (storage + offset); shape and strides (in elements,
 * ndim <= 8) describe the view; dst receives the elements in row-major order. */
BEE_B200_API int bee_b200_strided_copy(int dt, const void* src, int ndim, const int64_t* shape, const int64_t* strides,
                                       void* dst, bee_b200_stream_t stream);

/* ------------------------------------------------- multi-GPU (split-K GEMM)
 * New: the reference has no multi-GPU code.  One process per GPU.  C = A . B
 * with K sharded over `world` GPUs: rank r holds A[:, K_r] (a column block of
 * the row-major A, row stride `lda`) and B[K_r, :].  The product tiles are
 * 256x256; tile t is owned by rank t % world.
 *
 * 1. bee_b200_gemm_splitk_scatter: every rank computes its fp32 partial on the
 *    tensor cores and the GEMM epilogue stores each partial tile straight into
 *    the owner's receive buffer over NVLink (plain peer stores, slot = source
 *    rank).  recv_peers[r] is rank r's receive buffer as mapped in this process
 *    (bee_b200_ipc_open), each bee_b200_splitk_recv_bytes(M, N, world) bytes.
 * 2. A cross-GPU barrier on the stream (e.g. an all-reduce of one element).
 * 3. bee_b200_gemm_splitk_reduce: each rank sums the world partials of its
 *    own tiles in fixed slot order, rounds to bf16 and writes the tile into
 *    every rank's C (c_peers[r]: rank r's C mapped in this process, [M, N]).
 * 4. Another barrier before C is read on another GPU.
 * Requirements: world <= 8; K, N, lda multiples of 8; 16-byte aligned buffers. */
BEE_B200_API size_t bee_b200_splitk_recv_bytes(size_t M, size_t N, int world);
BEE_B200_API int bee_b200_gemm_splitk_scatter(const void* A, size_t lda, const void* B, size_t M, size_t K, size_t N,
                                              void* const* recv_peers, int world, int rank, bee_b200_stream_t stream);
BEE_B200_API int bee_b200_gemm_splitk_reduce(const void* recv_local, void* const* c_peers, size_t M, size_t N, int world,
                                             int rank, bee_b200_stream_t stream);

/* Device buffers shareable between the processes of one box (CUDA IPC):
 * allocate (cudaMalloc, so the buffer can be exported), export a 64-byte
 * handle, open a peer's handle into this process, close / free. */
BEE_B200_API int bee_b200_ipc_alloc(void** out_ptr, size_t nbytes);
BEE_B200_API int bee_b200_ipc_free(void* ptr);
BEE_B200_API int bee_b200_ipc_handle(const void* ptr, void* handle_out);
BEE_B200_API int bee_b200_ipc_open(const void* handle, void** out_ptr);
BEE_B200_API int bee_b200_ipc_close(void* ptr);

/* Reads and clears the device status word of the tensor-core kernels on the
 * current device: 0, or the code of the first bounded pipeline wait that gave
 * up (the kernel then abandons its remaining tiles instead of hanging).
 * Synchronous. */
BEE_B200_API int bee_b200_device_status(int* out_code);

#ifdef __cplusplus
}
#endif

#endif /* BEE_B200_H */
