// C++ host bridge over the bee_b200 C ABI: the functions of the reference's
// bee::tensor::cuda boundary (Bee/Tensor/Cuda/Backend.hpp:20-84) with the same
// names, argument meaning and error behaviour, plus the operators the
// reference lacks (softmax, RMSNorm, RoPE, batched matmul).
//
// Semantics mirrored from the reference (Bee/CUDA/Api.cpp):
//   * every call is synchronous: work is issued on the per-thread default
//     stream and the stream is synchronised before returning (:45-48, :121);
//   * size-0 elementwise / cast / scale / matmul calls succeed without work,
//     size-0 reduces fail (:213-214, :237-238, :245-246);
//   * a CUDA failure becomes Error{Recoverable, errc = cudaError_t} with the
//     message "<op> 失败: <error name> (<error string>)" (:59-64).
// Result<T> is std::expected<T, Error>, the reference's own alias
// (Bee/Base/Diagnostics/Error.hpp:79); Error carries the fields the Tensor
// layer reads (message, errc, severity).
#pragma once

#include <cstddef>
#include <cstdint>
#include <expected>
#include <string>

namespace bee_b200::tensor_cuda {

enum class Severity : std::uint8_t { Recoverable, Transient, Fatal, Bug };

struct Error {
    std::string message;
    int errc = 0;
    Severity severity = Severity::Recoverable;
    std::string detail;  // bee_b200_last_error() at the time of failure
};

template <typename T> using Result = std::expected<T, Error>;

// ---- execution mode
// Synchronous (the default) is the reference's contract: every call has
// finished when it returns.  Asynchronous mode (a process-wide switch, like the
// reference's backend choice, Bee/CUDA/Api.cpp:327-344) removes the per-call
// synchronisation that the reference pays on every allocation, copy and kernel
// (Bee/CUDA/Api.cpp:131-133, 188-190): calls are only enqueued on the calling
// thread's per-thread stream, allocations come from the stream-ordered pool, and
// synchronize() is the fence (kernel faults surface there).  Copies stay ordered
// with the kernels of the same thread; memcpy_d2h waits in both modes, since
// the host reads the data next.
auto set_synchronous(bool on) -> void;
[[nodiscard]] auto is_synchronous() -> bool;

// ---- memory (Backend.hpp:20-46, 84)
[[nodiscard]] auto allocate(std::size_t nbytes, std::size_t alignment) -> Result<void*>;
auto deallocate(void* p, std::size_t nbytes, std::size_t alignment) -> void;
[[nodiscard]] auto memcpy_h2d(void* dst, const void* src, std::size_t nbytes) -> Result<void>;
[[nodiscard]] auto memcpy_d2h(void* dst, const void* src, std::size_t nbytes) -> Result<void>;
[[nodiscard]] auto memcpy_d2d(void* dst, const void* src, std::size_t nbytes) -> Result<void>;
[[nodiscard]] auto memset(void* ptr, int value, std::size_t nbytes) -> Result<void>;
[[nodiscard]] auto synchronize() -> Result<void>;

// ---- operators on the path (Backend.hpp:51-70)
[[nodiscard]] auto ew_binary(int op, int dt, const void* a, const void* b, void* out, std::size_t n) -> Result<void>;
[[nodiscard]] auto ew_unary(int op, int dt, const void* src, void* dst, std::size_t n) -> Result<void>;
[[nodiscard]] auto ew_cast(int src_dt, const void* src, int dst_dt, void* dst, std::size_t n) -> Result<void>;
[[nodiscard]] auto reduce_global(int op, int dt, const void* src, void* dst, std::size_t n) -> Result<void>;
[[nodiscard]] auto reduce_axis(int op, int dt, const void* src, void* dst, std::size_t outer, std::size_t axis,
                               std::size_t inner) -> Result<void>;
[[nodiscard]] auto scale_fp(int dt, void* buf, double factor, std::size_t n) -> Result<void>;
[[nodiscard]] auto matmul(int dt, const void* A, const void* B, void* C, std::size_t M, std::size_t K, std::size_t N)
    -> Result<void>;

// 2-D transpose dst[i, j] = src[j, i] (Backend.hpp:72-73)
[[nodiscard]] auto transpose_2d(int dt, const void* src, void* dst, std::size_t rows, std::size_t cols) -> Result<void>;

// ---- new operators
// Tensor::contiguous() of any view (shape / strides in elements, ndim <= 8; src at the first element)
[[nodiscard]] auto strided_copy(int dt, const void* src, int ndim, const std::int64_t* shape, const std::int64_t* strides,
                                void* dst) -> Result<void>;
// a op b with broadcasting: out contiguous of `shape`, a and b strided views of it (stride 0 broadcasts)
[[nodiscard]] auto ew_binary_strided(int op, int dt, int ndim, const std::int64_t* shape, const void* a,
                                     const std::int64_t* a_strides, const void* b, const std::int64_t* b_strides,
                                     void* out) -> Result<void>;
// mean over `axis` of an I32 / I64 [outer, axis, inner] tensor into F64 [outer, inner]
[[nodiscard]] auto reduce_mean_int(int dt, const void* src, double* dst, std::size_t outer, std::size_t axis,
                                   std::size_t inner) -> Result<void>;
[[nodiscard]] auto bmm_strided(int dt_in, int dt_out, const void* A, std::int64_t lda, std::int64_t stride_a,
                               const void* B, std::int64_t ldb, std::int64_t stride_b, void* C, std::int64_t ldc,
                               std::int64_t stride_c, std::size_t batch, std::size_t M, std::size_t K, std::size_t N,
                               bool b_transposed, float alpha) -> Result<void>;
[[nodiscard]] auto bmm(int dt_in, int dt_out, const void* A, const void* B, void* C, std::size_t batch, std::size_t M,
                       std::size_t K, std::size_t N, bool b_transposed, float alpha) -> Result<void>;
[[nodiscard]] auto softmax_rows(int dt, const void* src, void* dst, std::size_t rows, std::size_t cols) -> Result<void>;
[[nodiscard]] auto rms_norm_rows(int dt, const void* x, const void* w, void* y, std::size_t rows, std::size_t cols,
                                 float eps) -> Result<void>;
[[nodiscard]] auto rope(int dt, const void* x, void* y, std::size_t rows, std::size_t seq, std::size_t heads,
                        std::size_t head_dim, double theta, std::size_t pos_offset) -> Result<void>;
[[nodiscard]] auto rms_norm_rope(int dt, const void* x, const void* w, void* y, std::size_t rows, std::size_t seq,
                                 std::size_t heads, std::size_t head_dim, float eps, double theta,
                                 std::size_t pos_offset) -> Result<void>;

// fused O = softmax(scale * Q K^T) V per head: q, k, v, o [heads, seq, head_dim] bf16
[[nodiscard]] auto attention(int dt, const void* q, const void* k, const void* v, void* o, std::size_t heads,
                             std::size_t seq, std::size_t head_dim, float scale) -> Result<void>;

}  // namespace bee_b200::tensor_cuda
