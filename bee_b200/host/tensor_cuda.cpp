// Implementation of the bee::tensor::cuda mirror over the bee_b200 C ABI.
// Every call runs on the per-thread default stream and (in the default,
// synchronous mode) synchronises it before returning, which is the observable
// contract of the reference's bridge.
#include "tensor_cuda.hpp"

#include <cuda_runtime_api.h>

#include <atomic>
#include <format>

#include "bee_b200.h"

namespace bee_b200::tensor_cuda {

namespace {

bee_b200_stream_t per_thread_stream() { return reinterpret_cast<bee_b200_stream_t>(cudaStreamPerThread); }

std::atomic<bool> g_synchronous{true};

Error make_error(int err, const char* op) {
    Error e;
    e.errc = err;
    e.severity = Severity::Recoverable;
    e.message = std::format("{} 失败: {} ({})", op, cudaGetErrorName(static_cast<cudaError_t>(err)),
                            cudaGetErrorString(static_cast<cudaError_t>(err)));
    e.detail = bee_b200_last_error();
    return e;
}

Error plain_error(const char* msg) {
    Error e;
    e.message = msg;
    return e;
}

// Converts a status into Result and, on success in synchronous mode,
// synchronises the stream so the call is complete when it returns.
Result<void> finish(int err, const char* op) {
    if (err == 0 && g_synchronous.load(std::memory_order_relaxed))
        err = bee_b200_stream_synchronize(per_thread_stream());
    if (err != 0) return std::unexpected(make_error(err, op));
    return {};
}

}  // namespace

auto set_synchronous(bool on) -> void { g_synchronous.store(on, std::memory_order_relaxed); }

auto is_synchronous() -> bool { return g_synchronous.load(std::memory_order_relaxed); }

auto allocate(std::size_t nbytes, std::size_t alignment) -> Result<void*> {
    void* p = nullptr;
    int err = bee_b200_allocate(&p, nbytes, alignment, per_thread_stream());
    if (err == 0 && is_synchronous()) err = bee_b200_stream_synchronize(per_thread_stream());
    if (err != 0) return std::unexpected(make_error(err, "cuda::allocate"));
    return p;
}

auto deallocate(void* p, std::size_t, std::size_t) -> void {
    if (!p) return;
    (void)bee_b200_deallocate(p, per_thread_stream());
    if (is_synchronous()) (void)bee_b200_stream_synchronize(per_thread_stream());
}

auto memcpy_h2d(void* dst, const void* src, std::size_t nbytes) -> Result<void> {
    return finish(bee_b200_memcpy_h2d(dst, src, nbytes, per_thread_stream()), "cuda::memcpy_h2d");
}

auto memcpy_d2h(void* dst, const void* src, std::size_t nbytes) -> Result<void> {
    // waits in both modes: the host reads the data next
    int err = bee_b200_memcpy_d2h(dst, src, nbytes, per_thread_stream());
    if (err == 0) err = bee_b200_stream_synchronize(per_thread_stream());
    if (err != 0) return std::unexpected(make_error(err, "cuda::memcpy_d2h"));
    return {};
}

auto memcpy_d2d(void* dst, const void* src, std::size_t nbytes) -> Result<void> {
    return finish(bee_b200_memcpy_d2d(dst, src, nbytes, per_thread_stream()), "cuda::memcpy_d2d");
}

auto memset(void* ptr, int value, std::size_t nbytes) -> Result<void> {
    return finish(bee_b200_memset(ptr, value, nbytes, per_thread_stream()), "cuda::memset");
}

auto synchronize() -> Result<void> {
    const cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return std::unexpected(make_error(static_cast<int>(e), "cuda::device_synchronize"));
    return {};
}

auto ew_binary(int op, int dt, const void* a, const void* b, void* out, std::size_t n) -> Result<void> {
    if (n == 0) return {};
    return finish(bee_b200_ew_binary(op, dt, a, b, out, n, per_thread_stream()), "cuda::ops::binary");
}

auto ew_unary(int op, int dt, const void* src, void* dst, std::size_t n) -> Result<void> {
    if (n == 0) return {};
    return finish(bee_b200_ew_unary(op, dt, src, dst, n, per_thread_stream()), "cuda::ops::unary");
}

auto ew_cast(int src_dt, const void* src, int dst_dt, void* dst, std::size_t n) -> Result<void> {
    if (n == 0) return {};
    return finish(bee_b200_ew_cast(src_dt, src, dst_dt, dst, n, per_thread_stream()), "cuda::ops::cast");
}

auto reduce_global(int op, int dt, const void* src, void* dst, std::size_t n) -> Result<void> {
    if (n == 0) return std::unexpected(plain_error("cuda::ops::reduce_global: n == 0"));
    return finish(bee_b200_reduce_global(op, dt, src, dst, n, per_thread_stream()), "cuda::ops::reduce_global");
}

auto reduce_axis(int op, int dt, const void* src, void* dst, std::size_t outer, std::size_t axis, std::size_t inner)
    -> Result<void> {
    if (outer == 0 || inner == 0 || axis == 0) return std::unexpected(plain_error("cuda::ops::reduce_axis: 维度含 0"));
    return finish(bee_b200_reduce_axis(op, dt, src, dst, outer, axis, inner, per_thread_stream()),
                  "cuda::ops::reduce_axis");
}

auto scale_fp(int dt, void* buf, double factor, std::size_t n) -> Result<void> {
    if (n == 0) return {};
    return finish(bee_b200_scale_fp(dt, buf, factor, n, per_thread_stream()), "cuda::ops::scale_fp");
}

auto matmul(int dt, const void* A, const void* B, void* C, std::size_t M, std::size_t K, std::size_t N)
    -> Result<void> {
    if (M == 0 || N == 0) return {};
    return finish(bee_b200_matmul(dt, A, B, C, M, K, N, per_thread_stream()), "cuda::ops::matmul");
}

auto transpose_2d(int dt, const void* src, void* dst, std::size_t rows, std::size_t cols) -> Result<void> {
    if (rows == 0 || cols == 0) return {};
    return finish(bee_b200_transpose_2d(dt, src, dst, rows, cols, per_thread_stream()), "cuda::ops::transpose_2d");
}

auto strided_copy(int dt, const void* src, int ndim, const std::int64_t* shape, const std::int64_t* strides, void* dst)
    -> Result<void> {
    return finish(bee_b200_strided_copy(dt, src, ndim, shape, strides, dst, per_thread_stream()),
                  "cuda::ops::strided_copy");
}

auto ew_binary_strided(int op, int dt, int ndim, const std::int64_t* shape, const void* a, const std::int64_t* a_strides,
                       const void* b, const std::int64_t* b_strides, void* out) -> Result<void> {
    return finish(bee_b200_ew_binary_strided(op, dt, ndim, shape, a, a_strides, b, b_strides, out, per_thread_stream()),
                  "cuda::ops::binary_strided");
}

auto reduce_mean_int(int dt, const void* src, double* dst, std::size_t outer, std::size_t axis, std::size_t inner)
    -> Result<void> {
    return finish(bee_b200_reduce_mean_int(dt, src, dst, outer, axis, inner, per_thread_stream()),
                  "cuda::ops::reduce_mean_int");
}

auto bmm_strided(int dt_in, int dt_out, const void* A, std::int64_t lda, std::int64_t stride_a, const void* B,
                 std::int64_t ldb, std::int64_t stride_b, void* C, std::int64_t ldc, std::int64_t stride_c,
                 std::size_t batch, std::size_t M, std::size_t K, std::size_t N, bool b_transposed, float alpha)
    -> Result<void> {
    return finish(bee_b200_bmm_strided(dt_in, dt_out, A, lda, stride_a, B, ldb, stride_b, C, ldc, stride_c, batch, M, K,
                                       N, b_transposed ? 1 : 0, alpha, per_thread_stream()),
                  "cuda::ops::bmm_strided");
}

auto bmm(int dt_in, int dt_out, const void* A, const void* B, void* C, std::size_t batch, std::size_t M, std::size_t K,
         std::size_t N, bool b_transposed, float alpha) -> Result<void> {
    return finish(bee_b200_bmm(dt_in, dt_out, A, B, C, batch, M, K, N, b_transposed ? 1 : 0, alpha, per_thread_stream()),
                  "cuda::ops::bmm");
}

auto softmax_rows(int dt, const void* src, void* dst, std::size_t rows, std::size_t cols) -> Result<void> {
    return finish(bee_b200_softmax_rows(dt, src, dst, rows, cols, per_thread_stream()), "cuda::ops::softmax_rows");
}

auto rms_norm_rows(int dt, const void* x, const void* w, void* y, std::size_t rows, std::size_t cols, float eps)
    -> Result<void> {
    return finish(bee_b200_rms_norm_rows(dt, x, w, y, rows, cols, eps, per_thread_stream()), "cuda::ops::rms_norm_rows");
}

auto rope(int dt, const void* x, void* y, std::size_t rows, std::size_t seq, std::size_t heads, std::size_t head_dim,
          double theta, std::size_t pos_offset) -> Result<void> {
    return finish(bee_b200_rope(dt, x, y, rows, seq, heads, head_dim, theta, pos_offset, per_thread_stream()),
                  "cuda::ops::rope");
}

auto rms_norm_rope(int dt, const void* x, const void* w, void* y, std::size_t rows, std::size_t seq, std::size_t heads,
                   std::size_t head_dim, float eps, double theta, std::size_t pos_offset) -> Result<void> {
    return finish(bee_b200_rms_norm_rope(dt, x, w, y, rows, seq, heads, head_dim, eps, theta, pos_offset,
                                         per_thread_stream()),
                  "cuda::ops::rms_norm_rope");
}

}  // namespace bee_b200::tensor_cuda

namespace bee_b200::tensor_cuda {

auto attention(int dt, const void* q, const void* k, const void* v, void* o, std::size_t heads, std::size_t seq,
               std::size_t head_dim, float scale) -> Result<void> {
    return finish(bee_b200_attention(dt, q, k, v, o, heads, seq, head_dim, scale, per_thread_stream()),
                  "cuda::ops::attention");
}

}  // namespace bee_b200::tensor_cuda
