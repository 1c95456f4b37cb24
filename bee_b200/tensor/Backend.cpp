// Bee/Tensor/Cuda/Backend.cpp for a Bee tree built on bee_b200: the bodies of
// the reference's CUDA boundary (Bee/Tensor/Cuda/Backend.hpp:20-84) forward to
// bee_b200's C++ bridge (bee_b200/host/tensor_cuda.hpp) instead of Bee::CUDA.
// The Tensor layer above (Bee/Tensor/Ops/*.cpp, Core/*.cpp) is compiled
// unchanged with BEE_TENSOR_WITH_CUDA defined.
//
// Every function keeps the reference's name, argument meaning and error
// behaviour: the bridge is synchronous (work done when the call returns), its
// failures become bee::Error{Recoverable, errc = cudaError_t} with the
// reference's "<op> 失败: <name> (<string>)" text, and integer dtype/op codes
// pass through unchanged (bee_b200 uses bee::DType's codes).  The added
// entries of BackendExt.hpp serve the new Tensor ops of Nn.hpp.
#include "Tensor/Cuda/Backend.hpp"

#include "BackendExt.hpp"
#include "tensor_cuda.hpp"

#include <type_traits>

namespace bee::tensor::cuda
{

namespace
{

namespace b2 = ::bee_b200::tensor_cuda;

template <typename T>
auto to_bee(b2::Result<T> r) -> Result<T>
{
    if (r) {
        if constexpr (std::is_void_v<T>)
            return {};
        else
            return *r;
    }
    return std::unexpected(make_error(r.error().message, Severity::Recoverable, r.error().errc));
}

auto not_on_path(const char* what) -> Error
{
    return make_error(std::string("CUDA 后端不可用：") + what + " (device-side random generation is not part of bee_b200)",
                      Severity::Recoverable);
}

} // namespace

auto allocate(std::size_t nbytes, std::size_t alignment) -> Result<void*>
{
    return to_bee(b2::allocate(nbytes, alignment));
}

auto deallocate(void* p, std::size_t nbytes, std::size_t alignment) -> void
{
    b2::deallocate(p, nbytes, alignment);
}

auto memcpy_h2d(void* dst, const void* src, std::size_t nbytes) -> Result<void>
{
    return to_bee(b2::memcpy_h2d(dst, src, nbytes));
}

auto memcpy_d2h(void* dst, const void* src, std::size_t nbytes) -> Result<void>
{
    return to_bee(b2::memcpy_d2h(dst, src, nbytes));
}

auto memcpy_d2d(void* dst, const void* src, std::size_t nbytes) -> Result<void>
{
    return to_bee(b2::memcpy_d2d(dst, src, nbytes));
}

auto memset(void* ptr, int value, std::size_t nbytes) -> Result<void>
{
    return to_bee(b2::memset(ptr, value, nbytes));
}

auto ew_binary(int op, int dt, const void* a, const void* b, void* out, std::size_t n) -> Result<void>
{
    return to_bee(b2::ew_binary(op, dt, a, b, out, n));
}

auto ew_unary(int op, int dt, const void* src, void* dst, std::size_t n) -> Result<void>
{
    return to_bee(b2::ew_unary(op, dt, src, dst, n));
}

auto ew_cast(int src_dt, const void* src, int dst_dt, void* dst, std::size_t n) -> Result<void>
{
    return to_bee(b2::ew_cast(src_dt, src, dst_dt, dst, n));
}

auto reduce_global(int op, int dt, const void* src, void* dst, std::size_t n) -> Result<void>
{
    return to_bee(b2::reduce_global(op, dt, src, dst, n));
}

auto reduce_axis(int op, int dt, const void* src, void* dst, std::size_t outer, std::size_t axis, std::size_t inner) -> Result<void>
{
    return to_bee(b2::reduce_axis(op, dt, src, dst, outer, axis, inner));
}

auto scale_fp(int dt, void* buf, double factor, std::size_t n) -> Result<void>
{
    return to_bee(b2::scale_fp(dt, buf, factor, n));
}

auto matmul(int dt, const void* A, const void* B, void* C, std::size_t M, std::size_t K, std::size_t N) -> Result<void>
{
    return to_bee(b2::matmul(dt, A, B, C, M, K, N));
}

auto transpose_2d(int dt, const void* src, void* dst, std::size_t rows, std::size_t cols) -> Result<void>
{
    return to_bee(b2::transpose_2d(dt, src, dst, rows, cols));
}

auto random_uniform(int, void*, std::size_t, std::uint64_t) -> Result<void>
{
    return std::unexpected(not_on_path("random_uniform"));
}

auto random_normal(int, void*, std::size_t, std::uint64_t) -> Result<void>
{
    return std::unexpected(not_on_path("random_normal"));
}

auto random_int(int, void*, std::size_t, std::int64_t, std::int64_t, std::uint64_t) -> Result<void>
{
    return std::unexpected(not_on_path("random_int"));
}

auto synchronize() -> Result<void>
{
    return to_bee(b2::synchronize());
}

// ── entries added for the new Tensor ops (BackendExt.hpp) ───────────────────

auto softmax_rows(int dt, const void* src, void* dst, std::size_t rows, std::size_t cols) -> Result<void>
{
    return to_bee(b2::softmax_rows(dt, src, dst, rows, cols));
}

auto rms_norm_rows(int dt, const void* x, const void* w, void* y, std::size_t rows, std::size_t cols, float eps) -> Result<void>
{
    return to_bee(b2::rms_norm_rows(dt, x, w, y, rows, cols, eps));
}

auto rope(int dt, const void* x, void* y, std::size_t rows, std::size_t seq, std::size_t heads, std::size_t head_dim, double theta,
          std::size_t pos_offset) -> Result<void>
{
    return to_bee(b2::rope(dt, x, y, rows, seq, heads, head_dim, theta, pos_offset));
}

auto rms_norm_rope(int dt, const void* x, const void* w, void* y, std::size_t rows, std::size_t seq, std::size_t heads,
                   std::size_t head_dim, float eps, double theta, std::size_t pos_offset) -> Result<void>
{
    return to_bee(b2::rms_norm_rope(dt, x, w, y, rows, seq, heads, head_dim, eps, theta, pos_offset));
}

auto bmm(int dt_in, int dt_out, const void* A, const void* B, void* C, std::size_t batch, std::size_t M, std::size_t K,
         std::size_t N, bool b_transposed, float alpha) -> Result<void>
{
    return to_bee(b2::bmm(dt_in, dt_out, A, B, C, batch, M, K, N, b_transposed, alpha));
}

auto attention(int dt, const void* q, const void* k, const void* v, void* o, std::size_t heads, std::size_t seq,
               std::size_t head_dim, float scale) -> Result<void>
{
    return to_bee(b2::attention(dt, q, k, v, o, heads, seq, head_dim, scale));
}

auto strided_copy(int dt, const void* src, int ndim, const std::int64_t* shape, const std::int64_t* strides, void* dst)
    -> Result<void>
{
    return to_bee(b2::strided_copy(dt, src, ndim, shape, strides, dst));
}

} // namespace bee::tensor::cuda
