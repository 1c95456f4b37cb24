#pragma once

// Entries added to the reference's CUDA boundary (Bee/Tensor/Cuda/Backend.hpp)
// for the Tensor ops the reference lacks (Nn.hpp).  Same conventions as the
// existing entries: host-only, contiguous device buffers, integer dtype codes
// equal to bee::DType's, synchronous, Result<void> with a Recoverable error
// carrying the cudaError_t in errc.  Bodies: Backend.cpp, forwarding to
// bee_b200's C ABI (include/bee_b200.h).

#include "Base/Diagnostics/Error.hpp"

#include <cstddef>
#include <cstdint>

namespace bee::tensor::cuda
{

// Row softmax over `cols` of a [rows, cols] tensor (F32 or BF16, fp32 math).
[[nodiscard]] auto softmax_rows(int dt, const void* src, void* dst, std::size_t rows, std::size_t cols) -> Result<void>;

// y = x / sqrt(mean(x^2) + eps) * w over the last dim of [rows, cols] (F32 or BF16).
[[nodiscard]] auto rms_norm_rows(int dt, const void* x, const void* w, void* y, std::size_t rows, std::size_t cols, float eps)
    -> Result<void>;

// Rotate-half RoPE of [rows = batch * seq, heads, head_dim]; position of row r is
// pos_offset + r % seq; angle_i = pos * theta^(-2i / head_dim).
[[nodiscard]] auto rope(int dt, const void* x, void* y, std::size_t rows, std::size_t seq, std::size_t heads, std::size_t head_dim,
                        double theta, std::size_t pos_offset) -> Result<void>;

// rms_norm_rows then rope in one pass (cols = heads * head_dim).
[[nodiscard]] auto rms_norm_rope(int dt, const void* x, const void* w, void* y, std::size_t rows, std::size_t seq,
                                 std::size_t heads, std::size_t head_dim, float eps, double theta, std::size_t pos_offset)
    -> Result<void>;

// C[b] = alpha * A[b] . op(B[b]) over contiguous [batch, M, K] x [batch, K, N]
// (B as [batch, N, K] when b_transposed); BF16 / F16 in -> same or F32 out on the
// tensor cores, other dtypes in == out.
[[nodiscard]] auto bmm(int dt_in, int dt_out, const void* A, const void* B, void* C, std::size_t batch, std::size_t M,
                       std::size_t K, std::size_t N, bool b_transposed, float alpha) -> Result<void>;

// O = softmax(scale * Q K^T) V per head, q, k, v, o [heads, seq, head_dim] BF16.
[[nodiscard]] auto attention(int dt, const void* q, const void* k, const void* v, void* o, std::size_t heads, std::size_t seq,
                             std::size_t head_dim, float scale) -> Result<void>;

// dst (contiguous) = the strided view (shape, strides in elements, ndim <= 8) at src.
[[nodiscard]] auto strided_copy(int dt, const void* src, int ndim, const std::int64_t* shape, const std::int64_t* strides,
                                void* dst) -> Result<void>;

} // namespace bee::tensor::cuda
