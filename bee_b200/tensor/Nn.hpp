#pragma once

// Tensor ops the reference lacks, in its free-function Result<Tensor> style
// (Bee/Tensor/Ops/Matmul.hpp, Reduce.hpp): softmax, RMSNorm, RoPE (and the
// two fused), batched matmul and fused attention.  A maintainer adds this file
// as Bee/Tensor/Ops/Nn.hpp.
//
// Device rules match the reference's ops: all operands on one device, the
// result on that device, errors Recoverable.  On CUDA each op is one bee_b200
// kernel (through BackendExt.hpp); on the CPU each op is the composition of
// the reference's public CPU ops a user would otherwise write (max, sub, exp,
// sum, div, mul, mean, sqrt, slice, matmul, ...), so CPU results are the
// reference's own arithmetic.  CPU dtypes: F32, F64 (the reference computes
// nothing in BF16/F16 on the CPU, Tensor/Core/DType.hpp:10-15); CUDA dtypes:
// F32 and BF16 for the row-wise ops, BF16 and F16 (plus F32, F64, I32, I64 on
// the SIMT path) for bmm, BF16 for attention.

#include "Base/Diagnostics/Error.hpp"
#include "Tensor/Core/Tensor.hpp"

#include <cstdint>

namespace bee
{

// exp(x - max) / sum(exp(x - max)) along `dim` (negative counts from the end).
[[nodiscard]] auto softmax(const Tensor& x, int dim) -> Result<Tensor>;

// x / sqrt(mean(x^2 over the last dim) + eps) * weight; weight is 1-D with the
// last dim's size, same dtype and device as x.
[[nodiscard]] auto rms_norm(const Tensor& x, const Tensor& weight, double eps = 1e-6) -> Result<Tensor>;

// Rotate-half rotary embedding of x [batch, seq, heads, head_dim] (head_dim
// even): for pair (i, i + head_dim/2) at position p = pos_offset + s,
// angle = p * theta^(-2i / head_dim), out_i = x_i cos - x_{i+h} sin,
// out_{i+h} = x_{i+h} cos + x_i sin.
[[nodiscard]] auto rope(const Tensor& x, double theta = 10000.0, int64_t pos_offset = 0) -> Result<Tensor>;

// rope(rms_norm(x viewed [batch, seq, heads * head_dim], weight, eps)) of
// x [batch, seq, heads, head_dim]; one pass over HBM on CUDA.
[[nodiscard]] auto rms_norm_rope(const Tensor& x, const Tensor& weight, double eps = 1e-6, double theta = 10000.0,
                                 int64_t pos_offset = 0) -> Result<Tensor>;

// Batched matmul: a [B, M, K] . b [B, K, N] -> [B, M, N], same dtype.  The
// reference's matmul stays 2-D only (Tensor/Ops/Matmul.cpp:63-64).
[[nodiscard]] auto bmm(const Tensor& a, const Tensor& b) -> Result<Tensor>;

// O = softmax(scale * Q K^T) V per head, q, k, v [heads, seq, head_dim] ->
// [heads, seq, head_dim].  CUDA: BF16, head_dim 128, seq a multiple of 128
// (scores never leave the chip); CPU: F32/F64 composition per head.
[[nodiscard]] auto attention(const Tensor& q, const Tensor& k, const Tensor& v, double scale) -> Result<Tensor>;

} // namespace bee
