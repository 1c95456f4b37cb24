// The Tensor ops of Nn.hpp.  CUDA: argument checks, contiguous operands, one
// bee_b200 kernel through the added backend entries (BackendExt.hpp).  CPU:
// the composition of the reference's public ops (Tensor/Ops/*.hpp), so the CPU
// result is the reference's own arithmetic.
#include "Nn.hpp"

#include "BackendExt.hpp"
#include "Tensor/Tensor.hpp"

#include <cmath>
#include <format>
#include <string_view>
#include <utility>
#include <vector>

namespace bee
{

namespace
{

#define NN_TRY(name, expr)                                                                                                       \
    auto name##_res = (expr);                                                                                                    \
    if (!name##_res)                                                                                                             \
        return std::unexpected(std::move(name##_res.error()));                                                                   \
    auto name = std::move(*name##_res)

#define NN_CHECK(expr)                                                                                                           \
    do {                                                                                                                         \
        auto nn_check_res = (expr);                                                                                              \
        if (!nn_check_res)                                                                                                       \
            return std::unexpected(std::move(nn_check_res.error()));                                                             \
    } while (0)

auto fail(std::string_view op, std::string_view why) -> Error
{
    return make_error(std::format("{}: {}", op, why), Severity::Recoverable);
}

auto dtype_name(DType dt) -> std::string_view
{
    switch (dt) {
    case DType::F32: return "F32";
    case DType::F64: return "F64";
    case DType::F16: return "F16";
    case DType::BF16: return "BF16";
    case DType::I32: return "I32";
    case DType::I64: return "I64";
    default: return "unsupported";
    }
}

// A contiguous copy of t (t itself when already contiguous).  CUDA views are
// gathered on the device by one strided-copy kernel, where the reference's
// Tensor::contiguous() goes device -> host -> device for anything but a 2-D
// transpose (Tensor/Core/Tensor.cpp:501-508).
auto contiguous_of(const Tensor& t) -> Result<Tensor>
{
    if (t.is_contiguous())
        return t;
    if (t.device() != Device::CUDA || t.ndim() > 8)
        return t.contiguous();
    NN_TRY(out, Tensor::empty(t.shape(), t.dtype(), Device::CUDA));
    NN_CHECK(tensor::cuda::strided_copy(static_cast<int>(t.dtype()), t.data_ptr(), static_cast<int>(t.ndim()),
                                        t.shape().data(), t.strides().data(), out.data_ptr()));
    return out;
}

auto same_device(std::string_view op, std::initializer_list<const Tensor*> ts) -> Result<void>
{
    const Tensor* first = *ts.begin();
    for (const Tensor* t : ts) {
        if (!t->defined())
            return std::unexpected(fail(op, "undefined tensor"));
        if (t->device() != first->device())
            return std::unexpected(fail(op, "operands on different devices"));
    }
    return {};
}

auto cpu_float(std::string_view op, DType dt) -> Result<void>
{
    if (dt != DType::F32 && dt != DType::F64)
        return std::unexpected(fail(op, std::format("CPU path computes in F32 or F64, got {}", dtype_name(dt))));
    return {};
}

auto cuda_rowwise(std::string_view op, DType dt) -> Result<void>
{
    if (dt != DType::F32 && dt != DType::BF16)
        return std::unexpected(fail(op, std::format("CUDA path takes F32 or BF16, got {}", dtype_name(dt))));
    return {};
}

auto scalar_like(double v, DType dt) -> Result<Tensor>
{
    return Tensor::full({1}, dt, v);
}

// cos / sin of the rotary angles as [1, seq, 1, half] tensors of dtype dt
// (angles in double, rounded once), to broadcast over batch and heads.
auto rope_tables(int64_t seq, int64_t head_dim, double theta, int64_t pos_offset, DType dt) -> Result<std::pair<Tensor, Tensor>>
{
    const int64_t half = head_dim / 2;
    NN_TRY(c, Tensor::empty({1, seq, 1, half}, dt));
    NN_TRY(s, Tensor::empty({1, seq, 1, half}, dt));
    for (int64_t p = 0; p < seq; ++p) {
        const double pos = static_cast<double>(p + pos_offset);
        for (int64_t i = 0; i < half; ++i) {
            const double ang = pos * std::pow(theta, -2.0 * static_cast<double>(i) / static_cast<double>(head_dim));
            const int64_t at = p * half + i;
            if (dt == DType::F32) {
                static_cast<float*>(c.data_ptr())[at] = static_cast<float>(std::cos(ang));
                static_cast<float*>(s.data_ptr())[at] = static_cast<float>(std::sin(ang));
            } else {
                static_cast<double*>(c.data_ptr())[at] = std::cos(ang);
                static_cast<double*>(s.data_ptr())[at] = std::sin(ang);
            }
        }
    }
    return std::pair<Tensor, Tensor>{std::move(c), std::move(s)};
}

auto rope_cpu(const Tensor& x, double theta, int64_t pos_offset) -> Result<Tensor>
{
    const int64_t seq = x.shape()[1], hd = x.shape()[3], half = hd / 2;
    NN_TRY(tables, rope_tables(seq, hd, theta, pos_offset, x.dtype()));
    const auto& [c, s] = tables;
    NN_TRY(x1, x.slice(3, 0, half));
    NN_TRY(x2, x.slice(3, half, hd));
    NN_TRY(a, mul(x1, c));
    NN_TRY(b, mul(x2, s));
    NN_TRY(o1, sub(a, b));
    NN_TRY(d, mul(x2, c));
    NN_TRY(e, mul(x1, s));
    NN_TRY(o2, add(d, e));
    NN_TRY(out, Tensor::zeros(x.shape(), x.dtype()));
    NN_TRY(y1, out.slice(3, 0, half));
    NN_TRY(y2, out.slice(3, half, hd));
    NN_CHECK(add_inplace(y1, o1));
    NN_CHECK(add_inplace(y2, o2));
    return out;
}

auto rms_norm_cpu(const Tensor& x, const Tensor& w, double eps) -> Result<Tensor>
{
    NN_TRY(sq, mul(x, x));
    NN_TRY(ms, mean(sq, -1, true));
    NN_TRY(e, scalar_like(eps, x.dtype()));
    NN_TRY(me, add(ms, e));
    NN_TRY(rt, sqrt(me));
    NN_TRY(xn, div(x, rt));
    return mul(xn, w);
}

auto check_rope_shape(std::string_view op, const Tensor& x) -> Result<void>
{
    if (x.ndim() != 4)
        return std::unexpected(fail(op, std::format("x must be [batch, seq, heads, head_dim], got ndim={}", x.ndim())));
    if (x.shape()[3] % 2 != 0)
        return std::unexpected(fail(op, "head_dim must be even"));
    return {};
}

auto check_norm_weight(std::string_view op, const Tensor& x, const Tensor& w, int64_t cols) -> Result<void>
{
    if (w.ndim() != 1 || w.shape()[0] != cols)
        return std::unexpected(fail(op, std::format("weight must be 1-D of size {}", cols)));
    if (w.dtype() != x.dtype())
        return std::unexpected(fail(op, "weight dtype differs from x"));
    return {};
}

} // namespace

auto softmax(const Tensor& x, int dim) -> Result<Tensor>
{
    constexpr std::string_view op = "softmax";
    NN_CHECK(same_device(op, {&x}));
    const int64_t nd = x.ndim();
    if (nd == 0)
        return std::unexpected(fail(op, "0-d input"));
    const int64_t d = dim < 0 ? dim + nd : dim;
    if (d < 0 || d >= nd)
        return std::unexpected(fail(op, std::format("dim {} out of range for ndim {}", dim, nd)));
    if (x.numel() == 0)
        return Tensor::empty(x.shape(), x.dtype(), x.device());

    if (x.device() == Device::CUDA) {
        NN_CHECK(cuda_rowwise(op, x.dtype()));
        if (d != nd - 1) {
            // move `dim` innermost, reduce rows, move it back
            std::vector<int> perm;
            for (int64_t i = 0; i < nd; ++i)
                if (i != d)
                    perm.push_back(static_cast<int>(i));
            perm.push_back(static_cast<int>(d));
            std::vector<int> inv(static_cast<std::size_t>(nd));
            for (int64_t i = 0; i < nd; ++i)
                inv[static_cast<std::size_t>(perm[static_cast<std::size_t>(i)])] = static_cast<int>(i);
            NN_TRY(moved, x.permute(std::span<const int>(perm)));
            NN_TRY(inner, softmax(moved, -1));
            NN_TRY(back, inner.permute(std::span<const int>(inv)));
            return contiguous_of(back);
        }
        NN_TRY(cx, contiguous_of(x));
        NN_TRY(out, Tensor::empty(x.shape(), x.dtype(), Device::CUDA));
        const auto cols = static_cast<std::size_t>(x.shape()[static_cast<std::size_t>(d)]);
        NN_CHECK(tensor::cuda::softmax_rows(static_cast<int>(x.dtype()), cx.data_ptr(), out.data_ptr(),
                                            static_cast<std::size_t>(x.numel()) / cols, cols));
        return out;
    }

    NN_CHECK(cpu_float(op, x.dtype()));
    NN_TRY(m, max(x, static_cast<int>(d), true));
    NN_TRY(t, sub(x, m));
    NN_TRY(e, exp(t));
    NN_TRY(s, sum(e, static_cast<int>(d), true));
    return div(e, s);
}

auto rms_norm(const Tensor& x, const Tensor& weight, double eps) -> Result<Tensor>
{
    constexpr std::string_view op = "rms_norm";
    NN_CHECK(same_device(op, {&x, &weight}));
    if (x.ndim() == 0)
        return std::unexpected(fail(op, "0-d input"));
    const int64_t cols = x.shape().back();
    NN_CHECK(check_norm_weight(op, x, weight, cols));
    if (x.numel() == 0)
        return Tensor::empty(x.shape(), x.dtype(), x.device());

    if (x.device() == Device::CUDA) {
        NN_CHECK(cuda_rowwise(op, x.dtype()));
        NN_TRY(cx, contiguous_of(x));
        NN_TRY(cw, contiguous_of(weight));
        NN_TRY(out, Tensor::empty(x.shape(), x.dtype(), Device::CUDA));
        NN_CHECK(tensor::cuda::rms_norm_rows(static_cast<int>(x.dtype()), cx.data_ptr(), cw.data_ptr(), out.data_ptr(),
                                             static_cast<std::size_t>(x.numel() / cols), static_cast<std::size_t>(cols),
                                             static_cast<float>(eps)));
        return out;
    }
    NN_CHECK(cpu_float(op, x.dtype()));
    return rms_norm_cpu(x, weight, eps);
}

auto rope(const Tensor& x, double theta, int64_t pos_offset) -> Result<Tensor>
{
    constexpr std::string_view op = "rope";
    NN_CHECK(same_device(op, {&x}));
    NN_CHECK(check_rope_shape(op, x));
    if (x.numel() == 0)
        return Tensor::empty(x.shape(), x.dtype(), x.device());
    if (pos_offset < 0)
        return std::unexpected(fail(op, "negative pos_offset"));

    if (x.device() == Device::CUDA) {
        NN_CHECK(cuda_rowwise(op, x.dtype()));
        const auto& s = x.shape();
        NN_TRY(cx, contiguous_of(x));
        NN_TRY(out, Tensor::empty(s, x.dtype(), Device::CUDA));
        NN_CHECK(tensor::cuda::rope(static_cast<int>(x.dtype()), cx.data_ptr(), out.data_ptr(),
                                    static_cast<std::size_t>(s[0] * s[1]), static_cast<std::size_t>(s[1]),
                                    static_cast<std::size_t>(s[2]), static_cast<std::size_t>(s[3]), theta,
                                    static_cast<std::size_t>(pos_offset)));
        return out;
    }
    NN_CHECK(cpu_float(op, x.dtype()));
    return rope_cpu(x, theta, pos_offset);
}

auto rms_norm_rope(const Tensor& x, const Tensor& weight, double eps, double theta, int64_t pos_offset) -> Result<Tensor>
{
    constexpr std::string_view op = "rms_norm_rope";
    NN_CHECK(same_device(op, {&x, &weight}));
    NN_CHECK(check_rope_shape(op, x));
    const auto& s = x.shape();
    NN_CHECK(check_norm_weight(op, x, weight, s[2] * s[3]));
    if (x.numel() == 0)
        return Tensor::empty(s, x.dtype(), x.device());
    if (pos_offset < 0)
        return std::unexpected(fail(op, "negative pos_offset"));

    if (x.device() == Device::CUDA) {
        NN_CHECK(cuda_rowwise(op, x.dtype()));
        NN_TRY(cx, contiguous_of(x));
        NN_TRY(cw, contiguous_of(weight));
        NN_TRY(out, Tensor::empty(s, x.dtype(), Device::CUDA));
        NN_CHECK(tensor::cuda::rms_norm_rope(static_cast<int>(x.dtype()), cx.data_ptr(), cw.data_ptr(), out.data_ptr(),
                                             static_cast<std::size_t>(s[0] * s[1]), static_cast<std::size_t>(s[1]),
                                             static_cast<std::size_t>(s[2]), static_cast<std::size_t>(s[3]),
                                             static_cast<float>(eps), theta, static_cast<std::size_t>(pos_offset)));
        return out;
    }
    NN_CHECK(cpu_float(op, x.dtype()));
    NN_TRY(flat, contiguous_of(x));
    NN_TRY(rows, flat.reshape({s[0], s[1], s[2] * s[3]}));
    NN_TRY(normed, rms_norm_cpu(rows, weight, eps));
    NN_TRY(heads, normed.reshape(s));
    return rope_cpu(heads, theta, pos_offset);
}

auto bmm(const Tensor& a, const Tensor& b) -> Result<Tensor>
{
    constexpr std::string_view op = "bmm";
    NN_CHECK(same_device(op, {&a, &b}));
    if (a.ndim() != 3 || b.ndim() != 3)
        return std::unexpected(fail(op, "operands must be [B, M, K] and [B, K, N]"));
    if (a.dtype() != b.dtype())
        return std::unexpected(fail(op, "dtype mismatch"));
    const int64_t B = a.shape()[0], M = a.shape()[1], K = a.shape()[2], N = b.shape()[2];
    if (b.shape()[0] != B || b.shape()[1] != K)
        return std::unexpected(fail(op, std::format("shape mismatch: [{}, {}, {}] . [{}, {}, {}]", B, M, K, b.shape()[0],
                                                    b.shape()[1], N)));

    if (a.device() == Device::CUDA) {
        const DType dt = a.dtype();
        if (dt != DType::BF16 && dt != DType::F16 && dt != DType::F32 && dt != DType::F64 && dt != DType::I32 &&
            dt != DType::I64)
            return std::unexpected(fail(op, std::format("CUDA path does not take {}", dtype_name(dt))));
        NN_TRY(out, Tensor::empty({B, M, N}, dt, Device::CUDA));
        if (out.numel() == 0)
            return out;
        NN_TRY(ca, contiguous_of(a));
        NN_TRY(cb, contiguous_of(b));
        NN_CHECK(tensor::cuda::bmm(static_cast<int>(dt), static_cast<int>(dt), ca.data_ptr(), cb.data_ptr(), out.data_ptr(),
                                   static_cast<std::size_t>(B), static_cast<std::size_t>(M), static_cast<std::size_t>(K),
                                   static_cast<std::size_t>(N), false, 1.0f));
        return out;
    }

    NN_TRY(out, Tensor::zeros({B, M, N}, a.dtype()));
    for (int64_t i = 0; i < B; ++i) {
        NN_TRY(ai, a.slice(0, i, i + 1));
        NN_TRY(bi, b.slice(0, i, i + 1));
        NN_TRY(a2, ai.squeeze(0));
        NN_TRY(b2, bi.squeeze(0));
        NN_TRY(prod, matmul(a2, b2));
        NN_TRY(oi, out.slice(0, i, i + 1));
        NN_TRY(o2, oi.squeeze(0));
        NN_CHECK(add_inplace(o2, prod));
    }
    return out;
}

auto attention(const Tensor& q, const Tensor& k, const Tensor& v, double scale) -> Result<Tensor>
{
    constexpr std::string_view op = "attention";
    NN_CHECK(same_device(op, {&q, &k, &v}));
    if (q.ndim() != 3 || q.shape() != k.shape() || q.shape() != v.shape())
        return std::unexpected(fail(op, "q, k, v must all be [heads, seq, head_dim]"));
    if (q.dtype() != k.dtype() || q.dtype() != v.dtype())
        return std::unexpected(fail(op, "dtype mismatch"));
    const int64_t H = q.shape()[0], S = q.shape()[1], D = q.shape()[2];
    if (q.numel() == 0)
        return Tensor::empty(q.shape(), q.dtype(), q.device());

    if (q.device() == Device::CUDA) {
        if (q.dtype() != DType::BF16)
            return std::unexpected(fail(op, std::format("CUDA path takes BF16, got {}", dtype_name(q.dtype()))));
        NN_TRY(cq, contiguous_of(q));
        NN_TRY(ck, contiguous_of(k));
        NN_TRY(cv, contiguous_of(v));
        NN_TRY(out, Tensor::empty(q.shape(), q.dtype(), Device::CUDA));
        NN_CHECK(tensor::cuda::attention(static_cast<int>(q.dtype()), cq.data_ptr(), ck.data_ptr(), cv.data_ptr(),
                                         out.data_ptr(), static_cast<std::size_t>(H), static_cast<std::size_t>(S),
                                         static_cast<std::size_t>(D), static_cast<float>(scale)));
        return out;
    }

    NN_CHECK(cpu_float(op, q.dtype()));
    NN_TRY(sc, scalar_like(scale, q.dtype()));
    NN_TRY(out, Tensor::zeros(q.shape(), q.dtype()));
    for (int64_t h = 0; h < H; ++h) {
        NN_TRY(qh3, q.slice(0, h, h + 1));
        NN_TRY(kh3, k.slice(0, h, h + 1));
        NN_TRY(vh3, v.slice(0, h, h + 1));
        NN_TRY(qh, qh3.squeeze(0));
        NN_TRY(kh, kh3.squeeze(0));
        NN_TRY(vh, vh3.squeeze(0));
        NN_TRY(kt, kh.transpose(0, 1));
        NN_TRY(ktc, kt.contiguous());
        NN_TRY(s, matmul(qh, ktc));
        NN_TRY(ss, mul(s, sc));
        NN_TRY(p, softmax(ss, -1));
        NN_TRY(oh, matmul(p, vh));
        NN_TRY(oi3, out.slice(0, h, h + 1));
        NN_TRY(oi, oi3.squeeze(0));
        NN_CHECK(add_inplace(oi, oh));
    }
    return out;
}

#undef NN_TRY
#undef NN_CHECK

} // namespace bee
