// The reference's Tensor layer on bee_b200: bee::* ops on Device::CUDA tensors,
// through the reference's own Tensor sources compiled with
// BEE_TENSOR_WITH_CUDA and bee_b200/tensor/Backend.cpp as the CUDA boundary,
// checked against the same ops on Device::CPU tensors (the reference's CPU
// path).  The CUDA cases restate Tests/Tensor/CudaStubTests.cpp:42-571 (the
// BEE_TENSOR_WITH_CUDA=ON half) with that file's sizes and tolerances, plus the
// ops and dtypes bee_b200 adds (BF16 / F16 matmul and cast, 1024^3 fp32
// matmul on the tensor cores, softmax, rms_norm, rope, rms_norm_rope, bmm,
// attention from bee_b200/tensor/Nn.hpp).
//
//   test_bee_tensor_cuda        every case (needs a GPU)
//   test_bee_tensor_cuda cpu    only the CPU-path cases of the new ops
// Prints one line per case; exits 0 when all pass.  Built by
// `make -C oracle tensor-cuda`, run by tests/test_gpu_bee_tensor.py and
// tests/test_bee_tensor_cpu.py.
#include "Nn.hpp"
#include "Tensor/Cuda/CudaAllocator.hpp"
#include "Tensor/Tensor.hpp"
#include "bee_b200.h"

#include <cmath>
#include <cstdio>
#include <cstring>
#include <functional>
#include <random>
#include <string>
#include <vector>

using namespace bee;

namespace
{

std::string g_fail;

#define EXPECT(cond, ...)                                                                                                        \
    do {                                                                                                                         \
        if (!(cond)) {                                                                                                           \
            char buf_[512];                                                                                                      \
            std::snprintf(buf_, sizeof(buf_), __VA_ARGS__);                                                                      \
            g_fail = std::string(__FILE__ ":") + std::to_string(__LINE__) + ": " + buf_;                                         \
            return false;                                                                                                        \
        }                                                                                                                        \
    } while (0)

template <typename T>
auto get(Result<T> r, const char* what) -> T
{
    if (!r) {
        std::fprintf(stderr, "%s failed: %s\n", what, std::string(r.error().message.view()).c_str());
        throw std::runtime_error(what);
    }
    return std::move(*r);
}

inline void get(Result<void> r, const char* what)
{
    if (!r) {
        std::fprintf(stderr, "%s failed: %s\n", what, std::string(r.error().message.view()).c_str());
        throw std::runtime_error(what);
    }
}

#define OK(expr) get((expr), #expr)

auto host_f32(const Tensor& t) -> std::vector<float>
{
    Tensor f = t.dtype() == DType::F32 ? t : OK(cast(t, DType::F32));
    Tensor c = OK(OK(f.to(Device::CPU)).contiguous());
    const auto* p = static_cast<const float*>(c.data_ptr());
    return std::vector<float>(p, p + c.numel());
}

template <typename T>
auto host_vec(const Tensor& t) -> std::vector<T>
{
    Tensor c = OK(OK(t.to(Device::CPU)).contiguous());
    const auto* p = static_cast<const T*>(c.data_ptr());
    return std::vector<T>(p, p + c.numel());
}

auto cpu_tensor(Shape s, const std::vector<float>& v) -> Tensor
{
    Tensor t = OK(Tensor::empty(std::move(s), DType::F32));
    std::memcpy(t.data_ptr(), v.data(), v.size() * sizeof(float));
    return t;
}

auto normals(std::size_t n, std::uint64_t seed, float scale = 1.f) -> std::vector<float>
{
    std::mt19937_64 rng(seed);
    std::normal_distribution<float> nd(0.f, 1.f);
    std::vector<float> v(n);
    for (auto& x : v)
        x = nd(rng) * scale;
    return v;
}

// bf16-rounded copy of an fp32 CPU tensor, made on the device (the reference's
// CPU cast to BF16 writes nothing, Tensor/Cpu/CastCpu.hpp:348)
auto bf16_rounded(const Tensor& cpu, DType half = DType::BF16) -> std::pair<Tensor, Tensor>
{
    Tensor h = OK(cast(OK(cpu.to(Device::CUDA)), half));
    Tensor back = OK(OK(cast(h, DType::F32)).to(Device::CPU));
    return {h, back};
}

// max |got - want| / max(|want|, rms(want)): the stated tolerances on the output's own scale
auto out_err(const std::vector<float>& got, const std::vector<float>& want) -> double
{
    double ss = 0;
    for (float w : want)
        ss += double(w) * w;
    const double rms = std::sqrt(ss / double(want.size() ? want.size() : 1));
    double e = 0;
    for (std::size_t i = 0; i < want.size(); ++i) {
        const double sc = std::max(std::abs(double(want[i])), rms);
        if (sc > 0)
            e = std::max(e, std::abs(double(got[i]) - want[i]) / sc);
    }
    return e;
}

bool equal_f32(const std::vector<float>& a, const std::vector<float>& b)
{
    return a.size() == b.size() && std::memcmp(a.data(), b.data(), a.size() * sizeof(float)) == 0;
}

// ── CudaStubTests.cpp:56-157: storage, factories, transfers ─────────────────

bool allocator_device()
{
    EXPECT(CudaAllocator::instance().device() == Device::CUDA, "CudaAllocator device");
    return true;
}

bool empty_on_cuda()
{
    auto t = OK(Tensor::empty({16, 8}, DType::F32, Device::CUDA));
    EXPECT(t.device() == Device::CUDA && t.numel() == 128 && t.is_contiguous() && t.data_ptr() != nullptr, "empty");
    return true;
}

bool zeros_on_cuda()
{
    auto v = host_f32(OK(Tensor::zeros({64}, DType::F32, Device::CUDA)));
    for (float x : v)
        EXPECT(x == 0.f, "zeros: %g", x);
    return true;
}

bool to_device_round_trip()
{
    auto cpu = OK(Tensor::arange(0, 128, 1, DType::F32, Device::CPU));
    auto cu = OK(cpu.to(Device::CUDA));
    EXPECT(cu.device() == Device::CUDA, "device");
    EXPECT(equal_f32(host_f32(cu), host_f32(cpu)), "values changed on the round trip");
    return true;
}

bool arange_on_cuda()
{
    auto v = host_vec<std::int32_t>(OK(Tensor::arange(0, 32, 1, DType::I32, Device::CUDA)));
    for (int i = 0; i < 32; ++i)
        EXPECT(v[std::size_t(i)] == i, "arange[%d] = %d", i, v[std::size_t(i)]);
    return true;
}

bool clone_on_cuda()
{
    auto a = OK(Tensor::arange(0, 16, 1, DType::F32, Device::CUDA));
    auto b = OK(a.clone());
    EXPECT(b.device() == Device::CUDA && b.data_ptr() != a.data_ptr(), "clone shares storage");
    EXPECT(equal_f32(host_f32(a), host_f32(b)), "clone values");
    return true;
}

bool to_same_device_is_shallow()
{
    auto t = OK(Tensor::zeros({4}, DType::F32, Device::CUDA));
    EXPECT(OK(t.to(Device::CUDA)).data_ptr() == t.data_ptr(), "to(CUDA) copied");
    return true;
}

// ── CudaStubTests.cpp:158-330: elementwise, cast ────────────────────────────

bool binary_f32_matches_cpu()
{
    const std::int64_t n = 257;
    auto a = OK(Tensor::arange(1, n + 1, 1, DType::F32, Device::CPU));
    auto b = OK(Tensor::full({n}, DType::F32, 2.0, Device::CPU));
    auto ac = OK(a.to(Device::CUDA)), bc = OK(b.to(Device::CUDA));
    using Fn = Result<Tensor> (*)(const Tensor&, const Tensor&);
    for (Fn f : {Fn(&add), Fn(&sub), Fn(&mul), Fn(&div)}) {
        auto c = OK(f(ac, bc));
        EXPECT(c.device() == Device::CUDA, "result device");
        EXPECT(equal_f32(host_f32(c), host_f32(OK(f(a, b)))), "binary op differs from the CPU");
    }
    return true;
}

bool unary_f32_matches_cpu()
{
    auto src = OK(Tensor::arange(1, 65, 1, DType::F32, Device::CPU));
    auto cu = OK(src.to(Device::CUDA));
    using Fn = Result<Tensor> (*)(const Tensor&);
    const Fn fns[] = {&neg, &abs, &sqrt, &exp, &log};
    const float tol[] = {0.f, 0.f, 0.f, 3e-7f, 3e-7f};  // relative; exp/log within 2 ulp of the CPU's
    for (int i = 0; i < 5; ++i) {
        auto s = i == 3 ? OK(Tensor::arange(0, 8, 1, DType::F32, Device::CPU)) : src;  // exp on small arguments
        auto g = host_f32(OK(fns[i](OK(s.to(Device::CUDA)))));
        auto w = host_f32(OK(fns[i](s)));
        for (std::size_t k = 0; k < w.size(); ++k)
            EXPECT(std::abs(g[k] - w[k]) <= tol[i] * std::abs(w[k]), "unary %d at %zu: %g vs %g", i, k, g[k], w[k]);
    }
    (void)cu;
    return true;
}

bool inplace_add_matches_cpu()
{
    auto a = OK(Tensor::arange(0, 100, 1, DType::F32, Device::CPU));
    auto b = OK(Tensor::full({100}, DType::F32, 3.0, Device::CPU));
    auto ac = OK(a.to(Device::CUDA)), bc = OK(b.to(Device::CUDA));
    OK(add_inplace(ac, bc));
    OK(add_inplace(a, b));
    EXPECT(equal_f32(host_f32(ac), host_f32(a)), "add_inplace");
    return true;
}

bool cast_matches_cpu()
{
    auto f = OK(Tensor::arange(0, 100, 1, DType::F32, Device::CPU));
    auto got = host_vec<std::int32_t>(OK(cast(OK(f.to(Device::CUDA)), DType::I32)));
    auto want = host_vec<std::int32_t>(OK(cast(f, DType::I32)));
    EXPECT(got == want, "F32 -> I32");
    auto i = OK(Tensor::arange(-16, 84, 1, DType::I32, Device::CPU));
    auto gd = host_vec<double>(OK(cast(OK(i.to(Device::CUDA)), DType::F64)));
    auto wd = host_vec<double>(OK(cast(i, DType::F64)));
    EXPECT(gd == wd, "I32 -> F64");
    return true;
}

bool shape_mismatch_is_an_error()
{
    auto a = OK(Tensor::zeros({4, 3}, DType::F32, Device::CUDA));
    auto b = OK(Tensor::zeros({3}, DType::F32, Device::CUDA));
    EXPECT(!add(a, b).has_value(), "broadcast add on CUDA must fail as in the reference");
    return true;
}

// ── CudaStubTests.cpp:331-470: reductions ───────────────────────────────────

bool reduce_global_matches_cpu()
{
    auto f = OK(Tensor::arange(0, 1000, 1, DType::F32, Device::CPU));
    auto fc = OK(f.to(Device::CUDA));
    const float s = host_f32(OK(sum(fc)))[0], sw = host_f32(OK(sum(f)))[0];
    EXPECT(std::abs(s - sw) <= 1e-5f * std::abs(sw), "sum %g vs %g", s, sw);
    const float m = host_f32(OK(mean(fc)))[0], mw = host_f32(OK(mean(f)))[0];
    EXPECT(std::abs(m - mw) <= 1e-5f * std::abs(mw), "mean %g vs %g", m, mw);
    auto i = OK(Tensor::arange(1, 13, 1, DType::I32, Device::CPU));
    auto ic = OK(i.to(Device::CUDA));
    EXPECT(host_vec<std::int32_t>(OK(min(ic)))[0] == 1, "min");
    EXPECT(host_vec<std::int32_t>(OK(max(ic)))[0] == 12, "max");
    EXPECT(host_vec<std::int32_t>(OK(prod(ic)))[0] == host_vec<std::int32_t>(OK(prod(i)))[0], "prod");
    return true;
}

bool reduce_axis_matches_cpu()
{
    auto x = OK(OK(Tensor::arange(0, 60, 1, DType::F32, Device::CPU)).reshape({3, 4, 5}));
    auto xc = OK(x.to(Device::CUDA));
    for (int dim : {0, 1, 2, -1}) {
        auto g = host_f32(OK(sum(xc, dim)));
        auto w = host_f32(OK(sum(x, dim)));
        EXPECT(g.size() == w.size(), "shape");
        for (std::size_t k = 0; k < w.size(); ++k)
            EXPECT(std::abs(g[k] - w[k]) <= 1e-5f * std::abs(w[k]), "sum dim %d at %zu", dim, k);
    }
    auto y = OK(OK(Tensor::arange(0, 24, 1, DType::F64, Device::CPU)).reshape({2, 3, 4}));
    auto gm = OK(mean(OK(y.to(Device::CUDA)), 1, true));
    EXPECT(gm.shape() == Shape({2, 1, 4}), "keepdim shape");
    EXPECT(host_vec<double>(gm) == host_vec<double>(OK(mean(y, 1, true))), "mean F64 keepdim");
    return true;
}

bool integer_mean_on_cuda_is_an_error()
{
    auto x = OK(Tensor::arange(0, 10, 1, DType::I32, Device::CUDA));
    EXPECT(!mean(x).has_value(), "the reference's Reduce.cpp rejects I32 mean on CUDA");
    return true;
}

// ── CudaStubTests.cpp:471-571: matmul, transpose ───────────────────────────

bool matmul_matches_cpu()
{
    {  // F32 17 x 33 x 21, randn, 1e-3 as in the reference
        auto a = OK(randn({17, 33}, DType::F32, 1)), b = OK(randn({33, 21}, DType::F32, 2));
        auto g = host_f32(OK(matmul(OK(a.to(Device::CUDA)), OK(b.to(Device::CUDA)))));
        auto w = host_f32(OK(matmul(a, b)));
        for (std::size_t k = 0; k < w.size(); ++k)
            EXPECT(std::abs(g[k] - w[k]) <= 1e-3f, "F32 matmul at %zu", k);
    }
    {  // F64 1e-9
        auto a = OK(randn({9, 7}, DType::F64, 5)), b = OK(randn({7, 11}, DType::F64, 6));
        auto g = host_vec<double>(OK(matmul(OK(a.to(Device::CUDA)), OK(b.to(Device::CUDA)))));
        auto w = host_vec<double>(OK(matmul(a, b)));
        for (std::size_t k = 0; k < w.size(); ++k)
            EXPECT(std::abs(g[k] - w[k]) <= 1e-9, "F64 matmul at %zu", k);
    }
    {  // I32 exact
        auto a = OK(randint(-3, 3, {13, 17}, DType::I32, 11)), b = OK(randint(-3, 3, {17, 19}, DType::I32, 12));
        EXPECT(host_vec<std::int32_t>(OK(matmul(OK(a.to(Device::CUDA)), OK(b.to(Device::CUDA))))) ==
                   host_vec<std::int32_t>(OK(matmul(a, b))),
               "I32 matmul");
    }
    {  // sizes on and around the tile boundary
        auto a = OK(randn({64, 16}, DType::F32, 7)), b = OK(randn({16, 65}, DType::F32, 8));
        auto g = host_f32(OK(matmul(OK(a.to(Device::CUDA)), OK(b.to(Device::CUDA)))));
        auto w = host_f32(OK(matmul(a, b)));
        for (std::size_t k = 0; k < w.size(); ++k)
            EXPECT(std::abs(g[k] - w[k]) <= 1e-3f, "boundary matmul at %zu", k);
    }
    return true;
}

bool transpose_via_contiguous()
{
    auto h = OK(randn({7, 13}, DType::F32, 42));
    auto gt = host_f32(OK(OK(OK(h.to(Device::CUDA)).transpose(0, 1)).contiguous()));
    auto wt = host_f32(OK(OK(h.transpose(0, 1)).contiguous()));
    EXPECT(equal_f32(gt, wt), "F32 transpose");
    auto hi = OK(randint(-100, 100, {11, 5}, DType::I64, 77));
    EXPECT(host_vec<std::int64_t>(OK(OK(OK(hi.to(Device::CUDA)).transpose(0, 1)).contiguous())) ==
               host_vec<std::int64_t>(OK(OK(hi.transpose(0, 1)).contiguous())),
           "I64 transpose");
    return true;
}

// ── added by bee_b200: the config sizes and dtypes of the path ──────────────

bool matmul_f32_1024_tensor_cores()
{
    std::mt19937_64 rng(1024);
    std::uniform_real_distribution<float> u(-1.f, 1.f);
    std::vector<float> av(1024 * 1024), bv(1024 * 1024);
    for (auto& x : av)
        x = u(rng);
    for (auto& x : bv)
        x = u(rng);
    auto a = cpu_tensor({1024, 1024}, av), b = cpu_tensor({1024, 1024}, bv);
    auto g = host_f32(OK(matmul(OK(a.to(Device::CUDA)), OK(b.to(Device::CUDA)))));
    auto w = host_f32(OK(matmul(a, b)));
    const double e = out_err(g, w);
    std::printf("  fp32 1024^3 through bee::matmul: max error %.3e of max(|ref|, rms)\n", e);
    EXPECT(e <= 1e-4, "fp32 1024^3: %.3e > 1e-4", e);
    return true;
}

bool matmul_16bit_and_cast()
{
    for (DType half : {DType::BF16, DType::F16}) {
        auto a32 = cpu_tensor({384, 256}, normals(384 * 256, 3));
        auto b32 = cpu_tensor({256, 520}, normals(256 * 520, 4));
        auto [ah, ar] = bf16_rounded(a32, half);
        auto [bh, br] = bf16_rounded(b32, half);
        auto c = OK(matmul(ah, bh));  // the reference's unchanged bee::matmul, CUDA path
        EXPECT(c.dtype() == half && c.shape() == Shape({384, 520}), "16-bit matmul result");
        const double e = out_err(host_f32(c), host_f32(OK(matmul(ar, br))));
        std::printf("  %s matmul 384x256x520: max error %.3e\n", half == DType::BF16 ? "bf16" : "f16", e);
        EXPECT(e <= 1e-2, "16-bit matmul error %.3e", e);
    }
    return true;
}

bool softmax_matches_cpu()
{
    auto x = cpu_tensor({37, 300}, normals(37 * 300, 9, 3.f));
    auto xc = OK(x.to(Device::CUDA));
    for (int dim : {1, -1, 0}) {
        const double e = out_err(host_f32(OK(softmax(xc, dim))), host_f32(OK(softmax(x, dim))));
        EXPECT(e <= 1e-5, "softmax dim %d: %.3e", dim, e);
    }
    // BF16 on the device against the fp32 CPU composition of the rounded input
    auto [xh, xr] = bf16_rounded(x);
    const double eb = out_err(host_f32(OK(softmax(xh, -1))), host_f32(OK(softmax(xr, -1))));
    EXPECT(eb <= 1e-2, "bf16 softmax %.3e", eb);
    return true;
}

bool rms_norm_rope_match_cpu()
{
    const std::int64_t B = 2, S = 16, H = 4, D = 128;
    auto x = cpu_tensor({B, S, H, D}, normals(std::size_t(B * S * H * D), 21));
    std::vector<float> wv = normals(std::size_t(H * D), 22, 0.02f);
    for (auto& w : wv)
        w += 1.f;
    auto w = cpu_tensor({H * D}, wv);
    auto xc = OK(x.to(Device::CUDA)), wc = OK(w.to(Device::CUDA));
    auto xrow = OK(x.reshape({B * S, H * D}));
    auto e1 = out_err(host_f32(OK(rms_norm(OK(xrow.to(Device::CUDA)), wc, 1e-6))), host_f32(OK(rms_norm(xrow, w, 1e-6))));
    EXPECT(e1 <= 1e-5, "rms_norm F32 %.3e", e1);
    auto e2 = out_err(host_f32(OK(rope(xc, 10000.0, 3))), host_f32(OK(rope(x, 10000.0, 3))));
    EXPECT(e2 <= 1e-5, "rope F32 %.3e", e2);
    auto e3 = out_err(host_f32(OK(rms_norm_rope(xc, wc, 1e-6, 10000.0, 0))), host_f32(OK(rms_norm_rope(x, w, 1e-6, 10000.0, 0))));
    EXPECT(e3 <= 1e-5, "rms_norm_rope F32 %.3e", e3);
    auto [xh, xr] = bf16_rounded(x);
    auto [wh, wr] = bf16_rounded(w);
    auto e4 = out_err(host_f32(OK(rms_norm_rope(xh, wh, 1e-6, 10000.0, 0))), host_f32(OK(rms_norm_rope(xr, wr, 1e-6, 10000.0, 0))));
    std::printf("  bf16 rms_norm_rope: max error %.3e\n", e4);
    EXPECT(e4 <= 1e-2, "rms_norm_rope BF16 %.3e", e4);
    return true;
}

bool bmm_and_attention_match_cpu()
{
    auto a = cpu_tensor({3, 130, 72}, normals(3 * 130 * 72, 31));
    auto b = cpu_tensor({3, 72, 136}, normals(3 * 72 * 136, 32));
    const double e1 = out_err(host_f32(OK(bmm(OK(a.to(Device::CUDA)), OK(b.to(Device::CUDA))))), host_f32(OK(bmm(a, b))));
    EXPECT(e1 <= 1e-4, "bmm F32 %.3e", e1);
    auto [ah, ar] = bf16_rounded(a);
    auto [bh, br] = bf16_rounded(b);
    const double e2 = out_err(host_f32(OK(bmm(ah, bh))), host_f32(OK(bmm(ar, br))));
    EXPECT(e2 <= 1e-2, "bmm BF16 %.3e", e2);
    const std::int64_t H = 2, S = 256, D = 128;
    auto [qh, qr] = bf16_rounded(cpu_tensor({H, S, D}, normals(std::size_t(H * S * D), 41)));
    auto [kh, kr] = bf16_rounded(cpu_tensor({H, S, D}, normals(std::size_t(H * S * D), 42)));
    auto [vh, vr] = bf16_rounded(cpu_tensor({H, S, D}, normals(std::size_t(H * S * D), 43)));
    const double scale = 1.0 / std::sqrt(double(D));
    const double e3 = out_err(host_f32(OK(attention(qh, kh, vh, scale))), host_f32(OK(attention(qr, kr, vr, scale))));
    std::printf("  bf16 attention 2x256x128: max error %.3e\n", e3);
    EXPECT(e3 <= 1e-2, "attention BF16 %.3e", e3);
    return true;
}

bool new_ops_reject_bad_arguments()
{
    auto x = OK(Tensor::zeros({2, 3}, DType::F32, Device::CUDA));
    auto w = OK(Tensor::zeros({4}, DType::F32, Device::CUDA));
    EXPECT(!rms_norm(x, w).has_value(), "weight size");
    EXPECT(!rope(x).has_value(), "rope needs 4-D");
    EXPECT(!softmax(x, 2).has_value(), "dim range");
    auto xi = OK(Tensor::zeros({2, 3}, DType::I32, Device::CUDA));
    EXPECT(!softmax(xi, 1).has_value(), "integer softmax");
    auto cpu = OK(Tensor::zeros({2, 3}, DType::F32));
    EXPECT(!bmm(OK(x.reshape({1, 2, 3})), OK(cpu.reshape({1, 3, 2}))).has_value(), "mixed devices");
    return true;
}

// ── CPU path of the new ops (no GPU needed) ─────────────────────────────────

bool cpu_softmax_known_values()
{
    auto x = cpu_tensor({2, 3}, {0.f, 0.f, 0.f, 1.f, 2.f, 3.f});
    auto v = host_vec<float>(OK(softmax(x, 1)));
    const double z = std::exp(1.0) + std::exp(2.0) + std::exp(3.0);
    for (int i = 0; i < 3; ++i)
        EXPECT(std::abs(v[std::size_t(i)] - 1.0 / 3) < 1e-6, "uniform row");
    for (int i = 0; i < 3; ++i)
        EXPECT(std::abs(v[std::size_t(3 + i)] - std::exp(1.0 + i) / z) < 1e-6, "row 1");
    auto c = host_vec<float>(OK(softmax(x, 0)));  // columns: softmax of (0, 1), (0, 2), (0, 3)
    EXPECT(std::abs(c[0] - 1.0 / (1.0 + std::exp(1.0))) < 1e-6, "dim 0");
    return true;
}

bool cpu_rms_norm_and_rope_known_values()
{
    auto x = cpu_tensor({1, 4}, {1.f, -2.f, 3.f, -4.f});
    auto w = cpu_tensor({4}, {1.f, 1.f, 2.f, 0.5f});
    auto v = host_vec<float>(OK(rms_norm(x, w, 0.0)));
    const double r = std::sqrt((1 + 4 + 9 + 16) / 4.0);
    const double want[4] = {1 / r, -2 / r, 6 / r, -2 / r};
    for (int i = 0; i < 4; ++i)
        EXPECT(std::abs(v[std::size_t(i)] - want[i]) < 1e-6, "rms_norm[%d]", i);
    // one head of 4 at position 1: pairs (0, 2) and (1, 3), angles 1 and 1/100 (theta 1e4)
    auto q = cpu_tensor({1, 2, 1, 4}, {1.f, 2.f, 3.f, 4.f, 1.f, 2.f, 3.f, 4.f});
    auto o = host_vec<float>(OK(rope(q, 10000.0, 0)));
    for (int i = 0; i < 4; ++i)
        EXPECT(o[std::size_t(i)] == float(i + 1), "position 0 is the identity");
    const double a0 = 1.0, a1 = 0.01;
    EXPECT(std::abs(o[4] - (1 * std::cos(a0) - 3 * std::sin(a0))) < 1e-6, "rope pair 0 first");
    EXPECT(std::abs(o[6] - (3 * std::cos(a0) + 1 * std::sin(a0))) < 1e-6, "rope pair 0 second");
    EXPECT(std::abs(o[5] - (2 * std::cos(a1) - 4 * std::sin(a1))) < 1e-6, "rope pair 1 first");
    return true;
}

bool cpu_bmm_and_attention_known_values()
{
    auto a = cpu_tensor({2, 2, 2}, {1, 2, 3, 4, 1, 0, 0, 1});
    auto b = cpu_tensor({2, 2, 2}, {5, 6, 7, 8, 2, 3, 4, 5});
    auto c = host_vec<float>(OK(bmm(a, b)));
    const float want[8] = {19, 22, 43, 50, 2, 3, 4, 5};  // Tests/Tensor/MatmulTests.cpp:31-62 per batch
    for (int i = 0; i < 8; ++i)
        EXPECT(c[std::size_t(i)] == want[i], "bmm[%d]", i);
    // equal keys: uniform attention, the output is the mean of V's rows
    auto q = cpu_tensor({1, 2, 2}, {1, 0, 0, 1});
    auto k = cpu_tensor({1, 2, 2}, {1, 1, 1, 1});
    auto v = cpu_tensor({1, 2, 2}, {2, 4, 6, 8});
    auto o = host_vec<float>(OK(attention(q, k, v, 0.5)));
    const float mean_v[4] = {4, 6, 4, 6};
    for (int i = 0; i < 4; ++i)
        EXPECT(std::abs(o[std::size_t(i)] - mean_v[i]) < 1e-6, "attention[%d]", i);
    return true;
}

struct Case
{
    const char* name;
    bool (*fn)();
    bool cuda;
};

const Case kCases[] = {
    {"cpu_softmax_known_values", cpu_softmax_known_values, false},
    {"cpu_rms_norm_and_rope_known_values", cpu_rms_norm_and_rope_known_values, false},
    {"cpu_bmm_and_attention_known_values", cpu_bmm_and_attention_known_values, false},
    {"allocator_device", allocator_device, true},
    {"empty_on_cuda", empty_on_cuda, true},
    {"zeros_on_cuda", zeros_on_cuda, true},
    {"to_device_round_trip", to_device_round_trip, true},
    {"arange_on_cuda", arange_on_cuda, true},
    {"clone_on_cuda", clone_on_cuda, true},
    {"to_same_device_is_shallow", to_same_device_is_shallow, true},
    {"binary_f32_matches_cpu", binary_f32_matches_cpu, true},
    {"unary_f32_matches_cpu", unary_f32_matches_cpu, true},
    {"inplace_add_matches_cpu", inplace_add_matches_cpu, true},
    {"cast_matches_cpu", cast_matches_cpu, true},
    {"shape_mismatch_is_an_error", shape_mismatch_is_an_error, true},
    {"reduce_global_matches_cpu", reduce_global_matches_cpu, true},
    {"reduce_axis_matches_cpu", reduce_axis_matches_cpu, true},
    {"integer_mean_on_cuda_is_an_error", integer_mean_on_cuda_is_an_error, true},
    {"matmul_matches_cpu", matmul_matches_cpu, true},
    {"transpose_via_contiguous", transpose_via_contiguous, true},
    {"matmul_f32_1024_tensor_cores", matmul_f32_1024_tensor_cores, true},
    {"matmul_16bit_and_cast", matmul_16bit_and_cast, true},
    {"softmax_matches_cpu", softmax_matches_cpu, true},
    {"rms_norm_rope_match_cpu", rms_norm_rope_match_cpu, true},
    {"bmm_and_attention_match_cpu", bmm_and_attention_match_cpu, true},
    {"new_ops_reject_bad_arguments", new_ops_reject_bad_arguments, true},
};

} // namespace

int main(int argc, char** argv)
{
    const bool cpu_only = argc > 1 && std::string(argv[1]) == "cpu";
    int devices = 0;
    if (!cpu_only && (bee_b200_device_count(&devices) != 0 || devices < 1)) {
        std::fprintf(stderr, "no CUDA device (run with `cpu` for the CPU cases)\n");
        return 2;
    }
    int failed = 0, ran = 0;
    for (const Case& c : kCases) {
        if (c.cuda && cpu_only)
            continue;
        g_fail.clear();
        bool ok = false;
        try {
            ok = c.fn();
        } catch (const std::exception& e) {
            g_fail = e.what();
        }
        ++ran;
        std::printf("%s %s%s%s\n", ok ? "PASS" : "FAIL", c.name, ok ? "" : ": ", ok ? "" : g_fail.c_str());
        failed += ok ? 0 : 1;
    }
    std::printf("%d of %d cases passed\n", ran - failed, ran);
    return failed == 0 ? 0 : 1;
}
