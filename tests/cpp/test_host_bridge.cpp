// GPU test of the C++ host bridge (bee_b200/host/tensor_cuda.hpp): the calls a
// Bee::Tensor maintainer would make from Bee/Tensor/Cuda/Backend.cpp, with the
// reference's synchronous semantics and error behaviour.  Exits 0 on success,
// prints the first failing check otherwise.  Run by tests/test_gpu_host_bridge.py.
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <random>
#include <string>
#include <vector>

#include "tensor_cuda.hpp"

namespace tc = bee_b200::tensor_cuda;

static int failures = 0;
#define CHECK(cond, ...)                                   \
    do {                                                   \
        if (!(cond)) {                                     \
            std::fprintf(stderr, "FAIL %s:%d: ", __FILE__, __LINE__); \
            std::fprintf(stderr, __VA_ARGS__);             \
            std::fprintf(stderr, "\n");                    \
            ++failures;                                    \
        }                                                  \
    } while (0)

template <typename T> static T* dev_alloc(size_t n) {
    auto r = tc::allocate(n * sizeof(T), 64);
    if (!r) {
        std::fprintf(stderr, "allocate failed: %s\n", r.error().message.c_str());
        std::exit(2);
    }
    return static_cast<T*>(*r);
}

int main() {
    constexpr int F32 = 4, I32 = 2, BF16 = 8;
    std::mt19937 rng(42);
    std::uniform_real_distribution<float> uni(-1.f, 1.f);

    // elementwise add, bit-exact
    const size_t n = 100003;
    std::vector<float> a(n), b(n), c(n);
    for (size_t i = 0; i < n; ++i) a[i] = uni(rng), b[i] = uni(rng);
    float *da = dev_alloc<float>(n), *db = dev_alloc<float>(n), *dc = dev_alloc<float>(n);
    CHECK(tc::memcpy_h2d(da, a.data(), n * 4).has_value(), "h2d a");
    CHECK(tc::memcpy_h2d(db, b.data(), n * 4).has_value(), "h2d b");
    CHECK(tc::ew_binary(0, F32, da, db, dc, n).has_value(), "add");
    CHECK(tc::memcpy_d2h(c.data(), dc, n * 4).has_value(), "d2h");
    for (size_t i = 0; i < n; ++i)
        if (c[i] != a[i] + b[i]) {
            CHECK(false, "add mismatch at %zu", i);
            break;
        }

    // matmul 2x2 known answer (Tests/Tensor/MatmulTests.cpp:31-62)
    float ha[4] = {1, 2, 3, 4}, hb[4] = {5, 6, 7, 8}, hc[4] = {0, 0, 0, 0};
    CHECK(tc::memcpy_h2d(da, ha, 16).has_value() && tc::memcpy_h2d(db, hb, 16).has_value(), "h2d 2x2");
    CHECK(tc::matmul(F32, da, db, dc, 2, 2, 2).has_value(), "matmul");
    CHECK(tc::memcpy_d2h(hc, dc, 16).has_value(), "d2h 2x2");
    CHECK(hc[0] == 19 && hc[1] == 22 && hc[2] == 43 && hc[3] == 50, "matmul KAT got %g %g %g %g", hc[0], hc[1], hc[2],
          hc[3]);

    // int32 full sum, bit-exact
    std::vector<int32_t> xi(n);
    std::uniform_int_distribution<int32_t> ui(-1000, 1000);
    int64_t want = 0;
    for (auto& v : xi) v = ui(rng), want += v;
    int32_t* dxi = dev_alloc<int32_t>(n);
    int32_t* dsum = dev_alloc<int32_t>(1);
    CHECK(tc::memcpy_h2d(dxi, xi.data(), n * 4).has_value(), "h2d ints");
    CHECK(tc::reduce_global(0, I32, dxi, dsum, n).has_value(), "reduce_global");
    int32_t got = 0;
    CHECK(tc::memcpy_d2h(&got, dsum, 4).has_value(), "d2h sum");
    CHECK(got == static_cast<int32_t>(want), "int32 sum %d != %lld", got, static_cast<long long>(want));

    // cast fp32 -> bf16 then back: |x - bf16(x)| <= 2^-9 |x|
    uint16_t* dbf = dev_alloc<uint16_t>(n);
    CHECK(tc::ew_cast(F32, da, BF16, dbf, n).has_value(), "cast to bf16");
    CHECK(tc::ew_cast(BF16, dbf, F32, dc, n).has_value(), "cast to f32");
    std::vector<float> back(n);
    CHECK(tc::memcpy_h2d(da, a.data(), n * 4).has_value(), "restore a");
    CHECK(tc::ew_cast(F32, da, BF16, dbf, n).has_value() && tc::ew_cast(BF16, dbf, F32, dc, n).has_value(), "round trip");
    CHECK(tc::memcpy_d2h(back.data(), dc, n * 4).has_value(), "d2h round trip");
    for (size_t i = 0; i < n; ++i)
        if (std::fabs(back[i] - a[i]) > std::ldexp(std::fabs(a[i]), -8)) {
            CHECK(false, "bf16 round trip at %zu: %g vs %g", i, back[i], a[i]);
            break;
        }

    // softmax rows sum to one
    const size_t rows = 7, cols = 1000;
    CHECK(tc::softmax_rows(F32, da, dc, rows, cols).has_value(), "softmax");
    std::vector<float> sm(rows * cols);
    CHECK(tc::memcpy_d2h(sm.data(), dc, rows * cols * 4).has_value(), "d2h softmax");
    for (size_t r = 0; r < rows; ++r) {
        double s = 0;
        for (size_t j = 0; j < cols; ++j) s += sm[r * cols + j];
        CHECK(std::fabs(s - 1.0) < 1e-4, "softmax row %zu sums to %g", r, s);
    }

    // error behaviour mirrored from Bee/CUDA/Api.cpp
    auto e0 = tc::reduce_global(0, I32, dxi, dsum, 0);
    CHECK(!e0.has_value() && e0.error().message.find("n == 0") != std::string::npos, "empty reduce must fail");
    CHECK(tc::ew_binary(0, F32, nullptr, nullptr, nullptr, 0).has_value(), "size-0 binary is a no-op");
    auto e1 = tc::ew_binary(0, 99, da, db, dc, n);
    CHECK(!e1.has_value() && e1.error().errc == 1 &&
              e1.error().message.find("cudaErrorInvalidValue") != std::string::npos && !e1.error().detail.empty(),
          "unknown dtype must give cudaErrorInvalidValue with a detail message");

    // transpose_2d (Tests/CUDA/TransposeTests.cu:79-92: 3x5 f64, i * 0.5) and contiguous() of its view
    {
        std::vector<double> t(15), tt(15), tv(15);
        for (int i = 0; i < 15; ++i) t[i] = i * 0.5;
        auto rs = tc::allocate(15 * 8, 64), rd = tc::allocate(15 * 8, 64);
        CHECK(rs.has_value() && rd.has_value(), "allocate transpose");
        CHECK(tc::memcpy_h2d(*rs, t.data(), 15 * 8).has_value(), "h2d transpose");
        CHECK(tc::transpose_2d(5, *rs, *rd, 3, 5).has_value(), "transpose_2d");
        CHECK(tc::memcpy_d2h(tt.data(), *rd, 15 * 8).has_value(), "d2h transpose");
        const std::int64_t shape[2] = {5, 3}, strides[2] = {1, 5};
        CHECK(tc::strided_copy(5, *rs, 2, shape, strides, *rd).has_value(), "strided_copy");
        CHECK(tc::memcpy_d2h(tv.data(), *rd, 15 * 8).has_value(), "d2h strided");
        for (int i = 0; i < 5; ++i)
            for (int j = 0; j < 3; ++j) {
                CHECK(tt[i * 3 + j] == t[j * 5 + i], "transpose (%d, %d)", i, j);
                CHECK(tv[i * 3 + j] == t[j * 5 + i], "strided copy (%d, %d)", i, j);
            }
        tc::deallocate(*rs, 0, 64);
        tc::deallocate(*rd, 0, 64);
    }

    // asynchronous mode: the same calls only enqueue; synchronize() is the fence
    CHECK(tc::is_synchronous(), "synchronous is the default");
    tc::set_synchronous(false);
    {
        std::vector<float> a2(n), c2(n);
        for (size_t i = 0; i < n; ++i) a2[i] = uni(rng);
        auto rt = tc::allocate(n * 4, 64);
        CHECK(rt.has_value(), "async allocate");
        float* dt2 = static_cast<float*>(*rt);
        CHECK(tc::memcpy_h2d(da, a2.data(), n * 4).has_value(), "async h2d");
        CHECK(tc::ew_binary(2, F32, da, da, dt2, n).has_value(), "async mul");
        CHECK(tc::ew_binary(0, F32, dt2, da, dc, n).has_value(), "async add");
        CHECK(tc::memcpy_d2h(c2.data(), dc, n * 4).has_value(), "async d2h (waits)");
        for (size_t i = 0; i < n; ++i) {
            volatile float sq = a2[i] * a2[i];  // two roundings, as the two kernels do
            if (c2[i] != sq + a2[i]) {
                CHECK(false, "async chain mismatch at %zu", i);
                break;
            }
        }
        tc::deallocate(dt2, n * 4, 64);
        CHECK(tc::synchronize().has_value(), "async synchronize");
    }
    tc::set_synchronous(true);

    for (void* p : {static_cast<void*>(da), static_cast<void*>(db), static_cast<void*>(dc), static_cast<void*>(dxi),
                    static_cast<void*>(dsum), static_cast<void*>(dbf)})
        tc::deallocate(p, 0, 64);
    CHECK(tc::synchronize().has_value(), "synchronize");
    if (failures == 0) std::printf("host bridge ok\n");
    return failures == 0 ? 0 : 1;
}
