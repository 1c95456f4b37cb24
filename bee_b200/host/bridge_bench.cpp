// Measures what the Tensor layer pays around a CUDA matmul (the plumbing cost of
// Bee/Tensor/Ops/Matmul.cpp:36-179 on the CUDA backend) through the C++ bridge:
//
//   reference sequence, synchronous: allocate C, zero it (Matmul.cpp:73), matmul,
//     free C, each call synchronising as the reference's bridge does
//     (Bee/CUDA/Api.cpp:131-133, 188-190);
//   asynchronous, one fence per call: allocate from the stream-ordered pool,
//     matmul (no zero fill: the kernel writes every element of C), free, then
//     one synchronize();
//   asynchronous, pipelined: the same calls back to back, one synchronize() at
//     the end (the kernel-bound floor).
//
// Prints one JSON line with the wall-clock microseconds per call of each.  Run
// by bench.py (extra "bridge_matmul") on the GPU it is given.
#include <chrono>
#include <cstdio>
#include <cstdint>
#include <random>
#include <vector>

#include "tensor_cuda.hpp"

namespace tc = bee_b200::tensor_cuda;
using clk = std::chrono::steady_clock;

static bool ok_or_die(bool ok, const char* what) {
    if (!ok) {
        std::fprintf(stderr, "bridge_bench: %s failed\n", what);
        std::exit(2);
    }
    return ok;
}

struct Times {
    double sync_ref, async_fenced, async_pipelined;
};

static Times measure(int dt, size_t elem, size_t M, size_t K, size_t N, int iters) {
    tc::set_synchronous(true);
    auto ra = tc::allocate(M * K * elem, 64), rb = tc::allocate(K * N * elem, 64);
    ok_or_die(ra.has_value() && rb.has_value(), "allocate A, B");
    void *A = *ra, *B = *rb;
    std::vector<uint8_t> host(std::max(M * K, K * N) * elem);
    std::mt19937 rng(7);
    for (size_t i = 0; i + 1 < host.size(); i += 2) {
        // small finite values of either type: bf16 1.0 +- or fp32 low-mantissa patterns
        const uint16_t v = static_cast<uint16_t>(0x3f80u + (rng() & 0x7fu));
        host[i] = static_cast<uint8_t>(v & 0xff);
        host[i + 1] = static_cast<uint8_t>(v >> 8);
    }
    ok_or_die(tc::memcpy_h2d(A, host.data(), M * K * elem).has_value(), "h2d A");
    ok_or_die(tc::memcpy_h2d(B, host.data(), K * N * elem).has_value(), "h2d B");

    auto one_ref = [&] {
        auto rc = tc::allocate(M * N * elem, 64);
        ok_or_die(rc.has_value(), "allocate C");
        ok_or_die(tc::memset(*rc, 0, M * N * elem).has_value(), "memset C");
        ok_or_die(tc::matmul(dt, A, B, *rc, M, K, N).has_value(), "matmul");
        tc::deallocate(*rc, M * N * elem, 64);
    };
    auto one_async = [&] {
        auto rc = tc::allocate(M * N * elem, 64);
        ok_or_die(rc.has_value(), "allocate C");
        ok_or_die(tc::matmul(dt, A, B, *rc, M, K, N).has_value(), "matmul");
        tc::deallocate(*rc, M * N * elem, 64);
    };
    auto per_call_us = [&](auto&& body, bool fence_each, bool fence_end) {
        for (int i = 0; i < 3; ++i) body();
        ok_or_die(tc::synchronize().has_value(), "synchronize");
        const auto t0 = clk::now();
        for (int i = 0; i < iters; ++i) {
            body();
            if (fence_each) ok_or_die(tc::synchronize().has_value(), "synchronize");
        }
        if (fence_end) ok_or_die(tc::synchronize().has_value(), "synchronize");
        return std::chrono::duration<double, std::micro>(clk::now() - t0).count() / iters;
    };
    Times t{};
    t.sync_ref = per_call_us(one_ref, false, false);
    tc::set_synchronous(false);
    t.async_fenced = per_call_us(one_async, true, false);
    t.async_pipelined = per_call_us(one_async, false, true);
    tc::set_synchronous(true);
    tc::deallocate(A, M * K * elem, 64);
    tc::deallocate(B, K * N * elem, 64);
    return t;
}

int main() {
    constexpr int F32 = 4, BF16 = 8;
    const Times f = measure(F32, 4, 1024, 1024, 1024, 50);
    const Times h = measure(BF16, 2, 4096, 4096, 4096, 50);
    std::printf(
        "{\"unit\": \"us per call\", \"f32_1024\": {\"sync_reference\": %.1f, \"async_fenced\": %.1f, "
        "\"async_pipelined\": %.1f}, \"bf16_4096\": {\"sync_reference\": %.1f, \"async_fenced\": %.1f, "
        "\"async_pipelined\": %.1f}}\n",
        f.sync_ref, f.async_fenced, f.async_pipelined, h.sync_ref, h.async_fenced, h.async_pipelined);
    return 0;
}
