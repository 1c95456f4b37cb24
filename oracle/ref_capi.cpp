// C entry points over the reference's own CPU path (Bee::Tensor public ops),
// compiled together with the reference sources into oracle/_ref/libbee_ref.so
// by oracle/Makefile.  Test infrastructure only: the parity tests use it to pin
// the oracle restatement, and bench.py's reference arm times it on the host.
//
// Every function copies the host inputs into bee::Tensor objects, runs the
// reference op `reps` times (only the op is timed, wall clock per call),
// copies the last result out and returns the median seconds per call, or a
// negative value when the reference reports an error (message on stderr).
// Ops the reference lacks (softmax, RMSNorm, RoPE, attention) are the
// compositions of public ops that the reference's users would write.
#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <thread>
#include <vector>

#include "SIMD/Detect.hpp"
#include "Tensor/Tensor.hpp"

using namespace bee;

namespace {

template <typename R> bool okr(const R& r, const char* what) {
    if (!r.has_value()) {
        std::fprintf(stderr, "bee reference: %s failed: %s\n", what, r.error().format().c_str());
        return false;
    }
    return true;
}

Tensor make(Shape s, DType dt, const void* src) {
    auto t = Tensor::empty(std::move(s), dt);
    if (!okr(t, "Tensor::empty")) return Tensor{};
    if (src) std::memcpy(t->data_ptr(), src, static_cast<size_t>(t->numel()) * dtype_size(dt));
    return *t;
}

void copy_out(const Tensor& t, void* dst) {
    auto c = t.contiguous();
    if (!okr(c, "contiguous")) return;
    std::memcpy(dst, c->data_ptr(), static_cast<size_t>(c->numel()) * dtype_size(c->dtype()));
}

template <typename F> double timed(int reps, F&& f) {
    std::vector<double> ts;
    for (int i = 0; i < std::max(reps, 1); ++i) {
        auto t0 = std::chrono::steady_clock::now();
        if (!f()) return -1.0;
        auto t1 = std::chrono::steady_clock::now();
        ts.push_back(std::chrono::duration<double>(t1 - t0).count());
    }
    std::sort(ts.begin(), ts.end());
    return ts[ts.size() / 2];
}

Tensor scalar_f32(float v) {
    auto t = Tensor::full({1}, DType::F32, static_cast<double>(v));
    okr(t, "Tensor::full");
    return t.has_value() ? *t : Tensor{};
}

// softmax over dim 1 of a 2-D fp32 tensor, from public ops.
Result<Tensor> softmax_rows(const Tensor& x) {
    auto m = max(x, 1, true);
    if (!m) return m;
    auto t = sub(x, *m);
    if (!t) return t;
    auto e = exp(*t);
    if (!e) return e;
    auto s = sum(*e, 1, true);
    if (!s) return s;
    return div(*e, *s);
}

}  // namespace

extern "C" {

int bref_threads(void) { return static_cast<int>(std::thread::hardware_concurrency()); }

// The SIMD level the reference's runtime dispatch picked on this host
// (Bee/SIMD/Detect.hpp:18-28).
const char* bref_isa(void) { return bee::simd::isa_name(bee::simd::current_isa()); }

double bref_matmul_f32(const float* a, const float* b, float* c, int64_t m, int64_t k, int64_t n, int reps) {
    Tensor A = make({m, k}, DType::F32, a), B = make({k, n}, DType::F32, b);
    Tensor C;
    double t = timed(reps, [&] {
        auto r = matmul(A, B);
        if (!okr(r, "matmul")) return false;
        C = *r;
        return true;
    });
    if (t >= 0) copy_out(C, c);
    return t;
}

// One step of the memory-bound sweep on the reference's CPU path: add, mul,
// row sum, row max, row softmax (the composition of public ops above) and the
// int32 full sum of [rows, cols] inputs.  The input Tensors are built on the
// first call for these pointers and kept, so a step times only the ops;
// seconds per op go to times[0..5] in that order; returns their total, or -1.
double bref_sweep(const float* x, const float* y, const int32_t* xi, int64_t rows, int64_t cols, double* times) {
    static const void* key[3] = {nullptr, nullptr, nullptr};
    static int64_t key_rows = -1, key_cols = -1;
    static Tensor X, Y, XI;
    if (key[0] != x || key[1] != y || key[2] != xi || key_rows != rows || key_cols != cols) {
        X = make({rows, cols}, DType::F32, x);
        Y = make({rows, cols}, DType::F32, y);
        XI = make({rows * cols}, DType::I32, xi);
        key[0] = x, key[1] = y, key[2] = xi, key_rows = rows, key_cols = cols;
    }
    auto clock = [](auto&& f) {
        auto t0 = std::chrono::steady_clock::now();
        const bool ok = f();
        auto t1 = std::chrono::steady_clock::now();
        return ok ? std::chrono::duration<double>(t1 - t0).count() : -1.0;
    };
    times[0] = clock([&] { return okr(add(X, Y), "add"); });
    times[1] = clock([&] { return okr(mul(X, Y), "mul"); });
    times[2] = clock([&] { return okr(sum(X, 1), "row sum"); });
    times[3] = clock([&] { return okr(max(X, 1), "row max"); });
    times[4] = clock([&] { return okr(softmax_rows(X), "softmax"); });
    times[5] = clock([&] { return okr(sum(XI), "int32 sum"); });
    double total = 0;
    for (int i = 0; i < 6; ++i) {
        if (times[i] < 0) return -1.0;
        total += times[i];
    }
    return total;
}

// op: 0 add, 1 sub, 2 mul, 3 div (same-shape fp32)
double bref_binary_f32(int op, const float* a, const float* b, float* out, int64_t rows, int64_t cols, int reps) {
    Tensor A = make({rows, cols}, DType::F32, a), B = make({rows, cols}, DType::F32, b);
    Tensor C;
    double t = timed(reps, [&] {
        auto r = op == 0 ? add(A, B) : op == 1 ? sub(A, B) : op == 2 ? mul(A, B) : div(A, B);
        if (!okr(r, "binary")) return false;
        C = *r;
        return true;
    });
    if (t >= 0) copy_out(C, out);
    return t;
}

// op: 0 sum, 1 min, 2 max over dim 1 of [rows, cols] fp32
double bref_reduce_rows_f32(int op, const float* x, float* out, int64_t rows, int64_t cols, int reps) {
    Tensor X = make({rows, cols}, DType::F32, x);
    Tensor R;
    double t = timed(reps, [&] {
        auto r = op == 0 ? sum(X, 1) : op == 1 ? min(X, 1) : max(X, 1);
        if (!okr(r, "reduce rows")) return false;
        R = *r;
        return true;
    });
    if (t >= 0) copy_out(R, out);
    return t;
}

// global sum / min / max of an int32 buffer (op as above)
double bref_reduce_global_i32(int op, const int32_t* x, int64_t n, int32_t* out, int reps) {
    Tensor X = make({n}, DType::I32, x);
    Tensor R;
    double t = timed(reps, [&] {
        auto r = op == 0 ? sum(X) : op == 1 ? min(X) : max(X);
        if (!okr(r, "reduce global")) return false;
        R = *r;
        return true;
    });
    if (t >= 0) copy_out(R, out);
    return t;
}

double bref_reduce_global_f32(int op, const float* x, int64_t n, float* out, int reps) {
    Tensor X = make({n}, DType::F32, x);
    Tensor R;
    double t = timed(reps, [&] {
        auto r = op == 0 ? sum(X) : op == 1 ? min(X) : max(X);
        if (!okr(r, "reduce global")) return false;
        R = *r;
        return true;
    });
    if (t >= 0) copy_out(R, out);
    return t;
}

double bref_softmax_f32(const float* x, float* y, int64_t rows, int64_t cols, int reps) {
    Tensor X = make({rows, cols}, DType::F32, x);
    Tensor Y;
    double t = timed(reps, [&] {
        auto r = softmax_rows(X);
        if (!okr(r, "softmax")) return false;
        Y = *r;
        return true;
    });
    if (t >= 0) copy_out(Y, y);
    return t;
}

// y = x / sqrt(mean(x*x, 1) + eps) * w
double bref_rms_norm_f32(const float* x, const float* w, float* y, int64_t rows, int64_t cols, float eps, int reps) {
    Tensor X = make({rows, cols}, DType::F32, x), W = make({cols}, DType::F32, w);
    Tensor E = scalar_f32(eps);
    Tensor Y;
    double t = timed(reps, [&] {
        auto sq = mul(X, X);
        if (!okr(sq, "mul")) return false;
        auto ms = mean(*sq, 1, true);
        if (!okr(ms, "mean")) return false;
        auto me = add(*ms, E);
        if (!okr(me, "add")) return false;
        auto d = sqrt(*me);
        if (!okr(d, "sqrt")) return false;
        auto xn = div(X, *d);
        if (!okr(xn, "div")) return false;
        auto r = mul(*xn, W);
        if (!okr(r, "mul w")) return false;
        Y = *r;
        return true;
    });
    if (t >= 0) copy_out(Y, y);
    return t;
}

// Rotate-half RoPE on x viewed [rows, heads, hd]; cos/sin tables are host
// doubles rounded to fp32, broadcast over heads as [rows, 1, hd/2].
double bref_rope_f32(const float* x, float* y, int64_t rows, int64_t seq, int64_t heads, int64_t hd, double theta,
                     int64_t pos_offset, int reps) {
    const int64_t half = hd / 2;
    std::vector<float> cosv(static_cast<size_t>(rows * half)), sinv(static_cast<size_t>(rows * half));
    for (int64_t r = 0; r < rows; ++r) {
        const double p = static_cast<double>(r % seq + pos_offset);
        for (int64_t i = 0; i < half; ++i) {
            const double f = std::pow(theta, -2.0 * static_cast<double>(i) / static_cast<double>(hd));
            cosv[static_cast<size_t>(r * half + i)] = static_cast<float>(std::cos(p * f));
            sinv[static_cast<size_t>(r * half + i)] = static_cast<float>(std::sin(p * f));
        }
    }
    Tensor X = make({rows, heads, hd}, DType::F32, x);
    Tensor C = make({rows, 1, half}, DType::F32, cosv.data()), S = make({rows, 1, half}, DType::F32, sinv.data());
    Tensor Y;
    double t = timed(reps, [&] {
        auto x1 = X.slice(2, 0, half);
        auto x2 = X.slice(2, half, hd);
        if (!okr(x1, "slice") || !okr(x2, "slice")) return false;
        auto a = mul(*x1, C), b = mul(*x2, S), c = mul(*x2, C), d = mul(*x1, S);
        if (!okr(a, "mul") || !okr(b, "mul") || !okr(c, "mul") || !okr(d, "mul")) return false;
        auto o1 = sub(*a, *b);
        auto o2 = add(*c, *d);
        if (!okr(o1, "sub") || !okr(o2, "add")) return false;
        auto out = Tensor::zeros({rows, heads, hd}, DType::F32);
        if (!okr(out, "zeros")) return false;
        auto y1 = out->slice(2, 0, half);
        auto y2 = out->slice(2, half, hd);
        if (!okr(y1, "slice") || !okr(y2, "slice")) return false;
        if (!okr(add_inplace(*y1, *o1), "add_inplace")) return false;
        if (!okr(add_inplace(*y2, *o2), "add_inplace")) return false;
        Y = *out;
        return true;
    });
    if (t >= 0) copy_out(Y, y);
    return t;
}

// Attention chain per head: S = Q K^T * scale, P = softmax(S), O = P V.
// q, k, v, o are [heads, seq, hd] fp32.
double bref_attention_f32(const float* q, const float* k, const float* v, float* o, int64_t heads, int64_t seq,
                          int64_t hd, float scale, int reps) {
    std::vector<Tensor> Q, K, V;
    for (int64_t h = 0; h < heads; ++h) {
        Q.push_back(make({seq, hd}, DType::F32, q + h * seq * hd));
        K.push_back(make({seq, hd}, DType::F32, k + h * seq * hd));
        V.push_back(make({seq, hd}, DType::F32, v + h * seq * hd));
    }
    Tensor Sc = scalar_f32(scale);
    std::vector<Tensor> O(static_cast<size_t>(heads));
    double t = timed(reps, [&] {
        for (int64_t h = 0; h < heads; ++h) {
            auto kt = K[static_cast<size_t>(h)].transpose(0, 1);
            if (!okr(kt, "transpose")) return false;
            auto ktc = kt->contiguous();
            if (!okr(ktc, "contiguous")) return false;
            auto s = matmul(Q[static_cast<size_t>(h)], *ktc);
            if (!okr(s, "matmul")) return false;
            auto ss = mul(*s, Sc);
            if (!okr(ss, "scale")) return false;
            auto p = softmax_rows(*ss);
            if (!okr(p, "softmax")) return false;
            auto oh = matmul(*p, V[static_cast<size_t>(h)]);
            if (!okr(oh, "matmul")) return false;
            O[static_cast<size_t>(h)] = *oh;
        }
        return true;
    });
    if (t >= 0)
        for (int64_t h = 0; h < heads; ++h) copy_out(O[static_cast<size_t>(h)], o + h * seq * hd);
    return t;
}


// permute(perm) then, for each dim d with step[d] > 0, slice(d, start[d],
// end[d], step[d]), then contiguous() — the reference's CPU view
// materialisation (Bee/Tensor/Core/Tensor.cpp:468-546) of an fp32 tensor.
double bref_view_copy_f32(const float* x, int ndim, const int64_t* shape, const int* perm, const int64_t* start,
                          const int64_t* end, const int64_t* step, float* out, int reps) {
    Shape s(shape, shape + ndim);
    Tensor t = make(s, DType::F32, x);
    Tensor res;
    double sec = timed(reps, [&] {
        auto v = t.permute(std::span<const int>(perm, static_cast<size_t>(ndim)));
        if (!okr(v, "permute")) return false;
        Tensor cur = *v;
        for (int d = 0; d < ndim; ++d) {
            if (step[d] <= 0) continue;
            auto sl = cur.slice(d, start[d], end[d], step[d]);
            if (!okr(sl, "slice")) return false;
            cur = *sl;
        }
        auto c = cur.contiguous();
        if (!okr(c, "contiguous")) return false;
        res = *c;
        return true;
    });
    if (sec >= 0) std::memcpy(out, res.data_ptr(), static_cast<size_t>(res.numel()) * sizeof(float));
    return sec;
}


// Broadcasting binary op on the reference's CPU path (Bee/Tensor/Ops/ElementWise.cpp,
// shapes aligned from the right as in Bee/Tensor/Ops/Broadcast.cpp); the
// output shape is the broadcast of a_shape and b_shape (both of rank ndim).
double bref_binary_bcast_f32(int op, const float* a, const int64_t* a_shape, const float* b, const int64_t* b_shape,
                             int ndim, float* out, int reps) {
    Tensor A = make(Shape(a_shape, a_shape + ndim), DType::F32, a);
    Tensor B = make(Shape(b_shape, b_shape + ndim), DType::F32, b);
    Tensor C;
    double t = timed(reps, [&] {
        auto r = op == 0 ? add(A, B) : op == 1 ? sub(A, B) : op == 2 ? mul(A, B) : div(A, B);
        if (!okr(r, "binary broadcast")) return false;
        C = *r;
        return true;
    });
    if (t >= 0) copy_out(C, out);
    return t;
}


// Integer mean over dim 1 of [outer, axis, inner] (axis < 0: global mean of
// all elements) on the reference's CPU path; out is F64.  dt: 2 I32, 3 I64.
double bref_mean_int(int dt, const void* x, int64_t outer, int64_t axis, int64_t inner, int global, double* out,
                     int reps) {
    Tensor X = make({outer, axis, inner}, dt == 2 ? DType::I32 : DType::I64, x);
    Tensor R;
    double t = timed(reps, [&] {
        auto r = global ? mean(X) : mean(X, 1);
        if (!okr(r, "mean")) return false;
        R = *r;
        return true;
    });
    if (t >= 0) copy_out(R, out);
    return t;
}

}  // extern "C"
