/*
 * bee_oracle.c — CPU restatement of the reference's Bee::Tensor compute path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker for the CUDA kernels:
 * only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may load
 * it, and never as the thing measured or shipped.
 *
 * Each function restates the reference algorithm it cites (paths relative to
 * the reference project).  Loop orders and accumulator types follow the
 * reference's scalar paths so that results agree to rounding; where the
 * reference has no op (softmax, RMSNorm, RoPE, attention, fp32->bf16 cast) the
 * function restates the composition of public ops a reference user would
 * write, and says so.  The compiled reference itself (oracle/_ref) pins these
 * functions in the CPU test suite.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* bf16 bits -> fp32 (exact). */
static inline float bf16_to_f32(uint16_t b) {
    uint32_t u = (uint32_t)b << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

/* fp32 -> bf16 bits, IEEE round-to-nearest-even on the bit pattern; NaN maps
 * to the canonical quiet NaN 0x7fff (sign dropped), matching cvt.rn.bf16.f32.
 * The reference's CPU cast to BF16 writes nothing (Bee/Tensor/Cpu/CastCpu.hpp:348),
 * so this is restated from the IEEE definition. */
static inline uint16_t f32_to_bf16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return 0x7fff;
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

void oracle_cast_f32_bf16(const float* x, uint16_t* y, int64_t n) {
    for (int64_t i = 0; i < n; ++i) y[i] = f32_to_bf16(x[i]);
}

void oracle_cast_bf16_f32(const uint16_t* x, float* y, int64_t n) {
    for (int64_t i = 0; i < n; ++i) y[i] = bf16_to_f32(x[i]);
}

/* C = A.B, row-major, fp32 accumulation in k order: the scalar reference GEMM
 * of Tests/Tensor/GemmTests.cpp:31-40 (i-j-k with a T accumulator). */
void oracle_matmul_f32(const float* A, const float* B, float* C, int64_t M, int64_t K, int64_t N) {
    /* i-k-j traversal with a row accumulator: each C[i][j] still sums its
     * products in k order, exactly as the i-j-k loop, but B is read by rows. */
    for (int64_t i = 0; i < M; ++i) {
        float* c = C + i * N;
        for (int64_t j = 0; j < N; ++j) c[j] = 0.0f;
        for (int64_t k = 0; k < K; ++k) {
            const float a = A[i * K + k];
            const float* b = B + k * N;
            for (int64_t j = 0; j < N; ++j) c[j] = c[j] + a * b[j];
        }
    }
}

/* Batched bf16 GEMM with fp32 math: C[b] = alpha * A[b] . op(B[b]), where
 * op(B) = B ([K,N]) or B^T (B stored [N,K] when b_trans).  Products of bf16
 * values are exact in fp32; accumulation is in double so the oracle is the
 * exactly-rounded fp32 result up to one rounding.  (The reference has no bf16
 * compute: Bee/Tensor/Core/DType.hpp:57-69; this is the fp32 matmul of the
 * bf16-rounded inputs.) */
void oracle_bmm_bf16(const uint16_t* A, const uint16_t* B, float* C, int64_t batch, int64_t M, int64_t K, int64_t N,
                     int b_trans, float alpha) {
    double* row = (double*)malloc((size_t)N * sizeof(double));
    float* bf = (float*)malloc((size_t)K * (size_t)N * sizeof(float));
    for (int64_t b = 0; b < batch; ++b) {
        const uint16_t* a = A + b * M * K;
        const uint16_t* bb = B + b * K * N;
        float* c = C + b * M * N;
        /* B as fp32 in [K, N] order (transposing when stored [N, K]) */
        for (int64_t k = 0; k < K; ++k)
            for (int64_t j = 0; j < N; ++j) bf[k * N + j] = bf16_to_f32(b_trans ? bb[j * K + k] : bb[k * N + j]);
        for (int64_t i = 0; i < M; ++i) {
            for (int64_t j = 0; j < N; ++j) row[j] = 0.0;
            for (int64_t k = 0; k < K; ++k) {
                const float av = bf16_to_f32(a[i * K + k]);
                const float* br = bf + k * N;
                for (int64_t j = 0; j < N; ++j) row[j] += (double)(av * br[j]);
            }
            for (int64_t j = 0; j < N; ++j) c[i * N + j] = (float)(row[j] * (double)alpha);
        }
    }
    free(bf);
    free(row);
}

/* Row reduce of [rows, cols] fp32 (op 0 sum, 1 min, 2 max), sequential fp32
 * accumulation: cpu_reduce_axis_dispatch's contiguous path
 * (Bee/Tensor/Cpu/ReduceCpu.hpp:496-506) with OpReduceSum/Min/Max scalars
 * (:177-250). */
void oracle_reduce_rows_f32(int op, const float* x, float* out, int64_t rows, int64_t cols) {
    for (int64_t r = 0; r < rows; ++r) {
        const float* p = x + r * cols;
        float acc = op == 0 ? 0.0f : op == 1 ? INFINITY : -INFINITY;
        if (op == 1) acc = 3.402823466e38f;
        if (op == 2) acc = -3.402823466e38f;
        for (int64_t k = 0; k < cols; ++k) {
            const float v = p[k];
            if (op == 0) acc = acc + v;
            else if (op == 1) acc = acc < v ? acc : v;
            else acc = acc > v ? acc : v;
        }
        out[r] = acc;
    }
}

/* Global int32 reduce (op 0 sum, 1 min, 2 max).  The reference accumulates in
 * int32 (OpReduceSum::scalar, Bee/Tensor/Cpu/ReduceCpu.hpp:190-193); the sum
 * is done in uint32 here so that wrap-around is defined, giving the same bits. */
int32_t oracle_reduce_global_i32(int op, const int32_t* x, int64_t n) {
    if (op == 0) {
        uint32_t acc = 0;
        for (int64_t i = 0; i < n; ++i) acc += (uint32_t)x[i];
        return (int32_t)acc;
    }
    int32_t acc = op == 1 ? INT32_MAX : INT32_MIN;
    for (int64_t i = 0; i < n; ++i) {
        if (op == 1) acc = acc < x[i] ? acc : x[i];
        else acc = acc > x[i] ? acc : x[i];
    }
    return acc;
}

/* Global fp32 sum, sequential fp32. */
float oracle_sum_f32(const float* x, int64_t n) {
    float acc = 0.0f;
    for (int64_t i = 0; i < n; ++i) acc += x[i];
    return acc;
}

/* Softmax over rows as the reference composition max(x,1,true) -> sub ->
 * exp -> sum(.,1,true) -> div: fp32 max and sequential fp32 sum
 * (ReduceCpu.hpp:496-506), exp through double then rounded to fp32
 * (OpExp::scalar, Bee/Tensor/Cpu/ElementWiseCpu.hpp:468-471), fp32 divide. */
void oracle_softmax_f32(const float* x, float* y, int64_t rows, int64_t cols) {
    for (int64_t r = 0; r < rows; ++r) {
        const float* p = x + r * cols;
        float* q = y + r * cols;
        float m = -3.402823466e38f;
        for (int64_t k = 0; k < cols; ++k) m = m > p[k] ? m : p[k];
        float s = 0.0f;
        for (int64_t k = 0; k < cols; ++k) {
            const float t = p[k] - m;
            q[k] = (float)exp((double)t);
            s += q[k];
        }
        for (int64_t k = 0; k < cols; ++k) q[k] = q[k] / s;
    }
}

/* RMSNorm as the composition mul(x,x) -> mean(.,1,true) -> add(eps) -> sqrt
 * -> div(x, .) -> mul(., w): the axis mean is the sequential fp32 sum divided
 * by (float)cols (Bee/Tensor/Ops/Reduce.cpp:331-335). */
void oracle_rms_norm_f32(const float* x, const float* w, float* y, int64_t rows, int64_t cols, float eps) {
    for (int64_t r = 0; r < rows; ++r) {
        const float* p = x + r * cols;
        float* q = y + r * cols;
        float s = 0.0f;
        for (int64_t k = 0; k < cols; ++k) s += p[k] * p[k];
        const float ms = s / (float)cols;
        const float d = sqrtf(ms + eps);
        for (int64_t k = 0; k < cols; ++k) q[k] = (p[k] / d) * w[k];
    }
}

/* Rotate-half RoPE on x viewed [rows, heads, hd] (position r % seq + offset):
 * the composition of slice views and mul/sub/add with host cos/sin tables
 * computed in double and rounded to fp32. */
void oracle_rope_f32(const float* x, float* y, int64_t rows, int64_t seq, int64_t heads, int64_t hd, double theta,
                     int64_t pos_offset) {
    const int64_t half = hd / 2;
    for (int64_t r = 0; r < rows; ++r) {
        const double p = (double)(r % seq + pos_offset);
        for (int64_t i = 0; i < half; ++i) {
            const double f = pow(theta, -2.0 * (double)i / (double)hd);
            const float c = (float)cos(p * f), s = (float)sin(p * f);
            for (int64_t h = 0; h < heads; ++h) {
                const float* xp = x + (r * heads + h) * hd;
                float* yp = y + (r * heads + h) * hd;
                const float x1 = xp[i], x2 = xp[i + half];
                const float a = x1 * c, b = x2 * s, cc = x2 * c, d = x1 * s;
                yp[i] = a - b;
                yp[i + half] = cc + d;
            }
        }
    }
}

/* Attention chain per head in fp32 from fp32 inputs: S = Q K^T * scale
 * (fp32 dot products in k order), row softmax as oracle_softmax_f32, O = P V. */
void oracle_attention_f32(const float* Q, const float* K, const float* V, float* O, int64_t heads, int64_t seq,
                          int64_t hd, float scale, float* work /* seq*seq floats */) {
    for (int64_t h = 0; h < heads; ++h) {
        const float* q = Q + h * seq * hd;
        const float* k = K + h * seq * hd;
        const float* v = V + h * seq * hd;
        float* o = O + h * seq * hd;
        for (int64_t i = 0; i < seq; ++i)
            for (int64_t j = 0; j < seq; ++j) {
                float acc = 0.0f;
                for (int64_t t = 0; t < hd; ++t) acc += q[i * hd + t] * k[j * hd + t];
                work[i * seq + j] = acc * scale;
            }
        oracle_softmax_f32(work, work, seq, seq);
        for (int64_t i = 0; i < seq; ++i)
            for (int64_t t = 0; t < hd; ++t) {
                float acc = 0.0f;
                for (int64_t j = 0; j < seq; ++j) acc += work[i * seq + j] * v[j * hd + t];
                o[i * hd + t] = acc;
            }
    }
}
