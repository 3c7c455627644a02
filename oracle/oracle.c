/*
 * CPU oracle for the cppinf tensor-op hot path. TEST INFRASTRUCTURE ONLY: used by tests/, by the smoke check and by
 * bench.py's CPU-baseline leg as the checker. Nothing in the product path calls it.
 *
 * Each function restates one reference op (cited file:line in mscprojects/cppinf) in plain C, with f32 arithmetic
 * rounded after every operation (built with -ffp-contract=off, no FMA), as the reference's x86-64 build does.
 * Storage dtypes: 0 = bf16 (uint16 bit patterns), 1 = f32.
 *
 * Where the reference delegates to oneDNN (rms_norm's reduction_mean, softmax_accurate, eltwise_swish, binary,
 * reorder) the summation order and exp implementation are oneDNN's and unspecified. The oracle then fixes:
 *  - sums of squares (RMSNorm): the device library's canonical order (see oracle_rms_norm), so device results are
 *    compared bit for bit; oracle_rms_norm with chunk == 0 instead sums in double, an order-free value used to show
 *    that any f32 order stays within one bf16 ulp;
 *  - exp: glibc expf.
 * Parity pins: the reference's own golden vectors (tests/ops/ops_test.cpp, tests/nn/rope_test.cpp,
 * tests/nn/qwen_mlp_test.cpp, tests/tensors/tensor_test.cpp) and, for softmax/RoPE/add/mul/silu/cast, the reference
 * source itself compiled under oracle/_ref (see oracle/Makefile).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define DT_BF16 0
#define DT_F32 1

/* src/tensors/bfloat16.cpp:17-22 */
static inline float bf16_to_f32(uint16_t bits) {
    const uint32_t u = (uint32_t)bits << 16;
    float f;
    memcpy(&f, &u, sizeof f);
    return f;
}

/* src/tensors/bfloat16.cpp:8-15: round to nearest even via bits + 0x7fff + lsb. */
static inline uint16_t f32_to_bf16(float value) {
    uint32_t bits;
    memcpy(&bits, &value, sizeof bits);
    const uint32_t lsb = (bits >> 16) & 1u;
    bits += 0x7fffu + lsb;
    return (uint16_t)(bits >> 16);
}

/* ops::detail::load_float_value / store_float_value, src/ops/op_utils.h:28-43, 70-83 */
static inline float load(int dtype, const void* base, int64_t i) {
    if (dtype == DT_BF16) {
        return bf16_to_f32(((const uint16_t*)base)[i]);
    }
    return ((const float*)base)[i];
}

static inline void store(int dtype, void* base, int64_t i, float v) {
    if (dtype == DT_BF16) {
        ((uint16_t*)base)[i] = f32_to_bf16(v);
    } else {
        ((float*)base)[i] = v;
    }
}

/* The value a tensor of `dtype` holds after storing v. */
static inline float quantize(int dtype, float v) {
    return dtype == DT_BF16 ? bf16_to_f32(f32_to_bf16(v)) : v;
}

void oracle_f32_to_bf16(const float* x, uint16_t* y, int64_t n) {
    for (int64_t i = 0; i < n; ++i) {
        y[i] = f32_to_bf16(x[i]);
    }
}

void oracle_bf16_to_f32(const uint16_t* x, float* y, int64_t n) {
    for (int64_t i = 0; i < n; ++i) {
        y[i] = bf16_to_f32(x[i]);
    }
}

/* ops::cast, src/ops/tensor_ops.cpp:138-143 (oneDNN reorder: f32 <-> bf16 round to nearest even). */
void oracle_cast(int src_dtype, const void* x, int dst_dtype, void* y, int64_t n) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) {
        store(dst_dtype, y, i, load(src_dtype, x, i));
    }
}

/* ops::add / ops::mul, src/ops/elementwise_ops.cpp:28-36 -> binary_with_one_dnn, src/ops/one_dnn_utils.cpp:125-149:
 * inputs already in the output dtype, f32 arithmetic, result stored in the output dtype. */
void oracle_add(int dtype, const void* a, const void* b, void* out, int64_t n) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) {
        store(dtype, out, i, load(dtype, a, i) + load(dtype, b, i));
    }
}

void oracle_mul(int dtype, const void* a, const void* b, void* out, int64_t n) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) {
        store(dtype, out, i, load(dtype, a, i) * load(dtype, b, i));
    }
}

/* ops::silu, src/ops/nn_ops.cpp:44-48: oneDNN eltwise_swish with alpha = 1, x / (1 + exp(-x)). */
static inline float silu_f32(float x) {
    return x / (1.0f + expf(-x));
}

void oracle_silu(int dtype, const void* x, void* y, int64_t n) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) {
        store(dtype, y, i, silu_f32(load(dtype, x, i)));
    }
}

/* qwen_mlp's ops::mul(ops::silu(gate), up), src/nn/qwen_mlp.cpp:65-66: the silu tensor is stored in the model dtype
 * before the product (two roundings for bf16, as tests/nn/qwen_mlp_oracle.py:26-31 quantises after each op).
 *
 * `out_alt` (may be NULL) receives the result obtained with the other bf16 neighbour of silu(gate) whenever the f32
 * silu value lies within 2^-20 (relative) of a bf16 rounding boundary; elsewhere it equals `out`. exp
 * implementations differ by a few f32 ulps, so in that band the reference's rounding of the intermediate is not
 * determined by the formula alone, and either product is a faithful result. */
void oracle_silu_mul(int dtype, const void* gate, const void* up, void* out, void* out_alt, int64_t n) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) {
        const float s = silu_f32(load(dtype, gate, i));
        const float u = load(dtype, up, i);
        const float sq = quantize(dtype, s);
        store(dtype, out, i, sq * u);
        if (out_alt != NULL) {
            float alt = sq;
            if (dtype == DT_BF16) {
                const float lo = quantize(DT_BF16, (float)((double)s * (1.0 - 0x1p-20)));
                const float hi = quantize(DT_BF16, (float)((double)s * (1.0 + 0x1p-20)));
                alt = (lo != sq) ? lo : hi;
            }
            store(dtype, out_alt, i, alt * u);
        }
    }
}

/* Sum of squares of one row in the device library's canonical order: the row is cut into chunks of `chunk`
 * consecutive elements; lane l (0..31) sums, in increasing element order, chunks l, l+32, l+64, ...; the 32 partials
 * are combined by a butterfly over lane distances 16, 8, 4, 2, 1 (partial[l] + partial[l ^ d]). chunk == 0 returns
 * the exactly rounded f32 of the double-precision sum instead. `fused`: each step is fmaf(v, v, s), as every bf16
 * RMSNorm and q/k-norm kernel of the device library does (the square of a bf16 value is exact in f32 where it is
 * normal, |v| >= 2^-63, so the two forms differ only below that); otherwise (f32) a separately rounded product and
 * sum, as the reference's rms_norm. */
static float row_sum_squares(int dtype, const void* x, int64_t base, int64_t width, int chunk, int fused) {
    if (chunk == 0) {
        double acc = 0.0;
        for (int64_t e = 0; e < width; ++e) {
            const double v = load(dtype, x, base + e);
            acc += v * v;
        }
        return (float)acc;
    }
    float partial[32];
    float next[32];
    const int64_t nchunks = width / chunk;
    for (int lane = 0; lane < 32; ++lane) {
        float s = 0.0f;
        for (int64_t c = lane; c < nchunks; c += 32) {
            for (int j = 0; j < chunk; ++j) {
                const float v = load(dtype, x, base + c * chunk + j);
                s = fused ? fmaf(v, v, s) : s + v * v;
            }
        }
        partial[lane] = s;
    }
    for (int d = 16; d > 0; d >>= 1) {
        for (int lane = 0; lane < 32; ++lane) {
            next[lane] = partial[lane] + partial[lane ^ d];
        }
        memcpy(partial, next, sizeof partial);
    }
    return partial[0];
}

/* ops::rms_norm, src/ops/nn_ops.cpp:140-201, per row of `width` elements:
 * mean = sum(x^2) / width (reduction_mean), var = mean + eps, rms = sqrt(var), inv = 1 / rms, n = x * inv,
 * r = n * w, stored in the input dtype. Row r of x starts at r * x_row_stride; y is dense. */
void oracle_rms_norm(int dtype, const void* x, int64_t x_row_stride, const void* w, void* y, int64_t rows,
                     int64_t width, float eps, int chunk) {
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; ++r) {
        const int64_t base = r * x_row_stride;
        const float ss = row_sum_squares(dtype, x, base, width, chunk, dtype == DT_BF16);
        const float mean = ss / (float)width;
        const float var = mean + eps;
        const float rms = sqrtf(var);
        const float inv = 1.0f / rms;
        for (int64_t e = 0; e < width; ++e) {
            const float n = load(dtype, x, base + e) * inv;
            store(dtype, y, r * width + e, n * load(dtype, w, e));
        }
    }
}

/* ops::add then ops::rms_norm on the stored sum (src/nn/qwen_decoder_block.cpp:80-84). */
void oracle_add_rms_norm(int dtype, const void* a, const void* b, const void* w, void* sum, void* y, int64_t rows,
                         int64_t width, float eps, int chunk) {
    oracle_add(dtype, a, b, sum, rows * width);
    oracle_rms_norm(dtype, sum, width, w, y, rows, width, eps, chunk);
}

/* ops::softmax_last_dim, src/ops/nn_ops.cpp:50-75 (oneDNN softmax_accurate in the input dtype, computed in f32):
 * y = exp(x - max) / sum. oneDNN's summation order is unspecified; the oracle sums the f32 exponentials in double
 * and rounds once, the order-free value every f32 order approximates. */
void oracle_softmax_last_dim(int dtype, const void* x, void* y, int64_t rows, int64_t width) {
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; ++r) {
        const int64_t base = r * width;
        float m = -INFINITY;
        for (int64_t k = 0; k < width; ++k) {
            const float v = load(dtype, x, base + k);
            m = (m < v) ? v : m;
        }
        double acc = 0.0;
        for (int64_t k = 0; k < width; ++k) {
            acc += (double)expf(load(dtype, x, base + k) - m);
        }
        const float sum = (float)acc;
        for (int64_t k = 0; k < width; ++k) {
            store(dtype, y, base + k, expf(load(dtype, x, base + k) - m) / sum);
        }
    }
}

/* ops::scaled_causal_softmax_last_dim, src/ops/nn_ops.cpp:77-138, f32 [matrices, Q, K]. */
void oracle_scaled_causal_softmax(const float* x, float* y, int64_t matrices, int64_t query_len, int64_t key_len,
                                  float scale) {
#pragma omp parallel for schedule(dynamic, 16)
    for (int64_t row = 0; row < matrices * query_len; ++row) {
        const int64_t q = row % query_len;
        const int64_t off = row * key_len;
        float max_value = -INFINITY;
        for (int64_t k = 0; k <= q; ++k) {
            const float v = x[off + k] * scale;
            max_value = (max_value < v) ? v : max_value; /* std::max(max_value, v) */
        }
        float sum = 0.0f;
        for (int64_t k = 0; k < key_len; ++k) {
            const float v = k <= q ? expf(x[off + k] * scale - max_value) : 0.0f;
            y[off + k] = v;
            sum += v;
        }
        for (int64_t k = 0; k < key_len; ++k) {
            y[off + k] = y[off + k] / sum;
        }
    }
}

/* scaled_position_causal_softmax_last_dim, src/nn/qwen_attention.cpp:193-232, f32 [B, H, Qcap, Kcap]. Rows with
 * q >= query_lengths[b] keep the zero initialisation of the reference's result tensor. */
void oracle_position_causal_softmax(const float* x, float* y, int64_t batch, int64_t heads, int64_t query_cap,
                                    int64_t key_cap, float scale, const int64_t* query_offsets,
                                    const int64_t* query_lengths, const int64_t* key_lengths) {
#pragma omp parallel for schedule(dynamic, 16)
    for (int64_t row = 0; row < batch * heads * query_cap; ++row) {
        const int64_t q = row % query_cap;
        const int64_t b = row / query_cap / heads;
        const int64_t off = row * key_cap;
        if (q >= query_lengths[b]) {
            for (int64_t k = 0; k < key_cap; ++k) {
                y[off + k] = 0.0f;
            }
            continue;
        }
        const int64_t position = query_offsets[b] + q;
        float max_value = -INFINITY;
        for (int64_t k = 0; k < key_lengths[b]; ++k) {
            if (k <= position) {
                const float v = x[off + k] * scale;
                max_value = (max_value < v) ? v : max_value;
            }
        }
        float sum = 0.0f;
        for (int64_t k = 0; k < key_cap; ++k) {
            const int visible = k < key_lengths[b] && k <= position;
            const float v = visible ? expf(x[off + k] * scale - max_value) : 0.0f;
            y[off + k] = v;
            sum += v;
        }
        for (int64_t k = 0; k < key_cap; ++k) {
            y[off + k] = sum == 0.0f ? 0.0f : y[off + k] / sum;
        }
    }
}

/* Angles of src/nn/rope.cpp:70-74, 84-88 laid out [positions][head_dim]: cos in [0, D/2), sin in [D/2, D). */
void oracle_rope_table(float base, int64_t head_dim, int64_t positions, float* table) {
    const int64_t half = head_dim / 2;
    for (int64_t p = 0; p < positions; ++p) {
        for (int64_t i = 0; i < half; ++i) {
            const float inv_freq = powf(base, -(float)i / (float)half);
            const float angle = (float)p * inv_freq;
            table[p * head_dim + i] = cosf(angle);
            table[p * head_dim + half + i] = sinf(angle);
        }
    }
}

/* nn::apply_rope, src/nn/rope.cpp:58-109: rank-3 view [d0, d1, D] with element strides, sequence axis seq_dim,
 * positions from `offset`. f32 math, result stored in the input dtype (dense). */
void oracle_rope(int dtype, const void* x, int64_t d0, int64_t d1, int64_t head_dim, int64_t s0, int64_t s1,
                 int64_t s2, int64_t seq_dim, int64_t offset, float base, void* y) {
    const int64_t half = head_dim / 2;
    float inv_freq[4096];
    for (int64_t i = 0; i < half && i < 4096; ++i) {
        inv_freq[i] = powf(base, -(float)i / (float)half);
    }
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < d0 * d1; ++r) {
        const int64_t i0 = r / d1;
        const int64_t i1 = r % d1;
        const float position = (float)(offset + (seq_dim == 0 ? i0 : i1));
        for (int64_t i = 0; i < half; ++i) {
            const float angle = position * inv_freq[i];
            const float c = cosf(angle);
            const float s = sinf(angle);
            const float first = load(dtype, x, i0 * s0 + i1 * s1 + i * s2);
            const float second = load(dtype, x, i0 * s0 + i1 * s1 + (i + half) * s2);
            store(dtype, y, r * head_dim + i, first * c - second * s);
            store(dtype, y, r * head_dim + i + half, second * c + first * s);
        }
    }
}

/* The attention block's q/k path, src/nn/qwen_attention.cpp:383-390: ops::rms_norm per head vector (stored in the
 * model dtype), then RoPE at position offset + t. q [T, Hq, D], k [T, Hk, D] dense. `chunk` as in oracle_rms_norm. */
void oracle_qk_norm_rope(int dtype, const void* q, const void* k, const void* qw, const void* kw, void* q_out,
                         void* k_out, int64_t tokens, int64_t q_heads, int64_t k_heads, int64_t head_dim,
                         int64_t offset, float eps, float base, int chunk) {
    const int64_t half = head_dim / 2;
    float inv_freq[4096];
    for (int64_t i = 0; i < half && i < 4096; ++i) {
        inv_freq[i] = powf(base, -(float)i / (float)half);
    }
    const int64_t heads = q_heads + k_heads;
#pragma omp parallel for schedule(static)
    for (int64_t hv = 0; hv < tokens * heads; ++hv) {
        const int64_t t = hv / heads;
        const int64_t h = hv % heads;
        const void* src = h < q_heads ? q : k;
        void* dst = h < q_heads ? q_out : k_out;
        const void* w = h < q_heads ? qw : kw;
        const int64_t base_idx = h < q_heads ? (t * q_heads + h) * head_dim : (t * k_heads + (h - q_heads)) * head_dim;
        float normed[8192];
        const float ss = row_sum_squares(dtype, src, base_idx, head_dim, chunk, dtype == DT_BF16);
        const float mean = ss / (float)head_dim;
        const float var = mean + eps;
        const float rms = sqrtf(var);
        const float inv = 1.0f / rms;
        for (int64_t e = 0; e < head_dim && e < 8192; ++e) {
            normed[e] = quantize(dtype, (load(dtype, src, base_idx + e) * inv) * load(dtype, w, e));
        }
        const float position = (float)(offset + t);
        for (int64_t i = 0; i < half; ++i) {
            const float angle = position * inv_freq[i];
            const float c = cosf(angle);
            const float s = sinf(angle);
            const float first = normed[i];
            const float second = normed[i + half];
            store(dtype, dst, base_idx + i, first * c - second * s);
            store(dtype, dst, base_idx + i + half, second * c + first * s);
        }
    }
}

/* cli::detail::select_argmax_token_id, src/cli/cli_app.cpp:72-94, applied to each row. */
void oracle_row_argmax(int dtype, const void* x, int64_t rows, int64_t cols, int64_t row_stride, int64_t* out) {
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; ++r) {
        const int64_t base = r * row_stride;
        int64_t best_id = 0;
        float best = load(dtype, x, base);
        for (int64_t i = 1; i < cols; ++i) {
            const float v = load(dtype, x, base + i);
            if (v > best) {
                best = v;
                best_id = i;
            }
        }
        out[r] = best_id;
    }
}

/* x [rows, in] times weight [out, in] transposed, f32 accumulation in index order, stored in `dtype`: the
 * linear_project of src/nn/qwen_common.cpp:15-37 at golden-test sizes. */
void oracle_linear(int dtype, const void* x, const void* weight, void* y, int64_t rows, int64_t in, int64_t out) {
    for (int64_t r = 0; r < rows; ++r) {
        for (int64_t o = 0; o < out; ++o) {
            float acc = 0.0f;
            for (int64_t i = 0; i < in; ++i) {
                acc += load(dtype, x, r * in + i) * load(dtype, weight, o * in + i);
            }
            store(dtype, y, r * out + o, acc);
        }
    }
}

/* ==== Qwen3 decoder (src/nn/qwen_decoder_block.cpp, qwen_attention.cpp, qwen_mlp.cpp, models/qwen3) =============
 *
 * The reference runs its decoder through oneDNN matmul/eltwise primitives whose accumulation order and exp are
 * unspecified. The device decoder fixes both, and these functions restate exactly what it computes:
 *  - linear (src/nn/qwen_common.cpp:15-37, ops::matmul src/ops/matmul.cpp:85-114 with bf16 in and out): each output
 *    is a dot product in the canonical lane order (chunk 8 when K % 8 == 0, else 1; lane l adds chunks l, l+32, ...
 *    in increasing element order, starting from +0; butterfly over lane distances 16..1), rounded to bf16 once;
 *  - exp: the portable exponential below, in the attention softmax and in SiLU;
 *  - attention (qwen_attention.cpp:236-333 with the softmax of :164-235): the fixed partition order of
 *    oracle_decoder_attention.
 * Every product-accumulate of two bf16 values (a probability is a bf16 value too) is a fused multiply-add, fmaf,
 * as on the device (fma.rn.f32.bf16). The product has at most 16 significant bits, so in the f32 normal range it is
 * exact and the FMA equals `acc + a * b` with a separately rounded product; fmaf agrees with the device for every
 * operand, subnormal products included. */

/* Portable exp, written from the mathematics: Cody-Waite argument reduction x = n ln2 + r with ln2 split into a
 * 12-bit head (so n * head is exact for |n| <= 2^12) and an f32 tail, e^r by its Taylor polynomial to degree 7 in
 * Horner form (|r| <= ln2/2, truncation error below 6e-9 relative), then scaling by 2^n through the exponent field.
 * Every step is one IEEE f32 operation, so the device evaluates the same value bit for bit. */
#define PEXP_LOG2E 0x1.715476p+0f
#define PEXP_LN2_HI 0x1.62ep-1f
#define PEXP_LN2_LO 0x1.0bfbe8p-15f

static inline float pow2i(int e) { /* 2^e for -126 <= e <= 127 */
    const uint32_t bits = (uint32_t)(e + 127) << 23;
    float f;
    memcpy(&f, &bits, sizeof f);
    return f;
}

float oracle_pexp(float x) {
    if (x != x) {
        return x;
    }
    if (x > 88.8f) {
        return INFINITY;
    }
    if (x < -104.0f) {
        return 0.0f;
    }
    const float n = rintf(x * PEXP_LOG2E);
    const float r = (x - n * PEXP_LN2_HI) - n * PEXP_LN2_LO;
    float p = 0x1.a01a02p-13f;
    p = p * r + 0x1.6c16c2p-10f;
    p = p * r + 0x1.111112p-7f;
    p = p * r + 0x1.555556p-5f;
    p = p * r + 0x1.555556p-3f;
    p = p * r + 0.5f;
    p = p * r + 1.0f;
    p = p * r + 1.0f;
    int e = (int)n;
    if (e > 127) {
        p = p * 2.0f;
        e -= 1;
    }
    if (e < -126) {
        p = p * 0x1p-64f;
        e += 64;
    }
    return p * pow2i(e);
}

void oracle_pexp_array(const float* x, float* y, int64_t n) {
    for (int64_t i = 0; i < n; ++i) {
        y[i] = oracle_pexp(x[i]);
    }
}

/* SiLU (src/ops/nn_ops.cpp:44-48, x / (1 + exp(-x))) with the portable exp, stored in bf16, times up, stored in
 * bf16: the decoder's gate/up epilogue (src/nn/qwen_mlp.cpp:65-66). */
void oracle_silu_mul_pexp(const uint16_t* gate, const uint16_t* up, uint16_t* out, int64_t n) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) {
        const float g = bf16_to_f32(gate[i]);
        const float s = bf16_to_f32(f32_to_bf16(g / (1.0f + oracle_pexp(-g))));
        out[i] = f32_to_bf16(s * bf16_to_f32(up[i]));
    }
}

static void butterfly32(float* partial) {
    float next[32];
    for (int d = 16; d > 0; d >>= 1) {
        for (int lane = 0; lane < 32; ++lane) {
            next[lane] = partial[lane] + partial[lane ^ d];
        }
        memcpy(partial, next, sizeof next);
    }
}

/* y[m, n] = sum_k x[m, k] w[n, k] in the canonical lane order; x [M, K] with row stride x_stride, w [N, K] dense.
 * Results go to y_bf16 [M, N] (rounded once) and/or y_f32 [M, N] (unrounded) when non-null. Rows of x are processed
 * in blocks of 64 with the block transposed, so the inner loop runs over rows and vectorises. */
void oracle_linear_canonical(const uint16_t* x, int64_t x_stride, const uint16_t* w, int64_t M, int64_t K, int64_t N,
                             uint16_t* y_bf16, float* y_f32) {
    enum { MB = 64 };
    const int64_t chunk = K % 8 == 0 ? 8 : 1;
    const int64_t nchunks = K / chunk;
    if (M == 1) {
        float* xf = (float*)malloc(sizeof(float) * (size_t)K);
        for (int64_t k = 0; k < K; ++k) {
            xf[k] = bf16_to_f32(x[k]);
        }
#pragma omp parallel for schedule(static)
        for (int64_t n = 0; n < N; ++n) {
            float partial[32] = {0};
            const uint16_t* wr = w + n * K;
            for (int64_t c = 0; c < nchunks; ++c) {
                float a = partial[c & 31];
                for (int64_t e = c * chunk; e < (c + 1) * chunk; ++e) {
                    a = fmaf(xf[e], bf16_to_f32(wr[e]), a);
                }
                partial[c & 31] = a;
            }
            butterfly32(partial);
            if (y_bf16) {
                y_bf16[n] = f32_to_bf16(partial[0]);
            }
            if (y_f32) {
                y_f32[n] = partial[0];
            }
        }
        free(xf);
        return;
    }
    float* xt = (float*)malloc(sizeof(float) * (size_t)K * MB);
    for (int64_t m0 = 0; m0 < M; m0 += MB) {
        const int64_t mb = M - m0 < MB ? M - m0 : MB;
        for (int64_t k = 0; k < K; ++k) {
            for (int64_t mm = 0; mm < MB; ++mm) {
                xt[k * MB + mm] = mm < mb ? bf16_to_f32(x[(m0 + mm) * x_stride + k]) : 0.0f;
            }
        }
#pragma omp parallel for schedule(static)
        for (int64_t n = 0; n < N; ++n) {
            float acc[32][MB];
            memset(acc, 0, sizeof acc);
            const uint16_t* wr = w + n * K;
            for (int64_t c = 0; c < nchunks; ++c) {
                float* a = acc[c & 31];
                for (int64_t e = c * chunk; e < (c + 1) * chunk; ++e) {
                    const float wv = bf16_to_f32(wr[e]);
                    const float* xk = xt + e * MB;
                    for (int mm = 0; mm < MB; ++mm) {
                        a[mm] = fmaf(xk[mm], wv, a[mm]);
                    }
                }
            }
            for (int64_t mm = 0; mm < mb; ++mm) {
                float partial[32];
                for (int lane = 0; lane < 32; ++lane) {
                    partial[lane] = acc[lane][mm];
                }
                butterfly32(partial);
                if (y_bf16) {
                    y_bf16[(m0 + mm) * N + n] = f32_to_bf16(partial[0]);
                }
                if (y_f32) {
                    y_f32[(m0 + mm) * N + n] = partial[0];
                }
            }
        }
    }
    free(xt);
}

/* Causal grouped-query attention of one sequence in the device decoder's order. q [T, Hq, D] bf16 (after q-norm and
 * RoPE); key/value caches [cap, Hkv, D] bf16; query t sits at position pos0 + t and sees keys 0 .. pos0 + t; query
 * head h reads key/value head h / (Hq / Hkv) (ops::repeat_interleave, src/ops/tensor_ops.cpp). ctx [T, Hq, D] bf16.
 *
 * Per (t, h), with L visible keys:
 *  - score s_j: the head vector is cut into G segments of D / G consecutive dims (G = 8, 4, 2 or 1, the largest
 *    dividing D), each summed in order from +0, the G partials combined by a butterfly over distances G/2 .. 1;
 *  - x_j = s_j * scale, scale = 1 / sqrt(D) (qwen_attention.cpp:205-222 scales then takes the max);
 *  - the keys are split into 8 parts of P = ceil(L / 8) consecutive keys (part c: [cP, min(L, cP + P)));
 *  - part c: m_c = max of its x_j (-inf when empty); S_c: slot i (0..127) adds pexp(x_j - m_c) for j = lo + i,
 *    lo + i + 128, ... in order, slots 32w .. 32w+31 are combined by a butterfly, the 4 results added in order;
 *  - M = max_c m_c; sum = S_0 pexp(m_0 - M) + S_1 pexp(m_1 - M) + ... + S_7 pexp(m_7 - M), added in order;
 *  - p_j = bf16(pexp(x_j - M) / sum) (the probabilities' bf16 cast, qwen_attention.cpp:321-327);
 *  - ctx_d: in each part, group w (0..3) adds p_j v_jd for j = lo + w, lo + w + 4, ... in order; the 4 group sums,
 *    then the 8 part sums, are added in order; stored in bf16. */
void oracle_decoder_attention(const uint16_t* q, const uint16_t* kc, const uint16_t* vc, uint16_t* ctx, int64_t T,
                              int64_t hq, int64_t hkv, int64_t D, int64_t pos0) {
    enum { PARTS = 8, SLOTS = 128, WARPS = 4 };
    const float scale = 1.0f / sqrtf((float)D);
    const int64_t group = hq / hkv;
    const int64_t G = D % 8 == 0 ? 8 : D % 4 == 0 ? 4 : D % 2 == 0 ? 2 : 1;
    const int64_t seg = D / G;
#pragma omp parallel for schedule(dynamic)
    for (int64_t th = 0; th < T * hq; ++th) {
        const int64_t t = th / hq;
        const int64_t h = th % hq;
        const int64_t kvh = h / group;
        const int64_t L = pos0 + t + 1;
        const uint16_t* qv = q + (t * hq + h) * D;
        float* e = (float*)malloc(sizeof(float) * (size_t)L);
        float* acc = (float*)calloc((size_t)D, sizeof(float));
        float* grp = (float*)malloc(sizeof(float) * (size_t)D * WARPS);
        for (int64_t j = 0; j < L; ++j) {
            const uint16_t* kv = kc + (j * hkv + kvh) * D;
            float partial[8];
            for (int64_t g = 0; g < G; ++g) {
                float s = 0.0f;
                for (int64_t d = g * seg; d < (g + 1) * seg; ++d) {
                    s = fmaf(bf16_to_f32(qv[d]), bf16_to_f32(kv[d]), s);
                }
                partial[g] = s;
            }
            for (int64_t dist = G / 2; dist > 0; dist >>= 1) {
                float next[8];
                for (int64_t g = 0; g < G; ++g) {
                    next[g] = partial[g] + partial[g ^ dist];
                }
                memcpy(partial, next, sizeof next);
            }
            e[j] = partial[0] * scale;
        }
        const int64_t P = (L + PARTS - 1) / PARTS;
        float part_max[PARTS];
        float part_sum[PARTS];
        float mx = -INFINITY;
        for (int c = 0; c < PARTS; ++c) {
            const int64_t lo = c * P < L ? c * P : L;
            const int64_t hi = lo + P < L ? lo + P : L;
            float m = -INFINITY;
            for (int64_t j = lo; j < hi; ++j) {
                m = e[j] > m ? e[j] : m;
            }
            float slots[SLOTS];
            for (int i = 0; i < SLOTS; ++i) {
                float s = 0.0f;
                for (int64_t j = lo + i; j < hi; j += SLOTS) {
                    s = s + oracle_pexp(e[j] - m);
                }
                slots[i] = s;
            }
            float part = 0.0f;
            for (int w = 0; w < WARPS; ++w) {
                butterfly32(slots + 32 * w);
                part = w == 0 ? slots[0] : part + slots[32 * w];
            }
            part_max[c] = m;
            part_sum[c] = part;
            mx = m > mx ? m : mx;
        }
        float sum = 0.0f;
        for (int c = 0; c < PARTS; ++c) {
            const float term = part_sum[c] * oracle_pexp(part_max[c] - mx);
            sum = c == 0 ? term : sum + term;
        }
        for (int64_t j = 0; j < L; ++j) {
            e[j] = oracle_pexp(e[j] - mx);
        }
        for (int64_t j = 0; j < L; ++j) {
            e[j] = bf16_to_f32(f32_to_bf16(e[j] / sum));
        }
        for (int c = 0; c < PARTS; ++c) {
            const int64_t lo = c * P < L ? c * P : L;
            const int64_t hi = lo + P < L ? lo + P : L;
            for (int w = 0; w < WARPS; ++w) {
                float* a = grp + w * D;
                for (int64_t d = 0; d < D; ++d) {
                    a[d] = 0.0f;
                }
                for (int64_t j = lo + w; j < hi; j += WARPS) {
                    const uint16_t* vv = vc + (j * hkv + kvh) * D;
                    for (int64_t d = 0; d < D; ++d) {
                        a[d] = fmaf(e[j], bf16_to_f32(vv[d]), a[d]);
                    }
                }
            }
            for (int64_t d = 0; d < D; ++d) {
                float p = grp[d];
                for (int w = 1; w < WARPS; ++w) {
                    p = p + grp[w * D + d];
                }
                acc[d] = c == 0 ? p : acc[d] + p;
            }
        }
        for (int64_t d = 0; d < D; ++d) {
            ctx[(t * hq + h) * D + d] = f32_to_bf16(acc[d]);
        }
        free(e);
        free(acc);
        free(grp);
    }
}

/* ops::matmul (src/ops/matmul.cpp:85-114) in the device library's order for any operand types: lhs [batch, m, k]
 * and rhs [batch, k, n] with element strides (batch, row, column), every element read as f32 (bf16 widened
 * exactly), y[b, i, j] = sum_p lhs[b, i, p] rhs[b, p, j] in the canonical lane order (chunk 8 when k % 8 == 0, else
 * 1; lane l adds chunks l, l+32, ... in element order from +0; butterfly over lane distances 16..1), stored once in
 * y_dtype, y dense [batch, m, n]. Each step is a fused multiply-add when both operands are bf16 (their product is
 * exact in f32 in the normal range; the device fuses it too), else a separately rounded multiply and add. */
void oracle_matmul_canonical(int x_dtype, const void* x, const int64_t* xs, int w_dtype, const void* w,
                             const int64_t* ws, int y_dtype, void* y, int64_t batch, int64_t m, int64_t k,
                             int64_t n) {
    const int64_t chunk = k % 8 == 0 ? 8 : 1;
    const int64_t nchunks = k / chunk;
    const int fused = x_dtype == DT_BF16 && w_dtype == DT_BF16;
#pragma omp parallel for schedule(static)
    for (int64_t idx = 0; idx < batch * m * n; ++idx) {
        const int64_t b = idx / (m * n);
        const int64_t i = (idx / n) % m;
        const int64_t j = idx % n;
        float partial[32] = {0};
        for (int64_t c = 0; c < nchunks; ++c) {
            float a = partial[c & 31];
            for (int64_t e = c * chunk; e < (c + 1) * chunk; ++e) {
                const float xv = load(x_dtype, x, b * xs[0] + i * xs[1] + e * xs[2]);
                const float wv = load(w_dtype, w, b * ws[0] + e * ws[1] + j * ws[2]);
                a = fused ? fmaf(xv, wv, a) : a + xv * wv;
            }
            partial[c & 31] = a;
        }
        butterfly32(partial);
        store(y_dtype, y, idx, partial[0]);
    }
}
