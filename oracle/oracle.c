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

/* ops::add / ops::mul, src/ops/elementwise_ops.cpp:44-52 -> binary_with_one_dnn, src/ops/one_dnn_utils.cpp:125-149:
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

/* ops::silu, src/ops/nn_ops.cpp:68-72: oneDNN eltwise_swish with alpha = 1, x / (1 + exp(-x)). */
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
 * the exactly rounded f32 of the double-precision sum instead. */
static float row_sum_squares(int dtype, const void* x, int64_t base, int64_t width, int chunk) {
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
                s = s + v * v;
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

/* ops::rms_norm, src/ops/nn_ops.cpp:164-225, per row of `width` elements:
 * mean = sum(x^2) / width (reduction_mean), var = mean + eps, rms = sqrt(var), inv = 1 / rms, n = x * inv,
 * r = n * w, stored in the input dtype. Row r of x starts at r * x_row_stride; y is dense. */
void oracle_rms_norm(int dtype, const void* x, int64_t x_row_stride, const void* w, void* y, int64_t rows,
                     int64_t width, float eps, int chunk) {
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; ++r) {
        const int64_t base = r * x_row_stride;
        const float ss = row_sum_squares(dtype, x, base, width, chunk);
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

/* ops::softmax_last_dim, src/ops/nn_ops.cpp:74-99 (oneDNN softmax_accurate in the input dtype, computed in f32):
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

/* ops::scaled_causal_softmax_last_dim, src/ops/nn_ops.cpp:133-159, f32 [matrices, Q, K]. */
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

/* Angles of src/nn/rope.cpp:85-103 laid out [positions][head_dim]: cos in [0, D/2), sin in [D/2, D). */
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

/* nn::apply_rope, src/nn/rope.cpp:73-124: rank-3 view [d0, d1, D] with element strides, sequence axis seq_dim,
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
        const float ss = row_sum_squares(dtype, src, base_idx, head_dim, chunk);
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
