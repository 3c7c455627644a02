/*
 * cppinf_b200 C ABI: sm_100a kernels for the elementwise, broadcast and row-reduction ops that the Qwen3 decoder of
 * cppinf calls (src/ops, src/nn/rope.cpp, the CLI argmax).
 *
 * Conventions shared by every entry point:
 *  - Pointers named x, y, out, ... are DEVICE pointers on the device that is current for the calling thread. Host
 *    pointers are accepted only where a parameter says "host".
 *  - Sizes are element counts (int64_t). Strides are in ELEMENTS, not bytes.
 *  - `stream` is a cudaStream_t cast to void*. NULL means the legacy default stream. Work is enqueued and the call
 *    returns without synchronising, so results are ready once the stream has reached that point.
 *  - Every call returns CPPINF_OK (0) or a negative cppinf_status. On failure cppinf_last_error() returns the
 *    message for the calling thread. The messages reuse the reference's validation texts where one exists.
 *  - No entry point allocates device memory and none falls back to the CPU.
 *  - Results are written to dense (contiguous) outputs. Outputs must not alias inputs unless the entry point says so.
 */
#ifndef CPPINF_B200_H
#define CPPINF_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define CPPINF_ABI_VERSION 1

/* Every entry point is exported from the shared library; everything else in it is hidden. */
#if defined(__GNUC__)
#define CPPINF_API __attribute__((visibility("default")))
#else
#define CPPINF_API
#endif

/* Element types, as in cppinf::tensors::DType (src/tensors/dtype.h:8-11). */
typedef enum cppinf_dtype {
    CPPINF_DTYPE_BF16 = 0,
    CPPINF_DTYPE_F32 = 1,
} cppinf_dtype;

/* Status codes. The first three mirror the exception types the reference throws from the same checks
 * (src/common/checked.cpp:10-49, src/ops/nn_ops.cpp:54-64). */
typedef enum cppinf_status {
    CPPINF_OK = 0,
    CPPINF_ERR_INVALID_ARGUMENT = -1, /* std::invalid_argument */
    CPPINF_ERR_OUT_OF_RANGE = -2,     /* std::out_of_range */
    CPPINF_ERR_OVERFLOW = -3,         /* std::overflow_error */
    CPPINF_ERR_UNSUPPORTED = -4,      /* a layout no device kernel handles, e.g. a misaligned vector operand */
    CPPINF_ERR_CUDA = -5,             /* a CUDA runtime call or kernel launch failed */
} cppinf_status;

/* Library metadata. */
CPPINF_API int cppinf_abi_version(void);
CPPINF_API const char* cppinf_last_error(void);
CPPINF_API const char* cppinf_status_name(int status);

/* Number of kernel launches this library has issued from any thread since load (for launch accounting). */
CPPINF_API uint64_t cppinf_launch_count(void);

/* ---------------------------------------------------------------------------------------------------------------
 * Elementwise ops.
 * ------------------------------------------------------------------------------------------------------------- */

/* ops::add, src/ops/elementwise_ops.h:10 (impl src/ops/elementwise_ops.cpp:44-47 -> one_dnn_utils.cpp:125-149).
 * out[i] = dtype(lhs[i] + rhs[i]) computed in f32, rounded to nearest-even for bf16. `out` may alias an input. */
CPPINF_API int cppinf_add(cppinf_dtype dtype, const void* lhs, const void* rhs, void* out, int64_t count, void* stream);

/* ops::mul, src/ops/elementwise_ops.h:14 (impl src/ops/elementwise_ops.cpp:49-52). Same rules as cppinf_add. */
CPPINF_API int cppinf_mul(cppinf_dtype dtype, const void* lhs, const void* rhs, void* out, int64_t count, void* stream);

/* ops::silu, src/ops/nn_ops.h:9 (impl src/ops/nn_ops.cpp:68-72, oneDNN eltwise_swish with alpha 1).
 * y[i] = dtype(x[i] / (1 + exp(-x[i]))). `y` may alias `x`. */
CPPINF_API int cppinf_silu(cppinf_dtype dtype, const void* x, void* y, int64_t count, void* stream);

/* ops::cast, src/ops/tensor_ops.h:15 (impl src/ops/tensor_ops.cpp:138-143 -> one_dnn_utils.cpp:94-105).
 * bf16 <-> f32 with round-to-nearest-even. src_dtype == dst_dtype is a copy. */
CPPINF_API int cppinf_cast(cppinf_dtype src_dtype, const void* x, cppinf_dtype dst_dtype, void* y, int64_t count, void* stream);

/* Fused ops::silu + ops::mul as the Qwen MLP calls them (src/nn/qwen_mlp.cpp:65-66).
 * out[i] = dtype(dtype(silu(gate[i])) * up[i]): the silu result is rounded to `dtype` before the product, exactly
 * like the two separate reference ops. */
CPPINF_API int cppinf_silu_mul(cppinf_dtype dtype, const void* gate, const void* up, void* out, int64_t count, void* stream);

/* Gather of a strided view of rank <= 8 into a dense buffer (the materialisation that
 * tensors::materialize_tensor, src/tensors/tensor_utils.h:83, and the strided loads of op_utils.h:45-68 imply).
 * `dims` and `strides` (elements) are HOST arrays of length `rank`. */
CPPINF_API int cppinf_strided_copy(cppinf_dtype dtype, const void* x, int64_t rank, const int64_t* dims, const int64_t* strides,
                        void* y, void* stream);

/* ---------------------------------------------------------------------------------------------------------------
 * Row reductions.
 * ------------------------------------------------------------------------------------------------------------- */

/* ops::rms_norm, src/ops/nn_ops.h:22 (impl src/ops/nn_ops.cpp:164-225) over rows of `width` elements.
 * y[r, i] = dtype((x[r, i] * (1 / sqrt(mean_i(x[r, i]^2) + eps))) * w[i]), all in f32.
 * Row r of x starts at x + r * x_row_stride; y is dense [rows, width]. Requires eps >= 0. */
CPPINF_API int cppinf_rms_norm(cppinf_dtype dtype, const void* x, int64_t x_row_stride, const void* weight, void* y,
                    int64_t rows, int64_t width, float eps, void* stream);

/* Residual add followed by RMSNorm, the pair the decoder block runs (src/nn/qwen_decoder_block.cpp:80-84, :89 and
 * the next layer's :73). sum = dtype(a + b) is written (it is the residual stream) and y = rms_norm(sum, w, eps).
 * All of a, b, sum, y are dense [rows, width]. `sum` may alias `a` or `b`. */
CPPINF_API int cppinf_add_rms_norm(cppinf_dtype dtype, const void* a, const void* b, const void* weight, void* sum, void* y,
                        int64_t rows, int64_t width, float eps, void* stream);

/* ops::softmax_last_dim, src/ops/nn_ops.h:13 (impl src/ops/nn_ops.cpp:74-99, oneDNN softmax_accurate).
 * Computed in f32, result rounded to `dtype`. x and y are dense [rows, width]. */
CPPINF_API int cppinf_softmax_last_dim(cppinf_dtype dtype, const void* x, void* y, int64_t rows, int64_t width, void* stream);

/* ops::scaled_causal_softmax_last_dim, src/ops/nn_ops.h:17 (impl src/ops/nn_ops.cpp:101-162).
 * x, y f32 dense [matrices, query_len, key_len] with query_len == key_len as the reference requires.
 * For row q: keys k <= q are visible, y = exp(x*scale - max) / sum over them, masked keys are written as 0. */
CPPINF_API int cppinf_scaled_causal_softmax_f32(const float* x, float* y, int64_t matrices, int64_t query_len, int64_t key_len,
                                     float scale, void* stream);

/* Position-aware variant used by attention, scaled_position_causal_softmax_last_dim
 * (src/nn/qwen_attention.cpp:164-235). x, y f32 dense [batch, heads, query_cap, key_cap].
 * query_offsets, query_lengths, key_lengths are HOST arrays of `batch` entries (batch <= 64).
 * Row (b, h, q) with q >= query_lengths[b] is written as zeros. Otherwise key k is visible when
 * k < key_lengths[b] and k <= query_offsets[b] + q, and a row with no visible key is all zeros. */
CPPINF_API int cppinf_scaled_position_causal_softmax_f32(const float* x, float* y, int64_t batch, int64_t heads,
                                              int64_t query_cap, int64_t key_cap, float scale,
                                              const int64_t* query_offsets, const int64_t* query_lengths,
                                              const int64_t* key_lengths, void* stream);

/* Row argmax, cli::detail::select_argmax_token_id (src/cli/cli_app.cpp:72-94) applied to every row.
 * out[r] = the lowest index of the largest value of row r, compared as f32. NaN is never selected, except that a
 * row whose element 0 is NaN yields 0 (the reference's strict '>' scan). Rows start at x + r * row_stride.
 * `out` is a device int64 array of `rows` entries. cols must be < 2^31. */
CPPINF_API int cppinf_row_argmax(cppinf_dtype dtype, const void* x, int64_t rows, int64_t cols, int64_t row_stride,
                      int64_t* out, void* stream);

/* ---------------------------------------------------------------------------------------------------------------
 * RoPE.
 * ------------------------------------------------------------------------------------------------------------- */

/* Host function: fills the HOST buffer `table` ([positions][head_dim] f32) with the split-half RoPE angles of
 * src/nn/rope.cpp:85-103: for pair i < head_dim/2 at position p,
 *   inv_freq[i] = powf(base, -(float)i / (float)(head_dim/2)), angle = (float)p * inv_freq[i],
 *   table[p][i] = cosf(angle), table[p][head_dim/2 + i] = sinf(angle).
 * The same libm calls the reference makes, so device results match it bit for bit. */
CPPINF_API int cppinf_rope_table(float base, int64_t head_dim, int64_t positions, float* table);

/* nn::apply_rope, src/nn/rope.h:12 (impl src/nn/rope.cpp:73-124) on a rank-3 view [dim0, dim1, head_dim] with
 * element strides (s0, s1, s2), sequence axis `seq_dim` (0 or 1), positions starting at `position_offset`.
 * `table` is a DEVICE copy of cppinf_rope_table(base, head_dim, >= position_offset + seq_len).
 * f32 math, result rounded to dtype; y is dense. */
CPPINF_API int cppinf_rope(cppinf_dtype dtype, const void* x, int64_t dim0, int64_t dim1, int64_t head_dim, int64_t s0,
                int64_t s1, int64_t s2, int64_t seq_dim, int64_t position_offset, const float* table,
                int64_t table_positions, void* y, void* stream);

/* Fused per-head q/k RMSNorm + RoPE, the sequence in src/nn/qwen_attention.cpp:383-390
 * (ops::rms_norm per head, result rounded to dtype, then apply_rope_batched at the token's position).
 * q: dense [tokens, q_heads, head_dim], k: dense [tokens, k_heads, head_dim], q_weight/k_weight: [head_dim].
 * Token t sits at position position_offset + t. q_out/k_out are dense and may alias q/k.
 * head_dim must be a multiple of 2 * (16 / element size) and at most 32 * (16 / element size). */
CPPINF_API int cppinf_qk_norm_rope(cppinf_dtype dtype, const void* q, const void* k, const void* q_weight,
                        const void* k_weight, void* q_out, void* k_out, int64_t tokens, int64_t q_heads,
                        int64_t k_heads, int64_t head_dim, int64_t position_offset, float eps, const float* table,
                        int64_t table_positions, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* CPPINF_B200_H */
