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
 *  - No entry point allocates device memory (except cppinf_qwen3_create, which allocates a model's weights, cache
 *    and workspace once) and none falls back to the CPU.
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
 * (src/common/checked.cpp:10-49, src/ops/nn_ops.cpp:30-40). */
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

/* Failure detection (no counterpart in the reference, whose ops run on the CPU). The decoder's kernels that stage
 * weights or cached rows by bulk copies wait on a shared-memory barrier for the copies to land; each such wait polls
 * at most `polls` times (default 2^24, far longer than any copy takes) before the kernel gives up, sets the model's
 * device error word (cppinf_qwen3_decode then returns CPPINF_ERR_CUDA) and, after a second wait with the default
 * limit that lets its copies land, exits without using the data.
 * The setting is process-wide and applies to kernels launched (or graphs captured) after the call; 0 makes every
 * first wait give up at once, which is how the tests exercise the error path without a fault. Returns the previous
 * limit. */
CPPINF_API uint32_t cppinf_set_wait_poll_limit(uint32_t polls);

/* ---------------------------------------------------------------------------------------------------------------
 * Elementwise ops.
 * ------------------------------------------------------------------------------------------------------------- */

/* ops::add, src/ops/elementwise_ops.h:10 (impl src/ops/elementwise_ops.cpp:28-31 -> one_dnn_utils.cpp:125-149).
 * out[i] = dtype(lhs[i] + rhs[i]) computed in f32, rounded to nearest-even for bf16. `out` may alias an input. */
CPPINF_API int cppinf_add(cppinf_dtype dtype, const void* lhs, const void* rhs, void* out, int64_t count, void* stream);

/* ops::mul, src/ops/elementwise_ops.h:14 (impl src/ops/elementwise_ops.cpp:33-36). Same rules as cppinf_add. */
CPPINF_API int cppinf_mul(cppinf_dtype dtype, const void* lhs, const void* rhs, void* out, int64_t count, void* stream);

/* ops::silu, src/ops/nn_ops.h:9 (impl src/ops/nn_ops.cpp:44-48, oneDNN eltwise_swish with alpha 1).
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

/* ops::rms_norm, src/ops/nn_ops.h:22 (impl src/ops/nn_ops.cpp:140-201) over rows of `width` elements.
 * y[r, i] = dtype((x[r, i] * (1 / sqrt(mean_i(x[r, i]^2) + eps))) * w[i]), all in f32.
 * Row r of x starts at x + r * x_row_stride; y is dense [rows, width]. Requires eps >= 0. */
CPPINF_API int cppinf_rms_norm(cppinf_dtype dtype, const void* x, int64_t x_row_stride, const void* weight, void* y,
                    int64_t rows, int64_t width, float eps, void* stream);

/* Residual add followed by RMSNorm, the pair the decoder block runs (src/nn/qwen_decoder_block.cpp:80-84, :89 and
 * the next layer's :73). sum = dtype(a + b) is written (it is the residual stream) and y = rms_norm(sum, w, eps).
 * All of a, b, sum, y are dense [rows, width]. `sum` may alias `a` or `b`. */
CPPINF_API int cppinf_add_rms_norm(cppinf_dtype dtype, const void* a, const void* b, const void* weight, void* sum, void* y,
                        int64_t rows, int64_t width, float eps, void* stream);

/* ops::softmax_last_dim, src/ops/nn_ops.h:13 (impl src/ops/nn_ops.cpp:50-75, oneDNN softmax_accurate).
 * Computed in f32, result rounded to `dtype`. x and y are dense [rows, width]. */
CPPINF_API int cppinf_softmax_last_dim(cppinf_dtype dtype, const void* x, void* y, int64_t rows, int64_t width, void* stream);

/* ops::scaled_causal_softmax_last_dim, src/ops/nn_ops.h:17 (impl src/ops/nn_ops.cpp:77-138).
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
 * src/nn/rope.cpp:70-74, 84-88: for pair i < head_dim/2 at position p,
 *   inv_freq[i] = powf(base, -(float)i / (float)(head_dim/2)), angle = (float)p * inv_freq[i],
 *   table[p][i] = cosf(angle), table[p][head_dim/2 + i] = sinf(angle).
 * The same libm calls the reference makes, so device results match it bit for bit. */
CPPINF_API int cppinf_rope_table(float base, int64_t head_dim, int64_t positions, float* table);

/* nn::apply_rope, src/nn/rope.h:12 (impl src/nn/rope.cpp:58-109) on a rank-3 view [dim0, dim1, head_dim] with
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

/* ---------------------------------------------------------------------------------------------------------------
 * Qwen3 decoder (bf16). Linear projections, attention and the model runtime on the device.
 *
 * Accumulation orders are fixed so that a CPU restatement reproduces every bit, and with it every greedy token:
 *  - linear: each output is a dot product whose in_features are cut into 16-byte chunks of 8; lane l (0..31) adds
 *    the products of chunks l, l+32, ... in element order starting from +0; the 32 partials are combined by a
 *    butterfly over lane distances 16..1; the sum is rounded to bf16 once. in_features must be a multiple of 8.
 *  - exp (softmax, SiLU): Cody-Waite reduction with a 12-bit ln2 head, degree-7 Taylor polynomial, exponent-field
 *    scaling, each step one IEEE f32 operation.
 *  - attention: see cppinf_decoder_attention.
 * The reference computes the same quantities through oneDNN, whose order is unspecified; these results agree with
 * it within a bf16 ulp per op, not bit for bit.
 * ------------------------------------------------------------------------------------------------------------- */

/* ops::matmul (src/ops/matmul.cpp:85-114, decl src/ops/matmul.h): y[b, i, j] = sum_p x[b, i, p] * w[b, p, j] for
 * x [batch, m, k] and w [batch, k, n] of any f32/bf16 types with element strides {batch, row, column} (HOST
 * arrays of 3), every element read as f32, the sum in the fixed lane order above (chunks of 8 when k % 8 == 0, of 1
 * otherwise), stored once in y_dtype; y dense [batch, m, n]. (The reference's dtype rules -- same-dtype inputs keep
 * it, bf16 inputs may ask for f32, mixed inputs give f32 -- are applied by its callers and by the C++ drop-in.)
 * bf16 operands with w the transposed view of a row-major [n, k] weight take the vector kernels; any other layout
 * a warp-per-output kernel with the same order. */
CPPINF_API int cppinf_matmul(cppinf_dtype x_dtype, const void* x, const int64_t* x_strides, cppinf_dtype w_dtype,
                             const void* w, const int64_t* w_strides, cppinf_dtype y_dtype, void* y, int64_t batch,
                             int64_t m, int64_t k, int64_t n, void* stream);

/* y[rows, out] = bf16(x[rows, in] * weight[out, in]^T): nn::detail::linear_project (src/nn/qwen_common.cpp:15-37)
 * over ops::matmul with bf16 operands and result (src/ops/matmul.cpp:85-114). Row r of x starts at r * x_row_stride;
 * y is dense. x, weight and x_row_stride * 2 bytes must be 16-byte aligned. */
CPPINF_API int cppinf_linear(const void* x, int64_t x_row_stride, const void* weight, void* y, int64_t rows,
                             int64_t in_features, int64_t out_features, void* stream);

/* y = bf16(residual + bf16(x * weight^T)): a projection followed by the residual ops::add of
 * src/nn/qwen_decoder_block.cpp:80-89. residual and y are dense [rows, out]; y may alias residual. */
CPPINF_API int cppinf_linear_residual(const void* x, int64_t x_row_stride, const void* weight, const void* residual,
                                      void* y, int64_t rows, int64_t in_features, int64_t out_features, void* stream);

/* y = bf16(bf16(silu(bf16(x * gate^T))) * bf16(x * up^T)): the gated MLP front of src/nn/qwen_mlp.cpp:58-66
 * (gate_proj, up_proj, ops::silu, ops::mul), fused. gate and up are [out, in]. */
CPPINF_API int cppinf_linear_silu_mul(const void* x, int64_t x_row_stride, const void* gate, const void* up, void* y,
                                      int64_t rows, int64_t in_features, int64_t out_features, void* stream);

/* The three projections above on the tensor cores (tcgen05.mma, TMA-staged tiles, f32 accumulation in tensor memory):
 * epilogue 0 = cppinf_linear (w1, residual unused), 1 = cppinf_linear_residual (y may alias residual),
 * 2 = cppinf_linear_silu_mul (w0 = gate, w1 = up). Opt-in: the accumulation order inside the tensor cores is not
 * the library's restated order, so results agree with cppinf_linear* to tolerance (a few bf16 ulps), not bit for
 * bit. Needs out_features % 32 == 0, in_features and x_row_stride % 8 == 0 and 16-byte aligned operands
 * (CPPINF_ERR_UNSUPPORTED otherwise). `error` (device, may be NULL) is set to 1 when a wait of the kernel ran out of
 * its poll limit (cppinf_set_wait_poll_limit). */
CPPINF_API int cppinf_linear_tc(int epilogue, const void* x, int64_t x_row_stride, const void* w0, const void* w1,
                                const void* residual, void* y, int64_t rows, int64_t in_features,
                                int64_t out_features, unsigned int* error, void* stream);

/* Greedy token of one logits row computed on the fly: out_token (DEVICE int64) = argmax over n of
 * bf16(x * weight[n]^T), the LM head of src/models/qwen3/qwen3_model.cpp:306-311 followed by
 * cli::detail::select_argmax_token_id (src/cli/cli_app.cpp:72-94: first maximum, NaN never selected unless at
 * index 0). x is one row [in]; if logits is non-NULL the bf16 logits [out] are stored too. Needs a DEVICE
 * scratch of cppinf_linear_argmax_scratch_bytes(out, in) bytes, 16-byte aligned, whose first 16 bytes are zero
 * before the first call (each call leaves them zero again); calls sharing a scratch must not overlap. */
CPPINF_API int cppinf_linear_argmax(const void* x, const void* weight, void* logits, int64_t in_features,
                                    int64_t out_features, int64_t* out_token, void* scratch, void* stream);
CPPINF_API int64_t cppinf_linear_argmax_scratch_bytes(int64_t out_features, int64_t in_features);

/* cppinf_linear_argmax without a caller-provided scratch, for callers that cannot allocate device memory: hosts
 * whose allocator owns the whole device budget (a framework's caching allocator, a fixed memory plan) and FFI
 * bindings that have no way to obtain a device buffer. The per-CTA maxima and the arrival counter live in a static
 * device array of this library (one per device, held until the process exits, zero-filled when the module loads;
 * every call leaves the counter at zero again). Nothing is allocated. The first call on a device looks up the array's
 * device address (cudaGetSymbolAddress) with that device current; make that first call before any stream capture.
 * This entry point has no counterpart in the reference (its CLI argmax runs on host logits and needs no scratch). Limits: the launch must fit the static scratch (1024 CTAs,
 * 8208 bytes; CPPINF_ERR_UNSUPPORTED with the sizes in the message otherwise). Calls on one device share the
 * scratch, so two calls that overlap in time -- on different streams, or from different threads without ordering
 * -- race and may return a wrong token; issue them on one stream or synchronise between them. */
CPPINF_API int cppinf_linear_argmax_noalloc(const void* x, const void* weight, void* logits, int64_t in_features,
                                            int64_t out_features, int64_t* out_token, void* stream);

/* Causal grouped-query attention of one sequence over its KV cache: fused_causal_attention of
 * src/nn/qwen_attention.cpp:236-333 with the position-causal softmax of :164-235. q [tokens, q_heads, head_dim]
 * (after q-norm and RoPE), k_cache/v_cache [capacity, kv_heads, head_dim], ctx [tokens, q_heads, head_dim], all
 * bf16. Query t sits at position `position` + t and sees keys 0 .. position + t; query head h reads kv head
 * h / (q_heads / kv_heads). Scores in f32, probabilities rounded to bf16, context rounded to bf16.
 * Order: per (query, head) the visible keys are split into 8 parts of ceil(L/8); score dot products in 8 segments
 * of head_dim/8 dims combined by a butterfly; parts, warps and slots summed in the fixed order of
 * oracle_decoder_attention. head_dim 64, 128 or 256; position + tokens <= capacity. */
CPPINF_API int cppinf_decoder_attention(const void* q, const void* k_cache, const void* v_cache, void* ctx,
                                        int64_t tokens, int64_t q_heads, int64_t kv_heads, int64_t head_dim,
                                        int64_t position, int64_t capacity, void* stream);

/* cppinf_decoder_attention on the tensor cores (tcgen05: S = Q K^T and P V as UMMAs with tensor-memory accumulators,
 * the causal softmax with bf16 probabilities in between), for head_dim 128. Opt-in, like cppinf_linear_tc: contexts
 * agree with cppinf_decoder_attention to tolerance (the running softmax sum and the tensor cores' accumulation order
 * are not the restated order), not bit for bit. `error` (device, may be NULL) is set to 1 when a wait of the kernel
 * ran out of its poll limit (cppinf_set_wait_poll_limit). No counterpart in the reference beyond the attention it
 * computes (src/nn/qwen_attention.cpp:237-333). */
CPPINF_API int cppinf_decoder_attention_tc(const void* q, const void* k_cache, const void* v_cache, void* ctx,
                                           int64_t tokens, int64_t q_heads, int64_t kv_heads, int64_t head_dim,
                                           int64_t position, int64_t capacity, unsigned int* error, void* stream);

/* Embedding lookup (src/models/qwen3/qwen3_model.cpp:132-165): out[t] = table[token_ids[t]], table [vocab, hidden]
 * bf16, token_ids a DEVICE int64 array. Ids are validated on the host by the model; here they are clamped into
 * range. hidden must be a multiple of 8. */
CPPINF_API int cppinf_embedding(const void* table, int64_t vocab, int64_t hidden, const int64_t* token_ids,
                                int64_t count, void* out, void* stream);

/* The Qwen3 model (src/models/qwen3/qwen3_model.h): tied embeddings, bf16 weights, one cached sequence. */
typedef struct cppinf_qwen3_config {
    int64_t vocab_size;
    int64_t hidden_size;
    int64_t intermediate_size;
    int64_t num_hidden_layers;
    int64_t num_attention_heads;
    int64_t num_key_value_heads;
    int64_t head_dim;
    float rms_norm_eps;
    float rope_theta;
} cppinf_qwen3_config;

typedef struct cppinf_qwen3 cppinf_qwen3;

/* Creates a model on the current device with room for `max_sequence_length` cached tokens (make_cache,
 * qwen3_model.cpp:222-245). Weights start zeroed; load them with cppinf_qwen3_set_weight. Validation follows
 * validate_model_config (qwen3_model.cpp:44-61): hidden and intermediate sizes multiples of 8, head_dim 64/128/256,
 * query heads a multiple of key-value heads. */
CPPINF_API int cppinf_qwen3_create(const cppinf_qwen3_config* config, int64_t max_sequence_length,
                                   cppinf_qwen3** model);
CPPINF_API void cppinf_qwen3_destroy(cppinf_qwen3* model);

/* Copies one checkpoint tensor (Hugging Face name, e.g. "model.layers.3.mlp.up_proj.weight", bf16, exactly the
 * tensor's bytes) from `data` (HOST memory when on_device == 0, DEVICE memory otherwise) into the model. */
CPPINF_API int cppinf_qwen3_set_weight(cppinf_qwen3* model, const char* name, const void* data, int64_t bytes,
                                       int on_device);

/* Loads a safetensors checkpoint (the format of src/files/safetensors_file.cpp: 8-byte little-endian header length,
 * JSON header of {dtype, shape, data_offsets} per tensor, tensor bytes) into the model: the file is memory-mapped and
 * each tensor the model uses is copied from the mapping to its device slot, so no host copy of the file is made.
 * The header is checked as the reference does (same messages); every tensor the model uses must be present and bf16
 * (validate_required_tensors, qwen3_model.cpp:63-90); tensors it does not use are skipped. `loaded` (HOST, may be
 * NULL) receives the number of tensors copied. */
CPPINF_API int cppinf_qwen3_load_safetensors(cppinf_qwen3* model, const char* path, int64_t* loaded);

/* Host-only check of a safetensors file's header (the same parse and checks as cppinf_qwen3_load_safetensors):
 * number of tensors and byte offset of the tensor data. */
CPPINF_API int cppinf_safetensors_info(const char* path, int64_t* tensor_count, int64_t* data_offset);

/* Qwen3Model::forward_cached (qwen3_model.cpp:275-311): appends `count` HOST token ids to the cached sequence.
 * logits (DEVICE bf16, may be NULL) receives [count, vocab] when all_rows != 0, else the last row [vocab].
 * next_token (HOST, may be NULL) receives the greedy token of the last row (cli_app.cpp:72-94); the call then
 * synchronises `stream`. */
CPPINF_API int cppinf_qwen3_forward(cppinf_qwen3* model, const int64_t* token_ids, int64_t count, void* logits,
                                    int all_rows, int64_t* next_token, void* stream);

/* Greedy decoding from the cached state: `steps` decode steps, each feeding the previous greedy token (the last
 * cppinf_qwen3_forward's, then each step's own). Writes the `steps` generated tokens to the HOST array `tokens` and
 * synchronises `stream`. One step is a captured CUDA graph of the whole decoder (the device-side sequence length
 * selects the cache row, the rotary position and the input token). Returns CPPINF_ERR_CUDA when a device wait ran
 * out of its poll limit (cppinf_set_wait_poll_limit); the model then refuses forward/decode until
 * cppinf_qwen3_reset. The step graph is captured again when the poll limit has changed since its capture. */
CPPINF_API int cppinf_qwen3_decode(cppinf_qwen3* model, int64_t steps, int64_t* tokens, void* stream);

/* A batch of cached sequences: Qwen3Model::make_cache(batch_size, max_sequence_length) (qwen3_model.cpp:222-245),
 * per layer and sequence a K and a V cache [capacity, kv_heads, head_dim] in device memory, every length 0.
 * `capacity` may not exceed the model's max_sequence_length. Independent of the model's own cached sequence. */
typedef struct cppinf_qwen3_cache cppinf_qwen3_cache;
CPPINF_API int cppinf_qwen3_cache_create(const cppinf_qwen3* model, int64_t batch, int64_t capacity,
                                         cppinf_qwen3_cache** cache);
CPPINF_API void cppinf_qwen3_cache_destroy(cppinf_qwen3_cache* cache);
CPPINF_API int64_t cppinf_qwen3_cache_batch(const cppinf_qwen3_cache* cache);
/* Qwen3Cache::sequence_lengths: `lengths` (HOST, cppinf_qwen3_cache_batch entries). */
CPPINF_API int cppinf_qwen3_cache_lengths(const cppinf_qwen3_cache* cache, int64_t* lengths);

/* Qwen3Model::forward_cached(const TokenIdBatch&, Qwen3Cache&) (qwen3_model.cpp:275-311, the right-padded packing of
 * pack_token_id_batch :104-130): sequence b appends its lengths[b] HOST token ids token_ids[b * max_length ..] to
 * its cached rows. logits (DEVICE bf16 [batch, max_length, vocab]) receives each sequence's rows; right-padded rows
 * are set to zero. Every row equals, bit for bit, the same row of a forward of that sequence alone (the reference's
 * mixed-length batch test, qwen3_model_test.cpp:459-486): the projections and the MLP run over the rows of all
 * sequences at once, the q/k norm + RoPE, cache appends and attention per sequence. Errors follow the reference
 * (empty batch, empty sequence, cache batch mismatch, cache too small, token out of range). */
CPPINF_API int cppinf_qwen3_forward_batch(cppinf_qwen3* model, cppinf_qwen3_cache* cache, const int64_t* token_ids,
                                          const int64_t* lengths, int64_t batch, int64_t max_length, void* logits,
                                          void* stream);

/* Forgets the cached sequence (a fresh make_cache) and clears a device error reported by cppinf_qwen3_decode. */
CPPINF_API int cppinf_qwen3_reset(cppinf_qwen3* model, void* stream);

/* Projections of prompt rows (cppinf_qwen3_forward): mode 0 (default) runs them on the CUDA cores in the library's
 * restated accumulation order, so logits and greedy tokens equal the CPU oracle's bit for bit; mode 1 runs the
 * eligible ones on the tensor cores (cppinf_linear_tc), several times faster, with logits that agree to tolerance.
 * Decode steps are unaffected. No counterpart in the reference (its matmul is one oneDNN path). */
CPPINF_API int cppinf_qwen3_set_prefill(cppinf_qwen3* model, int mode);

/* Number of cached tokens. */
CPPINF_API int64_t cppinf_qwen3_length(const cppinf_qwen3* model);

/* Kernel launches of one decode step (for launch accounting). */
CPPINF_API int64_t cppinf_qwen3_step_launches(const cppinf_qwen3* model);

#ifdef __cplusplus
}
#endif

#endif /* CPPINF_B200_H */
