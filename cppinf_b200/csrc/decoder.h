// Internal interface of the decoder kernels (linear.cu, attention.cu) used by the model runtime (qwen3.cu) and by
// the C ABI entry points. Host and device share these parameter blocks; all pointers are device pointers.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <string>
#include <vector>

#include "cppinf_b200.h"

namespace cppinf::device {

// What a linear kernel does with each finished dot product (bf16-rounded once, as the reference's bf16 matmul
// result):
//  kStore     out segment k gets the value (rows [seg[k], seg[k+1]) of the weight matrix go to segment k);
//  kResidual  out0 = bf16(residual + value), the residual edge of src/nn/qwen_decoder_block.cpp:80-89;
//  kSiluMul   two weight matrices (gate, up): out0 = bf16(bf16(silu(gate)) * up), src/nn/qwen_mlp.cpp:61-66;
//  kArgmax    the greedy token of the row (src/cli/cli_app.cpp:72-94), optionally also storing the logits.
enum class LinearEpilogue : int { kStore = 0, kResidual = 1, kSiluMul = 2, kArgmax = 3 };

struct LinearParams {
    LinearEpilogue epilogue;
    // Input rows x[m, 0..K): x + m * x_stride, or, when `tokens` is set, the embedding row
    // x + tokens[token_base + m] * x_stride (token_base read from *position when `position` is set).
    const __nv_bfloat16* x;
    int64_t x_stride;
    const int64_t* tokens;
    int64_t vocab;             // rows of the embedding table (token ids are clamped into range on the device)
    __nv_bfloat16* x_copy;     // single-row kernel only: the raw input row is also stored here (residual stream)
    const __nv_bfloat16* norm_weight;  // single-row kernel only: x is RMS-normalised first (ops::rms_norm)
    float eps;

    const __nv_bfloat16* w0;   // [N, K] row-major ([out_features, in_features], the checkpoint layout)
    const __nv_bfloat16* w1;   // second [N, K] matrix for kSiluMul
    int64_t M;
    int64_t N;
    int64_t K;

    // Output segments: row n of the weights with seg[k] <= n < seg[k + 1] is stored at
    // out[k] + (m + row_offset[k]) * ld[k] + (n - seg[k]); segment 2's row offset adds *position when set.
    __nv_bfloat16* out[3];
    int64_t ld[3];
    int64_t seg[4];
    int64_t row_offset[3];
    const int* position;       // device sequence length (decode steps)

    const __nv_bfloat16* residual;  // kResidual: [M, N] with row stride res_ld
    int64_t res_ld;

    // kArgmax: tokens_out[*position + advance] = argmax over the row; *position += advance. `partial` holds one
    // 64-bit key per CTA and `counter` must be zero before the launch (the last CTA resets it).
    int64_t* tokens_out;
    int* position_out;
    int64_t advance;
    unsigned long long* partial;
    unsigned int* counter;

    // Single-row kernel only: when set, the CTA's slice of weight rows is staged in shared memory by bulk copies
    // issued before griddepcontrol.wait (if it fits), and a bounded wait that runs out sets *error to 1.
    unsigned int* error;
    uint32_t poll_limit = 1u << 24;  // polls of that wait (cppinf_set_wait_poll_limit)
};

// Single-row (decode) linear: one warp per output row at a time, the weights streamed once. Supports every
// epilogue, the embedding gather and the RMSNorm prologue. Requires K % 8 == 0 and 16-byte aligned rows.
cudaError_t launch_gemv(const LinearParams& p, cudaStream_t s);

// Grid the single-row kernel uses for `p` (the size the kArgmax scratch `partial` must have).
int gemv_grid(const LinearParams& p);

// Multi-row linear (prefill): tiles of up to 16 input rows staged in shared memory, kStore / kResidual / kSiluMul.
// Requires K % 8 == 0 and 16-byte aligned rows.
cudaError_t launch_linear_rows(const LinearParams& p, cudaStream_t s);

// Multi-row linear on the tensor cores (gemm_tc.cu: tcgen05, tolerance parity, not the restated order):
// kStore / kResidual / kSiluMul with N % 32 == 0, K % 8 == 0, segment starts multiples of 32, 16-byte aligned
// operands, no embedding gather, RMSNorm prologue or device position. cudaErrorNotSupported otherwise.
bool linear_tc_supported(const LinearParams& p);
cudaError_t launch_linear_tc(const LinearParams& p, cudaStream_t s);

struct AttentionParams {
    const __nv_bfloat16* q;        // [T, Hq, D]
    const __nv_bfloat16* k_cache;  // [cap, Hkv, D]
    const __nv_bfloat16* v_cache;  // [cap, Hkv, D]
    __nv_bfloat16* ctx;            // [T, Hq, D]
    int64_t T;
    int q_heads;
    int kv_heads;
    int head_dim;
    int64_t pos0;                  // position of query 0 (added to *position when set)
    const int* position;
    int64_t capacity;              // cache rows; queries past it are skipped
    // Decode steps (T = 1): when q_norm is set, q and k_new are the raw projections of the new token; the kernel
    // applies the per-head q/k RMSNorm + RoPE itself (rope.cu's arithmetic), writes the new key row to k_cache and
    // uses it for the last position.
    const __nv_bfloat16* k_new;    // [Hkv, D]
    const __nv_bfloat16* q_norm;
    const __nv_bfloat16* k_norm;
    const float* rope_table;       // [capacity, D]
    float eps;
    // Decode steps: when set (and the part's rows fit in shared memory), the cached key/value rows before the new
    // token are staged into shared memory by TMA tensor copies issued before griddepcontrol.wait (the sequence
    // length is then read before the wait too, so the preceding kernel must not write it); a bounded wait that runs
    // out sets *error to 1.
    unsigned int* error;
    int64_t queries_per_cluster = 1;  // consecutive queries one cluster takes in turn (prefill)
    uint32_t poll_limit = 1u << 24;   // polls of the staging wait (cppinf_set_wait_poll_limit)
    // Decode steps with the q|k|v projection fused in (when wqkv is set and decode_projection_fused() holds): the
    // kernel RMS-normalises the input row x (or, when `tokens` is set, the embedding row tokens[*position], which
    // it also copies to x_copy) with in_norm, and computes the new token's q, k and v rows from the fused
    // [(Hq + 2 Hkv) D, hidden] weight matrix itself; q and k_new above are then unused, and the v row is written to
    // v_cache at the position.
    const __nv_bfloat16* x = nullptr;
    const int64_t* tokens = nullptr;
    int64_t vocab = 0;
    __nv_bfloat16* x_copy = nullptr;
    const __nv_bfloat16* in_norm = nullptr;
    const __nv_bfloat16* wqkv = nullptr;
    int hidden = 0;
};

// Whether the decode attention can take the q|k|v projection of a model with these sizes (head_dim 64 or 128,
// hidden 256, 512 or 1024); otherwise the projection runs as its own kernel.
bool decode_projection_fused(int64_t head_dim, int64_t hidden, int64_t capacity);

// Causal GQA attention of one sequence in the fixed partition order (see attention.cu). head_dim 64, 128 or 256.
cudaError_t launch_decoder_attention(const AttentionParams& p, int64_t max_keys, cudaStream_t s);

// The same attention on the tensor cores for cached keys (attention_tc.cu: tcgen05, tolerance parity): head_dim 128,
// no device position, no fused q/k norm. cudaErrorNotSupported otherwise.
bool attention_tc_supported(const AttentionParams& p);
cudaError_t launch_attention_tc(const AttentionParams& p, cudaStream_t s);

// Embedding lookup (src/models/qwen3/qwen3_model.cpp:132-165): out[t] = table[tokens[t]], ids clamped into range.
cudaError_t launch_embedding(const __nv_bfloat16* table, int64_t vocab, int64_t hidden, const int64_t* tokens,
                             int64_t count, __nv_bfloat16* out, cudaStream_t s);

// Host side of the model (qwen3.cu): bytes of the named checkpoint tensor the model uses (-1 if it does not use it),
// and how many tensors it uses.
int64_t qwen3_tensor_bytes(const cppinf_qwen3* model, const std::string& name);

// The shape the model expects for a checkpoint tensor it uses ([rows, cols] or [size]); false if it does not use it.
bool qwen3_tensor_shape(const cppinf_qwen3* model, const std::string& name, std::vector<int64_t>* shape);
int64_t qwen3_shape_elements(const std::vector<int64_t>& shape);
int64_t qwen3_tensor_count(const cppinf_qwen3* model);

}  // namespace cppinf::device
