// The Qwen3 model on one device: weights, KV cache and activations resident in HBM, the decoder of
// src/models/qwen3/qwen3_model.cpp:275-311 and src/nn/qwen_decoder_block.cpp:65-90 issued as device kernels.
//
// Layout in HBM (one allocation each, every tensor 256-byte aligned):
//  - weights: per layer the norms, q|k|v projections concatenated into one [(Hq + 2 Hkv) D, H] matrix, o_proj,
//    gate_proj, up_proj, down_proj (checkpoint row-major layout), then the tied embedding and the final norm;
//  - cache: per layer K [cap, Hkv, D] and V [cap, Hkv, D] (src/nn/qwen_cache.cpp's layout, batch 1);
//  - state: the device-side sequence length and the token history tokens[0 .. cap], where tokens[len] is the next
//    input; workspace for up to 512 prompt rows.
//
// forward(): prompt rows in chunks of up to 512 -- embedding gather, then per layer rms_norm, the multi-row q|k|v
// projection (v rows written straight into the cache), fused q/k-norm + RoPE (k rows into the cache), attention,
// o_proj with the residual add, rms_norm, gate/up with SiLU * up, down_proj with the residual add -- and finally
// the last row's final norm + LM head + argmax in one kernel.
// decode(): one step is 4 kernels per layer + 1 (attention with the input norm, the q|k|v projection -- in layer 0
// after the embedding gather -- and the q/k-norm + RoPE of the new token fused in; o_proj + residual; gate/up with
// the post-attention norm and SiLU * up; down_proj + residual; final norm + LM head + argmax), captured once as a
// CUDA graph. Sizes the fused attention does not take (decode_projection_fused) run the projection as a fifth kernel
// per layer. Every kernel reads the sequence length from device memory, and the last one advances it, so the same
// graphs are replayed for every step: one of eight consecutive steps (no graph-launch gap between them) and one of a
// single step for the remainder.
#include <cstring>
#include <optional>
#include <string>
#include <vector>

#include "cppinf_b200.h"
#include "decoder.h"
#include "runtime.h"

namespace rt = cppinf::runtime;
using cppinf::device::AttentionParams;
using cppinf::device::LinearEpilogue;
using cppinf::device::LinearParams;
using bf16 = __nv_bfloat16;

namespace {

constexpr int64_t kChunkRows = 512;
constexpr std::size_t kAlign = 256;

std::size_t align_up(std::size_t v) {
    return (v + kAlign - 1) / kAlign * kAlign;
}

struct Layer {
    bf16* in_norm;
    bf16* post_norm;
    bf16* q_norm;
    bf16* k_norm;
    bf16* wqkv;
    bf16* wo;
    bf16* wg;
    bf16* wu;
    bf16* wd;
    bf16* k_cache;
    bf16* v_cache;
};

}  // namespace

struct cppinf_qwen3 {
    cppinf_qwen3_config c{};
    int64_t cap = 0;
    int64_t q_dim = 0;
    int64_t kv_dim = 0;
    int64_t qkv_rows = 0;
    char* weights = nullptr;
    std::size_t weight_bytes = 0;
    char* cache = nullptr;
    std::size_t cache_bytes = 0;
    char* work = nullptr;
    std::vector<Layer> layers;
    bf16* embed = nullptr;
    bf16* final_norm = nullptr;
    float* rope = nullptr;
    int* d_len = nullptr;
    int64_t* d_tokens = nullptr;
    unsigned int* d_counter = nullptr;
    unsigned int* d_error = nullptr;  // set by a decode kernel whose bounded wait ran out
    unsigned long long* d_partial = nullptr;
    bf16* h = nullptr;
    bf16* xn = nullptr;
    bf16* q = nullptr;
    bf16* k = nullptr;
    bf16* qr = nullptr;
    bf16* ctx = nullptr;
    bf16* act = nullptr;
    int64_t len = 0;
    cudaGraphExec_t step = nullptr;
    int64_t step_launches = 0;
    cudaGraphExec_t step_block = nullptr;  // kBlockSteps steps in one graph
    int64_t step_block_launches = 0;
    uint32_t step_poll_limit = 0;  // the wait poll limit the decode-step graph was captured with
    int prefill_mode = 0;          // 0: CUDA-core projections (restated order), 1: tensor cores (tolerance parity)
    bool failed = false;           // a decode step reported a device error; cleared by cppinf_qwen3_reset
};

namespace {

#define QWEN3_TRY(expr, name)                                        \
    do {                                                             \
        const cudaError_t qwen3_err_ = (expr);                       \
        const int qwen3_st_ = rt::launched(qwen3_err_, (name));      \
        if (qwen3_st_ != CPPINF_OK) {                                \
            return qwen3_st_;                                        \
        }                                                            \
    } while (0)

#define QWEN3_CHECK(call)                                            \
    do {                                                             \
        const int qwen3_st_ = (call);                                \
        if (qwen3_st_ != CPPINF_OK) {                                \
            return qwen3_st_;                                        \
        }                                                            \
    } while (0)

LinearParams params_for(LinearEpilogue epi, const bf16* x, int64_t x_stride, const bf16* w0, const bf16* w1,
                        int64_t rows, int64_t n, int64_t k) {
    LinearParams p{};
    p.epilogue = epi;
    p.x = x;
    p.x_stride = x_stride;
    p.w0 = w0;
    p.w1 = w1;
    p.M = rows;
    p.N = n;
    p.K = k;
    p.seg[0] = 0;
    p.seg[1] = p.seg[2] = p.seg[3] = n;
    p.poll_limit = rt::wait_poll_limit();
    return p;
}

// The q|k|v projection: q rows to q, k rows to k, v rows into the cache at row (m + row0 [+ *position]).
void set_qkv_outputs(const cppinf_qwen3* m, const Layer& l, LinearParams& p, int64_t row0, const int* position) {
    p.out[0] = m->q;
    p.out[1] = m->k;
    p.out[2] = l.v_cache;
    p.ld[0] = m->q_dim;
    p.ld[1] = m->kv_dim;
    p.ld[2] = m->kv_dim;
    p.seg[0] = 0;
    p.seg[1] = m->q_dim;
    p.seg[2] = m->q_dim + m->kv_dim;
    p.seg[3] = m->qkv_rows;
    p.row_offset[2] = row0;
    p.position = position;
}

LinearParams lm_head_params(const cppinf_qwen3* m, const bf16* x, int64_t advance, bf16* logits) {
    const auto& c = m->c;
    LinearParams p = params_for(LinearEpilogue::kArgmax, x, c.hidden_size, m->embed, nullptr, 1, c.vocab_size,
                                c.hidden_size);
    p.norm_weight = m->final_norm;
    p.eps = c.rms_norm_eps;
    p.out[0] = logits;
    p.ld[0] = c.vocab_size;
    p.tokens_out = m->d_tokens;
    p.position_out = m->d_len;
    p.advance = advance;
    p.partial = m->d_partial;
    p.counter = m->d_counter;
    return p;
}

// Whether the decode step's attention kernel takes the input norm and the q|k|v projection (decoder.h).
bool projection_fused(const cppinf_qwen3* m) {
    return cppinf::device::decode_projection_fused(m->c.head_dim, m->c.hidden_size, m->cap);
}

// One decode step at the device-side position (see the file comment). Returns the number of launches. With
// `after_step` (a step enqueued right behind another in one graph) the step's first kernel starts only once the
// previous step's last kernel has completed: the attention kernel reads the sequence length before its dependency
// wait, and the LM head before it advances that length.
int enqueue_step(cppinf_qwen3* m, cudaStream_t s, int64_t* launches, bool after_step = false) {
    const auto& c = m->c;
    const int64_t H = c.hidden_size;
    const bool fused = projection_fused(m);
    int64_t n = 0;
    for (std::size_t i = 0; i < m->layers.size(); ++i) {
        const Layer& l = m->layers[i];
        if (!fused) {
            LinearParams qkv = params_for(LinearEpilogue::kStore, i == 0 ? m->embed : m->h, H, l.wqkv, nullptr, 1,
                                          m->qkv_rows, H);
            if (i == 0) {
                qkv.tokens = m->d_tokens;
                qkv.vocab = c.vocab_size;
                qkv.x_copy = m->h;
            }
            qkv.norm_weight = l.in_norm;
            qkv.eps = c.rms_norm_eps;
            set_qkv_outputs(m, l, qkv, 0, m->d_len);
            qkv.error = m->d_error;
            {
                const std::optional<rt::SerialLaunch> serial =
                    after_step && i == 0 ? std::optional<rt::SerialLaunch>(std::in_place) : std::nullopt;
                QWEN3_TRY(cppinf::device::launch_gemv(qkv, s), "qwen3_qkv");
            }
            ++n;
        }
        // q/k-norm + RoPE and the new key's cache row are fused into the attention kernel, and with `fused` the
        // input norm and the q|k|v projection too (the first layer's embedding gather included).
        AttentionParams ap{m->q, l.k_cache, l.v_cache, m->ctx, 1,
                           static_cast<int>(c.num_attention_heads), static_cast<int>(c.num_key_value_heads),
                           static_cast<int>(c.head_dim), 0, m->d_len, m->cap,
                           m->k, l.q_norm, l.k_norm, m->rope, c.rms_norm_eps, m->d_error};
        ap.poll_limit = rt::wait_poll_limit();
        if (fused) {
            ap.x = i == 0 ? m->embed : m->h;
            ap.tokens = i == 0 ? m->d_tokens : nullptr;
            ap.vocab = c.vocab_size;
            ap.x_copy = i == 0 ? m->h : nullptr;
            ap.in_norm = l.in_norm;
            ap.wqkv = l.wqkv;
            ap.hidden = static_cast<int>(H);
        }
        {
            const std::optional<rt::SerialLaunch> serial =
                after_step && i == 0 && fused ? std::optional<rt::SerialLaunch>(std::in_place) : std::nullopt;
            QWEN3_TRY(cppinf::device::launch_decoder_attention(ap, m->cap, s), "qwen3_attention");
        }
        LinearParams o = params_for(LinearEpilogue::kResidual, m->ctx, m->q_dim, l.wo, nullptr, 1, H, m->q_dim);
        o.residual = m->h;
        o.res_ld = H;
        o.out[0] = m->h;
        o.ld[0] = H;
        o.error = m->d_error;
        QWEN3_TRY(cppinf::device::launch_gemv(o, s), "qwen3_o_proj");
        LinearParams gu = params_for(LinearEpilogue::kSiluMul, m->h, H, l.wg, l.wu, 1, c.intermediate_size, H);
        gu.norm_weight = l.post_norm;
        gu.eps = c.rms_norm_eps;
        gu.out[0] = m->act;
        gu.ld[0] = c.intermediate_size;
        gu.error = m->d_error;
        QWEN3_TRY(cppinf::device::launch_gemv(gu, s), "qwen3_gate_up");
        LinearParams d = params_for(LinearEpilogue::kResidual, m->act, c.intermediate_size, l.wd, nullptr, 1, H,
                                    c.intermediate_size);
        d.residual = m->h;
        d.res_ld = H;
        d.out[0] = m->h;
        d.ld[0] = H;
        d.error = m->d_error;
        QWEN3_TRY(cppinf::device::launch_gemv(d, s), "qwen3_down_proj");
        n += 4;
    }
    QWEN3_TRY(cppinf::device::launch_gemv(lm_head_params(m, m->h, 1, nullptr), s), "qwen3_lm_head_argmax");
    *launches = n + 1;
    return CPPINF_OK;
}

// Decode steps replayed per graph launch when a call asks for at least this many: consecutive steps in one graph
// leave out the graph-launch gap between them.
constexpr int64_t kBlockSteps = 8;

// Captures `count` consecutive decode steps into one executable graph.
int capture_steps(cppinf_qwen3* m, int64_t count, cudaGraphExec_t* exec, int64_t* launches) {
    cudaStream_t cap_stream = nullptr;
    CPPINF_CUDA_TRY(cudaStreamCreateWithFlags(&cap_stream, cudaStreamNonBlocking));
    cudaGraph_t graph = nullptr;
    cudaError_t err = cudaStreamBeginCapture(cap_stream, cudaStreamCaptureModeThreadLocal);
    int64_t total = 0;
    int st = CPPINF_OK;
    if (err == cudaSuccess) {
        for (int64_t k = 0; k < count && st == CPPINF_OK; ++k) {
            int64_t n = 0;
            st = enqueue_step(m, cap_stream, &n, k > 0);
            total += n;
        }
        err = cudaStreamEndCapture(cap_stream, &graph);
    }
    if (err == cudaSuccess && st == CPPINF_OK) {
        err = cudaGraphInstantiate(exec, graph, 0);
    }
    if (graph != nullptr) {
        cudaGraphDestroy(graph);
    }
    cudaStreamDestroy(cap_stream);
    if (st != CPPINF_OK) {
        return st;
    }
    if (err != cudaSuccess) {
        *exec = nullptr;
        return rt::cuda_fail(err, "qwen3_decode graph capture");
    }
    *launches = total;
    rt::count_launches(-total);  // captured, not executed: each replay counts them
    return CPPINF_OK;
}

// A prompt-row projection: on the tensor cores when the model asks for them and the layout allows it, otherwise the
// CUDA-core kernel with the restated order.
cudaError_t launch_rows(const cppinf_qwen3* m, LinearParams p, cudaStream_t s) {
    if (m->prefill_mode == 1) {
        p.error = m->d_error;
        if (cppinf::device::linear_tc_supported(p)) {
            return cppinf::device::launch_linear_tc(p, s);
        }
    }
    return cppinf::device::launch_linear_rows(p, s);
}

// Prompt rows [pos0, pos0 + T) whose ids are already in d_tokens; writes logits of all rows to `logits` when set.
int enqueue_chunk(cppinf_qwen3* m, int64_t pos0, int64_t T, bf16* logits, cudaStream_t s) {
    const auto& c = m->c;
    const int64_t H = c.hidden_size;
    QWEN3_TRY(cppinf::device::launch_embedding(m->embed, c.vocab_size, H, m->d_tokens + pos0, T, m->h, s),
              "qwen3_embedding");
    for (const Layer& l : m->layers) {
        QWEN3_CHECK(cppinf_rms_norm(CPPINF_DTYPE_BF16, m->h, H, l.in_norm, m->xn, T, H, c.rms_norm_eps, s));
        LinearParams qkv = params_for(LinearEpilogue::kStore, m->xn, H, l.wqkv, nullptr, T, m->qkv_rows, H);
        set_qkv_outputs(m, l, qkv, pos0, nullptr);
        QWEN3_TRY(launch_rows(m, qkv, s), "qwen3_qkv_rows");
        QWEN3_CHECK(cppinf_qk_norm_rope(CPPINF_DTYPE_BF16, m->q, m->k, l.q_norm, l.k_norm, m->qr,
                                        l.k_cache + pos0 * m->kv_dim, T, c.num_attention_heads,
                                        c.num_key_value_heads, c.head_dim, pos0, c.rms_norm_eps, m->rope, m->cap, s));
        if (m->prefill_mode == 1) {
            AttentionParams ap{};
            ap.q = m->qr;
            ap.k_cache = l.k_cache;
            ap.v_cache = l.v_cache;
            ap.ctx = m->ctx;
            ap.T = T;
            ap.q_heads = static_cast<int>(c.num_attention_heads);
            ap.kv_heads = static_cast<int>(c.num_key_value_heads);
            ap.head_dim = static_cast<int>(c.head_dim);
            ap.pos0 = pos0;
            ap.capacity = m->cap;
            ap.error = m->d_error;
            ap.poll_limit = rt::wait_poll_limit();
            if (cppinf::device::attention_tc_supported(ap)) {
                QWEN3_TRY(cppinf::device::launch_attention_tc(ap, s), "qwen3_attention_tc");
            } else {
                QWEN3_CHECK(cppinf_decoder_attention(m->qr, l.k_cache, l.v_cache, m->ctx, T, c.num_attention_heads,
                                                     c.num_key_value_heads, c.head_dim, pos0, m->cap, s));
            }
        } else {
            QWEN3_CHECK(cppinf_decoder_attention(m->qr, l.k_cache, l.v_cache, m->ctx, T, c.num_attention_heads,
                                                 c.num_key_value_heads, c.head_dim, pos0, m->cap, s));
        }
        LinearParams o = params_for(LinearEpilogue::kResidual, m->ctx, m->q_dim, l.wo, nullptr, T, H, m->q_dim);
        o.residual = m->h;
        o.res_ld = H;
        o.out[0] = m->h;
        o.ld[0] = H;
        QWEN3_TRY(launch_rows(m, o, s), "qwen3_o_proj_rows");
        QWEN3_CHECK(cppinf_rms_norm(CPPINF_DTYPE_BF16, m->h, H, l.post_norm, m->xn, T, H, c.rms_norm_eps, s));
        LinearParams gu = params_for(LinearEpilogue::kSiluMul, m->xn, H, l.wg, l.wu, T, c.intermediate_size, H);
        gu.out[0] = m->act;
        gu.ld[0] = c.intermediate_size;
        QWEN3_TRY(launch_rows(m, gu, s), "qwen3_gate_up_rows");
        LinearParams d = params_for(LinearEpilogue::kResidual, m->act, c.intermediate_size, l.wd, nullptr, T, H,
                                    c.intermediate_size);
        d.residual = m->h;
        d.res_ld = H;
        d.out[0] = m->h;
        d.ld[0] = H;
        QWEN3_TRY(launch_rows(m, d, s), "qwen3_down_proj_rows");
    }
    if (logits != nullptr) {
        QWEN3_CHECK(cppinf_rms_norm(CPPINF_DTYPE_BF16, m->h, H, m->final_norm, m->xn, T, H, c.rms_norm_eps, s));
        LinearParams lm = params_for(LinearEpilogue::kStore, m->xn, H, m->embed, nullptr, T, c.vocab_size, H);
        lm.out[0] = logits;
        lm.ld[0] = c.vocab_size;
        QWEN3_TRY(T == 1 ? cppinf::device::launch_gemv(lm, s) : launch_rows(m, lm, s),
                  "qwen3_lm_head_rows");
    }
    return CPPINF_OK;
}

}  // namespace

// A batch of cached sequences (Qwen3Cache of src/models/qwen3/qwen3_model.cpp:222-245): per layer and sequence a K
// and a V cache [capacity, kv_heads, head_dim], and each sequence's length on the host.
struct cppinf_qwen3_cache {
    int64_t batch = 0;
    int64_t cap = 0;
    int64_t layers = 0;
    int64_t kv_dim = 0;
    std::size_t per_cache = 0;  // bytes of one K or V cache of one sequence and layer
    char* mem = nullptr;
    std::size_t bytes = 0;
    int64_t* d_ids = nullptr;  // the token ids of one chunk of rows
    std::vector<int64_t> lens;

    bf16* k(int64_t layer, int64_t b) const {
        return reinterpret_cast<bf16*>(mem + per_cache * static_cast<std::size_t>((layer * batch + b) * 2));
    }
    bf16* v(int64_t layer, int64_t b) const {
        return reinterpret_cast<bf16*>(mem + per_cache * static_cast<std::size_t>((layer * batch + b) * 2 + 1));
    }
};

namespace {

// Rows [start, start + n) of sequence b, at rows [row, row + n) of a chunk.
struct Piece {
    int64_t b;
    int64_t start;
    int64_t n;
    int64_t row;
};

// One chunk of a batched forward: the rows of `pieces` (at most the workspace's rows, one piece per sequence) go
// through the decoder together -- embedding, norms, projections and the MLP over all rows at once, the q/k norm +
// RoPE, the cache appends and the attention per sequence -- so each row is computed exactly as in a forward of its
// own sequence. Logits of each piece go to logits[b, start .. start + n).
int enqueue_batch_chunk(cppinf_qwen3* m, cppinf_qwen3_cache* kc, const std::vector<Piece>& pieces,
                        const int64_t* host_ids, int64_t max_length, bf16* logits, cudaStream_t s) {
    const auto& c = m->c;
    const int64_t H = c.hidden_size;
    const int64_t V = c.vocab_size;
    const int64_t R = pieces.back().row + pieces.back().n;
    std::vector<int64_t> ids(static_cast<std::size_t>(R));
    for (const Piece& p : pieces) {
        for (int64_t i = 0; i < p.n; ++i) {
            ids[static_cast<std::size_t>(p.row + i)] = host_ids[p.b * max_length + p.start + i];
        }
    }
    CPPINF_CUDA_TRY(cudaMemcpyAsync(kc->d_ids, ids.data(), static_cast<std::size_t>(R) * 8, cudaMemcpyHostToDevice,
                                    s));
    QWEN3_TRY(cppinf::device::launch_embedding(m->embed, V, H, kc->d_ids, R, m->h, s), "qwen3_embedding");
    for (std::size_t li = 0; li < m->layers.size(); ++li) {
        const Layer& l = m->layers[li];
        const auto layer = static_cast<int64_t>(li);
        QWEN3_CHECK(cppinf_rms_norm(CPPINF_DTYPE_BF16, m->h, H, l.in_norm, m->xn, R, H, c.rms_norm_eps, s));
        LinearParams qkv = params_for(LinearEpilogue::kStore, m->xn, H, l.wqkv, nullptr, R, m->qkv_rows, H);
        set_qkv_outputs(m, l, qkv, 0, nullptr);
        qkv.out[2] = m->ctx;  // v rows [R, kv_dim] staged in the context buffer, then appended to each cache
        QWEN3_TRY(launch_rows(m, qkv, s), "qwen3_qkv_rows");
        for (const Piece& p : pieces) {
            const int64_t pos = kc->lens[static_cast<std::size_t>(p.b)] + p.start;
            CPPINF_CUDA_TRY(cudaMemcpyAsync(kc->v(layer, p.b) + pos * m->kv_dim, m->ctx + p.row * m->kv_dim,
                                            static_cast<std::size_t>(p.n * m->kv_dim) * 2, cudaMemcpyDeviceToDevice,
                                            s));
        }
        for (const Piece& p : pieces) {
            const int64_t pos = kc->lens[static_cast<std::size_t>(p.b)] + p.start;
            bf16* kcache = kc->k(layer, p.b);
            bf16* vcache = kc->v(layer, p.b);
            bf16* qr = m->qr + p.row * m->q_dim;
            bf16* ctx = m->ctx + p.row * m->q_dim;
            QWEN3_CHECK(cppinf_qk_norm_rope(CPPINF_DTYPE_BF16, m->q + p.row * m->q_dim, m->k + p.row * m->kv_dim,
                                            l.q_norm, l.k_norm, qr, kcache + pos * m->kv_dim, p.n,
                                            c.num_attention_heads, c.num_key_value_heads, c.head_dim, pos,
                                            c.rms_norm_eps, m->rope, m->cap, s));
            AttentionParams ap{};
            ap.q = qr;
            ap.k_cache = kcache;
            ap.v_cache = vcache;
            ap.ctx = ctx;
            ap.T = p.n;
            ap.q_heads = static_cast<int>(c.num_attention_heads);
            ap.kv_heads = static_cast<int>(c.num_key_value_heads);
            ap.head_dim = static_cast<int>(c.head_dim);
            ap.pos0 = pos;
            ap.capacity = kc->cap;
            ap.error = m->d_error;
            ap.poll_limit = rt::wait_poll_limit();
            if (m->prefill_mode == 1 && cppinf::device::attention_tc_supported(ap)) {
                QWEN3_TRY(cppinf::device::launch_attention_tc(ap, s), "qwen3_attention_tc");
            } else {
                QWEN3_CHECK(cppinf_decoder_attention(qr, kcache, vcache, ctx, p.n, c.num_attention_heads,
                                                     c.num_key_value_heads, c.head_dim, pos, kc->cap, s));
            }
        }
        LinearParams o = params_for(LinearEpilogue::kResidual, m->ctx, m->q_dim, l.wo, nullptr, R, H, m->q_dim);
        o.residual = m->h;
        o.res_ld = H;
        o.out[0] = m->h;
        o.ld[0] = H;
        QWEN3_TRY(launch_rows(m, o, s), "qwen3_o_proj_rows");
        QWEN3_CHECK(cppinf_rms_norm(CPPINF_DTYPE_BF16, m->h, H, l.post_norm, m->xn, R, H, c.rms_norm_eps, s));
        LinearParams gu = params_for(LinearEpilogue::kSiluMul, m->xn, H, l.wg, l.wu, R, c.intermediate_size, H);
        gu.out[0] = m->act;
        gu.ld[0] = c.intermediate_size;
        QWEN3_TRY(launch_rows(m, gu, s), "qwen3_gate_up_rows");
        LinearParams d = params_for(LinearEpilogue::kResidual, m->act, c.intermediate_size, l.wd, nullptr, R, H,
                                    c.intermediate_size);
        d.residual = m->h;
        d.res_ld = H;
        d.out[0] = m->h;
        d.ld[0] = H;
        QWEN3_TRY(launch_rows(m, d, s), "qwen3_down_proj_rows");
    }
    QWEN3_CHECK(cppinf_rms_norm(CPPINF_DTYPE_BF16, m->h, H, m->final_norm, m->xn, R, H, c.rms_norm_eps, s));
    // The LM head once per run of pieces that are consecutive in logits [batch, max_length, vocab].
    std::size_t i = 0;
    while (i < pieces.size()) {
        std::size_t j = i + 1;
        int64_t rows = pieces[i].n;
        while (j < pieces.size() && pieces[j - 1].start + pieces[j - 1].n == max_length && pieces[j].start == 0 &&
               pieces[j].b == pieces[j - 1].b + 1) {
            rows += pieces[j].n;
            ++j;
        }
        const Piece& first = pieces[i];
        LinearParams lm = params_for(LinearEpilogue::kStore, m->xn + first.row * H, H, m->embed, nullptr, rows, V, H);
        lm.out[0] = logits + (first.b * max_length + first.start) * V;
        lm.ld[0] = V;
        QWEN3_TRY(rows == 1 ? cppinf::device::launch_gemv(lm, s) : launch_rows(m, lm, s), "qwen3_lm_head_rows");
        i = j;
    }
    return CPPINF_OK;
}

// Where a checkpoint tensor goes and the shape the model expects: [rows, cols] for matrices, [rows] when cols == 0.
struct WeightSlot {
    bf16* dst;
    int64_t elements;
    int64_t rows;
    int64_t cols;
};

int find_weight(cppinf_qwen3* m, const std::string& name, WeightSlot* slot) {
    const auto& c = m->c;
    const int64_t H = c.hidden_size;
    if (name == "model.embed_tokens.weight") {
        *slot = {m->embed, c.vocab_size * H, c.vocab_size, H};
        return CPPINF_OK;
    }
    if (name == "model.norm.weight") {
        *slot = {m->final_norm, H, H, 0};
        return CPPINF_OK;
    }
    const std::string prefix = "model.layers.";
    if (name.compare(0, prefix.size(), prefix) == 0) {
        std::size_t i = prefix.size();
        int64_t layer = 0;
        bool digits = false;
        while (i < name.size() && name[i] >= '0' && name[i] <= '9' && layer < (int64_t{1} << 40)) {
            layer = layer * 10 + (name[i] - '0');
            digits = true;
            ++i;
        }
        if (digits && i < name.size() && name[i] == '.' && layer < c.num_hidden_layers) {
            const std::string field = name.substr(i + 1);
            const Layer& l = m->layers[static_cast<std::size_t>(layer)];
            const int64_t I = c.intermediate_size;
            if (field == "input_layernorm.weight") {
                *slot = {l.in_norm, H, H, 0};
            } else if (field == "post_attention_layernorm.weight") {
                *slot = {l.post_norm, H, H, 0};
            } else if (field == "self_attn.q_norm.weight") {
                *slot = {l.q_norm, c.head_dim, c.head_dim, 0};
            } else if (field == "self_attn.k_norm.weight") {
                *slot = {l.k_norm, c.head_dim, c.head_dim, 0};
            } else if (field == "self_attn.q_proj.weight") {
                *slot = {l.wqkv, m->q_dim * H, m->q_dim, H};
            } else if (field == "self_attn.k_proj.weight") {
                *slot = {l.wqkv + m->q_dim * H, m->kv_dim * H, m->kv_dim, H};
            } else if (field == "self_attn.v_proj.weight") {
                *slot = {l.wqkv + (m->q_dim + m->kv_dim) * H, m->kv_dim * H, m->kv_dim, H};
            } else if (field == "self_attn.o_proj.weight") {
                *slot = {l.wo, H * m->q_dim, H, m->q_dim};
            } else if (field == "mlp.gate_proj.weight") {
                *slot = {l.wg, I * H, I, H};
            } else if (field == "mlp.up_proj.weight") {
                *slot = {l.wu, I * H, I, H};
            } else if (field == "mlp.down_proj.weight") {
                *slot = {l.wd, H * I, H, I};
            } else {
                return rt::fail(CPPINF_ERR_INVALID_ARGUMENT, "Qwen3Model does not use tensor '" + name + "'.");
            }
            return CPPINF_OK;
        }
    }
    return rt::fail(CPPINF_ERR_INVALID_ARGUMENT, "Qwen3Model does not use tensor '" + name + "'.");
}

void release(cppinf_qwen3* m) {
    if (m->step != nullptr) {
        cudaGraphExecDestroy(m->step);
    }
    if (m->step_block != nullptr) {
        cudaGraphExecDestroy(m->step_block);
    }
    cudaFree(m->weights);
    cudaFree(m->cache);
    cudaFree(m->work);
}

}  // namespace

namespace cppinf::device {

int64_t qwen3_tensor_bytes(const cppinf_qwen3* model, const std::string& name) {
    std::vector<int64_t> shape;
    return qwen3_tensor_shape(model, name, &shape) ? qwen3_shape_elements(shape) * 2 : -1;
}

bool qwen3_tensor_shape(const cppinf_qwen3* model, const std::string& name, std::vector<int64_t>* shape) {
    WeightSlot slot{};
    // find_weight records an error message for unknown names; this probe must not disturb the caller's.
    const std::string saved = cppinf_last_error();
    const int st = find_weight(const_cast<cppinf_qwen3*>(model), name, &slot);
    if (st != CPPINF_OK) {
        rt::fail(CPPINF_ERR_INVALID_ARGUMENT, saved);
        return false;
    }
    *shape = slot.cols == 0 ? std::vector<int64_t>{slot.rows} : std::vector<int64_t>{slot.rows, slot.cols};
    return true;
}

int64_t qwen3_shape_elements(const std::vector<int64_t>& shape) {
    int64_t n = 1;
    for (const int64_t d : shape) {
        n *= d;
    }
    return n;
}

int64_t qwen3_tensor_count(const cppinf_qwen3* model) {
    return 11 * model->c.num_hidden_layers + 2;
}

}  // namespace cppinf::device

extern "C" {

int cppinf_qwen3_create(const cppinf_qwen3_config* config, int64_t max_sequence_length, cppinf_qwen3** model) {
    CPPINF_REQUIRE(config && model, CPPINF_ERR_INVALID_ARGUMENT, "qwen3_create received a null pointer.");
    *model = nullptr;
    const cppinf_qwen3_config c = *config;
    CPPINF_REQUIRE(c.num_hidden_layers > 0 && c.num_attention_heads > 0 && c.num_key_value_heads > 0 &&
                       c.head_dim > 0,
                   CPPINF_ERR_INVALID_ARGUMENT, "Qwen3Model requires non-zero layer and head configuration.");
    CPPINF_REQUIRE(c.num_attention_heads % c.num_key_value_heads == 0, CPPINF_ERR_INVALID_ARGUMENT,
                   "Qwen3Model requires num_attention_heads to divide by num_key_value_heads.");
    CPPINF_REQUIRE(c.vocab_size > 0 && c.hidden_size > 0 && c.intermediate_size > 0, CPPINF_ERR_INVALID_ARGUMENT,
                   "Qwen3Model requires non-zero vocabulary, hidden and intermediate sizes.");
    CPPINF_REQUIRE(max_sequence_length > 0, CPPINF_ERR_INVALID_ARGUMENT,
                   "Qwen3Model cache requires non-zero batch and sequence dimensions.");
    CPPINF_REQUIRE(c.head_dim == 64 || c.head_dim == 128 || c.head_dim == 256, CPPINF_ERR_UNSUPPORTED,
                   "the device decoder supports head_dim 64, 128 or 256.");
    CPPINF_REQUIRE(c.hidden_size % 8 == 0 && c.intermediate_size % 8 == 0, CPPINF_ERR_UNSUPPORTED,
                   "the device decoder requires hidden and intermediate sizes that are multiples of 8.");
    CPPINF_REQUIRE(c.hidden_size <= 6144 && c.intermediate_size <= 6144 &&
                       c.num_attention_heads * c.head_dim <= 6144,
                   CPPINF_ERR_UNSUPPORTED, "the device decoder supports projection inputs of up to 6144 features.");
    CPPINF_REQUIRE(c.vocab_size < (int64_t{1} << 31) && max_sequence_length < (int64_t{1} << 24),
                   CPPINF_ERR_UNSUPPORTED, "the device decoder supports vocabularies below 2^31 and caches below 2^24.");
    CPPINF_REQUIRE(c.rms_norm_eps >= 0.0f && c.rope_theta > 0.0f, CPPINF_ERR_INVALID_ARGUMENT,
                   "qwen_decoder_block requires a non-negative finite norm epsilon and a positive rope base.");

    auto* m = new cppinf_qwen3();
    m->c = c;
    m->cap = max_sequence_length;
    m->q_dim = c.num_attention_heads * c.head_dim;
    m->kv_dim = c.num_key_value_heads * c.head_dim;
    m->qkv_rows = m->q_dim + 2 * m->kv_dim;
    const int64_t H = c.hidden_size;
    const int64_t I = c.intermediate_size;
    const int64_t L = c.num_hidden_layers;

    // Weights.
    std::vector<std::size_t> offsets;
    std::size_t off = 0;
    auto take = [&](int64_t elements) {
        const std::size_t at = off;
        off = align_up(off + static_cast<std::size_t>(elements) * 2);
        return at;
    };
    struct LayerOffsets {
        std::size_t in_norm, post_norm, q_norm, k_norm, wqkv, wo, wg, wu, wd;
    };
    std::vector<LayerOffsets> lo(static_cast<std::size_t>(L));
    for (auto& x : lo) {
        x.in_norm = take(H);
        x.post_norm = take(H);
        x.q_norm = take(c.head_dim);
        x.k_norm = take(c.head_dim);
        x.wqkv = take(m->qkv_rows * H);
        x.wo = take(H * m->q_dim);
        x.wg = take(I * H);
        x.wu = take(I * H);
        x.wd = take(H * I);
    }
    const std::size_t embed_off = take(c.vocab_size * H);
    const std::size_t final_off = take(H);
    m->weight_bytes = off;

    // Cache.
    const std::size_t per_cache = align_up(static_cast<std::size_t>(m->cap * m->kv_dim) * 2);
    m->cache_bytes = per_cache * 2 * static_cast<std::size_t>(L);

    // State and workspace.
    LinearParams lm{};
    lm.N = c.vocab_size;
    lm.K = H;
    const int partials = cppinf::device::gemv_grid(lm);
    std::size_t w = 0;
    auto wtake = [&](std::size_t bytes) {
        const std::size_t at = w;
        w = align_up(w + bytes);
        return at;
    };
    const std::size_t rope_off = wtake(static_cast<std::size_t>(m->cap * c.head_dim) * sizeof(float));
    const std::size_t len_off = wtake(sizeof(int));
    const std::size_t counter_off = wtake(sizeof(unsigned int));
    const std::size_t error_off = wtake(sizeof(unsigned int));
    const std::size_t partial_off = wtake(static_cast<std::size_t>(partials) * 8);
    const std::size_t tokens_off = wtake(static_cast<std::size_t>(m->cap + 1) * 8);
    const int64_t rows = kChunkRows < m->cap ? kChunkRows : m->cap;
    const std::size_t h_off = wtake(static_cast<std::size_t>(rows * H) * 2);
    const std::size_t xn_off = wtake(static_cast<std::size_t>(rows * H) * 2);
    const std::size_t q_off = wtake(static_cast<std::size_t>(rows * m->q_dim) * 2);
    const std::size_t k_off = wtake(static_cast<std::size_t>(rows * m->kv_dim) * 2);
    const std::size_t qr_off = wtake(static_cast<std::size_t>(rows * m->q_dim) * 2);
    const std::size_t ctx_off = wtake(static_cast<std::size_t>(rows * m->q_dim) * 2);
    const std::size_t act_off = wtake(static_cast<std::size_t>(rows * I) * 2);

    cudaError_t err = cudaMalloc(&m->weights, m->weight_bytes);
    if (err == cudaSuccess) {
        err = cudaMalloc(&m->cache, m->cache_bytes);
    }
    if (err == cudaSuccess) {
        err = cudaMalloc(&m->work, w);
    }
    if (err == cudaSuccess) {
        err = cudaMemset(m->weights, 0, m->weight_bytes);
    }
    if (err == cudaSuccess) {
        err = cudaMemset(m->cache, 0, m->cache_bytes);
    }
    if (err == cudaSuccess) {
        err = cudaMemset(m->work, 0, w);
    }
    if (err != cudaSuccess) {
        release(m);
        delete m;
        return rt::cuda_fail(err, "qwen3_create allocation");
    }
    for (int64_t i = 0; i < L; ++i) {
        const auto& x = lo[static_cast<std::size_t>(i)];
        auto at = [&](std::size_t o) { return reinterpret_cast<bf16*>(m->weights + o); };
        Layer layer{at(x.in_norm), at(x.post_norm), at(x.q_norm), at(x.k_norm), at(x.wqkv), at(x.wo), at(x.wg),
                    at(x.wu),      at(x.wd),        nullptr,      nullptr};
        layer.k_cache = reinterpret_cast<bf16*>(m->cache + per_cache * static_cast<std::size_t>(2 * i));
        layer.v_cache = reinterpret_cast<bf16*>(m->cache + per_cache * static_cast<std::size_t>(2 * i + 1));
        m->layers.push_back(layer);
    }
    m->embed = reinterpret_cast<bf16*>(m->weights + embed_off);
    m->final_norm = reinterpret_cast<bf16*>(m->weights + final_off);
    m->rope = reinterpret_cast<float*>(m->work + rope_off);
    m->d_len = reinterpret_cast<int*>(m->work + len_off);
    m->d_counter = reinterpret_cast<unsigned int*>(m->work + counter_off);
    m->d_error = reinterpret_cast<unsigned int*>(m->work + error_off);
    m->d_partial = reinterpret_cast<unsigned long long*>(m->work + partial_off);
    m->d_tokens = reinterpret_cast<int64_t*>(m->work + tokens_off);
    m->h = reinterpret_cast<bf16*>(m->work + h_off);
    m->xn = reinterpret_cast<bf16*>(m->work + xn_off);
    m->q = reinterpret_cast<bf16*>(m->work + q_off);
    m->k = reinterpret_cast<bf16*>(m->work + k_off);
    m->qr = reinterpret_cast<bf16*>(m->work + qr_off);
    m->ctx = reinterpret_cast<bf16*>(m->work + ctx_off);
    m->act = reinterpret_cast<bf16*>(m->work + act_off);

    std::vector<float> table(static_cast<std::size_t>(m->cap * c.head_dim));
    int st = cppinf_rope_table(c.rope_theta, c.head_dim, m->cap, table.data());
    if (st == CPPINF_OK) {
        err = cudaMemcpy(m->rope, table.data(), table.size() * sizeof(float), cudaMemcpyHostToDevice);
        st = err == cudaSuccess ? CPPINF_OK : rt::cuda_fail(err, "qwen3_create rope table");
    }
    if (st != CPPINF_OK) {
        release(m);
        delete m;
        return st;
    }
    *model = m;
    return rt::ok();
}

void cppinf_qwen3_destroy(cppinf_qwen3* model) {
    if (model != nullptr) {
        release(model);
        delete model;
    }
}

int cppinf_qwen3_set_weight(cppinf_qwen3* model, const char* name, const void* data, int64_t bytes, int on_device) {
    CPPINF_REQUIRE(model && name && data, CPPINF_ERR_INVALID_ARGUMENT, "qwen3_set_weight received a null pointer.");
    WeightSlot slot{};
    QWEN3_CHECK(find_weight(model, name, &slot));
    CPPINF_REQUIRE(bytes == slot.elements * 2, CPPINF_ERR_INVALID_ARGUMENT,
                   std::string("Qwen3Model tensor '") + name + "' has an unexpected size.");
    CPPINF_CUDA_TRY(cudaMemcpy(slot.dst, data, static_cast<std::size_t>(bytes),
                               on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice));
    return rt::ok();
}

int cppinf_qwen3_reset(cppinf_qwen3* model, void* stream) {
    CPPINF_REQUIRE(model, CPPINF_ERR_INVALID_ARGUMENT, "qwen3_reset received a null pointer.");
    const auto s = rt::as_stream(stream);
    CPPINF_CUDA_TRY(cudaMemsetAsync(model->cache, 0, model->cache_bytes, s));
    CPPINF_CUDA_TRY(cudaMemsetAsync(model->d_len, 0, sizeof(int), s));
    CPPINF_CUDA_TRY(cudaMemsetAsync(model->d_error, 0, sizeof(unsigned int), s));
    model->len = 0;
    model->failed = false;
    return rt::ok();
}

int cppinf_qwen3_set_prefill(cppinf_qwen3* model, int mode) {
    CPPINF_REQUIRE(model, CPPINF_ERR_INVALID_ARGUMENT, "qwen3_set_prefill received a null pointer.");
    CPPINF_REQUIRE(mode == 0 || mode == 1, CPPINF_ERR_INVALID_ARGUMENT,
                   "qwen3_set_prefill mode must be 0 (CUDA cores) or 1 (tensor cores).");
    model->prefill_mode = mode;
    return rt::ok();
}

int64_t cppinf_qwen3_length(const cppinf_qwen3* model) {
    return model != nullptr ? model->len : -1;
}

int64_t cppinf_qwen3_step_launches(const cppinf_qwen3* model) {
    if (model == nullptr) {
        return 0;
    }
    return (projection_fused(model) ? 4 : 5) * model->c.num_hidden_layers + 1;
}

int cppinf_qwen3_forward(cppinf_qwen3* model, const int64_t* token_ids, int64_t count, void* logits, int all_rows,
                         int64_t* next_token, void* stream) {
    CPPINF_REQUIRE(model && token_ids, CPPINF_ERR_INVALID_ARGUMENT, "qwen3_forward received a null pointer.");
    CPPINF_REQUIRE(count > 0, CPPINF_ERR_INVALID_ARGUMENT,
                   "Qwen3Model session forward requires at least one uncached token.");
    CPPINF_REQUIRE(!model->failed, CPPINF_ERR_CUDA,
                   "qwen3 model state is invalid after a device error; call qwen3_reset first.");
    CPPINF_REQUIRE(model->len + count <= model->cap, CPPINF_ERR_OUT_OF_RANGE,
                   "qwen_attention cache is too small for the new tokens.");
    for (int64_t i = 0; i < count; ++i) {
        CPPINF_REQUIRE(token_ids[i] >= 0 && token_ids[i] < model->c.vocab_size, CPPINF_ERR_OUT_OF_RANGE,
                       "Qwen3Model token id is out of vocabulary range.");
    }
    const auto s = rt::as_stream(stream);
    const int len_now = static_cast<int>(model->len);
    CPPINF_CUDA_TRY(cudaMemcpyAsync(model->d_tokens + model->len, token_ids, static_cast<std::size_t>(count) * 8,
                                    cudaMemcpyHostToDevice, s));
    CPPINF_CUDA_TRY(cudaMemcpyAsync(model->d_len, &len_now, sizeof(int), cudaMemcpyHostToDevice, s));
    const int64_t V = model->c.vocab_size;
    int64_t last_rows = 0;
    for (int64_t done = 0; done < count; done += kChunkRows) {
        const int64_t T = count - done < kChunkRows ? count - done : kChunkRows;
        bf16* chunk_logits = (logits != nullptr && all_rows) ? static_cast<bf16*>(logits) + done * V : nullptr;
        QWEN3_CHECK(enqueue_chunk(model, model->len + done, T, chunk_logits, s));
        last_rows = T;
    }
    bf16* last_logits = (logits != nullptr && !all_rows) ? static_cast<bf16*>(logits) : nullptr;
    QWEN3_TRY(cppinf::device::launch_gemv(
                  lm_head_params(model, model->h + (last_rows - 1) * model->c.hidden_size, count, last_logits), s),
              "qwen3_lm_head_argmax");
    model->len += count;
    if (next_token != nullptr) {
        CPPINF_CUDA_TRY(cudaMemcpyAsync(next_token, model->d_tokens + model->len, 8, cudaMemcpyDeviceToHost, s));
        CPPINF_CUDA_TRY(cudaStreamSynchronize(s));
    }
    return rt::ok();
}

int cppinf_qwen3_cache_create(const cppinf_qwen3* model, int64_t batch, int64_t capacity, cppinf_qwen3_cache** cache) {
    CPPINF_REQUIRE(model && cache, CPPINF_ERR_INVALID_ARGUMENT, "qwen3_cache_create received a null pointer.");
    *cache = nullptr;
    CPPINF_REQUIRE(batch > 0 && capacity > 0, CPPINF_ERR_INVALID_ARGUMENT,
                   "Qwen3Model cache requires non-zero batch and sequence dimensions.");
    CPPINF_REQUIRE(capacity <= model->cap, CPPINF_ERR_UNSUPPORTED,
                   "a batch cache may hold at most the model's max_sequence_length positions (its rotary table).");
    auto* kc = new cppinf_qwen3_cache();
    kc->batch = batch;
    kc->cap = capacity;
    kc->layers = model->c.num_hidden_layers;
    kc->kv_dim = model->kv_dim;
    kc->per_cache = align_up(static_cast<std::size_t>(capacity * model->kv_dim) * 2);
    kc->bytes = kc->per_cache * 2 * static_cast<std::size_t>(batch * kc->layers);
    kc->lens.assign(static_cast<std::size_t>(batch), 0);
    cudaError_t err = cudaMalloc(&kc->mem, kc->bytes);
    if (err == cudaSuccess) {
        err = cudaMemset(kc->mem, 0, kc->bytes);
    }
    if (err == cudaSuccess) {
        err = cudaMalloc(&kc->d_ids, static_cast<std::size_t>(kChunkRows) * 8);
    }
    if (err != cudaSuccess) {
        cudaFree(kc->mem);
        cudaFree(kc->d_ids);
        delete kc;
        return rt::cuda_fail(err, "qwen3_cache_create allocation");
    }
    *cache = kc;
    return rt::ok();
}

void cppinf_qwen3_cache_destroy(cppinf_qwen3_cache* cache) {
    if (cache != nullptr) {
        cudaFree(cache->mem);
        cudaFree(cache->d_ids);
        delete cache;
    }
}

int cppinf_qwen3_cache_lengths(const cppinf_qwen3_cache* cache, int64_t* lengths) {
    CPPINF_REQUIRE(cache && lengths, CPPINF_ERR_INVALID_ARGUMENT, "qwen3_cache_lengths received a null pointer.");
    std::memcpy(lengths, cache->lens.data(), cache->lens.size() * sizeof(int64_t));
    return rt::ok();
}

int64_t cppinf_qwen3_cache_batch(const cppinf_qwen3_cache* cache) {
    return cache != nullptr ? cache->batch : -1;
}

int cppinf_qwen3_forward_batch(cppinf_qwen3* model, cppinf_qwen3_cache* cache, const int64_t* token_ids,
                               const int64_t* lengths, int64_t batch, int64_t max_length, void* logits,
                               void* stream) {
    CPPINF_REQUIRE(model && cache, CPPINF_ERR_INVALID_ARGUMENT, "qwen3_forward_batch received a null pointer.");
    CPPINF_REQUIRE(batch > 0, CPPINF_ERR_INVALID_ARGUMENT,
                   "Qwen3Model batched forward requires at least one sequence.");
    CPPINF_REQUIRE(token_ids && lengths && logits, CPPINF_ERR_INVALID_ARGUMENT,
                   "qwen3_forward_batch received a null pointer.");
    CPPINF_REQUIRE(cache->layers == model->c.num_hidden_layers && cache->kv_dim == model->kv_dim,
                   CPPINF_ERR_INVALID_ARGUMENT, "Qwen3Model cache must have one entry per decoder layer.");
    CPPINF_REQUIRE(cache->batch == batch, CPPINF_ERR_INVALID_ARGUMENT,
                   "Qwen3Model cache batch size must match the input batch size.");
    CPPINF_REQUIRE(!model->failed, CPPINF_ERR_CUDA,
                   "qwen3 model state is invalid after a device error; call qwen3_reset first.");
    int64_t longest = 0;
    for (int64_t b = 0; b < batch; ++b) {
        CPPINF_REQUIRE(lengths[b] > 0, CPPINF_ERR_INVALID_ARGUMENT,
                       "Qwen3Model batched forward requires each sequence to contain at least one token.");
        longest = lengths[b] > longest ? lengths[b] : longest;
    }
    CPPINF_REQUIRE(longest <= max_length, CPPINF_ERR_INVALID_ARGUMENT,
                   "qwen3_forward_batch: a sequence is longer than the padded length.");
    for (int64_t b = 0; b < batch; ++b) {
        CPPINF_REQUIRE(cache->lens[static_cast<std::size_t>(b)] + lengths[b] <= cache->cap, CPPINF_ERR_OUT_OF_RANGE,
                       "qwen_attention cache is too small for the new tokens.");
        for (int64_t i = 0; i < lengths[b]; ++i) {
            const int64_t t = token_ids[b * max_length + i];
            CPPINF_REQUIRE(t >= 0 && t < model->c.vocab_size, CPPINF_ERR_OUT_OF_RANGE,
                           "Qwen3Model token id is out of vocabulary range.");
        }
    }
    const auto s = rt::as_stream(stream);
    const int64_t V = model->c.vocab_size;
    bf16* out = static_cast<bf16*>(logits);
    for (int64_t b = 0; b < batch; ++b) {
        if (lengths[b] < max_length) {
            // Right-padded positions: zero logits rows (only the sequences' own rows are results).
            CPPINF_CUDA_TRY(cudaMemsetAsync(out + (b * max_length + lengths[b]) * V, 0,
                                            static_cast<std::size_t>((max_length - lengths[b]) * V) * 2, s));
        }
    }
    // Chunks of up to the workspace's rows, filled with the sequences' rows in order; a sequence longer than the
    // room left continues in the next chunk (its later rows read the earlier ones from the cache).
    const int64_t room = kChunkRows < model->cap ? kChunkRows : model->cap;
    std::vector<Piece> pieces;
    int64_t used = 0;
    for (int64_t b = 0; b < batch; ++b) {
        int64_t start = 0;
        while (start < lengths[b]) {
            const int64_t n = lengths[b] - start < room - used ? lengths[b] - start : room - used;
            pieces.push_back({b, start, n, used});
            start += n;
            used += n;
            if (used == room) {
                QWEN3_CHECK(enqueue_batch_chunk(model, cache, pieces, token_ids, max_length, out, s));
                pieces.clear();
                used = 0;
            }
        }
    }
    if (!pieces.empty()) {
        QWEN3_CHECK(enqueue_batch_chunk(model, cache, pieces, token_ids, max_length, out, s));
    }
    for (int64_t b = 0; b < batch; ++b) {
        cache->lens[static_cast<std::size_t>(b)] += lengths[b];
    }
    return rt::ok();
}

int cppinf_qwen3_decode(cppinf_qwen3* model, int64_t steps, int64_t* tokens, void* stream) {
    CPPINF_REQUIRE(model, CPPINF_ERR_INVALID_ARGUMENT, "qwen3_decode received a null pointer.");
    CPPINF_REQUIRE(steps >= 0, CPPINF_ERR_INVALID_ARGUMENT, "qwen3_decode requires a non-negative step count.");
    if (steps == 0) {
        return rt::ok();
    }
    CPPINF_REQUIRE(tokens, CPPINF_ERR_INVALID_ARGUMENT, "qwen3_decode received a null pointer.");
    CPPINF_REQUIRE(!model->failed, CPPINF_ERR_CUDA,
                   "qwen3 model state is invalid after a device error; call qwen3_reset first.");
    CPPINF_REQUIRE(model->len > 0, CPPINF_ERR_INVALID_ARGUMENT,
                   "qwen3_decode needs a forward call first (the cache is empty).");
    CPPINF_REQUIRE(model->len + steps <= model->cap, CPPINF_ERR_OUT_OF_RANGE,
                   "qwen_attention cache is too small for the new tokens.");
    const auto s = rt::as_stream(stream);
    if (model->step != nullptr && model->step_poll_limit != rt::wait_poll_limit()) {
        // The wait poll limit changed since the steps were captured: capture them again with the current one (an
        // executable graph still in flight is freed when it completes).
        cudaGraphExecDestroy(model->step);
        model->step = nullptr;
        if (model->step_block != nullptr) {
            cudaGraphExecDestroy(model->step_block);
            model->step_block = nullptr;
        }
    }
    if (model->step == nullptr) {
        model->step_poll_limit = rt::wait_poll_limit();
        if (const int st = capture_steps(model, 1, &model->step, &model->step_launches); st != CPPINF_OK) {
            return st;
        }
    }
    if (steps >= kBlockSteps && model->step_block == nullptr) {
        if (const int st = capture_steps(model, kBlockSteps, &model->step_block, &model->step_block_launches);
            st != CPPINF_OK) {
            return st;
        }
    }
    int64_t i = 0;
    for (; i + kBlockSteps <= steps; i += kBlockSteps) {
        CPPINF_CUDA_TRY(cudaGraphLaunch(model->step_block, s));
        rt::count_launches(model->step_block_launches);
    }
    for (; i < steps; ++i) {
        CPPINF_CUDA_TRY(cudaGraphLaunch(model->step, s));
        rt::count_launches(model->step_launches);
    }
    unsigned int error = 0;
    CPPINF_CUDA_TRY(cudaMemcpyAsync(tokens, model->d_tokens + model->len + 1, static_cast<std::size_t>(steps) * 8,
                                    cudaMemcpyDeviceToHost, s));
    CPPINF_CUDA_TRY(cudaMemcpyAsync(&error, model->d_error, sizeof(error), cudaMemcpyDeviceToHost, s));
    CPPINF_CUDA_TRY(cudaStreamSynchronize(s));
    if (error != 0) {
        // The device advanced its sequence length but the tokens are not valid: the model needs a reset.
        model->failed = true;
        return rt::fail(CPPINF_ERR_CUDA,
                        "qwen3_decode: a device wait for staged data ran out of its poll limit; results are invalid "
                        "(call qwen3_reset).");
    }
    model->len += steps;
    return rt::ok();
}

}  // extern "C"
