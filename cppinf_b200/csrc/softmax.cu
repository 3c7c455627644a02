// Row softmax kernels:
//  - ops::softmax_last_dim (src/ops/nn_ops.cpp:50-75, oneDNN softmax_accurate), bf16 or f32 in and out;
//  - ops::scaled_causal_softmax_last_dim (src/ops/nn_ops.cpp:77-138), f32 [matrices, Q, K] with Q == K;
//  - the position-aware variant of attention, scaled_position_causal_softmax_last_dim
//    (src/nn/qwen_attention.cpp:164-235), f32 [batch, heads, Qcap, Kcap] with per-batch offsets and lengths.
//
// One warp owns one row. Only the visible prefix of a row is read (32- or 16-byte chunks into registers); the whole row is
// written, masked columns included. Per row, following the reference: m = max over visible k of (x*scale),
// e_k = exp(x_k*scale - m) for visible k and 0 otherwise, sum = sum of e, out_k = e_k / sum. Masked columns hold
// 0 / sum, which is 0 unless the sum is NaN, as in the reference's division loop. The position-aware variant writes
// 0 everywhere when the sum is 0 (a row with no visible key, or a query row past the query length).
//
// The sum is a per-lane partial followed by a butterfly, so it differs from the reference's left-to-right f32 sum
// only by rounding (f32 results agree to about 1e-6 relative). exp is CUDA's expf (max 2 ulp), the reference's
// std::exp is glibc expf.
//
// Roofline: HBM-bound. Algorithmic bytes per row: visible elements read + the full row written.
#include <cmath>

#include "common.cuh"
#include "runtime.h"

namespace cppinf::device {
namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kMaxBatch = 64;

// Visibility rules: visible(row) is the number of leading visible columns, zero_row(row) says whether the row is
// written as zeros regardless of the sum.
struct FullRows {
    int64_t width;
    __device__ __forceinline__ int64_t visible(int64_t) const { return width; }
    static constexpr bool kZeroOnEmpty = false;
};

struct SquareCausalRows {
    int64_t query_len;
    __device__ __forceinline__ int64_t visible(int64_t row) const { return row % query_len + 1; }
    static constexpr bool kZeroOnEmpty = false;
};

struct PositionCausalRows {
    int64_t query_cap;
    int64_t key_cap;
    int64_t heads;
    int64_t query_offsets[kMaxBatch];
    int64_t query_lengths[kMaxBatch];
    int64_t key_lengths[kMaxBatch];
    __device__ __forceinline__ int64_t visible(int64_t row) const {
        const int64_t q = row % query_cap;
        const int64_t b = row / query_cap / heads;
        if (q >= query_lengths[b]) {
            return 0;
        }
        const int64_t causal = query_offsets[b] + q + 1;
        const int64_t keys = key_lengths[b];
        return causal < keys ? causal : keys;
    }
    static constexpr bool kZeroOnEmpty = true;
};

// Pairwise (tree) max / sum of one chunk of kN values (kN a power of two).
template <int kN>
__device__ __forceinline__ float tree_max(const float (&v)[kN]) {
    float t[kN];
#pragma unroll
    for (int i = 0; i < kN; ++i) {
        t[i] = v[i];
    }
#pragma unroll
    for (int width = kN / 2; width > 0; width /= 2) {
#pragma unroll
        for (int i = 0; i < width; ++i) {
            t[i] = fmaxf(t[2 * i], t[2 * i + 1]);
        }
    }
    return t[0];
}

template <int kN>
__device__ __forceinline__ float tree_sum(const float (&v)[kN]) {
    float t[kN];
#pragma unroll
    for (int i = 0; i < kN; ++i) {
        t[i] = v[i];
    }
#pragma unroll
    for (int width = kN / 2; width > 0; width /= 2) {
#pragma unroll
        for (int i = 0; i < width; ++i) {
            t[i] = t[2 * i] + t[2 * i + 1];
        }
    }
    return t[0];
}

// Rows of at most 32 * kChunks * kVec elements (<= 4096), so element indices fit 32 bits. At most 128 registers per
// thread (two blocks per SM): the row occupies kChunks * kVec of them.
template <typename T, int kBytes, int kChunks, typename Rows>
__global__ void __launch_bounds__(kThreads, 2) softmax_regs_kernel(const void* __restrict__ x, void* __restrict__ y,
                                                                   int64_t rows, int64_t width, float scale,
                                                                   Rows rule) {
    grid_dependency_begin();
    using V = Chunk<T, kBytes>;
    constexpr int kVec = V::kElems;
    const int lane = threadIdx.x & 31;
    const int64_t warp_stride = static_cast<int64_t>(gridDim.x) * kWarps;
    const int nchunks = static_cast<int>(width / kVec);

    for (int64_t row = static_cast<int64_t>(blockIdx.x) * kWarps + threadIdx.x / 32; row < rows; row += warp_stride) {
        const int n = static_cast<int>(rule.visible(row));
        const int vis_chunks = (n + kVec - 1) / kVec;
        const char* xr = static_cast<const char*>(x) + row * width * static_cast<int64_t>(sizeof(T));
        char* yr = static_cast<char*>(y) + row * width * static_cast<int64_t>(sizeof(T));

        float v[kChunks][kVec];
#pragma unroll
        for (int i = 0; i < kChunks; ++i) {
            const int c = lane + 32 * i;
            if (c < vis_chunks) {
                V::load(xr + c * kBytes, v[i]);
            }
        }
        // Scaled values; only the chunk that straddles the visibility boundary needs per-element masks. Each chunk
        // is reduced as a small tree into one of two running accumulators, which keeps dependency chains short.
        // The masked tail of the chunk that straddles the boundary becomes -inf, so exp turns it into 0 (or NaN
        // exactly when the row's maximum is -inf, where the reference's 0 / sum is NaN too).
        float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
        for (int i = 0; i < kChunks; ++i) {
            const int c = lane + 32 * i;
            if (c < vis_chunks) {
#pragma unroll
                for (int j = 0; j < kVec; ++j) {
                    v[i][j] = v[i][j] * scale;
                }
                if ((c + 1) * kVec > n) {
#pragma unroll
                    for (int j = 0; j < kVec; ++j) {
                        v[i][j] = c * kVec + j < n ? v[i][j] : -INFINITY;
                    }
                }
                mx[i & 1] = fmaxf(mx[i & 1], tree_max<kVec>(v[i]));
            }
        }
        const float m = group_max<32>(fmaxf(mx[0], mx[1]));

        float acc[2] = {0.0f, 0.0f};
#pragma unroll
        for (int i = 0; i < kChunks; ++i) {
            const int c = lane + 32 * i;
            if (c < vis_chunks) {
#pragma unroll
                for (int j = 0; j < kVec; ++j) {
                    v[i][j] = expf(v[i][j] - m);
                }
                acc[i & 1] = acc[i & 1] + tree_sum<kVec>(v[i]);
            }
        }
        const float sum = group_sum<32>(acc[0] + acc[1]);
        const bool zero_row = Rows::kZeroOnEmpty && sum == 0.0f;
        const float masked = zero_row ? 0.0f : 0.0f / sum;
        // One division per row; each probability is e * (1 / sum), within one f32 ulp of e / sum.
        const float inv = zero_row ? 0.0f : 1.0f / sum;

#pragma unroll
        for (int i = 0; i < kChunks; ++i) {
            const int c = lane + 32 * i;
            if (c < nchunks) {
                float out[kVec];
                if (c < vis_chunks) {
#pragma unroll
                    for (int j = 0; j < kVec; ++j) {
                        out[j] = v[i][j] * inv;
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < kVec; ++j) {
                        out[j] = masked;
                    }
                }
                V::store(yr + static_cast<int64_t>(c) * kBytes, out);
            }
        }
    }
}

// Any width or alignment: three passes over the row (max, sum, write), element by element. Later passes re-read
// the row from L2.
template <typename T, typename Rows>
__global__ void __launch_bounds__(kThreads) softmax_stream_kernel(const void* __restrict__ x, void* __restrict__ y,
                                                                  int64_t rows, int64_t width, float scale,
                                                                  Rows rule) {
    grid_dependency_begin();
    using V = Vec16<T>;
    const int lane = threadIdx.x & 31;
    const int64_t warp_stride = static_cast<int64_t>(gridDim.x) * kWarps;
    for (int64_t row = static_cast<int64_t>(blockIdx.x) * kWarps + threadIdx.x / 32; row < rows; row += warp_stride) {
        const int64_t n = rule.visible(row);
        const int64_t base = row * width;
        float m = -INFINITY;
        for (int64_t k = lane; k < n; k += 32) {
            m = fmaxf(m, V::load1(x, base + k) * scale);
        }
        m = group_max<32>(m);
        float sum = 0.0f;
        for (int64_t k = lane; k < n; k += 32) {
            sum = sum + expf(V::load1(x, base + k) * scale - m);
        }
        sum = group_sum<32>(sum);
        const bool zero_row = Rows::kZeroOnEmpty && sum == 0.0f;
        const float masked = zero_row ? 0.0f : 0.0f / sum;
        for (int64_t k = lane; k < width; k += 32) {
            float out = masked;
            if (k < n && !zero_row) {
                out = expf(V::load1(x, base + k) * scale - m) / sum;
            }
            V::store1(y, base + k, out);
        }
    }
}

template <typename T, typename Rows>
int launch_softmax(const void* x, void* y, int64_t rows, int64_t width, float scale, const Rows& rule, void* stream,
                   const char* name) {
    constexpr int kVec = Vec16<T>::kVec;
    const int64_t per_sm = runtime::max_threads_per_sm() / kThreads;
    const int64_t wave = static_cast<int64_t>(runtime::sm_count()) * (per_sm > 0 ? per_sm : 1) * 4;
    const int64_t needed = runtime::ceil_div(rows, kWarps);
    const auto blocks = static_cast<unsigned>(needed < wave ? needed : wave);
    const auto s = runtime::as_stream(stream);
    // 32-byte chunks when rows are 32-byte aligned, else 16-byte chunks, else the element-wise streaming kernel.
    // A lane holds at most 64 f32 row values in registers.
    const bool rows32 = width % (32 / static_cast<int64_t>(sizeof(T))) == 0 &&
                        (reinterpret_cast<std::uintptr_t>(x) & 31u) == 0 && (reinterpret_cast<std::uintptr_t>(y) & 31u) == 0;
    const bool rows16 = width % kVec == 0 && runtime::aligned16(x) && runtime::aligned16(y);
    constexpr int kElems32 = 32 / static_cast<int>(sizeof(T));
    const int64_t per_lane32 = runtime::ceil_div(width / kElems32, 32);
    const int64_t per_lane16 = runtime::ceil_div(width / kVec, 32);
    cudaError_t launch_err;
    if (rows32 && per_lane32 * kElems32 <= 64) {
        if (per_lane32 <= 1) {
            launch_err = runtime::launch(softmax_regs_kernel<T, 32, 1, Rows>, dim3(blocks), dim3(kThreads), s, 1u, x, y,
                                         rows, width, scale, rule);
        } else if (per_lane32 <= 2) {
            launch_err = runtime::launch(softmax_regs_kernel<T, 32, 2, Rows>, dim3(blocks), dim3(kThreads), s, 1u, x, y,
                                         rows, width, scale, rule);
        } else if (per_lane32 <= 4) {
            launch_err = runtime::launch(softmax_regs_kernel<T, 32, 4, Rows>, dim3(blocks), dim3(kThreads), s, 1u, x, y,
                                         rows, width, scale, rule);
        } else {
            constexpr int kMax = 64 / kElems32;  // 8 chunks of f32; bf16 never gets here (4 * 16 = 64)
            launch_err = runtime::launch(softmax_regs_kernel<T, 32, kMax, Rows>, dim3(blocks), dim3(kThreads), s, 1u, x,
                                         y, rows, width, scale, rule);
        }
    } else if (rows16 && per_lane16 * kVec <= 64) {
        if (per_lane16 <= 2) {
            launch_err = runtime::launch(softmax_regs_kernel<T, 16, 2, Rows>, dim3(blocks), dim3(kThreads), s, 1u, x, y,
                                         rows, width, scale, rule);
        } else {
            constexpr int kMax = 64 / kVec;  // 16 chunks of f32, 8 of bf16
            launch_err = runtime::launch(softmax_regs_kernel<T, 16, kMax, Rows>, dim3(blocks), dim3(kThreads), s, 1u, x,
                                         y, rows, width, scale, rule);
        }
    } else {
        launch_err = runtime::launch(softmax_stream_kernel<T, Rows>, dim3(blocks), dim3(kThreads), s, 1u, x, y, rows,
                                     width, scale, rule);
    }
    return runtime::launched(launch_err, name);
}

}  // namespace
}  // namespace cppinf::device

using namespace cppinf::device;
namespace rt = cppinf::runtime;

extern "C" {

int cppinf_softmax_last_dim(cppinf_dtype dtype, const void* x, void* y, int64_t rows, int64_t width, void* stream) {
    CPPINF_REQUIRE(rt::valid_dtype(dtype), CPPINF_ERR_INVALID_ARGUMENT,
                   "softmax_last_dim received an unsupported dtype.");
    CPPINF_REQUIRE(width > 0, CPPINF_ERR_INVALID_ARGUMENT, "softmax_last_dim requires a non-empty last dimension.");
    CPPINF_REQUIRE(rows >= 0, CPPINF_ERR_INVALID_ARGUMENT, "softmax_last_dim requires a non-negative row count.");
    if (rows == 0) {
        return rt::ok();
    }
    CPPINF_REQUIRE(x && y, CPPINF_ERR_INVALID_ARGUMENT, "softmax_last_dim received a null pointer.");
    const FullRows rule{width};
    if (dtype == CPPINF_DTYPE_BF16) {
        return launch_softmax<bf16>(x, y, rows, width, 1.0f, rule, stream, "softmax_last_dim");
    }
    return launch_softmax<float>(x, y, rows, width, 1.0f, rule, stream, "softmax_last_dim");
}

int cppinf_scaled_causal_softmax_f32(const float* x, float* y, int64_t matrices, int64_t query_len, int64_t key_len,
                                     float scale, void* stream) {
    CPPINF_REQUIRE(std::isfinite(scale), CPPINF_ERR_INVALID_ARGUMENT,
                   "scaled_causal_softmax_last_dim requires a finite scale.");
    CPPINF_REQUIRE(matrices >= 0 && query_len >= 0 && key_len >= 0, CPPINF_ERR_INVALID_ARGUMENT,
                   "scaled_causal_softmax_last_dim requires non-negative sizes.");
    CPPINF_REQUIRE(query_len > 0 && key_len > 0, CPPINF_ERR_INVALID_ARGUMENT,
                   "scaled_causal_softmax_last_dim requires non-empty attention dimensions.");
    CPPINF_REQUIRE(query_len == key_len, CPPINF_ERR_INVALID_ARGUMENT,
                   "scaled_causal_softmax_last_dim requires square attention score matrices.");
    if (matrices == 0) {
        return rt::ok();
    }
    CPPINF_REQUIRE(x && y, CPPINF_ERR_INVALID_ARGUMENT, "scaled_causal_softmax_last_dim received a null pointer.");
    const SquareCausalRows rule{query_len};
    return launch_softmax<float>(x, y, matrices * query_len, key_len, scale, rule, stream,
                                 "scaled_causal_softmax_last_dim");
}

int cppinf_scaled_position_causal_softmax_f32(const float* x, float* y, int64_t batch, int64_t heads,
                                              int64_t query_cap, int64_t key_cap, float scale,
                                              const int64_t* query_offsets, const int64_t* query_lengths,
                                              const int64_t* key_lengths, void* stream) {
    CPPINF_REQUIRE(std::isfinite(scale), CPPINF_ERR_INVALID_ARGUMENT,
                   "qwen_attention batched softmax requires a finite scale.");
    CPPINF_REQUIRE(batch > 0, CPPINF_ERR_INVALID_ARGUMENT, "qwen_attention batch size must be non-zero.");
    CPPINF_REQUIRE(heads > 0, CPPINF_ERR_INVALID_ARGUMENT, "qwen_attention head count must be non-zero.");
    CPPINF_REQUIRE(query_cap > 0, CPPINF_ERR_INVALID_ARGUMENT, "qwen_attention query length must be non-zero.");
    CPPINF_REQUIRE(key_cap > 0, CPPINF_ERR_INVALID_ARGUMENT, "qwen_attention key length must be non-zero.");
    CPPINF_REQUIRE(batch <= kMaxBatch, CPPINF_ERR_UNSUPPORTED,
                   "scaled_position_causal_softmax supports at most 64 batch rows per call.");
    CPPINF_REQUIRE(query_offsets && query_lengths && key_lengths, CPPINF_ERR_INVALID_ARGUMENT,
                   "qwen_attention sequence_lengths must match the batch size.");
    PositionCausalRows rule{};
    rule.query_cap = query_cap;
    rule.key_cap = key_cap;
    rule.heads = heads;
    for (int64_t b = 0; b < batch; ++b) {
        CPPINF_REQUIRE(query_offsets[b] >= 0, CPPINF_ERR_INVALID_ARGUMENT,
                       "qwen_attention query offsets must be non-negative.");
        CPPINF_REQUIRE(query_lengths[b] >= 0 && query_lengths[b] <= query_cap, CPPINF_ERR_INVALID_ARGUMENT,
                       "qwen_attention query lengths sequence length exceeds the padded sequence capacity.");
        CPPINF_REQUIRE(key_lengths[b] >= 0 && key_lengths[b] <= key_cap, CPPINF_ERR_INVALID_ARGUMENT,
                       "qwen_attention key lengths sequence length exceeds the padded sequence capacity.");
        rule.query_offsets[b] = query_offsets[b];
        rule.query_lengths[b] = query_lengths[b];
        rule.key_lengths[b] = key_lengths[b];
    }
    CPPINF_REQUIRE(x && y, CPPINF_ERR_INVALID_ARGUMENT, "qwen_attention batched softmax received a null pointer.");
    return launch_softmax<float>(x, y, batch * heads * query_cap, key_cap, scale, rule, stream,
                                 "scaled_position_causal_softmax_last_dim");
}

}  // extern "C"
