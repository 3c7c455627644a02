// RMSNorm over the last dimension, ops::rms_norm (src/ops/nn_ops.cpp:140-201), and the residual add + RMSNorm pair
// of the decoder block (src/nn/qwen_decoder_block.cpp:80-84 and :89 feeding the next layer's :73).
//
// The reference runs nine oneDNN passes: cast to f32, x*x, reduction_mean, +eps, sqrt, 1/rms, x*inv, *w, cast. Here
// one warp owns one row: the row is read once into registers (16-byte vectors), the sum of squares is reduced with a
// butterfly, and the normalised row is written once. Per element the arithmetic is the reference's, in its order,
// each step rounded to f32: mean = sum / width, var = mean + eps, rms = sqrt(var), inv = 1 / rms, n = x * inv,
// r = n * w, then r rounded to the output dtype.
//
// Reduction order (oneDNN leaves it unspecified): the row is cut into chunks of `chunk` consecutive elements
// (16 bytes on the vector path, 1 element on the scalar path). Lane l sums, in increasing element order, the squares
// of chunks l, l+32, l+64, ...; the 32 lane partials are then combined by a butterfly over lane distances 16, 8, 4,
// 2, 1. The CPU oracle restates exactly this order.
//
// Roofline: HBM-bound. Algorithmic bytes per row: read width*size (x) [+ width*size (b)], write width*size (y)
// [+ width*size (sum)], plus the weight once per launch.
#include "common.cuh"
#include "runtime.h"

namespace cppinf::device {
namespace {

constexpr int kThreads = 128;
constexpr int kWarps = kThreads / 32;

struct RmsParams {
    const void* x;  // rows of x (or addend a)
    const void* b;  // addend b (fused residual only)
    const void* w;  // weight [width]
    void* sum;      // residual output (fused residual only)
    void* y;        // output
    int64_t rows;
    int64_t x_stride;  // elements between consecutive rows of x
    int width;
    float eps;
};

// Register-resident variant: each lane holds kChunks 16-byte vectors of its row.
template <typename T, int kChunks, bool kAdd>
__global__ void __launch_bounds__(kThreads) rms_norm_regs_kernel(RmsParams p) {
    using V = Vec16<T>;
    constexpr int kVec = V::kVec;
    const int lane = threadIdx.x & 31;
    const int nchunks = p.width / kVec;
    const float width_f = static_cast<float>(p.width);
    const int64_t warp_stride = static_cast<int64_t>(gridDim.x) * kWarps;
    // Before the dependency wait (while the previous kernel still runs), lane 0 asks L2 for the warp's first row
    // (and its addend row). A prefetch returns no data and L2 is the point of coherence, so the loads after the wait
    // still see what the previous kernel writes. Also prefetching the row half a grid away (which helps the q/k
    // kernel) measured slower here: 6.75 -> 7.29 us on [4096, 1024] bf16.
    const int64_t first_row = static_cast<int64_t>(blockIdx.x) * kWarps + threadIdx.x / 32;
    if (lane == 0 && first_row < p.rows) {
        const auto row_bytes = static_cast<uint32_t>(p.width * static_cast<int>(sizeof(T)));
        bulk_prefetch_l2(static_cast<const char*>(p.x) + first_row * p.x_stride * static_cast<int64_t>(sizeof(T)),
                         row_bytes);
        if constexpr (kAdd) {
            bulk_prefetch_l2(static_cast<const char*>(p.b) + first_row * p.width * static_cast<int64_t>(sizeof(T)),
                             row_bytes);
        }
    }
    grid_dependency_begin();

    for (int64_t row = static_cast<int64_t>(blockIdx.x) * kWarps + threadIdx.x / 32; row < p.rows;
         row += warp_stride) {
        const char* xr = static_cast<const char*>(p.x) + row * p.x_stride * static_cast<int64_t>(sizeof(T));
        const char* br = kAdd ? static_cast<const char*>(p.b) + row * p.width * static_cast<int64_t>(sizeof(T)) : nullptr;
        uint4 raw[kChunks];
        uint4 raw_b[kChunks];
#pragma unroll
        for (int i = 0; i < kChunks; ++i) {
            const int c = lane + 32 * i;
            if (c < nchunks) {
                raw[i] = ld_stream(xr + c * 16);
                if constexpr (kAdd) {
                    raw_b[i] = ld_stream(br + c * 16);
                }
            }
        }

        float ss = 0.0f;
        float vals[kChunks][kVec];
#pragma unroll
        for (int i = 0; i < kChunks; ++i) {
            const int c = lane + 32 * i;
            if (c < nchunks) {
                V::unpack(raw[i], vals[i]);
                if constexpr (kAdd) {
                    float bv[kVec];
                    V::unpack(raw_b[i], bv);
#pragma unroll
                    for (int j = 0; j < kVec; ++j) {
                        vals[i][j] = V::quantize(vals[i][j] + bv[j]);
                    }
                    char* sr = static_cast<char*>(p.sum) + row * p.width * static_cast<int64_t>(sizeof(T));
                    st_stream(sr + c * 16, V::pack(vals[i]));
                }
#pragma unroll
                for (int j = 0; j < kVec; ++j) {
                    ss = sum_square<T>(ss, vals[i][j]);
                }
            }
        }
        ss = group_sum<32>(ss);
        const float mean = ss / width_f;
        const float rms = sqrtf(mean + p.eps);
        const float inv = 1.0f / rms;

        char* yr = static_cast<char*>(p.y) + row * p.width * static_cast<int64_t>(sizeof(T));
#pragma unroll
        for (int i = 0; i < kChunks; ++i) {
            const int c = lane + 32 * i;
            if (c < nchunks) {
                float wv[kVec];
                V::unpack(ld_cached(static_cast<const char*>(p.w) + c * 16), wv);
                float out[kVec];
#pragma unroll
                for (int j = 0; j < kVec; ++j) {
                    out[j] = (vals[i][j] * inv) * wv[j];
                }
                st_stream(yr + c * 16, V::pack(out));
            }
        }
    }
}

// Streaming variant for any width: pass 1 accumulates the squares (and writes the residual sum), pass 2 re-reads the
// row (from L2) and writes the output. `chunk` is the number of consecutive elements a lane takes per step: the
// 16-byte vector width, or 1 when the operands are not vector-aligned.
template <typename T, bool kAdd>
__global__ void __launch_bounds__(kThreads) rms_norm_stream_kernel(RmsParams p, int chunk) {
    grid_dependency_begin();
    using V = Vec16<T>;
    const int lane = threadIdx.x & 31;
    const float width_f = static_cast<float>(p.width);
    const int64_t warp_stride = static_cast<int64_t>(gridDim.x) * kWarps;
    const int nchunks = p.width / chunk;

    for (int64_t row = static_cast<int64_t>(blockIdx.x) * kWarps + threadIdx.x / 32; row < p.rows;
         row += warp_stride) {
        const int64_t x_base = row * p.x_stride;
        const int64_t d_base = row * static_cast<int64_t>(p.width);
        float ss = 0.0f;
        for (int c = lane; c < nchunks; c += 32) {
            for (int j = 0; j < chunk; ++j) {
                const int e = c * chunk + j;
                float v = V::load1(p.x, x_base + e);
                if constexpr (kAdd) {
                    v = V::quantize(v + V::load1(p.b, d_base + e));
                    V::store1(p.sum, d_base + e, v);
                }
                ss = sum_square<T>(ss, v);
            }
        }
        ss = group_sum<32>(ss);
        const float mean = ss / width_f;
        const float rms = sqrtf(mean + p.eps);
        const float inv = 1.0f / rms;
        __syncwarp();
        for (int e = lane; e < p.width; e += 32) {
            // The fused variant re-reads the rounded sum it wrote in pass 1 (same thread, program order).
            const float v = kAdd ? V::load1(p.sum, d_base + e) : V::load1(p.x, x_base + e);
            V::store1(p.y, d_base + e, (v * inv) * V::load1(p.w, e));
        }
    }
}

template <typename T, bool kAdd>
int launch_rms(const RmsParams& p, bool vector_ok, void* stream, const char* name) {
    constexpr int kVec = Vec16<T>::kVec;
    const int64_t per_sm = runtime::max_threads_per_sm() / kThreads;
    const int64_t wave = static_cast<int64_t>(runtime::sm_count()) * (per_sm > 0 ? per_sm : 1);
    const int64_t needed = runtime::ceil_div(p.rows, kWarps);
    const auto blocks = static_cast<unsigned>(needed < wave ? needed : wave);
    auto s = runtime::as_stream(stream);
    const int chunks_per_lane = static_cast<int>(runtime::ceil_div(p.width / kVec, 32));
    cudaError_t launch_err;
    if (vector_ok && chunks_per_lane <= 8) {
        if (chunks_per_lane <= 1) {
            launch_err = ::cppinf::runtime::launch(rms_norm_regs_kernel<T, 1, kAdd>, dim3(blocks), dim3(kThreads), s, 1u, p);
        } else if (chunks_per_lane <= 2) {
            launch_err = ::cppinf::runtime::launch(rms_norm_regs_kernel<T, 2, kAdd>, dim3(blocks), dim3(kThreads), s, 1u, p);
        } else if (chunks_per_lane <= 4) {
            launch_err = ::cppinf::runtime::launch(rms_norm_regs_kernel<T, 4, kAdd>, dim3(blocks), dim3(kThreads), s, 1u, p);
        } else {
            launch_err = ::cppinf::runtime::launch(rms_norm_regs_kernel<T, 8, kAdd>, dim3(blocks), dim3(kThreads), s, 1u, p);
        }
    } else {
        launch_err = ::cppinf::runtime::launch(rms_norm_stream_kernel<T, kAdd>, dim3(blocks), dim3(kThreads), s, 1u, p, vector_ok ? kVec : 1);
    }
    return runtime::launched(launch_err, name);
}

int validate_rows(cppinf_dtype dtype, int64_t rows, int64_t width, float eps, const char* op) {
    CPPINF_REQUIRE(runtime::valid_dtype(dtype), CPPINF_ERR_INVALID_ARGUMENT,
                   std::string(op) + " received an unsupported dtype.");
    CPPINF_REQUIRE(width > 0, CPPINF_ERR_INVALID_ARGUMENT,
                   std::string(op) + " requires a non-empty last dimension.");
    CPPINF_REQUIRE(width <= (int64_t{1} << 30), CPPINF_ERR_UNSUPPORTED,
                   std::string(op) + " supports rows of at most 2^30 elements.");
    CPPINF_REQUIRE(rows >= 0, CPPINF_ERR_INVALID_ARGUMENT, std::string(op) + " requires a non-negative row count.");
    CPPINF_REQUIRE(eps >= 0.0f, CPPINF_ERR_INVALID_ARGUMENT, "rms_norm requires a non-negative epsilon.");
    return CPPINF_OK;
}

}  // namespace
}  // namespace cppinf::device

using namespace cppinf::device;
namespace rt = cppinf::runtime;

extern "C" {

int cppinf_rms_norm(cppinf_dtype dtype, const void* x, int64_t x_row_stride, const void* weight, void* y,
                    int64_t rows, int64_t width, float eps, void* stream) {
    if (const int st = validate_rows(dtype, rows, width, eps, "rms_norm"); st != CPPINF_OK) {
        return st;
    }
    CPPINF_REQUIRE(rows <= 1 || x_row_stride >= width, CPPINF_ERR_INVALID_ARGUMENT,
                   "rms_norm requires a row stride of at least the width.");
    if (rows == 0) {
        return rt::ok();
    }
    CPPINF_REQUIRE(x && weight && y, CPPINF_ERR_INVALID_ARGUMENT, "rms_norm received a null pointer.");
    RmsParams p{x, nullptr, weight, nullptr, y, rows, x_row_stride, static_cast<int>(width), eps};
    const int vec = dtype == CPPINF_DTYPE_BF16 ? 8 : 4;
    const bool vector_ok = width % vec == 0 && x_row_stride % vec == 0 && rt::aligned16(x) && rt::aligned16(weight) &&
                           rt::aligned16(y);
    if (dtype == CPPINF_DTYPE_BF16) {
        return launch_rms<bf16, false>(p, vector_ok, stream, "rms_norm");
    }
    return launch_rms<float, false>(p, vector_ok, stream, "rms_norm");
}

int cppinf_add_rms_norm(cppinf_dtype dtype, const void* a, const void* b, const void* weight, void* sum, void* y,
                        int64_t rows, int64_t width, float eps, void* stream) {
    if (const int st = validate_rows(dtype, rows, width, eps, "add_rms_norm"); st != CPPINF_OK) {
        return st;
    }
    if (rows == 0) {
        return rt::ok();
    }
    CPPINF_REQUIRE(a && b && weight && sum && y, CPPINF_ERR_INVALID_ARGUMENT,
                   "add_rms_norm received a null pointer.");
    RmsParams p{a, b, weight, sum, y, rows, width, static_cast<int>(width), eps};
    const int vec = dtype == CPPINF_DTYPE_BF16 ? 8 : 4;
    const bool vector_ok = width % vec == 0 && rt::aligned16(a) && rt::aligned16(b) && rt::aligned16(weight) &&
                           rt::aligned16(sum) && rt::aligned16(y);
    if (dtype == CPPINF_DTYPE_BF16) {
        return launch_rms<bf16, true>(p, vector_ok, stream, "add_rms_norm");
    }
    return launch_rms<float, true>(p, vector_ok, stream, "add_rms_norm");
}

}  // extern "C"
