// Linear projections of the Qwen3 decoder: y = x W^T with W [out_features, in_features] in bf16, the
// linear_project of src/nn/qwen_common.cpp:15-37 (ops::matmul, src/ops/matmul.cpp:85-114, bf16 in, bf16 out).
//
// Accumulation order (shared with the CPU oracle, so greedy tokens are compared bit for bit): one warp owns an
// output; its row is cut into 16-byte chunks of 8 elements, lane l adds the products of chunks l, l + 32, ... in
// increasing element order starting from +0, and the 32 partials are combined by a butterfly over lane distances
// 16 .. 1 -- the same order as the RMSNorm sum of squares. A product of two bf16 values is exact in f32, so every
// step is one rounded f32 addition. The result is rounded to bf16 once.
//
// Two kernels:
//  - gemv_kernel (one input row, the decode step): each warp streams whole weight rows with 16 loads of 16 bytes
//    per lane in flight. The first batch of weights is loaded before griddepcontrol.wait, so under programmatic
//    dependent launch it overlaps the previous kernel's tail (weights never depend on it). Fused prologues: the
//    embedding gather of the token at the device-side position and ops::rms_norm of the input row; fused epilogues:
//    segment stores (q | k | v, v straight into the KV cache), residual add, SiLU(gate) * up, and the greedy argmax
//    over the vocabulary (the last CTA to finish combines the per-CTA maxima).
//  - linear_rows_kernel (prefill): tiles of 16 input rows staged in shared memory; each weight chunk a lane loads
//    is unpacked once and used for the 16 rows.
//
// Roofline: the decode projections are HBM-bound on the weights (N * K * 2 bytes per token); the prefill tiles are
// bound by f32 issue (two instructions per multiply-add with separately rounded operations).
#include <mutex>
#include <string>

#include <type_traits>

#include "common.cuh"
#include "decoder.h"
#include "pexp.cuh"
#include "runtime.h"

namespace cppinf::device {
namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kLoads = 16;  // 16-byte weight loads a lane keeps in flight in the single-row kernel
constexpr int kTileRows = 16;

// One 16-byte chunk of the canonical dot product: 8 fused multiply-adds in element order (fma_bf16x8, common.cuh).
__device__ __forceinline__ float dot_chunk(uint4 x, uint4 w, float acc) {
    return fma_bf16x8(x, w, acc);
}

// Same products with the weight chunk already unpacked (exact f32 copies of bf16 values).
__device__ __forceinline__ float dot_chunk(uint4 x, const float (&w)[8], float acc) {
    acc = __fmaf_rn(bf16_lo(x.x), w[0], acc);
    acc = __fmaf_rn(bf16_hi(x.x), w[1], acc);
    acc = __fmaf_rn(bf16_lo(x.y), w[2], acc);
    acc = __fmaf_rn(bf16_hi(x.y), w[3], acc);
    acc = __fmaf_rn(bf16_lo(x.z), w[4], acc);
    acc = __fmaf_rn(bf16_hi(x.z), w[5], acc);
    acc = __fmaf_rn(bf16_lo(x.w), w[6], acc);
    acc = __fmaf_rn(bf16_hi(x.w), w[7], acc);
    return acc;
}

__device__ __forceinline__ int64_t clamp_token(int64_t t, int64_t vocab) {
    return t < 0 ? 0 : (t >= vocab ? vocab - 1 : t);
}

// Start of input row m (after the optional embedding gather).
__device__ __forceinline__ const bf16* input_row(const LinearParams& p, int64_t m, int64_t token_base) {
    if (p.tokens != nullptr) {
        return reinterpret_cast<const bf16*>(p.x) + clamp_token(p.tokens[token_base + m], p.vocab) * p.x_stride;
    }
    return reinterpret_cast<const bf16*>(p.x) + m * p.x_stride;
}

__device__ __forceinline__ void store_segment(const LinearParams& p, int64_t m, int64_t n, float v, int64_t pos) {
    const int k = n >= p.seg[2] ? 2 : (n >= p.seg[1] ? 1 : 0);
    const int64_t row = m + p.row_offset[k] + (k == 2 ? pos : 0);
    Vec16<bf16>::store1(p.out[k], row * p.ld[k] + (n - p.seg[k]), v);
}

// Argmax key of a bf16 logit (the reference compares the stored bf16 values): larger value first, then lower index;
// NaN never wins; a NaN at index 0 forces index 0 (the reference's scan never replaces its starting element).
__device__ __forceinline__ unsigned long long logit_key(float v, int64_t n) {
    uint32_t u = __float_as_uint(v);
    if ((u & 0x7fffffffu) > 0x7f800000u) {
        return n == 0 ? ~0ull : 0ull;
    }
    if ((u & 0x7fffffffu) == 0u) {
        u = 0u;
    }
    const uint32_t ord = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return (static_cast<unsigned long long>(ord) << 32) | (0xffffffffull - static_cast<unsigned long long>(n));
}

__device__ __forceinline__ unsigned long long umax64(unsigned long long a, unsigned long long b) {
    return a > b ? a : b;
}

template <LinearEpilogue kEpi>
__host__ __device__ constexpr int mats_of() {
    return kEpi == LinearEpilogue::kSiluMul ? 2 : 1;
}

// Stores (or, for kArgmax, folds into `best`) the kRows finished dot products of row group g; every lane holds
// every sum, lane r stores row r.
template <LinearEpilogue kEpi, int kRows>
__device__ __forceinline__ void gemv_epilogue(const LinearParams& p, int64_t g, const float* acc, int lane,
                                              int64_t pos, unsigned long long& best) {
#pragma unroll
    for (int r = 0; r < kRows; ++r) {
        const int64_t n = g * kRows + r;
        if (n >= p.N) {
            break;
        }
        if constexpr (kEpi == LinearEpilogue::kArgmax) {
            const float logit = round_to_bf16(acc[r]);
            best = umax64(best, logit_key(logit, n));
            if (lane == r && p.out[0] != nullptr) {
                store_segment(p, 0, n, logit, 0);
            }
        } else if (lane == r) {
            if constexpr (kEpi == LinearEpilogue::kStore) {
                store_segment(p, 0, n, acc[r], pos);
            } else if constexpr (kEpi == LinearEpilogue::kResidual) {
                const float res = Vec16<bf16>::load1(p.residual, n);
                Vec16<bf16>::store1(p.out[0], n, res + round_to_bf16(acc[r]));
            } else {
                const float gate = round_to_bf16(acc[r * 2]);
                const float up = round_to_bf16(acc[r * 2 + 1]);
                Vec16<bf16>::store1(p.out[0], n, round_to_bf16(silu_pexp(gate)) * up);
            }
        }
    }
}

// kArgmax: combines the warps' keys, then the CTAs' (the last CTA to arrive writes the token, advances the
// position and re-arms the counter). `best` is the same in every lane of a warp.
__device__ __forceinline__ void argmax_finish(const LinearParams& p, unsigned long long best,
                                              unsigned long long* s_best, int* s_last) {
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    if (lane == 0) {
        s_best[warp] = best;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        unsigned long long b = s_best[0];
#pragma unroll
        for (int w = 1; w < kWarps; ++w) {
            b = umax64(b, s_best[w]);
        }
        p.partial[blockIdx.x] = b;
        __threadfence();
        const unsigned ticket = atomicAdd(p.counter, 1u);
        *s_last = ticket == gridDim.x - 1 ? 1 : 0;
    }
    __syncthreads();
    if (*s_last) {
        __threadfence();
        unsigned long long b = 0ull;
        for (int64_t i = threadIdx.x; i < gridDim.x; i += kThreads) {
            b = umax64(b, __ldcg(p.partial + i));
        }
#pragma unroll
        for (int offset = 16; offset > 0; offset >>= 1) {
            b = umax64(b, __shfl_xor_sync(0xffffffffu, b, offset));
        }
        __syncthreads();
        if (lane == 0) {
            s_best[warp] = b;
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            unsigned long long all = s_best[0];
#pragma unroll
            for (int w = 1; w < kWarps; ++w) {
                all = umax64(all, s_best[w]);
            }
            int64_t index = 0;
            if (all != ~0ull && all != 0ull) {
                index = static_cast<int64_t>(0xffffffffull - (all & 0xffffffffull));
            }
            const int base = *p.position_out;
            p.tokens_out[base + p.advance] = index;
            *p.position_out = base + static_cast<int>(p.advance);
            *p.counter = 0u;
        }
    }
}

// Fast single-row kernel for K = 256 * kC: every lane holds exactly kC chunks of the input (in registers) and of
// each weight row, so a warp's whole row group is one batch of loads. The input row is normalised inside each
// warp (the lane partial over its chunks is the canonical one), with no shared memory and no block barrier. One
// CTA per SM, so the next kernel in the stream (launched early) can prefetch its weights on the same SM.
template <LinearEpilogue kEpi, int kC, int kRows>
__global__ void __launch_bounds__(kThreads, 2) gemv_fast_kernel(const LinearParams p) {
    __shared__ unsigned long long s_best[kWarps];
    __shared__ int s_last;
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

    constexpr int kMats = mats_of<kEpi>();
    constexpr int kSlots = kRows * kMats;
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int64_t groups = (p.N + kRows - 1) / kRows;
    const int64_t gstride = static_cast<int64_t>(gridDim.x) * kWarps;
    int64_t g = static_cast<int64_t>(blockIdx.x) * kWarps + warp;
    constexpr int64_t kRowBytes = kC * 32 * 16;

    uint4 wv[kSlots][kC];
    auto issue = [&](int64_t grp) {
#pragma unroll
        for (int r = 0; r < kRows; ++r) {
            const int64_t n = grp * kRows + r;
#pragma unroll
            for (int mat = 0; mat < kMats; ++mat) {
                const char* wrow = reinterpret_cast<const char*>(mat == 0 ? p.w0 : p.w1) + n * kRowBytes;
#pragma unroll
                for (int i = 0; i < kC; ++i) {
                    wv[r * kMats + mat][i] = n < p.N ? ld_stream(wrow + (lane + 32 * i) * 16) : make_uint4(0u, 0u, 0u, 0u);
                }
            }
        }
    };
    if (g < groups) {
        issue(g);
    }

    asm volatile("griddepcontrol.wait;" ::: "memory");

    const int64_t pos = p.position != nullptr ? static_cast<int64_t>(*p.position) : 0;
    const bf16* xrow = input_row(p, 0, pos);
    // Up to 4 chunks per lane the input row stays in registers (and may be normalised); longer rows are re-read
    // from L1 chunk by chunk while multiplying.
    constexpr bool kHoldX = kC <= 4;
    uint4 xv[kHoldX ? kC : 1];
    if constexpr (kHoldX) {
#pragma unroll
        for (int i = 0; i < kC; ++i) {
            xv[i] = ld_cached(xrow + (lane + 32 * i) * 8);
        }
        if (p.x_copy != nullptr && blockIdx.x == 0 && warp == 0) {
#pragma unroll
            for (int i = 0; i < kC; ++i) {
                st_v4(p.x_copy + (lane + 32 * i) * 8, xv[i]);
            }
        }
        if (p.norm_weight != nullptr) {
            // ops::rms_norm of the row: lane l's chunks are l, l + 32, ..., so its partial is the canonical one.
            float s = 0.0f;
#pragma unroll
            for (int i = 0; i < kC; ++i) {
                float f[8];
                Vec16<bf16>::unpack(xv[i], f);
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    s = __fmaf_rn(f[e], f[e], s);  // a bf16 square: fused, as sum_square
                }
            }
            s = group_sum<32>(s);
            const float mean = s / static_cast<float>(kC * 256);
            const float rms = sqrtf(mean + p.eps);
            const float inv = 1.0f / rms;
#pragma unroll
            for (int i = 0; i < kC; ++i) {
                float f[8];
                float w[8];
                Vec16<bf16>::unpack(xv[i], f);
                Vec16<bf16>::unpack(ld_cached(p.norm_weight + (lane + 32 * i) * 8), w);
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    f[e] = (f[e] * inv) * w[e];
                }
                xv[i] = Vec16<bf16>::pack(f);
            }
        }
    }

    unsigned long long best = 0ull;
    bool first = true;
    for (; g < groups; g += gstride) {
        if (!first) {
            issue(g);
        }
        first = false;
        float acc[kSlots];
#pragma unroll
        for (int j = 0; j < kSlots; ++j) {
            acc[j] = 0.0f;
        }
#pragma unroll
        for (int i = 0; i < kC; ++i) {
            uint4 x;
            if constexpr (kHoldX) {
                x = xv[i];
            } else {
                x = ld_cached(xrow + (lane + 32 * i) * 8);
            }
#pragma unroll
            for (int j = 0; j < kSlots; ++j) {
                acc[j] = dot_chunk(x, wv[j][i], acc[j]);
            }
        }
#pragma unroll
        for (int j = 0; j < kSlots; ++j) {
            acc[j] = group_sum<32>(acc[j]);
        }
        gemv_epilogue<kEpi, kRows>(p, g, acc, lane, pos, best);
    }
    if constexpr (kEpi == LinearEpilogue::kArgmax) {
        argmax_finish(p, best, s_best, &s_last);
    }
}

// Single-row kernel with the CTA's slice of weight rows (rows_per_cta rows of every matrix, contiguous in the
// checkpoint layout) staged in shared memory by bulk copies that thread 0 issues before griddepcontrol.wait. Under
// programmatic dependent launch the CTA starts while the previous kernel is still running, so the slice streams
// from HBM during the previous kernel instead of after it. After the wait the input row is read (and normalised)
// as in gemv_fast_kernel and each warp takes rows r, r + kStagedWarps, ... of the slice from shared memory.
// 8 warps per CTA: measured on the Qwen3-0.6B decode step, 670 us per token against 692 with 16 warps, 892 with 4
// (8 rows per warp) and 759 with 32.
// At most 85 registers (3 CTAs per SM): the decode step's next kernels must fit beside a staged CTA to become
// resident early (Qwen3-0.6B decode: 1595 tok/s with 2 CTAs per SM, 1657 with 3; 4, spilling: 1640).
constexpr int kStagedThreads = 256;
constexpr int kStagedWarps = kStagedThreads / 32;
constexpr int kStagedRowIters = 4;  // rows a warp may own: kStagedWarps * 4 rows per CTA at most

template <LinearEpilogue kEpi, int kC>
__global__ void __launch_bounds__(kStagedThreads, 3) gemv_staged_kernel(const LinearParams p, int64_t rows_per_cta) {
    extern __shared__ __align__(128) uint4 s_w[];
    __shared__ __align__(8) uint64_t s_bar;
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

    constexpr int kMats = mats_of<kEpi>();
    constexpr int64_t kRowBytes = kC * 512;
    constexpr int64_t kRowChunks = kC * 32;
    constexpr int64_t kPiece = 32 * 1024;  // bytes per bulk copy
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int64_t r0 = static_cast<int64_t>(blockIdx.x) * rows_per_cta;
    const int64_t r1 = r0 + rows_per_cta < p.N ? r0 + rows_per_cta : p.N;
    const int64_t nrows = r1 > r0 ? r1 - r0 : 0;
    if (threadIdx.x == 0) {
        mbar_init(&s_bar, 1);
        const int64_t bytes = nrows * kRowBytes;
        mbar_arrive_expect_tx(&s_bar, static_cast<uint32_t>(bytes * kMats));
#pragma unroll
        for (int mat = 0; mat < kMats; ++mat) {
            const char* src = reinterpret_cast<const char*>(mat == 0 ? p.w0 : p.w1) + r0 * kRowBytes;
            char* dst = reinterpret_cast<char*>(s_w) + mat * rows_per_cta * kRowBytes;
            for (int64_t off = 0; off < bytes; off += kPiece) {
                const int64_t len = bytes - off < kPiece ? bytes - off : kPiece;
                bulk_copy_g2s(dst + off, src + off, static_cast<uint32_t>(len), &s_bar);
            }
        }
    }
    __syncthreads();  // the barrier is initialised before anyone polls it

    constexpr bool kHoldX = kC <= 4;
    // Constants the previous kernel does not write are read before the wait.
    uint4 nw[kHoldX ? kC : 1];
    if constexpr (kHoldX) {
        if (p.norm_weight != nullptr) {
#pragma unroll
            for (int i = 0; i < kC; ++i) {
                nw[i] = ld_cached(p.norm_weight + (lane + 32 * i) * 8);
            }
        }
    }

    // One warp waits for the previous grid; the others wait at the block barrier (which orders their reads after
    // that wait), so warps of this CTA that are resident early do not compete for issue slots with the kernel
    // still running on the SM.
    if (warp == 0) {
        asm volatile("griddepcontrol.wait;" ::: "memory");
    }
    __syncthreads();

    const int64_t pos = p.position != nullptr ? static_cast<int64_t>(*p.position) : 0;
    const bf16* xrow = input_row(p, 0, pos);
    // The residual values this warp's rows add are read now, in parallel with the input row.
    float res_pre[kEpi == LinearEpilogue::kResidual ? kStagedRowIters : 1];
    if constexpr (kEpi == LinearEpilogue::kResidual) {
#pragma unroll
        for (int k = 0; k < kStagedRowIters; ++k) {
            const int64_t r = warp + static_cast<int64_t>(k) * kStagedWarps;
            res_pre[k] = (lane == 0 && r < nrows) ? Vec16<bf16>::load1(p.residual, r0 + r) : 0.0f;
        }
    }
    // Without a held (and normalised) row, the whole input row (up to K = 2048: more would double the registers
    // of a CTA and keep the next kernels' CTAs from becoming resident early) is still loaded here, right after the
    // wait, so its latency overlaps the residual load and the wait for the staged slice.
    uint4 xraw[kHoldX || kC > 8 ? 1 : kC];
    if constexpr (!kHoldX && kC <= 8) {
#pragma unroll
        for (int i = 0; i < kC; ++i) {
            xraw[i] = ld_cached(xrow + (lane + 32 * i) * 8);
        }
    }
    uint4 xv[kHoldX ? kC : 1];
    if constexpr (kHoldX) {
        // With a norm, warp 0 alone loads and normalises the row and hands it to the other warps through shared
        // memory (every warp doing it made the prologue issue-bound: 32 warps per SM repeating the same chain).
        __shared__ uint4 s_xn[kC * 32];
        const bool norm = p.norm_weight != nullptr;
        if (!norm || warp == 0) {
#pragma unroll
            for (int i = 0; i < kC; ++i) {
                xv[i] = ld_cached(xrow + (lane + 32 * i) * 8);
            }
        }
        if (p.x_copy != nullptr && blockIdx.x == 0 && warp == 0) {
#pragma unroll
            for (int i = 0; i < kC; ++i) {
                st_v4(p.x_copy + (lane + 32 * i) * 8, xv[i]);
            }
        }
        if (norm && warp == 0) {
            // ops::rms_norm of the row: lane l's chunks are l, l + 32, ..., so its partial is the canonical one.
            float s = 0.0f;
#pragma unroll
            for (int i = 0; i < kC; ++i) {
                float f[8];
                Vec16<bf16>::unpack(xv[i], f);
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    s = __fmaf_rn(f[e], f[e], s);  // a bf16 square: fused, as sum_square
                }
            }
            s = group_sum<32>(s);
            const float mean = s / static_cast<float>(kC * 256);
            const float rms = sqrtf(mean + p.eps);
            const float inv = 1.0f / rms;
#pragma unroll
            for (int i = 0; i < kC; ++i) {
                float f[8];
                float w[8];
                Vec16<bf16>::unpack(xv[i], f);
                Vec16<bf16>::unpack(nw[i], w);
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    f[e] = (f[e] * inv) * w[e];
                }
                s_xn[lane + 32 * i] = Vec16<bf16>::pack(f);
            }
        }
        if (norm) {
            __syncthreads();
#pragma unroll
            for (int i = 0; i < kC; ++i) {
                xv[i] = s_xn[lane + 32 * i];
            }
        }
    }

    const bool arrived = mbar_wait_bounded(&s_bar, 0, p.poll_limit);
    if (__syncthreads_or(arrived ? 0 : 1)) {
        // The copies did not complete within the poll limit: report it, give them one more bounded wait so no
        // copy lands in shared memory after this CTA has left, and produce nothing.
        if (threadIdx.x == 0) {
            atomicOr(p.error, 1u);
        }
        mbar_wait_bounded(&s_bar, 0);
        return;
    }

    // Each warp takes rows warp, warp + kStagedWarps, ... of the slice, one at a time (measured on B200:
    // interleaving four rows per warp was slower).
#pragma unroll
    for (int k = 0; k < kStagedRowIters; ++k) {
        const int64_t r = warp + static_cast<int64_t>(k) * kStagedWarps;
        if (r >= nrows) {
            break;
        }
        float acc[kMats];
#pragma unroll
        for (int mat = 0; mat < kMats; ++mat) {
            acc[mat] = 0.0f;
        }
#pragma unroll
        for (int i = 0; i < kC; ++i) {
            uint4 xr;
            if constexpr (kHoldX) {
                xr = xv[i];
            } else if constexpr (kC <= 8) {
                xr = xraw[i];
            } else {
                xr = ld_cached(xrow + (lane + 32 * i) * 8);
            }
#pragma unroll
            for (int mat = 0; mat < kMats; ++mat) {
                acc[mat] = dot_chunk(xr, s_w[(mat * rows_per_cta + r) * kRowChunks + lane + 32 * i], acc[mat]);
            }
        }
#pragma unroll
        for (int mat = 0; mat < kMats; ++mat) {
            acc[mat] = group_sum<32>(acc[mat]);
        }
        if (lane == 0) {
            const int64_t n = r0 + r;
            if constexpr (kEpi == LinearEpilogue::kStore) {
                store_segment(p, 0, n, acc[0], pos);
            } else if constexpr (kEpi == LinearEpilogue::kResidual) {
                Vec16<bf16>::store1(p.out[0], n, res_pre[k] + round_to_bf16(acc[0]));
            } else {
                const float gate = round_to_bf16(acc[0]);
                const float up = round_to_bf16(acc[1]);
                Vec16<bf16>::store1(p.out[0], n, round_to_bf16(silu_pexp(gate)) * up);
            }
        }
    }
}

template <LinearEpilogue kEpi, int kRows>
__global__ void __launch_bounds__(kThreads, 2) gemv_kernel(const LinearParams p) {
    extern __shared__ uint4 smem_x[];  // the input row, K / 8 chunks
    __shared__ float s_inv;
    __shared__ unsigned long long s_best[kWarps];
    __shared__ int s_last;

    // Dependents may be scheduled at once: they only prefetch weights before their own wait.
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

    constexpr int kMats = kEpi == LinearEpilogue::kSiluMul ? 2 : 1;
    constexpr int kSlots = kRows * kMats;
    constexpr int kBatch = kLoads / kSlots;  // chunk iterations per lane per batch
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int64_t nchunks = p.K / 8;
    const int64_t iters = (nchunks + 31) / 32;  // chunk iterations of lane 0
    const int64_t groups = (p.N + kRows - 1) / kRows;
    const int64_t gstride = static_cast<int64_t>(gridDim.x) * kWarps;
    int64_t g = static_cast<int64_t>(blockIdx.x) * kWarps + warp;
    const int64_t row_bytes = p.K * 2;

    uint4 wreg[kSlots][kBatch];
    auto issue = [&](int64_t grp, int64_t i0) {
#pragma unroll
        for (int r = 0; r < kRows; ++r) {
            const int64_t n = grp * kRows + r;
#pragma unroll
            for (int mat = 0; mat < kMats; ++mat) {
                const char* wrow = reinterpret_cast<const char*>(mat == 0 ? p.w0 : p.w1) + n * row_bytes;
#pragma unroll
                for (int b = 0; b < kBatch; ++b) {
                    const int64_t c = lane + 32 * (i0 + b);
                    if (n < p.N && c < nchunks) {
                        wreg[r * kMats + mat][b] = ld_stream(wrow + c * 16);
                    } else {
                        wreg[r * kMats + mat][b] = make_uint4(0u, 0u, 0u, 0u);
                    }
                }
            }
        }
    };
    bool pending = g < groups;
    if (pending) {
        issue(g, 0);
    }

    asm volatile("griddepcontrol.wait;" ::: "memory");

    const int64_t pos = p.position != nullptr ? static_cast<int64_t>(*p.position) : 0;
    const bf16* xrow = input_row(p, 0, pos);
    for (int64_t i = threadIdx.x; i < nchunks; i += kThreads) {
        const uint4 v = ld_cached(xrow + i * 8);
        smem_x[i] = v;
        if (p.x_copy != nullptr && blockIdx.x == 0) {
            st_v4(p.x_copy + i * 8, v);
        }
    }
    __syncthreads();
    if (p.norm_weight != nullptr) {
        // ops::rms_norm of the row, sum of squares in the canonical lane order (identical to rms_norm.cu).
        if (warp == 0) {
            float s = 0.0f;
            for (int64_t c = lane; c < nchunks; c += 32) {
                float f[8];
                Vec16<bf16>::unpack(smem_x[c], f);
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    s = __fmaf_rn(f[e], f[e], s);  // a bf16 square: fused, as sum_square
                }
            }
            s = group_sum<32>(s);
            if (lane == 0) {
                const float mean = s / static_cast<float>(p.K);
                const float rms = sqrtf(mean + p.eps);
                s_inv = 1.0f / rms;
            }
        }
        __syncthreads();
        const float inv = s_inv;
        for (int64_t i = threadIdx.x; i < nchunks; i += kThreads) {
            float f[8];
            float w[8];
            Vec16<bf16>::unpack(smem_x[i], f);
            Vec16<bf16>::unpack(ld_cached(p.norm_weight + i * 8), w);
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                f[e] = (f[e] * inv) * w[e];
            }
            smem_x[i] = Vec16<bf16>::pack(f);
        }
        __syncthreads();
    }

    unsigned long long best = 0ull;
    for (; g < groups; g += gstride) {
        float acc[kSlots];
#pragma unroll
        for (int j = 0; j < kSlots; ++j) {
            acc[j] = 0.0f;
        }
        for (int64_t i0 = 0; i0 < iters; i0 += kBatch) {
            if (pending) {
                pending = false;
            } else {
                issue(g, i0);
            }
#pragma unroll
            for (int b = 0; b < kBatch; ++b) {
                const int64_t c = lane + 32 * (i0 + b);
                if (c < nchunks) {
                    const uint4 xv = smem_x[c];
#pragma unroll
                    for (int j = 0; j < kSlots; ++j) {
                        acc[j] = dot_chunk(xv, wreg[j][b], acc[j]);
                    }
                }
            }
        }
#pragma unroll
        for (int j = 0; j < kSlots; ++j) {
            acc[j] = group_sum<32>(acc[j]);
        }
        gemv_epilogue<kEpi, kRows>(p, g, acc, lane, pos, best);
    }
    if constexpr (kEpi == LinearEpilogue::kArgmax) {
        argmax_finish(p, best, s_best, &s_last);
    }
}

// Sums kTileRows (16) per-lane partials over the warp in the canonical butterfly order -- partial[l] +
// partial[l ^ d] for d = 16, 8, 4, 2, 1 -- and leaves the total of row (lane >> 1) in lanes 2r and 2r + 1. At each
// distance a lane keeps half of its rows and trades the other half with its partner, so the 16 rows take 16
// shuffles instead of 80, and the epilogue then runs on all lanes at once. Every addition is the same pair of
// operands as in the plain butterfly (IEEE addition is commutative), so the bits are the same.
__device__ __forceinline__ float reduce_rows16(const float (&acc)[kTileRows], int lane) {
    static_assert(kTileRows == 16, "reduce_rows16 takes 16 rows");
    float v8[8];
    const bool b4 = (lane & 16) != 0;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        const float keep = b4 ? acc[8 + k] : acc[k];
        const float send = b4 ? acc[k] : acc[8 + k];
        v8[k] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
    }
    float v4[4];
    const bool b3 = (lane & 8) != 0;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const float keep = b3 ? v8[4 + k] : v8[k];
        const float send = b3 ? v8[k] : v8[4 + k];
        v4[k] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
    }
    float v2[2];
    const bool b2 = (lane & 4) != 0;
#pragma unroll
    for (int k = 0; k < 2; ++k) {
        const float keep = b2 ? v4[2 + k] : v4[k];
        const float send = b2 ? v4[k] : v4[2 + k];
        v2[k] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
    }
    const bool b1 = (lane & 2) != 0;
    const float keep = b1 ? v2[1] : v2[0];
    const float send = b1 ? v2[0] : v2[1];
    const float v1 = keep + __shfl_xor_sync(0xffffffffu, send, 2);
    return v1 + __shfl_xor_sync(0xffffffffu, v1, 1);
}

template <LinearEpilogue kEpi>
__global__ void __launch_bounds__(kThreads) linear_rows_kernel(const LinearParams p) {
    extern __shared__ uint4 smem_x[];  // kTileRows rows of K / 8 chunks
    grid_dependency_begin();
    constexpr int kMats = kEpi == LinearEpilogue::kSiluMul ? 2 : 1;
    constexpr int kBatch = 4;
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int64_t nchunks = p.K / 8;
    const int64_t m0 = static_cast<int64_t>(blockIdx.y) * kTileRows;
    const int64_t mt = p.M - m0 < kTileRows ? p.M - m0 : kTileRows;
    const int64_t row_bytes = p.K * 2;

    for (int64_t i = threadIdx.x; i < kTileRows * nchunks; i += kThreads) {
        const int64_t m = i / nchunks;
        const int64_t c = i - m * nchunks;
        smem_x[i] = m < mt ? ld_cached(input_row(p, m0 + m, 0) + c * 8) : make_uint4(0u, 0u, 0u, 0u);
    }
    __syncthreads();

    for (int64_t n = static_cast<int64_t>(blockIdx.x) * kWarps + warp; n < p.N;
         n += static_cast<int64_t>(gridDim.x) * kWarps) {
        float acc[kMats][kTileRows];
#pragma unroll
        for (int mat = 0; mat < kMats; ++mat) {
#pragma unroll
            for (int m = 0; m < kTileRows; ++m) {
                acc[mat][m] = 0.0f;
            }
        }
        for (int64_t i0 = 0; lane + 32 * i0 < nchunks; i0 += kBatch) {
            uint4 wraw[kMats][kBatch];
#pragma unroll
            for (int mat = 0; mat < kMats; ++mat) {
                const char* wrow = reinterpret_cast<const char*>(mat == 0 ? p.w0 : p.w1) + n * row_bytes;
#pragma unroll
                for (int b = 0; b < kBatch; ++b) {
                    const int64_t c = lane + 32 * (i0 + b);
                    wraw[mat][b] = c < nchunks ? ld_stream(wrow + c * 16) : make_uint4(0u, 0u, 0u, 0u);
                }
            }
#pragma unroll
            for (int b = 0; b < kBatch; ++b) {
                const int64_t c = lane + 32 * (i0 + b);
                if (c < nchunks) {
#pragma unroll
                    for (int mat = 0; mat < kMats; ++mat) {
                        float w[8];
                        Vec16<bf16>::unpack(wraw[mat][b], w);
#pragma unroll
                        for (int m = 0; m < kTileRows; ++m) {
                            acc[mat][m] = dot_chunk(smem_x[m * nchunks + c], w, acc[mat][m]);
                        }
                    }
                }
            }
        }
        float total[kMats];
#pragma unroll
        for (int mat = 0; mat < kMats; ++mat) {
            total[mat] = reduce_rows16(acc[mat], lane);
        }
        const int r = (lane >> 1) & (kTileRows - 1);
        if ((lane & 1) == 0 && r < mt) {
            const int64_t row = m0 + r;
            if constexpr (kEpi == LinearEpilogue::kStore) {
                store_segment(p, row, n, total[0], 0);
            } else if constexpr (kEpi == LinearEpilogue::kResidual) {
                const float res = Vec16<bf16>::load1(p.residual, row * p.res_ld + n);
                Vec16<bf16>::store1(p.out[0], row * p.ld[0] + n, res + round_to_bf16(total[0]));
            } else {
                const float gate = round_to_bf16(total[0]);
                const float up = round_to_bf16(total[1]);
                Vec16<bf16>::store1(p.out[0], row * p.ld[0] + n, round_to_bf16(silu_pexp(gate)) * up);
            }
        }
    }
}

// Prefill projection with the 16-row input tile staged in shared memory as f32, interleaved by row pairs so that one
// packed f32x2 fused multiply-add advances two rows, and two weight rows (or the gate and up rows of one output) per
// warp, so each staged input chunk feeds 16 multiply-adds. Same per-output order as the other kernels.
template <LinearEpilogue kEpi>
__global__ void __launch_bounds__(kThreads, 2) linear_rows_f32x_kernel(const LinearParams p) {
    // [kTileRows / 2 row pairs][4 element pairs][K / 8 chunks]: float4 (x[2q][e], x[2q+1][e], x[2q][e+1],
    // x[2q+1][e+1]) for e = 8 c + 2 k, so one 16-byte read gives two (row 2q, row 2q+1) pairs of one element each
    // and a warp's reads of consecutive chunks are conflict-free.
    extern __shared__ float4 smem_xf[];
    grid_dependency_begin();
    constexpr int kMats = mats_of<kEpi>();
    constexpr int kSlots = 2;                      // weight rows a warp multiplies together
    constexpr int kRowsPerWarp = kSlots / kMats;   // outputs a warp finishes per pass
    constexpr int kBatch = 2;
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int64_t nchunks = p.K / 8;
    const int64_t m0 = static_cast<int64_t>(blockIdx.y) * kTileRows;
    const int64_t mt = p.M - m0 < kTileRows ? p.M - m0 : kTileRows;
    const int64_t row_bytes = p.K * 2;
    constexpr int kPairs = kTileRows / 2;

    for (int64_t i = threadIdx.x; i < kPairs * nchunks; i += kThreads) {
        const int64_t q = i / nchunks;
        const int64_t c = i - q * nchunks;
        float f0[8] = {0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f};
        float f1[8] = {0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f};
        if (2 * q < mt) {
            Vec16<bf16>::unpack(ld_cached(input_row(p, m0 + 2 * q, 0) + c * 8), f0);
        }
        if (2 * q + 1 < mt) {
            Vec16<bf16>::unpack(ld_cached(input_row(p, m0 + 2 * q + 1, 0) + c * 8), f1);
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            smem_xf[(q * 4 + k) * nchunks + c] = make_float4(f0[2 * k], f1[2 * k], f0[2 * k + 1], f1[2 * k + 1]);
        }
    }
    __syncthreads();

    const int64_t step = static_cast<int64_t>(gridDim.x) * kWarps * kRowsPerWarp;
    for (int64_t n0 = (static_cast<int64_t>(blockIdx.x) * kWarps + warp) * kRowsPerWarp; n0 < p.N; n0 += step) {
        const char* wrows[kSlots];
        bool valid[kSlots];
#pragma unroll
        for (int sl = 0; sl < kSlots; ++sl) {
            const int mat = kMats == 2 ? sl : 0;
            const int64_t n = kMats == 2 ? n0 : n0 + sl;
            valid[sl] = n < p.N;
            wrows[sl] = reinterpret_cast<const char*>(mat == 0 ? p.w0 : p.w1) + (valid[sl] ? n : 0) * row_bytes;
        }
        float acc[kSlots][kTileRows];
#pragma unroll
        for (int sl = 0; sl < kSlots; ++sl) {
#pragma unroll
            for (int m = 0; m < kTileRows; ++m) {
                acc[sl][m] = 0.0f;
            }
        }
        for (int64_t i0 = 0; lane + 32 * i0 < nchunks; i0 += kBatch) {
            uint4 wraw[kSlots][kBatch];
#pragma unroll
            for (int sl = 0; sl < kSlots; ++sl) {
#pragma unroll
                for (int b = 0; b < kBatch; ++b) {
                    const int64_t c = lane + 32 * (i0 + b);
                    wraw[sl][b] = (valid[sl] && c < nchunks) ? ld_stream(wrows[sl] + c * 16) : make_uint4(0u, 0u, 0u, 0u);
                }
            }
#pragma unroll
            for (int b = 0; b < kBatch; ++b) {
                const int64_t c = lane + 32 * (i0 + b);
                if (c < nchunks) {
                    float w[kSlots][8];
#pragma unroll
                    for (int sl = 0; sl < kSlots; ++sl) {
                        Vec16<bf16>::unpack(wraw[sl][b], w[sl]);
                    }
#pragma unroll
                    for (int q = 0; q < kPairs; ++q) {
                        float2 xp[8];
#pragma unroll
                        for (int k = 0; k < 4; ++k) {
                            const float4 v = smem_xf[(q * 4 + k) * nchunks + c];
                            xp[2 * k] = make_float2(v.x, v.y);
                            xp[2 * k + 1] = make_float2(v.z, v.w);
                        }
#pragma unroll
                        for (int sl = 0; sl < kSlots; ++sl) {
                            // Rows 2q and 2q + 1 are separate chains: one packed fused multiply-add advances
                            // both, each rounded once (fma_bf16x2's arithmetic; the inputs are exact f32 copies).
                            float2 a01 = make_float2(acc[sl][2 * q], acc[sl][2 * q + 1]);
#pragma unroll
                            for (int e = 0; e < 8; ++e) {
                                a01 = __ffma2_rn(xp[e], make_float2(w[sl][e], w[sl][e]), a01);
                            }
                            acc[sl][2 * q] = a01.x;
                            acc[sl][2 * q + 1] = a01.y;
                        }
                    }
                }
            }
        }
        const float total0 = reduce_rows16(acc[0], lane);
        const float total1 = reduce_rows16(acc[1], lane);
        // Lanes 2r and 2r + 1 hold row r: the even lane finishes slot 0, the odd lane slot 1 (SiLU * up: the even
        // lane alone, from both).
        const int r = (lane >> 1) & (kTileRows - 1);
        const int sl = lane & 1;
        if (r < mt) {
            const int64_t row = m0 + r;
            if constexpr (kEpi == LinearEpilogue::kSiluMul) {
                if (sl == 0) {
                    const float gate = round_to_bf16(total0);
                    const float up = round_to_bf16(total1);
                    Vec16<bf16>::store1(p.out[0], row * p.ld[0] + n0, round_to_bf16(silu_pexp(gate)) * up);
                }
            } else {
                const int64_t n = n0 + sl;
                if (valid[sl]) {
                    const float v = sl == 0 ? total0 : total1;
                    if constexpr (kEpi == LinearEpilogue::kStore) {
                        store_segment(p, row, n, v, 0);
                    } else {
                        const float res = Vec16<bf16>::load1(p.residual, row * p.res_ld + n);
                        Vec16<bf16>::store1(p.out[0], row * p.ld[0] + n, res + round_to_bf16(v));
                    }
                }
            }
        }
    }
}

// ops::matmul for any operand types and strides: one warp per output element, the canonical lane order with chunks
// of 8 when K % 8 == 0 and of 1 otherwise (the same order as the vector kernels, so a bf16 layout they accept gives
// the same bits either way). Used for shapes and layouts the vector kernels do not take.
struct MatmulArgs {
    const void* x;
    int64_t xs[3];
    const void* w;
    int64_t ws[3];
    void* y;
    int64_t batch;
    int64_t m;
    int64_t k;
    int64_t n;
};

template <typename Tx, typename Tw, typename Ty>
__global__ void __launch_bounds__(kThreads) matmul_generic_kernel(const MatmulArgs a) {
    grid_dependency_begin();
    const int lane = threadIdx.x & 31;
    const int64_t total = a.batch * a.m * a.n;
    const int64_t chunk = a.k % 8 == 0 ? 8 : 1;
    const int64_t nchunks = a.k / chunk;
    for (int64_t idx = (static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x) / 32; idx < total;
         idx += static_cast<int64_t>(gridDim.x) * kWarps) {
        const int64_t b = idx / (a.m * a.n);
        const int64_t i = (idx / a.n) % a.m;
        const int64_t j = idx % a.n;
        const int64_t xrow = b * a.xs[0] + i * a.xs[1];
        const int64_t wcol = b * a.ws[0] + j * a.ws[2];
        float acc = 0.0f;
        for (int64_t c = lane; c < nchunks; c += 32) {
            for (int64_t e = c * chunk; e < (c + 1) * chunk; ++e) {
                const float xv = Vec16<Tx>::load1(a.x, xrow + e * a.xs[2]);
                const float wv = Vec16<Tw>::load1(a.w, wcol + e * a.ws[1]);
                if constexpr (std::is_same_v<Tx, bf16> && std::is_same_v<Tw, bf16>) {
                    acc = __fmaf_rn(xv, wv, acc);  // bf16 operands: fused, as in the vector kernels
                } else {
                    acc = acc + xv * wv;  // an f32 operand: separately rounded product and sum
                }
            }
        }
        acc = group_sum<32>(acc);
        if (lane == 0) {
            Vec16<Ty>::store1(a.y, idx, acc);
        }
    }
}

__global__ void __launch_bounds__(kThreads) embedding_kernel(const bf16* table, int64_t vocab, int64_t hidden,
                                                             const int64_t* tokens, int64_t count, bf16* out) {
    grid_dependency_begin();
    const int64_t chunks = hidden / 8;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x; i < count * chunks;
         i += static_cast<int64_t>(gridDim.x) * kThreads) {
        const int64_t t = i / chunks;
        const int64_t c = i - t * chunks;
        const int64_t row = clamp_token(tokens[t], vocab);
        st_v4(out + t * hidden + c * 8, ld_cached(table + row * hidden + c * 8));
    }
}

// Launch plan of the single-row kernels. K = 256 * c with c in {1, 2, 3, 4, 6, 8, 12} (c <= 4 with the RMSNorm
// prologue or the input copy) takes the fast kernel with
// kRows rows per warp (a lane's whole row group, kRows * mats * c 16-byte loads, in flight at once); other K take
// the generic kernel. Grids: one CTA per SM, two for the vocabulary-sized argmax head and for the staged kernel.
struct GemvPlan {
    bool fast;
    bool staged;            // gemv_staged_kernel: the CTA's weight rows staged in shared memory
    int chunks;             // c
    int rows;               // kRows
    int grid;
    int64_t rows_per_cta;   // staged kernel
    std::size_t smem;       // staged kernel
};

// A staged slice up to this size leaves room in the 228 KB of shared memory of an SM for the next kernel's slice.
constexpr std::size_t kMaxStagedBytes = 100 * 1024;

GemvPlan plan_gemv(const LinearParams& p, int mats) {
    GemvPlan plan{};
    const int64_t c = p.K % 256 == 0 ? p.K / 256 : 0;
    plan.fast = c == 1 || c == 2 || c == 3 || c == 4 || c == 6 || c == 8 || (c == 12 && mats == 1);
    if (c > 4 && (p.norm_weight != nullptr || p.x_copy != nullptr)) {
        plan.fast = false;  // the fast kernel keeps (and normalises) the input in registers only up to K = 1024
    }
    if (plan.fast) {
        plan.chunks = static_cast<int>(c);
        const int64_t r = kLoads / (mats * c);
        plan.rows = r >= 4 ? 4 : (r >= 2 ? 2 : 1);
    } else {
        const int64_t per_lane = (p.K / 8 + 31) / 32;
        const int64_t r = kLoads / (mats * (per_lane < 1 ? 1 : per_lane));
        plan.rows = r >= 4 ? 4 : (r >= 2 ? 2 : 1);
    }
    if (plan.fast && p.error != nullptr && p.N > 0 && p.epilogue != LinearEpilogue::kArgmax) {
        // Slices for two CTAs per SM: half as many rows per warp after the wait (Qwen3-0.6B decode, measured on
        // B200: one CTA per SM 1884 tok/s, two 1909, three 1912, four 1609 -- past the register cap of three).
        const int64_t sms = runtime::sm_count();
        const int64_t rpc = (p.N + 2 * sms - 1) / (2 * sms);
        const std::size_t bytes = static_cast<std::size_t>(rpc) * mats * p.K * 2;
        if (bytes <= kMaxStagedBytes && rpc <= kStagedWarps * kStagedRowIters) {
            plan.staged = true;
            plan.rows_per_cta = rpc;
            plan.smem = bytes;
            plan.grid = static_cast<int>((p.N + rpc - 1) / rpc);
            return plan;
        }
    }
    const int64_t groups = (p.N + plan.rows - 1) / plan.rows;
    const int64_t want = (groups + kWarps - 1) / kWarps;
    const int64_t per_sm = p.epilogue == LinearEpilogue::kArgmax || !plan.fast ? 2 : 1;
    const int64_t cap = static_cast<int64_t>(runtime::sm_count()) * per_sm;
    plan.grid = static_cast<int>(want < cap ? want : cap);
    return plan;
}

template <LinearEpilogue kEpi, int kC, int kRows>
cudaError_t launch_fast(const LinearParams& p, int grid, cudaStream_t s) {
    return runtime::launch(gemv_fast_kernel<kEpi, kC, kRows>, dim3(grid), dim3(kThreads), s, 1u, p);
}

template <LinearEpilogue kEpi, int kC>
cudaError_t launch_fast_rows(const LinearParams& p, const GemvPlan& plan, cudaStream_t s) {
    if (plan.staged) {
        auto kernel = gemv_staged_kernel<kEpi, kC>;
        if (plan.smem > 48 * 1024) {
            const cudaError_t err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                         static_cast<int>(plan.smem));
            if (err != cudaSuccess) {
                return err;
            }
        }
        return runtime::launch_smem(kernel, dim3(plan.grid), dim3(kStagedThreads), plan.smem, s, 1u, p,
                                    plan.rows_per_cta);
    }
    constexpr int kMats = mats_of<kEpi>();
    constexpr int kR = kLoads / (kMats * kC) >= 4 ? 4 : (kLoads / (kMats * kC) >= 2 ? 2 : 1);
    return launch_fast<kEpi, kC, kR>(p, plan.grid, s);
}

template <LinearEpilogue kEpi>
cudaError_t launch_fast_epi(const LinearParams& p, const GemvPlan& plan, cudaStream_t s) {
    switch (plan.chunks) {
    case 1:
        return launch_fast_rows<kEpi, 1>(p, plan, s);
    case 2:
        return launch_fast_rows<kEpi, 2>(p, plan, s);
    case 3:
        return launch_fast_rows<kEpi, 3>(p, plan, s);
    case 4:
        return launch_fast_rows<kEpi, 4>(p, plan, s);
    case 6:
        return launch_fast_rows<kEpi, 6>(p, plan, s);
    case 8:
        return launch_fast_rows<kEpi, 8>(p, plan, s);
    default:
        if constexpr (mats_of<kEpi>() == 1) {
            return launch_fast_rows<kEpi, 12>(p, plan, s);
        }
        return cudaErrorInvalidValue;
    }
}

template <LinearEpilogue kEpi, int kRows>
cudaError_t launch_gemv_rows(const LinearParams& p, int grid, cudaStream_t s) {
    const std::size_t smem = static_cast<std::size_t>(p.K) * 2;
    auto kernel = gemv_kernel<kEpi, kRows>;
    if (smem > 48 * 1024) {
        const cudaError_t err =
            cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (err != cudaSuccess) {
            return err;
        }
    }
    return runtime::launch_smem(kernel, dim3(grid), dim3(kThreads), smem, s, 1u, p);
}

template <LinearEpilogue kEpi>
cudaError_t launch_gemv_epi(const LinearParams& p, cudaStream_t s) {
    const GemvPlan plan = plan_gemv(p, mats_of<kEpi>());
    if (plan.fast) {
        return launch_fast_epi<kEpi>(p, plan, s);
    }
    switch (plan.rows) {
    case 4:
        return launch_gemv_rows<kEpi, 4>(p, plan.grid, s);
    case 2:
        return launch_gemv_rows<kEpi, 2>(p, plan.grid, s);
    default:
        return launch_gemv_rows<kEpi, 1>(p, plan.grid, s);
    }
}

template <LinearEpilogue kEpi>
cudaError_t launch_rows_epi(const LinearParams& p, cudaStream_t s) {
    // f32 staging while the tile fits an SM's shared memory (K <= 3584), bf16 staging beyond.
    const bool f32x = static_cast<std::size_t>(kTileRows) * p.K * 4 <= 224 * 1024;
    const std::size_t smem = static_cast<std::size_t>(kTileRows) * p.K * (f32x ? 4 : 2);
    auto kernel = f32x ? linear_rows_f32x_kernel<kEpi> : linear_rows_kernel<kEpi>;
    if (smem > 48 * 1024) {
        const cudaError_t err =
            cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (err != cudaSuccess) {
            return err;
        }
    }
    // Every CTA stages one 16-row tile and walks its share of the N outputs, so CTAs are equal: size the grid to
    // whole waves of resident CTAs (a partial last wave would run alone). The fewest waves that use at least 95% of
    // the slots, up to 4; otherwise the best of those.
    const int64_t tiles = (p.M + kTileRows - 1) / kTileRows;
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kThreads, smem) != cudaSuccess || per_sm < 1) {
        per_sm = 1;
    }
    const int64_t slots = static_cast<int64_t>(per_sm) * runtime::sm_count();
    const int64_t row_blocks = (p.N + kWarps - 1) / kWarps;
    int64_t gx = 1;
    double best = 0.0;
    for (int64_t waves = 1; waves <= 4; ++waves) {
        int64_t g = waves * slots / tiles;
        g = g < row_blocks ? g : row_blocks;
        if (g < 1) {
            continue;
        }
        const double used = static_cast<double>(g * tiles) /
                            static_cast<double>(runtime::ceil_div(g * tiles, slots) * slots);
        if (used > best + 1e-9) {
            best = used;
            gx = g;
        }
        if (used >= 0.95) {
            break;
        }
    }
    return runtime::launch_smem(kernel, dim3(static_cast<unsigned>(gx), static_cast<unsigned>(tiles)),
                                dim3(kThreads), smem, s, 1u, p);
}

template <typename Tx, typename Tw>
cudaError_t launch_matmul_w(const MatmulArgs& a, cppinf_dtype y_dtype, unsigned grid, cudaStream_t s) {
    return y_dtype == CPPINF_DTYPE_BF16
               ? runtime::launch(matmul_generic_kernel<Tx, Tw, bf16>, dim3(grid), dim3(kThreads), s, 1u, a)
               : runtime::launch(matmul_generic_kernel<Tx, Tw, float>, dim3(grid), dim3(kThreads), s, 1u, a);
}

template <typename Tx>
cudaError_t launch_matmul_x(const MatmulArgs& a, cppinf_dtype w_dtype, cppinf_dtype y_dtype, unsigned grid,
                            cudaStream_t s) {
    return w_dtype == CPPINF_DTYPE_BF16 ? launch_matmul_w<Tx, bf16>(a, y_dtype, grid, s)
                                        : launch_matmul_w<Tx, float>(a, y_dtype, grid, s);
}

}  // namespace

int gemv_grid(const LinearParams& p) {
    LinearParams q = p;
    q.epilogue = LinearEpilogue::kArgmax;
    return plan_gemv(q, 1).grid;
}

cudaError_t launch_gemv(const LinearParams& p, cudaStream_t s) {
    switch (p.epilogue) {
    case LinearEpilogue::kStore:
        return launch_gemv_epi<LinearEpilogue::kStore>(p, s);
    case LinearEpilogue::kResidual:
        return launch_gemv_epi<LinearEpilogue::kResidual>(p, s);
    case LinearEpilogue::kSiluMul:
        return launch_gemv_epi<LinearEpilogue::kSiluMul>(p, s);
    default:
        return launch_gemv_epi<LinearEpilogue::kArgmax>(p, s);
    }
}

cudaError_t launch_linear_rows(const LinearParams& p, cudaStream_t s) {
    switch (p.epilogue) {
    case LinearEpilogue::kStore:
        return launch_rows_epi<LinearEpilogue::kStore>(p, s);
    case LinearEpilogue::kResidual:
        return launch_rows_epi<LinearEpilogue::kResidual>(p, s);
    case LinearEpilogue::kSiluMul:
        return launch_rows_epi<LinearEpilogue::kSiluMul>(p, s);
    default:
        return cudaErrorInvalidValue;
    }
}

cudaError_t launch_embedding(const bf16* table, int64_t vocab, int64_t hidden, const int64_t* tokens, int64_t count,
                             bf16* out, cudaStream_t s) {
    const int64_t work = count * (hidden / 8);
    const int64_t want = (work + kThreads - 1) / kThreads;
    const int64_t cap = static_cast<int64_t>(runtime::sm_count()) * 4;
    const int64_t blocks = want < cap ? want : cap;
    return runtime::launch(embedding_kernel, dim3(static_cast<unsigned>(blocks < 1 ? 1 : blocks)), dim3(kThreads), s,
                           1u, table, vocab, hidden, tokens, count, out);
}

}  // namespace cppinf::device

using namespace cppinf::device;
namespace rt = cppinf::runtime;

namespace {

constexpr int64_t kScratchHeader = 16;  // u32 counter, i32 position slot, padding; then one u64 per CTA

// Scratch of cppinf_linear_argmax_noalloc: one per device, in the module's static device memory, which the CUDA
// runtime zero-fills when it loads the module on a device (the counter and position slot must start at zero; each
// call leaves them zero). Room for 1024 CTAs, four times the grid of a 148-SM B200.
constexpr int64_t kStaticScratchCtas = 1024;
static __device__ __align__(256) unsigned char g_argmax_scratch[kScratchHeader + 8 * kStaticScratchCtas];

// Device address of g_argmax_scratch on the current device, looked up once per device.
cudaError_t static_argmax_scratch(void** out) {
    constexpr int kMaxDevices = 64;
    static std::mutex mu;
    static void* addresses[kMaxDevices] = {};
    int device = 0;
    cudaError_t err = cudaGetDevice(&device);
    if (err != cudaSuccess) {
        return err;
    }
    if (device < 0 || device >= kMaxDevices) {
        return cudaErrorInvalidDevice;
    }
    std::lock_guard<std::mutex> lock(mu);
    if (addresses[device] == nullptr) {
        err = cudaGetSymbolAddress(&addresses[device], g_argmax_scratch);
        if (err != cudaSuccess) {
            return err;
        }
    }
    *out = addresses[device];
    return cudaSuccess;
}

int check_linear(const void* x, int64_t x_row_stride, const void* weight, const void* y, int64_t rows,
                 int64_t in_features, int64_t out_features) {
    CPPINF_REQUIRE(rows >= 0 && in_features > 0 && out_features >= 0, CPPINF_ERR_INVALID_ARGUMENT,
                   "matmul requires non-negative dimensions and a non-empty inner dimension.");
    CPPINF_REQUIRE(rows <= 1 || x_row_stride >= in_features, CPPINF_ERR_INVALID_ARGUMENT,
                   "linear requires a row stride of at least in_features.");
    CPPINF_REQUIRE(in_features % 8 == 0, CPPINF_ERR_UNSUPPORTED, "linear requires in_features to be a multiple of 8.");
    CPPINF_REQUIRE(in_features <= (rows > 1 ? 6144 : 65536), CPPINF_ERR_UNSUPPORTED,
                   "linear supports in_features up to 6144 (65536 for a single row).");
    CPPINF_REQUIRE(out_features < (int64_t{1} << 31), CPPINF_ERR_OVERFLOW, "linear supports fewer than 2^31 outputs.");
    if (rows == 0 || out_features == 0) {
        return CPPINF_OK;
    }
    CPPINF_REQUIRE(x && weight && y, CPPINF_ERR_INVALID_ARGUMENT, "linear received a null pointer.");
    CPPINF_REQUIRE(rt::aligned16(x) && rt::aligned16(weight) && (rows <= 1 || (x_row_stride * 2) % 16 == 0),
                   CPPINF_ERR_UNSUPPORTED, "linear requires 16-byte aligned input rows and weights.");
    return CPPINF_OK;
}

LinearParams linear_params(LinearEpilogue epi, const void* x, int64_t x_row_stride, const void* w0, const void* w1,
                           void* y, int64_t rows, int64_t in_features, int64_t out_features) {
    LinearParams p{};
    p.epilogue = epi;
    p.x = static_cast<const bf16*>(x);
    p.x_stride = rows <= 1 ? in_features : x_row_stride;
    p.w0 = static_cast<const bf16*>(w0);
    p.w1 = static_cast<const bf16*>(w1);
    p.M = rows;
    p.N = out_features;
    p.K = in_features;
    p.out[0] = static_cast<bf16*>(y);
    p.ld[0] = out_features;
    p.seg[0] = 0;
    p.seg[1] = p.seg[2] = p.seg[3] = out_features;
    return p;
}

int run_linear(const LinearParams& p, void* stream, const char* name) {
    const auto s = rt::as_stream(stream);
    return rt::launched(p.M == 1 ? launch_gemv(p, s) : launch_linear_rows(p, s), name);
}

}  // namespace

extern "C" {

int cppinf_matmul(cppinf_dtype x_dtype, const void* x, const int64_t* x_strides, cppinf_dtype w_dtype, const void* w,
                  const int64_t* w_strides, cppinf_dtype y_dtype, void* y, int64_t batch, int64_t m, int64_t k,
                  int64_t n, void* stream) {
    CPPINF_REQUIRE(rt::valid_dtype(x_dtype) && rt::valid_dtype(w_dtype) && rt::valid_dtype(y_dtype),
                   CPPINF_ERR_INVALID_ARGUMENT, "matmul received an unsupported dtype.");
    CPPINF_REQUIRE(batch >= 0 && m >= 0 && k >= 0 && n >= 0, CPPINF_ERR_INVALID_ARGUMENT,
                   "matmul requires non-negative dimensions.");
    CPPINF_REQUIRE(batch * m * n < (int64_t{1} << 40), CPPINF_ERR_OVERFLOW, "matmul result is too large.");
    if (batch == 0 || m == 0 || n == 0) {
        return rt::ok();
    }
    CPPINF_REQUIRE(x_strides && w_strides && x && w && y, CPPINF_ERR_INVALID_ARGUMENT,
                   "matmul received a null pointer.");
    const auto s = rt::as_stream(stream);
    // Vector path: bf16 throughout, dense input rows, weight columns of rhs [k, n] contiguous in k (rhs is the
    // transposed view of a row-major [n, k] weight), aligned rows, k a multiple of 8.
    const bool bf16s = x_dtype == CPPINF_DTYPE_BF16 && w_dtype == CPPINF_DTYPE_BF16 && y_dtype == CPPINF_DTYPE_BF16;
    const bool layout = x_strides[2] == 1 && w_strides[1] == 1 && w_strides[2] == k && k % 8 == 0 && k > 0 &&
                        (m == 1 || (x_strides[1] % 8 == 0 && x_strides[1] >= k)) && rt::aligned16(x) &&
                        rt::aligned16(w) && (batch == 1 || (x_strides[0] % 8 == 0 && w_strides[0] % 8 == 0)) &&
                        k <= (m > 1 ? 6144 : 65536);
    if (bf16s && layout) {
        for (int64_t b = 0; b < batch; ++b) {
            LinearParams p = linear_params(LinearEpilogue::kStore, static_cast<const bf16*>(x) + b * x_strides[0],
                                           x_strides[1], static_cast<const bf16*>(w) + b * w_strides[0], nullptr,
                                           static_cast<bf16*>(y) + b * m * n, m, k, n);
            const int st = run_linear(p, stream, "matmul");
            if (st != CPPINF_OK) {
                return st;
            }
        }
        return rt::ok();
    }
    MatmulArgs a{x, {x_strides[0], x_strides[1], x_strides[2]}, w, {w_strides[0], w_strides[1], w_strides[2]},
                 y, batch, m, k, n};
    const int64_t warps = batch * m * n;
    const int64_t want = (warps + kWarps - 1) / kWarps;
    const int64_t cap = static_cast<int64_t>(rt::sm_count()) * 8;
    const auto grid = static_cast<unsigned>(want < cap ? want : cap);
    const cudaError_t err = x_dtype == CPPINF_DTYPE_BF16 ? launch_matmul_x<bf16>(a, w_dtype, y_dtype, grid, s)
                                                         : launch_matmul_x<float>(a, w_dtype, y_dtype, grid, s);
    return rt::launched(err, "matmul");
}

int cppinf_linear(const void* x, int64_t x_row_stride, const void* weight, void* y, int64_t rows, int64_t in_features,
                  int64_t out_features, void* stream) {
    const int st = check_linear(x, x_row_stride, weight, y, rows, in_features, out_features);
    if (st != CPPINF_OK || rows == 0 || out_features == 0) {
        return st == CPPINF_OK ? rt::ok() : st;
    }
    return run_linear(linear_params(LinearEpilogue::kStore, x, x_row_stride, weight, nullptr, y, rows, in_features,
                                    out_features),
                      stream, "linear");
}

int cppinf_linear_residual(const void* x, int64_t x_row_stride, const void* weight, const void* residual, void* y,
                           int64_t rows, int64_t in_features, int64_t out_features, void* stream) {
    const int st = check_linear(x, x_row_stride, weight, y, rows, in_features, out_features);
    if (st != CPPINF_OK || rows == 0 || out_features == 0) {
        return st == CPPINF_OK ? rt::ok() : st;
    }
    CPPINF_REQUIRE(residual, CPPINF_ERR_INVALID_ARGUMENT, "linear received a null pointer.");
    LinearParams p = linear_params(LinearEpilogue::kResidual, x, x_row_stride, weight, nullptr, y, rows, in_features,
                                   out_features);
    p.residual = static_cast<const bf16*>(residual);
    p.res_ld = out_features;
    return run_linear(p, stream, "linear_residual");
}

int cppinf_linear_silu_mul(const void* x, int64_t x_row_stride, const void* gate, const void* up, void* y, int64_t rows,
                           int64_t in_features, int64_t out_features, void* stream) {
    const int st = check_linear(x, x_row_stride, gate, y, rows, in_features, out_features);
    if (st != CPPINF_OK || rows == 0 || out_features == 0) {
        return st == CPPINF_OK ? rt::ok() : st;
    }
    CPPINF_REQUIRE(up, CPPINF_ERR_INVALID_ARGUMENT, "linear received a null pointer.");
    CPPINF_REQUIRE(rt::aligned16(up), CPPINF_ERR_UNSUPPORTED, "linear requires 16-byte aligned input rows and weights.");
    return run_linear(linear_params(LinearEpilogue::kSiluMul, x, x_row_stride, gate, up, y, rows, in_features,
                                    out_features),
                      stream, "linear_silu_mul");
}

int64_t cppinf_linear_argmax_scratch_bytes(int64_t out_features, int64_t in_features) {
    if (out_features <= 0 || in_features <= 0) {
        return kScratchHeader;
    }
    LinearParams p{};
    p.N = out_features;
    p.K = in_features;
    return kScratchHeader + 8 * static_cast<int64_t>(gemv_grid(p));
}

int cppinf_linear_argmax(const void* x, const void* weight, void* logits, int64_t in_features, int64_t out_features,
                         int64_t* out_token, void* scratch, void* stream) {
    CPPINF_REQUIRE(out_features > 0, CPPINF_ERR_INVALID_ARGUMENT, "logits vocab size must be non-zero.");
    const int st = check_linear(x, in_features, weight, out_token, 1, in_features, out_features);
    if (st != CPPINF_OK) {
        return st;
    }
    CPPINF_REQUIRE(scratch, CPPINF_ERR_INVALID_ARGUMENT, "linear_argmax received a null scratch pointer.");
    CPPINF_REQUIRE(rt::aligned16(scratch), CPPINF_ERR_UNSUPPORTED, "linear_argmax requires a 16-byte aligned scratch.");
    LinearParams p = linear_params(LinearEpilogue::kArgmax, x, in_features, weight, nullptr, logits, 1, in_features,
                                   out_features);
    char* base = static_cast<char*>(scratch);
    p.counter = reinterpret_cast<unsigned int*>(base);
    p.position_out = reinterpret_cast<int*>(base + 4);
    p.partial = reinterpret_cast<unsigned long long*>(base + kScratchHeader);
    p.tokens_out = out_token;
    p.advance = 0;
    return run_linear(p, stream, "linear_argmax");
}

int cppinf_linear_argmax_noalloc(const void* x, const void* weight, void* logits, int64_t in_features,
                                 int64_t out_features, int64_t* out_token, void* stream) {
    CPPINF_REQUIRE(out_features > 0, CPPINF_ERR_INVALID_ARGUMENT, "logits vocab size must be non-zero.");
    const int st = check_linear(x, in_features, weight, out_token, 1, in_features, out_features);
    if (st != CPPINF_OK) {
        return st;
    }
    const int64_t needed = cppinf_linear_argmax_scratch_bytes(out_features, in_features);
    const auto capacity = static_cast<int64_t>(sizeof(g_argmax_scratch));
    CPPINF_REQUIRE(needed <= capacity, CPPINF_ERR_UNSUPPORTED,
                   "linear_argmax_noalloc needs " + std::to_string(needed) + " bytes of scratch for this launch but "
                       "its static scratch holds " + std::to_string(capacity) + " bytes; use cppinf_linear_argmax "
                       "with a caller-provided scratch.");
    void* scratch = nullptr;
    CPPINF_CUDA_TRY(static_argmax_scratch(&scratch));
    return cppinf_linear_argmax(x, weight, logits, in_features, out_features, out_token, scratch, stream);
}

int cppinf_embedding(const void* table, int64_t vocab, int64_t hidden, const int64_t* token_ids, int64_t count,
                     void* out, void* stream) {
    CPPINF_REQUIRE(vocab > 0 && hidden > 0 && count >= 0, CPPINF_ERR_INVALID_ARGUMENT,
                   "embedding_lookup requires a non-empty rank-2 embedding table.");
    CPPINF_REQUIRE(hidden % 8 == 0, CPPINF_ERR_UNSUPPORTED, "embedding requires hidden to be a multiple of 8.");
    if (count == 0) {
        return rt::ok();
    }
    CPPINF_REQUIRE(table && token_ids && out, CPPINF_ERR_INVALID_ARGUMENT, "embedding received a null pointer.");
    CPPINF_REQUIRE(rt::aligned16(table) && rt::aligned16(out), CPPINF_ERR_UNSUPPORTED,
                   "embedding requires 16-byte aligned rows.");
    return rt::launched(launch_embedding(static_cast<const bf16*>(table), vocab, hidden, token_ids, count,
                                         static_cast<bf16*>(out), rt::as_stream(stream)),
                        "embedding");
}

}  // extern "C"
