// Tensor-core (tcgen05) projections for the prompt rows: the linear_project of src/nn/qwen_common.cpp:15-37
// (ops::matmul, src/ops/matmul.cpp:85-114: x [M, K] times weight [N, K] transposed) with the decoder's epilogues,
// for M >= 64 rows. This path is opt-in (cppinf_linear_tc, cppinf_qwen3_set_prefill): its f32 accumulation happens
// inside the tensor cores in an order the CPU cannot restate, so it is held to tolerance parity, while the CUDA-core
// kernels of linear.cu (fixed, restated order) stay the default for bit-exact greedy tokens.
//
// One CTA of 4 warps per 128 x kBN output tile (kBN = 32, 64 or 128, picked so the grid covers the SMs):
//  - warp 0, one lane: TMA producer. Per 64-wide K block it loads the x tile [128, 64] and the weight tile(s)
//    [kBN, 64] (two for SiLU * up: gate and up) with cp.async.bulk.tensor (128-byte swizzle, no multicast; rows past
//    M or N and columns past K read as zeros) into a ring of kStages shared-memory stages, each completed on its
//    `full` mbarrier;
//  - warp 1, one lane: MMA issuer. tcgen05.mma.cta_group::1.kind::f16 (bf16 inputs, f32 accumulator in tensor
//    memory, 128 x kBN x 16 per instruction, four per K block), then tcgen05.commit onto the stage's `empty` mbarrier
//    so the producer can refill it once the tensor cores have read it; a last commit marks the accumulator done;
//  - all 4 warps: epilogue. Warp w reads tensor-memory lanes 32w .. 32w + 31 (= tile rows) with tcgen05.ld, 32
//    columns at a time, and applies the decoder's epilogue in registers (bf16 store into the q|k|v segments, residual
//    add, or SiLU(gate) * up -- the latter with the hardware exponential, this path being held to tolerance).
// Every mbarrier wait polls a bounded number of times; a wait that runs out sets *error (when given), the kernel
// carries on with meaningless data so every barrier still completes, and it waits again with the default limit for
// the tensor cores before freeing tensor memory.
//
// Roofline: tensor-bound for M = 512 at the 0.6B shapes (2 M N K flops over (M K + N K + M N) * 2 bytes: 128-340
// flop per byte).
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"
#include "decoder.h"
#include "runtime.h"
#include "tcgen05.cuh"

namespace cppinf::device {
namespace {

using namespace tc;

constexpr int kTcThreads = 128;

// SiLU for this tolerance-held path: the hardware exponential and a fast division (the portable exponential and the
// IEEE division of the bit-exact kernels cost ~40 instructions an element, which made the SiLU * up epilogue the
// longest part of the kernel). The argument is clamped so the divisor stays below 2^126, where __fdividef is
// accurate; below -80 SiLU is ~0 either way.
__device__ __forceinline__ float silu_fast(float x) {
    return __fdividef(x, 1.0f + __expf(fminf(-x, 80.0f)));
}

template <int kBN, int kMats>
struct TcShape {
    static constexpr int kStages = kMats == 2 && kBN >= 64 ? 3 : 4;
    static constexpr uint32_t kABytes = kBM * kBK * 2;   // 16 KB
    static constexpr uint32_t kBBytes = kBN * kBK * 2;   // 4, 8 or 16 KB
    static constexpr uint32_t kStageBytes = kABytes + kMats * kBBytes;
    static constexpr uint32_t kTmemCols = kMats * kBN;   // 32 .. 256, a power of two
    // 1024 bytes of alignment slack, the stages, then the barriers and the tensor-memory address.
    static constexpr std::size_t kSmem = 1024 + kStages * kStageBytes + 256;
};

template <LinearEpilogue kEpi, int kBN>
__global__ void __launch_bounds__(kTcThreads, 1)
    linear_tc_kernel(const __grid_constant__ CUtensorMap map_x, const __grid_constant__ CUtensorMap map_w0,
                     const __grid_constant__ CUtensorMap map_w1, const LinearParams p) {
    constexpr int kMats = kEpi == LinearEpilogue::kSiluMul ? 2 : 1;
    using S = TcShape<kBN, kMats>;
    constexpr int kStages = S::kStages;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t{1023});
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * S::kStageBytes);
    uint64_t* empty = full + kStages;
    uint64_t* done = empty + kStages;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
    int* issued_slot = reinterpret_cast<int*>(tmem_slot + 1);  // K blocks the producer issued
    int* consumed_slot = issued_slot + 1;                        // K blocks the MMA issuer consumed
    int* failed_slot = consumed_slot + 1;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int m0 = blockIdx.x * kBM;
    const int n0 = blockIdx.y * kBN;
    const int num_kb = static_cast<int>((p.K + kBK - 1) / kBK);
    constexpr uint32_t idesc = idesc_bf16_f32(kBN);

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(done, 1);
        *failed_slot = 0;
        asm volatile("prefetch.tensormap [%0];" ::"l"(&map_x) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(&map_w0) : "memory");
    }
    if (warp == 0) {
        tmem_alloc(tmem_slot, S::kTmemCols);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    // Inputs may come from the previous kernel in the stream: every global read follows the dependency wait.
    grid_dependency_begin();

    bool failed = false;
    if (warp == 0 && lane == 0) {
        // Producer.
        int kb = 0;
        for (; kb < num_kb; ++kb) {
            const int s = kb % kStages;
            const auto use = static_cast<uint32_t>(kb / kStages);
            if (kb >= kStages && !mbar_wait_bounded(&empty[s], (use + 1) & 1u, p.poll_limit)) {
                failed = true;
                break;
            }
            unsigned char* stage = smem + s * S::kStageBytes;
            mbar_arrive_expect_tx(&full[s], S::kStageBytes);
            tma_load_2d(stage, &map_x, kb * kBK, m0, &full[s]);
            tma_load_2d(stage + S::kABytes, &map_w0, kb * kBK, n0, &full[s]);
            if constexpr (kMats == 2) {
                tma_load_2d(stage + S::kABytes + S::kBBytes, &map_w1, kb * kBK, n0, &full[s]);
            }
        }
        *issued_slot = kb;
    } else if (warp == 1 && lane == 0) {
        // MMA issuer.
        int kb = 0;
        for (; kb < num_kb; ++kb) {
            const int s = kb % kStages;
            if (!mbar_wait_bounded(&full[s], static_cast<uint32_t>(kb / kStages) & 1u, p.poll_limit)) {
                failed = true;
                break;
            }
            tc_fence_after();
            const unsigned char* stage = smem + s * S::kStageBytes;
#pragma unroll
            for (int k = 0; k < kBK / kUmmaK; ++k) {
                const uint64_t a = smem_desc_sw128(stage, k * kUmmaK * 2);
                const uint64_t b0 = smem_desc_sw128(stage + S::kABytes, k * kUmmaK * 2);
                const uint32_t acc = (kb > 0 || k > 0) ? 1u : 0u;
                umma_bf16(tmem, a, b0, idesc, acc);
                if constexpr (kMats == 2) {
                    const uint64_t b1 = smem_desc_sw128(stage + S::kABytes + S::kBBytes, k * kUmmaK * 2);
                    umma_bf16(tmem + kBN, a, b1, idesc, acc);
                }
            }
            umma_commit(&empty[s]);  // the stage is free once these MMAs have read it
        }
        umma_commit(done);  // the accumulator is complete once every MMA issued above has
        *consumed_slot = kb;
    }
    if (failed) {
        atomicOr(reinterpret_cast<unsigned int*>(failed_slot), 1u);
        if (p.error != nullptr) {
            atomicOr(p.error, 1u);
        }
    }
    __syncthreads();
    const bool any_failed = *failed_slot != 0;

    // Every thread waits for the accumulator (the default limit: on a failed run this is the cleanup wait that lets
    // the tensor cores finish before tensor memory is freed).
    bool ready = mbar_wait_bounded(done, 0u, any_failed ? kDefaultPollLimit : p.poll_limit);
    if (!ready) {
        if (p.error != nullptr && threadIdx.x == 0) {
            atomicOr(p.error, 1u);
        }
        mbar_wait_bounded(done, 0u);  // the tensor cores finish before tensor memory is freed
    }
    if (any_failed && threadIdx.x == 0) {
        // Copies issued but never consumed by an MMA must land before this CTA leaves.
        for (int kb = *consumed_slot; kb < *issued_slot; ++kb) {
            mbar_wait_bounded(&full[kb % kStages], static_cast<uint32_t>(kb / kStages) & 1u);
        }
    }
    const bool skip = __syncthreads_or(any_failed || !ready) != 0;
    tc_fence_after();

    if (!skip) {
        const int64_t m = m0 + warp * 32 + lane;  // this thread's tile row = tensor-memory lane
        const uint32_t lane_base = tmem + (static_cast<uint32_t>(warp * 32) << 16);
#pragma unroll 1
        for (int c0 = 0; c0 < kBN; c0 += 32) {
            float acc[32];
            tmem_load32(lane_base + c0, acc);
            const int64_t n = n0 + c0;
            uint32_t packed[16];
            if constexpr (kEpi == LinearEpilogue::kStore) {
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    packed[j] = pack_bf16x2(acc[2 * j], acc[2 * j + 1]);
                }
            } else if constexpr (kEpi == LinearEpilogue::kResidual) {
                uint4 res[4] = {};
                if (m < p.M && n < p.N) {
                    const bf16* rrow = p.residual + m * p.res_ld + n;
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        res[q] = ld_cached(rrow + 8 * q);
                    }
                }
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    float r[8];
                    Vec16<bf16>::unpack(res[q], r);
#pragma unroll
                    for (int e = 0; e < 8; e += 2) {
                        packed[4 * q + e / 2] = pack_bf16x2(r[e] + round_to_bf16(acc[8 * q + e]),
                                                            r[e + 1] + round_to_bf16(acc[8 * q + e + 1]));
                    }
                }
            } else {
                float up[32];
                tmem_load32(lane_base + kBN + c0, up);
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const float g0 = round_to_bf16(acc[2 * j]);
                    const float g1 = round_to_bf16(acc[2 * j + 1]);
                    packed[j] = pack_bf16x2(round_to_bf16(silu_fast(g0)) * round_to_bf16(up[2 * j]),
                                            round_to_bf16(silu_fast(g1)) * round_to_bf16(up[2 * j + 1]));
                }
            }
            if (m < p.M && n < p.N) {
                // The whole 32-column chunk lies in one output segment (segment starts are multiples of 32).
                const int k = kEpi == LinearEpilogue::kStore ? (n >= p.seg[2] ? 2 : (n >= p.seg[1] ? 1 : 0)) : 0;
                bf16* dst = p.out[k] + (m + p.row_offset[k]) * p.ld[k] + (n - p.seg[k]);
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    st_v4(dst + 8 * q, make_uint4(packed[4 * q], packed[4 * q + 1], packed[4 * q + 2], packed[4 * q + 3]));
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, S::kTmemCols);
    }
}

// ---- host side ---------------------------------------------------------------------------------------------------

// A [rows, cols] bf16 row-major matrix (row stride in elements) read in boxes of [box_rows, 64] with the 128-byte
// swizzle; out-of-range rows and columns read as zeros.
bool make_map(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, int64_t row_stride, int box_rows) {
    const EncodeTiled encode = encode_tiled();
    if (encode == nullptr) {
        return false;
    }
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_stride) * 2};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(kBK), static_cast<cuuint32_t>(box_rows)};
    const cuuint32_t elem_strides[2] = {1, 1};
    return encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, elem_strides,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <LinearEpilogue kEpi, int kBN>
cudaError_t launch_tc(const LinearParams& p, cudaStream_t s) {
    constexpr int kMats = kEpi == LinearEpilogue::kSiluMul ? 2 : 1;
    using S = TcShape<kBN, kMats>;
    CUtensorMap mx{};
    CUtensorMap mw0{};
    CUtensorMap mw1{};
    if (!make_map(&mx, p.x, p.M, p.K, p.x_stride, kBM) || !make_map(&mw0, p.w0, p.N, p.K, p.K, kBN) ||
        !make_map(&mw1, kMats == 2 ? p.w1 : p.w0, p.N, p.K, p.K, kBN)) {
        return cudaErrorInvalidValue;
    }
    auto kernel = linear_tc_kernel<kEpi, kBN>;
    const cudaError_t err =
        cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(S::kSmem));
    if (err != cudaSuccess) {
        return err;
    }
    const dim3 grid(static_cast<unsigned>((p.M + kBM - 1) / kBM), static_cast<unsigned>((p.N + kBN - 1) / kBN));
    return runtime::launch_smem(kernel, grid, dim3(kTcThreads), S::kSmem, s, 1u, mx, mw0, mw1, p);
}

// Tile width: the widest of 128, 64, 32 whose grid still gives most SMs a tile.
template <LinearEpilogue kEpi>
cudaError_t launch_tc_epi(const LinearParams& p, cudaStream_t s) {
    const int64_t tiles_m = (p.M + kBM - 1) / kBM;
    const int64_t want = runtime::sm_count() * 3 / 4;
    if (tiles_m * ((p.N + 127) / 128) >= want) {
        return launch_tc<kEpi, 128>(p, s);
    }
    if (tiles_m * ((p.N + 63) / 64) >= want) {
        return launch_tc<kEpi, 64>(p, s);
    }
    return launch_tc<kEpi, 32>(p, s);
}

bool aligned16(const void* ptr) {
    return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0;
}

}  // namespace

bool linear_tc_supported(const LinearParams& p) {
    if (p.epilogue == LinearEpilogue::kArgmax || p.tokens != nullptr || p.position != nullptr ||
        p.norm_weight != nullptr || p.x_copy != nullptr) {
        return false;
    }
    if (p.M < 1 || p.N < 32 || p.N % 32 != 0 || p.K < 8 || p.K % 8 != 0 || p.x_stride % 8 != 0 ||
        p.M > (int64_t{1} << 31) - kBM || p.N > (int64_t{1} << 31) - 128 || p.K > (int64_t{1} << 31)) {
        return false;
    }
    if (!aligned16(p.x) || !aligned16(p.w0) || (p.epilogue == LinearEpilogue::kSiluMul && !aligned16(p.w1))) {
        return false;
    }
    const int segments = p.epilogue == LinearEpilogue::kStore ? 3 : 1;
    for (int k = 0; k < segments; ++k) {
        if (k > 0 && p.seg[k] >= p.N) {
            break;
        }
        if (p.out[k] == nullptr || !aligned16(p.out[k]) || p.ld[k] % 8 != 0 || p.seg[k] % 32 != 0) {
            return false;
        }
    }
    if (p.epilogue == LinearEpilogue::kResidual && (!aligned16(p.residual) || p.res_ld % 8 != 0)) {
        return false;
    }
    return encode_tiled() != nullptr;
}

cudaError_t launch_linear_tc(const LinearParams& p, cudaStream_t s) {
    if (!linear_tc_supported(p)) {
        return cudaErrorNotSupported;
    }
    switch (p.epilogue) {
    case LinearEpilogue::kStore:
        return launch_tc_epi<LinearEpilogue::kStore>(p, s);
    case LinearEpilogue::kResidual:
        return launch_tc_epi<LinearEpilogue::kResidual>(p, s);
    case LinearEpilogue::kSiluMul:
        return launch_tc_epi<LinearEpilogue::kSiluMul>(p, s);
    default:
        return cudaErrorNotSupported;
    }
}

}  // namespace cppinf::device

using namespace cppinf::device;
namespace rt = cppinf::runtime;

extern "C" {

int cppinf_linear_tc(int epilogue, const void* x, int64_t x_row_stride, const void* w0, const void* w1,
                     const void* residual, void* y, int64_t rows, int64_t in_features, int64_t out_features,
                     unsigned int* error, void* stream) {
    CPPINF_REQUIRE(epilogue >= 0 && epilogue <= 2, CPPINF_ERR_INVALID_ARGUMENT,
                   "linear_tc epilogue must be 0 (store), 1 (residual add) or 2 (SiLU * up).");
    CPPINF_REQUIRE(rows >= 0 && in_features > 0 && out_features >= 0, CPPINF_ERR_INVALID_ARGUMENT,
                   "linear requires non-negative sizes and a non-empty input dimension.");
    CPPINF_REQUIRE(rows <= 1 || x_row_stride >= in_features, CPPINF_ERR_INVALID_ARGUMENT,
                   "linear requires an input row stride of at least in_features.");
    if (rows == 0 || out_features == 0) {
        return rt::ok();
    }
    CPPINF_REQUIRE(x && w0 && y && (epilogue != 2 || w1) && (epilogue != 1 || residual), CPPINF_ERR_INVALID_ARGUMENT,
                   "linear received a null pointer.");
    LinearParams p{};
    p.epilogue = static_cast<LinearEpilogue>(epilogue);
    p.x = static_cast<const bf16*>(x);
    p.x_stride = rows <= 1 ? in_features : x_row_stride;
    p.w0 = static_cast<const bf16*>(w0);
    p.w1 = static_cast<const bf16*>(w1);
    p.M = rows;
    p.N = out_features;
    p.K = in_features;
    p.out[0] = static_cast<bf16*>(y);
    p.ld[0] = out_features;
    p.seg[1] = p.seg[2] = p.seg[3] = out_features;
    p.residual = static_cast<const bf16*>(residual);
    p.res_ld = out_features;
    p.error = error;
    p.poll_limit = rt::wait_poll_limit();
    CPPINF_REQUIRE(linear_tc_supported(p), CPPINF_ERR_UNSUPPORTED,
                   "linear_tc needs out_features % 32 == 0, in_features and the row stride % 8 == 0, 16-byte aligned "
                   "operands and the driver's tensor-map encoder.");
    return rt::launched(launch_linear_tc(p, rt::as_stream(stream)), "linear_tc");
}

}  // extern "C"
