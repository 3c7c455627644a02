// Prompt attention on the tensor cores (tcgen05), for the opt-in tensor-core prefill (cppinf_qwen3_set_prefill 1):
// the fused_causal_attention of src/nn/qwen_attention.cpp:237-333 for queries whose keys are in the cache -- scores
// q k^T in f32, scaled by 1/sqrt(D), the causal softmax with the probabilities rounded to bf16 before they multiply
// V (:320-327), context in bf16 -- for head_dim 128. Like the tensor-core projections it is held to tolerance parity:
// the tensor cores' f32 accumulation order and the one-pass running sum below are not the restated order of
// attention.cu, which stays the default.
//
// One CTA of 4 warps per (tile of 128 queries, query head); thread r owns query row r, which is tensor-memory lane r.
// Keys go in tiles of 128:
//  - pass 1: S = Q K^T (TMA loads Q once and each K tile with the 128-byte swizzle; 8 UMMAs of 128 x 128 x 16 into
//    tensor-memory columns [0, 128)); each thread reads its row and keeps the running maximum M and the running
//    sum of exp(x - M) of its visible keys (x = S / sqrt(D); keys past its position are masked);
//  - pass 2: S again; p = bf16(exp(x - M) / sum) (0 when masked; the fast exponential and one reciprocal of the
//    sum, as this path is held to tolerance) is written into shared memory as the K-major A
//    operand (swizzled by hand, the layout TMA would produce); the V tile, loaded by TMA as [keys][dims], is
//    transposed in shared memory into the K-major B operand [dims][keys]; O += P V (8 UMMAs into columns
//    [128, 256)).
//  - the context rows come out of tensor memory by tcgen05.ld, rounded to bf16.
// Every step waits for the previous one (no overlap between tiles): the kernel's job is to take the attention's
// contractions off the CUDA cores, not yet to pipeline them. Waits poll a bounded number of times; one that runs out
// sets *error and waits again with the default limit, so the protocol always completes.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "common.cuh"
#include "decoder.h"
#include "runtime.h"
#include "tcgen05.cuh"

namespace cppinf::device {
namespace {

using namespace tc;

constexpr int kAttD = 128;      // head_dim
constexpr int kKeyTile = 128;   // keys per tile (UMMA N of the scores, K of P V)
constexpr int kAttThreads = 128;
constexpr uint32_t kAtom = kBM * 128;         // one [128 rows][64 bf16] swizzled atom: 16 KB
constexpr uint32_t kTile = 2 * kAtom;         // a [128 rows][128 bf16] operand: two atoms along its K
constexpr uint32_t kTmemCols = 256;           // S in [0, 128), O in [128, 256)

struct AttnTcParams {
    __nv_bfloat16* ctx;  // [T, Hq, D]
    int64_t T;
    int q_heads;
    int kv_heads;
    int64_t pos0;        // position of query 0
    int64_t capacity;    // cache rows
    unsigned int* error;
    uint32_t poll_limit;
};

// Shared memory, 1024-byte aligned: Q, K, V (as TMA writes them) and the two UMMA operands built by the threads.
struct AttnSmem {
    static constexpr uint32_t kQ = 0;
    static constexpr uint32_t kK = kQ + kTile;
    static constexpr uint32_t kV = kK + kTile;
    static constexpr uint32_t kVT = kV + kTile;
    static constexpr uint32_t kP = kVT + kTile;
    static constexpr uint32_t kBars = kP + kTile;
    static constexpr std::size_t kBytes = 1024 + kBars + 128;
};

// Byte offset of element (row, k) of a K-major operand [128 rows][128 k] stored as two 128-byte-swizzled atoms along
// k (k 0-63, 64-127): the 16-byte chunk index within the row is XORed with row % 8, the layout TMA's SWIZZLE_128B
// produces and the UMMA descriptors expect.
__device__ __forceinline__ uint32_t sw128_offset(int row, int k) {
    const int atom = k >> 6;
    const int chunk = (k & 63) >> 3;
    return static_cast<uint32_t>(atom) * kAtom + static_cast<uint32_t>(row) * 128u +
           static_cast<uint32_t>((chunk ^ (row & 7)) << 4) + static_cast<uint32_t>((k & 7) << 1);
}

// Waits for `phase` of `bar`; a wait that runs out of the poll limit records the error and waits again with the
// default limit, so the operation it waits for has completed either way.
__device__ __forceinline__ void att_wait(uint64_t* bar, uint32_t phase, const AttnTcParams& p) {
    if (!mbar_wait_bounded(bar, phase, p.poll_limit)) {
        if (p.error != nullptr) {
            atomicOr(p.error, 1u);
        }
        mbar_wait_bounded(bar, phase);
    }
}

__global__ void __launch_bounds__(kAttThreads, 1)
    attention_tc_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                        const __grid_constant__ CUtensorMap map_v, const AttnTcParams p) {
    extern __shared__ __align__(16) unsigned char att_raw[];
    // 1024-byte aligned base, derived from the shared array itself so accesses stay shared-memory instructions.
    unsigned char* sm = att_raw + ((1024u - (smem_addr(att_raw) & 1023u)) & 1023u);
    unsigned char* sQ = sm + AttnSmem::kQ;
    unsigned char* sK = sm + AttnSmem::kK;
    unsigned char* sV = sm + AttnSmem::kV;
    unsigned char* sVT = sm + AttnSmem::kVT;
    unsigned char* sP = sm + AttnSmem::kP;
    uint64_t* bar_q = reinterpret_cast<uint64_t*>(sm + AttnSmem::kBars);
    uint64_t* bar_k = bar_q + 1;
    uint64_t* bar_v = bar_q + 2;
    uint64_t* bar_mma = bar_q + 3;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_q + 4);

    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int h = static_cast<int>(blockIdx.y);
    const int kvh = h / (p.q_heads / p.kv_heads);
    const int64_t m0 = static_cast<int64_t>(blockIdx.x) * kBM;
    const int64_t t = m0 + tid;                       // this thread's query
    const int64_t pos = p.pos0 + t;
    const int64_t L = (t < p.T && pos < p.capacity) ? pos + 1 : 0;  // visible keys of the row
    const int64_t t_end = m0 + kBM < p.T ? m0 + kBM : p.T;
    const int64_t lmax_raw = p.pos0 + t_end;
    const int64_t lmax = lmax_raw < p.capacity ? lmax_raw : p.capacity;  // keys the tile needs
    const int ntiles = static_cast<int>((lmax + kKeyTile - 1) / kKeyTile);
    const float scale = 1.0f / sqrtf(static_cast<float>(kAttD));
    constexpr uint32_t idesc = idesc_bf16_f32(kKeyTile);  // N = 128 for both contractions (keys, then dims)

    if (tid == 0) {
        mbar_init(bar_q, 1);
        mbar_init(bar_k, 1);
        mbar_init(bar_v, 1);
        mbar_init(bar_mma, 1);
    }
    if (warp == 0) {
        tmem_alloc(tmem_slot, kTmemCols);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t tmem_s = tmem;
    const uint32_t tmem_o = tmem + kKeyTile;
    const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;

    grid_dependency_begin();  // q and the cache rows come from the previous kernels
    uint32_t ph_k = 0;
    uint32_t ph_v = 0;
    uint32_t ph_mma = 0;
    if (tid == 0) {
        mbar_arrive_expect_tx(bar_q, kTile);
        tma_load_3d(sQ, &map_q, 0, h, static_cast<int>(m0), bar_q);
        tma_load_3d(sQ + kAtom, &map_q, 64, h, static_cast<int>(m0), bar_q);
    }
    att_wait(bar_q, 0, p);

    // S = Q K^T of key tile `kt` into tensor-memory columns [0, 128) (issued by thread 0; all threads wait).
    const auto scores = [&](int kt) {
        if (tid == 0) {
            mbar_arrive_expect_tx(bar_k, kTile);
            tma_load_3d(sK, &map_k, 0, kvh, kt * kKeyTile, bar_k);
            tma_load_3d(sK + kAtom, &map_k, 64, kvh, kt * kKeyTile, bar_k);
        }
        att_wait(bar_k, ph_k, p);
        ph_k ^= 1u;
        if (tid == 0) {
            tc_fence_after();
#pragma unroll
            for (int k = 0; k < kAttD / kUmmaK; ++k) {
                const uint32_t off = static_cast<uint32_t>(k >> 2) * kAtom + static_cast<uint32_t>(k & 3) * 32u;
                umma_bf16(tmem_s, smem_desc_sw128(sQ, off), smem_desc_sw128(sK, off), idesc, k > 0 ? 1u : 0u);
            }
            umma_commit(bar_mma);
        }
        att_wait(bar_mma, ph_mma, p);
        ph_mma ^= 1u;
        tc_fence_after();
    };

    // ---- pass 1: running maximum and exp sum of each row's visible scores -----------------------------------------
    float run_max = -INFINITY;
    float run_sum = 0.0f;
    for (int kt = 0; kt < ntiles; ++kt) {
        scores(kt);
#pragma unroll 1
        for (int c = 0; c < kKeyTile / 32; ++c) {
            float x[32];
            tmem_load32(tmem_s + lane_base + c * 32, x);
            const int64_t key0 = static_cast<int64_t>(kt) * kKeyTile + c * 32;
            float cmax = -INFINITY;
#pragma unroll
            for (int j = 0; j < 32; ++j) {
                x[j] = key0 + j < L ? x[j] * scale : -INFINITY;
                cmax = fmaxf(cmax, x[j]);
            }
            // Masked scores are -inf and contribute exp(-inf) = 0; a row with no visible key yet keeps M = -inf.
            const float new_max = fmaxf(run_max, cmax);
            if (new_max != -INFINITY) {
                float csum = 0.0f;
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    csum += __expf(x[j] - new_max);
                }
                run_sum = (run_max == -INFINITY ? 0.0f : run_sum * __expf(run_max - new_max)) + csum;
                run_max = new_max;
            }
            __syncwarp();  // the next tcgen05.ld is warp-collective
        }
        tc_fence_before();
        __syncthreads();  // every row is read before the next tile's scores overwrite tensor memory
    }

    // ---- pass 2: probabilities, then O += P V ---------------------------------------------------------------------
    const float inv_sum = L > 0 ? 1.0f / run_sum : 0.0f;
    for (int kt = 0; kt < ntiles; ++kt) {
        if (tid == 0) {
            mbar_arrive_expect_tx(bar_v, kTile);
            tma_load_3d(sV, &map_v, 0, kvh, kt * kKeyTile, bar_v);
            tma_load_3d(sV + kAtom, &map_v, 64, kvh, kt * kKeyTile, bar_v);
        }
        scores(kt);
        // Row tid of P (keys of this tile), rounded to bf16 like the reference's probabilities.
#pragma unroll 1
        for (int c = 0; c < kKeyTile / 32; ++c) {
            float x[32];
            tmem_load32(tmem_s + lane_base + c * 32, x);
            const int64_t key0 = static_cast<int64_t>(kt) * kKeyTile + c * 32;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                uint32_t w[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int j = q * 8 + 2 * e;
                    const float p0 = key0 + j < L ? __expf(x[j] * scale - run_max) * inv_sum : 0.0f;
                    const float p1 = key0 + j + 1 < L ? __expf(x[j + 1] * scale - run_max) * inv_sum : 0.0f;
                    w[e] = pack_bf16x2(p0, p1);
                }
                *reinterpret_cast<uint4*>(sP + sw128_offset(tid, c * 32 + q * 8)) = make_uint4(w[0], w[1], w[2], w[3]);
            }
        }
        // V tile [keys][dims] -> V^T [dims][keys]: thread tid builds dim row tid; keys past the tile's needed range
        // are zeros (their rows may hold anything).
        att_wait(bar_v, ph_v, p);
        ph_v ^= 1u;
#pragma unroll 1
        for (int kc = 0; kc < kKeyTile / 8; ++kc) {
            uint32_t w[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int k0 = kc * 8 + 2 * e;
                const int64_t g0 = static_cast<int64_t>(kt) * kKeyTile + k0;
                const uint16_t lo = g0 < lmax ? *reinterpret_cast<const uint16_t*>(sV + sw128_offset(k0, tid)) : 0;
                const uint16_t hi =
                    g0 + 1 < lmax ? *reinterpret_cast<const uint16_t*>(sV + sw128_offset(k0 + 1, tid)) : 0;
                w[e] = static_cast<uint32_t>(lo) | (static_cast<uint32_t>(hi) << 16);
            }
            *reinterpret_cast<uint4*>(sVT + sw128_offset(tid, kc * 8)) = make_uint4(w[0], w[1], w[2], w[3]);
        }
        fence_proxy_async_smem();  // the threads' operand writes, before the tensor cores read them
        tc_fence_before();
        __syncthreads();
        if (tid == 0) {
            tc_fence_after();
#pragma unroll
            for (int k = 0; k < kKeyTile / kUmmaK; ++k) {
                const uint32_t off = static_cast<uint32_t>(k >> 2) * kAtom + static_cast<uint32_t>(k & 3) * 32u;
                umma_bf16(tmem_o, smem_desc_sw128(sP, off), smem_desc_sw128(sVT, off), idesc,
                          (kt > 0 || k > 0) ? 1u : 0u);
            }
            umma_commit(bar_mma);
        }
        att_wait(bar_mma, ph_mma, p);  // P, V^T and S are free again once these have completed
        ph_mma ^= 1u;
        tc_fence_after();
    }

    // ---- context rows ----------------------------------------------------------------------------------------------
    if (ntiles > 0) {
#pragma unroll 1
        for (int c = 0; c < kAttD / 32; ++c) {
            float o[32];
            tmem_load32(tmem_o + lane_base + c * 32, o);
            if (L > 0) {
                bf16* dst = p.ctx + (t * p.q_heads + h) * kAttD + c * 32;
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    st_v4(dst + 8 * q, make_uint4(pack_bf16x2(o[8 * q], o[8 * q + 1]), pack_bf16x2(o[8 * q + 2], o[8 * q + 3]),
                                                  pack_bf16x2(o[8 * q + 4], o[8 * q + 5]),
                                                  pack_bf16x2(o[8 * q + 6], o[8 * q + 7])));
                }
            }
            __syncwarp();  // the next tcgen05.ld is warp-collective
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

// [rows, heads, 128] bf16 (head stride 128, row stride heads * 128) read in boxes of [128 rows][1 head][64 dims] with
// the 128-byte swizzle; rows past `rows` read as zeros.
bool make_head_map(CUtensorMap* map, const void* base, int64_t rows, int heads) {
    const EncodeTiled encode = encode_tiled();
    if (encode == nullptr) {
        return false;
    }
    const cuuint64_t dims[3] = {static_cast<cuuint64_t>(kAttD), static_cast<cuuint64_t>(heads),
                                static_cast<cuuint64_t>(rows)};
    const cuuint64_t strides[2] = {static_cast<cuuint64_t>(kAttD) * 2, static_cast<cuuint64_t>(heads) * kAttD * 2};
    const cuuint32_t box[3] = {64, 1, static_cast<cuuint32_t>(kBM)};
    const cuuint32_t elem_strides[3] = {1, 1, 1};
    return encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box,
                  elem_strides, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

bool attention_tc_supported(const AttentionParams& p) {
    const auto a16 = [](const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; };
    return p.head_dim == kAttD && p.position == nullptr && p.q_norm == nullptr && p.T >= 1 && p.q_heads > 0 &&
           p.kv_heads > 0 && p.q_heads % p.kv_heads == 0 && p.capacity < (int64_t{1} << 30) &&
           p.T < (int64_t{1} << 30) && a16(p.q) && a16(p.k_cache) && a16(p.v_cache) && a16(p.ctx) &&
           encode_tiled() != nullptr;
}

cudaError_t launch_attention_tc(const AttentionParams& p, cudaStream_t s) {
    if (!attention_tc_supported(p)) {
        return cudaErrorNotSupported;
    }
    CUtensorMap mq{};
    CUtensorMap mk{};
    CUtensorMap mv{};
    if (!make_head_map(&mq, p.q, p.T, p.q_heads) || !make_head_map(&mk, p.k_cache, p.capacity, p.kv_heads) ||
        !make_head_map(&mv, p.v_cache, p.capacity, p.kv_heads)) {
        return cudaErrorInvalidValue;
    }
    AttnTcParams ap{};
    ap.ctx = p.ctx;
    ap.T = p.T;
    ap.q_heads = p.q_heads;
    ap.kv_heads = p.kv_heads;
    ap.pos0 = p.pos0;
    ap.capacity = p.capacity;
    ap.error = p.error;
    ap.poll_limit = p.poll_limit;
    const cudaError_t err = cudaFuncSetAttribute(attention_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 static_cast<int>(AttnSmem::kBytes));
    if (err != cudaSuccess) {
        return err;
    }
    const dim3 grid(static_cast<unsigned>((p.T + kBM - 1) / kBM), static_cast<unsigned>(p.q_heads));
    return runtime::launch_smem(attention_tc_kernel, grid, dim3(kAttThreads), AttnSmem::kBytes, s, 1u, mq, mk, mv, ap);
}

}  // namespace cppinf::device

using namespace cppinf::device;
namespace rt = cppinf::runtime;

extern "C" {

int cppinf_decoder_attention_tc(const void* q, const void* k_cache, const void* v_cache, void* ctx, int64_t tokens,
                                int64_t q_heads, int64_t kv_heads, int64_t head_dim, int64_t position,
                                int64_t capacity, unsigned int* error, void* stream) {
    CPPINF_REQUIRE(tokens >= 0 && q_heads > 0 && kv_heads > 0 && head_dim > 0, CPPINF_ERR_INVALID_ARGUMENT,
                   "qwen_attention requires non-zero head configuration.");
    CPPINF_REQUIRE(q_heads % kv_heads == 0, CPPINF_ERR_INVALID_ARGUMENT,
                   "qwen_attention requires query heads to divide by key/value heads.");
    CPPINF_REQUIRE(position >= 0, CPPINF_ERR_INVALID_ARGUMENT, "qwen_attention query offsets must be non-negative.");
    CPPINF_REQUIRE(position + tokens <= capacity, CPPINF_ERR_OUT_OF_RANGE,
                   "qwen_attention key lengths exceed the cache capacity.");
    if (tokens == 0) {
        return rt::ok();
    }
    CPPINF_REQUIRE(q && k_cache && v_cache && ctx, CPPINF_ERR_INVALID_ARGUMENT,
                   "qwen_attention received a null pointer.");
    AttentionParams p{};
    p.q = static_cast<const bf16*>(q);
    p.k_cache = static_cast<const bf16*>(k_cache);
    p.v_cache = static_cast<const bf16*>(v_cache);
    p.ctx = static_cast<bf16*>(ctx);
    p.T = tokens;
    p.q_heads = static_cast<int>(q_heads);
    p.kv_heads = static_cast<int>(kv_heads);
    p.head_dim = static_cast<int>(head_dim);
    p.pos0 = position;
    p.capacity = capacity;
    p.error = error;
    p.poll_limit = rt::wait_poll_limit();
    CPPINF_REQUIRE(attention_tc_supported(p), CPPINF_ERR_UNSUPPORTED,
                   "tensor-core attention needs head_dim 128, 16-byte aligned operands and the driver's tensor-map "
                   "encoder.");
    return rt::launched(launch_attention_tc(p, rt::as_stream(stream)), "decoder_attention_tc");
}

}  // extern "C"
