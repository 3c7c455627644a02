// Causal grouped-query attention of the Qwen3 decoder over the KV cache: fused_causal_attention of
// src/nn/qwen_attention.cpp:236-333 (scores q k^T in f32, the position-causal softmax of :164-235, probabilities
// cast to bf16, probabilities times V in bf16) for one sequence, query t at position pos0 + t seeing keys
// 0 .. pos0 + t, query head h reading key/value head h / (Hq / Hkv) (the repeat_interleave of :290-291).
//
// One thread-block cluster of 8 CTAs per (query, head) -- for a prompt, per (run of consecutive queries, head), the
// queries taken one after another; CTA c owns the c-th of 8 parts of the visible keys (P = ceil(L / 8) consecutive
// keys each). The order of every sum is fixed in terms of 128 slots and 4 warp chains per part, and the CPU oracle
// restates it (oracle_decoder_attention); a CTA runs it with 8 warps (the score loop over all of them, each warp
// chain's P·V split into two halves of the dims):
//  - score: the head vector is cut into 8 segments of D / 8 dims, each summed in order by one lane, the 8 partials
//    combined by a butterfly over lane distances 4, 2, 1; x_j = score * (1 / sqrt(D));
//  - per part: m_c = max x_j; S_c: thread i adds exp(x_j - m_c) for j = lo + i, lo + i + 128, ... in order, warp
//    butterfly, the 4 warp sums in order (exp is the portable exp of pexp.cuh);
//  - every part pushes (m_c, S_c) into every CTA's shared memory (DSMEM stores), one cluster barrier, then
//    M = max m_c and total = sum over c in order of S_c * exp(m_c - M);
//  - p_j = bf16(exp(x_j - M) / total);
//  - context: warp w adds p_j v_j for j = lo + w, lo + w + 4, ... in order; the 4 warp sums in order; each part
//    pushes its partial of dims [cD/8, (c+1)D/8) to CTA c, one cluster barrier, CTA c adds the 8 partials in order;
//    stored in bf16.
// Only DSMEM stores carry partial results (no remote loads, no global scratch); two cluster barriers in all (three
// with the fused projection below). Every product-accumulate (scores, P·V) is a fused multiply-add of bf16 values.
//
// Queries whose keys are all in the cache already (prompt chunks, the C ABI entry) with up to 16384 visible keys take
// attention_rows_kernel instead: one CTA of 8 warps per (query, head), warp c playing part c with the same order of
// every sum, and shared memory plus block barriers in place of the cluster (measured on B200: the 512-token prompt of
// Qwen3-0.6B 45.2 -> 35.2 ms). The decode step keeps the cluster kernel: it stages each part's cached K/V rows with
// two TMA tensor copies before its dependency wait, fuses the new token's q/k norm and RoPE, and (for the model's
// common sizes) the input RMSNorm and the q|k|v projection too (kProjC below).
//
// Roofline: latency-bound in decode (a chain of dependent L2 round trips, block and cluster barriers); the bytes are
// 2 * L * D * 2 per query head (shared by the heads of a group through L2) plus, with the fused projection, this
// head's slice of the q|k|v weights.
#include <cooperative_groups.h>

#include "common.cuh"
#include "decoder.h"
#include "pexp.cuh"
#include "runtime.h"
#include "tcgen05.cuh"

namespace cg = cooperative_groups;

namespace cppinf::device {
namespace {

constexpr int kParts = 8;
constexpr int kThreads = 128;
constexpr int kWarps = kThreads / 32;
constexpr int kSegments = 8;  // lanes per key in the score dot product
// The cluster kernel's CTA: 8 warps play the 128 slots and the 4 warp chains of a part (kThreads, kWarps above are
// the restated order's), so each warp's share of the score and P·V loops is half as long.
// Registers are capped at 3 CTAs per SM (80 per thread): the decode step's kernels become resident early under
// programmatic dependent launch only while the neighbouring kernels' CTAs fit beside them (measured on the
// Qwen3-0.6B decode step: uncapped, 118 registers, 1496 tok/s; capped 1657; capped at 4 CTAs, spilling, 1560).
constexpr int kCtaThreads = 256;
constexpr int kCtaWarps = kCtaThreads / 32;

// A lane's kD / 32 values of one V row, loaded raw (so several rows can be in flight) and unpacked at use.
template <int kD>
struct VRow;

template <>
struct VRow<64> {
    using Raw = uint32_t;
    static __device__ __forceinline__ Raw load(const bf16* p) { return __ldg(reinterpret_cast<const unsigned int*>(p)); }
    static __device__ __forceinline__ void unpack(Raw w, float (&v)[2]) {
        v[0] = bf16_lo(w);
        v[1] = bf16_hi(w);
    }
};

template <>
struct VRow<128> {
    using Raw = uint2;
    static __device__ __forceinline__ Raw load(const bf16* p) { return __ldg(reinterpret_cast<const uint2*>(p)); }
    static __device__ __forceinline__ void unpack(Raw w, float (&v)[4]) {
        v[0] = bf16_lo(w.x);
        v[1] = bf16_hi(w.x);
        v[2] = bf16_lo(w.y);
        v[3] = bf16_hi(w.y);
    }
};

// P·V with two hardware warps per warp chain: a lane's kD / 64 values of one V row (the chain's half of the dims).
template <int kD>
struct VHalf;

template <>
struct VHalf<64> {
    using Raw = unsigned short;
    static __device__ __forceinline__ Raw load(const bf16* p) { return __ldg(reinterpret_cast<const unsigned short*>(p)); }
    static __device__ __forceinline__ void unpack(Raw w, float (&v)[1]) { v[0] = __uint_as_float(static_cast<uint32_t>(w) << 16); }
};

template <>
struct VHalf<128> {
    using Raw = uint32_t;
    static __device__ __forceinline__ Raw load(const bf16* p) { return __ldg(reinterpret_cast<const unsigned int*>(p)); }
    static __device__ __forceinline__ void unpack(Raw w, float (&v)[2]) {
        v[0] = bf16_lo(w);
        v[1] = bf16_hi(w);
    }
};

template <>
struct VHalf<256> {
    using Raw = uint2;
    static __device__ __forceinline__ Raw load(const bf16* p) { return __ldg(reinterpret_cast<const uint2*>(p)); }
    static __device__ __forceinline__ void unpack(Raw w, float (&v)[4]) {
        v[0] = bf16_lo(w.x);
        v[1] = bf16_hi(w.x);
        v[2] = bf16_lo(w.y);
        v[3] = bf16_hi(w.y);
    }
};

template <>
struct VRow<256> {
    using Raw = uint4;
    static __device__ __forceinline__ Raw load(const bf16* p) { return ld_cached(p); }
    static __device__ __forceinline__ void unpack(Raw w, float (&v)[8]) { Vec16<bf16>::unpack(w, v); }
};

// Eight elements of a score segment: fused multiply-adds in element order (fma_bf16x8, common.cuh).
__device__ __forceinline__ float dot8(uint4 a, uint4 b, float acc) {
    return fma_bf16x8(a, b, acc);
}

// Per-head RMSNorm + RoPE of one raw head vector into shared memory, with exactly the arithmetic of
// qk_norm_rope_kernel (rope.cu): kD / 16 lanes, lane hl holding dims [8 hl, 8 hl + 8) and the matching dims of the
// second half; the sum of squares in the canonical lane order; normalised values rounded to bf16; then
// (first * cos - second * sin, second * cos + first * sin) rounded to bf16 (src/nn/rope.cpp:100-103). The weights
// (w_first, w_second) and the angles (c, s) of the lane's pairs are loaded by the caller.
// kShared: `src` is in this CTA's shared memory (the fused projection's gathered rows) rather than global memory.
template <int kD, bool kShared = false>
__device__ __forceinline__ void norm_rope_head(const bf16* src, uint4 w_first, uint4 w_second, const float (&c)[8],
                                               const float (&s)[8], float eps, bf16* dst, int lane) {
    constexpr int kLanes = kD / 16;
    constexpr int kHalf = kD / 2;
    const int hl = lane % kLanes;
    float a[8];
    float b[8];
    if constexpr (kShared) {
        Vec16<bf16>::unpack(*reinterpret_cast<const uint4*>(src + hl * 8), a);
        Vec16<bf16>::unpack(*reinterpret_cast<const uint4*>(src + kHalf + hl * 8), b);
    } else {
        Vec16<bf16>::unpack(ld_cached(src + hl * 8), a);
        Vec16<bf16>::unpack(ld_cached(src + kHalf + hl * 8), b);
    }
    // Products as packed f32x2 pairs (first-half element, second-half element), the norm and rotation sums and
    // differences scalar in the same order as rope.cu.
    float2 s2 = make_float2(0.0f, 0.0f);  // the two halves' sums of squares as fused multiply-adds (rope.cu's bf16 path)
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const float2 v = make_float2(a[j], b[j]);
        s2 = __ffma2_rn(v, v, s2);
    }
    const float ss = group_sum<kLanes>(s2.x + s2.y);
    const float mean = ss / static_cast<float>(kD);
    const float rms = sqrtf(mean + eps);
    const float inv = 1.0f / rms;
    const float2 inv2 = make_float2(inv, inv);
    float wa[8];
    float wb[8];
    Vec16<bf16>::unpack(w_first, wa);
    Vec16<bf16>::unpack(w_second, wb);
    float out_a[8];
    float out_b[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const float2 x = __fmul2_rn(__fmul2_rn(make_float2(a[j], b[j]), inv2), make_float2(wa[j], wb[j]));
        const float n1 = round_to_bf16(x.x);
        const float n2 = round_to_bf16(x.y);
        const float2 nc = __fmul2_rn(make_float2(n1, n2), make_float2(c[j], c[j]));  // n1 * c, n2 * c
        const float2 ns = __fmul2_rn(make_float2(n2, n1), make_float2(s[j], s[j]));  // n2 * s, n1 * s
        out_a[j] = nc.x - ns.x;
        out_b[j] = nc.y + ns.y;
    }
    if (lane < kLanes) {
        *reinterpret_cast<uint4*>(dst + hl * 8) = Vec16<bf16>::pack(out_a);
        *reinterpret_cast<uint4*>(dst + kHalf + hl * 8) = Vec16<bf16>::pack(out_b);
    }
}

// Row `row` of the fused q|k|v weight matrix's part m (0: W_q rows of head h, 1: W_k, 2: W_v rows of key/value head
// kvh), counted from the head's first row.
template <int kD>
__device__ __forceinline__ const bf16* proj_row(const AttentionParams& p, int m, int h, int kvh, int row) {
    const int64_t q_dim = static_cast<int64_t>(p.q_heads) * kD;
    const int64_t kv_dim = static_cast<int64_t>(p.kv_heads) * kD;
    const int64_t first = m == 0 ? static_cast<int64_t>(h) * kD
                                 : (m == 1 ? q_dim : q_dim + kv_dim) + static_cast<int64_t>(kvh) * kD;
    return p.wqkv + (first + row) * p.hidden;
}

// The decode kernel's staging copies: TMA maps of the K and V caches, each a 3-D tensor [cap][Hkv][D] with a box of
// {D, 1, rows} (one head's rows of a part, 2 KB apart in the cache, in one copy).
struct StageMaps {
    CUtensorMap k;
    CUtensorMap v;
};

// kProjC > 0 (decode only, with kFused and kStage): the q|k|v projection of the new token is fused in, for a hidden
// size of 256 * kProjC. CTA c of head h's cluster computes dims [c D/8, (c+1) D/8) of the head's q row and of its
// key/value head's k and v rows: its D/8 rows of each weight matrix (contiguous in the fused matrix) are brought into
// L2 before the dependency wait and into registers right after it, while warp 0 RMS-normalises the input row as the
// staged projection does (same order); each of the 3 D/8 dot products runs in the canonical lane order on one warp,
// and the slices are gathered into every CTA of the cluster through DSMEM behind one cluster barrier -- the
// projection kernel, its launch boundary and the round trip of q and k through global memory are gone. (Staging the
// rows in shared memory instead, 96 KB per CTA, kept the clusters from becoming resident beside the running
// kernels: 1430 tok/s against 1930 unfused.)
template <int kD, bool kFused, bool kStage, int kProjC = 0>
__global__ void __launch_bounds__(kCtaThreads, kProjC > 0 ? 2 : 3)
    decoder_attention_kernel(const AttentionParams p, int64_t max_part, const __grid_constant__ StageMaps maps) {
    constexpr bool kProj = kProjC > 0;
    static_assert(!kProj || (kFused && kStage), "the fused projection runs in the staged decode kernel");
    constexpr int kProjRows = kD / 8;          // rows of each of q, k, v a CTA computes
    constexpr int kProjAll = 3 * kProjRows;
    constexpr int kSeg = kD / kSegments;       // dims per score segment
    constexpr int kSegChunks = kSeg / 8;       // 16-byte chunks per segment
    constexpr int kKeysPerIter = 32 / kSegments;
    constexpr int kDimsPerLane = kD / 64;      // P·V: a lane's dims of its chain's half
    constexpr int kFinal = kD / kParts;        // context dims each CTA finishes
    // Loads issued together: warp iterations of score loads, and V rows per warp. Measured on the Qwen3-0.6B decode
    // step: 2 and 4 took 691 us per token, 4 and 8 took 699; 4 and 16, or 2 and 2, were slower still.
    constexpr int kScoreBatch = 2;
    constexpr int kValueBatch = 4;
    // Dynamic shared memory: this part's scores (then exp values, then probabilities), and with kStage the part's
    // cached key and value rows.
    extern __shared__ __align__(16) float s_e[];
    __shared__ float s_red[kCtaWarps];    // per-warp maxima of this part's scores
    __shared__ float s_wsum[kWarps];      // per-warp exp sums of the 4 slot warps
    __shared__ float s_m[kParts];         // every part's max and exp sum, pushed here by each part
    __shared__ float s_s[kParts];
    __shared__ float s_acc[kWarps][kD];
    __shared__ float s_recv[kParts][kFinal];  // the parts' P·V partials of the dims this CTA finishes
    __shared__ __align__(16) bf16 s_q[kFused ? kD : 8];
    __shared__ __align__(16) bf16 s_knew[kFused ? kD : 8];
    __shared__ __align__(16) uint4 s_xn[kProj ? kProjC * 32 : 1];  // the normalised input row
    __shared__ __align__(16) bf16 s_proj[kProj ? kProjAll : 8];    // this CTA's q, k, v values
    __shared__ __align__(16) bf16 s_qraw[kProj ? kD : 8];          // the gathered raw q, k, v rows
    __shared__ __align__(16) bf16 s_kraw[kProj ? kD : 8];
    __shared__ __align__(16) bf16 s_vraw[kProj ? kD : 8];
    __shared__ __align__(16) float s_angles[kProj ? kD : 4];       // kProj: the position's RoPE row (cos, sin)
    __shared__ __align__(16) bf16 s_qnw[kProj ? kD : 8];           // kProj: the q and k norm weights
    __shared__ __align__(16) bf16 s_knw[kProj ? kD : 8];
    __shared__ __align__(8) uint64_t s_bar;

    cg::cluster_group cluster = cg::this_cluster();
    const int rank = static_cast<int>(cluster.block_rank());
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    if constexpr (!kStage) {
        grid_dependency_begin();
    }
    // The sequence position first (one memory round trip; the decode variant reads it before its wait, the previous
    // kernel does not write it), then the index math in 32 bits while it is in flight (the grid has < 2^31 CTAs).
    const int64_t pos_base = p.pos0 + (p.position != nullptr ? static_cast<int64_t>(*p.position) : 0);
    const int unit = static_cast<int>(blockIdx.x / kParts);
    const int tb = unit / p.q_heads;
    const int h = unit - tb * p.q_heads;
    const int64_t t_begin = static_cast<int64_t>(tb) * p.queries_per_cluster;
    const int64_t t_end = t_begin + p.queries_per_cluster < p.T ? t_begin + p.queries_per_cluster : p.T;
    const int group = p.q_heads / p.kv_heads;
    const int kvh = h / group;
    // Every CTA of the cluster has started once this barrier phase completes (waited on before the first DSMEM
    // store below).
    asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
    bool started = false;
    // The cluster takes queries t_begin .. t_end - 1 of head h one after another, each with the same arithmetic.
    // Between two queries every CTA has passed the previous query's last cluster barrier, so no DSMEM store of the
    // next query lands in shared memory that is still being read.
    for (int64_t t = t_begin; t < t_end; ++t) {
        const int64_t pos = pos_base + t;
        if (pos >= p.capacity) {
            if constexpr (kStage) {
                grid_dependency_begin();
            }
            break;  // the whole cluster leaves together (same t, later queries lie further out)
        }
        const int64_t L = pos + 1;
        const int64_t P = (L + kParts - 1) / kParts;
        const int64_t lo = rank * P < L ? rank * P : L;
        const int64_t hi = lo + P < L ? lo + P : L;
        // Keys of this part are addressed by their 32-bit index i in [0, n), key j = lo + i (64-bit index math in
        // these loops cost ~0.6 us per layer of the decode step, measured on B200).
        const int n = static_cast<int>(hi - lo);
        const int i_new = static_cast<int>(L - 1 - lo);  // the new token's key (outside [0, n) in other parts)
        const int64_t kv_row = static_cast<int64_t>(p.kv_heads) * kD;
        const float scale = 1.0f / sqrtf(static_cast<float>(kD));

        // kStage: rows [lo, staged_hi) (every cached row of this part before the new token) go to shared memory now;
        // the previous kernel in the stream writes neither them nor the sequence length.
        // The staged tiles start on a 128-byte boundary (TMA destinations), after the scores.
        char* const s_tiles = reinterpret_cast<char*>(s_e + ((max_part + 3) / 4) * 4);
        bf16* s_kt = reinterpret_cast<bf16*>(s_tiles + ((128u - (smem_addr(s_tiles) & 127u)) & 127u));
        bf16* s_vt = s_kt + max_part * kD;
        const int64_t staged_hi = hi < pos ? hi : pos;
        const int64_t staged = staged_hi > lo ? staged_hi - lo : 0;
        uint4 v_new = make_uint4(0u, 0u, 0u, 0u);
        float c_rope[kFused ? 8 : 1];
        float s_rope[kFused ? 8 : 1];
        uint4 wq_a, wq_b, wk_a, wk_b;
        if constexpr (kStage) {
            // Two TMA copies of max_part rows each (the box), from row lo: rows past the part's cached ones (the new
            // token's, later positions, or zeros past the cache) arrive too and are never read -- the new key comes
            // from s_knew and the new value row is written over its slot after this wait. Measured on B200: one
            // 256-byte bulk copy per row kept warp 0 issuing for ~6 us, past the end of the previous kernel.
            if (threadIdx.x == 0) {
                mbar_init(&s_bar, 1);
                mbar_arrive_expect_tx(&s_bar, staged > 0 ? static_cast<uint32_t>(max_part * kD * 2 * 2) : 0u);
                if (staged > 0) {
                    tc::tma_load_3d(s_kt, &maps.k, 0, kvh, static_cast<int>(lo), &s_bar);
                    tc::tma_load_3d(s_vt, &maps.v, 0, kvh, static_cast<int>(lo), &s_bar);
                }
                if constexpr (kProj) {
                    // This CTA's rows of W_q (head h), W_k and W_v (key/value head kvh), D/8 contiguous rows each,
                    // brought into L2 while the previous kernel runs.
    #pragma unroll
                    for (int m = 0; m < 3; ++m) {
                        bulk_prefetch_l2(proj_row<kD>(p, m, h, kvh, rank * kProjRows), kProjRows * p.hidden * 2);
                    }
                }
            }
            __syncthreads();
        }
        // RoPE angles of this position and the q/k norm weights: constants, read before the wait (with the fused
        // projection only brought into L1 then, and read after the projection, which needs the registers).
        constexpr int kLanes = kD / 16;
        const int hl = lane % kLanes;
        const float* trow = p.rope_table + pos * kD;
        auto load_constants = [&]() {
            if constexpr (kProj) {
    #pragma unroll
                for (int j = 0; j < 8; ++j) {
                    c_rope[j] = s_angles[hl * 8 + j];
                    s_rope[j] = s_angles[kD / 2 + hl * 8 + j];
                }
                wq_a = *reinterpret_cast<const uint4*>(s_qnw + hl * 8);
                wq_b = *reinterpret_cast<const uint4*>(s_qnw + kD / 2 + hl * 8);
                wk_a = *reinterpret_cast<const uint4*>(s_knw + hl * 8);
                wk_b = *reinterpret_cast<const uint4*>(s_knw + kD / 2 + hl * 8);
            } else {
    #pragma unroll
                for (int j = 0; j < 8; ++j) {
                    c_rope[j] = trow[hl * 8 + j];
                    s_rope[j] = trow[kD / 2 + hl * 8 + j];
                }
                wq_a = ld_cached(p.q_norm + hl * 8);
                wq_b = ld_cached(p.q_norm + kD / 2 + hl * 8);
                wk_a = ld_cached(p.k_norm + hl * 8);
                wk_b = ld_cached(p.k_norm + kD / 2 + hl * 8);
            }
        };
        if constexpr (kFused && !kProj) {
            load_constants();
        }
        uint4 nw[kProj ? kProjC : 1];  // kProj: warp 0's chunks of the input norm weight (a constant)
        if constexpr (kProj) {
            if (warp == 0) {
    #pragma unroll
                for (int i = 0; i < kProjC; ++i) {
                    nw[i] = ld_cached(p.in_norm + (lane + 32 * i) * 8);
                }
            }
        }
        if constexpr (kStage) {
            // One warp waits for the previous grid; the others wait at the block barrier, which orders their reads
            // after that wait (waiting warps would otherwise take issue slots from the kernel still running).
            if (warp == 0) {
                asm volatile("griddepcontrol.wait;" ::: "memory");
            }
            __syncthreads();
            asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
        }

        bool stage_failed = false;
        if constexpr (kProj) {
            // The input row: warp 0 loads it (the embedding row of the token at this position in the first layer,
            // which it also copies to the residual stream) and RMS-normalises it exactly as the staged projection
            // does (lane l's chunks l, l + 32, ..., canonical order), for every warp through shared memory.
            if (warp != 0) {
                // The RoPE row and the q/k norm weights into shared memory, for after the projection (registers
                // are short during it); warps 1.. do it while warp 0 normalises the input row.
                for (int i = threadIdx.x - 32; i < kD; i += kCtaThreads - 32) {
                    s_angles[i] = trow[i];
                    s_qnw[i] = p.q_norm[i];
                    s_knw[i] = p.k_norm[i];
                }
            }
            if (warp == 0) {
                const bf16* xrow = p.x;
                if (p.tokens != nullptr) {
                    const int64_t tok = p.tokens[pos];
                    xrow += (tok < 0 ? 0 : (tok >= p.vocab ? p.vocab - 1 : tok)) * p.hidden;
                }
                uint4 xv[kProjC];
    #pragma unroll
                for (int i = 0; i < kProjC; ++i) {
                    xv[i] = ld_cached(xrow + (lane + 32 * i) * 8);
                }
                if (p.x_copy != nullptr && blockIdx.x == 0) {
    #pragma unroll
                    for (int i = 0; i < kProjC; ++i) {
                        st_v4(p.x_copy + (lane + 32 * i) * 8, xv[i]);
                    }
                }
                float ssq = 0.0f;
    #pragma unroll
                for (int i = 0; i < kProjC; ++i) {
                    float f[8];
                    Vec16<bf16>::unpack(xv[i], f);
    #pragma unroll
                    for (int e = 0; e < 8; ++e) {
                        ssq = __fmaf_rn(f[e], f[e], ssq);  // a bf16 square: fused, as sum_square
                    }
                }
                ssq = group_sum<32>(ssq);
                const float mean = ssq / static_cast<float>(kProjC * 256);
                const float rms = sqrtf(mean + p.eps);
                const float inv = 1.0f / rms;
    #pragma unroll
                for (int i = 0; i < kProjC; ++i) {
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
            // Each warp takes rows warp, warp + 8, ... of the 3 D/8, three at a time in registers; its first three
            // are requested before the barrier, so they arrive while warp 0 normalises the row (measured on B200:
            // batches of 2 rows 1955 tok/s, 3 rows 1971; all 6 spilled; the first batch loaded before the dependency
            // wait 1913; double-buffered batches of 2 1900).
            constexpr int kRowsPerWarp = kProjAll / kCtaWarps;
            static_assert(kProjAll % kCtaWarps == 0, "whole rows per warp");
            constexpr int kBatch = kRowsPerWarp < 3 ? kRowsPerWarp : 3;
            uint4 wreg[kBatch][kProjC];
            auto load_rows = [&](int k0) {
    #pragma unroll
                for (int b = 0; b < kBatch; ++b) {
                    if (k0 + b < kRowsPerWarp) {
                        const int r = warp + (k0 + b) * kCtaWarps;
                        const bf16* wrow = proj_row<kD>(p, r / kProjRows, h, kvh, rank * kProjRows + r % kProjRows);
    #pragma unroll
                        for (int i = 0; i < kProjC; ++i) {
                            wreg[b][i] = ld_cached(wrow + (lane + 32 * i) * 8);
                        }
                    }
                }
            };
            load_rows(0);
            __syncthreads();
            const bool arrived = mbar_wait_bounded(&s_bar, 0, p.poll_limit);
            // On a timeout the kernel still runs every cluster barrier below (with meaningless values), so no CTA of
            // the cluster is left waiting; the host sees the error flag.
            stage_failed = __syncthreads_or(arrived ? 0 : 1) != 0;
            if (stage_failed && threadIdx.x == 0) {
                atomicOr(p.error, 1u);
            }
            // The 3 D/8 dot products, one warp each at a time: fused multiply-adds in the canonical lane order and a
            // butterfly, rounded to bf16 once (the staged projection's arithmetic).
    #pragma unroll
            for (int k0 = 0; k0 < kRowsPerWarp; k0 += kBatch) {
                if (k0 > 0) {
                    load_rows(k0);
                }
    #pragma unroll
                for (int b = 0; b < kBatch; ++b) {
                    if (k0 + b < kRowsPerWarp) {
                        float acc = 0.0f;
    #pragma unroll
                        for (int i = 0; i < kProjC; ++i) {
                            acc = fma_bf16x8(s_xn[lane + 32 * i], wreg[b][i], acc);
                        }
                        acc = group_sum<32>(acc);
                        if (lane == 0) {
                            s_proj[warp + (k0 + b) * kCtaWarps] = __float2bfloat16_rn(acc);
                        }
                    }
                }
            }
            __syncthreads();
            if (!started) {
                asm volatile("barrier.cluster.wait.aligned;" ::: "memory");  // every CTA has started: DSMEM is usable
                started = true;
            }
            // Gather: value r of this CTA goes to dim rank * D/8 + r % (D/8) of the q, k or v row of every CTA.
            for (int idx = threadIdx.x; idx < kProjAll * kParts; idx += kCtaThreads) {
                const int r = idx / kParts;
                const int m = r / kProjRows;
                bf16* row = m == 0 ? s_qraw : (m == 1 ? s_kraw : s_vraw);
                *cluster.map_shared_rank(row + rank * kProjRows + r % kProjRows, idx % kParts) = s_proj[r];
            }
            if (h % group == 0 && threadIdx.x < kProjRows) {
                // One cluster per key/value head stores the new token's value row (for the steps that follow).
                const_cast<bf16*>(p.v_cache)[pos * kv_row + kvh * kD + rank * kProjRows + threadIdx.x] =
                    s_proj[2 * kProjRows + threadIdx.x];
            }
            cluster.sync();
            // q-norm + RoPE of this head and k-norm + RoPE of the new key from the gathered rows; the new value row
            // into the staged tile (the copies have landed).
            if (warp < 2) {
                load_constants();
            }
            if (warp == 0) {
                norm_rope_head<kD, true>(s_qraw, wq_a, wq_b, c_rope, s_rope, p.eps, s_q, lane);
            } else if (warp == 1) {
                norm_rope_head<kD, true>(s_kraw, wk_a, wk_b, c_rope, s_rope, p.eps, s_knew, lane);
            } else if (warp == 2 && i_new >= 0 && i_new < n && lane < kD / 8) {
                *reinterpret_cast<uint4*>(s_vt + i_new * kD + lane * 8) =
                    *reinterpret_cast<const uint4*>(s_vraw + lane * 8);
            }
            __syncthreads();
            if (rank == 0 && h % group == 0 && threadIdx.x < kD / 8) {
                // One CTA per key/value head stores the new key row; nobody reads that row in this launch.
                st_v4(const_cast<bf16*>(p.k_cache) + pos * kv_row + kvh * kD + threadIdx.x * 8,
                      *reinterpret_cast<const uint4*>(s_knew + threadIdx.x * 8));
            }
        } else if constexpr (kFused) {
            // q-norm + RoPE of this head and k-norm + RoPE of the new key (computed by every CTA that needs them).
            if (warp == 0) {
                norm_rope_head<kD>(p.q + (t * p.q_heads + h) * kD, wq_a, wq_b, c_rope, s_rope, p.eps, s_q, lane);
            } else if (warp == 1) {
                norm_rope_head<kD>(p.k_new + (t * p.kv_heads + kvh) * kD, wk_a, wk_b, c_rope, s_rope, p.eps, s_knew,
                                   lane);
            } else if (kStage && warp == 2 && i_new >= 0 && i_new < n && lane < kD / 8) {
                // The new token's value row (written to the cache by the previous kernel), stored into the staged
                // tile after the copies have landed, so the P·V loop reads shared memory only.
                v_new = ld_cached(p.v_cache + pos * kv_row + kvh * kD + lane * 8);
            }
            __syncthreads();
            if (rank == 0 && h % group == 0 && threadIdx.x < kD / 8) {
                // One CTA per key/value head stores the new key row; nobody reads that row in this launch.
                st_v4(const_cast<bf16*>(p.k_cache) + pos * kv_row + kvh * kD + threadIdx.x * 8,
                      *reinterpret_cast<const uint4*>(s_knew + threadIdx.x * 8));
            }
        }
        if constexpr (kStage && !kProj) {
            const bool arrived = mbar_wait_bounded(&s_bar, 0, p.poll_limit);
            // On a timeout the kernel still runs every cluster barrier below (with meaningless values), so no CTA of
            // the cluster is left waiting; the host sees the error flag.
            stage_failed = __syncthreads_or(arrived ? 0 : 1) != 0;
            if (warp == 2 && i_new >= 0 && i_new < n && lane < kD / 8) {
                *reinterpret_cast<uint4*>(s_vt + i_new * kD + lane * 8) = v_new;  // read after later barriers
            }
            if (stage_failed && threadIdx.x == 0) {
                atomicOr(p.error, 1u);
            }
        }

        // Scores: 4 keys per warp iteration, 8 lanes per key, all warps of the CTA; kScoreBatch iterations' loads
        // in flight.
        const int sub = lane % kSegments;
        const int slot = lane / kSegments;
        uint4 qv[kSegChunks];
    #pragma unroll
        for (int c = 0; c < kSegChunks; ++c) {
            if constexpr (kFused) {
                qv[c] = *reinterpret_cast<const uint4*>(s_q + sub * kSeg + c * 8);
            } else {
                qv[c] = ld_cached(p.q + (t * p.q_heads + h) * kD + sub * kSeg + c * 8);
            }
        }
        constexpr int kIterKeys = kCtaWarps * kKeysPerIter;
        for (int i0 = warp * kKeysPerIter; i0 < n; i0 += kIterKeys * kScoreBatch) {
            uint4 kv[kScoreBatch][kSegChunks];
    #pragma unroll
            for (int u = 0; u < kScoreBatch; ++u) {
                const int i = i0 + u * kIterKeys + slot;
    #pragma unroll
                for (int c = 0; c < kSegChunks; ++c) {
                    if (i >= n) {
                        kv[u][c] = make_uint4(0u, 0u, 0u, 0u);
                    } else if (kFused && i == i_new) {
                        kv[u][c] = *reinterpret_cast<const uint4*>(s_knew + sub * kSeg + c * 8);
                    } else if (kStage) {
                        kv[u][c] = *reinterpret_cast<const uint4*>(s_kt + i * kD + sub * kSeg + c * 8);
                    } else {
                        kv[u][c] = ld_cached(p.k_cache + (lo + i) * kv_row + kvh * kD + sub * kSeg + c * 8);
                    }
                }
            }
    #pragma unroll
            for (int u = 0; u < kScoreBatch; ++u) {
                const int i = i0 + u * kIterKeys + slot;
                float s = 0.0f;
    #pragma unroll
                for (int c = 0; c < kSegChunks; ++c) {
                    s = dot8(qv[c], kv[u][c], s);
                }
    #pragma unroll
                for (int offset = kSegments / 2; offset > 0; offset >>= 1) {
                    s = s + __shfl_xor_sync(0xffffffffu, s, offset);
                }
                if (i < n && sub == 0) {
                    s_e[i] = s * scale;
                }
            }
        }
        __syncthreads();

        // This part's maximum and its sum of exp(x - max) (slot order, warp butterfly, warps in order).
        float mx = -INFINITY;
        for (int i = threadIdx.x; i < n; i += kCtaThreads) {
            mx = fmaxf(mx, s_e[i]);
        }
        mx = group_max<32>(mx);
        if (lane == 0) {
            s_red[warp] = mx;
        }
        __syncthreads();
        // Every thread folds the warp maxima itself (the max is exact in any order; no second barrier).
        float local_max = s_red[0];
    #pragma unroll
        for (int w = 1; w < kCtaWarps; ++w) {
            local_max = fmaxf(local_max, s_red[w]);
        }
        // The 128 slot chains are the first 4 warps' lanes (the order restated by the oracle).
        float sum = 0.0f;
        if (threadIdx.x < kThreads) {
            for (int i = threadIdx.x; i < n; i += kThreads) {
                sum = sum + pexp(s_e[i] - local_max);
            }
        }
        sum = group_sum<32>(sum);
        if (lane == 0 && warp < kWarps) {
            s_wsum[warp] = sum;
        }
        __syncthreads();
        if (!started) {
            asm volatile("barrier.cluster.wait.aligned;" ::: "memory");  // every CTA has started: DSMEM is usable
            started = true;
        }
        if (threadIdx.x < kParts) {
            float part_sum = s_wsum[0];
    #pragma unroll
            for (int w = 1; w < kWarps; ++w) {
                part_sum = part_sum + s_wsum[w];
            }
            // Push (max, sum) of this part to every CTA of the cluster, this one included.
            *cluster.map_shared_rank(&s_m[rank], static_cast<int>(threadIdx.x)) = local_max;
            *cluster.map_shared_rank(&s_s[rank], static_cast<int>(threadIdx.x)) = part_sum;
        }
        cluster.sync();
        // Global max M and total = sum over parts (in order) of part_sum * exp(part_max - M).
        float gmax = s_m[0];
    #pragma unroll
        for (int r = 1; r < kParts; ++r) {
            gmax = fmaxf(gmax, s_m[r]);
        }
        // Lane r forms part r's term; every lane then adds the terms in part order from the shuffled values (one
        // exponential per lane instead of kParts).
        const int tr = lane % kParts;
        const float term = s_s[tr] * pexp(s_m[tr] - gmax);
        float total = __shfl_sync(0xffffffffu, term, 0);
    #pragma unroll
        for (int r = 1; r < kParts; ++r) {
            total = total + __shfl_sync(0xffffffffu, term, r);
        }

        for (int i = threadIdx.x; i < n; i += kCtaThreads) {
            s_e[i] = round_to_bf16(pexp(s_e[i] - gmax) / total);
        }
        __syncthreads();

        // Probabilities times V: warp chain w = warp % 4 takes keys lo + w, lo + w + 4, ... in order (the restated
        // order); the two hardware warps of a chain take half of the dims each; kValueBatch rows in flight.
        const int chain = warp % kWarps;
        const int dim0 = (warp / kWarps) * (kD / 2) + lane * kDimsPerLane;
        float a[kDimsPerLane];
    #pragma unroll
        for (int d = 0; d < kDimsPerLane; ++d) {
            a[d] = 0.0f;
        }
        const bf16* vbase = p.v_cache + kvh * kD + dim0;
        for (int i0 = chain; i0 < n; i0 += kWarps * kValueBatch) {
            typename VHalf<kD>::Raw raw[kValueBatch];
    #pragma unroll
            for (int u = 0; u < kValueBatch; ++u) {
                const int i = i0 + u * kWarps;
                if (i < n) {
                    if constexpr (kStage) {
                        raw[u] = *reinterpret_cast<const typename VHalf<kD>::Raw*>(s_vt + i * kD + dim0);
                    } else {
                        raw[u] = VHalf<kD>::load(vbase + (lo + i) * kv_row);
                    }
                }
            }
    #pragma unroll
            for (int u = 0; u < kValueBatch; ++u) {
                const int i = i0 + u * kWarps;
                if (i < n) {
                    const float pj = s_e[i];
                    float v[kDimsPerLane];
                    VHalf<kD>::unpack(raw[u], v);
                    // a[d] = fma(p_j, v_j[d], a[d]) (p_j is a bf16 value, so each product is exact as in
                    // fma_bf16x2); neighbouring dims are separate chains, advanced two at a time.
                    if constexpr (kDimsPerLane >= 2) {
    #pragma unroll
                        for (int d = 0; d < kDimsPerLane; d += 2) {
                            const float2 r = __ffma2_rn(make_float2(pj, pj), make_float2(v[d], v[d + 1]),
                                                        make_float2(a[d], a[d + 1]));
                            a[d] = r.x;
                            a[d + 1] = r.y;
                        }
                    } else {
                        a[0] = __fmaf_rn(pj, v[0], a[0]);
                    }
                }
            }
        }
    #pragma unroll
        for (int d = 0; d < kDimsPerLane; ++d) {
            s_acc[chain][dim0 + d] = a[d];
        }
        __syncthreads();
        for (int d = threadIdx.x; d < kD; d += kCtaThreads) {
            float part = s_acc[0][d];
    #pragma unroll
            for (int w = 1; w < kWarps; ++w) {
                part = part + s_acc[w][d];
            }
            // Push the partial of dim d to the CTA that finishes it.
            *cluster.map_shared_rank(&s_recv[rank][d % kFinal], d / kFinal) = part;
        }
        cluster.sync();  // after this no CTA touches another's shared memory
        if (threadIdx.x < kFinal) {
            float c = s_recv[0][threadIdx.x];
    #pragma unroll
            for (int r = 1; r < kParts; ++r) {
                c = c + s_recv[r][threadIdx.x];
            }
            Vec16<bf16>::store1(p.ctx, (t * p.q_heads + h) * kD + rank * kFinal + threadIdx.x, c);
        }
        if (kStage && stage_failed) {
            mbar_wait_bounded(&s_bar, 0);  // no bulk copy may land after this CTA has left
        }
    }
    if (!started) {
        asm volatile("barrier.cluster.wait.aligned;" ::: "memory");
    }
}

// The same attention for queries whose keys are already in the cache (prompt chunks, and the C ABI), in one CTA per
// (query, head) instead of a cluster: warp c plays part c, and each lane plays the four slots (lane + 32 k) and the
// four warps of that part in registers, so every sum above is formed from the same operands in the same order --
// the score segments and their butterfly, the 128 slot chains of exp values and their per-warp butterflies added
// in warp order, the per-warp P·V chains over keys lo + w, lo + w + 4, ... added in warp order, and the 8 part
// partials added in part order. The exchanges between parts go through shared memory with two block barriers.
constexpr int kRowWarps = kParts;
constexpr int kRowThreads = kRowWarps * 32;

template <int kD>
__global__ void __launch_bounds__(kRowThreads, kD >= 256 ? 2 : 3) attention_rows_kernel(const AttentionParams p, int64_t max_part) {
    constexpr int kSeg = kD / kSegments;
    constexpr int kSegChunks = kSeg / 8;
    constexpr int kKeysPerIter = 32 / kSegments;
    constexpr int kDimsPerLane = kD / 32;
    constexpr int kScoreBatch = 2;  // measured on the 512-token prompt: 2 and 4 took 27.3 ms, 4 and 8 took 28.0
    constexpr int kValueBatch = 4;
    extern __shared__ __align__(16) float s_scores[];  // [kParts][stride]: each part's scores, then probabilities
    __shared__ float s_m[kParts];
    __shared__ float s_s[kParts];
    __shared__ float s_part[kParts][kD];

    grid_dependency_begin();
    const int lane = threadIdx.x & 31;
    const int part = threadIdx.x >> 5;
    const int64_t t = blockIdx.x / p.q_heads;
    const int h = static_cast<int>(blockIdx.x - t * p.q_heads);
    const int kvh = h / (p.q_heads / p.kv_heads);
    const int64_t pos = p.pos0 + (p.position != nullptr ? static_cast<int64_t>(*p.position) : 0) + t;
    if (pos >= p.capacity) {
        return;  // the whole CTA leaves together
    }
    const int64_t L = pos + 1;
    const int64_t P = (L + kParts - 1) / kParts;
    const int64_t lo = part * P < L ? part * P : L;
    const int64_t hi = lo + P < L ? lo + P : L;
    const int64_t n = hi - lo;
    const int64_t kv_row = static_cast<int64_t>(p.kv_heads) * kD;
    const float scale = 1.0f / sqrtf(static_cast<float>(kD));
    float* e = s_scores + part * ((max_part + 3) / 4 * 4);

    // Scores: 4 keys per iteration, 8 lanes per key (lane % 8 = segment), kScoreBatch iterations in flight.
    const int sub = lane % kSegments;
    const int slot = lane / kSegments;
    uint4 qv[kSegChunks];
#pragma unroll
    for (int c = 0; c < kSegChunks; ++c) {
        qv[c] = ld_cached(p.q + (t * p.q_heads + h) * kD + sub * kSeg + c * 8);
    }
    for (int64_t j0 = lo; j0 < hi; j0 += kKeysPerIter * kScoreBatch) {
        uint4 kv[kScoreBatch][kSegChunks];
#pragma unroll
        for (int u = 0; u < kScoreBatch; ++u) {
            const int64_t j = j0 + u * kKeysPerIter + slot;
#pragma unroll
            for (int c = 0; c < kSegChunks; ++c) {
                kv[u][c] = j < hi ? ld_cached(p.k_cache + j * kv_row + kvh * kD + sub * kSeg + c * 8)
                                  : make_uint4(0u, 0u, 0u, 0u);
            }
        }
#pragma unroll
        for (int u = 0; u < kScoreBatch; ++u) {
            const int64_t j = j0 + u * kKeysPerIter + slot;
            float sc = 0.0f;
#pragma unroll
            for (int c = 0; c < kSegChunks; ++c) {
                sc = dot8(qv[c], kv[u][c], sc);
            }
#pragma unroll
            for (int offset = kSegments / 2; offset > 0; offset >>= 1) {
                sc = sc + __shfl_xor_sync(0xffffffffu, sc, offset);
            }
            if (j < hi && sub == 0) {
                e[j - lo] = sc * scale;
            }
        }
    }
    __syncwarp();

    // The part's maximum, then its exp sum: slot i = 32 k + lane adds keys lo + i, lo + i + 128, ... in order; each
    // virtual warp k sums its 32 slots by a butterfly; the four warp sums are added in order.
    float mx = -INFINITY;
    for (int64_t i = lane; i < n; i += 32) {
        mx = fmaxf(mx, e[i]);
    }
    mx = group_max<32>(mx);
    float wsum[kWarps];
#pragma unroll
    for (int k = 0; k < kWarps; ++k) {
        float acc = 0.0f;
        for (int64_t i = k * 32 + lane; i < n; i += kThreads) {
            acc = acc + pexp(e[i] - mx);
        }
        wsum[k] = group_sum<32>(acc);
    }
    float part_sum = wsum[0];
#pragma unroll
    for (int k = 1; k < kWarps; ++k) {
        part_sum = part_sum + wsum[k];
    }
    if (lane == 0) {
        s_m[part] = mx;
        s_s[part] = part_sum;
    }
    __syncthreads();
    float gmax = s_m[0];
#pragma unroll
    for (int r = 1; r < kParts; ++r) {
        gmax = fmaxf(gmax, s_m[r]);
    }
    float total = s_s[0] * pexp(s_m[0] - gmax);
#pragma unroll
    for (int r = 1; r < kParts; ++r) {
        total = total + s_s[r] * pexp(s_m[r] - gmax);
    }
    for (int64_t i = lane; i < n; i += 32) {
        e[i] = round_to_bf16(pexp(e[i] - gmax) / total);
    }
    __syncwarp();

    // Probabilities times V: virtual warp w takes keys lo + w, lo + w + 4, ... (a[w]), the lane's kD / 32 dims.
    float a[kWarps][kDimsPerLane];
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
#pragma unroll
        for (int d = 0; d < kDimsPerLane; ++d) {
            a[w][d] = 0.0f;
        }
    }
    const bf16* vbase = p.v_cache + kvh * kD + lane * kDimsPerLane;
    static_assert(kValueBatch % kWarps == 0, "a batch covers whole rounds of the four virtual warps");
    for (int64_t j0 = lo; j0 < hi; j0 += kValueBatch) {
        typename VRow<kD>::Raw raw[kValueBatch];
#pragma unroll
        for (int u = 0; u < kValueBatch; ++u) {
            if (j0 + u < hi) {
                raw[u] = VRow<kD>::load(vbase + (j0 + u) * kv_row);
            }
        }
#pragma unroll
        for (int u = 0; u < kValueBatch; ++u) {
            if (j0 + u < hi) {
                const float pj = e[j0 + u - lo];
                float v[kDimsPerLane];
                VRow<kD>::unpack(raw[u], v);
#pragma unroll
                for (int d = 0; d < kDimsPerLane; ++d) {
                    a[u % kWarps][d] = __fmaf_rn(pj, v[d], a[u % kWarps][d]);
                }
            }
        }
    }
#pragma unroll
    for (int d = 0; d < kDimsPerLane; ++d) {
        float sum_w = a[0][d];
#pragma unroll
        for (int w = 1; w < kWarps; ++w) {
            sum_w = sum_w + a[w][d];
        }
        s_part[part][lane * kDimsPerLane + d] = sum_w;
    }
    __syncthreads();
    for (int d = threadIdx.x; d < kD; d += kRowThreads) {
        float c = s_part[0][d];
#pragma unroll
        for (int r = 1; r < kParts; ++r) {
            c = c + s_part[r][d];
        }
        Vec16<bf16>::store1(p.ctx, (t * p.q_heads + h) * kD + d, c);
    }
}

// Scores of all 8 parts up to this size stay in one CTA (contexts of up to 16384 keys); longer contexts take the
// cluster kernel, whose CTAs hold one part each.
constexpr std::size_t kMaxRowScoreBytes = 64 * 1024;

// Staged parts up to this size leave room in the SM's shared memory for the neighbouring kernels' CTAs.
constexpr std::size_t kMaxStagedBytes = 110 * 1024;



template <int kD, bool kFused, bool kStage, int kProjC = 0>
cudaError_t launch_attention_variant(const AttentionParams& p, int64_t max_part, std::size_t smem, cudaStream_t s,
                                     const StageMaps& maps = StageMaps{}) {
    auto kernel = decoder_attention_kernel<kD, kFused, kStage, kProjC>;
    // Opted in for every size: static and dynamic shared memory together may pass 48 KB before the dynamic part does.
    const cudaError_t err =
        cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (err != cudaSuccess) {
        return err;
    }
    const int64_t blocks = (p.T + p.queries_per_cluster - 1) / p.queries_per_cluster * p.q_heads * kParts;
    return runtime::launch_smem(kernel, dim3(static_cast<unsigned>(blocks)), dim3(kCtaThreads), smem, s,
                                static_cast<unsigned>(kParts), p, max_part, maps);
}

// TMA map of one cache [capacity][kv_heads][kD] with a box of one head's `rows` rows.
template <int kD>
bool make_stage_map(CUtensorMap* map, const bf16* cache, int64_t capacity, int kv_heads, int64_t rows) {
    const tc::EncodeTiled encode = tc::encode_tiled();
    if (encode == nullptr || (reinterpret_cast<uintptr_t>(cache) & 15u) != 0) {
        return false;
    }
    const cuuint64_t dims[3] = {static_cast<cuuint64_t>(kD), static_cast<cuuint64_t>(kv_heads),
                                static_cast<cuuint64_t>(capacity)};
    const cuuint64_t strides[2] = {static_cast<cuuint64_t>(kD) * 2, static_cast<cuuint64_t>(kv_heads) * kD * 2};
    const cuuint32_t box[3] = {static_cast<cuuint32_t>(kD), 1, static_cast<cuuint32_t>(rows)};
    const cuuint32_t elem_strides[3] = {1, 1, 1};
    return encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<bf16*>(cache), dims, strides, box,
                  elem_strides, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Prefill: a cluster takes several consecutive queries of one head in turn, so that a long prompt launches a few
// waves of clusters instead of one short-lived cluster per (query, head).
constexpr int64_t kTargetClusters = 1024;
constexpr int64_t kMaxQueriesPerCluster = 16;

int64_t queries_per_cluster(int64_t tokens, int64_t heads) {
    const int64_t q = tokens * heads / kTargetClusters;
    return q < 1 ? 1 : (q > kMaxQueriesPerCluster ? kMaxQueriesPerCluster : q);
}

template <int kD>
cudaError_t launch_attention_dim(const AttentionParams& p, int64_t max_keys, cudaStream_t s) {
    const int64_t per_part = (max_keys + kParts - 1) / kParts;
    const int64_t max_part = per_part < 1 ? 1 : per_part;
    const std::size_t score_bytes = static_cast<std::size_t>((max_part + 3) / 4 * 4) * sizeof(float);
    // Staged tiles: 128 bytes of alignment slack after the scores, then max_part rows of K and of V.
    const std::size_t staged_bytes = score_bytes + 128 + static_cast<std::size_t>(max_part) * kD * 2 * 2;
    if (p.q_norm != nullptr) {
        StageMaps maps{};
        const bool maps_ok = p.error != nullptr && p.T == 1 && max_part <= 256 &&
                             make_stage_map<kD>(&maps.k, p.k_cache, p.capacity, p.kv_heads, max_part) &&
                             make_stage_map<kD>(&maps.v, p.v_cache, p.capacity, p.kv_heads, max_part);
        if (p.wqkv != nullptr) {
            // The caller left the projection to this kernel (decode_projection_fused): no fallback exists.
            if constexpr (kD <= 128) {
                const std::size_t bytes = staged_bytes;
                if (maps_ok && bytes <= kMaxStagedBytes) {
                    switch (p.hidden) {
                    case 256:
                        return launch_attention_variant<kD, true, true, 1>(p, max_part, bytes, s, maps);
                    case 512:
                        return launch_attention_variant<kD, true, true, 2>(p, max_part, bytes, s, maps);
                    case 1024:
                        return launch_attention_variant<kD, true, true, 4>(p, max_part, bytes, s, maps);
                    default:
                        break;
                    }
                }
            }
            return cudaErrorNotSupported;
        }
        if (maps_ok && staged_bytes <= kMaxStagedBytes) {
            return launch_attention_variant<kD, true, true>(p, max_part, staged_bytes, s, maps);
        }
        return launch_attention_variant<kD, true, false>(p, max_part, score_bytes, s);
    }
    const std::size_t row_bytes = kParts * score_bytes;
    if (row_bytes <= kMaxRowScoreBytes) {
        auto kernel = attention_rows_kernel<kD>;
        if (row_bytes > 48 * 1024) {
            const cudaError_t err =
                cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(row_bytes));
            if (err != cudaSuccess) {
                return err;
            }
        }
        return runtime::launch_smem(kernel, dim3(static_cast<unsigned>(p.T * p.q_heads)), dim3(kRowThreads),
                                    row_bytes, s, 1u, p, max_part);
    }
    AttentionParams walk = p;
    walk.queries_per_cluster = queries_per_cluster(p.T, p.q_heads);
    return launch_attention_variant<kD, false, false>(walk, max_part, score_bytes, s);
}

}  // namespace

bool decode_projection_fused(int64_t head_dim, int64_t hidden, int64_t capacity) {
    if ((head_dim != 64 && head_dim != 128) || (hidden != 256 && hidden != 512 && hidden != 1024) || capacity < 1) {
        return false;
    }
    // The same sizes launch_attention_dim checks for the staged decode kernel with max_keys = capacity.
    const int64_t max_part = (capacity + kParts - 1) / kParts;
    const std::size_t score_bytes = static_cast<std::size_t>((max_part + 3) / 4 * 4) * sizeof(float);
    const std::size_t bytes = score_bytes + 128 + static_cast<std::size_t>(max_part) * head_dim * 2 * 2;
    return max_part <= 256 && bytes <= kMaxStagedBytes && tc::encode_tiled() != nullptr;
}

cudaError_t launch_decoder_attention(const AttentionParams& p, int64_t max_keys, cudaStream_t s) {
    switch (p.head_dim) {
    case 64:
        return launch_attention_dim<64>(p, max_keys, s);
    case 128:
        return launch_attention_dim<128>(p, max_keys, s);
    case 256:
        return launch_attention_dim<256>(p, max_keys, s);
    default:
        return cudaErrorInvalidValue;
    }
}

}  // namespace cppinf::device

using namespace cppinf::device;
namespace rt = cppinf::runtime;

extern "C" {

int cppinf_decoder_attention(const void* q, const void* k_cache, const void* v_cache, void* ctx, int64_t tokens,
                             int64_t q_heads, int64_t kv_heads, int64_t head_dim, int64_t position, int64_t capacity,
                             void* stream) {
    CPPINF_REQUIRE(tokens >= 0 && q_heads > 0 && kv_heads > 0 && head_dim > 0, CPPINF_ERR_INVALID_ARGUMENT,
                   "qwen_attention requires non-zero head configuration.");
    CPPINF_REQUIRE(q_heads % kv_heads == 0, CPPINF_ERR_INVALID_ARGUMENT,
                   "qwen_attention requires query heads to divide by key/value heads.");
    CPPINF_REQUIRE(head_dim == 64 || head_dim == 128 || head_dim == 256, CPPINF_ERR_UNSUPPORTED,
                   "decoder attention supports head_dim 64, 128 or 256.");
    CPPINF_REQUIRE(position >= 0, CPPINF_ERR_INVALID_ARGUMENT, "qwen_attention query offsets must be non-negative.");
    CPPINF_REQUIRE(position + tokens <= capacity, CPPINF_ERR_OUT_OF_RANGE,
                   "qwen_attention key lengths exceed the cache capacity.");
    CPPINF_REQUIRE(tokens * q_heads * 8 < (int64_t{1} << 31), CPPINF_ERR_UNSUPPORTED,
                   "decoder attention supports fewer than 2^28 query heads in one call.");
    CPPINF_REQUIRE((capacity + 7) / 8 * 4 <= 200 * 1024, CPPINF_ERR_UNSUPPORTED,
                   "decoder attention supports caches of up to 409600 positions.");
    if (tokens == 0) {
        return rt::ok();
    }
    CPPINF_REQUIRE(q && k_cache && v_cache && ctx, CPPINF_ERR_INVALID_ARGUMENT,
                   "qwen_attention received a null pointer.");
    CPPINF_REQUIRE(rt::aligned16(q) && rt::aligned16(k_cache) && rt::aligned16(v_cache), CPPINF_ERR_UNSUPPORTED,
                   "decoder attention requires 16-byte aligned operands.");
    AttentionParams p{static_cast<const bf16*>(q),
                      static_cast<const bf16*>(k_cache),
                      static_cast<const bf16*>(v_cache),
                      static_cast<bf16*>(ctx),
                      tokens,
                      static_cast<int>(q_heads),
                      static_cast<int>(kv_heads),
                      static_cast<int>(head_dim),
                      position,
                      nullptr,
                      capacity,
                      nullptr,
                      nullptr,
                      nullptr,
                      nullptr,
                      0.0f,
                      nullptr};
    return rt::launched(launch_decoder_attention(p, position + tokens, rt::as_stream(stream)), "decoder_attention");
}

}  // extern "C"
