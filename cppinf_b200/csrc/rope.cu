// Split-half RoPE, nn::apply_rope (src/nn/rope.cpp:58-109), and the fused per-head q/k RMSNorm + RoPE that the
// attention block runs (src/nn/qwen_attention.cpp:383-390: ops::rms_norm on [B, T, H, D] head views, result rounded
// to the model dtype, then apply_rope_batched at position cache_length + t).
//
// Angles: the reference evaluates powf/cosf/sinf on the host for every (head, token, pair). Here the host builds the
// same values once into a [positions][D] f32 table (cos in [0, D/2), sin in [D/2, D)) with the same libm calls, and
// the kernels read the row of the token's position. Device results therefore equal the reference's bit for bit: the
// rotation first*cos - second*sin / second*cos + first*sin is evaluated with separately rounded f32 products and
// sums (the library is built with --fmad=false).
//
// Fused kernel layout: q [T, Hq, D] and k [T, Hk, D] dense. A head vector is held by L = D / (2 * kVec) lanes; lane
// l holds chunk l of the first half (elements l*kVec ..) and chunk l of the second half (D/2 + l*kVec ..), one 16-byte
// vector each, so every RoPE pair (i, i + D/2) sits in one lane and no shuffle is needed for the rotation. One warp
// unit covers kIters groups of 32/L heads of one token, all q or all k heads (a token has ceil(Hq / unit) q units
// then ceil(Hk / unit) k units), so the unit's rows are contiguous and share one norm weight vector and one angle
// row: each lane holds the angles of its pairs in registers as f32 and the two weight chunks packed, for the whole
// unit. The unit index is split into (token, unit of the token) by a multiply-high division (FastDiv). When every
// unit is full (Hq and Hk multiples of the unit's heads: the Qwen3 shapes), the per-head bounds checks are compiled
// out (kFull). Measured on B200 for [2048, 16 + 8, 128] bf16 against the layout whose units could mix q and k heads
// and staged the angles and weights in shared memory: 6.43 -> 5.99 us; holding the weights as f32 (more registers,
// fewer CTAs per SM) 6.36 us. Later, with the packed products below, packed fused multiply-adds for the bf16 sum
// of squares: 5.92 -> 5.82 us; each unit's rows asked of L2 before the dependency wait, so that back-to-back
// launches overlap: 5.82 -> 5.23 us; each warp also prefetching the unit half a grid away: 5.41 -> 5.19 us
// (three or four partners: 5.27 / 5.54 us; the same for the residual add + RMSNorm rows was slower).
//
// Reduction order: the sum of squares of a head equals the library's canonical order (lane c sums chunk c, then a
// butterfly over lane distances 16, 8, ..., 1 over the D/kVec chunks): here a lane adds its first-half partial to its
// second-half partial, which is the canonical step at distance D/(2 kVec), and then runs the remaining butterfly
// steps across the head's L lanes.
//
// Roofline: HBM-bound. Algorithmic bytes per token: (Hq + Hk) * D * size read + the same written; the table row
// (D * 4 bytes per position) and the two weight vectors are shared by all heads and come from L1/L2.
#include <cmath>
#include <vector>

#include <type_traits>

#include "common.cuh"
#include "decoder.h"
#include "runtime.h"

namespace cppinf::device {
namespace {

constexpr int kThreads = 256;
constexpr int kQkThreads = 64;  // two warp units per CTA
constexpr int kQkWarps = kQkThreads / 32;
constexpr int kPrefetchUnits = 2;  // warp units whose rows each warp prefetches before the dependency wait

struct QkParams {
    const void* q;
    const void* k;
    const void* qw;
    const void* kw;
    void* q_out;
    void* k_out;
    const float* table;
    int64_t position_offset;
    uint32_t units;      // tokens * units_per_token (< 2^31)
    FastDiv per_token;   // units_per_token = q_units + k_units
    int q_units;         // ceil(q_heads / heads per unit): units [0, q_units) of a token hold q heads
    int q_heads;
    int k_heads;
    float eps;
};

// A warp unit is kIters groups of 32/L heads, all q heads or all k heads of one token, so the unit's source rows
// are one contiguous block and every head of the unit uses the same norm weights and the same angle row. Each lane
// loads its weights and angles once per unit into registers; the head vectors arrive by asynchronous copies
// into the warp's shared-memory slot (lane-major: each lane reads back exactly what it copied, no barrier but the
// copy-group wait), one copy group per iteration, and each iteration starts as soon as its own group has landed.
// At most 64 registers, so 16 CTAs fit an SM (measured 5.98 -> 5.93 us on [2048, 16 + 8, 128] bf16).
template <typename T, int kLanes, int kIters, bool kFull>
__global__ void __launch_bounds__(kQkThreads, 16) qk_norm_rope_kernel(const QkParams p) {
    using V = Vec16<T>;
    constexpr int kVec = V::kVec;
    constexpr int kHalf = kLanes * kVec;  // D / 2
    constexpr int kDim = 2 * kHalf;
    constexpr int kHeadsPerIter = 32 / kLanes;
    constexpr int kHeadsPerUnit = kHeadsPerIter * kIters;
    constexpr int kHeadBytes = kDim * static_cast<int>(sizeof(T));
    constexpr int kHalfBytes = kHalf * static_cast<int>(sizeof(T));
    __shared__ uint4 s_data[kQkWarps][kIters][2][32];

    const int lane = threadIdx.x & 31;
    const int hl = lane % kLanes;  // lane within the head
    const int slot = lane / kLanes;
    const uint32_t unit = blockIdx.x * kQkWarps + threadIdx.x / 32;
    if (unit >= p.units) {
        grid_dependency_begin();
        return;  // the whole warp leaves together
    }
    const uint32_t t = p.per_token.quot(unit);
    const int u = static_cast<int>(unit - t * p.per_token.d);
    const bool is_q = u < p.q_units;
    const int heads = is_q ? p.q_heads : p.k_heads;
    const int h0 = (is_q ? u : u - p.q_units) * kHeadsPerUnit;
    const int64_t row0 = static_cast<int64_t>(t) * heads + h0;  // first head row of the unit
    const char* src = static_cast<const char*>(is_q ? p.q : p.k) + row0 * kHeadBytes + hl * 16;
    char* dst = static_cast<char*>(is_q ? p.q_out : p.k_out) + row0 * kHeadBytes + hl * 16;
    const char* wsrc = static_cast<const char*>(is_q ? p.qw : p.kw) + hl * 16;
    const float* trow = p.table + (p.position_offset + t) * kDim + hl * kVec;

    // Before the dependency wait (while the previous kernel still runs), lanes 0 .. kPrefetchUnits - 1 ask L2 for the
    // head rows (contiguous) of this unit and of kPrefetchUnits - 1 partner units spread over the grid, so the warps
    // that become resident first also cover those that cannot yet. A prefetch returns no data and L2 is the point of
    // coherence, so the loads below still see what the previous kernel writes; everything that reads memory follows
    // the wait, since the op does not know which of its inputs the previous kernel of the stream wrote.
    if (lane < kPrefetchUnits) {
        const uint32_t step = (p.units + kPrefetchUnits - 1) / kPrefetchUnits;
        const uint32_t pu = (unit + static_cast<uint32_t>(lane) * step) % p.units;
        const uint32_t pt = p.per_token.quot(pu);
        const int pk = static_cast<int>(pu - pt * p.per_token.d);
        const bool pq = pk < p.q_units;
        const int pheads = pq ? p.q_heads : p.k_heads;
        const int ph0 = (pq ? pk : pk - p.q_units) * kHeadsPerUnit;
        const int unit_heads = kFull ? kHeadsPerUnit : min(kHeadsPerUnit, pheads - ph0);
        const char* psrc = static_cast<const char*>(pq ? p.q : p.k) +
                           (static_cast<int64_t>(pt) * pheads + ph0) * kHeadBytes;
        bulk_prefetch_l2(psrc, static_cast<uint32_t>(unit_heads * kHeadBytes));
    }
    grid_dependency_begin();
#pragma unroll
    for (int i = 0; i < kIters; ++i) {
        if (kFull || h0 + i * kHeadsPerIter + slot < heads) {
            const char* s = src + (i * kHeadsPerIter + slot) * kHeadBytes;
            cp_async16(&s_data[threadIdx.x / 32][i][0][lane], s);
            cp_async16(&s_data[threadIdx.x / 32][i][1][lane], s + kHalfBytes);
        }
        cp_async_commit();
    }
    const uint4 wpa = ld_cached(wsrc);
    const uint4 wpb = ld_cached(wsrc + kHalfBytes);
    float cs[kVec];
    float sn[kVec];
#pragma unroll
    for (int j = 0; j < kVec; j += 4) {
        const float4 c4 = ld_cached_f4(trow + j);
        const float4 s4 = ld_cached_f4(trow + kHalf + j);
        cs[j] = c4.x, cs[j + 1] = c4.y, cs[j + 2] = c4.z, cs[j + 3] = c4.w;
        sn[j] = s4.x, sn[j + 1] = s4.y, sn[j + 2] = s4.z, sn[j + 3] = s4.w;
    }

#pragma unroll
    for (int i = 0; i < kIters; ++i) {
        cp_async_wait_pending(kIters - 1 - i);
        const bool active = h0 + i * kHeadsPerIter + slot < heads;
        float a[kVec];
        float b[kVec];
        V::unpack(s_data[threadIdx.x / 32][i][0][lane], a);  // inactive lanes read stale bytes and store nothing
        V::unpack(s_data[threadIdx.x / 32][i][1][lane], b);
        // Sums of squares in element order, the two halves' chains side by side. bf16: one packed fused
        // multiply-add advances both chains; the square of a bf16 value is exact in f32 wherever it is a normal
        // number (|x| >= 2^-63), so this equals the separately rounded `sa + a*a` there (the oracle restates it with
        // fmaf). f32: packed products then scalar adds (a packed product feeding a packed add would be contracted
        // into a fused multiply-add by the code generator, which rounds once and changes the result).
        float sa = 0.0f;
        float sb = 0.0f;
        if constexpr (std::is_same_v<T, bf16>) {
            float2 s2 = make_float2(0.0f, 0.0f);
#pragma unroll
            for (int j = 0; j < kVec; ++j) {
                const float2 v = make_float2(a[j], b[j]);
                s2 = __ffma2_rn(v, v, s2);
            }
            sa = s2.x;
            sb = s2.y;
        } else {
#pragma unroll
            for (int j = 0; j < kVec; ++j) {
                const float2 v = make_float2(a[j], b[j]);
                const float2 sq = __fmul2_rn(v, v);
                sa = sa + sq.x;
                sb = sb + sq.y;
            }
        }
        // Every lane of the warp takes part; offsets below kLanes never leave the head's lane group.
        const float ss = group_sum<kLanes>(sa + sb);
        const float mean = ss / static_cast<float>(kDim);
        const float rms = sqrtf(mean + p.eps);
        const float inv = 1.0f / rms;
        const float2 inv2 = make_float2(inv, inv);
        float wa[kVec];
        float wb[kVec];
        V::unpack(wpa, wa);
        V::unpack(wpb, wb);
        float out_a[kVec];
        float out_b[kVec];
#pragma unroll
        for (int j = 0; j < kVec; j += 2) {
            // (x * inv) * w, separately rounded, then stored in the model dtype: the reference's rms_norm returns a
            // tensor of the input dtype and RoPE reads those rounded values.
            const float2 x = __fmul2_rn(__fmul2_rn(make_float2(a[j], a[j + 1]), inv2), make_float2(wa[j], wa[j + 1]));
            const float2 y = __fmul2_rn(__fmul2_rn(make_float2(b[j], b[j + 1]), inv2), make_float2(wb[j], wb[j + 1]));
            const float2 n1 = V::quantize2(x.x, x.y);  // first-half elements j, j + 1
            const float2 n2 = V::quantize2(y.x, y.y);  // second-half elements j, j + 1
            const float2 c = make_float2(cs[j], cs[j + 1]);
            const float2 s = make_float2(sn[j], sn[j + 1]);
            const float2 n1c = __fmul2_rn(n1, c);
            const float2 n2s = __fmul2_rn(n2, s);
            const float2 n2c = __fmul2_rn(n2, c);
            const float2 n1s = __fmul2_rn(n1, s);
            out_a[j] = n1c.x - n2s.x;  // first  * cos - second * sin  (src/nn/rope.cpp:100-101)
            out_a[j + 1] = n1c.y - n2s.y;
            out_b[j] = n2c.x + n1s.x;  // second * cos + first  * sin  (src/nn/rope.cpp:102-103)
            out_b[j + 1] = n2c.y + n1s.y;
        }
        if (kFull || active) {
            char* d = dst + (i * kHeadsPerIter + slot) * kHeadBytes;
            st_stream(d, V::pack(out_a));
            st_stream(d + kHalfBytes, V::pack(out_b));
        }
    }
}

struct RopeParams {
    const void* x;
    void* y;
    const float* table;
    int64_t dim0, dim1;
    int64_t s0, s1, s2;
    int64_t position_offset;
    int head_dim;
    int seq_dim;
};

// Standalone apply_rope on a strided rank-3 view: one thread per (dim0, dim1, pair).
template <typename T>
__global__ void __launch_bounds__(kThreads) rope_kernel(RopeParams p, int64_t total_pairs) {
    grid_dependency_begin();
    using V = Vec16<T>;
    const int half = p.head_dim / 2;
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; idx < total_pairs;
         idx += stride) {
        const int pair = static_cast<int>(idx % half);
        const int64_t r = idx / half;
        const int64_t i1 = r % p.dim1;
        const int64_t i0 = r / p.dim1;
        const int64_t seq = p.seq_dim == 0 ? i0 : i1;
        const float* row = p.table + (p.position_offset + seq) * p.head_dim;
        const float c = __ldg(row + pair);
        const float s = __ldg(row + half + pair);
        const int64_t base = i0 * p.s0 + i1 * p.s1;
        const float first = V::load1(p.x, base + pair * p.s2);
        const float second = V::load1(p.x, base + (pair + half) * p.s2);
        const int64_t out_base = r * p.head_dim;
        V::store1(p.y, out_base + pair, first * c - second * s);
        V::store1(p.y, out_base + pair + half, second * c + first * s);
    }
}

template <typename T, int kLanes, int kIters>
cudaError_t launch_qk_units(QkParams p, int64_t tokens, cudaStream_t s) {
    constexpr int kHeadsPerUnit = (32 / kLanes) * kIters;
    p.q_units = (p.q_heads + kHeadsPerUnit - 1) / kHeadsPerUnit;
    const int per_token = p.q_units + (p.k_heads + kHeadsPerUnit - 1) / kHeadsPerUnit;
    const int64_t units = tokens * per_token;
    if (units >= (int64_t{1} << 31)) {
        return cudaErrorInvalidConfiguration;  // the entry point rejects such sizes before this
    }
    p.units = static_cast<uint32_t>(units);
    p.per_token = FastDiv(static_cast<uint32_t>(per_token));
    const auto blocks = static_cast<unsigned>(runtime::ceil_div(units, kQkWarps));
    if (p.q_heads % kHeadsPerUnit == 0 && p.k_heads % kHeadsPerUnit == 0) {
        return ::cppinf::runtime::launch(qk_norm_rope_kernel<T, kLanes, kIters, true>, dim3(blocks), dim3(kQkThreads),
                                         s, 1u, p);
    }
    return ::cppinf::runtime::launch(qk_norm_rope_kernel<T, kLanes, kIters, false>, dim3(blocks), dim3(kQkThreads), s,
                                     1u, p);
}

// A warp unit covers 8 heads (two iterations of 4 heads at D = 128 bf16): measured on B200 against units of 4, 12
// and 24 heads for the [2048, 16 + 8, 128] configuration, it balances loads in flight per warp against warps per SM
// best.
template <typename T, int kLanes>
cudaError_t launch_qk(const QkParams& p, int64_t tokens, cudaStream_t s) {
    constexpr int kHeadsPerIter = 32 / kLanes;
    constexpr int kIters = kHeadsPerIter >= 8 ? 1 : 8 / kHeadsPerIter;
    return launch_qk_units<T, kLanes, kIters>(p, tokens, s);
}

template <typename T>
cudaError_t dispatch_qk(const QkParams& p, int64_t tokens, int lanes, cudaStream_t s) {
    switch (lanes) {
    case 1:
        return launch_qk<T, 1>(p, tokens, s);
    case 2:
        return launch_qk<T, 2>(p, tokens, s);
    case 4:
        return launch_qk<T, 4>(p, tokens, s);
    case 8:
        return launch_qk<T, 8>(p, tokens, s);
    default:
        return launch_qk<T, 16>(p, tokens, s);
    }
}

}  // namespace
}  // namespace cppinf::device

using namespace cppinf::device;
namespace rt = cppinf::runtime;

extern "C" {

int cppinf_rope_table(float base, int64_t head_dim, int64_t positions, float* table) {
    CPPINF_REQUIRE(std::isfinite(base) && base > 0.0f, CPPINF_ERR_INVALID_ARGUMENT,
                   "apply_rope requires a positive finite rope base.");
    CPPINF_REQUIRE(head_dim > 0, CPPINF_ERR_INVALID_ARGUMENT, "rope head size must be non-zero.");
    CPPINF_REQUIRE(head_dim % 2 == 0, CPPINF_ERR_INVALID_ARGUMENT, "apply_rope requires an even head size.");
    CPPINF_REQUIRE(positions >= 0, CPPINF_ERR_INVALID_ARGUMENT, "rope table positions must be non-negative.");
    CPPINF_REQUIRE(positions == 0 || table, CPPINF_ERR_INVALID_ARGUMENT, "rope table received a null pointer.");
    const int64_t half = head_dim / 2;
    // One inverse frequency per feature pair, as src/nn/rope.cpp:70-74 computes it.
    std::vector<float> inverse_frequencies(static_cast<std::size_t>(half));
    for (int64_t i = 0; i < half; ++i) {
        inverse_frequencies[static_cast<std::size_t>(i)] =
            std::pow(base, -static_cast<float>(i) / static_cast<float>(half));
    }
    for (int64_t pos = 0; pos < positions; ++pos) {
        const auto position = static_cast<float>(pos);
        float* row = table + pos * head_dim;
        for (int64_t i = 0; i < half; ++i) {
            const float angle = position * inverse_frequencies[static_cast<std::size_t>(i)];
            row[i] = std::cos(angle);
            row[half + i] = std::sin(angle);
        }
    }
    return rt::ok();
}

int cppinf_rope(cppinf_dtype dtype, const void* x, int64_t dim0, int64_t dim1, int64_t head_dim, int64_t s0,
                int64_t s1, int64_t s2, int64_t seq_dim, int64_t position_offset, const float* table,
                int64_t table_positions, void* y, void* stream) {
    CPPINF_REQUIRE(rt::valid_dtype(dtype), CPPINF_ERR_INVALID_ARGUMENT, "apply_rope received an unsupported dtype.");
    CPPINF_REQUIRE(seq_dim == 0 || seq_dim == 1, CPPINF_ERR_INVALID_ARGUMENT,
                   "apply_rope requires the sequence dimension to be 0 or 1.");
    CPPINF_REQUIRE(dim0 > 0, CPPINF_ERR_INVALID_ARGUMENT, "rope dim 0 must be non-zero.");
    CPPINF_REQUIRE(dim1 > 0, CPPINF_ERR_INVALID_ARGUMENT, "rope dim 1 must be non-zero.");
    CPPINF_REQUIRE(head_dim > 0, CPPINF_ERR_INVALID_ARGUMENT, "rope head size must be non-zero.");
    CPPINF_REQUIRE(head_dim % 2 == 0, CPPINF_ERR_INVALID_ARGUMENT, "apply_rope requires an even head size.");
    CPPINF_REQUIRE(head_dim <= (int64_t{1} << 30), CPPINF_ERR_UNSUPPORTED, "apply_rope head size is too large.");
    CPPINF_REQUIRE(s0 >= 0 && s1 >= 0 && s2 >= 0, CPPINF_ERR_INVALID_ARGUMENT,
                   "apply_rope strides must be non-negative.");
    CPPINF_REQUIRE(position_offset >= 0, CPPINF_ERR_INVALID_ARGUMENT, "apply_rope position offset must be >= 0.");
    const int64_t seq_len = seq_dim == 0 ? dim0 : dim1;
    CPPINF_REQUIRE(position_offset + seq_len <= table_positions, CPPINF_ERR_OUT_OF_RANGE,
                   "apply_rope positions exceed the rope table.");
    CPPINF_REQUIRE(x && y && table, CPPINF_ERR_INVALID_ARGUMENT, "apply_rope received a null pointer.");
    RopeParams p{x, y, table, dim0, dim1, s0, s1, s2, position_offset, static_cast<int>(head_dim),
                 static_cast<int>(seq_dim)};
    const int64_t total_pairs = dim0 * dim1 * (head_dim / 2);
    const int64_t per_sm = rt::max_threads_per_sm() / kThreads;
    const int64_t wave = static_cast<int64_t>(rt::sm_count()) * (per_sm > 0 ? per_sm : 1);
    const int64_t needed = rt::ceil_div(total_pairs, kThreads);
    const auto blocks = static_cast<unsigned>(needed < wave ? needed : wave);
    cudaError_t launch_err;
    if (dtype == CPPINF_DTYPE_BF16) {
        launch_err = ::cppinf::runtime::launch(rope_kernel<bf16>, dim3(blocks), dim3(kThreads), rt::as_stream(stream), 1u, p, total_pairs);
    } else {
        launch_err = ::cppinf::runtime::launch(rope_kernel<float>, dim3(blocks), dim3(kThreads), rt::as_stream(stream), 1u, p, total_pairs);
    }
    return rt::launched(launch_err, "rope");
}

int cppinf_qk_norm_rope(cppinf_dtype dtype, const void* q, const void* k, const void* q_weight,
                        const void* k_weight, void* q_out, void* k_out, int64_t tokens, int64_t q_heads,
                        int64_t k_heads, int64_t head_dim, int64_t position_offset, float eps, const float* table,
                        int64_t table_positions, void* stream) {
    CPPINF_REQUIRE(rt::valid_dtype(dtype), CPPINF_ERR_INVALID_ARGUMENT, "qk_norm_rope received an unsupported dtype.");
    CPPINF_REQUIRE(tokens >= 0 && q_heads >= 0 && k_heads >= 0, CPPINF_ERR_INVALID_ARGUMENT,
                   "qk_norm_rope requires non-negative sizes.");
    CPPINF_REQUIRE(q_heads + k_heads <= (int64_t{1} << 20), CPPINF_ERR_UNSUPPORTED,
                   "qk_norm_rope supports at most 2^20 heads.");
    CPPINF_REQUIRE(tokens < (int64_t{1} << 31) / (q_heads + k_heads + 2), CPPINF_ERR_UNSUPPORTED,
                   "qk_norm_rope supports fewer than 2^31 head vectors per call.");
    CPPINF_REQUIRE(head_dim > 0, CPPINF_ERR_INVALID_ARGUMENT, "rms_norm requires a non-empty last dimension.");
    CPPINF_REQUIRE(head_dim % 2 == 0, CPPINF_ERR_INVALID_ARGUMENT, "apply_rope requires an even head size.");
    CPPINF_REQUIRE(eps >= 0.0f, CPPINF_ERR_INVALID_ARGUMENT, "rms_norm requires a non-negative epsilon.");
    CPPINF_REQUIRE(position_offset >= 0, CPPINF_ERR_INVALID_ARGUMENT, "qk_norm_rope position offset must be >= 0.");
    CPPINF_REQUIRE(position_offset + tokens <= table_positions, CPPINF_ERR_OUT_OF_RANGE,
                   "qk_norm_rope positions exceed the rope table.");
    const int vec = dtype == CPPINF_DTYPE_BF16 ? 8 : 4;
    const int64_t lanes = head_dim / (2 * vec);
    CPPINF_REQUIRE(head_dim % (2 * vec) == 0 && lanes >= 1 && lanes <= 16 && (lanes & (lanes - 1)) == 0,
                   CPPINF_ERR_UNSUPPORTED,
                   "qk_norm_rope needs head_dim / (2 * (16 / element size)) to be a power of two from 1 to 16.");
    if (tokens == 0 || q_heads + k_heads == 0) {
        return rt::ok();
    }
    CPPINF_REQUIRE(table && (q_heads == 0 || (q && q_weight && q_out)) && (k_heads == 0 || (k && k_weight && k_out)),
                   CPPINF_ERR_INVALID_ARGUMENT, "qk_norm_rope received a null pointer.");
    CPPINF_REQUIRE(rt::aligned16(table) && (q_heads == 0 || (rt::aligned16(q) && rt::aligned16(q_weight) &&
                                                             rt::aligned16(q_out))) &&
                       (k_heads == 0 || (rt::aligned16(k) && rt::aligned16(k_weight) && rt::aligned16(k_out))),
                   CPPINF_ERR_UNSUPPORTED, "qk_norm_rope requires 16-byte aligned operands.");
    QkParams p{};
    p.q = q;
    p.k = k;
    p.qw = q_weight;
    p.kw = k_weight;
    p.q_out = q_out;
    p.k_out = k_out;
    p.table = table;
    p.position_offset = position_offset;
    p.q_heads = static_cast<int>(q_heads);
    p.k_heads = static_cast<int>(k_heads);
    p.eps = eps;
    const auto s = rt::as_stream(stream);
    const cudaError_t launch_err = dtype == CPPINF_DTYPE_BF16
                                       ? dispatch_qk<bf16>(p, tokens, static_cast<int>(lanes), s)
                                       : dispatch_qk<float>(p, tokens, static_cast<int>(lanes), s);
    return rt::launched(launch_err, "qk_norm_rope");
}

}  // extern "C"
