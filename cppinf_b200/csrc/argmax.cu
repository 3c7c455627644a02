// Row argmax over logits, the greedy pick of cli::detail::select_argmax_token_id (src/cli/cli_app.cpp:72-94) applied
// to every row of a [rows, cols] bf16/f32 matrix (the reference scans the last row of [seq, vocab] logits).
//
// Semantics of the reference's scan (best = x[0]; for i >= 1: if (x[i] > best) take i):
//  - the largest value wins, ties go to the lowest index (strict '>'), +0 and -0 compare equal;
//  - NaN never wins, except that a NaN at index 0 is never replaced, so the result is 0.
// Each thread keeps a running (value, index) over the elements it visits in increasing index order with the same
// strict '>' rule. Across threads the partial results are combined with an order-independent key,
// key(i) = (orderable(x[i]) << 32) | (2^32 - 1 - i), where orderable() maps floats to unsigned integers monotonically
// (after folding -0 into +0): max(key) is the lowest index of the largest value. A row whose element 0 is NaN
// yields 0.
//
// Layout: a row is split across a thread-block cluster of up to 8 CTAs of 256 threads, each CTA scanning a contiguous
// column range (scalar loads when the rows are not aligned for 16-byte vectors). Before its dependency wait each CTA
// asks L2 for its range (`cp.async.bulk.prefetch.L2`): back-to-back launches then overlap, the next launch's CTAs (20
// KB of shared memory each, so a whole second grid fits beside the running one) pulling their rows from HBM while the
// previous launch finishes. The range then streams through shared memory by per-thread asynchronous copies and through
// registers, all of a chunk requested before any is read; each 16-byte vector is first reduced with packed max
// instructions; a vector that would replace the thread's running maximum is kept whole and searched for its index once,
// after the last vector. Measured on B200 ([64, 151936] bf16, graph-replayed launches over buffers larger than L2):
// 6.19 us before the prefetch, 5.56-5.69 with it at 512 threads x 5 vectors, 5.23-5.26 at 256 x 5; 256 x 3, 256 x 4,
// 192 x 5 (more chunks per thread), 256 x 10 and 128 x 10 (fewer CTAs beside the running grid) 5.42-6.47. Each CTA also
// prefetching the range of the CTA half a grid away (the first CTAs to become resident then cover the rest): 6.03 ->
// 5.35 and 5.79-5.90 -> 5.47 us on two further boxes (four partners: 6.69). Five of each thread's ten vectors loaded
// into registers beside the five copied to shared memory, so a thread's whole range is one round trip: 5.33-5.42 ->
// 5.10-5.12 us on two boxes (7 + 3, 6 + 4: 6.3-6.4 us; 4 + 6 and more in registers, past 64 registers and so two waves:
// 8.5-9.0 us). With one round trip the partner prefetch no longer pays: one range per CTA 5.07 us against 5.60 with the
// partner's. Before the prefetch, register loads in batches of 5, 32-byte loads, clusters of 16 and bulk copies (TMA)
// of 2-8 KB chunks per CTA on mbarriers were slower too. CTA partials are combined through distributed shared memory:
// each CTA stores its key into cluster rank 0's shared array, one cluster barrier makes them visible, rank 0 combines
// them. No global scratch and no second launch are needed, and no thread waits on a flag (the copy-group waits are
// hardware waits).
//
// Roofline: HBM-bound. Algorithmic bytes per row: cols * size read + 8 bytes written.
#include <cooperative_groups.h>

#include "common.cuh"
#include "runtime.h"

namespace cg = cooperative_groups;

namespace cppinf::device {
namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kStaged = 5;  // 16-byte vectors per thread per shared-memory chunk (20 KB per CTA)
constexpr int kHeld = 5;    // 16-byte vectors per thread per chunk loaded into registers
constexpr int kCtasPerSmMin = 4;  // register cap of 64: one wave of 4 CTAs per SM (more registers: two waves)
constexpr int kMaxCluster = 8;
constexpr int64_t kPrefetchBytes = 64 * 1024;  // per CTA range, issued before the dependency wait
constexpr int kPrefetchSlices = 1;             // CTA ranges each CTA prefetches (see the file comment)
constexpr int kCtasPerSm = 4;                  // grid target: rows * cluster CTAs up to this many per SM

__device__ __forceinline__ unsigned long long argmax_key(float v, uint32_t index) {
    uint32_t u = __float_as_uint(v);
    if ((u & 0x7fffffffu) > 0x7f800000u) {
        return 0ull;  // NaN: never a candidate
    }
    if ((u & 0x7fffffffu) == 0u) {
        u = 0u;  // -0 == +0
    }
    const uint32_t ord = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return (static_cast<unsigned long long>(ord) << 32) | static_cast<unsigned long long>(0xffffffffu - index);
}

__device__ __forceinline__ unsigned long long umax64(unsigned long long a, unsigned long long b) {
    return a > b ? a : b;
}

// Per-thread running maximum over elements visited in increasing index order: strict '>' keeps the first of equal
// values (+0 and -0 included) and never takes NaN; `index < 0` marks "no candidate yet" so a leading -inf counts.
// A 16-byte vector that takes the maximum is kept whole (`vec`, with its first index in `index`) and searched for the
// position of the maximum only once, at the end (`resolve`): later vectors replace it only with a strictly larger
// value, so the first equal element of the kept vector is the answer, and the per-vector cost is a few packed max
// instructions and one compare.
struct Running {
    float value = -INFINITY;
    int index = -1;
    bool pending = false;  // `index` is the first index of `vec`, not yet resolved to the element
    uint4 vec = make_uint4(0u, 0u, 0u, 0u);

    __device__ __forceinline__ void visit(float v, int i) {
        if (v > value || (index < 0 && v == v)) {
            value = v;
            index = i;
            pending = false;
        }
    }

    template <typename T>
    __device__ __forceinline__ void resolve() {
        if (pending) {
            float v[Vec16<T>::kVec];
            Vec16<T>::unpack(vec, v);
            int j = Vec16<T>::kVec - 1;
#pragma unroll
            for (int k = Vec16<T>::kVec - 2; k >= 0; --k) {
                j = v[k] == value ? k : j;
            }
            index += j;
            pending = false;
        }
    }

    __device__ __forceinline__ unsigned long long key() const {
        return index < 0 ? 0ull : argmax_key(value, static_cast<uint32_t>(index));
    }

    // The kVec elements first .. first + kVec - 1 of one 16-byte vector, with the same result as visiting them one
    // by one: m = the vector's largest non-NaN value (packed max instructions: NaN loses to any number, and an
    // all-NaN vector gives NaN, which is never taken); when m is taken the vector is kept for `resolve`.
    template <typename T>
    __device__ __forceinline__ void visit_vector(uint4 r, int first) {
        float m;
        if constexpr (sizeof(T) == 2) {
            const __nv_bfloat162 m01 = __hmax2(as_bf162(r.x), as_bf162(r.y));
            const __nv_bfloat162 m23 = __hmax2(as_bf162(r.z), as_bf162(r.w));
            const uint32_t mw = bf162_bits(__hmax2(m01, m23));
            m = fmaxf(bf16_lo(mw), bf16_hi(mw));
        } else {
            m = fmaxf(fmaxf(__uint_as_float(r.x), __uint_as_float(r.y)),
                      fmaxf(__uint_as_float(r.z), __uint_as_float(r.w)));
        }
        if (m > value || (index < 0 && m == m)) {
            value = m;
            index = first;
            vec = r;
            pending = true;
        }
    }

    __device__ __forceinline__ static __nv_bfloat162 as_bf162(uint32_t w) {
        __nv_bfloat162 h;
        memcpy(&h, &w, sizeof(w));
        return h;
    }
    __device__ __forceinline__ static uint32_t bf162_bits(__nv_bfloat162 h) {
        uint32_t w;
        memcpy(&w, &h, sizeof(w));
        return w;
    }
};

// kBytes: 32 or 16 for vector loads of the row, 0 for element loads.
template <typename T, int kBytes>
__global__ void __launch_bounds__(kThreads, kCtasPerSmMin) row_argmax_kernel(const void* __restrict__ x, int64_t cols,
                                                              int64_t row_stride, int64_t* __restrict__ out) {
    // Every CTA of the cluster has started once this barrier phase completes; it is waited on right before the one
    // DSMEM store below, long after every CTA has arrived.
    asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
    constexpr int kVec = kBytes == 0 ? 1 : kBytes / static_cast<int>(sizeof(T));
    __shared__ unsigned long long warp_best[kWarps];
    __shared__ unsigned long long cluster_best[kMaxCluster];  // rank 0's copy receives every CTA's key

    cg::cluster_group cluster = cg::this_cluster();
    const unsigned rank = cluster.block_rank();
    const unsigned csize = cluster.num_blocks();     // a power of two (1 .. 8)
    const unsigned cshift = __ffs(csize) - 1;
    const int64_t row = blockIdx.x >> cshift;
    const char* xr = static_cast<const char*>(x) + row * row_stride * static_cast<int64_t>(sizeof(T));

    // Column range of this CTA, cut at vector boundaries so every vector load stays aligned (cols < 2^31, so the
    // column arithmetic is 32-bit).
    const int ncols = static_cast<int>(cols);
    const int per_cta = ((((ncols - 1) >> cshift) + 1 + kVec - 1) / kVec) * kVec;
    const int lo = per_cta * static_cast<int>(rank) < ncols ? per_cta * static_cast<int>(rank) : ncols;
    const int hi = lo + per_cta < ncols ? lo + per_cta : ncols;

    // Before the dependency wait (while the previous kernel still runs): ask L2 for the first kPrefetchBytes of the
    // whole vectors of kPrefetchSlices CTAs' ranges, this CTA's and those of kPrefetchSlices - 1 partners spread over
    // the grid (the CTAs that become resident first then also cover those that cannot yet). A prefetch returns no
    // data and L2 is the point of coherence, so values the previous kernel writes after it are still the ones read
    // below.
    if constexpr (kBytes > 0) {
        if (threadIdx.x < kPrefetchSlices) {
            const unsigned step = (gridDim.x + kPrefetchSlices - 1) / kPrefetchSlices;
            const unsigned c = (blockIdx.x + threadIdx.x * step) % gridDim.x;
            const int c_rank = static_cast<int>(c & (csize - 1));
            const int c_lo = per_cta * c_rank < ncols ? per_cta * c_rank : ncols;
            const int c_hi = c_lo + per_cta < ncols ? c_lo + per_cta : ncols;
            const int64_t whole = static_cast<int64_t>((c_hi - c_lo) / kVec) * kBytes;
            const uint32_t bytes = static_cast<uint32_t>(whole < kPrefetchBytes ? whole : kPrefetchBytes);
            if (bytes > 0) {
                const char* c_row = static_cast<const char*>(x) +
                                    static_cast<int64_t>(c >> cshift) * row_stride * static_cast<int64_t>(sizeof(T));
                bulk_prefetch_l2(c_row + static_cast<int64_t>(c_lo) * static_cast<int64_t>(sizeof(T)), bytes);
            }
        }
    }
    grid_dependency_begin();
    // Element 0 of the row decides the NaN-at-index-0 case; its load is issued now and lands during the scan.
    const float first = rank == 0 && threadIdx.x == 0 ? Vec16<T>::load1(xr, 0) : 0.0f;

    // Each thread visits its elements in increasing index order (vectors v, v + kThreads, ...; then the tail).
    Running run;
    if constexpr (kBytes > 0) {
        const int nvec = (hi - lo) / kVec;
        const char* base = xr + static_cast<int64_t>(lo) * static_cast<int64_t>(sizeof(T));
        // The slice streams in chunks of kStaged + kHeld vectors per thread: the first kStaged by asynchronous copies
        // into shared memory, the next kHeld by loads into registers, all of a chunk requested before the thread
        // waits for any of them, so a whole chunk (the whole slice, for the 151936-column vocabulary) is one round
        // trip. Each thread reads back only the shared-memory slots it filled, so no block barrier is needed; the
        // vectors are visited in increasing index order (shared-memory ones first).
        __shared__ uint4 staged[kStaged][kThreads];
        for (int c0 = 0; c0 < nvec; c0 += (kStaged + kHeld) * kThreads) {
#pragma unroll
            for (int u = 0; u < kStaged; ++u) {
                const int v = c0 + u * kThreads + static_cast<int>(threadIdx.x);
                if (v < nvec) {
                    cp_async16(&staged[u][threadIdx.x], base + static_cast<int64_t>(v) * kBytes);
                }
                cp_async_commit();
            }
            uint4 held[kHeld];
#pragma unroll
            for (int u = 0; u < kHeld; ++u) {
                const int v = c0 + (kStaged + u) * kThreads + static_cast<int>(threadIdx.x);
                if (v < nvec) {
                    held[u] = ld_stream(base + static_cast<int64_t>(v) * kBytes);
                }
            }
            // Vector u is visited as soon as its own copy group has landed (the later ones keep arriving).
#pragma unroll
            for (int u = 0; u < kStaged; ++u) {
                cp_async_wait_pending(kStaged - 1 - u);
                const int v = c0 + u * kThreads + static_cast<int>(threadIdx.x);
                if (v < nvec) {
                    run.visit_vector<T>(staged[u][threadIdx.x], lo + v * kVec);
                }
            }
#pragma unroll
            for (int u = 0; u < kHeld; ++u) {
                const int v = c0 + (kStaged + u) * kThreads + static_cast<int>(threadIdx.x);
                if (v < nvec) {
                    run.visit_vector<T>(held[u], lo + v * kVec);
                }
            }
        }
        run.resolve<T>();
        for (int e = lo + nvec * kVec + static_cast<int>(threadIdx.x); e < hi; e += kThreads) {
            run.visit(Vec16<T>::load1(xr, e), e);
        }
    } else {
        for (int e = lo + static_cast<int>(threadIdx.x); e < hi; e += kThreads) {
            run.visit(Vec16<T>::load1(xr, e), e);
        }
    }
    unsigned long long best = run.key();

#pragma unroll
    for (int offset = 16; offset > 0; offset >>= 1) {
        best = umax64(best, __shfl_xor_sync(0xffffffffu, best, offset));
    }
    const int warp = threadIdx.x / 32;
    if ((threadIdx.x & 31) == 0) {
        warp_best[warp] = best;
    }
    __syncthreads();
    asm volatile("barrier.cluster.wait.aligned;" ::: "memory");  // every CTA has started: DSMEM is usable
    if (threadIdx.x == 0) {
        unsigned long long b = warp_best[0];
#pragma unroll
        for (int w = 1; w < kWarps; ++w) {
            b = umax64(b, warp_best[w]);
        }
        // Push this CTA's key into rank 0's shared memory (a remote store, no remote load).
        *cluster.map_shared_rank(&cluster_best[rank], 0) = b;
    }
    // The pushes are visible to rank 0 after this barrier; no CTA touches another's shared memory after it, so the
    // other ranks may leave while rank 0 finishes.
    cluster.sync();
    if (rank == 0 && threadIdx.x == 0) {
        unsigned long long b = cluster_best[0];
        for (unsigned r = 1; r < csize; ++r) {
            b = umax64(b, cluster_best[r]);
        }
        int64_t index = 0;
        if (first == first && b != 0ull) {
            index = static_cast<int64_t>(0xffffffffu - static_cast<uint32_t>(b & 0xffffffffull));
        }
        out[row] = index;
    }
}

template <typename T>
cudaError_t launch_argmax(const void* x, int64_t rows, int64_t cols, int64_t row_stride, int64_t* out,
                          unsigned cluster, cudaStream_t s) {
    const auto base = reinterpret_cast<std::uintptr_t>(x);
    const int64_t stride_bytes = row_stride * static_cast<int64_t>(sizeof(T));
    const bool rows16 = (base & 15u) == 0 && (rows <= 1 || stride_bytes % 16 == 0);
    const dim3 grid(static_cast<unsigned>(rows * cluster));
    if (rows16) {
        return runtime::launch(row_argmax_kernel<T, 16>, grid, dim3(kThreads), s, cluster, x, cols, row_stride, out);
    }
    return runtime::launch(row_argmax_kernel<T, 0>, grid, dim3(kThreads), s, cluster, x, cols, row_stride, out);
}

}  // namespace
}  // namespace cppinf::device

using namespace cppinf::device;
namespace rt = cppinf::runtime;

extern "C" {

int cppinf_row_argmax(cppinf_dtype dtype, const void* x, int64_t rows, int64_t cols, int64_t row_stride,
                      int64_t* out, void* stream) {
    CPPINF_REQUIRE(rt::valid_dtype(dtype), CPPINF_ERR_INVALID_ARGUMENT, "row_argmax received an unsupported dtype.");
    CPPINF_REQUIRE(rows >= 0, CPPINF_ERR_INVALID_ARGUMENT, "logits sequence length must be non-negative.");
    CPPINF_REQUIRE(cols > 0, CPPINF_ERR_INVALID_ARGUMENT, "logits vocab size must be non-zero.");
    CPPINF_REQUIRE(cols < (int64_t{1} << 31), CPPINF_ERR_OVERFLOW, "row_argmax supports fewer than 2^31 columns.");
    CPPINF_REQUIRE(rows <= 1 || row_stride >= cols, CPPINF_ERR_INVALID_ARGUMENT,
                   "row_argmax requires a row stride of at least the column count.");
    if (rows == 0) {
        return rt::ok();
    }
    CPPINF_REQUIRE(x && out, CPPINF_ERR_INVALID_ARGUMENT, "row_argmax received a null pointer.");
    CPPINF_REQUIRE(rows <= (int64_t{1} << 27), CPPINF_ERR_UNSUPPORTED, "row_argmax supports at most 2^27 rows.");

    // Enough CTAs to cover the SMs a few times, but no CTA with fewer than ~4K columns.
    const int64_t target_ctas = static_cast<int64_t>(rt::sm_count()) * kCtasPerSm;
    int64_t cluster = 1;
    while (cluster < kMaxCluster && rows * cluster < target_ctas && cols / (cluster * 2) >= 4096) {
        cluster *= 2;
    }
    const auto s = rt::as_stream(stream);
    const cudaError_t launch_err =
        dtype == CPPINF_DTYPE_BF16
            ? launch_argmax<bf16>(x, rows, cols, row_stride, out, static_cast<unsigned>(cluster), s)
            : launch_argmax<float>(x, rows, cols, row_stride, out, static_cast<unsigned>(cluster), s);
    return rt::launched(launch_err, "row_argmax");
}

}  // extern "C"
