// Shared device-side helpers for the cppinf_b200 kernels: 128-bit global loads/stores, bf16 <-> f32 conversion,
// warp reductions and the launch bookkeeping every entry point uses.
//
// Numerics: every kernel in this library is compiled with --fmad=false, so each f32 multiply and add is rounded
// separately, the same as the reference's x86-64 SSE code (built without -mfma). f32 -> bf16 conversion is IEEE
// round-to-nearest-even (cvt.rn.bf16x2.f32), which equals the reference's `bits + 0x7fff + lsb` rounding
// (src/tensors/bfloat16.cpp:8-15) for every non-NaN value. NaN stays NaN (the reference helper's payload-dependent
// NaN handling is not reproduced).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace cppinf::device {

using bf16 = __nv_bfloat16;

// ---- programmatic dependent launch -------------------------------------------------------------------------------

// First statement of every kernel: waits until the previous grid in the stream has completed and its memory writes
// are visible (a no-op when the launch did not allow programmatic overlap), then lets the next grid be scheduled
// as soon as all CTAs of this one have started.
__device__ __forceinline__ void grid_dependency_begin() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---- 128-bit memory access -------------------------------------------------------------------------------------

// Read-only, streaming load: bypasses L1 allocation (the data is touched once) and asks L2 for 256-byte sectors so
// neighbouring warps' requests share DRAM bursts.
__device__ __forceinline__ uint4 ld_stream(const void* ptr) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(ptr));
    return r;
}

// Read-only load that is expected to hit in L1/L2 (norm weights, RoPE table rows).
__device__ __forceinline__ uint4 ld_cached(const void* ptr) {
    return __ldg(reinterpret_cast<const uint4*>(ptr));
}

__device__ __forceinline__ float4 ld_cached_f4(const float* ptr) {
    return __ldg(reinterpret_cast<const float4*>(ptr));
}

// 256-bit (32-byte) accesses, sm_100: one instruction moves a whole 32-byte sector, which halves the memory
// instructions of a streaming kernel and lets a copy reach the measured HBM peak. Addresses must be 32-byte aligned.
struct U8 {
    uint32_t r[8];
};

__device__ __forceinline__ U8 ld_stream32(const void* ptr) {
    U8 v;
    asm volatile("ld.global.nc.L1::no_allocate.v8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=r"(v.r[0]), "=r"(v.r[1]), "=r"(v.r[2]), "=r"(v.r[3]), "=r"(v.r[4]), "=r"(v.r[5]), "=r"(v.r[6]),
                   "=r"(v.r[7])
                 : "l"(ptr));
    return v;
}

__device__ __forceinline__ void st_stream32(void* ptr, const U8& v) {
    asm volatile("st.global.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(ptr), "r"(v.r[0]), "r"(v.r[1]),
                 "r"(v.r[2]), "r"(v.r[3]), "r"(v.r[4]), "r"(v.r[5]), "r"(v.r[6]), "r"(v.r[7])
                 : "memory");
}

// Plain 128-bit store.
__device__ __forceinline__ void st_v4(void* ptr, uint4 v) {
    asm volatile("st.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(ptr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                 : "memory");
}

// Streaming (evict-first) 128-bit store for outputs that are not read again by this kernel.
__device__ __forceinline__ void st_stream(void* ptr, uint4 v) {
    asm volatile("st.global.cs.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(ptr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                 : "memory");
}

// ---- bulk asynchronous copies (TMA engine) into shared memory, completed on an mbarrier ---------------------------
// Plain global -> shared bulk copies of one CTA (no multicast). Addresses and sizes must be multiples of 16 bytes.

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// One arrival that also announces `bytes` of bulk-copy data the barrier's current phase must receive.
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
                 : "memory");
}

// Per-thread asynchronous 16-byte copy global -> shared (L2 only, no L1 allocation, 256-byte L2 prefetch). The
// data lands in shared memory without passing through registers; cp_async_wait_all() waits for the calling
// thread's copies (a hardware wait, like a load's scoreboard), after which a __syncwarp()/__syncthreads() makes
// them visible to the other threads.
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global.L2::256B [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}

__device__ __forceinline__ void cp_async_wait_all() {
    asm volatile("cp.async.wait_all;" ::: "memory");
}

// Closes the calling thread's current group of asynchronous copies.
__device__ __forceinline__ void cp_async_commit() {
    asm volatile("cp.async.commit_group;" ::: "memory");
}

// Waits until at most `pending` (0..15) of the calling thread's committed copy groups are still in flight; larger
// values wait for all. In unrolled loops the switch folds to one instruction.
__device__ __forceinline__ void cp_async_wait_pending(int pending) {
    switch (pending) {
#define CPPINF_WAIT_GROUP(n)                                       \
    case n:                                                        \
        asm volatile("cp.async.wait_group " #n ";" ::: "memory"); \
        break;
        CPPINF_WAIT_GROUP(0)
        CPPINF_WAIT_GROUP(1)
        CPPINF_WAIT_GROUP(2)
        CPPINF_WAIT_GROUP(3)
        CPPINF_WAIT_GROUP(4)
        CPPINF_WAIT_GROUP(5)
        CPPINF_WAIT_GROUP(6)
        CPPINF_WAIT_GROUP(7)
        CPPINF_WAIT_GROUP(8)
        CPPINF_WAIT_GROUP(9)
        CPPINF_WAIT_GROUP(10)
        CPPINF_WAIT_GROUP(11)
        CPPINF_WAIT_GROUP(12)
        CPPINF_WAIT_GROUP(13)
        CPPINF_WAIT_GROUP(14)
        CPPINF_WAIT_GROUP(15)
#undef CPPINF_WAIT_GROUP
    default:
        asm volatile("cp.async.wait_all;" ::: "memory");
        break;
    }
}

// Brings `bytes` (a multiple of 16, 16-byte aligned) of global memory into L2 without waiting (no data returned).
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

__device__ __forceinline__ void bulk_copy_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t phase) {
    uint32_t done;
    asm volatile(
        "{\n"
        ".reg .pred p;\n"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        "selp.u32 %0, 1, 0, p;\n"
        "}\n"
        : "=r"(done)
        : "r"(smem_addr(bar)), "r"(phase)
        : "memory");
    return done != 0;
}

// Default poll limit of the bounded mbarrier waits: each try_wait may itself suspend the thread for a short,
// hardware-chosen time, so 2^24 polls is far longer than any copy of this library takes.
constexpr uint32_t kDefaultPollLimit = 1u << 24;

// Waits for phase `phase` of `bar` with at most `max_polls` polls (0: give up at once). Returns false if the limit
// ran out; the caller records the error and must not use the copied data.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t phase, uint32_t max_polls = kDefaultPollLimit) {
    for (uint32_t i = 0; i < max_polls; ++i) {
        if (mbar_try_wait(bar, phase)) {
            return true;
        }
    }
    return false;
}

// ---- bf16 / f32 packing ------------------------------------------------------------------------------------------

__device__ __forceinline__ float bf16_lo(uint32_t packed) {
    return __uint_as_float(packed << 16);
}

__device__ __forceinline__ float bf16_hi(uint32_t packed) {
    return __uint_as_float(packed & 0xffff0000u);
}

// One step of an RMSNorm sum of squares: s + v * v, fused for bf16 inputs (the square of a bf16 value is exact in f32
// wherever it is normal, |v| >= 2^-63, so this equals the separately rounded form there; the oracle restates it with
// fmaf), separately rounded for f32 inputs (whose squares are not exact).
template <typename T>
__device__ __forceinline__ float sum_square(float s, float v) {
    if constexpr (sizeof(T) == 2) {
        return __fmaf_rn(v, v, s);
    } else {
        return s + v * v;
    }
}

// Dot-product accumulation of bf16 operands: acc = fma(a, b, acc), rounded once. A product of two bf16 values has at
// most 16 significant bits, so wherever it lies in the f32 normal range it is exact and the fused multiply-add equals
// the separately rounded `acc + a * b`; the CPU oracle restates it with fmaf, which agrees for every operand.
// Mixed-precision form (bf16 operands straight from the packed words, f32 accumulator): one instruction per element.
__device__ __forceinline__ float fma_bf16x2(uint32_t a, uint32_t b, float acc) {  // low halves, then high halves
    asm("{\n\t.reg .b16 al, ah, bl, bh;\n\tmov.b32 {al, ah}, %1;\n\tmov.b32 {bl, bh}, %2;\n\t"
        "fma.rn.f32.bf16 %0, al, bl, %0;\n\tfma.rn.f32.bf16 %0, ah, bh, %0;\n\t}"
        : "+f"(acc)
        : "r"(a), "r"(b));
    return acc;
}

// Eight elements of two 16-byte bf16 vectors, accumulated in element order.
__device__ __forceinline__ float fma_bf16x8(uint4 a, uint4 b, float acc) {
    acc = fma_bf16x2(a.x, b.x, acc);
    acc = fma_bf16x2(a.y, b.y, acc);
    acc = fma_bf16x2(a.z, b.z, acc);
    acc = fma_bf16x2(a.w, b.w, acc);
    return acc;
}

// Packs two f32 values into a bf16x2 word (lo in the low half), round-to-nearest-even.
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
    uint32_t r;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}

__device__ __forceinline__ float round_to_bf16(float v) {
    return bf16_lo(pack_bf16x2(v, 0.0f));
}

// Element traits: a 16-byte vector holds kVec elements of T, read or written as f32.
template <typename T>
struct Vec16;

template <>
struct Vec16<bf16> {
    static constexpr int kVec = 8;
    __device__ __forceinline__ static void unpack(uint4 v, float (&f)[8]) {
        f[0] = bf16_lo(v.x);
        f[1] = bf16_hi(v.x);
        f[2] = bf16_lo(v.y);
        f[3] = bf16_hi(v.y);
        f[4] = bf16_lo(v.z);
        f[5] = bf16_hi(v.z);
        f[6] = bf16_lo(v.w);
        f[7] = bf16_hi(v.w);
    }
    __device__ __forceinline__ static uint4 pack(const float (&f)[8]) {
        return make_uint4(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]), pack_bf16x2(f[4], f[5]),
                          pack_bf16x2(f[6], f[7]));
    }
    // Value as stored: rounds f32 to bf16 and back.
    __device__ __forceinline__ static float quantize(float v) { return round_to_bf16(v); }
    // Two values as stored (one rounding instruction for both).
    __device__ __forceinline__ static float2 quantize2(float x, float y) {
        const uint32_t w = pack_bf16x2(x, y);
        return make_float2(bf16_lo(w), bf16_hi(w));
    }
    __device__ __forceinline__ static float load1(const void* base, int64_t i) {
        const uint16_t bits = __ldg(reinterpret_cast<const unsigned short*>(base) + i);
        return __uint_as_float(static_cast<uint32_t>(bits) << 16);
    }
    __device__ __forceinline__ static void store1(void* base, int64_t i, float v) {
        reinterpret_cast<unsigned short*>(base)[i] = static_cast<unsigned short>(pack_bf16x2(v, 0.0f) & 0xffffu);
    }
};

template <>
struct Vec16<float> {
    static constexpr int kVec = 4;
    __device__ __forceinline__ static void unpack(uint4 v, float (&f)[4]) {
        f[0] = __uint_as_float(v.x);
        f[1] = __uint_as_float(v.y);
        f[2] = __uint_as_float(v.z);
        f[3] = __uint_as_float(v.w);
    }
    __device__ __forceinline__ static uint4 pack(const float (&f)[4]) {
        return make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]), __float_as_uint(f[2]), __float_as_uint(f[3]));
    }
    __device__ __forceinline__ static float quantize(float v) { return v; }
    __device__ __forceinline__ static float2 quantize2(float x, float y) { return make_float2(x, y); }
    __device__ __forceinline__ static float load1(const void* base, int64_t i) {
        return __ldg(reinterpret_cast<const float*>(base) + i);
    }
    __device__ __forceinline__ static void store1(void* base, int64_t i, float v) {
        reinterpret_cast<float*>(base)[i] = v;
    }
};

// ---- 16- or 32-byte chunks of T as f32 ---------------------------------------------------------------------------

template <typename T, int kBytes>
struct Chunk {
    static constexpr int kElems = kBytes / static_cast<int>(sizeof(T));

    __device__ __forceinline__ static void load(const void* p, float (&f)[kElems]) {
        if constexpr (kBytes == 32) {
            const U8 v = ld_stream32(p);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                unpack_word(v.r[i], f, i);
            }
        } else {
            const uint4 v = ld_stream(p);
            unpack_word(v.x, f, 0);
            unpack_word(v.y, f, 1);
            unpack_word(v.z, f, 2);
            unpack_word(v.w, f, 3);
        }
    }

    __device__ __forceinline__ static void store(void* p, const float (&f)[kElems]) {
        if constexpr (kBytes == 32) {
            U8 v;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                v.r[i] = pack_word(f, i);
            }
            st_stream32(p, v);
        } else {
            st_stream(p, make_uint4(pack_word(f, 0), pack_word(f, 1), pack_word(f, 2), pack_word(f, 3)));
        }
    }

  private:
    __device__ __forceinline__ static void unpack_word(uint32_t w, float (&f)[kElems], int i) {
        if constexpr (sizeof(T) == 2) {
            f[2 * i] = bf16_lo(w);
            f[2 * i + 1] = bf16_hi(w);
        } else {
            f[i] = __uint_as_float(w);
        }
    }

    __device__ __forceinline__ static uint32_t pack_word(const float (&f)[kElems], int i) {
        if constexpr (sizeof(T) == 2) {
            return pack_bf16x2(f[2 * i], f[2 * i + 1]);
        } else {
            return __float_as_uint(f[i]);
        }
    }
};

// ---- integer division by a launch-time constant ------------------------------------------------------------------

// n / d for 0 <= n < 2^31 and 1 <= d < 2^31 by a multiply-high and a shift (Granlund-Montgomery round-up method):
// with l = ceil(log2 d) and m = floor(2^32 (2^l - d) / d) + 1, n / d = (umulhi(n, m) + n) >> l, and the sum stays
// below 2^32 because umulhi(n, m) <= n < 2^31. The host builds it once per launch; the device pays 3 instructions
// instead of a 32- or 64-bit division routine.
struct FastDiv {
    uint32_t d = 1;
    uint32_t m = 1;
    uint32_t l = 0;

    FastDiv() = default;
    __host__ explicit FastDiv(uint32_t divisor) : d(divisor) {
        while ((uint64_t{1} << l) < divisor) {
            ++l;
        }
        m = static_cast<uint32_t>((((uint64_t{1} << 32) * ((uint64_t{1} << l) - divisor)) / divisor) + 1);
    }
    __device__ __forceinline__ uint32_t quot(uint32_t n) const { return (__umulhi(n, m) + n) >> l; }
};

// ---- warp reductions ---------------------------------------------------------------------------------------------

// Butterfly sum over groups of `kLanes` consecutive lanes (a power of two <= 32). Every lane of a group ends with
// the same bits: step s adds the partner's partial, and f32 addition is commutative, so partners agree.
template <int kLanes>
__device__ __forceinline__ float group_sum(float v) {
#pragma unroll
    for (int offset = kLanes / 2; offset > 0; offset >>= 1) {
        v = v + __shfl_xor_sync(0xffffffffu, v, offset);
    }
    return v;
}

template <int kLanes>
__device__ __forceinline__ float group_max(float v) {
#pragma unroll
    for (int offset = kLanes / 2; offset > 0; offset >>= 1) {
        v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, offset));
    }
    return v;
}

}  // namespace cppinf::device
