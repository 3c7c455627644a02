// tcgen05 / TMA building blocks shared by the tensor-core kernels (gemm_tc.cu, attention_tc.cu): 2-D and 3-D TMA
// tile loads, tensor-memory allocation, the bf16 UMMA with its commit, 32-column tensor-memory loads, and the
// shared-memory and instruction descriptors of K-major tiles written by TMA with the 128-byte swizzle.
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include "common.cuh"

namespace cppinf::device::tc {

constexpr int kBM = 128;  // UMMA rows = tensor-memory lanes
constexpr int kBK = 64;   // one 128-byte swizzle row of bf16
constexpr int kUmmaK = 16;

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
        "[%4];" ::"r"(smem_addr(dst)),
        "l"(map), "r"(x), "r"(y), "r"(smem_addr(bar))
        : "memory");
}

__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t cols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(dst_smem)),
                 "r"(cols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t cols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, both K-major; `accumulate` = 0 overwrites D.
__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
    asm volatile(
        "{\n"
        ".reg .pred p;\n"
        "setp.ne.b32 p, %4, 0;\n"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n"
        "}\n" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrives once on `bar` when every tcgen05.mma this thread issued before has completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
                 : "memory");
}

// 32 consecutive f32 columns of this thread's tensor-memory lane.
__device__ __forceinline__ void tmem_load32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
          "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) {
        v[i] = __uint_as_float(r[i]);
    }
}

// Shared-memory matrix descriptor of a K-major tile written by TMA with the 128-byte swizzle: rows of 64 bf16
// (128 bytes), 8-row groups 1024 bytes apart (stride byte offset), layout type 2 (SWIZZLE_128B) in bits 61-63,
// descriptor version 1 in bits 46-47. The leading byte offset is not used by swizzled K-major layouts. Moving along
// K inside the 128-byte row adds the byte offset to the start address (the swizzle is a function of the address
// bits, and every tile starts 1024-byte aligned).
__device__ __forceinline__ uint64_t smem_desc_sw128(const void* tile, uint32_t k_byte_offset) {
    const uint32_t addr = smem_addr(tile) + k_byte_offset;
    uint64_t d = 0;
    d |= static_cast<uint64_t>((addr >> 4) & 0x3fffu);       // start address, bits 0-13
    d |= static_cast<uint64_t>(1u) << 16;                     // leading byte offset (unused), bits 16-29
    d |= static_cast<uint64_t>((1024u >> 4) & 0x3fffu) << 32;  // stride byte offset, bits 32-45
    d |= static_cast<uint64_t>(1u) << 46;                     // version, bits 46-47
    d |= static_cast<uint64_t>(2u) << 61;                     // SWIZZLE_128B, bits 61-63
    return d;
}

// Instruction descriptor of kind::f16 with bf16 A and B, f32 D, both K-major, M = 128, N = n:
// D format bits 4-5 (1 = f32), A format bits 7-9 and B format bits 10-12 (1 = bf16), N >> 3 in bits 17-22,
// M >> 4 in bits 24-28.
__host__ __device__ constexpr uint32_t idesc_bf16_f32(int n) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((static_cast<uint32_t>(n) >> 3) << 17) |
           ((static_cast<uint32_t>(kBM) >> 4) << 24);
}

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int x, int y, int z, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
        "[%5];" ::"r"(smem_addr(dst)),
        "l"(map), "r"(x), "r"(y), "r"(z), "r"(smem_addr(bar))
        : "memory");
}

// Makes this thread's generic-proxy shared-memory writes visible to the async proxy (tcgen05.mma operands).
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---- host side ----------------------------------------------------------------------------------------------

using EncodeTiled = PFN_cuTensorMapEncodeTiled_v12000;

// cuTensorMapEncodeTiled from the driver, looked up once through the runtime (no link against libcuda).
inline EncodeTiled encode_tiled() {
    static EncodeTiled fn = [] {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess) {
            return static_cast<EncodeTiled>(nullptr);
        }
        return reinterpret_cast<EncodeTiled>(ptr);
    }();
    return fn;
}

}  // namespace cppinf::device::tc
