// Streaming elementwise kernels: ops::add / ops::mul (src/ops/elementwise_ops.cpp:28-36), ops::silu
// (src/ops/nn_ops.cpp:44-48), ops::cast (src/ops/tensor_ops.cpp:138-143), the fused silu*up product of the Qwen MLP
// (src/nn/qwen_mlp.cpp:65-66) and the strided gather that materialises non-contiguous views.
//
// Every kernel is HBM-bound (<= 1 flop per byte). Layout: dense arrays walked in packs of 32 bytes (256-bit loads
// and stores, when every operand is 32-byte aligned), else 16 bytes, else single elements; the result is the same on
// every path because each element is computed alone. The grid is two waves of resident blocks striding over the
// packs, kUnroll independent packs per thread per iteration, so each thread keeps several loads in flight.
#include <type_traits>

#include "common.cuh"
#include "runtime.h"

namespace cppinf::device {
namespace {

constexpr int kThreads = 256;
constexpr int kUnroll = 2;

// kBytes of consecutive elements held as 32-bit words.
template <int kBytes>
struct Words {
    static constexpr int kCount = kBytes / 4;
    uint32_t w[kCount];

    __device__ __forceinline__ static Words load(const void* p) {
        Words out;
        if constexpr (kBytes == 32) {
            const U8 v = ld_stream32(p);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                out.w[i] = v.r[i];
            }
        } else {
            const uint4 v = ld_stream(p);
            out.w[0] = v.x;
            out.w[1] = v.y;
            out.w[2] = v.z;
            out.w[3] = v.w;
        }
        return out;
    }

    __device__ __forceinline__ void store(void* p) const {
        if constexpr (kBytes == 32) {
            U8 v;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                v.r[i] = w[i];
            }
            st_stream32(p, v);
        } else {
            st_stream(p, make_uint4(w[0], w[1], w[2], w[3]));
        }
    }
};

// Elements of T in a pack, as f32.
template <typename T, int kBytes>
struct PackOf {
    static constexpr int kElems = kBytes / static_cast<int>(sizeof(T));

    __device__ __forceinline__ static void unpack(const Words<kBytes>& p, float (&f)[kElems]) {
#pragma unroll
        for (int i = 0; i < Words<kBytes>::kCount; ++i) {
            if constexpr (sizeof(T) == 2) {
                f[2 * i] = bf16_lo(p.w[i]);
                f[2 * i + 1] = bf16_hi(p.w[i]);
            } else {
                f[i] = __uint_as_float(p.w[i]);
            }
        }
    }

    __device__ __forceinline__ static Words<kBytes> pack(const float (&f)[kElems]) {
        Words<kBytes> p;
#pragma unroll
        for (int i = 0; i < Words<kBytes>::kCount; ++i) {
            if constexpr (sizeof(T) == 2) {
                p.w[i] = pack_bf16x2(f[2 * i], f[2 * i + 1]);
            } else {
                p.w[i] = __float_as_uint(f[i]);
            }
        }
        return p;
    }
};

enum class BinaryOp { Add, Mul };

template <BinaryOp op>
__device__ __forceinline__ float apply_binary(float a, float b) {
    if constexpr (op == BinaryOp::Add) {
        return a + b;
    } else {
        return a * b;
    }
}

// x / (1 + exp(-x)), oneDNN eltwise_swish with alpha = 1 as ops::silu configures it (src/ops/nn_ops.cpp:46-47).
// The quotient uses the fast division (reciprocal approximation and one multiply, within 2 ulp): the IEEE division
// sequence made the SiLU kernels issue-bound (the [4096, 3072] bf16 SiLU * up took 16.0 us with it, 13.2 us now).
// Its reciprocal flushes to zero for divisors of 2^126 and above (x < -87.3), where the IEEE quotient is still a
// tiny normal number, so there both operands are scaled by 1/4 first (exact: x is then below -87, d finite or inf).
__device__ __forceinline__ float silu_f32(float x) {
    const float d = 1.0f + expf(-x);
    const float scale = d < 0x1p126f ? 1.0f : 0.25f;
    return __fdividef(x * scale, d * scale);
}

// Two bf16 products, each rounded to nearest even (packed bf16 multiply).
__device__ __forceinline__ uint32_t mul_bf16x2(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}

// Whether a functor asks L2 for its operands before the dependency wait (`prefetch<kBytes>(pack, bytes)`).
template <typename F, typename = void>
struct HasPrefetch : std::false_type {};
template <typename F>
struct HasPrefetch<F, std::void_t<decltype(&F::template prefetch<32>)>> : std::true_type {};

// Grid-stride rounds of packs prefetched per warp. SiLU * up on [4096, 3072] bf16, measured on B200: none 13.40 us,
// one round 12.93, two 13.45.
constexpr int kPrefetchRounds = 1;

// Generic grid-stride driver. `Functor::load<kBytes>(i)` / `compute_store<kBytes>(i, loaded)` handle pack i,
// `Functor::scalar(e)` element e.
template <typename Functor, int kBytes>
__global__ void __launch_bounds__(kThreads) elementwise_kernel(Functor f, int64_t n_vec, int64_t vec_elems,
                                                               int64_t count) {
    if constexpr (HasPrefetch<Functor>::value && kPrefetchRounds > 0) {
        // Before the dependency wait (while the previous kernel still runs), lane 0 of each warp asks L2 for the
        // warp's first kPrefetchRounds groups of 32 consecutive packs. A prefetch returns no data and L2 is the
        // point of coherence, so the loads after the wait still see what the previous kernel writes.
        if ((threadIdx.x & 31) == 0) {
            const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
            const int64_t first = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
#pragma unroll
            for (int r = 0; r < kPrefetchRounds; ++r) {
                const int64_t i = first + r * stride;
                if (i < n_vec) {
                    const int64_t packs = n_vec - i < 32 ? n_vec - i : 32;
                    f.template prefetch<kBytes>(i, static_cast<uint32_t>(packs * kBytes));
                }
            }
        }
    }
    grid_dependency_begin();
    using Loaded = typename Functor::template Loaded<kBytes>;
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    int64_t i = tid;
    for (; i + (kUnroll - 1) * stride < n_vec; i += kUnroll * stride) {
        Loaded loaded[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            loaded[u] = f.template load<kBytes>(i + u * stride);
        }
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            f.template compute_store<kBytes>(i + u * stride, loaded[u]);
        }
    }
    for (; i < n_vec; i += stride) {
        f.template compute_store<kBytes>(i, f.template load<kBytes>(i));
    }
    // Scalar tail (or the whole array when the vector path is off).
    for (int64_t e = n_vec * vec_elems + tid; e < count; e += stride) {
        f.scalar(e);
    }
}

template <typename T, BinaryOp op>
struct BinaryFunctor {
    template <int kBytes>
    struct Loaded {
        Words<kBytes> a, b;
    };
    const char* lhs;
    const char* rhs;
    char* out;

    template <int kBytes>
    __device__ __forceinline__ Loaded<kBytes> load(int64_t i) const {
        return {Words<kBytes>::load(lhs + i * kBytes), Words<kBytes>::load(rhs + i * kBytes)};
    }
    template <int kBytes>
    __device__ __forceinline__ void compute_store(int64_t i, const Loaded<kBytes>& l) const {
        using P = PackOf<T, kBytes>;
        float a[P::kElems], b[P::kElems];
        P::unpack(l.a, a);
        P::unpack(l.b, b);
#pragma unroll
        for (int j = 0; j < P::kElems; ++j) {
            a[j] = apply_binary<op>(a[j], b[j]);
        }
        P::pack(a).store(out + i * kBytes);
    }
    __device__ __forceinline__ void scalar(int64_t e) const {
        Vec16<T>::store1(out, e, apply_binary<op>(Vec16<T>::load1(lhs, e), Vec16<T>::load1(rhs, e)));
    }
};

template <typename T>
struct SiluFunctor {
    template <int kBytes>
    using Loaded = Words<kBytes>;
    const char* x;
    char* y;

    template <int kBytes>
    __device__ __forceinline__ Loaded<kBytes> load(int64_t i) const {
        return Words<kBytes>::load(x + i * kBytes);
    }
    template <int kBytes>
    __device__ __forceinline__ void compute_store(int64_t i, const Loaded<kBytes>& l) const {
        using P = PackOf<T, kBytes>;
        float a[P::kElems];
        P::unpack(l, a);
#pragma unroll
        for (int j = 0; j < P::kElems; ++j) {
            a[j] = silu_f32(a[j]);
        }
        P::pack(a).store(y + i * kBytes);
    }
    __device__ __forceinline__ void scalar(int64_t e) const { Vec16<T>::store1(y, e, silu_f32(Vec16<T>::load1(x, e))); }
};

// out = T(T(silu(gate)) * up): the reference rounds the silu tensor to T before ops::mul reads it.
template <typename T>
struct SiluMulFunctor {
    template <int kBytes>
    struct Loaded {
        Words<kBytes> g, u;
    };
    const char* gate;
    const char* up;
    char* out;

    template <int kBytes>
    __device__ __forceinline__ Loaded<kBytes> load(int64_t i) const {
        return {Words<kBytes>::load(gate + i * kBytes), Words<kBytes>::load(up + i * kBytes)};
    }
    template <int kBytes>
    __device__ __forceinline__ void prefetch(int64_t i, uint32_t bytes) const {
        bulk_prefetch_l2(gate + i * kBytes, bytes);
        bulk_prefetch_l2(up + i * kBytes, bytes);
    }
    template <int kBytes>
    __device__ __forceinline__ void compute_store(int64_t i, const Loaded<kBytes>& l) const {
        if constexpr (sizeof(T) == 2) {
            // bf16: the silu values are rounded to bf16 in pairs and multiplied by up as packed bf16. A product of
            // two bf16 values is exact in f32, so one bf16 rounding of it equals the f32 product rounded to bf16.
            Words<kBytes> o;
#pragma unroll
            for (int k = 0; k < Words<kBytes>::kCount; ++k) {
                const uint32_t s = pack_bf16x2(silu_f32(bf16_lo(l.g.w[k])), silu_f32(bf16_hi(l.g.w[k])));
                o.w[k] = mul_bf16x2(s, l.u.w[k]);
            }
            o.store(out + i * kBytes);
        } else {
            using P = PackOf<T, kBytes>;
            float g[P::kElems], u[P::kElems];
            P::unpack(l.g, g);
            P::unpack(l.u, u);
#pragma unroll
            for (int j = 0; j < P::kElems; ++j) {
                g[j] = silu_f32(g[j]) * u[j];
            }
            P::pack(g).store(out + i * kBytes);
        }
    }
    __device__ __forceinline__ void scalar(int64_t e) const {
        const float s = Vec16<T>::quantize(silu_f32(Vec16<T>::load1(gate, e)));
        Vec16<T>::store1(out, e, s * Vec16<T>::load1(up, e));
    }
};

// bf16 -> f32: a pack of kBytes of bf16 produces two packs of f32.
struct CastBf16ToF32Functor {
    template <int kBytes>
    using Loaded = Words<kBytes>;
    const char* x;
    char* y;

    template <int kBytes>
    __device__ __forceinline__ Loaded<kBytes> load(int64_t i) const {
        return Words<kBytes>::load(x + i * kBytes);
    }
    template <int kBytes>
    __device__ __forceinline__ void compute_store(int64_t i, const Loaded<kBytes>& l) const {
        Words<kBytes> lo, hi;
        constexpr int kHalf = Words<kBytes>::kCount / 2;
#pragma unroll
        for (int k = 0; k < kHalf; ++k) {
            lo.w[2 * k] = l.w[k] << 16;
            lo.w[2 * k + 1] = l.w[k] & 0xffff0000u;
            hi.w[2 * k] = l.w[kHalf + k] << 16;
            hi.w[2 * k + 1] = l.w[kHalf + k] & 0xffff0000u;
        }
        lo.store(y + 2 * i * kBytes);
        hi.store(y + 2 * i * kBytes + kBytes);
    }
    __device__ __forceinline__ void scalar(int64_t e) const { Vec16<float>::store1(y, e, Vec16<bf16>::load1(x, e)); }
};

// f32 -> bf16: two packs of f32 produce one pack of bf16.
struct CastF32ToBf16Functor {
    template <int kBytes>
    struct Loaded {
        Words<kBytes> a, b;
    };
    const char* x;
    char* y;

    template <int kBytes>
    __device__ __forceinline__ Loaded<kBytes> load(int64_t i) const {
        return {Words<kBytes>::load(x + 2 * i * kBytes), Words<kBytes>::load(x + 2 * i * kBytes + kBytes)};
    }
    template <int kBytes>
    __device__ __forceinline__ void compute_store(int64_t i, const Loaded<kBytes>& l) const {
        Words<kBytes> o;
        constexpr int kHalf = Words<kBytes>::kCount / 2;
#pragma unroll
        for (int k = 0; k < kHalf; ++k) {
            o.w[k] = pack_bf16x2(__uint_as_float(l.a.w[2 * k]), __uint_as_float(l.a.w[2 * k + 1]));
            o.w[kHalf + k] = pack_bf16x2(__uint_as_float(l.b.w[2 * k]), __uint_as_float(l.b.w[2 * k + 1]));
        }
        o.store(y + i * kBytes);
    }
    __device__ __forceinline__ void scalar(int64_t e) const { Vec16<bf16>::store1(y, e, Vec16<float>::load1(x, e)); }
};

struct CopyFunctor {
    template <int kBytes>
    using Loaded = Words<kBytes>;
    const char* x;
    char* y;

    template <int kBytes>
    __device__ __forceinline__ Loaded<kBytes> load(int64_t i) const {
        return Words<kBytes>::load(x + i * kBytes);
    }
    template <int kBytes>
    __device__ __forceinline__ void compute_store(int64_t i, const Loaded<kBytes>& l) const {
        l.store(y + i * kBytes);
    }
    __device__ __forceinline__ void scalar(int64_t e) const {
        reinterpret_cast<unsigned char*>(y)[e] = reinterpret_cast<const unsigned char*>(x)[e];
    }
};

// Strided gather of a rank <= 8 view into dense storage; one thread per output element.
struct StridedParams {
    int64_t dims[8];
    int64_t strides[8];
    int rank;
};

template <typename E>
__global__ void __launch_bounds__(kThreads) strided_copy_kernel(const E* __restrict__ x, E* __restrict__ y,
                                                                StridedParams p, int64_t count) {
    grid_dependency_begin();
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t e = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; e < count; e += stride) {
        int64_t rem = e;
        int64_t offset = 0;
        for (int axis = p.rank - 1; axis >= 0; --axis) {
            const int64_t coord = rem % p.dims[axis];
            rem /= p.dims[axis];
            offset += coord * p.strides[axis];
        }
        y[e] = x[offset];
    }
}

// Two waves of resident blocks, or fewer when the work is small.
int64_t grid_blocks(int64_t work_items) {
    const int64_t per_sm = runtime::max_threads_per_sm() / kThreads;
    const int64_t waves = 2 * static_cast<int64_t>(runtime::sm_count()) * (per_sm > 0 ? per_sm : 1);
    const int64_t needed = runtime::ceil_div(work_items, kThreads);
    return needed < waves ? (needed > 0 ? needed : 1) : waves;
}

bool aligned32(const void* p) {
    return (reinterpret_cast<std::uintptr_t>(p) & 31u) == 0;
}

// Picks the widest pack every operand is aligned for: 32 bytes, 16 bytes, or none (scalar). `elems16` is the number
// of elements in 16 bytes of the functor's pack unit (32-byte packs hold twice as many).
template <typename Functor>
int launch_elementwise(const Functor& f, std::initializer_list<const void*> operands, int64_t elems16, int64_t count,
                       void* stream, const char* name) {
    bool a32 = true;
    bool a16 = true;
    for (const void* p : operands) {
        a32 = a32 && aligned32(p);
        a16 = a16 && runtime::aligned16(p);
    }
    const auto s = runtime::as_stream(stream);
    cudaError_t launch_err;
    if (a32) {
        const int64_t n_vec = count / (2 * elems16);
        const int64_t work = n_vec > 0 ? n_vec : count;
        launch_err = runtime::launch(elementwise_kernel<Functor, 32>, dim3(static_cast<unsigned>(grid_blocks(work))),
                                     dim3(kThreads), s, 1u, f, n_vec, 2 * elems16, count);
    } else {
        const int64_t n_vec = a16 ? count / elems16 : 0;
        const int64_t work = n_vec > 0 ? n_vec : count;
        launch_err = runtime::launch(elementwise_kernel<Functor, 16>, dim3(static_cast<unsigned>(grid_blocks(work))),
                                     dim3(kThreads), s, 1u, f, n_vec, elems16, count);
    }
    return runtime::launched(launch_err, name);
}

int check_common(cppinf_dtype dtype, int64_t count, const char* op) {
    CPPINF_REQUIRE(runtime::valid_dtype(dtype), CPPINF_ERR_INVALID_ARGUMENT,
                   std::string(op) + " received an unsupported dtype.");
    CPPINF_REQUIRE(count >= 0, CPPINF_ERR_INVALID_ARGUMENT, std::string(op) + " requires a non-negative count.");
    return CPPINF_OK;
}

template <BinaryOp op>
int binary_entry(cppinf_dtype dtype, const void* lhs, const void* rhs, void* out, int64_t count, void* stream,
                 const char* name) {
    if (const int st = check_common(dtype, count, name); st != CPPINF_OK) {
        return st;
    }
    if (count == 0) {
        return runtime::ok();
    }
    CPPINF_REQUIRE(lhs && rhs && out, CPPINF_ERR_INVALID_ARGUMENT, std::string(name) + " received a null pointer.");
    const auto* a = static_cast<const char*>(lhs);
    const auto* b = static_cast<const char*>(rhs);
    auto* o = static_cast<char*>(out);
    if (dtype == CPPINF_DTYPE_BF16) {
        return launch_elementwise(BinaryFunctor<bf16, op>{a, b, o}, {lhs, rhs, out}, 8, count, stream, name);
    }
    return launch_elementwise(BinaryFunctor<float, op>{a, b, o}, {lhs, rhs, out}, 4, count, stream, name);
}

}  // namespace
}  // namespace cppinf::device

using namespace cppinf::device;
namespace rt = cppinf::runtime;

extern "C" {

int cppinf_add(cppinf_dtype dtype, const void* lhs, const void* rhs, void* out, int64_t count, void* stream) {
    return binary_entry<BinaryOp::Add>(dtype, lhs, rhs, out, count, stream, "add");
}

int cppinf_mul(cppinf_dtype dtype, const void* lhs, const void* rhs, void* out, int64_t count, void* stream) {
    return binary_entry<BinaryOp::Mul>(dtype, lhs, rhs, out, count, stream, "mul");
}

int cppinf_silu(cppinf_dtype dtype, const void* x, void* y, int64_t count, void* stream) {
    if (const int st = check_common(dtype, count, "silu"); st != CPPINF_OK) {
        return st;
    }
    if (count == 0) {
        return rt::ok();
    }
    CPPINF_REQUIRE(x && y, CPPINF_ERR_INVALID_ARGUMENT, "silu received a null pointer.");
    const auto* xs = static_cast<const char*>(x);
    auto* ys = static_cast<char*>(y);
    if (dtype == CPPINF_DTYPE_BF16) {
        return launch_elementwise(SiluFunctor<bf16>{xs, ys}, {x, y}, 8, count, stream, "silu");
    }
    return launch_elementwise(SiluFunctor<float>{xs, ys}, {x, y}, 4, count, stream, "silu");
}

int cppinf_silu_mul(cppinf_dtype dtype, const void* gate, const void* up, void* out, int64_t count, void* stream) {
    if (const int st = check_common(dtype, count, "silu_mul"); st != CPPINF_OK) {
        return st;
    }
    if (count == 0) {
        return rt::ok();
    }
    CPPINF_REQUIRE(gate && up && out, CPPINF_ERR_INVALID_ARGUMENT, "silu_mul received a null pointer.");
    const auto* g = static_cast<const char*>(gate);
    const auto* u = static_cast<const char*>(up);
    auto* o = static_cast<char*>(out);
    if (dtype == CPPINF_DTYPE_BF16) {
        return launch_elementwise(SiluMulFunctor<bf16>{g, u, o}, {gate, up, out}, 8, count, stream, "silu_mul");
    }
    return launch_elementwise(SiluMulFunctor<float>{g, u, o}, {gate, up, out}, 4, count, stream, "silu_mul");
}

int cppinf_cast(cppinf_dtype src_dtype, const void* x, cppinf_dtype dst_dtype, void* y, int64_t count, void* stream) {
    CPPINF_REQUIRE(rt::valid_dtype(src_dtype) && rt::valid_dtype(dst_dtype), CPPINF_ERR_INVALID_ARGUMENT,
                   "cast received an unsupported dtype.");
    CPPINF_REQUIRE(count >= 0, CPPINF_ERR_INVALID_ARGUMENT, "cast requires a non-negative count.");
    if (count == 0) {
        return rt::ok();
    }
    CPPINF_REQUIRE(x && y, CPPINF_ERR_INVALID_ARGUMENT, "cast received a null pointer.");
    const auto* xs = static_cast<const char*>(x);
    auto* ys = static_cast<char*>(y);
    if (src_dtype == dst_dtype) {
        const int64_t bytes = count * static_cast<int64_t>(rt::dtype_size(src_dtype));
        return launch_elementwise(CopyFunctor{xs, ys}, {x, y}, 16, bytes, stream, "cast_copy");
    }
    // The pack unit is counted on the bf16 side: 16 bytes of bf16 are 8 elements.
    if (src_dtype == CPPINF_DTYPE_BF16) {
        return launch_elementwise(CastBf16ToF32Functor{xs, ys}, {x, y}, 8, count, stream, "cast_bf16_f32");
    }
    return launch_elementwise(CastF32ToBf16Functor{xs, ys}, {x, y}, 8, count, stream, "cast_f32_bf16");
}

int cppinf_strided_copy(cppinf_dtype dtype, const void* x, int64_t rank, const int64_t* dims, const int64_t* strides,
                        void* y, void* stream) {
    CPPINF_REQUIRE(rt::valid_dtype(dtype), CPPINF_ERR_INVALID_ARGUMENT, "strided_copy received an unsupported dtype.");
    CPPINF_REQUIRE(rank >= 0 && rank <= 8, CPPINF_ERR_UNSUPPORTED, "strided_copy supports rank 0 to 8.");
    CPPINF_REQUIRE(rank == 0 || (dims && strides), CPPINF_ERR_INVALID_ARGUMENT,
                   "strided_copy received a null dims or strides array.");
    StridedParams p{};
    p.rank = static_cast<int>(rank);
    int64_t count = 1;
    for (int64_t a = 0; a < rank; ++a) {
        CPPINF_REQUIRE(dims[a] >= 0, CPPINF_ERR_INVALID_ARGUMENT, "strided_copy dims must be non-negative.");
        CPPINF_REQUIRE(strides[a] >= 0, CPPINF_ERR_INVALID_ARGUMENT, "strided_copy strides must be non-negative.");
        p.dims[a] = dims[a];
        p.strides[a] = strides[a];
        count *= dims[a];
    }
    if (count == 0) {
        return rt::ok();
    }
    CPPINF_REQUIRE(x && y, CPPINF_ERR_INVALID_ARGUMENT, "strided_copy received a null pointer.");
    const auto blocks = static_cast<unsigned>(grid_blocks(count));
    cudaError_t launch_err;
    if (dtype == CPPINF_DTYPE_BF16) {
        launch_err = rt::launch(strided_copy_kernel<unsigned short>, dim3(blocks), dim3(kThreads),
                                rt::as_stream(stream), 1u, static_cast<const unsigned short*>(x),
                                static_cast<unsigned short*>(y), p, count);
    } else {
        launch_err = rt::launch(strided_copy_kernel<float>, dim3(blocks), dim3(kThreads), rt::as_stream(stream), 1u,
                                static_cast<const float*>(x), static_cast<float*>(y), p, count);
    }
    return rt::launched(launch_err, "strided_copy");
}

}  // extern "C"
