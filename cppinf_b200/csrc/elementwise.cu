// Streaming elementwise kernels: ops::add / ops::mul (src/ops/elementwise_ops.cpp:44-52), ops::silu
// (src/ops/nn_ops.cpp:68-72), ops::cast (src/ops/tensor_ops.cpp:138-143), the fused silu*up product of the Qwen MLP
// (src/nn/qwen_mlp.cpp:65-66) and the strided gather that materialises non-contiguous views.
//
// Every kernel is HBM-bound (<= 1 flop per byte). Layout: dense arrays, 16-byte vectors, a grid of one full wave of
// resident blocks (SM count x blocks per SM) striding over the vectors with kUnroll independent vectors per thread
// per iteration so each thread keeps several 16-byte loads in flight. A misaligned operand or a ragged tail runs the
// scalar path of the same kernel.
#include "common.cuh"
#include "runtime.h"

namespace cppinf::device {
namespace {

constexpr int kThreads = 256;
constexpr int kUnroll = 4;

enum class BinaryOp { Add, Mul };

template <BinaryOp op>
__device__ __forceinline__ float apply_binary(float a, float b) {
    if constexpr (op == BinaryOp::Add) {
        return a + b;
    } else {
        return a * b;
    }
}

// x / (1 + exp(-x)), oneDNN eltwise_swish with alpha = 1 as ops::silu configures it (src/ops/nn_ops.cpp:70-71).
__device__ __forceinline__ float silu_f32(float x) {
    return x / (1.0f + expf(-x));
}

// Generic grid-stride driver. `Functor::vec(i)` handles 16-byte vector i, `Functor::scalar(i)` element i.
template <typename Functor>
__global__ void __launch_bounds__(kThreads) elementwise_kernel(Functor f, int64_t n_vec, int64_t vec_elems,
                                                               int64_t count) {
    grid_dependency_begin();
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    int64_t i = tid;
    for (; i + (kUnroll - 1) * stride < n_vec; i += kUnroll * stride) {
        typename Functor::Loaded loaded[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            loaded[u] = f.load(i + u * stride);
        }
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            f.compute_store(i + u * stride, loaded[u]);
        }
    }
    for (; i < n_vec; i += stride) {
        f.compute_store(i, f.load(i));
    }
    // Scalar tail (or the whole array when the vector path is off).
    for (int64_t e = n_vec * vec_elems + tid; e < count; e += stride) {
        f.scalar(e);
    }
}

template <typename T, BinaryOp op>
struct BinaryFunctor {
    using V = Vec16<T>;
    struct Loaded {
        uint4 a, b;
    };
    const uint4* lhs;
    const uint4* rhs;
    uint4* out;
    const void* lhs_s;
    const void* rhs_s;
    void* out_s;

    __device__ __forceinline__ Loaded load(int64_t i) const { return {ld_stream(lhs + i), ld_stream(rhs + i)}; }
    __device__ __forceinline__ void compute_store(int64_t i, const Loaded& l) const {
        float a[V::kVec], b[V::kVec];
        V::unpack(l.a, a);
        V::unpack(l.b, b);
#pragma unroll
        for (int j = 0; j < V::kVec; ++j) {
            a[j] = apply_binary<op>(a[j], b[j]);
        }
        st_stream(out + i, V::pack(a));
    }
    __device__ __forceinline__ void scalar(int64_t e) const {
        V::store1(out_s, e, apply_binary<op>(V::load1(lhs_s, e), V::load1(rhs_s, e)));
    }
};

template <typename T>
struct SiluFunctor {
    using V = Vec16<T>;
    using Loaded = uint4;
    const uint4* x;
    uint4* y;
    const void* x_s;
    void* y_s;

    __device__ __forceinline__ Loaded load(int64_t i) const { return ld_stream(x + i); }
    __device__ __forceinline__ void compute_store(int64_t i, const Loaded& l) const {
        float a[V::kVec];
        V::unpack(l, a);
#pragma unroll
        for (int j = 0; j < V::kVec; ++j) {
            a[j] = silu_f32(a[j]);
        }
        st_stream(y + i, V::pack(a));
    }
    __device__ __forceinline__ void scalar(int64_t e) const { V::store1(y_s, e, silu_f32(V::load1(x_s, e))); }
};

// out = T(T(silu(gate)) * up): the reference rounds the silu tensor to T before ops::mul reads it.
template <typename T>
struct SiluMulFunctor {
    using V = Vec16<T>;
    struct Loaded {
        uint4 g, u;
    };
    const uint4* gate;
    const uint4* up;
    uint4* out;
    const void* gate_s;
    const void* up_s;
    void* out_s;

    __device__ __forceinline__ Loaded load(int64_t i) const { return {ld_stream(gate + i), ld_stream(up + i)}; }
    __device__ __forceinline__ void compute_store(int64_t i, const Loaded& l) const {
        float g[V::kVec], u[V::kVec];
        V::unpack(l.g, g);
        V::unpack(l.u, u);
#pragma unroll
        for (int j = 0; j < V::kVec; ++j) {
            g[j] = V::quantize(silu_f32(g[j])) * u[j];
        }
        st_stream(out + i, V::pack(g));
    }
    __device__ __forceinline__ void scalar(int64_t e) const {
        const float s = V::quantize(silu_f32(V::load1(gate_s, e)));
        V::store1(out_s, e, s * V::load1(up_s, e));
    }
};

// bf16 -> f32: one 16-byte load of 8 bf16 produces two 16-byte stores.
struct CastBf16ToF32Functor {
    using Loaded = uint4;
    const uint4* x;
    uint4* y;
    const void* x_s;
    void* y_s;

    __device__ __forceinline__ Loaded load(int64_t i) const { return ld_stream(x + i); }
    __device__ __forceinline__ void compute_store(int64_t i, const Loaded& l) const {
        st_stream(y + 2 * i, make_uint4(l.x << 16, l.x & 0xffff0000u, l.y << 16, l.y & 0xffff0000u));
        st_stream(y + 2 * i + 1, make_uint4(l.z << 16, l.z & 0xffff0000u, l.w << 16, l.w & 0xffff0000u));
    }
    __device__ __forceinline__ void scalar(int64_t e) const { Vec16<float>::store1(y_s, e, Vec16<bf16>::load1(x_s, e)); }
};

// f32 -> bf16: two 16-byte loads of 4 f32 produce one 16-byte store.
struct CastF32ToBf16Functor {
    struct Loaded {
        uint4 a, b;
    };
    const uint4* x;
    uint4* y;
    const void* x_s;
    void* y_s;

    __device__ __forceinline__ Loaded load(int64_t i) const { return {ld_stream(x + 2 * i), ld_stream(x + 2 * i + 1)}; }
    __device__ __forceinline__ void compute_store(int64_t i, const Loaded& l) const {
        st_stream(y + i, make_uint4(pack_bf16x2(__uint_as_float(l.a.x), __uint_as_float(l.a.y)),
                                    pack_bf16x2(__uint_as_float(l.a.z), __uint_as_float(l.a.w)),
                                    pack_bf16x2(__uint_as_float(l.b.x), __uint_as_float(l.b.y)),
                                    pack_bf16x2(__uint_as_float(l.b.z), __uint_as_float(l.b.w))));
    }
    __device__ __forceinline__ void scalar(int64_t e) const { Vec16<bf16>::store1(y_s, e, Vec16<float>::load1(x_s, e)); }
};

struct CopyFunctor {
    using Loaded = uint4;
    const uint4* x;
    uint4* y;
    const unsigned char* x_s;
    unsigned char* y_s;

    __device__ __forceinline__ Loaded load(int64_t i) const { return ld_stream(x + i); }
    __device__ __forceinline__ void compute_store(int64_t i, const Loaded& l) const { st_stream(y + i, l); }
    __device__ __forceinline__ void scalar(int64_t e) const { y_s[e] = x_s[e]; }
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

int64_t wave_blocks(int64_t work_items) {
    const int64_t per_sm = runtime::max_threads_per_sm() / kThreads;
    const int64_t wave = static_cast<int64_t>(runtime::sm_count()) * (per_sm > 0 ? per_sm : 1);
    const int64_t needed = runtime::ceil_div(work_items, kThreads);
    return needed < wave ? (needed > 0 ? needed : 1) : wave;
}

template <typename Functor>
int launch_elementwise(const Functor& f, bool vector_ok, int64_t vec_elems, int64_t count, void* stream,
                       const char* name) {
    const int64_t n_vec = vector_ok ? count / vec_elems : 0;
    const int64_t work = n_vec > 0 ? n_vec : count;
    const cudaError_t launch_err = ::cppinf::runtime::launch(elementwise_kernel<Functor>, dim3(static_cast<unsigned>(wave_blocks(work))), dim3(kThreads), runtime::as_stream(stream), 1u, 
        f, n_vec, vec_elems, count);
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
    const bool vec = runtime::aligned16(lhs) && runtime::aligned16(rhs) && runtime::aligned16(out);
    if (dtype == CPPINF_DTYPE_BF16) {
        BinaryFunctor<bf16, op> f{static_cast<const uint4*>(lhs), static_cast<const uint4*>(rhs),
                                  static_cast<uint4*>(out), lhs, rhs, out};
        return launch_elementwise(f, vec, 8, count, stream, name);
    }
    BinaryFunctor<float, op> f{static_cast<const uint4*>(lhs), static_cast<const uint4*>(rhs), static_cast<uint4*>(out),
                               lhs, rhs, out};
    return launch_elementwise(f, vec, 4, count, stream, name);
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
    const bool vec = rt::aligned16(x) && rt::aligned16(y);
    if (dtype == CPPINF_DTYPE_BF16) {
        SiluFunctor<bf16> f{static_cast<const uint4*>(x), static_cast<uint4*>(y), x, y};
        return launch_elementwise(f, vec, 8, count, stream, "silu");
    }
    SiluFunctor<float> f{static_cast<const uint4*>(x), static_cast<uint4*>(y), x, y};
    return launch_elementwise(f, vec, 4, count, stream, "silu");
}

int cppinf_silu_mul(cppinf_dtype dtype, const void* gate, const void* up, void* out, int64_t count, void* stream) {
    if (const int st = check_common(dtype, count, "silu_mul"); st != CPPINF_OK) {
        return st;
    }
    if (count == 0) {
        return rt::ok();
    }
    CPPINF_REQUIRE(gate && up && out, CPPINF_ERR_INVALID_ARGUMENT, "silu_mul received a null pointer.");
    const bool vec = rt::aligned16(gate) && rt::aligned16(up) && rt::aligned16(out);
    if (dtype == CPPINF_DTYPE_BF16) {
        SiluMulFunctor<bf16> f{static_cast<const uint4*>(gate), static_cast<const uint4*>(up), static_cast<uint4*>(out),
                               gate, up, out};
        return launch_elementwise(f, vec, 8, count, stream, "silu_mul");
    }
    SiluMulFunctor<float> f{static_cast<const uint4*>(gate), static_cast<const uint4*>(up), static_cast<uint4*>(out),
                            gate, up, out};
    return launch_elementwise(f, vec, 4, count, stream, "silu_mul");
}

int cppinf_cast(cppinf_dtype src_dtype, const void* x, cppinf_dtype dst_dtype, void* y, int64_t count, void* stream) {
    CPPINF_REQUIRE(rt::valid_dtype(src_dtype) && rt::valid_dtype(dst_dtype), CPPINF_ERR_INVALID_ARGUMENT,
                   "cast received an unsupported dtype.");
    CPPINF_REQUIRE(count >= 0, CPPINF_ERR_INVALID_ARGUMENT, "cast requires a non-negative count.");
    if (count == 0) {
        return rt::ok();
    }
    CPPINF_REQUIRE(x && y, CPPINF_ERR_INVALID_ARGUMENT, "cast received a null pointer.");
    const bool vec = rt::aligned16(x) && rt::aligned16(y);
    if (src_dtype == dst_dtype) {
        const int64_t bytes = count * static_cast<int64_t>(rt::dtype_size(src_dtype));
        CopyFunctor f{static_cast<const uint4*>(x), static_cast<uint4*>(y), static_cast<const unsigned char*>(x),
                      static_cast<unsigned char*>(y)};
        return launch_elementwise(f, vec, 16, bytes, stream, "cast_copy");
    }
    if (src_dtype == CPPINF_DTYPE_BF16) {
        CastBf16ToF32Functor f{static_cast<const uint4*>(x), static_cast<uint4*>(y), x, y};
        return launch_elementwise(f, vec, 8, count, stream, "cast_bf16_f32");
    }
    CastF32ToBf16Functor f{static_cast<const uint4*>(x), static_cast<uint4*>(y), x, y};
    return launch_elementwise(f, vec, 8, count, stream, "cast_f32_bf16");
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
    const auto blocks = static_cast<unsigned>(wave_blocks(count));
    cudaError_t launch_err;
    if (dtype == CPPINF_DTYPE_BF16) {
        launch_err = ::cppinf::runtime::launch(strided_copy_kernel<unsigned short>, dim3(blocks), dim3(kThreads), rt::as_stream(stream), 1u, 
            static_cast<const unsigned short*>(x), static_cast<unsigned short*>(y), p, count);
    } else {
        launch_err = ::cppinf::runtime::launch(strided_copy_kernel<float>, dim3(blocks), dim3(kThreads), rt::as_stream(stream), 1u, static_cast<const float*>(x),
                                                                                   static_cast<float*>(y), p, count);
    }
    return rt::launched(launch_err, "strided_copy");
}

}  // extern "C"
