/*
 * Link stubs for the oneDNN C API entry points that the reference's inline dnnl.hpp wrappers reference. TEST
 * INFRASTRUCTURE ONLY (part of the oracle/_ref build of the reference sources).
 *
 * No oneDNN library exists in this environment (the reference fetches oneDNN v3.11 at configure time). Every stub
 * reports dnnl_unimplemented, so a reference function that really needs a oneDNN primitive (rms_norm's
 * reduction, softmax_last_dim, matmul, transposes) throws dnnl::error instead of computing anything; the functions
 * the oracle calls (scaled causal softmax loops, RoPE, argmax-free helpers) never reach these stubs.
 */
#include <oneapi/dnnl/dnnl.h>

dnnl_status_t dnnl_engine_destroy(dnnl_engine_t engine) {
    (void)engine;
    return dnnl_unimplemented;
}

dnnl_status_t dnnl_matmul_primitive_desc_create(dnnl_primitive_desc_t* primitive_desc, dnnl_engine_t engine,
                                                const_dnnl_memory_desc_t src_desc,
                                                const_dnnl_memory_desc_t weights_desc,
                                                const_dnnl_memory_desc_t bias_desc,
                                                const_dnnl_memory_desc_t dst_desc, const_dnnl_primitive_attr_t attr) {
    (void)primitive_desc, (void)engine, (void)src_desc, (void)weights_desc, (void)bias_desc, (void)dst_desc;
    (void)attr;
    return dnnl_unimplemented;
}

dnnl_status_t dnnl_memory_desc_clone(dnnl_memory_desc_t* memory_desc, const_dnnl_memory_desc_t existing) {
    (void)memory_desc, (void)existing;
    return dnnl_unimplemented;
}

dnnl_status_t dnnl_memory_desc_create_with_strides(dnnl_memory_desc_t* memory_desc, int ndims, const dnnl_dims_t dims,
                                                   dnnl_data_type_t data_type, const dnnl_dims_t strides) {
    (void)memory_desc, (void)ndims, (void)dims, (void)data_type, (void)strides;
    return dnnl_unimplemented;
}

dnnl_status_t dnnl_memory_desc_destroy(dnnl_memory_desc_t memory_desc) {
    (void)memory_desc;
    return dnnl_unimplemented;
}

dnnl_status_t dnnl_memory_get_engine(const_dnnl_memory_t memory, dnnl_engine_t* engine) {
    (void)memory, (void)engine;
    return dnnl_unimplemented;
}

dnnl_status_t dnnl_memory_get_memory_desc(const_dnnl_memory_t memory, const_dnnl_memory_desc_t* memory_desc) {
    (void)memory, (void)memory_desc;
    return dnnl_unimplemented;
}

dnnl_status_t dnnl_primitive_attr_create(dnnl_primitive_attr_t* attr) {
    (void)attr;
    return dnnl_unimplemented;
}

dnnl_status_t dnnl_primitive_attr_destroy(dnnl_primitive_attr_t attr) {
    (void)attr;
    return dnnl_unimplemented;
}

dnnl_status_t dnnl_primitive_create(dnnl_primitive_t* primitive, const_dnnl_primitive_desc_t primitive_desc) {
    (void)primitive, (void)primitive_desc;
    return dnnl_unimplemented;
}

dnnl_status_t dnnl_primitive_desc_destroy(dnnl_primitive_desc_t primitive_desc) {
    (void)primitive_desc;
    return dnnl_unimplemented;
}

dnnl_status_t dnnl_primitive_destroy(dnnl_primitive_t primitive) {
    (void)primitive;
    return dnnl_unimplemented;
}

dnnl_status_t dnnl_primitive_execute(const_dnnl_primitive_t primitive, dnnl_stream_t stream, int nargs,
                                     const dnnl_exec_arg_t* args) {
    (void)primitive, (void)stream, (void)nargs, (void)args;
    return dnnl_unimplemented;
}

dnnl_status_t dnnl_reduction_primitive_desc_create(dnnl_primitive_desc_t* primitive_desc, dnnl_engine_t engine,
                                                   dnnl_alg_kind_t alg_kind, const_dnnl_memory_desc_t src_desc,
                                                   const_dnnl_memory_desc_t dst_desc, float p, float eps,
                                                   const_dnnl_primitive_attr_t attr) {
    (void)primitive_desc, (void)engine, (void)alg_kind, (void)src_desc, (void)dst_desc, (void)p, (void)eps;
    (void)attr;
    return dnnl_unimplemented;
}

dnnl_status_t dnnl_reorder_primitive_desc_create(dnnl_primitive_desc_t* reorder_primitive_desc,
                                                 const_dnnl_memory_desc_t src_desc, dnnl_engine_t src_engine,
                                                 const_dnnl_memory_desc_t dst_desc, dnnl_engine_t dst_engine,
                                                 const_dnnl_primitive_attr_t attr) {
    (void)reorder_primitive_desc, (void)src_desc, (void)src_engine, (void)dst_desc, (void)dst_engine, (void)attr;
    return dnnl_unimplemented;
}

dnnl_status_t dnnl_softmax_forward_primitive_desc_create(dnnl_primitive_desc_t* primitive_desc, dnnl_engine_t engine,
                                                         dnnl_prop_kind_t prop_kind, dnnl_alg_kind_t alg_kind,
                                                         const_dnnl_memory_desc_t src_desc,
                                                         const_dnnl_memory_desc_t dst_desc, int softmax_axis,
                                                         const_dnnl_primitive_attr_t attr) {
    (void)primitive_desc, (void)engine, (void)prop_kind, (void)alg_kind, (void)src_desc, (void)dst_desc;
    (void)softmax_axis, (void)attr;
    return dnnl_unimplemented;
}

dnnl_status_t dnnl_stream_create(dnnl_stream_t* stream, dnnl_engine_t engine, unsigned flags) {
    (void)stream, (void)engine, (void)flags;
    return dnnl_unimplemented;
}

dnnl_status_t dnnl_stream_destroy(dnnl_stream_t stream) {
    (void)stream;
    return dnnl_unimplemented;
}

dnnl_status_t dnnl_stream_wait(dnnl_stream_t stream) {
    (void)stream;
    return dnnl_unimplemented;
}
