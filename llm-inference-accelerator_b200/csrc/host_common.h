// Host-side validation and launch helpers shared by the C ABI entry points.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "sdc_common.cuh"
#include "specdecode_cuda.h"

namespace sdc {

inline cudaStream_t as_stream(uintptr_t stream) { return reinterpret_cast<cudaStream_t>(stream); }

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

// Streaming multiprocessors of the current device, queried once per device.
inline int device_sms() {
    static int counts[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    if (counts[dev] <= 0) {
        int sms = 0;
        if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0) sms = 148;
        counts[dev] = sms;
    }
    return counts[dev];
}

inline int dtype_size(int dtype) {
    switch (dtype) {
        case SDC_DTYPE_F32: return 4;
        case SDC_DTYPE_BF16: return 2;
        case SDC_DTYPE_F16: return 2;
        case SDC_DTYPE_F64: return 8;
        default: return 0;
    }
}

// Lanes that handle one head vector: one lane per 16 elements, rounded up to
// a power of two so vector groups tile the warp.
inline int lanes_per_vector(int64_t head_dim) {
    const int64_t chunks = head_dim / 16;
    int lanes = 1;
    while (lanes < chunks) lanes <<= 1;
    return lanes;
}

// Checks a pool descriptor: positive geometry, non-null pointers, 16-byte
// aligned code rows (head_dim % 16 == 0, strides multiples of 16 bytes) and
// 4-byte aligned scales, and that the largest index stays inside int64.
inline sdc_status_t validate_pool(const sdc_page_pool_t* pool) {
    if (pool == nullptr) return SDC_STATUS_NULL_ARGUMENT;
    if (pool->keys == nullptr || pool->values == nullptr || pool->key_scales == nullptr ||
        pool->value_scales == nullptr) {
        return SDC_STATUS_NULL_ARGUMENT;
    }
    if (pool->num_blocks < 1 || pool->block_size < 1 || pool->num_layers < 1 ||
        pool->num_heads < 1 || pool->head_dim < 1) {
        return SDC_STATUS_INVALID_SIZE;
    }
    if (pool->head_dim % 16 != 0 || pool->head_dim > 512) return SDC_STATUS_UNSUPPORTED;
    if (pool->code_block_stride < 1 || pool->code_layer_stride < 1 || pool->code_head_stride < 1 ||
        pool->scale_block_stride < 1 || pool->scale_layer_stride < 1 || pool->scale_head_stride < 1) {
        return SDC_STATUS_INVALID_SIZE;
    }
    if (pool->code_block_stride % 16 || pool->code_layer_stride % 16 || pool->code_head_stride % 16) {
        return SDC_STATUS_MISALIGNED;
    }
    if (!aligned16(pool->keys) || !aligned16(pool->values)) return SDC_STATUS_MISALIGNED;
    if ((reinterpret_cast<uintptr_t>(pool->key_scales) & 3u) ||
        (reinterpret_cast<uintptr_t>(pool->value_scales) & 3u)) {
        return SDC_STATUS_MISALIGNED;
    }
    return SDC_STATUS_OK;
}

inline Pool to_pool(const sdc_page_pool_t* p) {
    Pool q;
    q.keys = p->keys;
    q.values = p->values;
    q.key_scales = p->key_scales;
    q.value_scales = p->value_scales;
    q.num_blocks = p->num_blocks;
    q.block_size = p->block_size;
    q.num_layers = p->num_layers;
    q.num_heads = p->num_heads;
    q.head_dim = p->head_dim;
    q.cbs = p->code_block_stride;
    q.cls = p->code_layer_stride;
    q.chs = p->code_head_stride;
    q.sbs = p->scale_block_stride;
    q.sls = p->scale_layer_stride;
    q.shs = p->scale_head_stride;
    return q;
}

inline sdc_status_t validate_edits(const sdc_table_edits_t* e, TableEdits* out) {
    *out = TableEdits{nullptr, 0, 0, nullptr, nullptr, 0, nullptr, 0};
    if (e == nullptr) return SDC_STATUS_OK;
    if (e->num_entries < 0 || e->num_lengths < 0) return SDC_STATUS_INVALID_SIZE;
    if (e->num_entries > 0 && (e->block_tables == nullptr || e->entries == nullptr)) {
        return SDC_STATUS_NULL_ARGUMENT;
    }
    if (e->num_lengths > 0 && (e->context_lens == nullptr || e->lengths == nullptr)) {
        return SDC_STATUS_NULL_ARGUMENT;
    }
    if ((e->num_entries > 0 || e->num_lengths > 0) && (e->table_rows < 1 || e->table_stride < 1)) {
        return SDC_STATUS_INVALID_SIZE;
    }
    *out = TableEdits{e->block_tables, e->table_stride, e->table_rows, e->context_lens,
                      e->entries,      e->num_entries,  e->lengths,    e->num_lengths};
    return SDC_STATUS_OK;
}

inline sdc_status_t launch_status() {
    const cudaError_t err = cudaGetLastError();
    return err == cudaSuccess ? SDC_STATUS_OK : SDC_STATUS_CUDA_ERROR;
}

}  // namespace sdc
