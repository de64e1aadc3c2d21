// C ABI entry points of kernel (c): argument validation, work planning and
// workspace layout, then the launch.

#include <cmath>

#include "host_common.h"
#include "paged_attention.h"

namespace sdc {
namespace {

constexpr int64_t kSimtChunk = 512;

struct Plan {
    int64_t rows;
    int64_t chunk;
    int64_t max_chunks;
    bool tensor_cores;  // shape served by the tcgen05 item kernel
    size_t part_o_bytes;
    size_t part_ml_bytes;
    size_t extra_bytes;
    size_t total;
};

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Work planning depends on the shape only, so the workspace sized here fits
// whichever item kernel the pool layout selects at launch.
sdc_status_t make_plan(int64_t batch, int64_t hq, int64_t hkv, int64_t d, int64_t window, int64_t max_ctx,
                       Plan* p) {
    if (batch < 1 || hq < 1 || hkv < 1 || d < 1 || window < 1 || max_ctx < 1) return SDC_STATUS_INVALID_SIZE;
    if (hq % hkv) return SDC_STATUS_INVALID_ARGUMENT;
    if (window > max_ctx) return SDC_STATUS_INVALID_SIZE;
    p->rows = (hq / hkv) * window;
    if (!simt_supports(d, p->rows)) return SDC_STATUS_UNSUPPORTED;
    p->tensor_cores = tc::shape_supported(d, p->rows);
    p->chunk = p->tensor_cores ? tc::chunk_for(batch, hkv, max_ctx, p->rows) : kSimtChunk;
    p->max_chunks = ceil_div(max_ctx, p->chunk);
    if (!combine_fits(p->max_chunks, p->rows)) return SDC_STATUS_UNSUPPORTED;
    const double items = static_cast<double>(batch) * hkv * p->max_chunks;
    if (items * p->rows * (d + 2) * 4.0 > 9.0e18) return SDC_STATUS_OVERFLOW;
    p->part_o_bytes = align_up(static_cast<size_t>(batch * hkv * p->max_chunks * p->rows * d) * 4, 256);
    p->part_ml_bytes = align_up(static_cast<size_t>(batch * hkv * p->max_chunks * p->rows * 2) * 4, 256);
    p->extra_bytes = p->tensor_cores ? align_up(tc::extra_workspace(batch, hkv, p->max_chunks, p->rows), 256) : 0;
    p->total = p->part_o_bytes + p->part_ml_bytes + p->extra_bytes;
    return SDC_STATUS_OK;
}

}  // namespace
}  // namespace sdc

using namespace sdc;

extern "C" {

SDC_API sdc_status_t sdc_paged_attention_workspace_size(int64_t batch, int64_t num_query_heads,
                                                        int64_t num_kv_heads, int64_t head_dim, int64_t window,
                                                        int64_t max_context_len, size_t* bytes) {
    try {
        if (bytes == nullptr) return SDC_STATUS_NULL_ARGUMENT;
        Plan p;
        const sdc_status_t rc =
            make_plan(batch, num_query_heads, num_kv_heads, head_dim, window, max_context_len, &p);
        if (rc != SDC_STATUS_OK) return rc;
        *bytes = p.total;
        return SDC_STATUS_OK;
    } catch (...) {
        return SDC_STATUS_INTERNAL_ERROR;
    }
}

SDC_API sdc_status_t sdc_paged_verify_attention(const sdc_page_pool_t* pool, int64_t layer, const void* query,
                                                int query_dtype, int64_t batch, int64_t num_query_heads,
                                                int64_t window, const int32_t* block_tables, int64_t table_stride,
                                                const int32_t* context_lens, int64_t max_context_len, void* out,
                                                void* workspace, size_t workspace_bytes, int32_t* device_status,
                                                uintptr_t stream) {
    try {
        sdc_status_t rc = validate_pool(pool);
        if (rc != SDC_STATUS_OK) return rc;
        if (query == nullptr || out == nullptr || block_tables == nullptr || context_lens == nullptr ||
            device_status == nullptr || workspace == nullptr) {
            return SDC_STATUS_NULL_ARGUMENT;
        }
        if (layer < 0 || layer >= pool->num_layers) return SDC_STATUS_INVALID_SIZE;
        if (table_stride < 1) return SDC_STATUS_INVALID_SIZE;
        if (query_dtype != SDC_DTYPE_BF16 && query_dtype != SDC_DTYPE_F16 && query_dtype != SDC_DTYPE_F32) {
            return SDC_STATUS_UNSUPPORTED;
        }
        if (!aligned16(query) || !aligned16(out) || !aligned16(workspace)) return SDC_STATUS_MISALIGNED;
        Plan p;
        rc = make_plan(batch, num_query_heads, pool->num_heads, pool->head_dim, window, max_context_len, &p);
        if (rc != SDC_STATUS_OK) return rc;
        if (workspace_bytes < p.total) return SDC_STATUS_INVALID_SIZE;
        if (p.max_chunks > 65535 || batch * pool->num_heads > 65535) return SDC_STATUS_UNSUPPORTED;

        AttnArgs a;
        a.pool = to_pool(pool);
        a.layer = layer;
        a.query = query;
        a.query_dtype = query_dtype;
        a.out = out;
        a.batch = batch;
        a.query_heads = num_query_heads;
        a.kv_heads = pool->num_heads;
        a.group = num_query_heads / pool->num_heads;
        a.window = window;
        a.rows = p.rows;
        a.head_dim = pool->head_dim;
        a.block_tables = block_tables;
        a.table_stride = table_stride;
        a.context_lens = context_lens;
        a.chunk = p.chunk;
        a.max_chunks = p.max_chunks;
        a.part_o = static_cast<float*>(workspace);
        a.part_ml = reinterpret_cast<float*>(static_cast<char*>(workspace) + p.part_o_bytes);
        a.status = device_status;
        a.qk_scale = static_cast<float>(1.4426950408889634 / std::sqrt(static_cast<double>(pool->head_dim)));
        if (p.tensor_cores && tc::supports(a)) {
            void* extra = static_cast<char*>(workspace) + p.part_o_bytes + p.part_ml_bytes;
            return tc::launch(a, extra, as_stream(stream));
        }
        return launch_attention_simt(a, as_stream(stream));
    } catch (...) {
        return SDC_STATUS_INTERNAL_ERROR;
    }
}

}  // extern "C"
