// Internal interface between the attention entry point and its kernels.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "sdc_common.cuh"

namespace sdc {

// Destinations one call may write its output rows to: the caller's buffer,
// or, with the KV-head all-gather, every rank's gathered output.
constexpr int kMaxOutputs = 8;

struct AttnArgs {
    Pool pool;
    int64_t layer;
    const void* query;
    int query_dtype;
    // Element (b, query head h, window row w, d) of this call goes to
    // outs[i] + b * out_seq_stride + ((out_head0 + h) * window + w) * head_dim + d
    // in every destination i < num_outs.
    void* outs[kMaxOutputs];
    int32_t num_outs;
    int64_t out_seq_stride;  // elements between sequences of a destination
    int64_t out_head0;       // first query head of this call in a destination
    int64_t batch;
    int64_t query_heads;
    int64_t kv_heads;
    int64_t group;   // query heads per KV head
    int64_t window;  // query rows per head (speculative window)
    int64_t rows;    // group * window: query rows served per KV head
    int64_t head_dim;
    const int32_t* block_tables;
    int64_t table_stride;
    const int32_t* context_lens;
    int64_t chunk;       // key positions per work item
    int64_t max_chunks;  // ceil(max_context_len / chunk)
    float* part_o;       // [batch * kv_heads][max_chunks][rows][head_dim]
    float* part_ml;      // [batch * kv_heads][max_chunks][rows][2]
    int32_t* status;
    float qk_scale;      // log2(e) / sqrt(head_dim)
};

// Element offset, in every destination, of the first output row of KV head
// h of sequence b (its group x window rows follow contiguously).
__host__ __device__ __forceinline__ int64_t out_rows_offset(const AttnArgs& a, int64_t b, int64_t h) {
    return b * a.out_seq_stride + (a.out_head0 + h * a.group) * a.window * a.head_dim;
}

bool simt_supports(int64_t head_dim, int64_t rows);
sdc_status_t launch_attention_simt(const AttnArgs& a, cudaStream_t stream);
// Merges the per-chunk partials into the output (used by both item kernels).
// `programmatic`: launched as a programmatic dependent of the item kernel
// (it waits for that grid's results with griddepcontrol.wait).
sdc_status_t launch_attention_combine(const AttnArgs& a, cudaStream_t stream, bool programmatic = false);
// Whether max_chunks * rows chunk weights fit the combine's shared buffer.
bool combine_fits(int64_t max_chunks, int64_t rows);

namespace tc {
// Shapes the tensor-core item kernel serves: head_dim 128 and at most 64
// query rows per KV head (more than 32 are split over two items).
bool shape_supported(int64_t head_dim, int64_t rows);
// Pool layouts it can read with TMA (page rows of 128 bytes, aligned scales).
bool supports(const AttnArgs& a);
int64_t chunk_for(int64_t batch, int64_t kv_heads, int64_t max_context_len, int64_t rows);
size_t extra_workspace(int64_t batch, int64_t kv_heads, int64_t max_chunks, int64_t rows);
sdc_status_t launch(const AttnArgs& a, void* extra, cudaStream_t stream);
// Cycles a bounded wait may take before it gives up (about a second unless
// sdc_test_attention_waits set a shorter limit).
long long wait_limit_cycles();
}  // namespace tc

}  // namespace sdc
