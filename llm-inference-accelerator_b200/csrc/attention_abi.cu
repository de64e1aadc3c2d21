// C ABI entry points of kernel (c): argument validation, work planning and
// workspace layout, then the launch.

#include <cmath>
#include <cstring>

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

// Where a call's output rows go (see AttnArgs).
struct Outputs {
    void* ptrs[kMaxOutputs] = {};
    int32_t count = 0;
    int64_t seq_stride = 0;
    int64_t head0 = 0;
};

sdc_status_t run_attention(const sdc_page_pool_t* pool, int64_t layer, const void* query, int query_dtype,
                           int64_t batch, int64_t num_query_heads, int64_t window, const int32_t* block_tables,
                           int64_t table_stride, const int32_t* context_lens, int64_t max_context_len,
                           const Outputs& o, void* workspace, size_t workspace_bytes, int32_t* device_status,
                           cudaStream_t stream) {
    sdc_status_t rc = validate_pool(pool);
    if (rc != SDC_STATUS_OK) return rc;
    if (query == nullptr || block_tables == nullptr || context_lens == nullptr || device_status == nullptr ||
        workspace == nullptr) {
        return SDC_STATUS_NULL_ARGUMENT;
    }
    if (layer < 0 || layer >= pool->num_layers) return SDC_STATUS_INVALID_SIZE;
    if (table_stride < 1) return SDC_STATUS_INVALID_SIZE;
    if (query_dtype != SDC_DTYPE_BF16 && query_dtype != SDC_DTYPE_F16 && query_dtype != SDC_DTYPE_F32) {
        return SDC_STATUS_UNSUPPORTED;
    }
    if (!aligned16(query) || !aligned16(workspace)) return SDC_STATUS_MISALIGNED;
    for (int i = 0; i < o.count; ++i) {
        if (!aligned16(o.ptrs[i])) return SDC_STATUS_MISALIGNED;
    }
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
    for (int i = 0; i < kMaxOutputs; ++i) a.outs[i] = i < o.count ? o.ptrs[i] : nullptr;
    a.num_outs = o.count;
    a.out_seq_stride = o.seq_stride;
    a.out_head0 = o.head0;
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
        return tc::launch(a, extra, stream);
    }
    return launch_attention_simt(a, stream);
}

// Completion of the KV-head all-gather: thread p < world stores `epoch` into
// rank p's flag word for this rank (a release at system scope, after the
// output launches' stores, which each made visible system-wide), then waits
// for its own flag word of rank p to read `epoch` (acquire).  A wait gives up
// after a bounded number of cycles and records SDC_FAULT_WAIT_TIMEOUT.
struct SignalArgs {
    uint32_t* flags[kMaxOutputs];
    int32_t world;
    int32_t rank;
    uint32_t epoch;
    long long wait_limit;
    int32_t* status;
};

__global__ void __launch_bounds__(32) gather_signal_kernel(SignalArgs s) {
    // launched as a programmatic dependent of the output launch: this waits
    // until that grid has finished and its stores are performed
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int p = threadIdx.x;
    if (p >= s.world) return;
    __threadfence_system();
    uint32_t* to = s.flags[p] + s.rank;
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(to), "r"(s.epoch) : "memory");
    const uint32_t* mine = s.flags[s.rank] + p;
    const long long t0 = clock64();
    while (true) {
        uint32_t v;
        asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(mine) : "memory");
        if (v == s.epoch) break;
        if (clock64() - t0 > s.wait_limit) {
            atomicOr(s.status, SDC_FAULT_WAIT_TIMEOUT);
            break;
        }
        __nanosleep(64);
    }
}

sdc_status_t launch_gather_signal(uint32_t* const* flags, int32_t world, int32_t rank, uint32_t epoch,
                                  int32_t* status, cudaStream_t stream) {
    SignalArgs s;
    for (int i = 0; i < kMaxOutputs; ++i) s.flags[i] = i < world ? flags[i] : nullptr;
    s.world = world;
    s.rank = rank;
    s.epoch = epoch;
    // ranks reach this point at different times (each rank's own host work
    // comes first), so the default bound is eight times the pipeline
    // waits' (about 9 s); a shorter test limit applies as set
    const long long limit = tc::wait_limit_cycles();
    s.wait_limit = limit >= (1ll << 31) ? (1ll << 34) : limit;
    s.status = status;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1);
    cfg.blockDim = dim3(32);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, gather_signal_kernel, s) != cudaSuccess) return SDC_STATUS_CUDA_ERROR;
    return launch_status();
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
        if (out == nullptr) return SDC_STATUS_NULL_ARGUMENT;
        Outputs o;
        o.ptrs[0] = out;
        o.count = 1;
        o.seq_stride = num_query_heads * window * (pool != nullptr ? pool->head_dim : 0);
        o.head0 = 0;
        return run_attention(pool, layer, query, query_dtype, batch, num_query_heads, window, block_tables,
                             table_stride, context_lens, max_context_len, o, workspace, workspace_bytes,
                             device_status, as_stream(stream));
    } catch (...) {
        return SDC_STATUS_INTERNAL_ERROR;
    }
}

SDC_API sdc_status_t sdc_paged_verify_attention_gather(
    const sdc_page_pool_t* pool, int64_t layer, const void* query, int query_dtype, int64_t batch,
    int64_t num_query_heads, int64_t window, const int32_t* block_tables, int64_t table_stride,
    const int32_t* context_lens, int64_t max_context_len, void* const* rank_outputs, uint32_t* const* rank_flags,
    int32_t world, int32_t rank, uint32_t epoch, void* workspace, size_t workspace_bytes, int32_t* device_status,
    uintptr_t stream) {
    try {
        if (rank_outputs == nullptr || rank_flags == nullptr || device_status == nullptr) {
            return SDC_STATUS_NULL_ARGUMENT;
        }
        if (world < 1 || world > kMaxOutputs || rank < 0 || rank >= world || epoch == 0) {
            return SDC_STATUS_INVALID_ARGUMENT;
        }
        Outputs o;
        for (int i = 0; i < world; ++i) {
            if (rank_outputs[i] == nullptr || rank_flags[i] == nullptr) return SDC_STATUS_NULL_ARGUMENT;
            if (!aligned16(rank_outputs[i]) || (reinterpret_cast<uintptr_t>(rank_flags[i]) & 3u)) {
                return SDC_STATUS_MISALIGNED;
            }
            o.ptrs[i] = rank_outputs[i];
        }
        o.count = world;
        o.seq_stride = static_cast<int64_t>(world) * num_query_heads * window * (pool != nullptr ? pool->head_dim : 0);
        o.head0 = static_cast<int64_t>(rank) * num_query_heads;
        cudaStream_t st = as_stream(stream);
        const sdc_status_t rc = run_attention(pool, layer, query, query_dtype, batch, num_query_heads, window,
                                              block_tables, table_stride, context_lens, max_context_len, o,
                                              workspace, workspace_bytes, device_status, st);
        if (rc != SDC_STATUS_OK) return rc;
        return launch_gather_signal(rank_flags, world, rank, epoch, device_status, st);
    } catch (...) {
        return SDC_STATUS_INTERNAL_ERROR;
    }
}

SDC_API sdc_status_t sdc_peer_buffer_alloc(size_t bytes, void** ptr) {
    try {
        if (ptr == nullptr) return SDC_STATUS_NULL_ARGUMENT;
        *ptr = nullptr;
        if (bytes == 0) return SDC_STATUS_INVALID_SIZE;
        void* p = nullptr;
        if (cudaMalloc(&p, bytes) != cudaSuccess) return SDC_STATUS_CUDA_ERROR;
        if (cudaMemset(p, 0, bytes) != cudaSuccess) {
            cudaFree(p);
            return SDC_STATUS_CUDA_ERROR;
        }
        *ptr = p;
        return SDC_STATUS_OK;
    } catch (...) {
        return SDC_STATUS_INTERNAL_ERROR;
    }
}

SDC_API sdc_status_t sdc_peer_buffer_free(void* ptr) {
    if (ptr == nullptr) return SDC_STATUS_OK;
    return cudaFree(ptr) == cudaSuccess ? SDC_STATUS_OK : SDC_STATUS_CUDA_ERROR;
}

SDC_API sdc_status_t sdc_peer_buffer_export(void* ptr, void* handle, size_t handle_bytes) {
    try {
        if (ptr == nullptr || handle == nullptr) return SDC_STATUS_NULL_ARGUMENT;
        if (handle_bytes < sizeof(cudaIpcMemHandle_t)) return SDC_STATUS_INVALID_SIZE;
        cudaIpcMemHandle_t h;
        if (cudaIpcGetMemHandle(&h, ptr) != cudaSuccess) return SDC_STATUS_CUDA_ERROR;
        std::memcpy(handle, &h, sizeof(h));
        return SDC_STATUS_OK;
    } catch (...) {
        return SDC_STATUS_INTERNAL_ERROR;
    }
}

SDC_API sdc_status_t sdc_peer_buffer_open(const void* handle, size_t handle_bytes, void** ptr) {
    try {
        if (handle == nullptr || ptr == nullptr) return SDC_STATUS_NULL_ARGUMENT;
        *ptr = nullptr;
        if (handle_bytes < sizeof(cudaIpcMemHandle_t)) return SDC_STATUS_INVALID_SIZE;
        cudaIpcMemHandle_t h;
        std::memcpy(&h, handle, sizeof(h));
        void* p = nullptr;
        if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) return SDC_STATUS_CUDA_ERROR;
        *ptr = p;
        return SDC_STATUS_OK;
    } catch (...) {
        return SDC_STATUS_INTERNAL_ERROR;
    }
}

SDC_API sdc_status_t sdc_peer_buffer_close(void* ptr) {
    if (ptr == nullptr) return SDC_STATUS_OK;
    return cudaIpcCloseMemHandle(ptr) == cudaSuccess ? SDC_STATUS_OK : SDC_STATUS_CUDA_ERROR;
}

}  // extern "C"
