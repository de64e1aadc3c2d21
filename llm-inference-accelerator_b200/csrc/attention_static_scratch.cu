// sdc_paged_verify_attention_no_alloc: paged verify attention with its
// scratch in a fixed device array that the library owns, for callers that
// must not allocate device memory themselves.
//
// Who needs it: code that runs where a cudaMalloc (or an allocating library
// call such as torch.empty) is not allowed or not safe, for example a
// serving loop whose memory is fully reserved up front by another allocator,
// a plugin host that hands the plugin only its input and output buffers, or
// a callback that must not synchronize the device (cudaMalloc / cudaFree can).
// Those callers still pass their own inputs and outputs; only the workspace
// (split-K partial sums, the work list and the quantized query images) comes
// from here.
//
// The scratch is SDC_NO_ALLOC_SCRATCH_BYTES (16 MiB) of device memory that
// every GPU which loads this library keeps until the process exits.  Shapes
// whose workspace is larger are rejected with SDC_STATUS_SCRATCH_EXCEEDED
// before anything is launched.  Nothing in it has to start at zero: the
// kernels write every workspace byte they read within the same call, exactly
// as with the caller-provided workspace of sdc_paged_verify_attention.
//
// All calls on a device share the one array and it keeps the last call's
// contents, so two calls whose kernels overlap on the GPU (on different
// streams, or from different threads) race on it; order such calls on one
// stream.  The first call on each device looks up the array's device
// address (cudaGetSymbolAddress, with that device current) and caches it;
// make that first call before any stream capture.  The cached address is
// never refreshed, so after cudaDeviceReset (or anything else that destroys
// and recreates the device's primary context) this entry point must not be
// called again on that device in the same process.

#include <mutex>

#include "host_common.h"

namespace {

constexpr size_t kScratchBytes = SDC_NO_ALLOC_SCRATCH_BYTES;

static __device__ __align__(256) unsigned char g_attention_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_setup_mutex;
void* g_scratch_address[kMaxDevices] = {};

// Device address of the scratch array on the current device.  Host code
// cannot use the symbol itself: on the host it names a stand-in variable, not
// device memory.
sdc_status_t scratch_on_current_device(void** address) {
    int device = 0;
    if (cudaGetDevice(&device) != cudaSuccess) return SDC_STATUS_CUDA_ERROR;
    if (device < 0 || device >= kMaxDevices) return SDC_STATUS_UNSUPPORTED;
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    if (g_scratch_address[device] == nullptr) {
        void* ptr = nullptr;
        if (cudaGetSymbolAddress(&ptr, g_attention_scratch) != cudaSuccess || ptr == nullptr) {
            return SDC_STATUS_CUDA_ERROR;
        }
        g_scratch_address[device] = ptr;
    }
    *address = g_scratch_address[device];
    return SDC_STATUS_OK;
}

}  // namespace

extern "C" {

SDC_API sdc_status_t sdc_paged_verify_attention_no_alloc(const sdc_page_pool_t* pool, int64_t layer,
                                                         const void* query, int query_dtype, int64_t batch,
                                                         int64_t num_query_heads, int64_t window,
                                                         const int32_t* block_tables, int64_t table_stride,
                                                         const int32_t* context_lens, int64_t max_context_len,
                                                         void* out, int32_t* device_status, uintptr_t stream) {
    try {
        if (pool == nullptr) return SDC_STATUS_NULL_ARGUMENT;
        size_t need = 0;
        sdc_status_t rc = sdc_paged_attention_workspace_size(batch, num_query_heads, pool->num_heads,
                                                             pool->head_dim, window, max_context_len, &need);
        if (rc != SDC_STATUS_OK) return rc;
        if (need > kScratchBytes) return SDC_STATUS_SCRATCH_EXCEEDED;
        void* scratch = nullptr;
        rc = scratch_on_current_device(&scratch);
        if (rc != SDC_STATUS_OK) return rc;
        return sdc_paged_verify_attention(pool, layer, query, query_dtype, batch, num_query_heads, window,
                                          block_tables, table_stride, context_lens, max_context_len, out, scratch,
                                          kScratchBytes, device_status, stream);
    } catch (...) {
        return SDC_STATUS_INTERNAL_ERROR;
    }
}

}  // extern "C"
