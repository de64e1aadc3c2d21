#ifndef SPECDECODE_CUDA_H
#define SPECDECODE_CUDA_H

/*
 * C ABI of libspecdecode_cuda.so: the paged INT8 KV-cache hot path on B200
 * (sm_100a).  The library is the device-side replacement for the reference
 * project's CPU quantizer library (native/include/specdecode/native.h) and for
 * the PyTorch ops its packed CUDA storage and unfused attention use
 * (src/specdecode/cuda_kv_cache.py).
 *
 * Conventions, kept from native/include/specdecode/native.h and
 * docs/native.md:41-56 of the reference:
 *   - every function returns an sdc_status_t; outputs go through caller-owned
 *     pointers; nothing returned is ever allocated by the library;
 *   - arguments are validated on the host before any launch or output write;
 *   - C++ exceptions never cross the boundary;
 *   - no fast-math anywhere.
 * Additions for device work:
 *   - device buffers are plain pointers into the current CUDA device's
 *     memory; `stream` is a cudaStream_t passed as uintptr_t (0 = legacy
 *     default stream); launches are asynchronous on that stream;
 *   - faults that only the kernel can see (a slot or block id outside the
 *     pool, a non-finite input, an invalid scale, a wait that gave up) are
 *     OR-ed into a caller-provided device status word (int32, SDC_FAULT_*
 *     bits) instead of trapping; the host reads it when it next synchronizes;
 *   - calls are thread-safe when callers use distinct streams, status words
 *     and workspaces.
 */

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__) || defined(__clang__)
#define SDC_API __attribute__((visibility("default")))
#else
#define SDC_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define SDC_ABI_VERSION UINT32_C(0x00020003)

/* Values 0-10 keep the meaning they have in the reference's sd_status_t
 * (native/include/specdecode/native.h:25-37). */
typedef enum sdc_status {
    SDC_STATUS_OK = 0,
    SDC_STATUS_NULL_ARGUMENT = 1,
    SDC_STATUS_INVALID_SIZE = 2,
    SDC_STATUS_NONFINITE_VALUE = 3,
    SDC_STATUS_NEGATIVE_PROBABILITY = 4,
    SDC_STATUS_ZERO_MASS = 5,
    SDC_STATUS_TOKEN_OUT_OF_RANGE = 6,
    SDC_STATUS_INVALID_UNIFORM = 7,
    SDC_STATUS_OVERFLOW = 8,
    SDC_STATUS_INTERNAL_ERROR = 9,
    SDC_STATUS_INVALID_SCALE = 10,
    SDC_STATUS_CUDA_ERROR = 11,
    SDC_STATUS_UNSUPPORTED = 12,
    SDC_STATUS_MISALIGNED = 13,
    SDC_STATUS_DEVICE_FAULT = 14,
    SDC_STATUS_INVALID_ARGUMENT = 15,
    SDC_STATUS_SCRATCH_EXCEEDED = 16
} sdc_status_t;

/* Bits a kernel ORs into the device status word. */
#define SDC_FAULT_NONFINITE_VALUE  0x01
#define SDC_FAULT_INVALID_SCALE    0x02
#define SDC_FAULT_SLOT_RANGE       0x04
#define SDC_FAULT_BLOCK_RANGE      0x08
#define SDC_FAULT_CONTEXT_RANGE    0x10
#define SDC_FAULT_WAIT_TIMEOUT     0x20
#define SDC_FAULT_TABLE_RANGE      0x40
/* Sampling kernels (the reference's status for the same input in brackets). */
#define SDC_FAULT_NEGATIVE_WEIGHT  0x80   /* a weight < 0, or a probability outside [0, 1] [4] */
#define SDC_FAULT_ZERO_MASS        0x100  /* a row whose weights sum to 0 [5] */
#define SDC_FAULT_TOKEN_RANGE      0x200  /* a proposed token outside the vocabulary [6] */
#define SDC_FAULT_INVALID_UNIFORM  0x400  /* a uniform outside [0, 1) [7] */
#define SDC_FAULT_PROPOSAL_COUNT   0x800  /* a proposal count outside [1, proposals] */
/* Device page allocator. */
#define SDC_FAULT_CAPACITY         0x1000 /* an append needs more free blocks than the pool has */

typedef enum sdc_dtype {
    SDC_DTYPE_F32 = 0,
    SDC_DTYPE_BF16 = 1,
    SDC_DTYPE_F16 = 2,
    SDC_DTYPE_F64 = 3
} sdc_dtype_t;

/*
 * The paged pool.  Codes are int8, scales float32, one scale per
 * (block, offset, layer, head) for keys and one for values.  Within a page a
 * (block, layer, head) holds block_size token rows of head_dim codes
 * back to back (token stride = head_dim) and block_size scales back to back
 * (token stride = 1); the other strides are free, in elements.  The library's
 * own allocation uses [block][layer][head][offset][dim]; the reference's
 * logical view [block][offset][layer][head][dim] is a permutation of it.
 */
typedef struct sdc_page_pool {
    int8_t* keys;
    int8_t* values;
    float* key_scales;
    float* value_scales;
    int64_t num_blocks;
    int64_t block_size;
    int64_t num_layers;
    int64_t num_heads;
    int64_t head_dim;
    int64_t code_block_stride;
    int64_t code_layer_stride;
    int64_t code_head_stride;
    int64_t scale_block_stride;
    int64_t scale_layer_stride;
    int64_t scale_head_stride;
} sdc_page_pool_t;

/*
 * Device block tables and lengths, plus a list of edits to apply.
 * entries: [num_entries][3] int32 (row, logical block, physical block; -1 clears)
 * lengths: [num_lengths][2] int32 (row, new context length)
 */
typedef struct sdc_table_edits {
    int32_t* block_tables;
    int64_t table_stride;
    int64_t table_rows;
    int32_t* context_lens;
    const int32_t* entries;
    int64_t num_entries;
    const int32_t* lengths;
    int64_t num_lengths;
} sdc_table_edits_t;

SDC_API uint32_t sdc_abi_version(void);
SDC_API const char* sdc_status_string(sdc_status_t status);

/*
 * Host-buffer drop-ins for the reference's per-vector quantizer, with the
 * reference's exact signatures and semantics:
 *   replaces sd_quantize_symmetric_int8_f64   (native/include/specdecode/native.h:93-98,
 *                                              native/src/native.cpp:275-319)
 *   replaces sd_dequantize_symmetric_int8_f64 (native/include/specdecode/native.h:101-106,
 *                                              native/src/native.cpp:321-353)
 * The arithmetic runs on the current CUDA device; inputs are copied in and
 * results copied back before return, and outputs are written only on success.
 */
SDC_API sdc_status_t sdc_quantize_symmetric_int8_f64(
    const double* values, size_t count, int8_t* output_values, double* output_scale);
SDC_API sdc_status_t sdc_dequantize_symmetric_int8_f64(
    const int8_t* values, size_t count, double scale, double* output_values);

/*
 * Quantize `rows` device vectors of `count` elements (row-major, dtype
 * `src_dtype`) with the reference rule; per-row status codes (sd_status_t
 * numbering) go to `row_status`.  Rows with a non-zero status are not written.
 * Batched form of the same per-vector rule (src/specdecode/kv_cache.py:130-146).
 */
SDC_API sdc_status_t sdc_quantize_rows(
    const void* source, int src_dtype, int64_t rows, int64_t count,
    int8_t* codes, float* scales, int32_t* row_status, uintptr_t stream);

/*
 * Kernel (a): fused quantize-and-append.  For every token i, every layer in
 * [layer_begin, layer_begin + num_src_layers) and every head, quantizes
 * keys[i][layer - layer_begin][head][:] and values[...] (dtype src_dtype,
 * element strides src_token_stride / src_layer_stride / src_head_stride, dim
 * contiguous) and writes codes + scale into physical slot slot_mapping[i]
 * (block = slot / block_size, offset = slot % block_size) with 16-byte stores.
 * Optional `edits` (may be NULL) are applied in the same launch.
 * Replaces: PagedKVCache.append_many's quantize+write (src/specdecode/kv_cache.py:298-336)
 * and CudaPagedKVCacheStorage's scatter upload (src/specdecode/cuda_kv_cache.py:343-348).
 * Requires head_dim % 16 == 0 and head_dim <= 512.
 */
SDC_API sdc_status_t sdc_quantize_append(
    const sdc_page_pool_t* pool, int64_t layer_begin, int64_t num_src_layers,
    const void* keys, const void* values, int src_dtype,
    int64_t num_tokens, int64_t src_token_stride, int64_t src_layer_stride,
    int64_t src_head_stride, const int64_t* slot_mapping, const sdc_table_edits_t* edits,
    int32_t* device_status, uintptr_t stream);

/*
 * Kernel (b): rollback.  Zeroes codes and scales of every layer and head in
 * the `num_clear` physical slots of `clear_slots`, then applies `edits`
 * (rewound block-table entries set to -1, new context lengths).
 * Replaces: PagedKVCache.truncate / rollback (src/specdecode/kv_cache.py:382-420)
 * and the stale-slot clearing of src/specdecode/cuda_kv_cache.py:336-342.
 */
SDC_API sdc_status_t sdc_rollback(
    const sdc_page_pool_t* pool, const int64_t* clear_slots, int64_t num_clear,
    const sdc_table_edits_t* edits, int32_t* device_status, uintptr_t stream);

/* Workspace bytes sdc_paged_verify_attention needs for this shape. */
SDC_API sdc_status_t sdc_paged_attention_workspace_size(
    int64_t batch, int64_t num_query_heads, int64_t num_kv_heads, int64_t head_dim,
    int64_t window, int64_t max_context_len, size_t* bytes);

/*
 * Kernel (c): fused paged verify/decode attention (split-K flash decoding).
 * query/out: [batch][num_query_heads][window][head_dim], dtype query_dtype
 * (bf16, f16 or f32), contiguous.  The window holds the last `window` cached
 * positions of each sequence; query head h reads KV head h / (Hq / Hkv); a
 * query at position p sees keys at positions <= p; softmax scale 1/sqrt(D).
 * block_tables: device int32 [batch][table_stride]; context_lens: device int32
 * [batch]; max_context_len: a host-side upper bound on every context length.
 * Replaces: submit_paged_attention's gather/dequantize/GQA/mask/SDPA
 * (src/specdecode/cuda_kv_cache.py:370-503, computation at :452-497) and the
 * CPU reconstruct path feeding attention (src/specdecode/hf_paged_cache.py:247-313).
 */
SDC_API sdc_status_t sdc_paged_verify_attention(
    const sdc_page_pool_t* pool, int64_t layer, const void* query, int query_dtype,
    int64_t batch, int64_t num_query_heads, int64_t window, const int32_t* block_tables,
    int64_t table_stride, const int32_t* context_lens, int64_t max_context_len, void* out,
    void* workspace, size_t workspace_bytes, int32_t* device_status, uintptr_t stream);

/*
 * sdc_paged_verify_attention for one rank of a KV-head split (the long-context
 * configuration: rank r of `world` holds KV heads [r Hkv/world, (r+1)
 * Hkv/world) of every page and the matching num_query_heads query heads),
 * with the all-gather of the outputs fused into the attention's own output
 * stores.  rank_outputs[i] (i < world) is rank i's gathered output
 * [batch, world * num_query_heads, window, head_dim] in the query dtype,
 * mapped into this process (sdc_peer_buffer_open for the other ranks');
 * the kernel that writes this rank's output rows stores each row into every
 * rank's buffer, at head offset rank * num_query_heads, over NVLink.
 * rank_flags[i] is rank i's array of `world` uint32 flag words.  After the
 * output launches, one more launch stores `epoch` into flag `rank` of every
 * rank (release, system scope) and waits until this rank's flags all read
 * `epoch` (acquire): when it ends, this rank's buffer holds every rank's rows.
 * A wait that runs past about nine seconds records SDC_FAULT_WAIT_TIMEOUT in
 * device_status and ends.  `epoch` must differ from the previous call's (a
 * per-call counter starting at 1; flag words start at 0).  Every rank must
 * make the same calls in the same order.  No counterpart in the reference,
 * which runs on one device; it replaces an all-gather collective after
 * sdc_paged_verify_attention.
 */
SDC_API sdc_status_t sdc_paged_verify_attention_gather(
    const sdc_page_pool_t* pool, int64_t layer, const void* query, int query_dtype,
    int64_t batch, int64_t num_query_heads, int64_t window, const int32_t* block_tables,
    int64_t table_stride, const int32_t* context_lens, int64_t max_context_len,
    void* const* rank_outputs, uint32_t* const* rank_flags, int32_t world, int32_t rank,
    uint32_t epoch, void* workspace, size_t workspace_bytes, int32_t* device_status,
    uintptr_t stream);

/* Device buffers other processes of the node can map (the gathered outputs
 * and flag words of sdc_paged_verify_attention_gather): allocate (zeroed) on
 * the current device, export an inter-process handle (SDC_PEER_HANDLE_BYTES
 * bytes), map another process's buffer from its handle, unmap, free. */
#define SDC_PEER_HANDLE_BYTES 64
SDC_API sdc_status_t sdc_peer_buffer_alloc(size_t bytes, void** ptr);
SDC_API sdc_status_t sdc_peer_buffer_free(void* ptr);
SDC_API sdc_status_t sdc_peer_buffer_export(void* ptr, void* handle, size_t handle_bytes);
SDC_API sdc_status_t sdc_peer_buffer_open(const void* handle, size_t handle_bytes, void** ptr);
SDC_API sdc_status_t sdc_peer_buffer_close(void* ptr);

/* Bytes of the library-owned scratch of sdc_paged_verify_attention_no_alloc. */
#define SDC_NO_ALLOC_SCRATCH_BYTES ((size_t)16 << 20)

/*
 * sdc_paged_verify_attention without a caller workspace, for callers that may
 * not allocate device memory (a serving loop whose memory another allocator
 * has reserved up front, a plugin host that hands over only its input and
 * output buffers, a callback that must not synchronize the device as
 * cudaMalloc / cudaFree can).  Same arguments, results and errors as
 * sdc_paged_verify_attention minus workspace / workspace_bytes; the workspace
 * is a SDC_NO_ALLOC_SCRATCH_BYTES device array that each GPU loading the
 * library holds until exit.  Shapes needing more (see
 * sdc_paged_attention_workspace_size) return SDC_STATUS_SCRATCH_EXCEEDED
 * before any launch.  Calls on one device share the array: calls that overlap
 * on the GPU race, so keep them on one stream.  The first call on a device
 * looks up the array's address with that device current; make it before any
 * stream capture.  That address is cached for the life of the process: do not
 * call this entry point on a device again after cudaDeviceReset.  No
 * counterpart in the reference.
 */
SDC_API sdc_status_t sdc_paged_verify_attention_no_alloc(
    const sdc_page_pool_t* pool, int64_t layer, const void* query, int query_dtype,
    int64_t batch, int64_t num_query_heads, int64_t window, const int32_t* block_tables,
    int64_t table_stride, const int32_t* context_lens, int64_t max_context_len, void* out,
    int32_t* device_status, uintptr_t stream);

/*
 * Test hook of kernel (c)'s bounded pipeline waits, for the launches that
 * follow in this process: every wait of the tensor-core item kernel gives up
 * after wait_limit_cycles SM cycles (<= 0: the default, about one second),
 * records SDC_FAULT_WAIT_TIMEOUT in device_status and winds its block down
 * (its copies and MMAs drained, tensor memory freed); stall = 1 makes the
 * softmax warps wait on a barrier that nothing completes, so that wait runs
 * out.  A timed-out launch writes no output rows.  Not for production use:
 * it changes every later launch until called again with (0, 0).  No
 * counterpart in the reference.
 */
SDC_API sdc_status_t sdc_test_attention_waits(int64_t wait_limit_cycles, int32_t stall);

/*
 * Gather and dequantize cached tokens: for every slot i and layer in
 * [layer_begin, layer_begin + num_layers) and head, writes code * scale to
 * out_keys / out_values at i*out_token_stride + (layer-layer_begin)*out_layer_stride
 * + head*out_head_stride (dim contiguous) in out_dtype.  f64 output is exact;
 * f32 is the correctly rounded product; bf16/f16 narrow through float32, as
 * torch.tensor does for Python floats.
 * Replaces: PagedKVCache.read_token / read_sequence dequantization
 * (src/specdecode/kv_cache.py:349-380) and the CPU reconstruct of
 * HuggingFacePagedCacheMirror.materialize_legacy_cache (src/specdecode/hf_paged_cache.py:247-313).
 */
SDC_API sdc_status_t sdc_gather_dequantize(
    const sdc_page_pool_t* pool, int64_t layer_begin, int64_t num_layers,
    const int64_t* slot_mapping, int64_t num_tokens, void* out_keys, void* out_values,
    int out_dtype, int64_t out_token_stride, int64_t out_layer_stride, int64_t out_head_stride,
    int32_t* device_status, uintptr_t stream);

/*
 * Device-resident acceptance and sampling (batched device forms of the
 * reference's sampling functions, native/include/specdecode/native.h:43-87,
 * native/src/native.cpp:84-273).
 *
 * Probability rows are device arrays of non-negative weights in dtype
 * SDC_DTYPE_F32 or SDC_DTYPE_F64, `vocab` (1 .. 2^21) weights per row, rows
 * `row_stride` elements apart; they need not be normalised.  Each function
 * validates its weights as the reference does (finite, non-negative, positive
 * sum), but on the device: a row that fails ORs the SDC_FAULT_* bit into
 * `device_status` and gets the marker output stated below instead of a
 * result.  Host-visible arguments (pointers, sizes, strides) are checked
 * before any launch.
 *
 * Arithmetic: sums are double-double (error below 2^-100 of the sum), the
 * per-row quotients double-double, so every decision (threshold < running
 * sum, uniform < probability) equals the reference's except for a draw
 * within about 1e-16 relative of the boundary, and every probability output
 * is within 2 ulp of the reference's extended-precision result.
 */

/* out[r][v] = weights[r][v] / sum(weights[r]), f64.  Replaces sd_normalize_f64
 * (native.h:43, native.cpp:84-102).  Faulted rows are not written. */
SDC_API sdc_status_t sdc_normalize_rows(
    const void* weights, int dtype, int64_t rows, int64_t vocab, int64_t row_stride,
    double* output, int64_t output_stride, int32_t* device_status, uintptr_t stream);

/* output_tokens[r] = the first v with uniforms[r] * sum(weights[r]) < weights[r][0] + ... +
 * weights[r][v], or vocab - 1 if there is none; -1 for a faulted row.
 * Replaces sd_sample_categorical_f64 (native.h:46-51, native.cpp:104-136). */
SDC_API sdc_status_t sdc_sample_categorical_rows(
    const void* weights, int dtype, int64_t rows, int64_t vocab, int64_t row_stride,
    const double* uniforms, int64_t* output_tokens, int32_t* device_status, uintptr_t stream);

/* out[r][v] = max(0, target[r][v] / sum(target[r]) - draft[r][v] / sum(draft[r])), or
 * target[r][v] / sum(target[r]) when those sum to at most 1e-15.  Faulted rows are
 * not written.  Replaces sd_residual_weights_f64 (native.h:57-62, native.cpp:138-177). */
SDC_API sdc_status_t sdc_residual_weights_rows(
    const void* target, const void* draft, int dtype, int64_t rows, int64_t vocab,
    int64_t target_stride, int64_t draft_stride, double* output, int64_t output_stride,
    int32_t* device_status, uintptr_t stream);

/* out[r] = 1 if draft[r][t] == 0, else min(1, (target[r][t] / sum(target[r])) /
 * (draft[r][t] / sum(draft[r]))) with t = proposed_tokens[r]; NaN for a faulted row.
 * Replaces sd_acceptance_probabilities_f64 (native.h:68-75, native.cpp:179-232). */
SDC_API sdc_status_t sdc_acceptance_probabilities_rows(
    const void* target, const void* draft, int dtype, int64_t rows, int64_t vocab,
    int64_t target_stride, int64_t draft_stride, const int64_t* proposed_tokens,
    double* output_probabilities, int32_t* device_status, uintptr_t stream);

/* For each of `sequences` rows of `proposals` acceptance probabilities and
 * uniforms (both `row_stride` apart): output_accepted[s] = the first i with
 * !(uniforms[s][i] < probabilities[s][i]), or `proposals` if none; -1 for a
 * faulted row.  Replaces sd_first_rejection_f64 (native.h:81-87,
 * native.cpp:234-273), whose two outputs are both this index. */
SDC_API sdc_status_t sdc_first_rejection_rows(
    const double* acceptance_probabilities, const double* uniforms, int64_t sequences,
    int64_t proposals, int64_t row_stride, int64_t* output_accepted, int32_t* device_status,
    uintptr_t stream);

/*
 * One verification round of speculative sampling for a batch: sequence s
 * proposed tokens proposed_tokens[s][0 .. n_s), drawn from the draft rows
 * (s, 0 .. n_s); the target rows (s, 0 .. n_s] are the target's distributions
 * at the same positions plus the bonus position.  Row (s, i) of the target
 * starts at target_rows + s * target_sequence_stride + i * target_row_stride
 * elements, likewise for the draft.
 *
 * uniforms[s][0 .. n_s] hold the sequence's draws in the reference decoder's
 * order (src/specdecode/decoder.py:206-257, docs/native.md:58-73): draw i
 * decides proposal i (accepted iff draw < its acceptance probability); after
 * a rejection at j, draw j + 1 samples the correction from the residual
 * weights of row j; after a full acceptance, draw n_s samples the bonus
 * token from target row n_s.  A caller holding one uniform stream per
 * sequence therefore consumes exactly output_accepted[s] + 2 draws after a
 * rejection and n_s + 1 (or n_s, without a bonus) after a full acceptance.
 *
 * n_s = proposal_counts[s] (1 .. proposals), or `proposals` when
 * proposal_counts is NULL.  bonus_allowed[s] == 0 means a full acceptance
 * ends the round without a bonus draw (the reference stops at an accepted
 * end-of-sequence token or at the token budget); NULL allows every bonus.
 *
 * Outputs: output_probabilities[s][i] (stride `proposals`) for i < n_s;
 * output_accepted[s] = accepted proposals; output_tokens[s] = the correction
 * or bonus token, or -1 after a full acceptance without a bonus.  A faulted
 * sequence gets -1 in both.  Two launches: one block per (sequence,
 * proposal) for the acceptance probabilities, then one per sequence for the
 * decision and the sample.  row_sums (optional, NULL allowed) is device
 * scratch of sequences * proposals * 4 doubles through which the first
 * launch hands its row sums to the second, which then reads only the
 * rejected rows' residual instead of summing both rows again.
 */
typedef struct sdc_verify_batch {
    const void* target_rows;
    const void* draft_rows;
    int dtype;
    int64_t sequences;
    int64_t proposals;
    int64_t vocab;
    int64_t target_sequence_stride;
    int64_t target_row_stride;
    int64_t draft_sequence_stride;
    int64_t draft_row_stride;
    const int64_t* proposed_tokens;  /* [sequences][token_stride] */
    int64_t token_stride;
    const double* uniforms;          /* [sequences][uniform_stride], uniform_stride > proposals */
    int64_t uniform_stride;
    const int64_t* proposal_counts;  /* [sequences] or NULL */
    const uint8_t* bonus_allowed;    /* [sequences] or NULL */
} sdc_verify_batch_t;

SDC_API sdc_status_t sdc_speculative_verify(
    const sdc_verify_batch_t* batch, double* output_probabilities, int64_t* output_accepted,
    int64_t* output_tokens, double* row_sums, int32_t* device_status, uintptr_t stream);

/*
 * Device-resident page allocation: the reference's lowest-free-block-first
 * allocator (the min-heap of src/specdecode/kv_cache.py:220-221, :327, :418,
 * whose order the block tables follow exactly) held on the device, so append
 * and rollback plan their blocks without a host round trip; plus prefix
 * sharing -- a forked sequence shares its source's blocks, reference-counted
 * -- with copy-on-write of a shared, partly filled last block on the next
 * append.  The reference defers sharing (docs/kv-cache.md:105-108); the
 * sharing semantics are this library's own.
 *
 * State, all device memory the caller owns: free_bits (bit h % 32 of word
 * h / 32 set = heap id h free; bits past num_blocks clear), refcount per
 * physical block (0 when free), high_water per physical block (rows
 * [0, high_water) of the page may be non-zero; 0 initially), block_order
 * (heap id -> physical block) and
 * heap_of (its inverse), the block tables (-1 = no block) and the context
 * lengths.  Rows passed to one call must be distinct.  A call that fails
 * validation on the device sets a fault bit and changes nothing.
 */
typedef struct sdc_page_allocator {
    uint32_t* free_bits;
    int32_t* refcount;
    int32_t* high_water;
    const int32_t* block_order;
    const int32_t* heap_of;
    int32_t* block_tables;
    int32_t* context_lens;
    int64_t num_blocks;
    int64_t block_size;
    int64_t table_rows;
    int64_t table_stride;
} sdc_page_allocator_t;

/* Workspace bytes of sdc_pages_append for this many sequences (1 .. 1024) and tokens. */
SDC_API sdc_status_t sdc_pages_append_workspace_size(
    int64_t sequences, int64_t total_tokens, int64_t block_size, size_t* bytes);

/*
 * Reserves room for counts[s] more tokens in table row rows[s] (device int32
 * arrays of `sequences` entries, total_tokens = their sum) and writes the
 * physical slot of every new token to slot_mapping (int64, sequence order
 * then token order), ready for sdc_quantize_append.  New blocks are the
 * lowest free heap ids, taken in sequence order; a shared partly filled last
 * block is first copied (rows below the old length; the rest zeroed) into a
 * private block.  Faults: SDC_FAULT_CAPACITY (the pool is short of blocks),
 * SDC_FAULT_TABLE_RANGE (a row out of range, a table row too short, counts
 * not summing to total_tokens); a faulted call changes no state and sets
 * every slot to -1, which sdc_quantize_append refuses to write.
 * Replaces PagedKVCache.append_many's block allocation (src/specdecode/kv_cache.py:298-336).
 */
SDC_API sdc_status_t sdc_pages_append(
    const sdc_page_allocator_t* allocator, const sdc_page_pool_t* pool, const int32_t* rows,
    const int32_t* counts, int64_t sequences, int64_t total_tokens, int64_t* slot_mapping,
    void* workspace, size_t workspace_bytes, int32_t* device_status, uintptr_t stream);

/*
 * Truncates table row rows[s] to new_lengths[s] tokens (device int32
 * arrays; at most max_removed tokens removed from any row): blocks past the
 * new length drop a reference and return to the free set when none is left,
 * their written rows zeroed; in a partly kept last page held by this row
 * alone the rows past the new length are zeroed (codes and scales of every
 * layer and head), as the reference's rollback leaves released slots.
 * Faults: SDC_FAULT_CONTEXT_RANGE (a new length above the old one or more
 * than max_removed below it; that row is left unchanged).
 * Replaces PagedKVCache.truncate / rollback (src/specdecode/kv_cache.py:382-420).
 */
SDC_API sdc_status_t sdc_pages_truncate(
    const sdc_page_allocator_t* allocator, const sdc_page_pool_t* pool, const int32_t* rows,
    const int32_t* new_lengths, int64_t sequences, int64_t max_removed, int32_t* device_status,
    uintptr_t stream);

/*
 * Prefix sharing: destination_rows[i] (empty) takes every block and the
 * length of source_rows[i]; each shared block gains a reference.  No
 * counterpart in the reference.
 */
SDC_API sdc_status_t sdc_pages_fork(
    const sdc_page_allocator_t* allocator, const int32_t* source_rows, const int32_t* destination_rows,
    int64_t pairs, int32_t* device_status, uintptr_t stream);

#ifdef __cplusplus
}
#endif

#endif
