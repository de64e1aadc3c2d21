// Device-resident page allocation: the reference's lowest-free-block-first
// allocator (the min-heap of src/specdecode/kv_cache.py:220-221, :327, :418)
// kept on the device as a free bitmap over heap ids, so an append or a
// rollback plans its blocks without a host round trip; plus prefix sharing
// (a forked sequence shares its source's blocks, reference-counted) with
// copy-on-write of a shared, partly filled last block on the next append.
// The reference defers sharing (docs/kv-cache.md:105-108); its semantics here
// are this file's own.
//
// State (sdc_page_allocator_t): free_bits (bit h of word h / 32 set = heap id
// h free), refcount per physical block, block_order (heap id -> physical
// block) and heap_of (its inverse), the block tables and context lengths.
//
// Launch shapes: planning runs in one 1024-thread block (one thread per
// sequence, at most 1024 sequences a call; the free bitmap is split into one
// run of words per thread and the lowest free ids found by a block-wide scan
// of per-thread popcounts).  Page copies and slot zeroing run on a grid.

#include <algorithm>
#include <cub/block/block_reduce.cuh>
#include <cub/block/block_scan.cuh>

#include "host_common.h"

namespace sdc {
namespace {

constexpr int kPlanThreads = 1024;
constexpr int kCopyThreads = 128;

struct Alloc {
    uint32_t* free_bits;
    int32_t* refcount;
    int32_t* high_water;  // per physical block: rows [0, high_water) may be non-zero
    const int32_t* block_order;
    const int32_t* heap_of;
    int32_t* tables;
    int32_t* lens;
    int64_t num_blocks, block_size, rows, stride;
};

__device__ __forceinline__ int64_t blocks_for(int64_t tokens, int64_t bs) { return (tokens + bs - 1) / bs; }

struct AppendPlanArgs {
    Alloc a;
    const int32_t* rows;
    const int32_t* counts;
    int32_t sequences;
    int64_t total_tokens;
    int64_t* slots;     // [total_tokens]
    int32_t* copies;    // [sequences][4]: old block, new block, rows kept, unused
    int32_t* picked;    // [picked_cap] heap ids in allocation order
    int64_t picked_cap;
    int32_t* status;
};

// One block: validates the call, reserves every new block (the lowest free
// heap ids, in sequence order, each sequence's copy-on-write block first and
// then its new logical blocks in order -- the order in which the reference
// pops its heap), writes the tables, lengths and reference counts, and the
// slot of every appended token.  A call that fails validation changes
// nothing.
//
// Copy-on-write: a sequence whose partly filled last block is shared
// (reference count above 1) reserves one block for a private copy.  The
// decision is taken with an atomic decrement of the shared block's count, so
// when every holder of a block appends in the same call the last of them
// keeps the block in place; its reserved copy block goes back to the free set.
__global__ void __launch_bounds__(kPlanThreads) append_plan_kernel(AppendPlanArgs p) {
    using Scan = cub::BlockScan<int64_t, kPlanThreads>;
    using Reduce = cub::BlockReduce<int64_t, kPlanThreads>;
    __shared__ union {
        typename Scan::TempStorage scan;
        typename Reduce::TempStorage reduce;
    } tmp;
    __shared__ int64_t tok_base[kPlanThreads + 1];
    __shared__ int32_t old_len[kPlanThreads];
    __shared__ int64_t s_total_blocks, s_total_tokens, s_free;
    __shared__ int s_faults;
    const Alloc& a = p.a;
    const int tid = threadIdx.x;
    if (tid == 0) s_faults = 0;
    if (tid < p.sequences) p.copies[static_cast<int64_t>(tid) * 4] = -1;  // no copy unless decided below
    __syncthreads();

    int faults = 0;
    int64_t need = 0, count = 0;
    int32_t row = -1, cow = 0;
    if (tid < p.sequences) {
        row = p.rows[tid];
        count = p.counts[tid];
        if (row < 0 || row >= a.rows || count < 0) {
            faults |= SDC_FAULT_TABLE_RANGE;
        } else {
            const int64_t old = a.lens[row];
            const int64_t now = old + count;
            if (blocks_for(now, a.block_size) > a.stride) faults |= SDC_FAULT_TABLE_RANGE;
            if (!faults && count > 0 && old % a.block_size != 0) {
                const int32_t phys = a.tables[row * a.stride + old / a.block_size];
                if (phys < 0 || phys >= a.num_blocks) faults |= SDC_FAULT_BLOCK_RANGE;
                else if (a.refcount[phys] > 1) cow = 1;
            }
            need = blocks_for(now, a.block_size) - blocks_for(old, a.block_size) + cow;
            old_len[tid] = static_cast<int32_t>(old);
        }
    }
    if (faults) atomicOr(&s_faults, faults);
    int64_t blk_base, total_blocks;
    Scan(tmp.scan).ExclusiveSum(need, blk_base, total_blocks);
    __syncthreads();
    int64_t tok, total_tokens;
    Scan(tmp.scan).ExclusiveSum(count, tok, total_tokens);
    tok_base[tid] = tok;
    if (tid == 0) {
        s_total_blocks = total_blocks;
        s_total_tokens = total_tokens;
    }
    __syncthreads();

    // free blocks: a run of bitmap words per thread
    const int64_t words = (a.num_blocks + 31) / 32;
    const int64_t per = (words + kPlanThreads - 1) / kPlanThreads;
    const int64_t w0 = tid * per;
    const int64_t w1 = min(words, w0 + per);
    int64_t mine = 0;
    for (int64_t w = w0; w < w1; ++w) mine += __popc(a.free_bits[w]);
    const int64_t free_total = Reduce(tmp.reduce).Sum(mine);
    if (tid == 0) s_free = free_total;
    __syncthreads();
    if (tid == 0) {
        int f = s_faults;
        if (s_total_tokens != p.total_tokens) f |= SDC_FAULT_TABLE_RANGE;
        if (s_total_blocks > p.picked_cap) f |= SDC_FAULT_TABLE_RANGE;
        if (!f && s_total_blocks > s_free) f |= SDC_FAULT_CAPACITY;
        s_faults = f;
        if (f) report_fault(p.status, f);
    }
    __syncthreads();
    if (s_faults) {
        // no slot for any token: the append that follows skips every write
        for (int64_t i = tid; i < p.total_tokens; i += kPlanThreads) p.slots[i] = -1;
        return;
    }
    total_blocks = s_total_blocks;

    // the lowest `total_blocks` free heap ids, in increasing order
    int64_t rank;
    Scan(tmp.scan).ExclusiveSum(mine, rank);
    for (int64_t w = w0; w < w1 && rank < total_blocks; ++w) {
        uint32_t bits = a.free_bits[w];
        uint32_t taken = 0;
        while (bits != 0 && rank < total_blocks) {
            const int b = __ffs(bits) - 1;
            bits &= bits - 1;
            taken |= 1u << b;
            p.picked[rank++] = static_cast<int32_t>(w * 32 + b);
        }
        a.free_bits[w] &= ~taken;
    }
    __syncthreads();

    if (tid < p.sequences) {
        int64_t r = blk_base;
        const int64_t old = old_len[tid];
        const int64_t first_new = blocks_for(old, a.block_size);
        const int64_t last_new = blocks_for(old + count, a.block_size);
        int32_t* table = a.tables + row * a.stride;
        int32_t* copy = p.copies + static_cast<int64_t>(tid) * 4;
        if (cow) {
            const int32_t heap = p.picked[r++];
            const int32_t shared = table[old / a.block_size];
            if (atomicSub(a.refcount + shared, 1) > 1) {
                const int32_t fresh = a.block_order[heap];
                table[old / a.block_size] = fresh;
                a.refcount[fresh] = 1;
                a.high_water[fresh] = static_cast<int32_t>(old % a.block_size);
                copy[1] = fresh;
                copy[2] = static_cast<int32_t>(old % a.block_size);
                copy[0] = shared;
            } else {
                // every other holder copied it away in this call: keep it
                atomicAdd(a.refcount + shared, 1);
                atomicOr(a.free_bits + (heap >> 5), 1u << (heap & 31));
            }
        }
        for (int64_t b = first_new; b < last_new; ++b) {
            const int32_t fresh = a.block_order[p.picked[r++]];
            table[b] = fresh;
            a.refcount[fresh] = 1;
        }
        a.lens[row] = static_cast<int32_t>(old + count);
    }
    if (tid == 0) tok_base[p.sequences] = p.total_tokens;
    __syncthreads();

    // slot of every appended token, in sequence order then token order
    for (int64_t i = tid; i < p.total_tokens; i += kPlanThreads) {
        int lo = 0, hi = p.sequences - 1;  // the last sequence whose base <= i
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (tok_base[mid] <= i) lo = mid;
            else hi = mid - 1;
        }
        const int64_t pos = old_len[lo] + (i - tok_base[lo]);
        const int32_t r = p.rows[lo];
        const int64_t blk = a.tables[r * a.stride + pos / a.block_size];
        p.slots[i] = blk * a.block_size + pos % a.block_size;
        atomicMax(a.high_water + blk, static_cast<int32_t>(pos % a.block_size) + 1);
    }
}

// Rows [first, last) of one page (every layer and head, keys and values,
// codes and scales) in page `to`: rows below `keep` copied from page `from`,
// the others zeroed (from < 0 zeroes them all).  In a page the rows of one
// (layer, key|value, head) are contiguous, so each such span is one run of
// 16-byte stores; warps take spans in turn, lanes the run's chunks.
__device__ void page_rows(const Pool& pool, int32_t from, int32_t to, int64_t first, int64_t last,
                          int64_t keep) {
    if (last <= first) return;
    const int64_t D = pool.head_dim;
    const int H = static_cast<int>(pool.num_heads), L = static_cast<int>(pool.num_layers);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, warps = blockDim.x >> 5;
    const int64_t copy_end = from >= 0 ? max(first, min(keep, last)) : first;
    const int copy_chunks = static_cast<int>((copy_end - first) * D / 16);
    const int zero_chunks = static_cast<int>((last - copy_end) * D / 16);
    // spans in (layer, key|value, head) order without divisions: the warp
    // walks its heads of every layer
    for (int layer = 0; layer < L; ++layer) {
        for (int kvh = warp; kvh < 2 * H; kvh += warps) {
            const bool value_side = kvh >= H;
            const int head = value_side ? kvh - H : kvh;
            int8_t* codes = (value_side ? pool.values : pool.keys) + layer * pool.cls + head * pool.chs;
            float* scales =
                (value_side ? pool.value_scales : pool.key_scales) + layer * pool.sls + head * pool.shs;
            if (copy_chunks > 0) {
                const uint4* src = reinterpret_cast<const uint4*>(codes + from * pool.cbs + first * D);
                uint4* dst = reinterpret_cast<uint4*>(codes + to * pool.cbs + first * D);
                for (int c = lane; c < copy_chunks; c += 32) dst[c] = src[c];
                for (int64_t r = first + lane; r < copy_end; r += 32) {
                    scales[to * pool.sbs + r] = scales[from * pool.sbs + r];
                }
            }
            uint4* dst = reinterpret_cast<uint4*>(codes + to * pool.cbs + copy_end * D);
            for (int c = lane; c < zero_chunks; c += 32) dst[c] = make_uint4(0u, 0u, 0u, 0u);
            for (int64_t r = copy_end + lane; r < last; r += 32) scales[to * pool.sbs + r] = 0.0f;
        }
    }
}

// Copy-on-write: block s copies the kept rows of sequence s's shared page
// into its fresh page and zeroes the rest, so a page's slots beyond its
// sequence's length hold zeros.  Sequences without a copy return at once.
__global__ void __launch_bounds__(kCopyThreads) page_copy_kernel(Pool pool, const int32_t* copies) {
    const int32_t* c = copies + static_cast<int64_t>(blockIdx.x) * 4;
    const int32_t from = c[0];
    const int32_t to = c[1];
    if (from < 0 || from >= pool.num_blocks || to < 0 || to >= pool.num_blocks) return;
    page_rows(pool, from, to, 0, pool.block_size, c[2]);
}

struct TruncateArgs {
    Alloc a;
    Pool pool;
    const int32_t* rows;
    const int32_t* lengths;
    int32_t sequences;
    int64_t max_removed;
    int32_t* status;
    int64_t span;      // layers one zeroing block clears
    FastDiv div_pairs;  // 2 x heads: a (layer, key/value head) pair index into its parts
};

__device__ __forceinline__ bool truncate_valid(const TruncateArgs& t, int s, int32_t* row, int64_t* old, int64_t* now) {
    *row = t.rows[s];
    if (*row < 0 || *row >= t.a.rows) return false;
    *old = t.a.lens[*row];
    *now = t.lengths[s];
    return *now >= 0 && *now <= *old && *old - *now <= t.max_removed;
}

// Truncation runs in three launches so that pages released by several rows
// of one call are found free exactly once and zeroed:
//   1. truncate_mark_kernel (a thread per row): drops one reference from
//      every block past the new length; a block whose last reference goes
//      is marked -1 (released in this call) instead of 0;
//   2. truncate_zero_kernel (a block per touched page, row and layer):
//      zeroes a released page's written rows, and the rows past the new
//      length of the partly kept last page when this row alone holds it (a
//      shared page's rows still belong to the other rows) -- up to the
//      page's high-water mark, the rows any holder has written -- so freed
//      pages and slots past a length hold zeros, as the reference's
//      rollback leaves them;
//   3. truncate_finish_kernel (a thread per row): lowers the high-water
//      marks of the zeroed pages, returns the marked blocks to the free set
//      (the first row to claim a block does it), clears the table entries
//      and sets the length.
__global__ void __launch_bounds__(kPlanThreads) truncate_mark_kernel(TruncateArgs t) {
    const int s = blockIdx.x * blockDim.x + threadIdx.x;
    if (s >= t.sequences) return;
    int32_t row;
    int64_t old, now;
    if (!truncate_valid(t, s, &row, &old, &now)) {
        report_fault(t.status, SDC_FAULT_CONTEXT_RANGE);
        return;
    }
    const Alloc& a = t.a;
    const int32_t* table = a.tables + row * a.stride;
    for (int64_t b = blocks_for(now, a.block_size); b < blocks_for(old, a.block_size); ++b) {
        const int32_t blk = table[b];
        if (blk < 0 || blk >= a.num_blocks) {
            report_fault(t.status, SDC_FAULT_BLOCK_RANGE);
            continue;
        }
        if (atomicSub(a.refcount + blk, 1) == 1) a.refcount[blk] = -1;
    }
}

// (layer, key/value head) pairs one zeroing block clears at most.
constexpr int kZeroPairs = 512;

// Block (touched page j, row s, layer span z) zeroes the rows to clear of
// that page in the span's layers -- every head, keys and values, codes and
// scales.  The page's checks are made once per block; the host sizes the
// spans so that the grid still covers every SM several times over.
__global__ void __launch_bounds__(kCopyThreads) truncate_zero_kernel(TruncateArgs t) {
    const Alloc& a = t.a;
    const Pool& pool = t.pool;
    const int s = blockIdx.y;
    const int64_t layer0 = static_cast<int64_t>(blockIdx.z) * t.span;
    const int layers = static_cast<int>(pool.num_layers - layer0 < t.span ? pool.num_layers - layer0 : t.span);
    int32_t row;
    int64_t old, now;
    if (!truncate_valid(t, s, &row, &old, &now) || now == old) return;
    const int64_t bs = a.block_size;
    const int64_t b = now / bs + blockIdx.x;
    if (b >= blocks_for(old, bs)) return;
    const int32_t blk = a.tables[row * a.stride + b];
    if (blk < 0 || blk >= a.num_blocks) return;
    int first;
    if (b < blocks_for(now, bs)) {
        if (a.refcount[blk] != 1) return;  // a shared kept page's rows belong to its other holders
        first = static_cast<int>(now % bs);
    } else if (a.refcount[blk] == -1) {
        first = 0;  // released in this call
    } else {
        return;
    }
    const int rows = a.high_water[blk] - first;
    if (rows <= 0) return;
    // The span's (layer, key/value head) pairs each hold `rows` contiguous
    // rows to clear (rows x head_dim bytes) and `rows` scales.  The block
    // first lays out every pair's code and scale addresses in shared memory;
    // then threads walk the flattened (pair, 16-byte chunk) space in
    // block-strided order with incremental indices, so a store costs one
    // shared load and an add.
    __shared__ int8_t* code_at[kZeroPairs];
    __shared__ float* scale_at[kZeroPairs];
    const int H = static_cast<int>(pool.num_heads);
    const int pairs = layers * 2 * H;  // <= kZeroPairs (the host sizes the span)
    for (int pr = static_cast<int>(threadIdx.x); pr < pairs; pr += static_cast<int>(blockDim.x)) {
        uint32_t layer, kvh;
        t.div_pairs.divmod(static_cast<uint32_t>(pr), layer, kvh);
        const bool value_side = static_cast<int>(kvh) >= H;
        const int64_t head = value_side ? static_cast<int>(kvh) - H : static_cast<int>(kvh);
        const int64_t l = layer0 + layer;
        code_at[pr] = (value_side ? pool.values : pool.keys) + blk * pool.cbs + l * pool.cls + head * pool.chs +
                      first * pool.head_dim;
        scale_at[pr] = (value_side ? pool.value_scales : pool.key_scales) + blk * pool.sbs + l * pool.sls +
                       head * pool.shs + first;
    }
    __syncthreads();
    auto walk = [&](int per_pair, auto&& store) {
        const int step = static_cast<int>(blockDim.x);
        const int dq = step / per_pair, dr = step - dq * per_pair;
        int pr = static_cast<int>(threadIdx.x) / per_pair;
        int j = static_cast<int>(threadIdx.x) - pr * per_pair;
        while (pr < pairs) {
            store(pr, j);
            j += dr;
            pr += dq;
            if (j >= per_pair) {
                j -= per_pair;
                ++pr;
            }
        }
    };
    walk(rows * static_cast<int>(pool.head_dim / 16),
         [&](int pr, int c) { *reinterpret_cast<uint4*>(code_at[pr] + c * 16) = make_uint4(0u, 0u, 0u, 0u); });
    walk(rows, [&](int pr, int r) { scale_at[pr][r] = 0.0f; });
}

__global__ void __launch_bounds__(kPlanThreads) truncate_finish_kernel(TruncateArgs t) {
    const int s = blockIdx.x * blockDim.x + threadIdx.x;
    if (s >= t.sequences) return;
    int32_t row;
    int64_t old, now;
    if (!truncate_valid(t, s, &row, &old, &now)) return;
    const Alloc& a = t.a;
    int32_t* table = a.tables + row * a.stride;
    if (now < old && now % a.block_size != 0) {
        // the kept page's rows past the new length were zeroed if this row alone holds it
        const int32_t blk = table[now / a.block_size];
        if (blk >= 0 && blk < a.num_blocks && a.refcount[blk] == 1) {
            a.high_water[blk] = min(a.high_water[blk], static_cast<int32_t>(now % a.block_size));
        }
    }
    for (int64_t b = blocks_for(now, a.block_size); b < blocks_for(old, a.block_size); ++b) {
        const int32_t blk = table[b];
        table[b] = -1;
        if (blk < 0 || blk >= a.num_blocks) continue;
        if (atomicCAS(a.refcount + blk, -1, 0) == -1) {
            a.high_water[blk] = 0;  // zeroed by the previous launch
            const int32_t h = a.heap_of[blk];
            atomicOr(a.free_bits + (h >> 5), 1u << (h & 31));
        }
    }
    a.lens[row] = static_cast<int32_t>(now);
}

// One thread per (source, destination) pair: the destination (empty) shares
// every block of the source and takes its length.
__global__ void __launch_bounds__(kPlanThreads) fork_kernel(Alloc a, const int32_t* src, const int32_t* dst,
                                                             int32_t pairs, int32_t* status) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= pairs) return;
    const int32_t from = src[i], to = dst[i];
    if (from < 0 || from >= a.rows || to < 0 || to >= a.rows || from == to || a.lens[to] != 0) {
        report_fault(status, SDC_FAULT_TABLE_RANGE);
        return;
    }
    const int64_t len = a.lens[from];
    for (int64_t b = 0; b < blocks_for(len, a.block_size); ++b) {
        const int32_t blk = a.tables[from * a.stride + b];
        a.tables[to * a.stride + b] = blk;
        if (blk >= 0 && blk < a.num_blocks) atomicAdd(a.refcount + blk, 1);
    }
    a.lens[to] = static_cast<int32_t>(len);
}

sdc_status_t to_alloc(const sdc_page_allocator_t* in, Alloc* out) {
    if (in == nullptr || in->free_bits == nullptr || in->refcount == nullptr || in->high_water == nullptr ||
        in->block_order == nullptr ||
        in->heap_of == nullptr || in->block_tables == nullptr || in->context_lens == nullptr) {
        return SDC_STATUS_NULL_ARGUMENT;
    }
    if (in->num_blocks < 1 || in->block_size < 1 || in->table_rows < 1 || in->table_stride < 1) {
        return SDC_STATUS_INVALID_SIZE;
    }
    if (in->num_blocks > (int64_t(1) << 31) - 1 || in->table_rows > (int64_t(1) << 31) - 1 ||
        in->table_stride > (int64_t(1) << 31) / in->table_rows ||
        in->block_size > (int64_t(1) << 31) / in->table_stride) {
        return SDC_STATUS_OVERFLOW;
    }
    *out = Alloc{in->free_bits, in->refcount, in->high_water, in->block_order, in->heap_of, in->block_tables,
                 in->context_lens, in->num_blocks, in->block_size, in->table_rows, in->table_stride};
    return SDC_STATUS_OK;
}

sdc_status_t check_pool_matches(const sdc_page_pool_t* pool, const Alloc& a) {
    const sdc_status_t st = validate_pool(pool);
    if (st != SDC_STATUS_OK) return st;
    if (pool->num_blocks != a.num_blocks || pool->block_size != a.block_size) return SDC_STATUS_INVALID_ARGUMENT;
    return SDC_STATUS_OK;
}

int64_t picked_capacity(int64_t sequences, int64_t total_tokens, int64_t block_size) {
    // a sequence appending n tokens takes at most ceil(n / bs) + 1 new blocks
    // (the partial block it starts in can end a block early) plus one copy
    return total_tokens / block_size + 3 * sequences;
}

template <typename F>
sdc_status_t guarded(F&& f) {
    try {
        return f();
    } catch (...) {
        return SDC_STATUS_INTERNAL_ERROR;
    }
}

}  // namespace
}  // namespace sdc

using namespace sdc;

extern "C" {

SDC_API sdc_status_t sdc_pages_append_workspace_size(int64_t sequences, int64_t total_tokens, int64_t block_size,
                                                     size_t* bytes) {
    if (bytes == nullptr) return SDC_STATUS_NULL_ARGUMENT;
    if (sequences < 1 || sequences > kPlanThreads || total_tokens < 0 || block_size < 1) return SDC_STATUS_INVALID_SIZE;
    if (total_tokens > (int64_t(1) << 40)) return SDC_STATUS_OVERFLOW;
    const int64_t copies = sequences * 4 * 4;
    *bytes = static_cast<size_t>(copies + picked_capacity(sequences, total_tokens, block_size) * 4);
    return SDC_STATUS_OK;
}

SDC_API sdc_status_t sdc_pages_append(const sdc_page_allocator_t* allocator, const sdc_page_pool_t* pool,
                                      const int32_t* rows, const int32_t* counts, int64_t sequences,
                                      int64_t total_tokens, int64_t* slot_mapping, void* workspace,
                                      size_t workspace_bytes, int32_t* device_status, uintptr_t stream) {
    return guarded([&]() -> sdc_status_t {
        Alloc a;
        sdc_status_t st = to_alloc(allocator, &a);
        if (st != SDC_STATUS_OK) return st;
        st = check_pool_matches(pool, a);
        if (st != SDC_STATUS_OK) return st;
        if (rows == nullptr || counts == nullptr || workspace == nullptr) return SDC_STATUS_NULL_ARGUMENT;
        if (total_tokens > 0 && slot_mapping == nullptr) return SDC_STATUS_NULL_ARGUMENT;
        size_t need = 0;
        st = sdc_pages_append_workspace_size(sequences, total_tokens, a.block_size, &need);
        if (st != SDC_STATUS_OK) return st;
        if (workspace_bytes < need) return SDC_STATUS_INVALID_SIZE;
        if (reinterpret_cast<uintptr_t>(workspace) % 16) return SDC_STATUS_MISALIGNED;
        int32_t* copies = static_cast<int32_t*>(workspace);
        AppendPlanArgs p{a, rows, counts, static_cast<int32_t>(sequences), total_tokens, slot_mapping, copies,
                         copies + sequences * 4, picked_capacity(sequences, total_tokens, a.block_size),
                         device_status};
        cudaStream_t s = as_stream(stream);
        append_plan_kernel<<<1, kPlanThreads, 0, s>>>(p);
        page_copy_kernel<<<static_cast<unsigned>(sequences), kCopyThreads, 0, s>>>(to_pool(pool), copies);
        return launch_status();
    });
}

SDC_API sdc_status_t sdc_pages_truncate(const sdc_page_allocator_t* allocator, const sdc_page_pool_t* pool,
                                        const int32_t* rows, const int32_t* new_lengths, int64_t sequences,
                                        int64_t max_removed, int32_t* device_status, uintptr_t stream) {
    return guarded([&]() -> sdc_status_t {
        Alloc a;
        sdc_status_t st = to_alloc(allocator, &a);
        if (st != SDC_STATUS_OK) return st;
        st = check_pool_matches(pool, a);
        if (st != SDC_STATUS_OK) return st;
        if (rows == nullptr || new_lengths == nullptr) return SDC_STATUS_NULL_ARGUMENT;
        if (sequences < 1 || sequences > 65535 || max_removed < 0) return SDC_STATUS_INVALID_SIZE;
        if (max_removed > 65535) return SDC_STATUS_OVERFLOW;
        TruncateArgs t{a, to_pool(pool), rows, new_lengths, static_cast<int32_t>(sequences), max_removed,
                       device_status, 1, FastDiv(static_cast<uint32_t>(2 * pool->num_heads))};
        // zeroing grid, checked before anything launches: pages a truncation
        // of at most max_removed tokens touches, and layers per block -- as
        // many as keep the grid at four blocks per SM or more
        const int64_t pages = (max_removed + a.block_size - 1) / a.block_size + 1;
        int64_t spans = 1;
        if (max_removed > 0) {
            if (2 * pool->num_heads > kZeroPairs) return SDC_STATUS_UNSUPPORTED;
            const int64_t L = pool->num_layers;
            const int64_t splits = std::min<int64_t>(L, ceil_div(4 * static_cast<int64_t>(device_sms()),
                                                                 pages * sequences));
            t.span = std::min<int64_t>(ceil_div(L, splits), kZeroPairs / (2 * pool->num_heads));
            spans = ceil_div(L, t.span);
            if (spans > 65535 || pages > INT32_MAX) return SDC_STATUS_UNSUPPORTED;
            if (t.span * 2 * pool->num_heads * a.block_size * (pool->head_dim / 16) >= INT32_MAX) {
                return SDC_STATUS_OVERFLOW;
            }
        }
        cudaStream_t s = as_stream(stream);
        const unsigned row_blocks = static_cast<unsigned>(ceil_div(sequences, kPlanThreads));
        truncate_mark_kernel<<<row_blocks, kPlanThreads, 0, s>>>(t);
        if (max_removed > 0) {
            truncate_zero_kernel<<<dim3(static_cast<unsigned>(pages), static_cast<unsigned>(sequences),
                                        static_cast<unsigned>(spans)),
                                   kCopyThreads, 0, s>>>(t);
        }
        truncate_finish_kernel<<<row_blocks, kPlanThreads, 0, s>>>(t);
        return launch_status();
    });
}

SDC_API sdc_status_t sdc_pages_fork(const sdc_page_allocator_t* allocator, const int32_t* source_rows,
                                    const int32_t* destination_rows, int64_t pairs, int32_t* device_status,
                                    uintptr_t stream) {
    return guarded([&]() -> sdc_status_t {
        Alloc a;
        const sdc_status_t st = to_alloc(allocator, &a);
        if (st != SDC_STATUS_OK) return st;
        if (source_rows == nullptr || destination_rows == nullptr) return SDC_STATUS_NULL_ARGUMENT;
        if (pairs < 1 || pairs > (int64_t(1) << 31) - 1) return SDC_STATUS_INVALID_SIZE;
        fork_kernel<<<static_cast<unsigned>(ceil_div(pairs, kPlanThreads)), kPlanThreads, 0, as_stream(stream)>>>(
            a, source_rows, destination_rows, static_cast<int32_t>(pairs), device_status);
        return launch_status();
    });
}

}  // extern "C"
