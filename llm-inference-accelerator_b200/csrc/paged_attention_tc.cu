// Kernel (c) on the 5th-generation tensor cores: paged verify attention with
// INT8 pages fed straight from TMA to tcgen05.mma (kind::i8), accumulators
// in tensor memory.  head_dim 128; any block size that divides 128 (>= 8).
//
// Same computation and work decomposition as paged_attention.cu (split-K
// items of (sequence, KV head, chunk), un-normalised partials, a combine
// pass); what changes is how one item walks its chunk, 128 tokens per tile:
//
//   S^T[t, n] = sum_d K[t, d] * Qi8[n, d]      (M = 128 tokens, N = 2*RMAX cols)
//   O^T[d, n] = sum_t V[t, d] * Pi8[n, t]      (M = 128 = head_dim, same N)
//
// The query rows are split into two INT8 parts, q ~ s1 * (hi + lo / 254)
// with s1 = max|q| / 127 per row (columns [0, RMAX) hold hi, [RMAX, 2 RMAX)
// lo), so the integer products are exact and the row's score is
// (254 * S_hi + S_lo) * s1 / 254 * scale_k: the query carries 15 bits of
// relative precision, finer than its bf16 input.  Probabilities are split
// the same way after folding in the value scale: u = p * scale_v / max(scale_v)
// in [0, 1], hi = rint(127 u), lo = rint(254 (127 u - hi)), an absolute error
// below 1.6e-5.  K is the A operand in K-major form and V the A operand in
// MN-major form of the same 128-byte rows: every page goes from HBM to
// shared memory exactly once, by one TMA box per page, and is never
// converted.
//
// Warp roles (192 threads): warps 0-3 run softmax (thread = token of S^T,
// TMEM lane) and the O epilogue (thread = head_dim row of O^T); warp 4
// issues TMA; warp 5 allocates tensor memory and issues the MMAs.  Every
// mbarrier wait gives up after one second, records SDC_FAULT_WAIT_TIMEOUT in
// the status word, and lets the block wind down: it waits (bounded) for its
// own copies and MMAs, frees tensor memory and returns.

#include <cuda.h>

#include <cub/block/block_scan.cuh>
#include <mutex>

#include "host_common.h"
#include "paged_attention.h"

namespace sdc {
namespace tc {
namespace {

constexpr int kTile = 128;     // tokens per tile (MMA M for S^T)
constexpr int kHeadDim = 128;  // MMA M for O^T, and the K extent of S^T
constexpr int kCodeTileBytes = kTile * kHeadDim;                    // 16 KiB
constexpr int kStageBytes = 2 * kCodeTileBytes + 2 * kTile * 4;     // K, V codes + scales
constexpr int kSoftmaxWarps = 4;
constexpr int kThreads = (kSoftmaxWarps + 2) * 32;
constexpr int kProducerWarp = 4;
constexpr int kMmaWarp = 5;
constexpr unsigned long long kWaitLimitNs = 1000000000ull;  // one second

constexpr int pow2_at_least(int v) {
    int p = 32;
    while (p < v) p <<= 1;
    return p;
}

template <int RMAX, int STAGES>
struct Layout {
    static constexpr int N = ((2 * RMAX + 15) / 16) * 16;                  // MMA N
    static constexpr int kQCodes = N * kHeadDim;                           // query image codes
    static constexpr int kQBytes = kQCodes + ((RMAX * 4 + 15) / 16) * 16;   // + per-row factors
    static constexpr int kPBytes = N * kTile;
    static constexpr int kTmemStride = pow2_at_least(N);                   // columns per buffer
    static constexpr int kTmemCols = 4 * kTmemStride;                      // S0 S1 O0 O1
    // shared-memory offsets (bytes, from a 1024-aligned base)
    static constexpr int kStages = 0;
    static constexpr int kQ = kStages + STAGES * kStageBytes;
    static constexpr int kP = kQ + 2 * ((kQBytes + 127) / 128) * 128;
    static constexpr int kRed = kP + 2 * kPBytes;                 // [2][4][RMAX + 1] per-warp exchange
    static constexpr int kAlpha = kRed + 2 * 4 * (RMAX + 1) * 4;  // [2][RMAX] rescale factors per tile parity
    static constexpr int kVfac = kAlpha + 2 * RMAX * 4;           // [2]
    static constexpr int kBar = ((kVfac + 8 + 7) / 8) * 8;        // mbarriers
    static constexpr int kNumBars = 2 * STAGES + 2 * 8;
    static constexpr int kMisc = kBar + kNumBars * 8;             // tmem base, abort flag
    static constexpr int kTotal = kMisc + 16;
    static constexpr int kDynamicSmem = kTotal + 1024;            // room to align the base
};

// Pipeline depth and blocks per SM by row bucket: 24 rows fit two blocks per
// SM (256 TMEM columns and ~93 KB of shared memory each); 40 rows take the
// whole tensor memory (512 columns), so one block with a deeper pipeline.
template <int RMAX>
constexpr int kStagesFor = RMAX <= 24 ? 2 : 3;
template <int RMAX>
constexpr int kMinBlocksFor = RMAX <= 24 ? 2 : 1;

struct WorkItem {
    int32_t b, h, t0, t1;
};

struct TcArgs {
    AttnArgs a;
    const uint8_t* qimg;    // [B * Hkv][q_bytes]
    int32_t q_bytes;
    const WorkItem* items;  // [max_items]
    const int32_t* item_count;
    int32_t rows;           // query rows per KV head (<= RMAX)
};

// ---------------------------------------------------------------- PTX helpers

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long globaltimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(bar), "r"(parity)
        : "memory");
    return done != 0;
}

// Bounded wait on an mbarrier phase.  Returns false when the block is
// aborting (this wait gave up, or another one already did).
__device__ __forceinline__ bool wait_phase(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                           int32_t* status) {
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long start = globaltimer();
    while (true) {
        if (mbar_try_wait(bar, parity)) return true;
        if (*abort_flag) return false;
        if (globaltimer() - start > kWaitLimitNs) {
            *abort_flag = 1;
            report_fault(status, SDC_FAULT_WAIT_TIMEOUT);
            return false;
        }
    }
}

// The same wait taken by a whole warp with one outcome: either every lane
// observed the phase (and so holds its acquire ordering) or all give up.
__device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag, int32_t* status) {
    return __all_sync(kFullMask, wait_phase(bar, parity, abort_flag, status));
}

// Wait used while winding down: bounded, ignores the abort flag.
__device__ __forceinline__ void drain_phase(uint32_t bar, uint32_t parity) {
    const unsigned long long start = globaltimer();
    while (!mbar_try_wait(bar, parity)) {
        if (globaltimer() - start > kWaitLimitNs) return;
    }
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int32_t x, int32_t y,
                                            uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
        "[%4];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
        : "memory");
}

__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
                 "l"(src), "r"(bytes), "r"(bar)
                 : "memory");
}

__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory matrix descriptor (tcgen05): start, leading and stride byte
// offsets in 16-byte units, descriptor version 1, layout (0 none, 2 = 128B swizzle).
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo, uint32_t layout) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((addr >> 4) & 0x3FFFu);
    d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
    d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
    d |= 1ull << 46;
    d |= static_cast<uint64_t>(layout) << 61;
    return d;
}

// Instruction descriptor for kind::i8: s32 accumulate, signed A and B.
__host__ __device__ constexpr uint32_t idesc_i8(int m, int n, int a_mn_major, int b_mn_major) {
    return (2u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(a_mn_major) << 15) |
           (static_cast<uint32_t>(b_mn_major) << 16) | (static_cast<uint32_t>(n >> 3) << 17) |
           (static_cast<uint32_t>(m >> 4) << 24);
}

__device__ __forceinline__ void mma_i8(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, bool accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(a), "l"(b), "r"(idesc), "r"(static_cast<uint32_t>(accumulate))
        : "memory");
}

__device__ __forceinline__ void mma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}

// 16 consecutive 32-bit TMEM columns of this thread's lane.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16], int base) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15}, [%16];"
        : "=r"(r[base + 0]), "=r"(r[base + 1]), "=r"(r[base + 2]), "=r"(r[base + 3]), "=r"(r[base + 4]),
          "=r"(r[base + 5]), "=r"(r[base + 6]), "=r"(r[base + 7]), "=r"(r[base + 8]), "=r"(r[base + 9]),
          "=r"(r[base + 10]), "=r"(r[base + 11]), "=r"(r[base + 12]), "=r"(r[base + 13]), "=r"(r[base + 14]),
          "=r"(r[base + 15])
        : "r"(taddr));
}

template <int N>
__device__ __forceinline__ void tmem_ld_row(uint32_t taddr, uint32_t (&r)[N]) {
    static_assert(N % 16 == 0, "columns come in groups of 16");
#pragma unroll
    for (int c = 0; c < N; c += 16) {
        uint32_t chunk[16];
        tmem_ld16(taddr + c, chunk, 0);
#pragma unroll
        for (int i = 0; i < 16; ++i) r[c + i] = chunk[i];
    }
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ float redux_max(float v) {
    float r;
    asm volatile("redux.sync.max.f32 %0, %1, 0xffffffff;" : "=f"(r) : "f"(v));
    return r;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(kFullMask, v, off);
    return v;
}

__device__ __forceinline__ uint32_t byte_of(int v, int i) { return (static_cast<uint32_t>(v) & 0xffu) << (8 * i); }

// ---------------------------------------------------------------- main kernel

template <int RMAX, int STAGES, int MIN_BLOCKS>
__global__ void __launch_bounds__(kThreads, MIN_BLOCKS)
    attn_tc_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap, TcArgs t) {
    using LY = Layout<RMAX, STAGES>;
    constexpr int N = LY::N;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const AttnArgs& a = t.a;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int count = __ldg(t.item_count);
    if (static_cast<int>(blockIdx.x) >= count) return;  // whole block: no work

    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + LY::kBar);
    auto bar = [&](int i) { return smem_u32(bars + i); };
    // barrier indices
    const int kvFull = 0, kvEmpty = STAGES, qFull = 2 * STAGES, qEmpty = qFull + 2, sFull = qEmpty + 2,
              sEmpty = sFull + 2, pFull = sEmpty + 2, oFull = pFull + 2, oEmpty = oFull + 2, xch = oEmpty + 2;
    volatile uint32_t* tmem_base_slot = reinterpret_cast<volatile uint32_t*>(smem + LY::kMisc);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + LY::kMisc + 4);

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(bar(kvFull + s), 1);
            mbar_init(bar(kvEmpty + s), 1 + kSoftmaxWarps);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(bar(qFull + i), 1);
            mbar_init(bar(qEmpty + i), 1 + kSoftmaxWarps);
            mbar_init(bar(sFull + i), 1);
            mbar_init(bar(sEmpty + i), kSoftmaxWarps);
            mbar_init(bar(pFull + i), kSoftmaxWarps * 32);
            mbar_init(bar(oFull + i), 1);
            mbar_init(bar(oEmpty + i), kSoftmaxWarps);
            mbar_init(bar(xch + i), kSoftmaxWarps);
        }
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == kMmaWarp) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(const_cast<uint32_t*>(tmem_base_slot))),
                     "n"(LY::kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_base_slot;

    const uint32_t stage_base = smem_u32(smem + LY::kStages);
    const uint32_t q_base = smem_u32(smem + LY::kQ);
    constexpr uint32_t kQStride = ((LY::kQBytes + 127) / 128) * 128;
    const uint32_t p_base = smem_u32(smem + LY::kP);
    const int R = t.rows;
    const int64_t bs = a.pool.block_size;
    const int pages_per_tile = static_cast<int>(kTile / bs);

    if (warp == kProducerWarp) {
        // ------------------------------------------------------------ TMA producer
        uint32_t g = 0, li = 0;
        for (int item = blockIdx.x; item < count; item += gridDim.x, ++li) {
            const WorkItem it = t.items[item];
            const uint32_t qb = li & 1;
            if (!warp_wait(bar(qEmpty + qb), ((li >> 1) & 1) ^ 1, abort_flag, a.status)) break;
            if (lane == 0) {
                mbar_arrive_expect_tx(bar(qFull + qb), t.q_bytes);
                bulk_load(q_base + qb * kQStride,
                          t.qimg + (static_cast<int64_t>(it.b) * a.kv_heads + it.h) * t.q_bytes, t.q_bytes,
                          bar(qFull + qb));
            }
            const int32_t* table = a.block_tables + static_cast<int64_t>(it.b) * a.table_stride;
            const int64_t code_base = a.layer * a.pool.cls + it.h * a.pool.chs;
            const int64_t scale_base = a.layer * a.pool.sls + it.h * a.pool.shs;
            bool stop = false;
            for (int tile0 = it.t0; tile0 < it.t1; tile0 += kTile, ++g) {
                const uint32_t s = g % STAGES;
                if (!warp_wait(bar(kvEmpty + s), ((g / STAGES) & 1) ^ 1, abort_flag, a.status)) {
                    stop = true;
                    break;
                }
                const int64_t page_token = tile0 + static_cast<int64_t>(lane) * bs;
                bool valid = lane < pages_per_tile && page_token < it.t1;
                int64_t blk = 0;
                if (valid) {
                    blk = __ldg(table + page_token / bs);
                    if (blk < 0 || blk >= a.pool.num_blocks) {
                        report_fault(a.status, SDC_FAULT_BLOCK_RANGE);
                        valid = false;
                    }
                }
                const uint32_t mask = __ballot_sync(kFullMask, valid);
                const uint32_t page_bytes = static_cast<uint32_t>(bs) * (2 * kHeadDim + 8);
                if (lane == 0) mbar_arrive_expect_tx(bar(kvFull + s), __popc(mask) * page_bytes);
                __syncwarp();
                if (valid) {
                    const uint32_t st = stage_base + s * kStageBytes;
                    const int64_t code_off = blk * a.pool.cbs + code_base;
                    const int32_t row = static_cast<int32_t>(code_off / kHeadDim);
                    const uint32_t dst = static_cast<uint32_t>(lane * bs * kHeadDim);
                    tma_load_2d(st + dst, &kmap, 0, row, bar(kvFull + s));
                    tma_load_2d(st + kCodeTileBytes + dst, &vmap, 0, row, bar(kvFull + s));
                    const int64_t scale_off = blk * a.pool.sbs + scale_base;
                    const uint32_t sdst = static_cast<uint32_t>(lane * bs * 4);
                    bulk_load(st + 2 * kCodeTileBytes + sdst, a.pool.key_scales + scale_off,
                              static_cast<uint32_t>(bs * 4), bar(kvFull + s));
                    bulk_load(st + 2 * kCodeTileBytes + kTile * 4 + sdst, a.pool.value_scales + scale_off,
                              static_cast<uint32_t>(bs * 4), bar(kvFull + s));
                }
            }
            if (stop) break;
        }
        // wind down: every copy this warp issued has landed before the block exits
        if (*abort_flag && lane == 0) {
            for (uint32_t k = 0; k < STAGES && k < g; ++k) {
                const uint32_t gg = g - 1 - k;
                drain_phase(bar(kvFull + gg % STAGES), (gg / STAGES) & 1);
            }
        }
    } else if (warp == kMmaWarp) {
        // ------------------------------------------------------------ MMA issuer
        constexpr uint32_t kIdescS = idesc_i8(kTile, N, 0, 0);
        constexpr uint32_t kIdescO = idesc_i8(kHeadDim, N, 1, 1);
        uint32_t g = 0, li = 0;
        bool have_prev = false;
        uint32_t prev = 0;
        uint32_t last_s_commit = 0, last_o_commit = 0;
        bool any_s = false, any_o = false;
        auto issue_pv = [&](uint32_t gp) -> bool {
            const uint32_t sb = gp & 1;
            const uint32_t s = gp % STAGES;
            if (!warp_wait(bar(pFull + sb), (gp >> 1) & 1, abort_flag, a.status)) return false;
            if (!warp_wait(bar(oEmpty + sb), ((gp >> 1) & 1) ^ 1, abort_flag, a.status)) return false;
            tc_fence_after();
            if (lane == 0) {
                const uint32_t v_tile = stage_base + s * kStageBytes + kCodeTileBytes;
                const uint32_t p_tile = p_base + sb * LY::kPBytes;
#pragma unroll
                for (int ks = 0; ks < kTile / 32; ++ks) {
                    const uint64_t da = smem_desc(v_tile + ks * 4096, kCodeTileBytes, 1024, 2);
                    const uint64_t db = smem_desc(p_tile + ks * 512, 128, 2048, 0);
                    mma_i8(tmem + (2 + sb) * LY::kTmemStride, da, db, kIdescO, ks > 0);
                }
                mma_commit(bar(oFull + sb));
                mma_commit(bar(kvEmpty + s));
            }
            __syncwarp();
            last_o_commit = gp;
            any_o = true;
            return true;
        };
        bool ok = true;
        for (int item = blockIdx.x; item < count && ok; item += gridDim.x, ++li) {
            const WorkItem it = t.items[item];
            const uint32_t qb = li & 1;
            if (!warp_wait(bar(qFull + qb), (li >> 1) & 1, abort_flag, a.status)) break;
            for (int tile0 = it.t0; tile0 < it.t1; tile0 += kTile, ++g) {
                const uint32_t s = g % STAGES;
                const uint32_t sb = g & 1;
                if (!warp_wait(bar(kvFull + s), (g / STAGES) & 1, abort_flag, a.status) ||
                    !warp_wait(bar(sEmpty + sb), ((g >> 1) & 1) ^ 1, abort_flag, a.status)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                if (lane == 0) {
                    const uint32_t k_tile = stage_base + s * kStageBytes;
                    const uint32_t q_tile = q_base + qb * kQStride;
#pragma unroll
                    for (int ks = 0; ks < kHeadDim / 32; ++ks) {
                        const uint64_t da = smem_desc(k_tile + ks * 32, 16, 1024, 2);
                        const uint64_t db = smem_desc(q_tile + ks * 256, 128, 1024, 0);
                        mma_i8(tmem + sb * LY::kTmemStride, da, db, kIdescS, ks > 0);
                    }
                    mma_commit(bar(sFull + sb));
                    if (tile0 + kTile >= it.t1) mma_commit(bar(qEmpty + qb));
                }
                __syncwarp();
                last_s_commit = g;
                any_s = true;
                if (have_prev && !issue_pv(prev)) {
                    ok = false;
                    have_prev = false;
                    break;
                }
                prev = g;
                have_prev = true;
            }
        }
        if (ok && have_prev) issue_pv(prev);
        if (*abort_flag && lane == 0) {
            if (any_s) drain_phase(bar(sFull + (last_s_commit & 1)), (last_s_commit >> 1) & 1);
            if (any_o) drain_phase(bar(oFull + (last_o_commit & 1)), (last_o_commit >> 1) & 1);
        }
    } else {
        // ------------------------------------------------------------ softmax + O epilogue
        // Cross-warp exchanges go through shared memory guarded by the xch
        // mbarriers (one arrival per warp), double-buffered by exchange
        // parity: a buffer is rewritten two exchanges later, by which time
        // every warp has arrived at the exchange in between and so has
        // finished reading it.
        float* red = reinterpret_cast<float*>(smem + LY::kRed);      // [2][4][RMAX + 1]
        float* alpha_s = reinterpret_cast<float*>(smem + LY::kAlpha);
        float* vfac_s = reinterpret_cast<float*>(smem + LY::kVfac);
        constexpr int kRedStride = RMAX + 1;
        const int tid = threadIdx.x;  // 0..127: token row of S^T, head_dim row of O^T
        const uint32_t lane_addr = static_cast<uint32_t>(warp * 32) << 16;
        uint32_t g = 0, li = 0, xc = 0;
        // publish this warp's slice of red[xc], wait for all four warps
        auto exchange = [&]() -> bool {
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(xch + (xc & 1)));
            const bool ok = warp_wait(bar(xch + (xc & 1)), (xc >> 1) & 1, abort_flag, a.status);
            return ok;
        };
        auto epilogue = [&](uint32_t gp, float (&o_acc)[RMAX]) -> bool {
            const uint32_t ob = gp & 1;
            if (!warp_wait(bar(oFull + ob), (gp >> 1) & 1, abort_flag, a.status)) return false;
            tc_fence_after();
            uint32_t oreg[N];
            tmem_ld_row<N>(tmem + lane_addr + (2 + ob) * LY::kTmemStride, oreg);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(oEmpty + ob));
            const float vf = vfac_s[ob];
#pragma unroll
            for (int r = 0; r < RMAX; ++r) {
                const int32_t combined = static_cast<int32_t>(oreg[r]) * 254 + static_cast<int32_t>(oreg[RMAX + r]);
                o_acc[r] = o_acc[r] * alpha_s[ob * RMAX + r] + static_cast<float>(combined) * vf;
            }
            return true;
        };
        bool ok = true;
        for (int item = blockIdx.x; item < count && ok; item += gridDim.x, ++li) {
            const WorkItem it = t.items[item];
            const uint32_t qb = li & 1;
            if (!warp_wait(bar(qFull + qb), (li >> 1) & 1, abort_flag, a.status)) break;
            const float* qfac = reinterpret_cast<const float*>(smem + LY::kQ + qb * kQStride + LY::kQCodes);
            const int64_t T = __ldg(a.context_lens + it.b);
            const int64_t window = a.window;
            float m_run[RMAX], l_thr[RMAX], o_acc[RMAX];
#pragma unroll
            for (int r = 0; r < RMAX; ++r) {
                m_run[r] = -INFINITY;
                l_thr[r] = 0.0f;
                o_acc[r] = 0.0f;
            }
            const uint32_t first_g = g;
            for (int tile0 = it.t0; tile0 < it.t1; tile0 += kTile, ++g) {
                const uint32_t sb = g & 1;
                const uint32_t s = g % STAGES;
                if (!warp_wait(bar(sFull + sb), (g >> 1) & 1, abort_flag, a.status) ||
                    !warp_wait(bar(kvFull + s), (g / STAGES) & 1, abort_flag, a.status)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                uint32_t sreg[N];
                tmem_ld_row<N>(tmem + lane_addr + sb * LY::kTmemStride, sreg);
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(bar(sEmpty + sb));

                const int64_t tok = tile0 + tid;
                const bool tvalid = tok < it.t1;
                const float* stage_scales =
                    reinterpret_cast<const float*>(smem + LY::kStages + s * kStageBytes + 2 * kCodeTileBytes);
                const float kscale = stage_scales[tid];
                const float vscale = tvalid ? stage_scales[kTile + tid] : 0.0f;
                __syncwarp();
                if (lane == 0) mbar_arrive(bar(kvEmpty + s));

                // a query at window row i sees keys up to T - window + i; only
                // tiles reaching into the window need the per-row test
                const bool causal_tile = tile0 + kTile > T - window;
                auto visible = [&](int r) {
                    if (!tvalid || r >= R) return false;
                    return !causal_tile || tok <= T - window + (r % window);
                };
                float* red_x = red + (xc & 1) * 4 * kRedStride;
#pragma unroll
                for (int r = 0; r < RMAX; ++r) {
                    float sc = -INFINITY;
                    if (visible(r)) {
                        const int32_t combined =
                            static_cast<int32_t>(sreg[r]) * 254 + static_cast<int32_t>(sreg[RMAX + r]);
                        sc = static_cast<float>(combined) * (qfac[r] * kscale);
                    }
                    const float wm = redux_max(sc);
                    if (lane == 0) red_x[warp * kRedStride + r] = wm;
                }
                const float wv = redux_max(vscale);
                if (lane == 0) red_x[warp * kRedStride + RMAX] = wv;
                if (!exchange()) {
                    ok = false;
                    break;
                }
                ++xc;
                const float vmax = fmaxf(fmaxf(red_x[RMAX], red_x[kRedStride + RMAX]),
                                         fmaxf(red_x[2 * kRedStride + RMAX], red_x[3 * kRedStride + RMAX]));
                const float u_scale = vmax > 0.0f ? 127.0f * vscale / vmax : 0.0f;
                uint32_t row_words[N / 4];
#pragma unroll
                for (int w = 0; w < N / 4; ++w) row_words[w] = 0u;
#pragma unroll
                for (int r = 0; r < RMAX; ++r) {
                    const float tmax = fmaxf(fmaxf(red_x[r], red_x[kRedStride + r]),
                                             fmaxf(red_x[2 * kRedStride + r], red_x[3 * kRedStride + r]));
                    const float m_new = fmaxf(m_run[r], tmax);
                    const float alpha = (m_new == -INFINITY) ? 1.0f : exp2f(m_run[r] - m_new);
                    m_run[r] = m_new;
                    float p = 0.0f;
                    if (visible(r)) {
                        const int32_t combined =
                            static_cast<int32_t>(sreg[r]) * 254 + static_cast<int32_t>(sreg[RMAX + r]);
                        p = exp2f(static_cast<float>(combined) * (qfac[r] * kscale) - m_new);
                    }
                    l_thr[r] = l_thr[r] * alpha + p;
                    const float x = p * u_scale;  // in [0, 127]
                    const float hi = rintf(x);
                    const float lo = rintf((x - hi) * 254.0f);
                    row_words[r / 4] |= byte_of(static_cast<int>(hi), r % 4);
                    row_words[(RMAX + r) / 4] |= byte_of(static_cast<int>(lo), (RMAX + r) % 4);
                    if (tid == r) alpha_s[sb * RMAX + r] = alpha;
                }
                if (tid == 0) vfac_s[sb] = vmax / (127.0f * 254.0f);
                // P^T row of this token (columns [0, RMAX) hi, [RMAX, 2 RMAX) lo,
                // rest zero) in the MN-major no-swizzle layout: a 128-byte core
                // matrix holds 16 columns x 8 tokens; 8-token groups are 128 bytes
                // apart, 16-column groups 2048 bytes apart.
                unsigned char* prow = smem + LY::kP + sb * LY::kPBytes + (tid >> 3) * 128 + (tid & 7) * 16;
#pragma unroll
                for (int c = 0; c < N / 16; ++c) {
                    *reinterpret_cast<uint4*>(prow + c * 2048) =
                        make_uint4(row_words[4 * c], row_words[4 * c + 1], row_words[4 * c + 2], row_words[4 * c + 3]);
                }
                fence_proxy_async();
                mbar_arrive(bar(pFull + sb));

                if (g > first_g && !epilogue(g - 1, o_acc)) {  // previous tile of this item
                    ok = false;
                    break;
                }
            }
            if (!ok) break;
            // publish the last tile's alpha / vfac, then its epilogue
            if (!exchange()) break;
            ++xc;
            if (!epilogue(g - 1, o_acc)) break;
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(qEmpty + qb));
            // partial result of this chunk: m, l (summed over all 128 tokens) and O
            float* red_x = red + (xc & 1) * 4 * kRedStride;
#pragma unroll
            for (int r = 0; r < RMAX; ++r) {
                const float ws = warp_sum(l_thr[r]);
                if (lane == 0) red_x[warp * kRedStride + r] = ws;
            }
            if (!exchange()) break;
            ++xc;
            const int64_t bh = static_cast<int64_t>(it.b) * a.kv_heads + it.h;
            const int64_t chunk = it.t0 / a.chunk;
            float* part_o = a.part_o + (bh * a.max_chunks + chunk) * R * kHeadDim;
            float* part_ml = a.part_ml + (bh * a.max_chunks + chunk) * R * 2;
#pragma unroll
            for (int r = 0; r < RMAX; ++r) {
                if (r < R) {
                    part_o[r * kHeadDim + tid] = o_acc[r];
                    if (tid == r) {
                        part_ml[2 * r + 0] = m_run[r];
                        part_ml[2 * r + 1] = red_x[r] + red_x[kRedStride + r] + red_x[2 * kRedStride + r] +
                                             red_x[3 * kRedStride + r];
                    }
                }
            }
        }
    }

    // ------------------------------------------------------------ teardown
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == kMmaWarp) {
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "n"(LY::kTmemCols)
                     : "memory");
    }
}

// ---------------------------------------------------------------- query images

// Splits each query row into INT8 hi/lo parts laid out as the B operand of
// the score MMA (K-major, no swizzle: 8 rows x 16 bytes per 128-byte core
// matrix, 16-byte K chunks 128 bytes apart, 8-row groups 1024 bytes apart),
// followed by the per-row factor s1 / 254 * log2(e) / sqrt(D).
template <typename QT, int RMAX>
__global__ void __launch_bounds__(256) query_image_kernel(TcArgs t) {
    using LY = Layout<RMAX, kStagesFor<RMAX>>;
    const AttnArgs& a = t.a;
    const int64_t bh = blockIdx.x;
    const int64_t b = bh / a.kv_heads;
    const int64_t h = bh - b * a.kv_heads;
    uint8_t* img = const_cast<uint8_t*>(t.qimg) + bh * t.q_bytes;
    for (int i = threadIdx.x; i < t.q_bytes / 16; i += blockDim.x) {
        reinterpret_cast<uint4*>(img)[i] = make_uint4(0u, 0u, 0u, 0u);
    }
    __syncthreads();
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const QT* q = static_cast<const QT*>(a.query) + ((b * a.query_heads + h * a.group) * a.window) * kHeadDim;
    float* factors = reinterpret_cast<float*>(img + LY::kQCodes);
    for (int r = warp; r < t.rows; r += blockDim.x / 32) {
        float x[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) x[i] = static_cast<float>(q[r * kHeadDim + lane * 4 + i]);
        float m = fmaxf(fmaxf(fabsf(x[0]), fabsf(x[1])), fmaxf(fabsf(x[2]), fabsf(x[3])));
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(kFullMask, m, off));
        uint32_t hi_word = 0, lo_word = 0;
        float factor = 0.0f;
        if (m > 0.0f) {
            const float s1 = m / 127.0f;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float hi = fminf(fmaxf(rintf(x[i] / s1), -127.0f), 127.0f);
                const float lo = fminf(fmaxf(rintf((x[i] - hi * s1) * (254.0f / s1)), -127.0f), 127.0f);
                hi_word |= byte_of(static_cast<int>(hi), i);
                lo_word |= byte_of(static_cast<int>(lo), i);
            }
            factor = s1 / 254.0f * a.qk_scale;
        }
        const int d = lane * 4;
        auto offset = [&](int n) { return (n >> 3) * 1024 + (d >> 4) * 128 + (n & 7) * 16 + (d & 15); };
        *reinterpret_cast<uint32_t*>(img + offset(r)) = hi_word;
        *reinterpret_cast<uint32_t*>(img + offset(RMAX + r)) = lo_word;
        if (lane == 0) factors[r] = factor;
    }
}

// Work list: (sequence, KV head, chunk) items, sequences in order; sequences
// whose context length is invalid get no items (the combine writes zeros).
__global__ void __launch_bounds__(1024) plan_items_kernel(TcArgs t, int32_t* first) {
    using Scan = cub::BlockScan<int32_t, 1024>;
    __shared__ typename Scan::TempStorage temp;
    __shared__ int32_t carry;
    const AttnArgs& a = t.a;
    if (threadIdx.x == 0) carry = 0;
    __syncthreads();
    for (int64_t base = 0; base < a.batch; base += 1024) {
        const int64_t b = base + threadIdx.x;
        int32_t n = 0;
        if (b < a.batch) {
            const int64_t T = __ldg(a.context_lens + b);
            const bool valid = T >= a.window && T <= a.table_stride * a.pool.block_size &&
                               T <= a.max_chunks * a.chunk;
            if (!valid) report_fault(a.status, SDC_FAULT_CONTEXT_RANGE);
            n = valid ? static_cast<int32_t>(((T + a.chunk - 1) / a.chunk) * a.kv_heads) : 0;
        }
        int32_t off, total;
        Scan(temp).ExclusiveSum(n, off, total);
        if (b < a.batch) first[b] = carry + off;
        __syncthreads();
        if (threadIdx.x == 0) carry += total;
        __syncthreads();
    }
    if (threadIdx.x == 0) *const_cast<int32_t*>(t.item_count) = carry;
    for (int64_t b = threadIdx.x; b < a.batch; b += blockDim.x) {
        const int64_t T = __ldg(a.context_lens + b);
        const bool valid = T >= a.window && T <= a.table_stride * a.pool.block_size && T <= a.max_chunks * a.chunk;
        if (!valid) continue;
        const int64_t chunks = (T + a.chunk - 1) / a.chunk;
        WorkItem* out = const_cast<WorkItem*>(t.items) + first[b];
        for (int64_t c = 0; c < chunks; ++c) {
            for (int64_t h = 0; h < a.kv_heads; ++h) {
                WorkItem w;
                w.b = static_cast<int32_t>(b);
                w.h = static_cast<int32_t>(h);
                w.t0 = static_cast<int32_t>(c * a.chunk);
                w.t1 = static_cast<int32_t>(min(T, (c + 1) * a.chunk));
                out[c * a.kv_heads + h] = w;
            }
        }
    }
}

// ---------------------------------------------------------------- host side

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static std::once_flag once;
    static EncodeTiledFn fn = nullptr;
    std::call_once(once, [] {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess) {
            fn = reinterpret_cast<EncodeTiledFn>(ptr);
        }
    });
    return fn;
}

bool make_page_map(CUtensorMap* map, const int8_t* codes, const Pool& p) {
    EncodeTiledFn fn = encode_fn();
    if (fn == nullptr) return false;
    const int64_t last = (p.num_blocks - 1) * p.cbs + (p.num_layers - 1) * p.cls + (p.num_heads - 1) * p.chs;
    const uint64_t rows = static_cast<uint64_t>(last / kHeadDim + p.block_size);
    if (rows > (uint64_t(1) << 32)) return false;
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(kHeadDim), static_cast<cuuint64_t>(rows)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(kHeadDim)};
    cuuint32_t box[2] = {static_cast<cuuint32_t>(kHeadDim), static_cast<cuuint32_t>(p.block_size)};
    cuuint32_t elem[2] = {1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<int8_t*>(codes), dims, strides, box, elem,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int rmax_for(int64_t rows) {
    if (rows <= 24) return 24;
    if (rows <= 40) return 40;
    return 0;
}


int num_sms() {
    static int sms = 0;
    if (sms == 0) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (sms <= 0) sms = 148;
    }
    return sms;
}

template <typename QT, int RMAX>
sdc_status_t launch_typed(const TcArgs& t, const CUtensorMap& kmap, const CUtensorMap& vmap, int32_t* first,
                          cudaStream_t st) {
    constexpr int STAGES = kStagesFor<RMAX>;
    constexpr int MINB = kMinBlocksFor<RMAX>;
    using LY = Layout<RMAX, STAGES>;
    const int64_t bh = t.a.batch * t.a.kv_heads;
    query_image_kernel<QT, RMAX><<<static_cast<unsigned>(bh), 256, 0, st>>>(t);
    plan_items_kernel<<<1, 1024, 0, st>>>(t, first);
    auto kernel = attn_tc_kernel<RMAX, STAGES, MINB>;
    static bool configured = false;
    if (!configured) {
        if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, LY::kDynamicSmem) !=
            cudaSuccess) {
            return SDC_STATUS_CUDA_ERROR;
        }
        configured = true;
    }
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kThreads, LY::kDynamicSmem) != cudaSuccess ||
        per_sm < 1) {
        return SDC_STATUS_CUDA_ERROR;
    }
    per_sm = per_sm > MINB ? MINB : per_sm;  // never more blocks per SM than tensor memory holds
    const int64_t max_items = bh * t.a.max_chunks;
    const int64_t grid = std::min<int64_t>(static_cast<int64_t>(num_sms()) * per_sm, max_items);
    kernel<<<static_cast<unsigned>(grid), kThreads, LY::kDynamicSmem, st>>>(kmap, vmap, t);
    return launch_status();
}

}  // namespace

bool shape_supported(int64_t head_dim, int64_t rows) { return head_dim == kHeadDim && rmax_for(rows) != 0; }

bool supports(const AttnArgs& a) {
    const Pool& p = a.pool;
    const int64_t bs = p.block_size;
    return p.head_dim == kHeadDim && rmax_for(a.rows) != 0 && bs >= 8 && bs <= kTile && (kTile % bs) == 0 &&
           p.cbs % kHeadDim == 0 && p.cls % kHeadDim == 0 && p.chs % kHeadDim == 0 && p.sbs % 4 == 0 &&
           p.sls % 4 == 0 && p.shs % 4 == 0 && (reinterpret_cast<uintptr_t>(p.key_scales) & 15) == 0 &&
           (reinterpret_cast<uintptr_t>(p.value_scales) & 15) == 0 && encode_fn() != nullptr;
}

int64_t chunk_for(int64_t batch, int64_t kv_heads, int64_t max_context_len) {
    // about four items per resident block when every sequence is at the
    // maximum length; a multiple of the tile
    const int64_t slots = static_cast<int64_t>(num_sms()) * 2 * 4;
    int64_t c = (batch * kv_heads * max_context_len + slots - 1) / slots;
    c = (c + kTile - 1) / kTile * kTile;
    if (c < 512) c = 512;
    if (c > 16384) c = 16384;
    return c;
}

size_t extra_workspace(int64_t batch, int64_t kv_heads, int64_t max_chunks, int64_t rows) {
    const int rmax = rmax_for(rows);
    const int64_t q_bytes = rmax == 24 ? Layout<24, kStagesFor<24>>::kQBytes : Layout<40, kStagesFor<40>>::kQBytes;
    const int64_t bh = batch * kv_heads;
    auto up = [](int64_t v) { return static_cast<size_t>((v + 255) / 256 * 256); };
    return up(bh * q_bytes) + up(bh * max_chunks * static_cast<int64_t>(sizeof(WorkItem))) + up(16) + up(batch * 4);
}

sdc_status_t launch(const AttnArgs& a, void* extra, cudaStream_t st) {
    const int rmax = rmax_for(a.rows);
    auto up = [](int64_t v) { return (v + 255) / 256 * 256; };
    const int64_t q_bytes = rmax == 24 ? Layout<24, kStagesFor<24>>::kQBytes : Layout<40, kStagesFor<40>>::kQBytes;
    const int64_t bh = a.batch * a.kv_heads;
    char* base = static_cast<char*>(extra);
    TcArgs t;
    t.a = a;
    t.qimg = reinterpret_cast<const uint8_t*>(base);
    t.q_bytes = static_cast<int32_t>(q_bytes);
    base += up(bh * q_bytes);
    t.items = reinterpret_cast<const WorkItem*>(base);
    base += up(bh * a.max_chunks * static_cast<int64_t>(sizeof(WorkItem)));
    t.item_count = reinterpret_cast<const int32_t*>(base);
    base += up(16);
    int32_t* first = reinterpret_cast<int32_t*>(base);
    t.rows = static_cast<int32_t>(a.rows);
    CUtensorMap kmap, vmap;
    if (!make_page_map(&kmap, a.pool.keys, a.pool) || !make_page_map(&vmap, a.pool.values, a.pool)) {
        return SDC_STATUS_CUDA_ERROR;
    }
    sdc_status_t rc;
    switch (a.query_dtype) {
        case SDC_DTYPE_BF16:
            rc = rmax == 24 ? launch_typed<__nv_bfloat16, 24>(t, kmap, vmap, first, st)
                            : launch_typed<__nv_bfloat16, 40>(t, kmap, vmap, first, st);
            break;
        case SDC_DTYPE_F16:
            rc = rmax == 24 ? launch_typed<__half, 24>(t, kmap, vmap, first, st)
                            : launch_typed<__half, 40>(t, kmap, vmap, first, st);
            break;
        case SDC_DTYPE_F32:
            rc = rmax == 24 ? launch_typed<float, 24>(t, kmap, vmap, first, st)
                            : launch_typed<float, 40>(t, kmap, vmap, first, st);
            break;
        default: return SDC_STATUS_UNSUPPORTED;
    }
    if (rc != SDC_STATUS_OK) return rc;
    return launch_attention_combine(a, st);
}

}  // namespace tc
}  // namespace sdc
