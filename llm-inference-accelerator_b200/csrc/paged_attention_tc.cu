// Kernel (c) on the 5th-generation tensor cores: paged verify attention with
// INT8 pages fed straight from TMA to tcgen05.mma (kind::i8), accumulators
// in tensor memory.  head_dim 64 or 128; any block size that divides 128
// (>= 8).
//
// Same computation and work decomposition as paged_attention.cu (split-K
// items of (sequence, KV head, chunk), un-normalised partials, a combine
// pass); what changes is how one item walks its chunk, 128 tokens per tile:
//
//   S^T[t, n] = sum_d K[t, d] * Qi8[n, d]      (M = 128 tokens, N columns)
//   O^T[d, n] = sum_t V[t, d] * Pi8[n, t]      (M = head_dim, same N)
//
// Query rows are split into two INT8 parts, q ~ s1 * (hi + lo / 254) with
// s1 = max|q| / 127 per row (columns [0, RB) hold hi, [RB, 2 RB) lo, RB = the
// row bucket), so the integer products are exact and a row's score is
// (254 S_hi + S_lo) * s1 / 254 * scale_k: 15 bits of relative precision,
// finer than the bf16 input.  Probabilities are split the same way after
// folding in the value scale: x = 127 p scale_v / max(scale_v) in [0, 127],
// hi = rint(x), lo = rint(254 (x - hi)), an absolute error below 1.6e-5 of
// the tile's largest weight.  K is the A operand in K-major form and V the A
// operand in MN-major form of the same page rows: every page goes from HBM
// to shared memory exactly once, one TMA box per page, and is never
// converted.
//
// The planning launch quantizes every (sequence, KV head)'s query rows once;
// items of the same pair share that image.  Warp roles of the item kernel
// (one block per SM, persistent over its items): G softmax warpgroups take
// the tiles in turn (tile g goes to warpgroup g % G, which owns S/P/O
// buffer g % G; a thread is a token row of S^T and a head_dim row of O^T,
// its TMEM lane), each with its own online softmax state; at the end of an
// item the warpgroup that took its last tile receives the others' states
// through tensor memory (each depositor writes its O sums into its own O
// buffer) and writes the result.  Four control warps follow the softmax
// warps: the key-code copies, the MMA issuer (which also allocates tensor
// memory), the value-code copies, and the scale / query-image copies.  With
// G = 3 the control warpgroup gives registers to the softmax warpgroups
// (setmaxnreg): the softmax chain of one tile is a long run of dependent
// steps, so a third warpgroup in flight hides its latency.
// Every mbarrier wait gives up after a bounded number of cycles (one second
// unless a test asks for less), records SDC_FAULT_WAIT_TIMEOUT in the
// status word, and lets the block wind down: it waits (bounded) for its own
// copies and MMAs, frees tensor memory and returns.  No named barriers: a
// warp that gives up can never strand another.

#include <cuda.h>

#include <atomic>
#include <cub/block/block_scan.cuh>
#include <mutex>

#include "host_common.h"
#include "paged_attention.h"

namespace sdc {
namespace tc {
namespace {

constexpr int kTile = 128;  // tokens per tile (MMA M for S^T)
constexpr float kRoundMagic = 12582912.0f;                  // 1.5 * 2^23
// A KV head's query rows (GQA group x window) beyond 32 are split over up
// to kMaxSplits items per chunk, each serving at most 32 rows.
constexpr int kMaxSplits = 2;
// Largest work item in tiles (the chunk size is clamped to 16384 tokens).
constexpr int kMaxItemTiles = 16384 / kTile;
// What starting a work item costs an SM, in tiles (chunk sizing for long
// contexts over few heads; measured on the 70B shards of one to eight GPUs).
constexpr int64_t kItemStartTiles = 4;
// Shared memory one block may use.
constexpr int kSmemLimit = 232448;

// Warp roles for G softmax warpgroups: warps [0, 4 G) run the softmax, then
// the four control warps.
template <int G>
struct Roles {
    static_assert(G == 2 || G == 3, "two or three softmax warpgroups");
    static constexpr int kKeyWarp = 4 * G;        // key codes of every page
    static constexpr int kMmaWarp = 4 * G + 1;    // tensor memory and the MMAs
    static constexpr int kValueWarp = 4 * G + 2;  // value codes of every page
    static constexpr int kScaleWarp = 4 * G + 3;  // key and value scales, query images
    static constexpr int kThreads = (4 * G + 4) * 32;
    // Register split with three softmax warpgroups: the block launches at
    // 128 registers a thread (65 536 in all); the control warpgroup drops
    // to 56 and the softmax warpgroups rise to 152:
    // 128 x 56 + 384 x 152 = 65 536, exactly the launch's registers (and
    // per SM sub-partition 56 + 3 x 152 = 512 a lane).
    static constexpr int kControlRegs = 56;
    static constexpr int kSoftmaxRegs = 152;
    static_assert(G != 3 || 128 * kControlRegs + 384 * kSoftmaxRegs == kThreads * 128, "register split");
};

// Layout of the kernel for RB query rows per item, head_dim HD (64 or 128)
// and G softmax warpgroups: HD is the MMA M of O^T and the K extent of S^T.
// A page row is HD bytes; key / value tiles use the 128-byte swizzle at HD
// 128 and the 64-byte swizzle at HD 64, which is also how TMA writes them.
// One query image (written by the planning launch, read by the item
// kernel): the codes of RB rows split into hi / lo parts, then the RB row
// factors; global images are kQStride bytes apart.
template <int RB, int HD>
struct QImage {
    static constexpr int N = ((2 * RB + 15) / 16) * 16;  // MMA N
    static constexpr int kQCodes = N * HD;
    static constexpr int kQCopyBytes = kQCodes + RB * 4;
    static constexpr int kQStride = ((kQCopyBytes + 127) / 128) * 128;
};

template <int RB, int HD, int G>
struct Rows {
    static_assert(HD == 64 || HD == 128, "head_dim 64 or 128");
    static constexpr int kCodeTileBytes = kTile * HD;                       // one K or V tile
    static constexpr int kStageBytes = 2 * kCodeTileBytes + 2 * kTile * 4;  // K, V codes + scales
    static constexpr uint32_t kSwizzle = HD == 128 ? 2u : 4u;  // descriptor layout: 128B / 64B swizzle
    static constexpr int N = QImage<RB, HD>::N;
    static constexpr int kQCodes = QImage<RB, HD>::kQCodes;
    static constexpr int kQCopyBytes = QImage<RB, HD>::kQCopyBytes;
    static constexpr int kQStride = QImage<RB, HD>::kQStride;
    static constexpr int kQBufBytes = ((kQCopyBytes + 1023) / 1024) * 1024;  // shared-memory buffer
    static constexpr int kPBytes = N * kTile;
    // P tiles per warpgroup: two let a warpgroup store P of its next tile
    // while the tensor core still reads the previous one; one leaves room
    // for the third warpgroup's buffers.
    static constexpr int kPBufs = G == 2 ? 2 : 1;
    static constexpr int kTmemStride = N <= 64 ? 64 : 128;  // columns per S / O buffer
    static constexpr int kTmemCols = 2 * G * kTmemStride <= 256 ? 256 : 512;  // S[G] then O[G]
    static_assert(2 * G * kTmemStride <= 512, "tensor memory columns");
    static constexpr int kRedStride = RB + 4;  // RB row maxima, the value-scale maximum, padding
    // shared memory after the stages, from a 1024-aligned base
    static constexpr int kQRel = 0;                                    // 2 query images
    static constexpr int kPRel = kQRel + 2 * kQBufBytes;               // [group][buffer] P tiles
    static constexpr int kRedRel = kPRel + G * kPBufs * kPBytes;       // [group][parity][warp][kRedStride]
    static constexpr int kWarpRel = kRedRel + G * 2 * 4 * kRedStride * 4;  // [warp][-m[RB], alpha[2][RB]]
    static constexpr int kMergeRel = kWarpRel + 4 * G * 3 * RB * 4;        // [group][RB][m, l]
    static constexpr int kBarRel = ((kMergeRel + G * RB * 8 + 7) / 8) * 8;
    static constexpr int kNumBars = 2 * 8 + 5 + 9 * G;  // stages (at most 8), query, stall, per-group barriers
    static constexpr int kMiscRel = kBarRel + kNumBars * 8;
    static constexpr int kCausalRel = kMiscRel + 16;  // [split][32] row masks of the causal window
    static constexpr int kTailBytes = kCausalRel + kMaxSplits * 32 * 4;
    // as many pipeline stages as fit (a stage holds one tile's pages)
    static constexpr int kFitStages = (kSmemLimit - 1024 - kTailBytes) / kStageBytes;
    static constexpr int kStages = kFitStages < (HD == 64 ? 8 : 5) ? kFitStages : (HD == 64 ? 8 : 5);
    static_assert(kStages >= 3, "pipeline depth");
    static constexpr int kStageOff = 0;
    static constexpr int kTailOff = kStages * kStageBytes;
    static constexpr int kQOff = kTailOff + kQRel;
    static constexpr int kPOff = kTailOff + kPRel;
    static constexpr int kRedOff = kTailOff + kRedRel;
    static constexpr int kWarpOff = kTailOff + kWarpRel;
    static constexpr int kMergeOff = kTailOff + kMergeRel;
    static constexpr int kBarOff = kTailOff + kBarRel;
    static constexpr int kMiscOff = kTailOff + kMiscRel;
    static constexpr int kCausalOff = kTailOff + kCausalRel;
    static constexpr int kDynamicSmem = kTailOff + kTailBytes + 1024;
    static_assert(kDynamicSmem <= kSmemLimit, "shared memory per block");
    static_assert(RB <= 32, "row masks are 32 bits");
    static_assert(RB % 4 == 0, "row factors fill whole 16-byte words");
};

// Softmax warpgroups of a bucket.  Three warpgroups (register split 152 /
// 56) were measured slower on the 8B verify shape (0.099 against 0.089 ms
// a call): each tile's softmax chain grew from 3 500 to 6 300 cycles, so the
// sub-partitions' pipes, not the chain's latency, bound the third
// warpgroup; two stay the default.
template <int RB, int HD>
constexpr int groups_for() {
    return 2;
}

// Bytes between two (sequence, KV head) query images for row bucket rb and
// head_dim hd.
constexpr int64_t query_image_stride(int rb, int hd) {
    return ((((2 * rb + 15) / 16) * 16 * hd + rb * 4 + 127) / 128) * 128;
}

// One unit of work: tokens [t0, t1) of sequence b (context length ctx) for
// query-row split `split` of KV head h; chunk = t0 / chunk size, the
// partial's slot.
struct __align__(32) WorkItem {
    int32_t b, h, t0, t1, ctx, chunk, split, pad;
};

struct TcArgs {
    AttnArgs a;
    const WorkItem* items;
    const int32_t* item_count;
    // per (sequence, KV head): the query rows split into INT8 hi / lo parts
    // in the score MMA's B layout, then the row factors (written by the
    // planning launch)
    unsigned char* qimg;
    int32_t rows;        // query rows per split (<= RB); the last split may hold fewer
    int32_t splits;      // row splits per KV head
    int32_t total_rows;  // query rows per KV head (group x window)
    int32_t gather4;     // scales fetched four pages per copy through the scale maps
    int32_t direct;      // one chunk per sequence: items write the output rows, no partials
    // Test hooks (sdc_test_attention_waits): cycles a pipeline wait may take
    // before it gives up, and a flag that makes the softmax warps wait on a
    // barrier nothing completes, so that wait gives up and the block winds
    // down through its error path.
    int32_t stall;
    long long wait_limit;
};

// ---------------------------------------------------------------- PTX helpers

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// Timeouts count SM clock cycles: reading the cycle counter is cheap, unlike
// the global nanosecond timer, so a spinning wait notices a completed phase
// at once.  2^31 cycles is about one second at B200 clocks.
constexpr long long kWaitLimitCycles = 1ll << 31;

__device__ __forceinline__ long long cycles() { return clock64(); }

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

// Non-blocking probe of a phase (polling loops).
__device__ __forceinline__ bool mbar_test(uint32_t bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(bar), "r"(parity)
        : "memory");
    return done != 0;
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
// aborting (this wait gave up after `limit` cycles, or another one already
// did).
__device__ __forceinline__ bool wait_phase(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                           int32_t* status, long long limit) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long start = cycles();
    while (true) {
        if (mbar_try_wait(bar, parity)) return true;
        if (*abort_flag) return false;
        if (cycles() - start > limit) {
            *abort_flag = 1;
            report_fault(status, SDC_FAULT_WAIT_TIMEOUT);
            return false;
        }
    }
}

// The same wait taken by a whole warp with one outcome: either every lane
// observed the phase (and so holds its acquire ordering) or all give up.
__device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag, int32_t* status,
                                          long long limit) {
    return __all_sync(kFullMask, wait_phase(bar, parity, abort_flag, status, limit));
}

// Wait used while winding down: bounded, ignores the abort flag.
__device__ __forceinline__ void drain_phase(uint32_t bar, uint32_t parity) {
    const long long start = cycles();
    while (!mbar_try_wait(bar, parity)) {
        if (cycles() - start > kWaitLimitCycles) return;
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

// Four rows of a 2-D map (box one row high) at independent row coordinates,
// stored back to back.
__device__ __forceinline__ void tma_gather4(uint32_t dst, const CUtensorMap* map, int32_t y0, int32_t y1, int32_t y2,
                                            int32_t y3, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile::gather4.mbarrier::complete_tx::bytes [%0], [%1, {%2, "
        "%3, %4, %5, %6}], [%7];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(0), "r"(y0), "r"(y1), "r"(y2), "r"(y3), "r"(bar)
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
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t* r) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}

template <int N>
__device__ __forceinline__ void tmem_ld_row(uint32_t taddr, uint32_t (&r)[N]) {
    static_assert(N % 16 == 0, "columns come in groups of 16");
#pragma unroll
    for (int c = 0; c < N; c += 16) tmem_ld16(taddr + c, r + c);
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Four consecutive 32-bit TMEM columns of this thread's lane, written from
// registers; tmem_st_wait orders them before a fence and a barrier.
__device__ __forceinline__ void tmem_st4(uint32_t taddr, uint32_t r0, uint32_t r1, uint32_t r2, uint32_t r3) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1, %2, %3, %4};" ::"r"(taddr), "r"(r0), "r"(r1),
                 "r"(r2), "r"(r3)
                 : "memory");
}

__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ float redux_max(float v) {
    float r;
    asm volatile("redux.sync.max.f32 %0, %1, 0xffffffff;" : "=f"(r) : "f"(v));
    return r;
}

__device__ __forceinline__ float fast_exp2(float x) {
    float r;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
    return r;
}

// Low bytes of four words packed into one word (byte i from w_i).
__device__ __forceinline__ uint32_t pack_low_bytes(uint32_t w0, uint32_t w1, uint32_t w2, uint32_t w3) {
    return __byte_perm(__byte_perm(w0, w1, 0x0040), __byte_perm(w2, w3, 0x0040), 0x5410);
}

// One output element in the query's dtype, in every destination of the call.
__device__ __forceinline__ void store_output(const AttnArgs& a, int64_t index, float v) {
    for (int i = 0; i < a.num_outs; ++i) {
        if (a.query_dtype == SDC_DTYPE_BF16) {
            static_cast<__nv_bfloat16*>(a.outs[i])[index] = __float2bfloat16_rn(v);
        } else if (a.query_dtype == SDC_DTYPE_F16) {
            static_cast<__half*>(a.outs[i])[index] = __float2half_rn(v);
        } else {
            static_cast<float*>(a.outs[i])[index] = v;
        }
    }
}

// ---------------------------------------------------------------- main kernel

template <int RB, int HD, int G>
__global__ void __launch_bounds__(Roles<G>::kThreads, 1)
    attn_tc_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap,
                   const __grid_constant__ CUtensorMap ksmap, const __grid_constant__ CUtensorMap vsmap, TcArgs t) {
    using LY = Rows<RB, HD, G>;
    using RO = Roles<G>;
    constexpr int N = LY::N;
    constexpr int STAGES = LY::kStages;
    constexpr int PB = LY::kPBufs;
    constexpr int kCodeTileBytes = LY::kCodeTileBytes;
    constexpr int kStageBytes = LY::kStageBytes;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char* smem =
        reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const AttnArgs& a = t.a;
    const long long limit = t.wait_limit;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    // launched programmatically after the planning launch: set up barriers
    // and tensor memory while it finishes, read its outputs only after
    // griddepcontrol.wait; the combine launch may start its own set-up now
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + LY::kBarOff);
    auto bar = [&](int i) { return smem_u32(bars + i); };
    // per-group barriers are indexed [group] (P tiles [group][buffer], the
    // exchange [group][parity])
    const int kvFull = 0, kvEmpty = STAGES, qFull = 2 * STAGES, qEmpty = qFull + 2, sFull = qEmpty + 2,
              sEmpty = sFull + G, pFull = sEmpty + G, oFull = pFull + G * PB, oEmpty = oFull + G, xch = oEmpty + G,
              mergeFull = xch + 2 * G, stallBar = mergeFull + G;
    static_assert(2 * STAGES + 5 + 7 * G + G * PB <= LY::kNumBars, "barrier slots");
    volatile uint32_t* tmem_base_slot = reinterpret_cast<volatile uint32_t*>(smem + LY::kMiscOff);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + LY::kMiscOff + 4);

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(bar(kvFull + s), 3);       // the three copy warps
            mbar_init(bar(kvEmpty + s), 1 + 4);  // MMA commit + the consuming warpgroup
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(bar(qFull + i), 1);
            mbar_init(bar(qEmpty + i), 1 + 4 * G);
        }
        for (int c = 0; c < G; ++c) {
            mbar_init(bar(sFull + c), 1);
            mbar_init(bar(sEmpty + c), 4);
            for (int b = 0; b < PB; ++b) mbar_init(bar(pFull + c * PB + b), 4);  // one arrival per warp
            mbar_init(bar(oFull + c), 1);
            mbar_init(bar(oEmpty + c), 4);
            mbar_init(bar(xch + 2 * c), 4);
            mbar_init(bar(xch + 2 * c + 1), 4);
            mbar_init(bar(mergeFull + c), 4);
        }
        mbar_init(bar(stallBar), 1);  // never completed: the test hook's wait
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (threadIdx.x < kMaxSplits * 32) {
        // causal[split][j]: the split's rows that a key j positions past the
        // last fully visible one stays visible to (query row q = group row *
        // window + i sees i >= j)
        const int sp = threadIdx.x >> 5, j = threadIdx.x & 31;
        uint32_t m = 0;
        for (int r = 0; r < t.rows; ++r) {
            const int q = sp * t.rows + r;
            if (q < t.total_rows && q % a.window >= j) m |= 1u << r;
        }
        reinterpret_cast<uint32_t*>(smem + LY::kCausalOff)[threadIdx.x] = m;
    }
    if (warp == RO::kMmaWarp) {
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
    asm volatile("griddepcontrol.wait;" ::: "memory");  // the work list and query images are written
    const int count = __ldg(t.item_count);
    // The work list is sorted by size, largest first; block c takes
    // positions c, 2 grid - 1 - c, 2 grid + c, ... (snake order), which
    // balances the blocks' total work.
    auto item_pos = [&](int k) -> int {
        const int grid = static_cast<int>(gridDim.x);
        return k * grid + ((k & 1) ? grid - 1 - static_cast<int>(blockIdx.x) : static_cast<int>(blockIdx.x));
    };

    const uint32_t stage_base = smem_u32(smem + LY::kStageOff);
    const uint32_t q_base = smem_u32(smem + LY::kQOff);
    const uint32_t p_base = smem_u32(smem + LY::kPOff);
    const int64_t bs = a.pool.block_size;
    const int pages_per_tile = static_cast<int>(kTile / bs);

    auto control_copies = [&]() {
        // ------------------------------------------------------------ copies
        // Three warps share the copies of a tile, each arriving on the
        // stage's full barrier with its own bytes: the key warp the key
        // codes and the value warp the value codes (lane j copies page j),
        // the scale warp the key and value scales (four pages per gather
        // when a tile holds a multiple of four pages) and, once per item,
        // the query image.
        const bool scale_side = warp == RO::kScaleWarp;
        const CUtensorMap* map = warp == RO::kValueWarp ? &vmap : &kmap;  // the scale warp uses neither
        const uint32_t code_dst = (warp == RO::kKeyWarp ? 0u : static_cast<uint32_t>(kCodeTileBytes)) +
                                  static_cast<uint32_t>(lane * bs * HD);
        const uint32_t code_bytes = static_cast<uint32_t>(bs * HD);
        const uint32_t scale_bytes = static_cast<uint32_t>(bs * 4);
        const int lg_bs = __ffs(static_cast<int>(bs)) - 1;  // block sizes are powers of two
        const bool gather = t.gather4 != 0;
        uint32_t g = 0, li = 0, q_issued = 0;
        WorkItem nxt = t.items[item_pos(0)];
        for (int k = 0, item = item_pos(0); item < count; ++k, item = item_pos(k), ++li) {
            const WorkItem it = nxt;
            if (item_pos(k + 1) < count) nxt = t.items[item_pos(k + 1)];
            if (scale_side) {
                const uint32_t qb = li & 1;
                if (!warp_wait(bar(qEmpty + qb), ((li >> 1) & 1) ^ 1, abort_flag, a.status, limit)) break;
                if (lane == 0) {
                    const int64_t image = (static_cast<int64_t>(it.b) * a.kv_heads + it.h) * t.splits + it.split;
                    mbar_arrive_expect_tx(bar(qFull + qb), LY::kQCopyBytes);
                    bulk_load(q_base + qb * LY::kQBufBytes, t.qimg + image * LY::kQStride, LY::kQCopyBytes,
                              bar(qFull + qb));
                }
                __syncwarp();
                ++q_issued;
            }
            const int32_t* table = a.block_tables + static_cast<int64_t>(it.b) * a.table_stride;
            const int64_t code_base = a.layer * a.pool.cls + it.h * a.pool.chs;
            const int64_t scale_base = a.layer * a.pool.sls + it.h * a.pool.shs;
            // a page's block id is fetched one tile ahead, so the table load
            // overlaps the wait for a free stage
            auto page_of = [&](int tile0) -> int64_t {
                const int page = (tile0 >> lg_bs) + lane;
                if (lane >= pages_per_tile || (page << lg_bs) >= it.t1) return -1;
                return __ldg(table + page);
            };
            int64_t next_blk = page_of(it.t0);
            bool stop = false;
            for (int tile0 = it.t0; tile0 < it.t1; tile0 += kTile, ++g) {
                const int64_t blk = next_blk;
                if (tile0 + kTile < it.t1) next_blk = page_of(tile0 + kTile);
                const uint32_t s = g % STAGES;
                if (!warp_wait(bar(kvEmpty + s), ((g / STAGES) & 1) ^ 1, abort_flag, a.status, limit)) {
                    stop = true;
                    break;
                }
                bool valid = lane < pages_per_tile && tile0 + (lane << lg_bs) < it.t1;
                if (valid && (blk < 0 || blk >= a.pool.num_blocks)) {
                    if (scale_side) report_fault(a.status, SDC_FAULT_BLOCK_RANGE);
                    valid = false;
                }
                const uint32_t mask = __ballot_sync(kFullMask, valid);
                const uint32_t st = stage_base + s * kStageBytes;
                if (!scale_side) {
                    if (lane == 0) mbar_arrive_expect_tx(bar(kvFull + s), __popc(mask) * code_bytes);
                    __syncwarp();
                    if (valid) {
                        const int32_t row = static_cast<int32_t>((blk * a.pool.cbs + code_base) / HD);
                        tma_load_2d(st + code_dst, map, 0, row, bar(kvFull + s));
                    }
                } else if (gather) {
                    // every group of four pages is copied whole; pages past
                    // the item read row 0 and are never used
                    const int32_t srow = valid ? static_cast<int32_t>((blk * a.pool.sbs + scale_base) >> lg_bs) : 0;
                    if (lane == 0) mbar_arrive_expect_tx(bar(kvFull + s), 2u * pages_per_tile * scale_bytes);
                    for (int q = 0; q < pages_per_tile; q += 4) {
                        const int32_t y0 = __shfl_sync(kFullMask, srow, q);
                        const int32_t y1 = __shfl_sync(kFullMask, srow, q + 1);
                        const int32_t y2 = __shfl_sync(kFullMask, srow, q + 2);
                        const int32_t y3 = __shfl_sync(kFullMask, srow, q + 3);
                        if (lane == 0) {
                            const uint32_t off = 2 * kCodeTileBytes + q * scale_bytes;
                            tma_gather4(st + off, &ksmap, y0, y1, y2, y3, bar(kvFull + s));
                            tma_gather4(st + off + kTile * 4, &vsmap, y0, y1, y2, y3, bar(kvFull + s));
                        }
                    }
                    __syncwarp();
                } else {
                    if (lane == 0) mbar_arrive_expect_tx(bar(kvFull + s), __popc(mask) * 2 * scale_bytes);
                    __syncwarp();
                    if (valid) {
                        const int64_t off = blk * a.pool.sbs + scale_base;
                        const uint32_t dst = st + 2 * kCodeTileBytes + lane * scale_bytes;
                        bulk_load(dst, a.pool.key_scales + off, scale_bytes, bar(kvFull + s));
                        bulk_load(dst + kTile * 4, a.pool.value_scales + off, scale_bytes, bar(kvFull + s));
                    }
                }
            }
            if (stop) break;
        }
        if (*abort_flag && lane == 0) {  // every copy issued has landed before the block exits
            for (uint32_t k = 0; k < STAGES && k < g; ++k) {
                const uint32_t gg = g - 1 - k;
                drain_phase(bar(kvFull + gg % STAGES), (gg / STAGES) & 1);
            }
            for (uint32_t k = 0; k < 2 && k < q_issued; ++k) {
                const uint32_t lq = q_issued - 1 - k;
                drain_phase(bar(qFull + (lq & 1)), (lq >> 1) & 1);
            }
        }
    };
    auto control_mma = [&]() {
        // ------------------------------------------------------------ MMA issuer
        // One thread issues both products as soon as their inputs are ready:
        // the score MMA of tile gs needs its stage, its S buffer (gs % G,
        // released once its warpgroup has read S of its previous tile) and
        // its item's query image; the P.V MMA of tile gp needs P of tile gp
        // and its O buffer.  Scores therefore run ahead of P.V instead of
        // queueing behind it.  Both waits are polled; the thread gives up
        // after the wait limit without progress.
        constexpr uint32_t kIdescS = idesc_i8(kTile, N, 0, 0);
        constexpr uint32_t kIdescO = idesc_i8(HD, N, 1, 1);
        if (lane == 0) {
            uint32_t gs = 0, gp = 0, li = 0;
            int k = 0;
            int item = item_pos(0);
            WorkItem it = t.items[item];
            WorkItem nxt = it;
            if (item_pos(1) < count) nxt = t.items[item_pos(1)];
            int tile0 = it.t0;
            bool s_done = false, q_ready = false;
            long long idle_since = cycles();
            while (true) {
                bool progress = false;
                if (!s_done) {
                    const uint32_t qb = li & 1;
                    const uint32_t s = gs % STAGES;
                    const uint32_t sb = gs % G;
                    if (!q_ready) q_ready = mbar_test(bar(qFull + qb), (li >> 1) & 1);
                    if (q_ready && mbar_test(bar(kvFull + s), (gs / STAGES) & 1) &&
                        mbar_test(bar(sEmpty + sb), ((gs / G) & 1) ^ 1)) {
                        tc_fence_after();
                        const uint32_t k_tile = stage_base + s * kStageBytes;
                        const uint32_t q_tile = q_base + qb * LY::kQBufBytes;
#pragma unroll
                        for (int ks = 0; ks < HD / 32; ++ks) {
                            const uint64_t da = smem_desc(k_tile + ks * 32, 16, 8 * HD, LY::kSwizzle);
                            const uint64_t db = smem_desc(q_tile + ks * 256, 128, 8 * HD, 0);
                            mma_i8(tmem + sb * LY::kTmemStride, da, db, kIdescS, ks > 0);
                        }
                        mma_commit(bar(sFull + sb));
                        ++gs;
                        progress = true;
                        tile0 += kTile;
                        if (tile0 >= it.t1) {  // the item's last tile: its query image is free once this lands
                            mma_commit(bar(qEmpty + qb));
                            item = item_pos(++k);
                            ++li;
                            q_ready = false;
                            if (item >= count) {
                                s_done = true;
                            } else {
                                it = nxt;
                                if (item_pos(k + 1) < count) nxt = t.items[item_pos(k + 1)];
                                tile0 = it.t0;
                            }
                        }
                    }
                }
                if (gp < gs) {
                    const uint32_t sb = gp % G;
                    const uint32_t use = gp / G;  // the warpgroup's own tile index
                    const uint32_t pb = use % PB;
                    const uint32_t s = gp % STAGES;
                    // P buffer pb of the owning warpgroup completes once per
                    // PB of its tiles, and its next phase needs this product
                    // complete, so the parity cannot be a phase behind
                    if (mbar_test(bar(pFull + sb * PB + pb), (use / PB) & 1) &&
                        mbar_test(bar(oEmpty + sb), (use & 1) ^ 1)) {
                        tc_fence_after();
                        const uint32_t v_tile = stage_base + s * kStageBytes + kCodeTileBytes;
                        const uint32_t p_tile = p_base + (sb * PB + pb) * LY::kPBytes;
#pragma unroll
                        for (int ks = 0; ks < kTile / 32; ++ks) {
                            const uint64_t da = smem_desc(v_tile + ks * 32 * HD, kCodeTileBytes, 8 * HD, LY::kSwizzle);
                            const uint64_t db = smem_desc(p_tile + ks * 512, 128, 2048, 0);
                            mma_i8(tmem + (G + sb) * LY::kTmemStride, da, db, kIdescO, ks > 0);
                        }
                        mma_commit(bar(oFull + sb));
                        mma_commit(bar(kvEmpty + s));
                        ++gp;
                        progress = true;
                    }
                } else if (s_done) {
                    break;
                }
                if (progress) {
                    idle_since = cycles();
                } else {
                    if (*abort_flag) break;
                    if (cycles() - idle_since > limit) {
                        *abort_flag = 1;
                        report_fault(a.status, SDC_FAULT_WAIT_TIMEOUT);
                        break;
                    }
                }
            }
            if (*abort_flag) {  // the MMAs issued have completed before tensor memory is freed
                if (gs > 0) drain_phase(bar(sFull + (gs - 1) % G), ((gs - 1) / G) & 1);
                if (gp > 0) drain_phase(bar(oFull + (gp - 1) % G), ((gp - 1) / G) & 1);
            }
        }
        __syncwarp();
    };
    auto softmax = [&]() {
        // ------------------------------------------------------------ softmax + O epilogue
        // Warpgroup `grp` takes the tiles with g % G == grp.  Per tile each
        // warp reduces its 32 tokens' row maxima (and value-scale maximum)
        // into shared memory; after the group's exchange (an mbarrier with one
        // arrival per warp) lanes r < RB of every warp resolve row r's new
        // running max and rescale factor and hand them to their warp through
        // the warp's own shared-memory row, read back four rows per load.
        // Exchange buffers are double-buffered by exchange parity: a buffer
        // is rewritten two exchanges later, by which time every warp of the
        // group has arrived at the exchange in between and so has finished
        // reading it.  Row quantities go two rows at a time through the
        // packed f32x2 arithmetic of sm_100.
        const int grp = warp >> 2;
        const int qw = warp & 3;            // lane quarter = TMEM lanes [32 qw, 32 qw + 32)
        const int tid = threadIdx.x & 127;  // token row of S^T
        // head_dim row of O^T held by this thread: at HD 128 row tid; at HD
        // 64 (an M = 64 product) rows 16 qw .. 16 qw + 15 sit in lanes 0-15
        // of each warp's lane quarter and lanes 16-31 hold none
        const bool o_row = HD == 128 || lane < 16;
        const int dcol = HD == 128 ? tid : qw * 16 + lane;
        const uint32_t lane_addr = static_cast<uint32_t>(qw * 32) << 16;
        const uint32_t s_col = grp * LY::kTmemStride;
        const uint32_t o_col = (G + grp) * LY::kTmemStride;
        constexpr int RS = LY::kRedStride;
        float* red = reinterpret_cast<float*>(smem + LY::kRedOff) + grp * 2 * 4 * RS;
        float* wrow = reinterpret_cast<float*>(smem + LY::kWarpOff) + warp * 3 * RB;  // -m[RB], alpha[2][RB]
        float* merge_ml = reinterpret_cast<float*>(smem + LY::kMergeOff);               // [group][RB][m, l]
        uint32_t g = 0, li = 0, xc = 0, own = 0;
        uint32_t deposits[G];  // states each warpgroup has handed over so far (every group counts all)
#pragma unroll
        for (int c = 0; c < G; ++c) deposits[c] = 0;
        const float2 magic2 = make_float2(kRoundMagic, kRoundMagic);
        const float2 neg_magic2 = make_float2(-kRoundMagic, -kRoundMagic);
        const float2 minus_one2 = make_float2(-1.0f, -1.0f);
        const float2 c254 = make_float2(254.0f, 254.0f);

        auto exchange = [&]() -> bool {
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(xch + grp * 2 + (xc & 1)));
            return warp_wait(bar(xch + grp * 2 + (xc & 1)), (xc >> 1) & 1, abort_flag, a.status, limit);
        };
        // Folds O^T of own tile k into the running sums:
        // o = o * alpha_k + (254 O_hi + O_lo) * vf_k.  The group's k-th use
        // of its O buffer has parity k & 1.  `release` hands the O buffer
        // back to the MMA issuer; the last tile of an item keeps it when the
        // group's state is handed over through it.
        auto epilogue = [&](uint32_t k, float vf, bool release, float2 (&o_acc)[RB / 2]) -> bool {
            if (!warp_wait(bar(oFull + grp), k & 1, abort_flag, a.status, limit)) return false;
            tc_fence_after();
            uint32_t oreg[N];
            tmem_ld_row<N>(tmem + lane_addr + o_col, oreg);
            tc_fence_before();
            __syncwarp();
            if (release && lane == 0) mbar_arrive(bar(oEmpty + grp));
            const float4* al4 = reinterpret_cast<const float4*>(wrow + RB + (k & 1) * RB);
            const float2 vf2 = make_float2(vf, vf);
#pragma unroll
            for (int r4 = 0; r4 < RB; r4 += 4) {
                const float4 al = al4[r4 / 4];
#pragma unroll
                for (int j = 0; j < 4; j += 2) {
                    const int r = r4 + j;
                    const float c0 = static_cast<float>(static_cast<int32_t>(oreg[r]) * 254 +
                                                        static_cast<int32_t>(oreg[RB + r]));
                    const float c1 = static_cast<float>(static_cast<int32_t>(oreg[r + 1]) * 254 +
                                                        static_cast<int32_t>(oreg[RB + r + 1]));
                    const float2 a2 = j == 0 ? make_float2(al.x, al.y) : make_float2(al.z, al.w);
                    o_acc[r / 2] = __ffma2_rn(make_float2(c0, c1), vf2, __fmul2_rn(o_acc[r / 2], a2));
                }
            }
            return true;
        };

        bool ok = true;
        if (t.stall) {
            // test hook: a wait nothing completes, which gives up after the
            // wait limit and winds the block down
            ok = warp_wait(bar(stallBar), 0, abort_flag, a.status, limit);
        }
        WorkItem nxt = t.items[item_pos(0)];
        for (int k = 0, item = item_pos(0); item < count && ok; ++k, item = item_pos(k), ++li) {
            const WorkItem it = nxt;
            if (item_pos(k + 1) < count) nxt = t.items[item_pos(k + 1)];
            const uint32_t qb = li & 1;
            if (!warp_wait(bar(qFull + qb), (li >> 1) & 1, abort_flag, a.status, limit)) break;
            const float* qfac = reinterpret_cast<const float*>(smem + LY::kQOff + qb * LY::kQBufBytes + LY::kQCodes);
            const float qf_lane = lane < RB ? qfac[lane] : 0.0f;
            const int64_t T = it.ctx;
            const int64_t window = a.window;
            const int row0 = it.split * t.rows;               // first query row of this item
            const int R = min(t.rows, t.total_rows - row0);   // its rows
            const uint32_t row_mask = R >= 32 ? 0xffffffffu : (1u << R) - 1u;
            const uint32_t* causal = reinterpret_cast<const uint32_t*>(smem + LY::kCausalOff) + it.split * 32;
            const uint32_t g0 = g;  // the block's tile counter at the item's first tile
            const uint32_t ntiles = static_cast<uint32_t>((it.t1 - it.t0 + kTile - 1) / kTile);
            // lane r < RB holds row r's running max of (score * log2 e); the
            // scores held per token are K-scaled, the query factor applied later
            float m_lane = -INFINITY;
            float2 l_thr[RB / 2], o_acc[RB / 2];
#pragma unroll
            for (int r = 0; r < RB / 2; ++r) {
                l_thr[r] = make_float2(0.0f, 0.0f);
                o_acc[r] = make_float2(0.0f, 0.0f);
            }
            bool have_prev = false;
            uint32_t prev_own = 0;
            float vf_prev = 0.0f;
            for (int tile0 = it.t0; tile0 < it.t1; tile0 += kTile, ++g) {
                if (static_cast<int>(g % G) != grp) continue;
                const uint32_t s = g % STAGES;
                if (!warp_wait(bar(sFull + grp), own & 1, abort_flag, a.status, limit) ||
                    !warp_wait(bar(kvFull + s), (g / STAGES) & 1, abort_flag, a.status, limit)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                uint32_t sreg[N];
                tmem_ld_row<N>(tmem + lane_addr + s_col, sreg);
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(bar(sEmpty + grp));

                const float* sc_ptr =
                    reinterpret_cast<const float*>(smem + LY::kStageOff + s * kStageBytes + 2 * kCodeTileBytes);
                const float kscale = sc_ptr[tid];
                float vscale = sc_ptr[kTile + tid];
                __syncwarp();
                if (lane == 0) mbar_arrive(bar(kvEmpty + s));

                // Full tiles (every token inside the item and visible to every
                // row) skip the masking; a query at window row i sees keys up
                // to T - window + i.
                const bool full = tile0 + kTile <= it.t1 && tile0 + kTile <= T - window + 1;
                uint32_t vis_mask = row_mask;
                if (!full) {
                    const int64_t tok = tile0 + tid;
                    if (tok >= it.t1) {
                        vis_mask = 0u;
                        vscale = 0.0f;
                    }
                    const int64_t past = tok - (T - window);  // > 0: inside the window
                    if (past > 0) {
                        vis_mask &= past < window ? causal[past] : 0u;
                    }
                }
                float sc[RB];
                float* red_x = red + (xc & 1) * 4 * RS;
#pragma unroll
                for (int r4 = 0; r4 < RB; r4 += 4) {
                    float wm[4];
#pragma unroll
                    for (int j = 0; j < 4; j += 2) {
                        const int r = r4 + j;
                        const float c0 = static_cast<float>(static_cast<int32_t>(sreg[r]) * 254 +
                                                            static_cast<int32_t>(sreg[RB + r]));
                        const float c1 = static_cast<float>(static_cast<int32_t>(sreg[r + 1]) * 254 +
                                                            static_cast<int32_t>(sreg[RB + r + 1]));
                        const float2 s2 = __fmul2_rn(make_float2(c0, c1), make_float2(kscale, kscale));
                        sc[r] = s2.x;
                        sc[r + 1] = s2.y;
                        if (!full) {
                            if (!((vis_mask >> r) & 1u)) sc[r] = -INFINITY;
                            if (!((vis_mask >> (r + 1)) & 1u)) sc[r + 1] = -INFINITY;
                        }
                        wm[j] = redux_max(sc[r]);
                        wm[j + 1] = redux_max(sc[r + 1]);
                    }
                    if (lane == 0) {
                        *reinterpret_cast<float4*>(red_x + qw * RS + r4) = make_float4(wm[0], wm[1], wm[2], wm[3]);
                    }
                }
                {
                    const float wv = redux_max(vscale);
                    if (lane == 0) red_x[qw * RS + RB] = wv;
                }
                if (!exchange()) {
                    ok = false;
                    break;
                }
                ++xc;
                // lane r resolves row r: tile max over the four warps (times
                // the query factor, which is >= 0 and so commutes with max),
                // new running max, and the rescale factor of the old sums
                if (lane < RB) {
                    float tmax = fmaxf(fmaxf(red_x[lane], red_x[RS + lane]),
                                       fmaxf(red_x[2 * RS + lane], red_x[3 * RS + lane]));
                    tmax = tmax == -INFINITY ? -INFINITY : tmax * qf_lane;
                    const float m_new = fmaxf(m_lane, tmax);
                    float alpha = 1.0f;
                    if (m_new > m_lane) alpha = m_lane == -INFINITY ? 0.0f : fast_exp2(m_lane - m_new);
                    m_lane = m_new;
                    wrow[lane] = -m_new;
                    wrow[RB + (own & 1) * RB + lane] = alpha;
                }
                const float vmax = fmaxf(fmaxf(red_x[RB], red_x[RS + RB]), fmaxf(red_x[2 * RS + RB], red_x[3 * RS + RB]));
                const float u_scale = vmax > 0.0f ? vscale * __fdividef(127.0f, vmax) : 0.0f;
                const float2 u2 = make_float2(u_scale, u_scale);
                const float vf_cur = vmax * (1.0f / (127.0f * 254.0f));
                __syncwarp();
                static_assert(RB % 4 == 0, "rows are packed four to a word");
                uint32_t words[N / 4];  // P^T row: hi bytes in columns [0, RB), lo in [RB, 2 RB)
#pragma unroll
                for (int w = 0; w < N / 4; ++w) words[w] = 0u;
                const float4* nm4 = reinterpret_cast<const float4*>(wrow);
                const float4* al4 = reinterpret_cast<const float4*>(wrow + RB + (own & 1) * RB);
                const float4* qf4 = reinterpret_cast<const float4*>(qfac);
#pragma unroll
                for (int r4 = 0; r4 < RB; r4 += 4) {
                    const float4 nm = nm4[r4 / 4];
                    const float4 al = al4[r4 / 4];
                    const float4 qf = qf4[r4 / 4];
                    uint32_t th_bits[4], tl_bits[4];
#pragma unroll
                    for (int j = 0; j < 4; j += 2) {
                        const int r = r4 + j;
                        const float2 nm2 = j == 0 ? make_float2(nm.x, nm.y) : make_float2(nm.z, nm.w);
                        const float2 al2 = j == 0 ? make_float2(al.x, al.y) : make_float2(al.z, al.w);
                        const float2 qf2 = j == 0 ? make_float2(qf.x, qf.y) : make_float2(qf.z, qf.w);
                        float2 e = __ffma2_rn(make_float2(sc[r], sc[r + 1]), qf2, nm2);
                        if (!full) {
                            if (sc[r] == -INFINITY) e.x = -INFINITY;
                            if (sc[r + 1] == -INFINITY) e.y = -INFINITY;
                        }
                        const float2 p = make_float2(fast_exp2(e.x), fast_exp2(e.y));
                        l_thr[r / 2] = __ffma2_rn(l_thr[r / 2], al2, p);
                        // x in [0, 127]: hi = rint(x), lo = rint(254 (x - hi)); adding
                        // 1.5 * 2^23 leaves the rounded integer in the low mantissa bits
                        const float2 x = __fmul2_rn(p, u2);
                        const float2 th = __fadd2_rn(x, magic2);
                        const float2 hi = __fadd2_rn(th, neg_magic2);
                        const float2 tl = __ffma2_rn(__ffma2_rn(hi, minus_one2, x), c254, magic2);
                        th_bits[j] = __float_as_uint(th.x);
                        th_bits[j + 1] = __float_as_uint(th.y);
                        tl_bits[j] = __float_as_uint(tl.x);
                        tl_bits[j + 1] = __float_as_uint(tl.y);
                    }
                    words[r4 / 4] = pack_low_bytes(th_bits[0], th_bits[1], th_bits[2], th_bits[3]);
                    words[(RB + r4) / 4] = pack_low_bytes(tl_bits[0], tl_bits[1], tl_bits[2], tl_bits[3]);
                }
                // With one P buffer the previous tile's product must have
                // read it: fold that tile first (its O wait covers the P
                // buffer).  With two, P of own tile k is written once this
                // warp's epilogue of own tile k - 2 has seen that product
                // complete, and the fold follows.
                if (PB == 1 && have_prev && !epilogue(prev_own, vf_prev, true, o_acc)) {
                    ok = false;
                    break;
                }
                // P^T row of this token in the MN-major no-swizzle layout: a
                // 128-byte core matrix holds 16 columns x 8 tokens; 8-token
                // groups are 128 bytes apart, 16-column groups 2048 apart.
                const uint32_t pbuf = grp * PB + (own % PB);
                unsigned char* prow = smem + LY::kPOff + pbuf * LY::kPBytes + (tid >> 3) * 128 + (tid & 7) * 16;
#pragma unroll
                for (int c = 0; c < N / 16; ++c) {
                    *reinterpret_cast<uint4*>(prow + c * 2048) =
                        make_uint4(words[4 * c], words[4 * c + 1], words[4 * c + 2], words[4 * c + 3]);
                }
                // every thread orders its P stores before the tensor core's
                // reads; the warp's lane 0 then arrives for all 32
                fence_proxy_async();
                __syncwarp();
                if (lane == 0) mbar_arrive(bar(pFull + pbuf));

                if (PB == 2 && have_prev && !epilogue(prev_own, vf_prev, true, o_acc)) {
                    ok = false;
                    break;
                }
                have_prev = true;
                prev_own = own;
                vf_prev = vf_cur;
                ++own;
            }
            if (!ok) break;
            // the warpgroup that took the item's last tile receives the
            // others' states; a depositor keeps its O buffer after its last
            // fold and writes its sums into it, and the receiver hands the
            // buffer back to the MMA issuer once it has read them
            const int receiver = static_cast<int>((g0 + ntiles - 1) % G);
            const bool is_receiver = grp == receiver;
            const bool had_tiles = have_prev;
            if (have_prev && !epilogue(prev_own, vf_prev, is_receiver, o_acc)) break;
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(qEmpty + qb));
            // this group's row sums over all its tokens: a transposing
            // reduction (each exchange halves the rows a lane carries) leaves
            // row `lane`'s warp sum in lane `lane`
            float* red_x = red + (xc & 1) * 4 * RS;
            {
                float x[32];
#pragma unroll
                for (int r = 0; r < 32; ++r) x[r] = r < RB ? ((r & 1) ? l_thr[r / 2].y : l_thr[r / 2].x) : 0.0f;
#pragma unroll
                for (int w = 16; w >= 1; w >>= 1) {
                    const bool upper = (lane & w) != 0;
#pragma unroll
                    for (int i = 0; i < w; ++i) {
                        const float send = upper ? x[i] : x[i + w];
                        const float keep = upper ? x[i + w] : x[i];
                        x[i] = keep + __shfl_xor_sync(kFullMask, send, w);
                    }
                }
                if (lane < RB) red_x[qw * RS + lane] = x[0];
            }
            if (!exchange()) break;
            ++xc;
            float l_lane = 0.0f;
            if (lane < RB) {
                l_lane = red_x[lane] + red_x[RS + lane] + red_x[2 * RS + lane] + red_x[3 * RS + lane];
            }
            const uint32_t holders = ntiles < static_cast<uint32_t>(G) ? ntiles : static_cast<uint32_t>(G);
            if (!is_receiver) {
                if (had_tiles) {
                    // deposit: O sums into columns [0, RB) of this group's O
                    // buffer (this thread's lane), (m, l) per row into shared memory
                    const uint32_t dst = tmem + lane_addr + o_col;
#pragma unroll
                    for (int r = 0; r < RB; r += 4) {
                        tmem_st4(dst + r, __float_as_uint(o_acc[r / 2].x), __float_as_uint(o_acc[r / 2].y),
                                 __float_as_uint(o_acc[r / 2 + 1].x), __float_as_uint(o_acc[r / 2 + 1].y));
                    }
                    tmem_st_wait();
                    if (qw == 0 && lane < RB) {
                        merge_ml[(grp * RB + lane) * 2 + 0] = m_lane;
                        merge_ml[(grp * RB + lane) * 2 + 1] = l_lane;
                    }
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(bar(mergeFull + grp));
                }
            } else {
                bool merged = true;
                for (uint32_t i = 0; i < holders; ++i) {
                    const int c = static_cast<int>((g0 + i) % G);
                    if (c == grp) continue;
                    if (!warp_wait(bar(mergeFull + c), deposits[c] & 1, abort_flag, a.status, limit)) {
                        merged = false;
                        break;
                    }
                    tc_fence_after();
                    uint32_t dep[(RB + 15) / 16 * 16];
                    tmem_ld_row<(RB + 15) / 16 * 16>(tmem + lane_addr + (G + c) * LY::kTmemStride, dep);
                    float e0_lane = 0.0f, e1_lane = 0.0f;
                    if (lane < RB) {
                        const float m1 = merge_ml[(c * RB + lane) * 2 + 0];
                        const float l1 = merge_ml[(c * RB + lane) * 2 + 1];
                        const float m_tot = fmaxf(m_lane, m1);
                        if (m_tot != -INFINITY) {
                            e0_lane = m_lane == -INFINITY ? 0.0f : fast_exp2(m_lane - m_tot);
                            e1_lane = m1 == -INFINITY ? 0.0f : fast_exp2(m1 - m_tot);
                        }
                        l_lane = l_lane * e0_lane + l1 * e1_lane;
                        m_lane = m_tot;
                    }
                    // the deposit is read: group c's O buffer goes back to the MMA issuer
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(bar(oEmpty + c));
#pragma unroll
                    for (int r = 0; r < RB; r += 2) {
                        const float a0 = __shfl_sync(kFullMask, e0_lane, r);
                        const float a1 = __shfl_sync(kFullMask, e0_lane, r + 1);
                        const float b0 = __shfl_sync(kFullMask, e1_lane, r);
                        const float b1 = __shfl_sync(kFullMask, e1_lane, r + 1);
                        o_acc[r / 2] = __ffma2_rn(make_float2(__uint_as_float(dep[r]), __uint_as_float(dep[r + 1])),
                                                  make_float2(b0, b1), __fmul2_rn(o_acc[r / 2], make_float2(a0, a1)));
                    }
                }
                if (!merged) break;
                if (t.direct) {
                    // every item covers its sequence's whole context: it writes
                    // the normalised output rows itself (no partial, no combine);
                    // the row factors are gathered first so the stores issue
                    // back to back, and the dtype is branched on once
                    const float inv_lane = l_lane > 0.0f ? 1.0f / l_lane : 0.0f;
                    float v[RB];
#pragma unroll
                    for (int r = 0; r < RB; ++r) {
                        v[r] = ((r & 1) ? o_acc[r / 2].y : o_acc[r / 2].x) * __shfl_sync(kFullMask, inv_lane, r);
                    }
                    if (o_row) {
                        // every destination: the caller's buffer, or each rank's
                        // gathered output (stores to another GPU made visible
                        // system-wide before the completion signal)
                        const int64_t e0 = out_rows_offset(a, it.b, it.h) + row0 * HD + dcol;
                        for (int i = 0; i < a.num_outs; ++i) {
                            if (a.query_dtype == SDC_DTYPE_BF16) {
                                __nv_bfloat16* out = static_cast<__nv_bfloat16*>(a.outs[i]) + e0;
#pragma unroll
                                for (int r = 0; r < RB; ++r) {
                                    if (r < R) out[r * HD] = __float2bfloat16_rn(v[r]);
                                }
                            } else if (a.query_dtype == SDC_DTYPE_F16) {
                                __half* out = static_cast<__half*>(a.outs[i]) + e0;
#pragma unroll
                                for (int r = 0; r < RB; ++r) {
                                    if (r < R) out[r * HD] = __float2half_rn(v[r]);
                                }
                            } else {
                                float* out = static_cast<float*>(a.outs[i]) + e0;
#pragma unroll
                                for (int r = 0; r < RB; ++r) {
                                    if (r < R) out[r * HD] = v[r];
                                }
                            }
                        }
                        if (a.num_outs > 1) __threadfence_system();
                    }
                } else {
                    const int64_t bh = static_cast<int64_t>(it.b) * a.kv_heads + it.h;
                    const int64_t chunk = it.chunk;
                    float* part_o = a.part_o + ((bh * a.max_chunks + chunk) * t.total_rows + row0) * HD;
                    float* part_ml = a.part_ml + ((bh * a.max_chunks + chunk) * t.total_rows + row0) * 2;
#pragma unroll
                    for (int r = 0; r < RB; ++r) {
                        const float o0 = (r & 1) ? o_acc[r / 2].y : o_acc[r / 2].x;
                        if (r < R && o_row) part_o[r * HD + dcol] = o0;
                    }
                    if (qw == 0 && lane < R) {
                        part_ml[2 * lane + 0] = m_lane;
                        part_ml[2 * lane + 1] = l_lane;
                    }
                }
            }
            // every group counts the item's hand-overs
            for (uint32_t i = 0; i < holders; ++i) {
                const int c = static_cast<int>((g0 + i) % G);
                if (c != receiver) ++deposits[c];
            }
        }
    };

    if (static_cast<int>(blockIdx.x) >= count) {
        // no item for this block: straight to the teardown
    } else if (warp >= 4 * G) {
        // the control warpgroup; with three softmax warpgroups its registers
        // go to them (every warp of a warpgroup takes the same setmaxnreg)
        if constexpr (G == 3) asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(RO::kControlRegs));
        if (warp == RO::kMmaWarp) {
            control_mma();
        } else {
            control_copies();
        }
    } else {
        if constexpr (G == 3) asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(RO::kSoftmaxRegs));
        softmax();
    }

    // ------------------------------------------------------------ teardown
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == RO::kMmaWarp) {
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "n"(LY::kTmemCols)
                     : "memory");
    }
}

// Planning launch.  Block 0 writes the work list: (sequence, KV head, chunk,
// row split) items sorted by size, largest first; sequences whose context
// length is invalid get no items (the combine writes zeros).  Every other block quantizes query
// rows, one warp per (sequence, KV head, row): each row splits into INT8
// hi / lo parts written in the score MMA's B layout (K-major, no swizzle:
// 8 rows x 16 bytes per 128-byte core matrix, 16-byte K chunks 128 bytes
// apart, 8-row groups 8 x HD bytes apart), and its factor s1 / 254 * qk_scale.
// Rows past `rows`, and the padding rows of the MMA's N, are zero.  At HD
// 64 lanes 16-31 of a row's warp hold no elements.
template <int RB, int HD>
__global__ void __launch_bounds__(256) prep_kernel(TcArgs t, int32_t* first) {
    static_assert(kMaxItemTiles < 256, "one scan thread per size bin");
    using LY = QImage<RB, HD>;
    const AttnArgs& a = t.a;
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");  // the item kernel may start its set-up
    if (blockIdx.x > 0) {
        const int lane = threadIdx.x & 31;
        const int64_t w = static_cast<int64_t>(blockIdx.x - 1) * (blockDim.x >> 5) + (threadIdx.x >> 5);
        const int64_t image = w / RB;  // (sequence, KV head, split)
        const int r = static_cast<int>(w - image * RB);
        if (image >= a.batch * a.kv_heads * t.splits) return;
        const int64_t bh = image / t.splits;
        const int64_t row = (image - bh * t.splits) * t.rows + r;  // query row within the KV head
        const int64_t b = bh / a.kv_heads;
        const int64_t h = bh - b * a.kv_heads;
        unsigned char* img = t.qimg + image * LY::kQStride;
        const int d = lane * 4;
        const bool has_d = d < HD;
        {
            // a sequence whose context length is invalid gets no items: its
            // output rows are zero
            const int64_t T = __ldg(a.context_lens + b);
            const bool valid = T >= a.window && T <= a.table_stride * a.pool.block_size && T <= a.max_chunks * a.chunk;
            if (!valid && has_d && r < t.rows && row < t.total_rows) {
                const int64_t e0 = out_rows_offset(a, b, h) + row * HD + d;
                for (int i = 0; i < 4; ++i) store_output(a, e0 + i, 0.0f);
                if (a.num_outs > 1) __threadfence_system();
            }
        }
        float x[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        if (has_d && r < t.rows && row < t.total_rows) {
            const int64_t e = ((b * a.query_heads + h * a.group) * a.window + row) * HD + d;
            if (a.query_dtype == SDC_DTYPE_BF16) {
                const uint2 v = __ldg(reinterpret_cast<const uint2*>(static_cast<const __nv_bfloat16*>(a.query) + e));
                x[0] = __uint_as_float(v.x << 16);
                x[1] = __uint_as_float(v.x & 0xffff0000u);
                x[2] = __uint_as_float(v.y << 16);
                x[3] = __uint_as_float(v.y & 0xffff0000u);
            } else if (a.query_dtype == SDC_DTYPE_F16) {
                const uint2 v = __ldg(reinterpret_cast<const uint2*>(static_cast<const __half*>(a.query) + e));
                const float2 lo = __half22float2(*reinterpret_cast<const __half2*>(&v.x));
                const float2 hi = __half22float2(*reinterpret_cast<const __half2*>(&v.y));
                x[0] = lo.x;
                x[1] = lo.y;
                x[2] = hi.x;
                x[3] = hi.y;
            } else {
                const float4 v = __ldg(reinterpret_cast<const float4*>(static_cast<const float*>(a.query) + e));
                x[0] = v.x;
                x[1] = v.y;
                x[2] = v.z;
                x[3] = v.w;
            }
        }
        float m = fmaxf(fmaxf(fabsf(x[0]), fabsf(x[1])), fmaxf(fabsf(x[2]), fabsf(x[3])));
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(kFullMask, m, off));
        uint32_t hi_word = 0, lo_word = 0;
        float factor = 0.0f;
        if (m > 0.0f) {
            const float s1 = m / 127.0f;
            const float inv = 1.0f / s1;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float hi = fminf(fmaxf(rintf(x[i] * inv), -127.0f), 127.0f);
                const float lo = fminf(fmaxf(rintf((x[i] - hi * s1) * (254.0f * inv)), -127.0f), 127.0f);
                hi_word |= (static_cast<uint32_t>(static_cast<int>(hi)) & 0xffu) << (8 * i);
                lo_word |= (static_cast<uint32_t>(static_cast<int>(lo)) & 0xffu) << (8 * i);
            }
            factor = s1 / 254.0f * a.qk_scale;
        }
        auto offset = [&](int n) { return (n >> 3) * (8 * HD) + (d >> 4) * 128 + (n & 7) * 16 + (d & 15); };
        if (has_d) {
            *reinterpret_cast<uint32_t*>(img + offset(r)) = hi_word;
            *reinterpret_cast<uint32_t*>(img + offset(RB + r)) = lo_word;
            if (2 * RB + r < LY::N) *reinterpret_cast<uint32_t*>(img + offset(2 * RB + r)) = 0u;
        }
        if (lane == 0) reinterpret_cast<float*>(img + LY::kQCodes)[r] = factor;
        return;
    }

    // Work list sorted by size (tiles per item), largest first: a counting
    // sort over the at most kMaxItemTiles + 1 sizes.  A chunk's row splits
    // take adjacent positions, so they run on neighbouring SMs at about the
    // same time and the second reads its pages from L2.
    __shared__ int32_t hist[kMaxItemTiles + 1];
    for (int i = threadIdx.x; i <= kMaxItemTiles; i += blockDim.x) hist[i] = 0;
    __syncthreads();
    auto valid_len = [&](int64_t T) {
        return T >= a.window && T <= a.table_stride * a.pool.block_size && T <= a.max_chunks * a.chunk;
    };
    auto tiles_of = [&](int64_t T, int64_t c) {
        return static_cast<int>((min(T, (c + 1) * a.chunk) - c * a.chunk + kTile - 1) / kTile);
    };
    const int per_chunk = static_cast<int>(a.kv_heads) * t.splits;
    // one thread per (sequence, chunk); the trip count is uniform across the
    // block so every lane takes part in the warp-aggregated position counts
    const int lane = threadIdx.x & 31;
    const int64_t pairs = a.batch * a.max_chunks;
    const int64_t span = (pairs + blockDim.x - 1) / blockDim.x * blockDim.x;
    auto chunk_tiles = [&](int64_t i, int64_t& b, int64_t& c, int64_t& T) -> int {
        if (i >= pairs) return -1;
        b = i / a.max_chunks;
        c = i - b * a.max_chunks;
        T = __ldg(a.context_lens + b);
        if (!valid_len(T)) {
            if (c == 0) report_fault(a.status, SDC_FAULT_CONTEXT_RANGE);
            return -1;
        }
        return c * a.chunk < T ? tiles_of(T, c) : -1;
    };
    // adds `amount` to bin `key` (>= 0) for every lane of the warp that
    // shares it with one atomic, returning this lane's own start position
    auto add_to_bin = [&](int key, int32_t amount) -> int32_t {
        const unsigned peers = __match_any_sync(kFullMask, key);
        const int leader = __ffs(peers) - 1;
        int32_t base = 0;
        if (key >= 0 && lane == leader) base = atomicAdd(&hist[key], amount * __popc(peers));
        base = __shfl_sync(kFullMask, base, leader);
        return base + __popc(peers & ((1u << lane) - 1u)) * amount;
    };
    for (int64_t i = threadIdx.x; i < span; i += blockDim.x) {
        int64_t b = 0, c = 0, T = 0;
        add_to_bin(chunk_tiles(i, b, c, T), per_chunk);
    }
    __syncthreads();
    {  // bin start positions, largest size first: thread i owns bin kMaxItemTiles - i
        using Scan = cub::BlockScan<int32_t, 256>;
        __shared__ typename Scan::TempStorage scan_tmp;
        const int bin = kMaxItemTiles - static_cast<int>(threadIdx.x);
        const int32_t n = bin >= 1 ? hist[bin] : 0;
        int32_t start = 0, total = 0;
        Scan(scan_tmp).ExclusiveSum(n, start, total);
        if (bin >= 1) hist[bin] = start;
        if (threadIdx.x == 0) *const_cast<int32_t*>(t.item_count) = total;
    }
    __syncthreads();
    for (int64_t i = threadIdx.x; i < span; i += blockDim.x) {
        int64_t b = 0, c = 0, T = 0;
        const int tiles = chunk_tiles(i, b, c, T);
        const int32_t pos = add_to_bin(tiles, per_chunk);
        if (tiles < 0) continue;
        for (int64_t h = 0; h < a.kv_heads; ++h) {
            for (int sp = 0; sp < t.splits; ++sp) {
                WorkItem w;
                w.b = static_cast<int32_t>(b);
                w.h = static_cast<int32_t>(h);
                w.t0 = static_cast<int32_t>(c * a.chunk);
                w.t1 = static_cast<int32_t>(min(T, (c + 1) * a.chunk));
                w.ctx = static_cast<int32_t>(T);
                w.chunk = static_cast<int32_t>(c);
                w.split = sp;
                w.pad = 0;
                const_cast<WorkItem*>(t.items)[pos + h * t.splits + sp] = w;
            }
        }
    }
    (void)first;
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

// 2-D map over the pool's codes as rows of head_dim bytes; one box = one
// page (block_size rows), swizzled (128-byte rows: 128B, 64-byte rows: 64B)
// to match the MMA operand layout.
bool make_page_map(CUtensorMap* map, const int8_t* codes, const Pool& p) {
    EncodeTiledFn fn = encode_fn();
    if (fn == nullptr) return false;
    const int64_t hd = p.head_dim;
    const int64_t last = (p.num_blocks - 1) * p.cbs + (p.num_layers - 1) * p.cls + (p.num_heads - 1) * p.chs;
    const uint64_t rows = static_cast<uint64_t>(last / hd + p.block_size);
    if (rows > (uint64_t(1) << 31)) return false;
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(hd), static_cast<cuuint64_t>(rows)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(hd)};
    cuuint32_t box[2] = {static_cast<cuuint32_t>(hd), static_cast<cuuint32_t>(p.block_size)};
    cuuint32_t elem[2] = {1, 1};
    const CUtensorMapSwizzle swizzle = hd == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<int8_t*>(codes), dims, strides, box, elem,
              CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// 2-D map over a scale array as rows of block_size floats (one page's
// scales); one box = one row, read four rows at a time by tile::gather4.
// Needs every page's scales to start on a row boundary.
bool make_scale_map(CUtensorMap* map, const float* scales, const Pool& p) {
    EncodeTiledFn fn = encode_fn();
    if (fn == nullptr) return false;
    const int64_t bs = p.block_size;
    if (p.sbs % bs || p.sls % bs || p.shs % bs) return false;
    const int64_t last = (p.num_blocks - 1) * p.sbs + (p.num_layers - 1) * p.sls + (p.num_heads - 1) * p.shs;
    const uint64_t rows = static_cast<uint64_t>(last / bs + 1);
    if (rows > (uint64_t(1) << 31)) return false;
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(bs), static_cast<cuuint64_t>(rows)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(bs * 4)};
    cuuint32_t box[2] = {static_cast<cuuint32_t>(bs), 1};
    cuuint32_t elem[2] = {1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(scales), dims, strides, box, elem,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_64B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Row buckets with a compiled kernel; rows are padded up to the bucket.
int bucket_for(int64_t rows) {
    if (rows <= 0) return 0;
    if (rows <= 8) return 8;
    if (rows <= 16) return 16;
    if (rows <= 20) return 20;
    if (rows <= 24) return 24;
    if (rows <= 32) return 32;
    return 0;
}

// Query-row splits of a KV head's rows, and rows per split.
int64_t splits_for(int64_t rows) { return (rows + 31) / 32; }
int64_t split_rows(int64_t rows) {
    const int64_t sp = splits_for(rows);
    return sp > 0 ? (rows + sp - 1) / sp : 0;
}

int num_sms() { return device_sms(); }

// Test hooks of the pipeline waits (sdc_test_attention_waits): the limit in
// cycles and the stall flag that the next launches carry.
std::atomic<long long> g_wait_limit{kWaitLimitCycles};
std::atomic<int> g_stall{0};

// The item kernel's shared-memory opt-in is a per-device function attribute:
// set it once on every device that launches the kernel.
template <typename Kernel>
bool raise_smem_limit(Kernel kernel, int bytes, std::atomic<uint64_t>& done) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return false;
    const uint64_t bit = dev < 64 ? (uint64_t(1) << dev) : 0;
    if (bit != 0 && (done.load(std::memory_order_acquire) & bit)) return true;
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess) return false;
    if (bit != 0) done.fetch_or(bit, std::memory_order_acq_rel);
    return true;
}

template <int RB, int HD>
sdc_status_t launch_bucket(const TcArgs& t, const CUtensorMap& kmap, const CUtensorMap& vmap,
                           const CUtensorMap& ksmap, const CUtensorMap& vsmap, int32_t* first, cudaStream_t st) {
    constexpr int G = groups_for<RB, HD>();
    using LY = Rows<RB, HD, G>;
    const int64_t query_warps = t.a.batch * t.a.kv_heads * t.splits * RB;
    prep_kernel<RB, HD><<<static_cast<unsigned>(1 + (query_warps + 7) / 8), 256, 0, st>>>(t, first);
    auto kernel = attn_tc_kernel<RB, HD, G>;
    static std::atomic<uint64_t> configured{0};
    if (!raise_smem_limit(kernel, LY::kDynamicSmem, configured)) return SDC_STATUS_CUDA_ERROR;
    const int64_t max_items = t.a.batch * t.a.kv_heads * t.a.max_chunks * t.splits;
    const int64_t grid = std::min<int64_t>(num_sms(), max_items);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(grid));
    cfg.blockDim = dim3(Roles<G>::kThreads);
    cfg.dynamicSmemBytes = LY::kDynamicSmem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, kernel, kmap, vmap, ksmap, vsmap, t) != cudaSuccess) return SDC_STATUS_CUDA_ERROR;
    return launch_status();
}

}  // namespace

bool shape_supported(int64_t head_dim, int64_t rows) {
    return (head_dim == 64 || head_dim == 128) && rows >= 1 && splits_for(rows) <= kMaxSplits && bucket_for(split_rows(rows)) != 0;
}

bool supports(const AttnArgs& a) {
    const Pool& p = a.pool;
    const int64_t bs = p.block_size;
    return shape_supported(p.head_dim, a.rows) && bs >= 8 && bs <= kTile && (kTile % bs) == 0 &&
           p.cbs % p.head_dim == 0 && p.cls % p.head_dim == 0 && p.chs % p.head_dim == 0 && p.sbs % 4 == 0 &&
           p.sls % 4 == 0 && p.shs % 4 == 0 && (reinterpret_cast<uintptr_t>(p.key_scales) & 15) == 0 &&
           (reinterpret_cast<uintptr_t>(p.value_scales) & 15) == 0 && encode_fn() != nullptr;
}

int64_t chunk_for(int64_t batch, int64_t kv_heads, int64_t max_context_len, int64_t rows) {
    const int64_t sms = static_cast<int64_t>(num_sms());
    const int64_t pairs = batch * kv_heads * splits_for(rows);
    // Fewer (sequence, KV head, row split) pairs than SMs: long contexts over
    // few heads (a KV-head shard).  Every pair is taken to be at the maximum
    // length, and the number of chunks per pair is the one whose busiest SM
    // finishes first: ceil(pairs x n / SMs) items of ceil(tiles / n) tiles,
    // each item's start counted as kItemStartTiles tiles.  (Four items per
    // SM, the rule below, leaves some SMs a fifth item whenever the item
    // count is not a multiple of the SM count.)
    if (pairs < sms) {
        const int64_t tiles = (max_context_len + kTile - 1) / kTile;
        int64_t best_n = 0, best_cost = 0;
        for (int64_t n = 1; n <= 256; ++n) {
            const int64_t per = (tiles + n - 1) / n;
            if (per > kMaxItemTiles) continue;
            if (per * kTile < 512 && n > 1) break;
            const int64_t cost = ((pairs * n + sms - 1) / sms) * (per + kItemStartTiles);
            if (best_n == 0 || cost < best_cost) {
                best_n = n;
                best_cost = cost;
            }
        }
        if (best_n > 0) return ((tiles + best_n - 1) / best_n) * kTile;
    }
    // otherwise about four items per SM when every sequence is at the
    // maximum length; a multiple of the tile
    const int64_t slots = sms * 4;
    int64_t c = (batch * kv_heads * splits_for(rows) * max_context_len + slots - 1) / slots;
    c = (c + kTile - 1) / kTile * kTile;
    if (c < 512) c = 512;
    if (c > kMaxItemTiles * kTile) c = kMaxItemTiles * kTile;
    // with at least two (sequence, KV head) items per SM, whole contexts
    // balance well enough and need no combine
    if (pairs >= 2 * sms && max_context_len <= kMaxItemTiles * kTile) {
        c = (max_context_len + kTile - 1) / kTile * kTile;
    }
    return c;
}

size_t extra_workspace(int64_t batch, int64_t kv_heads, int64_t max_chunks, int64_t rows) {
    auto up = [](int64_t v) { return static_cast<size_t>((v + 255) / 256 * 256); };
    const int64_t sp = splits_for(rows);
    return up(batch * kv_heads * max_chunks * sp * static_cast<int64_t>(sizeof(WorkItem))) + up(16) +
           up(batch * 4) + up(batch * kv_heads * sp * query_image_stride(bucket_for(split_rows(rows)), 128));
}

sdc_status_t launch(const AttnArgs& a, void* extra, cudaStream_t st) {
    auto up = [](int64_t v) { return (v + 255) / 256 * 256; };
    char* base = static_cast<char*>(extra);
    TcArgs t;
    t.a = a;
    t.splits = static_cast<int32_t>(splits_for(a.rows));
    t.rows = static_cast<int32_t>(split_rows(a.rows));
    t.total_rows = static_cast<int32_t>(a.rows);
    t.direct = a.max_chunks == 1 ? 1 : 0;
    t.stall = g_stall.load(std::memory_order_relaxed);
    t.wait_limit = g_wait_limit.load(std::memory_order_relaxed);
    t.items = reinterpret_cast<const WorkItem*>(base);
    base += up(a.batch * a.kv_heads * a.max_chunks * t.splits * static_cast<int64_t>(sizeof(WorkItem)));
    t.item_count = reinterpret_cast<const int32_t*>(base);
    base += up(16);
    int32_t* first = reinterpret_cast<int32_t*>(base);
    base += up(a.batch * 4);
    t.qimg = reinterpret_cast<unsigned char*>(base);
    CUtensorMap kmap, vmap, ksmap, vsmap;
    if (!make_page_map(&kmap, a.pool.keys, a.pool) || !make_page_map(&vmap, a.pool.values, a.pool)) {
        return SDC_STATUS_CUDA_ERROR;
    }
    // gathers need whole groups of four pages per tile and row-aligned scales
    t.gather4 = (kTile / a.pool.block_size) % 4 == 0 && make_scale_map(&ksmap, a.pool.key_scales, a.pool) &&
                make_scale_map(&vsmap, a.pool.value_scales, a.pool);
    if (!t.gather4) {
        ksmap = kmap;  // unused
        vsmap = vmap;
    }
    sdc_status_t rc;
    const bool hd64 = a.pool.head_dim == 64;
#define SDC_TC_BUCKET(R)                                                                            \
    case R:                                                                                         \
        rc = hd64 ? launch_bucket<R, 64>(t, kmap, vmap, ksmap, vsmap, first, st)                    \
                  : launch_bucket<R, 128>(t, kmap, vmap, ksmap, vsmap, first, st);                  \
        break;
    switch (bucket_for(t.rows)) {
        SDC_TC_BUCKET(8)
        SDC_TC_BUCKET(16)
        SDC_TC_BUCKET(20)
        SDC_TC_BUCKET(24)
        SDC_TC_BUCKET(32)
        default: return SDC_STATUS_UNSUPPORTED;
    }
#undef SDC_TC_BUCKET
    if (rc != SDC_STATUS_OK) return rc;
    if (t.direct) return SDC_STATUS_OK;  // every item wrote its output rows
    return launch_attention_combine(a, st, /*programmatic=*/true);
}

long long wait_limit_cycles() { return g_wait_limit.load(std::memory_order_relaxed); }

}  // namespace tc
}  // namespace sdc

extern "C" {

SDC_API sdc_status_t sdc_test_attention_waits(int64_t wait_limit_cycles, int32_t stall) {
    if (stall != 0 && stall != 1) return SDC_STATUS_INVALID_ARGUMENT;
    sdc::tc::g_wait_limit.store(wait_limit_cycles > 0 ? wait_limit_cycles : sdc::tc::kWaitLimitCycles,
                                std::memory_order_relaxed);
    sdc::tc::g_stall.store(stall, std::memory_order_relaxed);
    return SDC_STATUS_OK;
}

}  // extern "C"
