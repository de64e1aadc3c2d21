// Kernels (a) quantize-and-append and (b) rollback, plus the per-vector
// quantizer and the gather/dequantize read path, with their C ABI entries.
//
// Work mapping shared by the page kernels: a "head vector" is the head_dim
// codes of one (token, layer, K|V, head).  A group of LPV lanes owns one head
// vector; lane j of the group owns elements [16j, 16j + 16), so every code
// store is one 16-byte store and a group writes the vector's row in one
// coalesced burst.  Vectors are enumerated with the head fastest, so
// neighbouring groups read neighbouring source rows.

#include <algorithm>
#include <cmath>
#include <cstring>
#include <new>
#include <type_traits>
#include <vector>

#include "host_common.h"

namespace sdc {
namespace {

template <typename Src>
struct AccOf {
    using type = float;
};
template <>
struct AccOf<double> {
    using type = double;
};

__device__ __forceinline__ float amax(float a, float b) { return fmaxf(a, b); }
__device__ __forceinline__ double amax(double a, double b) { return fmax(a, b); }

// max that propagates NaN, so one reduction finds both the vector maximum and
// any non-finite element (the result is then NaN or +inf).
__device__ __forceinline__ float max_nan(float a, float b) {
    float r;
    asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
    return r;
}

template <typename Src>
__device__ __forceinline__ int quant_one(typename AccOf<Src>::type x, float s, float rcp) {
    if constexpr (std::is_same<Src, double>::value) {
        return quant_code_f64(x, static_cast<double>(s));
    } else {
        return s >= kFloatPathMinScale ? quant_code_f32(x, s, rcp)
                                       : quant_code_f64(static_cast<double>(x), static_cast<double>(s));
    }
}

// Sixteen codes of a float-valued vector with scale s >= 2^-100 (rcp = 1/s
// rounded), packed four to a word: round_half_away(x / s) clamped to 127 in
// magnitude, the same integers as quant_code_f32 but with no conversion
// instruction.  The candidate rint(|x| * rcp) comes from adding and removing
// 1.5 * 2^23 (round to nearest even of a value below 2^22, exactly what rintf
// returns); it is within one of the answer and is corrected by the exact
// signs of |x| - (n +- 1/2) s, each from one fused multiply-add.  The signed
// code plus 1.5 * 2^23 holds the code's two's-complement byte in its low
// mantissa bits, which byte permutes pack.  Pairs of elements go through the
// packed f32x2 arithmetic.
__device__ __forceinline__ uint4 quant16_f32(const float (&x)[16], float s, float rcp) {
    constexpr float kMagic = 12582912.0f;  // 1.5 * 2^23
    const float2 rcp2 = make_float2(rcp, rcp), negs2 = make_float2(-s, -s);
    const float2 m2 = make_float2(kMagic, kMagic), negm2 = make_float2(-kMagic, -kMagic);
    const float2 half2 = make_float2(0.5f, 0.5f), neghalf2 = make_float2(-0.5f, -0.5f);
    uint32_t bits[16];
#pragma unroll
    for (int i = 0; i < 16; i += 2) {
        const float2 a = make_float2(fabsf(x[i]), fabsf(x[i + 1]));
        float2 n = __fadd2_rn(__fadd2_rn(__fmul2_rn(a, rcp2), m2), negm2);
        const float2 above = __ffma2_rn(__fadd2_rn(n, half2), negs2, a);     // a - (n + 1/2) s
        const float2 below = __ffma2_rn(__fadd2_rn(n, neghalf2), negs2, a);  // a - (n - 1/2) s
        n.x += (above.x >= 0.0f ? 1.0f : 0.0f) - (below.x < 0.0f ? 1.0f : 0.0f);
        n.y += (above.y >= 0.0f ? 1.0f : 0.0f) - (below.y < 0.0f ? 1.0f : 0.0f);
        // |x| <= m and s = fl(m / 127) give |x| / s < 127.5, so n <= 127 needs no clamp
        const float2 q = make_float2(copysignf(n.x, x[i]), copysignf(n.y, x[i + 1]));
        const float2 t = __fadd2_rn(q, m2);
        bits[i] = __float_as_uint(t.x);
        bits[i + 1] = __float_as_uint(t.y);
    }
    auto pack = [](uint32_t w0, uint32_t w1, uint32_t w2, uint32_t w3) {
        return __byte_perm(__byte_perm(w0, w1, 0x0040), __byte_perm(w2, w3, 0x0040), 0x5410);
    };
    return make_uint4(pack(bits[0], bits[1], bits[2], bits[3]), pack(bits[4], bits[5], bits[6], bits[7]),
                      pack(bits[8], bits[9], bits[10], bits[11]), pack(bits[12], bits[13], bits[14], bits[15]));
}

// Per-group maximum of |x| over 16 elements per lane and LPV lanes; for float
// sources a non-finite element makes the result NaN or +inf.
template <typename Src, int LPV, int H = 1>
__device__ __forceinline__ typename AccOf<Src>::type group_absmax(const typename AccOf<Src>::type (&x)[H][16],
                                                                  int& bad) {
    using Acc = typename AccOf<Src>::type;
    Acc m = Acc(0);
    if constexpr (std::is_same<Src, double>::value) {
        int b = 0;
#pragma unroll
        for (int h = 0; h < H; ++h) {
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                b |= !isfinite(x[h][i]);
                m = fmax(m, fabs(x[h][i]));
            }
        }
#pragma unroll
        for (int off = LPV / 2; off > 0; off >>= 1) {
            m = fmax(m, __shfl_xor_sync(kFullMask, m, off));
            b |= __shfl_xor_sync(kFullMask, b, off);
        }
        bad = b;
    } else {
#pragma unroll
        for (int h = 0; h < H; ++h) {
#pragma unroll
            for (int i = 0; i < 16; ++i) m = max_nan(m, fabsf(x[h][i]));
        }
#pragma unroll
        for (int off = LPV / 2; off > 0; off >>= 1) m = max_nan(m, __shfl_xor_sync(kFullMask, m, off));
        bad = !(m < INFINITY);
    }
    return m;
}

struct AppendArgs {
    Pool pool;
    const void* keys;
    const void* values;
    int64_t layer_begin;
    int64_t num_src_layers;
    int64_t s_tok, s_layer, s_head;
    const int64_t* slots;
    uint32_t total_vectors;
    uint32_t vector_blocks;
    FastDiv div_heads;   // num_heads
    FastDiv div_layers;  // num_src_layers
    FastDiv div_block;   // block_size
    TableEdits edits;
    int32_t* status;
};

// H 16-element halves per lane: lane j of a group owns elements
// [16 H j, 16 H (j + 1)) of its head vector.
// Four blocks per SM (at most 64 registers a thread): more loads in flight
// per SM measured 13 % faster than three blocks at 74 registers.
template <typename Src, int LPV, int H>
__global__ void __launch_bounds__(256, 4) quantize_append_kernel(AppendArgs a) {
    using Acc = typename AccOf<Src>::type;
    if (blockIdx.x >= a.vector_blocks) {  // the trailing block applies table edits
        apply_table_edits(a.edits, threadIdx.x, blockDim.x, a.status);
        return;
    }
    constexpr int VPW = 32 / LPV;
    const uint32_t lane = threadIdx.x & 31;
    const uint32_t sub = lane & (LPV - 1);
    const uint32_t warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const uint32_t v = warp * VPW + lane / LPV;
    const bool active = v < a.total_vectors;
    const uint32_t D = static_cast<uint32_t>(a.pool.head_dim);

    uint32_t head = 0, kv = 0, layer_rel = 0, token = 0;
    if (active) {
        uint32_t r;
        a.div_heads.divmod(v, r, head);
        kv = r & 1;
        a.div_layers.divmod(r >> 1, token, layer_rel);
    }
    const bool has_chunk = active && (sub * 16 * H < D);

    Acc x[H][16];
    if (has_chunk) {
        const Src* base = static_cast<const Src*>(kv ? a.values : a.keys) + token * a.s_tok +
                          layer_rel * a.s_layer + head * a.s_head + sub * 16 * H;
#pragma unroll
        for (int h = 0; h < H; ++h) load16(base + 16 * h, x[h]);
    } else {
#pragma unroll
        for (int h = 0; h < H; ++h) {
#pragma unroll
            for (int i = 0; i < 16; ++i) x[h][i] = Acc(0);
        }
    }
    int bad = 0;
    const Acc m = group_absmax<Src, LPV, H>(x, bad);
    if (!active) return;

    const int64_t slot = __ldg(a.slots + token);
    if (slot < 0 || slot >= a.pool.num_blocks * a.pool.block_size) {
        if (sub == 0) report_fault(a.status, SDC_FAULT_SLOT_RANGE);
        return;
    }
    if (bad) {
        if (sub == 0) report_fault(a.status, SDC_FAULT_NONFINITE_VALUE);
        return;
    }
    uint32_t blk, off;
    a.div_block.divmod(static_cast<uint32_t>(slot), blk, off);
    const int64_t layer = a.layer_begin + layer_rel;
    int8_t* codes = (kv ? a.pool.values : a.pool.keys) + blk * a.pool.cbs + layer * a.pool.cls +
                    head * a.pool.chs + off * D;
    float* scale_dst = (kv ? a.pool.value_scales : a.pool.key_scales) + blk * a.pool.sbs +
                       layer * a.pool.sls + head * a.pool.shs + off;

    float s = 0.0f;
    uint4 packed[H];
#pragma unroll
    for (int h = 0; h < H; ++h) packed[h] = make_uint4(0u, 0u, 0u, 0u);
    if (m != Acc(0)) {
        if constexpr (std::is_same<Src, double>::value) {
            s = scale_from_max(m);
        } else {
            // for a float maximum the reference's double quotient rounded to
            // float equals the correctly rounded float quotient (53 >= 2 * 24 + 2
            // bits: double rounding of a division is innocuous)
            s = __fdiv_rn(m, 127.0f);
        }
        if (!(s > 0.0f) || isinf(s)) {
            if (sub == 0) report_fault(a.status, SDC_FAULT_INVALID_SCALE);
            return;
        }
        const float rcp = 1.0f / s;
#pragma unroll
        for (int h = 0; h < H; ++h) {
            if (!std::is_same<Src, double>::value && s >= kFloatPathMinScale) {
                float xf[16];
#pragma unroll
                for (int i = 0; i < 16; ++i) xf[i] = static_cast<float>(x[h][i]);
                packed[h] = quant16_f32(xf, s, rcp);
            } else {
                int q[16];
#pragma unroll
                for (int i = 0; i < 16; ++i) q[i] = quant_one<Src>(x[h][i], s, rcp);
                packed[h].x = pack4(q[0], q[1], q[2], q[3]);
                packed[h].y = pack4(q[4], q[5], q[6], q[7]);
                packed[h].z = pack4(q[8], q[9], q[10], q[11]);
                packed[h].w = pack4(q[12], q[13], q[14], q[15]);
            }
        }
    }
    if (has_chunk) {
#pragma unroll
        for (int h = 0; h < H; ++h) *reinterpret_cast<uint4*>(codes + sub * 16 * H + 16 * h) = packed[h];
    }
    if (sub == 0) *scale_dst = s;
}

// One warp per row, any row length: the per-vector API and the
// KVQuantizer-protocol path use it.
template <typename Src>
__global__ void __launch_bounds__(256) quantize_rows_kernel(const Src* src, int64_t rows, int64_t count,
                                                            int8_t* codes, float* scales,
                                                            int32_t* row_status) {
    using Acc = typename AccOf<Src>::type;
    const int lane = threadIdx.x & 31;
    const int64_t row = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    if (row >= rows) return;
    const Src* x = src + row * count;
    Acc m = Acc(0);
    int bad = 0;
    for (int64_t i = lane; i < count; i += 32) {
        const Acc v = static_cast<Acc>(x[i]);
        bad |= !isfinite(v);
        m = amax(m, fabs(v));
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        m = amax(m, __shfl_xor_sync(kFullMask, m, off));
        bad |= __shfl_xor_sync(kFullMask, bad, off);
    }
    if (bad) {
        if (lane == 0) row_status[row] = SDC_STATUS_NONFINITE_VALUE;
        return;
    }
    int8_t* out = codes + row * count;
    if (m == Acc(0)) {
        for (int64_t i = lane; i < count; i += 32) out[i] = 0;
        if (lane == 0) {
            scales[row] = 0.0f;
            row_status[row] = SDC_STATUS_OK;
        }
        return;
    }
    const float s = scale_from_max(static_cast<double>(m));
    if (!(s > 0.0f) || isinf(s)) {
        if (lane == 0) row_status[row] = SDC_STATUS_INVALID_SCALE;
        return;
    }
    const float rcp = 1.0f / s;
    for (int64_t i = lane; i < count; i += 32) {
        out[i] = static_cast<int8_t>(quant_one<Src>(static_cast<Acc>(x[i]), s, rcp));
    }
    if (lane == 0) {
        scales[row] = s;
        row_status[row] = SDC_STATUS_OK;
    }
}

__global__ void dequantize_vector_kernel(const int8_t* codes, int64_t count, double scale, double* out) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < count) out[i] = static_cast<double>(codes[i]) * scale;
}

struct RollbackArgs {
    Pool pool;
    const int64_t* slots;
    uint32_t slot_blocks;  // cleared slots x layer spans: one block each
    uint32_t span;         // layers one block clears
    FastDiv div_spans;     // layer spans per slot
    FastDiv div_chunks;    // 16-byte code chunks of one layer: 2 x heads x head_dim / 16
    FastDiv div_vector;    // chunks of one head vector: head_dim / 16
    FastDiv div_scales;    // scales of one layer: 2 x heads
    FastDiv div_block;
    TableEdits edits;
    int32_t* status;
};

// One block clears one cleared slot over a span of layers: the key and value
// codes of every head, one 16-byte chunk per thread and step (consecutive
// threads fill a head vector's contiguous row, so each warp store writes four
// whole 128-byte rows at head_dim 128), then the span's 2 x heads scales per
// layer.  The slot is read once per block and every store after it is
// independent, so a block issues all of its writes back to back; the host
// sizes the spans so that the grid fills every SM with eight blocks.
__global__ void __launch_bounds__(256) rollback_kernel(RollbackArgs a) {
    if (blockIdx.x >= a.slot_blocks) {
        apply_table_edits(a.edits, threadIdx.x, blockDim.x, a.status);
        return;
    }
    uint32_t index, part;
    a.div_spans.divmod(blockIdx.x, index, part);
    const int64_t slot = __ldg(a.slots + index);
    if (slot < 0 || slot >= a.pool.num_blocks * a.pool.block_size) {
        if (threadIdx.x == 0) report_fault(a.status, SDC_FAULT_SLOT_RANGE);
        return;
    }
    uint32_t blk, off;
    a.div_block.divmod(static_cast<uint32_t>(slot), blk, off);
    const uint32_t L = static_cast<uint32_t>(a.pool.num_layers);
    const uint32_t H = static_cast<uint32_t>(a.pool.num_heads);
    const uint32_t l0 = part * a.span;
    const uint32_t layers = L - l0 < a.span ? L - l0 : a.span;
    const int64_t code_base = blk * a.pool.cbs + (int64_t)off * a.pool.head_dim;
    const uint32_t chunks = layers * a.div_chunks.divisor;
    for (uint32_t c = threadIdx.x; c < chunks; c += blockDim.x) {
        uint32_t layer, rem, row, ch;
        a.div_chunks.divmod(c, layer, rem);
        a.div_vector.divmod(rem, row, ch);  // row: kv * H + head
        const bool value_side = row >= H;
        const uint32_t head = value_side ? row - H : row;
        int8_t* codes = (value_side ? a.pool.values : a.pool.keys) + code_base + (l0 + layer) * a.pool.cls +
                        head * a.pool.chs + ch * 16;
        *reinterpret_cast<uint4*>(codes) = make_uint4(0u, 0u, 0u, 0u);
    }
    const int64_t scale_base = blk * a.pool.sbs + off;
    const uint32_t scales = layers * a.div_scales.divisor;
    for (uint32_t i = threadIdx.x; i < scales; i += blockDim.x) {
        uint32_t layer, r;
        a.div_scales.divmod(i, layer, r);
        const bool value_side = r >= H;
        const uint32_t head = value_side ? r - H : r;
        (value_side ? a.pool.value_scales : a.pool.key_scales)[scale_base + (l0 + layer) * a.pool.sls +
                                                              head * a.pool.shs] = 0.0f;
    }
}

struct GatherArgs {
    Pool pool;
    int64_t layer_begin;
    int64_t num_layers;
    const int64_t* slots;
    uint32_t total_vectors;
    FastDiv div_heads;
    FastDiv div_layers;
    FastDiv div_block;
    void* out_keys;
    void* out_values;
    int64_t o_tok, o_layer, o_head;
    int32_t* status;
};

__device__ __forceinline__ void store16(double* p, const int (&q)[16], float s) {
    double2* d = reinterpret_cast<double2*>(p);
    const double sd = static_cast<double>(s);
#pragma unroll
    for (int i = 0; i < 8; ++i) d[i] = make_double2(q[2 * i] * sd, q[2 * i + 1] * sd);
}
__device__ __forceinline__ void store16(float* p, const int (&q)[16], float s) {
    float4* d = reinterpret_cast<float4*>(p);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        d[i] = make_float4(__fmul_rn(static_cast<float>(q[4 * i]), s), __fmul_rn(static_cast<float>(q[4 * i + 1]), s),
                           __fmul_rn(static_cast<float>(q[4 * i + 2]), s), __fmul_rn(static_cast<float>(q[4 * i + 3]), s));
    }
}
__device__ __forceinline__ void store16(__nv_bfloat16* p, const int (&q)[16], float s) {
    uint32_t w[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        __nv_bfloat162 h = __floats2bfloat162_rn(__fmul_rn(static_cast<float>(q[2 * i]), s),
                                                 __fmul_rn(static_cast<float>(q[2 * i + 1]), s));
        w[i] = *reinterpret_cast<uint32_t*>(&h);
    }
    uint4* d = reinterpret_cast<uint4*>(p);
    d[0] = make_uint4(w[0], w[1], w[2], w[3]);
    d[1] = make_uint4(w[4], w[5], w[6], w[7]);
}
__device__ __forceinline__ void store16(__half* p, const int (&q)[16], float s) {
    uint32_t w[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        __half2 h = __floats2half2_rn(__fmul_rn(static_cast<float>(q[2 * i]), s),
                                      __fmul_rn(static_cast<float>(q[2 * i + 1]), s));
        w[i] = *reinterpret_cast<uint32_t*>(&h);
    }
    uint4* d = reinterpret_cast<uint4*>(p);
    d[0] = make_uint4(w[0], w[1], w[2], w[3]);
    d[1] = make_uint4(w[4], w[5], w[6], w[7]);
}

// Vectors each lane of the gather handles, a grid's width apart.
constexpr int kGatherVectors = 2;

// Each lane dequantizes 16 elements of a head vector (LPV lanes per vector)
// for kGatherVectors vectors a grid's width apart: every vector's slot read,
// then every code / scale read, is issued before any store, so that many
// dependent load chains are in flight per lane.
template <typename Out, int LPV>
__global__ void __launch_bounds__(256) gather_dequantize_kernel(GatherArgs a) {
    constexpr int VPW = 32 / LPV;
    const uint32_t lane = threadIdx.x & 31;
    const uint32_t sub = lane & (LPV - 1);
    const uint32_t warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const uint32_t pass = gridDim.x * (blockDim.x >> 5) * VPW;  // vectors one pass of the grid covers
    const uint32_t D = static_cast<uint32_t>(a.pool.head_dim);
    constexpr int K = kGatherVectors;
    uint32_t head[K], kv[K], token[K], layer_rel[K];
    int64_t slot[K];
    bool live[K];
#pragma unroll
    for (int j = 0; j < K; ++j) {
        const uint32_t v = warp * VPW + lane / LPV + j * pass;
        live[j] = v < a.total_vectors && sub * 16 < D;
        uint32_t r;
        a.div_heads.divmod(live[j] ? v : 0u, r, head[j]);
        kv[j] = r & 1;
        a.div_layers.divmod(r >> 1, token[j], layer_rel[j]);
        slot[j] = live[j] ? __ldg(a.slots + token[j]) : 0;
    }
    uint4 packed[K];
    float scale[K];
#pragma unroll
    for (int j = 0; j < K; ++j) {
        if (live[j] && (slot[j] < 0 || slot[j] >= a.pool.num_blocks * a.pool.block_size)) {
            if (sub == 0) report_fault(a.status, SDC_FAULT_SLOT_RANGE);
            live[j] = false;
        }
        if (!live[j]) continue;
        uint32_t blk, off;
        a.div_block.divmod(static_cast<uint32_t>(slot[j]), blk, off);
        const int64_t layer = a.layer_begin + layer_rel[j];
        const int8_t* codes = (kv[j] ? a.pool.values : a.pool.keys) + blk * a.pool.cbs + layer * a.pool.cls +
                              head[j] * a.pool.chs + off * D + sub * 16;
        scale[j] = __ldg((kv[j] ? a.pool.value_scales : a.pool.key_scales) + blk * a.pool.sbs +
                         layer * a.pool.sls + head[j] * a.pool.shs + off);
        packed[j] = __ldg(reinterpret_cast<const uint4*>(codes));
    }
#pragma unroll
    for (int j = 0; j < K; ++j) {
        if (!live[j]) continue;
        const uint32_t w[4] = {packed[j].x, packed[j].y, packed[j].z, packed[j].w};
        int q[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) q[i] = static_cast<int8_t>((w[i / 4] >> (8 * (i % 4))) & 0xffu);
        Out* dst = static_cast<Out*>(kv[j] ? a.out_values : a.out_keys) + token[j] * a.o_tok +
                   layer_rel[j] * a.o_layer + head[j] * a.o_head + sub * 16;
        store16(dst, q, scale[j]);
    }
}

constexpr int kThreads = 256;

template <typename Src>
sdc_status_t launch_append(int lpv, int halves, int64_t blocks, cudaStream_t stream, const AppendArgs& a) {
#define SDC_APPEND_CASE(L, H) \
    case L: quantize_append_kernel<Src, L, H><<<blocks, kThreads, 0, stream>>>(a); break;
    if (halves == 2) {
        switch (lpv) {
            SDC_APPEND_CASE(1, 2)
            SDC_APPEND_CASE(2, 2)
            SDC_APPEND_CASE(4, 2)
            SDC_APPEND_CASE(8, 2)
            SDC_APPEND_CASE(16, 2)
            default: return SDC_STATUS_UNSUPPORTED;
        }
    } else {
        switch (lpv) {
            SDC_APPEND_CASE(1, 1)
            SDC_APPEND_CASE(2, 1)
            SDC_APPEND_CASE(4, 1)
            SDC_APPEND_CASE(8, 1)
            SDC_APPEND_CASE(16, 1)
            SDC_APPEND_CASE(32, 1)
            default: return SDC_STATUS_UNSUPPORTED;
        }
    }
#undef SDC_APPEND_CASE
    return launch_status();
}

template <typename Out>
sdc_status_t launch_gather(int lpv, int64_t blocks, cudaStream_t stream, const GatherArgs& a) {
    switch (lpv) {
        case 1: gather_dequantize_kernel<Out, 1><<<blocks, kThreads, 0, stream>>>(a); break;
        case 2: gather_dequantize_kernel<Out, 2><<<blocks, kThreads, 0, stream>>>(a); break;
        case 4: gather_dequantize_kernel<Out, 4><<<blocks, kThreads, 0, stream>>>(a); break;
        case 8: gather_dequantize_kernel<Out, 8><<<blocks, kThreads, 0, stream>>>(a); break;
        case 16: gather_dequantize_kernel<Out, 16><<<blocks, kThreads, 0, stream>>>(a); break;
        case 32: gather_dequantize_kernel<Out, 32><<<blocks, kThreads, 0, stream>>>(a); break;
        default: return SDC_STATUS_UNSUPPORTED;
    }
    return launch_status();
}

sdc_status_t launch_rollback(int64_t blocks, cudaStream_t stream, const RollbackArgs& a) {
    rollback_kernel<<<blocks, kThreads, 0, stream>>>(a);
    return launch_status();
}

// Blocks needed for `vectors` head vectors at `lpv` lanes per vector.
int64_t vector_blocks(int64_t vectors, int lpv) {
    const int64_t per_block = (kThreads / 32) * (32 / lpv);
    return ceil_div(vectors, per_block);
}

template <typename Src>
sdc_status_t launch_rows(const void* src, int64_t rows, int64_t count, int8_t* codes, float* scales,
                         int32_t* status, cudaStream_t stream) {
    const int64_t blocks = ceil_div(rows, kThreads / 32);
    quantize_rows_kernel<Src><<<blocks, kThreads, 0, stream>>>(static_cast<const Src*>(src), rows, count, codes,
                                                               scales, status);
    return launch_status();
}

sdc_status_t dispatch_rows(const void* src, int dtype, int64_t rows, int64_t count, int8_t* codes, float* scales,
                           int32_t* status, cudaStream_t stream) {
    switch (dtype) {
        case SDC_DTYPE_F32: return launch_rows<float>(src, rows, count, codes, scales, status, stream);
        case SDC_DTYPE_BF16: return launch_rows<__nv_bfloat16>(src, rows, count, codes, scales, status, stream);
        case SDC_DTYPE_F16: return launch_rows<__half>(src, rows, count, codes, scales, status, stream);
        case SDC_DTYPE_F64: return launch_rows<double>(src, rows, count, codes, scales, status, stream);
        default: return SDC_STATUS_UNSUPPORTED;
    }
}

}  // namespace
}  // namespace sdc

using namespace sdc;

extern "C" {

SDC_API uint32_t sdc_abi_version(void) { return SDC_ABI_VERSION; }

SDC_API const char* sdc_status_string(sdc_status_t status) {
    switch (status) {
        case SDC_STATUS_OK: return "ok";
        case SDC_STATUS_NULL_ARGUMENT: return "null argument";
        case SDC_STATUS_INVALID_SIZE: return "invalid size";
        case SDC_STATUS_NONFINITE_VALUE: return "non-finite value";
        case SDC_STATUS_NEGATIVE_PROBABILITY: return "negative probability";
        case SDC_STATUS_ZERO_MASS: return "zero probability mass";
        case SDC_STATUS_TOKEN_OUT_OF_RANGE: return "token out of range";
        case SDC_STATUS_INVALID_UNIFORM: return "uniform must be finite and in [0, 1)";
        case SDC_STATUS_OVERFLOW: return "size overflow";
        case SDC_STATUS_INTERNAL_ERROR: return "internal error";
        case SDC_STATUS_INVALID_SCALE: return "invalid quantization scale";
        case SDC_STATUS_CUDA_ERROR: return "CUDA runtime error";
        case SDC_STATUS_UNSUPPORTED: return "unsupported shape or dtype";
        case SDC_STATUS_MISALIGNED: return "buffer or stride is not 16-byte aligned";
        case SDC_STATUS_DEVICE_FAULT: return "a kernel reported a fault in the device status word";
        case SDC_STATUS_INVALID_ARGUMENT: return "invalid argument";
        case SDC_STATUS_SCRATCH_EXCEEDED: return "workspace larger than the library's fixed scratch";
        default: return "unknown status";
    }
}

SDC_API sdc_status_t sdc_quantize_symmetric_int8_f64(const double* values, size_t count, int8_t* output_values,
                                                     double* output_scale) {
    try {
        if (values == nullptr || output_values == nullptr || output_scale == nullptr) {
            return SDC_STATUS_NULL_ARGUMENT;
        }
        if (count == 0) return SDC_STATUS_INVALID_SIZE;
        if (count > (size_t(1) << 40)) return SDC_STATUS_OVERFLOW;
        cudaStream_t stream = cudaStreamPerThread;
        const size_t in_bytes = count * sizeof(double);
        const size_t code_off = (in_bytes + 15) & ~size_t(15);
        const size_t scale_off = (code_off + count + 15) & ~size_t(15);
        const size_t total = scale_off + 16;
        char* dev = nullptr;
        if (cudaMallocAsync(reinterpret_cast<void**>(&dev), total, stream) != cudaSuccess) {
            return SDC_STATUS_CUDA_ERROR;
        }
        std::vector<int8_t> codes(count);
        float scale = 0.0f;
        int32_t status = SDC_STATUS_INTERNAL_ERROR;
        sdc_status_t rc = SDC_STATUS_OK;
        if (cudaMemcpyAsync(dev, values, in_bytes, cudaMemcpyHostToDevice, stream) != cudaSuccess) {
            rc = SDC_STATUS_CUDA_ERROR;
        }
        if (rc == SDC_STATUS_OK) {
            rc = launch_rows<double>(dev, 1, static_cast<int64_t>(count), reinterpret_cast<int8_t*>(dev + code_off),
                                     reinterpret_cast<float*>(dev + scale_off),
                                     reinterpret_cast<int32_t*>(dev + scale_off + 4), stream);
        }
        if (rc == SDC_STATUS_OK &&
            (cudaMemcpyAsync(codes.data(), dev + code_off, count, cudaMemcpyDeviceToHost, stream) != cudaSuccess ||
             cudaMemcpyAsync(&scale, dev + scale_off, 4, cudaMemcpyDeviceToHost, stream) != cudaSuccess ||
             cudaMemcpyAsync(&status, dev + scale_off + 4, 4, cudaMemcpyDeviceToHost, stream) != cudaSuccess)) {
            rc = SDC_STATUS_CUDA_ERROR;
        }
        cudaFreeAsync(dev, stream);
        if (cudaStreamSynchronize(stream) != cudaSuccess) return SDC_STATUS_CUDA_ERROR;
        if (rc != SDC_STATUS_OK) return rc;
        if (status != SDC_STATUS_OK) return static_cast<sdc_status_t>(status);
        std::memcpy(output_values, codes.data(), count);
        *output_scale = static_cast<double>(scale);
        return SDC_STATUS_OK;
    } catch (...) {
        return SDC_STATUS_INTERNAL_ERROR;
    }
}

SDC_API sdc_status_t sdc_dequantize_symmetric_int8_f64(const int8_t* values, size_t count, double scale,
                                                       double* output_values) {
    try {
        if (values == nullptr || output_values == nullptr) return SDC_STATUS_NULL_ARGUMENT;
        if (count == 0) return SDC_STATUS_INVALID_SIZE;
        if (count > (size_t(1) << 40)) return SDC_STATUS_OVERFLOW;
        if (!std::isfinite(scale) || scale < 0.0) return SDC_STATUS_INVALID_SCALE;
        if (scale == 0.0) {
            for (size_t i = 0; i < count; ++i) {
                if (values[i] != 0) return SDC_STATUS_INVALID_SCALE;
            }
        }
        cudaStream_t stream = cudaStreamPerThread;
        const size_t out_off = (count + 15) & ~size_t(15);
        char* dev = nullptr;
        if (cudaMallocAsync(reinterpret_cast<void**>(&dev), out_off + count * sizeof(double), stream) !=
            cudaSuccess) {
            return SDC_STATUS_CUDA_ERROR;
        }
        std::vector<double> out(count);
        sdc_status_t rc = SDC_STATUS_OK;
        if (cudaMemcpyAsync(dev, values, count, cudaMemcpyHostToDevice, stream) != cudaSuccess) {
            rc = SDC_STATUS_CUDA_ERROR;
        }
        if (rc == SDC_STATUS_OK) {
            const int64_t blocks = ceil_div(static_cast<int64_t>(count), kThreads);
            dequantize_vector_kernel<<<blocks, kThreads, 0, stream>>>(
                reinterpret_cast<const int8_t*>(dev), static_cast<int64_t>(count), scale,
                reinterpret_cast<double*>(dev + out_off));
            rc = launch_status();
        }
        if (rc == SDC_STATUS_OK && cudaMemcpyAsync(out.data(), dev + out_off, count * sizeof(double),
                                                   cudaMemcpyDeviceToHost, stream) != cudaSuccess) {
            rc = SDC_STATUS_CUDA_ERROR;
        }
        cudaFreeAsync(dev, stream);
        if (cudaStreamSynchronize(stream) != cudaSuccess) return SDC_STATUS_CUDA_ERROR;
        if (rc != SDC_STATUS_OK) return rc;
        std::memcpy(output_values, out.data(), count * sizeof(double));
        return SDC_STATUS_OK;
    } catch (...) {
        return SDC_STATUS_INTERNAL_ERROR;
    }
}

SDC_API sdc_status_t sdc_quantize_rows(const void* source, int src_dtype, int64_t rows, int64_t count,
                                       int8_t* codes, float* scales, int32_t* row_status, uintptr_t stream) {
    try {
        if (source == nullptr || codes == nullptr || scales == nullptr || row_status == nullptr) {
            return SDC_STATUS_NULL_ARGUMENT;
        }
        if (rows < 0 || count < 1) return SDC_STATUS_INVALID_SIZE;
        if (dtype_size(src_dtype) == 0) return SDC_STATUS_UNSUPPORTED;
        if (rows == 0) return SDC_STATUS_OK;
        return dispatch_rows(source, src_dtype, rows, count, codes, scales, row_status, as_stream(stream));
    } catch (...) {
        return SDC_STATUS_INTERNAL_ERROR;
    }
}

SDC_API sdc_status_t sdc_quantize_append(const sdc_page_pool_t* pool, int64_t layer_begin, int64_t num_src_layers,
                                         const void* keys, const void* values, int src_dtype, int64_t num_tokens,
                                         int64_t src_token_stride, int64_t src_layer_stride,
                                         int64_t src_head_stride, const int64_t* slot_mapping,
                                         const sdc_table_edits_t* edits, int32_t* device_status,
                                         uintptr_t stream) {
    try {
        sdc_status_t rc = validate_pool(pool);
        if (rc != SDC_STATUS_OK) return rc;
        TableEdits te;
        rc = validate_edits(edits, &te);
        if (rc != SDC_STATUS_OK) return rc;
        if (device_status == nullptr) return SDC_STATUS_NULL_ARGUMENT;
        if (num_tokens < 0 || num_src_layers < 1) return SDC_STATUS_INVALID_SIZE;
        if (layer_begin < 0 || layer_begin + num_src_layers > pool->num_layers) return SDC_STATUS_INVALID_SIZE;
        const int es = dtype_size(src_dtype);
        if (es == 0) return SDC_STATUS_UNSUPPORTED;
        const bool has_edits = te.num_entries > 0 || te.num_lengths > 0;
        if (num_tokens == 0 && !has_edits) return SDC_STATUS_OK;
        if (num_tokens > 0) {
            if (keys == nullptr || values == nullptr || slot_mapping == nullptr) return SDC_STATUS_NULL_ARGUMENT;
            if (src_token_stride < 0 || src_layer_stride < 0 || src_head_stride < 0) {
                return SDC_STATUS_INVALID_SIZE;
            }
            if (!aligned16(keys) || !aligned16(values) || (src_token_stride * es) % 16 ||
                (src_layer_stride * es) % 16 || (src_head_stride * es) % 16) {
                return SDC_STATUS_MISALIGNED;
            }
        }
        // float-valued sources take 32 elements per lane when head_dim allows
        const int halves = (src_dtype != SDC_DTYPE_F64 && pool->head_dim % 32 == 0) ? 2 : 1;
        const int lpv = lanes_per_vector(pool->head_dim / halves);
        AppendArgs a;
        a.pool = to_pool(pool);
        a.keys = keys;
        a.values = values;
        a.layer_begin = layer_begin;
        a.num_src_layers = num_src_layers;
        a.s_tok = src_token_stride;
        a.s_layer = src_layer_stride;
        a.s_head = src_head_stride;
        a.slots = slot_mapping;
        const int64_t vectors = num_tokens * num_src_layers * 2 * pool->num_heads;
        const int64_t nblocks = vector_blocks(vectors, lpv);
        if (vectors >= INT32_MAX || nblocks + 1 >= INT32_MAX) return SDC_STATUS_OVERFLOW;
        if (pool->num_blocks * pool->block_size >= INT32_MAX) return SDC_STATUS_OVERFLOW;
        a.total_vectors = static_cast<uint32_t>(vectors);
        a.vector_blocks = static_cast<uint32_t>(nblocks);
        a.div_heads = FastDiv(static_cast<uint32_t>(pool->num_heads));
        a.div_layers = FastDiv(static_cast<uint32_t>(num_src_layers));
        a.div_block = FastDiv(static_cast<uint32_t>(pool->block_size));
        a.edits = te;
        a.status = device_status;
        const int64_t blocks = nblocks + (has_edits ? 1 : 0);
        cudaStream_t st = as_stream(stream);
        switch (src_dtype) {
            case SDC_DTYPE_F32: return launch_append<float>(lpv, halves, blocks, st, a);
            case SDC_DTYPE_BF16: return launch_append<__nv_bfloat16>(lpv, halves, blocks, st, a);
            case SDC_DTYPE_F16: return launch_append<__half>(lpv, halves, blocks, st, a);
            case SDC_DTYPE_F64: return launch_append<double>(lpv, halves, blocks, st, a);
            default: return SDC_STATUS_UNSUPPORTED;
        }
    } catch (...) {
        return SDC_STATUS_INTERNAL_ERROR;
    }
}

SDC_API sdc_status_t sdc_rollback(const sdc_page_pool_t* pool, const int64_t* clear_slots, int64_t num_clear,
                                  const sdc_table_edits_t* edits, int32_t* device_status, uintptr_t stream) {
    try {
        sdc_status_t rc = validate_pool(pool);
        if (rc != SDC_STATUS_OK) return rc;
        TableEdits te;
        rc = validate_edits(edits, &te);
        if (rc != SDC_STATUS_OK) return rc;
        if (device_status == nullptr) return SDC_STATUS_NULL_ARGUMENT;
        if (num_clear < 0) return SDC_STATUS_INVALID_SIZE;
        if (num_clear > 0 && clear_slots == nullptr) return SDC_STATUS_NULL_ARGUMENT;
        const bool has_edits = te.num_entries > 0 || te.num_lengths > 0;
        if (num_clear == 0 && !has_edits) return SDC_STATUS_OK;
        RollbackArgs a;
        a.pool = to_pool(pool);
        a.slots = clear_slots;
        // layers per block: the whole slot when there are enough slots to
        // fill every SM with eight blocks, otherwise spans small enough that
        // they do (more resident warps hide the slot read before the stores)
        const int64_t L = pool->num_layers;
        const int64_t want = 8 * static_cast<int64_t>(device_sms());
        const int64_t splits = num_clear > 0 ? std::min<int64_t>(L, ceil_div(want, num_clear)) : 1;
        const int64_t span = ceil_div(L, splits);
        const int64_t spans = ceil_div(L, span);
        const int64_t nblocks = num_clear * spans;
        const int64_t chunks = 2 * pool->num_heads * (pool->head_dim / 16);
        if (nblocks + 1 >= INT32_MAX || chunks * span >= INT32_MAX || 2 * pool->num_heads * span >= INT32_MAX) {
            return SDC_STATUS_OVERFLOW;
        }
        if (pool->num_blocks * pool->block_size >= INT32_MAX) return SDC_STATUS_OVERFLOW;
        a.slot_blocks = static_cast<uint32_t>(nblocks);
        a.span = static_cast<uint32_t>(span);
        a.div_spans = FastDiv(static_cast<uint32_t>(spans));
        a.div_chunks = FastDiv(static_cast<uint32_t>(chunks));
        a.div_vector = FastDiv(static_cast<uint32_t>(pool->head_dim / 16));
        a.div_scales = FastDiv(static_cast<uint32_t>(2 * pool->num_heads));
        a.div_block = FastDiv(static_cast<uint32_t>(pool->block_size));
        a.edits = te;
        a.status = device_status;
        const int64_t blocks = nblocks + (has_edits ? 1 : 0);
        return launch_rollback(blocks, as_stream(stream), a);
    } catch (...) {
        return SDC_STATUS_INTERNAL_ERROR;
    }
}

SDC_API sdc_status_t sdc_gather_dequantize(const sdc_page_pool_t* pool, int64_t layer_begin, int64_t num_layers,
                                           const int64_t* slot_mapping, int64_t num_tokens, void* out_keys,
                                           void* out_values, int out_dtype, int64_t out_token_stride,
                                           int64_t out_layer_stride, int64_t out_head_stride,
                                           int32_t* device_status, uintptr_t stream) {
    try {
        sdc_status_t rc = validate_pool(pool);
        if (rc != SDC_STATUS_OK) return rc;
        if (device_status == nullptr) return SDC_STATUS_NULL_ARGUMENT;
        if (num_tokens < 0 || num_layers < 1) return SDC_STATUS_INVALID_SIZE;
        if (layer_begin < 0 || layer_begin + num_layers > pool->num_layers) return SDC_STATUS_INVALID_SIZE;
        if (num_tokens == 0) return SDC_STATUS_OK;
        if (slot_mapping == nullptr || out_keys == nullptr || out_values == nullptr) return SDC_STATUS_NULL_ARGUMENT;
        const int es = dtype_size(out_dtype);
        if (es == 0) return SDC_STATUS_UNSUPPORTED;
        if (out_token_stride < 0 || out_layer_stride < 0 || out_head_stride < 0) return SDC_STATUS_INVALID_SIZE;
        if (!aligned16(out_keys) || !aligned16(out_values) || (out_token_stride * es) % 16 ||
            (out_layer_stride * es) % 16 || (out_head_stride * es) % 16) {
            return SDC_STATUS_MISALIGNED;
        }
        const int lpv = lanes_per_vector(pool->head_dim);
        GatherArgs a;
        a.pool = to_pool(pool);
        a.layer_begin = layer_begin;
        a.num_layers = num_layers;
        a.slots = slot_mapping;
        const int64_t vectors = num_tokens * num_layers * 2 * pool->num_heads;
        if (vectors >= INT32_MAX) return SDC_STATUS_OVERFLOW;
        if (pool->num_blocks * pool->block_size >= INT32_MAX) return SDC_STATUS_OVERFLOW;
        a.total_vectors = static_cast<uint32_t>(vectors);
        a.div_heads = FastDiv(static_cast<uint32_t>(pool->num_heads));
        a.div_layers = FastDiv(static_cast<uint32_t>(num_layers));
        a.div_block = FastDiv(static_cast<uint32_t>(pool->block_size));
        a.out_keys = out_keys;
        a.out_values = out_values;
        a.o_tok = out_token_stride;
        a.o_layer = out_layer_stride;
        a.o_head = out_head_stride;
        a.status = device_status;
        // kGatherVectors vectors per lane, a grid's width apart
        const int64_t blocks = vector_blocks((vectors + kGatherVectors - 1) / kGatherVectors, lpv);
        cudaStream_t st = as_stream(stream);
        switch (out_dtype) {
            case SDC_DTYPE_F32: return launch_gather<float>(lpv, blocks, st, a);
            case SDC_DTYPE_BF16: return launch_gather<__nv_bfloat16>(lpv, blocks, st, a);
            case SDC_DTYPE_F16: return launch_gather<__half>(lpv, blocks, st, a);
            case SDC_DTYPE_F64: return launch_gather<double>(lpv, blocks, st, a);
            default: return SDC_STATUS_UNSUPPORTED;
        }
    } catch (...) {
        return SDC_STATUS_INTERNAL_ERROR;
    }
}

}  // extern "C"
