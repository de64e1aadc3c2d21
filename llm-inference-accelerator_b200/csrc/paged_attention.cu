// Kernel (c): fused paged verify/decode attention over INT8 pages.
//
// Computation (the reference's unfused op, src/specdecode/cuda_kv_cache.py:452-497):
//   for each sequence b and query head hq (KV head h = hq / G, G = Hq / Hkv),
//   for each window row i (query position p = T - window + i):
//     s_t = (q . k_t) / sqrt(D) for key positions t <= p,  out = softmax(s) . v
//   with k_t = code_t * scale_t and v_t likewise.
//
// Decomposition (split-K flash decoding): one work item is (sequence, KV head,
// chunk of `chunk` key positions).  An item serves all G * window query rows
// that read this KV head, so each page is read once per item.  Each item
// writes an un-normalised partial (running max m, sum l, O = sum p v) and a
// combine pass merges the chunks of a (sequence, KV head).
//
// This file holds the CUDA-core form of the item kernel: a 256-thread block
// walks the chunk in 32-token tiles staged in shared memory; warp w owns query
// rows w, w+8, ...; scores use lane = token, the P.V product uses lane = a
// slice of head_dim.  Softmax runs in the log2 domain (q pre-multiplied by
// log2(e)/sqrt(D)).  Scales are applied after the integer dot product:
// s = (q . code_k) * scale_k and P.V = sum (p * scale_v) * code_v.

#include <cmath>

#include "host_common.h"
#include "paged_attention.h"

namespace sdc {
namespace {

constexpr int kTile = 32;
constexpr int kWarps = 8;
constexpr int kThreadsAttn = kWarps * 32;

template <typename T>
__device__ __forceinline__ float to_float(T v);
template <>
__device__ __forceinline__ float to_float<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_float<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <>
__device__ __forceinline__ float to_float<__half>(__half v) { return __half2float(v); }

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v = fmaxf(v, __shfl_xor_sync(kFullMask, v, off));
    return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(kFullMask, v, off);
    return v;
}

__device__ __forceinline__ void unpack16(const uint4& c, float (&f)[16]) {
    const uint32_t w[4] = {c.x, c.y, c.z, c.w};
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        f[i] = static_cast<float>(static_cast<int8_t>((w[i >> 2] >> (8 * (i & 3))) & 0xffu));
    }
}

// Shared-memory carve-up for one block.
template <int D>
struct SimtSmem {
    static constexpr int kRow = D + 16;  // padded code row: conflict-free 16-byte reads
    static size_t bytes(int rows) {
        return sizeof(float) * rows * D            // q rows
               + 2 * kTile * kRow                  // K and V code tiles
               + 2 * sizeof(float) * kTile         // K and V scales
               + sizeof(float) * rows * kTile;     // probabilities (scaled by v scale)
    }
};

template <typename QT, int D, int RPW>
__global__ void __launch_bounds__(kThreadsAttn) attn_simt_kernel(AttnArgs a) {
    constexpr int kRow = SimtSmem<D>::kRow;
    constexpr int DPL = D >= 32 ? D / 32 : 1;  // head_dim elements per lane in the P.V product
    extern __shared__ __align__(16) unsigned char smem[];
    const int R = static_cast<int>(a.rows);
    float* q_s = reinterpret_cast<float*>(smem);
    int8_t* k_s = reinterpret_cast<int8_t*>(q_s + R * D);
    int8_t* v_s = k_s + kTile * kRow;
    float* ks_s = reinterpret_cast<float*>(v_s + kTile * kRow);
    float* vs_s = ks_s + kTile;
    float* p_s = vs_s + kTile;

    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int lane = tid & 31;
    const bool pv_lane = lane * DPL < D;  // head_dim < 32 leaves upper lanes idle in P.V
    const int64_t item = blockIdx.y;  // b * Hkv + h
    const int64_t b = item / a.kv_heads;
    const int64_t h = item - b * a.kv_heads;
    const int64_t chunk_index = blockIdx.x;

    const int64_t T = __ldg(a.context_lens + b);
    const bool valid_ctx = T >= a.window && T <= a.table_stride * a.pool.block_size &&
                           T <= a.max_chunks * a.chunk;
    const int64_t t0 = chunk_index * a.chunk;
    float* part_o = a.part_o + (item * a.max_chunks + chunk_index) * R * D;
    float* part_ml = a.part_ml + (item * a.max_chunks + chunk_index) * R * 2;
    if (!valid_ctx) {
        if (tid == 0 && chunk_index == 0) report_fault(a.status, SDC_FAULT_CONTEXT_RANGE);
        return;
    }
    if (t0 >= T) return;
    const int64_t t1 = min(T, t0 + a.chunk);

    // q rows for this (sequence, KV head) are contiguous: heads h*G .. h*G+G-1,
    // each with `window` rows of D, i.e. row r = g * window + i.
    const QT* q = static_cast<const QT*>(a.query) + ((b * a.query_heads + h * a.group) * a.window) * D;
    for (int idx = tid; idx < R * D; idx += kThreadsAttn) q_s[idx] = to_float(q[idx]) * a.qk_scale;

    float m_run[RPW], l_run[RPW], acc[RPW][DPL];
#pragma unroll
    for (int j = 0; j < RPW; ++j) {
        m_run[j] = -INFINITY;
        l_run[j] = 0.0f;
#pragma unroll
        for (int e = 0; e < DPL; ++e) acc[j][e] = 0.0f;
    }

    const int32_t* table = a.block_tables + b * a.table_stride;
    const int64_t bs = a.pool.block_size;
    const int64_t code_base = a.layer * a.pool.cls + h * a.pool.chs;
    const int64_t scale_base = a.layer * a.pool.sls + h * a.pool.shs;
    constexpr int kChunks16 = D / 16;

    for (int64_t tile = t0; tile < t1; tile += kTile) {
        __syncthreads();  // previous tile's shared data fully consumed
        for (int idx = tid; idx < 2 * kTile * kChunks16; idx += kThreadsAttn) {
            const int kv = idx / (kTile * kChunks16);
            const int rem = idx - kv * kTile * kChunks16;
            const int tok = rem / kChunks16;
            const int ch = rem - tok * kChunks16;
            const int64_t t = tile + tok;
            uint4 c = make_uint4(0u, 0u, 0u, 0u);
            if (t < t1) {
                const int64_t blk = __ldg(table + t / bs);
                if (blk >= 0 && blk < a.pool.num_blocks) {
                    const int8_t* src = (kv ? a.pool.values : a.pool.keys) + blk * a.pool.cbs + code_base +
                                        (t - (t / bs) * bs) * D + ch * 16;
                    c = __ldg(reinterpret_cast<const uint4*>(src));
                } else if (ch == 0 && kv == 0) {
                    report_fault(a.status, SDC_FAULT_BLOCK_RANGE);
                }
            }
            *reinterpret_cast<uint4*>((kv ? v_s : k_s) + tok * kRow + ch * 16) = c;
        }
        if (tid < 2 * kTile) {
            const int kv = tid / kTile;
            const int tok = tid - kv * kTile;
            const int64_t t = tile + tok;
            float sc = 0.0f;
            if (t < t1) {
                const int64_t blk = __ldg(table + t / bs);
                if (blk >= 0 && blk < a.pool.num_blocks) {
                    sc = __ldg((kv ? a.pool.value_scales : a.pool.key_scales) + blk * a.pool.sbs + scale_base +
                               (t - (t / bs) * bs));
                }
            }
            (kv ? vs_s : ks_s)[tok] = sc;
        }
        __syncthreads();

        // Scores: lane = token, rows r = warp + 8j.
        float s[RPW];
#pragma unroll
        for (int j = 0; j < RPW; ++j) s[j] = 0.0f;
#pragma unroll 2
        for (int ch = 0; ch < kChunks16; ++ch) {
            float kf[16];
            unpack16(*reinterpret_cast<const uint4*>(k_s + lane * kRow + ch * 16), kf);
#pragma unroll
            for (int j = 0; j < RPW; ++j) {
                const int r = warp + kWarps * j;
                if (r < R) {
                    const float4* qr = reinterpret_cast<const float4*>(q_s + r * D + ch * 16);
                    float acc_s = s[j];
#pragma unroll
                    for (int v4 = 0; v4 < 4; ++v4) {
                        const float4 qv = qr[v4];
                        acc_s = fmaf(qv.x, kf[4 * v4 + 0], acc_s);
                        acc_s = fmaf(qv.y, kf[4 * v4 + 1], acc_s);
                        acc_s = fmaf(qv.z, kf[4 * v4 + 2], acc_s);
                        acc_s = fmaf(qv.w, kf[4 * v4 + 3], acc_s);
                    }
                    s[j] = acc_s;
                }
            }
        }
        const int64_t t = tile + lane;
        const float kscale = ks_s[lane];
        const float vscale = vs_s[lane];
#pragma unroll
        for (int j = 0; j < RPW; ++j) {
            const int r = warp + kWarps * j;
            if (r < R) {  // warp-uniform
                const int i = r % static_cast<int>(a.window);
                const bool visible = t < t1 && t <= T - a.window + i;
                const float sc = visible ? s[j] * kscale : -INFINITY;
                const float m_new = fmaxf(m_run[j], warp_max(sc));
                const float alpha = (m_new == -INFINITY) ? 1.0f : exp2f(m_run[j] - m_new);
                const float p = visible ? exp2f(sc - m_new) : 0.0f;
                l_run[j] = l_run[j] * alpha + warp_sum(p);
                m_run[j] = m_new;
#pragma unroll
                for (int e = 0; e < DPL; ++e) acc[j][e] *= alpha;
                p_s[r * kTile + lane] = p * vscale;
            }
        }
        __syncwarp();

        // P.V: lane owns head_dim slice [lane*DPL, lane*DPL + DPL).
#pragma unroll 4
        for (int tok = 0; tok < kTile; ++tok) {
            if (!pv_lane) break;
            float vf[DPL];
            const int8_t* vrow = v_s + tok * kRow + lane * DPL;
            if constexpr (DPL == 4) {
                const uint32_t w = *reinterpret_cast<const uint32_t*>(vrow);
#pragma unroll
                for (int e = 0; e < 4; ++e) vf[e] = static_cast<float>(static_cast<int8_t>((w >> (8 * e)) & 0xffu));
            } else {
#pragma unroll
                for (int e = 0; e < DPL; ++e) vf[e] = static_cast<float>(vrow[e]);
            }
#pragma unroll
            for (int j = 0; j < RPW; ++j) {
                const int r = warp + kWarps * j;
                if (r < R) {
                    const float p = p_s[r * kTile + tok];
#pragma unroll
                    for (int e = 0; e < DPL; ++e) acc[j][e] = fmaf(p, vf[e], acc[j][e]);
                }
            }
        }
    }

#pragma unroll
    for (int j = 0; j < RPW; ++j) {
        const int r = warp + kWarps * j;
        if (r < R) {
            if (pv_lane) {
#pragma unroll
                for (int e = 0; e < DPL; ++e) part_o[r * D + lane * DPL + e] = acc[j][e];
            }
            if (lane == 0) {
                part_ml[2 * r + 0] = m_run[j];
                part_ml[2 * r + 1] = l_run[j];
            }
        }
    }
}

// Four consecutive output elements in one store (8 bytes for 16-bit types,
// 16 for float); the element offset is a multiple of 4.
template <typename QT>
__device__ __forceinline__ void store4(QT* dst, float x, float y, float z, float w);
template <>
__device__ __forceinline__ void store4<float>(float* dst, float x, float y, float z, float w) {
    *reinterpret_cast<float4*>(dst) = make_float4(x, y, z, w);
}
template <>
__device__ __forceinline__ void store4<__nv_bfloat16>(__nv_bfloat16* dst, float x, float y, float z, float w) {
    const __nv_bfloat162 lo = __floats2bfloat162_rn(x, y), hi = __floats2bfloat162_rn(z, w);
    *reinterpret_cast<uint2*>(dst) =
        make_uint2(*reinterpret_cast<const uint32_t*>(&lo), *reinterpret_cast<const uint32_t*>(&hi));
}
template <>
__device__ __forceinline__ void store4<__half>(__half* dst, float x, float y, float z, float w) {
    const __half2 lo = __floats2half2_rn(x, y), hi = __floats2half2_rn(z, w);
    *reinterpret_cast<uint2*>(dst) =
        make_uint2(*reinterpret_cast<const uint32_t*>(&lo), *reinterpret_cast<const uint32_t*>(&hi));
}

// The four elements at `offset` of every destination of the call (one, or
// every rank's gathered output).  Stores that reach another GPU's memory are
// made visible system-wide before the thread moves on to the completion
// signal, which the launch after this one raises.
template <typename QT>
__device__ __forceinline__ void put4(const AttnArgs& a, int64_t offset, float x, float y, float z, float w) {
    for (int i = 0; i < a.num_outs; ++i) store4<QT>(static_cast<QT*>(a.outs[i]) + offset, x, y, z, w);
    if (a.num_outs > 1) __threadfence_system();
}

// Merges the chunk partials of one (sequence, KV head) and a group of its
// query rows and writes the output.  D / 4 threads cover a row (4 columns
// each, 16-byte loads), so a block of kCombineThreads serves 4 * 128 / D
// rows (blockIdx.y picks the group).  One coalesced pass brings the rows'
// (m, l) of every chunk into shared memory, thread r < rows of the group turns
// them into weights exp2(m_c - m) / L, and every thread then sums its row's
// chunk partials with independent loads: about three memory round trips.
constexpr int kCombineThreads = 128;
constexpr int kCombineMaxWeights = 12 * 1024;  // chunks x rows the host admits

template <typename QT>
__global__ void __launch_bounds__(kCombineThreads) attn_combine_kernel(AttnArgs a) {
    extern __shared__ float csm[];  // ml [chunks][group rows][2], then weights [chunks][group rows]
    asm volatile("griddepcontrol.wait;" ::: "memory");  // partials of the item kernel (no-op for a plain launch)
    // a completion launch chained after this one (the KV-head gather's flags)
    // may be scheduled now; it waits for this grid's stores before it signals
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int64_t item = blockIdx.x;
    const int64_t b = item / a.kv_heads;
    const int64_t h = item - b * a.kv_heads;
    const int R = static_cast<int>(a.rows);
    const int D = static_cast<int>(a.head_dim);
    const int per_row = D / 4;
    const int rpb = kCombineThreads / per_row;  // rows of this block's group
    const int r0 = static_cast<int>(blockIdx.y) * rpb;
    const int nr = min(rpb, R - r0);
    if (nr <= 0) return;
    const int64_t T = __ldg(a.context_lens + b);
    const int64_t out = out_rows_offset(a, b, h);
    const bool valid_ctx = T >= a.window && T <= a.table_stride * a.pool.block_size &&
                           T <= a.max_chunks * a.chunk;
    const int rl = threadIdx.x / per_row;  // this thread's row within the group
    const int d4 = (threadIdx.x % per_row) * 4;
    if (!valid_ctx) {
        if (rl < nr) put4<QT>(a, out + (r0 + rl) * D + d4, 0.0f, 0.0f, 0.0f, 0.0f);
        return;
    }
    const int chunks = static_cast<int>((T + a.chunk - 1) / a.chunk);
    const float* ml = a.part_ml + item * a.max_chunks * R * 2;
    const float* po = a.part_o + item * a.max_chunks * R * D;
    float* weights = csm + 2 * chunks * rpb;
    for (int i = threadIdx.x; i < 2 * chunks * nr; i += blockDim.x) {
        const int c = i / (2 * nr), j = i - c * 2 * nr;
        csm[c * 2 * rpb + j] = __ldg(ml + (static_cast<int64_t>(c) * R + r0) * 2 + j);
    }
    __syncthreads();
    if (threadIdx.x < nr) {
        const int r = threadIdx.x;
        float m = -INFINITY;
        for (int c = 0; c < chunks; ++c) m = fmaxf(m, csm[(c * rpb + r) * 2]);
        float l = 0.0f;
        for (int c = 0; c < chunks; ++c) {
            const float mc = csm[(c * rpb + r) * 2];
            const float w = mc == -INFINITY ? 0.0f : exp2f(mc - m);
            weights[c * rpb + r] = w;
            l = fmaf(csm[(c * rpb + r) * 2 + 1], w, l);
        }
        const float inv = l > 0.0f ? 1.0f / l : 0.0f;
        for (int c = 0; c < chunks; ++c) weights[c * rpb + r] *= inv;
    }
    __syncthreads();
    if (rl >= nr) return;
    const int r = r0 + rl;
    float4 o = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll 4
    for (int c = 0; c < chunks; ++c) {
        const float4 v = __ldg(reinterpret_cast<const float4*>(po + (static_cast<int64_t>(c) * R + r) * D + d4));
        const float w = weights[c * rpb + rl];
        o.x = fmaf(v.x, w, o.x);
        o.y = fmaf(v.y, w, o.y);
        o.z = fmaf(v.z, w, o.z);
        o.w = fmaf(v.w, w, o.w);
    }
    put4<QT>(a, out + r * D + d4, o.x, o.y, o.z, o.w);
}

template <typename QT, int D>
sdc_status_t launch_simt_rows(const AttnArgs& a, int rpw, dim3 grid, size_t smem, cudaStream_t st) {
#define SDC_SIMT_CASE(N)                                                                                  \
    case N:                                                                                               \
        if (smem > 48 * 1024 &&                                                                           \
            cudaFuncSetAttribute(attn_simt_kernel<QT, D, N>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                                 static_cast<int>(smem)) != cudaSuccess) {                                \
            return SDC_STATUS_CUDA_ERROR;                                                                 \
        }                                                                                                 \
        attn_simt_kernel<QT, D, N><<<grid, kThreadsAttn, smem, st>>>(a);                                  \
        break;
    switch (rpw) {
        SDC_SIMT_CASE(1)
        SDC_SIMT_CASE(2)
        SDC_SIMT_CASE(3)
        SDC_SIMT_CASE(4)
        SDC_SIMT_CASE(5)
        SDC_SIMT_CASE(6)
        SDC_SIMT_CASE(7)
        SDC_SIMT_CASE(8)
        default: return SDC_STATUS_UNSUPPORTED;
    }
#undef SDC_SIMT_CASE
    return launch_status();
}

template <typename QT>
sdc_status_t launch_combine_typed(const AttnArgs& a, cudaStream_t st, bool programmatic) {
    const int rpb = kCombineThreads / static_cast<int>(a.head_dim / 4);
    const size_t smem = static_cast<size_t>(a.max_chunks * rpb) * 3 * sizeof(float);
    if (smem > 48 * 1024 && cudaFuncSetAttribute(attn_combine_kernel<QT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 static_cast<int>(smem)) != cudaSuccess) {
        return SDC_STATUS_CUDA_ERROR;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(a.batch * a.kv_heads), static_cast<unsigned>((a.rows + rpb - 1) / rpb));
    cfg.blockDim = dim3(kCombineThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = programmatic ? 1 : 0;
    if (cudaLaunchKernelEx(&cfg, attn_combine_kernel<QT>, a) != cudaSuccess) return SDC_STATUS_CUDA_ERROR;
    return launch_status();
}

template <typename QT>
sdc_status_t launch_simt_typed(const AttnArgs& a, cudaStream_t st) {
    const int rpw = static_cast<int>((a.rows + kWarps - 1) / kWarps);
    dim3 grid(static_cast<unsigned>(a.max_chunks), static_cast<unsigned>(a.batch * a.kv_heads));
    sdc_status_t rc;
    switch (a.head_dim) {
        case 16: rc = launch_simt_rows<QT, 16>(a, rpw, grid, SimtSmem<16>::bytes(static_cast<int>(a.rows)), st); break;
        case 32: rc = launch_simt_rows<QT, 32>(a, rpw, grid, SimtSmem<32>::bytes(static_cast<int>(a.rows)), st); break;
        case 64: rc = launch_simt_rows<QT, 64>(a, rpw, grid, SimtSmem<64>::bytes(static_cast<int>(a.rows)), st); break;
        case 128: rc = launch_simt_rows<QT, 128>(a, rpw, grid, SimtSmem<128>::bytes(static_cast<int>(a.rows)), st); break;
        case 256: rc = launch_simt_rows<QT, 256>(a, rpw, grid, SimtSmem<256>::bytes(static_cast<int>(a.rows)), st); break;
        default: return SDC_STATUS_UNSUPPORTED;
    }
    if (rc != SDC_STATUS_OK) return rc;
    return launch_combine_typed<QT>(a, st, false);
}

}  // namespace

bool combine_fits(int64_t max_chunks, int64_t rows) { return max_chunks * rows <= kCombineMaxWeights; }

bool simt_supports(int64_t head_dim, int64_t rows) {
    return (head_dim == 16 || head_dim == 32 || head_dim == 64 || head_dim == 128 || head_dim == 256) && rows >= 1 &&
           rows <= kWarps * 8;
}

sdc_status_t launch_attention_combine(const AttnArgs& a, cudaStream_t st, bool programmatic) {
    switch (a.query_dtype) {
        case SDC_DTYPE_BF16: return launch_combine_typed<__nv_bfloat16>(a, st, programmatic);
        case SDC_DTYPE_F16: return launch_combine_typed<__half>(a, st, programmatic);
        case SDC_DTYPE_F32: return launch_combine_typed<float>(a, st, programmatic);
        default: return SDC_STATUS_UNSUPPORTED;
    }
}

sdc_status_t launch_attention_simt(const AttnArgs& a, cudaStream_t st) {
    switch (a.query_dtype) {
        case SDC_DTYPE_BF16: return launch_simt_typed<__nv_bfloat16>(a, st);
        case SDC_DTYPE_F16: return launch_simt_typed<__half>(a, st);
        case SDC_DTYPE_F32: return launch_simt_typed<float>(a, st);
        default: return SDC_STATUS_UNSUPPORTED;
    }
}

}  // namespace sdc
