// Shared device helpers for libspecdecode_cuda (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "specdecode_cuda.h"

namespace sdc {

constexpr unsigned kFullMask = 0xffffffffu;

// Pool descriptor passed to kernels by value.
struct Pool {
    int8_t* keys;
    int8_t* values;
    float* key_scales;
    float* value_scales;
    int64_t num_blocks, block_size, num_layers, num_heads, head_dim;
    int64_t cbs, cls, chs;  // code block / layer / head strides (elements)
    int64_t sbs, sls, shs;  // scale block / layer / head strides (elements)
};

struct TableEdits {
    int32_t* block_tables;
    int64_t table_stride;
    int64_t table_rows;
    int32_t* context_lens;
    const int32_t* entries;
    int64_t num_entries;
    const int32_t* lengths;
    int64_t num_lengths;
};

__device__ __forceinline__ void report_fault(int32_t* status, int32_t bits) {
    if (status != nullptr) atomicOr(status, bits);
}

// Unsigned 32-bit division by a run-time constant (Granlund-Montgomery):
// q = (t + ((n - t) >> 1)) >> (shift - 1) with t = umulhi(n, mul).  Exact
// for every 32-bit n and divisor >= 1.
struct FastDiv {
    uint32_t divisor;
    uint32_t mul;
    uint32_t shift;

    FastDiv() = default;
    __host__ explicit FastDiv(uint32_t d) : divisor(d) {
        uint32_t l = 0;
        while ((uint64_t(1) << l) < d) ++l;
        shift = l;
        mul = static_cast<uint32_t>(((uint64_t(1) << 32) * ((uint64_t(1) << l) - d)) / d + 1);
    }
    __device__ __forceinline__ uint32_t div(uint32_t n) const {
        if (shift == 0) return n;  // divisor 1
        const uint32_t t = __umulhi(n, mul);
        return (t + ((n - t) >> 1)) >> (shift - 1);
    }
    __device__ __forceinline__ void divmod(uint32_t n, uint32_t& q, uint32_t& r) const {
        q = div(n);
        r = n - q * divisor;
    }
};

// Loads 16 consecutive source elements (16-byte aligned) as Acc values.
__device__ __forceinline__ void load16(const float* p, float (&x)[16]) {
    const float4* q = reinterpret_cast<const float4*>(p);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        float4 v = __ldg(q + i);
        x[4 * i + 0] = v.x; x[4 * i + 1] = v.y; x[4 * i + 2] = v.z; x[4 * i + 3] = v.w;
    }
}

__device__ __forceinline__ void load16(const __nv_bfloat16* p, float (&x)[16]) {
    const uint4* q = reinterpret_cast<const uint4*>(p);
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        uint4 v = __ldg(q + i);
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            // bf16 -> f32 is exact: the bf16 bits are the high half of the f32 bits.
            x[8 * i + 2 * j + 0] = __uint_as_float(w[j] << 16);
            x[8 * i + 2 * j + 1] = __uint_as_float(w[j] & 0xffff0000u);
        }
    }
}

__device__ __forceinline__ void load16(const __half* p, float (&x)[16]) {
    const uint4* q = reinterpret_cast<const uint4*>(p);
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        uint4 v = __ldg(q + i);
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            __half2 h = *reinterpret_cast<const __half2*>(&w[j]);
            float2 f = __half22float2(h);
            x[8 * i + 2 * j + 0] = f.x;
            x[8 * i + 2 * j + 1] = f.y;
        }
    }
}

__device__ __forceinline__ void load16(const double* p, double (&x)[16]) {
    const double2* q = reinterpret_cast<const double2*>(p);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        double2 v = __ldg(q + i);
        x[2 * i + 0] = v.x; x[2 * i + 1] = v.y;
    }
}

// ---------------------------------------------------------------------------
// The reference's quantization rule (native/src/native.cpp:289-315):
//   scale = (double)(float)(max|x| / 127.0)
//   q     = clamp(round_half_away_from_zero(x / scale), -127, 127)
// with the division and rounding done in double.
// ---------------------------------------------------------------------------

// Scale from the vector maximum: a double division rounded once to float.
__device__ __forceinline__ float scale_from_max(double maximum) {
    return __double2float_rn(maximum / 127.0);
}

// Double path: the reference arithmetic verbatim.  CUDA's round() rounds
// halfway cases away from zero, like std::round.
__device__ __forceinline__ int quant_code_f64(double x, double scale) {
    double r = round(x / scale);
    r = fmin(fmax(r, -127.0), 127.0);
    return static_cast<int>(r);
}

// Float path for inputs that are float32 values (f32 / bf16 / f16 sources).
// Returns round_half_away(x / s) of the *exact* quotient using only float
// arithmetic.  A candidate n0 = rint(|x| * rcp) is within one of the answer
// (rcp = 1/s rounded once, so |x|*rcp is within 2^-22 relative of |x|/s).  It
// is corrected by the signs of |x| - (n0 + 1/2) s and |x| - (n0 - 1/2) s,
// each computed with one fused multiply-add: a correctly rounded result has
// the sign of the exact residual, and the residual cannot round to zero
// because it is zero or a multiple of at least 2^-149 (true whenever
// s >= 2^-100; smaller scales take the double path).  For a quotient of two
// float32 values the double-rounded quotient the reference rounds lands on
// the same integer as the exact one, because such a quotient is never within
// 2^-26 of a half-integer without being one.
__device__ __forceinline__ float quant_mag_f32(float a, float s, float rcp) {
    float n = rintf(a * rcp);
    n += (__fmaf_rn(-(n + 0.5f), s, a) >= 0.0f) ? 1.0f : 0.0f;
    n -= (__fmaf_rn(-(n - 0.5f), s, a) < 0.0f) ? 1.0f : 0.0f;
    return fminf(n, 127.0f);
}

__device__ __forceinline__ int quant_code_f32(float x, float s, float rcp) {
    const int q = static_cast<int>(quant_mag_f32(fabsf(x), s, rcp));
    return x < 0.0f ? -q : q;
}

constexpr float kFloatPathMinScale = 0x1p-100f;

__device__ __forceinline__ uint32_t pack4(int a, int b, int c, int d) {
    return (static_cast<uint32_t>(a) & 0xffu) | ((static_cast<uint32_t>(b) & 0xffu) << 8) |
           ((static_cast<uint32_t>(c) & 0xffu) << 16) | ((static_cast<uint32_t>(d) & 0xffu) << 24);
}

__device__ __forceinline__ void apply_table_edits(const TableEdits& e, int64_t index, int64_t stride,
                                                  int32_t* status) {
    for (int64_t i = index; i < e.num_entries; i += stride) {
        const int32_t row = e.entries[3 * i + 0];
        const int32_t col = e.entries[3 * i + 1];
        const int32_t val = e.entries[3 * i + 2];
        if (row < 0 || row >= e.table_rows || col < 0 || col >= e.table_stride) {
            report_fault(status, SDC_FAULT_TABLE_RANGE);
            continue;
        }
        e.block_tables[static_cast<int64_t>(row) * e.table_stride + col] = val;
    }
    for (int64_t i = index; i < e.num_lengths; i += stride) {
        const int32_t row = e.lengths[2 * i + 0];
        const int32_t len = e.lengths[2 * i + 1];
        if (row < 0 || row >= e.table_rows || len < 0) {
            report_fault(status, SDC_FAULT_TABLE_RANGE);
            continue;
        }
        e.context_lens[row] = len;
    }
}

}  // namespace sdc
