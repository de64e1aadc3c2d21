// Device-resident acceptance and sampling for speculative decoding.
//
// Batched device forms of the reference's native sampling functions
// (native/src/native.cpp:84-273): normalisation, categorical sampling from an
// explicit uniform, residual weights, acceptance probabilities and the first
// rejection, plus sdc_speculative_verify, which applies one verification
// round of the reference decoder (src/specdecode/decoder.py:206-257) to every
// sequence of a batch in two launches.
//
// Work mapping.  One 1024-thread block per probability row (per sequence for
// the resolving launch).  A row is cut into tiles of 4096 weights; warp w sums
// tiles w, w + 32, ...; lane l owns weights 4l .. 4l + 3 of each 128-weight
// chunk of the tile, so a warp's loads are contiguous.  Sampling walks the
// tile sums to the tile where the running sum passes the threshold, sums
// that tile's 32 chunks (one warp each) to find the chunk, and scans the
// chunk across one warp to find the weight.
//
// Arithmetic.  The reference sums weights in x87 extended precision with
// Kahan compensation (native.cpp:20-42) and forms its quotients in extended
// precision.  Here every sum is a double-double accumulation (Knuth's TwoSum,
// renormalised by Dekker's Fast2Sum; T. J. Dekker, "A floating-point
// technique for extending the available precision", 1971), and quotients are
// double-double (a double quotient refined twice by the exact remainder, as
// in Dekker's division).  Both are closer to the exact values than the
// reference's, so a decision (threshold < running sum, uniform <
// probability) can differ from the reference's only for a draw within about
// 1e-16 relative of the boundary: the ambiguity the reference accepts
// between its own Python and native backends.  Intrinsics with explicit
// rounding keep the compiler from contracting the error-free transformations.

#include <math_constants.h>

#include <cmath>

#include "host_common.h"

namespace sdc {
namespace {

constexpr int kThreads = 1024;
constexpr int kWarps = kThreads / 32;
constexpr int kChunk = 128;                // weights per warp step, four per lane
constexpr int kTile = kWarps * kChunk;     // 4096 weights
constexpr int64_t kMaxVocab = int64_t(1) << 21;
constexpr int kMaxTiles = static_cast<int>(kMaxVocab / kTile);

// ---------------------------------------------------------------------------
// Double-double arithmetic.
// ---------------------------------------------------------------------------

struct DD {
    double hi, lo;
};

// s + e == a + b exactly (Knuth's TwoSum; any a, b).
__device__ __forceinline__ DD two_sum(double a, double b) {
    const double s = __dadd_rn(a, b);
    const double bb = __dsub_rn(s, a);
    const double e = __dadd_rn(__dsub_rn(a, __dsub_rn(s, bb)), __dsub_rn(b, bb));
    return {s, e};
}

// s + e == a + b exactly when |a| >= |b| (Dekker's Fast2Sum).
__device__ __forceinline__ DD fast_two_sum(double a, double b) {
    const double s = __dadd_rn(a, b);
    return {s, __dsub_rn(b, __dsub_rn(s, a))};
}

// p + e == a * b exactly (the error of the product from one fused multiply-add).
__device__ __forceinline__ DD two_prod(double a, double b) {
    const double p = __dmul_rn(a, b);
    return {p, __fma_rn(a, b, -p)};
}

__device__ __forceinline__ DD dd_add(DD a, DD b) {
    const DD s = two_sum(a.hi, b.hi);
    const DD t = two_sum(a.lo, b.lo);
    const DD u = fast_two_sum(s.hi, __dadd_rn(s.lo, t.hi));
    return fast_two_sum(u.hi, __dadd_rn(u.lo, t.lo));
}

__device__ __forceinline__ DD dd_add(DD a, double b) {
    const DD s = two_sum(a.hi, b);
    return fast_two_sum(s.hi, __dadd_rn(s.lo, a.lo));
}

__device__ __forceinline__ DD dd_neg(DD a) { return {-a.hi, -a.lo}; }

__device__ __forceinline__ DD dd_mul(DD a, double b) {
    const DD p = two_prod(a.hi, b);
    return fast_two_sum(p.hi, __fma_rn(a.lo, b, p.lo));
}

// a / b for b > 0: q1 = a.hi / b.hi, then two corrections from the remainder
// a - b * (q1 + ...), each remainder formed in double-double.
__device__ __forceinline__ DD dd_div(DD a, DD b) {
    const double q1 = __ddiv_rn(a.hi, b.hi);
    DD r = dd_add(a, dd_neg(dd_mul(b, q1)));
    const double q2 = __ddiv_rn(r.hi, b.hi);
    r = dd_add(r, dd_neg(dd_mul(b, q2)));
    const double q3 = __ddiv_rn(r.hi, b.hi);
    return dd_add(fast_two_sum(q1, q2), q3);
}

// a < b for renormalised values (hi is the double nearest to the value).
__device__ __forceinline__ bool dd_lt(DD a, DD b) { return a.hi < b.hi || (a.hi == b.hi && a.lo < b.lo); }

__device__ __forceinline__ DD warp_sum(DD x) {
    // dd_add is symmetric in its arguments, so every lane ends with the same value.
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const DD y{__shfl_xor_sync(kFullMask, x.hi, o), __shfl_xor_sync(kFullMask, x.lo, o)};
        x = dd_add(x, y);
    }
    return x;
}

__device__ __forceinline__ DD warp_exclusive_scan(DD x, int lane) {
    DD inc = x;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const DD y{__shfl_up_sync(kFullMask, inc.hi, o), __shfl_up_sync(kFullMask, inc.lo, o)};
        if (lane >= o) inc = dd_add(y, inc);
    }
    const DD prev{__shfl_up_sync(kFullMask, inc.hi, 1), __shfl_up_sync(kFullMask, inc.lo, 1)};
    return lane == 0 ? DD{0.0, 0.0} : prev;
}

// ---------------------------------------------------------------------------
// Weight views and validation.
// ---------------------------------------------------------------------------

// The reference's per-weight checks (native.cpp:29-34) on the bit patterns,
// off the double-precision pipe.  A lane keeps two running maxima: of the
// magnitude bits (all-ones exponent or more: not finite) and of the raw
// bits (above the pattern of -0: a set sign bit on a non-zero: negative).
// Only the high word of a double matters for either test.
struct WeightCheck {
    uint32_t mag = 0, raw = 0;
    __device__ __forceinline__ void add(float x) {
        const uint32_t b = __float_as_uint(x);
        mag = max(mag, b & 0x7fffffffu);
        raw = max(raw, b);
    }
    __device__ __forceinline__ void add(double x) {
        const uint32_t h = static_cast<uint32_t>(static_cast<uint64_t>(__double_as_longlong(x)) >> 32);
        const uint32_t l = static_cast<uint32_t>(__double_as_longlong(x));
        // f64 exponent all ones <=> high word magnitude >= 0x7ff00000; a
        // negative non-zero has a high word above 0x80000000, or exactly
        // 0x80000000 with a non-zero low word
        mag = max(mag, (h & 0x7fffffffu) >= 0x7ff00000u ? 0x7f800000u : 0u);
        raw = max(raw, h > 0x80000000u || (h == 0x80000000u && l != 0) ? 0x80000001u : 0u);
    }
    __device__ __forceinline__ int faults() const {
        if (mag >= 0x7f800000u) return SDC_FAULT_NONFINITE_VALUE;
        return raw > 0x80000000u ? SDC_FAULT_NEGATIVE_WEIGHT : 0;
    }
};

__device__ __forceinline__ bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Weights v0 .. v0 + 3 of a row (v0 a multiple of 4), zero past the
// vocabulary: one 16-byte load (two for f64) where the row is 16-byte
// aligned and all four exist, element loads otherwise.
template <typename T>
__device__ __forceinline__ void load_quad(const T* row, bool vec, int64_t v0, int64_t vocab, T (&q)[4]) {
    if (vec && v0 + 3 < vocab) {
        if constexpr (sizeof(T) == 4) {
            const float4 f = __ldg(reinterpret_cast<const float4*>(row + v0));
            q[0] = f.x, q[1] = f.y, q[2] = f.z, q[3] = f.w;
        } else {
            const double2 a = __ldg(reinterpret_cast<const double2*>(row + v0));
            const double2 b = __ldg(reinterpret_cast<const double2*>(row + v0 + 2));
            q[0] = a.x, q[1] = a.y, q[2] = b.x, q[3] = b.y;
        }
    } else {
#pragma unroll
        for (int e = 0; e < 4; ++e) q[e] = v0 + e < vocab ? row[v0 + e] : T(0);
    }
}

template <typename T>
struct Stored {  // the row as stored
    const T* row;
    bool vec;
    __device__ explicit Stored(const T* r) : row(r), vec(aligned16(r)) {}
    __device__ __forceinline__ double operator()(int64_t v) const { return static_cast<double>(row[v]); }
    // Raw quads kept in flight: four per lane for f32 rows, two for f64.
    struct Raw {
        T q[4];
    };
    static constexpr int kDepth = sizeof(T) == 4 ? 4 : 2;
    __device__ __forceinline__ void load_raw(int64_t v0, int64_t vocab, Raw& r) const {
        load_quad(row, vec, v0, vocab, r.q);
    }
    template <bool Check>
    __device__ __forceinline__ void convert(const Raw& r, double (&x)[4], WeightCheck& check) const {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            if (Check) check.add(r.q[e]);
            x[e] = static_cast<double>(r.q[e]);
        }
    }
    template <bool Check>
    __device__ __forceinline__ void load4(int64_t v0, int64_t vocab, double (&x)[4], WeightCheck& check) const {
        Raw r;
        load_raw(v0, vocab, r);
        convert<Check>(r, x, check);
    }
};

// max(0, t[v] / S_t - d[v] / S_d) rounded to double (native.cpp:155-160),
// from the double-double reciprocals of the row sums: p = t * inv_t and
// q = d * inv_d are each an exact product of the high parts plus the low
// parts' contribution; p - q is an exact TwoSum of the high terms plus the
// low terms, rounded once.
template <typename T>
struct Residual {
    const T* t;
    const T* d;
    DD inv_t, inv_d;
    bool vec_t, vec_d;
    __device__ Residual(const T* t_, const T* d_, DD it, DD id)
        : t(t_), d(d_), inv_t(it), inv_d(id), vec_t(aligned16(t_)), vec_d(aligned16(d_)) {}
    __device__ __forceinline__ double value(double x, double y) const {
        const DD p = two_prod(inv_t.hi, x);
        const DD q = two_prod(inv_d.hi, y);
        const DD s = two_sum(p.hi, -q.hi);
        const double lo = __dsub_rn(__fma_rn(inv_t.lo, x, p.lo), __fma_rn(inv_d.lo, y, q.lo));
        const double r = __dadd_rn(s.hi, __dadd_rn(s.lo, lo));
        return r > 0.0 ? r : 0.0;
    }
    __device__ __forceinline__ double operator()(int64_t v) const {
        return value(static_cast<double>(t[v]), static_cast<double>(d[v]));
    }
    struct Raw {
        T a[4], b[4];
    };
    static constexpr int kDepth = 2;
    __device__ __forceinline__ void load_raw(int64_t v0, int64_t vocab, Raw& r) const {
        load_quad(t, vec_t, v0, vocab, r.a);
        load_quad(d, vec_d, v0, vocab, r.b);
    }
    template <bool Check>
    __device__ __forceinline__ void convert(const Raw& r, double (&x)[4], WeightCheck&) const {
#pragma unroll
        for (int e = 0; e < 4; ++e) x[e] = value(static_cast<double>(r.a[e]), static_cast<double>(r.b[e]));
    }
    template <bool Check>
    __device__ __forceinline__ void load4(int64_t v0, int64_t vocab, double (&x)[4], WeightCheck& check) const {
        Raw r;
        load_raw(v0, vocab, r);
        convert<Check>(r, x, check);
    }
};

// native.cpp:44-46: a uniform must be finite and in [0, 1).
__device__ __forceinline__ int uniform_faults(double u) { return (u >= 0.0 && u < 1.0) ? 0 : SDC_FAULT_INVALID_UNIFORM; }

__device__ __forceinline__ DD reciprocal(DD s) { return dd_div(DD{1.0, 0.0}, s); }

// ---------------------------------------------------------------------------
// Block-level row sums and search.
// ---------------------------------------------------------------------------

struct RowShared {
    DD tile[kMaxTiles];
    DD chunk[kWarps];
    DD total;
    DD base;
    int pick;
    int faults;
    int64_t index;
};

// Compensated sum: sum + comp carries the exact running sum up to the
// rounding of comp itself -- every addition's exact error (TwoSum, seven
// additions in all, no comparisons) lands in comp, whose own rounding stays
// below 2^-99 of the sum for a lane's 128 weights.
__device__ __forceinline__ void accumulate(double& sum, double& comp, const double (&x)[4]) {
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        const DD s = two_sum(sum, x[e]);
        comp = __dadd_rn(comp, s.lo);
        sum = s.hi;
    }
}

// Sums the row's tiles into sh.tile[] and their in-order total into
// sh.total.  With Check, ORs the weights' faults into the returned word
// (the same on every thread).  All threads of the block must call it.
template <bool Check, class W>
__device__ int row_sums(const W& w, int64_t vocab, RowShared& sh) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tiles = static_cast<int>((vocab + kTile - 1) / kTile);
    __syncthreads();  // earlier readers of sh are done
    if (threadIdx.x == 0) sh.faults = 0;
    __syncthreads();
    WeightCheck check;
    constexpr int kChunks = kTile / kChunk;
    for (int t = warp; t < tiles; t += kWarps) {
        // W::kDepth chunks of raw weights in flight per lane: each slot is
        // refilled with the chunk kDepth ahead as soon as it is converted;
        // two chains (even and odd slots) halve the addition latency
        constexpr int kDepth = W::kDepth;
        double sum0 = 0.0, comp0 = 0.0, sum1 = 0.0, comp1 = 0.0;
        const int64_t first = static_cast<int64_t>(t) * kTile + lane * 4;
        typename W::Raw buf[kDepth];
#pragma unroll
        for (int j = 0; j < kDepth; ++j) w.load_raw(first + static_cast<int64_t>(j) * kChunk, vocab, buf[j]);
#pragma unroll 1
        for (int c = 0; c < kChunks; c += kDepth) {
#pragma unroll
            for (int j = 0; j < kDepth; ++j) {
                double x[4];
                w.template convert<Check>(buf[j], x, check);
                if (c + kDepth + j < kChunks) {
                    w.load_raw(first + static_cast<int64_t>(c + kDepth + j) * kChunk, vocab, buf[j]);
                }
                if (j % 2 == 0) {
                    accumulate(sum0, comp0, x);
                } else {
                    accumulate(sum1, comp1, x);
                }
            }
        }
        DD acc = dd_add(fast_two_sum(sum0, comp0), fast_two_sum(sum1, comp1));
        acc = warp_sum(acc);
        if (lane == 0) sh.tile[t] = acc;
    }
    const int faults = Check ? check.faults() : 0;
    if (faults) atomicOr(&sh.faults, faults);
    __syncthreads();
    if (threadIdx.x == 0) {
        DD s{0.0, 0.0};
        for (int t = 0; t < tiles; ++t) s = dd_add(s, sh.tile[t]);
        sh.total = s;
    }
    __syncthreads();
    return sh.faults;
}

// The first v whose running sum w[0] + ... + w[v] exceeds `thr`, or vocab - 1
// if none does (native.cpp:123-133), given sh.tile[] from row_sums over the
// same weights.  All threads of the block must call it; all get the index.
template <class W>
__device__ int64_t row_search(const W& w, int64_t vocab, DD thr, RowShared& sh) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tiles = static_cast<int>((vocab + kTile - 1) / kTile);
    if (threadIdx.x == 0) {
        DD run{0.0, 0.0};
        int pick = -1;
        for (int t = 0; t < tiles; ++t) {
            const DD next = dd_add(run, sh.tile[t]);
            if (dd_lt(thr, next)) {
                pick = t;
                break;
            }
            run = next;
        }
        sh.pick = pick;
        sh.base = run;
        sh.index = vocab - 1;
    }
    __syncthreads();
    const int tile = sh.pick;
    if (tile >= 0) {
        const int64_t tile_first = static_cast<int64_t>(tile) * kTile;
        {
            const int64_t first = tile_first + warp * kChunk + lane * 4;
            double x[4];
            WeightCheck unused;
            w.template load4<false>(first, vocab, x, unused);
            DD acc{0.0, 0.0};
#pragma unroll
            for (int e = 0; e < 4; ++e) acc = dd_add(acc, x[e]);
            acc = warp_sum(acc);
            if (lane == 0) sh.chunk[warp] = acc;
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            const int64_t left = (vocab - tile_first + kChunk - 1) / kChunk;
            const int chunks = left < kWarps ? static_cast<int>(left) : kWarps;
            DD run = sh.base;
            int pick = chunks - 1;
            for (int c = 0; c < chunks; ++c) {
                const DD next = dd_add(run, sh.chunk[c]);
                if (dd_lt(thr, next) || c == chunks - 1) {
                    pick = c;
                    break;
                }
                run = next;
            }
            sh.pick = pick;
            sh.base = run;
        }
        __syncthreads();
        if (warp == 0) {
            const int64_t chunk_first = tile_first + static_cast<int64_t>(sh.pick) * kChunk;
            const int64_t first = chunk_first + lane * 4;
            double x[4];
            WeightCheck unused;
            w.template load4<false>(first, vocab, x, unused);
            DD mine{0.0, 0.0};
#pragma unroll
            for (int e = 0; e < 4; ++e) mine = dd_add(mine, x[e]);
            DD run = dd_add(sh.base, warp_exclusive_scan(mine, lane));
            int hit = 4;
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                run = dd_add(run, x[e]);
                if (hit == 4 && first + e < vocab && dd_lt(thr, run)) hit = e;
            }
            const unsigned found = __ballot_sync(kFullMask, hit < 4);
            if (found) {
                const int src = __ffs(found) - 1;
                const int64_t index = __shfl_sync(kFullMask, first + hit, src);
                if (lane == 0) sh.index = index;
            } else {
                // The chunk-level sums passed the threshold but the per-weight
                // running sum (added in another order) did not: the chunk's
                // last index with a positive weight, where its running sum
                // reaches the chunk's total (never a zero-weight or padding
                // index).
                int64_t last = -1;
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    if (first + e < vocab && x[e] > 0.0) last = first + e;
                }
#pragma unroll
                for (int off = 16; off > 0; off >>= 1) {
                    const int64_t other = __shfl_xor_sync(kFullMask, last, off);
                    last = other > last ? other : last;
                }
                if (lane == 0) sh.index = last >= 0 ? last : min(vocab - 1, chunk_first + kChunk - 1);
            }
        }
    }
    __syncthreads();
    const int64_t index = sh.index;
    __syncthreads();
    return index;
}

// ---------------------------------------------------------------------------
// Kernels.
// ---------------------------------------------------------------------------

template <typename T>
__global__ void __launch_bounds__(kThreads) normalize_kernel(const T* weights, int64_t vocab, int64_t stride,
                                                              double* out, int64_t out_stride, int32_t* status) {
    __shared__ RowShared sh;
    const int64_t r = blockIdx.x;
    const Stored<T> w(weights + r * stride);
    int faults = row_sums<true>(w, vocab, sh);
    if (!(sh.total.hi > 0.0)) faults |= SDC_FAULT_ZERO_MASS;
    if (faults) {
        if (threadIdx.x == 0) report_fault(status, faults);
        return;
    }
    const DD inv = reciprocal(sh.total);
    for (int64_t v = threadIdx.x; v < vocab; v += kThreads) out[r * out_stride + v] = dd_mul(inv, w(v)).hi;
}

template <typename T>
__global__ void __launch_bounds__(kThreads) categorical_kernel(const T* weights, int64_t vocab, int64_t stride,
                                                                const double* uniforms, int64_t* out,
                                                                int32_t* status) {
    __shared__ RowShared sh;
    const int64_t r = blockIdx.x;
    const Stored<T> w(weights + r * stride);
    const double u = uniforms[r];
    int faults = row_sums<true>(w, vocab, sh) | uniform_faults(u);
    if (!(sh.total.hi > 0.0)) faults |= SDC_FAULT_ZERO_MASS;
    if (faults) {
        if (threadIdx.x == 0) {
            out[r] = -1;
            report_fault(status, faults);
        }
        return;
    }
    const int64_t index = row_search(w, vocab, dd_mul(sh.total, u), sh);
    if (threadIdx.x == 0) out[r] = index;
}

// Sums and validates a target and a draft row; returns the faults, with the
// sums in *st / *sd.
template <typename T>
__device__ int pair_sums(const T* t, const T* d, int64_t vocab, RowShared& sh, DD* st, DD* sd) {
    int faults = row_sums<true>(Stored<T>(t), vocab, sh);
    *st = sh.total;
    faults |= row_sums<true>(Stored<T>(d), vocab, sh);
    *sd = sh.total;
    if (!(st->hi > 0.0) || !(sd->hi > 0.0)) faults |= SDC_FAULT_ZERO_MASS;
    return faults;
}

// native.cpp:145-176: residual weights, with the normalised target when the
// residual mass is at most 1e-15.
template <typename T>
__global__ void __launch_bounds__(kThreads) residual_kernel(const T* target, int64_t t_stride, const T* draft,
                                                             int64_t d_stride, int64_t vocab, double* out,
                                                             int64_t out_stride, int32_t* status) {
    __shared__ RowShared sh;
    const int64_t r = blockIdx.x;
    const T* t = target + r * t_stride;
    const T* d = draft + r * d_stride;
    DD st, sd;
    const int faults = pair_sums(t, d, vocab, sh, &st, &sd);
    if (faults) {
        if (threadIdx.x == 0) report_fault(status, faults);
        return;
    }
    const Residual<T> res(t, d, reciprocal(st), reciprocal(sd));
    row_sums<false>(res, vocab, sh);
    const bool fallback = !dd_lt(DD{1.0e-15, 0.0}, sh.total);
    double* o = out + r * out_stride;
    if (fallback) {
        for (int64_t v = threadIdx.x; v < vocab; v += kThreads) o[v] = dd_mul(res.inv_t, static_cast<double>(t[v])).hi;
    } else {
        for (int64_t v = threadIdx.x; v < vocab; v += kThreads) o[v] = res(v);
    }
}

// min(1, (t / S_t) / (d / S_d)) = min(1, t * S_d / (d * S_t)); 1 when d == 0
// (native.cpp:222-228).
__device__ __forceinline__ double acceptance(double t, double d, DD st, DD sd) {
    if (d == 0.0) return 1.0;
    const DD ratio = dd_div(dd_mul(sd, t), dd_mul(st, d));
    return ratio.hi >= 1.0 ? 1.0 : ratio.hi;
}

struct AcceptArgs {
    const void* target;
    const void* draft;
    int64_t t_seq, t_row, d_seq, d_row;
    int64_t proposals, vocab;
    const int64_t* tokens;
    int64_t token_stride;
    const int64_t* counts;
    double* out;   // [sequences][proposals]
    double* sums;  // [sequences][proposals][4]: S_t, S_d as double-doubles, or null
    int32_t* status;
};

// One block per (sequence, proposal): the acceptance probability of the
// proposal (native.cpp:198-229, one row).
template <typename T>
__global__ void __launch_bounds__(kThreads) acceptance_kernel(AcceptArgs a) {
    __shared__ RowShared sh;
    const int64_t s = blockIdx.x, i = blockIdx.y;
    const int64_t n = a.counts != nullptr ? a.counts[s] : a.proposals;
    if (n < 1 || n > a.proposals || i >= n) return;  // the resolving launch reports bad counts
    const T* t = static_cast<const T*>(a.target) + s * a.t_seq + i * a.t_row;
    const T* d = static_cast<const T*>(a.draft) + s * a.d_seq + i * a.d_row;
    const int64_t token = a.tokens[s * a.token_stride + i];
    DD st, sd;
    int faults = pair_sums(t, d, a.vocab, sh, &st, &sd);
    if (token < 0 || token >= a.vocab) faults |= SDC_FAULT_TOKEN_RANGE;
    if (threadIdx.x != 0) return;
    double* out = a.out + s * a.proposals + i;
    if (faults) {
        *out = CUDART_NAN;
        report_fault(a.status, faults);
        return;
    }
    *out = acceptance(static_cast<double>(t[token]), static_cast<double>(d[token]), st, sd);
    if (a.sums != nullptr) {
        double* w = a.sums + (s * a.proposals + i) * 4;
        w[0] = st.hi, w[1] = st.lo, w[2] = sd.hi, w[3] = sd.lo;
    }
}

// native.cpp:247-272 for one row of probabilities and uniforms.
__device__ __forceinline__ int64_t first_rejection(const double* p, const double* u, int64_t n, int* faults) {
    for (int64_t i = 0; i < n; ++i) {
        if (!isfinite(p[i])) *faults |= SDC_FAULT_NONFINITE_VALUE;
        else if (p[i] < 0.0 || p[i] > 1.0) *faults |= SDC_FAULT_NEGATIVE_WEIGHT;
        *faults |= uniform_faults(u[i]);
    }
    if (*faults) return -1;
    for (int64_t i = 0; i < n; ++i) {
        if (!(u[i] < p[i])) return i;
    }
    return n;
}

__global__ void first_rejection_kernel(const double* p, const double* u, int64_t sequences, int64_t proposals,
                                       int64_t stride, int64_t* out, int32_t* status) {
    const int64_t s = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (s >= sequences) return;
    int faults = 0;
    out[s] = first_rejection(p + s * stride, u + s * stride, proposals, &faults);
    if (faults) report_fault(status, faults);
}

struct ResolveArgs {
    const void* target;
    const void* draft;
    int64_t t_seq, t_row, d_seq, d_row;
    int64_t proposals, vocab;
    const double* probs;  // [sequences][proposals]
    const double* uniforms;
    int64_t uniform_stride;
    const int64_t* counts;
    const uint8_t* bonus;
    const double* sums;  // written by acceptance_kernel, or null
    int64_t* accepted;
    int64_t* tokens;
    int32_t* status;
};

// One block per sequence: the first rejection, then the correction sample
// from the residual of the rejected row, or the bonus sample from the last
// target row (decoder.py:218-257).
template <typename T>
__global__ void __launch_bounds__(kThreads) resolve_kernel(ResolveArgs a) {
    __shared__ RowShared sh;
    __shared__ int64_t s_reject;
    __shared__ int s_faults;
    const int64_t s = blockIdx.x;
    const int64_t n = a.counts != nullptr ? a.counts[s] : a.proposals;
    const double* u = a.uniforms + s * a.uniform_stride;
    if (threadIdx.x == 0) {
        int faults = 0;
        int64_t j = -1;
        if (n < 1 || n > a.proposals) {
            faults = SDC_FAULT_PROPOSAL_COUNT;
        } else {
            j = first_rejection(a.probs + s * a.proposals, u, n, &faults);
            faults |= uniform_faults(u[n]);
        }
        s_reject = j;
        s_faults = faults;
    }
    __syncthreads();
    const int64_t j = s_reject;
    int faults = s_faults;
    int64_t token = -1;
    if (!faults && j < n) {
        const T* t = static_cast<const T*>(a.target) + s * a.t_seq + j * a.t_row;
        const T* d = static_cast<const T*>(a.draft) + s * a.d_seq + j * a.d_row;
        DD st, sd;
        if (a.sums != nullptr) {
            // validated, and the row sums formed, by the acceptance launch
            const double* w = a.sums + (s * a.proposals + j) * 4;
            st = DD{w[0], w[1]};
            sd = DD{w[2], w[3]};
        } else {
            faults |= pair_sums(t, d, a.vocab, sh, &st, &sd);
        }
        if (!faults) {
            const Residual<T> res(t, d, reciprocal(st), reciprocal(sd));
            row_sums<false>(res, a.vocab, sh);
            if (dd_lt(DD{1.0e-15, 0.0}, sh.total)) {
                token = row_search(res, a.vocab, dd_mul(sh.total, u[j + 1]), sh);
            } else {
                const Stored<T> w(t);
                row_sums<false>(w, a.vocab, sh);
                token = row_search(w, a.vocab, dd_mul(sh.total, u[j + 1]), sh);
            }
        }
    } else if (!faults && (a.bonus == nullptr || a.bonus[s] != 0)) {
        const Stored<T> w(static_cast<const T*>(a.target) + s * a.t_seq + n * a.t_row);
        faults |= row_sums<true>(w, a.vocab, sh);
        if (!(sh.total.hi > 0.0)) faults |= SDC_FAULT_ZERO_MASS;
        if (!faults) token = row_search(w, a.vocab, dd_mul(sh.total, u[n]), sh);
    }
    if (threadIdx.x == 0) {
        if (faults) {
            a.accepted[s] = -1;
            a.tokens[s] = -1;
            report_fault(a.status, faults);
        } else {
            a.accepted[s] = j;
            a.tokens[s] = token;
        }
    }
}

// ---------------------------------------------------------------------------
// Host validation.
// ---------------------------------------------------------------------------

sdc_status_t check_rows(const void* p, int dtype, int64_t rows, int64_t vocab, int64_t stride) {
    if (p == nullptr) return SDC_STATUS_NULL_ARGUMENT;
    if (dtype != SDC_DTYPE_F32 && dtype != SDC_DTYPE_F64) return SDC_STATUS_UNSUPPORTED;
    if (rows < 1 || vocab < 1) return SDC_STATUS_INVALID_SIZE;
    if (vocab > kMaxVocab) return SDC_STATUS_UNSUPPORTED;
    if (stride < vocab) return SDC_STATUS_INVALID_SIZE;
    if (rows > (int64_t(1) << 31) - 1 || stride > (int64_t(1) << 40) / rows) return SDC_STATUS_OVERFLOW;
    if (reinterpret_cast<uintptr_t>(p) % dtype_size(dtype)) return SDC_STATUS_MISALIGNED;
    return SDC_STATUS_OK;
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

SDC_API sdc_status_t sdc_normalize_rows(const void* weights, int dtype, int64_t rows, int64_t vocab,
                                        int64_t row_stride, double* output, int64_t output_stride,
                                        int32_t* device_status, uintptr_t stream) {
    return guarded([&]() -> sdc_status_t {
        sdc_status_t st = check_rows(weights, dtype, rows, vocab, row_stride);
        if (st != SDC_STATUS_OK) return st;
        if (output == nullptr) return SDC_STATUS_NULL_ARGUMENT;
        if (output_stride < vocab || output_stride > (int64_t(1) << 40) / rows) return SDC_STATUS_INVALID_SIZE;
        const dim3 grid(static_cast<unsigned>(rows));
        if (dtype == SDC_DTYPE_F32) {
            normalize_kernel<float><<<grid, kThreads, 0, as_stream(stream)>>>(
                static_cast<const float*>(weights), vocab, row_stride, output, output_stride, device_status);
        } else {
            normalize_kernel<double><<<grid, kThreads, 0, as_stream(stream)>>>(
                static_cast<const double*>(weights), vocab, row_stride, output, output_stride, device_status);
        }
        return launch_status();
    });
}

SDC_API sdc_status_t sdc_sample_categorical_rows(const void* weights, int dtype, int64_t rows, int64_t vocab,
                                                 int64_t row_stride, const double* uniforms, int64_t* output_tokens,
                                                 int32_t* device_status, uintptr_t stream) {
    return guarded([&]() -> sdc_status_t {
        sdc_status_t st = check_rows(weights, dtype, rows, vocab, row_stride);
        if (st != SDC_STATUS_OK) return st;
        if (uniforms == nullptr || output_tokens == nullptr) return SDC_STATUS_NULL_ARGUMENT;
        const dim3 grid(static_cast<unsigned>(rows));
        if (dtype == SDC_DTYPE_F32) {
            categorical_kernel<float><<<grid, kThreads, 0, as_stream(stream)>>>(
                static_cast<const float*>(weights), vocab, row_stride, uniforms, output_tokens, device_status);
        } else {
            categorical_kernel<double><<<grid, kThreads, 0, as_stream(stream)>>>(
                static_cast<const double*>(weights), vocab, row_stride, uniforms, output_tokens, device_status);
        }
        return launch_status();
    });
}

SDC_API sdc_status_t sdc_residual_weights_rows(const void* target, const void* draft, int dtype, int64_t rows,
                                               int64_t vocab, int64_t target_stride, int64_t draft_stride,
                                               double* output, int64_t output_stride, int32_t* device_status,
                                               uintptr_t stream) {
    return guarded([&]() -> sdc_status_t {
        sdc_status_t st = check_rows(target, dtype, rows, vocab, target_stride);
        if (st == SDC_STATUS_OK) st = check_rows(draft, dtype, rows, vocab, draft_stride);
        if (st != SDC_STATUS_OK) return st;
        if (output == nullptr) return SDC_STATUS_NULL_ARGUMENT;
        if (output_stride < vocab || output_stride > (int64_t(1) << 40) / rows) return SDC_STATUS_INVALID_SIZE;
        const dim3 grid(static_cast<unsigned>(rows));
        if (dtype == SDC_DTYPE_F32) {
            residual_kernel<float><<<grid, kThreads, 0, as_stream(stream)>>>(
                static_cast<const float*>(target), target_stride, static_cast<const float*>(draft), draft_stride,
                vocab, output, output_stride, device_status);
        } else {
            residual_kernel<double><<<grid, kThreads, 0, as_stream(stream)>>>(
                static_cast<const double*>(target), target_stride, static_cast<const double*>(draft), draft_stride,
                vocab, output, output_stride, device_status);
        }
        return launch_status();
    });
}

SDC_API sdc_status_t sdc_acceptance_probabilities_rows(const void* target, const void* draft, int dtype,
                                                       int64_t rows, int64_t vocab, int64_t target_stride,
                                                       int64_t draft_stride, const int64_t* proposed_tokens,
                                                       double* output_probabilities, int32_t* device_status,
                                                       uintptr_t stream) {
    return guarded([&]() -> sdc_status_t {
        sdc_status_t st = check_rows(target, dtype, rows, vocab, target_stride);
        if (st == SDC_STATUS_OK) st = check_rows(draft, dtype, rows, vocab, draft_stride);
        if (st != SDC_STATUS_OK) return st;
        if (proposed_tokens == nullptr || output_probabilities == nullptr) return SDC_STATUS_NULL_ARGUMENT;
        // rows independent proposals: `rows` sequences of one proposal each
        AcceptArgs a{target, draft, target_stride, 0, draft_stride, 0, 1, vocab, proposed_tokens, 1,
                     nullptr, output_probabilities, nullptr, device_status};
        const dim3 grid(static_cast<unsigned>(rows), 1);
        if (dtype == SDC_DTYPE_F32) {
            acceptance_kernel<float><<<grid, kThreads, 0, as_stream(stream)>>>(a);
        } else {
            acceptance_kernel<double><<<grid, kThreads, 0, as_stream(stream)>>>(a);
        }
        return launch_status();
    });
}

SDC_API sdc_status_t sdc_first_rejection_rows(const double* acceptance_probabilities, const double* uniforms,
                                              int64_t sequences, int64_t proposals, int64_t row_stride,
                                              int64_t* output_accepted, int32_t* device_status, uintptr_t stream) {
    return guarded([&]() -> sdc_status_t {
        if (acceptance_probabilities == nullptr || uniforms == nullptr || output_accepted == nullptr) {
            return SDC_STATUS_NULL_ARGUMENT;
        }
        if (sequences < 1 || proposals < 0 || row_stride < proposals) return SDC_STATUS_INVALID_SIZE;
        if (sequences > (int64_t(1) << 31) - 1 || row_stride > (int64_t(1) << 40) / sequences) {
            return SDC_STATUS_OVERFLOW;
        }
        const int threads = 128;
        first_rejection_kernel<<<static_cast<unsigned>(ceil_div(sequences, threads)), threads, 0,
                                 as_stream(stream)>>>(acceptance_probabilities, uniforms, sequences, proposals,
                                                      row_stride, output_accepted, device_status);
        return launch_status();
    });
}

SDC_API sdc_status_t sdc_speculative_verify(const sdc_verify_batch_t* batch, double* output_probabilities,
                                            int64_t* output_accepted, int64_t* output_tokens, double* row_sums,
                                            int32_t* device_status, uintptr_t stream) {
    return guarded([&]() -> sdc_status_t {
        if (batch == nullptr || output_probabilities == nullptr || output_accepted == nullptr ||
            output_tokens == nullptr || batch->proposed_tokens == nullptr || batch->uniforms == nullptr) {
            return SDC_STATUS_NULL_ARGUMENT;
        }
        const sdc_verify_batch_t& b = *batch;
        if (b.sequences < 1 || b.proposals < 1 || b.vocab < 1) return SDC_STATUS_INVALID_SIZE;
        if (b.proposals > 65535) return SDC_STATUS_OVERFLOW;
        // The target has proposals + 1 rows per sequence, the draft proposals.
        const int64_t t_span = b.proposals * b.target_row_stride + b.vocab;
        const int64_t d_span = (b.proposals - 1) * b.draft_row_stride + b.vocab;
        sdc_status_t st = check_rows(b.target_rows, b.dtype, b.sequences, b.vocab, b.target_sequence_stride);
        if (st == SDC_STATUS_OK) st = check_rows(b.draft_rows, b.dtype, b.sequences, b.vocab, b.draft_sequence_stride);
        if (st != SDC_STATUS_OK) return st;
        if (b.target_row_stride < b.vocab || b.draft_row_stride < b.vocab) return SDC_STATUS_INVALID_SIZE;
        if (b.target_row_stride > (int64_t(1) << 40) / (b.proposals + 1) ||
            b.draft_row_stride > (int64_t(1) << 40) / (b.proposals + 1)) {
            return SDC_STATUS_OVERFLOW;
        }
        if (b.target_sequence_stride < t_span || b.draft_sequence_stride < d_span) return SDC_STATUS_INVALID_SIZE;
        if (b.token_stride < b.proposals || b.uniform_stride < b.proposals + 1) return SDC_STATUS_INVALID_SIZE;
        if (b.token_stride > (int64_t(1) << 40) / b.sequences || b.uniform_stride > (int64_t(1) << 40) / b.sequences) {
            return SDC_STATUS_OVERFLOW;
        }
        AcceptArgs a{b.target_rows, b.draft_rows, b.target_sequence_stride, b.target_row_stride,
                     b.draft_sequence_stride, b.draft_row_stride, b.proposals, b.vocab, b.proposed_tokens,
                     b.token_stride, b.proposal_counts, output_probabilities, row_sums, device_status};
        ResolveArgs r{b.target_rows, b.draft_rows, b.target_sequence_stride, b.target_row_stride,
                      b.draft_sequence_stride, b.draft_row_stride, b.proposals, b.vocab, output_probabilities,
                      b.uniforms, b.uniform_stride, b.proposal_counts, b.bonus_allowed, row_sums, output_accepted,
                      output_tokens, device_status};
        const dim3 grid_a(static_cast<unsigned>(b.sequences), static_cast<unsigned>(b.proposals));
        const dim3 grid_r(static_cast<unsigned>(b.sequences));
        cudaStream_t s = as_stream(stream);
        if (b.dtype == SDC_DTYPE_F32) {
            acceptance_kernel<float><<<grid_a, kThreads, 0, s>>>(a);
            resolve_kernel<float><<<grid_r, kThreads, 0, s>>>(r);
        } else {
            acceptance_kernel<double><<<grid_a, kThreads, 0, s>>>(a);
            resolve_kernel<double><<<grid_r, kThreads, 0, s>>>(r);
        }
        return launch_status();
    });
}

}  // extern "C"
