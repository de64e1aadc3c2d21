/*
 * ORACLE — test infrastructure only. Nothing in the product links this file;
 * only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg load it,
 * and only as the checker.
 *
 * A plain-C restatement of the reference's per-head symmetric INT8 quantizer:
 *   native/src/native.cpp:275-319  sd_quantize_symmetric_int8_f64
 *   native/src/native.cpp:321-353  sd_dequantize_symmetric_int8_f64
 *   src/specdecode/kv_cache.py:119-151  PythonKVQuantizer (same arithmetic)
 *
 * Arithmetic, in IEEE double throughout (no fast-math):
 *   m     = max_i |x_i|
 *   m==0  -> every code 0, scale exactly 0.0
 *   scale = (double)(float)(m / 127.0)     double division, then round to float32
 *   q_i   = clamp(round_half_away_from_zero(x_i / scale), -127, 127)
 * Validation happens before any output is written; non-finite input returns
 * status 3 (NONFINITE_VALUE), a float32 scale that is 0 or not finite returns
 * status 10 (INVALID_SCALE).  Status numbers follow native/include/specdecode/
 * native.h:25-37.
 *
 * The row-batched entry points apply the same per-vector rule to each row of a
 * row-major matrix and record one status per row; they exist so that large
 * parity cases and the CPU baseline do not pay one foreign call per vector.
 */
#include <math.h>
#include <stddef.h>
#include <stdint.h>

enum {
    ORACLE_OK = 0,
    ORACLE_NULL_ARGUMENT = 1,
    ORACLE_INVALID_SIZE = 2,
    ORACLE_NONFINITE_VALUE = 3,
    ORACLE_INVALID_SCALE = 10
};

int oracle_quantize_f64(const double* values, size_t count, int8_t* out_values, double* out_scale) {
    if (values == NULL || out_values == NULL || out_scale == NULL) {
        return ORACLE_NULL_ARGUMENT;
    }
    if (count == 0) {
        return ORACLE_INVALID_SIZE;
    }
    double maximum = 0.0;
    for (size_t i = 0; i < count; ++i) {
        if (!isfinite(values[i])) {
            return ORACLE_NONFINITE_VALUE;
        }
        double a = fabs(values[i]);
        if (a > maximum) {
            maximum = a;
        }
    }
    if (maximum == 0.0) {
        for (size_t i = 0; i < count; ++i) {
            out_values[i] = 0;
        }
        *out_scale = 0.0;
        return ORACLE_OK;
    }
    float float_scale = (float)(maximum / 127.0);
    if (!isfinite(float_scale) || float_scale == 0.0f) {
        return ORACLE_INVALID_SCALE;
    }
    double scale = (double)float_scale;
    for (size_t i = 0; i < count; ++i) {
        double r = round(values[i] / scale); /* C round(): halfway cases away from zero */
        if (r > 127.0) r = 127.0;
        if (r < -127.0) r = -127.0;
        out_values[i] = (int8_t)r;
    }
    *out_scale = scale;
    return ORACLE_OK;
}

int oracle_dequantize_f64(const int8_t* values, size_t count, double scale, double* out_values) {
    if (values == NULL || out_values == NULL) {
        return ORACLE_NULL_ARGUMENT;
    }
    if (count == 0) {
        return ORACLE_INVALID_SIZE;
    }
    if (!isfinite(scale) || scale < 0.0) {
        return ORACLE_INVALID_SCALE;
    }
    if (scale == 0.0) {
        for (size_t i = 0; i < count; ++i) {
            if (values[i] != 0) {
                return ORACLE_INVALID_SCALE;
            }
        }
    }
    for (size_t i = 0; i < count; ++i) {
        out_values[i] = (double)values[i] * scale;
    }
    return ORACLE_OK;
}

/* rows x count matrix of doubles -> rows x count codes, rows float32 scales. */
void oracle_quantize_rows_f64(const double* values, size_t rows, size_t count,
                              int8_t* out_values, float* out_scales, int32_t* out_status) {
    for (size_t r = 0; r < rows; ++r) {
        double scale = 0.0;
        int status = oracle_quantize_f64(values + r * count, count, out_values + r * count, &scale);
        out_status[r] = status;
        out_scales[r] = status == ORACLE_OK ? (float)scale : 0.0f;
    }
}

/* Same rule over float32 rows (a float32 value widens to double exactly). */
void oracle_quantize_rows_f32(const float* values, size_t rows, size_t count,
                              int8_t* out_values, float* out_scales, int32_t* out_status) {
    double buffer[4096];
    for (size_t r = 0; r < rows; ++r) {
        int status;
        double scale = 0.0;
        if (count > 4096) {
            status = ORACLE_INVALID_SIZE;
        } else {
            for (size_t i = 0; i < count; ++i) {
                buffer[i] = (double)values[r * count + i];
            }
            status = oracle_quantize_f64(buffer, count, out_values + r * count, &scale);
        }
        out_status[r] = status;
        out_scales[r] = status == ORACLE_OK ? (float)scale : 0.0f;
    }
}
