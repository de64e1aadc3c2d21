/*
 * The reference's native sampling / quantization ABI, served by
 * libspecdecode_cuda.so on the GPU.
 *
 * The reference's Python loader (src/specdecode/native.py:77-160,
 * `_NativeLibrary`) binds nine `sd_*` functions from a shared library and
 * requires sd_abi_version() == 0x00010001 (native/include/specdecode/native.h:23-106).
 * libspecdecode_cuda.so exports those nine names with the same C signatures
 * and status numbering, so pointing the reference's loader at it
 * (SPECDECODE_NATIVE_LIBRARY, or NativeKVQuantizer.load(path)) runs the
 * reference's quantizer and sampling calls on the device unchanged.  Inputs
 * and outputs stay host buffers, as the reference's callers pass them: each
 * call copies its inputs to the device, runs the batched kernel of the
 * matching sdc_* entry point on one row, copies the results back and
 * synchronizes.
 *
 * Results equal the reference's: the same quantized codes and scale bits,
 * the same sampled index and first rejection, acceptance probabilities and
 * normalized / residual rows within the sdc_* functions' stated bounds.
 * Errors: host-side checks (null pointers, sizes, overflow, the sampling
 * uniform) come first and in the reference's order; value faults found on
 * the device (non-finite, negative, zero mass, token out of range, invalid
 * uniform) map to the reference's statuses.  When one call holds several
 * different faults, the status is the first of: invalid uniform, token out of
 * range, non-finite value, negative probability, zero mass -- where the
 * reference reports whichever it meets first while scanning.  A CUDA error,
 * or a sampling row longer than the kernels serve (2^21 entries), returns
 * SD_STATUS_INTERNAL_ERROR (9).
 */
#ifndef SPECDECODE_NATIVE_COMPAT_H
#define SPECDECODE_NATIVE_COMPAT_H

#include <stddef.h>
#include <stdint.h>

#include "specdecode_cuda.h"

#ifdef __cplusplus
extern "C" {
#endif

#define SDC_REFERENCE_NATIVE_ABI UINT32_C(0x00010001)

/* The reference's sd_status_t values are sdc_status_t values 0-10. */
SDC_API uint32_t sd_abi_version(void);
SDC_API const char* sd_status_string(int status);
SDC_API int sd_normalize_f64(const double* weights, size_t count, double* output);
SDC_API int sd_sample_categorical_f64(const double* weights, size_t count, double uniform_01,
                                      uint64_t* output_token);
SDC_API int sd_residual_weights_f64(const double* target, const double* draft, size_t vocabulary_size,
                                    double* output_weights);
SDC_API int sd_acceptance_probabilities_f64(const double* target_rows, const double* draft_rows,
                                            const uint64_t* proposed_tokens, size_t proposal_count,
                                            size_t vocabulary_size, double* output_probabilities);
SDC_API int sd_first_rejection_f64(const double* acceptance_probabilities, const double* uniforms,
                                   size_t proposal_count, size_t* output_accepted_count,
                                   size_t* output_rejection_index);
SDC_API int sd_quantize_symmetric_int8_f64(const double* values, size_t count, int8_t* output_values,
                                           double* output_scale);
SDC_API int sd_dequantize_symmetric_int8_f64(const int8_t* values, size_t count, double scale,
                                             double* output_values);

#ifdef __cplusplus
}
#endif

#endif /* SPECDECODE_NATIVE_COMPAT_H */
