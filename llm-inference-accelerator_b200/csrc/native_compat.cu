// The reference's nine sd_* native functions (native/include/specdecode/native.h,
// loaded by src/specdecode/native.py:77-160) served on the GPU: host buffers
// in and out, the computation in the batched sdc_* kernels on one row.  See
// include/specdecode_native_compat.h for the contract.

#include <algorithm>
#include <cmath>
#include <limits>
#include <vector>

#include "host_common.h"
#include "specdecode_native_compat.h"

namespace sdc {
namespace {

// The reference's status messages (its sd_status_string), which its Python
// loader puts into NativeBackendError.
const char* reference_message(int status) {
    switch (status) {
        case 0: return "ok";
        case 1: return "null argument";
        case 2: return "invalid size";
        case 3: return "non-finite value";
        case 4: return "negative probability";
        case 5: return "zero probability mass";
        case 6: return "token out of range";
        case 7: return "uniform must be finite and in [0, 1)";
        case 8: return "size overflow";
        case 9: return "internal error";
        case 10: return "quantization scale must be finite and non-negative";
        default: return "unknown status";
    }
}

bool bad_uniform(double u) { return !std::isfinite(u) || u < 0.0 || u >= 1.0; }

// Status of the device fault bits, in a fixed order.
int status_of_faults(int32_t bits) {
    if (bits == 0) return SDC_STATUS_OK;
    if (bits & SDC_FAULT_INVALID_UNIFORM) return SDC_STATUS_INVALID_UNIFORM;
    if (bits & SDC_FAULT_TOKEN_RANGE) return SDC_STATUS_TOKEN_OUT_OF_RANGE;
    if (bits & SDC_FAULT_NONFINITE_VALUE) return SDC_STATUS_NONFINITE_VALUE;
    if (bits & SDC_FAULT_NEGATIVE_WEIGHT) return SDC_STATUS_NEGATIVE_PROBABILITY;
    if (bits & SDC_FAULT_ZERO_MASS) return SDC_STATUS_ZERO_MASS;
    return SDC_STATUS_INTERNAL_ERROR;
}

// Device scratch of one call, carved into 16-byte aligned pieces, on the
// calling thread's default stream; freed (stream-ordered) on destruction.
class Scratch {
  public:
    explicit Scratch(size_t bytes) : stream_(cudaStreamPerThread) {
        ok_ = cudaMallocAsync(reinterpret_cast<void**>(&base_), bytes + 16, stream_) == cudaSuccess &&
              cudaMemsetAsync(base_, 0, 16, stream_) == cudaSuccess;  // the status word
        used_ = 16;
    }
    ~Scratch() {
        if (base_ != nullptr) cudaFreeAsync(base_, stream_);
    }
    Scratch(const Scratch&) = delete;
    Scratch& operator=(const Scratch&) = delete;

    bool ok() const { return ok_; }
    int32_t* status() { return reinterpret_cast<int32_t*>(base_); }
    uintptr_t stream() const { return reinterpret_cast<uintptr_t>(stream_); }
    template <typename T>
    T* take(size_t count) {
        T* p = reinterpret_cast<T*>(base_ + used_);
        used_ += (count * sizeof(T) + 15) & ~size_t(15);
        return p;
    }
    template <typename T>
    T* upload(const T* host, size_t count) {
        T* p = take<T>(count);
        if (ok_ && cudaMemcpyAsync(p, host, count * sizeof(T), cudaMemcpyHostToDevice, stream_) != cudaSuccess) {
            ok_ = false;
        }
        return p;
    }
    // Launch result of an sdc_* entry point: its host-side errors pass
    // through when the reference has the status (0-10); the others (a row
    // longer than the kernels serve, a CUDA error) are internal errors.
    int launched(sdc_status_t rc) {
        if (rc != SDC_STATUS_OK) ok_ = false;
        return rc <= SDC_STATUS_INVALID_SCALE ? rc : SDC_STATUS_INTERNAL_ERROR;
    }
    // Copies `count` T back, synchronizes, and returns the call's status.
    template <typename T>
    int finish(T* host, const T* device, size_t count) {
        int32_t bits = 0;
        if (ok_ && count > 0 &&
            cudaMemcpyAsync(host, device, count * sizeof(T), cudaMemcpyDeviceToHost, stream_) != cudaSuccess) {
            ok_ = false;
        }
        if (ok_ && cudaMemcpyAsync(&bits, base_, sizeof(bits), cudaMemcpyDeviceToHost, stream_) != cudaSuccess) {
            ok_ = false;
        }
        if (cudaStreamSynchronize(stream_) != cudaSuccess) ok_ = false;
        return ok_ ? status_of_faults(bits) : SDC_STATUS_INTERNAL_ERROR;
    }

  private:
    cudaStream_t stream_;
    char* base_ = nullptr;
    size_t used_ = 0;
    bool ok_ = false;
};

constexpr size_t kMaxElements = size_t(1) << 40;

}  // namespace
}  // namespace sdc

using namespace sdc;

extern "C" {

SDC_API uint32_t sd_abi_version(void) { return SDC_REFERENCE_NATIVE_ABI; }

SDC_API const char* sd_status_string(int status) { return reference_message(status); }

SDC_API int sd_normalize_f64(const double* weights, size_t count, double* output) {
    try {
        if (output == nullptr || weights == nullptr) return SDC_STATUS_NULL_ARGUMENT;
        if (count == 0) return SDC_STATUS_INVALID_SIZE;
        if (count > kMaxElements) return SDC_STATUS_OVERFLOW;
        Scratch s(2 * count * sizeof(double) + 64);
        if (!s.ok()) return SDC_STATUS_INTERNAL_ERROR;
        const double* w = s.upload(weights, count);
        double* out = s.take<double>(count);
        const int64_t n = static_cast<int64_t>(count);
        const int rc = s.launched(sdc_normalize_rows(w, SDC_DTYPE_F64, 1, n, n, out, n, s.status(), s.stream()));
        if (rc != SDC_STATUS_OK) return rc;
        // a faulted row is not written: copy back only a good result
        std::vector<double> result(count);
        const int st = s.finish(result.data(), out, count);
        if (st == SDC_STATUS_OK) std::copy(result.begin(), result.end(), output);
        return st;
    } catch (...) {
        return SDC_STATUS_INTERNAL_ERROR;
    }
}

SDC_API int sd_sample_categorical_f64(const double* weights, size_t count, double uniform_01, uint64_t* output_token) {
    try {
        if (output_token == nullptr) return SDC_STATUS_NULL_ARGUMENT;
        if (bad_uniform(uniform_01)) return SDC_STATUS_INVALID_UNIFORM;
        if (weights == nullptr) return SDC_STATUS_NULL_ARGUMENT;
        if (count == 0) return SDC_STATUS_INVALID_SIZE;
        if (count > kMaxElements) return SDC_STATUS_OVERFLOW;
        Scratch s(count * sizeof(double) + 64);
        if (!s.ok()) return SDC_STATUS_INTERNAL_ERROR;
        const double* w = s.upload(weights, count);
        const double* u = s.upload(&uniform_01, 1);
        int64_t* token = s.take<int64_t>(1);
        const int64_t n = static_cast<int64_t>(count);
        const int rc =
            s.launched(sdc_sample_categorical_rows(w, SDC_DTYPE_F64, 1, n, n, u, token, s.status(), s.stream()));
        if (rc != SDC_STATUS_OK) return rc;
        int64_t index = -1;
        const int st = s.finish(&index, token, 1);
        if (st == SDC_STATUS_OK) {
            if (index < 0) return SDC_STATUS_INTERNAL_ERROR;
            *output_token = static_cast<uint64_t>(index);
        }
        return st;
    } catch (...) {
        return SDC_STATUS_INTERNAL_ERROR;
    }
}

SDC_API int sd_residual_weights_f64(const double* target, const double* draft, size_t vocabulary_size,
                                    double* output_weights) {
    try {
        if (output_weights == nullptr || target == nullptr) return SDC_STATUS_NULL_ARGUMENT;
        if (vocabulary_size == 0) return SDC_STATUS_INVALID_SIZE;
        if (draft == nullptr) return SDC_STATUS_NULL_ARGUMENT;
        if (vocabulary_size > kMaxElements) return SDC_STATUS_OVERFLOW;
        Scratch s(3 * vocabulary_size * sizeof(double) + 64);
        if (!s.ok()) return SDC_STATUS_INTERNAL_ERROR;
        const double* t = s.upload(target, vocabulary_size);
        const double* d = s.upload(draft, vocabulary_size);
        double* out = s.take<double>(vocabulary_size);
        const int64_t n = static_cast<int64_t>(vocabulary_size);
        const int rc = s.launched(
            sdc_residual_weights_rows(t, d, SDC_DTYPE_F64, 1, n, n, n, out, n, s.status(), s.stream()));
        if (rc != SDC_STATUS_OK) return rc;
        std::vector<double> result(vocabulary_size);
        const int st = s.finish(result.data(), out, vocabulary_size);
        if (st == SDC_STATUS_OK) std::copy(result.begin(), result.end(), output_weights);
        return st;
    } catch (...) {
        return SDC_STATUS_INTERNAL_ERROR;
    }
}

SDC_API int sd_acceptance_probabilities_f64(const double* target_rows, const double* draft_rows,
                                            const uint64_t* proposed_tokens, size_t proposal_count,
                                            size_t vocabulary_size, double* output_probabilities) {
    try {
        if (target_rows == nullptr || draft_rows == nullptr || proposed_tokens == nullptr ||
            output_probabilities == nullptr) {
            return SDC_STATUS_NULL_ARGUMENT;
        }
        if (proposal_count == 0 || vocabulary_size == 0) return SDC_STATUS_INVALID_SIZE;
        if (proposal_count > std::numeric_limits<size_t>::max() / vocabulary_size) return SDC_STATUS_OVERFLOW;
        const size_t elements = proposal_count * vocabulary_size;
        if (elements > kMaxElements) return SDC_STATUS_OVERFLOW;
        // a token at or past the vocabulary (any uint64) becomes out of range
        std::vector<int64_t> tokens(proposal_count);
        for (size_t i = 0; i < proposal_count; ++i) {
            tokens[i] = proposed_tokens[i] >= vocabulary_size ? -1 : static_cast<int64_t>(proposed_tokens[i]);
        }
        Scratch s(2 * elements * sizeof(double) + 2 * proposal_count * 8 + 64);
        if (!s.ok()) return SDC_STATUS_INTERNAL_ERROR;
        const double* t = s.upload(target_rows, elements);
        const double* d = s.upload(draft_rows, elements);
        const int64_t* tok = s.upload(tokens.data(), proposal_count);
        double* out = s.take<double>(proposal_count);
        const int64_t rows = static_cast<int64_t>(proposal_count), v = static_cast<int64_t>(vocabulary_size);
        const int rc = s.launched(sdc_acceptance_probabilities_rows(t, d, SDC_DTYPE_F64, rows, v, v, v, tok, out,
                                                                    s.status(), s.stream()));
        if (rc != SDC_STATUS_OK) return rc;
        std::vector<double> result(proposal_count);
        const int st = s.finish(result.data(), out, proposal_count);
        if (st == SDC_STATUS_OK) std::copy(result.begin(), result.end(), output_probabilities);
        return st;
    } catch (...) {
        return SDC_STATUS_INTERNAL_ERROR;
    }
}

SDC_API int sd_first_rejection_f64(const double* acceptance_probabilities, const double* uniforms,
                                   size_t proposal_count, size_t* output_accepted_count,
                                   size_t* output_rejection_index) {
    try {
        if (output_accepted_count == nullptr || output_rejection_index == nullptr) return SDC_STATUS_NULL_ARGUMENT;
        if (proposal_count > 0 && (acceptance_probabilities == nullptr || uniforms == nullptr)) {
            return SDC_STATUS_NULL_ARGUMENT;
        }
        if (proposal_count == 0) {
            *output_accepted_count = 0;
            *output_rejection_index = 0;
            return SDC_STATUS_OK;
        }
        if (proposal_count > kMaxElements) return SDC_STATUS_OVERFLOW;
        Scratch s(2 * proposal_count * sizeof(double) + 64);
        if (!s.ok()) return SDC_STATUS_INTERNAL_ERROR;
        const double* p = s.upload(acceptance_probabilities, proposal_count);
        const double* u = s.upload(uniforms, proposal_count);
        int64_t* accepted = s.take<int64_t>(1);
        const int64_t n = static_cast<int64_t>(proposal_count);
        const int rc = s.launched(sdc_first_rejection_rows(p, u, 1, n, n, accepted, s.status(), s.stream()));
        if (rc != SDC_STATUS_OK) return rc;
        int64_t count = -1;
        const int st = s.finish(&count, accepted, 1);
        if (st == SDC_STATUS_OK) {
            if (count < 0) return SDC_STATUS_INTERNAL_ERROR;
            *output_accepted_count = static_cast<size_t>(count);
            *output_rejection_index = static_cast<size_t>(count);
        }
        return st;
    } catch (...) {
        return SDC_STATUS_INTERNAL_ERROR;
    }
}

SDC_API int sd_quantize_symmetric_int8_f64(const double* values, size_t count, int8_t* output_values,
                                           double* output_scale) {
    return sdc_quantize_symmetric_int8_f64(values, count, output_values, output_scale);
}

SDC_API int sd_dequantize_symmetric_int8_f64(const int8_t* values, size_t count, double scale,
                                             double* output_values) {
    return sdc_dequantize_symmetric_int8_f64(values, count, scale, output_values);
}

}  // extern "C"
