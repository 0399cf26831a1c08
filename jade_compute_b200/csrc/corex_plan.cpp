// Fixed-shape GEMM plan ABI (include/jade_corex.h), the drop-in for the
// reference's cuBLAS provider (native/jade_corex.h, loaded by src/corex.rs:55-84).
// A plan is a small object over this library's own C ABI: one jr context that
// owns the stream, events and the A, B, C buffers, and one compiled GEMM - the
// FP32 FFMA kernel (precision 0) or the tcgen05 FP16 x FP16 -> FP32 kernel
// (precision 1, inputs rounded to FP16 on upload). The exported functions keep
// the provider's symbols, validation order, result codes and message texts.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <climits>
#include <cmath>
#include <cstdio>
#include <memory>
#include <new>
#include <string>
#include <vector>

#include "cabi.hpp"
#include "jade_corex.h"
#include "jade_runtime.h"

namespace {

// Result codes of this ABI (jade_corex.h): they differ from jr_*'s numbering.
constexpr int kInvalid = 1, kRuntime = 2, kAllocation = 4;

[[noreturn]] void invalid(const char *message) { throw jade::Fault{kInvalid, message}; }

// Runs one jr_* call with a message buffer of its own; a failure is re-thrown in
// this ABI's numbering with the runtime's message.
template <class Call>
void via_runtime(Call &&call) {
    char message[512] = {0};
    const int rc = call(message, sizeof message);
    if (rc == JR_OK) return;
    throw jade::Fault{rc == JR_EINVAL ? kInvalid : rc == JR_ENOMEM ? kAllocation : kRuntime, message};
}

// Element count and byte size of an x-by-y matrix of `width`-byte values.
bool extent(uint64_t x, uint64_t y, size_t width, size_t &count, size_t &bytes) {
    return !__builtin_mul_overflow(x, y, &count) && !__builtin_mul_overflow(count, width, &bytes);
}

class Plan {
  public:
    Plan(uint32_t m, uint32_t n, uint32_t k, int device, uint32_t precision)
        : m_(m), n_(n), k_(k), device_(device), fp16_(precision == 1) {
        const size_t in = fp16_ ? sizeof(uint16_t) : sizeof(float);
        size_t host_a = 0, host_b = 0;  // the caller's FP32 arrays must be addressable too
        if (!extent(m, k, in, a_.count, a_.bytes) || !extent(k, n, in, b_.count, b_.bytes) ||
            !extent(m, n, sizeof(float), c_.count, c_.bytes) || !extent(m, k, sizeof(float), a_.count, host_a) ||
            !extent(k, n, sizeof(float), b_.count, host_b))
            invalid("matrix byte count overflows size_t");
    }

    ~Plan() {
        if (kernel_) jr_kernel_release(kernel_);
        if (!rt_) return;
        for (void *p : {a_.ptr, b_.ptr, c_.ptr})
            if (p) jr_free(rt_, p);
        jr_destroy(rt_);
    }

    // Device context, buffers and the compiled GEMM.
    void open() {
        const int visible = jr_device_count();
        if (device_ >= visible) jade::raise(kInvalid, "device %d outside detected count %d", device_, visible);
        via_runtime([&](char *e, size_t c) { return jr_create(device_, &rt_, e, c); });
        for (Matrix *mat : {&a_, &b_, &c_})
            via_runtime([&](char *e, size_t c) { return jr_alloc(rt_, mat->bytes, &mat->ptr, e, c); });
        const std::string spec = "{\"op\":\"gemm\",\"m\":" + std::to_string(m_) + ",\"n\":" + std::to_string(n_) +
                                 ",\"k\":" + std::to_string(k_) + ",\"tiled\":true" +
                                 (fp16_ ? ",\"dtype\":\"fp16\",\"out_dtype\":\"fp32\"}" : "}");
        via_runtime([&](char *e, size_t c) { return jr_compile(rt_, spec.c_str(), &kernel_, e, c); });
        if (fp16_) {
            try {
                half_a_.resize(a_.count);
                half_b_.resize(b_.count);
            } catch (const std::bad_alloc &) {
                throw jade::Fault{kAllocation, "FP16 staging allocation failed"};
            }
        }
    }

    bool accepts_inputs(size_t a_len, size_t b_len) const { return a_len == a_.count && b_len == b_.count; }
    bool accepts_output(size_t c_len) const { return c_len == c_.count; }

    void upload(const float *a, const float *b) {
        uploaded_ = computed_ = false;
        const void *src[2] = {a, b};
        if (fp16_) {  // round to nearest even, as the provider's fp16 conversion
            for (size_t i = 0; i < a_.count; ++i) half_a_[i] = __half_as_ushort(__float2half_rn(a[i]));
            for (size_t i = 0; i < b_.count; ++i) half_b_[i] = __half_as_ushort(__float2half_rn(b[i]));
            src[0] = half_a_.data();
            src[1] = half_b_.data();
        }
        via_runtime([&](char *e, size_t c) { return jr_upload(rt_, a_.ptr, src[0], a_.bytes, e, c); });
        via_runtime([&](char *e, size_t c) { return jr_upload(rt_, b_.ptr, src[1], b_.bytes, e, c); });
        uploaded_ = true;
    }

    double run(uint32_t iterations) {
        computed_ = false;
        if (!uploaded_) invalid("upload A/B before running");
        void *buffers[3] = {a_.ptr, b_.ptr, c_.ptr};
        const jr_dispatch job{kernel_, buffers, 3};
        double ms = 0;
        via_runtime([&](char *e, size_t c) { return jr_execute2(rt_, &job, 1, iterations, 0, &ms, nullptr, e, c); });
        if (!std::isfinite(ms) || ms < 0) throw jade::Fault{kRuntime, "invalid GPU event duration"};
        computed_ = true;
        return ms;
    }

    void download(float *out) {
        if (!computed_) invalid("run successfully before downloading C");
        via_runtime([&](char *e, size_t c) { return jr_download(rt_, c_.ptr, out, c_.bytes, e, c); });
    }

    // "device=.. name=.. memory_bytes=.. multiprocessors=.. runtime_api=..
    // driver_api=.. blas_api=0 precision=.. kernel=.."
    void describe(char *out, size_t out_cap) const {
        cudaError_t st = cudaSetDevice(device_);
        if (st != cudaSuccess) jade::raise(kRuntime, "cudaSetDevice: %s", cudaGetErrorString(st));
        cudaDeviceProp prop{};
        st = cudaGetDeviceProperties(&prop, device_);
        if (st != cudaSuccess) jade::raise(kRuntime, "cudaGetDeviceProperties: %s", cudaGetErrorString(st));
        int runtime = 0, driver = 0;
        if (cudaRuntimeGetVersion(&runtime) != cudaSuccess || cudaDriverGetVersion(&driver) != cudaSuccess)
            throw jade::Fault{kRuntime, "CUDA version query failed"};
        const int n = std::snprintf(out, out_cap,
                                    "device=%d name=%.255s memory_bytes=%llu multiprocessors=%d runtime_api=%d driver_api=%d "
                                    "blas_api=0 precision=%s kernel=%s",
                                    device_, prop.name, static_cast<unsigned long long>(prop.totalGlobalMem),
                                    prop.multiProcessorCount, runtime, driver, fp16_ ? "fp16_inputs_fp32_accum_output" : "fp32",
                                    kernel_impl().c_str());
        if (n < 0 || static_cast<size_t>(n) >= out_cap) {
            out[out_cap - 1] = '\0';
            invalid("device info output buffer too small");
        }
    }

  private:
    struct Matrix {
        size_t count = 0, bytes = 0;
        void *ptr = nullptr;
    };

    // The implementation name the runtime reports for the compiled GEMM.
    std::string kernel_impl() const {
        char info[2048];
        if (jr_kernel_info(kernel_, info, sizeof info, nullptr, 0) != JR_OK) return "unknown";
        const std::string text(info), key = "\"impl\":\"";
        const size_t at = text.find(key);
        if (at == std::string::npos) return "unknown";
        const size_t from = at + key.size();
        return text.substr(from, text.find('"', from) - from);
    }

    uint32_t m_, n_, k_;
    int device_;
    bool fp16_;
    Matrix a_, b_, c_;
    void *rt_ = nullptr;
    jr_kernel *kernel_ = nullptr;
    std::vector<uint16_t> half_a_, half_b_;
    bool uploaded_ = false, computed_ = false;
};

// c_entry with this ABI's allocation code for host allocation failures.
template <class Body>
int plan_entry(char *err, size_t cap, Body &&body) noexcept {
    return jade::c_entry(err, cap, [&] {
        try {
            body();
        } catch (const std::bad_alloc &) {
            throw jade::Fault{kAllocation, "context allocation failed"};
        }
    });
}

}  // namespace

extern "C" JC_API uint32_t jade_corex_abi_version(void) { return 1; }

extern "C" JC_API int jade_corex_create(uint32_t m, uint32_t n, uint32_t k, int device, uint32_t precision, void **out,
                                        char *err, size_t cap) {
    return plan_entry(err, cap, [&] {
        if (!out) invalid("null output handle");
        *out = nullptr;
        const bool dims_ok = m && n && k && m <= INT_MAX && n <= INT_MAX && k <= INT_MAX;
        if (!dims_ok || device < 0 || precision > 1) invalid("dimensions must be 1..INT_MAX; device >= 0; precision 0 or 1");
        auto plan = std::make_unique<Plan>(m, n, k, device, precision);
        plan->open();
        *out = plan.release();
    });
}

extern "C" JC_API int jade_corex_upload(void *handle, const float *a, size_t a_len, const float *b, size_t b_len,
                                        char *err, size_t cap) {
    return plan_entry(err, cap, [&] {
        auto *plan = static_cast<Plan *>(handle);
        if (!plan || !a || !b || !plan->accepts_inputs(a_len, b_len))
            invalid("upload requires non-null buffers and exact A/B element counts");
        plan->upload(a, b);
    });
}

extern "C" JC_API int jade_corex_run(void *handle, uint32_t iterations, double *elapsed_ms, char *err, size_t cap) {
    if (elapsed_ms) *elapsed_ms = 0;
    return plan_entry(err, cap, [&] {
        auto *plan = static_cast<Plan *>(handle);
        if (!plan || !iterations || !elapsed_ms) invalid("run requires context, iterations > 0 and elapsed output");
        *elapsed_ms = plan->run(iterations);
    });
}

extern "C" JC_API int jade_corex_download(void *handle, float *out, size_t out_len, char *err, size_t cap) {
    return plan_entry(err, cap, [&] {
        auto *plan = static_cast<Plan *>(handle);
        if (!plan || !out || !plan->accepts_output(out_len)) invalid("download requires exact C element count");
        plan->download(out);
    });
}

extern "C" JC_API int jade_corex_device_info(void *handle, char *out, size_t out_cap, char *err, size_t cap) {
    if (out && out_cap) out[0] = '\0';
    return plan_entry(err, cap, [&] {
        auto *plan = static_cast<Plan *>(handle);
        if (!plan || !out || !out_cap) invalid("device info requires context and output buffer");
        plan->describe(out, out_cap);
    });
}

extern "C" JC_API void jade_corex_destroy(void *handle) { delete static_cast<Plan *>(handle); }
