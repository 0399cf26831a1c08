// Fixed-shape GEMM plan ABI (include/jade_corex.h): the reference's cuBLAS
// provider contract (native/jade_corex.cpp:110-266) implemented on this
// library's own kernels through its C ABI (jr_create / jr_compile /
// jr_execute2). Validation order, error codes and messages follow the
// reference; the GEMM is the FP32 FFMA kernel (precision 0) or the tcgen05
// FP16 x FP16 -> FP32 kernel (precision 1).
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <climits>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <limits>
#include <new>
#include <string>
#include <vector>

#include "jade_corex.h"
#include "jade_runtime.h"

namespace {

struct Plan {
    uint32_t m = 0, n = 0, k = 0, precision = 0;
    int device = 0;
    size_t a_len = 0, b_len = 0, c_len = 0;
    size_t a_bytes = 0, b_bytes = 0, c_bytes = 0;
    void *rt = nullptr;  // jr context (owns the stream, events and buffers)
    void *a = nullptr, *b = nullptr, *c = nullptr;
    jr_kernel *kernel = nullptr;
    std::vector<uint16_t> host_a, host_b;  // FP16 staging (precision 1)
    bool uploaded = false, computed = false;
};

void clear_error(char *err, size_t cap) {
    if (err && cap) err[0] = '\0';
}

int fail(int code, char *err, size_t cap, const char *format, ...) {
    if (err && cap) {
        va_list args;
        va_start(args, format);
        std::vsnprintf(err, cap, format, args);
        va_end(args);
        err[cap - 1] = '\0';
    }
    return code;
}

// jr_* codes (1 invalid, 2 CUDA, 3 out of memory, 4 device timeout) to this
// ABI's (1 invalid, 2 runtime, 4 allocation); the message is already in err.
int map_code(int rc) {
    switch (rc) {
        case 0: return 0;
        case JR_EINVAL: return 1;
        case JR_ENOMEM: return 4;
        default: return 2;
    }
}

bool matrix_size(uint32_t x, uint32_t y, size_t element_size, size_t &count, size_t &bytes) {
    const auto maximum = std::numeric_limits<size_t>::max();
    if (!x || !y || static_cast<size_t>(x) > maximum / y) return false;
    count = static_cast<size_t>(x) * y;
    if (count > maximum / element_size) return false;
    bytes = count * element_size;
    return true;
}

void cleanup(Plan *p) {
    if (!p) return;
    if (p->kernel) jr_kernel_release(p->kernel);
    if (p->rt) {
        if (p->a) jr_free(p->rt, p->a);
        if (p->b) jr_free(p->rt, p->b);
        if (p->c) jr_free(p->rt, p->c);
        jr_destroy(p->rt);
    }
    delete p;
}

std::string gemm_spec(const Plan &p) {
    std::string s = "{\"op\":\"gemm\",\"m\":" + std::to_string(p.m) + ",\"n\":" + std::to_string(p.n) +
                    ",\"k\":" + std::to_string(p.k) + ",\"tiled\":true";
    if (p.precision) s += ",\"dtype\":\"fp16\",\"out_dtype\":\"fp32\"";
    return s + "}";
}

}  // namespace

extern "C" JC_API uint32_t jade_corex_abi_version(void) { return 1; }

extern "C" JC_API int jade_corex_create(uint32_t m, uint32_t n, uint32_t k, int device, uint32_t precision, void **out,
                                        char *err, size_t cap) {
    clear_error(err, cap);
    if (!out) return fail(1, err, cap, "null output handle");
    *out = nullptr;
    if (!m || !n || !k || m > INT_MAX || n > INT_MAX || k > INT_MAX || device < 0 || precision > 1)
        return fail(1, err, cap, "dimensions must be 1..INT_MAX; device >= 0; precision 0 or 1");
    Plan *p = new (std::nothrow) Plan();
    if (!p) return fail(4, err, cap, "context allocation failed");
    p->m = m;
    p->n = n;
    p->k = k;
    p->device = device;
    p->precision = precision;
    const size_t input_size = precision ? sizeof(uint16_t) : sizeof(float);
    if (!matrix_size(m, k, input_size, p->a_len, p->a_bytes) || !matrix_size(k, n, input_size, p->b_len, p->b_bytes) ||
        !matrix_size(m, n, sizeof(float), p->c_len, p->c_bytes) ||
        p->a_len > std::numeric_limits<size_t>::max() / sizeof(float) ||
        p->b_len > std::numeric_limits<size_t>::max() / sizeof(float)) {
        delete p;
        return fail(1, err, cap, "matrix byte count overflows size_t");
    }
    const auto initialize = [&]() -> int {
        const int count = jr_device_count();
        if (count < 0) return fail(2, err, cap, "cudaGetDeviceCount failed");
        if (device >= count) return fail(1, err, cap, "device %d outside detected count %d", device, count);
        int rc = jr_create(device, &p->rt, err, cap);
        if (rc) return map_code(rc);
        if ((rc = jr_alloc(p->rt, p->a_bytes, &p->a, err, cap)) || (rc = jr_alloc(p->rt, p->b_bytes, &p->b, err, cap)) ||
            (rc = jr_alloc(p->rt, p->c_bytes, &p->c, err, cap)))
            return map_code(rc);
        if ((rc = jr_compile(p->rt, gemm_spec(*p).c_str(), &p->kernel, err, cap))) return map_code(rc);
        if (precision) {
            try {
                p->host_a.resize(p->a_len);
                p->host_b.resize(p->b_len);
            } catch (...) {
                return fail(4, err, cap, "FP16 staging allocation failed");
            }
        }
        return 0;
    };
    const int rc = initialize();
    if (rc) {
        cleanup(p);
        return rc;
    }
    *out = p;
    return 0;
}

extern "C" JC_API int jade_corex_upload(void *handle, const float *a, size_t a_len, const float *b, size_t b_len,
                                        char *err, size_t cap) {
    clear_error(err, cap);
    auto *p = static_cast<Plan *>(handle);
    if (!p || !a || !b || a_len != p->a_len || b_len != p->b_len)
        return fail(1, err, cap, "upload requires non-null buffers and exact A/B element counts");
    p->uploaded = false;
    p->computed = false;
    const void *src_a = a, *src_b = b;
    if (p->precision) {
        for (size_t i = 0; i < a_len; ++i) p->host_a[i] = __half_as_ushort(__float2half_rn(a[i]));
        for (size_t i = 0; i < b_len; ++i) p->host_b[i] = __half_as_ushort(__float2half_rn(b[i]));
        src_a = p->host_a.data();
        src_b = p->host_b.data();
    }
    int rc = jr_upload(p->rt, p->a, src_a, p->a_bytes, err, cap);
    if (!rc) rc = jr_upload(p->rt, p->b, src_b, p->b_bytes, err, cap);
    if (rc) return map_code(rc);
    p->uploaded = true;
    return 0;
}

extern "C" JC_API int jade_corex_run(void *handle, uint32_t iterations, double *elapsed_ms, char *err, size_t cap) {
    clear_error(err, cap);
    if (elapsed_ms) *elapsed_ms = 0;
    auto *p = static_cast<Plan *>(handle);
    if (!p || !iterations || !elapsed_ms) return fail(1, err, cap, "run requires context, iterations > 0 and elapsed output");
    p->computed = false;
    if (!p->uploaded) return fail(1, err, cap, "upload A/B before running");
    void *buffers[3] = {p->a, p->b, p->c};
    const jr_dispatch job{p->kernel, buffers, 3};
    double ms = 0;
    const int rc = jr_execute2(p->rt, &job, 1, iterations, 0, &ms, nullptr, err, cap);
    if (rc) return map_code(rc);
    if (!std::isfinite(ms) || ms < 0) return fail(2, err, cap, "invalid GPU event duration");
    *elapsed_ms = ms;
    p->computed = true;
    return 0;
}

extern "C" JC_API int jade_corex_download(void *handle, float *out, size_t out_len, char *err, size_t cap) {
    clear_error(err, cap);
    auto *p = static_cast<Plan *>(handle);
    if (!p || !out || out_len != p->c_len) return fail(1, err, cap, "download requires exact C element count");
    if (!p->computed) return fail(1, err, cap, "run successfully before downloading C");
    return map_code(jr_download(p->rt, p->c, out, p->c_bytes, err, cap));
}

extern "C" JC_API int jade_corex_device_info(void *handle, char *out, size_t out_cap, char *err, size_t cap) {
    clear_error(err, cap);
    if (out && out_cap) out[0] = '\0';
    auto *p = static_cast<Plan *>(handle);
    if (!p || !out || !out_cap) return fail(1, err, cap, "device info requires context and output buffer");
    auto status = cudaSetDevice(p->device);
    if (status != cudaSuccess) return fail(2, err, cap, "cudaSetDevice: %s", cudaGetErrorString(status));
    cudaDeviceProp prop{};
    status = cudaGetDeviceProperties(&prop, p->device);
    if (status != cudaSuccess) return fail(2, err, cap, "cudaGetDeviceProperties: %s", cudaGetErrorString(status));
    int runtime = 0, driver = 0;
    if (cudaRuntimeGetVersion(&runtime) != cudaSuccess || cudaDriverGetVersion(&driver) != cudaSuccess)
        return fail(2, err, cap, "CUDA version query failed");
    char kinfo[1024];
    std::string impl = "unknown";
    if (jr_kernel_info(p->kernel, kinfo, sizeof kinfo, nullptr, 0) == 0) {
        const std::string s(kinfo);
        const auto at = s.find("\"impl\":\"");
        if (at != std::string::npos) impl = s.substr(at + 8, s.find('"', at + 8) - (at + 8));
    }
    const int needed = std::snprintf(
        out, out_cap,
        "device=%d name=%.255s memory_bytes=%llu multiprocessors=%d runtime_api=%d driver_api=%d blas_api=0 precision=%s "
        "kernel=%s",
        p->device, prop.name, static_cast<unsigned long long>(prop.totalGlobalMem), prop.multiProcessorCount, runtime,
        driver, p->precision ? "fp16_inputs_fp32_accum_output" : "fp32", impl.c_str());
    if (needed < 0 || static_cast<size_t>(needed) >= out_cap) {
        out[out_cap - 1] = '\0';
        return fail(1, err, cap, "device info output buffer too small");
    }
    return 0;
}

extern "C" JC_API void jade_corex_destroy(void *handle) { cleanup(static_cast<Plan *>(handle)); }
