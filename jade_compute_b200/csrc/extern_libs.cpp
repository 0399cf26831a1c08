// Runtime-loaded pieces: NVRTC lowering of elementwise expressions to sm_100a
// cubins, the cuBLAS SGEMM comparator behind `gemm_mps`, and NCCL collectives.
// NVRTC, cuBLAS and NCCL are opened with dlopen at first use so the library
// loads (and its IR/ABI can be tested) on hosts without them or without a GPU.
#include <cuda.h>
#include <cuda_runtime.h>
#include <dlfcn.h>

#include <cstring>
#include <string>
#include <vector>

#include "internal.hpp"

namespace jade {
namespace {

void *open_first(std::initializer_list<const char *> names) {
    for (const char *n : names)
        if (void *h = dlopen(n, RTLD_NOW | RTLD_GLOBAL)) return h;
    return nullptr;
}

// ------------------------------------------------------------------ NVRTC
typedef int nvrtcResult_t;
struct Nvrtc {
    void *lib = nullptr;
    nvrtcResult_t (*create)(void **, const char *, const char *, int, const char *const *, const char *const *) = nullptr;
    nvrtcResult_t (*compile)(void *, int, const char *const *) = nullptr;
    nvrtcResult_t (*log_size)(void *, size_t *) = nullptr;
    nvrtcResult_t (*log)(void *, char *) = nullptr;
    nvrtcResult_t (*cubin_size)(void *, size_t *) = nullptr;
    nvrtcResult_t (*cubin)(void *, char *) = nullptr;
    nvrtcResult_t (*destroy)(void **) = nullptr;
};
Nvrtc &nvrtc() {
    static Nvrtc n;
    static bool tried = false;
    if (!tried) {
        tried = true;
        n.lib = open_first({"libnvrtc.so.12", "libnvrtc.so", "/usr/local/cuda/lib64/libnvrtc.so.12"});
        if (n.lib) {
            n.create = (decltype(n.create))dlsym(n.lib, "nvrtcCreateProgram");
            n.compile = (decltype(n.compile))dlsym(n.lib, "nvrtcCompileProgram");
            n.log_size = (decltype(n.log_size))dlsym(n.lib, "nvrtcGetProgramLogSize");
            n.log = (decltype(n.log))dlsym(n.lib, "nvrtcGetProgramLog");
            n.cubin_size = (decltype(n.cubin_size))dlsym(n.lib, "nvrtcGetCUBINSize");
            n.cubin = (decltype(n.cubin))dlsym(n.lib, "nvrtcGetCUBIN");
            n.destroy = (decltype(n.destroy))dlsym(n.lib, "nvrtcDestroyProgram");
        }
    }
    return n;
}

struct Driver {
    CUresult (*load)(CUmodule *, const void *) = nullptr;
    CUresult (*get)(CUfunction *, CUmodule, const char *) = nullptr;
    CUresult (*launch)(CUfunction, unsigned, unsigned, unsigned, unsigned, unsigned, unsigned, unsigned, CUstream, void **, void **) = nullptr;
    CUresult (*unload)(CUmodule) = nullptr;
};
Driver &driver() {
    static Driver d;
    static bool tried = false;
    if (!tried) {
        tried = true;
        d.load = (decltype(d.load))driver_entry("cuModuleLoadData");
        d.get = (decltype(d.get))driver_entry("cuModuleGetFunction");
        d.launch = (decltype(d.launch))driver_entry("cuLaunchKernel");
        d.unload = (decltype(d.unload))driver_entry("cuModuleUnload");
    }
    return d;
}

}  // namespace

LaunchFn make_elementwise_rtc(Context *ctx, const Spec &s, std::string &impl) {
    const std::string src = cuda_elementwise_source(s);
    CUfunction fn = nullptr;
    {
        std::lock_guard<std::mutex> lock(ctx->rtc_mutex);
        auto it = ctx->rtc_modules.find(src);
        if (it != ctx->rtc_modules.end()) {
            fn = static_cast<CUfunction>(it->second.second);
        } else {
            Nvrtc &n = nvrtc();
            if (!n.lib || !n.create || !n.compile || !n.cubin) throw IrError("NVRTC (libnvrtc.so.12) is not available; elementwise IR cannot be lowered");
            Driver &d = driver();
            if (!d.load || !d.get || !d.launch) throw IrError("CUDA driver entry points unavailable");
            void *prog = nullptr;
            if (n.create(&prog, src.c_str(), "jade_elementwise.cu", 0, nullptr, nullptr) != 0) throw IrError("nvrtcCreateProgram failed");
            // IEEE FP32 throughout: no FMA contraction, accurate expf, no flush-to-zero.
            const char *opts[] = {"--gpu-architecture=sm_100a", "--fmad=false", "--ftz=false", "--prec-div=true", "--prec-sqrt=true", "-std=c++17"};
            const int rc = n.compile(prog, 6, opts);
            if (rc != 0) {
                size_t ls = 0;
                n.log_size(prog, &ls);
                std::string log(ls, '\0');
                n.log(prog, &log[0]);
                n.destroy(&prog);
                throw IrError("NVRTC compile failed: " + log);
            }
            size_t cs = 0;
            n.cubin_size(prog, &cs);
            std::vector<char> cubin(cs);
            n.cubin(prog, cubin.data());
            n.destroy(&prog);
            CUmodule mod = nullptr;
            if (d.load(&mod, cubin.data()) != CUDA_SUCCESS) throw IrError("cuModuleLoadData failed for the elementwise cubin");
            if (d.get(&fn, mod, "jade_elementwise") != CUDA_SUCCESS) throw IrError("cuModuleGetFunction failed");
            ctx->rtc_modules[src] = {mod, fn};
        }
    }
    const uint32_t ninputs = s.inputs;
    const unsigned long long n = s.len;
    const uint64_t vec = (n + 3) / 4;
    uint64_t blocks = (vec + 255) / 256;
    const uint64_t cap = (uint64_t)ctx->sm_count * 8;
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    const unsigned grid = (unsigned)blocks;
    impl = "elementwise_nvrtc_sm100a_v4";
    Driver *d = &driver();
    return [=](cudaStream_t st, void **b) {
        void *args[10];
        void *ptrs[9];
        unsigned long long count = n;
        for (uint32_t i = 0; i <= ninputs; ++i) {
            ptrs[i] = b[i];
            args[i] = &ptrs[i];
        }
        args[ninputs + 1] = &count;
        const CUresult r = d->launch(fn, grid, 1, 1, 256, 1, 1, 0, (CUstream)st, args, nullptr);
        return r == CUDA_SUCCESS ? cudaGetLastError() : cudaErrorLaunchFailure;
    };
}

void rtc_destroy(Context *ctx) {
    Driver &d = driver();
    for (auto &m : ctx->rtc_modules)
        if (d.unload) d.unload(static_cast<CUmodule>(m.second.first));
    ctx->rtc_modules.clear();
}

// ------------------------------------------------------------------ cuBLAS
namespace {
struct Cublas {
    void *lib = nullptr;
    int (*create)(void **) = nullptr;
    int (*destroy)(void *) = nullptr;
    int (*set_stream)(void *, cudaStream_t) = nullptr;
    int (*sgemm)(void *, int, int, int, int, int, const float *, const float *, int, const float *, int, const float *, float *, int) = nullptr;
    int (*set_math)(void *, int) = nullptr;
};
Cublas &cublas() {
    static Cublas c;
    static bool tried = false;
    if (!tried) {
        tried = true;
        c.lib = open_first({"libcublas.so.12", "libcublas.so", "/usr/local/cuda/lib64/libcublas.so.12"});
        if (c.lib) {
            c.create = (decltype(c.create))dlsym(c.lib, "cublasCreate_v2");
            c.destroy = (decltype(c.destroy))dlsym(c.lib, "cublasDestroy_v2");
            c.set_stream = (decltype(c.set_stream))dlsym(c.lib, "cublasSetStream_v2");
            c.sgemm = (decltype(c.sgemm))dlsym(c.lib, "cublasSgemm_v2");
            c.set_math = (decltype(c.set_math))dlsym(c.lib, "cublasSetMathMode");
        }
    }
    return c;
}
}  // namespace

// The reference's MPS GEMM (src/runtime/metal.rs:345-441) is a vendor-library
// FP32 GEMM. Its analogue here is cuBLAS SGEMM in pedantic FP32 mode: row-major
// C = A.B computed as column-major C^T = B^T.A^T (native/jade_corex.cpp:86-108).
LaunchFn make_cublas_gemm(Context *ctx, const Spec &s, std::string &impl) {
    Cublas &c = cublas();
    if (!c.lib || !c.create || !c.sgemm) throw IrError("cuBLAS (libcublas.so.12) is not available for gemm_mps");
    if (!ctx->cublas) {
        if (c.create(&ctx->cublas) != 0) throw IrError("cublasCreate failed");
        if (c.set_math) c.set_math(ctx->cublas, 2 /* CUBLAS_PEDANTIC_MATH */);
    }
    const int M = (int)s.m, N = (int)s.n, K = (int)s.k;
    void *h = ctx->cublas;
    impl = "cublas_sgemm_pedantic";
    return [=, &c](cudaStream_t st, void **b) {
        const float one = 1.0f, zero = 0.0f;
        c.set_stream(h, st);
        const int r = c.sgemm(h, 0, 0, N, M, K, &one, (const float *)b[1], N, (const float *)b[0], K, &zero, (float *)b[2], N);
        return r == 0 ? cudaSuccess : cudaErrorUnknown;
    };
}

void cublas_destroy(Context *ctx) {
    if (ctx->cublas && cublas().destroy) cublas().destroy(ctx->cublas);
    ctx->cublas = nullptr;
}

}  // namespace jade
