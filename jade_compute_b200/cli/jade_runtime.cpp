// jade-runtime: the reference's CLI (src/bin/jade-runtime.rs:41-314) on the B200
// backend. Subcommands keep their names and reports keep their keys:
//   info, verify, metal-verify, metal-gemm, metal-attention, mlp, emit, emit-suite
// The "metal-*" experiments run the CUDA kernels (the names are the reference's).
// Everything goes through the public C ABI of libjade_runtime.so, as an
// external caller would; the FP64 expectations are this tool's own restatement
// of the reference's workloads (src/runtime/workloads.rs, metal_lab.rs), used
// only to check results, never to produce them.
#include <sys/utsname.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <functional>
#include <map>
#include <memory>
#include <sstream>
#include <stdexcept>
#include <string>
#include <vector>

#include "../../include/jade_runtime.h"
#include "../csrc/json.hpp"

using jade::Json;

namespace {

[[noreturn]] void die(const std::string &m) { throw std::runtime_error(m); }
void check(int rc, const char *err) {
    if (rc) die("Jade runtime error " + std::to_string(rc) + ": " + err);
}

// ------------------------------------------------------------------ C ABI wrapper
struct Buf {
    void *ptr = nullptr;
    size_t bytes = 0;
    size_t elements() const { return bytes / 4; }
};

struct Exec {
    double host_ms, gpu_ms;
    uint64_t dispatches;
    uint32_t repeats;
    Json json() const {
        Json j = Json::object();
        j.set("host_ms", Json::f64(host_ms)).set("gpu_ms", gpu_ms > 0 ? Json::f64(gpu_ms) : Json::null());
        j.set("dispatches", Json::unsigned_(dispatches)).set("repeats", Json::unsigned_(repeats));
        return j;
    }
};

class Runtime {
  public:
    explicit Runtime(int device) {
        char err[1024];
        if (jr_version() != 1 || jr2_version() != 2) die("unsupported native runtime ABI");
        check(jr_create(device, &ctx_, err, sizeof err), err);
        char out[2048];
        check(jr_info(ctx_, out, sizeof out, err, sizeof err), err);
        info_ = out;
    }
    ~Runtime() {
        for (auto *k : kernels_) jr_kernel_release(k);
        for (auto &b : bufs_) jr_free(ctx_, b);
        jr_destroy(ctx_);
    }
    Json info() const {  // src/runtime/mod.rs:15-21
        Json j = Json::object();
        j.set("backend", Json::str("CUDA sm_100a built-in kernels"));
        j.set("device", Json::str(info_));
        j.set("execution", Json::str("ordered launches on one persistent non-blocking stream; optional CUDA-graph replay"));
        Json lim = Json::array();
        lim.push(Json::str("synchronous API at the public boundary"));
        lim.push(Json::str("FP32, TF32, BF16 and FP16 buffers"));
        j.set("limitations", lim);
        return j;
    }
    Buf alloc(size_t elements) {
        if (!elements) die("buffer allocation must be nonempty");
        char err[1024];
        Buf b;
        b.bytes = elements * 4;
        check(jr_alloc(ctx_, b.bytes, &b.ptr, err, sizeof err), err);
        bufs_.push_back(b.ptr);
        return b;
    }
    void upload(const Buf &b, const std::vector<float> &v) {
        if (v.size() != b.elements()) die("upload element count must match buffer exactly");
        char err[1024];
        check(jr_upload(ctx_, b.ptr, v.data(), b.bytes, err, sizeof err), err);
    }
    std::vector<float> download(const Buf &b) {
        std::vector<float> v(b.elements());
        char err[1024];
        check(jr_download(ctx_, b.ptr, v.data(), b.bytes, err, sizeof err), err);
        return v;
    }
    Buf resident(const std::vector<float> &v) {
        Buf b = alloc(v.size());
        upload(b, v);
        return b;
    }
    jr_kernel *compile(const Json &spec) {
        char err[2048];
        jr_kernel *k = nullptr;
        check(jr_compile(ctx_, jade::to_string_compact(spec).c_str(), &k, err, sizeof err), err);
        kernels_.push_back(k);
        return k;
    }
    Exec execute(const std::vector<std::pair<jr_kernel *, std::vector<Buf>>> &jobs, uint32_t repeats, bool graph = false) {
        if (jobs.empty() || !repeats) die("execution requires jobs and positive repeats");
        std::vector<std::vector<void *>> ptrs;
        std::vector<jr_dispatch> d;
        for (auto &j : jobs) {
            ptrs.emplace_back();
            for (auto &b : j.second) ptrs.back().push_back(b.ptr);
        }
        for (size_t i = 0; i < jobs.size(); ++i) d.push_back(jr_dispatch{jobs[i].first, ptrs[i].data(), ptrs[i].size()});
        char err[2048];
        double gpu = 0;
        const auto t0 = std::chrono::steady_clock::now();
        check(jr_execute2(ctx_, d.data(), d.size(), repeats, graph ? JR_EXEC_GRAPH : 0, &gpu, nullptr, err, sizeof err), err);
        const double host = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
        if (!std::isfinite(gpu) || gpu < 0) die("invalid GPU event time");
        return Exec{host, gpu, (uint64_t)jobs.size() * repeats, repeats};
    }
    bool execute_fails(const std::vector<std::pair<jr_kernel *, std::vector<Buf>>> &jobs, uint32_t repeats) {
        try {
            execute(jobs, repeats);
            return false;
        } catch (const std::exception &) {
            return true;
        }
    }

  private:
    void *ctx_ = nullptr;
    std::string info_;
    std::vector<jr_kernel *> kernels_;
    std::vector<void *> bufs_;
};

// ------------------------------------------------------------------ FP64 expectations
// workloads.rs:17-27
std::vector<float> values(size_t len, uint32_t seed, float scale) {
    std::vector<float> v(len);
    uint32_t s = seed;
    for (auto &x : v) {
        s ^= s << 13;
        s ^= s >> 17;
        s ^= s << 5;
        x = ((float)(s >> 8) / 16777216.0f * 2.0f - 1.0f) * scale;
    }
    return v;
}
std::vector<double> widen(const std::vector<float> &v) { return std::vector<double>(v.begin(), v.end()); }
// workloads.rs:28-32
std::vector<double> dot(size_t m, size_t n, size_t k, const std::vector<double> &a, const std::vector<double> &b) {
    std::vector<double> out(m * n);
    for (size_t i = 0; i < m * n; ++i) {
        double s = 0;
        for (size_t p = 0; p < k; ++p) s += a[i / n * k + p] * b[p * n + i % n];
        out[i] = s;
    }
    return out;
}
double sigmoid(double x) {  // workloads.rs:36-43
    if (x >= 0) return 1.0 / (1.0 + std::exp(-x));
    const double e = std::exp(x);
    return e / (1.0 + e);
}
// workloads.rs:44-55
std::vector<double> normalize(size_t rows, size_t cols, const std::vector<double> &x, const std::vector<double> &w, double eps) {
    std::vector<double> out(x.size());
    for (size_t r = 0; r < rows; ++r) {
        double sq = 0;
        for (size_t c = 0; c < cols; ++c) sq += x[r * cols + c] * x[r * cols + c];
        const double inv = 1.0 / std::sqrt(sq / (double)cols + eps);
        for (size_t c = 0; c < cols; ++c) out[r * cols + c] = x[r * cols + c] * inv * w[c];
    }
    return out;
}
// metal_lab.rs:18-31
std::vector<double> gemm_reference(size_t m, size_t n, size_t k, const std::vector<float> &a, const std::vector<float> &b) {
    std::vector<double> out(m * n, 0.0);
    for (size_t r = 0; r < m; ++r)
        for (size_t p = 0; p < k; ++p) {
            const double av = a[r * k + p];
            for (size_t c = 0; c < n; ++c) out[r * n + c] += av * (double)b[p * n + c];
        }
    return out;
}
// metal_lab.rs:33-73
std::vector<double> attention_reference(size_t h, size_t s, size_t d, bool causal, const std::vector<float> &q,
                                        const std::vector<float> &k, const std::vector<float> &v) {
    std::vector<double> out(h * s * d, 0.0);
    for (size_t hh = 0; hh < h; ++hh)
        for (size_t row = 0; row < s; ++row) {
            const size_t count = causal ? row + 1 : s;
            std::vector<double> sc(count);
            for (size_t col = 0; col < count; ++col) {
                double acc = 0;
                for (size_t e = 0; e < d; ++e) acc += (double)q[(hh * s + row) * d + e] * (double)k[(hh * s + col) * d + e];
                sc[col] = acc / std::sqrt((double)d);
            }
            double mx = -INFINITY;
            for (double x : sc) mx = std::fmax(mx, x);
            double den = 0;
            for (double &x : sc) {
                x = std::exp(x - mx);
                den += x;
            }
            for (size_t e = 0; e < d; ++e) {
                double acc = 0;
                for (size_t col = 0; col < count; ++col) acc += sc[col] / den * (double)v[(hh * s + col) * d + e];
                out[(hh * s + row) * d + e] = acc;
            }
        }
    return out;
}

// workloads.rs:224-243
Json compare(const std::vector<float> &actual, const std::vector<double> &expected, double atol, double rtol) {
    if (actual.size() != expected.size()) die("oracle length mismatch");
    double max_abs = 0, max_rel = 0;
    for (size_t i = 0; i < actual.size(); ++i) {
        const double a = actual[i], e = expected[i];
        if (!std::isfinite(a) || !std::isfinite(e)) die("nonfinite value at " + std::to_string(i));
        const double error = std::fabs(a - e);
        if (!(error <= atol + rtol * std::fabs(e))) {
            char m[256];
            snprintf(m, sizeof m, "mismatch at %zu: got %.9g, expected %.17g, error %.3g", i, a, e, error);
            die(m);
        }
        max_abs = std::max(max_abs, error);
        max_rel = std::max(max_rel, error / std::max(std::fabs(e), atol));
    }
    Json j = Json::object();
    j.set("elements", Json::unsigned_(actual.size())).set("max_abs_error", Json::f64(max_abs));
    j.set("max_relative_error", Json::f64(max_rel)).set("all_finite", Json::boolean(true));
    return j;
}

Json spec_json(const std::string &text) { return jade::parse_json(text); }

struct Case {
    std::string name;
    Json spec;
    std::vector<std::vector<float>> inputs;
    std::vector<double> expected;
};

Json relu_expr() {
    return spec_json(R"({"kind":"maximum","left":{"kind":"add","left":{"kind":"multiply","left":{"kind":"input","binding":0},)"
                     R"("right":{"kind":"constant","value":2.5}},"right":{"kind":"input","binding":1}},"right":{"kind":"constant","value":0.0}})");
}

// workloads.rs:56-215
std::vector<Case> cases() {
    std::vector<Case> all;
    for (size_t len : {1, 257, 1025}) {
        auto a = values(len, 0x1234, 2.0f), b = values(len, 0xabcd, 1.0f);
        std::vector<double> e(len);
        for (size_t i = 0; i < len; ++i) e[i] = -0.375 * a[i] + (double)b[i];
        all.push_back({"axpy_" + std::to_string(len), spec_json("{\"op\":\"axpy\",\"len\":" + std::to_string(len) + ",\"alpha\":-0.375}"), {a, b}, e});
    }
    {
        auto a = values(257, 0x1234, 2.0f), b = values(257, 0xabcd, 1.0f);
        std::vector<double> e(257);
        for (size_t i = 0; i < 257; ++i) e[i] = (double)a[i] + (double)b[i];
        all.push_back({"add_257", spec_json(R"({"op":"add","len":257})"), {a, b}, e});
    }
    {
        std::vector<float> gate = {-1000, -100, -20, -1, 0, 0.25, 1, 20, 100, 1000};
        auto up = values(gate.size(), 0xaacc, 2.0f);
        std::vector<double> e(gate.size());
        for (size_t i = 0; i < gate.size(); ++i) e[i] = (double)gate[i] * sigmoid(gate[i]) * (double)up[i];
        all.push_back({"swiglu_extreme", spec_json(R"({"op":"swi_glu","len":10})"), {gate, up}, e});
    }
    for (auto rc : std::vector<std::pair<size_t, size_t>>{{1, 1}, {3, 17}, {2, 257}}) {
        const size_t rows = rc.first, cols = rc.second;
        auto x = values(rows * cols, 0x1234, 2.0f), w = values(cols, 0xabcd, 1.0f);
        const float eps = 1e-5f;
        all.push_back({"rmsnorm_" + std::to_string(rows) + "_" + std::to_string(cols),
                       spec_json("{\"op\":\"rms_norm\",\"rows\":" + std::to_string(rows) + ",\"cols\":" + std::to_string(cols) + ",\"epsilon\":1e-5}"),
                       {x, w}, normalize(rows, cols, widen(x), widen(w), (double)eps)});
        std::vector<float> xs(rows * cols);
        for (size_t i = 0; i < xs.size(); ++i) xs[i] = i / cols == 0 ? 1000.0f : (float)(i % cols) * 0.25f - 10000.0f;
        std::vector<double> e(xs.size());
        for (size_t r = 0; r < rows; ++r) {
            float mx = -INFINITY;
            for (size_t c = 0; c < cols; ++c) mx = std::fmax(mx, xs[r * cols + c]);
            double sum = 0;
            for (size_t c = 0; c < cols; ++c) sum += std::exp((double)xs[r * cols + c] - mx);
            for (size_t c = 0; c < cols; ++c) e[r * cols + c] = std::exp((double)xs[r * cols + c] - mx) / sum;
        }
        all.push_back({"softmax_" + std::to_string(rows) + "_" + std::to_string(cols),
                       spec_json("{\"op\":\"softmax\",\"rows\":" + std::to_string(rows) + ",\"cols\":" + std::to_string(cols) + "}"), {xs}, e});
    }
    for (auto mnk : std::vector<std::array<size_t, 3>>{{1, 1, 1}, {31, 47, 19}, {8, 33, 65}})
        for (bool tiled : {false, true}) {
            const size_t m = mnk[0], n = mnk[1], k = mnk[2];
            auto a = values(m * k, 0x1234, 1.0f), b = values(k * n, 0xabcd, 1.0f);
            all.push_back({"gemm_" + std::to_string(m) + "_" + std::to_string(n) + "_" + std::to_string(k) + "_tiled_" + (tiled ? "true" : "false"),
                           spec_json("{\"op\":\"gemm\",\"m\":" + std::to_string(m) + ",\"n\":" + std::to_string(n) + ",\"k\":" + std::to_string(k) +
                                     ",\"tiled\":" + (tiled ? "true" : "false") + "}"),
                           {a, b}, dot(m, n, k, widen(a), widen(b))});
        }
    {
        auto a = values(257, 0x1234, 1.0f), b = values(257, 0xabcd, 1.0f);
        std::vector<double> e(257);
        for (size_t i = 0; i < 257; ++i) e[i] = std::fmax((double)a[i] * 2.5 + (double)b[i], 0.0);
        Json spec = spec_json(R"({"op":"elementwise","len":257,"inputs":2})");
        spec.set("expression", relu_expr());
        all.push_back({"custom_fused_axpy_relu", spec, {a, b}, e});
    }
    {
        auto x = values(73, 0x9988, 1.0f);
        std::vector<double> e(73);
        for (size_t i = 0; i < 73; ++i) e[i] = std::exp(-(double)x[i]);
        all.push_back({"custom_negate_exp",
                       spec_json(R"({"op":"elementwise","len":73,"inputs":1,"expression":{"kind":"exp","value":{"kind":"negate","value":{"kind":"input","binding":0}}}})"),
                       {x}, e});
    }
    return all;
}

double median(std::vector<double> v) {  // metal_lab.rs:75-83
    std::sort(v.begin(), v.end());
    const size_t n = v.size();
    return n % 2 == 0 ? (v[n / 2 - 1] + v[n / 2]) * 0.5 : v[n / 2];
}

Json samples_json(const std::vector<Exec> &s) {
    Json a = Json::array();
    for (auto &e : s) a.push(e.json());
    return a;
}
Json summary(const std::vector<Exec> &s) {  // metal_lab.rs:84-100
    std::vector<double> host, gpu;
    for (auto &e : s) {
        host.push_back(e.host_ms / e.repeats);
        gpu.push_back(e.gpu_ms / e.repeats);
    }
    Json j = Json::object();
    j.set("median_host_ms", Json::f64(median(host)));
    j.set("min_host_ms", Json::f64(*std::min_element(host.begin(), host.end())));
    j.set("max_host_ms", Json::f64(*std::max_element(host.begin(), host.end())));
    j.set("median_gpu_ms", Json::f64(median(gpu)));
    j.set("samples", samples_json(s));
    return j;
}
double med_host(const std::vector<Exec> &s) {
    std::vector<double> v;
    for (auto &e : s) v.push_back(e.host_ms / e.repeats);
    return median(v);
}
double med_gpu(const std::vector<Exec> &s) {
    std::vector<double> v;
    for (auto &e : s) v.push_back(e.gpu_ms / e.repeats);
    return median(v);
}

// ------------------------------------------------------------------ subcommands
// workloads.rs:245-320
Json verify(Runtime &rt) {
    Json checks = Json::array();
    for (auto &c : cases()) {
        jr_kernel *k = rt.compile(c.spec);
        std::vector<Buf> bufs;
        for (auto &in : c.inputs) bufs.push_back(rt.resident(in));
        Buf out = rt.alloc(c.expected.size());
        bufs.push_back(out);
        Exec t = rt.execute({{k, bufs}}, 2);
        Json chk;
        try {
            chk = compare(rt.download(out), c.expected, 3e-5, 3e-5);
        } catch (const std::exception &e) {
            die(c.name + ": " + e.what());
        }
        fprintf(stderr, "PASS native %s: %zu elements\n", c.name.c_str(), c.expected.size());
        Json j = Json::object();
        j.set("case", Json::str(c.name)).set("spec", c.spec).set("check", chk).set("execution", t.json());
        checks.push(j);
    }
    // Validation failures must be rejected before enqueueing any GPU work.
    jr_kernel *k = rt.compile(spec_json(R"({"op":"add","len":17})"));
    Buf a = rt.alloc(17), b = rt.alloc(17), wrong = rt.alloc(16);
    bool short_upload = false;
    try {
        rt.upload(a, std::vector<float>(16, 0.0f));
    } catch (const std::exception &) {
        short_upload = true;
    }
    if (!short_upload) die("short upload accepted");
    if (!rt.execute_fails({{k, {a, b, a}}}, 1)) die("aliased output accepted");
    if (!rt.execute_fails({{k, {a, b, wrong}}}, 1)) die("wrong output length accepted");
    if (!rt.execute_fails({}, 1)) die("empty job list accepted");
    if (!rt.execute_fails({{k, {a, b, wrong}}}, 0)) die("zero repeats accepted");
    Json r = Json::object();
    r.set("runtime", rt.info()).set("passed", Json::boolean(true)).set("checks", checks).set("rejected_invalid_calls", Json::integer(5));
    r.set("scope", Json::str("Native GPU execution against independent FP64 references; not full-model conformance"));
    return r;
}

// metal_lab.rs:114-230 on this backend: FP32 FFMA tiled GEMM, cuBLAS SGEMM, tcgen05 TF32
Json gemm(Runtime &rt, uint32_t m, uint32_t n, uint32_t k, uint32_t repeats, uint32_t samples) {
    if (repeats < 1 || repeats > 100) die("repeats must be 1..=100");
    if (samples < 3 || samples > 31) die("samples must be 3..=31");
    if ((uint64_t)m * n * k > 2147483648ull) die("GEMM experiment limited to 2^31 reference multiply-adds");
    if ((uint64_t)m * k + (uint64_t)k * n + 4ull * m * n > 32ull * 1024 * 1024) die("GEMM experiment limited to 128 MiB of GPU tensors");
    auto a = values((size_t)m * k, 0x1234, 1.0f), b = values((size_t)k * n, 0xabcd, 1.0f / std::sqrt((float)k));
    auto expected = gemm_reference(m, n, k, a, b);
    Buf ag = rt.resident(a), bg = rt.resident(b);
    const char *names[] = {"jade_ffma_fp32", "cublas_sgemm_fp32", "jade_tcgen05_tf32"};
    std::string dims = "\"m\":" + std::to_string(m) + ",\"n\":" + std::to_string(n) + ",\"k\":" + std::to_string(k);
    jr_kernel *ks[3] = {rt.compile(spec_json("{\"op\":\"gemm\"," + dims + ",\"tiled\":true}")),
                        rt.compile(spec_json("{\"op\":\"gemm_mps\"," + dims + "}")),
                        rt.compile(spec_json("{\"op\":\"gemm\"," + dims + ",\"tiled\":true,\"dtype\":\"tf32\"}"))};
    std::vector<Buf> outs;
    for (int i = 0; i < 3; ++i) outs.push_back(rt.alloc((size_t)m * n));
    // TF32 keeps 10 mantissa bits: its bound is validation.rs:73-78 with the
    // reduced-precision coefficient, expressed here as a relative tolerance.
    const double tol[3] = {5e-5, 5e-5, 2e-3};
    Json initial = Json::array(), final_ = Json::array();
    for (int i = 0; i < 3; ++i) {
        rt.execute({{ks[i], {ag, bg, outs[i]}}}, 3);
        initial.push(compare(rt.download(outs[i]), expected, tol[i], tol[i]));
    }
    std::vector<Exec> timings[3];
    Json order = Json::array();
    for (uint32_t r = 0; r < samples; ++r) {
        Json ro = Json::array();
        for (int off = 0; off < 3; ++off) {
            const int i = (r + off) % 3;
            timings[i].push_back(rt.execute({{ks[i], {ag, bg, outs[i]}}}, repeats));
            ro.push(Json::str(names[i]));
        }
        order.push(ro);
    }
    for (int i = 0; i < 3; ++i) final_.push(compare(rt.download(outs[i]), expected, tol[i], tol[i]));
    if (rt.download(ag) != a || rt.download(bg) != b) die("GEMM modified an input");
    Json variants = Json::array();
    for (int i = 0; i < 3; ++i) {
        Json v = Json::object();
        v.set("name", Json::str(names[i])).set("timing", summary(timings[i])).set("initial_check", initial.items[i]).set("final_check", final_.items[i]);
        const double tf = 2.0 * m * n * k / (med_gpu(timings[i]) * 1e-3) / 1e12;
        v.set("tflops_gpu", Json::f64(tf));
        variants.push(v);
    }
    Json shape = Json::object();
    shape.set("m", Json::unsigned_(m)).set("n", Json::unsigned_(n)).set("k", Json::unsigned_(k));
    Json r = Json::object();
    r.set("runtime", rt.info()).set("experiment", Json::str("native_fp32_gemm")).set("passed", Json::boolean(true)).set("shape", shape);
    r.set("variants", variants).set("ratio_ffma_to_cublas_gpu", Json::f64(med_gpu(timings[0]) / med_gpu(timings[1])));
    r.set("ratio_tf32_to_ffma_gpu", Json::f64(med_gpu(timings[2]) / med_gpu(timings[0])));
    r.set("sample_order", order).set("warmup_repeats_per_variant", Json::integer(3));
    r.set("validation", Json::str("All output elements against independent FP64 CPU reference before and after timing; input immutability checked"));
    return r;
}

// metal_lab.rs:232-396
Json attention(Runtime &rt, uint32_t heads, uint32_t seq, uint32_t dim, bool causal, uint32_t repeats, uint32_t samples, float amplitude,
               bool zeros) {
    if (repeats < 1 || repeats > 100) die("repeats must be 1..=100");
    if (samples < 3 || samples > 31) die("samples must be 3..=31");
    const size_t count = (size_t)heads * seq * dim, score_count = (size_t)heads * seq * seq;
    if (5 * count + 2 * score_count > 32ull * 1024 * 1024) die("attention experiment limited to 128 MiB of GPU tensors");
    if ((uint64_t)heads * seq * seq * dim > 536870912ull) die("attention experiment limited to 2^29 reference dot-product terms");
    auto q = zeros ? std::vector<float>(count, 0.0f) : values(count, 0x1111, amplitude);
    auto k = zeros ? std::vector<float>(count, 0.0f) : values(count, 0x2222, amplitude);
    auto v = values(count, 0x3333, 1.0f);
    auto expected = attention_reference(heads, seq, dim, causal, q, k, v);
    Buf qg = rt.resident(q), kg = rt.resident(k), vg = rt.resident(v);
    Buf scores = rt.alloc(score_count), probs = rt.alloc(score_count), out_m = rt.alloc(count), out_o = rt.alloc(count);
    const std::string hsd = "\"heads\":" + std::to_string(heads) + ",\"seq\":" + std::to_string(seq) + ",\"dim\":" + std::to_string(dim);
    const std::string c = causal ? "true" : "false";
    jr_kernel *ks = rt.compile(spec_json("{\"op\":\"attention_scores\"," + hsd + ",\"causal\":" + c + "}"));
    jr_kernel *sm = rt.compile(spec_json("{\"op\":\"softmax\",\"rows\":" + std::to_string(heads * seq) + ",\"cols\":" + std::to_string(seq) + "}"));
    jr_kernel *ap = rt.compile(spec_json("{\"op\":\"attention_apply\"," + hsd + "}"));
    jr_kernel *on = rt.compile(spec_json("{\"op\":\"attention_online\"," + hsd + ",\"causal\":" + c + "}"));
    std::vector<std::pair<jr_kernel *, std::vector<Buf>>> jobs[2] = {
        {{ks, {qg, kg, scores}}, {sm, {scores, probs}}, {ap, {probs, vg, out_m}}}, {{on, {qg, kg, vg, out_o}}}};
    const Buf outs[2] = {out_m, out_o};
    const char *names[2] = {"materialized_reference", "online_simt"};
    const double tol = amplitude > 1.0f ? 5e-4 : 5e-5;
    Json initial = Json::array(), final_ = Json::array(), order = Json::array();
    for (int i = 0; i < 2; ++i) {
        rt.execute(jobs[i], 3);
        initial.push(compare(rt.download(outs[i]), expected, tol, tol));
    }
    std::vector<Exec> t[2];
    for (uint32_t r = 0; r < samples; ++r) {
        const int idx[2] = {r % 2 == 0 ? 0 : 1, r % 2 == 0 ? 1 : 0};
        Json ro = Json::array();
        for (int i : idx) {
            t[i].push_back(rt.execute(jobs[i], repeats));
            ro.push(Json::str(names[i]));
        }
        order.push(ro);
    }
    for (int i = 0; i < 2; ++i) final_.push(compare(rt.download(outs[i]), expected, tol, tol));
    if (rt.download(qg) != q || rt.download(kg) != k || rt.download(vg) != v) die("attention modified an input");
    Json variants = Json::array();
    for (int i = 0; i < 2; ++i) {
        Json j = Json::object();
        j.set("name", Json::str(names[i])).set("timing", summary(t[i])).set("initial_check", initial.items[i]).set("final_check", final_.items[i]);
        variants.push(j);
    }
    Json shape = Json::object();
    shape.set("heads", Json::unsigned_(heads)).set("sequence", Json::unsigned_(seq)).set("head_dim", Json::unsigned_(dim)).set("causal", Json::boolean(causal));
    Json scratch = Json::object();
    scratch.set("materialized_reference", Json::unsigned_(2 * score_count * 4)).set("online_simt", Json::integer(0));
    Json r = Json::object();
    r.set("runtime", rt.info()).set("experiment", Json::str("native_fp32_self_attention")).set("passed", Json::boolean(true)).set("shape", shape);
    r.set("input_amplitude", Json::f64(amplitude)).set("zero_qk", Json::boolean(zeros)).set("variants", variants);
    r.set("ratio_materialized_to_online_host", Json::f64(med_host(t[0]) / med_host(t[1])));
    r.set("ratio_materialized_to_online_gpu", Json::f64(med_gpu(t[0]) / med_gpu(t[1])));
    r.set("sample_order", order).set("warmup_repeats_per_variant", Json::integer(3)).set("logical_global_scratch_bytes", scratch);
    Json tj = Json::object();
    tj.set("atol", Json::f64(tol)).set("rtol", Json::f64(tol));
    r.set("tolerance", tj);
    return r;
}

// metal_lab.rs:398-466
Json metal_verify(Runtime &rt) {
    Json g = Json::array(), a = Json::array(), p = Json::array();
    const uint32_t shapes[][3] = {{1, 1, 1}, {7, 9, 13}, {8, 8, 8}, {31, 47, 19}, {32, 32, 33}, {33, 31, 65},
                                  {65, 67, 63}, {1, 129, 33}, {64, 64, 64}, {127, 65, 129}, {256, 256, 65}, {257, 263, 67}};
    for (auto &s : shapes) {
        g.push(gemm(rt, s[0], s[1], s[2], 1, 3));
        fprintf(stderr, "PASS CUDA FP32 GEMM (%u,%u,%u) including cuBLAS and tcgen05 TF32\n", s[0], s[1], s[2]);
    }
    struct AC { uint32_t h, s, d; bool causal; float amp; bool zeros; };
    const AC configs[] = {{1, 1, 1, false, 1, false},   {1, 1, 128, true, 1, false},  {2, 7, 17, false, 1, false}, {2, 7, 17, true, 1, false},
                          {2, 33, 64, false, 1, false}, {2, 33, 64, true, 1, false},  {1, 65, 128, true, 1, false}, {3, 17, 33, false, 1, true},
                          {2, 17, 31, true, 1, true},   {2, 17, 64, false, 20, false}, {2, 17, 64, true, 20, false}};
    for (auto &c : configs) {
        a.push(attention(rt, c.h, c.s, c.d, c.causal, 1, 3, c.amp, c.zeros));
        fprintf(stderr, "PASS CUDA attention (%u,%u,%u), causal=%d, amplitude=%g, zero_qk=%d\n", c.h, c.s, c.d, c.causal, c.amp, c.zeros);
    }
    const float probes[][2] = {{1.0001f, 1.0003f}, {70000.25f, 1.0000312f}};
    for (auto &pr : probes) {
        Buf ag = rt.resident({pr[0]}), bg = rt.resident({pr[1]}), out = rt.alloc(1);
        for (const char *spec : {R"({"op":"gemm_simd","m":1,"n":1,"k":1})", R"({"op":"gemm_mps","m":1,"n":1,"k":1})"}) {
            jr_kernel *k = rt.compile(spec_json(spec));
            rt.execute({{k, {ag, bg, out}}}, 1);
            Json j = Json::object();
            j.set("spec", spec_json(spec)).set("a", Json::f32(pr[0])).set("b", Json::f32(pr[1]));
            j.set("check", compare(rt.download(out), {(double)pr[0] * (double)pr[1]}, 1e-5, 1e-6));
            p.push(j);
        }
    }
    Json r = Json::object();
    r.set("runtime", rt.info()).set("passed", Json::boolean(true)).set("gemm_shapes", g).set("attention_shapes", a).set("fp32_precision_probes", p);
    r.set("scope", Json::str("CUDA kernels and cuBLAS on B200, every output compared against independent FP64 references. Verification timings are diagnostic."));
    return r;
}

// workloads.rs:322-334
uint64_t mlp_elements(uint32_t batch, uint32_t width, uint32_t hidden) {
    const unsigned __int128 x = (unsigned __int128)batch * width * 4, w = (unsigned __int128)width * hidden * 3,
                            act = (unsigned __int128)batch * hidden * 3;
    const unsigned __int128 t = x + w + act + width;
    if (t > UINT64_MAX) die("MLP tensor size calculation overflow");
    return (uint64_t)t;
}

// workloads.rs:366-525 plus a CUDA-graph replay variant of the ordered batch
Json mlp(Runtime &rt, uint32_t batch, uint32_t width, uint32_t hidden, uint32_t repeats, uint32_t samples, const std::string &mode) {
    if (!(batch && width && hidden && repeats && repeats <= 1000 && samples >= 3 && samples <= 31)) die("invalid MLP dimensions/repeats/samples");
    if (mlp_elements(batch, width, hidden) > 32ull * 1024 * 1024) die("MLP experiment limited to 128 MiB of tensors");
    const size_t m = batch, w = width, h = hidden;
    auto x = values(m * w, 0x1234, 1.0f);
    std::vector<float> norm(w, 1.0f);
    auto wg = values(w * h, 0x3333, 1.0f / std::sqrt((float)w)), wu = values(w * h, 0x4444, 1.0f / std::sqrt((float)w));
    auto wd = values(h * w, 0x5555, 1.0f / std::sqrt((float)h));
    Buf xg = rt.resident(x), ng = rt.resident(norm), wgg = rt.resident(wg), wug = rt.resident(wu), wdg = rt.resident(wd);
    Buf normalized = rt.alloc(m * w), gate = rt.alloc(m * h), up = rt.alloc(m * h), act = rt.alloc(m * h), proj = rt.alloc(m * w), out = rt.alloc(m * w);
    auto gspec = [&](size_t mm, size_t nn, size_t kk) {
        const std::string d = "\"m\":" + std::to_string(mm) + ",\"n\":" + std::to_string(nn) + ",\"k\":" + std::to_string(kk);
        if (mode == "simd") return spec_json("{\"op\":\"gemm_simd\"," + d + "}");
        if (mode == "mps") return spec_json("{\"op\":\"gemm_mps\"," + d + "}");
        return spec_json("{\"op\":\"gemm\"," + d + ",\"tiled\":true}");
    };
    std::vector<Json> specs = {spec_json("{\"op\":\"rms_norm\",\"rows\":" + std::to_string(m) + ",\"cols\":" + std::to_string(w) + ",\"epsilon\":1e-5}"),
                               gspec(m, h, w), gspec(m, h, w), spec_json("{\"op\":\"swi_glu\",\"len\":" + std::to_string(m * h) + "}"),
                               gspec(m, w, h), spec_json("{\"op\":\"add\",\"len\":" + std::to_string(m * w) + "}")};
    std::vector<jr_kernel *> k;
    for (auto &s : specs) k.push_back(rt.compile(s));
    std::vector<std::pair<jr_kernel *, std::vector<Buf>>> jobs = {
        {k[0], {xg, ng, normalized}}, {k[1], {normalized, wgg, gate}}, {k[2], {normalized, wug, up}},
        {k[3], {gate, up, act}},      {k[4], {act, wdg, proj}},        {k[5], {proj, xg, out}}};
    const auto rn = normalize(m, w, widen(x), widen(norm), (double)1e-5f);
    const auto rg = dot(m, h, w, rn, widen(wg)), ru = dot(m, h, w, rn, widen(wu));
    std::vector<double> ra(rg.size());
    for (size_t i = 0; i < ra.size(); ++i) ra[i] = rg[i] * sigmoid(rg[i]) * ru[i];
    const auto rp = dot(m, w, h, ra, widen(wd));
    std::vector<double> expected(rp.size());
    for (size_t i = 0; i < rp.size(); ++i) expected[i] = rp[i] + (double)x[i];
    rt.execute(jobs, 3);
    Json initial = compare(rt.download(out), expected, 5e-5, 5e-5);
    std::vector<Exec> batched, separately, graphed;
    auto separate = [&]() {
        const auto t0 = std::chrono::steady_clock::now();
        double gpu = 0;
        for (uint32_t r = 0; r < repeats; ++r)
            for (auto &j : jobs) gpu += rt.execute({j}, 1).gpu_ms;
        return Exec{std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count(), gpu,
                    (uint64_t)repeats * jobs.size(), repeats};
    };
    for (uint32_t r = 0; r < samples; ++r) {  // rotating order, as workloads.rs:500-508 with a third variant
        for (int off = 0; off < 3; ++off) {
            switch ((r + off) % 3) {
                case 0: batched.push_back(rt.execute(jobs, repeats)); break;
                case 1: separately.push_back(separate()); break;
                default: graphed.push_back(rt.execute(jobs, repeats, true)); break;
            }
        }
    }
    Json final_ = compare(rt.download(out), expected, 5e-5, 5e-5);
    const double b = med_host(batched), s = med_host(separately), g = med_host(graphed);
    Json shape = Json::object();
    shape.set("batch", Json::unsigned_(batch)).set("width", Json::unsigned_(width)).set("hidden", Json::unsigned_(hidden));
    Json sp = Json::array();
    for (auto &x2 : specs) sp.push(x2);
    Json r = Json::object();
    r.set("runtime", rt.info()).set("workload", Json::str("synthetic residual MLP: RMSNorm -> gate/up GEMM -> SwiGLU -> down GEMM -> residual add"));
    r.set("trained_model", Json::boolean(false)).set("gemm_mode", Json::str(mode == "simd" ? "simd" : mode == "mps" ? "mps" : "register"));
    r.set("shape", shape).set("specs", sp).set("initial_check", initial).set("final_check", final_);
    r.set("batched_samples", samples_json(batched)).set("separate_submission_samples", samples_json(separately)).set("graph_samples", samples_json(graphed));
    r.set("median_batched_host_ms_per_block", Json::f64(b)).set("median_separate_host_ms_per_block", Json::f64(s));
    r.set("median_graph_host_ms_per_block", Json::f64(g)).set("ratio_separate_to_batched", Json::f64(s / b));
    r.set("ratio_batched_to_graph", Json::f64(b / g)).set("output_elements", Json::unsigned_(m * w));
    r.set("scope", Json::str("Same logical operations and resident tensors; one ordered batch versus synchronizing every dispatch versus "
                             "one CUDA-graph replay. Excludes compilation, allocation, upload and readback."));
    return r;
}

// ------------------------------------------------------------------ output
std::string read_file(const std::string &path, size_t limit) {
    std::ifstream f(path, std::ios::binary);
    if (!f) die("cannot read " + path);
    std::stringstream ss;
    ss << f.rdbuf();
    std::string s = ss.str();
    if (s.size() > limit) die("kernel JSON exceeds 64 KiB");
    return s;
}
void write_file(const std::string &path, const std::string &content) {  // jade-runtime.rs:135-141
    const auto slash = path.find_last_of('/');
    if (slash != std::string::npos && slash > 0) {
        const std::string dir = path.substr(0, slash);
        std::string cmd = "mkdir -p '" + dir + "'";
        if (system(cmd.c_str()) != 0) die("cannot create " + dir);
    }
    std::ofstream f(path, std::ios::binary);
    if (!f) die("cannot write " + path);
    f << content << "\n";
}
void emit_report(Json value, const std::string &path) {  // jade-runtime.rs:120-134
    utsname u{};
    uname(&u);
    value.set("schema_version", Json::integer(1));
    value.set("unix_time", Json::unsigned_((uint64_t)std::chrono::duration_cast<std::chrono::seconds>(
                                               std::chrono::system_clock::now().time_since_epoch()).count()));
    value.set("host_os", Json::str("linux")).set("host_arch", Json::str(u.machine));
    const std::string text = jade::to_string_pretty(value.sorted());
    if (!path.empty()) {
        write_file(path, text);
        fprintf(stderr, "Report: %s\n", path.c_str());
    }
    printf("%s\n", text.c_str());
}

std::string emit_text(const std::string &spec, const std::string &target) {
    char err[2048];
    size_t need = 0;
    std::string out(1 << 16, '\0');
    int rc = jr_spec_emit(spec.c_str(), target.c_str(), &out[0], out.size(), &need, err, sizeof err);
    if (rc && need > out.size()) {
        out.assign(need, '\0');
        rc = jr_spec_emit(spec.c_str(), target.c_str(), &out[0], out.size(), &need, err, sizeof err);
    }
    check(rc, err);
    return std::string(out.c_str());
}
Json spec_call(int (*fn)(const char *, char *, size_t, char *, size_t), const std::string &spec) {
    char err[2048];
    std::string out(1 << 16, '\0');
    check(fn(spec.c_str(), &out[0], out.size(), err, sizeof err), err);
    return jade::parse_json(out.c_str());
}

const char *kUsage =
    "jade-runtime [--backend cuda] [--device N] <command> [options]\n"
    "  info\n"
    "  verify [--report PATH]\n"
    "  metal-verify [--report PATH]\n"
    "  metal-gemm [--m 512 --n 512 --k 512 --repeats 10 --samples 9 --report PATH]\n"
    "  metal-attention [--heads 4 --sequence 256 --head-dim 64 --causal --repeats 10 --samples 9 --report PATH]\n"
    "  mlp [--simd-gemm|--mps-gemm] [--batch 8 --width 128 --hidden 256 --repeats 10 --samples 7 --report PATH]\n"
    "  emit --spec FILE.json --target corex|metal|cuda --output FILE\n"
    "  emit-suite --directory DIR\n";

}  // namespace

int main(int argc, char **argv) {
    try {
        std::vector<std::string> a(argv + 1, argv + argc);
        std::string backend = "cuda", command;
        int device = 0;
        std::map<std::string, std::string> opt;
        for (size_t i = 0; i < a.size(); ++i) {
            const std::string &x = a[i];
            if (x == "--help" || x == "-h") {
                printf("%s", kUsage);
                return 0;
            }
            if (x.rfind("--", 0) == 0) {
                const std::string key = x.substr(2);
                if (key == "causal" || key == "simd-gemm" || key == "mps-gemm") opt[key] = "1";
                else if (i + 1 < a.size()) opt[key] = a[++i];
                else die("missing value for " + x);
            } else if (command.empty()) command = x;
            else die("unexpected argument " + x);
        }
        if (opt.count("backend")) backend = opt["backend"];
        if (opt.count("device")) device = std::stoi(opt["device"]);
        auto num = [&](const char *k, uint32_t d) { return opt.count(k) ? (uint32_t)std::stoul(opt[k]) : d; };
        const std::string report = opt.count("report") ? opt["report"] : "";
        if (command.empty()) die(std::string("missing command\n") + kUsage);
        if (command == "emit") {
            const std::string spec = read_file(opt.at("spec"), 65536);
            write_file(opt.at("output"), emit_text(spec, opt.at("target")));
            printf("Generated %s (source only; no execution)\n", opt.at("output").c_str());
            return 0;
        }
        if (command == "emit-suite") {  // jade-runtime.rs:218-244
            const std::string dir = opt.at("directory");
            Json entries = Json::array();
            for (auto &c : cases()) {
                char err[2048];
                std::string canon(1 << 16, '\0');
                const std::string compact = jade::to_string_compact(c.spec);
                check(jr_spec_canonical(compact.c_str(), &canon[0], canon.size(), err, sizeof err), err);
                write_file(dir + "/" + c.name + ".json", canon.c_str());
                write_file(dir + "/" + c.name + ".metal", emit_text(compact, "metal"));
                write_file(dir + "/" + c.name + ".cu", emit_text(compact, "corex"));
                // this backend's sm_100a module of the case, beside the reference's CoreX text
                write_file(dir + "/" + c.name + ".sm100a.cu", emit_text(compact, "cuda"));
                // json! of the reference widens f32 fields to f64 (jade-runtime.rs:234)
                std::function<void(Json &)> widen_f32 = [&](Json &j) {
                    if (j.kind == Json::Number && j.text.find_first_of(".eE") != std::string::npos) j = Json::f64((double)(float)j.num);
                    for (auto &f : j.fields) widen_f32(f.second);
                    for (auto &x : j.items) widen_f32(x);
                };
                Json spec64 = jade::parse_json(canon.c_str());
                widen_f32(spec64);
                Json binds = Json::array();
                for (auto &b : spec_call(jr_spec_bindings, compact).items) {  // the reference's Binding has no dtype
                    Json nb = Json::object();
                    nb.set("name", *b.get("name")).set("elements", *b.get("elements")).set("write", *b.get("write"));
                    binds.push(nb);
                }
                Json e = Json::object();
                e.set("case", Json::str(c.name)).set("spec", spec64);
                e.set("launch", spec_call(jr_spec_launch, compact)).set("bindings", binds);
                entries.push(e);
            }
            Json m = Json::object();
            m.set("schema_version", Json::integer(1)).set("scope", Json::str("Generated source, not compilation or hardware validation")).set("cases", entries);
            write_file(dir + "/manifest.json", jade::to_string_pretty(m.sorted()));
            printf("Generated Metal + CoreX + CUDA sm_100a kernels in %s\n", dir.c_str());
            return 0;
        }
        if (backend == "metal") die("native Metal requires macOS");
        if (backend != "cuda" && backend != "corex") die("unknown backend " + backend);
        Runtime rt(device);
        if (command == "info") {
            Json j = Json::object();
            j.set("runtime", rt.info());
            emit_report(j, "");
        } else if (command == "verify") emit_report(verify(rt), report);
        else if (command == "metal-verify") emit_report(metal_verify(rt), report);
        else if (command == "metal-gemm") emit_report(gemm(rt, num("m", 512), num("n", 512), num("k", 512), num("repeats", 10), num("samples", 9)), report);
        else if (command == "metal-attention")
            emit_report(attention(rt, num("heads", 4), num("sequence", 256), num("head-dim", 64), opt.count("causal") > 0, num("repeats", 10),
                                  num("samples", 9), 1.0f, false),
                        report);
        else if (command == "mlp") {
            if (opt.count("simd-gemm") && opt.count("mps-gemm")) die("--simd-gemm conflicts with --mps-gemm");
            const std::string mode = opt.count("mps-gemm") ? "mps" : opt.count("simd-gemm") ? "simd" : "register";
            emit_report(mlp(rt, num("batch", 8), num("width", 128), num("hidden", 256), num("repeats", 10), num("samples", 7), mode), report);
        } else die("unknown command " + command + "\n" + kUsage);
        return 0;
    } catch (const std::exception &e) {
        fprintf(stderr, "Error: %s\n", e.what());
        return 1;
    }
}
