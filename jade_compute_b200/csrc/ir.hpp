// Checked operation/expression IR: the reference's KernelSpec and Expr
// (src/runtime/ir.rs:6-84) with the same JSON form (serde tag "op"/"kind",
// snake_case), the same validation limits and messages (ir.rs:85-110,193-268),
// bindings (ir.rs:269-339), binding validation (ir.rs:340-367), launch geometry
// (ir.rs:368-420) and the CoreX-dialect CUDA C++ emitter (ir.rs:458-575,
// reproduced byte for byte).
//
// Extensions (all optional, defaults keep the reference behaviour):
//   "dtype"      fp32 | tf32 | bf16 | fp16   compute/storage type of the op
//   "out_dtype"  output storage type (GEMM, attention)
//   "b_layout"   kn (reference row-major K x N, default) | nk (pre-transposed N x K)
//   "epilogue"   none | swiglu | residual   (GEMM epilogue fusion)
//   "row_scale"  bool, GEMM output rows scaled by a per-row FP32 vector
//   "batch"      attention batch (layout [batch, heads, seq, dim])
// and ops of this backend: rms_inv, all_reduce, copy, l2_flush, fill.
#pragma once
#include <cstdint>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include "json.hpp"

namespace jade {

struct IrError : std::runtime_error {
    using std::runtime_error::runtime_error;
};

enum class DType { F32, TF32, BF16, F16, U8 };
size_t dtype_size(DType d);
const char *dtype_name(DType d);
DType parse_dtype(const std::string &s);

struct Expr {
    enum Kind { Input, Constant, Add, Multiply, Maximum, Negate, Exp } kind = Input;
    uint32_t binding = 0;
    float value = 0;
    std::shared_ptr<Expr> left, right;  // unary ops use `left` as their value
};

enum class Op {
    Elementwise, Axpy, Add, Gemm, GemmSimd, GemmMps, AttentionScores, AttentionApply,
    AttentionOnline, RmsNorm, SwiGlu, Softmax,
    RmsInv, AllReduce, Copy, L2Flush, Fill, WaitProbe, ShardReduce, ShardGather
};

// Words of the per-rank flag buffer that the peer collectives share (arrivals
// per rank for two phases, two local epoch counters), as bytes.
constexpr uint32_t kPeerFlagBytes = 256;
constexpr uint32_t kMaxPeerRanks = 8;

struct Spec {
    Op op = Op::Add;
    uint32_t len = 0, inputs = 0;
    std::shared_ptr<Expr> expression;
    float alpha = 0;
    uint32_t m = 0, n = 0, k = 0;
    bool tiled = false;
    uint32_t heads = 0, seq = 0, dim = 0, batch = 1;
    bool causal = false;
    uint32_t rows = 0, cols = 0;
    float epsilon = 0;
    // extensions
    DType dtype = DType::F32;
    DType out_dtype = DType::F32;
    bool has_dtype = false, has_out_dtype = false, has_batch = false;
    bool b_nk = false, has_b_layout = false;
    std::string epilogue = "none";
    bool row_scale = false;
    uint64_t bytes = 0;
    std::string direction;  // copy: h2d | d2h | d2d
    std::string dist;       // fill: uniform | normal
    uint64_t seed = 0;
    uint32_t stream_id = 0;
    float lo = 0, hi = 1;
    uint64_t offset = 0;    // fill: generator index of element 0 (a slice of a larger fill)
    uint32_t sm_limit = 0;  // tcgen05 gemm: at most this many persistent CTAs (0 = one per SM)
    uint64_t limit_ns = 0;  // wait_probe: the bounded wait's time limit
    uint32_t ranks = 0, rank = 0;  // peer collectives and the gemm "scatter" epilogue
    bool residual = false;         // shard_reduce: add a residual to the reduced rows
    bool extended() const;
};

struct Binding {
    std::string name;
    uint64_t elements;
    bool write;
    DType dtype;
    bool host = false;  // copy endpoints that live in registered host memory
};

struct Launch {
    uint32_t grid[3];
    uint32_t block[3];
};

Spec parse_spec(const Json &j);
Spec parse_spec_text(const std::string &text);
Json spec_to_json(const Spec &s);  // serde derive order, f32 fields as f32
const char *spec_name(const Spec &s);
bool is_metal_specific(const Spec &s);
void validate(const Spec &s);
std::vector<Binding> bindings(const Spec &s);
// lengths are element counts per binding (the reference's contract); ids are
// buffer identities for the write-alias check.
void validate_bindings(const Spec &s, const std::vector<uint64_t> &lengths,
                       const std::vector<uint64_t> &ids);
Launch launch(const Spec &s);
std::string corex_source(const Spec &s);
// Metal Shading Language text of the same templates (ir.rs:421-449) for the
// reference operations emitted through source(); text only, never compiled here.
std::string metal_source(const Spec &s);
// sm_100a lowering of an elementwise expression: a vectorised grid-stride kernel
// named jade_elementwise(const float* input0.., float* out, unsigned long long n).
std::string cuda_elementwise_source(const Spec &s);
// Text of the "cuda" emit target (jr_spec_emit): an sm_100a translation unit for
// the spec with the ABI-1 launcher jade_generated_launch(stream, buffers).
std::string cuda_source(const Spec &s);
std::string expr_cuda_code(const Expr &e, const std::vector<std::string> &names);

Json binding_to_json(const Binding &b);
Json launch_to_json(const Launch &l);

}  // namespace jade
