// Checked operation/expression IR (see ir.hpp for the reference mapping).
#include "ir.hpp"

#include <cmath>
#include <climits>
#include <cstring>
#include <sstream>

namespace jade {

namespace {

[[noreturn]] void bail(const std::string &m) { throw IrError(m); }
void ensure(bool c, const std::string &m) { if (!c) bail(m); }

const Json &field(const Json &j, const char *k) {
    const Json *v = j.get(k);
    if (!v) bail(std::string("missing field `") + k + "`");
    return *v;
}

bool is_integer_text(const Json &v) {
    if (v.kind != Json::Number) return false;
    for (char c : v.text) if (c == '.' || c == 'e' || c == 'E') return false;
    return true;
}

uint64_t get_uint(const Json &j, const char *k, uint64_t maxv) {
    const Json &v = field(j, k);
    if (!is_integer_text(v)) bail(std::string("invalid type for `") + k + "`: expected an unsigned integer");
    if (!v.text.empty() && v.text[0] == '-') bail(std::string("invalid value for `") + k + "`: expected an unsigned integer");
    errno = 0;
    unsigned long long x = strtoull(v.text.c_str(), nullptr, 10);
    if (errno || x > maxv) bail(std::string("invalid value for `") + k + "`: out of range");
    return x;
}
uint32_t get_u32(const Json &j, const char *k) { return (uint32_t)get_uint(j, k, UINT32_MAX); }

float get_f32(const Json &j, const char *k) {
    const Json &v = field(j, k);
    if (v.kind != Json::Number) bail(std::string("invalid type for `") + k + "`: expected f32");
    return (float)v.num;  // serde_json: parse as f64, then narrow
}
bool get_bool(const Json &j, const char *k) {
    const Json &v = field(j, k);
    if (v.kind != Json::Bool) bail(std::string("invalid type for `") + k + "`: expected a boolean");
    return v.b;
}
std::string get_str(const Json &j, const char *k) {
    const Json &v = field(j, k);
    if (v.kind != Json::String) bail(std::string("invalid type for `") + k + "`: expected a string");
    return v.text;
}

std::shared_ptr<Expr> parse_expr(const Json &j, int depth) {
    if (depth > 200) bail("expression nesting too deep");
    if (j.kind != Json::Object) bail("invalid type: expected expression object");
    auto e = std::make_shared<Expr>();
    const std::string kind = get_str(j, "kind");
    if (kind == "input") { e->kind = Expr::Input; e->binding = get_u32(j, "binding"); }
    else if (kind == "constant") { e->kind = Expr::Constant; e->value = get_f32(j, "value"); }
    else if (kind == "add" || kind == "multiply" || kind == "maximum") {
        e->kind = kind == "add" ? Expr::Add : kind == "multiply" ? Expr::Multiply : Expr::Maximum;
        e->left = parse_expr(field(j, "left"), depth + 1);
        e->right = parse_expr(field(j, "right"), depth + 1);
    } else if (kind == "negate" || kind == "exp") {
        e->kind = kind == "negate" ? Expr::Negate : Expr::Exp;
        e->left = parse_expr(field(j, "value"), depth + 1);
    } else bail("unknown variant `" + kind + "`, expected one of `input`, `constant`, `add`, `multiply`, `maximum`, `negate`, `exp`");
    return e;
}

Json expr_to_json(const Expr &e) {
    Json j = Json::object();
    switch (e.kind) {
        case Expr::Input: j.set("kind", Json::str("input")).set("binding", Json::unsigned_(e.binding)); break;
        case Expr::Constant: j.set("kind", Json::str("constant")).set("value", Json::f32(e.value)); break;
        case Expr::Add: case Expr::Multiply: case Expr::Maximum:
            j.set("kind", Json::str(e.kind == Expr::Add ? "add" : e.kind == Expr::Multiply ? "multiply" : "maximum"));
            j.set("left", expr_to_json(*e.left)).set("right", expr_to_json(*e.right));
            break;
        case Expr::Negate: case Expr::Exp:
            j.set("kind", Json::str(e.kind == Expr::Negate ? "negate" : "exp")).set("value", expr_to_json(*e.left));
            break;
    }
    return j;
}

// ir.rs:86-110
void validate_expr(const Expr &e, uint32_t inputs, size_t depth, size_t &nodes) {
    nodes += 1;
    ensure(depth <= 32 && nodes <= 512, "expression exceeds compiler complexity limit");
    switch (e.kind) {
        case Expr::Input: ensure(e.binding < inputs, "expression input binding out of range"); break;
        case Expr::Constant: ensure(std::isfinite(e.value), "expression constant must be finite"); break;
        case Expr::Add: case Expr::Multiply: case Expr::Maximum:
            validate_expr(*e.left, inputs, depth + 1, nodes);
            validate_expr(*e.right, inputs, depth + 1, nodes);
            break;
        case Expr::Negate: case Expr::Exp: validate_expr(*e.left, inputs, depth + 1, nodes); break;
    }
}

void dim(uint32_t v) { ensure(v > 0 && v <= (uint32_t)INT_MAX, "dimension must be in 1..=INT_MAX"); }
void matrix(uint64_t x, uint64_t y) {
    ensure(x > 0 && x <= (uint64_t)INT_MAX && y > 0 && y <= (uint64_t)INT_MAX, "dimension must be in 1..=INT_MAX");
    ensure(x * y <= (uint64_t)INT_MAX, "tensor exceeds checked 31-bit indexing");
}

bool is16(DType d) { return d == DType::BF16 || d == DType::F16; }

void check_dtype(const Spec &s, std::initializer_list<DType> allowed) {
    for (DType d : allowed) if (d == s.dtype) return;
    bail(std::string(spec_name(s)) + " does not support dtype " + dtype_name(s.dtype));
}

std::string u(uint64_t v) { return std::to_string(v) + "u"; }

}  // namespace

size_t dtype_size(DType d) {
    switch (d) {
        case DType::F32: case DType::TF32: return 4;
        case DType::BF16: case DType::F16: return 2;
        case DType::U8: return 1;
    }
    return 4;
}
const char *dtype_name(DType d) {
    switch (d) {
        case DType::F32: return "fp32";
        case DType::TF32: return "tf32";
        case DType::BF16: return "bf16";
        case DType::F16: return "fp16";
        case DType::U8: return "u8";
    }
    return "?";
}
DType parse_dtype(const std::string &s) {
    if (s == "fp32" || s == "f32") return DType::F32;
    if (s == "tf32") return DType::TF32;
    if (s == "bf16") return DType::BF16;
    if (s == "fp16" || s == "f16") return DType::F16;
    bail("unknown dtype `" + s + "`, expected one of `fp32`, `tf32`, `bf16`, `fp16`");
}

bool Spec::extended() const {
    return has_dtype || has_out_dtype || has_batch || has_b_layout || epilogue != "none" || row_scale || sm_limit ||
           op == Op::RmsInv || op == Op::AllReduce || op == Op::Copy || op == Op::L2Flush || op == Op::Fill || op == Op::WaitProbe ||
           op == Op::ShardReduce || op == Op::ShardGather || ranks;
}

const char *spec_name(const Spec &s) {
    switch (s.op) {  // ir.rs:176-192
        case Op::Elementwise: return "elementwise";
        case Op::Axpy: return "axpy";
        case Op::Add: return "add";
        case Op::Gemm: return s.tiled ? "gemm_register32" : "gemm_naive";
        case Op::GemmSimd: return "gemm_simdgroup_fp32";
        case Op::GemmMps: return "gemm_mps_fp32";
        case Op::AttentionScores: return "attention_scores";
        case Op::AttentionApply: return "attention_apply";
        case Op::AttentionOnline: return "attention_online";
        case Op::RmsNorm: return "rms_norm";
        case Op::SwiGlu: return "swi_glu";
        case Op::Softmax: return "softmax";
        case Op::RmsInv: return "rms_inv";
        case Op::AllReduce: return "all_reduce";
        case Op::Copy: return "copy";
        case Op::L2Flush: return "l2_flush";
        case Op::WaitProbe: return "wait_probe";
        case Op::ShardReduce: return "shard_reduce";
        case Op::ShardGather: return "shard_gather";
        case Op::Fill: return "fill";
    }
    return "?";
}

bool is_metal_specific(const Spec &s) {  // ir.rs:166-175
    return s.op == Op::GemmSimd || s.op == Op::GemmMps || s.op == Op::AttentionScores ||
           s.op == Op::AttentionApply || s.op == Op::AttentionOnline;
}

Spec parse_spec(const Json &j) {
    if (j.kind != Json::Object) bail("invalid type: expected a kernel spec object");
    Spec s;
    const std::string op = get_str(j, "op");
    if (op == "elementwise") {
        s.op = Op::Elementwise;
        s.len = get_u32(j, "len");
        s.inputs = get_u32(j, "inputs");
        s.expression = parse_expr(field(j, "expression"), 0);
    } else if (op == "axpy") { s.op = Op::Axpy; s.len = get_u32(j, "len"); s.alpha = get_f32(j, "alpha"); }
    else if (op == "add") { s.op = Op::Add; s.len = get_u32(j, "len"); }
    else if (op == "gemm") {
        s.op = Op::Gemm; s.m = get_u32(j, "m"); s.n = get_u32(j, "n"); s.k = get_u32(j, "k"); s.tiled = get_bool(j, "tiled");
    } else if (op == "gemm_simd" || op == "gemm_mps") {
        s.op = op == "gemm_simd" ? Op::GemmSimd : Op::GemmMps;
        s.m = get_u32(j, "m"); s.n = get_u32(j, "n"); s.k = get_u32(j, "k");
    } else if (op == "attention_scores" || op == "attention_online") {
        s.op = op == "attention_scores" ? Op::AttentionScores : Op::AttentionOnline;
        s.heads = get_u32(j, "heads"); s.seq = get_u32(j, "seq"); s.dim = get_u32(j, "dim"); s.causal = get_bool(j, "causal");
    } else if (op == "attention_apply") {
        s.op = Op::AttentionApply; s.heads = get_u32(j, "heads"); s.seq = get_u32(j, "seq"); s.dim = get_u32(j, "dim");
    } else if (op == "rms_norm" || op == "rms_inv") {
        s.op = op == "rms_norm" ? Op::RmsNorm : Op::RmsInv;
        s.rows = get_u32(j, "rows"); s.cols = get_u32(j, "cols"); s.epsilon = get_f32(j, "epsilon");
    } else if (op == "swi_glu") { s.op = Op::SwiGlu; s.len = get_u32(j, "len"); }
    else if (op == "softmax") { s.op = Op::Softmax; s.rows = get_u32(j, "rows"); s.cols = get_u32(j, "cols"); }
    else if (op == "all_reduce") { s.op = Op::AllReduce; s.len = get_u32(j, "len"); }
    else if (op == "copy") { s.op = Op::Copy; s.bytes = get_uint(j, "bytes", UINT64_MAX); s.direction = get_str(j, "direction"); }
    else if (op == "l2_flush") { s.op = Op::L2Flush; s.bytes = get_uint(j, "bytes", UINT64_MAX); }
    else if (op == "wait_probe") { s.op = Op::WaitProbe; s.limit_ns = get_uint(j, "limit_ns", UINT64_MAX); }
    else if (op == "shard_reduce" || op == "shard_gather") {
        s.op = op == "shard_reduce" ? Op::ShardReduce : Op::ShardGather;
        s.rows = get_u32(j, "rows"); s.cols = get_u32(j, "cols");
        if (j.has("residual")) s.residual = get_bool(j, "residual");
    }
    else if (op == "fill") {
        s.op = Op::Fill; s.len = get_u32(j, "len"); s.dist = get_str(j, "dist");
        s.seed = get_uint(j, "seed", UINT64_MAX);
        if (j.has("stream")) s.stream_id = get_u32(j, "stream");
        if (j.has("lo")) s.lo = get_f32(j, "lo");
        if (j.has("hi")) s.hi = get_f32(j, "hi");
        if (j.has("offset")) s.offset = get_uint(j, "offset", UINT64_MAX);
    } else {
        bail("unknown variant `" + op + "`, expected one of `elementwise`, `axpy`, `add`, `gemm`, `gemm_simd`, `gemm_mps`, "
             "`attention_scores`, `attention_apply`, `attention_online`, `rms_norm`, `swi_glu`, `softmax`, "
             "`rms_inv`, `all_reduce`, `copy`, `l2_flush`, `fill`, `wait_probe`, `shard_reduce`, `shard_gather`");
    }
    if (const Json *d = j.get("dtype")) {
        if (d->kind != Json::String) bail("invalid type for `dtype`");
        s.dtype = parse_dtype(d->text);
        s.has_dtype = true;
    }
    s.out_dtype = s.dtype == DType::TF32 ? DType::F32 : s.dtype;
    if (s.op == Op::Gemm || s.op == Op::GemmSimd || s.op == Op::GemmMps) s.out_dtype = DType::F32;
    if (const Json *d = j.get("out_dtype")) {
        if (d->kind != Json::String) bail("invalid type for `out_dtype`");
        s.out_dtype = parse_dtype(d->text);
        s.has_out_dtype = true;
    }
    if (j.has("batch")) { s.batch = get_u32(j, "batch"); s.has_batch = true; }
    if (const Json *d = j.get("b_layout")) {
        if (d->kind != Json::String || (d->text != "kn" && d->text != "nk")) bail("`b_layout` must be \"kn\" or \"nk\"");
        s.b_nk = d->text == "nk";
        s.has_b_layout = true;
    }
    if (const Json *d = j.get("epilogue")) {
        if (d->kind != Json::String) bail("invalid type for `epilogue`");
        s.epilogue = d->text;
    }
    if (j.has("row_scale")) s.row_scale = get_bool(j, "row_scale");
    if (j.has("sm_limit")) s.sm_limit = get_u32(j, "sm_limit");
    if (j.has("ranks")) s.ranks = get_u32(j, "ranks");
    if (j.has("rank")) s.rank = get_u32(j, "rank");
    return s;
}

Spec parse_spec_text(const std::string &text) {
    Json j;
    try { j = parse_json(text); } catch (const std::exception &e) { bail(e.what()); }
    return parse_spec(j);
}

Json spec_to_json(const Spec &s) {
    Json j = Json::object();
    auto U = [](uint64_t v) { return Json::unsigned_(v); };
    switch (s.op) {
        case Op::Elementwise:
            j.set("op", Json::str("elementwise")).set("len", U(s.len)).set("inputs", U(s.inputs)).set("expression", expr_to_json(*s.expression));
            break;
        case Op::Axpy: j.set("op", Json::str("axpy")).set("len", U(s.len)).set("alpha", Json::f32(s.alpha)); break;
        case Op::Add: j.set("op", Json::str("add")).set("len", U(s.len)); break;
        case Op::Gemm: j.set("op", Json::str("gemm")).set("m", U(s.m)).set("n", U(s.n)).set("k", U(s.k)).set("tiled", Json::boolean(s.tiled)); break;
        case Op::GemmSimd: case Op::GemmMps:
            j.set("op", Json::str(s.op == Op::GemmSimd ? "gemm_simd" : "gemm_mps")).set("m", U(s.m)).set("n", U(s.n)).set("k", U(s.k));
            break;
        case Op::AttentionScores: case Op::AttentionOnline:
            j.set("op", Json::str(s.op == Op::AttentionScores ? "attention_scores" : "attention_online"))
                .set("heads", U(s.heads)).set("seq", U(s.seq)).set("dim", U(s.dim)).set("causal", Json::boolean(s.causal));
            break;
        case Op::AttentionApply: j.set("op", Json::str("attention_apply")).set("heads", U(s.heads)).set("seq", U(s.seq)).set("dim", U(s.dim)); break;
        case Op::RmsNorm: case Op::RmsInv:
            j.set("op", Json::str(s.op == Op::RmsNorm ? "rms_norm" : "rms_inv")).set("rows", U(s.rows)).set("cols", U(s.cols)).set("epsilon", Json::f32(s.epsilon));
            break;
        case Op::SwiGlu: j.set("op", Json::str("swi_glu")).set("len", U(s.len)); break;
        case Op::Softmax: j.set("op", Json::str("softmax")).set("rows", U(s.rows)).set("cols", U(s.cols)); break;
        case Op::AllReduce: j.set("op", Json::str("all_reduce")).set("len", U(s.len)); break;
        case Op::Copy: j.set("op", Json::str("copy")).set("bytes", U(s.bytes)).set("direction", Json::str(s.direction)); break;
        case Op::L2Flush: j.set("op", Json::str("l2_flush")).set("bytes", U(s.bytes)); break;
        case Op::WaitProbe: j.set("op", Json::str("wait_probe")).set("limit_ns", U(s.limit_ns)); break;
        case Op::ShardReduce: case Op::ShardGather:
            j.set("op", Json::str(s.op == Op::ShardReduce ? "shard_reduce" : "shard_gather")).set("rows", U(s.rows)).set("cols", U(s.cols));
            if (s.residual) j.set("residual", Json::boolean(true));
            break;
        case Op::Fill:
            j.set("op", Json::str("fill")).set("len", U(s.len)).set("dist", Json::str(s.dist)).set("seed", U(s.seed))
                .set("stream", U(s.stream_id)).set("lo", Json::f32(s.lo)).set("hi", Json::f32(s.hi));
            if (s.offset) j.set("offset", U(s.offset));
            break;
    }
    if (s.has_dtype) j.set("dtype", Json::str(dtype_name(s.dtype)));
    if (s.has_out_dtype) j.set("out_dtype", Json::str(dtype_name(s.out_dtype)));
    if (s.has_batch) j.set("batch", U(s.batch));
    if (s.has_b_layout) j.set("b_layout", Json::str(s.b_nk ? "nk" : "kn"));
    if (s.epilogue != "none") j.set("epilogue", Json::str(s.epilogue));
    if (s.row_scale) j.set("row_scale", Json::boolean(true));
    if (s.sm_limit) j.set("sm_limit", U(s.sm_limit));
    if (s.ranks) j.set("ranks", U(s.ranks)).set("rank", U(s.rank));
    return j;
}

void validate(const Spec &s) {  // ir.rs:193-268 plus the extensions
    switch (s.op) {
        case Op::Elementwise: {
            dim(s.len);
            ensure(s.inputs > 0 && s.inputs <= 8, "elementwise input count must be 1..8");
            size_t nodes = 0;
            validate_expr(*s.expression, s.inputs, 0, nodes);
            check_dtype(s, {DType::F32});
            break;
        }
        case Op::Axpy:
            dim(s.len);
            ensure(std::isfinite(s.alpha), "alpha must be finite");
            check_dtype(s, {DType::F32});
            break;
        case Op::Add: dim(s.len); check_dtype(s, {DType::F32}); break;
        case Op::SwiGlu: dim(s.len); check_dtype(s, {DType::F32, DType::BF16}); break;
        case Op::Gemm: case Op::GemmSimd: case Op::GemmMps:
            matrix(s.m, s.k);
            matrix(s.k, s.n);
            matrix(s.m, s.n);
            if (s.op == Op::Gemm) check_dtype(s, {DType::F32, DType::TF32, DType::BF16, DType::F16});
            else check_dtype(s, {DType::F32});
            ensure(s.out_dtype == DType::F32 || (is16(s.dtype) && s.out_dtype == s.dtype),
                   "gemm out_dtype must be fp32 or the 16-bit input type");
            if (s.epilogue != "none" || s.row_scale || s.b_nk || s.sm_limit)
                ensure(s.dtype != DType::F32, "GEMM fusion, b_layout nk and sm_limit need a tensor-core dtype (tf32, bf16, fp16)");
            ensure(s.epilogue == "none" || s.epilogue == "swiglu" || s.epilogue == "residual" || s.epilogue == "scatter",
                   "epilogue must be none, swiglu, residual or scatter");
            ensure((s.epilogue == "scatter") == (s.ranks > 0), "the scatter epilogue and ranks go together");
            if (s.epilogue == "scatter") {
                ensure(is16(s.dtype) && s.out_dtype == s.dtype && s.b_nk && !s.row_scale,
                       "scatter epilogue needs 16-bit inputs and outputs of the same type and b_layout nk");
                ensure(s.ranks <= kMaxPeerRanks && s.rank < s.ranks, "ranks must be 1..8 and rank below it");
                ensure(s.m % (128 * s.ranks) == 0, "scatter epilogue needs m to be a multiple of 128 * ranks");
            }
            if (s.epilogue == "swiglu") {
                ensure(is16(s.dtype) && s.b_nk, "swiglu epilogue needs 16-bit inputs and b_layout nk");
                ensure(s.n % 128 == 0, "swiglu epilogue needs n to be a multiple of 128");
                matrix(2ull * s.n, s.k);
            }
            break;
        case Op::AttentionScores: case Op::AttentionApply: case Op::AttentionOnline:
            if (s.dtype == DType::F32) {
                ensure(s.heads >= 1 && s.heads <= 32, "attention heads must be 1..=32");
                ensure(s.seq >= 1 && s.seq <= 2048, "attention sequence must be 1..=2048");
                ensure(s.dim >= 1 && s.dim <= 128, "attention head dimension must be 1..=128");
                matrix((uint64_t)s.heads * s.seq, s.dim);
                matrix((uint64_t)s.heads * s.seq, s.seq);
                ensure(s.batch >= 1 && s.batch <= 65535, "attention batch must be 1..=65535");
                ensure((uint64_t)s.batch * s.heads * s.seq * s.dim <= (uint64_t)INT_MAX, "tensor exceeds checked 31-bit indexing");
                ensure(s.out_dtype == DType::F32, "fp32 attention writes fp32");
            } else {
                ensure(s.op == Op::AttentionOnline, "only attention_online has a 16-bit path");
                check_dtype(s, {DType::BF16, DType::F16});
                ensure(s.heads >= 1 && s.heads <= 1024, "attention heads must be 1..=1024");
                ensure(s.seq >= 1 && s.seq <= 131072, "attention sequence must be 1..=131072");
                ensure(s.dim == 64 || s.dim == 128, "16-bit attention head dimension must be 64 or 128");
                ensure(s.batch >= 1 && s.batch <= 65535, "attention batch must be 1..=65535");
                ensure((uint64_t)s.batch * s.heads * s.seq * s.dim <= (uint64_t)INT_MAX, "tensor exceeds checked 31-bit indexing");
                ensure(s.out_dtype == DType::F32 || s.out_dtype == s.dtype, "attention out_dtype must be fp32 or the input type");
            }
            break;
        case Op::RmsNorm: case Op::RmsInv:
            matrix(s.rows, s.cols);
            ensure(std::isfinite(s.epsilon) && s.epsilon > 0.0f, "epsilon must be finite and positive");
            check_dtype(s, {DType::F32, DType::BF16});
            break;
        case Op::Softmax: matrix(s.rows, s.cols); check_dtype(s, {DType::F32, DType::BF16}); break;
        case Op::AllReduce: dim(s.len); check_dtype(s, {DType::F32, DType::BF16, DType::F16}); break;
        case Op::Copy:
            ensure(s.bytes > 0, "copy must be nonempty");
            ensure(s.direction == "h2d" || s.direction == "d2h" || s.direction == "d2d", "copy direction must be h2d, d2h or d2d");
            break;
        case Op::L2Flush: ensure(s.bytes >= (1u << 20), "l2_flush needs at least 1 MiB"); break;
        case Op::WaitProbe:
            ensure(s.limit_ns >= 1000 && s.limit_ns <= 10000000000ull, "wait_probe limit_ns must be 1e3..1e10");
            break;
        case Op::ShardReduce: case Op::ShardGather:
            matrix(s.rows, s.cols);
            check_dtype(s, {DType::BF16});
            ensure(s.ranks >= 1 && s.ranks <= kMaxPeerRanks && s.rank < s.ranks, "ranks must be 1..8 and rank below it");
            ensure(s.rows % s.ranks == 0, "rows must split evenly over the ranks");
            ensure(s.cols % 8 == 0, "cols must be a multiple of 8 (16-byte rows)");
            ensure(s.op == Op::ShardReduce || !s.residual, "residual applies to shard_reduce");
            break;
        case Op::Fill:
            dim(s.len);
            ensure(s.dist == "uniform" || s.dist == "normal", "fill dist must be uniform or normal");
            ensure(std::isfinite(s.lo) && std::isfinite(s.hi), "fill parameters must be finite");
            check_dtype(s, {DType::F32, DType::BF16, DType::F16});
            break;
    }
    if (s.op != Op::Gemm) {
        ensure(!s.has_b_layout && s.epilogue == "none" && !s.row_scale, std::string(spec_name(s)) + " has no GEMM fusion fields");
        ensure(!s.ranks || s.op == Op::ShardReduce || s.op == Op::ShardGather,
               std::string(spec_name(s)) + " has no ranks (gemm scatter and the shard collectives only)");
    }
    if (s.has_batch) ensure(s.op == Op::AttentionOnline || s.op == Op::AttentionScores || s.op == Op::AttentionApply, "batch applies to attention only");
}

std::vector<Binding> bindings(const Spec &s) {  // ir.rs:269-339
    validate(s);
    auto b = [](const char *n, uint64_t e, bool w, DType d) { return Binding{n, e, w, d, false}; };
    const DType d = s.dtype == DType::TF32 ? DType::F32 : s.dtype;
    std::vector<Binding> r;
    switch (s.op) {
        case Op::Elementwise: {
            static const char *names[] = {"input0", "input1", "input2", "input3", "input4", "input5", "input6", "input7"};
            for (uint32_t i = 0; i < s.inputs; ++i) r.push_back(b(names[i], s.len, false, d));
            r.push_back(b("out", s.len, true, d));
            break;
        }
        case Op::Axpy: case Op::Add:
            r = {b("a", s.len, false, d), b("b", s.len, false, d), b("out", s.len, true, d)};
            break;
        case Op::SwiGlu: r = {b("gate", s.len, false, d), b("up", s.len, false, d), b("out", s.len, true, d)}; break;
        case Op::Gemm: case Op::GemmSimd: case Op::GemmMps: {
            const uint64_t bn = s.epilogue == "swiglu" ? 2ull * s.n : s.n;
            r.push_back(b("a", (uint64_t)s.m * s.k, false, d));
            r.push_back(b("b", (uint64_t)s.k * bn, false, d));
            if (s.row_scale) r.push_back(b("row_scale", s.m, false, DType::F32));
            if (s.epilogue == "residual") r.push_back(b("residual", (uint64_t)s.m * s.n, false, s.out_dtype));
            r.push_back(b("out", (uint64_t)s.m * s.n, true, s.out_dtype));
            if (s.epilogue == "scatter") r.push_back(b("flags", kPeerFlagBytes, true, DType::U8));
            break;
        }
        case Op::AttentionScores: {
            const uint64_t bh = (uint64_t)s.batch * s.heads;
            r = {b("q", bh * s.seq * s.dim, false, d), b("k", bh * s.seq * s.dim, false, d), b("scores", bh * s.seq * s.seq, true, d)};
            break;
        }
        case Op::AttentionApply: {
            const uint64_t bh = (uint64_t)s.batch * s.heads;
            r = {b("probabilities", bh * s.seq * s.seq, false, d), b("v", bh * s.seq * s.dim, false, d), b("out", bh * s.seq * s.dim, true, d)};
            break;
        }
        case Op::AttentionOnline: {
            const uint64_t n = (uint64_t)s.batch * s.heads * s.seq * s.dim;
            r = {b("q", n, false, d), b("k", n, false, d), b("v", n, false, d), b("out", n, true, s.out_dtype)};
            break;
        }
        case Op::RmsNorm:
            r = {b("x", (uint64_t)s.rows * s.cols, false, d), b("weight", s.cols, false, d), b("out", (uint64_t)s.rows * s.cols, true, d)};
            break;
        case Op::RmsInv: r = {b("x", (uint64_t)s.rows * s.cols, false, d), b("out", s.rows, true, DType::F32)}; break;
        case Op::Softmax: r = {b("x", (uint64_t)s.rows * s.cols, false, d), b("out", (uint64_t)s.rows * s.cols, true, d)}; break;
        case Op::AllReduce: r = {b("data", s.len, true, d)}; break;
        case Op::Copy: {
            Binding src = b("src", s.bytes, false, DType::U8), dst = b("dst", s.bytes, true, DType::U8);
            src.host = s.direction == "h2d";
            dst.host = s.direction == "d2h";
            r = {src, dst};
            break;
        }
        case Op::L2Flush: r = {b("scratch", s.bytes, true, DType::U8)}; break;
        case Op::WaitProbe: r = {b("elapsed_ns", 2, true, DType::F32)}; break;
        case Op::ShardReduce: {
            const uint64_t n = (uint64_t)s.rows * s.cols;
            r = {b("partials", n, false, d)};
            if (s.residual) r.push_back(b("residual", n, false, d));
            r.push_back(b("out", n, true, d));
            r.push_back(b("flags", kPeerFlagBytes, true, DType::U8));
            break;
        }
        case Op::ShardGather:
            r = {b("out", (uint64_t)s.rows * s.cols, true, d), b("flags", kPeerFlagBytes, true, DType::U8)};
            break;
        case Op::Fill: r = {b("out", s.len, true, d)}; break;
    }
    return r;
}

void validate_bindings(const Spec &s, const std::vector<uint64_t> &lengths, const std::vector<uint64_t> &ids) {
    const auto expected = bindings(s);  // ir.rs:340-367
    ensure(lengths.size() == expected.size() && ids.size() == expected.size(),
           std::string(spec_name(s)) + " expects " + std::to_string(expected.size()) + " bindings");
    for (size_t i = 0; i < expected.size(); ++i) {
        ensure(lengths[i] == expected[i].elements,
               std::string(spec_name(s)) + " binding " + expected[i].name + " expected " + std::to_string(expected[i].elements) +
                   " floats, got " + std::to_string(lengths[i]));
        if (expected[i].write)
            for (size_t j = 0; j < ids.size(); ++j)
                ensure(i == j || ids[i] != ids[j], "output binding must not alias another binding");
    }
}

Launch launch(const Spec &s) {  // ir.rs:368-420 (reference geometry of the emitted kernels)
    validate(s);
    ensure(!s.extended(), std::string(spec_name(s)) + " with backend extensions owns its launch geometry");
    auto cdiv = [](uint32_t a, uint32_t b) { return (a + b - 1) / b; };
    switch (s.op) {
        case Op::GemmMps: bail("MPS library operations own their launch geometry");
        case Op::GemmSimd: return Launch{{cdiv(s.n, 32), cdiv(s.m, 32), 1}, {128, 1, 1}};   // metal_simd.rs:24-26
        case Op::AttentionOnline: return Launch{{s.seq, s.heads, 1}, {32, 1, 1}};           // metal_attention.rs:46-49
        case Op::AttentionScores: return Launch{{cdiv(s.seq, 8), cdiv(s.seq, 8), s.heads}, {8, 8, 1}};
        case Op::AttentionApply: return Launch{{cdiv(s.dim, 8), cdiv(s.seq, 8), s.heads}, {8, 8, 1}};
        case Op::Elementwise: case Op::Axpy: case Op::Add: case Op::SwiGlu:
            return Launch{{cdiv(s.len, 256), 1, 1}, {256, 1, 1}};
        case Op::RmsNorm: case Op::Softmax: return Launch{{s.rows, 1, 1}, {256, 1, 1}};
        case Op::Gemm: {
            const uint32_t tile = s.tiled ? 32 : 8;
            return Launch{{cdiv(s.n, tile), cdiv(s.m, tile), 1}, {8, 8, 1}};
        }
        default: bail("backend-owned launch geometry");
    }
}

namespace {

// The two text dialects of ir.rs:461-464: CoreX (CUDA C++) and Metal Shading Language.
struct Dialect {
    bool metal;
    const char *header, *signature, *prefix, *shared, *barrier, *exponential, *rsqrt_fn, *maximum, *fused;
};
const Dialect kCorex{false, "#include <cuda_runtime.h>\n#include <math.h>\n", "__global__ void jade_main",
                     "    const uint3 gid = make_uint3(blockIdx.x*blockDim.x+threadIdx.x, blockIdx.y*blockDim.y+threadIdx.y, 0);\n"
                     "    const uint3 tid = threadIdx;\n"
                     "    const uint3 group = blockIdx;\n",
                     "__shared__", "__syncthreads();", "expf", "rsqrtf", "fmaxf", "fmaf"};
const Dialect kMetal{true, "#include <metal_stdlib>\nusing namespace metal;\n", "kernel void jade_main", "", "threadgroup",
                     "threadgroup_barrier(mem_flags::mem_threadgroup);", "exp", "rsqrt", "fmax", "fma"};

// ir.rs:111-137
std::string expr_code(const Expr &e, const Dialect &d) {
    switch (e.kind) {
        case Expr::Input: return "input" + std::to_string(e.binding) + "[i]";
        case Expr::Constant: return rust_lower_exp_f32(e.value) + "f";
        case Expr::Add: return "(" + expr_code(*e.left, d) + "+" + expr_code(*e.right, d) + ")";
        case Expr::Multiply: return "(" + expr_code(*e.left, d) + "*" + expr_code(*e.right, d) + ")";
        case Expr::Maximum: return std::string(d.maximum) + "(" + expr_code(*e.left, d) + "," + expr_code(*e.right, d) + ")";
        case Expr::Negate: return "(-" + expr_code(*e.left, d) + ")";
        case Expr::Exp: return std::string(d.exponential) + "(" + expr_code(*e.left, d) + ")";
    }
    return "";
}

// ir.rs:458-575
std::string source(const Spec &s, const Dialect &d) {
    validate(s);
    ensure(!s.extended(), std::string(spec_name(s)) + " uses backend extensions; the emitted dialects cover reference FP32 operations only");
    const auto bs = bindings(s);
    std::string args;
    for (size_t i = 0; i < bs.size(); ++i) {
        if (i) args += ", ";
        const std::string q = bs[i].write ? "" : "const ";
        if (d.metal) args += "device " + q + "float* " + bs[i].name + " [[buffer(" + std::to_string(i) + ")]]";
        else args += q + "float* " + bs[i].name;
    }
    if (d.metal)
        args += ", uint3 gid [[thread_position_in_grid]], uint3 tid [[thread_position_in_threadgroup]], uint3 group [[threadgroup_position_in_grid]]";
    const std::string sh = d.shared, bar = d.barrier, ex = d.exponential, mx = d.maximum, fu = d.fused;
    std::string body;
    switch (s.op) {
        case Op::Elementwise:
            body = "    const unsigned i=gid.x;\n    if(i<" + u(s.len) + ") out[i]=" + expr_code(*s.expression, d) + ";\n";
            break;
        case Op::Axpy:
            body = "    const unsigned i=gid.x;\n    if(i<" + u(s.len) + ") out[i]=" + fu + "(" + rust_lower_exp_f32(s.alpha) + "f,a[i],b[i]);\n";
            break;
        case Op::Add: body = "    const unsigned i=gid.x;\n    if(i<" + u(s.len) + ") out[i]=a[i]+b[i];\n"; break;
        case Op::SwiGlu:
            body = "    const unsigned i=gid.x;\n    if(i<" + u(s.len) + ") {\n        const float v=gate[i];\n"
                   "        const float e=" + ex + "(-fabs(v));\n"
                   "        const float sigmoid=v>=0.0f?1.0f/(1.0f+e):e/(1.0f+e);\n"
                   "        out[i]=(v*sigmoid)*up[i];\n    }\n";
            break;
        case Op::RmsNorm: {
            const std::string c = std::to_string(s.cols);
            body = "    " + sh + " float partial[256];\n"
                   "    const unsigned row=group.x, lane=tid.x;\n"
                   "    float sum=0.0f;\n"
                   "    for(unsigned c=lane;c<" + c + "u;c+=256u) { float v=x[row*" + c + "u+c]; sum=" + fu + "(v,v,sum); }\n"
                   "    partial[lane]=sum;\n"
                   "    " + bar + "\n"
                   "    for(unsigned step=128u;step>0u;step/=2u) {\n"
                   "        if(lane<step) partial[lane]+=partial[lane+step];\n"
                   "        " + bar + "\n"
                   "    }\n"
                   "    const float inv=" + d.rsqrt_fn + "(partial[0]/" + c + ".0f+" + rust_lower_exp_f32(s.epsilon) + "f);\n"
                   "    for(unsigned c=lane;c<" + c + "u;c+=256u) out[row*" + c + "u+c]=x[row*" + c + "u+c]*inv*weight[c];\n";
            break;
        }
        case Op::Softmax: {
            const std::string c = std::to_string(s.cols);
            body = "    " + sh + " float partial[256];\n"
                   "    const unsigned row=group.x, lane=tid.x;\n"
                   "    float maxv=-INFINITY;\n"
                   "    for(unsigned c=lane;c<" + c + "u;c+=256u) maxv=" + mx + "(maxv,x[row*" + c + "u+c]);\n"
                   "    partial[lane]=maxv;\n"
                   "    " + bar + "\n"
                   "    for(unsigned step=128u;step>0u;step/=2u) {\n"
                   "        if(lane<step) partial[lane]=" + mx + "(partial[lane],partial[lane+step]);\n"
                   "        " + bar + "\n"
                   "    }\n"
                   "    maxv=partial[0];\n"
                   "    " + bar + "\n"
                   "    float sum=0.0f;\n"
                   "    for(unsigned c=lane;c<" + c + "u;c+=256u) sum+=" + ex + "(x[row*" + c + "u+c]-maxv);\n"
                   "    partial[lane]=sum;\n"
                   "    " + bar + "\n"
                   "    for(unsigned step=128u;step>0u;step/=2u) {\n"
                   "        if(lane<step) partial[lane]+=partial[lane+step];\n"
                   "        " + bar + "\n"
                   "    }\n"
                   "    const float denom=partial[0];\n"
                   "    for(unsigned c=lane;c<" + c + "u;c+=256u) out[row*" + c + "u+c]=" + ex + "(x[row*" + c + "u+c]-maxv)/denom;\n";
            break;
        }
        case Op::Gemm: {
            const std::string m = std::to_string(s.m), n = std::to_string(s.n), k = std::to_string(s.k);
            if (!s.tiled) {
                body = "    const unsigned row=gid.y,col=gid.x;\n"
                       "    if(row<" + m + "u && col<" + n + "u) {\n"
                       "        float sum=0.0f;\n"
                       "        for(unsigned p=0u;p<" + k + "u;++p) sum=" + fu + "(a[row*" + k + "u+p],b[p*" + n + "u+col],sum);\n"
                       "        out[row*" + n + "u+col]=sum;\n"
                       "    }\n";
            } else {
                body = "    " + sh + " float tile_a[512], tile_b[512];\n"
                       "    const unsigned linear_thread=tid.y*8u+tid.x;\n"
                       "    const unsigned tile_row=group.y*32u, tile_col=group.x*32u;\n"
                       "    const unsigned local_row=tid.y*4u, local_col=tid.x*4u;\n"
                       "    float acc[4][4]={};\n"
                       "    for(unsigned base=0u;base<" + k + "u;base+=16u) {\n"
                       "        for(unsigned load=0u;load<8u;++load) {\n"
                       "            const unsigned slot=linear_thread+load*64u;\n"
                       "            const unsigned ar=tile_row+slot/16u, ac=base+slot%16u;\n"
                       "            const unsigned br=base+slot/32u, bc=tile_col+slot%32u;\n"
                       "            tile_a[slot]=(ar<" + m + "u && ac<" + k + "u)?a[ar*" + k + "u+ac]:0.0f;\n"
                       "            tile_b[slot]=(br<" + k + "u && bc<" + n + "u)?b[br*" + n + "u+bc]:0.0f;\n"
                       "        }\n"
                       "        " + bar + "\n"
                       "        for(unsigned p=0u;p<16u;++p) {\n"
                       "            for(unsigned r=0u;r<4u;++r) {\n"
                       "                const float av=tile_a[(local_row+r)*16u+p];\n"
                       "                for(unsigned c=0u;c<4u;++c) acc[r][c]=" + fu + "(av,tile_b[p*32u+local_col+c],acc[r][c]);\n"
                       "            }\n"
                       "        }\n"
                       "        " + bar + "\n"
                       "    }\n"
                       "    for(unsigned r=0u;r<4u;++r) for(unsigned c=0u;c<4u;++c) {\n"
                       "        const unsigned row=tile_row+local_row+r, col=tile_col+local_col+c;\n"
                       "        if(row<" + m + "u && col<" + n + "u) out[row*" + n + "u+col]=acc[r][c];\n"
                       "    }\n";
            }
            break;
        }
        default: bail("Metal-specific operations use their own checked source emitters");
    }
    std::string src = std::string("// Generated by Jade checked operation IR: ") + spec_name(s) + "\n" + d.header + d.signature + "(" + args +
                      ") {\n" + d.prefix + body + "}\n";
    if (!d.metal) {
        const Launch l = launch(s);
        std::string casts;
        for (size_t i = 0; i < bs.size(); ++i) {
            if (i) casts += ",";
            casts += std::string("static_cast<") + (bs[i].write ? "" : "const ") + "float*>(buffers[" + std::to_string(i) + "])";
        }
        char head[256];
        snprintf(head, sizeof head, "    jade_main<<<dim3(%u,%u,%u),dim3(%u,%u,%u),0,static_cast<cudaStream_t>(stream)>>>(",
                 l.grid[0], l.grid[1], l.grid[2], l.block[0], l.block[1], l.block[2]);
        src += "extern \"C\" int jade_generated_launch(void* stream, void** buffers) {\n" + std::string(head) + casts +
               ");\n    return static_cast<int>(cudaGetLastError());\n}\n";
    }
    return src;
}

}  // namespace

std::string corex_source(const Spec &s) {  // ir.rs:450-457
    ensure(!is_metal_specific(s), std::string(spec_name(s)) + " is a Metal-only operation; CoreX lowering is not implemented");
    return source(s, kCorex);
}

std::string metal_source(const Spec &s) {  // ir.rs:421-449 for the operations whose MSL comes from source()
    ensure(!is_metal_specific(s), std::string(spec_name(s)) +
                                      " uses a Metal-specific source template (metal_simd.rs / metal_attention.rs), which this backend does not emit");
    return source(s, kMetal);
}

std::string expr_cuda_code(const Expr &e, const std::vector<std::string> &names) {
    // Every node is one correctly rounded FP32 operation in tree order; __fadd_rn
    // and __fmul_rn are never contracted into an FMA.
    switch (e.kind) {
        case Expr::Input: return names[e.binding];
        case Expr::Constant: {
            uint32_t bits;
            memcpy(&bits, &e.value, 4);
            char b[48];
            snprintf(b, sizeof b, "__uint_as_float(0x%08xu)", bits);
            return b;
        }
        case Expr::Add: return "__fadd_rn(" + expr_cuda_code(*e.left, names) + "," + expr_cuda_code(*e.right, names) + ")";
        case Expr::Multiply: return "__fmul_rn(" + expr_cuda_code(*e.left, names) + "," + expr_cuda_code(*e.right, names) + ")";
        case Expr::Maximum: return "fmaxf(" + expr_cuda_code(*e.left, names) + "," + expr_cuda_code(*e.right, names) + ")";
        case Expr::Negate: return "(-" + expr_cuda_code(*e.left, names) + ")";
        case Expr::Exp: return "expf(" + expr_cuda_code(*e.left, names) + ")";
    }
    return "";
}

std::string cuda_elementwise_source(const Spec &s) {
    validate(s);
    ensure(s.op == Op::Elementwise, "cuda_elementwise_source needs an elementwise spec");
    std::ostringstream o;
    const uint32_t ni = s.inputs;
    o << "// Jade elementwise IR lowered for sm_100a: 128-bit loads and stores, grid-stride, 4 vectors in flight.\n";
    o << "extern \"C\" __global__ void __launch_bounds__(256) jade_elementwise(";
    for (uint32_t i = 0; i < ni; ++i) o << "const float* __restrict__ input" << i << ", ";
    o << "float* __restrict__ out, unsigned long long n) {\n";
    o << "    const unsigned long long stride = (unsigned long long)gridDim.x * blockDim.x;\n";
    o << "    const unsigned long long nvec = n >> 2;\n";
    o << "    unsigned long long v = (unsigned long long)blockIdx.x * blockDim.x + threadIdx.x;\n";
    // main loop: 4 independent float4 per input per iteration
    o << "    for (; v + 3 * stride < nvec; v += 4 * stride) {\n";
    for (uint32_t i = 0; i < ni; ++i)
        for (int u = 0; u < 4; ++u)
            o << "        const float4 x" << i << "_" << u << " = __ldcs(reinterpret_cast<const float4*>(input" << i << ") + v + " << u << " * stride);\n";
    for (int u = 0; u < 4; ++u) {
        o << "        { float4 r;\n";
        for (const char *c : {"x", "y", "z", "w"}) {
            std::vector<std::string> names;
            for (uint32_t i = 0; i < ni; ++i) names.push_back("x" + std::to_string(i) + "_" + std::to_string(u) + "." + c);
            o << "          r." << c << " = " << expr_cuda_code(*s.expression, names) << ";\n";
        }
        o << "          __stcs(reinterpret_cast<float4*>(out) + v + " << u << " * stride, r); }\n";
    }
    o << "    }\n";
    o << "    for (; v < nvec; v += stride) {\n";
    for (uint32_t i = 0; i < ni; ++i)
        o << "        const float4 x" << i << " = __ldcs(reinterpret_cast<const float4*>(input" << i << ") + v);\n";
    o << "        float4 r;\n";
    for (const char *c : {"x", "y", "z", "w"}) {
        std::vector<std::string> names;
        for (uint32_t i = 0; i < ni; ++i) names.push_back("x" + std::to_string(i) + "." + c);
        o << "        r." << c << " = " << expr_cuda_code(*s.expression, names) << ";\n";
    }
    o << "        __stcs(reinterpret_cast<float4*>(out) + v, r);\n    }\n";
    o << "    const unsigned long long t = (unsigned long long)blockIdx.x * blockDim.x + threadIdx.x;\n";
    o << "    if (t < (n & 3ull)) {\n        const unsigned long long i = (nvec << 2) + t;\n";
    {
        std::vector<std::string> names;
        for (uint32_t i = 0; i < ni; ++i) names.push_back("input" + std::to_string(i) + "[i]");
        o << "        out[i] = " << expr_cuda_code(*s.expression, names) << ";\n";
    }
    o << "    }\n}\n";
    return o.str();
}

Json binding_to_json(const Binding &b) {
    Json j = Json::object();
    j.set("name", Json::str(b.name)).set("elements", Json::unsigned_(b.elements)).set("write", Json::boolean(b.write));
    j.set("dtype", Json::str(dtype_name(b.dtype)));
    if (b.host) j.set("host", Json::boolean(true));
    return j;
}
Json launch_to_json(const Launch &l) {
    Json j = Json::object();
    Json g = Json::array(), b = Json::array();
    for (int i = 0; i < 3; ++i) { g.push(Json::unsigned_(l.grid[i])); b.push(Json::unsigned_(l.block[i])); }
    j.set("grid", g).set("block", b);
    return j;
}

}  // namespace jade
