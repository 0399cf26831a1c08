// Minimal JSON value, parser and writer for kernel specs and reports.
//
// Objects keep insertion order (specs serialise like serde's derive order,
// src/runtime/ir.rs:6-84); `sorted()` gives the key-sorted form serde_json's
// json! macro produces (reports, manifest). Number text is kept so f32 fields
// can be parsed exactly (strtof of the original digits).
#pragma once
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

namespace jade {

struct Json {
    enum Kind { Null, Bool, Number, String, Array, Object } kind = Null;
    bool b = false;
    double num = 0;
    std::string text;  // number text or string value
    std::vector<Json> items;
    std::vector<std::pair<std::string, Json>> fields;
    int float_width = 64;  // number formatting when serialised: 32 or 64 bits

    static Json null() { return Json(); }
    static Json boolean(bool v) { Json j; j.kind = Bool; j.b = v; return j; }
    static Json integer(long long v) { Json j; j.kind = Number; j.num = (double)v; j.text = std::to_string(v); return j; }
    static Json unsigned_(unsigned long long v) { Json j; j.kind = Number; j.num = (double)v; j.text = std::to_string(v); return j; }
    static Json f32(float v) { Json j; j.kind = Number; j.num = v; j.float_width = 32; j.text.clear(); return j; }
    static Json f64(double v) { Json j; j.kind = Number; j.num = v; j.float_width = 64; j.text.clear(); return j; }
    static Json str(std::string v) { Json j; j.kind = String; j.text = std::move(v); return j; }
    static Json array() { Json j; j.kind = Array; return j; }
    static Json object() { Json j; j.kind = Object; return j; }

    Json &set(const std::string &k, Json v) {
        for (auto &f : fields) if (f.first == k) { f.second = std::move(v); return *this; }
        fields.emplace_back(k, std::move(v));
        return *this;
    }
    Json &push(Json v) { items.push_back(std::move(v)); return *this; }
    const Json *get(const std::string &k) const {
        for (auto &f : fields) if (f.first == k) return &f.second;
        return nullptr;
    }
    bool has(const std::string &k) const { return get(k) != nullptr; }
    Json sorted() const;
};

Json parse_json(const std::string &s);  // throws std::runtime_error
std::string to_string_pretty(const Json &j);
std::string to_string_compact(const Json &j);

// Rust `{:e}` formatting of an f32 (shortest round-trip digits), e.g. 2.5 -> "2.5e0".
std::string rust_lower_exp_f32(float v);
// serde_json/ryu formatting of a finite float (f32 or f64 shortest digits).
std::string ryu_like(double v, int width);

}  // namespace jade
