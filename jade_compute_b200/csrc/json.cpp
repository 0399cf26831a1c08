#include "json.hpp"

#include <algorithm>

namespace jade {
namespace {

struct Parser {
    const std::string &s;
    size_t i = 0;
    int depth = 0;
    explicit Parser(const std::string &src) : s(src) {}
    [[noreturn]] void fail(const char *what) {
        throw std::runtime_error(std::string("JSON parse error at byte ") + std::to_string(i) + ": " + what);
    }
    void ws() { while (i < s.size() && (s[i] == ' ' || s[i] == '\n' || s[i] == '\r' || s[i] == '\t')) ++i; }
    bool lit(const char *w) {
        size_t n = strlen(w);
        if (s.compare(i, n, w) == 0) { i += n; return true; }
        return false;
    }
    std::string string_body() {
        if (s[i] != '"') fail("expected string");
        ++i;
        std::string out;
        while (true) {
            if (i >= s.size()) fail("unterminated string");
            char c = s[i++];
            if (c == '"') break;
            if ((unsigned char)c < 0x20) fail("control character in string");
            if (c != '\\') { out.push_back(c); continue; }
            if (i >= s.size()) fail("bad escape");
            char e = s[i++];
            switch (e) {
                case '"': out.push_back('"'); break;
                case '\\': out.push_back('\\'); break;
                case '/': out.push_back('/'); break;
                case 'b': out.push_back('\b'); break;
                case 'f': out.push_back('\f'); break;
                case 'n': out.push_back('\n'); break;
                case 'r': out.push_back('\r'); break;
                case 't': out.push_back('\t'); break;
                case 'u': {
                    if (i + 4 > s.size()) fail("bad unicode escape");
                    unsigned cp = (unsigned)strtoul(s.substr(i, 4).c_str(), nullptr, 16);
                    i += 4;
                    if (cp < 0x80) out.push_back((char)cp);
                    else if (cp < 0x800) { out.push_back((char)(0xC0 | (cp >> 6))); out.push_back((char)(0x80 | (cp & 63))); }
                    else { out.push_back((char)(0xE0 | (cp >> 12))); out.push_back((char)(0x80 | ((cp >> 6) & 63))); out.push_back((char)(0x80 | (cp & 63))); }
                    break;
                }
                default: fail("bad escape");
            }
        }
        return out;
    }
    Json value() {
        if (++depth > 256) fail("nesting too deep");
        ws();
        if (i >= s.size()) fail("unexpected end");
        Json j;
        char c = s[i];
        if (c == '{') {
            ++i;
            j.kind = Json::Object;
            ws();
            if (i < s.size() && s[i] == '}') { ++i; --depth; return j; }
            while (true) {
                ws();
                std::string k = string_body();
                ws();
                if (i >= s.size() || s[i] != ':') fail("expected ':'");
                ++i;
                Json v = value();
                for (auto &f : j.fields) if (f.first == k) fail("duplicate field");
                j.fields.emplace_back(k, std::move(v));
                ws();
                if (i < s.size() && s[i] == ',') { ++i; continue; }
                if (i < s.size() && s[i] == '}') { ++i; break; }
                fail("expected ',' or '}'");
            }
        } else if (c == '[') {
            ++i;
            j.kind = Json::Array;
            ws();
            if (i < s.size() && s[i] == ']') { ++i; --depth; return j; }
            while (true) {
                j.items.push_back(value());
                ws();
                if (i < s.size() && s[i] == ',') { ++i; continue; }
                if (i < s.size() && s[i] == ']') { ++i; break; }
                fail("expected ',' or ']'");
            }
        } else if (c == '"') {
            j.kind = Json::String;
            j.text = string_body();
        } else if (lit("true")) { j.kind = Json::Bool; j.b = true; }
        else if (lit("false")) { j.kind = Json::Bool; j.b = false; }
        else if (lit("null")) { j.kind = Json::Null; }
        else if (c == '-' || (c >= '0' && c <= '9')) {
            size_t st = i;
            if (s[i] == '-') ++i;
            while (i < s.size() && (isdigit((unsigned char)s[i]) || s[i] == '.' || s[i] == 'e' || s[i] == 'E' || s[i] == '+' || s[i] == '-')) ++i;
            j.kind = Json::Number;
            j.text = s.substr(st, i - st);
            char *end = nullptr;
            j.num = strtod(j.text.c_str(), &end);
            if (!end || *end) fail("bad number");
        } else fail("unexpected character");
        --depth;
        return j;
    }
};

void escape(std::string &out, const std::string &v) {
    out.push_back('"');
    for (char c : v) {
        switch (c) {
            case '"': out += "\\\""; break;
            case '\\': out += "\\\\"; break;
            case '\n': out += "\\n"; break;
            case '\r': out += "\\r"; break;
            case '\t': out += "\\t"; break;
            default:
                if ((unsigned char)c < 0x20) { char b[8]; snprintf(b, sizeof b, "\\u%04x", c); out += b; }
                else out.push_back(c);
        }
    }
    out.push_back('"');
}

std::string number_text(const Json &j) {
    if (!j.text.empty()) return j.text;  // integers and parsed numbers keep their text
    if (!std::isfinite(j.num)) return "null";
    return ryu_like(j.num, j.float_width);
}

void write(std::string &out, const Json &j, int indent, int level) {
    auto nl = [&](int lv) {
        if (indent < 0) return;
        out.push_back('\n');
        out.append((size_t)(indent * lv), ' ');
    };
    switch (j.kind) {
        case Json::Null: out += "null"; break;
        case Json::Bool: out += j.b ? "true" : "false"; break;
        case Json::Number: out += number_text(j); break;
        case Json::String: escape(out, j.text); break;
        case Json::Array:
            if (j.items.empty()) { out += "[]"; break; }
            out.push_back('[');
            for (size_t k = 0; k < j.items.size(); ++k) {
                if (k) out.push_back(',');
                nl(level + 1);
                write(out, j.items[k], indent, level + 1);
            }
            nl(level);
            out.push_back(']');
            break;
        case Json::Object:
            if (j.fields.empty()) { out += "{}"; break; }
            out.push_back('{');
            for (size_t k = 0; k < j.fields.size(); ++k) {
                if (k) out.push_back(',');
                nl(level + 1);
                escape(out, j.fields[k].first);
                out += indent < 0 ? ":" : ": ";
                write(out, j.fields[k].second, indent, level + 1);
            }
            nl(level);
            out.push_back('}');
            break;
    }
}

// Shortest decimal digits d (no leading zeros) and exponent e with value = 0.d * 10^e
// that round-trip through strtof/strtod at the given width.
void shortest_digits(double v, int width, std::string &digits, int &point) {
    char buf[64];
    for (int p = 1; p <= 17; ++p) {
        snprintf(buf, sizeof buf, "%.*e", p - 1, v);
        bool ok = width == 32 ? (strtof(buf, nullptr) == (float)v) : (strtod(buf, nullptr) == v);
        if (ok) break;
    }
    // buf = "[-]d.ddde[+-]XX"
    const char *q = buf;
    if (*q == '-') ++q;
    digits.clear();
    while (*q && *q != 'e') { if (*q != '.') digits.push_back(*q); ++q; }
    int exp10 = atoi(q + 1);
    while (digits.size() > 1 && digits.back() == '0') digits.pop_back();
    point = exp10 + 1;  // value = 0.digits * 10^point
}

}  // namespace

Json Json::sorted() const {
    Json j = *this;
    if (kind == Object) {
        std::sort(j.fields.begin(), j.fields.end(), [](auto &a, auto &b) { return a.first < b.first; });
        for (auto &f : j.fields) f.second = f.second.sorted();
    } else if (kind == Array) {
        for (auto &x : j.items) x = x.sorted();
    }
    return j;
}

Json parse_json(const std::string &s) {
    Parser p(s);
    Json j = p.value();
    p.ws();
    if (p.i != s.size()) p.fail("trailing characters");
    return j;
}

std::string to_string_pretty(const Json &j) {
    std::string out;
    write(out, j, 2, 0);
    return out;
}
std::string to_string_compact(const Json &j) {
    std::string out;
    write(out, j, -1, 0);
    return out;
}

std::string rust_lower_exp_f32(float v) {
    std::string out;
    if (std::signbit(v)) out.push_back('-');
    if (v == 0.0f) return out + "0e0";
    std::string digits;
    int point;
    shortest_digits(std::fabs((double)v), 32, digits, point);
    out.push_back(digits[0]);
    if (digits.size() > 1) { out.push_back('.'); out.append(digits.substr(1)); }
    out += "e" + std::to_string(point - 1);
    return out;
}

std::string ryu_like(double v, int width) {
    std::string out;
    if (std::signbit(v)) out.push_back('-');
    if (v == 0.0) return out + "0.0";
    std::string d;
    int kk;  // value = 0.d * 10^kk, i.e. the decimal point sits after kk digits
    shortest_digits(std::fabs(v), width, d, kk);
    const int len = (int)d.size();
    const int k = kk - len;  // value = d * 10^k
    if (k >= 0 && kk <= 16) {
        out += d + std::string((size_t)k, '0') + ".0";
    } else if (kk > 0 && kk <= 16) {
        out += d.substr(0, (size_t)kk) + "." + d.substr((size_t)kk);
    } else if (kk > -5 && kk <= 0) {
        out += "0." + std::string((size_t)(-kk), '0') + d;
    } else if (len == 1) {
        out += d + "e" + std::to_string(kk - 1);
    } else {
        out += d.substr(0, 1) + "." + d.substr(1) + "e" + std::to_string(kk - 1);
    }
    return out;
}

}  // namespace jade
