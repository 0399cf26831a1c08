// Error transport across the extern "C" boundary.
//
// Library code reports a failure by throwing jade::Fault (a return code plus the
// message text). Every exported function runs its body through jade::c_entry,
// the one place where a Fault becomes the integer result and the NUL-terminated
// message in the caller's (err, cap) storage. No exception ever crosses into C.
#pragma once
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <exception>
#include <new>
#include <string>

#include "../../include/jade_runtime.h"

namespace jade {

struct Fault {
    int code;
    std::string text;
};

inline std::string vformat(const char *format, va_list args) {
    char small[512];
    va_list again;
    va_copy(again, args);
    const int n = std::vsnprintf(small, sizeof small, format, args);
    if (n < 0) {
        va_end(again);
        return "unformattable message";
    }
    if (static_cast<size_t>(n) < sizeof small) {
        va_end(again);
        return std::string(small, static_cast<size_t>(n));
    }
    std::string big(static_cast<size_t>(n) + 1, '\0');
    std::vsnprintf(&big[0], big.size(), format, again);
    va_end(again);
    big.resize(static_cast<size_t>(n));
    return big;
}

[[noreturn]] __attribute__((format(printf, 2, 3))) inline void raise(int code, const char *format, ...) {
    va_list args;
    va_start(args, format);
    std::string text = vformat(format, args);
    va_end(args);
    throw Fault{code, std::move(text)};
}

// Invalid input or state: JR_EINVAL with a fixed message.
inline void require(bool ok, const char *message) {
    if (!ok) throw Fault{JR_EINVAL, message};
}

// A failed CUDA runtime call: JR_ECUDA, "<operation>: <description> (<number>)".
inline void check_cuda(cudaError_t status, const char *operation) {
    if (status != cudaSuccess)
        raise(JR_ECUDA, "%s: %s (%d)", operation, cudaGetErrorString(status), static_cast<int>(status));
}

// Copies `text` into the caller's message storage, truncated and NUL-terminated.
inline void put_message(char *err, size_t cap, const std::string &text) {
    if (!err || !cap) return;
    const size_t n = text.size() < cap - 1 ? text.size() : cap - 1;
    std::memcpy(err, text.data(), n);
    err[n] = '\0';
}

// Runs `body` for an exported function: the message storage starts empty, a
// Fault becomes (code, message), an exhausted allocator JR_ENOMEM, any other
// exception JR_EINVAL with its text (spec parsing and validation throw those).
template <class Body>
int c_entry(char *err, size_t cap, Body &&body) noexcept {
    put_message(err, cap, std::string());
    try {
        body();
        return JR_OK;
    } catch (const Fault &f) {
        put_message(err, cap, f.text);
        return f.code;
    } catch (const std::bad_alloc &) {
        put_message(err, cap, "host allocation failed");
        return JR_ENOMEM;
    } catch (const std::exception &e) {
        put_message(err, cap, e.what());
        return JR_EINVAL;
    } catch (...) {
        put_message(err, cap, "unexpected failure");
        return JR_EINVAL;
    }
}

// Writes `text` (with its NUL) into a caller-owned output buffer, or fails with
// the byte count it needs.
inline void put_output(const std::string &text, char *out, size_t out_cap) {
    require(out && out_cap, "missing output buffer");
    if (text.size() + 1 > out_cap) {
        out[0] = '\0';
        raise(JR_EINVAL, "output buffer too small (%zu bytes needed)", text.size() + 1);
    }
    std::memcpy(out, text.c_str(), text.size() + 1);
}

}  // namespace jade
