// TEST INFRASTRUCTURE: a minimal registry and check macros for the native
// test libraries (GoogleTest is not available offline). A case throws
// Failure on the first failed check; qvp_*_run reports its text.
#pragma once

#include <cstdio>
#include <cmath>
#include <cstring>
#include <functional>
#include <map>
#include <sstream>
#include <string>

namespace native {

struct Failure {
    std::string what;
};

inline std::map<std::string, std::function<void()>>& registry() {
    static std::map<std::string, std::function<void()>> r;
    return r;
}

struct Register {
    Register(const char* name, std::function<void()> fn) { registry()[name] = std::move(fn); }
};

// Names of all cases, one per line; returns the count (or -1 if `cap` is short).
inline int list_cases(char* out, size_t cap) {
    std::string names;
    for (const auto& kv : registry()) names += kv.first + "\n";
    if (names.size() + 1 > cap) return -1;
    std::memcpy(out, names.c_str(), names.size() + 1);
    return static_cast<int>(registry().size());
}

// 0 = passed, 1 = failed (text in msg), 2 = unknown case.
inline int run_case(const char* name, char* msg, size_t cap) {
    const auto it = registry().find(name);
    std::string text;
    int rc = 0;
    if (it == registry().end()) {
        text = "unknown test";
        rc = 2;
    } else {
        try {
            it->second();
        } catch (const Failure& f) {
            text = f.what;
            rc = 1;
        }
    }
    std::snprintf(msg, cap, "%s", text.c_str());
    return rc;
}

}  // namespace native

#define CHECK(cond)                                                                         \
    do {                                                                                    \
        if (!(cond))                                                                        \
            throw ::native::Failure{std::string(__FILE__ ":") + std::to_string(__LINE__) + \
                                    ": " #cond};                                            \
    } while (0)

#define CHECK_NEAR(a, b, tol)                                                                       \
    do {                                                                                            \
        const double a_ = (a), b_ = (b);                                                            \
        if (!(std::fabs(a_ - b_) <= (tol))) {                                                       \
            std::ostringstream s_;                                                                  \
            s_ << __FILE__ << ":" << __LINE__ << ": " << a_ << " vs " << b_ << " (" #a " ~ " #b ")"; \
            throw ::native::Failure{s_.str()};                                                      \
        }                                                                                           \
    } while (0)

#define NATIVE_TEST(name)                                         \
    void name();                                                  \
    const ::native::Register reg_##name(#name, name);             \
    void name()
