// TEST INFRASTRUCTURE: a small stand-in for the part of the GoogleTest API
// that the reference's test files use (GoogleTest is not installed here).
// It lets those files compile unmodified against this project's headers:
// TEST, TEST_F, ::testing::Test, EXPECT_/ASSERT_ {EQ, NE, LT, LE, GT, GE,
// TRUE, FALSE}, EXPECT_FLOAT_EQ, EXPECT_NEAR, ASSERT_NO_FATAL_FAILURE and
// `<<` messages after any of them. The runner (gtest_main.cpp) runs every
// case in a child process, so a case that crashes fails alone.
#pragma once

#include <cmath>
#include <cstdint>
#include <cstring>
#include <functional>
#include <optional>
#include <ostream>
#include <sstream>
#include <string>
#include <type_traits>
#include <utility>
#include <vector>

namespace testing {

class Test {
public:
    virtual ~Test() = default;
    virtual void SetUp() {}
    virtual void TearDown() {}
    virtual void TestBody() = 0;
};

namespace internal {

template <class T, class = void>
struct Streamable : std::false_type {};
template <class T>
struct Streamable<T, std::void_t<decltype(std::declval<std::ostream&>() << std::declval<const T&>())>>
    : std::true_type {};

template <class T>
struct IsOptional : std::false_type {};
template <class T>
struct IsOptional<std::optional<T>> : std::true_type {};

template <class T>
void print(std::ostream& os, const T& v) {
    if constexpr (std::is_same_v<T, std::nullopt_t>) {
        os << "nullopt";
    } else if constexpr (IsOptional<T>::value) {
        if (v)
            print(os, *v);
        else
            os << "nullopt";
    } else if constexpr (std::is_enum_v<T>) {
        os << static_cast<long long>(static_cast<std::underlying_type_t<T>>(v));
    } else if constexpr (std::is_same_v<T, std::nullptr_t>) {
        os << "nullptr";
    } else if constexpr (std::is_pointer_v<T>) {
        os << static_cast<const void*>(v);
    } else if constexpr (std::is_same_v<T, bool>) {
        os << (v ? "true" : "false");
    } else if constexpr (Streamable<T>::value) {
        os << v;
    } else {
        os << "<" << sizeof(T) << "-byte object>";
    }
}

}  // namespace internal

class Message {
public:
    Message() = default;
    template <class T>
    Message& operator<<(const T& v) {
        internal::print(os_, v);
        return *this;
    }
    Message& operator<<(const char* s) {
        os_ << (s ? s : "(null)");
        return *this;
    }
    std::string str() const { return os_.str(); }

private:
    std::ostringstream os_;
};

namespace internal {

struct State {
    bool failed = false;
    bool fatal = false;
    std::string log;
};

inline State& state() {
    static State s;
    return s;
}

inline void record(const char* file, int line, const std::string& text, bool fatal) {
    State& s = state();
    s.failed = true;
    if (fatal) s.fatal = true;
    s.log += std::string(file) + ":" + std::to_string(line) + ": " + text + "\n";
}

struct Result {
    bool ok;
    std::string text;
    explicit operator bool() const { return ok; }
};

class Helper {
public:
    Helper(const char* file, int line, std::string text, bool fatal)
        : file_(file), line_(line), text_(std::move(text)), fatal_(fatal) {}
    void operator=(const Message& m) const {
        const std::string extra = m.str();
        record(file_, line_, extra.empty() ? text_ : text_ + " | " + extra, fatal_);
    }

private:
    const char* file_;
    int line_;
    std::string text_;
    bool fatal_;
};

template <class A, class B, class Op>
Result compare(Op op, const char* sym, const char* ea, const char* eb, const A& a, const B& b) {
    if (op(a, b)) return Result{true, {}};
    std::ostringstream os;
    os << "expected " << ea << " " << sym << " " << eb << ", got ";
    print(os, a);
    os << " vs ";
    print(os, b);
    return Result{false, os.str()};
}

inline Result boolean(bool v, bool want, const char* expr) {
    if (v == want) return Result{true, {}};
    return Result{false, std::string("expected ") + (want ? "true" : "false") + ": " + expr};
}

// Equal within 4 units in the last place (of float), as GoogleTest defines it.
inline Result float_eq(float a, float b, const char* ea, const char* eb) {
    auto biased = [](float f) {
        std::uint32_t u;
        std::memcpy(&u, &f, 4);
        return (u & 0x80000000u) ? 0x80000000u - (u & 0x7fffffffu) : 0x80000000u + u;
    };
    const bool nan = std::isnan(a) || std::isnan(b);
    const std::uint32_t x = biased(a), y = biased(b);
    if (!nan && (x > y ? x - y : y - x) <= 4u) return Result{true, {}};
    std::ostringstream os;
    os << "expected " << ea << " == " << eb << " (float, 4 ulp), got " << a << " vs " << b;
    return Result{false, os.str()};
}

inline Result near(double a, double b, double tol, const char* ea, const char* eb) {
    if (std::fabs(a - b) <= tol) return Result{true, {}};
    std::ostringstream os;
    os << "expected |" << ea << " - " << eb << "| <= " << tol << ", got " << a << " vs " << b;
    return Result{false, os.str()};
}

struct Case {
    std::string suite, name;
    std::function<Test*()> make;
};

inline std::vector<Case>& cases() {
    static std::vector<Case> c;
    return c;
}

inline bool add(const char* suite, const char* name, std::function<Test*()> make) {
    cases().push_back(Case{suite, name, std::move(make)});
    return true;
}

}  // namespace internal
}  // namespace testing

#define QVP_GT_CHECK_(res, fatal)                                      \
    switch (0)                                                         \
    case 0:                                                            \
    default:                                                           \
        if (const ::testing::internal::Result qvp_gt_r_ = (res)) {     \
        } else                                                         \
            QVP_GT_FAIL_##fatal(qvp_gt_r_)

#define QVP_GT_FAIL_1(r) return ::testing::internal::Helper(__FILE__, __LINE__, (r).text, true) = ::testing::Message()
#define QVP_GT_FAIL_0(r) ::testing::internal::Helper(__FILE__, __LINE__, (r).text, false) = ::testing::Message()

#define QVP_GT_CMP_(a, b, sym, fatal)                                                                           \
    QVP_GT_CHECK_(::testing::internal::compare([](const auto& x_, const auto& y_) { return x_ sym y_; }, #sym, #a, \
                                               #b, a, b),                                                       \
                  fatal)

#define EXPECT_EQ(a, b) QVP_GT_CMP_(a, b, ==, 0)
#define EXPECT_NE(a, b) QVP_GT_CMP_(a, b, !=, 0)
#define EXPECT_LT(a, b) QVP_GT_CMP_(a, b, <, 0)
#define EXPECT_LE(a, b) QVP_GT_CMP_(a, b, <=, 0)
#define EXPECT_GT(a, b) QVP_GT_CMP_(a, b, >, 0)
#define EXPECT_GE(a, b) QVP_GT_CMP_(a, b, >=, 0)
#define ASSERT_EQ(a, b) QVP_GT_CMP_(a, b, ==, 1)
#define ASSERT_NE(a, b) QVP_GT_CMP_(a, b, !=, 1)
#define ASSERT_LT(a, b) QVP_GT_CMP_(a, b, <, 1)
#define ASSERT_LE(a, b) QVP_GT_CMP_(a, b, <=, 1)
#define ASSERT_GT(a, b) QVP_GT_CMP_(a, b, >, 1)
#define ASSERT_GE(a, b) QVP_GT_CMP_(a, b, >=, 1)
#define EXPECT_TRUE(c) QVP_GT_CHECK_(::testing::internal::boolean(static_cast<bool>(c), true, #c), 0)
#define EXPECT_FALSE(c) QVP_GT_CHECK_(::testing::internal::boolean(static_cast<bool>(c), false, #c), 0)
#define ASSERT_TRUE(c) QVP_GT_CHECK_(::testing::internal::boolean(static_cast<bool>(c), true, #c), 1)
#define ASSERT_FALSE(c) QVP_GT_CHECK_(::testing::internal::boolean(static_cast<bool>(c), false, #c), 1)
#define EXPECT_FLOAT_EQ(a, b) \
    QVP_GT_CHECK_(::testing::internal::float_eq(static_cast<float>(a), static_cast<float>(b), #a, #b), 0)
#define ASSERT_FLOAT_EQ(a, b) \
    QVP_GT_CHECK_(::testing::internal::float_eq(static_cast<float>(a), static_cast<float>(b), #a, #b), 1)
#define EXPECT_NEAR(a, b, tol)                                                                                   \
    QVP_GT_CHECK_(::testing::internal::near(static_cast<double>(a), static_cast<double>(b), static_cast<double>(tol), \
                                            #a, #b),                                                             \
                  0)

#define ASSERT_NO_FATAL_FAILURE(stmt)                                                              \
    do {                                                                                           \
        const bool qvp_gt_before_ = ::testing::internal::state().fatal;                            \
        ::testing::internal::state().fatal = false;                                                \
        stmt;                                                                                      \
        const bool qvp_gt_now_ = ::testing::internal::state().fatal;                               \
        ::testing::internal::state().fatal = qvp_gt_before_ || qvp_gt_now_;                       \
        if (qvp_gt_now_) {                                                                         \
            ::testing::internal::record(__FILE__, __LINE__, "fatal failure inside " #stmt, true); \
            return;                                                                                \
        }                                                                                          \
    } while (0)

#define QVP_GT_TEST_(suite, name, base)                                                               \
    class suite##_##name##_Test : public base {                                                       \
    public:                                                                                           \
        void TestBody() override;                                                                     \
    };                                                                                                \
    static const bool suite##_##name##_registered_ =                                                  \
        ::testing::internal::add(#suite, #name, []() -> ::testing::Test* { return new suite##_##name##_Test; }); \
    void suite##_##name##_Test::TestBody()

#define TEST(suite, name) QVP_GT_TEST_(suite, name, ::testing::Test)
#define TEST_F(fixture, name) QVP_GT_TEST_(fixture, name, fixture)
