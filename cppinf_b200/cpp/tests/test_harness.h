// A small GoogleTest-style harness (GoogleTest is not available in this toolchain): TEST registration,
// EXPECT_/ASSERT_ macros and a main that runs every test, or only those marked host-only with --host-only (no GPU).
#pragma once

#include <cmath>
#include <cstdio>
#include <exception>
#include <functional>
#include <sstream>
#include <string>
#include <string_view>
#include <vector>

namespace test_harness {

struct TestCase {
    std::string name;
    bool needs_gpu;
    std::function<void()> body;
};

inline std::vector<TestCase>& registry() {
    static std::vector<TestCase> tests;
    return tests;
}

inline int& failures() {
    static int count = 0;
    return count;
}

struct Registrar {
    Registrar(std::string name, bool needs_gpu, std::function<void()> body) {
        registry().push_back({std::move(name), needs_gpu, std::move(body)});
    }
};

struct FatalFailure {};

inline void report(const char* file, int line, const std::string& what) {
    ++failures();
    std::fprintf(stderr, "%s:%d: Failure\n  %s\n", file, line, what.c_str());
}

template <typename T>
std::string show(const T& v) {
    if constexpr (requires(std::ostream& os, const T& x) { os << x; }) {
        std::ostringstream os;
        os << v;
        return os.str();
    } else {
        return "<value>";
    }
}

inline int run_all(int argc, char** argv) {
    bool host_only = false;
    std::string filter;
    for (int i = 1; i < argc; ++i) {
        const std::string_view arg = argv[i];
        if (arg == "--host-only") {
            host_only = true;
        } else if (arg.rfind("--filter=", 0) == 0) {
            filter = std::string(arg.substr(9));
        }
    }
    int run = 0;
    int failed = 0;
    for (const auto& t : registry()) {
        if ((host_only && t.needs_gpu) || (!filter.empty() && t.name.find(filter) == std::string::npos)) {
            continue;
        }
        const int before = failures();
        ++run;
        try {
            t.body();
        } catch (const FatalFailure&) {
        } catch (const std::exception& e) {
            report(__FILE__, __LINE__, std::string("uncaught exception: ") + e.what());
        }
        const bool ok = failures() == before;
        failed += ok ? 0 : 1;
        std::printf("[%s] %s\n", ok ? "       OK " : "  FAILED  ", t.name.c_str());
    }
    std::printf("%d tests run, %d failed\n", run, failed);
    return failed == 0 ? 0 : 1;
}

} // namespace test_harness

#define HARNESS_CONCAT2(a, b) a##b
#define HARNESS_CONCAT(a, b) HARNESS_CONCAT2(a, b)

// TEST runs on the GPU (device tensors, or host tensors staged through the GPU); HOST_TEST needs no GPU.
#define HARNESS_DEFINE(fixture, name, gpu)                                                                   \
    static void HARNESS_CONCAT(fixture##_##name, _body)();                                                   \
    static test_harness::Registrar HARNESS_CONCAT(fixture##_##name, _registrar)(#fixture "." #name, gpu,     \
                                                                                &HARNESS_CONCAT(fixture##_##name, _body)); \
    static void HARNESS_CONCAT(fixture##_##name, _body)()
#define TEST(fixture, name) HARNESS_DEFINE(fixture, name, true)
#define HOST_TEST(fixture, name) HARNESS_DEFINE(fixture, name, false)

#define HARNESS_CHECK(cond, text, fatal)                                                                     \
    do {                                                                                                     \
        if (!(cond)) {                                                                                       \
            test_harness::report(__FILE__, __LINE__, text);                                                  \
            if (fatal) {                                                                                     \
                throw test_harness::FatalFailure{};                                                          \
            }                                                                                                \
        }                                                                                                    \
    } while (0)

#define EXPECT_TRUE(c) HARNESS_CHECK((c), "EXPECT_TRUE(" #c ")", false)
#define EXPECT_EQ(a, b)                                                                                      \
    HARNESS_CHECK((a) == (b), "EXPECT_EQ(" #a ", " #b "): " + test_harness::show(a) + " vs " +               \
                                  test_harness::show(b), false)
#define ASSERT_EQ(a, b)                                                                                      \
    HARNESS_CHECK((a) == (b), "ASSERT_EQ(" #a ", " #b "): " + test_harness::show(a) + " vs " +               \
                                  test_harness::show(b), true)
#define EXPECT_NEAR(a, b, tol)                                                                               \
    HARNESS_CHECK(std::fabs(static_cast<double>(a) - static_cast<double>(b)) <= static_cast<double>(tol),    \
                  "EXPECT_NEAR(" #a ", " #b "): " + test_harness::show(a) + " vs " + test_harness::show(b),  \
                  false)
#define EXPECT_THROW(stmt, exc)                                                                              \
    do {                                                                                                     \
        bool caught_ = false;                                                                                \
        try {                                                                                                \
            (void)(stmt);                                                                                    \
        } catch (const exc&) {                                                                               \
            caught_ = true;                                                                                  \
        } catch (...) {                                                                                      \
        }                                                                                                    \
        HARNESS_CHECK(caught_, "EXPECT_THROW(" #stmt ", " #exc ")", false);                                  \
    } while (0)
