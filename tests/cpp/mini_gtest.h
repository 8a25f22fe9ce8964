// mini_gtest.h -- TEST INFRASTRUCTURE ONLY: a small self-contained test runner
// whose console output follows GoogleTest's format ("[ RUN      ]",
// "[       OK ]", "[  FAILED  ]", "[  PASSED  ] N tests."), so scripts that
// grade a gtest binary by its summary lines work on these suites unchanged.
// Written for this repository (GoogleTest itself is not in the image); it
// implements only what the suites here use:
//   TEST(Suite, Name) { ... }
//   mini_gtest::add(full_name, fn)          -- register a generated case
//   EXPECT_TRUE(c) << msg; EXPECT_LE(a, b) << msg; ASSERT_TRUE(c);
//   flags --gtest_filter=PAT (':'-separated, '*' wildcards, '-' negatives)
//   and --gtest_list_tests.
#pragma once
#include <chrono>
#include <cstdio>
#include <cstring>
#include <functional>
#include <sstream>
#include <string>
#include <vector>

namespace mini_gtest {

struct Case {
    std::string name;
    std::function<void()> fn;
};

inline std::vector<Case>& registry() {
    static std::vector<Case> r;
    return r;
}
inline bool& current_failed() {
    static bool f = false;
    return f;
}
inline void add(const std::string& name, std::function<void()> fn) {
    registry().push_back({name, std::move(fn)});
}

struct Registrar {
    Registrar(const char* suite, const char* name, void (*fn)()) {
        add(std::string(suite) + "." + name, fn);
    }
};

// Collects a failure message; reports it when the statement ends.
class Failure {
  public:
    Failure(const char* file, int line, const char* what) {
        os_ << file << ":" << line << ": Failure\n" << what << "\n";
    }
    template <class T>
    Failure& operator<<(const T& v) {
        os_ << v;
        return *this;
    }
    ~Failure() {
        current_failed() = true;
        std::fputs(os_.str().c_str(), stdout);
        std::fputs("\n", stdout);
    }

  private:
    std::ostringstream os_;
};

struct FatalFailure {};  // thrown by ASSERT_* to end the test body

inline bool glob(const char* p, const char* s) {
    if (*p == '\0') return *s == '\0';
    if (*p == '*') return glob(p + 1, s) || (*s && glob(p, s + 1));
    return *s && (*p == '?' || *p == *s) && glob(p + 1, s + 1);
}

// gtest filter semantics: positive patterns before '-', negative after.
inline bool selected(const std::string& name, const std::string& filter) {
    std::string pos = filter, neg;
    const size_t dash = filter.find('-');
    if (dash != std::string::npos) {
        pos = filter.substr(0, dash);
        neg = filter.substr(dash + 1);
    }
    auto any = [&](const std::string& pats) {
        size_t start = 0;
        while (start <= pats.size()) {
            size_t end = pats.find(':', start);
            if (end == std::string::npos) end = pats.size();
            const std::string pat = pats.substr(start, end - start);
            if (!pat.empty() && glob(pat.c_str(), name.c_str())) return true;
            start = end + 1;
        }
        return false;
    };
    if (pos.empty()) pos = "*";
    return any(pos) && !(neg.size() && any(neg));
}

inline int run_all(int argc, char** argv) {
    std::string filter = "*";
    bool list = false;
    for (int i = 1; i < argc; ++i) {
        if (std::strncmp(argv[i], "--gtest_filter=", 15) == 0) filter = argv[i] + 15;
        if (std::strcmp(argv[i], "--gtest_list_tests") == 0) list = true;
    }
    if (list) {
        for (auto& c : registry())
            if (selected(c.name, filter)) std::printf("%s\n", c.name.c_str());
        return 0;
    }
    std::vector<Case*> todo;
    for (auto& c : registry())
        if (selected(c.name, filter)) todo.push_back(&c);
    std::vector<std::string> failed;
    std::printf("[==========] Running %zu tests.\n", todo.size());
    const auto t_all = std::chrono::steady_clock::now();
    for (Case* c : todo) {
        std::printf("[ RUN      ] %s\n", c->name.c_str());
        std::fflush(stdout);
        current_failed() = false;
        const auto t0 = std::chrono::steady_clock::now();
        try {
            c->fn();
        } catch (const FatalFailure&) {
        } catch (const std::exception& e) {
            Failure(__FILE__, __LINE__, "uncaught exception") << e.what();
        }
        const long ms = (long)std::chrono::duration_cast<std::chrono::milliseconds>(
                            std::chrono::steady_clock::now() - t0).count();
        if (current_failed()) {
            std::printf("[  FAILED  ] %s (%ld ms)\n", c->name.c_str(), ms);
            failed.push_back(c->name);
        } else {
            std::printf("[       OK ] %s (%ld ms)\n", c->name.c_str(), ms);
        }
        std::fflush(stdout);
    }
    const long total = (long)std::chrono::duration_cast<std::chrono::milliseconds>(
                           std::chrono::steady_clock::now() - t_all).count();
    std::printf("[==========] %zu tests ran. (%ld ms total)\n", todo.size(), total);
    std::printf("[  PASSED  ] %zu tests.\n", todo.size() - failed.size());
    if (!failed.empty()) {
        std::printf("[  FAILED  ] %zu tests, listed below:\n", failed.size());
        for (auto& n : failed) std::printf("[  FAILED  ] %s\n", n.c_str());
        return 1;
    }
    return 0;
}

}  // namespace mini_gtest

#define TEST(suite, name)                                                           \
    static void suite##_##name##_body();                                            \
    static mini_gtest::Registrar suite##_##name##_reg(#suite, #name,                \
                                                      suite##_##name##_body);       \
    static void suite##_##name##_body()

#define EXPECT_TRUE(c) \
    if (c) {           \
    } else             \
        mini_gtest::Failure(__FILE__, __LINE__, "Expected: " #c)
#define EXPECT_LE(a, b) \
    if ((a) <= (b)) {   \
    } else              \
        mini_gtest::Failure(__FILE__, __LINE__, "Expected: " #a " <= " #b)
#define EXPECT_EQ(a, b) \
    if ((a) == (b)) {   \
    } else              \
        mini_gtest::Failure(__FILE__, __LINE__, "Expected: " #a " == " #b)
#define ASSERT_TRUE(c)                                                   \
    do {                                                                 \
        if (!(c)) {                                                      \
            mini_gtest::Failure(__FILE__, __LINE__, "Expected: " #c);   \
            throw mini_gtest::FatalFailure{};                            \
        }                                                                \
    } while (0)
