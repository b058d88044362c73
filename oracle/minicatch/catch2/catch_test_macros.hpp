// A minimal, from-scratch stand-in for the part of Catch2 v3's <catch2/catch_test_macros.hpp>
// that the reference's attention tests use (TEST_CASE, SECTION, REQUIRE, CHECK, INFO). Catch2 is
// not available offline; this header lets ROCmKernels.Tests/AttentionTests.cpp compile unchanged.
// TEST INFRASTRUCTURE: built only into the oracle/_ref test binary.
//
// Semantics kept from Catch2: a TEST_CASE body is run once per SECTION, each run entering exactly
// one section (sections are flat here: nesting is not supported); CHECK records a failure and
// continues; REQUIRE records a failure and leaves the current run; INFO messages in scope are
// printed with a failure. Command line: `-c <section>` runs one section, `-s` also prints INFO
// messages of passing checks, `--list` lists test names.
#pragma once

#include <cstdio>
#include <exception>
#include <functional>
#include <sstream>
#include <string>
#include <vector>

namespace minicatch {

struct TestCase {
    const char *name;
    void (*body)();
};

inline std::vector<TestCase> &registry() {
    static std::vector<TestCase> cases;
    return cases;
}

struct Registrar {
    Registrar(const char *name, void (*body)()) { registry().push_back(TestCase{name, body}); }
};

struct RunState {
    int encountered = 0;       // sections seen in this run
    int target = 0;            // index of the section this run enters
    std::string filter;        // only enter sections with this name (empty = all)
    std::string current;       // name of the section entered in this run
    bool show_success = false; // print INFO for passing checks too
    int failed_checks = 0;
    int passed_checks = 0;
    std::vector<std::string> info;
};

inline RunState &state() {
    static RunState run;
    return run;
}

struct Section {
    bool active;
    explicit Section(const char *name) {
        RunState &s = state();
        active = s.encountered == s.target && (s.filter.empty() || s.filter == name);
        if (active) s.current = name;
        ++s.encountered;
    }
    explicit operator bool() const { return active; }
};

struct ScopedInfo {
    explicit ScopedInfo(std::string message) { state().info.push_back(std::move(message)); }
    ~ScopedInfo() { state().info.pop_back(); }
};

struct AbortRun {};

inline void record(bool passed, const char *macro, const char *expression, const char *file, int line, bool fatal) {
    RunState &s = state();
    if (passed) {
        ++s.passed_checks;
        if (s.show_success)
            for (const std::string &message : s.info) std::printf("  [%s] passed: %s\n", s.current.c_str(), message.c_str());
        return;
    }
    ++s.failed_checks;
    std::printf("%s:%d: FAILED %s(%s) in section '%s'\n", file, line, macro, expression, s.current.c_str());
    for (const std::string &message : s.info) std::printf("  with message: %s\n", message.c_str());
    if (fatal) throw AbortRun{};
}

inline int run(int argc, char **argv) {
    RunState &s = state();
    for (int i = 1; i < argc; ++i) {
        const std::string argument = argv[i];
        if (argument == "-c" && i + 1 < argc) s.filter = argv[++i];
        else if (argument == "-s") s.show_success = true;
        else if (argument == "--list") {
            for (const TestCase &test : registry()) std::printf("%s\n", test.name);
            return 0;
        }
    }
    int sections_run = 0;
    for (const TestCase &test : registry()) {
        for (int target = 0;; ++target) {
            s.encountered = 0;
            s.target = target;
            s.current.clear();
            s.info.clear();
            const int failed_before = s.failed_checks;
            try {
                test.body();
            } catch (const AbortRun &) {
            } catch (const std::exception &error) {
                ++s.failed_checks;
                std::printf("FAILED: '%s' section '%s' threw: %s\n", test.name, s.current.c_str(), error.what());
            }
            if (!s.current.empty()) {
                ++sections_run;
                std::printf("%s: %s / %s\n", s.failed_checks == failed_before ? "PASS" : "FAIL", test.name, s.current.c_str());
            }
            if (s.encountered == 0 || target + 1 >= s.encountered) break;
        }
    }
    std::printf("%d section(s), %d check(s) passed, %d failed\n", sections_run, s.passed_checks, s.failed_checks);
    return s.failed_checks == 0 && sections_run > 0 ? 0 : 1;
}

}  // namespace minicatch

#define MINICATCH_JOIN2(a, b) a##b
#define MINICATCH_JOIN(a, b) MINICATCH_JOIN2(a, b)

#define TEST_CASE(name, ...)                                                                                 \
    static void MINICATCH_JOIN(minicatch_body_, __LINE__)();                                                 \
    static const ::minicatch::Registrar MINICATCH_JOIN(minicatch_registrar_, __LINE__)(                      \
            name, &MINICATCH_JOIN(minicatch_body_, __LINE__));                                               \
    static void MINICATCH_JOIN(minicatch_body_, __LINE__)()

#define SECTION(name) if (const ::minicatch::Section MINICATCH_JOIN(minicatch_section_, __LINE__){name}; \
                          MINICATCH_JOIN(minicatch_section_, __LINE__))

#define CHECK(...) ::minicatch::record(static_cast<bool>(__VA_ARGS__), "CHECK", #__VA_ARGS__, __FILE__, __LINE__, false)
#define REQUIRE(...) ::minicatch::record(static_cast<bool>(__VA_ARGS__), "REQUIRE", #__VA_ARGS__, __FILE__, __LINE__, true)

#define INFO(message)                                                                                        \
    const ::minicatch::ScopedInfo MINICATCH_JOIN(minicatch_info_, __LINE__)([&] {                            \
        std::ostringstream minicatch_stream;                                                                 \
        minicatch_stream << message;                                                                         \
        return minicatch_stream.str();                                                                       \
    }())
