// A minimal, from-scratch stand-in for the part of Catch2 v3's <catch2/catch_test_macros.hpp>
// that the reference's attention, generic-attention and positional tests use (TEST_CASE, SECTION,
// REQUIRE, CHECK, INFO). Catch2 is not available offline; this header lets those test files
// (ROCmKernels.Tests/AttentionTests.cpp, Generic/AttentionGenericTests.cpp, PositionalTests.cpp)
// compile unchanged.
// TEST INFRASTRUCTURE: built only into the oracle/_ref test binary.
//
// Semantics kept from Catch2: a TEST_CASE body is run once per leaf SECTION (once if it has
// none); each run enters, at every nesting level, the first section that is not complete yet and
// skips its siblings (a section is complete once it has run without discovering unfinished
// child sections). CHECK records a failure and continues; REQUIRE records a failure and leaves
// the current run; INFO messages in scope are printed with a failure. Command line: `-c <section>` runs only the
// sections of that name (and everything inside them), `-s` also prints INFO messages of passing
// checks, `--list` lists test names.
#pragma once

#include <cstdio>
#include <exception>
#include <functional>
#include <map>
#include <set>
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
    // Section paths are the names from the test case down, joined by " / ".
    std::set<std::string> completed;                     // sections finished (this test case)
    std::map<std::string, std::set<std::string>> children;  // section path -> child paths seen
    std::set<std::string> entered_parents;               // this run: parents that entered a child
    std::vector<std::string> stack;                      // this run: entered sections, outermost first
    std::vector<bool> matched;                           // per stack entry: inside a filtered section
    std::string filter;        // only enter sections with this name (empty = all)
    std::string current;       // deepest section entered in this run
    bool show_success = false; // print INFO for passing checks too
    int failed_checks = 0;
    int passed_checks = 0;
    std::vector<std::string> info;
};

inline RunState &state() {
    static RunState run;
    return run;
}

inline std::string join(const std::vector<std::string> &names) {
    std::string path;
    for (const std::string &name : names) path += (path.empty() ? "" : " / ") + name;
    return path;
}

struct Section {
    bool active = false;
    std::string path;
    explicit Section(const char *name) {
        RunState &s = state();
        const std::string parent = join(s.stack);
        path = parent.empty() ? std::string(name) : parent + " / " + name;
        s.children[parent].insert(path);
        const bool inside = !s.matched.empty() && s.matched.back();
        const bool matches = s.filter.empty() || inside || s.filter == name;
        if (!matches) {
            s.completed.insert(path);  // filtered out: never entered
            return;
        }
        active = !s.completed.count(path) && !s.entered_parents.count(parent);
        if (!active) return;
        s.entered_parents.insert(parent);
        s.stack.push_back(name);
        s.matched.push_back(inside || s.filter == name);
        s.current = path;
    }
    ~Section() {
        if (!active) return;
        RunState &s = state();
        bool done = true;
        for (const std::string &child : s.children[path]) done = done && s.completed.count(child) > 0;
        if (done) s.completed.insert(path);
        s.stack.pop_back();
        s.matched.pop_back();
    }
    Section(const Section &) = delete;
    Section &operator=(const Section &) = delete;
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
        s.completed.clear();
        s.children.clear();
        for (;;) {
            s.entered_parents.clear();
            s.stack.clear();
            s.matched.clear();
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
            if (!s.current.empty() || s.children[""].empty()) {  // a leaf section, or a test case without sections
                ++sections_run;
                std::printf("%s: %s%s%s\n", s.failed_checks == failed_before ? "PASS" : "FAIL", test.name,
                            s.current.empty() ? "" : " / ", s.current.c_str());
            }
            bool finished = true;  // every top-level section complete (or none exists)
            for (const std::string &child : s.children[""]) finished = finished && s.completed.count(child) > 0;
            if (finished || s.current.empty()) break;
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
