// main() of the minimal GoogleTest stand-in (gtest/gtest.h beside it).  Runs every registered
// test whose name contains the optional --gtest_filter=SUBSTRING and prints one
// "RESULT <name> PASSED|FAILED|SKIPPED" line per test; exits 1 if any test failed.
#include "gtest/gtest.h"

#include <cstring>
#include <string>


int main(int argc, char** argv) {
    std::string filter;
    for (int i = 1; i < argc; ++i)
        if (!std::strncmp(argv[i], "--gtest_filter=", 15)) filter = argv[i] + 15;
    int failed = 0, passed = 0, skipped = 0;
    for (auto& e : ::testing::internal::registry()) {
        if (!filter.empty() && e.name.find(filter) == std::string::npos) continue;
        ::testing::internal::state() = ::testing::internal::State();
        std::printf("[ RUN      ] %s\n", e.name.c_str());
        std::fflush(stdout);
        e.run();
        const auto& st = ::testing::internal::state();
        const char* r = st.failed ? "FAILED" : (st.skipped ? "SKIPPED" : "PASSED");
        (st.failed ? failed : (st.skipped ? skipped : passed))++;
        std::printf("RESULT %s %s\n", e.name.c_str(), r);
        std::fflush(stdout);
    }
    std::printf("%d passed, %d failed, %d skipped\n", passed, failed, skipped);
    return failed ? 1 : 0;
}
