// A minimal stand-in for the GoogleTest API subset that GPT-SoVITS.cpp's T2S tests use (TEST,
// TEST_P, TestWithParam, Values, INSTANTIATE_TEST_SUITE_P, ASSERT_* / EXPECT_* with streamed
// messages, GTEST_SKIP), so those test files compile and run against include/gpt_sovits/t2s.h
// here, where GoogleTest is not installed.  Test infrastructure only; main() is gtest_main.cpp.
#pragma once

#include <cstdio>
#include <functional>
#include <memory>
#include <ostream>
#include <sstream>
#include <string>
#include <type_traits>
#include <vector>

namespace testing {

class Message {
public:
    template <class T>
    Message& operator<<(const T& v) {
        ss_ << v;
        return *this;
    }
    std::string str() const { return ss_.str(); }

private:
    std::ostringstream ss_;
};

class Test {
public:
    virtual ~Test() = default;
    virtual void SetUp() {}
    virtual void TearDown() {}
    virtual void TestBody() = 0;
};

template <class T>
class TestWithParam : public Test {
public:
    using ParamType = T;
    static const T*& param_slot() {
        static const T* p = nullptr;
        return p;
    }
    const T& GetParam() const { return *param_slot(); }
};

template <class T>
struct TestParamInfo {
    T param;
    size_t index;
};

template <class T, class... Ts>
std::vector<T> Values(T v, Ts... vs) {
    return std::vector<T>{v, T(vs)...};
}

namespace internal {

struct State {
    bool failed = false;
    bool skipped = false;
};
inline State& state() {
    static State s;
    return s;
}

struct Entry {
    std::string name;
    std::function<void()> run;
};
inline std::vector<Entry>& registry() {
    static std::vector<Entry> r;
    return r;
}

class AssertHelper {
public:
    AssertHelper(const char* file, int line, const char* text) : file_(file), line_(line), text_(text) {}
    void operator=(const Message& m) const {
        std::printf("%s:%d: Failure: %s %s\n", file_, line_, text_, m.str().c_str());
        state().failed = true;
    }

private:
    const char* file_;
    int line_;
    const char* text_;
};

class SkipHelper {
public:
    void operator=(const Message& m) const {
        std::printf("  skipped: %s\n", m.str().c_str());
        state().skipped = true;
    }
};

inline void run_test(Test* t) {
    t->SetUp();
    t->TestBody();
    t->TearDown();
    delete t;
}

inline int add_test(const char* name, std::function<Test*()> make) {
    registry().push_back(Entry{name, [make] { run_test(make()); }});
    return 0;
}

template <class F>
std::vector<std::pair<std::string, std::function<Test*()>>>& param_bodies() {
    static std::vector<std::pair<std::string, std::function<Test*()>>> b;
    return b;
}

template <class F>
int add_param_test(const char* name, std::function<Test*()> make) {
    param_bodies<F>().push_back({name, make});
    return 0;
}

template <class F, class Namer>
int instantiate(const char* prefix, const char* fixture, std::vector<typename F::ParamType> vals, Namer namer) {
    auto shared = std::make_shared<std::vector<typename F::ParamType>>(std::move(vals));
    for (auto& body : param_bodies<F>())
        for (size_t i = 0; i < shared->size(); ++i) {
            TestParamInfo<typename F::ParamType> info{(*shared)[i], i};
            const std::string name = std::string(prefix) + "/" + fixture + "." + body.first + "/" + namer(info);
            auto make = body.second;
            registry().push_back(Entry{name, [shared, i, make] {
                                           F::param_slot() = &(*shared)[i];
                                           run_test(make());
                                       }});
        }
    return 0;
}

template <class F>
int instantiate(const char* prefix, const char* fixture, std::vector<typename F::ParamType> vals) {
    return instantiate<F>(prefix, fixture, std::move(vals),
                          [](const TestParamInfo<typename F::ParamType>& info) { return std::to_string(info.index); });
}

}  // namespace internal
}  // namespace testing

int RUN_ALL_TESTS_MIN(int argc, char** argv);

#define TEST(suite, name)                                                                              \
    class suite##_##name##_Test : public ::testing::Test {                                             \
    public:                                                                                            \
        void TestBody() override;                                                                      \
    };                                                                                                 \
    static int suite##_##name##_reg = ::testing::internal::add_test(                                   \
        #suite "." #name, []() -> ::testing::Test* { return new suite##_##name##_Test(); });           \
    void suite##_##name##_Test::TestBody()

#define TEST_P(fixture, name)                                                                          \
    class fixture##_##name##_Test : public fixture {                                                   \
    public:                                                                                            \
        void TestBody() override;                                                                      \
    };                                                                                                 \
    static int fixture##_##name##_reg = ::testing::internal::add_param_test<fixture>(                  \
        #name, []() -> ::testing::Test* { return new fixture##_##name##_Test(); });                    \
    void fixture##_##name##_Test::TestBody()

#define INSTANTIATE_TEST_SUITE_P(prefix, fixture, ...) \
    static int prefix##_##fixture##_inst = ::testing::internal::instantiate<fixture>(#prefix, #fixture, __VA_ARGS__)

#define GTEST_MIN_CHECK_(cond, text, on_fail) \
    switch (0)                                \
    case 0:                                   \
    default:                                  \
        if (cond)                             \
            ;                                 \
        else                                  \
            on_fail ::testing::internal::AssertHelper(__FILE__, __LINE__, text) = ::testing::Message()

#define ASSERT_TRUE(c) GTEST_MIN_CHECK_((c), "ASSERT_TRUE(" #c ")", return)
#define ASSERT_FALSE(c) GTEST_MIN_CHECK_(!(c), "ASSERT_FALSE(" #c ")", return)
#define ASSERT_EQ(a, b) GTEST_MIN_CHECK_((a) == (b), "ASSERT_EQ(" #a ", " #b ")", return)
#define ASSERT_NE(a, b) GTEST_MIN_CHECK_((a) != (b), "ASSERT_NE(" #a ", " #b ")", return)
#define ASSERT_LT(a, b) GTEST_MIN_CHECK_((a) < (b), "ASSERT_LT(" #a ", " #b ")", return)
#define ASSERT_LE(a, b) GTEST_MIN_CHECK_((a) <= (b), "ASSERT_LE(" #a ", " #b ")", return)
#define ASSERT_GT(a, b) GTEST_MIN_CHECK_((a) > (b), "ASSERT_GT(" #a ", " #b ")", return)
#define ASSERT_GE(a, b) GTEST_MIN_CHECK_((a) >= (b), "ASSERT_GE(" #a ", " #b ")", return)
#define EXPECT_TRUE(c) GTEST_MIN_CHECK_((c), "EXPECT_TRUE(" #c ")", )
#define EXPECT_FALSE(c) GTEST_MIN_CHECK_(!(c), "EXPECT_FALSE(" #c ")", )
#define EXPECT_EQ(a, b) GTEST_MIN_CHECK_((a) == (b), "EXPECT_EQ(" #a ", " #b ")", )
#define EXPECT_NE(a, b) GTEST_MIN_CHECK_((a) != (b), "EXPECT_NE(" #a ", " #b ")", )
#define EXPECT_LT(a, b) GTEST_MIN_CHECK_((a) < (b), "EXPECT_LT(" #a ", " #b ")", )
#define EXPECT_LE(a, b) GTEST_MIN_CHECK_((a) <= (b), "EXPECT_LE(" #a ", " #b ")", )
#define EXPECT_GT(a, b) GTEST_MIN_CHECK_((a) > (b), "EXPECT_GT(" #a ", " #b ")", )
#define EXPECT_GE(a, b) GTEST_MIN_CHECK_((a) >= (b), "EXPECT_GE(" #a ", " #b ")", )
#define GTEST_SKIP() return ::testing::internal::SkipHelper() = ::testing::Message()
