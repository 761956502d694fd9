// A minimal stand-in for <gtest/gtest.h>. TEST INFRASTRUCTURE ONLY.
//
// gtest is not installed here, and the reference's CMake would fetch it over the
// network. This header provides just what tests/golden_kernel_test.cpp of the
// reference uses (TEST, ASSERT_EQ, ASSERT_NE, EXPECT_TRUE, AssertionResult) so
// that file compiles unmodified and its Golden.MatMulQ body -- the reference's
// own int8 packer -- can run from oracle/ref_packer_pin.cpp.
#pragma once

#include <functional>
#include <iostream>
#include <sstream>
#include <string>
#include <utility>
#include <vector>

namespace testing {

class Message {
 public:
  template <typename T>
  Message& operator<<(const T& v) {
    ss_ << v;
    return *this;
  }
  std::string str() const { return ss_.str(); }

 private:
  std::ostringstream ss_;
};

class AssertionResult {
 public:
  explicit AssertionResult(bool ok) : ok_(ok) {}
  AssertionResult(const AssertionResult& o) : ok_(o.ok_), msg_(o.msg_) {}
  explicit operator bool() const { return ok_; }
  template <typename T>
  AssertionResult& operator<<(const T& v) {
    std::ostringstream ss;
    ss << v;
    msg_ += ss.str();
    return *this;
  }
  const std::string& message() const { return msg_; }

 private:
  bool ok_;
  std::string msg_;
};

inline AssertionResult AssertionSuccess() { return AssertionResult(true); }
inline AssertionResult AssertionFailure() { return AssertionResult(false); }

namespace shim {

struct TestCase {
  std::string name;  // "Suite.Name"
  std::function<void()> body;
};

inline std::vector<TestCase>& registry() {
  static std::vector<TestCase> r;
  return r;
}

inline int& failures() {
  static int n = 0;
  return n;
}

struct Registrar {
  Registrar(const char* suite, const char* name, void (*fn)()) {
    registry().push_back({std::string(suite) + "." + name, fn});
  }
};

// Records one failed check; `= Message() << ...` appends the streamed context.
class Failure {
 public:
  Failure(const char* file, int line, std::string what) {
    ++failures();
    std::cerr << file << ":" << line << ": check failed: " << what;
  }
  void operator=(const Message& m) const { std::cerr << " " << m.str() << "\n"; }
};

inline std::string describe(const AssertionResult& r) { return r.message(); }
inline std::string describe(bool) { return std::string(); }

// Runs the test named `full_name`; returns the number of failed checks, or -1 if
// no such test is registered.
inline int run(const std::string& full_name) {
  for (const TestCase& t : registry()) {
    if (t.name == full_name) {
      failures() = 0;
      t.body();
      return failures();
    }
  }
  return -1;
}

}  // namespace shim
}  // namespace testing

#define TEST(suite, name)                                                            \
  static void suite##_##name##_body();                                               \
  static ::testing::shim::Registrar suite##_##name##_registrar(#suite, #name,        \
                                                               &suite##_##name##_body); \
  static void suite##_##name##_body()

#define GTEST_SHIM_CHECK_(ok, what, on_fail) \
  if (ok)                                    \
    ;                                        \
  else                                       \
    on_fail ::testing::shim::Failure(__FILE__, __LINE__, what) = ::testing::Message()

#define ASSERT_EQ(a, b) GTEST_SHIM_CHECK_((a) == (b), #a " == " #b, return)
#define ASSERT_NE(a, b) GTEST_SHIM_CHECK_((a) != (b), #a " != " #b, return)
#define EXPECT_TRUE(c)                                                                           \
  if (const auto& gtest_shim_r_ = (c))                                                           \
    ;                                                                                            \
  else                                                                                           \
    ::testing::shim::Failure(__FILE__, __LINE__, std::string(#c) + " " +                         \
                                                     ::testing::shim::describe(gtest_shim_r_)) = \
        ::testing::Message()
