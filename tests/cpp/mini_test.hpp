// mini_test.hpp — a minimal test runner standing in for GoogleTest (absent
// here): TEST(group, name) registers a case, EXPECT_* record failures,
// main() runs the cases whose group matches argv[1] ("cpu", "gpu" or "all").
#pragma once
#include <cmath>
#include <cstdio>
#include <cstring>
#include <functional>
#include <string>
#include <vector>

namespace mini {
struct Case {
  std::string group, name;
  std::function<void()> fn;
};
inline std::vector<Case>& registry() {
  static std::vector<Case> r;
  return r;
}
inline int& failures() {
  static int f = 0;
  return f;
}
struct Reg {
  Reg(const char* g, const char* n, std::function<void()> fn) { registry().push_back({g, n, std::move(fn)}); }
};
inline void fail(const char* file, int line, const std::string& what) {
  std::printf("  FAILED %s:%d: %s\n", file, line, what.c_str());
  ++failures();
}
}  // namespace mini

#define MT_CAT2(a, b) a##b
#define MT_CAT(a, b) MT_CAT2(a, b)
#define TEST(group, name)                                                      \
  static void MT_CAT(test_, MT_CAT(group, MT_CAT(_, name)))();                 \
  static mini::Reg MT_CAT(reg_, MT_CAT(group, MT_CAT(_, name)))(#group, #name, \
      MT_CAT(test_, MT_CAT(group, MT_CAT(_, name))));                          \
  static void MT_CAT(test_, MT_CAT(group, MT_CAT(_, name)))()

#define EXPECT_TRUE(c) do { if (!(c)) mini::fail(__FILE__, __LINE__, #c); } while (0)
#define EXPECT_FALSE(c) EXPECT_TRUE(!(c))
#define EXPECT_EQ(a, b) do { if (!((a) == (b))) mini::fail(__FILE__, __LINE__, #a " == " #b); } while (0)
#define EXPECT_NE(a, b) do { if (!((a) != (b))) mini::fail(__FILE__, __LINE__, #a " != " #b); } while (0)
#define EXPECT_LE(a, b) do { if (!((a) <= (b))) mini::fail(__FILE__, __LINE__, #a " <= " #b); } while (0)
#define EXPECT_GE(a, b) do { if (!((a) >= (b))) mini::fail(__FILE__, __LINE__, #a " >= " #b); } while (0)
#define EXPECT_LT(a, b) do { if (!((a) < (b))) mini::fail(__FILE__, __LINE__, #a " < " #b); } while (0)
#define EXPECT_NEAR(a, b, tol) do { if (!(std::fabs((double)(a) - (double)(b)) <= (tol))) \
    mini::fail(__FILE__, __LINE__, #a " ~= " #b " (" + std::to_string((double)(a)) + " vs " + std::to_string((double)(b)) + ")"); } while (0)
#define EXPECT_THROW(stmt, ex) do { bool caught_ = false; try { stmt; } catch (const ex&) { caught_ = true; } catch (...) {} \
    if (!caught_) mini::fail(__FILE__, __LINE__, "expected " #ex " from " #stmt); } while (0)
#define EXPECT_NO_THROW(stmt) do { try { stmt; } catch (const std::exception& e_) { \
    mini::fail(__FILE__, __LINE__, std::string("unexpected exception: ") + e_.what()); } } while (0)

inline int mini_main(int argc, char** argv) {
  const std::string want = argc > 1 ? argv[1] : "all";
  int ran = 0;
  for (auto& c : mini::registry()) {
    if (want != "all" && c.group.rfind(want, 0) != 0) continue;
    const int before = mini::failures();
    std::printf("[ RUN  ] %s.%s\n", c.group.c_str(), c.name.c_str());
    try {
      c.fn();
    } catch (const std::exception& e) {
      mini::fail(__FILE__, __LINE__, std::string("uncaught exception: ") + e.what());
    }
    std::printf("[ %s ] %s.%s\n", mini::failures() == before ? " OK " : "FAIL", c.group.c_str(), c.name.c_str());
    ++ran;
  }
  std::printf("%d cases, %d failures\n", ran, mini::failures());
  return mini::failures() == 0 && ran > 0 ? 0 : 1;
}
