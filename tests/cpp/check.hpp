// Minimal test harness for the C++ API tests (same shape as pkt's
// tests/test_utils.cuh: named cases, a pass/fail summary, non-zero exit on failure).
// Device tests FAIL when no CUDA device is present (pkt's returned "pass").
#pragma once

#include <cmath>
#include <cstdio>
#include <cstdlib>

#define CHECK(cond, msg)                                                      \
  do {                                                                        \
    if (!(cond)) {                                                            \
      std::fprintf(stderr, "CHECK failed %s:%d: %s\n", __FILE__, __LINE__, msg); \
      return false;                                                           \
    }                                                                         \
  } while (0)

struct Case {
  const char* name;
  bool (*fn)();
};

inline int run_cases(const Case* cs, int n) {
  int failed = 0;
  for (int i = 0; i < n; ++i) {
    const bool ok = cs[i].fn();
    std::printf("[%d/%d] %s %s\n", i + 1, n, cs[i].name, ok ? "PASSED" : "FAILED");
    failed += ok ? 0 : 1;
  }
  std::printf("Results: %d passed, %d failed\n", n - failed, failed);
  return failed ? 1 : 0;
}
