// Host check of the launch-constant division of the GEMM tile schedules
// (FastDiv / fdiv in open-pacho_b200/csrc/pb_internal.cuh): the same
// multiply-high formula the kernels run, compared with plain division on
// boundary and random operands.  Built and run by tests/test_fastdiv.py.
#include <cstdint>
#include <cstdio>
#include <random>
#include <vector>

#include "pb_internal.cuh"

int main() {
  std::mt19937_64 rng(7);
  long long bad = 0, checked = 0;
  auto check = [&](int64_t n, const pb::FastDiv& f) {
    ++checked;
    if (pb::fdiv(n, f) != n / f.d && bad++ < 10)
      std::printf("mismatch: n=%lld d=%lld got %lld\n", (long long)n, (long long)f.d,
                  (long long)pb::fdiv(n, f));
  };
  const int64_t top = (int64_t(1) << 31) - 1;
  std::vector<int64_t> ds;
  for (int64_t d = 1; d <= 4096; ++d) ds.push_back(d);
  for (int k = 1; k <= 31; ++k)
    for (int e = -1; e <= 1; ++e) ds.push_back((int64_t(1) << k) + e);
  ds.push_back(int64_t(1) << 31);
  for (int i = 0; i < 20000; ++i) ds.push_back(1 + (int64_t)(rng() % (uint64_t(1) << 31)));
  ds.push_back(3000000000ll);  // above 2^31: plain division
  ds.push_back(int64_t(1) << 40);
  for (const int64_t d : ds) {
    const pb::FastDiv f = pb::make_fastdiv(d);
    const int64_t edge[] = {0, 1, d - 1, d, d + 1, 2 * d - 1, 2 * d, top, top - 1, top - d,
                            top / d * d, top / d * d - 1, top + 1, (int64_t(1) << 40) + 12345};
    for (const int64_t n : edge)
      if (n >= 0) check(n, f);
    for (int i = 0; i < 64; ++i) check((int64_t)(rng() % (uint64_t(1) << 31)), f);
    for (int i = 0; i < 8; ++i) check((int64_t)(rng() >> 2), f);
  }
  std::printf("checked %lld, mismatches %lld\n", checked, bad);
  return bad != 0;
}
