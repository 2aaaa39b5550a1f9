// Host-side check of the tensor-core engine's index arithmetic
// (mlx-cross-entropy_b200/csrc/schedule.cuh), built and run by
// tests/test_schedule_cpu.py with nvcc on the CPU:
//   * Sched::coords maps the unit ids 0 .. units()-1 one-to-one onto
//     (mb, nb, ks) for every raster (M- or N-fast, grouped or not) and split;
//   * Sched::krange cuts [0, num_kb) into splits() consecutive ranges;
//   * MaskView::next / field give the same answers over the bit copy and the
//     byte mask, and agree with a direct scan.
// Prints "SCHEDULE_OK" and exits 0, or prints the first mismatch and exits 1.
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <vector>

#include "schedule.cuh"

using cce::tc::MaskView;
using cce::tc::Sched;

static uint64_t rng_state = 0x9E3779B97F4A7C15ull;
static uint32_t rnd(uint32_t n) {
  rng_state ^= rng_state << 13;
  rng_state ^= rng_state >> 7;
  rng_state ^= rng_state << 17;
  return (uint32_t)(rng_state % n);
}

static int fail(const char* what, int a, int b, int c) {
  std::printf("MISMATCH %s (%d, %d, %d)\n", what, a, b, c);
  return 1;
}

int main() {
  for (int it = 0; it < 3000; ++it) {
    Sched s{};
    s.num_m = 1 + (int)rnd(40);
    s.num_n = 1 + (int)rnd(40);
    s.num_kb = (int)rnd(300);
    s.m_fast = (int)rnd(2);
    s.group = rnd(3) == 0 ? 0 : 1 + (int)rnd(20);
    s.ksplit = (int)rnd(4);
    std::vector<int> seen((size_t)s.units(), 0);
    for (int u = 0; u < s.units(); ++u) {
      int mb, nb, ks;
      s.coords(u, mb, nb, ks);
      if (mb < 0 || mb >= s.num_m || nb < 0 || nb >= s.num_n || ks < 0 || ks >= s.splits())
        return fail("coords range", u, mb, nb);
      int& slot = seen[((size_t)ks * s.num_m + mb) * s.num_n + nb];
      if (slot++) return fail("coords duplicate", u, mb, nb);
    }
    int expect = 0;
    for (int ks = 0; ks < s.splits(); ++ks) {
      int kb0, kb1;
      s.krange(ks, kb0, kb1);
      if (kb0 != expect || kb1 < kb0 || kb1 > s.num_kb) return fail("krange", ks, kb0, kb1);
      expect = kb1;
    }
    if (expect != s.num_kb) return fail("krange cover", expect, s.num_kb, 0);
  }
  for (int it = 0; it < 2000; ++it) {
    const int rows = 1 + (int)rnd(8), cols = 1 + (int)rnd(300);
    const int wpr = (cols + 31) / 32;
    const int density = (int)rnd(10);  // 0: empty rows, 9: dense rows
    std::vector<uint8_t> bytes((size_t)rows * cols);
    std::vector<uint32_t> bits((size_t)rows * wpr, 0u);
    for (int r = 0; r < rows; ++r)
      for (int c = 0; c < cols; ++c) {
        const uint8_t v = (int)rnd(10) < density ? 1 : 0;
        bytes[(size_t)r * cols + c] = v;
        if (v) bits[(size_t)r * wpr + c / 32] |= 1u << (c % 32);
      }
    MaskView vb{bits.data(), nullptr, 0, wpr, cols};
    MaskView vy{nullptr, bytes.data(), cols, 0, cols};
    for (int q = 0; q < 50; ++q) {
      const int r = (int)rnd(rows);
      const int c = (int)rnd(cols + 1);
      const int c1 = c + (int)rnd(cols + 1 - c);
      int ref = c1;
      for (int k = c; k < c1; ++k)
        if (bytes[(size_t)r * cols + k]) { ref = k; break; }
      if (vb.next(r, c, c1) != ref) return fail("next(bits)", r, c, c1);
      if (vy.next(r, c, c1) != ref) return fail("next(bytes)", r, c, c1);
      const int n = 1 << (int)rnd(6);  // 1 .. 32
      const int cf = (int)rnd((cols + n - 1) / n) * n;
      uint32_t fref = 0;
      for (int i = 0; i < n && cf + i < cols; ++i)
        if (bytes[(size_t)r * cols + cf + i]) fref |= 1u << i;
      if (vb.field(r, cf, n) != fref) return fail("field(bits)", r, cf, n);
      if (vy.field(r, cf, n) != fref) return fail("field(bytes)", r, cf, n);
    }
  }
  std::printf("SCHEDULE_OK\n");
  return 0;
}
