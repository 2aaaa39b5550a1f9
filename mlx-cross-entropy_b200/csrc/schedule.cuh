// Work-unit schedule and filter-mask view of the tensor-core engine
// (tc_kernels.cu), kept host-callable so that tests/sched_check.cu can check
// the index arithmetic on the CPU.
#pragma once

#include <cstdint>

namespace cce {
namespace tc {

// 1-based index of the lowest set bit (0 for 0), on the device and the host.
__host__ __device__ __forceinline__ int ffs32(uint32_t x) {
#ifdef __CUDA_ARCH__
  return __ffs(x);
#else
  return __builtin_ffs((int)x);
#endif
}

struct Sched {
  int num_m, num_n, num_kb;
  int m_fast;    // consecutive tile ids walk M first (1) or N first (0)
  int a3d, b3d;  // MN-major operand loaded as one 3-D box (else one 2-D box per 64 columns)
  int* counter;  // dynamic scheduling: next tile id (zeroed before the launch); nullptr = static
  int group;     // grouped raster: blocks of the fast dimension per group (<= 0: all)
  int ksplit;    // K splits per output tile (<= 1: none); split s is its own work unit
  int span;      // K-major B: one MMA over the span of a tile's kept column groups
  const int* list;        // claims index this list of unit ids (nullptr: claim = unit id)
  const int* list_count;  // its length, read at the kernel's start
  __host__ __device__ __forceinline__ int splits() const { return ksplit > 1 ? ksplit : 1; }
  __host__ __device__ __forceinline__ int units() const { return num_m * num_n * splits(); }
  // Unit id -> (mb, nb, ks).  All units of split 0 come first, then split 1, ...
  // Within a split, ids walk the fast dimension inside groups of `group`
  // blocks, then the slow dimension, then the next group: the ~148 tiles in
  // flight cover group x (148 / group) blocks, so both operand panels of the
  // window stay in L2 even when one operand as a whole does not.
  __host__ __device__ __forceinline__ void coords(int unit, int& mb, int& nb, int& ks) const {
    const int per_split = num_m * num_n;
    ks = unit / per_split;
    const int tile = unit - ks * per_split;
    const int fast = m_fast ? num_m : num_n;
    const int slow = m_fast ? num_n : num_m;
    const int gsz0 = (group > 0 && group < fast) ? group : fast;
    const int per_group = gsz0 * slow;
    const int g = tile / per_group;
    const int r = tile - g * per_group;
    const int gsz = gsz0 < fast - g * gsz0 ? gsz0 : fast - g * gsz0;
    const int f = g * gsz0 + r % gsz;
    const int sl = r / gsz;
    if (m_fast) {
      mb = f;
      nb = sl;
    } else {
      nb = f;
      mb = sl;
    }
  }
  // K-blocks [kb0, kb1) of split ks.
  __host__ __device__ __forceinline__ void krange(int ks, int& kb0, int& kb1) const {
    const int per = (num_kb + splits() - 1) / splits();
    kb0 = ks * per < num_kb ? ks * per : num_kb;
    kb1 = kb0 + per < num_kb ? kb0 + per : num_kb;
  }
};

// Fast-dimension group size: all blocks when that operand fits comfortably in
// L2 (it is then read from DRAM once however the tiles are ordered), else 16.
__host__ __device__ inline int raster_group(int64_t fast_operand_bytes) {
  return fast_operand_bytes <= (40ll << 20) ? 0 : 16;
}

// Read-only view of a vocabulary chunk's filter-mask slice [row block][stat
// tile]: bits in shared memory (row-aligned 32-bit words, `wpr` per row) when
// they fit, else the bytes in global memory (row stride `ld`).
struct MaskView {
  const uint32_t* bits;  // row-aligned words (zero past `cols`), shared or global memory
  const uint8_t* bytes;
  int64_t ld;
  int wpr;
  int cols;
  // Bits [c, c + n) of row r (n <= 32 divides 32, c a multiple of n).
  __host__ __device__ __forceinline__ uint32_t field(int r, int c, int n) const {
    const uint32_t lo = n == 32 ? 0xffffffffu : (1u << n) - 1u;
    if (bits) return (bits[r * wpr + (c >> 5)] >> (c & 31)) & lo;
    uint32_t m = 0;
    for (int i = 0; i < n && c + i < cols; ++i) m |= (bytes[(int64_t)r * ld + c + i] != 0 ? 1u : 0u) << i;
    return m;
  }
  // First set column of row r in [c, c1), else c1.
  __host__ __device__ __forceinline__ int next(int r, int c, int c1) const {
    if (bits) {
      const uint32_t* row = bits + r * wpr;
      while (c < c1) {
        const uint32_t w = row[c >> 5] >> (c & 31);
        if (w) {
          c += ffs32(w) - 1;
          return c < c1 ? c : c1;
        }
        c = (c | 31) + 1;
      }
      return c1;
    }
    for (; c < c1; ++c)
      if (bytes[(int64_t)r * ld + c]) return c;
    return c1;
  }
};

}  // namespace tc
}  // namespace cce
