// tcgen05 / TMEM / TMA kernels for 16-bit inputs (the hot path).
//
// One persistent, warp-specialised GEMM engine drives four epilogues:
//
//   K1 forward : S = e @ c^T per (128-row, 256-column) tile; the epilogue adds
//                the bias, picks the target logit, writes each row's max over
//                every 32-column statistics tile (the backward filter's input)
//                and one online (max, sum-exp) pair per row for the whole tile
//                (the LSE partial).  Replaces the tile kernel of
//                csrc/cce/cce.metal:19-135 (which does the same per 32x32 tile
//                on 8x8 simdgroup MMAs).
//   K4 dlogits : the same S for one vocabulary chunk, then
//                w = d_nll * (exp(S + b - lse) - [v == t]) stored as bf16
//                (cce.metal:274-282), with blocks the filter rejects
//                (cce.metal:190-204) never computed; grad_bias column sums.
//   K5 grad_e  : grad_e[N, D] (+)= w[N, chunk] @ c[chunk, D]   (cce.metal:284-291)
//   K6 grad_c  : grad_c[chunk, D] = w^T @ e                    (cce.metal:292-304,
//                reference/_fused_backward.py:1549-1567)
//
// Engine: 192 threads, one CTA per SM, grid = min(#work units, #SMs).  Warp 0
// lane 0 takes work units (a tile, or a tile's K range for grad_e) from a
// static round-robin schedule (forward) or a global atomic counter (backward)
// and issues the TMA loads of the A and B K-slices (64 elements = one 128-byte
// swizzle row) into a 4-stage ring, skipping the K-blocks the filter rejects;
// warp 1 lane 0 issues tcgen05.mma (M=128, N=256 or fewer, K=16) into one of
// two 256-column fp32 TMEM accumulators and commits stage / accumulator
// barriers; warps 2-5 read the accumulator with tcgen05.ld (one TMEM lane =
// one output row per thread) and run the epilogue, which leaves through TMA
// box stores, while the next tile's MMAs proceed.
//
// An epilogue type supplies: kMask (reads a filter-mask slice) and, if so,
// kMaskBits (the slice is already a bit table) with mask_src / mask_ld /
// mask_rows / mask_cols; tile_active, next_kb and ksub_mask (which tiles,
// K-blocks and K=16 steps run); col_mask (the column groups the MMA computes,
// K-major B only); chunk_live (which 32-column chunks the epilogue reads from
// TMEM); begin / chunk / end (per tile, per 32-column chunk, per tile end).
#include <cuda.h>

#include <atomic>
#include <cstdlib>
#include <type_traits>

#include "kernels.cuh"
#include "schedule.cuh"
#include "tc_ptx.cuh"

namespace cce {
namespace tc {
namespace {

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int BK = 64;
constexpr int STAGES = 4;
constexpr int kThreads = 192;
constexpr uint32_t A_BYTES = BM * BK * 2;   // 16 KB
constexpr uint32_t B_BYTES = BN * BK * 2;   // 32 KB
constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;
constexpr uint32_t BOX_MN_BYTES = 64 * BK * 2;  // one 64 x 64 MN-major box (8 KB)
constexpr uint32_t TMEM_COLS = 512;
constexpr int RING = 4;                          // depth of the tile-id ring
// Statistics tiles (kStatTile vocabulary columns each, the filter's column
// granularity) per engine tile and per K-block.
constexpr int kGroups = BN / kStatTile;                // per 256-column output tile
constexpr uint32_t kAllGroups = (1u << kGroups) - 1u;
constexpr int kChunksPerStat = kStatTile / 32;         // epilogue 32-column chunks per statistics tile
constexpr int kStatsPerM = BM / kStatTile;             // per 128-row M tile (grad_c)
constexpr int kStepsPerStat = kStatTile / 16;          // K=16 MMA steps per statistics tile (grad_e)
static_assert(kStatTile % 32 == 0 && BK % kStatTile == 0 && kGroups <= 32, "statistics-tile layout");
static_assert(BN == kTcLseTile, "one LSE partial per output tile");
constexpr uint32_t SMASK_BYTES = 16384;   // shared copy of the chunk's filter-mask slice (bits)
constexpr uint32_t OUT_STAGE_BYTES = 4 * 4096;  // epilogue output staging, 4 KB per epilogue warp
constexpr size_t SMEM_BYTES = 1024 + STAGES * (size_t)STAGE_BYTES + OUT_STAGE_BYTES + 256 + SMASK_BYTES;
constexpr int kPushWaitCode = 8;  // status code: a push unit's epilogue threads never all arrived
// K-major B loaded as 32-row boxes (B32_BYTES each) when a tile's live column
// groups are one run of at most this many groups (kNarrowB epilogues): a box
// costs on its own, so longer runs load the whole tile in one box.
constexpr uint32_t kNarrowMaxGroups = 2;
constexpr uint32_t B32_BYTES = kStatTile * BK * 2;  // 4 KB: 32 rows x 128 bytes
// Narrow tiles two K-blocks per stage (kNarrowB epilogues with `dbl` set):
// the stage's A slot holds A(kb); its B slot holds A(kb + 1) in the first
// A_BYTES, then the live B rows of kb and of kb + 1, kNarrowMaxGroups boxes
// each -- half the load round trips of a tile that fills a third of a stage.
constexpr uint32_t kDblB0 = A_BYTES;                                 // B(kb) in the B slot
constexpr uint32_t kDblB1 = A_BYTES + kNarrowMaxGroups * B32_BYTES;  // B(kb + 1)
static_assert(kDblB1 + kNarrowMaxGroups * B32_BYTES <= B_BYTES, "two narrow K-blocks per stage");

// The single run of kept column groups [j, j + n) of a tile's column mask cm
// whose B rows are loaded alone (n <= kNarrowMaxGroups); false for a full or
// empty mask or more than one run.
__device__ __forceinline__ bool narrow_run(uint32_t cm, uint32_t& j, uint32_t& n) {
  if (cm == kAllGroups || cm == 0u) return false;
  j = __ffs(cm) - 1;
  n = __ffs(~(cm >> j)) - 1;
  return (cm >> (j + n)) == 0u && n <= kNarrowMaxGroups;
}
// Half K-blocks (kHalfK epilogues): a K-block whose only kept statistics tile
// is one of its two 32-row halves loads that half alone -- A as a 128 x 32
// box in the 64-byte swizzle (SW64 K-major), B as a 3-D box of 32 K-rows x
// 256 columns (four 4 KB slabs) -- into the first half of the stage.
constexpr uint32_t A_HALF_BYTES = BM * (BK / 2) * 2;  // 8 KB
constexpr uint32_t B_HALF_BYTES = BN * (BK / 2) * 2;  // 16 KB
constexpr uint32_t BOX_MN_HALF_BYTES = 64 * (BK / 2) * 2;  // one 64-column slab of a half box (4 KB)
static_assert(BK / 2 == kStatTile, "a half K-block is one statistics tile");

// Executed tensor-core work per kernel kind (0 forward, 1 dlogits, 2 grad_e,
// 3 grad_c): the sum of N over every issued M = 128, K = 16 MMA, added once
// per CTA; FLOPs = 2 * 128 * 16 * sum.  Read by cce_mma_flops().
__device__ unsigned long long g_mma_cols[4];

// ---------------------------------------------------------------------------
// helpers for the epilogues
// ---------------------------------------------------------------------------

// 32 bias values for columns [col0, col0 + 32), zero past `limit`.
template <typename TB>
__device__ __forceinline__ void load_bias32(const void* bias, int64_t col0, int64_t limit, float (&b)[32]) {
  const TB* p = reinterpret_cast<const TB*>(bias);
#pragma unroll
  for (int j = 0; j < 32; ++j) b[j] = (col0 + j < limit) ? to_f32(__ldg(p + col0 + j)) : 0.f;
}

// Sum each of 32 per-lane values across the warp's 32 lanes; afterwards lane
// j holds the total of value j (recursive-halving transpose-reduce, 31 shuffles).
__device__ __forceinline__ float warp_transpose_sum32(float (&v)[32]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int w = 16; w >= 1; w >>= 1) {
    const bool upper = (lane & w) != 0;
#pragma unroll
    for (int i = 0; i < w; ++i) {
      const float send = upper ? v[i] : v[i + w];
      const float keep = upper ? v[i + w] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, w);
    }
  }
  return v[0];
}

// Output staging of one epilogue warp: two 2 KB slots, each 32 rows x 64 bytes
// in the TMA 64-byte swizzle (16-byte unit u of row r sits at unit
// u ^ ((r >> 1) & 3), so a warp's 16-byte stores are free of bank conflicts).
// A filled slot goes to global memory as one TMA box store (or reduce-add)
// issued by lane 0, which also owns the bulk groups and their waits; the
// tensor map clips rows and columns past the output's extent.
struct Stager {
  const CUtensorMap* tm;
  uint8_t* buf;  // this warp's 4 KB (1 KB aligned)
  int slot;      // next slot of a 16-bit store

  __device__ __forceinline__ uint4* unit(int sl, int u) const {
    const int lane = threadIdx.x & 31;
    return reinterpret_cast<uint4*>(buf + sl * 2048 + lane * 64 + ((u ^ ((lane >> 1) & 3)) << 4));
  }
  // All lanes' shared-memory writes become visible to the TMA unit.
  __device__ __forceinline__ void publish() const {
    fence_proxy_async();
    __syncwarp();
  }
  // Slot reuse: wait until at most `N` committed groups still read shared memory.
  template <int N>
  __device__ __forceinline__ void acquire() const {
    if ((threadIdx.x & 31) == 0) bulk_wait_read<N>();
    __syncwarp();
  }
  __device__ __forceinline__ void drain() const {
    if ((threadIdx.x & 31) == 0) bulk_wait_all();
    __syncwarp();
  }

  // 32 values of this lane's row -> one 32 x 32 box of 16-bit T at (x, y).
  template <typename T>
  __device__ __forceinline__ void store16(const float (&v)[32], int x, int y) {
    acquire<1>();  // the slot's previous box (two stores back) has been read
    uint32_t w[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      T lo = from_f32<T>(v[2 * i]), hi = from_f32<T>(v[2 * i + 1]);
      w[i] = (uint32_t)(*reinterpret_cast<uint16_t*>(&lo)) | ((uint32_t)(*reinterpret_cast<uint16_t*>(&hi)) << 16);
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) *unit(slot, u) = make_uint4(w[4 * u], w[4 * u + 1], w[4 * u + 2], w[4 * u + 3]);
    publish();
    if ((threadIdx.x & 31) == 0) {
      tma_store_2d(tm, smem_u32(buf + slot * 2048), x, y);
      bulk_commit();
    }
    slot ^= 1;
  }

  // 32 fp32 values of this lane's row -> two 16 x 32 x 1 boxes at (x, y, z)
  // and (x + 16, y, z) of a 3-D map, stored or added to global memory.
  __device__ __forceinline__ void store_f32(const float (&v)[32], int x, int y, int z, bool add) {
    acquire<0>();
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
      for (int u = 0; u < 4; ++u)
        *unit(h, u) = make_uint4(__float_as_uint(v[16 * h + 4 * u]), __float_as_uint(v[16 * h + 4 * u + 1]),
                                 __float_as_uint(v[16 * h + 4 * u + 2]), __float_as_uint(v[16 * h + 4 * u + 3]));
    publish();
    if ((threadIdx.x & 31) == 0) {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        if (add) tma_reduce_add_3d(tm, smem_u32(buf + h * 2048), x + 16 * h, y, z);
        else tma_store_3d(tm, smem_u32(buf + h * 2048), x + 16 * h, y, z);
      }
      bulk_commit();
    }
  }
};

// ---------------------------------------------------------------------------
// K1: forward tile statistics
// ---------------------------------------------------------------------------

template <typename TB>  // bias element type; void = no bias
struct FwdEpi {
  static constexpr bool kNarrowB = false;  // B rows loaded for a tile's live column run only
  static constexpr bool kPairLd = false;  // the epilogue reads TMEM two 32-column chunks at a time
  __device__ __forceinline__ bool pair_ld() const { return false; }
  static constexpr bool kHalfK = false;  // half K-blocks loaded alone (see A_HALF_BYTES)
  static constexpr bool kWideCapable = false;  // may run as wide units (see GradEEpi)
  static constexpr int kKind = 0;  // slot in g_mma_cols
  const int32_t* targets;
  const void* bias;
  float* tile_max;  // [ceil(V / kStatTile)][N]
  float* part_m;    // [ceil(V / BN)][N]
  float* part_s;
  float* tgt;
  int64_t N, V, v_offset;

  struct State {
    int64_t row, tl, col0;
    float m, s;  // online max / sum-exp over the whole tile (the LSE partial)
    float mt;    // max over the current statistics tile
  };

  static constexpr bool kMask = false;
  static constexpr bool kZeroTiles = false;
  __device__ __forceinline__ bool tile_active(const MaskView&, int, int) const { return true; }
  __device__ __forceinline__ bool skip_unit(const MaskView&, int, int, int, int) const { return false; }
  __device__ __forceinline__ uint32_t col_mask(const MaskView&, int, int) const { return kAllGroups; }
  __device__ __forceinline__ int next_kb(const MaskView&, int, int, int kb, int) const { return kb; }
  __device__ __forceinline__ uint32_t ksub_mask(const MaskView&, int, int, int) const { return 0xFu; }
  __device__ __forceinline__ void inactive_tile(int, int, int) const {}
  template <class S>
  __device__ __forceinline__ bool chunk_live(const S&, int) const { return true; }

  __device__ __forceinline__ void begin(State& st, const MaskView&, int mb, int nb, int r, int) const {
    st.row = (int64_t)mb * BM + r;
    st.tl = st.row < N ? (int64_t)targets[st.row] - v_offset : -1;
    st.col0 = (int64_t)nb * BN;
    st.m = -INFINITY;
    st.s = 0.f;
    st.mt = -INFINITY;
  }

  __device__ __forceinline__ void chunk(State& st, int c, float (&v)[32], Stager& sg) const {
    const int64_t cb = st.col0 + c * 32;
    float b[32];
    if constexpr (!std::is_void<TB>::value) {
      load_bias32<TB>(bias, cb, V, b);
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j) b[j] = 0.f;
    }
    float mc = -INFINITY;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      v[j] = (cb + j < V) ? v[j] + b[j] : -INFINITY;
      mc = fmaxf(mc, v[j]);
      if (cb + j == st.tl && cb + j < V) tgt[st.row] = v[j];
    }
    const float nm = fmaxf(st.m, mc);
    if (nm != -INFINITY) {
      const float nml = nm * kLog2e;
      float acc = 0.f;
#pragma unroll
      for (int j = 0; j < 32; ++j) acc += exp2f(fmaf(v[j], kLog2e, -nml));
      st.s = st.s * exp2f(fmaf(st.m, kLog2e, -nml)) + acc;
      st.m = nm;
    }
    st.mt = fmaxf(st.mt, mc);
    if ((c + 1) % kChunksPerStat == 0) {  // end of a statistics tile
      const int h = c / kChunksPerStat;
      if (st.row < N && st.col0 + h * kStatTile < V) tile_max[(st.col0 / kStatTile + h) * N + st.row] = st.mt;
      st.mt = -INFINITY;
    }
  }

  __device__ __forceinline__ void end(State& st) const {
    if (st.row < N && st.col0 < V) {
      const int64_t idx = (st.col0 / BN) * N + st.row;
      part_m[idx] = st.m;
      part_s[idx] = st.s;
    }
  }
  __device__ __forceinline__ void after_unit(uint64_t*, uint32_t&) const {}
};

// ---------------------------------------------------------------------------
// K4: dlogits of one vocabulary chunk
// ---------------------------------------------------------------------------

template <typename T, typename TB>
struct DlogitsEpi {
  static constexpr bool kNarrowB = true;  // B rows loaded for a tile's live column run only
  static constexpr bool kPairLd = false;  // the epilogue reads TMEM two 32-column chunks at a time
  __device__ __forceinline__ bool pair_ld() const { return false; }
  static constexpr bool kHalfK = false;  // half K-blocks loaded alone (see A_HALF_BYTES)
  static constexpr bool kWideCapable = false;  // may run as wide units (see GradEEpi)
  static constexpr int kKind = 1;  // slot in g_mma_cols
  const int32_t* targets;
  const float* lse;
  const float* d_nll;
  const void* bias;
  T* dl;                // [N][ld], column 0 = local vocab row vc0
  float* grad_bias;     // [V] or nullptr
  const float* scale;   // fp16: {s, 1/s}, dl holds w / s; nullptr = unscaled (bf16)
  const void* mask_src;     // keep + vc0 / kStatTile: the chunk's columns of the [nRb][nVt] byte mask
  int64_t mask_ld;          // nVt
  int mask_rows, mask_cols; // nRb, statistics tiles in the chunk
  int64_t N, V, v_offset, vc0, vc_end, ld;
  int dbl = 0;     // narrow tiles load two K-blocks per stage (kDblB0)

  struct State {
    int64_t row, tl, col0;
    float g, L, s;   // g = d_nll / s
    uint32_t kmask;  // kept statistics-tile column groups of the tile
    int y0;          // first row of this warp's 32-row slab
  };

  // The tile's kGroups column groups are the chunk's statistics tiles kGroups nb + g.
  static constexpr bool kMask = true;
  static constexpr bool kZeroTiles = false;
  // Kept column groups of the tile (bit g = chunk statistics tile kGroups nb + g).
  __device__ __forceinline__ uint32_t group_mask(const MaskView& mk, int mb, int nb) const {
    return mb < mask_rows ? mk.field(mb, kGroups * nb, kGroups) : 0u;
  }
  __device__ __forceinline__ bool tile_active(const MaskView& mk, int mb, int nb) const {
    return group_mask(mk, mb, nb) != 0;
  }
  // Tiles without a kept block produce nothing: the producer passes them over.
  __device__ __forceinline__ bool skip_unit(const MaskView& mk, int mb, int nb, int, int) const {
    return !tile_active(mk, mb, nb);
  }
  // Column groups the MMA computes: only the kept ones (the epilogue never
  // reads the accumulator columns of the others).
  __device__ __forceinline__ uint32_t col_mask(const MaskView& mk, int mb, int nb) const {
    return group_mask(mk, mb, nb);
  }
  __device__ __forceinline__ bool chunk_live(const State& st, int c) const {
    return (st.kmask >> (c / kChunksPerStat)) & 1u;
  }
  static constexpr bool kMaskBits = false;
  __device__ __forceinline__ int next_kb(const MaskView&, int, int, int kb, int) const { return kb; }
  __device__ __forceinline__ uint32_t ksub_mask(const MaskView&, int, int, int) const { return 0xFu; }

  // Rejected tiles are not written: the grad GEMMs skip exactly those blocks.
  __device__ __forceinline__ void inactive_tile(int, int, int) const {}

  __device__ __forceinline__ void begin(State& st, const MaskView& mk, int mb, int nb, int r, int) const {
    st.row = (int64_t)mb * BM + r;
    st.col0 = vc0 + (int64_t)nb * BN;  // local vocab id of the tile's column 0
    const bool ok = st.row < N;
    st.s = scale ? scale[0] : 1.f;
    st.g = ok ? d_nll[st.row] * (scale ? scale[1] : 1.f) : 0.f;
    st.L = ok ? lse[st.row] : 0.f;
    st.tl = ok ? (int64_t)targets[st.row] - v_offset : -1;
    st.kmask = group_mask(mk, mb, nb);
    st.y0 = (int)(st.row - (threadIdx.x & 31));
  }

  __device__ __forceinline__ void chunk(State& st, int c, float (&v)[32], Stager& sg) const {
    const int64_t cb = st.col0 + c * 32;
    const bool kept = (st.kmask >> (c / kChunksPerStat)) & 1u;
    float b[32];
    if constexpr (!std::is_void<TB>::value) {
      load_bias32<TB>(bias, cb, vc_end, b);
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j) b[j] = 0.f;
    }
    const float Ll = st.L * kLog2e;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      float w = 0.f;
      if (kept && cb + j < vc_end) {
        w = st.g * exp2f(fmaf(v[j] + b[j], kLog2e, -Ll));
        if (cb + j == st.tl) w -= st.g;
      }
      v[j] = w;
    }
    // grad_c multiplies whole 128-column quarters (its M tiles): a quarter
    // with a kept group is stored whole (zeros in the others), the rest never
    // read; grad_e reads kept groups only.
    if ((st.kmask >> (kStatsPerM * (c >> 2))) & ((1u << kStatsPerM) - 1u))
      sg.store16<T>(v, (int)(cb - vc0), st.y0);
    // (kept is the same for the whole warp: a rejected group is all zeros)
    if (grad_bias != nullptr && kept) {
      const int lane = threadIdx.x & 31;
      const float colsum = warp_transpose_sum32(v);
      if (cb + lane < vc_end && colsum != 0.f) atomicAdd(grad_bias + cb + lane, colsum * st.s);
    }
  }

  __device__ __forceinline__ void end(State&) const {}
  __device__ __forceinline__ void after_unit(uint64_t*, uint32_t&) const {}
};

// ---------------------------------------------------------------------------
// K5: grad_e accumulation
// ---------------------------------------------------------------------------

// Each output tile's K range (the chunk's vocabulary rows) is split in two
// work units; split s adds into fp32 accumulator slab s of acc[2][N][D] (a TMA
// store in the first chunk, a TMA reduce-add after it), so every slab has one
// writer per chunk and the sums are deterministic.  The caller adds the two
// slabs into grad_e after the last chunk.
//
// Push mode (the last chunk of a vocabulary-sharded backward): a unit's result
// plus its slab's earlier chunks is stored straight into the receive slot
// (this rank, split) of the rank that owns its rows (peer.cuh), with plain
// 16-byte stores over NVLink while the MMAs of the next units run; the last
// unit raises the `pushed` flag on every rank.  The slabs are not written.
struct GradEEpi {
  static constexpr bool kNarrowB = false;  // B rows loaded for a tile's live column run only
  static constexpr bool kPairLd = false;  // the epilogue reads TMEM two 32-column chunks at a time
  __device__ __forceinline__ bool pair_ld() const { return false; }
  static constexpr bool kHalfK = true;  // half K-blocks loaded alone when half_k is set
  static constexpr bool kWideCapable = true;  // may run as wide units (see GradEEpi)
  static constexpr int kKind = 2;  // slot in g_mma_cols
  const float* scale;       // fp16: {s, 1/s}, the products are multiplied by s; else nullptr
  const void* mask_src;     // keep + vc0 / kStatTile: the chunk's columns of the [nRb][nVt] byte mask
  int64_t mask_ld;          // nVt
  int mask_rows, mask_cols; // nRb, statistics tiles in the chunk
  int accumulate;
  float* acc2;              // [2][N][D]: zero tiles of the first chunk are stored directly
  int64_t N, D;
  int push;                 // push mode (then the fields below are set)
  unsigned total_units;     // work units of the launch
  peer::Peers peers;
  peer::Layout layout;
  int half_k;               // the half-K maps are valid: load half K-blocks alone
  // Wide units: a unit is an output tile pair (nb = 2 np, 2 np + 1) of one
  // K range, accumulated in both 256-column TMEM accumulators at once from
  // one A stage, K stepping by statistics tile (32 rows: a 128 x 32 A box,
  // a 32 x 512 B box).  Each unit loads A once for 512 output columns, which
  // halves the A strips the ~148 units in flight stream from DRAM; the price
  // is no overlap of a unit's epilogue with the next unit's MMAs.
  int wide;

  struct State {
    int64_t col0;
    float s;
    int y0;  // first row of this warp's 32-row slab
    int ks;  // accumulator slab
  };
  // A work unit no K-block reached adds zeros: nothing to do after the first
  // chunk; in the first chunk its slab rows are zeroed (lane l: 8 columns).
  __device__ __forceinline__ void zero_tile(const State& st) const {
    if (accumulate) return;
    const int64_t c0 = st.col0 + 8 * (threadIdx.x & 31);
    if (c0 >= D) return;
    float* base = acc2 + (int64_t)st.ks * N * D + c0;
    for (int i = 0; i < 32 && (int64_t)st.y0 + i < N; ++i) {
      float4* dst = reinterpret_cast<float4*>(base + ((int64_t)st.y0 + i) * D);
      dst[0] = make_float4(0.f, 0.f, 0.f, 0.f);
      dst[1] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
  // K runs over the chunk's vocabulary rows: K-block kb (64 rows) holds the
  // chunk's statistics tiles BK / kStatTile * kb + i; the MMA skips the K=16
  // steps of the rejected ones.
  static constexpr bool kMask = true;
  static constexpr bool kZeroTiles = true;
  __device__ __forceinline__ bool tile_active(const MaskView&, int, int) const { return true; }
  static constexpr bool kMaskBits = false;
  static constexpr int kSpk = BK / kStatTile;  // statistics tiles per K-block
  // K=16 steps of K-block kb whose statistics tile the filter keeps (kb active).
  __device__ __forceinline__ uint32_t ksub_mask(const MaskView& mk, int mb, int, int kb) const {
    const uint32_t f = mk.field(mb, kSpk * kb, kSpk);
    uint32_t m = 0;
#pragma unroll
    for (int i = 0; i < kSpk; ++i)
      if ((f >> i) & 1u) m |= ((1u << kStepsPerStat) - 1u) << (i * kStepsPerStat);
    return m;
  }
  // First K-block in [kb, kb1) with a kept statistics tile in row block mb, else kb1.
  // (Wide units step by statistics tile: kb is a statistics-tile index.)
  __device__ __forceinline__ int next_kb(const MaskView& mk, int mb, int, int kb, int kb1) const {
    if (mb >= mask_rows) return kb1;
    if (wide) {
      const int lim = min(kb1, mask_cols);
      const int t = mk.next(mb, kb, lim);
      return t < lim ? t : kb1;
    }
    const int lim = min(kSpk * kb1, mask_cols);
    const int t = mk.next(mb, kSpk * kb, lim);
    return t < lim ? t / kSpk : kb1;
  }
  // A unit no K-block reaches adds zeros to the slab after the first chunk:
  // nothing to do, so the producer passes it over (not in push mode, where
  // every unit sends its slab, nor in the first chunk, which zeroes it).
  __device__ __forceinline__ bool skip_unit(const MaskView& mk, int mb, int nb, int kb0, int kb1) const {
    return accumulate && !push && next_kb(mk, mb, nb, kb0, kb1) >= kb1;
  }
  __device__ __forceinline__ void inactive_tile(int, int, int) const {}
  template <class S>
  __device__ __forceinline__ bool chunk_live(const S&, int) const { return true; }
  __device__ __forceinline__ void begin(State& st, const MaskView&, int mb, int nb, int r, int ks) const {
    st.col0 = (int64_t)nb * BN;
    st.s = scale ? scale[0] : 1.f;
    st.y0 = mb * BM + r - (int)(threadIdx.x & 31);
    st.ks = ks;
  }
  // Push mode has no zero-tile shortcut: an empty unit still sends its slab.
  __device__ __forceinline__ bool zero_shortcut() const { return push == 0; }
  __device__ __forceinline__ void chunk(State& st, int c, float (&v)[32], Stager& sg) const {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] *= st.s;
    if (push) {
      push_chunk(st, c, v, sg);
      return;
    }
    sg.store_f32(v, (int)(st.col0 + c * 32), st.y0, st.ks, accumulate != 0);
  }
  // The warp's 32 rows x 32 columns go through its 4 KB staging area (16-byte
  // units of row r at unit u ^ (r & 7): conflict-free both ways), then leave
  // as 4 rows x 128 contiguous bytes per store instruction.
  __device__ __forceinline__ void push_chunk(const State& st, int c, const float (&v)[32], Stager& sg) const {
    const int lane = threadIdx.x & 31;
    float4* buf = reinterpret_cast<float4*>(sg.buf);
    __syncwarp();  // the previous chunk's reads of the staging area are done
#pragma unroll
    for (int u = 0; u < 8; ++u)
      buf[lane * 8 + (u ^ (lane & 7))] = make_float4(v[4 * u], v[4 * u + 1], v[4 * u + 2], v[4 * u + 3]);
    __syncwarp();
    const int u = lane & 7;
    const int64_t col = st.col0 + c * 32 + 4 * u;
    const int owner = (int)((st.y0 / peer::kRows) / layout.mt_per);
    float* slot = reinterpret_cast<float*>(peers.bases[owner] + layout.recv_off) +
                  ((int64_t)(peers.rank * peer::kSlotsPerSrc + st.ks) * layout.R - (int64_t)owner * layout.R) * D;
    const float* slab = acc2 + (int64_t)st.ks * N * D;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int rr = 4 * i + (lane >> 3);
      const int64_t row = (int64_t)st.y0 + rr;
      float4 x = buf[rr * 8 + (u ^ (rr & 7))];
      if (row < N && col < D) {
        if (accumulate) {
          const float4 a = *reinterpret_cast<const float4*>(slab + row * D + col);
          x.x += a.x;
          x.y += a.y;
          x.z += a.z;
          x.w += a.w;
        }
        *reinterpret_cast<float4*>(slot + row * D + col) = x;
      }
    }
  }
  __device__ __forceinline__ void end(State&) const {}
  // Push mode: once all 128 epilogue threads' stores of the unit are issued
  // (they arrive on `ubar`; the wait is bounded), one thread publishes them
  // and counts the unit; the last unit of the launch raises `pushed`.
  __device__ __forceinline__ void after_unit(uint64_t* ubar, uint32_t& uphase) const {
    if (!push) return;
    mbar_arrive(ubar);
    if (threadIdx.x == 64 && mbar_wait(ubar, uphase, kPushWaitCode))
      peer::arrive_and_signal(peers, peer::kDoneUnitsOff, total_units, true, peer::kPushedOff);
    uphase ^= 1u;
  }
};

// ---------------------------------------------------------------------------
// K6: grad_c store
// ---------------------------------------------------------------------------

template <typename T>
struct GradCEpi {
  static constexpr bool kNarrowB = false;  // B rows loaded for a tile's live column run only
  static constexpr bool kPairLd = true;   // the epilogue reads TMEM two 32-column chunks at a time
  static constexpr bool kHalfK = false;  // half K-blocks loaded alone (see A_HALF_BYTES)
  static constexpr bool kWideCapable = false;  // may run as wide units (see GradEEpi)
  static constexpr int kKind = 3;  // slot in g_mma_cols
  T* out;        // grad_c + vc0 * D
  const float* scale;       // fp16: {s, 1/s}, the products are multiplied by s; else nullptr
  const void* mask_src;     // activity table rows of the chunk's M tiles: [ceil(V/128)][mask_ld] words
  int64_t mask_ld;          // words per table row
  int mask_rows, mask_cols; // M tiles in the chunk, nRb
  int64_t rows, D;
  int pair = 1;             // TMEM read two chunks per wait (kPairLd), else one
  __device__ __forceinline__ bool pair_ld() const { return pair != 0; }

  struct State {
    int64_t row, col0;
    float s;
    int y0;  // first row of this warp's 32-row slab
  };
  // M tile mb covers the chunk's statistics tiles kStatsPerM * mb + i; K-block
  // kb (64 rows) lies in row block kb / 2.
  static constexpr bool kMask = true;
  static constexpr bool kZeroTiles = true;
  __device__ __forceinline__ bool tile_active(const MaskView&, int, int) const { return true; }
  __device__ __forceinline__ uint32_t col_mask(const MaskView&, int, int) const { return kAllGroups; }
  // The mask view is the transposed activity table: row = the chunk's 128-row
  // M tile, bit = row block (the OR of the tile's statistics tiles there).
  static constexpr bool kMaskBits = true;
  static constexpr int kKpr = kRowBlock / BK;  // K-blocks per row block
  __device__ __forceinline__ uint32_t ksub_mask(const MaskView&, int, int, int) const { return 0xFu; }
  __device__ __forceinline__ int next_kb(const MaskView& mk, int mb, int, int kb, int kb1) const {
    if (mb >= mask_rows) return kb1;
    const int lim = min((kb1 + kKpr - 1) / kKpr, mask_cols);
    const int r = mk.next(mb, kb / kKpr, lim);
    if (r >= lim) return kb1;
    return max(kb, r * kKpr);
  }
  // Every tile is written (zero tiles with plain stores, see zero_tile).
  __device__ __forceinline__ bool skip_unit(const MaskView&, int, int, int, int) const { return false; }
  __device__ __forceinline__ void inactive_tile(int, int, int) const {}
  __device__ __forceinline__ bool zero_shortcut() const { return true; }
  // A tile no K-block reached is zero: lane l stores 8 columns of each row.
  __device__ __forceinline__ void zero_tile(const State& st) const {
    const int64_t c0 = st.col0 + 8 * (threadIdx.x & 31);
    if (c0 >= D) return;
    for (int i = 0; i < 32 && (int64_t)st.y0 + i < rows; ++i)
      *reinterpret_cast<uint4*>(out + ((int64_t)st.y0 + i) * D + c0) = make_uint4(0u, 0u, 0u, 0u);
  }
  template <class S>
  __device__ __forceinline__ bool chunk_live(const S&, int) const { return true; }
  __device__ __forceinline__ void begin(State& st, const MaskView&, int mb, int nb, int r, int) const {
    st.row = (int64_t)mb * BM + r;
    st.col0 = (int64_t)nb * BN;
    st.s = scale ? scale[0] : 1.f;
    st.y0 = (int)(st.row - (threadIdx.x & 31));
  }
  __device__ __forceinline__ void chunk(State& st, int c, float (&v)[32], Stager& sg) const {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] *= st.s;
    sg.store16<T>(v, (int)(st.col0 + c * 32), st.y0);
  }
  __device__ __forceinline__ void end(State&) const {}
  __device__ __forceinline__ void after_unit(uint64_t*, uint32_t&) const {}
};

// ---------------------------------------------------------------------------
// the engine
// ---------------------------------------------------------------------------

// The epilogue's mask slice as a MaskView: copied into shared memory as bits
// when it fits (all threads of the block take part; a __syncthreads follows
// before any use), else read in place.  kMaskBits: the source already holds
// row-aligned bit words (row stride mask_ld words); else one byte per entry
// (row stride mask_ld bytes).
template <class Epi>
__device__ __forceinline__ void load_mask_view(const Epi& epi, uint8_t* smask, MaskView& mk) {
  if constexpr (Epi::kMask) {
    const int rows = epi.mask_rows, cols = epi.mask_cols;
    const int wpr = (cols + 31) / 32;
    const bool fits = (int64_t)rows * wpr * 4 <= SMASK_BYTES;
    uint32_t* sb = reinterpret_cast<uint32_t*>(smask);
    mk.cols = cols;
    if constexpr (Epi::kMaskBits) {
      const uint32_t* src = static_cast<const uint32_t*>(epi.mask_src);
      if (fits) {
        for (int i = threadIdx.x; i < rows * wpr; i += blockDim.x)
          sb[i] = __ldg(src + (int64_t)(i / wpr) * epi.mask_ld + i % wpr);
        mk.bits = sb;
        mk.wpr = wpr;
      } else {
        mk.bits = src;
        mk.wpr = (int)epi.mask_ld;
      }
    } else {
      const uint8_t* src0 = static_cast<const uint8_t*>(epi.mask_src);
      if (fits) {
        // one thread per 32-column word, its 32 byte loads independent (a
        // warp-wide ballot per word serialised ~100 L2 round trips per warp
        // before the first tile)
        for (int i = threadIdx.x; i < rows * wpr; i += blockDim.x) {
          const int rr = i / wpr, w = i - rr * wpr;
          const uint8_t* src = src0 + (int64_t)rr * epi.mask_ld + w * 32;
          const int n = min(32, cols - w * 32);
          uint32_t word = 0;
#pragma unroll
          for (int b = 0; b < 32; ++b)
            if (b < n && __ldg(src + b) != 0) word |= 1u << b;
          sb[i] = word;
        }
        mk.bits = sb;
        mk.wpr = wpr;
      } else {
        mk.bytes = src0;
        mk.ld = epi.mask_ld;
      }
    }
  }
}

template <bool A_MN, bool B_MN, class Epi>
__global__ void __launch_bounds__(kThreads, 1)
tc_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
               const __grid_constant__ CUtensorMap tmAalt, const __grid_constant__ CUtensorMap tmBalt,
               const __grid_constant__ CUtensorMap tmC, const Sched sched, const Epi epi, const uint32_t idesc) {
  // tmBalt: K-major B in 32-row boxes (kNarrowB); tmAalt / tmBalt: the half
  // K-block boxes of A and B (kHalfK).
  extern __shared__ uint8_t smem_raw[];
  const uint32_t pad = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
  uint8_t* smem = smem_raw + pad;
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_BYTES;
  uint8_t* sOut = sB + STAGES * B_BYTES;   // epilogue staging (1 KB aligned)
  uint64_t* full = reinterpret_cast<uint64_t*>(sOut + OUT_STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* rfull = tempty + 2;      // tile-id ring: published by the producer
  uint64_t* rempty = rfull + RING;   // released by the MMA thread + 128 epilogue threads
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(rempty + RING);
  volatile int* ring = reinterpret_cast<volatile int*>(tmem_slot + 1);
  uint64_t* ubar = full + 23;        // epilogue unit barrier (bytes 184-191; the ring ends at 180)
  uint8_t* smask = reinterpret_cast<uint8_t*>(full) + 256;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_tiles = sched.units();

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(tfull + a, 1);
      mbar_init(tempty + a, 128);
    }
    for (int i = 0; i < RING; ++i) {
      mbar_init(rfull + i, 1);
      mbar_init(rempty + i, 129);
    }
    mbar_init(ubar, 128);
    fence_barrier_init();
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
    if constexpr (Epi::kNarrowB) prefetch_tmap(&tmBalt);
    if constexpr (Epi::kHalfK) {
      if (epi.half_k) {
        prefetch_tmap(&tmAalt);
        prefetch_tmap(&tmBalt);
      }
    }
  }
  // Filter-mask slice: copied to shared memory when it fits, else read in place.
  MaskView mk{nullptr, nullptr, 0, 0, 0};
  load_mask_view<Epi>(epi, smask, mk);
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer + tile scheduler ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      // Work units are claimed one id at a time from the global counter
      // (dynamic schedule) or in a fixed stride (static).  The next id is
      // claimed one unit ahead, so the atomic's latency overlaps the current
      // unit's loads.  A unit the epilogue has nothing to do for
      // (Epi::skip_unit) is passed over here and never reaches the MMA and
      // epilogue warps.  (Claiming several ids per atomic after dead units
      // measured slower: live tiles then bunch up on a few SMs.)
      // With a unit list (sched.list) a claim k is list entry k, a unit with
      // work; the entry is read when the claim is taken up.
      const int num_claims = sched.list ? min(*sched.list_count, num_tiles) : num_tiles;
      int next = sched.counter ? atomicAdd(sched.counter, 1) : (int)blockIdx.x;
      int sidx = 0;  // static schedule: claims made
      auto advance = [&]() {
        next = sched.counter ? atomicAdd(sched.counter, 1) : (int)blockIdx.x + (++sidx) * (int)gridDim.x;
      };
      for (int i = 0;; ++i) {
        const int slot = i & (RING - 1);
        if (!mbar_wait(rempty + slot, ((i / RING) & 1) ^ 1u, 5)) break;
        int tile = -1;
        int mb = 0, nb = 0, ks = 0, kb0 = 0, kb1 = 0;
        while (next < num_claims) {
          const int u = sched.list ? __ldg(sched.list + next) : next;
          sched.coords(u, mb, nb, ks);
          sched.krange(ks, kb0, kb1);
          const bool skip = epi.skip_unit(mk, mb, nb, kb0, kb1);
          advance();
          if (!skip) {
            tile = u;
            break;
          }
        }
        ring[slot] = tile;
        mbar_arrive(rfull + slot);
        if (tile < 0) break;
        if (!epi.tile_active(mk, mb, nb)) continue;
        // B rows to load: the whole tile, or (K-major B, kNarrowB) only a
        // short run of live 32-column groups [nj0, nj0 + nn0) -- the rows
        // the MMA of this tile reads (see the MMA issuer)
        uint32_t nj0 = 0, nn0 = kGroups;
        bool dbl = false;  // two K-blocks per stage (see kDblB0)
        if constexpr (Epi::kNarrowB && !B_MN) {
          uint32_t j, n;
          if (narrow_run(epi.col_mask(mk, mb, nb), j, n)) {
            nj0 = j;
            nn0 = n;
            dbl = epi.dbl != 0;
          }
        }
        const uint32_t tx_bytes = A_BYTES + (nn0 < (uint32_t)kGroups ? nn0 * B32_BYTES : B_BYTES);
        const int kstep = dbl ? 2 : 1;
        bool ok = true;
        for (int kb = epi.next_kb(mk, mb, nb, kb0, kb1); kb < kb1; kb = epi.next_kb(mk, mb, nb, kb + kstep, kb1)) {
          if (!mbar_wait(empty + stage, phase ^ 1u, 1)) { ok = false; break; }
          uint8_t* a = sA + stage * A_BYTES;
          uint8_t* b = sB + stage * B_BYTES;
          const int k0 = kb * BK;
          if constexpr (Epi::kNarrowB && !B_MN) {
            if (dbl) {
              const bool two = kb + 1 < kb1;
              mbar_arrive_expect_tx(full + stage, (two ? 2u : 1u) * tx_bytes);
              tma_load_2d(a, &tmA, full + stage, k0, mb * BM);
              for (uint32_t g = 0; g < nn0; ++g)
                tma_load_2d(b + kDblB0 + g * B32_BYTES, &tmBalt, full + stage, k0, nb * BN + (int)((nj0 + g) * kStatTile));
              if (two) {
                tma_load_2d(b, &tmA, full + stage, k0 + BK, mb * BM);
                for (uint32_t g = 0; g < nn0; ++g)
                  tma_load_2d(b + kDblB1 + g * B32_BYTES, &tmBalt, full + stage, k0 + BK,
                              nb * BN + (int)((nj0 + g) * kStatTile));
              }
              if (++stage == STAGES) {
                stage = 0;
                phase ^= 1u;
              }
              continue;
            }
          }
          if constexpr (Epi::kWideCapable) {
            if (epi.wide) {
              // one statistics tile of K for the tile pair nb = 2 np, 2 np + 1
              const int kt = kb * kStatTile;
              mbar_arrive_expect_tx(full + stage, A_HALF_BYTES + 2 * B_HALF_BYTES);
              tma_load_2d(a, &tmAalt, full + stage, kt, mb * BM);
              tma_load_3d(b, &tmBalt, full + stage, 0, kt, nb * (2 * BN / 64));
              if (++stage == STAGES) {
                stage = 0;
                phase ^= 1u;
              }
              continue;
            }
          }
          if constexpr (Epi::kHalfK) {
            // one kept statistics tile (ksub_mask 0x3 or 0xC): load that half only
            const uint32_t km = epi.half_k ? epi.ksub_mask(mk, mb, nb, kb) : 0xFu;
            if (km != 0xFu) {
              const int kh = k0 + (km == 0x3u ? 0 : BK / 2);
              mbar_arrive_expect_tx(full + stage, A_HALF_BYTES + B_HALF_BYTES);
              tma_load_2d(a, &tmAalt, full + stage, kh, mb * BM);
              tma_load_3d(b, &tmBalt, full + stage, 0, kh, nb * (BN / 64));
              if (++stage == STAGES) {
                stage = 0;
                phase ^= 1u;
              }
              continue;
            }
          }
          mbar_arrive_expect_tx(full + stage, tx_bytes);
          if (A_MN) {
            if (sched.a3d) {
              tma_load_3d(a, &tmA, full + stage, 0, k0, mb * (BM / 64));
            } else {
              tma_load_2d(a, &tmA, full + stage, mb * BM, k0);
              tma_load_2d(a + BOX_MN_BYTES, &tmA, full + stage, mb * BM + 64, k0);
            }
          } else {
            tma_load_2d(a, &tmA, full + stage, k0, mb * BM);
          }
          if (B_MN) {
            if (sched.b3d) {
              tma_load_3d(b, &tmB, full + stage, 0, k0, nb * (BN / 64));
            } else {
#pragma unroll
              for (int j = 0; j < BN / 64; ++j)
                tma_load_2d(b + j * BOX_MN_BYTES, &tmB, full + stage, nb * BN + j * 64, k0);
            }
          } else if (nn0 < (uint32_t)kGroups) {
            for (uint32_t g = nj0; g < nj0 + nn0; ++g)
              tma_load_2d(b + g * B32_BYTES, &tmBalt, full + stage, k0, nb * BN + (int)(g * kStatTile));
          } else {
            tma_load_2d(b, &tmB, full + stage, k0, nb * BN);
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      unsigned long long mma_cols = 0;  // sum of N over the issued M=128, K=16 MMAs
      // descriptors of stage 0, k-step 0; the start-address field (addr >> 4,
      // bits 0-13) is advanced by adding byte offsets >> 4
      const uint64_t adesc0 = A_MN ? smem_desc(smem_u32(sA), BOX_MN_BYTES, 1024)
                                   : smem_desc(smem_u32(sA), 16, 1024);
      const uint64_t bdesc0 = B_MN ? smem_desc(smem_u32(sB), BOX_MN_BYTES, 1024)
                                   : smem_desc(smem_u32(sB), 16, 1024);
      constexpr uint32_t a_kstep = (A_MN ? 2048u : 32u) >> 4;
      constexpr uint32_t b_kstep = (B_MN ? 2048u : 32u) >> 4;
      // half K-blocks (kHalfK: K-major A, MN-major B): A in the 64-byte
      // swizzle (8-row groups 512 bytes apart), B slabs 4 KB apart
      const uint64_t adesc_h = smem_desc_sw64(smem_u32(sA), 16, 512);
      const uint64_t bdesc_h = smem_desc(smem_u32(sB), BOX_MN_HALF_BYTES, 1024);
      for (int i = 0;; ++i) {
        const int slot = i & (RING - 1);
        if (!mbar_wait(rfull + slot, (i / RING) & 1, 6)) break;
        const int tile = ring[slot];
        mbar_arrive(rempty + slot);
        if (tile < 0) break;
        int mb, nb, ks, kb0, kb1;
        sched.coords(tile, mb, nb, ks);
        sched.krange(ks, kb0, kb1);
        if (!epi.tile_active(mk, mb, nb)) continue;
        if constexpr (Epi::kWideCapable) {
          if (epi.wide) {
            // both accumulators: columns [0, 256) for nb = 2 np, [256, 512) for 2 np + 1
            if (!mbar_wait(tempty + 0, acc_phase ^ 1u, 2) || !mbar_wait(tempty + 1, acc_phase ^ 1u, 2)) break;
            tc_fence_after();
            bool ok = true;
            uint32_t fresh = 1;
            constexpr uint32_t b_second = (4 * BOX_MN_HALF_BYTES) >> 4;  // slabs 4-7 of the B box
            for (int kb = epi.next_kb(mk, mb, nb, kb0, kb1); kb < kb1; kb = epi.next_kb(mk, mb, nb, kb + 1, kb1)) {
              mma_cols += 4ull * BN;
              if (!mbar_wait(full + stage, phase, 3)) { ok = false; break; }
              tc_fence_after();
              const uint64_t ad = adesc_h + (uint64_t)((stage * A_BYTES) >> 4);
              const uint64_t bd = bdesc_h + (uint64_t)((stage * B_BYTES) >> 4);
#pragma unroll
              for (int k = 0; k < kStatTile / 16; ++k) {
                mma_f16(tmem_base, ad + k * a_kstep, bd + k * b_kstep, idesc, fresh ^ 1u);
                mma_f16(tmem_base + BN, ad + k * a_kstep, bd + b_second + k * b_kstep, idesc, fresh ^ 1u);
                fresh = 0;
              }
              mma_commit(empty + stage);
              if (++stage == STAGES) {
                stage = 0;
                phase ^= 1u;
              }
            }
            if (!ok) break;
            mma_commit(tfull + 0);
            mma_commit(tfull + 1);
            acc_phase ^= 1u;
            continue;
          }
        }
        if (!mbar_wait(tempty + acc, acc_phase ^ 1u, 2)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
        // The tile's statistics-tile column groups to compute: the span from
        // the first to the last kept group (j0, n0) -- one MMA of N =
        // kStatTile n0 columns at B rows kStatTile j0 (K-major B: 128 bytes
        // per row); the columns of rejected groups inside the span are
        // computed and never read.  (Two runs as two MMAs re-read A from
        // shared memory and measured slower.)  sched.span = 0 narrows only a
        // single run of kept groups.
        uint32_t j0 = 0, n0 = kGroups;
        bool dbl = false;  // the producer's two-K-blocks-per-stage layout (kDblB0)
        if constexpr (!B_MN) {
          const uint32_t cm = epi.col_mask(mk, mb, nb);
          if (cm != kAllGroups && cm != 0u) {
            const uint32_t j = __ffs(cm) - 1;
            const uint32_t n = sched.span ? (32u - __clz(cm)) - j : __ffs(~(cm >> j)) - 1;
            if ((cm >> (j + n)) == 0u) {
              j0 = j;
              n0 = n;
            }
          }
          if constexpr (Epi::kNarrowB) {
            uint32_t j, n;
            dbl = epi.dbl != 0 && narrow_run(cm, j, n);  // then (j, n) == (j0, n0)
          }
        }
        const uint32_t idesc0 = idesc_with_n(idesc, kStatTile * n0);
        const uint32_t d0 = d_tmem + kStatTile * j0;
        const uint32_t boff = (kStatTile * 128u * j0) >> 4;
        bool ok = true;
        uint32_t fresh = 1;  // the tile's first MMA overwrites the accumulator
        if constexpr (Epi::kNarrowB && !B_MN) {
          if (dbl) {
            for (int kb = epi.next_kb(mk, mb, nb, kb0, kb1); kb < kb1; kb = epi.next_kb(mk, mb, nb, kb + 2, kb1)) {
              const bool two = kb + 1 < kb1;
              mma_cols += (unsigned long long)((two ? 2 : 1) * (BK / 16) * kStatTile * n0);
              if (!mbar_wait(full + stage, phase, 3)) { ok = false; break; }
              tc_fence_after();
              const uint32_t sb = smem_u32(sB + stage * B_BYTES);
              const uint64_t ad = adesc0 + (uint64_t)((stage * A_BYTES) >> 4);
              const uint64_t bd = smem_desc(sb + kDblB0, 16, 1024);
#pragma unroll
              for (int k = 0; k < BK / 16; ++k) {
                mma_f16(d0, ad + k * a_kstep, bd + k * b_kstep, idesc0, fresh ^ 1u);
                fresh = 0;
              }
              if (two) {
                const uint64_t ad1 = smem_desc(sb, 16, 1024);
                const uint64_t bd1 = smem_desc(sb + kDblB1, 16, 1024);
#pragma unroll
                for (int k = 0; k < BK / 16; ++k) mma_f16(d0, ad1 + k * a_kstep, bd1 + k * b_kstep, idesc0, 1u);
              }
              mma_commit(empty + stage);
              if (++stage == STAGES) {
                stage = 0;
                phase ^= 1u;
              }
            }
            if (!ok) break;
            mma_commit(tfull + acc);
            acc ^= 1;
            if (acc == 0) acc_phase ^= 1u;
            continue;
          }
        }
        for (int kb = epi.next_kb(mk, mb, nb, kb0, kb1); kb < kb1; kb = epi.next_kb(mk, mb, nb, kb + 1, kb1)) {
          const uint32_t km = epi.ksub_mask(mk, mb, nb, kb);  // K=16 steps to issue
          mma_cols += (unsigned long long)(__popc(km & 0xFu) * kStatTile * n0);
          if (!mbar_wait(full + stage, phase, 3)) { ok = false; break; }
          tc_fence_after();
          if constexpr (Epi::kHalfK) {
            if (epi.half_k && km != 0xFu) {
              // the stage holds the kept half: its two K=16 steps
              const uint64_t ad = adesc_h + (uint64_t)((stage * A_BYTES) >> 4);
              const uint64_t bd = bdesc_h + (uint64_t)((stage * B_BYTES) >> 4) + boff;
#pragma unroll
              for (int k = 0; k < BK / 32; ++k) {
                mma_f16(d0, ad + k * a_kstep, bd + k * b_kstep, idesc0, fresh ^ 1u);
                fresh = 0;
              }
              mma_commit(empty + stage);
              if (++stage == STAGES) {
                stage = 0;
                phase ^= 1u;
              }
              continue;
            }
          }
          const uint64_t ad = adesc0 + (uint64_t)((stage * A_BYTES) >> 4);
          const uint64_t bd = bdesc0 + (uint64_t)((stage * B_BYTES) >> 4) + boff;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            if ((km >> k) & 1u) {
              mma_f16(d0, ad + k * a_kstep, bd + k * b_kstep, idesc0, fresh ^ 1u);
              fresh = 0;
            }
          }
          mma_commit(empty + stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        mma_commit(tfull + acc);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1u;
      }
      atomicAdd(&g_mma_cols[Epi::kKind], mma_cols);
    }
    __syncwarp();
  } else {
    // ---------------- epilogue (warps 2..5) ----------------
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int r = q * 32 + lane;
    Stager sg{&tmC, sOut + q * 4096, 0};
    int acc = 0;
    uint32_t acc_phase = 0;
    uint32_t uphase = 0;
    for (int i = 0;; ++i) {
      const int slot = i & (RING - 1);
      if (!mbar_wait(rfull + slot, (i / RING) & 1, 7)) break;
      const int tile = ring[slot];
      mbar_arrive(rempty + slot);
      if (tile < 0) break;
      int mb, nb, ks, kb0, kb1;
      sched.coords(tile, mb, nb, ks);
      sched.krange(ks, kb0, kb1);
      if (!epi.tile_active(mk, mb, nb)) {
        epi.inactive_tile(mb, nb, r);
        continue;
      }
      const bool any_kb = !Epi::kMask || epi.next_kb(mk, mb, nb, kb0, kb1) < kb1;
      // One output tile from the accumulator at column `col`.
      auto drain_tile = [&](int nbt, uint32_t col) {
        typename Epi::State st;
        epi.begin(st, mk, mb, nbt, r, ks);
        const uint32_t tbase = tmem_base + ((uint32_t)(q * 32) << 16) + col;
        // a tile no K-block reached is all zeros: plain coalesced zero stores
        // (or nothing, when zeros would be added), not the staged path
        bool zero_tile = false;
        if constexpr (Epi::kZeroTiles) zero_tile = !any_kb && epi.zero_shortcut();
        if (zero_tile) {
          if constexpr (Epi::kZeroTiles) epi.zero_tile(st);
        } else if (Epi::kPairLd && epi.pair_ld() && any_kb) {
          // two chunks per TMEM wait: the loads of chunks 2p + 2, 2p + 3 are in
          // flight while chunks 2p, 2p + 1 are processed (every chunk live)
          uint32_t cur0[32], cur1[32], nxt0[32], nxt1[32];
          tmem_ld32_issue(tbase, cur0);
          tmem_ld32_issue(tbase + 32, cur1);
#pragma unroll 1
          for (int p = 0; p < BN / 64; ++p) {
            __syncwarp();
            tmem_ld_wait(cur0);
            tmem_ld_wait(cur1);
            const bool more = p + 1 < BN / 64;
            if (more) {
              tmem_ld32_issue(tbase + (2 * p + 2) * 32, nxt0);
              tmem_ld32_issue(tbase + (2 * p + 3) * 32, nxt1);
            }
            float v[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(cur0[j]);
            epi.chunk(st, 2 * p, v, sg);
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(cur1[j]);
            epi.chunk(st, 2 * p + 1, v, sg);
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              cur0[j] = nxt0[j];
              cur1[j] = nxt1[j];
            }
          }
        } else {
          // the TMEM load of chunk c + 1 is in flight while chunk c is processed
          uint32_t cur[32], nxt[32];
          bool cur_live = any_kb && epi.chunk_live(st, 0);
          if (cur_live) tmem_ld32_issue(tbase, cur);
#pragma unroll 1
          for (int c = 0; c < BN / 32; ++c) {
            __syncwarp();
            const bool nxt_live = c + 1 < BN / 32 && any_kb && epi.chunk_live(st, c + 1);
            if (cur_live) tmem_ld_wait(cur);
            if (nxt_live) tmem_ld32_issue(tbase + (c + 1) * 32, nxt);
            float v[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = cur_live ? __uint_as_float(cur[j]) : 0.f;
            epi.chunk(st, c, v, sg);
#pragma unroll
            for (int j = 0; j < 32; ++j) cur[j] = nxt[j];
            cur_live = nxt_live;
          }
        }
        epi.end(st);
      };
      if constexpr (Epi::kWideCapable) {
        if (epi.wide) {
          // the tile pair 2 nb, 2 nb + 1 from accumulators 0 and 1
          bool ok = true;
          for (int h = 0; h < 2; ++h) {
            if (!mbar_wait(tfull + h, acc_phase, 4)) { ok = false; break; }
            tc_fence_after();
            if ((int64_t)(2 * nb + h) * BN < epi.D) drain_tile(2 * nb + h, (uint32_t)(h * BN));
            __syncwarp();
            tc_fence_before();
            mbar_arrive(tempty + h);
          }
          if (!ok) break;
          epi.after_unit(ubar, uphase);
          acc_phase ^= 1u;
          continue;
        }
      }
      if (!mbar_wait(tfull + acc, acc_phase, 4)) break;
      tc_fence_after();
      drain_tile(nb, (uint32_t)(acc * BN));
      epi.after_unit(ubar, uphase);
      __syncwarp();
      tc_fence_before();
      mbar_arrive(tempty + acc);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1u;
    }
    sg.drain();  // output boxes written before the kernel ends
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}


// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = []() -> EncodeTiledFn {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return nullptr;
    return reinterpret_cast<EncodeTiledFn>(p);
  }();
  return fn;
}

int num_sms() {
  static std::atomic<int> cache[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (dev < 0 || dev >= 64) return 148;
  int n = cache[dev].load(std::memory_order_relaxed);
  if (n == 0) {
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cache[dev].store(n, std::memory_order_relaxed);
  }
  return n;
}

// Row-major [outer][inner] 16-bit matrix with row stride `ld` elements, read in
// (box_inner x box_outer) boxes with 128-byte swizzling and zero fill.
bool make_tmap(CUtensorMap* tm, const void* base, bool bf16, int64_t inner, int64_t outer, int64_t ld,
               uint32_t box_inner, uint32_t box_outer,
               CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)outer};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t es[2] = {1, 1};
  CUresult r = fn(tm, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                  const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// A/B switches for timing, read once from the environment:
// CCE_GRAD_E_WIDE=0 runs grad_e as single 128 x 256 tiles (64-row K-blocks)
// instead of wide units; CCE_GRAD_E_HALF_K=0 then loads whole K-blocks only.
bool env_on(const char* name) {
  const char* s = getenv(name);
  return !(s != nullptr && s[0] == '0');
}
// CCE_DLOGITS_SPAN=0: dlogits narrows its MMA only to a single run of kept
// column groups instead of the span of all of them (A/B switch).
bool dlogits_span() {
  static const bool v = env_on("CCE_DLOGITS_SPAN");
  return v;
}
bool half_k_enabled() {
  static const bool v = env_on("CCE_GRAD_E_HALF_K");
  return v;
}
bool wide_enabled() {
  static const bool v = env_on("CCE_GRAD_E_WIDE");
  return v;
}
// CCE_GRAD_C_PAIR_LD=0: the grad_c epilogue reads TMEM one 32-column chunk per wait.
bool grad_c_pair_ld() {
  static const bool v = env_on("CCE_GRAD_C_PAIR_LD");
  return v;
}
// CCE_DLOGITS_DOUBLE_K=0: narrow dlogits tiles load one K-block per stage.
bool dlogits_double_k() {
  static const bool v = env_on("CCE_DLOGITS_DOUBLE_K");
  return v;
}

// An MN-major operand [outer][inner] (inner contiguous, a multiple of 64) as a
// 3-D tensor [inner / 64 groups][outer rows][64]: one box of (64, box_rows,
// groups) lands in shared memory as `groups` consecutive 64-column slabs of
// box_rows x 128 bytes -- the same layout as `groups` separate 2-D boxes.
bool make_tmap_mn3d(CUtensorMap* tm, const void* base, bool bf16, int64_t inner, int64_t outer,
                    int64_t ld, uint32_t box_rows, uint32_t groups) {
  EncodeTiledFn fn = encode_fn();
  if (!fn || inner % 64 != 0) return false;
  cuuint64_t dims[3] = {64, (cuuint64_t)outer, (cuuint64_t)(inner / 64)};
  cuuint64_t strides[2] = {(cuuint64_t)(ld * 2), 128};
  cuuint32_t box[3] = {64, box_rows, groups};
  cuuint32_t es[3] = {1, 1, 1};
  CUresult r = fn(tm, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3,
                  const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// MN-major operand map: the 3-D form when the encoder accepts it, else 2-D boxes
// of 64 columns.  Returns false when neither can be encoded; *is3d tells which.
bool make_tmap_mn(CUtensorMap* tm, const void* base, bool bf16, int64_t inner, int64_t outer,
                  int64_t ld, uint32_t groups, int* is3d) {
  if (make_tmap_mn3d(tm, base, bf16, inner, outer, ld, BK, groups)) {
    *is3d = 1;
    return true;
  }
  *is3d = 0;
  return make_tmap(tm, base, bf16, inner, outer, ld, 64, BK);
}

// Epilogue output map: row-major [outer][inner] of `dtype` (CCE_F32 / F16 /
// BF16), row stride `ld` elements, written in (box_inner x 32) boxes of 64
// bytes per row with the 64-byte swizzle the Stager lays out.
bool make_tmap_out(CUtensorMap* tm, const void* base, int dtype, int64_t inner, int64_t outer, int64_t ld) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  const int es = dtype == CCE_F32 ? 4 : 2;
  const CUtensorMapDataType dt = dtype == CCE_F32   ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                 : dtype == CCE_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                    : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)outer};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * es)};
  cuuint32_t box[2] = {(cuuint32_t)(64 / es), 32};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(tm, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// The two fp32 grad_e accumulator slabs acc2[2][N][D] as a 3-D map, written in
// (16 x 32 x 1) boxes (64-byte rows, 64-byte swizzle); the slab index is the z
// coordinate, so rows past N of one slab are clipped rather than spilling
// into the other.
bool make_tmap_acc2(CUtensorMap* tm, const float* acc2, int64_t D, int64_t N) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[3] = {(cuuint64_t)D, (cuuint64_t)N, 2};
  cuuint64_t strides[2] = {(cuuint64_t)(D * 4), (cuuint64_t)(N * D * 4)};
  cuuint32_t box[3] = {16, 32, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float*>(acc2), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// Opt a kernel into `bytes` of dynamic shared memory, once per CUDA context
// (the attribute belongs to the context; `ctx_of` caches, per device ordinal,
// the id of the context it was last set in).
template <typename K>
cudaError_t ensure_smem_attr(K kern, size_t bytes, std::atomic<unsigned long long> (&ctx_of)[64]) {
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return err;
  const bool slot = dev >= 0 && dev < 64;
  unsigned long long ctx = 0;
  if (slot && current_context_id(&ctx) && ctx != 0 && ctx_of[dev].load(std::memory_order_acquire) == ctx)
    return cudaSuccess;
  err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
  if (err != cudaSuccess) return err;
  if (slot && current_context_id(&ctx) && ctx != 0) ctx_of[dev].store(ctx, std::memory_order_release);
  return cudaSuccess;
}

template <bool A_MN, bool B_MN, class Epi>
cudaError_t launch_gemm(const CUtensorMap& tmA, const CUtensorMap& tmB, const CUtensorMap& tmAalt,
                        const CUtensorMap& tmBalt, const CUtensorMap& tmC, const Sched& s, const Epi& epi,
                        bool bf16, cudaStream_t stream) {
  auto kern = tc_gemm_kernel<A_MN, B_MN, Epi>;
  static std::atomic<unsigned long long> attr_ctx[64];
  cudaError_t err = ensure_smem_attr(kern, SMEM_BYTES, attr_ctx);
  if (err != cudaSuccess) return err;
  const int tiles = s.units();
  if (tiles == 0) return cudaSuccess;
  const int grid = tiles < num_sms() ? tiles : num_sms();
  const uint32_t idesc = instr_desc(BM, BN, bf16, A_MN, B_MN);
  kern<<<grid, kThreads, SMEM_BYTES, stream>>>(tmA, tmB, tmAalt, tmBalt, tmC, s, epi, idesc);
  return launched();
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace
}  // namespace tc

using namespace tc;

bool tc_supported(const void* e, const void* c, int64_t D, int dtype) {
  return (dtype == CCE_BF16 || dtype == CCE_F16) && D % 8 == 0 && aligned16(e) && aligned16(c) &&
         encode_fn() != nullptr;
}

bool tc_backward_supported(const void* e, const void* c, int64_t D, int dtype) {
  return tc_supported(e, c, D, dtype);
}

namespace {

template <typename TB>
cudaError_t fwd_launch(const FwdArgs& a, cudaStream_t s) {
  const bool bf16 = a.dtype == CCE_BF16;
  CUtensorMap tmA, tmB;
  if (!make_tmap(&tmA, a.e, bf16, a.D, a.N, a.D, BK, BM)) return cudaErrorInvalidValue;
  if (!make_tmap(&tmB, a.c, bf16, a.D, a.V, a.D, BK, BN)) return cudaErrorInvalidValue;
  Sched sc{(int)ceil_div(a.N, BM), (int)ceil_div(a.V, BN), (int)ceil_div(a.D, BK), 1, 0, 0,
           nullptr, raster_group(a.N * a.D * 2)};
  FwdEpi<TB> epi{a.targets, a.bias, a.tile_max, a.part_m, a.part_s, a.tgt, a.N, a.V, a.v_offset};
  const CUtensorMap tmC{};  // the forward epilogue writes no tiles
  return launch_gemm<false, false>(tmA, tmB, tmA, tmB, tmC, sc, epi, bf16, s);
}

// The dlogits schedule of a chunk of vc_len rows (also the list builder's).
__host__ __device__ Sched dl_sched(int64_t N, int64_t D, int64_t vc_len, int* counter) {
  return Sched{(int)ceil_div(N, BM), (int)ceil_div(vc_len, BN), (int)ceil_div(D, BK), 1, 0, 0,
               counter, raster_group(N * D * 2)};
}

// One block per vocabulary chunk: thread t checks a run of consecutive unit
// ids (a tile's 8 mask bytes in one 8-byte load where they are aligned), a
// block-wide scan gives each run its place, so the list keeps the schedule
// order.
__global__ void __launch_bounds__(1024) dl_list_kernel(const uint8_t* keep, int64_t N, int64_t D, int64_t V,
                                                         int64_t vc, int* lists, int64_t list_len, int* counters) {
  static_assert(kGroups == 8, "one 8-byte mask load per tile");
  __shared__ int warp_tot[32];
  const int ch = blockIdx.x;
  const int64_t vc0 = (int64_t)ch * vc;
  const int64_t vlen = min(vc, V - vc0);
  const Sched sc = dl_sched(N, D, vlen, nullptr);
  const int units = sc.units();
  const int64_t nvt = ceil_div(V, (int64_t)kStatTile);
  const int64_t t0 = vc0 / kStatTile;
  const int tiles = (int)ceil_div(vlen, (int64_t)kStatTile);  // the chunk's statistics tiles
  const bool wide = ((nvt | t0) & 7) == 0 && (reinterpret_cast<uintptr_t>(keep) & 7) == 0;
  const int per = (units + (int)blockDim.x - 1) / (int)blockDim.x;
  const int u0 = min(units, (int)threadIdx.x * per), u1 = min(units, u0 + per);
  auto live = [&](int u) {
    int mb, nb, ks;
    sc.coords(u, mb, nb, ks);
    const uint8_t* row = keep + (int64_t)mb * nvt + t0;
    const int g0 = kGroups * nb, g1 = min(g0 + kGroups, tiles);
    if (wide && g1 - g0 == kGroups) return __ldg(reinterpret_cast<const unsigned long long*>(row + g0)) != 0ull;
    bool any = false;
    for (int g = g0; g < g1; ++g) any |= __ldg(row + g) != 0;
    return any;
  };
  // pass 1: count (live bits of the first 32 units kept in a register)
  uint32_t bits = 0;
  int cnt = 0;
#pragma unroll 8
  for (int i = 0; i < per; ++i) {
    const int u = u0 + i;
    if (u < u1 && live(u)) {
      ++cnt;
      if (i < 32) bits |= 1u << i;
    }
  }
  // exclusive scan of cnt over the block
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int incl = cnt;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  if (lane == 31) warp_tot[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    const int nw = (int)(blockDim.x >> 5);
    int w = lane < nw ? warp_tot[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    if (lane < nw) warp_tot[lane] = w;  // inclusive over warps
    if (lane == nw - 1) counters[4 * ch + 3] = w;
  }
  __syncthreads();
  // pass 2: write the ids
  int pos = incl - cnt + (warp > 0 ? warp_tot[warp - 1] : 0);
  int* list = lists + (int64_t)ch * list_len;
  for (int i = 0; i < per && u0 + i < u1; ++i)
    if (i < 32 ? ((bits >> i) & 1u) != 0 : live(u0 + i)) list[pos++] = u0 + i;
}

template <typename T, typename TB>
cudaError_t dl_launch(const BwdChunkArgs& a, cudaStream_t s) {
  const bool bf16 = a.dtype == CCE_BF16;
  CUtensorMap tmA, tmB;
  const void* cchunk = a.c_chunk;
  if (!make_tmap(&tmA, a.e, bf16, a.D, a.N, a.D, BK, BM)) return cudaErrorInvalidValue;
  if (!make_tmap(&tmB, cchunk, bf16, a.D, a.vc_len, a.D, BK, BN)) return cudaErrorInvalidValue;
  Sched sc = dl_sched(a.N, a.D, a.vc_len, a.counters ? a.counters + 0 : nullptr);
  if (a.dl_list != nullptr && a.counters != nullptr) {
    sc.list = a.dl_list;
    sc.list_count = a.counters + 3;
  }
  const int64_t vc_end = (a.vc0 + a.vc_len) < a.V ? (a.vc0 + a.vc_len) : a.V;
  sc.span = dlogits_span() ? 1 : 0;
  DlogitsEpi<T, TB> epi{a.targets, a.lse, a.d_nll, a.bias, static_cast<T*>(a.dlogits), a.grad_bias,
                        a.scale, a.keep + a.vc0 / kStatTile, ceil_div(a.V, kStatTile),
                        (int)ceil_div(a.N, kRowBlock), (int)ceil_div(a.vc_len, kStatTile),
                        a.N, a.V, a.v_offset, a.vc0, vc_end, a.vc_ld};
  epi.dbl = dlogits_double_k() ? 1 : 0;
  CUtensorMap tmC, tmB32;
  if (!make_tmap_out(&tmC, a.dlogits, a.dtype, a.vc_len, a.N, a.vc_ld)) return cudaErrorInvalidValue;
  if (!make_tmap(&tmB32, cchunk, bf16, a.D, a.vc_len, a.D, BK, kStatTile)) return cudaErrorInvalidValue;
  return launch_gemm<false, false>(tmA, tmB, tmA, tmB32, tmC, sc, epi, bf16, s);
}

}  // namespace

int64_t tc_dlogits_list_len(int64_t N, int64_t vc) { return ceil_div(N, (int64_t)BM) * ceil_div(vc, (int64_t)BN); }

cudaError_t tc_dlogits_lists(const uint8_t* keep, int64_t N, int64_t D, int64_t V, int64_t vc, int* lists,
                             int* counters, cudaStream_t s) {
  if (N == 0 || V == 0) return cudaSuccess;
  const int64_t nch = ceil_div(V, vc);
  dl_list_kernel<<<(unsigned)nch, 1024, 0, s>>>(keep, N, D, V, vc, lists, tc_dlogits_list_len(N, vc), counters);
  return cudaGetLastError();
}

cudaError_t tc_forward(const FwdArgs& a, cudaStream_t s) {
  if (a.N == 0 || a.V == 0) return cudaSuccess;
  switch (a.bias == nullptr ? -1 : a.bias_dtype) {
    case -1: return fwd_launch<void>(a, s);
    case CCE_F32: return fwd_launch<float>(a, s);
    case CCE_F16: return fwd_launch<__half>(a, s);
    case CCE_BF16: return fwd_launch<__nv_bfloat16>(a, s);
  }
  return cudaErrorInvalidValue;
}

template <typename T>
cudaError_t dl_dispatch(const BwdChunkArgs& a, cudaStream_t s) {
  switch (a.bias == nullptr ? -1 : a.bias_dtype) {
    case -1: return dl_launch<T, void>(a, s);
    case CCE_F32: return dl_launch<T, float>(a, s);
    case CCE_F16: return dl_launch<T, __half>(a, s);
    case CCE_BF16: return dl_launch<T, __nv_bfloat16>(a, s);
  }
  return cudaErrorInvalidValue;
}

cudaError_t tc_dlogits(const BwdChunkArgs& a, cudaStream_t s) {
  if (a.N == 0 || a.vc_len == 0) return cudaSuccess;
  if (a.dtype == CCE_BF16) return dl_dispatch<__nv_bfloat16>(a, s);
  if (a.dtype == CCE_F16) return dl_dispatch<__half>(a, s);
  return cudaErrorNotSupported;
}

namespace {

template <typename T>
cudaError_t grad_e_launch(const BwdChunkArgs& a, float* acc2, bool accumulate, const PeerPush* push,
                          cudaStream_t s) {
  const bool bf16 = std::is_same<T, __nv_bfloat16>::value;
  CUtensorMap tmA, tmB, tmC;
  const void* cchunk = a.c_chunk;
  if (!make_tmap(&tmA, a.dlogits, bf16, a.vc_len, a.N, a.vc_ld, BK, BM)) return cudaErrorInvalidValue;
  int b3d = 0;
  if (!make_tmap_mn(&tmB, cchunk, bf16, a.D, a.vc_len, a.D, (BN) / 64, &b3d))
    return cudaErrorInvalidValue;
  if (!make_tmap_acc2(&tmC, acc2, a.D, a.N)) return cudaErrorInvalidValue;
  Sched sc{(int)ceil_div(a.N, BM), (int)ceil_div(a.D, BN), (int)ceil_div(a.vc_len, BK), 1, 0, b3d,
           a.counters ? a.counters + 1 : nullptr, raster_group(a.N * a.vc_len * 2), 2};
  GradEEpi epi{a.scale, a.keep + a.vc0 / kStatTile, ceil_div(a.V, kStatTile), (int)ceil_div(a.N, kRowBlock),
               (int)ceil_div(a.vc_len, kStatTile), accumulate ? 1 : 0, acc2, a.N, a.D};
  if (push != nullptr) {
    epi.push = 1;
    epi.total_units = (unsigned)sc.units();
    epi.peers = push->peers;
    epi.layout = push->layout;
  }
  // A (dlogits) in boxes 32 columns wide in the 64-byte swizzle, and B (the
  // c chunk) in boxes of 32 rows of the 3-D MN-major form: 512 columns for
  // wide units, 256 for half K-blocks
  CUtensorMap tmAh = tmA, tmBh = tmB;
  const bool a_half = b3d && make_tmap(&tmAh, a.dlogits, bf16, a.vc_len, a.N, a.vc_ld, BK / 2, BM,
                                       CU_TENSOR_MAP_SWIZZLE_64B);
  if (a_half && wide_enabled() && make_tmap_mn3d(&tmBh, cchunk, bf16, a.D, a.vc_len, a.D, kStatTile, 2 * BN / 64)) {
    epi.wide = 1;
    sc.num_n = (int)ceil_div(ceil_div(a.D, BN), 2);
    sc.num_kb = (int)ceil_div(a.vc_len, kStatTile);
    if (push != nullptr) epi.total_units = (unsigned)sc.units();
  } else {
    epi.half_k = (a_half && half_k_enabled() &&
                  make_tmap_mn3d(&tmBh, cchunk, bf16, a.D, a.vc_len, a.D, BK / 2, BN / 64))
                     ? 1 : 0;
  }
  return launch_gemm<false, true>(tmA, tmB, tmAh, tmBh, tmC, sc, epi, bf16, s);
}

template <typename T>
cudaError_t grad_c_launch(const BwdChunkArgs& a, void* grad_c, cudaStream_t s) {
  const bool bf16 = std::is_same<T, __nv_bfloat16>::value;
  CUtensorMap tmA, tmB;
  int a3d = 0, b3d = 0;
  if (!make_tmap_mn(&tmA, a.dlogits, bf16, a.vc_len, a.N, a.vc_ld, BM / 64, &a3d)) return cudaErrorInvalidValue;
  if (!make_tmap_mn(&tmB, a.e, bf16, a.D, a.N, a.D, (BN) / 64, &b3d)) return cudaErrorInvalidValue;
  Sched sc{(int)ceil_div(a.vc_len, BM), (int)ceil_div(a.D, BN), (int)ceil_div(a.N, BK), 0, a3d, b3d,
           a.counters ? a.counters + 2 : nullptr, raster_group(a.N * a.D * 2)};
  GradCEpi<T> epi{static_cast<T*>(grad_c) + a.vc0 * a.D, a.scale,
                  a.keep_t + (a.vc0 / 128) * a.keep_t_ld, a.keep_t_ld,
                  (int)ceil_div(a.vc_len, (int64_t)128), (int)ceil_div(a.N, kRowBlock),
                  a.vc_len, a.D};
  epi.pair = grad_c_pair_ld() ? 1 : 0;
  CUtensorMap tmC;
  if (!make_tmap_out(&tmC, static_cast<uint16_t*>(grad_c) + a.vc0 * a.D, a.dtype, a.D, a.vc_len, a.D))
    return cudaErrorInvalidValue;
  return launch_gemm<true, true>(tmA, tmB, tmA, tmB, tmC, sc, epi, bf16, s);
}

}  // namespace

cudaError_t tc_grad_e(const BwdChunkArgs& a, float* acc2, bool accumulate, const PeerPush* push, cudaStream_t s) {
  if (a.N == 0 || a.D == 0) return cudaSuccess;
  if (a.dtype == CCE_BF16) return grad_e_launch<__nv_bfloat16>(a, acc2, accumulate, push, s);
  if (a.dtype == CCE_F16) return grad_e_launch<__half>(a, acc2, accumulate, push, s);
  return cudaErrorNotSupported;
}

cudaError_t tc_grad_c(const BwdChunkArgs& a, void* grad_c, cudaStream_t s) {
  if (a.vc_len == 0 || a.D == 0) return cudaSuccess;
  if (a.dtype == CCE_BF16) return grad_c_launch<__nv_bfloat16>(a, grad_c, s);
  if (a.dtype == CCE_F16) return grad_c_launch<__half>(a, grad_c, s);
  return cudaErrorNotSupported;
}

namespace {

// Diagnostic: one thread waits on a fresh mbarrier whose phase nothing
// completes, so the bounded wait runs out after limit_ns, records `code` in
// the status word and returns -- the path every pipeline wait takes when an
// arrival is lost.
__global__ void selftest_wait_kernel(uint64_t limit_ns, int code) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_barrier_init();
    (void)mbar_wait(&bar, 0, code, limit_ns);
  }
}

}  // namespace

cudaError_t tc_selftest_wait(uint64_t limit_ns, int code, cudaStream_t s) {
  selftest_wait_kernel<<<1, 32, 0, s>>>(limit_ns, code);
  return launched();
}

int tc_read_mma_flops(uint64_t* out4, bool reset) {
  unsigned long long v[4];
  if (cudaMemcpyFromSymbol(v, g_mma_cols, sizeof(v)) != cudaSuccess) return -1;
  for (int k = 0; k < 4; ++k) out4[k] = (uint64_t)v[k] * 2ull * 128ull * 16ull;
  if (reset) {
    const unsigned long long z[4] = {0, 0, 0, 0};
    if (cudaMemcpyToSymbol(g_mma_cols, z, sizeof(z)) != cudaSuccess) return -1;
  }
  return 0;
}

int tc_read_status(bool reset) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_status, sizeof(int)) != cudaSuccess) return -1;
  if (reset && v != 0) {
    const int z = 0;
    cudaMemcpyToSymbol(g_status, &z, sizeof(int));
  }
  return v;
}

}  // namespace cce
