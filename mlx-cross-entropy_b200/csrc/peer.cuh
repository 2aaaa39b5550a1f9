// The exchange buffer of the vocabulary-sharded backward and the device-side
// signalling shared by the grad_e push epilogue (tc_kernels.cu) and the
// exchange kernels (peer.cu).
//
// Every rank owns one buffer, allocated once per process group and mapped into
// every other rank's process (driver virtual memory shared through a file
// descriptor), so each rank reaches every buffer
// with plain loads and stores over NVLink:
//
//   [0, 4 KB)        control block (flags and counters, below)
//   recv             [world][2][R][D] fp32: slot (src, s) holds rank src's
//                    partial grad_e (K-split slab s) for the rows this rank owns
//   reduced          [R][D] in the output dtype: this rank's rows of the summed
//                    grad_e, read by every other rank
//
// Rows are owned in whole 128-row M tiles: rank p owns the rows of M tiles
// [p * mt_per, (p + 1) * mt_per), i.e. rows [p * R, min((p + 1) * R, N)) with
// R = 128 * mt_per and mt_per = ceil(ceil(N / 128) / world).
//
// Signalling: a writer publishes its stores with a system-scope fence, counts
// itself on a local counter, and the last writer of a launch raises a flag in
// every rank's control block with a release store; a reader acquires the flag
// before touching the data.  Flags carry the exchange's epoch (the rank's
// exchange count, advanced on the device by the last pushing writer), so they
// are never cleared and a CUDA graph replay gets a fresh epoch each time.
#pragma once

#include "common.cuh"

namespace cce {
namespace peer {

constexpr int kMaxWorld = CCE_PEER_MAX_WORLD;
constexpr int kRows = 128;  // ownership granularity: one M tile of the grad_e GEMM

// Control block offsets (bytes from the buffer's base); each on its own 128-byte line.
constexpr size_t kEpochOff = 0;          // u64: this rank's exchange count (local only)
constexpr size_t kDoneUnitsOff = 128;    // u32: pushing units / CTAs of the current launch done
constexpr size_t kDoneReduceOff = 256;   // u32: reduce CTAs of the current launch done
constexpr size_t kPushedOff = 512;       // u64[kMaxWorld]: pushed[src] = epoch of src's last push here
constexpr size_t kReducedOff = 1024;     // u64[kMaxWorld]: reduced[src] = epoch of src's last reduce
constexpr size_t kCtrlBytes = 4096;
constexpr int kSlotsPerSrc = 2;          // the grad_e GEMM's two K-split slabs

struct Layout {
  int64_t mt_per;      // M tiles per owner
  int64_t R;           // rows per owner = kRows * mt_per
  size_t recv_off;     // recv slots
  size_t reduced_off;  // reduced rows
  size_t bytes;        // whole buffer
};

__host__ __device__ inline Layout make_layout(int64_t N, int64_t D, int world, int out_esize) {
  Layout L;
  const int64_t mt = ceil_div(N > 0 ? N : 1, kRows);
  L.mt_per = ceil_div(mt, world);
  L.R = L.mt_per * kRows;
  L.recv_off = kCtrlBytes;
  const size_t recv = (size_t)world * kSlotsPerSrc * (size_t)L.R * (size_t)D * 4;
  L.reduced_off = L.recv_off + (size_t)round_up((int64_t)recv, 256);
  L.bytes = L.reduced_off + (size_t)round_up((int64_t)((size_t)L.R * (size_t)D * out_esize), 256);
  return L;
}

// The ranks' buffers as mapped in this process (bases[rank] is this rank's own).
struct Peers {
  char* bases[kMaxWorld];
  int rank, world;
};

__device__ __forceinline__ void st_release_sys(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ unsigned long long* flag(char* base, size_t off, int src) {
  return reinterpret_cast<unsigned long long*>(base + off) + src;
}

// One thread per writer (a grad_e unit or a CTA), after all of the writer's
// threads have finished their stores (bar.sync before the call): publishes
// them and counts the writer on `counter_off`.  The last of `total` writers of
// the launch resets the counter for the next launch, takes the epoch (advanced
// by one when `advance`), and raises flag[rank] at `flag_off` on every rank.
__device__ __forceinline__ void arrive_and_signal(const Peers& P, size_t counter_off, unsigned total,
                                                  bool advance, size_t flag_off) {
  char* own = P.bases[P.rank];
  unsigned* counter = reinterpret_cast<unsigned*>(own + counter_off);
  __threadfence_system();
  if (atomicAdd(counter, 1u) != total - 1u) return;
  *counter = 0u;
  unsigned long long* ep = reinterpret_cast<unsigned long long*>(own + kEpochOff);
  unsigned long long e = *ep;
  if (advance) {
    e += 1ull;
    *ep = e;
  }
  __threadfence_system();
  for (int p = 0; p < P.world; ++p) st_release_sys(flag(P.bases[p], flag_off, P.rank), e);
}

}  // namespace peer
}  // namespace cce
