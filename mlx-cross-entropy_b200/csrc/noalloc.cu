// cce_forward_noalloc: the forward pass for callers that cannot allocate
// device memory.
//
// cce_forward needs a workspace (the per-(vocabulary tile, row) sum-exp
// partials that the LSE fold reads) which the caller allocates.  Some callers
// have no way to do that: a host that hands the loss only its input and output
// buffers (a plugin or FFI slot with a fixed memory contract, a framework
// hook that forbids allocation while it executes), or code that must not
// allocate at all.  For them the partials live in a fixed device array owned
// by this library.
//
// The array is a file-scope __device__ symbol of kMaxScratchFloats floats
// (32 MiB): every GPU that loads the library holds it until the process
// exits, whether or not this entry point is used.  Host code cannot use the
// symbol's name as a device address, so the address is looked up with
// cudaGetSymbolAddress (the set-up below) and passed to the kernels as their
// workspace pointer.  An address belongs to a CUDA context, not to a device
// ordinal: a host that drives its own driver-API context, or that reset the
// device and so got a new primary context, needs a fresh lookup.  The cache
// is therefore keyed by the current context's process-unique id
// (cuCtxGetId), so the lookup runs once per context.
#include <cstdio>
#include <mutex>

#include "kernels.cuh"

namespace {

// Capacity in floats: the forward's LSE partials, 2 * ceil(V / 128) * N, must
// not exceed it (e.g. V = 128256 with N up to 4185, or V = 256000 with N up
// to 2097).
constexpr int64_t kMaxScratchFloats = 8ll << 20;

static __device__ __align__(256) float g_fwd_scratch[kMaxScratchFloats];

struct ScratchEntry {
  unsigned long long ctx_id;
  float* ptr;
};
constexpr int kCacheSlots = 64;
ScratchEntry g_cache[kCacheSlots];  // guarded by g_cache_mu; ids are never reused in a process
int g_cache_next = 0;
std::mutex g_cache_mu;

// Device address of g_fwd_scratch in the current context (looked up on the
// first call in each context, then cached).
int scratch_address(float** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess)
    return cce::report_error(CCE_ERR_CUDA, "cce_forward_noalloc: cudaGetDevice failed");
  unsigned long long id = 0;
  if (!cce::current_context_id(&id))
    return cce::report_error(CCE_ERR_CUDA, "cce_forward_noalloc: could not read the current CUDA context");
  std::lock_guard<std::mutex> lock(g_cache_mu);
  if (id != 0) {
    for (int i = 0; i < kCacheSlots; ++i)
      if (g_cache[i].ctx_id == id && g_cache[i].ptr != nullptr) {
        *out = g_cache[i].ptr;
        return CCE_OK;
      }
  }
  // Miss: the runtime call below also makes the device's primary context
  // current when no context was current yet.
  float* p = nullptr;
  const cudaError_t err = cudaGetSymbolAddress(reinterpret_cast<void**>(&p), g_fwd_scratch);
  if (err != cudaSuccess || p == nullptr)
    return cce::report_error(CCE_ERR_CUDA,
                             "cce_forward_noalloc: cudaGetSymbolAddress of the static scratch failed");
  if (id == 0 && !cce::current_context_id(&id))
    return cce::report_error(CCE_ERR_CUDA, "cce_forward_noalloc: could not read the current CUDA context");
  if (id != 0) {
    g_cache[g_cache_next] = ScratchEntry{id, p};
    g_cache_next = (g_cache_next + 1) % kCacheSlots;
  }
  *out = p;
  return CCE_OK;
}

}  // namespace

extern "C" {

int cce_forward_noalloc(const void* e, const void* c, const void* bias, int bias_dtype,
                        const int32_t* targets, int64_t N, int64_t D, int64_t V, int64_t v_offset,
                        int dtype, float* tile_max, float* lse, float* tgt, void* stream) {
  if (N < 0 || V < 0) return cce::report_error(CCE_ERR_SHAPE, "cce_forward_noalloc: negative size");
  const int64_t need = (int64_t)(cce_forward_workspace_bytes(N, D, V, dtype) / sizeof(float));
  if (need > kMaxScratchFloats) {
    char msg[256];
    snprintf(msg, sizeof(msg),
             "cce_forward_noalloc: 2 * ceil(V/128) * N = %lld partials exceed the static scratch of "
             "%lld floats (32 MiB); use cce_forward with a caller-allocated workspace",
             (long long)need, (long long)kMaxScratchFloats);
    return cce::report_error(CCE_ERR_WORKSPACE, msg);
  }
  float* scratch = nullptr;
  const int rc = scratch_address(&scratch);
  if (rc != CCE_OK) return rc;
  // Every partial the LSE fold reads is written by the forward kernel of the
  // same call first, so the array needs no clearing between calls.
  return cce_forward(e, c, bias, bias_dtype, targets, N, D, V, v_offset, dtype, tile_max, lse, tgt,
                     scratch, (size_t)kMaxScratchFloats * sizeof(float), stream);
}

}  // extern "C"
