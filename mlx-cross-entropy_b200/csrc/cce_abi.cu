// C-ABI layer: argument validation, workspace carving and kernel dispatch.
//
// Mirrors the host side of the reference's op layer: shape / dtype checks of
// csrc/cce/cce.cpp:41-73 (returned as status codes instead of thrown
// exceptions), output and zero-fill set-up of cce.cpp:243-246 and :316-340,
// and the dtype-keyed kernel choice of cce.cpp:221-231, :300-310.
#include <cuda.h>

#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <unordered_map>

#include "kernels.cuh"

namespace cce {

std::atomic<uint64_t> g_launches{0};

cudaError_t launched() {
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return cudaGetLastError();
}

namespace {

template <typename Fn>
Fn driver_fn(const char* name) {
  void* p = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint(name, &p, cudaEnableDefault, &q) != cudaSuccess || q != cudaDriverEntryPointSuccess)
    return nullptr;
  return reinterpret_cast<Fn>(p);
}

}  // namespace

bool current_context_id(unsigned long long* id) {
  using GetCurrentFn = CUresult (*)(CUcontext*);
  using GetIdFn = CUresult (*)(CUcontext, unsigned long long*);
  static const GetCurrentFn get_cur = driver_fn<GetCurrentFn>("cuCtxGetCurrent");
  static const GetIdFn get_id = driver_fn<GetIdFn>("cuCtxGetId");
  if (!get_cur || !get_id) return false;
  CUcontext ctx = nullptr;
  if (get_cur(&ctx) != CUDA_SUCCESS) return false;
  *id = 0;
  if (ctx == nullptr) return true;
  return get_id(ctx, id) == CUDA_SUCCESS;
}

}  // namespace cce

namespace {

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int cuda_fail(cudaError_t err, const char* where) {
  return fail(CCE_ERR_CUDA, "%s: CUDA error %d (%s)", where, (int)err, cudaGetErrorString(err));
}

#define CCE_CUDA_CHECK(expr, where)          \
  do {                                       \
    cudaError_t _e = (expr);                 \
    if (_e != cudaSuccess) return cuda_fail(_e, where); \
  } while (0)

constexpr size_t kAlign = 256;
// dlogits chunk buffer: aim for 32768 vocabulary rows per chunk within 128 MiB
// to 1 GiB of buffer.  Every chunk costs three kernel launches whatever its
// work (~70 us at N = 2048 when the filter rejects nearly every block), so
// N below 4096 grows its chunks up to 512 MiB of buffer, but never past half
// of the vocabulary: the buffer stays below half of the [N, V] logits, the
// memory bound of the whole method.  Measured on B200: config 3 (N = 4096)
// backward 8.71 ms at 16384 rows, 8.35 at 32768, 8.42 at 65536, 8.62 at
// 131072 (and, with the current grad_e, whole steps equal at 32768 and
// 65536 rows); config 4 (N = 2048) 1.44 ms in 8 chunks, 1.15 in 4, 1.01 in 2
// (whole steps 2.76 ms in 4 chunks, 2.63 in 2); config 2 (N = 1024) in 2
// chunks.  (Two buffers, so that a chunk's dlogits overlap the previous
// chunk's grads, measured no faster.)
constexpr int64_t kDlTargetRows = 32768;
constexpr int64_t kDlMaxBytes = 1ll << 30;
constexpr int64_t kDlMinBytes = 128ll << 20;
constexpr int64_t kDlSmallNBytes = 256ll << 20;  // N below this many bytes per 32768 rows is "small"
constexpr int64_t kDlSmallNGrowBytes = 512ll << 20;

size_t align_up(size_t x) { return (x + kAlign - 1) / kAlign * kAlign; }

bool dtype_ok(int d) { return d == CCE_F32 || d == CCE_F16 || d == CCE_BF16; }
size_t dtype_size(int d) { return d == CCE_F32 ? 4 : 2; }

std::atomic<int> g_arch[64];

int check_arch() {
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return cuda_fail(err, "cudaGetDevice");
  if (dev < 0 || dev >= 64) return CCE_OK;
  int cc = g_arch[dev].load(std::memory_order_relaxed);
  if (cc == 0) {
    int major = 0, minor = 0;
    err = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    if (err != cudaSuccess) return cuda_fail(err, "cudaDeviceGetAttribute");
    err = cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
    if (err != cudaSuccess) return cuda_fail(err, "cudaDeviceGetAttribute");
    cc = major * 10 + minor;
    g_arch[dev].store(cc, std::memory_order_relaxed);
  }
  if (cc != 100)
    return fail(CCE_ERR_ARCH, "device %d has compute capability %d.%d; this library is built for sm_100a (B200)",
                dev, cc / 10, cc % 10);
  return CCE_OK;
}

// Vocabulary rows per backward chunk and whether the tensor-core path runs.
struct BwdPlan {
  bool tc;
  int64_t vc;        // chunk rows (also the dlogits row stride)
  size_t keep_bytes, dl_bytes, acc_bytes, counter_bytes, scale_bytes;
  int64_t keep_t_ld;     // words per row of the transposed table (tensor-core path)
  size_t keep_t_bytes;
  int splits;            // CUDA-core path: K splits of grad_e (partials part_bytes)
  size_t part_bytes;
  size_t list_bytes;     // tensor-core path: the dlogits live-tile lists of every chunk
};

bool tc_candidate(int dtype, int64_t D) { return dtype != CCE_F32 && D % 8 == 0; }

// CCE_BWD_CHUNK_ROWS=<rows> in the environment overrides the target rows per
// backward vocabulary chunk (a tuning knob, also used by the tests to force
// several chunks; read on every call; the 1 GiB cap still applies, the 512 MiB
// floor does not).
int64_t target_chunk_rows() {
  const char* s = getenv("CCE_BWD_CHUNK_ROWS");
  const long long r = s ? atoll(s) : 0;
  return r >= 256 ? (int64_t)r : kDlTargetRows;
}

// CCE_DL_LIST=0 in the environment: the dlogits GEMM claims every tile id and
// passes over the dead ones instead of claiming from a list of live tiles
// (an A/B switch; read once, since it sizes the workspace).
bool dl_list_enabled() {
  static const bool v = [] {
    const char* s = getenv("CCE_DL_LIST");
    return !(s != nullptr && s[0] == '0');
  }();
  return v;
}

BwdPlan plan_backward(int64_t N, int64_t D, int64_t V, int dtype, int flags, bool tc) {
  BwdPlan p{};
  p.tc = tc;
  const int64_t gran = tc ? 256 : 128;
  const int64_t elt = tc ? 2 : 4;
  const int64_t nrow = N > 0 ? N : 1;
  const int64_t target = target_chunk_rows();
  // the budget is in 16-bit bytes for both paths (the CUDA-core path's fp32
  // dlogits get half the rows), so neither plan's workspace dominates the other's
  int64_t budget = nrow * 2 * target;
  if (budget > kDlMaxBytes) budget = kDlMaxBytes;
  if (budget < kDlMinBytes && target == kDlTargetRows) budget = kDlMinBytes;
  int64_t vc = (budget / (nrow * elt)) / gran * gran;
  if (vc < gran) vc = gran;
  if (target == kDlTargetRows && nrow * 2 * target < kDlSmallNBytes) {
    // small N: longer chunks, up to 512 MiB and half the vocabulary
    const int64_t half = cce::round_up(cce::ceil_div(V > 0 ? V : 1, 2), gran);
    int64_t grow = (kDlSmallNGrowBytes / (nrow * elt)) / gran * gran;
    if (grow > half) grow = half;
    if (grow > vc) vc = grow;
  }
  const int64_t vmax = cce::round_up(V > 0 ? V : 1, gran);
  if (vc > vmax) vc = vmax;
  p.vc = vc;
  p.keep_bytes = align_up((size_t)cce::ceil_div(N, cce::kRowBlock) * (size_t)cce::ceil_div(V, cce::kStatTile));
  // grad_c's view of the mask: per 128-column tile a bit per row block
  p.keep_t_ld = tc ? cce::ceil_div(cce::ceil_div(N, cce::kRowBlock), 32) : 0;
  p.keep_t_bytes = tc ? align_up((size_t)cce::ceil_div(V, 128) * (size_t)p.keep_t_ld * 4) : 0;
  p.dl_bytes = align_up((size_t)N * (size_t)vc * (size_t)elt);
  // grad_e accumulators: the tensor-core path keeps two fp32 slabs [2][N][D]
  // (the two K halves of every chunk's grad_e GEMM), summed into grad_e at the
  // end; the SIMT path one [N][D] (none when grad_e itself is fp32).
  if (!(flags & CCE_NEED_DE)) p.acc_bytes = 0;
  else if (tc) p.acc_bytes = align_up(2 * (size_t)N * (size_t)D * 4);
  else p.acc_bytes = (flags & CCE_DE_F32) ? 0 : align_up((size_t)N * (size_t)D * 4);
  // four counters per vocabulary chunk: the tile claims of the three
  // dynamically scheduled kernels and the dlogits live-tile count
  const int64_t nch = cce::ceil_div(V > 0 ? V : 1, vc);
  p.counter_bytes = align_up((size_t)nch * 4 * sizeof(int));
  p.list_bytes = (tc && dl_list_enabled()) ? align_up((size_t)nch * (size_t)cce::tc_dlogits_list_len(nrow, vc) * sizeof(int)) : 0;
  p.scale_bytes = (tc && dtype == CCE_F16) ? kAlign : 0;  // {s, 1/s} for fp16 dlogits
  p.splits = (!tc && (flags & CCE_NEED_DE)) ? cce::simt_grad_e_splits(N, D, vc) : 1;
  p.part_bytes = p.splits > 1 ? align_up((size_t)p.splits * (size_t)N * (size_t)D * 4) : 0;
  return p;
}

size_t plan_bytes(const BwdPlan& p) {
  return p.keep_bytes + p.dl_bytes + p.acc_bytes + p.counter_bytes + p.scale_bytes + p.keep_t_bytes + p.part_bytes +
         p.list_bytes;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// CCE_FORCE_SIMT=1 in the environment routes every call to the CUDA-core
// kernels (used by the tests to compare both kernel families).
bool force_simt() {
  static const bool v = [] {
    const char* s = getenv("CCE_FORCE_SIMT");
    return s != nullptr && s[0] == '1';
  }();
  return v;
}

int check_sizes(int64_t N, int64_t D, int64_t V, int dtype) {
  if (N < 0 || D <= 0 || V < 0) return fail(CCE_ERR_SHAPE, "bad sizes N=%lld D=%lld V=%lld", (long long)N, (long long)D, (long long)V);
  if (N > (1ll << 31) || V > (1ll << 31) || D > (1ll << 20))
    return fail(CCE_ERR_SHAPE, "sizes out of supported range N=%lld D=%lld V=%lld", (long long)N, (long long)D, (long long)V);
  if (!dtype_ok(dtype)) return fail(CCE_ERR_DTYPE, "unsupported dtype code %d", dtype);
  return CCE_OK;
}

// Side streams of the tensor-core backward: grad_e and grad_c of one chunk run
// concurrently (grad_e on the higher-priority stream, launched first), so
// grad_c's CTAs take the SMs that grad_e's last partial wave leaves idle.
// One set per (host thread, device), tagged with the CUDA context it was
// created in: a set from another context (the host's own driver-API context,
// or a primary context since reset) is replaced, not used.  Created on first
// use, never destroyed (a replaced set is left to its context).
struct SideStreams {
  unsigned long long ctx_id = 0;
  cudaStream_t se = nullptr, sc = nullptr;
  cudaStream_t sq = nullptr;  // dequantisation of a quantised head's next chunk
  cudaEvent_t start = nullptr, ev_l = nullptr, ev_e = nullptr, ev_c = nullptr;
  cudaEvent_t ev_q[2] = {nullptr, nullptr};  // chunk buffer b holds its dequantised chunk
  cudaEvent_t ev_r = nullptr;                // the other chunk buffer's readers are done
};

thread_local SideStreams g_side[64];

int side_streams(SideStreams** out) {
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return cuda_fail(err, "cudaGetDevice");
  if (dev < 0 || dev >= 64) return fail(CCE_ERR_CUDA, "device ordinal %d out of range", dev);
  unsigned long long ctx = 0;
  if (!cce::current_context_id(&ctx)) return fail(CCE_ERR_CUDA, "could not read the current CUDA context");
  SideStreams& ss = g_side[dev];
  if (ss.se == nullptr || ss.ctx_id != ctx) {
    int lo = 0, hi = 0;
    err = cudaDeviceGetStreamPriorityRange(&lo, &hi);
    if (err != cudaSuccess) return cuda_fail(err, "cudaDeviceGetStreamPriorityRange");
    SideStreams n;
    if ((err = cudaStreamCreateWithPriority(&n.se, cudaStreamNonBlocking, hi)) != cudaSuccess ||
        (err = cudaStreamCreateWithPriority(&n.sc, cudaStreamNonBlocking, lo)) != cudaSuccess ||
        (err = cudaStreamCreateWithPriority(&n.sq, cudaStreamNonBlocking, lo)) != cudaSuccess ||
        (err = cudaEventCreateWithFlags(&n.start, cudaEventDisableTiming)) != cudaSuccess ||
        (err = cudaEventCreateWithFlags(&n.ev_l, cudaEventDisableTiming)) != cudaSuccess ||
        (err = cudaEventCreateWithFlags(&n.ev_e, cudaEventDisableTiming)) != cudaSuccess ||
        (err = cudaEventCreateWithFlags(&n.ev_c, cudaEventDisableTiming)) != cudaSuccess ||
        (err = cudaEventCreateWithFlags(&n.ev_q[0], cudaEventDisableTiming)) != cudaSuccess ||
        (err = cudaEventCreateWithFlags(&n.ev_q[1], cudaEventDisableTiming)) != cudaSuccess ||
        (err = cudaEventCreateWithFlags(&n.ev_r, cudaEventDisableTiming)) != cudaSuccess)
      return cuda_fail(err, "creating the backward side streams");
    // creating them made a context current if none was
    if (!cce::current_context_id(&n.ctx_id)) return fail(CCE_ERR_CUDA, "could not read the current CUDA context");
    ss = n;
  }
  *out = &ss;
  return CCE_OK;
}

// ---- exchange buffers: driver virtual-memory API ----
//
// Each buffer is a physical allocation (cuMemCreate) exportable as a POSIX
// file descriptor, mapped into a reserved virtual range with access for the
// local device only.  A peer process imports the descriptor and maps the same
// physical memory into its own range, again with access for its own device.
// Unlike CUDA IPC this turns on no context-wide peer access, which would make
// every later cudaMalloc of the process map its memory into the peer device
// (measured: ~5 ms per new allocator segment on B200).

struct VmmApi {
  using CreateFn = CUresult (*)(CUmemGenericAllocationHandle*, size_t, const CUmemAllocationProp*, unsigned long long);
  using ReleaseFn = CUresult (*)(CUmemGenericAllocationHandle);
  using ReserveFn = CUresult (*)(CUdeviceptr*, size_t, size_t, CUdeviceptr, unsigned long long);
  using AddrFreeFn = CUresult (*)(CUdeviceptr, size_t);
  using MapFn = CUresult (*)(CUdeviceptr, size_t, size_t, CUmemGenericAllocationHandle, unsigned long long);
  using UnmapFn = CUresult (*)(CUdeviceptr, size_t);
  using SetAccessFn = CUresult (*)(CUdeviceptr, size_t, const CUmemAccessDesc*, size_t);
  using ExportFn = CUresult (*)(void*, CUmemGenericAllocationHandle, CUmemAllocationHandleType, unsigned long long);
  using ImportFn = CUresult (*)(CUmemGenericAllocationHandle*, void*, CUmemAllocationHandleType);
  using GranFn = CUresult (*)(size_t*, const CUmemAllocationProp*, CUmemAllocationGranularity_flags);
  CreateFn create = nullptr;
  ReleaseFn release = nullptr;
  ReserveFn reserve = nullptr;
  AddrFreeFn addr_free = nullptr;
  MapFn map = nullptr;
  UnmapFn unmap = nullptr;
  SetAccessFn set_access = nullptr;
  ExportFn export_fd = nullptr;
  ImportFn import_fd = nullptr;
  GranFn granularity = nullptr;
  bool ok = false;
};

template <typename Fn>
Fn entry(const char* name) {
  void* p = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint(name, &p, cudaEnableDefault, &q) != cudaSuccess || q != cudaDriverEntryPointSuccess)
    return nullptr;
  return reinterpret_cast<Fn>(p);
}

const VmmApi& vmm_api() {
  static const VmmApi api = [] {
    VmmApi a;
    a.create = entry<VmmApi::CreateFn>("cuMemCreate");
    a.release = entry<VmmApi::ReleaseFn>("cuMemRelease");
    a.reserve = entry<VmmApi::ReserveFn>("cuMemAddressReserve");
    a.addr_free = entry<VmmApi::AddrFreeFn>("cuMemAddressFree");
    a.map = entry<VmmApi::MapFn>("cuMemMap");
    a.unmap = entry<VmmApi::UnmapFn>("cuMemUnmap");
    a.set_access = entry<VmmApi::SetAccessFn>("cuMemSetAccess");
    a.export_fd = entry<VmmApi::ExportFn>("cuMemExportToShareableHandle");
    a.import_fd = entry<VmmApi::ImportFn>("cuMemImportFromShareableHandle");
    a.granularity = entry<VmmApi::GranFn>("cuMemGetAllocationGranularity");
    a.ok = a.create && a.release && a.reserve && a.addr_free && a.map && a.unmap && a.set_access &&
           a.export_fd && a.import_fd && a.granularity;
    return a;
  }();
  return api;
}

CUmemAllocationProp device_prop(int dev) {
  CUmemAllocationProp prop;
  memset(&prop, 0, sizeof(prop));
  prop.type = CU_MEM_ALLOCATION_TYPE_PINNED;
  prop.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
  prop.location.id = dev;
  prop.requestedHandleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
  return prop;
}

void unmap(const VmmApi& api, CUdeviceptr va, size_t size) {
  api.unmap(va, size);
  api.addr_free(va, size);
}

// Reserve a range, map `h` into it and give the local device read/write access.
int map_local(const VmmApi& api, CUmemGenericAllocationHandle h, size_t size, int dev, CUdeviceptr* out) {
  CUdeviceptr va = 0;
  CUresult r = api.reserve(&va, size, 0, 0, 0);
  if (r != CUDA_SUCCESS) return fail(CCE_ERR_CUDA, "cuMemAddressReserve of %zu bytes failed (%d)", size, (int)r);
  if ((r = api.map(va, size, 0, h, 0)) != CUDA_SUCCESS) {
    api.addr_free(va, size);
    return fail(CCE_ERR_CUDA, "cuMemMap failed (%d)", (int)r);
  }
  CUmemAccessDesc acc;
  memset(&acc, 0, sizeof(acc));
  acc.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
  acc.location.id = dev;
  acc.flags = CU_MEM_ACCESS_FLAGS_PROT_READWRITE;
  if ((r = api.set_access(va, size, &acc, 1)) != CUDA_SUCCESS) {
    unmap(api, va, size);
    return fail(CCE_ERR_CUDA, "cuMemSetAccess failed (%d)", (int)r);
  }
  *out = va;
  return CCE_OK;
}

// Mapped exchange buffers of this process: base address -> (handle, size).
struct Mapping {
  CUmemGenericAllocationHandle handle;
  size_t size;
};
std::mutex g_maps_mu;
std::unordered_map<uintptr_t, Mapping> g_maps;

void remember(CUdeviceptr va, CUmemGenericAllocationHandle h, size_t size) {
  std::lock_guard<std::mutex> lock(g_maps_mu);
  g_maps[(uintptr_t)va] = Mapping{h, size};
}

int forget_and_unmap(void* ptr, const char* what) {
  Mapping m;
  {
    std::lock_guard<std::mutex> lock(g_maps_mu);
    auto it = g_maps.find(reinterpret_cast<uintptr_t>(ptr));
    if (it == g_maps.end()) return fail(CCE_ERR_ARG, "%s: %p is not a mapped exchange buffer", what, ptr);
    m = it->second;
    g_maps.erase(it);
  }
  const VmmApi& api = vmm_api();
  const CUdeviceptr va = reinterpret_cast<CUdeviceptr>(ptr);
  const CUresult r1 = api.unmap(va, m.size);
  const CUresult r2 = api.addr_free(va, m.size);
  const CUresult r3 = api.release(m.handle);
  if (r1 != CUDA_SUCCESS || r2 != CUDA_SUCCESS || r3 != CUDA_SUCCESS)
    return fail(CCE_ERR_CUDA, "%s: unmapping failed (%d, %d, %d)", what, (int)r1, (int)r2, (int)r3);
  return CCE_OK;
}

}  // namespace

namespace cce {

// Records `msg` as this thread's cce_last_error() and returns `code`.
int report_error(int code, const char* msg) { return fail(code, "%s", msg); }

}  // namespace cce

extern "C" {

int cce_version(void) { return 100; }

const char* cce_last_error(void) { return g_last_error.c_str(); }

uint64_t cce_launch_count(void) { return cce::g_launches.load(std::memory_order_relaxed); }

int cce_device_status(int reset) {
  const int v = cce::tc_read_status(reset != 0);
  const int pv = cce::peer::read_status(reset != 0);
  if (v < 0 || pv < 0) return fail(CCE_ERR_CUDA, "cce_device_status: could not read the device status words");
  if (v > 0)
    return fail(CCE_ERR_CUDA, "a tensor-core kernel abandoned a pipeline wait after its time limit (code %d)", v);
  if (pv > 0)
    return fail(CCE_ERR_CUDA, "a grad_e exchange kernel gave up waiting for another rank (code %d)", pv);
  return CCE_OK;
}

int cce_mma_flops(uint64_t* flops4, int reset) {
  if (!flops4) return fail(CCE_ERR_ARG, "cce_mma_flops: NULL output");
  if (cce::tc_read_mma_flops(flops4, reset != 0) != 0)
    return fail(CCE_ERR_CUDA, "cce_mma_flops: could not read the device counters");
  return CCE_OK;
}

int cce_selftest_wait_timeout(int64_t limit_ns, void* stream) {
  if (limit_ns <= 0 || limit_ns > 2000000000ll)
    return fail(CCE_ERR_ARG, "cce_selftest_wait_timeout: limit_ns must be in (0, 2e9], got %lld", (long long)limit_ns);
  int rc = check_arch();
  if (rc) return rc;
  CCE_CUDA_CHECK(cce::tc_selftest_wait((uint64_t)limit_ns, CCE_SELFTEST_WAIT_CODE, (cudaStream_t)stream),
                 "cce_selftest_wait_timeout");
  return CCE_OK;
}

int64_t cce_num_stat_tiles(int64_t V) { return V <= 0 ? 0 : cce::ceil_div(V, cce::kStatTile); }

// A quantised head's arguments are usable for rows of width D.
static int check_head(const CceQuantHead* h, int64_t D, const char* what) {
  if (!h || !h->wq || !h->scales || !h->biases) return fail(CCE_ERR_ARG, "%s: NULL quantised-head pointer", what);
  if (h->bits != 2 && h->bits != 4 && h->bits != 8)
    return fail(CCE_ERR_ARG, "%s: bits must be 2, 4 or 8, got %d", what, h->bits);
  if (h->group_size != 32 && h->group_size != 64 && h->group_size != 128)
    return fail(CCE_ERR_ARG, "%s: group_size must be 32, 64 or 128, got %d", what, h->group_size);
  if (D % h->group_size != 0)
    return fail(CCE_ERR_SHAPE, "%s: D=%lld is not a multiple of group_size=%d", what, (long long)D, h->group_size);
  if (!dtype_ok(h->scale_dtype)) return fail(CCE_ERR_DTYPE, "%s: scale dtype code %d", what, h->scale_dtype);
  return CCE_OK;
}

// Rows [v0, v0 + rows) of a quantised head expanded into `out` (dtype), on `s`.
static cudaError_t dequant_rows(const CceQuantHead* h, int64_t v0, int64_t rows, int64_t D, int dtype, void* out,
                         cudaStream_t s) {
  const int64_t wpr = D * h->bits / 32;
  const int64_t gpr = D / h->group_size;
  const size_t ssz = dtype_size(h->scale_dtype);
  return cce::launch_dequantize(h->wq + v0 * wpr, static_cast<const char*>(h->scales) + v0 * gpr * ssz,
                                static_cast<const char*>(h->biases) + v0 * gpr * ssz, h->scale_dtype, rows, D,
                                h->group_size, h->bits, dtype, out, s);
}

// Bytes of one chunk buffer of a quantised head's expanded rows.
static size_t chunk_buf_bytes(const BwdPlan& p, int64_t D, int dtype) {
  return align_up((size_t)p.vc * (size_t)D * dtype_size(dtype));
}

static size_t backward_ws_bytes(int64_t N, int64_t D, int64_t V, int dtype, int flags, bool quant) {
  const BwdPlan ps = plan_backward(N, D, V, dtype, flags, false);
  size_t b = plan_bytes(ps) + (quant ? 2 * chunk_buf_bytes(ps, D, dtype) : 0);
  if (tc_candidate(dtype, D)) {
    const BwdPlan pt = plan_backward(N, D, V, dtype, flags, true);
    const size_t t = plan_bytes(pt) + (quant ? 2 * chunk_buf_bytes(pt, D, dtype) : 0);
    if (t > b) b = t;
  }
  return b;
}

// The LSE partials (max, sum-exp) per row per kernel tile: 2 x ceil(V / 128) x N
// floats covers both kernel families (tensor-core tiles are 256 columns wide).
size_t cce_forward_workspace_bytes(int64_t N, int64_t D, int64_t V, int dtype) {
  (void)D;
  (void)dtype;
  const int64_t P = V > 0 ? cce::ceil_div(V, cce::kSimtLseTile) : 0;
  return align_up(2 * (size_t)P * (size_t)(N > 0 ? N : 0) * sizeof(float));
}

int cce_forward(const void* e, const void* c, const void* bias, int bias_dtype,
                const int32_t* targets, int64_t N, int64_t D, int64_t V, int64_t v_offset,
                int dtype, float* tile_max, float* lse, float* tgt, void* workspace,
                size_t workspace_bytes, void* stream) {
  int rc = check_sizes(N, D, V, dtype);
  if (rc) return rc;
  if (bias && !dtype_ok(bias_dtype)) return fail(CCE_ERR_DTYPE, "unsupported bias dtype code %d", bias_dtype);
  if (N == 0) return CCE_OK;
  if (V == 0) return fail(CCE_ERR_SHAPE, "V must be positive");
  if (!e || !c || !targets || !tile_max || !lse || !tgt)
    return fail(CCE_ERR_ARG, "cce_forward: NULL required pointer");
  const size_t need = cce_forward_workspace_bytes(N, D, V, dtype);
  if (!workspace || workspace_bytes < need)
    return fail(CCE_ERR_WORKSPACE, "cce_forward: workspace %zu bytes < required %zu", workspace_bytes, need);
  rc = check_arch();
  if (rc) return rc;
  cudaStream_t s = (cudaStream_t)stream;
  const bool tc = !force_simt() && cce::tc_supported(e, c, D, dtype);
  const int64_t P = cce::ceil_div(V, tc ? cce::kTcLseTile : cce::kSimtLseTile);
  float* part_m = (float*)workspace;
  float* part_s = part_m + P * N;
  cce::FwdArgs a{e, c, bias, bias_dtype, targets, N, D, V, v_offset, dtype, tile_max, part_m, part_s, tgt};
  // Rows whose target is not in this call's vocabulary range keep tgt = 0.
  CCE_CUDA_CHECK(cudaMemsetAsync(tgt, 0, (size_t)N * sizeof(float), s), "cce_forward memset");
  if (tc) {
    CCE_CUDA_CHECK(cce::tc_forward(a, s), "cce_forward tc kernel");
  } else {
    CCE_CUDA_CHECK(cce::simt_forward(a, s), "cce_forward simt kernel");
  }
  CCE_CUDA_CHECK(cce::launch_lse_combine(part_m, part_s, nullptr, P, N, N, lse, nullptr, nullptr, s),
                 "cce_forward combine");
  return CCE_OK;
}

// Rows of a quantised head expanded per forward chunk (two buffers).
// Config 3 with a 4-bit head, frozen, fwd + grad_e against the same step on
// the dense head: 1.09x at 32768 rows, 1.10-1.11x at 16384.
#ifndef CCE_FWDQ_ROWS
#define CCE_FWDQ_ROWS 32768
#endif
constexpr int64_t kFwdQuantChunkRows = CCE_FWDQ_ROWS;

static size_t forward_q_ws_bytes(int64_t N, int64_t D, int64_t V, int dtype) {
  const int64_t rows = V < kFwdQuantChunkRows ? (V > 0 ? V : 1) : kFwdQuantChunkRows;
  return cce_forward_workspace_bytes(N, D, V, dtype) + 2 * align_up((size_t)rows * (size_t)D * dtype_size(dtype));
}

size_t cce_forward_q_workspace_bytes(int64_t N, int64_t D, int64_t V, int dtype) {
  return forward_q_ws_bytes(N, D, V, dtype);
}

int cce_forward_q(const void* e, const CceQuantHead* head, const void* bias, int bias_dtype,
                  const int32_t* targets, int64_t N, int64_t D, int64_t V, int64_t v_offset, int dtype,
                  float* tile_max, float* lse, float* tgt, void* workspace, size_t workspace_bytes, void* stream) {
  int rc = check_sizes(N, D, V, dtype);
  if (rc) return rc;
  rc = check_head(head, D, "cce_forward_q");
  if (rc) return rc;
  if (bias && !dtype_ok(bias_dtype)) return fail(CCE_ERR_DTYPE, "unsupported bias dtype code %d", bias_dtype);
  if (N == 0) return CCE_OK;
  if (V == 0) return fail(CCE_ERR_SHAPE, "V must be positive");
  if (!e || !targets || !tile_max || !lse || !tgt) return fail(CCE_ERR_ARG, "cce_forward_q: NULL required pointer");
  const size_t need = forward_q_ws_bytes(N, D, V, dtype);
  if (!workspace || workspace_bytes < need)
    return fail(CCE_ERR_WORKSPACE, "cce_forward_q: workspace %zu bytes < required %zu", workspace_bytes, need);
  rc = check_arch();
  if (rc) return rc;
  cudaStream_t s = (cudaStream_t)stream;
  const size_t part_bytes = cce_forward_workspace_bytes(N, D, V, dtype);
  char* cbuf[2] = {(char*)workspace + part_bytes, nullptr};
  const int64_t vq = V < kFwdQuantChunkRows ? V : kFwdQuantChunkRows;
  cbuf[1] = cbuf[0] + align_up((size_t)vq * (size_t)D * dtype_size(dtype));
  const bool tc = !force_simt() && cce::tc_supported(e, cbuf[0], D, dtype);
  const int64_t ptile = tc ? cce::kTcLseTile : cce::kSimtLseTile;
  const int64_t P = cce::ceil_div(V, ptile);
  float* part_m = (float*)workspace;
  float* part_s = part_m + P * N;
  SideStreams* ss = nullptr;
  rc = side_streams(&ss);
  if (rc) return rc;
  CCE_CUDA_CHECK(cudaMemsetAsync(tgt, 0, (size_t)N * sizeof(float), s), "cce_forward_q memset");
  CCE_CUDA_CHECK(cudaEventRecord(ss->start, s), "cce_forward_q fork");
  CCE_CUDA_CHECK(cudaStreamWaitEvent(ss->sq, ss->start, 0), "cce_forward_q fork");
  CCE_CUDA_CHECK(dequant_rows(head, 0, vq, D, dtype, cbuf[0], ss->sq), "cce_forward_q dequantise");
  CCE_CUDA_CHECK(cudaEventRecord(ss->ev_q[0], ss->sq), "cce_forward_q record");
  const int64_t nchunks = cce::ceil_div(V, vq);
  const size_t bsz = bias ? dtype_size(bias_dtype) : 0;
  for (int64_t k = 0; k < nchunks; ++k) {
    const int64_t v0 = k * vq;
    const int64_t rows = (V - v0) < vq ? (V - v0) : vq;
    if (k + 1 < nchunks) {
      // the buffer chunk k+1 goes into was read by forward(k-1), enqueued on `s` already
      CCE_CUDA_CHECK(cudaEventRecord(ss->ev_r, s), "cce_forward_q record");
      CCE_CUDA_CHECK(cudaStreamWaitEvent(ss->sq, ss->ev_r, 0), "cce_forward_q wait");
      const int64_t v1 = v0 + vq;
      const int64_t rows1 = (V - v1) < vq ? (V - v1) : vq;
      CCE_CUDA_CHECK(dequant_rows(head, v1, rows1, D, dtype, cbuf[(k + 1) & 1], ss->sq), "cce_forward_q dequantise");
      CCE_CUDA_CHECK(cudaEventRecord(ss->ev_q[(k + 1) & 1], ss->sq), "cce_forward_q record");
    }
    CCE_CUDA_CHECK(cudaStreamWaitEvent(s, ss->ev_q[k & 1], 0), "cce_forward_q wait");
    // this chunk's columns of the statistics and partials (vq is a multiple of both tile widths)
    cce::FwdArgs a{e, cbuf[k & 1], bias ? static_cast<const char*>(bias) + v0 * bsz : nullptr, bias_dtype, targets,
                   N, D, rows, v_offset + v0, dtype, tile_max + (v0 / cce::kStatTile) * N,
                   part_m + (v0 / ptile) * N, part_s + (v0 / ptile) * N, tgt};
    if (tc) {
      CCE_CUDA_CHECK(cce::tc_forward(a, s), "cce_forward_q tc kernel");
    } else {
      CCE_CUDA_CHECK(cce::simt_forward(a, s), "cce_forward_q simt kernel");
    }
  }
  CCE_CUDA_CHECK(cce::launch_lse_combine(part_m, part_s, nullptr, P, N, N, lse, nullptr, nullptr, s),
                 "cce_forward_q combine");
  return CCE_OK;
}

int cce_lse_combine(const float* part_lse, const float* part_tgt, int64_t P, int64_t N,
                    int64_t part_stride, float* lse, float* tgt, float* nll, void* stream) {
  if (P <= 0 || N < 0) return fail(CCE_ERR_SHAPE, "cce_lse_combine: bad P=%lld N=%lld", (long long)P, (long long)N);
  if (P > 1 && part_stride < N)
    return fail(CCE_ERR_SHAPE, "cce_lse_combine: part_stride %lld < N %lld", (long long)part_stride, (long long)N);
  if (N == 0) return CCE_OK;
  if (!part_lse || !lse) return fail(CCE_ERR_ARG, "cce_lse_combine: NULL required pointer");
  if (tgt && !part_tgt) return fail(CCE_ERR_ARG, "cce_lse_combine: tgt requested without part_tgt");
  if (nll && !part_tgt) return fail(CCE_ERR_ARG, "cce_lse_combine: nll requested without part_tgt");
  int rc = check_arch();
  if (rc) return rc;
  CCE_CUDA_CHECK(cce::launch_lse_combine(part_lse, nullptr, part_tgt, P, N, part_stride, lse, tgt,
                                         nll, (cudaStream_t)stream),
                 "cce_lse_combine");
  return CCE_OK;
}

size_t cce_backward_workspace_bytes(int64_t N, int64_t D, int64_t V, int dtype, int flags) {
  return backward_ws_bytes(N, D, V, dtype, flags, false);
}

// cce_backward, cce_backward_peer when `pg` is given (grad_e summed over the
// group through the exchange buffers), and cce_backward_q when `qh` is given
// (c is a quantised head: every vocabulary chunk is expanded into one of two
// workspace buffers on a side stream while the previous chunk's GEMMs run).
static int backward_impl(const void* e, const void* c, const CceQuantHead* qh, const void* bias, int bias_dtype,
                         const int32_t* targets, const float* lse, const float* d_nll,
                         const float* tile_max, int64_t N, int64_t D, int64_t V, int64_t v_offset,
                         int dtype, int flags, float filter_log_eps, void* grad_e, void* grad_c,
                         float* grad_bias, int64_t* skip_stats, void* workspace, size_t workspace_bytes,
                         const CcePeerGroup* pg, void* stream) {
  int rc = check_sizes(N, D, V, dtype);
  if (rc) return rc;
  if (bias && !dtype_ok(bias_dtype)) return fail(CCE_ERR_DTYPE, "unsupported bias dtype code %d", bias_dtype);
  if (flags & ~(CCE_NEED_DE | CCE_NEED_DC | CCE_NEED_DBIAS | CCE_DE_F32 | CCE_NO_FILTER))
    return fail(CCE_ERR_ARG, "cce_backward: unknown flag bits 0x%x", flags);
  const bool need_de = flags & CCE_NEED_DE, need_dc = flags & CCE_NEED_DC,
             need_db = flags & CCE_NEED_DBIAS;
  if (qh) {
    rc = check_head(qh, D, "cce_backward_q");
    if (rc) return rc;
    if (need_dc) return fail(CCE_ERR_ARG, "cce_backward_q: a quantised head is frozen (no CCE_NEED_DC)");
  }
  // A zero-size output may come with a NULL pointer (torch gives empty tensors none).
  if ((need_de && N > 0 && !grad_e) || (need_dc && V > 0 && !grad_c) || (need_db && V > 0 && !grad_bias))
    return fail(CCE_ERR_ARG, "cce_backward: a requested gradient has a NULL output pointer");
  if (need_db && !bias) return fail(CCE_ERR_ARG, "cce_backward: CCE_NEED_DBIAS without bias");
  if (!need_de && !need_dc && !need_db) return CCE_OK;
  if (V == 0) return fail(CCE_ERR_SHAPE, "V must be positive");
  cudaStream_t s = (cudaStream_t)stream;
  rc = check_arch();
  if (rc) return rc;
  if (N == 0) {
    // No rows: every requested gradient is zero.
    if (need_dc) CCE_CUDA_CHECK(cudaMemsetAsync(grad_c, 0, (size_t)V * D * dtype_size(dtype), s), "memset grad_c");
    if (need_db) CCE_CUDA_CHECK(cudaMemsetAsync(grad_bias, 0, (size_t)V * sizeof(float), s), "memset grad_bias");
    return CCE_OK;
  }
  if (!e || (!c && !qh) || !targets || !lse || !d_nll || !tile_max)
    return fail(CCE_ERR_ARG, "cce_backward: NULL required pointer");
  // (a quantised head's chunks live in the workspace: its alignment stands for c's)
  const bool tc = !force_simt() && cce::tc_backward_supported(e, qh ? workspace : c, D, dtype) &&
                  aligned16(workspace) && (!need_de || aligned16(grad_e)) && (!need_dc || aligned16(grad_c));
  const BwdPlan p = plan_backward(N, D, V, dtype, flags, tc);
  const size_t need = backward_ws_bytes(N, D, V, dtype, flags, qh != nullptr);
  if (!workspace || workspace_bytes < need)
    return fail(CCE_ERR_WORKSPACE, "cce_backward: workspace %zu bytes < required %zu", workspace_bytes, need);

  // the cross-rank exchange of grad_e (only when grad_e is requested)
  const bool exchange = pg != nullptr && need_de;
  cce::PeerPush push{};
  uint64_t wait_ns = 0;
  const int out_dtype = (flags & CCE_DE_F32) ? CCE_F32 : dtype;
  if (exchange) {
    push.layout = cce::peer::make_layout(N, D, pg->world, (int)dtype_size(out_dtype));
    if (pg->bytes < push.layout.bytes)
      return fail(CCE_ERR_WORKSPACE, "cce_backward_peer: exchange buffers of %zu bytes < required %zu", pg->bytes,
                  push.layout.bytes);
    push.peers.rank = pg->rank;
    push.peers.world = pg->world;
    for (int r = 0; r < pg->world; ++r) push.peers.bases[r] = static_cast<char*>(pg->bases[r]);
    wait_ns = pg->wait_limit_ns > 0 ? (uint64_t)pg->wait_limit_ns : 10000000000ull;
  }

  char* ws = (char*)workspace;
  uint8_t* keep = (uint8_t*)ws;
  void* dl = ws + p.keep_bytes;
  float* acc = nullptr;
  if (need_de)
    acc = (!p.tc && (flags & CCE_DE_F32)) ? (float*)grad_e : (float*)(ws + p.keep_bytes + p.dl_bytes);
  int* counters = (int*)(ws + p.keep_bytes + p.dl_bytes + p.acc_bytes);
  float* scale = p.scale_bytes ? (float*)(ws + p.keep_bytes + p.dl_bytes + p.acc_bytes + p.counter_bytes)
                               : nullptr;
  uint32_t* keep_t = p.keep_t_bytes
                         ? (uint32_t*)(ws + p.keep_bytes + p.dl_bytes + p.acc_bytes + p.counter_bytes + p.scale_bytes)
                         : nullptr;
  float* part = p.part_bytes ? (float*)(ws + p.keep_bytes + p.dl_bytes + p.acc_bytes + p.counter_bytes +
                                        p.scale_bytes + p.keep_t_bytes)
                             : nullptr;
  int* dl_lists = p.list_bytes ? (int*)(ws + p.keep_bytes + p.dl_bytes + p.acc_bytes + p.counter_bytes +
                                         p.scale_bytes + p.keep_t_bytes + p.part_bytes)
                               : nullptr;
  char* cbuf[2] = {nullptr, nullptr};  // a quantised head's expanded chunks
  if (qh) {
    cbuf[0] = ws + plan_bytes(p);
    cbuf[1] = cbuf[0] + chunk_buf_bytes(p, D, dtype);
  }
  if (p.tc) CCE_CUDA_CHECK(cudaMemsetAsync(counters, 0, p.counter_bytes, s), "cce_backward memset counters");
  if (keep_t) CCE_CUDA_CHECK(cudaMemsetAsync(keep_t, 0, p.keep_t_bytes, s), "cce_backward memset mask table");
  if (scale) CCE_CUDA_CHECK(cce::launch_pow2_absmax(d_nll, N, scale, s), "cce_backward scale");

  CCE_CUDA_CHECK(cce::launch_block_mask(tile_max, lse, targets, d_nll, N, V, v_offset, filter_log_eps,
                                        (flags & CCE_NO_FILTER) != 0, keep, keep_t, p.keep_t_ld, skip_stats, s),
                 "cce_backward mask");
  if (need_db) CCE_CUDA_CHECK(cudaMemsetAsync(grad_bias, 0, (size_t)V * sizeof(float), s), "memset grad_bias");
  if (dl_lists)
    CCE_CUDA_CHECK(cce::tc_dlogits_lists(keep, N, D, V, p.vc, dl_lists, counters, s), "cce_backward dlogits lists");

  cce::BwdChunkArgs a{e, c, nullptr, bias, bias_dtype, targets, lse, d_nll, keep, keep_t, p.keep_t_ld, N, D, V,
                      v_offset, dtype, 0, 0, p.vc, dl, need_db ? grad_bias : nullptr, nullptr, scale};
  const int64_t nchunks = cce::ceil_div(V, p.vc);
  const size_t esz = dtype_size(dtype);
  SideStreams* ss = nullptr;
  if (p.tc || qh) {
    rc = side_streams(&ss);
    if (rc) return rc;
    // fork: the side streams start after everything enqueued on `s` so far
    CCE_CUDA_CHECK(cudaEventRecord(ss->start, s), "cce_backward fork");
    if (p.tc) {
      CCE_CUDA_CHECK(cudaStreamWaitEvent(ss->se, ss->start, 0), "cce_backward fork");
      CCE_CUDA_CHECK(cudaStreamWaitEvent(ss->sc, ss->start, 0), "cce_backward fork");
    }
    if (qh) {
      CCE_CUDA_CHECK(cudaStreamWaitEvent(ss->sq, ss->start, 0), "cce_backward fork");
      const int64_t rows0 = V < p.vc ? V : p.vc;
      CCE_CUDA_CHECK(dequant_rows(qh, 0, rows0, D, dtype, cbuf[0], ss->sq), "cce_backward_q dequantise");
      CCE_CUDA_CHECK(cudaEventRecord(ss->ev_q[0], ss->sq), "cce_backward record");
    }
  }
  for (int64_t ch = 0; ch < nchunks; ++ch) {
    a.vc0 = ch * p.vc;
    a.vc_len = (V - a.vc0) < p.vc ? (V - a.vc0) : p.vc;
    const bool last = ch == nchunks - 1;
    a.counters = counters + 4 * ch;
    a.dl_list = dl_lists ? dl_lists + ch * cce::tc_dlogits_list_len(N, p.vc) : nullptr;
    // dlogits(ch) on `s` overwrites the buffer grad_e / grad_c of chunk ch-1 read
    if (p.tc && ch > 0) {
      CCE_CUDA_CHECK(cudaStreamWaitEvent(s, ss->ev_e, 0), "cce_backward join");
      CCE_CUDA_CHECK(cudaStreamWaitEvent(s, ss->ev_c, 0), "cce_backward join");
    }
    if (qh) {
      // chunk ch+1 goes into the buffer chunk ch-1 was read from (all of
      // whose readers `s` has now waited for); chunk ch was expanded already
      if (!last) {
        CCE_CUDA_CHECK(cudaEventRecord(ss->ev_r, s), "cce_backward record");
        CCE_CUDA_CHECK(cudaStreamWaitEvent(ss->sq, ss->ev_r, 0), "cce_backward wait");
        const int64_t v1 = a.vc0 + p.vc;
        const int64_t rows1 = (V - v1) < p.vc ? (V - v1) : p.vc;
        CCE_CUDA_CHECK(dequant_rows(qh, v1, rows1, D, dtype, cbuf[(ch + 1) & 1], ss->sq), "cce_backward_q dequantise");
        CCE_CUDA_CHECK(cudaEventRecord(ss->ev_q[(ch + 1) & 1], ss->sq), "cce_backward record");
      }
      CCE_CUDA_CHECK(cudaStreamWaitEvent(s, ss->ev_q[ch & 1], 0), "cce_backward wait");
      a.c_chunk = cbuf[ch & 1];
    } else {
      a.c_chunk = static_cast<const char*>(c) + (size_t)a.vc0 * (size_t)D * esz;
    }
    if (p.tc) {
      CCE_CUDA_CHECK(cce::tc_dlogits(a, s), "cce_backward tc dlogits");
      CCE_CUDA_CHECK(cudaEventRecord(ss->ev_l, s), "cce_backward record");
      CCE_CUDA_CHECK(cudaStreamWaitEvent(ss->se, ss->ev_l, 0), "cce_backward wait");
      CCE_CUDA_CHECK(cudaStreamWaitEvent(ss->sc, ss->ev_l, 0), "cce_backward wait");
      if (need_de) {
        const bool push_now = exchange && last;
        CCE_CUDA_CHECK(cce::tc_grad_e(a, acc, ch > 0, push_now ? &push : nullptr, ss->se), "cce_backward tc grad_e");
        if (push_now)
          CCE_CUDA_CHECK(cce::peer::launch_reduce_gather(push.peers, push.layout, cce::peer::kSlotsPerSrc, N, D,
                                                         out_dtype, grad_e, wait_ns, ss->se),
                         "cce_backward_peer exchange");
        else if (last)
          CCE_CUDA_CHECK(cce::launch_sum2_f32(acc, acc + N * D, grad_e, out_dtype, N * D, ss->se),
                         "cce_backward sum grad_e");
      }
      if (need_dc) CCE_CUDA_CHECK(cce::tc_grad_c(a, grad_c, ss->sc), "cce_backward tc grad_c");
      CCE_CUDA_CHECK(cudaEventRecord(ss->ev_e, ss->se), "cce_backward record");
      CCE_CUDA_CHECK(cudaEventRecord(ss->ev_c, ss->sc), "cce_backward record");
      if (last) {
        CCE_CUDA_CHECK(cudaStreamWaitEvent(s, ss->ev_e, 0), "cce_backward join");
        CCE_CUDA_CHECK(cudaStreamWaitEvent(s, ss->ev_c, 0), "cce_backward join");
      }
    } else {
      CCE_CUDA_CHECK(cce::simt_dlogits(a, s), "cce_backward simt dlogits");
      if (need_de) CCE_CUDA_CHECK(cce::simt_grad_e(a, acc, ch > 0, part, p.splits, s), "cce_backward simt grad_e");
      if (need_dc) CCE_CUDA_CHECK(cce::simt_grad_c(a, grad_c, s), "cce_backward simt grad_c");
      if (need_de && last && exchange) {
        CCE_CUDA_CHECK(cce::peer::launch_push(push.peers, push.layout, acc, 1, N, D, s), "cce_backward_peer push");
        CCE_CUDA_CHECK(cce::peer::launch_reduce_gather(push.peers, push.layout, 1, N, D, out_dtype, grad_e, wait_ns, s),
                       "cce_backward_peer exchange");
      } else if (need_de && last && !(flags & CCE_DE_F32)) {
        CCE_CUDA_CHECK(cce::launch_cast_f32(acc, grad_e, dtype, N * D, s), "cce_backward cast grad_e");
      }
    }
  }
  return CCE_OK;
}

int cce_backward(const void* e, const void* c, const void* bias, int bias_dtype,
                 const int32_t* targets, const float* lse, const float* d_nll,
                 const float* tile_max, int64_t N, int64_t D, int64_t V, int64_t v_offset,
                 int dtype, int flags, float filter_log_eps, void* grad_e, void* grad_c,
                 float* grad_bias, int64_t* skip_stats, void* workspace, size_t workspace_bytes,
                 void* stream) {
  return backward_impl(e, c, nullptr, bias, bias_dtype, targets, lse, d_nll, tile_max, N, D, V, v_offset, dtype,
                       flags, filter_log_eps, grad_e, grad_c, grad_bias, skip_stats, workspace, workspace_bytes,
                       nullptr, stream);
}

int cce_backward_peer(const void* e, const void* c, const void* bias, int bias_dtype,
                      const int32_t* targets, const float* lse, const float* d_nll,
                      const float* tile_max, int64_t N, int64_t D, int64_t V, int64_t v_offset,
                      int dtype, int flags, float filter_log_eps, void* grad_e, void* grad_c,
                      float* grad_bias, int64_t* skip_stats, void* workspace, size_t workspace_bytes,
                      const CcePeerGroup* group, void* stream) {
  if (!group) return fail(CCE_ERR_ARG, "cce_backward_peer: NULL group");
  if (group->world < 1 || group->world > CCE_PEER_MAX_WORLD || group->rank < 0 || group->rank >= group->world)
    return fail(CCE_ERR_ARG, "cce_backward_peer: rank %d / world %d out of range (world <= %d)", group->rank,
                group->world, CCE_PEER_MAX_WORLD);
  for (int r = 0; r < group->world; ++r)
    if (!group->bases[r] || !aligned16(group->bases[r]))
      return fail(CCE_ERR_ARG, "cce_backward_peer: buffer of rank %d is NULL or not 16-byte aligned", r);
  return backward_impl(e, c, nullptr, bias, bias_dtype, targets, lse, d_nll, tile_max, N, D, V, v_offset, dtype,
                       flags, filter_log_eps, grad_e, grad_c, grad_bias, skip_stats, workspace, workspace_bytes, group,
                       stream);
}

size_t cce_backward_q_workspace_bytes(int64_t N, int64_t D, int64_t V, int dtype, int flags) {
  return backward_ws_bytes(N, D, V, dtype, flags, true);
}

int cce_backward_q(const void* e, const CceQuantHead* head, const void* bias, int bias_dtype,
                   const int32_t* targets, const float* lse, const float* d_nll, const float* tile_max, int64_t N,
                   int64_t D, int64_t V, int64_t v_offset, int dtype, int flags, float filter_log_eps, void* grad_e,
                   float* grad_bias, int64_t* skip_stats, void* workspace, size_t workspace_bytes, void* stream) {
  if (!head) return fail(CCE_ERR_ARG, "cce_backward_q: NULL head");
  return backward_impl(e, nullptr, head, bias, bias_dtype, targets, lse, d_nll, tile_max, N, D, V, v_offset, dtype,
                       flags, filter_log_eps, grad_e, nullptr, grad_bias, skip_stats, workspace, workspace_bytes,
                       nullptr, stream);
}

size_t cce_peer_buffer_bytes(int64_t N, int64_t D, int world, int out_dtype) {
  if (N < 0 || D <= 0 || world < 1 || world > CCE_PEER_MAX_WORLD || !dtype_ok(out_dtype)) return 0;
  return cce::peer::make_layout(N, D, world, (int)dtype_size(out_dtype)).bytes;
}

int cce_peer_buffer_alloc(size_t bytes, void** ptr, int* fd) {
  if (!ptr || !fd) return fail(CCE_ERR_ARG, "cce_peer_buffer_alloc: NULL output pointer");
  if (bytes < cce::peer::kCtrlBytes) return fail(CCE_ERR_ARG, "cce_peer_buffer_alloc: %zu bytes is too small", bytes);
  int rc = check_arch();
  if (rc) return rc;
  const VmmApi& api = vmm_api();
  if (!api.ok) return fail(CCE_ERR_CUDA, "cce_peer_buffer_alloc: the driver's virtual-memory API is unavailable");
  int dev = 0;
  CCE_CUDA_CHECK(cudaGetDevice(&dev), "cudaGetDevice");
  CUmemAllocationProp prop = device_prop(dev);
  size_t gran = 0;
  CUresult r = api.granularity(&gran, &prop, CU_MEM_ALLOC_GRANULARITY_RECOMMENDED);
  if (r != CUDA_SUCCESS || gran == 0) return fail(CCE_ERR_CUDA, "cuMemGetAllocationGranularity failed (%d)", (int)r);
  const size_t size = (bytes + gran - 1) / gran * gran;
  CUmemGenericAllocationHandle h = 0;
  if ((r = api.create(&h, size, &prop, 0)) != CUDA_SUCCESS)
    return fail(CCE_ERR_CUDA, "cuMemCreate of %zu bytes failed (%d)", size, (int)r);
  CUdeviceptr va = 0;
  rc = map_local(api, h, size, dev, &va);
  if (rc) {
    api.release(h);
    return rc;
  }
  int shared = -1;
  if ((r = api.export_fd(&shared, h, CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR, 0)) != CUDA_SUCCESS) {
    unmap(api, va, size);
    api.release(h);
    return fail(CCE_ERR_CUDA, "cuMemExportToShareableHandle failed (%d)", (int)r);
  }
  // zero the whole buffer (the control block above all) before any rank maps it
  cudaError_t err = cudaMemset(reinterpret_cast<void*>(va), 0, size);
  if (err == cudaSuccess) err = cudaDeviceSynchronize();
  if (err != cudaSuccess) {
    unmap(api, va, size);
    api.release(h);
    return cuda_fail(err, "cce_peer_buffer_alloc memset");
  }
  remember(va, h, size);
  *ptr = reinterpret_cast<void*>(va);
  *fd = shared;
  return CCE_OK;
}

int cce_peer_buffer_open(int fd, size_t bytes, void** ptr) {
  if (!ptr || fd < 0) return fail(CCE_ERR_ARG, "cce_peer_buffer_open: NULL pointer or bad descriptor");
  const VmmApi& api = vmm_api();
  if (!api.ok) return fail(CCE_ERR_CUDA, "cce_peer_buffer_open: the driver's virtual-memory API is unavailable");
  int dev = 0;
  CCE_CUDA_CHECK(cudaGetDevice(&dev), "cudaGetDevice");
  CUmemAllocationProp prop = device_prop(dev);
  size_t gran = 0;
  CUresult r = api.granularity(&gran, &prop, CU_MEM_ALLOC_GRANULARITY_RECOMMENDED);
  if (r != CUDA_SUCCESS || gran == 0) return fail(CCE_ERR_CUDA, "cuMemGetAllocationGranularity failed (%d)", (int)r);
  const size_t size = (bytes + gran - 1) / gran * gran;
  CUmemGenericAllocationHandle h = 0;
  r = api.import_fd(&h, reinterpret_cast<void*>(static_cast<uintptr_t>(fd)), CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR);
  if (r != CUDA_SUCCESS) return fail(CCE_ERR_CUDA, "cuMemImportFromShareableHandle failed (%d)", (int)r);
  CUdeviceptr va = 0;
  int rc = map_local(api, h, size, dev, &va);
  if (rc) {
    api.release(h);
    return rc;
  }
  remember(va, h, size);
  *ptr = reinterpret_cast<void*>(va);
  return CCE_OK;
}

int cce_peer_buffer_close(void* ptr) {
  if (!ptr) return CCE_OK;
  return forget_and_unmap(ptr, "cce_peer_buffer_close");
}

int cce_peer_buffer_free(void* ptr) {
  if (!ptr) return CCE_OK;
  return forget_and_unmap(ptr, "cce_peer_buffer_free");
}

int cce_dequantize(const uint32_t* wq, const void* scales, const void* biases, int scale_dtype, int64_t rows,
                   int64_t D, int group_size, int bits, int out_dtype, void* out, void* stream) {
  if (rows < 0 || D < 0) return fail(CCE_ERR_SHAPE, "cce_dequantize: negative size");
  if (bits != 2 && bits != 4 && bits != 8) return fail(CCE_ERR_ARG, "cce_dequantize: bits must be 2, 4 or 8, got %d", bits);
  if (group_size != 32 && group_size != 64 && group_size != 128)
    return fail(CCE_ERR_ARG, "cce_dequantize: group_size must be 32, 64 or 128, got %d", group_size);
  if (D % group_size != 0)
    return fail(CCE_ERR_SHAPE, "cce_dequantize: D=%lld is not a multiple of group_size=%d", (long long)D, group_size);
  if (!dtype_ok(scale_dtype) || !dtype_ok(out_dtype))
    return fail(CCE_ERR_DTYPE, "cce_dequantize: dtype codes %d / %d", scale_dtype, out_dtype);
  if (rows == 0 || D == 0) return CCE_OK;
  if (!wq || !scales || !biases || !out) return fail(CCE_ERR_ARG, "cce_dequantize: NULL pointer");
  int rc = check_arch();
  if (rc) return rc;
  CCE_CUDA_CHECK(cce::launch_dequantize(wq, scales, biases, scale_dtype, rows, D, group_size, bits, out_dtype, out,
                                        (cudaStream_t)stream),
                 "cce_dequantize");
  return CCE_OK;
}

}  // extern "C"
