// Exchange kernels of the vocabulary-sharded backward: the cross-rank sum of
// grad_e over NVLink peer memory, with no collective library in the loop.
//
// Each rank holds a partial grad_e (the product of its vocabulary shard's
// dlogits with its shard of c).  The reduction is a reduce-scatter followed by
// an all-gather, both as plain loads and stores into the ranks' exchange
// buffers (layout and signalling in peer.cuh):
//
//   push    every rank stores its partial rows into the owner rank's receive
//           slots.  The tensor-core path does this inside the grad_e GEMM's
//           epilogue of the last vocabulary chunk (tc_kernels.cu), so the
//           NVLink transfer overlaps the MMAs tile by tile; push_kernel below
//           does it for partials that are already in memory (CUDA-core path).
//   reduce  the owner waits for every rank's `pushed` flag, sums the slots of
//           its rows in a fixed order (rank 0 first, so the result does not
//           depend on arrival order), writes them to its grad_e and to its
//           reduced area, and raises `reduced` on every rank.
//   gather  every rank waits for the other ranks' `reduced` flags and copies
//           their rows from their reduced areas into its own grad_e.
//
// Waits are bounded: after the limit the kernel records a code in the status
// word read by cce_device_status() and returns, so a rank that never arrives
// ends the call with an error instead of hanging the GPU.  The kernels use no
// shared memory, so they run beside the persistent grad_c kernel of the same
// chunk, which holds almost all of every SM's shared memory.
#include "kernels.cuh"
#include "peer.cuh"

namespace cce {
namespace peer {
namespace {

__device__ int g_peer_status = 0;

__device__ __forceinline__ uint64_t now_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Waits (one thread) until flag[src] >= epoch for every src != skip.  Returns
// false after limit_ns, having recorded `code`.
__device__ bool wait_flags(char* own, size_t off, int world, int skip, unsigned long long epoch,
                           uint64_t limit_ns, int code) {
  const uint64_t t0 = now_ns();
  for (int src = 0; src < world; ++src) {
    if (src == skip) continue;
    const unsigned long long* f = flag(own, off, src);
    while (ld_acquire_sys(f) < epoch) {
      if (now_ns() - t0 > limit_ns) {
        atomicCAS(&g_peer_status, 0, code);
        return false;
      }
      __nanosleep(200);
    }
  }
  return true;
}

__device__ __forceinline__ unsigned long long own_epoch(const Peers& P) {
  return *reinterpret_cast<volatile unsigned long long*>(P.bases[P.rank] + kEpochOff);
}

template <typename T> struct Vec;
template <> struct Vec<float> { static constexpr int n = 4; };
template <> struct Vec<__half> { static constexpr int n = 8; };
template <> struct Vec<__nv_bfloat16> { static constexpr int n = 8; };

// Partial rows src[s][row][:] (fp32, nslab slabs) -> slot (rank, s) of the
// row's owner.  The last CTA raises `pushed` with a new epoch.
__global__ void push_kernel(Peers P, Layout L, const float* __restrict__ src, int nslab, int64_t N, int64_t D) {
  const int64_t step = (int64_t)gridDim.x * blockDim.x;
  const int64_t i0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const bool vec = (D & 3) == 0;
  const int w = vec ? 4 : 1;
  const int64_t per_row = D / w;
  const int64_t items = (int64_t)nslab * N * per_row;
  for (int64_t i = i0; i < items; i += step) {
    const int64_t s = i / (N * per_row);
    const int64_t rem = i - s * N * per_row;
    const int64_t row = rem / per_row;
    const int64_t col = (rem - row * per_row) * w;
    const int owner = (int)((row / kRows) / L.mt_per);
    const int64_t lrow = row - (int64_t)owner * L.R;
    float* dst = reinterpret_cast<float*>(P.bases[owner] + L.recv_off) +
                 (((int64_t)P.rank * kSlotsPerSrc + s) * L.R + lrow) * D + col;
    const float* from = src + (s * N + row) * D + col;
    if (vec) *reinterpret_cast<float4*>(dst) = *reinterpret_cast<const float4*>(from);
    else *dst = *from;
  }
  __syncthreads();
  if (threadIdx.x == 0) arrive_and_signal(P, kDoneUnitsOff, gridDim.x, true, kPushedOff);
}

template <typename TO>
__device__ __forceinline__ void store_out(TO* p, const float* v, int n) {
  for (int j = 0; j < n; ++j) p[j] = from_f32<TO>(v[j]);
}

// Vec<TO>::n values converted to TO, packed into 16 bytes (element 0 lowest).
template <typename TO>
__device__ __forceinline__ uint4 pack16(const float* v);
template <>
__device__ __forceinline__ uint4 pack16<float>(const float* v) {
  return make_uint4(__float_as_uint(v[0]), __float_as_uint(v[1]), __float_as_uint(v[2]), __float_as_uint(v[3]));
}
template <typename T16>
__device__ __forceinline__ uint32_t pack2(float a, float b) {
  const T16 lo = from_f32<T16>(a), hi = from_f32<T16>(b);
  return (uint32_t)__builtin_bit_cast(uint16_t, lo) | ((uint32_t)__builtin_bit_cast(uint16_t, hi) << 16);
}
template <>
__device__ __forceinline__ uint4 pack16<__half>(const float* v) {
  return make_uint4(pack2<__half>(v[0], v[1]), pack2<__half>(v[2], v[3]), pack2<__half>(v[4], v[5]),
                    pack2<__half>(v[6], v[7]));
}
template <>
__device__ __forceinline__ uint4 pack16<__nv_bfloat16>(const float* v) {
  return make_uint4(pack2<__nv_bfloat16>(v[0], v[1]), pack2<__nv_bfloat16>(v[2], v[3]),
                    pack2<__nv_bfloat16>(v[4], v[5]), pack2<__nv_bfloat16>(v[6], v[7]));
}

// This rank's rows: sum of the nslot slots of every source rank (rank 0
// first), written to out and to the reduced area; the last CTA raises
// `reduced` on every rank.
template <typename TO>
__global__ void reduce_kernel(Peers P, Layout L, int nslot, int64_t N, int64_t D, TO* __restrict__ out,
                              uint64_t limit_ns) {
  char* own = P.bases[P.rank];
  const unsigned long long epoch = own_epoch(P);
  int ok = 1;
  if (threadIdx.x == 0) ok = wait_flags(own, kPushedOff, P.world, -1, epoch, limit_ns, CCE_PEER_WAIT_PUSH);
  if (!__syncthreads_and(ok)) return;  // the flags stay down: every other rank's wait runs out too
  constexpr int VN = Vec<TO>::n;
  const bool vec = D % VN == 0;
  const int w = vec ? VN : 1;
  const int64_t r0 = (int64_t)P.rank * L.R;
  const int64_t rows = N - r0 < L.R ? (N - r0 > 0 ? N - r0 : 0) : L.R;
  const int64_t per_row = D / w;
  const int64_t items = rows * per_row;
  const float* recv = reinterpret_cast<const float*>(own + L.recv_off);
  TO* red = reinterpret_cast<TO*>(own + L.reduced_off);
  const int64_t slot_stride = L.R * D;
  const int64_t step = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < items; i += step) {
    const int64_t lrow = i / per_row;
    const int64_t col = (i - lrow * per_row) * w;
    float acc[VN];
#pragma unroll
    for (int j = 0; j < VN; ++j) acc[j] = 0.f;
    for (int k = 0; k < P.world * nslot; ++k) {
      const int src = k / nslot, s = k - src * nslot;
      const float* p = recv + (int64_t)(src * kSlotsPerSrc + s) * slot_stride + lrow * D + col;
      if (vec) {
#pragma unroll
        for (int j = 0; j < VN; j += 4) {
          const float4 x = *reinterpret_cast<const float4*>(p + j);
          acc[j] += x.x;
          acc[j + 1] += x.y;
          acc[j + 2] += x.z;
          acc[j + 3] += x.w;
        }
      } else {
        acc[0] += *p;
      }
    }
    if (vec) {
      const uint4 o = pack16<TO>(acc);
      *reinterpret_cast<uint4*>(out + (r0 + lrow) * D + col) = o;
      *reinterpret_cast<uint4*>(red + lrow * D + col) = o;
    } else {
      store_out(out + (r0 + lrow) * D + col, acc, 1);
      store_out(red + lrow * D + col, acc, 1);
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) arrive_and_signal(P, kDoneReduceOff, gridDim.x, false, kReducedOff);
}

// The other ranks' reduced rows -> out.
template <typename TO>
__global__ void gather_kernel(Peers P, Layout L, int64_t N, int64_t D, TO* __restrict__ out, uint64_t limit_ns) {
  char* own = P.bases[P.rank];
  const unsigned long long epoch = own_epoch(P);
  int ok = 1;
  if (threadIdx.x == 0) ok = wait_flags(own, kReducedOff, P.world, P.rank, epoch, limit_ns, CCE_PEER_WAIT_REDUCE);
  if (!__syncthreads_and(ok)) return;
  constexpr int VN = Vec<TO>::n;
  const bool vec = D % VN == 0;
  const int w = vec ? VN : 1;
  const int64_t per_row = D / w;
  const int64_t items = N * per_row;
  const int64_t step = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < items; i += step) {
    const int64_t row = i / per_row;
    const int src = (int)(row / L.R);
    if (src == P.rank) continue;
    const int64_t col = (i - row * per_row) * w;
    const TO* from = reinterpret_cast<const TO*>(P.bases[src] + L.reduced_off) + (row - (int64_t)src * L.R) * D + col;
    if (vec) *reinterpret_cast<uint4*>(out + row * D + col) = *reinterpret_cast<const uint4*>(from);
    else out[row * D + col] = *from;
  }
}

// At most 2 CTAs of 256 threads per SM: these kernels run on the grad_e
// stream, which has the higher priority, while the persistent grad_c kernel
// of the same chunk waits for SMs; two of them (2 x ~14K registers) still
// leave room on an SM for one grad_c CTA (~14K registers, 225 KB of shared
// memory), so waiting on another rank never keeps grad_c off the GPU.
int grid_for(int64_t items) {
  const int64_t g = ceil_div(items > 0 ? items : 1, 256);
  return (int)(g < 296 ? g : 296);
}

}  // namespace

cudaError_t launch_push(const Peers& P, const Layout& L, const float* src, int nslab, int64_t N, int64_t D,
                        cudaStream_t s) {
  const int64_t items = (int64_t)nslab * N * ((D & 3) == 0 ? D / 4 : D);
  push_kernel<<<grid_for(items), 256, 0, s>>>(P, L, src, nslab, N, D);
  return launched();
}

template <typename TO>
cudaError_t reduce_gather_t(const Peers& P, const Layout& L, int nslot, int64_t N, int64_t D, void* out,
                            uint64_t limit_ns, cudaStream_t s) {
  const int64_t R = L.R;
  const int64_t own = N - (int64_t)P.rank * R;
  const int64_t rows = own < 0 ? 0 : (own < R ? own : R);
  reduce_kernel<TO><<<grid_for(rows * D / 4), 256, 0, s>>>(P, L, nslot, N, D, static_cast<TO*>(out), limit_ns);
  cudaError_t err = launched();
  if (err != cudaSuccess) return err;
  gather_kernel<TO><<<grid_for(N * D / 8), 256, 0, s>>>(P, L, N, D, static_cast<TO*>(out), limit_ns);
  return launched();
}

cudaError_t launch_reduce_gather(const Peers& P, const Layout& L, int nslot, int64_t N, int64_t D, int out_dtype,
                                 void* out, uint64_t limit_ns, cudaStream_t s) {
  switch (out_dtype) {
    case CCE_F32: return reduce_gather_t<float>(P, L, nslot, N, D, out, limit_ns, s);
    case CCE_F16: return reduce_gather_t<__half>(P, L, nslot, N, D, out, limit_ns, s);
    case CCE_BF16: return reduce_gather_t<__nv_bfloat16>(P, L, nslot, N, D, out, limit_ns, s);
  }
  return cudaErrorInvalidValue;
}

int read_status(bool reset) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_peer_status, sizeof(int)) != cudaSuccess) return -1;
  if (reset && v != 0) {
    const int z = 0;
    cudaMemcpyToSymbol(g_peer_status, &z, sizeof(int));
  }
  return v;
}

}  // namespace peer
}  // namespace cce
