// Auxiliary kernels: LSE combine, backward block mask, casts.
//
// - lse_combine_kernel: per row, fold P partial (max, sum-exp) pairs -- the
//   vocabulary tiles of one call, or the vocabulary shards of several ranks --
//   into lse = M + log(sum_p s_p * exp(m_p - M)) with M = max_p m_p.  This is
//   reduce_tile_to_lse of the reference (csrc/cce/cce.metal:332-355), with the
//   target-logit sum and nll = lse - tgt (mlx_cce/__init__.py:32) fused in.
// - block_mask_kernel: the reference's per-tile skip decision
//   (csrc/cce/cce.metal:190-204) taken once per (128-row block, 32-column
//   vocabulary tile) instead of inside the backward kernel.
#include "kernels.cuh"

namespace cce {

namespace {

constexpr int kCombRows = 32;    // rows per block (threadIdx.x): a warp reads 128 contiguous bytes
constexpr int kCombSlices = 32;  // partial slices per row (threadIdx.y)

// Fold (mp, sp) into the running (m, s): s * 2^(m - M) + sp * 2^(mp - M), M = max.
__device__ __forceinline__ void fold(float& m, float& s, float mp, float sp) {
  const float M = fmaxf(m, mp);
  if (M == -INFINITY) return;
  s = s * exp2f((m - M) * kLog2e) + sp * exp2f((mp - M) * kLog2e);
  m = M;
}

__global__ void __launch_bounds__(kCombRows * kCombSlices)
lse_combine_kernel(const float* __restrict__ part_max, const float* __restrict__ part_sum,
                   const float* __restrict__ part_tgt, int64_t P, int64_t N, int64_t ld,
                   float* __restrict__ lse, float* __restrict__ tgt, float* __restrict__ nll) {
  __shared__ float sm[kCombSlices][kCombRows];
  __shared__ float ss[kCombSlices][kCombRows];
  __shared__ float st[kCombSlices][kCombRows];
  const int64_t row = (int64_t)blockIdx.x * kCombRows + threadIdx.x;
  float m = -INFINITY, s = 0.f, t = 0.f;
  if (row < N) {
    int64_t p = threadIdx.y;
    // four independent partials per step so their loads overlap
    for (; p + 3 * kCombSlices < P; p += 4 * kCombSlices) {
      float mp[4], sp[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int64_t q = (p + u * kCombSlices) * ld + row;
        mp[u] = part_max[q];
        sp[u] = part_sum ? part_sum[q] : 1.0f;
        if (part_tgt) t += part_tgt[q];
      }
      const float M = fmaxf(fmaxf(fmaxf(mp[0], mp[1]), fmaxf(mp[2], mp[3])), m);
      if (M != -INFINITY) {
        float acc = s * exp2f((m - M) * kLog2e);
#pragma unroll
        for (int u = 0; u < 4; ++u) acc += sp[u] * exp2f((mp[u] - M) * kLog2e);
        s = acc;
        m = M;
      }
    }
    for (; p < P; p += kCombSlices) {
      const int64_t q = p * ld + row;
      fold(m, s, part_max[q], part_sum ? part_sum[q] : 1.0f);
      if (part_tgt) t += part_tgt[q];
    }
  }
  sm[threadIdx.y][threadIdx.x] = m;
  ss[threadIdx.y][threadIdx.x] = s;
  st[threadIdx.y][threadIdx.x] = t;
  __syncthreads();
  // tree fold over the slices
  for (int h = kCombSlices / 2; h >= 1; h >>= 1) {
    if (threadIdx.y < h) {
      float M = sm[threadIdx.y][threadIdx.x], S = ss[threadIdx.y][threadIdx.x];
      fold(M, S, sm[threadIdx.y + h][threadIdx.x], ss[threadIdx.y + h][threadIdx.x]);
      sm[threadIdx.y][threadIdx.x] = M;
      ss[threadIdx.y][threadIdx.x] = S;
      st[threadIdx.y][threadIdx.x] += st[threadIdx.y + h][threadIdx.x];
    }
    __syncthreads();
  }
  if (threadIdx.y == 0 && row < N) {
    const float L = sm[0][threadIdx.x] + logf(ss[0][threadIdx.x]);
    const float T = st[0][threadIdx.x];
    lse[row] = L;
    if (tgt) tgt[row] = T;
    if (nll) nll[row] = L - T;
  }
}

// One block = one 128-row block x kMaskRounds x kMaskTiles statistics tiles;
// in each round every warp decides kMaskTiles / 8 tiles, its lane l covering
// rows l, l + 32, l + 64 and l + 96 (coalesced tile_max loads, per-row inputs
// read once per block).  Besides the byte mask keep[row block][tile], the
// block ORs its decisions per 128-column tile into the transposed bit table
// keep_t[128-column tile][row block bits] (zeroed by the caller; nullable).
// The skip counters take one atomic pair per block: blocks span 256 tiles so
// that there are few of them (at 32 tiles per block the ~4000 blocks of
// config 3 serialised on the two counter addresses).
constexpr int kMaskTiles = 32;
constexpr int kMaskRounds = 8;
constexpr int kMaskWarps = 8;
constexpr int kTilesPer128 = 128 / kStatTile;
static_assert(kMaskTiles % kTilesPer128 == 0, "whole 128-column tiles per round");

__global__ void __launch_bounds__(kMaskWarps * 32, 4)
block_mask_kernel(const float* __restrict__ tile_max, const float* __restrict__ lse,
                  const int32_t* __restrict__ targets, const float* __restrict__ d_nll, int64_t N,
                  int64_t V, int64_t v_offset, float log_eps, int no_filter, uint8_t* __restrict__ keep,
                  uint32_t* __restrict__ keep_t, int64_t keep_t_ld,
                  unsigned long long* __restrict__ skip_stats) {
  constexpr int kGroups = kMaskRounds * kMaskTiles / kTilesPer128;  // 128-column tiles per block
  __shared__ uint32_t any128[kGroups];
  __shared__ int cnt[2];
  if (threadIdx.x < kGroups) any128[threadIdx.x] = 0;
  if (threadIdx.x == 0) cnt[0] = cnt[1] = 0;
  __syncthreads();
  const int64_t nVt = ceil_div(V, kStatTile);
  const int64_t i = blockIdx.y;  // row block
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int kRowsPerLane = kRowBlock / 32;
  // Per row: its LSE, whether it is live, and the statistics tile holding its
  // target in this call's vocabulary range (-1: none), kept in few registers
  // so that four blocks fit on an SM.
  float L[kRowsPerLane];
  int tt[kRowsPerLane];
  bool live[kRowsPerLane];
  const float* tm0 = tile_max + i * kRowBlock + lane;  // + 32 u + j N: row lane + 32 u, tile j
#pragma unroll
  for (int u = 0; u < kRowsPerLane; ++u) {
    const int64_t row = i * kRowBlock + lane + 32 * u;
    live[u] = row < N && d_nll[row] != 0.f;  // rows with a zero cotangent contribute nothing
    L[u] = live[u] ? lse[row] : 0.f;
    const int64_t tl = live[u] ? (int64_t)targets[row] - v_offset : -1;
    tt[u] = (tl >= 0 && tl < V) ? (int)(tl / kStatTile) : -1;
  }
  constexpr int kTilesPerWarp = kMaskTiles / kMaskWarps;
  int skipped = 0, total = 0;
  const int64_t tile0 = (int64_t)blockIdx.x * kMaskRounds * kMaskTiles;
#pragma unroll 1
  for (int r = 0; r < kMaskRounds; ++r) {
    const int64_t base = tile0 + (int64_t)r * kMaskTiles;
    if (base >= nVt) break;
    // all of this warp's tile maxima of the round are loaded before any is
    // tested, so the loads overlap
    float x[kTilesPerWarp][kRowsPerLane];
#pragma unroll
    for (int q = 0; q < kTilesPerWarp; ++q) {
      const int64_t j = base + warp + q * kMaskWarps;
#pragma unroll
      for (int u = 0; u < kRowsPerLane; ++u) x[q][u] = (live[u] && j < nVt) ? __ldg(tm0 + 32 * u + j * N) : -INFINITY;
    }
#pragma unroll
    for (int q = 0; q < kTilesPerWarp; ++q) {
      const int w = warp + q * kMaskWarps;
      const int64_t j = base + w;  // vocabulary tile
      if (j >= nVt) break;
      bool k = false;
#pragma unroll
      for (int u = 0; u < kRowsPerLane; ++u) {
        if (live[u]) k = k || no_filter || tt[u] == (int)j || (x[q][u] - L[u] >= log_eps);
      }
      k = __any_sync(0xffffffffu, k);
      if (lane == 0) {
        keep[i * nVt + j] = (uint8_t)k;
        if (k) any128[(r * kMaskTiles + w) / kTilesPer128] = 1u;  // benign race: every writer stores 1
      }
      ++total;
      skipped += k ? 0 : 1;
    }
  }
  if (skip_stats && lane == 0 && total) {
    atomicAdd(&cnt[0], skipped);
    atomicAdd(&cnt[1], total);
  }
  __syncthreads();
  if (keep_t && threadIdx.x < kGroups && any128[threadIdx.x]) {
    const int64_t m = tile0 / kTilesPer128 + threadIdx.x;  // 128-column tile
    atomicOr(&keep_t[m * keep_t_ld + (i >> 5)], 1u << (i & 31));
  }
  if (skip_stats && threadIdx.x == 0 && cnt[1]) {
    atomicAdd(&skip_stats[0], (unsigned long long)cnt[0]);
    atomicAdd(&skip_stats[1], (unsigned long long)cnt[1]);
  }
}

template <typename T>
__global__ void cast_f32_kernel(const float* __restrict__ src, T* __restrict__ dst, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    dst[i] = from_f32<T>(src[i]);
}

// dst = a + b; four elements per thread step when n is a multiple of 4 (all
// pointers are then 16-byte aligned by the caller's contract), else one.
template <typename T>
__global__ void sum2_f32_kernel(const float* __restrict__ a, const float* __restrict__ b, T* __restrict__ dst,
                                int64_t n) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const int64_t i0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if ((n & 3) == 0) {
    for (int64_t i = i0; i < n / 4; i += stride) {
      const float4 x = reinterpret_cast<const float4*>(a)[i];
      const float4 y = reinterpret_cast<const float4*>(b)[i];
      dst[4 * i] = from_f32<T>(x.x + y.x);
      dst[4 * i + 1] = from_f32<T>(x.y + y.y);
      dst[4 * i + 2] = from_f32<T>(x.z + y.z);
      dst[4 * i + 3] = from_f32<T>(x.w + y.w);
    }
  } else {
    for (int64_t i = i0; i < n; i += stride) dst[i] = from_f32<T>(a[i] + b[i]);
  }
}

__global__ void fill_f32_kernel(float* __restrict__ dst, float v, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    dst[i] = v;
}

// One block: s = smallest power of two >= max |x| (exact scaling for fp16
// dlogits, which then lie in [-1, 1]); s = 1 when every x is zero.
__global__ void __launch_bounds__(1024) pow2_absmax_kernel(const float* __restrict__ x, int64_t n,
                                                           float* __restrict__ out) {
  __shared__ float red[32];
  float m = 0.f;
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) m = fmaxf(m, fabsf(x[i]));
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x < 32) {
    m = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (threadIdx.x == 0) {
      float s = 1.f;
      if (m > 0.f && isfinite(m)) {
        int ex;
        const float f = frexpf(m, &ex);  // m = f * 2^ex, f in [0.5, 1)
        s = ldexpf(1.f, f == 0.5f ? ex - 1 : ex);
      }
      out[0] = s;
      out[1] = 1.f / s;
    }
  }
}

int grid_for(int64_t n, int threads) {
  int64_t b = ceil_div(n, threads);
  if (b > 148 * 16) b = 148 * 16;
  if (b < 1) b = 1;
  return (int)b;
}

}  // namespace

cudaError_t launch_lse_combine(const float* part_max, const float* part_sum, const float* part_tgt,
                               int64_t P, int64_t N, int64_t ld, float* lse, float* tgt, float* nll,
                               cudaStream_t stream) {
  if (N == 0) return cudaSuccess;
  dim3 block(kCombRows, kCombSlices);
  dim3 grid((unsigned)ceil_div(N, kCombRows));
  lse_combine_kernel<<<grid, block, 0, stream>>>(part_max, part_sum, part_tgt, P, N, ld, lse, tgt, nll);
  return launched();
}

cudaError_t launch_block_mask(const float* tile_max, const float* lse, const int32_t* targets,
                              const float* d_nll, int64_t N, int64_t V, int64_t v_offset,
                              float log_eps, bool no_filter, uint8_t* keep, uint32_t* keep_t,
                              int64_t keep_t_ld, int64_t* skip_stats, cudaStream_t stream) {
  if (N == 0 || V == 0) return cudaSuccess;
  dim3 grid((unsigned)ceil_div(ceil_div(V, kStatTile), (int64_t)(kMaskTiles * kMaskRounds)),
            (unsigned)ceil_div(N, kRowBlock));
  block_mask_kernel<<<grid, kMaskWarps * 32, 0, stream>>>(tile_max, lse, targets, d_nll, N, V, v_offset,
                                                    log_eps, no_filter ? 1 : 0, keep, keep_t, keep_t_ld,
                                                    reinterpret_cast<unsigned long long*>(skip_stats));
  return launched();
}

cudaError_t launch_cast_f32(const float* src, void* dst, int dtype, int64_t n, cudaStream_t stream) {
  if (n == 0) return cudaSuccess;
  const int threads = 256;
  const int grid = grid_for(n, threads);
  switch (dtype) {
    case CCE_F32:
      return cudaMemcpyAsync(dst, src, n * sizeof(float), cudaMemcpyDeviceToDevice, stream);
    case CCE_F16:
      cast_f32_kernel<__half><<<grid, threads, 0, stream>>>(src, (__half*)dst, n);
      break;
    case CCE_BF16:
      cast_f32_kernel<__nv_bfloat16><<<grid, threads, 0, stream>>>(src, (__nv_bfloat16*)dst, n);
      break;
    default:
      return cudaErrorInvalidValue;
  }
  return launched();
}

cudaError_t launch_sum2_f32(const float* a, const float* b, void* dst, int dtype, int64_t n, cudaStream_t stream) {
  if (n == 0) return cudaSuccess;
  const int threads = 256;
  const int grid = grid_for((n & 3) == 0 ? n / 4 : n, threads);
  switch (dtype) {
    case CCE_F32:
      sum2_f32_kernel<float><<<grid, threads, 0, stream>>>(a, b, (float*)dst, n);
      break;
    case CCE_F16:
      sum2_f32_kernel<__half><<<grid, threads, 0, stream>>>(a, b, (__half*)dst, n);
      break;
    case CCE_BF16:
      sum2_f32_kernel<__nv_bfloat16><<<grid, threads, 0, stream>>>(a, b, (__nv_bfloat16*)dst, n);
      break;
    default:
      return cudaErrorInvalidValue;
  }
  return launched();
}

// The kPer values of one packed word written to dst: one or two 16-byte
// stores (8-byte for 8-bit words into 16-bit outputs) when `vec` (dst is
// aligned to the word's output bytes), else element by element.
template <typename TO, int kPer>
__device__ __forceinline__ void store_values(TO* dst, const float (&v)[kPer], bool vec) {
  constexpr int kBytes = kPer * (int)sizeof(TO);
  if (vec) {
    uint32_t u[kBytes / 4];
    if constexpr (sizeof(TO) == 4) {
#pragma unroll
      for (int i = 0; i < kPer; ++i) u[i] = __float_as_uint(v[i]);
    } else {
#pragma unroll
      for (int i = 0; i < kPer / 2; ++i) {
        TO lo = from_f32<TO>(v[2 * i]), hi = from_f32<TO>(v[2 * i + 1]);
        u[i] = (uint32_t)(*reinterpret_cast<uint16_t*>(&lo)) | ((uint32_t)(*reinterpret_cast<uint16_t*>(&hi)) << 16);
      }
    }
    if constexpr (kBytes % 16 == 0) {
#pragma unroll
      for (int k = 0; k < kBytes / 16; ++k)
        reinterpret_cast<uint4*>(dst)[k] = make_uint4(u[4 * k], u[4 * k + 1], u[4 * k + 2], u[4 * k + 3]);
    } else {
      static_assert(kBytes % 8 == 0, "a packed word's values fill whole 8-byte units");
#pragma unroll
      for (int k = 0; k < kBytes / 8; ++k) reinterpret_cast<uint2*>(dst)[k] = make_uint2(u[2 * k], u[2 * k + 1]);
    }
  } else {
#pragma unroll
    for (int i = 0; i < kPer; ++i) dst[i] = from_f32<TO>(v[i]);
  }
}

// Affine group dequantisation.  A block walks whole rows; thread t takes
// packed words t, t + blockDim.x, ... of a row, so a warp reads 128
// contiguous bytes and writes its values as contiguous vector stores.  A
// word's 32 / BITS values share one group (group_size >= 32 >= 32 / BITS):
// one scale and one bias, found by a shift (group_size is a power of two).
template <int BITS, typename TS, typename TO>
__global__ void __launch_bounds__(256)
dequant_kernel(const uint32_t* __restrict__ wq, const TS* __restrict__ scales, const TS* __restrict__ biases,
               int64_t rows, int wpr, int gpr, int gshift, bool vec, TO* __restrict__ out) {
  constexpr int kPer = 32 / BITS;
  constexpr uint32_t kMask = (1u << BITS) - 1u;
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const uint32_t* src = wq + r * wpr;
    const TS* sr = scales + r * gpr;
    const TS* br = biases + r * gpr;
    TO* dst = out + r * (int64_t)wpr * kPer;
    for (int w = threadIdx.x; w < wpr; w += blockDim.x) {
      const int g = (w * kPer) >> gshift;
      const float s = to_f32(sr[g]), b = to_f32(br[g]);
      const uint32_t q = __ldg(src + w);
      float v[kPer];
#pragma unroll
      for (int i = 0; i < kPer; ++i) v[i] = fmaf(s, (float)((q >> (i * BITS)) & kMask), b);
      store_values<TO, kPer>(dst + w * kPer, v, vec);
    }
  }
}

template <typename TS, typename TO>
cudaError_t dequant_dispatch(const uint32_t* wq, const void* scales, const void* biases, int64_t rows,
                             int64_t D, int group, int bits, void* out, cudaStream_t stream) {
  const int wpr = (int)(D * bits / 32), gpr = (int)(D / group);
  const int gshift = group == 32 ? 5 : group == 64 ? 6 : 7;
  // rows start on 16-byte boundaries when the output does (D is a multiple
  // of the group size, >= 32 values)
  const bool vec = (reinterpret_cast<uintptr_t>(out) & 15u) == 0;
  int64_t grid = rows < 148 * 8 ? rows : 148 * 8;
  if (grid < 1) grid = 1;
  const TS* s = static_cast<const TS*>(scales);
  const TS* b = static_cast<const TS*>(biases);
  TO* o = static_cast<TO*>(out);
  switch (bits) {
    case 2: dequant_kernel<2, TS, TO><<<(unsigned)grid, 256, 0, stream>>>(wq, s, b, rows, wpr, gpr, gshift, vec, o); break;
    case 4: dequant_kernel<4, TS, TO><<<(unsigned)grid, 256, 0, stream>>>(wq, s, b, rows, wpr, gpr, gshift, vec, o); break;
    case 8: dequant_kernel<8, TS, TO><<<(unsigned)grid, 256, 0, stream>>>(wq, s, b, rows, wpr, gpr, gshift, vec, o); break;
    default: return cudaErrorInvalidValue;
  }
  return launched();
}

template <typename TS>
cudaError_t dequant_out(const uint32_t* wq, const void* scales, const void* biases, int64_t rows, int64_t D,
                        int group, int bits, int out_dtype, void* out, cudaStream_t stream) {
  switch (out_dtype) {
    case CCE_F32: return dequant_dispatch<TS, float>(wq, scales, biases, rows, D, group, bits, out, stream);
    case CCE_F16: return dequant_dispatch<TS, __half>(wq, scales, biases, rows, D, group, bits, out, stream);
    case CCE_BF16: return dequant_dispatch<TS, __nv_bfloat16>(wq, scales, biases, rows, D, group, bits, out, stream);
  }
  return cudaErrorInvalidValue;
}

cudaError_t launch_dequantize(const uint32_t* wq, const void* scales, const void* biases, int scale_dtype,
                              int64_t rows, int64_t D, int group, int bits, int out_dtype, void* out,
                              cudaStream_t stream) {
  if (rows == 0 || D == 0) return cudaSuccess;
  switch (scale_dtype) {
    case CCE_F32: return dequant_out<float>(wq, scales, biases, rows, D, group, bits, out_dtype, out, stream);
    case CCE_F16: return dequant_out<__half>(wq, scales, biases, rows, D, group, bits, out_dtype, out, stream);
    case CCE_BF16: return dequant_out<__nv_bfloat16>(wq, scales, biases, rows, D, group, bits, out_dtype, out, stream);
  }
  return cudaErrorInvalidValue;
}

cudaError_t launch_pow2_absmax(const float* x, int64_t n, float* out, cudaStream_t stream) {
  pow2_absmax_kernel<<<1, 1024, 0, stream>>>(x, n, out);
  return launched();
}

cudaError_t launch_fill_f32(float* dst, float v, int64_t n, cudaStream_t stream) {
  if (n == 0) return cudaSuccess;
  fill_f32_kernel<<<grid_for(n, 256), 256, 0, stream>>>(dst, v, n);
  return launched();
}

}  // namespace cce
