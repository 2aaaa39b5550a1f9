// Auxiliary kernels: LSE combine, backward block mask, casts.
//
// - lse_combine_kernel: per row, fold P partial (max, sum-exp) pairs -- the
//   vocabulary tiles of one call, or the vocabulary shards of several ranks --
//   into lse = M + log(sum_p s_p * exp(m_p - M)) with M = max_p m_p.  This is
//   reduce_tile_to_lse of the reference (csrc/cce/cce.metal:332-355), with the
//   target-logit sum and nll = lse - tgt (mlx_cce/__init__.py:32) fused in.
// - block_mask_kernel: the reference's per-tile skip decision
//   (csrc/cce/cce.metal:190-204) taken once per (128-row block, 64-column
//   vocabulary tile) instead of inside the backward kernel.
#include "kernels.cuh"

namespace cce {

namespace {

constexpr int kCombRows = 32;    // rows per block (threadIdx.x)
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
  __shared__ float sm[kCombSlices][kCombRows + 1];
  __shared__ float ss[kCombSlices][kCombRows + 1];
  __shared__ float st[kCombSlices][kCombRows + 1];
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
  if (threadIdx.y == 0 && row < N) {
    float M = -INFINITY, S = 0.f, T = 0.f;
    for (int i = 0; i < kCombSlices; ++i) {
      fold(M, S, sm[i][threadIdx.x], ss[i][threadIdx.x]);
      T += st[i][threadIdx.x];
    }
    const float L = M + logf(S);
    lse[row] = L;
    if (tgt) tgt[row] = T;
    if (nll) nll[row] = L - T;
  }
}

__global__ void __launch_bounds__(kRowBlock)
block_mask_kernel(const float* __restrict__ tile_max, const float* __restrict__ lse,
                  const int32_t* __restrict__ targets, const float* __restrict__ d_nll, int64_t N,
                  int64_t V, int64_t v_offset, float log_eps, int no_filter, uint8_t* __restrict__ keep,
                  unsigned long long* __restrict__ skip_stats) {
  const int64_t j = blockIdx.x;   // vocabulary tile
  const int64_t i = blockIdx.y;   // row block
  const int64_t row = i * kRowBlock + threadIdx.x;
  const int64_t nVt = gridDim.x;
  int k = 0;
  if (row < N) {
    const float g = d_nll[row];
    if (g != 0.f) {  // rows with a zero cotangent contribute nothing
      if (no_filter) {
        k = 1;
      } else {
        const int64_t tl = (int64_t)targets[row] - v_offset;
        const bool hit = tl >= j * kStatTile && tl < (j + 1) * kStatTile && tl < V;
        k = hit || (tile_max[j * N + row] - lse[row] >= log_eps);
      }
    }
  }
  k = __syncthreads_or(k);
  if (threadIdx.x == 0) {
    keep[i * nVt + j] = (uint8_t)k;
    if (skip_stats) {
      atomicAdd(&skip_stats[1], 1ull);
      if (!k) atomicAdd(&skip_stats[0], 1ull);
    }
  }
}

template <typename T>
__global__ void cast_f32_kernel(const float* __restrict__ src, T* __restrict__ dst, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    dst[i] = from_f32<T>(src[i]);
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
                              float log_eps, bool no_filter, uint8_t* keep, int64_t* skip_stats,
                              cudaStream_t stream) {
  if (N == 0 || V == 0) return cudaSuccess;
  dim3 grid((unsigned)ceil_div(V, kStatTile), (unsigned)ceil_div(N, kRowBlock));
  block_mask_kernel<<<grid, kRowBlock, 0, stream>>>(tile_max, lse, targets, d_nll, N, V, v_offset,
                                                    log_eps, no_filter ? 1 : 0, keep,
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
