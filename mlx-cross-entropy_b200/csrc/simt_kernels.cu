// SIMT (CUDA-core FFMA) kernels: the fp32 path and the path for shapes the
// tensor-core kernels cannot take (16-bit rows not 16-byte aligned).
//
// Arithmetic follows the reference's tile kernels with fp32 accumulation:
//  - forward: csrc/cce/cce.metal:19-135 (tile logits, tile max, tile sum-exp,
//    target logit), here on 64-row x 128-column tiles;
//  - backward: csrc/cce/cce.metal:146-326, split into a dlogits pass
//    (w = d_nll * (exp(logit - lse) - [v == t]), cce.metal:276-281) and two
//    plain GEMMs (dE += w @ c, dC = w^T @ e, cce.metal:284-304) instead of
//    per-element atomics.
#include "kernels.cuh"

namespace cce {
namespace {

constexpr int BM = 64;     // rows of a forward / dlogits tile
constexpr int BN = 128;    // vocabulary columns of a tile
constexpr int SG = BN / kStatTile;  // statistics tiles per tile
static_assert(BN == kSimtLseTile, "one LSE partial per tile");
static_assert(kStatTile % 16 == 0 && BN % kStatTile == 0, "tile / statistics-tile layout");
// statistics tile (within the tile) of thread column tx + 16 j, tx < 16
__device__ __forceinline__ constexpr int gof(int j) { return (16 * j) / kStatTile; }
constexpr int BK = 16;
constexpr int THREADS = 256;

// Load a BM x BK tile of e and a BN x BK tile of c (rows contiguous in K) into
// shared memory transposed to [k][row], converting to fp32.
template <typename T>
__device__ __forceinline__ void load_ec_tiles(const T* __restrict__ e, const T* __restrict__ c,
                                              int64_t N, int64_t D, int64_t V, int64_t r0, int64_t v0,
                                              int64_t k0, float (*As)[BM + 4], float (*Bs)[BN + 4]) {
  const int tid = threadIdx.x;
#pragma unroll
  for (int it = 0; it < (BM * BK) / THREADS; ++it) {
    const int idx = tid + it * THREADS;
    const int r = idx / BK, k = idx % BK;
    const int64_t gr = r0 + r, gk = k0 + k;
    As[k][r] = (gr < N && gk < D) ? to_f32(e[gr * D + gk]) : 0.f;
  }
#pragma unroll
  for (int it = 0; it < (BN * BK) / THREADS; ++it) {
    const int idx = tid + it * THREADS;
    const int r = idx / BK, k = idx % BK;
    const int64_t gv = v0 + r, gk = k0 + k;
    Bs[k][r] = (gv < V && gk < D) ? to_f32(c[gv * D + gk]) : 0.f;
  }
}

// acc[i][j] = logit(row r0 + ty + 16 i, column v0 + tx + 16 j)
template <typename T>
__device__ __forceinline__ void tile_logits(const T* __restrict__ e, const T* __restrict__ c,
                                            int64_t N, int64_t D, int64_t V, int64_t r0, int64_t v0,
                                            float acc[4][8]) {
  __shared__ float As[BK][BM + 4];
  __shared__ float Bs[BK][BN + 4];
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;
  for (int64_t k0 = 0; k0 < D; k0 += BK) {
    load_ec_tiles<T>(e, c, N, D, V, r0, v0, k0, As, Bs);
    __syncthreads();
#pragma unroll
    for (int k = 0; k < BK; ++k) {
      float a[4], b[8];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = As[k][ty + 16 * i];
#pragma unroll
      for (int j = 0; j < 8; ++j) b[j] = Bs[k][tx + 16 * j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
}

template <typename TB>
__device__ __forceinline__ float bias_at(const void* bias, int64_t v) {
  return to_f32(reinterpret_cast<const TB*>(bias)[v]);
}

template <typename T, typename TB>
__global__ void __launch_bounds__(THREADS)
simt_fwd_kernel(const T* __restrict__ e, const T* __restrict__ c, const void* __restrict__ bias,
                const int32_t* __restrict__ targets, int64_t N, int64_t D, int64_t V, int64_t v_offset,
                float* __restrict__ tile_max, float* __restrict__ part_m, float* __restrict__ part_s,
                float* __restrict__ tgt) {
  const int64_t r0 = (int64_t)blockIdx.x * BM;
  const int64_t tile = blockIdx.y;
  const int64_t v0 = tile * BN;
  float acc[4][8];
  tile_logits<T>(e, c, N, D, V, r0, v0, acc);
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  float bv[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int64_t v = v0 + tx + 16 * j;
    bv[j] = (bias != nullptr && v < V) ? bias_at<TB>(bias, v) : 0.f;
  }
  // column tx + 16 j (tx < 16) lies in the tile's statistics tile 16 j / kStatTile
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t row = r0 + ty + 16 * i;
    float x[8];
    float m[SG];
#pragma unroll
    for (int g = 0; g < SG; ++g) m[g] = -INFINITY;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int64_t v = v0 + tx + 16 * j;
      x[j] = (v < V) ? acc[i][j] + bv[j] : -INFINITY;
      m[gof(j)] = fmaxf(m[gof(j)], x[j]);
    }
#pragma unroll
    for (int g = 0; g < SG; ++g)
#pragma unroll
      for (int o = 8; o >= 1; o >>= 1) m[g] = fmaxf(m[g], __shfl_xor_sync(0xffffffffu, m[g], o));
    float s[SG];
#pragma unroll
    for (int g = 0; g < SG; ++g) s[g] = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (m[gof(j)] != -INFINITY) s[gof(j)] += exp2f((x[j] - m[gof(j)]) * kLog2e);
#pragma unroll
    for (int g = 0; g < SG; ++g)
#pragma unroll
      for (int o = 8; o >= 1; o >>= 1) s[g] += __shfl_xor_sync(0xffffffffu, s[g], o);
    if (row < N) {
      if (tx == 0) {
#pragma unroll
        for (int g = 0; g < SG; ++g)
          if (v0 + g * kStatTile < V) tile_max[(SG * tile + g) * N + row] = m[g];
        // the tile's LSE partial: fold the statistics tiles' (max, sum-exp)
        float M = -INFINITY;
#pragma unroll
        for (int g = 0; g < SG; ++g) M = fmaxf(M, m[g]);
        float S = 0.f;
#pragma unroll
        for (int g = 0; g < SG; ++g)
          if (m[g] != -INFINITY) S += s[g] * exp2f((m[g] - M) * kLog2e);
        part_m[tile * N + row] = M;
        part_s[tile * N + row] = S;
      }
      const int64_t tl = (int64_t)targets[row] - v_offset;
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (tl == v0 + tx + 16 * j && tl < V) tgt[row] = x[j];
    }
  }
}

template <typename T, typename TB>
__global__ void __launch_bounds__(THREADS)
simt_dlogits_kernel(const T* __restrict__ e, const T* __restrict__ c, const void* __restrict__ bias,
                    const int32_t* __restrict__ targets, const float* __restrict__ lse,
                    const float* __restrict__ d_nll, const uint8_t* __restrict__ keep, int64_t N,
                    int64_t D, int64_t V, int64_t v_offset, int64_t vc0, int64_t vc_len, int64_t ld,
                    float* __restrict__ dl, float* __restrict__ grad_bias) {
  const int64_t r0 = (int64_t)blockIdx.x * BM;
  const int64_t v0 = vc0 + (int64_t)blockIdx.y * BN;   // local vocab id of column 0
  const int64_t vend = min(vc0 + vc_len, V);
  const int64_t nVt = ceil_div(V, kStatTile);
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  // the tile's SG statistics tiles
  const uint8_t* kr = keep + (r0 / kRowBlock) * nVt + v0 / kStatTile;
  uint32_t kmask = 0;
#pragma unroll
  for (int g = 0; g < SG; ++g)
    if (v0 / kStatTile + g < nVt && kr[g] != 0) kmask |= 1u << g;
  if (kmask == 0) {
    for (int idx = threadIdx.x; idx < BM * BN; idx += THREADS) {
      const int r = idx / BN, cc = idx % BN;
      const int64_t row = r0 + r, v = v0 + cc;
      if (row < N && v < vend) dl[row * ld + (v - vc0)] = 0.f;
    }
    return;
  }
  float acc[4][8];
  // c holds the chunk's rows: row 0 = local vocab id vc0
  tile_logits<T>(e, c, N, D, vend - vc0, r0, v0 - vc0, acc);
  __shared__ float colsum[BN];
  if (grad_bias) {
    for (int idx = threadIdx.x; idx < BN; idx += THREADS) colsum[idx] = 0.f;
    __syncthreads();
  }
  float bv[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int64_t v = v0 + tx + 16 * j;
    bv[j] = (bias != nullptr && v < V) ? bias_at<TB>(bias, v) : 0.f;
  }
  float cs[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) cs[j] = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t row = r0 + ty + 16 * i;
    if (row >= N) continue;
    const float g = d_nll[row];
    const float L = lse[row];
    const int64_t tl = (int64_t)targets[row] - v_offset;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int64_t v = v0 + tx + 16 * j;
      if (v < vend) {
        float w = 0.f;
        if ((kmask >> gof(j)) & 1u) {
          w = g * exp2f((acc[i][j] + bv[j] - L) * kLog2e);
          if (v == tl) w -= g;
        }
        dl[row * ld + (v - vc0)] = w;
        cs[j] += w;
      }
    }
  }
  if (grad_bias) {
#pragma unroll
    for (int j = 0; j < 8; ++j) atomicAdd(&colsum[tx + 16 * j], cs[j]);
    __syncthreads();
    for (int idx = threadIdx.x; idx < BN; idx += THREADS) {
      const int64_t v = v0 + idx;
      if (v < vend) atomicAdd(&grad_bias[v], colsum[idx]);
    }
  }
}

// Generic SIMT GEMM: out[m, n] (+)= sum_k A(m, k) * B(k, n), fp32 accumulate.
//   A(m, k) = A[m * a_sm + k * a_sk] (fp32), B(k, n) = B[k * b_sk + n * b_sn] (TB)
// A_M_CONTIG selects the coalesced load mapping for A.  Split K: block z
// covers k in [z * k_per, (z + 1) * k_per) and writes out + z * out_z.
constexpr int GM = 64, GN = 64, GK = 16;

template <typename TB, typename TO, bool A_M_CONTIG>
__global__ void __launch_bounds__(THREADS)
simt_gemm_kernel(const float* __restrict__ A, int64_t a_sm, int64_t a_sk, const TB* __restrict__ B,
                 int64_t b_sk, int64_t b_sn, int64_t M, int64_t Nn, int64_t K, TO* __restrict__ out,
                 int64_t ld_out, bool accumulate, int64_t k_per, int64_t out_z) {
  __shared__ float As[GK][GM + 4];
  __shared__ float Bs[GK][GN + 4];
  const int64_t m0 = (int64_t)blockIdx.y * GM, n0 = (int64_t)blockIdx.x * GN;
  const int64_t kbeg = (int64_t)blockIdx.z * k_per;
  const int64_t kend = kbeg + k_per < K ? kbeg + k_per : K;
  out += (int64_t)blockIdx.z * out_z;
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
  for (int64_t k0 = kbeg; k0 < kend; k0 += GK) {
#pragma unroll
    for (int it = 0; it < (GM * GK) / THREADS; ++it) {
      const int idx = threadIdx.x + it * THREADS;
      int m, k;
      if (A_M_CONTIG) { m = idx % GM; k = idx / GM; } else { k = idx % GK; m = idx / GK; }
      const int64_t gm = m0 + m, gk = k0 + k;
      As[k][m] = (gm < M && gk < kend) ? A[gm * a_sm + gk * a_sk] : 0.f;
    }
#pragma unroll
    for (int it = 0; it < (GN * GK) / THREADS; ++it) {
      const int idx = threadIdx.x + it * THREADS;
      const int n = idx % GN, k = idx / GN;
      const int64_t gn = n0 + n, gk = k0 + k;
      Bs[k][n] = (gn < Nn && gk < kend) ? to_f32(B[gk * b_sk + gn * b_sn]) : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < GK; ++k) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = As[k][ty + 16 * i];
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = Bs[k][tx + 16 * j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t m = m0 + ty + 16 * i;
    if (m >= M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t n = n0 + tx + 16 * j;
      if (n >= Nn) continue;
      float v = acc[i][j];
      if (accumulate) v += to_f32(out[m * ld_out + n]);
      out[m * ld_out + n] = from_f32<TO>(v);
    }
  }
}

// acc[i] = (accumulate ? acc[i] : 0) + part[0][i] + part[1][i] + ... in that
// order: the split-K partials summed deterministically.
__global__ void sum_splits_kernel(const float* __restrict__ part, int splits, int64_t n, float* __restrict__ acc,
                                  bool accumulate) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    float v = accumulate ? acc[i] : 0.f;
    for (int z = 0; z < splits; ++z) v += part[(int64_t)z * n + i];
    acc[i] = v;
  }
}

template <typename T>
cudaError_t fwd_dispatch_bias(const FwdArgs& a, cudaStream_t s) {
  dim3 grid((unsigned)ceil_div(a.N, BM), (unsigned)ceil_div(a.V, BN));
  const T* e = (const T*)a.e;
  const T* c = (const T*)a.c;
  switch (a.bias == nullptr ? CCE_F32 : a.bias_dtype) {
    case CCE_F32:
      simt_fwd_kernel<T, float><<<grid, THREADS, 0, s>>>(e, c, a.bias, a.targets, a.N, a.D, a.V,
                                                          a.v_offset, a.tile_max, a.part_m, a.part_s, a.tgt);
      break;
    case CCE_F16:
      simt_fwd_kernel<T, __half><<<grid, THREADS, 0, s>>>(e, c, a.bias, a.targets, a.N, a.D, a.V,
                                                           a.v_offset, a.tile_max, a.part_m, a.part_s, a.tgt);
      break;
    case CCE_BF16:
      simt_fwd_kernel<T, __nv_bfloat16><<<grid, THREADS, 0, s>>>(
          e, c, a.bias, a.targets, a.N, a.D, a.V, a.v_offset, a.tile_max, a.part_m, a.part_s, a.tgt);
      break;
    default:
      return cudaErrorInvalidValue;
  }
  return launched();
}

template <typename T>
cudaError_t dl_dispatch_bias(const BwdChunkArgs& a, cudaStream_t s) {
  dim3 grid((unsigned)ceil_div(a.N, BM), (unsigned)ceil_div(a.vc_len, BN));
  const T* e = (const T*)a.e;
  const T* c = (const T*)a.c_chunk;
  float* dl = (float*)a.dlogits;
#define CCE_DL_LAUNCH(TB)                                                                        \
  simt_dlogits_kernel<T, TB><<<grid, THREADS, 0, s>>>(e, c, a.bias, a.targets, a.lse, a.d_nll,    \
                                                      a.keep, a.N, a.D, a.V, a.v_offset, a.vc0, \
                                                      a.vc_len, a.vc_ld, dl, a.grad_bias)
  switch (a.bias == nullptr ? CCE_F32 : a.bias_dtype) {
    case CCE_F32: CCE_DL_LAUNCH(float); break;
    case CCE_F16: CCE_DL_LAUNCH(__half); break;
    case CCE_BF16: CCE_DL_LAUNCH(__nv_bfloat16); break;
    default: return cudaErrorInvalidValue;
  }
#undef CCE_DL_LAUNCH
  return launched();
}

}  // namespace

cudaError_t simt_forward(const FwdArgs& a, cudaStream_t s) {
  if (a.N == 0 || a.V == 0) return cudaSuccess;
  switch (a.dtype) {
    case CCE_F32: return fwd_dispatch_bias<float>(a, s);
    case CCE_F16: return fwd_dispatch_bias<__half>(a, s);
    case CCE_BF16: return fwd_dispatch_bias<__nv_bfloat16>(a, s);
  }
  return cudaErrorInvalidValue;
}

cudaError_t simt_dlogits(const BwdChunkArgs& a, cudaStream_t s) {
  if (a.N == 0 || a.vc_len == 0) return cudaSuccess;
  switch (a.dtype) {
    case CCE_F32: return dl_dispatch_bias<float>(a, s);
    case CCE_F16: return dl_dispatch_bias<__half>(a, s);
    case CCE_BF16: return dl_dispatch_bias<__nv_bfloat16>(a, s);
  }
  return cudaErrorInvalidValue;
}

int simt_grad_e_splits(int64_t N, int64_t D, int64_t vc) {
  // enough blocks for two waves of 148 SMs, at most 8 splits of >= 1024 rows
  const int64_t tiles = ceil_div(N, GM) * ceil_div(D, GN);
  int64_t sp = ceil_div(2 * 148, tiles > 0 ? tiles : 1);
  if (sp > 8) sp = 8;
  if (sp > vc / 1024) sp = vc / 1024;
  return sp < 1 ? 1 : (int)sp;
}

cudaError_t simt_grad_e(const BwdChunkArgs& a, float* grad_e_acc, bool accumulate, float* part, int splits,
                        cudaStream_t s) {
  if (a.N == 0 || a.D == 0) return cudaSuccess;
  // A(m = row, k = v) = dl[row * ld + v]; B(k = v, n = d) = c_chunk[v * D + d] (row vc0 + v of c)
  // Few output tiles (small N x D) leave most SMs idle over a long K: the K
  // range is then split over `splits` blocks per tile writing partials that
  // sum_splits_kernel adds in split order.
  const bool split = splits > 1 && part != nullptr;
  const int sp = split ? splits : 1;
  const int64_t k_per = split ? ceil_div(ceil_div(a.vc_len, sp), GK) * GK : a.vc_len;
  dim3 grid((unsigned)ceil_div(a.D, GN), (unsigned)ceil_div(a.N, GM), (unsigned)sp);
  const float* dl = (const float*)a.dlogits;
  float* out = split ? part : grad_e_acc;
  const bool acc_in = split ? false : accumulate;
  const int64_t out_z = a.N * a.D;
#define CCE_GE_LAUNCH(T)                                                                       \
  simt_gemm_kernel<T, float, false><<<grid, THREADS, 0, s>>>(                                  \
      dl, a.vc_ld, 1, (const T*)a.c_chunk, a.D, 1, a.N, a.D, a.vc_len, out, a.D, acc_in, k_per, out_z)
  switch (a.dtype) {
    case CCE_F32: CCE_GE_LAUNCH(float); break;
    case CCE_F16: CCE_GE_LAUNCH(__half); break;
    case CCE_BF16: CCE_GE_LAUNCH(__nv_bfloat16); break;
    default: return cudaErrorInvalidValue;
  }
#undef CCE_GE_LAUNCH
  cudaError_t err = launched();
  if (err != cudaSuccess || !split) return err;
  const int64_t n = a.N * a.D;
  int64_t blocks = ceil_div(n, 256);
  if (blocks > 148 * 8) blocks = 148 * 8;
  sum_splits_kernel<<<(unsigned)blocks, 256, 0, s>>>(part, sp, n, grad_e_acc, accumulate);
  return launched();
}

cudaError_t simt_grad_c(const BwdChunkArgs& a, void* grad_c, cudaStream_t s) {
  if (a.vc_len == 0 || a.D == 0) return cudaSuccess;
  // A(m = v, k = row) = dl[row * ld + v]; B(k = row, n = d) = e[row * D + d]
  dim3 grid((unsigned)ceil_div(a.D, GN), (unsigned)ceil_div(a.vc_len, GM));
  const float* dl = (const float*)a.dlogits;
#define CCE_GC_LAUNCH(T)                                                                     \
  simt_gemm_kernel<T, T, true><<<grid, THREADS, 0, s>>>(dl, 1, a.vc_ld, (const T*)a.e, a.D, 1, \
                                                        a.vc_len, a.D, a.N,                    \
                                                        (T*)grad_c + a.vc0 * a.D, a.D, false, a.N, 0)
  switch (a.dtype) {
    case CCE_F32: CCE_GC_LAUNCH(float); break;
    case CCE_F16: CCE_GC_LAUNCH(__half); break;
    case CCE_BF16: CCE_GC_LAUNCH(__nv_bfloat16); break;
    default: return cudaErrorInvalidValue;
  }
#undef CCE_GC_LAUNCH
  return launched();
}

}  // namespace cce
