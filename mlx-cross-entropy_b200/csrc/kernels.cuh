// Internal launch interface between the C-ABI layer (cce_abi.cu) and the
// kernel translation units.  All launchers enqueue on `stream` and return the
// cudaError_t of the launch.
#pragma once

#include "common.cuh"
#include "peer.cuh"

namespace cce {

// Counts one kernel launch (cce_launch_count) and returns cudaGetLastError().
cudaError_t launched();

// Records `msg` as this thread's cce_last_error() and returns `code`.
int report_error(int code, const char* msg);

// Process-unique id of the CUDA context current on this thread (cuCtxGetId);
// *id = 0 when no context is current yet.  False if the driver calls fail.
// Per-context host state (device addresses of symbols, streams) is keyed by
// it: device ordinals are not enough once a host runs its own driver-API
// context or resets a device.
bool current_context_id(unsigned long long* id);

struct FwdArgs {
  const void* e;
  const void* c;
  const void* bias;
  int bias_dtype;
  const int32_t* targets;
  int64_t N, D, V, v_offset;
  int dtype;
  float* tile_max;  // [ceil(V / kStatTile)][N]: row max over each statistics tile (filter input)
  float* part_m;    // [P][N] (workspace): row max over each kernel tile, P = ceil(V / lse_tile)
  float* part_s;    // [P][N] (workspace): row sum of exp(logit - part_m) over the same columns
  float* tgt;       // [N]
};

struct BwdChunkArgs {
  const void* e;
  const void* c;         // row 0 of this call's c (the dense head; nullptr for a quantised one)
  const void* c_chunk;   // row vc0 of c: the chunk's vc_len rows (the dequantised chunk buffer
                         // for a quantised head); the chunk kernels read c through it
  const void* bias;
  int bias_dtype;
  const int32_t* targets;
  const float* lse;
  const float* d_nll;
  const uint8_t* keep;   // [nRb][nVt] block mask
  const uint32_t* keep_t;  // [ceil(V/128)][keep_t_ld] words: bit r of row m = a kept block of
                           // row block r in the 128 vocabulary columns of m (grad_c's M tiles)
  int64_t keep_t_ld;
  int64_t N, D, V, v_offset;
  int dtype;
  int64_t vc0;           // first local vocab row of the chunk
  int64_t vc_len;        // rows in the chunk
  int64_t vc_ld;         // row stride of the dlogits buffer (elements)
  void* dlogits;         // [N][vc_ld], fp32 (SIMT path) or 16-bit (tensor-core path)
  float* grad_bias;      // [V] fp32 or nullptr
  int* counters;         // 4 zeroed counters of this chunk (dlogits, grad_e, grad_c tile claims; the
                         // dlogits live-tile count) or nullptr
  const float* scale;    // fp16 tensor-core path: {s, 1/s} with s = 2^ceil(log2 max|d_nll|); else nullptr
  const int* dl_list = nullptr;  // the chunk's live dlogits tiles (tc_dlogits_lists), count in counters[3]
};

// ---- auxiliary kernels (aux_kernels.cu) ----
// (max, sum-exp) pairs, row p at part_max + p * ld (part_sum == nullptr: the
// entries are LSEs, i.e. pairs with sum 1)
cudaError_t launch_lse_combine(const float* part_max, const float* part_sum, const float* part_tgt,
                               int64_t P, int64_t N, int64_t ld, float* lse, float* tgt, float* nll,
                               cudaStream_t stream);
cudaError_t launch_block_mask(const float* tile_max, const float* lse, const int32_t* targets,
                              const float* d_nll, int64_t N, int64_t V, int64_t v_offset,
                              float log_eps, bool no_filter, uint8_t* keep, uint32_t* keep_t,
                              int64_t keep_t_ld, int64_t* skip_stats, cudaStream_t stream);
cudaError_t launch_cast_f32(const float* src, void* dst, int dtype, int64_t n, cudaStream_t stream);
// out[r][j] = scales[r][j / group] * q[r][j] + biases[r][j / group]  (cce_dequantize)
cudaError_t launch_dequantize(const uint32_t* wq, const void* scales, const void* biases, int scale_dtype,
                              int64_t rows, int64_t D, int group, int bits, int out_dtype, void* out,
                              cudaStream_t stream);
// dst[i] = a[i] + b[i], written in dtype (CCE_F32 / F16 / BF16)
cudaError_t launch_sum2_f32(const float* a, const float* b, void* dst, int dtype, int64_t n, cudaStream_t stream);
// out[0] = s = the power of two >= max |x| (1 if all zero), out[1] = 1 / s
cudaError_t launch_pow2_absmax(const float* x, int64_t n, float* out, cudaStream_t stream);
cudaError_t launch_fill_f32(float* dst, float v, int64_t n, cudaStream_t stream);

// ---- SIMT kernels (simt_kernels.cu): any dtype, any shape ----
cudaError_t simt_forward(const FwdArgs& a, cudaStream_t stream);
// vocabulary columns per LSE partial of simt_forward / tc_forward
constexpr int64_t kSimtLseTile = 128;
constexpr int64_t kTcLseTile = 256;
cudaError_t simt_dlogits(const BwdChunkArgs& a, cudaStream_t stream);
// grad_e_acc[N, D] (+)= dl[N, vc_len] @ c[v_offset-local rows vc0.., D]; with
// splits > 1 the K range is split over that many partial slabs part[splits][N][D]
// (workspace), summed in split order
cudaError_t simt_grad_e(const BwdChunkArgs& a, float* grad_e_acc, bool accumulate, float* part, int splits,
                        cudaStream_t stream);
// K splits simt_grad_e uses for an N x D output over chunks of vc rows
int simt_grad_e_splits(int64_t N, int64_t D, int64_t vc);
// grad_c[vc0 .. vc0+vc_len, D] = dl^T @ e, written in dtype
cudaError_t simt_grad_c(const BwdChunkArgs& a, void* grad_c, cudaStream_t stream);

// ---- tcgen05 kernels (tc_kernels.cu): 16-bit dtypes, D % 8 == 0 ----
bool tc_supported(const void* e, const void* c, int64_t D, int dtype);
bool tc_backward_supported(const void* e, const void* c, int64_t D, int dtype);
// Reads (and optionally clears) the tensor-core kernels' device status word:
// 0 = ok, > 0 = code of a bounded wait that timed out, -1 = read failed.
int tc_read_status(bool reset);
// Executed MMA FLOPs per kernel kind (forward, dlogits, grad_e, grad_c) since
// the last reset; 0 = ok, -1 = read failed.
int tc_read_mma_flops(uint64_t* out4, bool reset);
cudaError_t tc_forward(const FwdArgs& a, cudaStream_t stream);
cudaError_t tc_dlogits(const BwdChunkArgs& a, cudaStream_t stream);
// Lists, per vocabulary chunk of vc rows, the dlogits work units with a kept
// block in schedule order: chunk ch's ids at lists + ch * tc_dlogits_list_len(N, vc),
// their count in counters[4 ch + 3] (zeroed before).  One block per chunk.
int64_t tc_dlogits_list_len(int64_t N, int64_t vc);
cudaError_t tc_dlogits_lists(const uint8_t* keep, int64_t N, int64_t D, int64_t V, int64_t vc, int* lists,
                             int* counters, cudaStream_t stream);
// acc2[2][N][D] fp32: each output tile's two K halves of this chunk are
// stored (accumulate = false) or added into slabs 0 and 1; grad_e is
// acc2[0] + acc2[1] after the last chunk (launch_sum2_f32).  With `push`
// (the last chunk of a vocabulary-sharded backward) each half, plus its slab
// when accumulating, goes to its rows' owner rank instead (peer.cuh).
struct PeerPush {
  peer::Peers peers;
  peer::Layout layout;
};
cudaError_t tc_grad_e(const BwdChunkArgs& a, float* acc2, bool accumulate, const PeerPush* push,
                      cudaStream_t stream);
cudaError_t tc_grad_c(const BwdChunkArgs& a, void* grad_c, cudaStream_t stream);
// one bounded pipeline wait that nothing satisfies: records `code` after limit_ns
cudaError_t tc_selftest_wait(uint64_t limit_ns, int code, cudaStream_t stream);

// ---- cross-rank grad_e exchange (peer.cu) ----
namespace peer {
// partial rows src[nslab][N][D] fp32 -> their owners' receive slots; raises `pushed`
cudaError_t launch_push(const Peers& P, const Layout& L, const float* src, int nslab, int64_t N, int64_t D,
                        cudaStream_t stream);
// reduce this rank's rows (nslot slots per source) into out (out_dtype) and the
// reduced area, then gather the other ranks' rows into out
cudaError_t launch_reduce_gather(const Peers& P, const Layout& L, int nslot, int64_t N, int64_t D, int out_dtype,
                                 void* out, uint64_t limit_ns, cudaStream_t stream);
// status word of the exchange kernels' bounded waits (0 = ok, -1 = read failed)
int read_status(bool reset);
}  // namespace peer

}  // namespace cce
