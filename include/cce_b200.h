/*
 * cce_b200.h -- C ABI of the B200 (sm_100a) Cut Cross-Entropy library.
 *
 * This ABI replaces the nanobind module of the reference
 * (csrc/bindings.cpp:12-87) and the MLX primitives behind it
 * (csrc/cce/cce.h:10-101, csrc/cce/cce.cpp:123-375).  Everything crossing it
 * is a plain pointer or integer: no torch, no MLX, no C++ types, and no
 * exception ever crosses it.
 *
 * Conventions
 *   - Every tensor pointer is DEVICE memory on the current CUDA device,
 *     contiguous and row-major.  The caller allocates every input, output
 *     and workspace; the library never calls cudaMalloc on these paths.
 *   - ``stream`` is a cudaStream_t passed as void* (NULL = legacy default
 *     stream).  All work is enqueued asynchronously on it.
 *   - Return value: CCE_OK (0) or a negative CCE_ERR_* code; the message is in
 *     cce_last_error() (thread-local, valid until the next call on the thread).
 *   - Rows: N flattened tokens.  D: hidden size.  V: number of vocabulary rows
 *     of ``c`` handled by THIS call (a shard of the full vocabulary when the
 *     vocabulary is split across ranks); global vocab id = v_offset + local id.
 *   - targets are int32, already sanitised (ignored rows replaced by 0, as in
 *     mlx_cce/__init__.py:59-64 of the reference), with values in
 *     [0, V_total).  A target outside [v_offset, v_offset + V) is "not on this
 *     shard" and contributes a target logit of 0.
 */
#ifndef CCE_B200_H
#define CCE_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define CCE_API __attribute__((visibility("default")))
#else
#define CCE_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* status codes */
#define CCE_OK             0
#define CCE_ERR_SHAPE     -1  /* bad N / D / V / sizes                         */
#define CCE_ERR_DTYPE     -2  /* unsupported dtype code                         */
#define CCE_ERR_ALIGN     -3  /* pointer misaligned for the selected kernel     */
#define CCE_ERR_CUDA      -4  /* a CUDA runtime call or launch failed           */
#define CCE_ERR_ARCH      -5  /* device is not sm_100 (B200)                    */
#define CCE_ERR_WORKSPACE -6  /* workspace NULL or smaller than required        */
#define CCE_ERR_ARG       -7  /* NULL required pointer or bad flag combination  */

/* dtype codes (inputs e, c; bias has its own code) */
#define CCE_F32  0
#define CCE_F16  1
#define CCE_BF16 2

/* Vocabulary columns summarised by one tile statistic.  tile_max is laid out
 * [ceil(V / CCE_STAT_TILE)][N] (tile-major, rows contiguous). */
#define CCE_STAT_TILE 32

/* backward flags */
#define CCE_NEED_DE     1   /* write grad_e                                       */
#define CCE_NEED_DC     2   /* write grad_c                                       */
#define CCE_NEED_DBIAS  4   /* write grad_bias (fp32)                             */
#define CCE_DE_F32      8   /* grad_e is fp32 [N, D] (for a cross-rank sum), else e's dtype */
#define CCE_NO_FILTER  16   /* exact gradients: never skip a block                */

/* ln(2^-12): the reference's gradient-filter threshold (csrc/cce/cce.metal:143). */
#define CCE_FILTER_LOG_EPS (-8.3177661667f)

/* Library version (major * 10000 + minor * 100 + patch). */
CCE_API int cce_version(void);

/* Thread-local message describing the last failed call on this thread. */
CCE_API const char* cce_last_error(void);

/* Number of CUDA kernels this library has launched in this process (all
 * devices, all threads).  Instrumentation only; no counterpart in the
 * reference. */
CCE_API uint64_t cce_launch_count(void);

/* Tensor-core work the library's GEMM kernels actually issued on the current
 * device since the last reset: flops4[k] = 2 * 128 * 16 * (sum of N over the
 * M = 128, K = 16 MMAs issued) for k = 0 forward, 1 dlogits, 2 grad_e,
 * 3 grad_c.  Blocks skipped by the filter and MMA columns left out of a tile
 * are not counted; padding of partial tiles is.  Synchronous; reset != 0
 * clears the counters after reading.  Instrumentation only; no counterpart in
 * the reference. */
CCE_API int cce_mma_flops(uint64_t* flops4, int reset);

/* Synchronous health check of the current device: CCE_OK, or CCE_ERR_CUDA if
 * a tensor-core kernel gave up on a pipeline wait after its time limit (it then
 * returns instead of hanging; its outputs are invalid).  reset != 0 clears the
 * recorded state.  No counterpart in the reference (Metal kernels there cannot
 * time out). */
CCE_API int cce_device_status(int reset);

/* Diagnostic of that failure path: launches one thread that waits on a
 * pipeline barrier nothing completes, with a limit of limit_ns (at most 2 s);
 * the wait runs out, records CCE_SELFTEST_WAIT_CODE in the device status
 * word and returns, so cce_device_status then reports it and the context
 * stays usable.  No fault, trap or hang is involved. */
#define CCE_SELFTEST_WAIT_CODE 99
CCE_API int cce_selftest_wait_timeout(int64_t limit_ns, void* stream);

/* Number of vocabulary tile statistics per row: ceil(V / CCE_STAT_TILE). */
CCE_API int64_t cce_num_stat_tiles(int64_t V);

/*
 * Forward workspace size in bytes for cce_forward with these sizes.
 */
CCE_API size_t cce_forward_workspace_bytes(int64_t N, int64_t D, int64_t V, int dtype);

/*
 * cce_forward -- fused logits + per-tile max / sum-exp + target logit + LSE.
 *
 * Replaces cce_forward_raw (csrc/bindings.cpp:58-69, csrc/cce/cce.cpp:123-145)
 * and CutCrossEntropy::eval_gpu (csrc/cce/cce.cpp:207-277): the forward tile
 * kernel (csrc/cce/cce.metal:19-135) followed by reduce_tile_to_lse
 * (csrc/cce/cce.metal:332-355).  The [N, V] logits are never stored.
 *
 *   e        [N, D]   dtype          c [V, D] dtype
 *   bias     [V]      bias_dtype or NULL
 *   targets  [N]      int32 sanitised global ids
 *   tile_max [ceil(V/32)][N] fp32 out: max logit (+bias) of each row over
 *            each 32-column vocabulary tile (the backward's filter input)
 *   lse      [N] fp32 out: log-sum-exp over this call's V columns
 *   tgt      [N] fp32 out: logit (+bias) of the row's target when the target
 *            lies in [v_offset, v_offset + V), else 0
 *   workspace >= cce_forward_workspace_bytes(N, D, V, dtype)
 */
CCE_API int cce_forward(const void* e, const void* c, const void* bias, int bias_dtype,
                const int32_t* targets, int64_t N, int64_t D, int64_t V,
                int64_t v_offset, int dtype,
                float* tile_max, float* lse, float* tgt,
                void* workspace, size_t workspace_bytes, void* stream);

/*
 * cce_forward_noalloc -- cce_forward for callers that cannot allocate device
 * memory.  No counterpart in the reference (whose MLX runtime allocates every
 * buffer itself).
 *
 * Same arguments and results as cce_forward minus the workspace: the sum-exp
 * partials live in a static 32 MiB device array inside this library (held on
 * every GPU that loads the library, until the process exits).  For callers
 * that can pass inputs and outputs but own no allocator: a plugin or FFI slot
 * with a fixed memory contract, or a host that forbids allocation while it
 * runs.  It calls no cudaMalloc / cudaFree.
 *   - limit: 2 * ceil(V / 128) * N <= 8388608 (e.g. V = 128256, N <= 4185);
 *     larger calls return CCE_ERR_WORKSPACE and do nothing.
 *   - the first call in each CUDA context (normally: per device, in the
 *     device's primary context) looks up the array's device address with
 *     cudaGetSymbolAddress, with that device current; make that first call
 *     before any stream capture.  The address is cached per context id, so a
 *     host running its own driver-API context, or one that reset the device,
 *     gets the address that is valid in its current context.
 *   - all calls on a device share the array: calls that overlap on the GPU
 *     (different streams, or different host threads without ordering) race.
 *     Each call writes every partial it reads, so nothing carries over.
 */
CCE_API int cce_forward_noalloc(const void* e, const void* c, const void* bias, int bias_dtype,
                                const int32_t* targets, int64_t N, int64_t D, int64_t V,
                                int64_t v_offset, int dtype, float* tile_max, float* lse,
                                float* tgt, void* stream);

/*
 * cce_lse_combine -- merge P partial (lse, target-logit) rows into one.
 *
 *   part_lse, part_tgt: P rows of N fp32 values, row p starting at
 *   part_lse + p * part_stride (e.g. gathered from P vocabulary shards).
 *   lse[n] = log sum_p exp(part_lse[p][n]); tgt[n] = sum_p part_tgt[p][n]
 *   (tgt nullable); nll[n] (nullable) = lse[n] - tgt[n].  The outputs may
 *   alias no input.
 * The per-rank fold of reduce_tile_to_lse (csrc/cce/cce.metal:332-355) lifted
 * one level up, plus nll = lse + neg_target_logit of mlx_cce/__init__.py:32.
 */
CCE_API int cce_lse_combine(const float* part_lse, const float* part_tgt, int64_t P, int64_t N,
                    int64_t part_stride, float* lse, float* tgt, float* nll, void* stream);

/*
 * Backward workspace size in bytes for cce_backward with these sizes/flags.
 */
CCE_API size_t cce_backward_workspace_bytes(int64_t N, int64_t D, int64_t V, int dtype, int flags);

/*
 * cce_backward -- filtered recompute of softmax - onehot and the grad GEMMs.
 *
 * Replaces cce_backward_raw (csrc/bindings.cpp:71-86, csrc/cce/cce.cpp:152-179)
 * and CutCrossEntropyBwd::eval_gpu (csrc/cce/cce.cpp:283-375) running the
 * backward kernel (csrc/cce/cce.metal:146-326) with COMPUTE_DC, i.e. the
 * compute_all_grads path of reference/_fused_backward.py:1618-1655.
 *
 *   lse       [N] fp32: GLOBAL log-sum-exp (after any cross-shard combine)
 *   d_nll     [N] fp32: cotangent of each row's NLL (0 for ignored rows)
 *   tile_max  [ceil(V/32)][N] fp32 from cce_forward
 *   grad_e    [N, D] e's dtype, or fp32 with CCE_DE_F32 (overwritten)
 *   grad_c    [V, D] c's dtype (overwritten; NULL unless CCE_NEED_DC)
 *   grad_bias [V] fp32 (overwritten; NULL unless CCE_NEED_DBIAS)
 *   skip_stats device int64[2] (nullable): accumulates (skipped, total)
 *            (128-row x 32-column) blocks of this call
 *   filter_log_eps: a block whose every row has tile_max - lse below it and
 *            holds no target is skipped (CCE_FILTER_LOG_EPS = the reference's).
 */
CCE_API int cce_backward(const void* e, const void* c, const void* bias, int bias_dtype,
                 const int32_t* targets, const float* lse, const float* d_nll,
                 const float* tile_max, int64_t N, int64_t D, int64_t V,
                 int64_t v_offset, int dtype, int flags, float filter_log_eps,
                 void* grad_e, void* grad_c, float* grad_bias, int64_t* skip_stats,
                 void* workspace, size_t workspace_bytes, void* stream);

/*
 * cce_dequantize -- expand rows of an affine group-quantised classifier.
 *
 * No counterpart in the reference's library: its mlx-lm recipe dequantises
 * the whole [V, D] head with MLX before every call (README.md:84-95).  The
 * quantised layout is MLX's affine one for bits in {2, 4, 8}:
 *   wq     [rows][D * bits / 32] uint32: 32 / bits values per word, value j
 *          of a row in bits [(j * bits) % 32, +bits) of word (j * bits) / 32
 *   scales, biases [rows][D / group_size] in scale_dtype (F32 / F16 / BF16)
 *   out[r][j] = scales[r][j / group_size] * q + biases[r][j / group_size],
 *          written in out_dtype (F32 / F16 / BF16), [rows][D] row-major.
 * group_size in {32, 64, 128}, D a multiple of group_size.  Pass the first
 * row's pointers to expand a range of rows (a vocabulary chunk).
 */
CCE_API int cce_dequantize(const uint32_t* wq, const void* scales, const void* biases, int scale_dtype,
                           int64_t rows, int64_t D, int group_size, int bits, int out_dtype, void* out,
                           void* stream);

/* ---------------------------------------------------------------------------
 * Quantised classifier.  No counterpart in the reference's library: its
 * mlx-lm recipe (README.md:84-95) dequantises the whole [V, D] head with MLX
 * before every call.  Here the head stays quantised in HBM and the forward /
 * backward expand one vocabulary chunk at a time into a workspace buffer (two
 * buffers: the next chunk is expanded on a side stream while the current
 * chunk's GEMMs run), in e's dtype.  The head is frozen: no gradient for it.
 * --------------------------------------------------------------------------- */

typedef struct CceQuantHead {
  const uint32_t* wq;      /* [V][D * bits / 32] words, MLX's affine layout (see cce_dequantize) */
  const void* scales;      /* [V][D / group_size] in scale_dtype                                 */
  const void* biases;      /* [V][D / group_size] in scale_dtype                                 */
  int32_t scale_dtype;     /* CCE_F32 / F16 / BF16                                               */
  int32_t group_size;      /* 32, 64 or 128 (D must be a multiple)                               */
  int32_t bits;            /* 2, 4 or 8                                                          */
} CceQuantHead;

/* cce_forward with the classifier given as a quantised head (V rows). */
CCE_API size_t cce_forward_q_workspace_bytes(int64_t N, int64_t D, int64_t V, int dtype);
CCE_API int cce_forward_q(const void* e, const CceQuantHead* head, const void* bias, int bias_dtype,
                          const int32_t* targets, int64_t N, int64_t D, int64_t V, int64_t v_offset,
                          int dtype, float* tile_max, float* lse, float* tgt, void* workspace,
                          size_t workspace_bytes, void* stream);
/* cce_backward with a quantised head: CCE_NEED_DE and / or CCE_NEED_DBIAS
 * (CCE_NEED_DC is refused: the head is frozen). */
CCE_API size_t cce_backward_q_workspace_bytes(int64_t N, int64_t D, int64_t V, int dtype, int flags);
CCE_API int cce_backward_q(const void* e, const CceQuantHead* head, const void* bias, int bias_dtype,
                           const int32_t* targets, const float* lse, const float* d_nll,
                           const float* tile_max, int64_t N, int64_t D, int64_t V, int64_t v_offset,
                           int dtype, int flags, float filter_log_eps, void* grad_e, float* grad_bias,
                           int64_t* skip_stats, void* workspace, size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------------------
 * Vocabulary-sharded backward over NVLink peer memory.  No counterpart in the
 * reference (it has no multi-device code); this is the cross-rank sum of
 * grad_e that the sharded path needs, done with the ranks' own loads and
 * stores instead of a collective library.
 *
 * Every rank of a group (one process per GPU of one node) allocates one
 * exchange buffer with cce_peer_buffer_alloc, which returns a POSIX file
 * descriptor of the buffer's physical memory; sends it to every other rank of
 * the node (file descriptors travel between processes only through a Unix
 * socket, SCM_RIGHTS); maps the others' buffers with cce_peer_buffer_open;
 * and passes all of them in a CcePeerGroup.  The buffers are driver
 * virtual-memory allocations mapped with access for each rank's own device
 * only: no context-wide peer access is turned on, so the process's other
 * allocations stay as cheap as without the group.  Buffers are allocated once
 * per group, not per call (this is set-up, the only place this library
 * allocates device memory).
 * --------------------------------------------------------------------------- */

#define CCE_PEER_MAX_WORLD    16
/* cce_device_status codes of the exchange's bounded waits */
#define CCE_PEER_WAIT_PUSH    201  /* a rank's partial grad_e never arrived      */
#define CCE_PEER_WAIT_REDUCE  202  /* a rank's reduced rows never became ready   */

typedef struct CcePeerGroup {
  int32_t rank;            /* this rank, in [0, world)                              */
  int32_t world;           /* ranks in the group, 1..CCE_PEER_MAX_WORLD              */
  int64_t wait_limit_ns;   /* bound of each wait on another rank (<= 0: 10 s)        */
  size_t bytes;            /* size of every rank's buffer (all equal)                */
  void* bases[CCE_PEER_MAX_WORLD]; /* each rank's buffer as mapped in this process;
                                      bases[rank] = this rank's own                  */
} CcePeerGroup;

/* Exchange-buffer size for N rows of grad_e [N, D] over `world` ranks, the
 * result written in out_dtype (CCE_F32 / F16 / BF16). */
CCE_API size_t cce_peer_buffer_bytes(int64_t N, int64_t D, int world, int out_dtype);

/* Allocates a zero-initialised exchange buffer of at least `bytes` on the
 * current device, maps it at *ptr, and writes to *fd a new POSIX file
 * descriptor that shares it (the caller sends it to the other ranks and
 * closes it). */
CCE_API int cce_peer_buffer_alloc(size_t bytes, void** ptr, int* fd);
/* Maps another rank's buffer (its descriptor, received in this process, and
 * the same `bytes`) at *ptr with access for the current device.  The caller
 * may close `fd` afterwards. */
CCE_API int cce_peer_buffer_open(int fd, size_t bytes, void** ptr);
/* Unmaps a buffer mapped with cce_peer_buffer_open. */
CCE_API int cce_peer_buffer_close(void* ptr);
/* Unmaps and releases a buffer from cce_peer_buffer_alloc (its memory lives
 * on while another process still maps it). */
CCE_API int cce_peer_buffer_free(void* ptr);

/*
 * cce_backward_peer -- cce_backward for one vocabulary shard, with grad_e
 * summed over the group: on return (in stream order) every rank's grad_e holds
 * the full sum of all ranks' partials, in e's dtype (fp32 with CCE_DE_F32).
 * Arguments as cce_backward (c, bias, V, v_offset are this rank's shard; lse
 * the global one); grad_c / grad_bias stay sharded.  Every rank of the group
 * must make the same sequence of calls with the same N, D, dtype and flags.
 *
 * The last vocabulary chunk's grad_e GEMM stores each output tile straight
 * into the owning rank's buffer over NVLink (rows are owned in 128-row tiles),
 * each owner sums its rows in rank order (deterministic), and every rank
 * copies the other ranks' summed rows.  Waits on other ranks are bounded by
 * group->wait_limit_ns; when one runs out the call's grad_e is invalid,
 * cce_device_status reports CCE_PEER_WAIT_PUSH / _REDUCE, and the group's
 * buffers must be re-created.
 */
CCE_API int cce_backward_peer(const void* e, const void* c, const void* bias, int bias_dtype,
                              const int32_t* targets, const float* lse, const float* d_nll,
                              const float* tile_max, int64_t N, int64_t D, int64_t V,
                              int64_t v_offset, int dtype, int flags, float filter_log_eps,
                              void* grad_e, void* grad_c, float* grad_bias, int64_t* skip_stats,
                              void* workspace, size_t workspace_bytes, const CcePeerGroup* group,
                              void* stream);

#ifdef __cplusplus
}
#endif

#endif /* CCE_B200_H */
