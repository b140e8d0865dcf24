/*
 * quipsharp_b200 -- C ABI of the B200 (sm_100a) kernels behind QuIP#'s
 * quantized-linear forward path.
 *
 * Every entry point takes plain device pointers owned by the caller, sizes,
 * and a CUDA stream (cudaStream_t passed as qs_stream_t; NULL = legacy default
 * stream).  Work is enqueued on that stream; nothing synchronises unless the
 * comment says so.  No entry point allocates device memory: buffers that a
 * path needs beyond its inputs and outputs ("workspace") are passed in by the
 * caller, who asks for their size with the matching *_bytes() function.
 *
 * Return value: QS_OK (0) or one of the qs_status codes; qs_last_error()
 * gives a message for the last failing call on the calling thread.  The
 * status codes map onto the exceptions the reference raises for the same
 * conditions (see each entry point).
 *
 * Reference citations are `path:line` inside the reference project
 * (numbersletter/quipsharp).
 */
#ifndef QUIPSHARP_B200_H
#define QUIPSHARP_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st *qs_stream_t; /* == cudaStream_t */

typedef enum qs_status {
  QS_OK = 0,
  QS_ERR_INVALID_ARG = 1, /* bad pointer / size / enum value                     */
  QS_ERR_NOT_POW2 = 2,    /* fwht on a non-power-of-two size (ValueError, hadamard.py:28-29) */
  QS_ERR_ODD_DIM = 3,     /* RFFT on an odd size (AssertionError, rfft.py:42, rfft.py:55)   */
  QS_ERR_INDEX = 4,       /* 1-bit codebook index outside [-256, 256) (IndexError, e8_1bit.py:87) */
  QS_ERR_UNSUPPORTED = 5, /* size beyond what the kernels handle                  */
  QS_ERR_ALIGNMENT = 6,   /* pointer not aligned as the kernel requires           */
  QS_ERR_CUDA = 7,        /* a CUDA runtime call or launch failed                 */
  QS_ERR_WORKSPACE = 8,   /* workspace missing or smaller than *_bytes() asked for */
  QS_ERR_TIMEOUT = 9      /* a kernel gave up a bounded pipeline wait (see qs_device_status) */
} qs_status;

/* Codebook kinds (one per RVQ stage). */
typedef enum qs_codebook_kind {
  QS_CB_E8P = 0,    /* 16-bit E8P code per 8 weights, quipsharp/codebooks/e8p.py */
  QS_CB_E8_1BIT = 1 /* 8-bit index per 8 weights, quipsharp/codebooks/e8_1bit.py */
} qs_codebook_kind;

/* Element types. */
typedef enum qs_dtype {
  QS_F32 = 0, QS_F16 = 1, QS_BF16 = 2, QS_I16 = 3, QS_I32 = 4, QS_I64 = 5
} qs_dtype;

/* Incoherence transform of a layer (quipsharp/incoherence.py:115-131). */
typedef enum qs_transform { QS_RHT = 0, QS_RFFT = 1 } qs_transform;

const char *qs_version(void);
const char *qs_last_error(void);

/* Synchronises the stream and reports whether any kernel of this library gave
 * up a bounded wait inside its pipeline since the last call (QS_ERR_TIMEOUT;
 * the results of that launch are invalid).  The kernels never spin without a
 * limit: a stalled pipeline ends the kernel with this flag set instead of
 * hanging the GPU.  No counterpart in the reference (pure Python). */
int qs_device_status(qs_stream_t stream);

/* Limit, in nanoseconds, of the bounded waits between the warps of the
 * pipelined kernels (default 4 s; 0 restores the default), applied to launches
 * made after the call, process-wide.  A wait that runs out ends its kernel
 * early with the qs_device_status flag set; the kernel still waits for its own
 * copies and tensor-core work in flight (fixed 4 s limit) before it exits.
 * Lower it to detect a stalled pipeline sooner.  No counterpart in the
 * reference (pure Python). */
int qs_set_wait_limit_ns(uint64_t ns);
uint64_t qs_wait_limit_ns(void);

/* Host-only.  Writes the 256x8 float32 table of `kind` (row-major) to host
 * memory: E8P = build_abs_table() (quipsharp/codebooks/e8p.py:84-89),
 * E8_1BIT = build_table() (quipsharp/codebooks/e8_1bit.py:67-71). */
int qs_codebook_table(int kind, float *out_host);

/* E8PCodebook.dequantize (quipsharp/codebooks/e8p.py:197-199) and
 * E8OneBitCodebook.dequantize (quipsharp/codebooks/e8_1bit.py:86-87):
 * out[i*8 + j] = decode(codes[i])[j], bit-exact float32.  codes has element
 * type code_dtype (QS_I16, QS_I32 or QS_I64); E8P uses the low 16 bits of
 * each code (e8p.py:174-180).  For E8_1BIT an index outside [-256, 256)
 * returns QS_ERR_INDEX (this check synchronises the stream). */
int qs_decode(int kind, const void *codes, int code_dtype, int64_t count, float *out,
              qs_stream_t stream);

/* rvq_dequantize (quipsharp/rvq.py:83-88) through RVQCodebookAdapter.dequantize
 * (quipsharp/quantize.py:43-45): out = sum_s fl32(decode_s(codes[s][i]) *
 * stage_scales[s]), accumulated in stage order.  stage_scales is host memory
 * (float32 per stage). */
int qs_rvq_decode(int stages, const int *kinds, const void *const *codes, int code_dtype,
                  const float *stage_scales, int64_t count, float *out, qs_stream_t stream);

/* dequantize_linear (quipsharp/quantize.py:107-113) on the QuantizedLinear
 * int16 buffer (quipsharp/checkpoint.py:99-103, :132-139):
 * codes is int16 (stages, m, n/8), out is float32 (m, n).  stage_scales is
 * host memory or NULL for a plain (non-RVQ) codebook; layer_scale points to
 * the float32 `scale` buffer on the device. */
int qs_dequantize_linear(const int16_t *codes, int stages, const int *kinds,
                         const float *stage_scales, const float *layer_scale, int64_t m,
                         int64_t n, float *out, qs_stream_t stream);

/* fwht (quipsharp/hadamard.py:17-40) over rows of length n (a power of two,
 * n <= 32768), fused with the sign vectors of transform_input / transform_output
 * (quipsharp/incoherence.py:86-93): y = post * H_n(pre * x) / sqrt(n).
 * pre/post are float32 device vectors of length n or NULL.  x and y have
 * element type dtype (QS_F32, QS_F16, QS_BF16), row strides ld_x / ld_y
 * elements; computation is float32. */
int qs_fwht(const void *x, int64_t ld_x, void *y, int64_t ld_y, int dtype, int64_t rows,
            int64_t n, const float *pre, const float *post, qs_stream_t stream);

/* to_transformed_space (inverse = 0, quipsharp/rfft.py:37-47) and
 * from_transformed_space (inverse = 1, quipsharp/rfft.py:50-60) over rows of
 * length n (even, n/2 <= 32768, prime factors of n/2 at most 43):
 * forward: y = view_as_real(FFT_ortho(view_as_complex(x) * phase));
 * inverse: y = view_as_real(IFFT_ortho(view_as_complex(x)) * conj(phase)).
 * phase is complex64 (interleaved float2) of length n/2 on the device. */
int qs_rfft(int inverse, const void *x, int64_t ld_x, void *y, int64_t ld_y, int dtype,
            int64_t rows, int64_t n, const void *phase, qs_stream_t stream);

/* Size in bytes of the kernel-ready weight stream for a layer of `stages`
 * codebooks (kinds) with m outputs and n inputs, as written by qs_pack_codes. */
int64_t qs_packed_bytes(int stages, const int *kinds, int64_t m, int64_t n);

/* Re-lays the QuantizedLinear int16 codes (stages, m, n/8) into the tiled
 * bit-sliced stream the fused kernels read.  The mapping is a bijection of
 * the code bits (no information is dropped); 1-bit stages are narrowed to
 * uint8 (an index >= 256 returns QS_ERR_INDEX, as table indexing does in
 * e8_1bit.py:87; this check synchronises the stream). */
int qs_pack_codes(const int16_t *codes, int stages, const int *kinds, int64_t m, int64_t n,
                  void *packed, int64_t packed_bytes, qs_stream_t stream);

/* Workspace bytes qs_linear_fwd needs for `batch` rows of a layer (m, n). */
int64_t qs_linear_workspace_bytes(int64_t batch, int64_t m, int64_t n);

/* QuantizedLinear.forward (quipsharp/checkpoint.py:141-146) ->
 * linear_forward (quipsharp/quantize.py:116-124):
 *   y = cast(transform_out(transform_in(float(x)) @ What^T) + bias)
 * x: (batch, n) of x_dtype (QS_F32/F16/BF16), y: (batch, m) of the same type.
 * packed: from qs_pack_codes.  stage_scales: host float32 per stage or NULL
 * for a plain codebook.  layer_scale: device pointer to the float32 `scale`.
 * transform QS_RHT uses su (m) / sv (n) float32; QS_RFFT uses phase_u (m/2) /
 * phase_v (n/2) complex64.  bias: float32 (m) or NULL.  workspace: device
 * buffer of qs_linear_workspace_bytes(batch, m, n) bytes (256-byte aligned). */
int qs_linear_fwd(const void *x, int x_dtype, int64_t batch, int64_t n, int64_t m,
                  const void *packed, int stages, const int *kinds, const float *stage_scales,
                  const float *layer_scale, int transform, const float *su, const float *sv,
                  const void *phase_u, const void *phase_v, const float *bias, void *y,
                  void *workspace, int64_t workspace_bytes, qs_stream_t stream);

/* qs_linear_fwd for callers that cannot allocate device memory (no
 * counterpart in the reference).  Same arguments and result as qs_linear_fwd
 * without the workspace: it uses a built-in 8 MiB device array instead, which
 * every GPU that loads the library holds until exit, so a caller whose memory
 * is owned by a fixed-budget allocator (a server that reserved HBM up front, a
 * plugin host) or that must avoid cudaMalloc's implicit synchronisation needs
 * no allocation.  Returns QS_ERR_WORKSPACE when qs_linear_workspace_bytes(batch,
 * m, n) exceeds 8 MiB.  The first call on a device looks up the array's device
 * address (make it before any CUDA graph capture).  Calls share the array:
 * calls that overlap on the GPU (other streams or threads) race. */
int qs_linear_fwd_noalloc(const void *x, int x_dtype, int64_t batch, int64_t n, int64_t m,
                          const void *packed, int stages, const int *kinds,
                          const float *stage_scales, const float *layer_scale, int transform,
                          const float *su, const float *sv, const void *phase_u,
                          const void *phase_v, const float *bias, void *y, qs_stream_t stream);

/* One layer of qs_linear_fwd_group: the arguments of qs_linear_fwd that
 * follow (x, x_dtype, batch, n), which the layers of a group share. */
typedef struct qs_linear_layer {
  int64_t m;
  const void *packed;
  int stages;
  const int *kinds;
  const float *stage_scales;
  const float *layer_scale;
  int transform;
  const float *su;
  const float *sv;
  const void *phase_u;
  const void *phase_v;
  const float *bias;
  void *y;
  void *workspace;
  int64_t workspace_bytes;
} qs_linear_layer;

#define QS_GROUP_MAX_LAYERS 8
/* The layers of a decoder that read one input ([q,k,v], [gate,up]; the
 * reference groups them in architectures.py:52-94 get_linear_groups) in one
 * call: y_i = qs_linear_fwd(x, layers[i]) for each of `count` layers
 * (1..QS_GROUP_MAX_LAYERS).  At batches of at most 32 tokens layer 0 runs on
 * `stream` and the others on side streams of this library that fork from
 * `stream` and join back into it, so the group's latency-bound transform steps
 * and its matmuls overlap on the GPU; larger batches, whose kernels each fill
 * the GPU, run the layers one after another on `stream`.  Work queued on
 * `stream` after the call sees every y_i.  The call may
 * be captured in a CUDA graph (the side streams join the capture); make the
 * first call on a device outside capture (it creates the side streams).
 * Every layer is validated before anything is launched.  Workspaces and
 * outputs must not overlap one another (the layers run concurrently).
 * Calls from several host threads are serialised. */
int qs_linear_fwd_group(const void *x, int x_dtype, int64_t batch, int64_t n, int count,
                        const qs_linear_layer *layers, qs_stream_t stream);

/* The three steps of qs_linear_fwd, for callers that put a collective between
 * the matmul and the output transform (column-sharded tensor parallelism:
 * each rank runs qs_linear_input + qs_linear_matmul on its rows of the
 * weight, the y1 shards are all-gathered, then every rank runs
 * qs_linear_output on the full y1).
 * Batches above 32 tokens run the prefill matmul (fused decode + tcgen05
 * tensor-core GEMM); smaller ones the decode-regime kernel.
 *  - qs_linear_input: x -> x2 (fp16 tiles + per-row scale in workspace) and
 *    zeroes y1 (batch, m_local) float32.
 *  - qs_linear_matmul: y1 += x2 @ What_local^T * scales (rows m_local).
 *  - qs_linear_output: y = cast(transform_out(y1) + bias).  With shards == 1,
 *    y1 is float32 (batch, m) with row stride ld_y1.  With shards = P > 1, y1
 *    is the rank-major result of an all-gather of P shards of (batch, m/P):
 *    element (b, c) sits at ((c / (m/P)) * batch + b) * (m/P) + c % (m/P)
 *    (ld_y1 is ignored), so no re-layout copy is needed after the gather.
 *    y1 is consumed: for many rows of an RFFT layer (shards == 1, ld_y1 == m)
 *    the transform runs in two passes and uses y1 as its scratch, so its
 *    contents are unspecified afterwards. */
/* Bytes of the x2 workspace of qs_linear_input / qs_linear_matmul: the fp16
 * operand, the per-row scales and, for RFFT widths that transform in two passes
 * (n/2 = P * 2^a >= 4096), a float32 scratch row per token. */
int64_t qs_linear_input_bytes(int64_t batch, int64_t n);
int qs_linear_input(const void *x, int x_dtype, int64_t batch, int64_t n, int transform,
                    const float *sv, const void *phase_v, void *x2_workspace,
                    int64_t x2_workspace_bytes, float *y1, int64_t m_local, qs_stream_t stream);
int qs_linear_matmul(const void *x2_workspace, int64_t batch, int64_t n, int64_t m_local,
                     const void *packed, int stages, const int *kinds,
                     const float *stage_scales, const float *layer_scale, float *y1,
                     qs_stream_t stream);
int qs_linear_output(float *y1, int64_t ld_y1, int64_t shards, int64_t batch, int64_t m,
                     int transform, const float *su, const void *phase_u, const float *bias,
                     void *y, int y_dtype, qs_stream_t stream);

/* ---- codebook construction: stage-scale sweeps ----------------------------
 * build_codebook (quipsharp/checkpoint.py:60-77) rebuilds an RVQ codebook from
 * (bits, seed) by sweeping candidate scales (quipsharp/rvq.py:28-66):
 *   fit_stage_scale:          mse(s) = mean ||x - s Q(x / s)||^2
 *   fit_residual_stage_scale: the same on x - RVQ_prev(x)
 * over Gaussian samples x (samples x 8 float32, device).  Q is one codebook
 * (rvq == 0: kinds[0]) or an RVQ of `stages` codebooks with stage_scales
 * (rvq == 1, quipsharp/rvq.py:69-80); prev_stages (0..2) codebooks with
 * prev_scales are quantized away first.  candidates: host float32 array of
 * ncand (1..128) scales.  Writes mse (device double[ncand]) and best (device
 * int: the first candidate with the smallest mse).  Kinds and scales are host
 * arrays.  workspace: qs_fit_workspace_bytes(samples, ncand) bytes. */
int64_t qs_fit_workspace_bytes(int64_t samples, int ncand);
int qs_fit_scale_sweep(const float *x, int64_t samples, int prev_stages, const int *prev_kinds,
                       const float *prev_scales, int rvq, int stages, const int *kinds,
                       const float *stage_scales, const float *candidates, int ncand,
                       void *workspace, int64_t workspace_bytes, double *mse, int *best,
                       qs_stream_t stream);

/* ---- column-sharded tensor parallelism over peer memory -------------------
 * No counterpart in the reference (it places whole decoder layers on devices,
 * quipsharp/checkpoint.py:236-262); this is the scale-out of one layer over the
 * GPUs of a node.  Rank r of `world` holds weight rows [r m/world, (r+1)
 * m/world) (its own qs_pack_codes stream of those rows).  Every rank allocates
 * (zeroed) a float32 receive buffer of two regions of recv_floats each, an
 * int32 flag array [2][world] and four uint32 control words; it exports the
 * receive buffer and the flags with qs_ipc_export, exchanges the handles with
 * its peers (any host channel) and maps theirs with qs_ipc_import; qs_tp_peers
 * then lists every rank's buffers as mapped in this process.  Each call pushes
 * this rank's y1 shard into every rank's receive buffer (stores over NVLink)
 * and announces it through the flags; the region a call uses follows a call
 * counter kept in the control words on the device, so calls may be captured
 * in CUDA graphs and replayed in any mix with direct calls.  All ranks must
 * make the same sequence of calls on one peer set; calls are stream-ordered;
 * ranks synchronise only through the flags, whose waits are bounded
 * (qs_set_wait_limit_ns; a wait that runs out sets the qs_device_status flag
 * and the call's output is invalid). */
#define QS_TP_MAX_RANKS 8
typedef struct qs_tp_peers {
  int world;                            /* ranks, 1..QS_TP_MAX_RANKS */
  int rank;                             /* this process's rank */
  float *recv[QS_TP_MAX_RANKS];         /* every rank's receive buffer (float32 [2][recv_floats]) */
  int *flags[QS_TP_MAX_RANKS];          /* every rank's flags (int32 [2][world]) */
  unsigned *ctl;                        /* this rank's control words (uint32 [4], zeroed, 16-byte aligned) */
  int64_t recv_floats;                  /* floats per region (>= batch * m of every call, twice
                                           that for batches of at most 32 tokens, which travel
                                           as 8-byte words {value, call number}) */
} qs_tp_peers;

/* CUDA IPC of a device pointer (any pointer into a cudaMalloc allocation):
 * handle is 64 bytes (cudaIpcMemHandle_t), offset the pointer's offset in its
 * allocation.  qs_ipc_import maps a peer's allocation (peer access enabled
 * lazily) and returns the pointer at the same offset; qs_ipc_close unmaps it. */
int qs_ipc_export(const void *ptr, void *handle, int64_t *offset);
int qs_ipc_import(const void *handle, int64_t offset, void **ptr);
int qs_ipc_close(void *ptr, int64_t offset);

/* Workspace bytes of qs_linear_fwd_tp: the x2 workspace of qs_linear_input
 * and this rank's private y1 shard (batch, m_local) float32. */
int64_t qs_linear_tp_workspace_bytes(int64_t batch, int64_t n, int64_t m_local);

/* QuantizedLinear.forward of one column-sharded layer on this rank
 * (quipsharp/checkpoint.py:141-146 -> quipsharp/quantize.py:116-124, the rows
 * split over ranks): input step, fused decode + matmul of this rank's rows
 * (packed: this rank's row shard, m / world rows) into a private y1 shard,
 * push of the shard to every rank, output step over the gathered y1.  m, su,
 * phase_u, bias and y are the full layer's (every rank ends with the whole
 * output).  workspace: qs_linear_tp_workspace_bytes(batch, n, m / world)
 * bytes, 256-byte aligned. */
int qs_linear_fwd_tp(const void *x, int x_dtype, int64_t batch, int64_t n, int64_t m,
                     const void *packed, int stages, const int *kinds, const float *stage_scales,
                     const float *layer_scale, int transform, const float *su, const float *sv,
                     const void *phase_u, const void *phase_v, const float *bias, void *y,
                     void *workspace, int64_t workspace_bytes, const qs_tp_peers *peers,
                     qs_stream_t stream);
/* The last two steps alone, for callers that compute the shard themselves:
 * qs_tp_push copies this rank's y1 shard (batch, m_local) float32 into every
 * rank's receive buffer (after the work before it on the stream) and
 * announces it; qs_linear_output_peers waits for all ranks' shards of the
 * call and applies the output step to the gathered y1 (m = m_local * world). */
int qs_tp_push(const qs_tp_peers *peers, const float *y1, int64_t batch, int64_t m_local,
               qs_stream_t stream);
/* qs_linear_matmul followed by qs_tp_push of its y1 shard, fused for batches
 * of at most 32 tokens (after a grid barrier every CTA of the matmul pushes its
 * slice of the shard as self-validating words, saving a kernel); larger
 * batches run the two in sequence. */
int qs_linear_matmul_tp(const void *x2_workspace, int64_t batch, int64_t n, int64_t m_local,
                        const void *packed, int stages, const int *kinds, const float *stage_scales,
                        const float *layer_scale, float *y1, const qs_tp_peers *peers,
                        qs_stream_t stream);
int qs_linear_output_peers(const qs_tp_peers *peers, int64_t batch, int64_t m, int transform,
                           const float *su, const void *phase_u, const float *bias, void *y,
                           int y_dtype, qs_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* QUIPSHARP_B200_H */
