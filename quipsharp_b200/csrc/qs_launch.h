// Internal launchers shared between the translation units of the library.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/quipsharp_b200.h"

struct CUtensorMap_st;  // CUtensorMap (cuda.h)

namespace qs {

// qs_decode.cu
int launch_decode(int kind, const void *codes, int code_dtype, int64_t count, float *out,
                  cudaStream_t s);
int launch_rvq_decode(int stages, const int *kinds, const void *const *codes, int code_dtype,
                      const float *stage_scales, int64_t count, float *out, cudaStream_t s);
int launch_dequantize_linear(const int16_t *codes, int stages, const int *kinds,
                             const float *stage_scales, const float *layer_scale, int64_t m,
                             int64_t n, float *out, cudaStream_t s);

// qs_transform.cu
int launch_fwht(const void *x, int64_t ld_x, void *y, int64_t ld_y, int dtype, int64_t rows,
                int64_t n, const float *pre, const float *post, cudaStream_t s);
int launch_rfft(int inverse, const void *x, int64_t ld_x, void *y, int64_t ld_y, int dtype,
                int64_t rows, int64_t n, const void *phase, cudaStream_t s);
int64_t linear_input_bytes(int64_t batch, int64_t n);
int launch_linear_input(const void *x, int x_dtype, int64_t batch, int64_t n, int transform,
                        const float *sv, const void *phase_v, void *x2ws, float *y1,
                        int64_t m_local, cudaStream_t s);
struct XPeerGather;
struct TpPush;
int launch_linear_output(float *y1, int64_t ld_y1, int64_t shards, int64_t batch, int64_t m,
                         int transform, const float *su, const void *phase_u, const float *bias,
                         void *y, int y_dtype, cudaStream_t s, const XPeerGather *pg = nullptr);
int check_fft_size(int64_t n_complex);
int check_fwht_size(int64_t n);

// qs_xform2.cu: two-pass RFFT of the linear input / output steps
bool two_pass_rfft(int64_t n_complex, int64_t rows, int *P, int *lgN1);
int64_t two_pass_input_scratch_bytes(int64_t batch, int64_t n);
int launch_two_pass_input(const void *x, int dtype, int64_t batch, int64_t n, const float2 *phase, float scale,
                          __half *x2h, float *rowscale, int n_pad, void *scratch, float *y1, int64_t m_local,
                          cudaStream_t s);
int launch_two_pass_output(float *y1, int64_t batch, int64_t m, const float2 *phase, const float *bias, float scale,
                           void *y, int dtype, cudaStream_t s);

// qs_xsmall.cu: decode-batch FWHT row kernels of the linear input / output steps
constexpr int64_t kSmallRhtMaxRows = 32;
bool small_rht_ok(int64_t n, int64_t rows);
int launch_small_input_rht(const void *x, int dtype, int64_t rows, int64_t n, const float *sv, float scale,
                           __half *x2h, float *rowscale, int n_pad, float *y1, int64_t m_local, cudaStream_t s);
int launch_small_output_rht(const float *y1, int64_t ld_y1, int64_t shards, int64_t batch, int64_t m,
                            const float *su, const float *bias, float scale, void *y, int y_dtype,
                            const XPeerGather *pg, cudaStream_t s);
bool small_rfft_ok(int64_t n_complex, int64_t rows);
int launch_small_input_rfft(const void *x, int dtype, int64_t rows, int64_t n, const float2 *phase, float scale,
                            __half *x2h, float *rowscale, int n_pad, float *y1, int64_t m_local, cudaStream_t s);
int launch_small_output_rfft(const float *y1, int64_t ld_y1, int64_t shards, int64_t batch, int64_t m,
                             const float2 *phase, const float *bias, float scale, void *y, int y_dtype,
                             const XPeerGather *pg, cudaStream_t s);

// qs_fit.cu: stage-scale sweeps of RVQ codebook construction
constexpr int kFitMaxStages = 2;
constexpr int kFitMaxCandidates = 128;
int64_t fit_workspace_bytes(int64_t samples, int ncand);
int launch_fit_sweep(const float *x, int64_t samples, int nprev, const int *prev_kinds, const float *prev_scales,
                     int rvq, int nst, const int *kinds, const float *stage_scales, const float *candidates,
                     int ncand, void *workspace, double *mse, int *best, cudaStream_t s);

// qs_tp.cu: column-sharded tensor parallelism over peer memory
int ipc_export(const void *ptr, void *handle, int64_t *offset);
int ipc_import(const void *handle, int64_t offset, void **ptr);
int ipc_close(void *ptr, int64_t offset);
int64_t tp_workspace_bytes(int64_t batch, int64_t n, int64_t m_local);
int launch_tp_push(const qs_tp_peers *pe, const float *y1, int64_t batch, int64_t m_local, cudaStream_t s);
int launch_matmul_tp(const void *x2ws, int64_t batch, int64_t n, int64_t m_local, const void *packed, int stages,
                     const int *kinds, const float *stage_scales, const float *layer_scale, float *y1,
                     const qs_tp_peers *pe, cudaStream_t s);
int launch_output_peers(const qs_tp_peers *pe, int64_t batch, int64_t m, int transform, const float *su,
                        const void *phase_u, const float *bias, void *y, int y_dtype, cudaStream_t s);
int launch_linear_fwd_tp(const void *x, int x_dtype, int64_t batch, int64_t n, int64_t m, const void *packed,
                         int stages, const int *kinds, const float *stage_scales, const float *layer_scale,
                         int transform, const float *su, const float *sv, const void *phase_u, const void *phase_v,
                         const float *bias, void *y, void *workspace, const qs_tp_peers *pe, cudaStream_t s);

// qs_pack.cu
int launch_pack(const int16_t *codes, int stages, const int *kinds, int64_t m, int64_t n,
                void *packed, cudaStream_t s);

// qs_gemv.cu: fused decode + matmul; batches below kTcMinBatch run the
// decode-regime kernel of this file, larger ones launch_matmul_tc.  push
// (decode batches only): after a grid barrier the CTAs push y1 to every rank.
int launch_matmul(const void *x2ws, int64_t batch, int64_t n, int64_t m, const void *packed,
                  int stages, const int *kinds, const float *stage_scales,
                  const float *layer_scale, float *y1, cudaStream_t s, const TpPush *push = nullptr);

// qs_gemm_tc.cu
int launch_matmul_tc(const void *x2ws, int64_t batch, int64_t n, int64_t m, const void *packed, int stages,
                     const int *kinds, const float *stage_scales, const float *layer_scale, float *y1,
                     cudaStream_t s);
int device_status(cudaStream_t s);
// Device address (current device) of the error flag qs_device_status reports.
int *device_error_flag();
// 2-D tensor map over fp16 rows (rows x n_pad, row stride n_pad elements) with
// a box of box_x elements x box_y rows; 128-byte swizzle or none.
int encode_fp16_rows_map(::CUtensorMap_st *map, const void *x2h, int64_t n_pad, int64_t rows, int box_x, int box_y,
                         bool swizzle128);
// Limit (ns) of every bounded wait between the warps of a pipelined kernel
// (mbarrier waits); a wait that runs out sets the device error flag.  Drains of
// a CTA's own asynchronous copies and tensor-core work keep a fixed 4 s limit.
constexpr uint64_t kDefaultWaitNs = 4000000000ull;
uint64_t pipeline_wait_ns();
void set_pipeline_wait_ns(uint64_t ns);
// Batches of at least this many tokens use the tcgen05 GEMM (128 x 256 tiles,
// decoded weights in shared memory); smaller ones the mma.sync decode-regime
// kernel (weights decoded in registers, passes of 8 or 16 tokens).
constexpr int64_t kTcMinBatch = 33;

}  // namespace qs
