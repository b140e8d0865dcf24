// extern "C" entry points of libquipsharp_b200: argument validation, error
// reporting and dispatch to the launchers of the other translation units.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "qs_common.cuh"
#include "qs_launch.h"

#define QS_API extern "C" __attribute__((visibility("default")))

namespace qs {

static thread_local char g_last_error[512] = "";

void set_error(const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
}

int fail(int status, const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return status;
}

int check_launch(const char *what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(QS_ERR_CUDA, "%s launch failed: %s", what, cudaGetErrorString(e));
  return QS_OK;
}

static bool valid_kind(int k) { return k == QS_CB_E8P || k == QS_CB_E8_1BIT; }
static bool valid_io_dtype(int d) { return d == QS_F32 || d == QS_F16 || d == QS_BF16; }
static bool valid_code_dtype(int d) { return d == QS_I16 || d == QS_I32 || d == QS_I64; }

static int check_kinds(int stages, const int *kinds) {
  if (stages < 1 || stages > 2 || kinds == nullptr)
    return fail(QS_ERR_INVALID_ARG, "stages must be 1 or 2 (got %d) with a kinds array", stages);
  for (int i = 0; i < stages; ++i)
    if (!valid_kind(kinds[i])) return fail(QS_ERR_INVALID_ARG, "bad codebook kind %d", kinds[i]);
  return QS_OK;
}

static bool aligned(const void *p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

}  // namespace qs

using namespace qs;

QS_API const char *qs_version(void) { return "quipsharp_b200 0.1 (sm_100a)"; }

QS_API const char *qs_last_error(void) { return g_last_error; }

QS_API int qs_device_status(qs_stream_t stream) { return device_status((cudaStream_t)stream); }

QS_API int qs_set_wait_limit_ns(uint64_t ns) {
  set_pipeline_wait_ns(ns);
  return QS_OK;
}

QS_API uint64_t qs_wait_limit_ns(void) { return pipeline_wait_ns(); }

QS_API int qs_codebook_table(int kind, float *out_host) {
  if (!out_host) return fail(QS_ERR_INVALID_ARG, "null output");
  if (kind == QS_CB_E8P) memcpy(out_host, kE8pAbsF32Host, sizeof(kE8pAbsF32Host));
  else if (kind == QS_CB_E8_1BIT) memcpy(out_host, kE81BitF32Host, sizeof(kE81BitF32Host));
  else return fail(QS_ERR_INVALID_ARG, "bad codebook kind %d", kind);
  return QS_OK;
}

QS_API int qs_decode(int kind, const void *codes, int code_dtype, int64_t count, float *out,
                     qs_stream_t stream) {
  if (!valid_kind(kind)) return fail(QS_ERR_INVALID_ARG, "bad codebook kind %d", kind);
  if (!valid_code_dtype(code_dtype)) return fail(QS_ERR_INVALID_ARG, "bad code dtype %d", code_dtype);
  if (count < 0) return fail(QS_ERR_INVALID_ARG, "negative count");
  if (count == 0) return QS_OK;
  if (!codes || !out) return fail(QS_ERR_INVALID_ARG, "null pointer");
  return launch_decode(kind, codes, code_dtype, count, out, (cudaStream_t)stream);
}

QS_API int qs_rvq_decode(int stages, const int *kinds, const void *const *codes, int code_dtype,
                         const float *stage_scales, int64_t count, float *out,
                         qs_stream_t stream) {
  int st = check_kinds(stages, kinds);
  if (st) return st;
  if (!valid_code_dtype(code_dtype)) return fail(QS_ERR_INVALID_ARG, "bad code dtype %d", code_dtype);
  if (count < 0) return fail(QS_ERR_INVALID_ARG, "negative count");
  if (count == 0) return QS_OK;
  if (!codes || !out || !stage_scales) return fail(QS_ERR_INVALID_ARG, "null pointer");
  for (int i = 0; i < stages; ++i)
    if (!codes[i]) return fail(QS_ERR_INVALID_ARG, "null codes for stage %d", i);
  return launch_rvq_decode(stages, kinds, codes, code_dtype, stage_scales, count, out,
                           (cudaStream_t)stream);
}

QS_API int qs_dequantize_linear(const int16_t *codes, int stages, const int *kinds,
                                const float *stage_scales, const float *layer_scale, int64_t m,
                                int64_t n, float *out, qs_stream_t stream) {
  int st = check_kinds(stages, kinds);
  if (st) return st;
  if (m < 0 || n < 0 || n % 8) return fail(QS_ERR_INVALID_ARG, "bad shape (%lld, %lld)", (long long)m, (long long)n);
  if (m == 0 || n == 0) return QS_OK;
  if (!codes || !out || !layer_scale) return fail(QS_ERR_INVALID_ARG, "null pointer");
  return launch_dequantize_linear(codes, stages, kinds, stage_scales, layer_scale, m, n, out,
                                  (cudaStream_t)stream);
}

QS_API int qs_fwht(const void *x, int64_t ld_x, void *y, int64_t ld_y, int dtype, int64_t rows,
                   int64_t n, const float *pre, const float *post, qs_stream_t stream) {
  if (!valid_io_dtype(dtype)) return fail(QS_ERR_INVALID_ARG, "bad dtype %d", dtype);
  if (n <= 0 || (n & (n - 1)))
    return fail(QS_ERR_NOT_POW2, "fwht requires a power-of-two size along dim, got %lld", (long long)n);
  int st = check_fwht_size(n);
  if (st) return st;
  if (rows < 0 || ld_x < n || ld_y < n) return fail(QS_ERR_INVALID_ARG, "bad rows/strides");
  if (rows == 0) return QS_OK;
  if (!x || !y) return fail(QS_ERR_INVALID_ARG, "null pointer");
  return launch_fwht(x, ld_x, y, ld_y, dtype, rows, n, pre, post, (cudaStream_t)stream);
}

QS_API int qs_rfft(int inverse, const void *x, int64_t ld_x, void *y, int64_t ld_y, int dtype,
                   int64_t rows, int64_t n, const void *phase, qs_stream_t stream) {
  if (!valid_io_dtype(dtype)) return fail(QS_ERR_INVALID_ARG, "bad dtype %d", dtype);
  if (n <= 0 || (n % 2)) return fail(QS_ERR_ODD_DIM, "RFFT requires an even size, got %lld", (long long)n);
  int st = check_fft_size(n / 2);
  if (st) return st;
  if (rows < 0 || ld_x < n || ld_y < n) return fail(QS_ERR_INVALID_ARG, "bad rows/strides");
  if (rows == 0) return QS_OK;
  if (!x || !y || !phase) return fail(QS_ERR_INVALID_ARG, "null pointer");
  if (!aligned(phase, 8)) return fail(QS_ERR_ALIGNMENT, "phase must be 8-byte aligned");
  return launch_rfft(inverse, x, ld_x, y, ld_y, dtype, rows, n, phase, (cudaStream_t)stream);
}

QS_API int64_t qs_packed_bytes(int stages, const int *kinds, int64_t m, int64_t n) {
  if (check_kinds(stages, kinds) || m <= 0 || n <= 0 || n % 8) return -1;
  int64_t total = 0;
  for (int s = 0; s < stages; ++s) total += round_up(stage_bytes(kinds[s], m, n), 256);
  return total;
}

QS_API int qs_pack_codes(const int16_t *codes, int stages, const int *kinds, int64_t m, int64_t n,
                         void *packed, int64_t packed_bytes, qs_stream_t stream) {
  int st = check_kinds(stages, kinds);
  if (st) return st;
  if (m <= 0 || n <= 0 || n % 8) return fail(QS_ERR_INVALID_ARG, "bad shape (%lld, %lld)", (long long)m, (long long)n);
  if (!codes || !packed) return fail(QS_ERR_INVALID_ARG, "null pointer");
  if (packed_bytes < qs_packed_bytes(stages, kinds, m, n))
    return fail(QS_ERR_WORKSPACE, "packed buffer too small");
  if (!aligned(packed, 256)) return fail(QS_ERR_ALIGNMENT, "packed buffer must be 256-byte aligned");
  return launch_pack(codes, stages, kinds, m, n, packed, (cudaStream_t)stream);
}

static int64_t ws_align(int64_t b) { return round_up(b, 256); }

QS_API int64_t qs_linear_input_bytes(int64_t batch, int64_t n) {
  if (batch < 0 || n <= 0) return -1;
  return linear_input_bytes(batch, n);
}

QS_API int64_t qs_linear_workspace_bytes(int64_t batch, int64_t m, int64_t n) {
  if (batch < 0 || m <= 0 || n <= 0) return -1;
  return ws_align(linear_input_bytes(batch, n)) + ws_align(batch * m * (int64_t)sizeof(float));
}

static int check_transform_args(int transform, int64_t m, int64_t n, const float *su,
                                const float *sv, const void *phase_u, const void *phase_v) {
  if (transform == QS_RHT) {
    if (n <= 0 || (n & (n - 1)) || m <= 0 || (m & (m - 1)))
      return fail(QS_ERR_NOT_POW2, "RHT needs power-of-two dims, got (%lld, %lld)", (long long)m, (long long)n);
    int st = check_fwht_size(n);
    if (st) return st;
    if ((st = check_fwht_size(m))) return st;
    if (!su || !sv) return fail(QS_ERR_INVALID_ARG, "RHT needs su and sv");
  } else if (transform == QS_RFFT) {
    if (n % 2 || m % 2) return fail(QS_ERR_ODD_DIM, "RFFT needs even dims, got (%lld, %lld)", (long long)m, (long long)n);
    int st = check_fft_size(n / 2);
    if (st) return st;
    st = check_fft_size(m / 2);
    if (st) return st;
    if (!phase_u || !phase_v) return fail(QS_ERR_INVALID_ARG, "RFFT needs phase_u and phase_v");
  } else {
    return fail(QS_ERR_INVALID_ARG, "bad transform %d", transform);
  }
  return QS_OK;
}

QS_API int qs_linear_input(const void *x, int x_dtype, int64_t batch, int64_t n, int transform,
                           const float *sv, const void *phase_v, void *x2_workspace,
                           int64_t x2_workspace_bytes, float *y1, int64_t m_local,
                           qs_stream_t stream) {
  if (!valid_io_dtype(x_dtype)) return fail(QS_ERR_INVALID_ARG, "bad dtype %d", x_dtype);
  int st = check_transform_args(transform, transform == QS_RHT ? 1 : 2, n, sv, sv, phase_v, phase_v);
  if (st) return st;
  if (batch < 0 || m_local < 0) return fail(QS_ERR_INVALID_ARG, "bad batch / m_local");
  if (batch == 0) return QS_OK;
  if (!x || !x2_workspace) return fail(QS_ERR_INVALID_ARG, "null pointer");
  if (x2_workspace_bytes < linear_input_bytes(batch, n)) return fail(QS_ERR_WORKSPACE, "x2 workspace too small");
  if (!aligned(x2_workspace, 256)) return fail(QS_ERR_ALIGNMENT, "workspace must be 256-byte aligned");
  return launch_linear_input(x, x_dtype, batch, n, transform, sv, phase_v, x2_workspace, y1,
                             m_local, (cudaStream_t)stream);
}

QS_API int qs_linear_matmul(const void *x2_workspace, int64_t batch, int64_t n, int64_t m_local,
                            const void *packed, int stages, const int *kinds,
                            const float *stage_scales, const float *layer_scale, float *y1,
                            qs_stream_t stream) {
  int st = check_kinds(stages, kinds);
  if (st) return st;
  if (batch < 0 || n <= 0 || n % 8 || m_local <= 0) return fail(QS_ERR_INVALID_ARG, "bad shape");
  if (batch == 0) return QS_OK;
  if (!x2_workspace || !packed || !layer_scale || !y1) return fail(QS_ERR_INVALID_ARG, "null pointer");
  if (stages == 2 && !stage_scales) return fail(QS_ERR_INVALID_ARG, "RVQ needs stage scales");
  if (!aligned(packed, 256)) return fail(QS_ERR_ALIGNMENT, "packed buffer must be 256-byte aligned");
  return launch_matmul(x2_workspace, batch, n, m_local, packed, stages, kinds, stage_scales,
                       layer_scale, y1, (cudaStream_t)stream);
}

QS_API int qs_linear_matmul_tp(const void *x2_workspace, int64_t batch, int64_t n, int64_t m_local,
                               const void *packed, int stages, const int *kinds, const float *stage_scales,
                               const float *layer_scale, float *y1, const qs_tp_peers *peers, qs_stream_t stream) {
  int st = check_kinds(stages, kinds);
  if (st) return st;
  if (batch < 0 || n <= 0 || n % 8 || m_local <= 0) return fail(QS_ERR_INVALID_ARG, "bad shape");
  if (batch == 0) return launch_tp_push(peers, y1, 0, m_local, (cudaStream_t)stream);  // the call still counts
  if (!x2_workspace || !packed || !layer_scale || !y1) return fail(QS_ERR_INVALID_ARG, "null pointer");
  if (stages == 2 && !stage_scales) return fail(QS_ERR_INVALID_ARG, "RVQ needs stage scales");
  if (!aligned(packed, 256)) return fail(QS_ERR_ALIGNMENT, "packed buffer must be 256-byte aligned");
  return launch_matmul_tp(x2_workspace, batch, n, m_local, packed, stages, kinds, stage_scales, layer_scale, y1,
                          peers, (cudaStream_t)stream);
}

QS_API int qs_linear_output(float *y1, int64_t ld_y1, int64_t shards, int64_t batch,
                            int64_t m, int transform, const float *su, const void *phase_u,
                            const float *bias, void *y, int y_dtype, qs_stream_t stream) {
  if (!valid_io_dtype(y_dtype)) return fail(QS_ERR_INVALID_ARG, "bad dtype %d", y_dtype);
  int st = check_transform_args(transform, m, transform == QS_RHT ? 1 : 2, su, su, phase_u, phase_u);
  if (st) return st;
  if (shards < 1 || m % shards) return fail(QS_ERR_INVALID_ARG, "m=%lld not divisible by %lld shards", (long long)m, (long long)shards);
  if (shards > 1 && transform == QS_RFFT && (m / shards) % 2)
    return fail(QS_ERR_INVALID_ARG, "RFFT shards must hold an even number of columns");
  if (batch < 0 || (shards == 1 && ld_y1 < m)) return fail(QS_ERR_INVALID_ARG, "bad batch / ld_y1");
  if (batch == 0) return QS_OK;
  if (!y1 || !y) return fail(QS_ERR_INVALID_ARG, "null pointer");
  return launch_linear_output(y1, shards == 1 ? ld_y1 : m, shards, batch, m, transform, su, phase_u,
                              bias, y, y_dtype, (cudaStream_t)stream);
}

QS_API int64_t qs_fit_workspace_bytes(int64_t samples, int ncand) {
  if (samples < 1 || ncand < 1 || ncand > kFitMaxCandidates) return -1;
  return fit_workspace_bytes(samples, ncand);
}

QS_API int qs_fit_scale_sweep(const float *x, int64_t samples, int prev_stages, const int *prev_kinds,
                              const float *prev_scales, int rvq, int stages, const int *kinds,
                              const float *stage_scales, const float *candidates, int ncand, void *workspace,
                              int64_t workspace_bytes, double *mse, int *best, qs_stream_t stream) {
  if (!x || !candidates || !mse || !best || !workspace || !kinds) return fail(QS_ERR_INVALID_ARG, "null pointer");
  if (samples < 1 || samples > (int64_t(1) << 31) / 8) return fail(QS_ERR_INVALID_ARG, "bad sample count");
  if (ncand < 1 || ncand > kFitMaxCandidates) return fail(QS_ERR_INVALID_ARG, "1..%d candidates", kFitMaxCandidates);
  if (prev_stages < 0 || prev_stages > kFitMaxStages || (prev_stages && (!prev_kinds || !prev_scales)))
    return fail(QS_ERR_INVALID_ARG, "bad previous stages");
  if (rvq != 0 && rvq != 1) return fail(QS_ERR_INVALID_ARG, "rvq must be 0 or 1");
  if (stages < 1 || stages > (rvq ? kFitMaxStages : 1) || (rvq && !stage_scales))
    return fail(QS_ERR_INVALID_ARG, "bad swept stages");
  int st = check_kinds(stages, kinds);
  if (st) return st;
  if (prev_stages && (st = check_kinds(prev_stages, prev_kinds))) return st;
  for (int i = 0; i < prev_stages; ++i)
    if (!(prev_scales[i] != 0.f)) return fail(QS_ERR_INVALID_ARG, "zero previous-stage scale");
  for (int c = 0; c < ncand; ++c)
    if (!(candidates[c] != 0.f)) return fail(QS_ERR_INVALID_ARG, "zero candidate scale");
  if (workspace_bytes < fit_workspace_bytes(samples, ncand)) return fail(QS_ERR_WORKSPACE, "workspace too small");
  if (!aligned(workspace, 8)) return fail(QS_ERR_ALIGNMENT, "workspace must be 8-byte aligned");
  return launch_fit_sweep(x, samples, prev_stages, prev_kinds, prev_scales, rvq, stages, kinds, stage_scales,
                          candidates, ncand, workspace, mse, best, (cudaStream_t)stream);
}

QS_API int qs_ipc_export(const void *ptr, void *handle, int64_t *offset) {
  if (!ptr || !handle || !offset) return fail(QS_ERR_INVALID_ARG, "null pointer");
  return ipc_export(ptr, handle, offset);
}

QS_API int qs_ipc_import(const void *handle, int64_t offset, void **ptr) {
  if (!handle || !ptr || offset < 0) return fail(QS_ERR_INVALID_ARG, "bad argument");
  return ipc_import(handle, offset, ptr);
}

QS_API int qs_ipc_close(void *ptr, int64_t offset) {
  if (!ptr || offset < 0) return fail(QS_ERR_INVALID_ARG, "bad argument");
  return ipc_close(ptr, offset);
}

QS_API int64_t qs_linear_tp_workspace_bytes(int64_t batch, int64_t n, int64_t m_local) {
  if (batch < 0 || n <= 0 || m_local <= 0) return -1;
  return tp_workspace_bytes(batch, n, m_local);
}

QS_API int qs_tp_push(const qs_tp_peers *peers, const float *y1, int64_t batch, int64_t m_local,
                      qs_stream_t stream) {
  if (batch < 0 || m_local <= 0) return fail(QS_ERR_INVALID_ARG, "bad shape");
  if (batch > 0 && !y1) return fail(QS_ERR_INVALID_ARG, "null pointer");
  return launch_tp_push(peers, y1, batch, m_local, (cudaStream_t)stream);
}

QS_API int qs_linear_output_peers(const qs_tp_peers *peers, int64_t batch, int64_t m, int transform,
                                  const float *su, const void *phase_u, const float *bias, void *y, int y_dtype,
                                  qs_stream_t stream) {
  if (!valid_io_dtype(y_dtype)) return fail(QS_ERR_INVALID_ARG, "bad dtype %d", y_dtype);
  int st = check_transform_args(transform, m, transform == QS_RHT ? 1 : 2, su, su, phase_u, phase_u);
  if (st) return st;
  if (batch < 0) return fail(QS_ERR_INVALID_ARG, "bad batch");
  if (batch == 0) return QS_OK;  // nothing to read (the matching push still counted the call)
  if (!y) return fail(QS_ERR_INVALID_ARG, "null pointer");
  return launch_output_peers(peers, batch, m, transform, su, phase_u, bias, y, y_dtype, (cudaStream_t)stream);
}

QS_API int qs_linear_fwd_tp(const void *x, int x_dtype, int64_t batch, int64_t n, int64_t m, const void *packed,
                            int stages, const int *kinds, const float *stage_scales, const float *layer_scale,
                            int transform, const float *su, const float *sv, const void *phase_u,
                            const void *phase_v, const float *bias, void *y, void *workspace,
                            int64_t workspace_bytes, const qs_tp_peers *peers, qs_stream_t stream) {
  int st = check_kinds(stages, kinds);
  if (st) return st;
  if (!valid_io_dtype(x_dtype)) return fail(QS_ERR_INVALID_ARG, "bad dtype %d", x_dtype);
  if (!peers || peers->world < 1 || peers->world > QS_TP_MAX_RANKS || peers->rank < 0 || peers->rank >= peers->world)
    return fail(QS_ERR_INVALID_ARG, "bad peers");
  if (batch < 0 || n <= 0 || m <= 0 || n % 8 || m % peers->world) return fail(QS_ERR_INVALID_ARG, "bad shape");
  st = check_transform_args(transform, m, n, su, sv, phase_u, phase_v);
  if (st) return st;
  if (transform == QS_RFFT && (m / peers->world) % 2)
    return fail(QS_ERR_INVALID_ARG, "RFFT shards must hold an even number of columns");
  if (batch == 0) return QS_OK;  // every rank skips the call: no push, no wait
  if (!x || !y || !packed || !layer_scale || !workspace) return fail(QS_ERR_INVALID_ARG, "null pointer");
  if (stages == 2 && !stage_scales) return fail(QS_ERR_INVALID_ARG, "RVQ needs stage scales");
  if (workspace_bytes < tp_workspace_bytes(batch, n, m / peers->world))
    return fail(QS_ERR_WORKSPACE, "workspace too small");
  if (!aligned(workspace, 256) || !aligned(packed, 256))
    return fail(QS_ERR_ALIGNMENT, "workspace/packed must be 256-byte aligned");
  if (batch * m * (batch < kTcMinBatch ? 2 : 1) > peers->recv_floats)
    return fail(QS_ERR_WORKSPACE, "receive buffers too small");
  return launch_linear_fwd_tp(x, x_dtype, batch, n, m, packed, stages, kinds, stage_scales, layer_scale, transform,
                              su, sv, phase_u, phase_v, bias, y, workspace, peers, (cudaStream_t)stream);
}

// Checks of one layer of qs_linear_fwd / qs_linear_fwd_group (nothing launched).
static int check_linear(const void *x, int x_dtype, int64_t batch, int64_t n, const qs_linear_layer &L) {
  int st = check_kinds(L.stages, L.kinds);
  if (st) return st;
  if (!valid_io_dtype(x_dtype)) return fail(QS_ERR_INVALID_ARG, "bad dtype %d", x_dtype);
  if (batch < 0 || n <= 0 || L.m <= 0 || n % 8) return fail(QS_ERR_INVALID_ARG, "bad shape");
  st = check_transform_args(L.transform, L.m, n, L.su, L.sv, L.phase_u, L.phase_v);
  if (st) return st;
  if (batch == 0) return QS_OK;
  if (!x || !L.y || !L.packed || !L.layer_scale || !L.workspace) return fail(QS_ERR_INVALID_ARG, "null pointer");
  if (L.stages == 2 && !L.stage_scales) return fail(QS_ERR_INVALID_ARG, "RVQ needs stage scales");
  if (L.workspace_bytes < qs_linear_workspace_bytes(batch, L.m, n)) return fail(QS_ERR_WORKSPACE, "workspace too small");
  if (!aligned(L.workspace, 256) || !aligned(L.packed, 256))
    return fail(QS_ERR_ALIGNMENT, "workspace/packed must be 256-byte aligned");
  return QS_OK;
}

// Step `step` (0 input, 1 matmul, 2 output) of one checked layer on stream s.
static int launch_linear_step(int step, const void *x, int x_dtype, int64_t batch, int64_t n,
                              const qs_linear_layer &L, cudaStream_t s) {
  const int64_t x2b = ws_align(linear_input_bytes(batch, n));
  float *y1 = reinterpret_cast<float *>(static_cast<char *>(L.workspace) + x2b);
  // the prefill matmul writes every y1 element; only the decode-regime kernel accumulates
  const bool tc = batch >= kTcMinBatch;
  if (step == 0)
    return launch_linear_input(x, x_dtype, batch, n, L.transform, L.sv, L.phase_v, L.workspace, tc ? nullptr : y1,
                               L.m, s);
  if (step == 1)
    return launch_matmul(L.workspace, batch, n, L.m, L.packed, L.stages, L.kinds, L.stage_scales, L.layer_scale,
                         y1, s);
  return launch_linear_output(y1, L.m, 1, batch, L.m, L.transform, L.su, L.phase_u, L.bias, L.y, x_dtype, s);
}

QS_API int qs_linear_fwd(const void *x, int x_dtype, int64_t batch, int64_t n, int64_t m,
                         const void *packed, int stages, const int *kinds,
                         const float *stage_scales, const float *layer_scale, int transform,
                         const float *su, const float *sv, const void *phase_u,
                         const void *phase_v, const float *bias, void *y, void *workspace,
                         int64_t workspace_bytes, qs_stream_t stream) {
  const qs_linear_layer L{m, packed, stages, kinds, stage_scales, layer_scale, transform, su, sv, phase_u, phase_v,
                          bias, y, workspace, workspace_bytes};
  int st = check_linear(x, x_dtype, batch, n, L);
  if (st || batch == 0) return st;
  for (int step = 0; step < 3; ++step)
    if ((st = launch_linear_step(step, x, x_dtype, batch, n, L, (cudaStream_t)stream))) return st;
  return QS_OK;
}

// Side streams and events of qs_linear_fwd_group, per device, made on first use
// and kept until exit (guarded by g_group_mutex, which also serialises the
// calls: the events are reused by every call).
namespace {
struct GroupStreams {
  bool have_fork = false;
  int made = 0;  // side streams (with their join events) created so far
  cudaStream_t side[QS_GROUP_MAX_LAYERS - 1];
  cudaEvent_t fork;
  cudaEvent_t join[QS_GROUP_MAX_LAYERS - 1];
};
constexpr int kGroupDevices = 64;
std::mutex g_group_mutex;
GroupStreams g_group[kGroupDevices];

int group_streams(GroupStreams **out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kGroupDevices)
    return fail(QS_ERR_CUDA, "no usable current device for the group's side streams");
  GroupStreams &g = g_group[dev];
  if (!g.have_fork) {
    if (cudaEventCreateWithFlags(&g.fork, cudaEventDisableTiming) != cudaSuccess)
      return fail(QS_ERR_CUDA, "cannot create the group's fork event");
    g.have_fork = true;
  }
  // a failed creation is retried by the next call from where it stopped
  for (; g.made < QS_GROUP_MAX_LAYERS - 1; ++g.made) {
    if (cudaStreamCreateWithFlags(&g.side[g.made], cudaStreamNonBlocking) != cudaSuccess)
      return fail(QS_ERR_CUDA, "cannot create the group's side streams");
    if (cudaEventCreateWithFlags(&g.join[g.made], cudaEventDisableTiming) != cudaSuccess) {
      cudaStreamDestroy(g.side[g.made]);
      return fail(QS_ERR_CUDA, "cannot create the group's join events");
    }
  }
  *out = &g;
  return QS_OK;
}

bool overlaps(const void *a, int64_t na, const void *b, int64_t nb) {
  const uintptr_t pa = reinterpret_cast<uintptr_t>(a), pb = reinterpret_cast<uintptr_t>(b);
  return pa < pb + static_cast<uintptr_t>(nb) && pb < pa + static_cast<uintptr_t>(na);
}
}  // namespace

QS_API int qs_linear_fwd_group(const void *x, int x_dtype, int64_t batch, int64_t n, int count,
                               const qs_linear_layer *layers, qs_stream_t stream) {
  if (count < 1 || count > QS_GROUP_MAX_LAYERS || !layers)
    return fail(QS_ERR_INVALID_ARG, "a group has 1 to %d layers (got %d) and a layers array", QS_GROUP_MAX_LAYERS,
                count);
  for (int i = 0; i < count; ++i) {
    const int st = check_linear(x, x_dtype, batch, n, layers[i]);
    if (st) return st;
  }
  if (batch == 0) return QS_OK;
  const int64_t esz = x_dtype == QS_F32 ? 4 : 2;
  for (int i = 0; i < count; ++i)
    for (int j = i + 1; j < count; ++j) {
      const qs_linear_layer &a = layers[i], &b = layers[j];
      const int64_t wa = qs_linear_workspace_bytes(batch, a.m, n), wb = qs_linear_workspace_bytes(batch, b.m, n);
      const int64_t ya = batch * a.m * esz, yb = batch * b.m * esz;
      if (overlaps(a.workspace, wa, b.workspace, wb) || overlaps(a.y, ya, b.y, yb) ||
          overlaps(a.workspace, wa, b.y, yb) || overlaps(a.y, ya, b.workspace, wb))
        return fail(QS_ERR_INVALID_ARG, "layers %d and %d of the group share workspace or output memory", i, j);
    }
  cudaStream_t s = (cudaStream_t)stream;
  // Prefill batches: every kernel of a layer fills the GPU (and the tensor-core
  // GEMM holds all of an SM's tensor memory), so the layers follow one another.
  if (count == 1 || batch >= kTcMinBatch) {
    for (int i = 0; i < count; ++i)
      for (int step = 0; step < 3; ++step) {
        const int st = launch_linear_step(step, x, x_dtype, batch, n, layers[i], s);
        if (st) return st;
      }
    return QS_OK;
  }
  std::lock_guard<std::mutex> lock(g_group_mutex);
  GroupStreams *g = nullptr;
  int st = group_streams(&g);
  if (st) return st;
  if (cudaEventRecord(g->fork, s) != cudaSuccess) return fail(QS_ERR_CUDA, "group fork: event record failed");
  int forked = 1;  // layers with a stream: 0 on s, i on side[i - 1]
  for (; forked < count; ++forked)
    if (cudaStreamWaitEvent(g->side[forked - 1], g->fork, 0) != cudaSuccess) {
      st = fail(QS_ERR_CUDA, "group fork: stream wait failed");
      break;
    }
  // step by step across the layers, so every layer's first kernel is queued early
  for (int step = 0; step < 3 && !st; ++step)
    for (int i = 0; i < forked && !st; ++i)
      st = launch_linear_step(step, x, x_dtype, batch, n, layers[i], i ? g->side[i - 1] : s);
  // join every forked stream whatever happened: a capture must end with all of them joined
  for (int i = 1; i < forked; ++i)
    if ((cudaEventRecord(g->join[i - 1], g->side[i - 1]) != cudaSuccess ||
         cudaStreamWaitEvent(s, g->join[i - 1], 0) != cudaSuccess) && !st)
      st = fail(QS_ERR_CUDA, "group join failed");
  return st;
}
