// qs_linear_fwd_noalloc: the quantized-linear forward for callers that must not
// allocate device memory.
//
// Who needs it: host programs that hand all device memory to their own
// allocator up front (inference servers that reserve most of HBM for their KV
// cache, or plugin hosts with a fixed per-plugin budget), where an extra
// cudaMalloc either fails or steps outside the budget; and latency-critical
// loops where cudaMalloc / cudaFree may synchronise the device.  Such a caller
// cannot provide the workspace qs_linear_fwd asks for, so this entry point
// brings its own: a file-scope __device__ array of kStaticWorkspaceBytes that
// every GPU which loads the library holds until the process exits.
//
// The array's name is only a host-side stand-in for the device symbol; the
// device address comes from cudaGetSymbolAddress, looked up once per device
// (with that device current) on the first call made on it.  Make that first
// call before any CUDA graph capture.  All calls share the one array and it
// keeps whatever the last call left: the forward zeroes the part that must
// start at zero (its float32 accumulator) itself, but calls that overlap on
// the GPU (different streams, or different host threads) would race on it.
#include <mutex>

#include "qs_common.cuh"

#define QS_API extern "C" __attribute__((visibility("default")))

namespace qs {

constexpr int64_t kStaticWorkspaceBytes = int64_t(8) << 20;  // 8 MiB
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_static_workspace[kStaticWorkspaceBytes];

static std::mutex g_static_ws_mutex;
static void *g_static_ws_addr[kMaxDevices] = {nullptr};

// Device address of g_static_workspace on the current device (looked up once).
static int static_workspace(void **out) {
  int dev = 0;
  QS_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return fail(QS_ERR_INVALID_ARG, "device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_static_ws_mutex);
  if (!g_static_ws_addr[dev]) {
    void *p = nullptr;
    QS_CUDA_TRY(cudaGetSymbolAddress(&p, g_static_workspace));
    g_static_ws_addr[dev] = p;
  }
  *out = g_static_ws_addr[dev];
  return QS_OK;
}

}  // namespace qs

using namespace qs;

QS_API int64_t qs_linear_workspace_bytes(int64_t batch, int64_t m, int64_t n);
QS_API int qs_linear_fwd(const void *x, int x_dtype, int64_t batch, int64_t n, int64_t m,
                         const void *packed, int stages, const int *kinds,
                         const float *stage_scales, const float *layer_scale, int transform,
                         const float *su, const float *sv, const void *phase_u,
                         const void *phase_v, const float *bias, void *y, void *workspace,
                         int64_t workspace_bytes, qs_stream_t stream);

QS_API int qs_linear_fwd_noalloc(const void *x, int x_dtype, int64_t batch, int64_t n, int64_t m,
                                 const void *packed, int stages, const int *kinds,
                                 const float *stage_scales, const float *layer_scale, int transform,
                                 const float *su, const float *sv, const void *phase_u,
                                 const void *phase_v, const float *bias, void *y,
                                 qs_stream_t stream) {
  const int64_t need = qs_linear_workspace_bytes(batch, m, n);
  if (need < 0) return fail(QS_ERR_INVALID_ARG, "bad shape (batch %lld, m %lld, n %lld)",
                            (long long)batch, (long long)m, (long long)n);
  if (need > kStaticWorkspaceBytes)
    return fail(QS_ERR_WORKSPACE,
                "batch %lld of a %lld x %lld layer needs %lld bytes of workspace; the built-in "
                "workspace of qs_linear_fwd_noalloc holds %lld bytes (use qs_linear_fwd with a "
                "caller-provided workspace, or split the batch)",
                (long long)batch, (long long)m, (long long)n, (long long)need,
                (long long)kStaticWorkspaceBytes);
  void *ws = nullptr;
  int st = static_workspace(&ws);
  if (st) return st;
  return qs_linear_fwd(x, x_dtype, batch, n, m, packed, stages, kinds, stage_scales, layer_scale,
                       transform, su, sv, phase_u, phase_v, bias, y, ws, kStaticWorkspaceBytes, stream);
}
