// Decode-batch FWHT row kernels for the linear input / output steps of RHT
// layers (quipsharp/incoherence.py:86-93: x2 = fwht(x * sv), y = fwht(y1) * su,
// the normalised Sylvester Hadamard transform of quipsharp/hadamard.py:17-40).
//
// A decode step transforms a handful of rows, so one row's latency is the
// cost.  One CTA per row of n = 2^(5 + LV + LW) points, 32 * 2^LW threads,
// each thread holding V = 2^LV points:
//   layout A: point i = lane + 32 * (r + V * w)  (r: register, w: warp);
//   1. butterflies over the register bits of i, in registers;
//   2. butterflies over the lane bits, by warp shuffles;
//   3. one shared-memory transpose: thread (w', lane) takes, for the V / W
//      register indices r = w' + W * j, all W points along the warp bits
//      (W = 2^LW <= V), and the butterflies over the warp bits run in registers.
// A butterfly maps (a, b) to (a + b, a - b) with a the point whose bit is 0;
// any bit order gives the same transform.  Loads and stores are coalesced
// (consecutive lanes, consecutive points); shared-memory accesses are
// conflict-free.  Layer constants (signs, bias) are loaded before the
// dependent-launch wait, so their latency hides behind the previous kernel.
#include "qs_common.cuh"
#include "qs_launch.h"
#include "qs_xform.cuh"

namespace qs {

namespace {

template <int N>
__device__ __forceinline__ void fwht_regs(float (&v)[N]) {
#pragma unroll
  for (int h = 1; h < N; h <<= 1)
#pragma unroll
    for (int j = 0; j < N; ++j)
      if (!(j & h)) {
        const float a = v[j], b = v[j + h];
        v[j] = a + b;
        v[j + h] = a - b;
      }
}

template <int V>
__device__ __forceinline__ void fwht_lanes(float (&v)[V], int lane) {
#pragma unroll
  for (int m = 1; m < 32; m <<= 1) {
    const float s = (lane & m) ? -1.f : 1.f;
#pragma unroll
    for (int r = 0; r < V; ++r) {
      const float p = __shfl_xor_sync(0xffffffffu, v[r], m);
      v[r] = fmaf(s, v[r], p);  // bit 0: v + p; bit 1: p - v
    }
  }
}

// Steps 1-3 on the values of layout A; on return v[j * W + k] holds point
// lane + 32 * ((w' + W * j) + V * k) of the transformed row.
template <int LV, int LW>
__device__ __forceinline__ void fwht_row_small(float (&v)[1 << LV], float *sm) {
  constexpr int V = 1 << LV, W = 1 << LW;
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  fwht_regs(v);
  fwht_lanes(v, lane);
#pragma unroll
  for (int r = 0; r < V; ++r) sm[lane + 32 * (r + V * w)] = v[r];
  __syncthreads();
#pragma unroll
  for (int j = 0; j < V / W; ++j) {
    float u[W];
#pragma unroll
    for (int k = 0; k < W; ++k) u[k] = sm[lane + 32 * ((w + W * j) + V * k)];
    fwht_regs(u);
#pragma unroll
    for (int k = 0; k < W; ++k) v[j * W + k] = u[k];
  }
}

// Point index of v[j * W + k] after fwht_row_small.
template <int LV, int LW>
__device__ __forceinline__ int point_b(int j, int k) {
  constexpr int V = 1 << LV, W = 1 << LW;
  return (threadIdx.x & 31) + 32 * (((threadIdx.x >> 5) + W * j) + V * k);
}

template <int LV>
__device__ __forceinline__ int point_a(int r) {
  constexpr int V = 1 << LV;
  return (threadIdx.x & 31) + 32 * (r + V * (threadIdx.x >> 5));
}

struct SmallIn {
  const void *x;
  int dtype;
  const float *sv;
  float scale;  // 1 / sqrt(n)
  __half *x2h;
  float *rowscale;
  int n_pad;
  float *y1;
  int64_t m_local;
};

template <int LV, int LW>
__global__ void __launch_bounds__(32 << LW) xsmall_input_rht_kernel(SmallIn a) {
  constexpr int V = 1 << LV, W = 1 << LW, n = 32 * V * W;
  extern __shared__ float sm_small[];
  __shared__ float red[W];
  pdl_launch_dependents();
  const int64_t row = blockIdx.x;
  float sg[V];
#pragma unroll
  for (int r = 0; r < V; ++r) sg[r] = __ldg(a.sv + point_a<LV>(r));  // layer constant
  pdl_wait();  // x may be the previous kernel's output; y1 may still be read by it
  if (a.y1) xzero_row(a.y1, row, a.m_local, 0, a.m_local);
  float v[V];
#pragma unroll
  for (int r = 0; r < V; ++r) v[r] = load_as_float(a.x, row * n + point_a<LV>(r), a.dtype) * sg[r];
  fwht_row_small<LV, LW>(v, sm_small);
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < V; ++i) {
    v[i] *= a.scale;
    amax = fmaxf(amax, fabsf(v[i]));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
  __syncthreads();
#pragma unroll
  for (int k = 0; k < W; ++k) amax = fmaxf(amax, red[k]);
  float sc, inv;
  xpow2_scale(amax, sc, inv);
  __half *out = a.x2h + row * a.n_pad;
#pragma unroll
  for (int j = 0; j < V / W; ++j)
#pragma unroll
    for (int k = 0; k < W; ++k) out[point_b<LV, LW>(j, k)] = __float2half_rn(v[j * W + k] * sc);
  if (threadIdx.x == 0) a.rowscale[row] = inv;
}

struct SmallOut {
  const float *y1;
  int64_t ld_y1;      // shards == 1: row stride of y1
  int64_t batch;
  int shard_log2;     // shards > 1: log2(m / shards) (rank-major gathered layout); else -1
  const float *su;
  const float *bias;
  float scale;        // 1 / sqrt(m)
  void *y;
  int dtype;
  int *busy;          // dry-pass hint flag of the library's input steps
  XPeerGather pg;     // flags != null: y1 is the pushed receive buffer
};

template <int LV, int LW>
__global__ void __launch_bounds__(32 << LW) xsmall_output_rht_kernel(SmallOut a) {
  constexpr int V = 1 << LV, W = 1 << LW, m = 32 * V * W;
  extern __shared__ float sm_small[];
  const int64_t row = blockIdx.x;
  const bool flag = row == 0 && threadIdx.x == 0;
  if (flag) xbusy_set(a.busy, 1);  // before the release: the next input step reads it at its start
  pdl_launch_dependents();
  float sg[V], bb[V];
#pragma unroll
  for (int j = 0; j < V / W; ++j)
#pragma unroll
    for (int k = 0; k < W; ++k) {
      const int i = point_b<LV, LW>(j, k);
      sg[j * W + k] = __ldg(a.su + i) * a.scale;  // layer constants
      bb[j * W + k] = a.bias ? __ldg(a.bias + i) : 0.f;
    }
  pdl_wait();  // y1 comes from the matmul (or the ranks' pushes)
  const float *src = a.pg.flags ? xwait_peers(a.pg) : a.y1;
  float v[V];
#pragma unroll
  for (int r = 0; r < V; ++r) {
    const int i = point_a<LV>(r);
    int64_t off;
    if (a.shard_log2 < 0) off = row * a.ld_y1 + i;
    else off = ((static_cast<int64_t>(i >> a.shard_log2) * a.batch + row) << a.shard_log2) + (i & ((1 << a.shard_log2) - 1));
    v[r] = src ? src[off] : 0.f;
  }
  fwht_row_small<LV, LW>(v, sm_small);
#pragma unroll
  for (int j = 0; j < V / W; ++j)
#pragma unroll
    for (int k = 0; k < W; ++k) {
      const int i = point_b<LV, LW>(j, k);
      store_from_float(a.y, row * m + i, a.dtype, fmaf(v[j * W + k], sg[j * W + k], bb[j * W + k]));
    }
  if (flag) xbusy_set(a.busy, 0);
}

// (LV, LW) per log2(n): W <= V, at most 512 threads.
template <template <int, int> class F, typename... Args>
int dispatch_small(int lg, Args &&...args) {
  switch (lg) {
    case 10: return F<3, 2>::run(args...);
    case 11: return F<3, 3>::run(args...);
    case 12: return F<4, 3>::run(args...);
    case 13: return F<4, 4>::run(args...);
    case 14: return F<5, 4>::run(args...);
    default: return fail(QS_ERR_UNSUPPORTED, "no decode-batch FWHT for 2^%d points", lg);
  }
}

template <int LV, int LW>
struct RunIn {
  static int run(const SmallIn &a, int64_t rows, cudaStream_t s) {
    constexpr int n = 32 << (LV + LW);
    auto k = xsmall_input_rht_kernel<LV, LW>;
    QS_CUDA_TRY(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, n * 4));
    return launch_pdl("xsmall_input_rht", k, dim3(static_cast<unsigned>(rows)), dim3(32 << LW), n * 4, s, a);
  }
};

template <int LV, int LW>
struct RunOut {
  static int run(const SmallOut &a, int64_t rows, cudaStream_t s) {
    constexpr int n = 32 << (LV + LW);
    auto k = xsmall_output_rht_kernel<LV, LW>;
    QS_CUDA_TRY(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, n * 4));
    return launch_pdl("xsmall_output_rht", k, dim3(static_cast<unsigned>(rows)), dim3(32 << LW), n * 4, s, a);
  }
};

int log2_exact(int64_t n) {
  int lg = 0;
  while ((int64_t(1) << lg) < n) ++lg;
  return (int64_t(1) << lg) == n ? lg : -1;
}

}  // namespace

bool small_rht_ok(int64_t n, int64_t rows) {
  const int lg = log2_exact(n);
  return lg >= 10 && lg <= 14 && rows >= 1 && rows <= kSmallRhtMaxRows;
}

int launch_small_input_rht(const void *x, int dtype, int64_t rows, int64_t n, const float *sv, float scale,
                           __half *x2h, float *rowscale, int n_pad, float *y1, int64_t m_local, cudaStream_t s) {
  SmallIn a{x, dtype, sv, scale, x2h, rowscale, n_pad, y1, m_local};
  return dispatch_small<RunIn>(log2_exact(n), a, rows, s);
}

int launch_small_output_rht(const float *y1, int64_t ld_y1, int64_t shards, int64_t batch, int64_t m,
                            const float *su, const float *bias, float scale, void *y, int y_dtype,
                            const XPeerGather *pg, cudaStream_t s) {
  SmallOut a{};
  a.y1 = y1;
  a.ld_y1 = ld_y1;
  a.batch = batch;
  a.shard_log2 = -1;
  if (shards > 1) {
    a.shard_log2 = log2_exact(m / shards);
    if (a.shard_log2 < 0) return fail(QS_ERR_UNSUPPORTED, "shard width is not a power of two");
  }
  a.su = su;
  a.bias = bias;
  a.scale = scale;
  a.y = y;
  a.dtype = y_dtype;
  a.busy = xbusy_flag();
  if (pg) a.pg = *pg;
  return dispatch_small<RunOut>(log2_exact(m), a, batch, s);
}

}  // namespace qs
