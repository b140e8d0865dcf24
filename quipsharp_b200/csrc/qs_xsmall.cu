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

// Zeroing of the y1 row the matmul accumulates into.  Plain stores from the
// row's CTA competed with its loads (a 28672-float row cost more than the
// transform); instead one thread hands the row to the bulk-copy engine as
// asynchronous copies of a zeroed shared-memory block (no multicast; 16-byte
// aligned, sizes in multiples of 16 bytes) and waits for them at the end.
constexpr int kZeroBlockBytes = 4096;

struct BulkZero {
  bool pending = false;

  // Call with all threads after the dependent-launch wait; zblk: kZeroBlockBytes of
  // shared memory this CTA does not otherwise use.
  __device__ __forceinline__ void start(float *row, int64_t floats, float4 *zblk) {
    const bool bulk = (reinterpret_cast<uintptr_t>(row) & 15) == 0 && (floats & 3) == 0;
    if (!bulk) {
      for (int64_t i = threadIdx.x; i < floats; i += blockDim.x) row[i] = 0.f;
      return;
    }
    for (int i = threadIdx.x; i < kZeroBlockBytes / 16; i += blockDim.x) zblk[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // the zeros, to the bulk-copy engine
    __syncthreads();
    if (threadIdx.x == 0) {
      const uint32_t src = static_cast<uint32_t>(__cvta_generic_to_shared(zblk));
      char *dst = reinterpret_cast<char *>(row);
      for (int64_t off = 0, bytes = floats * 4; off < bytes; off += kZeroBlockBytes) {
        const uint32_t n = static_cast<uint32_t>(bytes - off < kZeroBlockBytes ? bytes - off : kZeroBlockBytes);
        asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst + off), "r"(src), "r"(n)
                     : "memory");
      }
      asm volatile("cp.async.bulk.commit_group;" ::: "memory");
      pending = true;
    }
  }
  __device__ __forceinline__ void finish() {
    if (pending) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
  }
};

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
  int64_t rows;
};

template <int LV, int LW>
__global__ void __launch_bounds__(32 << LW) xsmall_input_rht_kernel(SmallIn a) {
  constexpr int V = 1 << LV, W = 1 << LW, n = 32 * V * W;
  extern __shared__ float sm_small[];
  __shared__ float red[W];
  __shared__ float4 zblk[kZeroBlockBytes / 16];
  pdl_launch_dependents();
  const int64_t row = blockIdx.x;
  float sg[V];
#pragma unroll
  for (int r = 0; r < V; ++r) sg[r] = __ldg(a.sv + point_a<LV>(r));  // layer constant
  pdl_wait();  // x may be the previous kernel's output; y1 may still be read by it
  float v[V];
#pragma unroll
  for (int r = 0; r < V; ++r) v[r] = load_as_float(a.x, row * n + point_a<LV>(r), a.dtype) * sg[r];
  BulkZero bz;
  if (a.y1) bz.start(a.y1 + row * a.m_local, a.m_local, zblk);
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
  bz.finish();
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
__global__ void __maxnreg__(128) xsmall_output_rht_kernel(SmallOut a) {  // 512 threads at most
  constexpr int V = 1 << LV, W = 1 << LW, m = 32 * V * W;
  extern __shared__ float sm_small[];
  const int64_t row = blockIdx.x;
  const bool flag = row == 0 && threadIdx.x == 0;
  if (flag) xbusy_set(a.busy, 1);  // before the release: the next input step reads it at its start
  pdl_launch_dependents();
  constexpr bool kBiasEarly = V <= 16;  // registers: 32 points per thread leave no room for the bias
  float sg[V], bb[kBiasEarly ? V : 1];
#pragma unroll
  for (int j = 0; j < V / W; ++j)
#pragma unroll
    for (int k = 0; k < W; ++k) {
      const int i = point_b<LV, LW>(j, k);
      sg[j * W + k] = __ldg(a.su + i) * a.scale;  // layer constants
      if constexpr (kBiasEarly) bb[j * W + k] = a.bias ? __ldg(a.bias + i) : 0.f;
    }
  pdl_wait();  // y1 comes from the matmul (or the ranks' pushes)
  const XPeerSrc src = a.pg.flags ? xwait_peers(a.pg) : xplain_src(a.y1);
  auto off = [&](int r) -> int64_t {
    const int i = point_a<LV>(r);
    if (a.shard_log2 < 0) return row * a.ld_y1 + i;
    return ((static_cast<int64_t>(i >> a.shard_log2) * a.batch + row) << a.shard_log2) + (i & ((1 << a.shard_log2) - 1));
  };
  float v[V];
  if (!src.base) {
#pragma unroll
    for (int r = 0; r < V; ++r) v[r] = 0.f;
  } else if (src.words) {  // verified words, read from L2
    src.verify<V>(off, false);
#pragma unroll
    for (int r = 0; r < V; ++r) v[r] = __ldcg(src.base + 2 * off(r));
  } else {
#pragma unroll
    for (int r = 0; r < V; ++r) v[r] = src.base[off(r)];
  }
  fwht_row_small<LV, LW>(v, sm_small);
#pragma unroll
  for (int j = 0; j < V / W; ++j)
#pragma unroll
    for (int k = 0; k < W; ++k) {
      const int i = point_b<LV, LW>(j, k);
      float b;
      if constexpr (kBiasEarly) b = bb[j * W + k];
      else b = a.bias ? __ldg(a.bias + i) : 0.f;
      store_from_float(a.y, row * m + i, a.dtype, fmaf(v[j * W + k], sg[j * W + k], b));
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

// ---- decode-batch FFT rows (RFFT layers, quipsharp/rfft.py:37-60) -----------
// N = 2^(5 + LV + LW) complex points, one CTA of T = 32 * 2^LW threads per row,
// V = 2^LV points per thread.  Three-factor Cooley-Tukey with the input index
// i = t + T r (t the thread, register digit r slowest) and the output index
// k = k_r + V (k_w + W k_l):
//   1. V-point DFT over r in registers, then twiddle w_N^{t k_r};
//   2. shared-memory transpose: thread (w', lane) takes k_r = w' + W j and all w;
//   3. W-point DFT over w in registers, then twiddle w_N^{V lane k_w};
//   4. 32-point DFT over the lanes by warp shuffles (radix-2 decimation in
//      frequency: lane l ends with k_l = bitreverse5(l));
//   5. the results are staged in shared memory by k (padded one slot per V W
//      points, so a warp's stores hit distinct bank pairs) and leave in natural
//      order: thread t handles k = t + T i, so global loads of the layer's
//      phases / bias and stores of the result are coalesced.
// The in-register DFTs are radix-2 decimation in frequency (natural input,
// bit-reversed output positions) with w_32^e constants from the constant bank.
// Twiddles of steps 1, 3 and 4 come from a table of w_8192^e rounded from
// double and are loaded before the dependent-launch wait, with the layer's
// phases; the inverse transform uses conjugates.

#include "qs_twiddle_gen.inc"  // kTwiddle8192, kTw32

constexpr int kTwLog = 13;

__device__ __forceinline__ float2 cadd(float2 a, float2 b) { return make_float2(a.x + b.x, a.y + b.y); }
__device__ __forceinline__ float2 csub(float2 a, float2 b) { return make_float2(a.x - b.x, a.y - b.y); }
__device__ __forceinline__ float2 cmul(float2 a, float2 b) {
  return make_float2(fmaf(a.x, b.x, -a.y * b.y), fmaf(a.x, b.y, a.y * b.x));
}
template <bool INV>
__device__ __forceinline__ float2 cj(float2 t) { return INV ? make_float2(t.x, -t.y) : t; }

// A read-only load the compiler issues where it stands and keeps in registers
// (a plain __ldg may be re-issued after the dependent-launch wait instead).
__device__ __forceinline__ float2 ldg_pinned(const float2 *p) {
  float2 v;
  asm volatile("ld.global.nc.v2.f32 {%0, %1}, [%2];" : "=f"(v.x), "=f"(v.y) : "l"(p));
  return v;
}

template <bool INV>
__device__ __forceinline__ float2 twiddle(int e, int lgN) {  // w_N^e, e in [0, N)
  return cj<INV>(__ldg(&kTwiddle8192[e << (kTwLog - lgN)]));
}

template <bool INV>
__device__ __forceinline__ float2 twiddle_pinned(int e, int lgN) {
  return cj<INV>(ldg_pinned(&kTwiddle8192[e << (kTwLog - lgN)]));
}

__host__ __device__ constexpr int bitrev(int x, int bits) {
  int r = 0;
  for (int b = 0; b < bits; ++b) r |= ((x >> b) & 1) << (bits - 1 - b);
  return r;
}

// In-register DFT of R <= 32 points (radix-2 DIF): v[p] ends holding k = bitrev(p).
template <int R, bool INV>
__device__ __forceinline__ void dft_regs(float2 (&v)[R]) {
#pragma unroll
  for (int h = R / 2; h >= 1; h >>= 1)
#pragma unroll
    for (int j = 0; j < R; ++j)
      if (!(j & h)) {
        const float2 a = v[j], b = v[j + h];
        v[j] = cadd(a, b);
        const int e = (j & (h - 1)) * (16 / h);  // w_{2h}^(j mod h) = w_32^e
        v[j + h] = e ? cmul(csub(a, b), cj<INV>(kTw32[e])) : csub(a, b);
      }
}

template <int LV, int LW, bool INV>
struct FftRow {
  static constexpr int V = 1 << LV, W = 1 << LW, T = 32 * W, N = T * V, LN = 5 + LV + LW;
  static constexpr int kStage = N + N / (V * W);  // staging slots (padded)
  // w_N^{t k_r}, by register position p (k_r = bitrev(p)); with 32 points per
  // thread they are loaded where used (registers)
  static constexpr bool kT1Early = V <= 16;
  float2 t1[kT1Early ? V : 1];
  float2 t3[W];  // w_N^{V lane k_w}, by position q (k_w = bitrev(q))
  float2 tl[5];  // lane stages: w_{2m}^{lane mod m}, m = 16, 8, 4, 2, 1

  __device__ __forceinline__ void prefetch_twiddles() {
    const int lane = threadIdx.x & 31, t = threadIdx.x;
#pragma unroll
    for (int p = 0; p < (kT1Early ? V : 0); ++p) t1[p] = twiddle_pinned<INV>((t * bitrev(p, LV)) & (N - 1), LN);
#pragma unroll
    for (int q = 0; q < W; ++q) t3[q] = twiddle_pinned<INV>((V * lane * bitrev(q, LW)) & (N - 1), LN);
#pragma unroll
    for (int s = 0; s < 5; ++s) {
      const int m = 16 >> s;
      tl[s] = twiddle_pinned<INV>((lane & (m - 1)) * (N / (2 * m)), LN);
    }
  }

  __device__ __forceinline__ static int slot(int k) { return k + (k >> (LV + LW)); }

  // v: v[r] = input point t + T r.  Leaves output k at stage[slot(k)] (call
  // __syncthreads before reading it); sm and stage are distinct buffers.
  __device__ __forceinline__ void run(float2 (&v)[V], float2 *sm, float2 *stage) const {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    dft_regs<V, INV>(v);
#pragma unroll
    for (int p = 1; p < V; ++p) {
      float2 tw;
      if constexpr (kT1Early) tw = t1[p];
      else tw = twiddle<INV>((static_cast<int>(threadIdx.x) * bitrev(p, LV)) & (N - 1), LN);
      v[p] = cmul(v[p], tw);
    }
#pragma unroll
    for (int p = 0; p < V; ++p) sm[lane + 32 * (w + W * bitrev(p, LV))] = v[p];
    __syncthreads();
#pragma unroll
    for (int j = 0; j < V / W; ++j) {
      float2 u[W];
#pragma unroll
      for (int ww = 0; ww < W; ++ww) u[ww] = sm[lane + 32 * (ww + W * (w + W * j))];
      dft_regs<W, INV>(u);
#pragma unroll
      for (int q = 0; q < W; ++q) v[j * W + q] = q ? cmul(u[q], t3[q]) : u[q];
    }
#pragma unroll
    for (int s = 0; s < 5; ++s) {
      const int m = 16 >> s;
      const bool hi = lane & m;
#pragma unroll
      for (int i = 0; i < V; ++i) {
        const float2 pv = make_float2(__shfl_xor_sync(0xffffffffu, v[i].x, m), __shfl_xor_sync(0xffffffffu, v[i].y, m));
        v[i] = hi ? cmul(csub(pv, v[i]), tl[s]) : cadd(v[i], pv);
      }
    }
    const int kl = V * W * bitrev(lane, 5);
#pragma unroll
    for (int j = 0; j < V / W; ++j)
#pragma unroll
      for (int q = 0; q < W; ++q) stage[slot((w + W * j) + V * bitrev(q, LW) + kl)] = v[j * W + q];
  }
};

__device__ __forceinline__ float2 load_pair(const void *p, int64_t i, int dtype) {  // elements i, i + 1
  if (dtype == QS_F16) return __half22float2(*reinterpret_cast<const __half2 *>(static_cast<const __half *>(p) + i));
  if (dtype == QS_BF16)
    return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(static_cast<const __nv_bfloat16 *>(p) + i));
  return *reinterpret_cast<const float2 *>(static_cast<const float *>(p) + i);
}

__device__ __forceinline__ void store_pair(void *p, int64_t i, int dtype, float2 v) {
  if (dtype == QS_F16) *reinterpret_cast<__half2 *>(static_cast<__half *>(p) + i) = __floats2half2_rn(v.x, v.y);
  else if (dtype == QS_BF16)
    *reinterpret_cast<__nv_bfloat162 *>(static_cast<__nv_bfloat16 *>(p) + i) = __floats2bfloat162_rn(v.x, v.y);
  else *reinterpret_cast<float2 *>(static_cast<float *>(p) + i) = v;
}

struct SmallInF {
  const void *x;
  int dtype;
  const float2 *phase;  // phase_v (N)
  float scale;          // 1 / sqrt(N)
  __half *x2h;
  float *rowscale;
  int n_pad;
  float *y1;
  int64_t m_local;
  int64_t rows;
};

template <int LV, int LW>
__global__ void __launch_bounds__(32 << LW) xsmall_input_rfft_kernel(SmallInF a) {
  using F = FftRow<LV, LW, false>;
  constexpr int V = F::V, W = F::W, T = F::T, N = F::N;
  extern __shared__ float2 smf_small[];
  float2 *const stage = smf_small + N;
  __shared__ float red[W];
  __shared__ float4 zblk[kZeroBlockBytes / 16];
  pdl_launch_dependents();
  const int64_t row = blockIdx.x;
  const int t = threadIdx.x;
  F f;
  f.prefetch_twiddles();
  float2 ph[V];
#pragma unroll
  for (int r = 0; r < V; ++r) ph[r] = ldg_pinned(a.phase + t + T * r);  // layer constant
  pdl_wait();  // x may be the previous kernel's output; y1 may still be read by it
  float2 v[V];
#pragma unroll
  for (int r = 0; r < V; ++r) v[r] = cmul(load_pair(a.x, row * (2 * N) + 2 * (t + T * r), a.dtype), ph[r]);
  BulkZero bz;
  if (a.y1) bz.start(a.y1 + row * a.m_local, a.m_local, zblk);
  f.run(v, smf_small, stage);
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < V; ++i) amax = fmaxf(amax, fmaxf(fabsf(v[i].x), fabsf(v[i].y)));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  if ((t & 31) == 0) red[t >> 5] = amax;
  __syncthreads();  // the row maximum and the staged results
#pragma unroll
  for (int k = 0; k < W; ++k) amax = fmaxf(amax, red[k]);
  float sc, inv;
  xpow2_scale(amax * a.scale, sc, inv);
  sc *= a.scale;
  __half2 *out = reinterpret_cast<__half2 *>(a.x2h + row * a.n_pad);
#pragma unroll
  for (int i = 0; i < V; ++i) {
    const int k = t + T * i;
    const float2 z = stage[F::slot(k)];
    out[k] = __floats2half2_rn(z.x * sc, z.y * sc);
  }
  if (t == 0) a.rowscale[row] = inv;
  bz.finish();
}

struct SmallOutF {
  const float *y1;
  int64_t ld_y1;
  int64_t batch;
  int shard_log2;       // shards > 1: log2(m / shards); else -1
  const float2 *phase;  // phase_u (N)
  const float *bias;
  float scale;          // 1 / sqrt(N)
  void *y;
  int dtype;
  int *busy;
  XPeerGather pg;
};

template <int LV, int LW>
__global__ void __launch_bounds__(32 << LW) xsmall_output_rfft_kernel(SmallOutF a) {
  using F = FftRow<LV, LW, true>;
  constexpr int V = F::V, T = F::T, N = F::N;
  extern __shared__ float2 smf_small[];
  float2 *const stage = smf_small + N;
  const int64_t row = blockIdx.x;
  const int t = threadIdx.x;
  const bool flag = row == 0 && t == 0;
  if (flag) xbusy_set(a.busy, 1);  // before the release: the next input step reads it at its start
  pdl_launch_dependents();
  F f;
  f.prefetch_twiddles();
  constexpr bool kBiasEarly = V <= 16;  // registers: 32 points per thread leave no room for the bias
  const float2 *bias2 = reinterpret_cast<const float2 *>(a.bias);
  float2 ph[V], bb[kBiasEarly ? V : 1];
#pragma unroll
  for (int i = 0; i < V; ++i) {  // layer constants of the outputs k = t + T i
    const float2 p = ldg_pinned(a.phase + t + T * i);
    ph[i] = make_float2(p.x * a.scale, -p.y * a.scale);  // scale * conj(phase)
    if constexpr (kBiasEarly) bb[i] = bias2 ? ldg_pinned(bias2 + t + T * i) : make_float2(0.f, 0.f);
  }
  pdl_wait();  // y1 comes from the matmul (or the ranks' pushes)
  const XPeerSrc src = a.pg.flags ? xwait_peers(a.pg) : xplain_src(a.y1);
  auto off = [&](int r) -> int64_t {
    const int c = 2 * (t + T * r);  // real index of the complex point's first half
    if (a.shard_log2 < 0) return row * a.ld_y1 + c;
    return ((static_cast<int64_t>(c >> a.shard_log2) * a.batch + row) << a.shard_log2) + (c & ((1 << a.shard_log2) - 1));
  };
  float2 v[V];
  if (!src.base) {
#pragma unroll
    for (int r = 0; r < V; ++r) v[r] = make_float2(0.f, 0.f);
  } else if (src.words) {  // verified words, read from L2
    src.verify<V>(off, true);
#pragma unroll
    for (int r = 0; r < V; ++r) {
      const float4 q = __ldcg(reinterpret_cast<const float4 *>(src.base + 2 * off(r)));
      v[r] = make_float2(q.x, q.z);
    }
  } else {
#pragma unroll
    for (int r = 0; r < V; ++r) v[r] = *reinterpret_cast<const float2 *>(src.base + off(r));
  }
  f.run(v, smf_small, stage);
  __syncthreads();
#pragma unroll
  for (int i = 0; i < V; ++i) {
    const int k = t + T * i;
    const float2 z = cmul(stage[F::slot(k)], ph[i]);
    float2 b2;
    if constexpr (kBiasEarly) b2 = bb[i];
    else b2 = bias2 ? __ldg(bias2 + k) : make_float2(0.f, 0.f);
    store_pair(a.y, row * (2 * N) + 2 * k, a.dtype, make_float2(z.x + b2.x, z.y + b2.y));
  }
  if (flag) xbusy_set(a.busy, 0);
}

template <int LV, int LW>
struct RunInF {
  static int run(const SmallInF &a, int64_t rows, cudaStream_t s) {
    constexpr int bytes = 8 * ((32 << (LV + LW)) + FftRow<LV, LW, false>::kStage);
    auto k = xsmall_input_rfft_kernel<LV, LW>;
    QS_CUDA_TRY(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
    return launch_pdl("xsmall_input_rfft", k, dim3(static_cast<unsigned>(rows)), dim3(32 << LW), bytes, s, a);
  }
};

template <int LV, int LW>
struct RunOutF {
  static int run(const SmallOutF &a, int64_t rows, cudaStream_t s) {
    constexpr int bytes = 8 * ((32 << (LV + LW)) + FftRow<LV, LW, true>::kStage);
    auto k = xsmall_output_rfft_kernel<LV, LW>;
    QS_CUDA_TRY(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
    return launch_pdl("xsmall_output_rfft", k, dim3(static_cast<unsigned>(rows)), dim3(32 << LW), bytes, s, a);
  }
};

// (LV, LW) per log2(N) of the complex length: 2^10 .. 2^13.
template <template <int, int> class F, typename... Args>
int dispatch_small_fft(int lg, Args &&...args) {
  switch (lg) {
    case 10: return F<3, 2>::run(args...);
    case 11: return F<3, 3>::run(args...);
    case 12: return F<4, 3>::run(args...);
    case 13: return F<5, 3>::run(args...);
    default: return fail(QS_ERR_UNSUPPORTED, "no decode-batch FFT for 2^%d points", lg);
  }
}

}  // namespace

bool small_rfft_ok(int64_t n_complex, int64_t rows) {
  const int lg = log2_exact(n_complex);
  return lg >= 10 && lg <= 13 && rows >= 1 && rows <= kSmallRhtMaxRows;
}

int launch_small_input_rfft(const void *x, int dtype, int64_t rows, int64_t n, const float2 *phase, float scale,
                            __half *x2h, float *rowscale, int n_pad, float *y1, int64_t m_local, cudaStream_t s) {
  SmallInF a{x, dtype, phase, scale, x2h, rowscale, n_pad, y1, m_local, rows};
  return dispatch_small_fft<RunInF>(log2_exact(n / 2), a, rows, s);
}

int launch_small_output_rfft(const float *y1, int64_t ld_y1, int64_t shards, int64_t batch, int64_t m,
                             const float2 *phase, const float *bias, float scale, void *y, int y_dtype,
                             const XPeerGather *pg, cudaStream_t s) {
  SmallOutF a{};
  a.y1 = y1;
  a.ld_y1 = ld_y1;
  a.batch = batch;
  a.shard_log2 = -1;
  if (shards > 1) {
    a.shard_log2 = log2_exact(m / shards);
    if (a.shard_log2 < 1) return fail(QS_ERR_UNSUPPORTED, "shard width is not an even power of two");
  }
  a.phase = phase;
  a.bias = bias;
  a.scale = scale;
  a.y = y;
  a.dtype = y_dtype;
  a.busy = xbusy_flag();
  if (pg) a.pg = *pg;
  return dispatch_small_fft<RunOutF>(log2_exact(m / 2), a, batch, s);
}

bool small_rht_ok(int64_t n, int64_t rows) {
  const int lg = log2_exact(n);
  return lg >= 10 && lg <= 14 && rows >= 1 && rows <= kSmallRhtMaxRows;
}

int launch_small_input_rht(const void *x, int dtype, int64_t rows, int64_t n, const float *sv, float scale,
                           __half *x2h, float *rowscale, int n_pad, float *y1, int64_t m_local, cudaStream_t s) {
  SmallIn a{x, dtype, sv, scale, x2h, rowscale, n_pad, y1, m_local, rows};
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
