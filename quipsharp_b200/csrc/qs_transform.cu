// Incoherence transforms on rows held in shared memory:
//   * FWHT (quipsharp/hadamard.py:17-40) for the randomized Hadamard transform
//     (quipsharp/incoherence.py:86-93);
//   * mixed-radix Stockham FFT for the RFFT transform (quipsharp/rfft.py:37-60).
// One CTA owns one row; the whole row lives in shared memory, so every pass
// runs at shared-memory speed and the row is read and written in HBM once.
// The "linear" kernels fuse the transforms with the producer/consumer steps of
// the quantized-linear forward: input cast + sign/phase + transform + fp16
// packing for the matmul (with a per-row power-of-two scale) + zeroing of the
// y1 accumulator; and y1 -> transform -> sign/conj-phase -> bias -> cast.
#include <cmath>

#include "qs_fft.cuh"

namespace qs {

// ============================================================================
// FWHT
// ============================================================================
constexpr int kFwhtMaxE = 32;  // elements per thread per pass (upper bound)

__device__ __forceinline__ int fpad(int i) { return i + (i >> 5); }

template <typename Load, typename Store>
__device__ __forceinline__ void fwht_pass(Load load, Store store, int n, int lo, int w) {
  const int G = 1 << w;
  const int groups = n >> w;
  for (int gi = threadIdx.x; gi < groups; gi += blockDim.x) {
    const int base = (gi & ((1 << lo) - 1)) | ((gi >> lo) << (lo + w));
    float v[kFwhtMaxE];
#pragma unroll
    for (int j = 0; j < kFwhtMaxE; ++j)
      if (j < G) v[j] = load(base + (j << lo));
#pragma unroll
    for (int h = 1; h < kFwhtMaxE; h <<= 1) {
      if (h < G) {
#pragma unroll
        for (int j = 0; j < kFwhtMaxE; ++j) {
          if (j < G && !(j & h)) {
            const float a = v[j], b = v[j + h];
            v[j] = a + b;
            v[j + h] = a - b;
          }
        }
      }
    }
#pragma unroll
    for (int j = 0; j < kFwhtMaxE; ++j)
      if (j < G) store(base + (j << lo), v[j]);
  }
}

// Unnormalised Walsh-Hadamard transform of the row gload(i), i < 2^L, handed
// to gstore(i, v).  Index bits are processed in passes of log2(E) bits; in a
// pass each thread owns groups of E elements that differ only in those bits
// and transforms them in registers.  The first pass reads global memory, the
// last writes through gstore; passes in between use buf[fpad(.)].
template <typename GLoad, typename GStore>
__device__ __forceinline__ void fwht_row(GLoad gload, GStore gstore, float *buf, int L, int E) {
  const int n = 1 << L;
  const int e = 31 - __clz(E);
  auto sload = [&](int i) { return buf[fpad(i)]; };
  auto sstore = [&](int i, float v) { buf[fpad(i)] = v; };
  if (L <= e) {  // one pass (also n == 1)
    fwht_pass(gload, gstore, n, 0, L);
    return;
  }
  fwht_pass(gload, sstore, n, 0, e);
  __syncthreads();
  int lo = e;
  for (; lo + e < L; lo += e) {
    fwht_pass(sload, sstore, n, lo, e);
    __syncthreads();
  }
  fwht_pass(sload, gstore, n, lo, L - lo);
}

struct FwhtGeom {
  int L, E, threads;
  size_t smem;
};

static FwhtGeom fwht_geom(int64_t n) {
  FwhtGeom g;
  g.L = 0;
  while ((int64_t(1) << g.L) < n) ++g.L;
  int threads = static_cast<int>(std::min<int64_t>(1024, std::max<int64_t>(32, n / 16)));
  g.threads = threads;
  // 16 (or 32 for the largest rows) elements per group; tiny rows use one group.
  g.E = static_cast<int>(std::min<int64_t>(n, std::max<int64_t>(16, std::min<int64_t>(kFwhtMaxE, n / threads))));
  g.smem = static_cast<size_t>(n + (n >> 5) + 1) * sizeof(float);
  return g;
}

__global__ void __launch_bounds__(1024) fwht_rows_kernel(const void *x, int64_t ld_x, void *y,
                                                         int64_t ld_y, int dtype, int L, int E,
                                                         const float *pre, const float *post,
                                                         float scale) {
  extern __shared__ float fsm[];
  const int64_t row = blockIdx.x;
  const void *xr = static_cast<const char *>(x) + row * ld_x * (dtype == QS_F32 ? 4 : 2);
  void *yr = static_cast<char *>(y) + row * ld_y * (dtype == QS_F32 ? 4 : 2);
  auto gload = [&](int i) {
    float v = load_as_float(xr, i, dtype);
    return pre ? v * pre[i] : v;
  };
  auto gstore = [&](int i, float v) {
    v *= scale;
    if (post) v *= post[i];
    store_from_float(yr, i, dtype, v);
  };
  fwht_row(gload, gstore, fsm, L, E);
}

template <typename K>
static int set_smem(K kern, size_t bytes) {
  QS_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   static_cast<int>(bytes)));
  return QS_OK;
}

static float inv_sqrt_f32(int64_t n) { return static_cast<float>(1.0 / std::sqrt(static_cast<double>(n))); }

int launch_fwht(const void *x, int64_t ld_x, void *y, int64_t ld_y, int dtype, int64_t rows,
                int64_t n, const float *pre, const float *post, cudaStream_t s) {
  FwhtGeom g = fwht_geom(n);
  QS_CUDA_TRY(cudaFuncSetAttribute(fwht_rows_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   static_cast<int>(g.smem)));
  fwht_rows_kernel<<<rows, g.threads, g.smem, s>>>(x, ld_x, y, ld_y, dtype, g.L, g.E, pre, post,
                                                  inv_sqrt_f32(n));
  return check_launch("fwht");
}

// ============================================================================
// FFT plans and dispatch (kernels: qs_fft.cuh, instantiated in qs_fft_*.cu)
// ============================================================================
static int make_plan(int64_t N, FftPlan &p) {
  if (N < 1 || N > kFftMaxN) return fail(QS_ERR_UNSUPPORTED, "FFT length %lld outside [1, %d]", (long long)N, kFftMaxN);
  p.N = static_cast<int>(N);
  p.nst = 0;
  int64_t rem = N;
  int big = 0;
  for (int P : {43, 41, 37, 31, 29, 23, 19, 17, 13, 11}) {
    while (rem % P == 0) {
      if (big) return fail(QS_ERR_UNSUPPORTED, "FFT length %lld has two prime factors >= 11", (long long)N);
      big = P;
      rem /= P;
    }
  }
  p.big = big;
  if (big) p.radix[p.nst++] = big;
  for (int P : {7, 5, 3}) {
    while (rem % P == 0) {
      p.radix[p.nst++] = P;
      rem /= P;
    }
  }
  for (int P : {16, 8, 4, 2}) {
    while (rem % P == 0) {
      p.radix[p.nst++] = P;
      rem /= P;
    }
  }
  if (rem != 1)
    return fail(QS_ERR_UNSUPPORTED, "FFT length %lld has a prime factor above 43", (long long)N);
  if (p.nst == 0) p.radix[p.nst++] = 1;  // N == 1
  if (p.nst > kMaxStages) return fail(QS_ERR_UNSUPPORTED, "FFT plan too deep");
  p.pingpong = N <= kFftPingPongMax;
  if (p.pingpong) {
    int threads = 64;
    while (threads < 512 && threads * 8 < N) threads *= 2;
    p.threads = threads;
  } else {
    if (big) return fail(QS_ERR_UNSUPPORTED, "FFT length %lld: prime factors >= 11 need N <= %d", (long long)N, kFftPingPongMax);
    p.threads = 1024;  // N / 1024 <= kFftIpE values per thread
  }
  return QS_OK;
}

int check_fft_size(int64_t n_complex) {
  FftPlan p;
  return make_plan(n_complex, p);
}

static size_t fft_smem_bytes(const FftPlan &p) {
  return (p.pingpong ? 2 : 1) * static_cast<size_t>(fft_buf_elems(p.N)) * sizeof(float2);
}

int launch_rfft(int inverse, const void *x, int64_t ld_x, void *y, int64_t ld_y, int dtype,
                int64_t rows, int64_t n, const void *phase, cudaStream_t s) {
  FftPlan p;
  int st = make_plan(n / 2, p);
  if (st) return st;
  const size_t smem = fft_smem_bytes(p);
  const float2 *ph = static_cast<const float2 *>(phase);
  const float sc = inv_sqrt_f32(n / 2);
  if (!p.pingpong) return run_rfft_rows<false, 0>(inverse, x, ld_x, y, ld_y, dtype, rows, p, ph, sc, smem, s);
  switch (p.big) {
#define QS_CASE(B) \
  case B: return run_rfft_rows<true, B>(inverse, x, ld_x, y, ld_y, dtype, rows, p, ph, sc, smem, s);
    QS_FOR_EACH_BIG(QS_CASE)
#undef QS_CASE
    default: return fail(QS_ERR_UNSUPPORTED, "bad FFT plan");
  }
}

// ============================================================================
// Quantized-linear input / output steps
// ============================================================================
// x2 workspace layout: [x2h: batch x n_pad fp16][rowscale: batch float32],
// n_pad = round_up(n, 256) (zero filled beyond n).  x2h[r] = fp16(x2[r] * 2^k_r)
// with 2^k_r chosen so max|x2[r]| * 2^k_r lies in [2^11, 2^12); rowscale[r] =
// 2^-k_r undoes it in the matmul epilogue.  The power-of-two scaling is exact
// and keeps every row inside fp16 range whatever the activation magnitudes.
static int64_t n_padded(int64_t n) { return padded_T(n) * 8; }

int64_t linear_input_bytes(int64_t batch, int64_t n) {
  return round_up(batch * n_padded(n) * 2, 256) + round_up(batch * 4, 256);
}

__global__ void __launch_bounds__(1024) linear_input_rht_kernel(
    const void *x, int dtype, int L, int E, const float *sv, float scale, __half *x2h,
    float *rowscale, int n_pad, float *y1, int64_t m_local) {
  extern __shared__ float fsm[];
  __shared__ float red[32];
  pdl_launch_dependents();
  pdl_wait();  // x may be the previous kernel's output; y1 may still be read by it
  const int n = 1 << L;
  const int64_t row = blockIdx.x;
  for (int64_t i = threadIdx.x; i < m_local; i += blockDim.x) y1[row * m_local + i] = 0.f;
  float amax = 0.f;
  auto gload = [&](int i) { return load_as_float(x, row * n + i, dtype) * sv[i]; };
  auto rstore = [&](int i, float v) {
    v *= scale;
    amax = fmaxf(amax, fabsf(v));
    fsm[fpad(i)] = v;
  };
  fwht_row(gload, rstore, fsm, L, E);
  __syncthreads();
  emit_x2h([&](int i) { return fsm[fpad(i)]; }, amax, n, n_pad, x2h + row * n_pad, rowscale + row, red);
}

// Buffer (0/1) that receives the result of fft_row when its store functor
// writes shared memory: the one the last stage does not read.
static int fft_result_buf(const FftPlan &p) {
  if (!p.pingpong) return 0;
  if (p.nst == 1) return 0;
  return ((p.nst - 2) % 2) ^ 1;
}

int launch_linear_input(const void *x, int x_dtype, int64_t batch, int64_t n, int transform,
                        const float *sv, const void *phase_v, void *x2ws, float *y1,
                        int64_t m_local, cudaStream_t s) {
  const int64_t n_pad = n_padded(n);
  __half *x2h = static_cast<__half *>(x2ws);
  float *rowscale = reinterpret_cast<float *>(static_cast<char *>(x2ws) + round_up(batch * n_pad * 2, 256));
  if (!y1) m_local = 0;
  int st;
  if (transform == QS_RHT) {
    FwhtGeom g = fwht_geom(n);
    if ((st = set_smem(linear_input_rht_kernel, g.smem))) return st;
    return launch_pdl("linear_input_rht", linear_input_rht_kernel, dim3(batch), dim3(g.threads), g.smem, s,
                      x, x_dtype, g.L, g.E, sv, inv_sqrt_f32(n), x2h, rowscale, static_cast<int>(n_pad), y1,
                      m_local);
  }
  FftPlan p;
  if ((st = make_plan(n / 2, p))) return st;
  const size_t smem = fft_smem_bytes(p);
  const float2 *ph = static_cast<const float2 *>(phase_v);
  const float sc = inv_sqrt_f32(n / 2);
  const int rb = fft_result_buf(p), np = static_cast<int>(n_pad);
  if (!p.pingpong)
    return run_linear_input_rfft<false, 0>(x, x_dtype, batch, p, ph, sc, x2h, rowscale, np, y1, m_local, rb, smem, s);
  switch (p.big) {
#define QS_CASE(B) \
  case B: return run_linear_input_rfft<true, B>(x, x_dtype, batch, p, ph, sc, x2h, rowscale, np, y1, m_local, rb, smem, s);
    QS_FOR_EACH_BIG(QS_CASE)
#undef QS_CASE
    default: return fail(QS_ERR_UNSUPPORTED, "bad FFT plan");
  }
}

__global__ void __launch_bounds__(1024) linear_output_rht_kernel(const float *y1, int64_t ld_y1,
                                                                 int64_t shards, int64_t batch,
                                                                 int L, int E, const float *su,
                                                                 const float *bias, float scale,
                                                                 void *y, int dtype) {
  extern __shared__ float fsm[];
  pdl_launch_dependents();
  pdl_wait();  // y1 comes from the matmul kernel
  const int m = 1 << L;
  const int64_t mp = m / shards;
  const int64_t row = blockIdx.x;
  auto gload = [&](int i) { return y1[y1_offset(row, i, ld_y1, shards, mp, batch)]; };
  auto gstore = [&](int i, float v) {
    v = v * scale * su[i];
    if (bias) v += bias[i];
    store_from_float(y, row * m + i, dtype, v);
  };
  fwht_row(gload, gstore, fsm, L, E);
}

int launch_linear_output(const float *y1, int64_t ld_y1, int64_t shards, int64_t batch, int64_t m,
                         int transform, const float *su, const void *phase_u, const float *bias,
                         void *y, int y_dtype, cudaStream_t s) {
  int st;
  if (transform == QS_RHT) {
    FwhtGeom g = fwht_geom(m);
    if ((st = set_smem(linear_output_rht_kernel, g.smem))) return st;
    return launch_pdl("linear_output_rht", linear_output_rht_kernel, dim3(batch), dim3(g.threads), g.smem, s,
                      y1, ld_y1, shards, batch, g.L, g.E, su, bias, inv_sqrt_f32(m), y, y_dtype);
  }
  if (ld_y1 % 2) return fail(QS_ERR_ALIGNMENT, "RFFT y1 row stride must be even");
  FftPlan p;
  if ((st = make_plan(m / 2, p))) return st;
  const size_t smem = fft_smem_bytes(p);
  const float2 *ph = static_cast<const float2 *>(phase_u);
  const float sc = inv_sqrt_f32(m / 2);
  if (!p.pingpong)
    return run_linear_output_rfft<false, 0>(y1, ld_y1, shards, batch, p, ph, bias, sc, y, y_dtype, smem, s);
  switch (p.big) {
#define QS_CASE(B) \
  case B: return run_linear_output_rfft<true, B>(y1, ld_y1, shards, batch, p, ph, bias, sc, y, y_dtype, smem, s);
    QS_FOR_EACH_BIG(QS_CASE)
#undef QS_CASE
    default: return fail(QS_ERR_UNSUPPORTED, "bad FFT plan");
  }
}

}  // namespace qs
