// Host side of the incoherence transforms: plans (stage radices, cluster
// size, threads, shared memory) and dispatch of the qs_xform.cuh kernels for
//   * the standalone FWHT (quipsharp/hadamard.py:17-40) and RFFT transform
//     (quipsharp/rfft.py:37-60) entry points;
//   * the input / output steps of the quantized-linear forward
//     (quipsharp/incoherence.py:86-115, quipsharp/rfft.py:62-100): input cast +
//     sign / phase + transform + fp16 packing for the matmul (per-row power-of-two
//     scale) + zeroing of the y1 accumulator; and y1 -> transform -> sign /
//     conjugate phase -> bias -> cast.
#include <algorithm>
#include <cmath>

#include "qs_xform.cuh"

namespace qs {

// Largest dynamic shared memory a plan may ask for (two row buffers); the
// kernels' static shared memory (twiddle tables, reductions) is below 4 KB.
constexpr size_t kXSmemCap = 220 * 1024;

static int xnum_sms() {
  static int cached[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && cached[dev]) return cached[dev];
  int n = 148;
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  if (dev < 64) cached[dev] = n;
  return n;
}

// The dry-pass hint flag (see xbusy_flag in qs_xform.cuh): one int per device,
// its address looked up once per device.
__device__ int g_qs_xbusy;

int *xbusy_flag() {
  static int *cached[64] = {nullptr};
  static bool tried[64] = {false};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  if (!tried[dev]) {
    void *p = nullptr;
    if (cudaGetSymbolAddress(&p, g_qs_xbusy) != cudaSuccess) {
      p = nullptr;
      cudaGetLastError();
    }
    cached[dev] = static_cast<int *>(p);
    tried[dev] = true;
  }
  return cached[dev];
}

static float inv_sqrt_f32(int64_t n) { return static_cast<float>(1.0 / std::sqrt(static_cast<double>(n))); }

static size_t plan_smem(int N, int C, int elem_bytes) {
  const int E = N / C;
  return 2 * static_cast<size_t>(elem_bytes) *
         static_cast<size_t>(elem_bytes == 8 ? xbuf_elems<float2>(E) : xbuf_elems<float>(E));
}

// Points per CTA above which a few-row transform is spread over a cluster:
// one CTA is fastest while its share stays small (a cluster costs barriers
// and leaves each SM a single warp or two).
constexpr int kXLatencyPointsFft = 2048;
constexpr int kXLatencyPointsFwht = 4096;

// Few rows: the rows alone cannot fill the SMs; plans minimise one row's latency.
static bool few_rows(int64_t rows) { return rows * 2 <= xnum_sms(); }

// CTAs per row wanted before the stages are known: the fewest whose share of
// the two row buffers fits kXSmemCap (a cluster across SMs costs a many-row
// transform more in barriers and remote stores than it gains); then, while the
// rows alone leave SMs idle, doubled (up to 16) while each CTA's share is above
// `latency_points`.
static int wanted_cluster(int N, int elem_bytes, int64_t rows, int latency_points) {
  int C = 1;
  while (plan_smem(N, C, elem_bytes) > kXSmemCap && C < kXMaxCluster) C *= 2;
  const int64_t sms = xnum_sms();
  while (C < kXMaxCluster && rows * 2 * C <= sms && N / C > latency_points) C *= 2;
  return C;
}

// Largest power-of-two radix (log2) of a plan.  Many rows: `cap` (few stages,
// each thread a long independent chain; other rows fill the SM).  Few rows:
// small enough that every stage still has kXLatencyTasks butterflies per CTA,
// so the SM runs several warps per scheduler while one row is in flight.
constexpr int kXLatencyTasks = 256;
static int max_radix_log(int N, int C, int64_t rows, int cap) {
  if (!few_rows(rows)) return cap;
  int w = 1;
  while (w < cap && (N / C) >> (w + 1) >= kXLatencyTasks) ++w;
  return w;
}

// Fixes C (at most `want`, a power of two dividing every stage's butterfly
// count, so each butterfly's inputs sit in one CTA), then the per-CTA task
// counts and the launch shape.
static int finish_plan(XPlan &p, XLaunch &L, int elem_bytes, int64_t rows, int want) {
  int C = want;
  for (bool ok = false; !ok && C > 1;) {
    ok = true;
    for (int s = 0; s < p.nst; ++s) ok = ok && (p.st[s].nb % C == 0);
    if (!ok) C /= 2;
  }
  if (plan_smem(p.N, C, elem_bytes) > kXSmemCap)
    return fail(QS_ERR_UNSUPPORTED, "transform of %d points does not fit the shared memory of %d CTAs", p.N, C);
  p.C = C;
  p.cl = 0;
  while ((1 << p.cl) < C) ++p.cl;
  p.E = p.N / C;
  int most = 128;
  for (int s = 0; s < p.nst; ++s) {
    XStage &S = p.st[s];
    S.nbC = S.nb / C;
    // odd radices: few rows across a cluster run compact rolled code with one
    // output pair per task, or two when one pair per task would need more
    // than one round of kXMaxThreads; otherwise unrolled groups of up to six
    S.compact = 0;
    if ((S.R & 1) && S.R > 1) {
      const int H = (S.R - 1) / 2;
      if (C > 1 && few_rows(rows) && H > 1) {
        S.compact = S.nbC * H <= kXMaxThreads ? 1 : 2;
        S.G = (H + S.compact - 1) / S.compact;
      } else {
        S.G = xodd_groups(S.R);
      }
    }
    S.dnbC = make_fastdiv(static_cast<uint32_t>(S.nbC));
    most = std::max(most, S.nbC * S.G);
  }
  L.threads = std::min(kXMaxThreads, (most + 31) / 32 * 32);
  L.smem = plan_smem(p.N, C, elem_bytes);
  L.rows = rows;
  return QS_OK;
}

// Complex FFT of N points: the prime >= 11 (at most one, once), 7 / 5 / 3, then
// the power-of-two part in balanced stages (radices up to 16; smaller for few
// rows, see max_radix_log); a copy stage follows an odd last radix (the
// last stage writes the sink).
static int make_fft_plan(int64_t N64, int64_t rows, XPlan &p, XLaunch &L) {
  if (N64 < 1 || N64 > kXMaxN)
    return fail(QS_ERR_UNSUPPORTED, "FFT length %lld outside [1, %d]", (long long)N64, kXMaxN);
  const int N = static_cast<int>(N64);
  int rem = N, big = 0, nr = 0;
  int radix[kXMaxStages];
  for (int P : {43, 41, 37, 31, 29, 23, 19, 17, 13, 11}) {
    if (rem % P == 0) {
      if (big || (rem / P) % P == 0)
        return fail(QS_ERR_UNSUPPORTED, "FFT length %lld has more than one prime factor >= 11", (long long)N);
      big = P;
      rem /= P;
    }
  }
  if (big) radix[nr++] = big;
  for (int P : {7, 5, 3}) {
    while (rem % P == 0) {
      if (nr >= kXMaxStages - 1) return fail(QS_ERR_UNSUPPORTED, "FFT plan too deep");
      radix[nr++] = P;
      rem /= P;
    }
  }
  int a = 0;
  while (rem % 2 == 0) {
    rem /= 2;
    ++a;
  }
  if (rem != 1) return fail(QS_ERR_UNSUPPORTED, "FFT length %lld has a prime factor above 43", (long long)N);
  const int want = wanted_cluster(N, 8, rows, kXLatencyPointsFft);
  if (a > 0) {
    const int maxlog = max_radix_log(N, want, rows, 4);
    const int ns = (a + maxlog - 1) / maxlog, base = a / ns, extra = a % ns;
    if (nr + ns >= kXMaxStages) return fail(QS_ERR_UNSUPPORTED, "FFT plan too deep");
    for (int i = 0; i < ns; ++i) radix[nr++] = 1 << (base + (i < extra ? 1 : 0));
  }
  if (nr == 0) radix[nr++] = 1;              // N == 1
  if (radix[nr - 1] & 1 && radix[nr - 1] > 1) radix[nr++] = 1;
  p.N = N;
  p.nst = nr;
  p.big = big;
  int Ns = 1;
  for (int s = 0; s < nr; ++s) {
    XStage &S = p.st[s];
    S.R = radix[s];
    S.G = 1;
    S.compact = 0;
    S.Ns = Ns;
    S.nb = N / S.R;
    S.twstep = N / (Ns * S.R);
    S.dNs = make_fastdiv(static_cast<uint32_t>(Ns));
    Ns *= S.R;
  }
  return finish_plan(p, L, 8, rows, want);
}

// FWHT of n = 2^Lb points: balanced passes of the rotating form, up to 5 bits
// each for one CTA per row, up to 3 across a cluster.
static int make_fwht_plan(int64_t n, int64_t rows, XPlan &p, XLaunch &L) {
  if (n < 1 || (n & (n - 1)))
    return fail(QS_ERR_NOT_POW2, "fwht requires a power-of-two size along dim, got %lld", (long long)n);
  if (n > kXMaxN) return fail(QS_ERR_UNSUPPORTED, "fwht size %lld exceeds %d", (long long)n, kXMaxN);
  int Lb = 0;
  while ((int64_t(1) << Lb) < n) ++Lb;
  const int want = wanted_cluster(static_cast<int>(n), 4, rows, kXLatencyPointsFwht);
  int widths[kXMaxStages], np = 0;
  if (Lb == 0) {
    widths[np++] = 0;
  } else {
    const int maxw = max_radix_log(static_cast<int>(n), want, rows, 5);
    const int ns = (Lb + maxw - 1) / maxw, base = Lb / ns, extra = Lb % ns;
    for (int i = 0; i < ns; ++i) widths[np++] = base + (i < extra ? 1 : 0);
  }
  p.N = static_cast<int>(n);
  p.nst = np;
  p.big = 0;
  for (int s = 0; s < np; ++s) {
    XStage &S = p.st[s];
    S.R = 1 << widths[s];
    S.G = 1;
    S.compact = 0;
    S.Ns = 1;
    S.nb = p.N / S.R;
    S.twstep = 0;
    S.dNs = make_fastdiv(1);
  }
  return finish_plan(p, L, 4, rows, want);
}

int check_fft_size(int64_t n_complex) {
  XPlan p;
  XLaunch L;
  return make_fft_plan(n_complex, 1, p, L);
}

int check_fwht_size(int64_t n) {
  XPlan p;
  XLaunch L;
  return make_fwht_plan(n, 1, p, L);
}

// ============================================================================
// Standalone transforms
// ============================================================================
int launch_fwht(const void *x, int64_t ld_x, void *y, int64_t ld_y, int dtype, int64_t rows, int64_t n,
                const float *pre, const float *post, cudaStream_t s) {
  XPlan p;
  XLaunch L;
  int st = make_fwht_plan(n, rows, p, L);
  if (st) return st;
  if (rows == 0) return QS_OK;
  const float sc = inv_sqrt_f32(n);
  return p.C > 1 ? run_xfwht_rows<true>(L, s, x, ld_x, y, ld_y, dtype, p, pre, post, sc)
                 : run_xfwht_rows<false>(L, s, x, ld_x, y, ld_y, dtype, p, pre, post, sc);
}

int launch_rfft(int inverse, const void *x, int64_t ld_x, void *y, int64_t ld_y, int dtype, int64_t rows, int64_t n,
                const void *phase, cudaStream_t s) {
  XPlan p;
  XLaunch L;
  int st = make_fft_plan(n / 2, rows, p, L);
  if (st) return st;
  if (rows == 0) return QS_OK;
  const float2 *ph = static_cast<const float2 *>(phase);
  const float sc = inv_sqrt_f32(n / 2);
  switch (p.big) {
#define QS_CASE(B)                                                                                   \
  case B:                                                                                            \
    return p.C > 1 ? run_xrfft_rows<B, true>(L, s, inverse, x, ld_x, y, ld_y, dtype, p, ph, sc)     \
                   : run_xrfft_rows<B, false>(L, s, inverse, x, ld_x, y, ld_y, dtype, p, ph, sc);
    QS_FOR_EACH_XBIG(QS_CASE)
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

// Pointer aligned for loads / stores of element pairs of `dtype` (null passes).
static bool pair_aligned(const void *p, int dtype) {
  const uintptr_t a = dtype == QS_F32 ? 8 : 4;
  return (reinterpret_cast<uintptr_t>(p) % a) == 0;
}

// Layout: [x2h][rowscale][two-pass scratch (float32 rows + L1 partial sums),
// only for batches and sizes that use the two-pass RFFT].
int64_t linear_input_bytes(int64_t batch, int64_t n) {
  return round_up(batch * n_padded(n) * 2, 256) + round_up(batch * 4, 256) + two_pass_input_scratch_bytes(batch, n);
}

int launch_linear_input(const void *x, int x_dtype, int64_t batch, int64_t n, int transform, const float *sv,
                        const void *phase_v, void *x2ws, float *y1, int64_t m_local, cudaStream_t s) {
  const int64_t n_pad = n_padded(n);
  __half *x2h = static_cast<__half *>(x2ws);
  float *rowscale = reinterpret_cast<float *>(static_cast<char *>(x2ws) + round_up(batch * n_pad * 2, 256));
  if (!y1) m_local = 0;
  const int np = static_cast<int>(n_pad);
  XPlan p;
  XLaunch L;
  L.warm = 1;
  int st;
  if (transform == QS_RHT) {
    if (small_rht_ok(n, batch))  // decode batches: one-barrier row kernel
      return launch_small_input_rht(x, x_dtype, batch, n, sv, inv_sqrt_f32(n), x2h, rowscale, np, y1, m_local, s);
    if ((st = make_fwht_plan(n, batch, p, L))) return st;
    const float sc = inv_sqrt_f32(n);
    return p.C > 1 ? run_xinput_rht<true>(L, s, x, x_dtype, p, sv, sc, x2h, rowscale, np, y1, m_local)
                   : run_xinput_rht<false>(L, s, x, x_dtype, p, sv, sc, x2h, rowscale, np, y1, m_local);
  }
  const float2 *ph = static_cast<const float2 *>(phase_v);
  const float sc = inv_sqrt_f32(n / 2);
  if (small_rfft_ok(n / 2, batch) && pair_aligned(x, x_dtype))  // decode batches: one-barrier row kernel
    return launch_small_input_rfft(x, x_dtype, batch, n, ph, sc, x2h, rowscale, np, y1, m_local, s);
  if (two_pass_rfft(n / 2, batch, nullptr, nullptr) && (!y1 || few_rows(batch))) {
    void *scratch = static_cast<char *>(x2ws) + round_up(batch * n_pad * 2, 256) + round_up(batch * 4, 256);
    return launch_two_pass_input(x, x_dtype, batch, n, ph, sc, x2h, rowscale, np, scratch, y1, m_local, s);
  }
  if ((st = make_fft_plan(n / 2, batch, p, L))) return st;
  switch (p.big) {
#define QS_CASE(B)                                                                                             \
  case B:                                                                                                      \
    return p.C > 1 ? run_xinput_rfft<B, true>(L, s, x, x_dtype, p, ph, sc, x2h, rowscale, np, y1, m_local)    \
                   : run_xinput_rfft<B, false>(L, s, x, x_dtype, p, ph, sc, x2h, rowscale, np, y1, m_local);
    QS_FOR_EACH_XBIG(QS_CASE)
#undef QS_CASE
    default: return fail(QS_ERR_UNSUPPORTED, "bad FFT plan");
  }
}

int launch_linear_output(float *y1, int64_t ld_y1, int64_t shards, int64_t batch, int64_t m, int transform,
                         const float *su, const void *phase_u, const float *bias, void *y, int y_dtype,
                         cudaStream_t s, const XPeerGather *pg) {
  XPlan p;
  XLaunch L;
  int st;
  if (transform == QS_RHT) {
    const int64_t mp = m / shards;
    if (small_rht_ok(m, batch) && (shards == 1 || (mp & (mp - 1)) == 0))  // decode batches
      return launch_small_output_rht(y1, ld_y1, shards, batch, m, su, bias, inv_sqrt_f32(m), y, y_dtype, pg, s);
    if ((st = make_fwht_plan(m, batch, p, L))) return st;
    if (pg) L.pg = *pg;
    const float sc = inv_sqrt_f32(m);
    return p.C > 1 ? run_xoutput_rht<true>(L, s, y1, ld_y1, shards, batch, p, su, bias, sc, y, y_dtype)
                   : run_xoutput_rht<false>(L, s, y1, ld_y1, shards, batch, p, su, bias, sc, y, y_dtype);
  }
  if (ld_y1 % 2) return fail(QS_ERR_ALIGNMENT, "RFFT y1 row stride must be even");
  const float2 *ph = static_cast<const float2 *>(phase_u);
  const float sc = inv_sqrt_f32(m / 2);
  const int64_t mp = m / shards;
  if (small_rfft_ok(m / 2, batch) && (shards == 1 || (mp >= 2 && (mp & (mp - 1)) == 0)) &&
      (pg || pair_aligned(y1, QS_F32)) && pair_aligned(bias, QS_F32) && pair_aligned(y, y_dtype))
    return launch_small_output_rfft(y1, ld_y1, shards, batch, m, ph, bias, sc, y, y_dtype, pg, s);
  // the two-pass store loop reads phase / bias and writes y two complex values at a time
  const bool aligned16 = (reinterpret_cast<uintptr_t>(ph) & 15) == 0 && (reinterpret_cast<uintptr_t>(bias) & 15) == 0 &&
                         (reinterpret_cast<uintptr_t>(y) & 15) == 0;
  if (!pg && shards == 1 && ld_y1 == m && aligned16 && two_pass_rfft(m / 2, batch, nullptr, nullptr))
    return launch_two_pass_output(y1, batch, m, ph, bias, sc, y, y_dtype, s);
  if ((st = make_fft_plan(m / 2, batch, p, L))) return st;
  if (pg) L.pg = *pg;
  switch (p.big) {
#define QS_CASE(B)                                                                                                \
  case B:                                                                                                         \
    return p.C > 1 ? run_xoutput_rfft<B, true>(L, s, y1, ld_y1, shards, batch, p, ph, bias, sc, y, y_dtype)      \
                   : run_xoutput_rfft<B, false>(L, s, y1, ld_y1, shards, batch, p, ph, bias, sc, y, y_dtype);
    QS_FOR_EACH_XBIG(QS_CASE)
#undef QS_CASE
    default: return fail(QS_ERR_UNSUPPORTED, "bad FFT plan");
  }
}

}  // namespace qs
