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

#include "qs_common.cuh"
#include "qs_launch.h"

namespace qs {

// ============================================================================
// FWHT
// ============================================================================
constexpr int kFwhtMaxE = 32;  // elements per thread per pass (upper bound)

__device__ __forceinline__ int fpad(int i) { return i + (i >> 5); }

// In-place unnormalised Walsh-Hadamard transform of buf[fpad(0..n-1)].
// Bits of the index are processed in passes of log2(E) bits; within a pass each
// thread owns groups of E elements that differ only in those bits and
// transforms them in registers.
__device__ __forceinline__ void fwht_smem(float *buf, int L, int E) {
  const int n = 1 << L;
  int e = 31 - __clz(E);
  for (int lo = 0; lo < L; lo += e) {
    const int w = min(e, L - lo);
    const int G = 1 << w;
    const int groups = n >> w;
    for (int gi = threadIdx.x; gi < groups; gi += blockDim.x) {
      const int base = (gi & ((1 << lo) - 1)) | ((gi >> lo) << (lo + w));
      float v[kFwhtMaxE];
#pragma unroll
      for (int j = 0; j < kFwhtMaxE; ++j)
        if (j < G) v[j] = buf[fpad(base + (j << lo))];
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
        if (j < G) buf[fpad(base + (j << lo))] = v[j];
    }
    __syncthreads();
  }
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
  const int n = 1 << L;
  const int64_t row = blockIdx.x;
  const void *xr = static_cast<const char *>(x) + row * ld_x * (dtype == QS_F32 ? 4 : 2);
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    float v = load_as_float(xr, i, dtype);
    if (pre) v *= pre[i];
    fsm[fpad(i)] = v;
  }
  __syncthreads();
  fwht_smem(fsm, L, E);
  void *yr = static_cast<char *>(y) + row * ld_y * (dtype == QS_F32 ? 4 : 2);
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    float v = fsm[fpad(i)] * scale;
    if (post) v *= post[i];
    store_from_float(yr, i, dtype, v);
  }
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
// FFT
// ============================================================================
// Two layouts of the same Stockham algorithm:
//  * ping-pong (N <= kFftPingPongMax): two row buffers; every butterfly reads
//    from one and writes the other, so a thread handles one butterfly at a
//    time and register pressure stays low;
//  * in place (kFftPingPongMax < N <= kFftMaxN, radices <= 16 only): one
//    buffer; each thread holds at most kFftIpE values across the stage barrier.
constexpr int kFftMaxN = 16384;
constexpr int kFftPingPongMax = 12288;
constexpr int kFftIpE = 16;
constexpr int kMaxStages = 16;

struct FftPlan {
  int N;
  int nst;
  int radix[kMaxStages];
  int threads;
  int pingpong;
};

__device__ __forceinline__ int cpad(int i) { return i + (i >> 4); }

__device__ __forceinline__ float2 cmul(float2 a, float2 b) {
  return make_float2(a.x * b.x - a.y * b.y, a.x * b.y + a.y * b.x);
}
__device__ __forceinline__ float2 cadd(float2 a, float2 b) { return make_float2(a.x + b.x, a.y + b.y); }
__device__ __forceinline__ float2 csub(float2 a, float2 b) { return make_float2(a.x - b.x, a.y - b.y); }

// exp(-+2*pi*i*num/den): forward uses the negative exponent.
__device__ __forceinline__ float2 twiddle(int num, int den, bool inverse) {
  float s, c;
  sincospif(2.0f * static_cast<float>(num) / static_cast<float>(den), &s, &c);
  return make_float2(c, inverse ? s : -s);
}

// cos/sin(2*pi*k/16), k < 16, for the power-of-two butterflies.
__device__ __forceinline__ float2 tw16(int k, bool inverse) {
  constexpr float c[16] = {1.0f, 0.92387953251128674f, 0.70710678118654752f, 0.38268343236508977f,
                           0.0f, -0.38268343236508977f, -0.70710678118654752f, -0.92387953251128674f,
                           -1.0f, -0.92387953251128674f, -0.70710678118654752f, -0.38268343236508977f,
                           0.0f, 0.38268343236508977f, 0.70710678118654752f, 0.92387953251128674f};
  const float cs = c[k & 15];
  const float sn = c[(k + 12) & 15];  // sin(2*pi*k/16) = cos(2*pi*(k-4)/16)
  return make_float2(cs, inverse ? sn : -sn);
}

// In-register DFT of R = 2^k points (natural order in and out), radix-2 DIT.
template <int R>
__device__ __forceinline__ void dft_pow2(float2 (&v)[R], bool inverse) {
#pragma unroll
  for (int i = 0; i < R; ++i) {
    int j = 0;
#pragma unroll
    for (int b = 1, t = i; b < R; b <<= 1, t >>= 1) j = (j << 1) | (t & 1);
    if (i < j) {
      float2 tmp = v[i];
      v[i] = v[j];
      v[j] = tmp;
    }
  }
#pragma unroll
  for (int len = 2; len <= R; len <<= 1) {
    const int half = len / 2;
#pragma unroll
    for (int i = 0; i < R; i += len) {
#pragma unroll
      for (int k = 0; k < half; ++k) {
        const float2 w = tw16(k * (16 / len), inverse);
        const float2 u = v[i + k];
        const float2 t = k == 0 ? v[i + k + half] : cmul(w, v[i + k + half]);
        v[i + k] = cadd(u, t);
        v[i + k + half] = csub(u, t);
      }
    }
  }
}

// In-register DFT of an odd prime number R of points, using the conjugate-pair
// symmetry X_k, X_{R-k} = A_k -+ i B_k with A_k = x0 + sum_j (x_j + x_{R-j}) cos,
// B_k = sum_j (x_j - x_{R-j}) sin.
template <int R>
__device__ __forceinline__ void dft_odd(float2 (&v)[R], bool inverse) {
  constexpr int H = (R - 1) / 2;
  constexpr int off = prime_offset(R);
  float2 a[H], b[H];
#pragma unroll
  for (int j = 1; j <= H; ++j) {
    a[j - 1] = cadd(v[j], v[R - j]);
    b[j - 1] = csub(v[j], v[R - j]);
  }
  float2 out[R];
  float2 s0 = v[0];
#pragma unroll
  for (int j = 0; j < H; ++j) s0 = cadd(s0, a[j]);
  out[0] = s0;
#pragma unroll
  for (int k = 1; k <= H; ++k) {
    float2 A = v[0], B = make_float2(0.f, 0.f);
#pragma unroll
    for (int j = 1; j <= H; ++j) {
      const float c = kDftCos[off + (j * k) % R];
      const float s = kDftSin[off + (j * k) % R];
      A.x = fmaf(a[j - 1].x, c, A.x);
      A.y = fmaf(a[j - 1].y, c, A.y);
      B.x = fmaf(b[j - 1].x, s, B.x);
      B.y = fmaf(b[j - 1].y, s, B.y);
    }
    // forward: X_k = A - iB, X_{R-k} = A + iB   (-iB = (B.y, -B.x))
    const float2 miB = make_float2(B.y, -B.x);
    out[k] = inverse ? csub(A, miB) : cadd(A, miB);
    out[R - k] = inverse ? cadd(A, miB) : csub(A, miB);
  }
#pragma unroll
  for (int i = 0; i < R; ++i) v[i] = out[i];
}

template <int R>
__device__ __forceinline__ void dft_small(float2 (&v)[R], bool inverse) {
  if constexpr ((R & (R - 1)) == 0) dft_pow2<R>(v, inverse);
  else dft_odd<R>(v, inverse);
}

// Stockham butterfly j of radix R with Ns = product of the previous radices:
// reads in[j + r*N/R], twiddles by W_{Ns*R}^{r*(j mod Ns)}, DFT, writes
// out[(j - j mod Ns)*R + j mod Ns + r*Ns].
template <int R>
__device__ __forceinline__ void butterfly_load(const float2 *in, int nb, int Ns, int j,
                                               bool inverse, float2 (&v)[R]) {
#pragma unroll
  for (int r = 0; r < R; ++r) v[r] = in[cpad(j + r * nb)];
  if (Ns > 1) {
    const int k = j % Ns;
#pragma unroll
    for (int r = 1; r < R; ++r) v[r] = cmul(v[r], twiddle(r * k, Ns * R, inverse));
  }
  dft_small<R>(v, inverse);
}

template <int R>
__device__ __forceinline__ void butterfly_store(float2 *out, int Ns, int j, const float2 (&v)[R]) {
  const int k = j % Ns;
  const int base = (j - k) * R + k;
#pragma unroll
  for (int r = 0; r < R; ++r) out[cpad(base + r * Ns)] = v[r];
}

template <int R>
__device__ __forceinline__ void fft_stage_pp(const float2 *in, float2 *out, int N, int Ns, bool inverse) {
  const int nb = N / R;
  for (int j = threadIdx.x; j < nb; j += blockDim.x) {
    float2 v[R];
    butterfly_load<R>(in, nb, Ns, j, inverse, v);
    butterfly_store<R>(out, Ns, j, v);
  }
}

template <int R>
__device__ __forceinline__ void fft_stage_ip(float2 *buf, int N, int Ns, bool inverse) {
  constexpr int J = (kFftIpE + R - 1) / R;
  const int nb = N / R;
  float2 v[J][R];
#pragma unroll
  for (int jj = 0; jj < J; ++jj) {
    const int j = threadIdx.x + jj * blockDim.x;
    if (j < nb) butterfly_load<R>(buf, nb, Ns, j, inverse, v[jj]);
  }
  __syncthreads();
#pragma unroll
  for (int jj = 0; jj < J; ++jj) {
    const int j = threadIdx.x + jj * blockDim.x;
    if (j < nb) butterfly_store<R>(buf, Ns, j, v[jj]);
  }
}

// First stage for an odd prime P >= 11 (Ns = 1, no twiddles), ping-pong only.
// The conjugate-pair outputs of each of the N/P sequences are split into 4
// groups so several threads share one sequence; each thread reads the P
// inputs once and writes its outputs straight to the other buffer.
__host__ __device__ constexpr int prime_per(int P) { return ((P - 1) / 2 + 3) / 4; }

template <int P, int G>
__device__ __forceinline__ void prime_group(const float2 *in, float2 *out, int nb, int j,
                                            bool inverse) {
  constexpr int H = (P - 1) / 2;
  constexpr int per = prime_per(P);
  constexpr int off = prime_offset(P);
  constexpr int klo = G * per + 1;
  constexpr int khi = (G + 1) * per < H ? (G + 1) * per : H;
  const float2 x0 = in[cpad(j)];
  float2 A[per], B[per];
#pragma unroll
  for (int q = 0; q < per; ++q) {
    A[q] = x0;
    B[q] = make_float2(0.f, 0.f);
  }
  float2 s0 = x0;
#pragma unroll
  for (int r = 1; r <= H; ++r) {
    const float2 xa = in[cpad(j + r * nb)], xb = in[cpad(j + (P - r) * nb)];
    const float2 a = cadd(xa, xb), b = csub(xa, xb);
    if (G == 0) s0 = cadd(s0, a);
#pragma unroll
    for (int q = 0; q < per; ++q) {
      const int k = klo + q;
      if (k <= khi) {
        const float c = kDftCos[off + (r * k) % P];
        const float s = kDftSin[off + (r * k) % P];
        A[q].x = fmaf(a.x, c, A[q].x);
        A[q].y = fmaf(a.y, c, A[q].y);
        B[q].x = fmaf(b.x, s, B[q].x);
        B[q].y = fmaf(b.y, s, B[q].y);
      }
    }
  }
  // Stockham output with Ns = 1: X_k of sequence j goes to j*P + k.
#pragma unroll
  for (int q = 0; q < per; ++q) {
    const int k = klo + q;
    if (k <= khi) {
      const float2 miB = make_float2(B[q].y, -B[q].x);
      out[cpad(j * P + k)] = inverse ? csub(A[q], miB) : cadd(A[q], miB);
      out[cpad(j * P + P - k)] = inverse ? cadd(A[q], miB) : csub(A[q], miB);
    }
  }
  if (G == 0) out[cpad(j * P)] = s0;
}

template <int P>
__device__ __forceinline__ void fft_prime_pp(const float2 *in, float2 *out, int N, bool inverse) {
  const int nb = N / P;
  for (int t = threadIdx.x; t < 4 * nb; t += blockDim.x) {
    const int g = t / nb, j = t % nb;
    switch (g) {
      case 0: prime_group<P, 0>(in, out, nb, j, inverse); break;
      case 1: prime_group<P, 1>(in, out, nb, j, inverse); break;
      case 2: prime_group<P, 2>(in, out, nb, j, inverse); break;
      default: prime_group<P, 3>(in, out, nb, j, inverse); break;
    }
  }
}

// Unnormalised DFT (forward: exp(-2*pi*i*jk/N), inverse: exp(+...)) of
// buf0[cpad(0..N-1)]; returns the buffer holding the result (buf0 or buf1).
template <bool PP>
__device__ __forceinline__ float2 *fft_smem(float2 *buf0, float2 *buf1, const FftPlan &p,
                                            bool inverse) {
  int Ns = 1;
  float2 *src = buf0, *dst = buf1;
  for (int s = 0; s < p.nst; ++s) {
    const int R = p.radix[s];
    if constexpr (PP) {
      switch (R) {
        case 2: fft_stage_pp<2>(src, dst, p.N, Ns, inverse); break;
        case 3: fft_stage_pp<3>(src, dst, p.N, Ns, inverse); break;
        case 4: fft_stage_pp<4>(src, dst, p.N, Ns, inverse); break;
        case 5: fft_stage_pp<5>(src, dst, p.N, Ns, inverse); break;
        case 7: fft_stage_pp<7>(src, dst, p.N, Ns, inverse); break;
        case 8: fft_stage_pp<8>(src, dst, p.N, Ns, inverse); break;
        case 16: fft_stage_pp<16>(src, dst, p.N, Ns, inverse); break;
        case 11: fft_prime_pp<11>(src, dst, p.N, inverse); break;
        case 13: fft_prime_pp<13>(src, dst, p.N, inverse); break;
        case 17: fft_prime_pp<17>(src, dst, p.N, inverse); break;
        case 19: fft_prime_pp<19>(src, dst, p.N, inverse); break;
        case 23: fft_prime_pp<23>(src, dst, p.N, inverse); break;
        case 29: fft_prime_pp<29>(src, dst, p.N, inverse); break;
        case 31: fft_prime_pp<31>(src, dst, p.N, inverse); break;
        case 37: fft_prime_pp<37>(src, dst, p.N, inverse); break;
        case 41: fft_prime_pp<41>(src, dst, p.N, inverse); break;
        case 43: fft_prime_pp<43>(src, dst, p.N, inverse); break;
        default: break;  // rejected by make_plan
      }
      float2 *t = src;
      src = dst;
      dst = t;
    } else {
      switch (R) {
        case 2: fft_stage_ip<2>(src, p.N, Ns, inverse); break;
        case 3: fft_stage_ip<3>(src, p.N, Ns, inverse); break;
        case 4: fft_stage_ip<4>(src, p.N, Ns, inverse); break;
        case 5: fft_stage_ip<5>(src, p.N, Ns, inverse); break;
        case 7: fft_stage_ip<7>(src, p.N, Ns, inverse); break;
        case 8: fft_stage_ip<8>(src, p.N, Ns, inverse); break;
        case 16: fft_stage_ip<16>(src, p.N, Ns, inverse); break;
        default: break;  // rejected by make_plan
      }
    }
    __syncthreads();
    Ns *= R;
  }
  return src;
}

// Radix order: at most one prime >= 11 (first: Ns = 1 so it needs no
// twiddles), then 7/5/3, then 16/8/4/2.
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

__host__ __device__ __forceinline__ int fft_buf_elems(int N) { return N + (N >> 4) + 1; }
static size_t fft_smem_bytes(const FftPlan &p) {
  return (p.pingpong ? 2 : 1) * fft_buf_elems(p.N) * sizeof(float2);
}

template <bool PP>
__global__ void __launch_bounds__(PP ? 512 : 1024) rfft_rows_kernel(
    int inverse, const void *x, int64_t ld_x, void *y, int64_t ld_y, int dtype, FftPlan plan,
    const float2 *phase, float scale) {
  extern __shared__ float2 csm[];
  float2 *buf1 = csm + fft_buf_elems(plan.N);
  const int N = plan.N;
  const int64_t row = blockIdx.x;
  const int esz = dtype == QS_F32 ? 4 : 2;
  const void *xr = static_cast<const char *>(x) + row * ld_x * esz;
  for (int i = threadIdx.x; i < N; i += blockDim.x) {
    float2 z = make_float2(load_as_float(xr, 2 * i, dtype), load_as_float(xr, 2 * i + 1, dtype));
    if (!inverse) z = cmul(z, phase[i]);
    csm[cpad(i)] = z;
  }
  __syncthreads();
  const float2 *res = fft_smem<PP>(csm, buf1, plan, inverse != 0);
  void *yr = static_cast<char *>(y) + row * ld_y * esz;
  for (int i = threadIdx.x; i < N; i += blockDim.x) {
    float2 z = res[cpad(i)];
    z.x *= scale;
    z.y *= scale;
    if (inverse) {
      const float2 ph = phase[i];
      z = cmul(z, make_float2(ph.x, -ph.y));
    }
    store_from_float(yr, 2 * i, dtype, z.x);
    store_from_float(yr, 2 * i + 1, dtype, z.y);
  }
}

template <typename K>
static int set_smem(K kern, size_t bytes) {
  QS_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   static_cast<int>(bytes)));
  return QS_OK;
}

int launch_rfft(int inverse, const void *x, int64_t ld_x, void *y, int64_t ld_y, int dtype,
                int64_t rows, int64_t n, const void *phase, cudaStream_t s) {
  FftPlan p;
  int st = make_plan(n / 2, p);
  if (st) return st;
  const size_t smem = fft_smem_bytes(p);
  const float2 *ph = static_cast<const float2 *>(phase);
  if (p.pingpong) {
    if ((st = set_smem(rfft_rows_kernel<true>, smem))) return st;
    rfft_rows_kernel<true><<<rows, p.threads, smem, s>>>(inverse, x, ld_x, y, ld_y, dtype, p, ph,
                                                          inv_sqrt_f32(n / 2));
  } else {
    if ((st = set_smem(rfft_rows_kernel<false>, smem))) return st;
    rfft_rows_kernel<false><<<rows, p.threads, smem, s>>>(inverse, x, ld_x, y, ld_y, dtype, p, ph,
                                                           inv_sqrt_f32(n / 2));
  }
  return check_launch("rfft");
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

__device__ float block_absmax(float v, float *red) {
  v = fabsf(v);
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int w = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[w] = v;
  __syncthreads();
  float r = 0.f;
  for (int i = 0; i < nw; ++i) r = fmaxf(r, red[i]);
  return r;
}

__device__ __forceinline__ void pow2_scale(float amax, float &scale, float &inv) {
  if (!(amax > 0.f) || !isfinite(amax)) {
    scale = 1.f;
    inv = 1.f;
    return;
  }
  int e;
  frexpf(amax, &e);  // amax = f * 2^e, f in [0.5, 1)
  scale = ldexpf(1.f, 12 - e);
  inv = ldexpf(1.f, e - 12);
}

// Writes x2h for one row from values v(i) = smem value * post-scale, i < n.
template <typename GetV>
__device__ void write_x2h(GetV getv, int n, int n_pad, __half *x2h_row, float *rowscale_r,
                          float *red) {
  float amax = 0.f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) amax = fmaxf(amax, fabsf(getv(i)));
  amax = block_absmax(amax, red);
  float sc, inv;
  pow2_scale(amax, sc, inv);
  for (int i = threadIdx.x; i < n_pad; i += blockDim.x)
    x2h_row[i] = __float2half_rn(i < n ? getv(i) * sc : 0.f);
  if (threadIdx.x == 0) *rowscale_r = inv;
}

__global__ void __launch_bounds__(1024) linear_input_rht_kernel(
    const void *x, int dtype, int L, int E, const float *sv, float scale, __half *x2h,
    float *rowscale, int n_pad, float *y1, int64_t m_local) {
  extern __shared__ float fsm[];
  __shared__ float red[32];
  const int n = 1 << L;
  const int64_t row = blockIdx.x;
  for (int64_t i = threadIdx.x; i < m_local; i += blockDim.x) y1[row * m_local + i] = 0.f;
  for (int i = threadIdx.x; i < n; i += blockDim.x)
    fsm[fpad(i)] = load_as_float(x, row * n + i, dtype) * sv[i];
  __syncthreads();
  fwht_smem(fsm, L, E);
  write_x2h([&](int i) { return fsm[fpad(i)] * scale; }, n, n_pad, x2h + row * n_pad,
            rowscale + row, red);
}

template <bool PP>
__global__ void __launch_bounds__(PP ? 512 : 1024) linear_input_rfft_kernel(
    const void *x, int dtype, FftPlan plan, const float2 *phase, float scale, __half *x2h,
    float *rowscale, int n_pad, float *y1, int64_t m_local) {
  extern __shared__ float2 csm[];
  __shared__ float red[32];
  float2 *buf1 = csm + fft_buf_elems(plan.N);
  const int N = plan.N;
  const int64_t row = blockIdx.x;
  for (int64_t i = threadIdx.x; i < m_local; i += blockDim.x) y1[row * m_local + i] = 0.f;
  for (int i = threadIdx.x; i < N; i += blockDim.x) {
    const float2 z = make_float2(load_as_float(x, row * 2 * N + 2 * i, dtype),
                                 load_as_float(x, row * 2 * N + 2 * i + 1, dtype));
    csm[cpad(i)] = cmul(z, phase[i]);
  }
  __syncthreads();
  const float *f = reinterpret_cast<const float *>(fft_smem<PP>(csm, buf1, plan, false));
  write_x2h([&](int i) { return f[2 * cpad(i >> 1) + (i & 1)] * scale; }, 2 * N, n_pad,
            x2h + row * n_pad, rowscale + row, red);
}

int launch_linear_input(const void *x, int x_dtype, int64_t batch, int64_t n, int transform,
                        const float *sv, const void *phase_v, void *x2ws, float *y1,
                        int64_t m_local, cudaStream_t s) {
  const int64_t n_pad = n_padded(n);
  __half *x2h = static_cast<__half *>(x2ws);
  float *rowscale = reinterpret_cast<float *>(static_cast<char *>(x2ws) + round_up(batch * n_pad * 2, 256));
  if (!y1) m_local = 0;
  if (transform == QS_RHT) {
    FwhtGeom g = fwht_geom(n);
    QS_CUDA_TRY(cudaFuncSetAttribute(linear_input_rht_kernel,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     static_cast<int>(g.smem)));
    linear_input_rht_kernel<<<batch, g.threads, g.smem, s>>>(x, x_dtype, g.L, g.E, sv,
                                                            inv_sqrt_f32(n), x2h, rowscale,
                                                            static_cast<int>(n_pad), y1, m_local);
    return check_launch("linear_input_rht");
  }
  FftPlan p;
  int st = make_plan(n / 2, p);
  if (st) return st;
  const size_t smem = fft_smem_bytes(p);
  const float2 *ph = static_cast<const float2 *>(phase_v);
  if (p.pingpong) {
    if ((st = set_smem(linear_input_rfft_kernel<true>, smem))) return st;
    linear_input_rfft_kernel<true><<<batch, p.threads, smem, s>>>(
        x, x_dtype, p, ph, inv_sqrt_f32(n / 2), x2h, rowscale, static_cast<int>(n_pad), y1, m_local);
  } else {
    if ((st = set_smem(linear_input_rfft_kernel<false>, smem))) return st;
    linear_input_rfft_kernel<false><<<batch, p.threads, smem, s>>>(
        x, x_dtype, p, ph, inv_sqrt_f32(n / 2), x2h, rowscale, static_cast<int>(n_pad), y1, m_local);
  }
  return check_launch("linear_input_rfft");
}

// Offset of y1 element (row, col): plain row-major with stride ld_y1 when
// shards == 1, else the rank-major layout of an all-gather of `shards` column
// blocks of (batch, mp): ((col / mp) * batch + row) * mp + col % mp.
__device__ __forceinline__ int64_t y1_offset(int64_t row, int64_t col, int64_t ld_y1, int64_t shards,
                                             int64_t mp, int64_t batch) {
  if (shards == 1) return row * ld_y1 + col;
  return ((col / mp) * batch + row) * mp + col % mp;
}

__global__ void __launch_bounds__(1024) linear_output_rht_kernel(const float *y1, int64_t ld_y1,
                                                                 int64_t shards, int64_t batch,
                                                                 int L, int E, const float *su,
                                                                 const float *bias, float scale,
                                                                 void *y, int dtype) {
  extern __shared__ float fsm[];
  const int m = 1 << L;
  const int64_t mp = m / shards;
  const int64_t row = blockIdx.x;
  for (int i = threadIdx.x; i < m; i += blockDim.x) fsm[fpad(i)] = y1[y1_offset(row, i, ld_y1, shards, mp, batch)];
  __syncthreads();
  fwht_smem(fsm, L, E);
  for (int i = threadIdx.x; i < m; i += blockDim.x) {
    float v = fsm[fpad(i)] * scale * su[i];
    if (bias) v += bias[i];
    store_from_float(y, row * m + i, dtype, v);
  }
}

template <bool PP>
__global__ void __launch_bounds__(PP ? 512 : 1024) linear_output_rfft_kernel(
    const float *y1, int64_t ld_y1, int64_t shards, int64_t batch, FftPlan plan, const float2 *phase,
    const float *bias, float scale, void *y, int dtype) {
  extern __shared__ float2 csm[];
  float2 *buf1 = csm + fft_buf_elems(plan.N);
  const int N = plan.N;
  const int64_t mp = 2 * N / shards;
  const int64_t row = blockIdx.x;
  for (int i = threadIdx.x; i < N; i += blockDim.x)
    csm[cpad(i)] = *reinterpret_cast<const float2 *>(y1 + y1_offset(row, 2 * i, ld_y1, shards, mp, batch));
  __syncthreads();
  const float2 *res = fft_smem<PP>(csm, buf1, plan, true);
  for (int i = threadIdx.x; i < N; i += blockDim.x) {
    float2 z = res[cpad(i)];
    z.x *= scale;
    z.y *= scale;
    const float2 ph = phase[i];
    z = cmul(z, make_float2(ph.x, -ph.y));
    if (bias) {
      z.x += bias[2 * i];
      z.y += bias[2 * i + 1];
    }
    store_from_float(y, row * 2 * N + 2 * i, dtype, z.x);
    store_from_float(y, row * 2 * N + 2 * i + 1, dtype, z.y);
  }
}

int launch_linear_output(const float *y1, int64_t ld_y1, int64_t shards, int64_t batch, int64_t m,
                         int transform, const float *su, const void *phase_u, const float *bias,
                         void *y, int y_dtype, cudaStream_t s) {
  if (transform == QS_RHT) {
    FwhtGeom g = fwht_geom(m);
    QS_CUDA_TRY(cudaFuncSetAttribute(linear_output_rht_kernel,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     static_cast<int>(g.smem)));
    linear_output_rht_kernel<<<batch, g.threads, g.smem, s>>>(y1, ld_y1, shards, batch, g.L, g.E, su,
                                                             bias, inv_sqrt_f32(m), y, y_dtype);
    return check_launch("linear_output_rht");
  }
  if (ld_y1 % 2) return fail(QS_ERR_ALIGNMENT, "RFFT y1 row stride must be even");
  FftPlan p;
  int st = make_plan(m / 2, p);
  if (st) return st;
  const size_t smem = fft_smem_bytes(p);
  const float2 *ph = static_cast<const float2 *>(phase_u);
  if (p.pingpong) {
    if ((st = set_smem(linear_output_rfft_kernel<true>, smem))) return st;
    linear_output_rfft_kernel<true><<<batch, p.threads, smem, s>>>(y1, ld_y1, shards, batch, p, ph,
                                                                   bias, inv_sqrt_f32(m / 2), y, y_dtype);
  } else {
    if ((st = set_smem(linear_output_rfft_kernel<false>, smem))) return st;
    linear_output_rfft_kernel<false><<<batch, p.threads, smem, s>>>(y1, ld_y1, shards, batch, p, ph,
                                                                    bias, inv_sqrt_f32(m / 2), y, y_dtype);
  }
  return check_launch("linear_output_rfft");
}

}  // namespace qs
