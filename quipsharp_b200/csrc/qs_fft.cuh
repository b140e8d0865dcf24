// Mixed-radix shared-memory FFT (device code and kernel templates) shared by
// qs_transform.cu (plans, dispatch) and the qs_fft_*.cu instantiation units.
#pragma once

#include "qs_common.cuh"
#include "qs_launch.h"

namespace qs {

__device__ __forceinline__ float block_absmax(float v, float *red) {
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

// Writes x2h / rowscale of one row from the transform result held in
// shared memory (value(i), i < n) and the thread-local |max| seen while it
// was produced.
template <typename Val>
__device__ __forceinline__ void emit_x2h(Val value, float local_amax, int n, int n_pad, __half *x2h_row,
                                         float *rowscale_r, float *red) {
  const float amax = block_absmax(local_amax, red);
  float sc, inv;
  pow2_scale(amax, sc, inv);
  for (int i = threadIdx.x; i < n_pad; i += blockDim.x)
    x2h_row[i] = __float2half_rn(i < n ? value(i) * sc : 0.f);
  if (threadIdx.x == 0) *rowscale_r = inv;
}

// ============================================================================
// FFT
// ============================================================================
// Mixed-radix Stockham FFT of one row (N complex points) per CTA, written for
// small code: with few rows (decode batch) one CTA runs the program once, so
// the kernel must not be a long unrolled instruction stream.
//  * Stage order: at most one prime >= 11 (the "big" prime), then 7/5/3, then
//    16/8/4/2.  Each radix is instantiated once (shared -> shared).
//  * The row is loaded into shared memory by a separate pass (cast, phase
//    multiply) and stored by another (scale, conjugate phase, bias, cast).
//  * Twiddles W_N^e come from two shared tables built at kernel start:
//    W_N^e = C[e >> 7] * F[e & 127] with F[j] = W_N^j (j < 128) and
//    C[j] = W_N^(128 j) (j < N/128): two loads and one complex product each.
//  * Ping-pong buffers (N <= kFftPingPongMax): each butterfly reads one buffer
//    and writes the other.  Larger rows (N <= kFftMaxN, radices <= 16 only) run
//    in place with at most kFftIpE values per thread held across the barrier.
constexpr int kFftMaxN = 16384;
constexpr int kFftPingPongMax = 12288;
constexpr int kFftIpE = 16;
constexpr int kMaxStages = 16;
constexpr int kTwFine = 128;
constexpr int kTwCoarseMax = kFftMaxN / kTwFine;

struct FftPlan {
  int N;
  int nst;
  int radix[kMaxStages];
  int threads;
  int pingpong;
  int big;  // prime >= 11 dividing N, or 0
};

__device__ __forceinline__ int cpad(int i) { return i + (i >> 4); }
__host__ __device__ __forceinline__ int fft_buf_elems(int N) { return N + (N >> 4) + 1; }

__device__ __forceinline__ float2 cmul(float2 a, float2 b) {
  return make_float2(a.x * b.x - a.y * b.y, a.x * b.y + a.y * b.x);
}
__device__ __forceinline__ float2 cadd(float2 a, float2 b) { return make_float2(a.x + b.x, a.y + b.y); }
__device__ __forceinline__ float2 csub(float2 a, float2 b) { return make_float2(a.x - b.x, a.y - b.y); }
__device__ __forceinline__ float2 conjf2(float2 a) { return make_float2(a.x, -a.y); }

// Runs body(i) for i = threadIdx.x + k*blockDim.x < n in batches of U with
// all U loads of a batch issued before their results are used: load(i)
// produces a value, use(i, value) consumes it.  Keeps several global loads in
// flight per thread instead of one L2 round trip per element.
template <int U, typename T, typename Load, typename Use>
__device__ __forceinline__ void batched_rows(int n, Load load, Use use) {
  for (int base = threadIdx.x; base < n; base += U * blockDim.x) {
    T v[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int i = base + u * blockDim.x;
      if (i < n) v[u] = load(i);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int i = base + u * blockDim.x;
      if (i < n) use(i, v[u]);
    }
  }
}

// Shared twiddle tables of the forward transform (the inverse conjugates).
struct Twiddles {
  float2 fine[kTwFine];
  float2 coarse[kTwCoarseMax];
};

__device__ __forceinline__ void build_twiddles(Twiddles &tw, int N) {
  const int nc = (N + kTwFine - 1) / kTwFine;
  for (int j = threadIdx.x; j < kTwFine + nc; j += blockDim.x) {
    const int e = j < kTwFine ? j : (j - kTwFine) * kTwFine;
    float s, c;
    sincospif(2.0f * static_cast<float>(e % N) / static_cast<float>(N), &s, &c);
    if (j < kTwFine) tw.fine[j] = make_float2(c, -s);
    else tw.coarse[j - kTwFine] = make_float2(c, -s);
  }
}

// W_N^e (forward) or its conjugate (inverse), 0 <= e < N.
__device__ __forceinline__ float2 tw_lookup(const Twiddles &tw, int e, bool inverse) {
  const float2 w = cmul(tw.coarse[e >> 7], tw.fine[e & (kTwFine - 1)]);
  return inverse ? conjf2(w) : w;
}

// cos(2*pi*k/16) for the power-of-two butterflies (k is a compile-time constant).
__host__ __device__ constexpr float cos16(int k) {
  return (k & 15) == 0 ? 1.0f : (k & 15) == 1 ? 0.92387953251128674f : (k & 15) == 2 ? 0.70710678118654752f
       : (k & 15) == 3 ? 0.38268343236508977f : (k & 15) == 4 ? 0.0f : (k & 15) == 5 ? -0.38268343236508977f
       : (k & 15) == 6 ? -0.70710678118654752f : (k & 15) == 7 ? -0.92387953251128674f : (k & 15) == 8 ? -1.0f
       : (k & 15) == 9 ? -0.92387953251128674f : (k & 15) == 10 ? -0.70710678118654752f
       : (k & 15) == 11 ? -0.38268343236508977f : (k & 15) == 12 ? 0.0f : (k & 15) == 13 ? 0.38268343236508977f
       : (k & 15) == 14 ? 0.70710678118654752f : 0.92387953251128674f;
}

template <int K>
__device__ __forceinline__ float2 tw16(bool inverse) {
  constexpr float cs = cos16(K), sn = cos16(K + 12);  // sin(2*pi*k/16) = cos(2*pi*(k-4)/16)
  return make_float2(cs, inverse ? sn : -sn);
}

template <int R, int LEN, int K>
__device__ __forceinline__ void pow2_butterflies(float2 (&v)[R], bool inverse) {
  if constexpr (K < LEN / 2) {
#pragma unroll
    for (int i = 0; i < R; i += LEN) {
      const float2 u = v[i + K];
      const float2 t = K == 0 ? v[i + K + LEN / 2] : cmul(tw16<K * (16 / LEN)>(inverse), v[i + K + LEN / 2]);
      v[i + K] = cadd(u, t);
      v[i + K + LEN / 2] = csub(u, t);
    }
    pow2_butterflies<R, LEN, K + 1>(v, inverse);
  }
}

template <int R, int LEN>
__device__ __forceinline__ void pow2_levels(float2 (&v)[R], bool inverse) {
  if constexpr (LEN <= R) {
    pow2_butterflies<R, LEN, 0>(v, inverse);
    pow2_levels<R, LEN * 2>(v, inverse);
  }
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
  pow2_levels<R, 2>(v, inverse);
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
  float2 s0 = v[0];
#pragma unroll
  for (int j = 0; j < H; ++j) s0 = cadd(s0, a[j]);
  const float2 x0 = v[0];
  v[0] = s0;
#pragma unroll
  for (int k = 1; k <= H; ++k) {
    float2 A = x0, B = make_float2(0.f, 0.f);
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
    v[k] = inverse ? csub(A, miB) : cadd(A, miB);
    v[R - k] = inverse ? cadd(A, miB) : csub(A, miB);
  }
}

template <int R>
__device__ __forceinline__ void dft_small(float2 (&v)[R], bool inverse) {
  if constexpr ((R & (R - 1)) == 0) dft_pow2<R>(v, inverse);
  else dft_odd<R>(v, inverse);
}

// Butterfly j of a Stockham stage of radix R with Ns = product of the previous
// radices: reads in[j + r*N/R], twiddles by W_{Ns*R}^{r*(j mod Ns)} = W_N^{r*k*N/(Ns*R)},
// DFT, writes out[(j - j mod Ns)*R + j mod Ns + r*Ns].
template <int R>
__device__ __forceinline__ void butterfly_load(const float2 *in, const Twiddles &tw, int N, int nb, int Ns,
                                               int j, bool inverse, float2 (&v)[R]) {
#pragma unroll
  for (int r = 0; r < R; ++r) v[r] = in[cpad(j + r * nb)];
  if (Ns > 1) {
    const int step = (j % Ns) * (N / (Ns * R));
    int e = step;
#pragma unroll
    for (int r = 1; r < R; ++r) {
      v[r] = cmul(v[r], tw_lookup(tw, e, inverse));
      e += step;
    }
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
__device__ __noinline__ void stage_pp(const float2 *in, float2 *out, const Twiddles &tw, int N, int Ns,
                                      bool inverse) {
  const int nb = N / R;
  for (int j = threadIdx.x; j < nb; j += blockDim.x) {
    float2 v[R];
    butterfly_load<R>(in, tw, N, nb, Ns, j, inverse, v);
    butterfly_store<R>(out, Ns, j, v);
  }
}

template <int R>
__device__ __noinline__ void stage_ip(float2 *buf, const Twiddles &tw, int N, int Ns, bool inverse) {
  constexpr int J = (kFftIpE + R - 1) / R;
  const int nb = N / R;
  float2 v[J][R];
#pragma unroll
  for (int jj = 0; jj < J; ++jj) {
    const int j = threadIdx.x + jj * blockDim.x;
    if (j < nb) butterfly_load<R>(buf, tw, N, nb, Ns, j, inverse, v[jj]);
  }
  __syncthreads();
#pragma unroll
  for (int jj = 0; jj < J; ++jj) {
    const int j = threadIdx.x + jj * blockDim.x;
    if (j < nb) butterfly_store<R>(buf, Ns, j, v[jj]);
  }
}

// Big-prime first stage (Ns = 1, no twiddles), ping-pong only.  The
// (P-1)/2 conjugate-pair outputs of each of the N/P sequences are split into 4
// groups of kPrimePer pairs; each thread takes one (group, sequence), reads
// the P inputs once (loop, not unrolled), and keeps kPrimePer accumulator
// pairs.  Threads of a warp share the group (N/P is a multiple of 32 for the
// layer shapes), so the cos/sin reads are warp-uniform constant-cache hits.
constexpr int kPrimePer = 6;  // ceil(21 / 4) for P = 43, the largest prime handled

template <int P>
__device__ __noinline__ void prime_stage(const float2 *in, float2 *out, int N, bool inverse) {
  constexpr int H = (P - 1) / 2;
  constexpr int per = (H + 3) / 4;
  static_assert(per <= kPrimePer, "prime too large");
  constexpr int off = prime_offset(P);
  const int nb = N / P;
  for (int t = threadIdx.x; t < 4 * nb; t += blockDim.x) {
    const int g = t / nb, j = t % nb;
    const int klo = g * per + 1;
    const float2 x0 = in[cpad(j)];
    float2 A[per], B[per];
    int idx[per];
#pragma unroll
    for (int q = 0; q < per; ++q) {
      A[q] = x0;
      B[q] = make_float2(0.f, 0.f);
      idx[q] = 0;
    }
    float2 s0 = x0;
#pragma unroll 1
    for (int r = 1; r <= H; ++r) {
      const float2 xa = in[cpad(j + r * nb)], xb = in[cpad(j + (P - r) * nb)];
      const float2 a = cadd(xa, xb), b = csub(xa, xb);
      s0 = cadd(s0, a);
#pragma unroll
      for (int q = 0; q < per; ++q) {
        idx[q] += klo + q;  // (r * k) mod P, kept incrementally
        if (idx[q] >= P) idx[q] -= P;
        const float c = kDftCos[off + idx[q]];
        const float s = kDftSin[off + idx[q]];
        A[q].x = fmaf(a.x, c, A[q].x);
        A[q].y = fmaf(a.y, c, A[q].y);
        B[q].x = fmaf(b.x, s, B[q].x);
        B[q].y = fmaf(b.y, s, B[q].y);
      }
    }
#pragma unroll
    for (int q = 0; q < per; ++q) {
      const int k = klo + q;
      if (k <= H) {
        const float2 miB = make_float2(B[q].y, -B[q].x);
        out[cpad(j * P + k)] = inverse ? csub(A[q], miB) : cadd(A[q], miB);
        out[cpad(j * P + P - k)] = inverse ? cadd(A[q], miB) : csub(A[q], miB);
      }
    }
    if (g == 0) out[cpad(j * P)] = s0;
  }
}

template <bool PP>
__device__ __forceinline__ void small_stage(int R, float2 *src, float2 *dst, const Twiddles &tw, int N, int Ns,
                                            bool inverse) {
  switch (R) {
#define QS_STAGE(RR) \
  case RR: if constexpr (PP) stage_pp<RR>(src, dst, tw, N, Ns, inverse); else stage_ip<RR>(src, tw, N, Ns, inverse); break;
    QS_STAGE(2) QS_STAGE(3) QS_STAGE(4) QS_STAGE(5) QS_STAGE(7) QS_STAGE(8) QS_STAGE(16)
#undef QS_STAGE
    default: break;  // rejected by make_plan
  }
}

// Unnormalised DFT (forward: exp(-2*pi*i*jk/N), inverse: exp(+...)) of the row
// in buf0[cpad(.)]; returns the buffer holding the result.  Ends with a barrier.
// The caller builds the twiddle tables (build_twiddles) before the barrier
// that precedes this call.
template <bool PP, int BIG>
__device__ __forceinline__ float2 *fft_row(float2 *buf0, float2 *buf1, Twiddles &tw, const FftPlan &p,
                                           bool inverse) {
  float2 *src = buf0, *dst = buf1;
  int Ns = 1;
  for (int s = 0; s < p.nst; ++s) {
    const int R = p.radix[s];
    if (R == 1) break;  // N == 1
    if constexpr (BIG != 0) {
      if (s == 0) prime_stage<BIG>(src, dst, p.N, inverse);
      else small_stage<PP>(R, src, dst, tw, p.N, Ns, inverse);
    } else {
      small_stage<PP>(R, src, dst, tw, p.N, Ns, inverse);
    }
    __syncthreads();
    if constexpr (PP) {
      float2 *t = src;
      src = dst;
      dst = t;
    }
    Ns *= R;
  }
  return src;
}

template <bool PP, int BIG>
__global__ void __launch_bounds__(PP ? 512 : 1024) rfft_rows_kernel(
    int inverse, const void *x, int64_t ld_x, void *y, int64_t ld_y, int dtype, FftPlan plan,
    const float2 *phase, float scale) {
  extern __shared__ float2 csm[];
  __shared__ Twiddles tw;
  float2 *buf1 = csm + fft_buf_elems(plan.N);
  const int N = plan.N;
  const int64_t row = blockIdx.x;
  const int esz = dtype == QS_F32 ? 4 : 2;
  const void *xr = static_cast<const char *>(x) + row * ld_x * esz;
  void *yr = static_cast<char *>(y) + row * ld_y * esz;
  build_twiddles(tw, N);
  batched_rows<8, float4>(N, [&](int i) {
    return make_float4(load_as_float(xr, 2 * i, dtype), load_as_float(xr, 2 * i + 1, dtype),
                       inverse ? 1.f : phase[i].x, inverse ? 0.f : phase[i].y);
  }, [&](int i, float4 v) { csm[cpad(i)] = cmul(make_float2(v.x, v.y), make_float2(v.z, v.w)); });
  __syncthreads();
  const float2 *res = fft_row<PP, BIG>(csm, buf1, tw, plan, inverse != 0);
  batched_rows<8, float2>(N, [&](int i) { return inverse ? conjf2(phase[i]) : make_float2(1.f, 0.f); },
                          [&](int i, float2 ph) {
    float2 z = res[cpad(i)];
    z.x *= scale;
    z.y *= scale;
    z = cmul(z, ph);
    store_from_float(yr, 2 * i, dtype, z.x);
    store_from_float(yr, 2 * i + 1, dtype, z.y);
  });
}

template <bool PP, int BIG>
__global__ void __launch_bounds__(PP ? 512 : 1024) linear_input_rfft_kernel(
    const void *x, int dtype, FftPlan plan, const float2 *phase, float scale, __half *x2h,
    float *rowscale, int n_pad, float *y1, int64_t m_local, int resbuf) {
  extern __shared__ float2 csm[];
  __shared__ Twiddles tw;
  __shared__ float red[32];
  float2 *buf1 = csm + fft_buf_elems(plan.N);
  const int N = plan.N;
  const int64_t row = blockIdx.x;
  pdl_launch_dependents();
  build_twiddles(tw, N);
  pdl_wait();  // x may be the previous kernel's output; y1 may still be read by it
  for (int64_t i = threadIdx.x; i < m_local; i += blockDim.x) y1[row * m_local + i] = 0.f;
  if (dtype == QS_F16 || dtype == QS_BF16) {
    const uint32_t *xr = reinterpret_cast<const uint32_t *>(static_cast<const char *>(x) + row * 4 * N);
    const bool f16 = dtype == QS_F16;
    batched_rows<8, float4>(N, [&](int i) {
      const uint32_t w = xr[i];
      const float2 z = f16 ? __half22float2(*reinterpret_cast<const __half2 *>(&w))
                           : __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&w));
      const float2 ph = phase[i];
      return make_float4(z.x, z.y, ph.x, ph.y);
    }, [&](int i, float4 v) { csm[cpad(i)] = cmul(make_float2(v.x, v.y), make_float2(v.z, v.w)); });
  } else {
    const float2 *xr = reinterpret_cast<const float2 *>(static_cast<const char *>(x) + row * 8 * N);
    batched_rows<8, float4>(N, [&](int i) {
      const float2 z = xr[i], ph = phase[i];
      return make_float4(z.x, z.y, ph.x, ph.y);
    }, [&](int i, float4 v) { csm[cpad(i)] = cmul(make_float2(v.x, v.y), make_float2(v.z, v.w)); });
  }
  __syncthreads();
  const float2 *res = fft_row<PP, BIG>(csm, buf1, tw, plan, false);
  float amax = 0.f;
  for (int i = threadIdx.x; i < N; i += blockDim.x) {
    const float2 z = res[cpad(i)];
    amax = fmaxf(amax, fmaxf(fabsf(z.x), fabsf(z.y)));
  }
  const float *f = reinterpret_cast<const float *>(res);
  emit_x2h([&](int i) { return f[2 * cpad(i >> 1) + (i & 1)] * scale; }, amax * scale, 2 * N, n_pad,
           x2h + row * n_pad, rowscale + row, red);
}

// Offset of y1 element (row, col): plain row-major with stride ld_y1 when
// shards == 1, else the rank-major layout of an all-gather of `shards` column
// blocks of (batch, mp): ((col / mp) * batch + row) * mp + col % mp.
__device__ __forceinline__ int64_t y1_offset(int64_t row, int64_t col, int64_t ld_y1, int64_t shards,
                                             int64_t mp, int64_t batch) {
  if (shards == 1) return row * ld_y1 + col;
  return ((col / mp) * batch + row) * mp + col % mp;
}

template <bool PP, int BIG>
__global__ void __launch_bounds__(PP ? 512 : 1024) linear_output_rfft_kernel(
    const float *y1, int64_t ld_y1, int64_t shards, int64_t batch, FftPlan plan, const float2 *phase,
    const float *bias, float scale, void *y, int dtype) {
  extern __shared__ float2 csm[];
  __shared__ Twiddles tw;
  float2 *buf1 = csm + fft_buf_elems(plan.N);
  const int N = plan.N;
  const int64_t mp = 2 * N / shards;
  const int64_t row = blockIdx.x;
  pdl_launch_dependents();
  build_twiddles(tw, N);
  pdl_wait();  // y1 comes from the matmul (or the all-gather)
  batched_rows<8, float2>(N, [&](int i) {
    return *reinterpret_cast<const float2 *>(y1 + y1_offset(row, 2 * i, ld_y1, shards, mp, batch));
  }, [&](int i, float2 v) { csm[cpad(i)] = v; });
  __syncthreads();
  const float2 *res = fft_row<PP, BIG>(csm, buf1, tw, plan, true);
  batched_rows<8, float4>(N, [&](int i) {
    const float2 ph = phase[i];
    const float2 bb = bias ? reinterpret_cast<const float2 *>(bias)[i] : make_float2(0.f, 0.f);
    return make_float4(ph.x, -ph.y, bb.x, bb.y);
  }, [&](int i, float4 pb) {
    float2 z = res[cpad(i)];
    z.x *= scale;
    z.y *= scale;
    z = cmul(z, make_float2(pb.x, pb.y));
    z.x += pb.z;
    z.y += pb.w;
    if (dtype == QS_F16) reinterpret_cast<__half2 *>(y)[row * N + i] = __floats2half2_rn(z.x, z.y);
    else if (dtype == QS_BF16) reinterpret_cast<__nv_bfloat162 *>(y)[row * N + i] = __floats2bfloat162_rn(z.x, z.y);
    else reinterpret_cast<float2 *>(y)[row * N + i] = z;
  });
}

// Host launchers of the FFT kernels for one big prime (explicitly instantiated
// in the qs_fft_*.cu units).
template <bool PP, int BIG>
int run_rfft_rows(int inverse, const void *x, int64_t ld_x, void *y, int64_t ld_y, int dtype, int64_t rows,
                  const FftPlan &p, const float2 *phase, float scale, size_t smem, cudaStream_t s);
template <bool PP, int BIG>
int run_linear_input_rfft(const void *x, int dtype, int64_t batch, const FftPlan &p, const float2 *phase,
                          float scale, __half *x2h, float *rowscale, int n_pad, float *y1, int64_t m_local,
                          int resbuf, size_t smem, cudaStream_t s);
template <bool PP, int BIG>
int run_linear_output_rfft(const float *y1, int64_t ld_y1, int64_t shards, int64_t batch, const FftPlan &p,
                           const float2 *phase, const float *bias, float scale, void *y, int dtype, size_t smem,
                           cudaStream_t s);

#define QS_FOR_EACH_BIG(X) X(0) X(11) X(13) X(17) X(19) X(23) X(29) X(31) X(37) X(41) X(43)

#define QS_DEFINE_FFT_RUNNERS(PP, BIG)                                                                    \
  template <>                                                                                             \
  int run_rfft_rows<PP, BIG>(int inverse, const void *x, int64_t ld_x, void *y, int64_t ld_y, int dtype,  \
                             int64_t rows, const FftPlan &p, const float2 *phase, float scale, size_t smem, \
                             cudaStream_t s) {                                                            \
    QS_CUDA_TRY(cudaFuncSetAttribute(rfft_rows_kernel<PP, BIG>,                                           \
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));            \
    rfft_rows_kernel<PP, BIG><<<rows, p.threads, smem, s>>>(inverse, x, ld_x, y, ld_y, dtype, p, phase, scale); \
    return check_launch("rfft");                                                                          \
  }                                                                                                       \
  template <>                                                                                             \
  int run_linear_input_rfft<PP, BIG>(const void *x, int dtype, int64_t batch, const FftPlan &p,           \
                                     const float2 *phase, float scale, __half *x2h, float *rowscale,      \
                                     int n_pad, float *y1, int64_t m_local, int resbuf, size_t smem,      \
                                     cudaStream_t s) {                                                    \
    QS_CUDA_TRY(cudaFuncSetAttribute(linear_input_rfft_kernel<PP, BIG>,                                   \
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));            \
    return launch_pdl("linear_input_rfft", linear_input_rfft_kernel<PP, BIG>, dim3(batch), dim3(p.threads), \
                      smem, s, x, dtype, p, phase, scale, x2h, rowscale, n_pad, y1, m_local, resbuf);       \
  }                                                                                                       \
  template <>                                                                                             \
  int run_linear_output_rfft<PP, BIG>(const float *y1, int64_t ld_y1, int64_t shards, int64_t batch,      \
                                      const FftPlan &p, const float2 *phase, const float *bias,           \
                                      float scale, void *y, int dtype, size_t smem, cudaStream_t s) {     \
    QS_CUDA_TRY(cudaFuncSetAttribute(linear_output_rfft_kernel<PP, BIG>,                                  \
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));            \
    return launch_pdl("linear_output_rfft", linear_output_rfft_kernel<PP, BIG>, dim3(batch),                \
                      dim3(p.threads), smem, s, y1, ld_y1, shards, batch, p, phase, bias, scale, y, dtype); \
  }

}  // namespace qs
