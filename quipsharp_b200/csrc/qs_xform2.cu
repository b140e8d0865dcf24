// Two-pass ("four-step") RFFT transforms of the quantized-linear input and
// output steps for many rows (prefill), N = P * N1 complex points with P an odd
// prime <= 43 and N1 = 2^a >= 64:
//
//   X[k + P*k1] = sum_{j1} W_N1^{j1 k1} [ W_N^{j1 k} sum_{j2} x[j1 + N1*j2] W_P^{j2 k} ]
//
// Pass A (xcol_kernel): one thread per (row, column j1) loads the P points
// x[j1 + N1*j2] (a warp reads 32 consecutive columns: coalesced), computes
// their P-point DFT in registers (conjugate pairs, compile-time cos / sin),
// multiplies by the twiddles W_N^{j1 k} and stores them to j1 + N1*k.  No
// shared memory, no barriers: a streaming kernel with many rows in flight.
// Pass B (xblk_kernel): one CTA per row runs the P contiguous N1-point FFTs
// (a warp per block for N1 <= 512, the whole CTA otherwise) with the stages of
// qs_xform.cuh, writes each result to its final position k + P*k1 of a
// shared-memory copy of the output row (sign / conjugate phase, bias, cast, or
// the fp16 matmul operand), and stores the row with coalesced 16-byte writes.
//
// Output step: pass A works in place on y1 (consumed).  Input step: pass A
// writes a float32 scratch after the x2 workspace and per-warp L1 sums of the
// phase-multiplied input; the row's power-of-two fp16 scale comes from the
// bound max|X| <= sum |x| (power-of-two scaling commutes with fp16 rounding, so
// the stored operand times its row scale is the same as with the exact max).
#include <cmath>

#include "qs_xform.cuh"

namespace qs {

// ---- pass A ---------------------------------------------------------------------
template <int P, bool OUT>
__global__ void __launch_bounds__(256, OUT ? 1 : 2) xcol_kernel(const void *x, int dtype, const float2 *phase, float2 *y,
                                                   float *partial, int N, int lgN1, int64_t cols) {
  // many rows: the dependent kernel is released only at exit (its CTAs would
  // otherwise take SMs this grid still needs)
  pdl_wait();  // OUT: y1 comes from the matmul; IN: x may be the previous kernel's output
  const int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (t >= cols) return;  // cols is a multiple of 32 (N1 >= 64): whole warps leave together
  constexpr int H = (P - 1) / 2;
  constexpr int off = prime_offset(P);
  const int64_t b = t >> lgN1;
  const int j1 = static_cast<int>(t & ((int64_t(1) << lgN1) - 1));
  // column j1 of row b: element j2 at [j2 << lgN1]; every load of the column
  // precedes every store (output step: in place), so the two views never
  // touch one location in the other order
  const float2 *__restrict__ cin = y + b * N + j1;
  float2 *__restrict__ col = y + b * N + j1;
  float2 v[P];
  float l1 = 0.f;
#pragma unroll
  for (int j2 = 0; j2 < P; ++j2) {
    const int o = j2 << lgN1;
    if constexpr (OUT) {
      v[j2] = cin[o];
    } else {
      const int64_t e = b * N + j1 + o;
      float2 z;
      if (dtype == QS_F16) z = __half22float2(reinterpret_cast<const __half2 *>(x)[e]);
      else if (dtype == QS_BF16) z = __bfloat1622float2(reinterpret_cast<const __nv_bfloat162 *>(x)[e]);
      else z = reinterpret_cast<const float2 *>(x)[e];
      v[j2] = xcmul(z, phase[j1 + o]);
      l1 += fabsf(v[j2].x) + fabsf(v[j2].y);
    }
  }
  // conjugate pairs: a_r = x_r + x_{P-r}, b_r = x_r - x_{P-r} (kept in v[r], v[P-r])
  float2 s0 = v[0];
#pragma unroll
  for (int r = 1; r <= H; ++r) {
    const float2 a = xcadd(v[r], v[P - r]), d = xcsub(v[r], v[P - r]);
    v[r] = a;
    v[P - r] = d;
    s0 = xcadd(s0, a);
  }
  // twiddles W_N^{j1 k} (forward) / conjugate (inverse): w^k by repeated products,
  // w^(P-k) = w^P * conj(w^k) with w^P = W_N1^{j1}
  float sn, cs;
  sincospif(2.0f * static_cast<float>(j1) / static_cast<float>(N), &sn, &cs);
  const float2 w = make_float2(cs, OUT ? sn : -sn);
  sincospif(2.0f * static_cast<float>(j1) / static_cast<float>(1 << lgN1), &sn, &cs);
  const float2 wP = make_float2(cs, OUT ? sn : -sn);
  float2 wk = make_float2(1.f, 0.f);
  col[0] = s0;
#pragma unroll
  for (int k = 1; k <= H; ++k) {
    float2 A = v[0], B = make_float2(0.f, 0.f);
#pragma unroll
    for (int r = 1; r <= H; ++r) {
      const float c = kDftCos[off + (r * k) % P];
      const float s = kDftSin[off + (r * k) % P];
      A.x = fmaf(v[r].x, c, A.x);
      A.y = fmaf(v[r].y, c, A.y);
      B.x = fmaf(v[P - r].x, s, B.x);
      B.y = fmaf(v[P - r].y, s, B.y);
    }
    // forward: X_k = A - iB, X_{P-k} = A + iB (-iB = (B.y, -B.x)); inverse swapped
    const float2 miB = make_float2(B.y, -B.x);
    const float2 Xk = OUT ? xcsub(A, miB) : xcadd(A, miB);
    const float2 Xm = OUT ? xcadd(A, miB) : xcsub(A, miB);
    wk = xcmul(wk, w);
    col[k << lgN1] = xcmul(Xk, wk);
    col[(P - k) << lgN1] = xcmul(Xm, xcmul(wP, xconj(wk)));
  }
  if constexpr (!OUT) {
    for (int o = 16; o > 0; o >>= 1) l1 += __shfl_xor_sync(0xffffffffu, l1, o);
    if ((threadIdx.x & 31) == 0) partial[t >> 5] = l1;
  }
}

// ---- pass B ---------------------------------------------------------------------
template <typename Src, typename Dst>
__device__ __forceinline__ void xwarp_stage(const XStage &S, const Src &src, const Dst &dst, const XTw &tw,
                                            bool inverse, int lane) {
  for (int j = lane; j < S.nb; j += 32) {
    switch (S.R) {
      case 2: xbutterfly_pow2<2>(S, src, dst, tw, inverse, j); break;
      case 4: xbutterfly_pow2<4>(S, src, dst, tw, inverse, j); break;
      case 8: xbutterfly_pow2<8>(S, src, dst, tw, inverse, j); break;
      case 16: xbutterfly_pow2<16>(S, src, dst, tw, inverse, j); break;
      default: break;
    }
  }
  __syncwarp();
}

// One warp runs the N1-point FFT of one block.  The plan's first stage has
// radix R0 = N1 / 32, so lane j owns first-stage butterfly j and its R0 inputs
// blk[j + 32 r], which the caller loaded into v0 ahead of time (while the
// previous block was being transformed).
template <int R0, typename Sink>
__device__ __forceinline__ void xfft_block_warp(const XPlan &p, float2 (&v0)[R0], float2 *buf0, float2 *buf1,
                                                const XTw &tw, bool inverse, int lane, const Sink &sink) {
  const XSrc<float2, false> s0{buf0, 0}, s1{buf1, 0};
  const XDst<float2, false> d0{buf0, 0}, d1{buf1, 0};
  xbutterfly_pow2_vals<R0>(p.st[0], v0, d1, tw, inverse, lane);
  __syncwarp();
  for (int s = 1; s + 1 < p.nst; ++s) {
    if (s & 1) xwarp_stage(p.st[s], s1, d0, tw, inverse, lane);
    else xwarp_stage(p.st[s], s0, d1, tw, inverse, lane);
  }
  if ((p.nst - 1) & 1) xwarp_stage(p.st[p.nst - 1], s1, sink, tw, inverse, lane);
  else xwarp_stage(p.st[p.nst - 1], s0, sink, tw, inverse, lane);
}

struct XBlkArgs {
  const float2 *y;     // pass-A result, rows x N complex
  int N, P, N1, warp_mode;
  // output step
  const float2 *phase;
  const float *bias;
  float scale;
  void *out;
  int dtype;
  // input step
  const float *partial;
  int nparts;
  __half *x2h;
  float *rowscale;
  int n_pad;
};

// Block source (CTA per block): element e1 of the contiguous pass-A block.
struct XBlockSrc {
  const float2 *blk;
  __device__ __forceinline__ float2 operator()(int e1) const { return blk[e1]; }
};

// Block sink: FFT output k1 of block k is element k + P*k1 of the row, staged
// in shared memory (output step: scaled float32, finished in the coalesced
// store loop where sign / phase and bias loads are contiguous; input step: the
// fp16 matmul operand).
template <bool OUT>
struct XBlockSink {
  unsigned char *row;
  float scale;
  int k, P;
  __device__ __forceinline__ void operator()(int k1, float2 z) const {
    const int e = k + P * k1;
    z.x *= scale;
    z.y *= scale;
    if constexpr (OUT) reinterpret_cast<float2 *>(row)[e] = z;
    else reinterpret_cast<__half2 *>(row)[e] = __floats2half2_rn(z.x, z.y);
  }
};

template <bool OUT>
__global__ void __launch_bounds__(256) xblk_kernel(XPlan p1, XBlkArgs a) {
  extern __shared__ __align__(16) unsigned char xsm2[];
  __shared__ XTw tw;
  __shared__ float red[8];
  // many rows: the dependent kernel is released only at exit
  build_xtw(tw, a.N1);
  pdl_wait();  // the pass-A result
  const int64_t b = blockIdx.x;
  const int N = a.N, P = a.P, N1 = a.N1;
  const int bufE = xbuf_elems<float2>(N1);
  // staging row (final order; output step float32, input step fp16) after the FFT buffers
  const int nbufs = a.warp_mode ? 2 * (blockDim.x >> 5) : 2;
  unsigned char *stage_row = xsm2 + round_up(static_cast<int64_t>(nbufs) * bufE * sizeof(float2), 16);
  float sc = a.scale, inv = 1.f;
  if constexpr (!OUT) {
    // row scale from the L1 bound of the transformed row
    float part = 0.f;
    for (int i = threadIdx.x; i < a.nparts; i += blockDim.x) part += a.partial[b * a.nparts + i];
    for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = part;
    __syncthreads();
    float l1 = 0.f;
    for (int i = 0; i < static_cast<int>(blockDim.x >> 5); ++i) l1 += red[i];
    float s2;
    xpow2_scale(l1 * a.scale, s2, inv);
    sc = a.scale * s2;
  }
  __syncthreads();  // twiddle tables
  const float2 *yrow = a.y + b * N;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  if (a.warp_mode) {
    float2 *b0 = reinterpret_cast<float2 *>(xsm2) + static_cast<size_t>(2 * warp) * bufE;
    switch (N1 >> 5) {
#define QS_WARP_BLOCKS(R0)                                                                    \
  case R0: {                                                                                  \
    float2 nxt[R0];                                                                           \
    if (warp < P) {                                                                           \
      _Pragma("unroll") for (int r = 0; r < R0; ++r) nxt[r] = yrow[warp * N1 + lane + 32 * r]; \
    }                                                                                         \
    for (int k = warp; k < P; k += nw) {                                                      \
      float2 cur[R0];                                                                         \
      _Pragma("unroll") for (int r = 0; r < R0; ++r) cur[r] = nxt[r];                         \
      if (k + nw < P) {                                                                       \
        _Pragma("unroll") for (int r = 0; r < R0; ++r) nxt[r] = yrow[(k + nw) * N1 + lane + 32 * r]; \
      }                                                                                       \
      XBlockSink<OUT> sink{stage_row, sc, k, P};                                              \
      xfft_block_warp<R0>(p1, cur, b0, b0 + bufE, tw, OUT, lane, sink);                       \
      __syncwarp();                                                                           \
    }                                                                                         \
  } break;
      QS_WARP_BLOCKS(2) QS_WARP_BLOCKS(4) QS_WARP_BLOCKS(8) QS_WARP_BLOCKS(16)
#undef QS_WARP_BLOCKS
      default: break;
    }
  } else {
    float2 *b0 = reinterpret_cast<float2 *>(xsm2);
    for (int k = 0; k < P; ++k) {
      XBlockSink<OUT> sink{stage_row, sc, k, P};
      XBlockSrc gsrc{yrow + static_cast<int64_t>(k) * N1};
      xfft_row<0, false>(p1, b0, b0 + bufE, tw, OUT, 0, gsrc, sink);
      __syncthreads();
    }
  }
  __syncthreads();
  if constexpr (OUT) {
    // y = staged * conj(phase) + bias, cast; two complex values per step,
    // contiguous in the staged row, the phases, the bias and the output
    const float4 *st4 = reinterpret_cast<const float4 *>(stage_row);
    const float4 *ph4 = reinterpret_cast<const float4 *>(a.phase);
    const float4 *bi4 = reinterpret_cast<const float4 *>(a.bias);
    for (int i = threadIdx.x; i < N / 2; i += blockDim.x) {
      float4 z = st4[i];
      const float4 ph = ph4[i];
      float4 r = make_float4(z.x * ph.x + z.y * ph.y, z.y * ph.x - z.x * ph.y, z.z * ph.z + z.w * ph.w,
                             z.w * ph.z - z.z * ph.w);
      if (a.bias) {
        const float4 bb = bi4[i];
        r.x += bb.x;
        r.y += bb.y;
        r.z += bb.z;
        r.w += bb.w;
      }
      if (a.dtype == QS_F16) {
        const __half2 h0 = __floats2half2_rn(r.x, r.y), h1 = __floats2half2_rn(r.z, r.w);
        reinterpret_cast<uint2 *>(a.out)[b * (N / 2) + i] =
            make_uint2(*reinterpret_cast<const uint32_t *>(&h0), *reinterpret_cast<const uint32_t *>(&h1));
      } else if (a.dtype == QS_BF16) {
        const __nv_bfloat162 h0 = __floats2bfloat162_rn(r.x, r.y), h1 = __floats2bfloat162_rn(r.z, r.w);
        reinterpret_cast<uint2 *>(a.out)[b * (N / 2) + i] =
            make_uint2(*reinterpret_cast<const uint32_t *>(&h0), *reinterpret_cast<const uint32_t *>(&h1));
      } else {
        reinterpret_cast<float4 *>(a.out)[b * (N / 2) + i] = r;
      }
    }
  } else {
    // coalesced 16-byte stores of the staged fp16 row
    const int row_bytes = N * 4;
    unsigned char *dst = reinterpret_cast<unsigned char *>(a.x2h + b * a.n_pad);
    const int nv = row_bytes >> 4;
    for (int i = threadIdx.x; i < nv; i += blockDim.x)
      reinterpret_cast<uint4 *>(dst)[i] = reinterpret_cast<const uint4 *>(stage_row)[i];
    for (int i = nv * 16 + threadIdx.x; i < row_bytes; i += blockDim.x) dst[i] = stage_row[i];
  }
  if constexpr (!OUT) {
    for (int i = 2 * N + threadIdx.x; i < a.n_pad; i += blockDim.x) a.x2h[b * a.n_pad + i] = __float2half_rn(0.f);
    if (threadIdx.x == 0) a.rowscale[b] = inv;
  }
}

// ---- few rows ("spread" mode) ---------------------------------------------------
// When the rows alone cannot fill the GPU (decode), pass A splits each column's
// output pairs over G = spread_groups(P) lanes of a warp (all lanes load the column, a warp
// barrier, then each lane stores its pairs: in place is safe), and pass B
// gives each block to its own warp (N1 <= 512) or CTA, across as many CTAs as
// there are blocks, writing the output straight to global memory.
// Lanes per column in spread mode: a power of two up to 4, at most the number
// of output pairs (P - 1) / 2 (more lanes repeat the column loads and the
// per-group code without shortening the chain enough).
__host__ __device__ constexpr int spread_groups(int P) {
  int G = 1;
  while (G * 2 <= (P - 1) / 2 && G < 4) G *= 2;
  return G;
}
constexpr int kSpreadGroupsMax = 4;
// Largest prime whose spread pass A splits a column over lanes (xcol_spread_kernel);
// larger primes take a warp per column (xcol_warp_kernel).
constexpr int kSpreadMaxPrime = 13;

template <int P, bool OUT, int G, int g>
__device__ __forceinline__ void xcol_group(const float2 (&v)[P], float2 *__restrict__ col, int lgN1, int j1, int N) {
  constexpr int H = (P - 1) / 2;
  constexpr int per = (H + G - 1) / G;
  constexpr int klo = g * per + 1;
  constexpr int off = prime_offset(P);
  if constexpr (klo <= H) {
    float sn, cs;
    sincospif(2.0f * static_cast<float>(j1) / static_cast<float>(N), &sn, &cs);
    const float2 w = make_float2(cs, OUT ? sn : -sn);
    sincospif(2.0f * static_cast<float>(j1) / static_cast<float>(1 << lgN1), &sn, &cs);
    const float2 wP = make_float2(cs, OUT ? sn : -sn);
    sincospif(2.0f * static_cast<float>((j1 * klo) % N) / static_cast<float>(N), &sn, &cs);
    float2 wk = make_float2(cs, OUT ? sn : -sn);  // w^klo
#pragma unroll
    for (int q = 0; q < per; ++q) {
          const int k = klo + q;
      if (k <= H) {
        float2 A = v[0], B = make_float2(0.f, 0.f);
#pragma unroll
        for (int r = 1; r <= H; ++r) {
          const float c = kDftCos[off + (r * (klo + q)) % P];
          const float s = kDftSin[off + (r * (klo + q)) % P];
          A.x = fmaf(v[r].x, c, A.x);
          A.y = fmaf(v[r].y, c, A.y);
          B.x = fmaf(v[P - r].x, s, B.x);
          B.y = fmaf(v[P - r].y, s, B.y);
        }
        const float2 miB = make_float2(B.y, -B.x);
        const float2 Xk = OUT ? xcsub(A, miB) : xcadd(A, miB);
        const float2 Xm = OUT ? xcadd(A, miB) : xcsub(A, miB);
        col[k << lgN1] = xcmul(Xk, wk);
        col[(P - k) << lgN1] = xcmul(Xm, xcmul(wP, xconj(wk)));
        wk = xcmul(wk, w);
      }
    }
  }
}

template <int P, bool OUT, int G, int g = 0>
__device__ __forceinline__ void xcol_group_dispatch(int gi, const float2 (&v)[P], float2 *__restrict__ col, int lgN1,
                                                    int j1, int N) {
  if constexpr (g < G) {
    if (gi == g) xcol_group<P, OUT, G, g>(v, col, lgN1, j1, N);
    else xcol_group_dispatch<P, OUT, G, g + 1>(gi, v, col, lgN1, j1, N);
  }
}

template <int P, bool OUT>
__global__ void __launch_bounds__(256) xcol_spread_kernel(const void *x, int dtype, const float2 *phase, float2 *y,
                                                          float *partial, int N, int lgN1, int64_t tasks) {
  constexpr int G = spread_groups(P);
  pdl_launch_dependents();
  if constexpr (!OUT) xprefetch_l2(phase, 8 * static_cast<int64_t>(N), blockIdx.x, gridDim.x);
  pdl_wait();
  const int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (t >= tasks) return;  // tasks = rows * N1 * G, a multiple of 32: whole warps leave together
  constexpr int H = (P - 1) / 2;
  const int g = static_cast<int>(t & (G - 1));
  const int64_t c = t / G;
  const int64_t b = c >> lgN1;
  const int j1 = static_cast<int>(c & ((int64_t(1) << lgN1) - 1));
  const float2 *__restrict__ cin = y + b * N + j1;
  float2 *__restrict__ col = y + b * N + j1;
  float2 v[P];
  float l1 = 0.f;
#pragma unroll
  for (int j2 = 0; j2 < P; ++j2) {
    const int o = j2 << lgN1;
    if constexpr (OUT) {
      v[j2] = cin[o];
    } else {
      const int64_t e = b * N + j1 + o;
      float2 z;
      if (dtype == QS_F16) z = __half22float2(reinterpret_cast<const __half2 *>(x)[e]);
      else if (dtype == QS_BF16) z = __bfloat1622float2(reinterpret_cast<const __nv_bfloat162 *>(x)[e]);
      else z = reinterpret_cast<const float2 *>(x)[e];
      v[j2] = xcmul(z, phase[j1 + o]);
      if (g == 0) l1 += fabsf(v[j2].x) + fabsf(v[j2].y);
    }
  }
  __syncwarp();  // every lane of the column has read it before any lane stores into it
  float2 s0 = v[0];
#pragma unroll
  for (int r = 1; r <= H; ++r) {
    const float2 a = xcadd(v[r], v[P - r]), d = xcsub(v[r], v[P - r]);
    v[r] = a;
    v[P - r] = d;
    s0 = xcadd(s0, a);
  }
  if (g == 0) col[0] = s0;
  xcol_group_dispatch<P, OUT, G>(g, v, col, lgN1, j1, N);
  if constexpr (!OUT) {
    for (int o = 16; o > 0; o >>= 1) l1 += __shfl_xor_sync(0xffffffffu, l1, o);
    if ((threadIdx.x & 31) == 0) partial[t >> 5] = l1;
  }
}

// Spread pass A for the primes above kSpreadMaxPrime: a warp per column
// (columns j1 of the rows' N1 x P layout, inputs j1 + j2 * N1), lane k computing
// output pair k (lane 0 the DC term).  Lane l loads inputs l and l + 32, the
// conjugate-pair sums a_r = x_r + x_{P-r}, b_r = x_r - x_{P-r} (one shuffle) are
// staged per warp in shared memory and read back as broadcasts, and lane k
// holds its H cos / sin coefficients in registers, formed by rotation before
// the dependent-launch wait.  Outputs get the four-step twiddles and land in
// place (every lane loads the column before any lane stores).  The input step
// also writes the column's L1 norm to partial[column].
constexpr int kColWarpsMax = 4;

template <int P, bool OUT>
__global__ void __launch_bounds__(32 * kColWarpsMax) xcol_warp_kernel(const void *x, int dtype, const float2 *phase,
                                                                     float2 *y, float *partial, int N, int lgN1,
                                                                     int64_t cols) {
  constexpr int H = (P - 1) / 2;
  __shared__ float4 stage_all[kColWarpsMax][H + 1];
  pdl_launch_dependents();
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  float cr[H], sr[H];
  {
    float sk, ck;
    sincospif(2.0f * static_cast<float>(lane <= H ? lane : 0) / static_cast<float>(P), &sk, &ck);
    float2 z = make_float2(ck, sk);
#pragma unroll
    for (int r = 0; r < H; ++r) {
      cr[r] = z.x;
      sr[r] = z.y;
      z = xcmul(z, make_float2(ck, sk));
    }
  }
  if constexpr (!OUT) xprefetch_l2(phase, 8 * static_cast<int64_t>(N), blockIdx.x, gridDim.x);
  pdl_wait();  // OUT: y1 comes from the matmul; IN: x may be the previous kernel's output
  const int64_t c = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + w;
  if (c >= cols) return;  // whole warps leave together
  const int64_t b = c >> lgN1;
  const int j1 = static_cast<int>(c & ((int64_t(1) << lgN1) - 1));
  float2 *__restrict__ col = y + b * N + j1;
  auto load = [&](int j2) -> float2 {
    const int o = j2 << lgN1;
    if constexpr (OUT) {
      return col[o];
    } else {
      const int64_t e = b * N + j1 + o;
      float2 z;
      if (dtype == QS_F16) z = __half22float2(reinterpret_cast<const __half2 *>(x)[e]);
      else if (dtype == QS_BF16) z = __bfloat1622float2(reinterpret_cast<const __nv_bfloat162 *>(x)[e]);
      else z = reinterpret_cast<const float2 *>(x)[e];
      return xcmul(z, phase[j1 + o]);
    }
  };
  const float2 v0 = lane < P ? load(lane) : make_float2(0.f, 0.f);
  const float2 v1 = lane + 32 < P ? load(lane + 32) : make_float2(0.f, 0.f);
  if constexpr (!OUT) {
    float l1 = fabsf(v0.x) + fabsf(v0.y) + fabsf(v1.x) + fabsf(v1.y);
    for (int o = 16; o > 0; o >>= 1) l1 += __shfl_xor_sync(0xffffffffu, l1, o);
    if (lane == 0) partial[c] = l1;
  }
  const int src = (P - lane) & 31;  // lane holding x_{P - lane}, in its second register when P - lane >= 32
  const float2 u0 = make_float2(__shfl_sync(0xffffffffu, v0.x, src), __shfl_sync(0xffffffffu, v0.y, src));
  const float2 u1 = make_float2(__shfl_sync(0xffffffffu, v1.x, src), __shfl_sync(0xffffffffu, v1.y, src));
  const float2 xm = (lane >= 1 && P - lane >= 32) ? u1 : u0;
  float4 *st = stage_all[w];
  if (lane == 0) st[0] = make_float4(v0.x, v0.y, 0.f, 0.f);
  else if (lane <= H) st[lane] = make_float4(v0.x + xm.x, v0.y + xm.y, v0.x - xm.x, v0.y - xm.y);
  __syncwarp();  // the column is in registers / shared memory: stores into it may start
  const float4 x0 = st[0];
  float2 A = make_float2(x0.x, x0.y), A2 = make_float2(0.f, 0.f), B = A2, B2 = A2;
#pragma unroll
  for (int r = 0; r < H; ++r) {
    const float4 ab = st[1 + r];
    if (r & 1) {
      A2.x = fmaf(ab.x, cr[r], A2.x);
      A2.y = fmaf(ab.y, cr[r], A2.y);
      B2.x = fmaf(ab.z, sr[r], B2.x);
      B2.y = fmaf(ab.w, sr[r], B2.y);
    } else {
      A.x = fmaf(ab.x, cr[r], A.x);
      A.y = fmaf(ab.y, cr[r], A.y);
      B.x = fmaf(ab.z, sr[r], B.x);
      B.y = fmaf(ab.w, sr[r], B.y);
    }
  }
  A = xcadd(A, A2);
  B = xcadd(B, B2);
  if (lane == 0) {
    col[0] = A;  // k = 0: every coefficient is 1, twiddle 1
  } else if (lane <= H) {
    const int k = lane;
    float sn, cs;
    sincospif(2.0f * static_cast<float>((j1 * k) % N) / static_cast<float>(N), &sn, &cs);
    const float2 wk = make_float2(cs, OUT ? sn : -sn);  // W_N^(j1 k) (conjugate for the inverse)
    sincospif(2.0f * static_cast<float>(j1) / static_cast<float>(1 << lgN1), &sn, &cs);
    const float2 wP = make_float2(cs, OUT ? sn : -sn);  // W_N^(j1 P) = W_N1^j1
    const float2 miB = make_float2(B.y, -B.x);          // -iB
    const float2 Xk = OUT ? xcsub(A, miB) : xcadd(A, miB);
    const float2 Xm = OUT ? xcadd(A, miB) : xcsub(A, miB);
    col[k << lgN1] = xcmul(Xk, wk);
    col[(P - k) << lgN1] = xcmul(Xm, xcmul(wP, xconj(wk)));
  }
}

// Global sink of a spread block: element k + P*k1 of row b.
template <bool OUT>
struct XSpreadSink {
  const float2 *phase;
  const float *bias;
  void *out;
  int dtype;
  __half *x2h;
  int64_t n_pad;
  int64_t b;
  int N, k, P;
  float scale;
  __device__ __forceinline__ void operator()(int k1, float2 z) const {
    const int e = k + P * k1;
    z.x *= scale;
    z.y *= scale;
    if constexpr (OUT) {
      z = xcmul(z, xconj(phase[e]));
      if (bias) {
        const float2 bb = reinterpret_cast<const float2 *>(bias)[e];
        z.x += bb.x;
        z.y += bb.y;
      }
      const int64_t o = b * N + e;
      if (dtype == QS_F16) reinterpret_cast<__half2 *>(out)[o] = __floats2half2_rn(z.x, z.y);
      else if (dtype == QS_BF16) reinterpret_cast<__nv_bfloat162 *>(out)[o] = __floats2bfloat162_rn(z.x, z.y);
      else reinterpret_cast<float2 *>(out)[o] = z;
    } else {
      reinterpret_cast<__half2 *>(x2h + b * n_pad)[e] = __floats2half2_rn(z.x, z.y);
    }
  }
};

// Input step: the row's fp16 scale from its L1 partial sums (every warp of the row computes it).
__device__ __forceinline__ void xrow_scale_from_l1(const float *partial, int nparts, int64_t b, float scale, int lane,
                                                   float &sc, float &inv) {
  float part = 0.f;
  for (int i = lane; i < nparts; i += 32) part += partial[b * nparts + i];
  for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
  float s2;
  xpow2_scale(part * scale, s2, inv);
  sc = scale * s2;
}

struct XSpreadArgs {
  int64_t rows;
  float *y1;        // input step of a decode-sized batch: y1 (rows, m_local) to zero, or null
  int64_t m_local;
  int *busy;        // output step: the dry-pass hint flag (xbusy_flag), set while it runs
};

template <bool OUT, int R0>
__global__ void __launch_bounds__(256) xblk_spread_kernel(XPlan p1, XBlkArgs a, XSpreadArgs sa) {
  extern __shared__ float2 xsm3[];
  __shared__ XTw tw;
  constexpr int RW = R0 ? R0 : 1;
  const bool flag = OUT && blockIdx.x == 0 && threadIdx.x == 0;
  if (flag) xbusy_set(sa.busy, 1);  // dry-pass hint for the next input step (xbusy_flag)
  pdl_launch_dependents();
  if constexpr (OUT) {  // layer constants of the sink, into L2 while pass A still runs
    xprefetch_l2(a.phase, 8 * static_cast<int64_t>(a.N), blockIdx.x, gridDim.x);
    xprefetch_l2(a.bias, 8 * static_cast<int64_t>(a.N), blockIdx.x, gridDim.x);
  }
  build_xtw(tw, a.N1);
  pdl_wait();
  if (!OUT && sa.y1) {  // zero y1 for the decode matmul: a slice per CTA
    const int64_t total = sa.rows * sa.m_local;
    const int64_t z0 = total * blockIdx.x / gridDim.x, z1 = total * (blockIdx.x + 1) / gridDim.x;
    for (int64_t i = z0 + threadIdx.x; i < z1; i += blockDim.x) sa.y1[i] = 0.f;
  }
  __syncthreads();  // twiddle tables
  const int N = a.N, P = a.P, N1 = a.N1;
  const int bufE = xbuf_elems<float2>(N1);
  const int lane = threadIdx.x & 31;
  int64_t blk_id;
  float2 *b0;
  if constexpr (R0 != 0) {
    const int warp = threadIdx.x >> 5;
    blk_id = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + warp;
    if (blk_id >= sa.rows * P) return;  // no CTA barrier follows
    b0 = xsm3 + static_cast<size_t>(2 * warp) * bufE;
  } else {
    blk_id = blockIdx.x;
    b0 = xsm3;
  }
  const int64_t b = blk_id / P;
  const int k = static_cast<int>(blk_id - b * P);
  const float2 *blk = a.y + b * N + static_cast<int64_t>(k) * N1;
  float sc = a.scale, inv = 1.f;
  if constexpr (!OUT) xrow_scale_from_l1(a.partial, a.nparts, b, a.scale, lane, sc, inv);
  XSpreadSink<OUT> sink{a.phase, a.bias, a.out, a.dtype, a.x2h, a.n_pad, b, N, k, P, sc};
  if constexpr (R0 != 0) {
    float2 cur[RW];
#pragma unroll
    for (int r = 0; r < RW; ++r) cur[r] = blk[lane + 32 * r];
    xfft_block_warp<RW>(p1, cur, b0, b0 + bufE, tw, OUT, lane, sink);
  } else {
    xfft_row<0, false>(p1, b0, b0 + bufE, tw, OUT, 0, XBlockSrc{blk}, sink);
  }
  if constexpr (!OUT) {
    if (k == 0) {
      for (int i = 2 * N + lane; i < a.n_pad; i += 32) a.x2h[b * a.n_pad + i] = __float2half_rn(0.f);
      if (lane == 0) a.rowscale[b] = inv;
    }
  }
  if (flag) xbusy_set(sa.busy, 0);
}

// ---- host -----------------------------------------------------------------------
static int xnum_sms2() {
  static int cached[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && cached[dev]) return cached[dev];
  int n = 148;
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  if (dev < 64) cached[dev] = n;
  return n;
}

// Half widths that use the two-pass path: N = P * 2^a >= 4096, P an odd prime
// <= 43, 2^a >= 64.
static bool spread_mode(int64_t rows) { return rows * 2 <= xnum_sms2(); }

bool two_pass_rfft(int64_t N, int64_t rows, int *P_out, int *lgN1_out) {
  if (N < 4096) return false;
  int P = 0;
  for (int q : {43, 41, 37, 31, 29, 23, 19, 17, 13, 11, 7, 5, 3}) {
    if (N % q == 0) {
      if (P) return false;  // more than one odd prime
      P = q;
    }
  }
  if (!P || (N / P) % P == 0) return false;
  const int64_t N1 = N / P;
  if (N1 < 64 || (N1 & (N1 - 1))) return false;
  int lg = 0;
  while ((int64_t(1) << lg) < N1) ++lg;
  if (P_out) *P_out = P;
  if (lgN1_out) *lgN1_out = lg;
  return true;
}

int64_t two_pass_input_scratch_bytes(int64_t batch, int64_t n) {
  int P, lg;
  if (n % 2 || !two_pass_rfft(n / 2, batch, &P, &lg)) return 0;
  const int64_t N = n / 2, N1 = int64_t(1) << lg;
  // L1 partial sums: N1 / 32 * G per row (lane-split columns), N1 per row (a warp per column)
  return round_up(batch * N * 8, 256) + round_up(batch * N1 * 4, 256);
}

// Plan of the N1-point block FFT.  Warp per block (N1 <= 512): first radix
// N1 / 32 (one first-stage butterfly per lane), then the remaining 5 bits in
// radix-8 and radix-4 stages.  CTA per block: power-of-two stages with at
// least 256 butterflies each.
static void block_plan(int N1, bool warp_mode, XPlan &p) {
  int a = 0;
  while ((1 << a) < N1) ++a;
  int logs[kXMaxStages], ns = 0;
  if (warp_mode) {
    logs[ns++] = a - 5;
    logs[ns++] = 3;
    logs[ns++] = 2;
  } else {
    int maxlog = 1;
    while (maxlog < 4 && (N1 >> (maxlog + 1)) >= 256) ++maxlog;
    const int cnt = (a + maxlog - 1) / maxlog, base = a / cnt, extra = a % cnt;
    for (int s = 0; s < cnt; ++s) logs[ns++] = base + (s < extra ? 1 : 0);
  }
  p.N = N1;
  p.nst = ns;
  p.C = 1;
  p.cl = 0;
  p.E = N1;
  p.big = 0;
  int Ns = 1;
  for (int s = 0; s < ns; ++s) {
    XStage &S = p.st[s];
    S.R = 1 << logs[s];
    S.G = 1;
    S.compact = 0;
    S.Ns = Ns;
    S.nb = N1 / S.R;
    S.nbC = S.nb;
    S.twstep = N1 / (Ns * S.R);
    S.dNs = make_fastdiv(static_cast<uint32_t>(Ns));
    S.dnbC = make_fastdiv(static_cast<uint32_t>(S.nbC));
    Ns *= S.R;
  }
}

template <bool OUT>
static int launch_col(int P, const void *x, int dtype, const float2 *phase, float2 *y, float *partial, int N,
                      int lgN1, int64_t cols, cudaStream_t s) {
  const dim3 grid(static_cast<unsigned>(ceil_div(cols, 256)));
  switch (P) {
#define QS_COL(Q) \
  case Q: return launch_pdl("two_pass_columns", xcol_kernel<Q, OUT>, grid, dim3(256), 0, s, x, dtype, phase, y, partial, N, lgN1, cols);
    QS_COL(3) QS_COL(5) QS_COL(7) QS_COL(11) QS_COL(13) QS_COL(17) QS_COL(19) QS_COL(23) QS_COL(29) QS_COL(31)
    QS_COL(37) QS_COL(41) QS_COL(43)
#undef QS_COL
    default: return fail(QS_ERR_UNSUPPORTED, "two-pass FFT: bad prime %d", P);
  }
}

template <bool OUT>
static int launch_col_spread(int P, const void *x, int dtype, const float2 *phase, float2 *y, float *partial, int N,
                             int lgN1, int64_t tasks, cudaStream_t s) {
  const dim3 grid(static_cast<unsigned>(ceil_div(tasks, 256)));
  switch (P) {
#define QS_COL(Q) \
  case Q: return launch_pdl("two_pass_columns", xcol_spread_kernel<Q, OUT>, grid, dim3(256), 0, s, x, dtype, phase, y, partial, N, lgN1, tasks);
    QS_COL(3) QS_COL(5) QS_COL(7) QS_COL(11) QS_COL(13)
#undef QS_COL
    default: return fail(QS_ERR_UNSUPPORTED, "two-pass FFT: bad prime %d", P);
  }
}

template <bool OUT>
static int launch_col_warp(int P, const void *x, int dtype, const float2 *phase, float2 *y, float *partial, int N,
                           int lgN1, int64_t cols, cudaStream_t s) {
  // one warp per CTA while the columns alone leave SMs idle (latency), else kColWarpsMax
  const int wpc = cols <= xnum_sms2() ? 1 : kColWarpsMax;
  const dim3 grid(static_cast<unsigned>(ceil_div(cols, wpc)));
  switch (P) {
#define QS_COL(Q) \
  case Q: return launch_pdl("two_pass_columns", xcol_warp_kernel<Q, OUT>, grid, dim3(32 * wpc), 0, s, x, dtype, phase, y, partial, N, lgN1, cols);
    QS_COL(17) QS_COL(19) QS_COL(23) QS_COL(29) QS_COL(31) QS_COL(37) QS_COL(41) QS_COL(43)
#undef QS_COL
    default: return fail(QS_ERR_UNSUPPORTED, "two-pass FFT: bad prime %d", P);
  }
}

// Spread pass B: a warp per block (N1 <= 512) in CTAs of 8 warps, else a CTA per block.
template <bool OUT>
static int launch_blk_spread(const XBlkArgs &a0, const XSpreadArgs &sa, cudaStream_t s) {
  XBlkArgs a = a0;
  const bool warp = a.N1 <= 512;
  a.warp_mode = warp;
  XPlan p1;
  block_plan(a.N1, warp, p1);
  const int64_t nblocks = sa.rows * a.P;
  const size_t smem = static_cast<size_t>(warp ? 16 : 2) * xbuf_elems<float2>(a.N1) * sizeof(float2);
  auto kern = xblk_spread_kernel<OUT, 0>;
  if (warp) {
    switch (a.N1 >> 5) {
      case 2: kern = xblk_spread_kernel<OUT, 2>; break;
      case 4: kern = xblk_spread_kernel<OUT, 4>; break;
      case 8: kern = xblk_spread_kernel<OUT, 8>; break;
      case 16: kern = xblk_spread_kernel<OUT, 16>; break;
      default: return fail(QS_ERR_UNSUPPORTED, "two-pass FFT: block of %d points", a.N1);
    }
  }
  QS_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  const int64_t grid = warp ? ceil_div(nblocks, 8) : nblocks;
  return launch_pdl("two_pass_blocks", kern, dim3(static_cast<unsigned>(grid)), dim3(256), smem, s, p1, a, sa);
}

template <bool OUT>
static int launch_blk(int64_t rows, const XBlkArgs &a0, cudaStream_t s) {
  XBlkArgs a = a0;
  const int threads = 256;
  a.warp_mode = a.N1 <= 512;
  XPlan p1;
  block_plan(a.N1, a.warp_mode != 0, p1);
  const int nbufs = a.warp_mode ? 2 * (threads / 32) : 2;
  const size_t smem = round_up(static_cast<int64_t>(nbufs) * xbuf_elems<float2>(a.N1) * sizeof(float2), 16) +
                      static_cast<size_t>(a.N) * (OUT ? 8 : 4);
  if (smem > 220 * 1024) return fail(QS_ERR_UNSUPPORTED, "two-pass FFT: row of %d points too large", a.N);
  QS_CUDA_TRY(cudaFuncSetAttribute(xblk_kernel<OUT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  return launch_pdl("two_pass_blocks", xblk_kernel<OUT>, dim3(static_cast<unsigned>(rows)), dim3(threads), smem, s,
                    p1, a);
}

int launch_two_pass_output(float *y1, int64_t batch, int64_t m, const float2 *phase, const float *bias, float scale,
                           void *y, int dtype, cudaStream_t s) {
  int P, lg;
  const int64_t N = m / 2;
  if (!two_pass_rfft(N, batch, &P, &lg)) return fail(QS_ERR_INVALID_ARG, "two-pass FFT not applicable");
  float2 *yc = reinterpret_cast<float2 *>(y1);
  const bool spread = spread_mode(batch);
  int st = !spread ? launch_col<true>(P, nullptr, 0, nullptr, yc, nullptr, static_cast<int>(N), lg, batch << lg, s)
           : P > kSpreadMaxPrime
               ? launch_col_warp<true>(P, nullptr, 0, nullptr, yc, nullptr, static_cast<int>(N), lg, batch << lg, s)
               : launch_col_spread<true>(P, nullptr, 0, nullptr, yc, nullptr, static_cast<int>(N), lg,
                                         (batch << lg) * spread_groups(P), s);
  if (st) return st;
  XBlkArgs a{};
  a.y = yc;
  a.N = static_cast<int>(N);
  a.P = P;
  a.N1 = 1 << lg;
  a.phase = phase;
  a.bias = bias;
  a.scale = scale;
  a.out = y;
  a.dtype = dtype;
  if (spread) return launch_blk_spread<true>(a, XSpreadArgs{batch, nullptr, 0, xbusy_flag()}, s);
  return launch_blk<true>(batch, a, s);
}

int launch_two_pass_input(const void *x, int dtype, int64_t batch, int64_t n, const float2 *phase, float scale,
                          __half *x2h, float *rowscale, int n_pad, void *scratch, float *y1, int64_t m_local,
                          cudaStream_t s) {
  int P, lg;
  const int64_t N = n / 2;
  if (!two_pass_rfft(N, batch, &P, &lg)) return fail(QS_ERR_INVALID_ARG, "two-pass FFT not applicable");
  float2 *yc = static_cast<float2 *>(scratch);
  float *partial = reinterpret_cast<float *>(static_cast<char *>(scratch) + round_up(batch * N * 8, 256));
  const bool spread = spread_mode(batch);
  if (!spread && y1) return fail(QS_ERR_INVALID_ARG, "two-pass FFT: y1 zeroing only in spread mode");
  const bool colwarp = spread && P > kSpreadMaxPrime;
  int st = !spread ? launch_col<false>(P, x, dtype, phase, yc, partial, static_cast<int>(N), lg, batch << lg, s)
           : colwarp ? launch_col_warp<false>(P, x, dtype, phase, yc, partial, static_cast<int>(N), lg, batch << lg, s)
                     : launch_col_spread<false>(P, x, dtype, phase, yc, partial, static_cast<int>(N), lg,
                                                (batch << lg) * spread_groups(P), s);
  if (st) return st;
  XBlkArgs a{};
  a.y = yc;
  a.N = static_cast<int>(N);
  a.P = P;
  a.N1 = 1 << lg;
  a.scale = scale;
  a.partial = partial;
  a.nparts = colwarp ? (1 << lg) : (1 << lg) / 32 * (spread ? spread_groups(P) : 1);
  a.x2h = x2h;
  a.rowscale = rowscale;
  a.n_pad = n_pad;
  if (spread) return launch_blk_spread<false>(a, XSpreadArgs{batch, y1, y1 ? m_local : 0, nullptr}, s);
  return launch_blk<false>(batch, a, s);
}

}  // namespace qs
