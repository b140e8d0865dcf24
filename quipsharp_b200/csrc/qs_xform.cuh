// Row transforms of the incoherence processing -- the RFFT transform's
// complex FFT (quipsharp/rfft.py:37-60) and the randomized Hadamard
// transform's FWHT (quipsharp/hadamard.py:17-40) -- as one engine of
// register-resident Stockham stages.
//
// Execution model
//  * One row of N points is transformed by a group of C CTAs (C = 1, or a
//    thread-block cluster of 2..16 CTAs exchanging data through distributed
//    shared memory).  Few rows (decode) spread a long row over a cluster so
//    its latency is divided over several SMs; many rows (prefill) run one CTA
//    per row, or a small cluster when a row does not fit one SM's shared
//    memory twice.  (The RFFT's N = P * 2^a >= 4096 widths use the two-pass
//    kernels of qs_xform2.cu instead, for few rows and many.)
//  * The row lives in two shared buffers (ping-pong), distributed cyclically:
//    element e sits in CTA e mod C at local index e / C, so butterfly j, whose
//    inputs are j + r * nb with C dividing nb, finds them all in CTA j mod C;
//    stages read their own CTA's buffer and store to the owners' buffers.
//  * A stage is a set of independent tasks (butterflies, or output groups of
//    one); each CTA runs the tasks of its own butterflies.  A thread loads a
//    task's values, transforms them in registers and stores them; a barrier
//    (CTA or cluster) separates stages.
//  * A power-of-two first stage reads the row from global memory (the cast and
//    the sign / phase multiply fused into the load); an odd first stage reads
//    a copy made by a coalesced load pass.  For the output steps the last
//    stage writes global memory (scale, sign / conjugate phase, bias and cast
//    fused into the store), so HBM sees the row once in and once out.
//
// FFT: mixed-radix Stockham, radices {16, 8, 4, 2} (in-register DIT), odd
// primes 3..43.  Stage order: the prime >= 11 (at most one, first), then
// 7 / 5 / 3, then the power-of-two stages.  The odd-prime DFT uses the
// conjugate-pair form X_k, X_{P-k} = A_k -+ i B_k; its (P-1)/2 output pairs are
// split into G groups that run as separate tasks (warp-uniform): unrolled with
// compile-time cos / sin operands, or (few rows in a cluster) compact rolled
// code with one or two pairs per task.  Twiddles W_N^e come from two small
// shared tables (W_N^e = C[e >> 7] * F[e & 127]); the powers a butterfly needs
// are formed by a product tree.
//
// FWHT: passes of up to 5 index bits (groups of 2^W values in registers) in
// a rotating form: a pass transforms the top W bits of the index and writes
// them at the bottom, so after passes covering all bits every element is back
// in place.
#pragma once

#include "qs_common.cuh"
#include "qs_launch.h"

namespace qs {

// ---- limits ------------------------------------------------------------------
constexpr int kXMaxStages = 16;
constexpr int kXMaxN = 32768;            // complex FFT points / FWHT points per row
constexpr int kXFine = 128;
constexpr int kXCoarse = kXMaxN / kXFine;
constexpr int kXMaxCluster = 16;
constexpr int kXMaxThreads = 512;

// ---- division by a runtime constant (x < 2^31) -------------------------------
// q = (umulhi(x, m) + x) >> l with l = ceil(log2 d), m = floor(2^32 (2^l - d) / d) + 1.
struct FastDiv {
  uint32_t d, m, l;
};

inline FastDiv make_fastdiv(uint32_t d) {
  FastDiv f;
  f.d = d;
  uint32_t l = 0;
  while ((uint64_t(1) << l) < d) ++l;
  f.l = l;
  f.m = static_cast<uint32_t>(((uint64_t(1) << 32) * ((uint64_t(1) << l) - d)) / d + 1);
  return f;
}

__device__ __forceinline__ int fdiv(int x, const FastDiv &f) {
  return static_cast<int>((__umulhi(static_cast<uint32_t>(x), f.m) + static_cast<uint32_t>(x)) >> f.l);
}

// ---- plans ----------------------------------------------------------------
struct XStage {
  int R;       // radix (FFT: 1 = copy, 2..16 powers of two, odd primes; FWHT: 2^W, 1 = copy)
  int G;       // task groups per butterfly (odd radices), else 1
  int Ns;      // FFT: product of the previous radices (FWHT: unused)
  int nb;      // butterflies: N / R
  int nbC;     // butterflies per CTA: nb / C
  int twstep;  // N / (Ns * R)
  int compact;  // odd radices in cluster kernels: 1 / 2 output pairs per task, rolled code (0: unrolled groups)
  FastDiv dNs, dnbC;
};

struct XPlan {
  int N;     // points (complex for the FFT, real for the FWHT)
  int nst;   // stages (>= 1)
  int C;     // CTAs per row (power of two, divides every stage's nb)
  int cl;    // log2(C)
  int E;     // points per CTA (N / C)
  int big;   // prime >= 11 of the FFT (0: none)
  XStage st[kXMaxStages];
};

// ---- small complex helpers -----------------------------------------------------
__device__ __forceinline__ float2 xcmul(float2 a, float2 b) {
  return make_float2(a.x * b.x - a.y * b.y, a.x * b.y + a.y * b.x);
}
__device__ __forceinline__ float2 xcadd(float2 a, float2 b) { return make_float2(a.x + b.x, a.y + b.y); }
__device__ __forceinline__ float2 xcsub(float2 a, float2 b) { return make_float2(a.x - b.x, a.y - b.y); }
__device__ __forceinline__ float2 xconj(float2 a) { return make_float2(a.x, -a.y); }

// Padded shared offsets (break the power-of-two strides of the butterflies).
__device__ __forceinline__ int xpad(int i, float2) { return i + (i >> 4); }
__device__ __forceinline__ int xpad(int i, float) { return i + (i >> 5); }
template <typename T>
__host__ __device__ constexpr int xbuf_elems(int E) {
  return sizeof(T) == 8 ? E + (E >> 4) + 1 : E + (E >> 5) + 1;
}

// ---- cluster primitives --------------------------------------------------------
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}

__device__ __forceinline__ float2 ld_dsmem(uint32_t addr, float2) {
  float2 v;
  asm volatile("ld.shared::cluster.v2.f32 {%0, %1}, [%2];" : "=f"(v.x), "=f"(v.y) : "r"(addr) : "memory");
  return v;
}
__device__ __forceinline__ float ld_dsmem(uint32_t addr, float) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
}
__device__ __forceinline__ void st_dsmem(uint32_t addr, float2 v) {
  asm volatile("st.shared::cluster.v2.f32 [%0], {%1, %2};" ::"r"(addr), "f"(v.x), "f"(v.y) : "memory");
}
__device__ __forceinline__ void st_dsmem(uint32_t addr, float v) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}

template <bool CL>
__device__ __forceinline__ void xsync() {
  if constexpr (CL) cluster_sync();
  else __syncthreads();
}

// Row layout: element e lives in CTA e & (C - 1) at local index e >> cl
// (cyclic), so a butterfly j whose inputs are j + r * nb (C divides nb) finds
// all of them in CTA j & (C - 1).  Stages read their own CTA's buffer and
// write the owners' buffers (remote stores through distributed shared memory,
// which do not stall the thread).
template <typename T, bool CL>
struct XSrc {  // elements owned by this CTA
  const T *p;
  int cl;
  __device__ __forceinline__ T operator()(int e) const { return p[xpad(CL ? (e >> cl) : e, T())]; }
};

template <typename T, bool CL>
struct XDst {  // any element: stored into its owner's buffer
  T *p;
  int cl;
  __device__ __forceinline__ void operator()(int e, T v) const {
    if constexpr (CL) {
      const uint32_t a = mapa_shared(smem_u32(p + xpad(e >> cl, T())), static_cast<uint32_t>(e & ((1 << cl) - 1)));
      st_dsmem(a, v);
    } else {
      p[xpad(e, T())] = v;
    }
  }
};

// ---- twiddles ----------------------------------------------------------------
struct XTw {
  float2 fine[kXFine];
  float2 coarse[kXCoarse];
};

__device__ __forceinline__ void build_xtw(XTw &tw, int N) {
  const int nc = (N + kXFine - 1) / kXFine;
  for (int j = threadIdx.x; j < kXFine + nc; j += blockDim.x) {
    const int e = j < kXFine ? j : (j - kXFine) * kXFine;
    float s, c;
    sincospif(2.0f * static_cast<float>(e % N) / static_cast<float>(N), &s, &c);
    if (j < kXFine) tw.fine[j] = make_float2(c, -s);
    else tw.coarse[j - kXFine] = make_float2(c, -s);
  }
}

// W_N^e (forward) or its conjugate (inverse), 0 <= e < N.
__device__ __forceinline__ float2 xtw(const XTw &tw, int e, bool inverse) {
  const float2 w = xcmul(tw.coarse[e >> 7], tw.fine[e & (kXFine - 1)]);
  return inverse ? xconj(w) : w;
}

// ---- in-register DFTs ----------------------------------------------------------
__host__ __device__ constexpr float xcos16(int k) {
  return (k & 15) == 0 ? 1.0f : (k & 15) == 1 ? 0.92387953251128674f : (k & 15) == 2 ? 0.70710678118654752f
       : (k & 15) == 3 ? 0.38268343236508977f : (k & 15) == 4 ? 0.0f : (k & 15) == 5 ? -0.38268343236508977f
       : (k & 15) == 6 ? -0.70710678118654752f : (k & 15) == 7 ? -0.92387953251128674f : (k & 15) == 8 ? -1.0f
       : (k & 15) == 9 ? -0.92387953251128674f : (k & 15) == 10 ? -0.70710678118654752f
       : (k & 15) == 11 ? -0.38268343236508977f : (k & 15) == 12 ? 0.0f : (k & 15) == 13 ? 0.38268343236508977f
       : (k & 15) == 14 ? 0.70710678118654752f : 0.92387953251128674f;
}

// Multiplies by W_16^K (forward) / W_16^-K (inverse); the K = 4 (-+i) case is a swap.
template <int K>
__device__ __forceinline__ float2 xrot16(float2 v, bool inverse) {
  constexpr int k = K & 15;
  if constexpr (k == 0) return v;
  else if constexpr (k == 4) return inverse ? make_float2(-v.y, v.x) : make_float2(v.y, -v.x);
  else {
    constexpr float cs = xcos16(k), sn = xcos16(k + 12);  // sin(2 pi k / 16)
    const float2 w = make_float2(cs, inverse ? sn : -sn);
    return xcmul(w, v);
  }
}

template <int R, int LEN, int K>
__device__ __forceinline__ void xpow2_butterflies(float2 (&v)[R], bool inverse) {
  if constexpr (K < LEN / 2) {
#pragma unroll
    for (int i = 0; i < R; i += LEN) {
      const float2 u = v[i + K];
      const float2 t = xrot16<K * (16 / LEN)>(v[i + K + LEN / 2], inverse);
      v[i + K] = xcadd(u, t);
      v[i + K + LEN / 2] = xcsub(u, t);
    }
    xpow2_butterflies<R, LEN, K + 1>(v, inverse);
  }
}

template <int R, int LEN>
__device__ __forceinline__ void xpow2_levels(float2 (&v)[R], bool inverse) {
  if constexpr (LEN <= R) {
    xpow2_butterflies<R, LEN, 0>(v, inverse);
    xpow2_levels<R, LEN * 2>(v, inverse);
  }
}

// DFT of R = 2^k points in registers (natural order in and out), radix-2 DIT.
template <int R>
__device__ __forceinline__ void xdft_pow2(float2 (&v)[R], bool inverse) {
#pragma unroll
  for (int i = 0; i < R; ++i) {
    int j = 0;
#pragma unroll
    for (int b = 1, t = i; b < R; b <<= 1, t >>= 1) j = (j << 1) | (t & 1);
    if (i < j) {
      const float2 tmp = v[i];
      v[i] = v[j];
      v[j] = tmp;
    }
  }
  xpow2_levels<R, 2>(v, inverse);
}

// ---- FFT stages ----------------------------------------------------------------
// Butterfly j of this CTA: j = rank + C * i, i < nbC.

// Power-of-two (or copy, R = 1) Stockham butterfly j: reads src[j + r*nb],
// twiddles by W_{Ns*R}^{r*k} (k = j mod Ns), transforms, writes
// dst[(j - k)*R + k + r*Ns].
// The same with the R input values already in registers (v[r] = src[j + r*nb]).
template <int R, typename Dst>
__device__ __forceinline__ void xbutterfly_pow2_vals(const XStage &S, float2 (&v)[R], const Dst &dst, const XTw &tw,
                                                     bool inverse, int j) {
  int k = 0;
  if (S.Ns > 1) {
    k = j - fdiv(j, S.dNs) * S.Ns;
    if constexpr (R > 1) {
      // powers w^r by a product tree (depth log2 R): w^r = w^(r/2) * w^(r - r/2)
      float2 pw[R];
      pw[1] = xtw(tw, k * S.twstep, inverse);
#pragma unroll
      for (int r = 2; r < R; ++r) pw[r] = xcmul(pw[r / 2], pw[r - r / 2]);
#pragma unroll
      for (int r = 1; r < R; ++r) v[r] = xcmul(v[r], pw[r]);
    }
  }
  if constexpr (R > 1) xdft_pow2<R>(v, inverse);
  const int base = (j - k) * R + k;
#pragma unroll
  for (int r = 0; r < R; ++r) dst(base + r * S.Ns, v[r]);
}

template <int R, typename Src, typename Dst>
__device__ __forceinline__ void xbutterfly_pow2(const XStage &S, const Src &src, const Dst &dst, const XTw &tw,
                                                bool inverse, int j) {
  float2 v[R];
#pragma unroll
  for (int r = 0; r < R; ++r) v[r] = src(j + r * S.nb);
  xbutterfly_pow2_vals<R>(S, v, dst, tw, inverse, j);
}

// Stage over this CTA's butterflies j = rank + C * i, i < nbC.
template <int R, typename Src, typename Dst>
__device__ __forceinline__ void xstage_pow2(const XStage &S, const Src &src, const Dst &dst, const XTw &tw,
                                            bool inverse, int rank, int C) {
  for (int i = threadIdx.x; i < S.nbC; i += blockDim.x) xbutterfly_pow2<R>(S, src, dst, tw, inverse, rank + C * i);
}

__host__ __device__ constexpr int xodd_groups(int P) {
  return ((P - 1) / 2 + 5) / 6;  // at most 6 output pairs per task
}
__host__ __device__ constexpr int xodd_per(int P) {
  return ((P - 1) / 2 + xodd_groups(P) - 1) / xodd_groups(P);
}

// Writes the outputs of output group (klo .. klo + per - 1) of an odd-prime
// butterfly: X_k = A - iB, X_{P-k} = A + iB (forward; swapped for the inverse).
template <int P, typename Dst>
__device__ __forceinline__ void xodd_store(const Dst &dst, int base, int Ns, int klo, const float2 (&A)[xodd_per(P)],
                                           const float2 (&B)[xodd_per(P)], bool inverse) {
  constexpr int H = (P - 1) / 2;
#pragma unroll
  for (int q = 0; q < xodd_per(P); ++q) {
    const int kk = klo + q;
    if (kk <= H) {
      const float2 miB = make_float2(B[q].y, -B[q].x);  // -iB
      dst(base + kk * Ns, inverse ? xcsub(A[q], miB) : xcadd(A[q], miB));
      dst(base + (P - kk) * Ns, inverse ? xcadd(A[q], miB) : xcsub(A[q], miB));
    }
  }
}

// Output group g of butterfly j, fully unrolled: cos / sin are compile-time
// constant-bank operands (throughput variant, one CTA per row).
template <int P, int g, typename Src, typename Dst>
__device__ __forceinline__ void xodd_group_unrolled(const XStage &S, const Src &src, const Dst &dst, int j, int k,
                                                    float2 w1, float2 wP, bool tw_on, bool inverse) {
  constexpr int H = (P - 1) / 2;
  constexpr int per = xodd_per(P);
  constexpr int klo = g * per + 1;
  constexpr int off = prime_offset(P);
  const float2 x0 = src(j);
  float2 A[per], B[per];
#pragma unroll
  for (int q = 0; q < per; ++q) {
    A[q] = x0;
    B[q] = make_float2(0.f, 0.f);
  }
  float2 s0 = x0;
  float2 tr = w1;
#pragma unroll
  for (int r = 1; r <= H; ++r) {
    float2 xa = src(j + r * S.nb), xb = src(j + (P - r) * S.nb);
    if (tw_on) {
      if (r > 1) tr = xcmul(tr, w1);
      xa = xcmul(xa, tr);
      xb = xcmul(xb, xcmul(wP, xconj(tr)));
    }
    const float2 a = xcadd(xa, xb), b = xcsub(xa, xb);
    if constexpr (g == 0) s0 = xcadd(s0, a);
#pragma unroll
    for (int q = 0; q < per; ++q) {
      if (klo + q <= H) {
        const float c = kDftCos[off + (r * (klo + q)) % P];
        const float s = kDftSin[off + (r * (klo + q)) % P];
        A[q].x = fmaf(a.x, c, A[q].x);
        A[q].y = fmaf(a.y, c, A[q].y);
        B[q].x = fmaf(b.x, s, B[q].x);
        B[q].y = fmaf(b.y, s, B[q].y);
      }
    }
  }
  const int base = (j - k) * P + k;
  xodd_store<P>(dst, base, S.Ns, klo, A, B, inverse);
  if constexpr (g == 0) dst(base, s0);
}

template <int P, int g, typename Src, typename Dst>
__device__ __forceinline__ void xodd_dispatch(int gi, const XStage &S, const Src &src, const Dst &dst, int j,
                                              int k, float2 w1, float2 wP, bool tw_on, bool inverse) {
  if constexpr (g < xodd_groups(P)) {
    if (gi == g) xodd_group_unrolled<P, g>(S, src, dst, j, k, w1, wP, tw_on, inverse);
    else xodd_dispatch<P, g + 1>(gi, S, src, dst, j, k, w1, wP, tw_on, inverse);
  }
}

// Output pairs k = g*PER + 1 .. g*PER + PER of butterfly j, compact: the
// loop over the inputs is rolled (by 3) and cos / sin come from the constant
// table (latency variant: a cluster per row runs this code once, so its
// length and the per-thread dependency chain, not the instruction count, set
// the time).
template <int P, int PER, typename Src, typename Dst>
__device__ __forceinline__ void xodd_pairs_compact(int g, const XStage &S, const Src &src, const Dst &dst, int j,
                                                   int k, float2 w1, float2 wP, bool tw_on, bool inverse) {
  constexpr int H = (P - 1) / 2;
  constexpr int off = prime_offset(P);
  const int klo = g * PER + 1;
  const float2 x0 = src(j);
  float2 A[PER], B[PER];
  int idx[PER];
#pragma unroll
  for (int q = 0; q < PER; ++q) {
    A[q] = x0;
    B[q] = make_float2(0.f, 0.f);
    idx[q] = 0;
  }
  float2 s0 = x0, tr = w1;
#pragma unroll 3
  for (int r = 1; r <= H; ++r) {
    float2 xa = src(j + r * S.nb), xb = src(j + (P - r) * S.nb);
    if (tw_on) {
      if (r > 1) tr = xcmul(tr, w1);
      xa = xcmul(xa, tr);
      xb = xcmul(xb, xcmul(wP, xconj(tr)));
    }
    const float2 a = xcadd(xa, xb), b = xcsub(xa, xb);
    if (g == 0) s0 = xcadd(s0, a);
#pragma unroll
    for (int q = 0; q < PER; ++q) {
      idx[q] += klo + q;  // (r * k) mod P, kept incrementally (k > H only in a partial last group)
      if (idx[q] >= P) idx[q] -= P;
      const float c = kDftCos[off + idx[q]];
      const float sn = kDftSin[off + idx[q]];
      A[q].x = fmaf(a.x, c, A[q].x);
      A[q].y = fmaf(a.y, c, A[q].y);
      B[q].x = fmaf(b.x, sn, B[q].x);
      B[q].y = fmaf(b.y, sn, B[q].y);
    }
  }
  const int base = (j - k) * P + k;
#pragma unroll
  for (int q = 0; q < PER; ++q) {
    const int kk = klo + q;
    if (kk <= H) {
      const float2 miB = make_float2(B[q].y, -B[q].x);  // -iB
      dst(base + kk * S.Ns, inverse ? xcsub(A[q], miB) : xcadd(A[q], miB));
      dst(base + (P - kk) * S.Ns, inverse ? xcadd(A[q], miB) : xcsub(A[q], miB));
    }
  }
  if (g == 0) dst(base, s0);
}

// Odd-prime stage: task t = g * nbC + i (output group g of butterfly
// j = rank + C * i; compact plans: output pairs g*PER + 1 .. g*PER + PER);
// tasks of a warp share g except at group boundaries.
template <int P, bool COMPACT, typename Src, typename Dst>
__device__ __forceinline__ void xstage_odd(const XStage &S, const Src &src, const Dst &dst, const XTw &tw,
                                           bool inverse, int rank, int C) {
  const int tasks = S.nbC * S.G;
  for (int t = threadIdx.x; t < tasks; t += blockDim.x) {
    const int g = fdiv(t, S.dnbC);
    const int j = rank + C * (t - g * S.nbC);
    int k = 0;
    float2 w1 = make_float2(1.f, 0.f), wP = w1;
    const bool tw_on = S.Ns > 1;
    if (tw_on) {
      k = j - fdiv(j, S.dNs) * S.Ns;
      w1 = xtw(tw, k * S.twstep, inverse);
      wP = xtw(tw, k * S.twstep * P, inverse);
    }
    // compact code only in cluster kernels and only when the plan asks for it (few rows)
    if (COMPACT && S.compact == 1) xodd_pairs_compact<P, 1>(g, S, src, dst, j, k, w1, wP, tw_on, inverse);
    else if (COMPACT && S.compact == 2) xodd_pairs_compact<P, 2>(g, S, src, dst, j, k, w1, wP, tw_on, inverse);
    else xodd_dispatch<P, 0>(g, S, src, dst, j, k, w1, wP, tw_on, inverse);
  }
}

// First stage of a compact plan (few rows in a cluster) with an odd radix P,
// straight from global memory: output pairs g*PER + 1 .. g*PER + PER (and the
// DC term for g == 0) of butterfly j.  All P inputs are loaded into registers
// at once (independent loads, one memory latency); the stage has no twiddles
// (Ns = 1), so output k of butterfly j lands at j * P + k.
template <int P, int PER, typename GSrc, typename Dst>
__device__ __forceinline__ void xodd_first_pairs(int g, int nb, const GSrc &gsrc, const Dst &dst, int j,
                                                 bool inverse) {
  constexpr int H = (P - 1) / 2;
  constexpr int off = prime_offset(P);
  const float2 x0 = gsrc(j);
  float2 a[H], b[H];
#pragma unroll
  for (int r = 1; r <= H; ++r) {
    const float2 xa = gsrc(j + r * nb), xb = gsrc(j + (P - r) * nb);
    a[r - 1] = xcadd(xa, xb);
    b[r - 1] = xcsub(xa, xb);
  }
  const int base = j * P;
  if (g == 0) {
    float2 s0 = x0, s1 = make_float2(0.f, 0.f);
#pragma unroll
    for (int r = 0; r < H; ++r) {
      if (r & 1) s1 = xcadd(s1, a[r]);
      else s0 = xcadd(s0, a[r]);
    }
    dst(base, xcadd(s0, s1));
  }
#pragma unroll
  for (int q = 0; q < PER; ++q) {
    const int kk = g * PER + 1 + q;
    if (kk <= H) {
      float2 A = x0, B = make_float2(0.f, 0.f);
      int idx = 0;
#pragma unroll
      for (int r = 0; r < H; ++r) {
        idx += kk;  // (r + 1) * kk mod P
        if (idx >= P) idx -= P;
        const float c = kDftCos[off + idx], sn = kDftSin[off + idx];
        A.x = fmaf(a[r].x, c, A.x);
        A.y = fmaf(a[r].y, c, A.y);
        B.x = fmaf(b[r].x, sn, B.x);
        B.y = fmaf(b[r].y, sn, B.y);
      }
      const float2 miB = make_float2(B.y, -B.x);  // -iB
      dst(base + kk, inverse ? xcsub(A, miB) : xcadd(A, miB));
      dst(base + P - kk, inverse ? xcadd(A, miB) : xcsub(A, miB));
    }
  }
}

template <int P, typename GSrc, typename Dst>
__device__ __forceinline__ void xodd_first_tasks(const XStage &S, const GSrc &gsrc, const Dst &dst, bool inverse,
                                                 int rank, int C) {
  const int tasks = S.nbC * S.G;
  for (int t = threadIdx.x; t < tasks; t += blockDim.x) {
    const int g = fdiv(t, S.dnbC);
    const int j = rank + C * (t - g * S.nbC);
    if (S.compact == 1) xodd_first_pairs<P, 1>(g, S.nb, gsrc, dst, j, inverse);
    else xodd_first_pairs<P, 2>(g, S.nb, gsrc, dst, j, inverse);
  }
}

// First stage of a compact plan with the prime P >= 11, straight from global
// memory: a warp per butterfly (column j, inputs j + r * nb), lane k computing
// output pair k (lane 0 the DC term).  Lane l loads inputs l and l + 32; the
// conjugate-pair sums a_r = x_r + x_{P-r}, b_r = x_r - x_{P-r} (one shuffle)
// are staged in a per-warp slot of `stage` as float4 (a_r, b_r), slot 0 = x0,
// and read back as broadcasts.  A warp issues the loads of up to 4 butterflies
// first, then forms its lane's H cos / sin coefficients by rotation
// (w^r = w^(r-1) * w, w = exp(2 pi i k / P)) while they are in flight.
template <int P, typename GSrc, typename Dst>
__device__ __forceinline__ void xbig_first_stage(const XStage &S, const GSrc &gsrc, const Dst &dst, float2 *stage,
                                                 int stage_cap, bool inverse, int rank, int C) {
  constexpr int H = (P - 1) / 2;
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int nb = S.nb, nbC = S.nbC;
  int nw = blockDim.x >> 5;
  if (nw * (H + 1) * 2 > stage_cap) nw = stage_cap / (2 * (H + 1));  // warps whose slots fit
  if (w >= nw) return;
  float4 *st = reinterpret_cast<float4 *>(stage) + w * (H + 1);
  const int src = (P - lane) & 31;              // lane holding x_{P - lane}
  const bool hi = lane >= 1 && P - lane >= 32;  // ... in its second register
  float cr[H], sr[H];
  for (int c0 = w; c0 < nbC; c0 += 4 * nw) {
    float2 v0[4], v1[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int ci = c0 + q * nw;
      v0[q] = v1[q] = make_float2(0.f, 0.f);
      if (ci < nbC) {
        const int j = rank + C * ci;
        if (lane < P) v0[q] = gsrc(j + lane * nb);
        if (lane + 32 < P) v1[q] = gsrc(j + (lane + 32) * nb);
      }
    }
    if (c0 == w) {
      // cos / sin (2 pi r k / P), r = 1..H, of this lane's pair k (lanes above H: k = 0, unused)
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
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int ci = c0 + q * nw;
      if (ci >= nbC) break;  // warp-uniform
      const float2 u0 = make_float2(__shfl_sync(0xffffffffu, v0[q].x, src), __shfl_sync(0xffffffffu, v0[q].y, src));
      const float2 u1 = make_float2(__shfl_sync(0xffffffffu, v1[q].x, src), __shfl_sync(0xffffffffu, v1[q].y, src));
      const float2 xm = hi ? u1 : u0;
      if (lane == 0) {
        st[0] = make_float4(v0[q].x, v0[q].y, 0.f, 0.f);
      } else if (lane <= H) {
        st[lane] = make_float4(v0[q].x + xm.x, v0[q].y + xm.y, v0[q].x - xm.x, v0[q].y - xm.y);
      }
      __syncwarp();
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
      __syncwarp();  // the slot is rewritten by the next butterfly
      const int base = (rank + C * ci) * P;
      if (lane == 0) {
        dst(base, A);  // k = 0: every coefficient is 1
      } else if (lane <= H) {
        const float2 miB = make_float2(B.y, -B.x);  // -iB
        dst(base + lane, inverse ? xcsub(A, miB) : xcadd(A, miB));
        dst(base + P - lane, inverse ? xcadd(A, miB) : xcsub(A, miB));
      }
    }
  }
}

// The same stage with the row read coalesced: this CTA takes the contiguous
// butterflies [rank * nbC, (rank + 1) * nbC) (any split works: the stage reads
// global memory and stores to the owners), its threads load (x_r, x_{P-r})
// with consecutive lanes on consecutive butterflies and stage (a_r, b_r) as a
// float4 tile [r][butterfly] (row 0: x0), a CTA barrier, then a warp per
// butterfly reads the tile as broadcasts.  The tile, (H + 1) * nbC float4,
// fits the row buffer when P >= 17.
template <int P, typename GSrc, typename Dst>
__device__ __forceinline__ void xbig_first_stage_tiled(const XStage &S, const GSrc &gsrc, const Dst &dst,
                                                       float2 *stage, bool inverse, int rank) {
  constexpr int H = (P - 1) / 2;
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const int nb = S.nb, nbC = S.nbC, j0 = rank * nbC;
  float4 *tile = reinterpret_cast<float4 *>(stage);
  const int items = (H + 1) * nbC;
  // loads of this thread's (r, butterfly) items, all issued before any use (at most 4 per thread)
  for (int i0 = threadIdx.x; i0 < items; i0 += 4 * blockDim.x) {
    float2 xa[4], xb[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int i = i0 + u * blockDim.x;
      xa[u] = xb[u] = make_float2(0.f, 0.f);
      if (i < items) {
        const int r = fdiv(i, S.dnbC), c = i - r * nbC;
        xa[u] = gsrc(j0 + c + r * nb);
        if (r > 0) xb[u] = gsrc(j0 + c + (P - r) * nb);
      }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int i = i0 + u * blockDim.x;
      if (i < items) {
        tile[i] = i < nbC ? make_float4(xa[u].x, xa[u].y, 0.f, 0.f)
                          : make_float4(xa[u].x + xb[u].x, xa[u].y + xb[u].y, xa[u].x - xb[u].x, xa[u].y - xb[u].y);
      }
    }
  }
  // cos / sin (2 pi r k / P), r = 1..H, of this lane's pair k = lane (lanes above H: k = 0, unused)
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
  __syncthreads();
  for (int c = w; c < nbC; c += nw) {
    const float4 x0 = tile[c];
    float2 A = make_float2(x0.x, x0.y), A2 = make_float2(0.f, 0.f), B = A2, B2 = A2;
#pragma unroll
    for (int r = 0; r < H; ++r) {
      const float4 ab = tile[(1 + r) * nbC + c];
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
    const int base = (j0 + c) * P;
    if (lane == 0) {
      dst(base, A);  // k = 0: every coefficient is 1
    } else if (lane <= H) {
      const float2 miB = make_float2(B.y, -B.x);  // -iB
      dst(base + lane, inverse ? xcsub(A, miB) : xcadd(A, miB));
      dst(base + P - lane, inverse ? xcadd(A, miB) : xcsub(A, miB));
    }
  }
}

// Odd first stage of a compact plan: radix 5 / 7 as output-pair tasks, the
// plan's prime >= 11 a warp per butterfly (`stage`: stage_cap float2 of
// scratch in this CTA's shared memory, 16-byte aligned).
template <int BIG, typename GSrc, typename Dst>
__device__ __forceinline__ void xstage_odd_first(const XStage &S, const GSrc &gsrc, const Dst &dst, float2 *stage,
                                                 int stage_cap, bool inverse, int rank, int C) {
  if (S.R == 5) xodd_first_tasks<5>(S, gsrc, dst, inverse, rank, C);
  else if (S.R == 7) xodd_first_tasks<7>(S, gsrc, dst, inverse, rank, C);
  else if constexpr (BIG != 0) {
    if (2 * ((BIG + 1) / 2) * S.nbC <= stage_cap) xbig_first_stage_tiled<BIG>(S, gsrc, dst, stage, inverse, rank);
    else xbig_first_stage<BIG>(S, gsrc, dst, stage, stage_cap, inverse, rank, C);
  }
}

// One stage, any radix of the plan (the prime >= 11 only as stage 0, odd radices
// never last: the host plan guarantees both).
template <int BIG, bool COMPACT, bool FIRST, bool LAST, typename Src, typename Dst>
__device__ __forceinline__ void xfft_stage(const XStage &S, const Src &src, const Dst &dst, const XTw &tw,
                                           bool inverse, int rank, int C) {
  switch (S.R) {
    case 1: xstage_pow2<1>(S, src, dst, tw, inverse, rank, C); break;
    case 2: xstage_pow2<2>(S, src, dst, tw, inverse, rank, C); break;
    case 4: xstage_pow2<4>(S, src, dst, tw, inverse, rank, C); break;
    case 8: xstage_pow2<8>(S, src, dst, tw, inverse, rank, C); break;
    case 16: xstage_pow2<16>(S, src, dst, tw, inverse, rank, C); break;
    default:
      if constexpr (!LAST) {
        if (S.R == 3) xstage_odd<3, COMPACT>(S, src, dst, tw, inverse, rank, C);
        else if (S.R == 5) xstage_odd<5, COMPACT>(S, src, dst, tw, inverse, rank, C);
        else if (S.R == 7) xstage_odd<7, COMPACT>(S, src, dst, tw, inverse, rank, C);
        else if constexpr (FIRST && BIG != 0) xstage_odd<BIG, COMPACT>(S, src, dst, tw, inverse, rank, C);
      }
      break;
  }
}

// Power-of-two (or copy) stage only: the first stage when it reads global memory.
template <bool CL, typename Src, typename Dst>
__device__ __forceinline__ void xfft_stage_pow2(const XStage &S, const Src &src, const Dst &dst, const XTw &tw,
                                                bool inverse, int rank, int C) {
  switch (S.R) {
    case 1: xstage_pow2<1>(S, src, dst, tw, inverse, rank, C); break;
    case 2: xstage_pow2<2>(S, src, dst, tw, inverse, rank, C); break;
    case 4: xstage_pow2<4>(S, src, dst, tw, inverse, rank, C); break;
    case 8: xstage_pow2<8>(S, src, dst, tw, inverse, rank, C); break;
    case 16: xstage_pow2<16>(S, src, dst, tw, inverse, rank, C); break;
    default: break;
  }
}

// Loads the row into buffer 0: this CTA reads the contiguous range
// [rank * E, (rank + 1) * E) (coalesced, U loads in flight per thread) and
// stores each element into its owner's buffer.
template <int U, typename T, typename GSrc, typename Dst>
__device__ __forceinline__ void xload_row(const GSrc &gsrc, const Dst &dst, int E, int rank) {
  const int e0 = rank * E;
  for (int base = threadIdx.x; base < E; base += U * blockDim.x) {
    T v[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int i = base + u * blockDim.x;
      if (i < E) v[u] = gsrc(e0 + i);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int i = base + u * blockDim.x;
      if (i < E) dst(e0 + i, v[u]);
    }
  }
}

// Unnormalised DFT of the row (forward exp(-2 pi i jk/N), inverse exp(+...)):
// gsrc(e) -> sink(e, v).  Group barriers separate the load pass and the
// stages; ends after the last stage's stores, without a barrier (the last stage
// reads only this CTA's own buffer, so no peer touches it afterwards).
template <int BIG, bool CL, typename GSrc, typename Sink>
__device__ __forceinline__ void xfft_row(const XPlan &p, float2 *buf0, float2 *buf1, const XTw &tw, bool inverse,
                                         int rank, const GSrc &gsrc, const Sink &sink) {
  const XDst<float2, CL> d0{buf0, p.cl}, d1{buf1, p.cl};
  // A power-of-two first stage reads the row straight from global memory (its
  // R loads per thread are independent), and so does an odd first stage of a
  // compact plan (each butterfly's P inputs loaded at once; buf0, unused until
  // stage 1, stages the prime's conjugate-pair sums); other odd first stages
  // (unrolled groups that consume their inputs one pair at a time) read a
  // shared copy made by a coalesced load pass.  Odd radices are never last, so
  // a one-stage plan is a power of two or a copy.
  const XStage &S0 = p.st[0];
  const bool odd0 = (S0.R & 1) && S0.R > 1;
  if (p.nst == 1) {
    xfft_stage_pow2<CL>(S0, gsrc, sink, tw, inverse, rank, p.C);
    return;
  }
  if (!odd0) {
    xfft_stage_pow2<CL>(S0, gsrc, d1, tw, inverse, rank, p.C);
  } else if (S0.compact) {
    xstage_odd_first<BIG>(S0, gsrc, d1, buf0, xbuf_elems<float2>(p.E), inverse, rank, p.C);
  } else {
    xload_row<8, float2>(gsrc, d0, p.E, rank);
    xsync<CL>();
    xfft_stage<BIG, CL, true, false>(S0, XSrc<float2, CL>{buf0, p.cl}, d1, tw, inverse, rank, p.C);
  }
  xsync<CL>();
  // Middle stages share one copy of the stage code (buffers picked at run
  // time): a stage whose radix an earlier stage had runs from a warm
  // instruction cache.
  for (int s = 1; s + 1 < p.nst; ++s) {
    const XSrc<float2, CL> si{(s & 1) ? buf1 : buf0, p.cl};
    const XDst<float2, CL> di{(s & 1) ? buf0 : buf1, p.cl};
    xfft_stage<BIG, CL, false, false>(p.st[s], si, di, tw, inverse, rank, p.C);
    xsync<CL>();
  }
  const XSrc<float2, CL> sl{((p.nst - 1) & 1) ? buf1 : buf0, p.cl};
  xfft_stage<BIG, CL, false, true>(p.st[p.nst - 1], sl, sink, tw, inverse, rank, p.C);
}

// Buffer the last stage reads (the other one receives its results when the
// sink is a buffer): stage s >= 1 reads buffer (s + 1) & 1 ... stage 0 reads
// global memory or, after the load pass, buffer 0.
__device__ __forceinline__ int xresult_buf(const XPlan &p) {
  if (p.nst == 1) return 1;
  return (p.nst - 1) & 1 ? 0 : 1;
}

// ---- FWHT passes ------------------------------------------------------------
// Pass of W bits on the top of the index, rotating them to the bottom:
// butterfly j reads src[j + r*nb] (r < 2^W), writes dst[j*2^W + r].  After
// passes whose widths sum to log2(N) every bit has been transformed once and
// rotated back to its place.
template <int W, typename Src, typename Dst>
__device__ __forceinline__ void xfwht_pass(const XStage &S, const Src &src, const Dst &dst, int rank, int C) {
  constexpr int R = 1 << W;
  for (int i = threadIdx.x; i < S.nbC; i += blockDim.x) {
    const int j = rank + C * i;
    float v[R];
#pragma unroll
    for (int r = 0; r < R; ++r) v[r] = src(j + r * S.nb);
#pragma unroll
    for (int h = 1; h < R; h <<= 1) {
#pragma unroll
      for (int q = 0; q < R; ++q) {
        if (!(q & h)) {
          const float a = v[q], b = v[q + h];
          v[q] = a + b;
          v[q + h] = a - b;
        }
      }
    }
#pragma unroll
    for (int r = 0; r < R; ++r) dst(j * R + r, v[r]);
  }
}

template <typename Src, typename Dst>
__device__ __forceinline__ void xfwht_stage(const XStage &S, const Src &src, const Dst &dst, int rank, int C) {
  switch (S.R) {
    case 1: xfwht_pass<0>(S, src, dst, rank, C); break;
    case 2: xfwht_pass<1>(S, src, dst, rank, C); break;
    case 4: xfwht_pass<2>(S, src, dst, rank, C); break;
    case 8: xfwht_pass<3>(S, src, dst, rank, C); break;
    case 16: xfwht_pass<4>(S, src, dst, rank, C); break;
    case 32: xfwht_pass<5>(S, src, dst, rank, C); break;
    default: break;
  }
}

// Unnormalised Walsh-Hadamard transform of the row gsrc(i) -> sink(i, v).
template <bool CL, typename GSrc, typename Sink>
__device__ __forceinline__ void xfwht_row(const XPlan &p, float *buf0, float *buf1, int rank, const GSrc &gsrc,
                                          const Sink &sink) {
  const XDst<float, CL> d1{buf1, p.cl};
  if (p.nst == 1) {  // the first pass reads global memory directly
    xfwht_stage(p.st[0], gsrc, sink, rank, p.C);
    return;
  }
  xfwht_stage(p.st[0], gsrc, d1, rank, p.C);
  xsync<CL>();
  for (int s = 1; s + 1 < p.nst; ++s) {  // one copy of the pass code for all middle passes
    const XSrc<float, CL> si{(s & 1) ? buf1 : buf0, p.cl};
    const XDst<float, CL> di{(s & 1) ? buf0 : buf1, p.cl};
    xfwht_stage(p.st[s], si, di, rank, p.C);
    xsync<CL>();
  }
  const XSrc<float, CL> sl{((p.nst - 1) & 1) ? buf1 : buf0, p.cl};
  xfwht_stage(p.st[p.nst - 1], sl, sink, rank, p.C);
}

// ---- row epilogue of the linear input step ------------------------------------------
// Row |max| over the group: block reduction, then (cluster) every CTA posts its
// value into every CTA's slot table.  Ends with a group barrier, after which
// every remote store made before it is visible.
template <bool CL>
__device__ __forceinline__ float xgroup_absmax(float v, float *red, float *slots, int rank, int C) {
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int w = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  if ((threadIdx.x & 31) == 0) red[w] = v;
  __syncthreads();
  float r = 0.f;
  for (int i = 0; i < nw; ++i) r = fmaxf(r, red[i]);
  if constexpr (CL) {
    if (static_cast<int>(threadIdx.x) < C) st_dsmem(mapa_shared(smem_u32(slots + rank), threadIdx.x), r);
    cluster_sync();
    r = 0.f;
    for (int i = 0; i < C; ++i) r = fmaxf(r, slots[i]);
  }
  return r;
}

__device__ __forceinline__ void xpow2_scale(float amax, float &scale, float &inv) {
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

// Zeroes floats [z0, z1) of row `row` of the (rows, m) matrix y1 with this
// CTA's threads (16-byte stores when the row is 16-byte aligned).
__device__ __forceinline__ void xzero_row(float *y1, int64_t row, int64_t m, int64_t z0, int64_t z1) {
  float *r = y1 + row * m;
  if ((m & 3) == 0 && (reinterpret_cast<uintptr_t>(y1) & 15) == 0) {
    const int v0 = static_cast<int>((z0 + 3) >> 2), v1 = static_cast<int>(z1 >> 2);
    float4 *r4 = reinterpret_cast<float4 *>(r);
    for (int i = v0 + threadIdx.x; i < v1; i += blockDim.x) r4[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int i = static_cast<int>(z0) + threadIdx.x; i < v0 * 4 && i < z1; i += blockDim.x) r[i] = 0.f;
    for (int i = v1 * 4 + threadIdx.x; i < z1; i += blockDim.x) r[i] = 0.f;
  } else {
    for (int i = static_cast<int>(z0) + threadIdx.x; i < z1; i += blockDim.x) r[i] = 0.f;
  }
}

// Few rows: pulls a layer constant (phases, signs, bias; never written by the
// previous kernel) into L2 before the kernel waits for its predecessor, so its
// HBM latency overlaps the wait.  The group's C CTAs split the 128-byte lines.
__device__ __forceinline__ void xprefetch_l2(const void *p, int64_t bytes, int rank, int C) {
  if (!p) return;
  const char *c = static_cast<const char *>(p);
  const int64_t step = static_cast<int64_t>(C) * blockDim.x * 128;
  for (int64_t o = (static_cast<int64_t>(rank) * blockDim.x + threadIdx.x) * 128; o < bytes; o += step)
    asm volatile("prefetch.global.L2 [%0];" ::"l"(c + o));
}

// Offset of y1 element (row, col): plain row-major with stride ld_y1 when
// shards == 1, else the rank-major layout of an all-gather of `shards` column
// blocks of (batch, mp): ((col / mp) * batch + row) * mp + col % mp.
__device__ __forceinline__ int64_t xy1_offset(int64_t row, int64_t col, int64_t ld_y1, int64_t shards,
                                              int64_t mp, int64_t batch) {
  if (shards == 1) return row * ld_y1 + col;
  return ((col / mp) * batch + row) * mp + col % mp;
}

// ---- kernels -----------------------------------------------------------------
// Grid: CL ? (C, rows) with cluster (C, 1, 1) : (rows).  Dynamic shared memory:
// two buffers of xbuf_elems<T>(E) elements.  A cluster needs no barrier before
// exit: after the row transform's last barrier every CTA reads only its own
// buffers (and, in the input kernels, the group reduction ends with a barrier).
// Output step of a column-sharded layer whose y1 shards every rank pushed into
// this rank's receive buffer (tensor parallelism over peer memory): the call's
// parity region base + (seq & 1) * stride holds the rank-major gathered layout
// of xy1_offset, seq being the call's sequence number.  Flagged format: plain
// floats, complete once every flags[(seq & 1) * nflags + r] has reached seq
// (set by rank r after its pushed data, system-scope release).  Word format
// (words = 1): value i is the 8-byte word i {float bits, seq of the call that
// wrote it}, valid once its seq matches.  flags == null: y1 is the kernel's y1
// argument.
constexpr int kMaxPeers = 8;
struct XPeerGather {
  const float *base;     // this rank's receive buffer (parity region 0): gathered rank-major shards
  int64_t stride;        // floats between the two parity regions
  const int *flags;       // this rank's arrival flags, int32 [2][nflags]
  const unsigned *seq;    // this rank's call sequence number (written by its push)
  int nflags;
  int words;              // 1: self-validating 8-byte words, no flags
  uint64_t wait_ns;
  int *error;  // set when a wait ran out
};

// Where an output step reads y1 from: the kernel's own y1 (plain floats) or a
// receive region.  In word format value i is word i: base[2 i] holds its bits
// and base[2 i + 1] the call number.  The decode-batch row kernels verify a
// thread's words with batched loads before plain reads (verify, get); the
// general row engine waits per word where it reads (get_wait).  A reader that gives up (wait limit)
// stops waiting and the error flag tells the host the output is invalid.
struct XPeerSrc {
  const float *base;
  unsigned seq;
  int words;
  uint64_t wait_ns;
  int *error;

  __device__ __forceinline__ bool expired(uint64_t &t0, bool &dead) const {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    if (!t0) t0 = t;
    if (t - t0 <= wait_ns) return false;
    atomicExch(error, 1);
    dead = true;
    return true;
  }
  // word i, loaded without waiting: {bits, call number}
  __device__ __forceinline__ uint2 load_word(int64_t i) const {
    uint2 w;
    asm volatile("ld.volatile.global.v2.u32 {%0, %1}, [%2];" : "=r"(w.x), "=r"(w.y) : "l"(base + 2 * i) : "memory");
    return w;
  }
  // waits (bounded) until word i holds this call; returns its value
  __device__ __forceinline__ float wait_word(int64_t i, uint2 w, bool &dead) const {
    uint64_t t0 = 0;
    while (w.y != seq && !dead && !expired(t0, dead)) w = load_word(i);
    return dead ? 0.f : __uint_as_float(w.x);
  }
  // Word format: waits until the words off(r) (and off(r) + 1 with pair), r < R,
  // hold this call.  The call-number halves of up to 16 values are loaded
  // together; only words not yet arrived are waited on.
  template <int R, typename Off>
  __device__ __forceinline__ void verify(Off off, bool pair) const {
    constexpr int kChunk = R < 16 ? R : 16;
    bool dead = false;
#pragma unroll 1
    for (int r0 = 0; r0 < R; r0 += kChunk) {
      uint32_t miss = 0;
#pragma unroll
      for (int j = 0; j < kChunk; ++j) {
        const float *w = base + 2 * off(r0 + j);
        uint32_t s0, s1 = seq;
        asm volatile("ld.volatile.global.u32 %0, [%1];" : "=r"(s0) : "l"(w + 1) : "memory");
        if (pair) asm volatile("ld.volatile.global.u32 %0, [%1];" : "=r"(s1) : "l"(w + 3) : "memory");
        if (s0 != seq || s1 != seq) miss |= 1u << j;
      }
      if (!miss) continue;
      const uint2 stale = make_uint2(0u, seq + 1u);  // forces a fresh load
#pragma unroll
      for (int j = 0; j < kChunk; ++j)
        if ((miss >> j) & 1u) {
          wait_word(off(r0 + j), stale, dead);
          if (pair) wait_word(off(r0 + j) + 1, stale, dead);
        }
    }
  }
  // value i of the word format, waiting (bounded) for its word
  __device__ __forceinline__ float get_wait(int64_t i, bool &dead) const {
    if (!base || dead) return 0.f;
    return wait_word(i, load_word(i), dead);
  }
  __device__ __forceinline__ float2 get2_wait(int64_t i, bool &dead) const {  // i even
    const float x = get_wait(i, dead);
    return make_float2(x, get_wait(i + 1, dead));
  }
  // value i (plain floats, or a verified word, read from L2); no base: zeros
  __device__ __forceinline__ float get(int64_t i) const {
    if (!base) return 0.f;
    return words ? __ldcg(base + 2 * i) : base[i];
  }
  __device__ __forceinline__ float2 get2(int64_t i) const {  // values i, i + 1 (i even)
    if (!base) return make_float2(0.f, 0.f);
    if (!words) return *reinterpret_cast<const float2 *>(base + i);
    const float4 q = __ldcg(reinterpret_cast<const float4 *>(base + 2 * i));
    return make_float2(q.x, q.z);
  }
};

__device__ __forceinline__ XPeerSrc xplain_src(const float *y1) { return XPeerSrc{y1, 0u, 0, 0, nullptr}; }

struct XRowArgs {
  int64_t row_base;
  int C;
  int early;  // release the dependent kernel at the start (few rows) or only at exit (many rows)
  int warm;   // input kernels, one CTA per row: may run a dry pass before waiting (see xinput_rfft_kernel)
  int *busy;  // device flag: set while a few-row output step runs (a hint, see xbusy_flag)
  XPeerGather pg;
};

// The receive region of this call (every thread of the CTA calls it).  The
// call's sequence number was written by this rank's push, complete before the
// caller's pdl_wait returned.  Flagged format: waits (thread 0, bounded) until
// every rank's flag of this call is set, else gives up (error flag set, base
// null: zeros are read).  Word format: no wait here; the reads wait per word.
__device__ __forceinline__ XPeerSrc xwait_peers(const XPeerGather &pg) {
  __shared__ int s_ok;
  __shared__ unsigned s_seq;
  if (threadIdx.x == 0) {
    const unsigned seq = *reinterpret_cast<const volatile unsigned *>(pg.seq);
    bool ok = true;
    if (!pg.words) {
      const int *fl = pg.flags + static_cast<int>(seq & 1u) * pg.nflags;
      uint64_t t0 = 0;
      for (int r = 0; r < pg.nflags && ok; ++r) {
        for (;;) {
          int v;
          asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(fl + r) : "memory");
          if (static_cast<int>(static_cast<unsigned>(v) - seq) >= 0) break;
          uint64_t t;
          asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
          if (!t0) t0 = t;
          if (t - t0 > pg.wait_ns) {
            ok = false;
            atomicExch(pg.error, 1);
            break;
          }
        }
      }
    }
    s_ok = ok;
    s_seq = seq;
  }
  __syncthreads();
  const unsigned seq = s_seq;
  return XPeerSrc{s_ok ? pg.base + (seq & 1u) * pg.stride : nullptr, seq, pg.words, pg.wait_ns, pg.error};
}

// Hint flag for the input kernels' dry pass: few-row output steps set it at
// their start (they release the next kernel at once) and clear it at their
// end, so an input kernel that finds it set was launched while an output step
// of this library still runs and has time to spare before its wait returns.
// Only a heuristic: a stale or missed value costs time, never correctness.
int *xbusy_flag();

__device__ __forceinline__ void xbusy_set(int *busy, int v) {
  if (busy) *reinterpret_cast<volatile int *>(busy) = v;
}

__device__ __forceinline__ int64_t xrow(const XRowArgs &a, bool cl) {
  return a.row_base + (cl ? blockIdx.y : blockIdx.x);
}

// Standalone RFFT rows (quipsharp/rfft.py:37-60): forward y = FFT(x * phase) * scale,
// inverse y = IFFT(x) * scale * conj(phase); x, y viewed as N complex values.
template <int BIG, bool CL>
__global__ void __launch_bounds__(kXMaxThreads, 1) xrfft_rows_kernel(
    int inverse, const void *x, int64_t ld_x, void *y, int64_t ld_y, int dtype, XPlan plan, const float2 *phase,
    float scale, XRowArgs ra) {
  extern __shared__ float2 xsm[];
  __shared__ XTw tw;
  const int rank = CL ? static_cast<int>(blockIdx.x) : 0;
  const int64_t row = xrow(ra, CL);
  float2 *b0 = xsm, *b1 = xsm + xbuf_elems<float2>(plan.E);
  build_xtw(tw, plan.N);
  pdl_wait();  // launched with programmatic serialization: x may be the previous kernel's output
  __syncthreads();
  const int esz = dtype == QS_F32 ? 4 : 2;
  const void *xr = static_cast<const char *>(x) + row * ld_x * esz;
  void *yr = static_cast<char *>(y) + row * ld_y * esz;
  auto gsrc = [&](int e) {
    const float2 z = make_float2(load_as_float(xr, 2 * e, dtype), load_as_float(xr, 2 * e + 1, dtype));
    return inverse ? z : xcmul(z, phase[e]);
  };
  auto sink = [&](int e, float2 z) {
    z.x *= scale;
    z.y *= scale;
    if (inverse) z = xcmul(z, xconj(phase[e]));
    store_from_float(yr, 2 * e, dtype, z.x);
    store_from_float(yr, 2 * e + 1, dtype, z.y);
  };
  xfft_row<BIG, CL>(plan, b0, b1, tw, inverse != 0, rank, gsrc, sink);
}

// Input step, RFFT: x2 = FFT(x * phase_v) * scale -> x2h (fp16, per-row
// power-of-two scale) + rowscale; zeroes the row's y1 accumulator (y1 != null).
template <int BIG, bool CL>
__global__ void __launch_bounds__(kXMaxThreads, 1) xinput_rfft_kernel(
    const void *x, int dtype, XPlan plan, const float2 *phase, float scale, __half *x2h, float *rowscale,
    int n_pad, float *y1, int64_t m_local, XRowArgs ra) {
  extern __shared__ float2 xsm[];
  __shared__ XTw tw;
  __shared__ float red[32];
  __shared__ float slots[kXMaxCluster];
  const int rank = CL ? static_cast<int>(blockIdx.x) : 0;
  const int C = plan.C;
  const int64_t row = xrow(ra, CL);
  float2 *const b0 = xsm, *const b1 = xsm + xbuf_elems<float2>(plan.E);
  if (ra.early) {
    pdl_launch_dependents();
    xprefetch_l2(phase, 8 * static_cast<int64_t>(plan.N), rank, C);
  }
  build_xtw(tw, plan.N);
  const int N = plan.N;
  const uint32_t *xh = reinterpret_cast<const uint32_t *>(static_cast<const char *>(x) + row * 4 * N);
  const float2 *xf = reinterpret_cast<const float2 *>(static_cast<const char *>(x) + row * 8 * N);
  __shared__ int s_dry;
  if (threadIdx.x == 0) s_dry = ra.warm && ra.busy && *reinterpret_cast<volatile int *>(ra.busy);
  auto gsrc_h = [&](int e) {
    const uint32_t w = xh[e];
    const float2 z = dtype == QS_F16 ? __half22float2(*reinterpret_cast<const __half2 *>(&w))
                                     : __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&w));
    return xcmul(z, phase[e]);
  };
  auto gsrc_f = [&](int e) { return xcmul(xf[e], phase[e]); };
  float amax = 0.f;
  const int rb = xresult_buf(plan);
  float2 *const rbuf = rb ? b1 : b0;
  const XDst<float2, CL> res{rbuf, plan.cl};
  auto sink = [&](int e, float2 z) {
    z.x *= scale;
    z.y *= scale;
    amax = fmaxf(amax, fmaxf(fabsf(z.x), fabsf(z.y)));
    res(e, z);
  };
  __syncthreads();  // twiddle tables (the first stage may use them), s_dry
  if (CL || !s_dry) {  // the plain path (many rows, clusters, no time to spare)
    pdl_wait();  // x may be the previous kernel's output; y1 may still be read by it
    if (y1) xzero_row(y1, row, m_local, m_local * rank / C, m_local * (rank + 1) / C);
    if (dtype == QS_F32) xfft_row<BIG, CL>(plan, b0, b1, tw, false, rank, gsrc_f, sink);
    else xfft_row<BIG, CL>(plan, b0, b1, tw, false, rank, gsrc_h, sink);
  } else if constexpr (!CL) {
    // Warm start (few rows, one CTA per row, launched while an output step of
    // this library still runs): the row transform first runs over zeros (x is
    // not read, phase is), through the same code as the real pass, so the real
    // pass finds its instructions and phase_v in this SM's caches.  Its results
    // are discarded.  A separate copy of the plain path, so the plain path
    // carries none of this.
    bool dry = true;
    auto wsrc_h = [&](int e) {
      const uint32_t w = dry ? 0u : xh[e];
      const float2 z = dtype == QS_F16 ? __half22float2(*reinterpret_cast<const __half2 *>(&w))
                                       : __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&w));
      return xcmul(z, phase[e]);
    };
    auto wsrc_f = [&](int e) { return xcmul(dry ? make_float2(0.f, 0.f) : xf[e], phase[e]); };
#pragma unroll 1
    for (int pass = 0; pass < 2; ++pass) {
      if (pass == 1) {
        __syncthreads();  // the dry pass's stores land before the real pass rewrites the buffers
        dry = false;
        amax = 0.f;
        pdl_wait();
        if (y1) xzero_row(y1, row, m_local, 0, m_local);
      }
      if (dtype == QS_F32) xfft_row<BIG, false>(plan, b0, b1, tw, false, 0, wsrc_f, sink);
      else xfft_row<BIG, false>(plan, b0, b1, tw, false, 0, wsrc_h, sink);
    }
  }
  const float row_max = xgroup_absmax<CL>(amax, red, slots, rank, C);
  float sc, inv;
  xpow2_scale(row_max, sc, inv);
  const float2 *mine = rbuf;
  __half2 *out = reinterpret_cast<__half2 *>(x2h + row * n_pad);
  for (int i = threadIdx.x; i < plan.E; i += blockDim.x) {
    const float2 z = mine[xpad(i, float2())];
    out[rank + C * i] = __floats2half2_rn(z.x * sc, z.y * sc);
  }
  if (rank == C - 1) {
    for (int i = 2 * N + threadIdx.x; i < n_pad; i += blockDim.x) x2h[row * n_pad + i] = __float2half_rn(0.f);
  }
  if (rank == 0 && threadIdx.x == 0) rowscale[row] = inv;
}

// Output step, RFFT: y = IFFT(y1) * scale * conj(phase_u) + bias, cast.
template <int BIG, bool CL>
__global__ void __launch_bounds__(kXMaxThreads, 1) xoutput_rfft_kernel(
    const float *y1, int64_t ld_y1, int64_t shards, int64_t batch, XPlan plan, const float2 *phase,
    const float *bias, float scale, void *y, int dtype, XRowArgs ra) {
  extern __shared__ float2 xsm[];
  __shared__ XTw tw;
  const int rank = CL ? static_cast<int>(blockIdx.x) : 0;
  const int64_t row = xrow(ra, CL);
  float2 *b0 = xsm, *b1 = xsm + xbuf_elems<float2>(plan.E);
  const int N = plan.N;
  const int64_t mp = 2 * static_cast<int64_t>(N) / shards;
  const bool flag = ra.early && row == 0 && rank == 0 && threadIdx.x == 0;
  if (ra.early) {
    if (flag) xbusy_set(ra.busy, 1);  // before the release: the next kernel reads it at its start
    pdl_launch_dependents();
    xprefetch_l2(phase, 8 * static_cast<int64_t>(N), rank, plan.C);
    xprefetch_l2(bias, 8 * static_cast<int64_t>(N), rank, plan.C);
  }
  build_xtw(tw, N);
  pdl_wait();  // y1 comes from the matmul (or the all-gather, or the ranks' pushes)
  const XPeerSrc src = ra.pg.flags ? xwait_peers(ra.pg) : xplain_src(y1);
  bool dead = false;
  auto gsrc = [&](int e) {
    const int64_t off = xy1_offset(row, 2 * e, ld_y1, shards, mp, batch);
    return src.words ? src.get2_wait(off, dead) : src.get2(off);
  };
  auto sink = [&](int e, float2 z) {
    z.x *= scale;
    z.y *= scale;
    z = xcmul(z, xconj(phase[e]));
    if (bias) {
      const float2 bb = reinterpret_cast<const float2 *>(bias)[e];
      z.x += bb.x;
      z.y += bb.y;
    }
    if (dtype == QS_F16) reinterpret_cast<__half2 *>(y)[row * N + e] = __floats2half2_rn(z.x, z.y);
    else if (dtype == QS_BF16) reinterpret_cast<__nv_bfloat162 *>(y)[row * N + e] = __floats2bfloat162_rn(z.x, z.y);
    else reinterpret_cast<float2 *>(y)[row * N + e] = z;
  };
  __syncthreads();  // twiddle tables
  xfft_row<BIG, CL>(plan, b0, b1, tw, true, rank, gsrc, sink);
  if (flag) xbusy_set(ra.busy, 0);
}

// Standalone FWHT rows: y = FWHT(x * pre) * scale * post (pre / post optional).
template <bool CL>
__global__ void __launch_bounds__(kXMaxThreads, 1) xfwht_rows_kernel(
    const void *x, int64_t ld_x, void *y, int64_t ld_y, int dtype, XPlan plan, const float *pre,
    const float *post, float scale, XRowArgs ra) {
  extern __shared__ float fsm_x[];
  const int rank = CL ? static_cast<int>(blockIdx.x) : 0;
  const int64_t row = xrow(ra, CL);
  float *b0 = fsm_x, *b1 = fsm_x + xbuf_elems<float>(plan.E);
  pdl_wait();  // launched with programmatic serialization: x may be the previous kernel's output
  const int esz = dtype == QS_F32 ? 4 : 2;
  const void *xr = static_cast<const char *>(x) + row * ld_x * esz;
  void *yr = static_cast<char *>(y) + row * ld_y * esz;
  auto gsrc = [&](int i) {
    const float v = load_as_float(xr, i, dtype);
    return pre ? v * pre[i] : v;
  };
  auto sink = [&](int i, float v) {
    v *= scale;
    if (post) v *= post[i];
    store_from_float(yr, i, dtype, v);
  };
  xfwht_row<CL>(plan, b0, b1, rank, gsrc, sink);
}

// Input step, RHT: x2 = FWHT(x * sv) * scale -> x2h + rowscale; zeroes y1.
template <bool CL>
__global__ void __launch_bounds__(kXMaxThreads, 1) xinput_rht_kernel(
    const void *x, int dtype, XPlan plan, const float *sv, float scale, __half *x2h, float *rowscale, int n_pad,
    float *y1, int64_t m_local, XRowArgs ra) {
  extern __shared__ float fsm_x[];
  __shared__ float red[32];
  __shared__ float slots[kXMaxCluster];
  const int rank = CL ? static_cast<int>(blockIdx.x) : 0;
  const int C = plan.C;
  const int64_t row = xrow(ra, CL);
  const int n = plan.N;
  float *const b0 = fsm_x, *const b1 = fsm_x + xbuf_elems<float>(plan.E);
  if (ra.early) {
    pdl_launch_dependents();
    xprefetch_l2(sv, 4 * static_cast<int64_t>(n), rank, C);
  }
  __shared__ int s_dry;  // warm start: see xinput_rfft_kernel
  if (threadIdx.x == 0) s_dry = ra.warm && ra.busy && *reinterpret_cast<volatile int *>(ra.busy);
  __syncthreads();
  auto gsrc = [&](int i) { return load_as_float(x, row * n + i, dtype) * sv[i]; };
  float amax = 0.f;
  const int rb = xresult_buf(plan);
  float *const rbuf = rb ? b1 : b0;
  const XDst<float, CL> res{rbuf, plan.cl};
  auto sink = [&](int i, float v) {
    v *= scale;
    amax = fmaxf(amax, fabsf(v));
    res(i, v);
  };
  if (CL || !s_dry) {
    pdl_wait();
    if (y1) xzero_row(y1, row, m_local, m_local * rank / C, m_local * (rank + 1) / C);
    xfwht_row<CL>(plan, b0, b1, rank, gsrc, sink);
  } else if constexpr (!CL) {
    bool dry = true;
    auto wsrc = [&](int i) { return (dry ? 0.f : load_as_float(x, row * n + i, dtype)) * sv[i]; };
#pragma unroll 1
    for (int pass = 0; pass < 2; ++pass) {
      if (pass == 1) {
        __syncthreads();
        dry = false;
        amax = 0.f;
        pdl_wait();
        if (y1) xzero_row(y1, row, m_local, 0, m_local);
      }
      xfwht_row<false>(plan, b0, b1, 0, wsrc, sink);
    }
  }
  const float row_max = xgroup_absmax<CL>(amax, red, slots, rank, C);
  float sc, inv;
  xpow2_scale(row_max, sc, inv);
  const float *mine = rbuf;
  for (int i = threadIdx.x; i < plan.E; i += blockDim.x)
    x2h[row * n_pad + rank + C * i] = __float2half_rn(mine[xpad(i, float())] * sc);
  if (rank == C - 1) {
    for (int i = n + threadIdx.x; i < n_pad; i += blockDim.x) x2h[row * n_pad + i] = __float2half_rn(0.f);
  }
  if (rank == 0 && threadIdx.x == 0) rowscale[row] = inv;
}

// Output step, RHT: y = FWHT(y1) * scale * su + bias, cast.
template <bool CL>
__global__ void __launch_bounds__(kXMaxThreads, 1) xoutput_rht_kernel(
    const float *y1, int64_t ld_y1, int64_t shards, int64_t batch, XPlan plan, const float *su, const float *bias,
    float scale, void *y, int dtype, XRowArgs ra) {
  extern __shared__ float fsm_x[];
  const int rank = CL ? static_cast<int>(blockIdx.x) : 0;
  const int64_t row = xrow(ra, CL);
  const int m = plan.N;
  const int64_t mp = m / shards;
  float *b0 = fsm_x, *b1 = fsm_x + xbuf_elems<float>(plan.E);
  const bool flag = ra.early && row == 0 && rank == 0 && threadIdx.x == 0;
  if (ra.early) {
    if (flag) xbusy_set(ra.busy, 1);  // before the release: the next kernel reads it at its start
    pdl_launch_dependents();
    xprefetch_l2(su, 4 * static_cast<int64_t>(m), rank, plan.C);
    xprefetch_l2(bias, 4 * static_cast<int64_t>(m), rank, plan.C);
  }
  pdl_wait();  // y1 comes from the matmul (or the all-gather, or the ranks' pushes)
  const XPeerSrc src = ra.pg.flags ? xwait_peers(ra.pg) : xplain_src(y1);
  bool dead = false;
  auto gsrc = [&](int i) {
    const int64_t off = xy1_offset(row, i, ld_y1, shards, mp, batch);
    return src.words ? src.get_wait(off, dead) : src.get(off);
  };
  auto sink = [&](int i, float v) {
    v = v * scale * su[i];
    if (bias) v += bias[i];
    store_from_float(y, row * m + i, dtype, v);
  };
  xfwht_row<CL>(plan, b0, b1, rank, gsrc, sink);
  if (flag) xbusy_set(ra.busy, 0);
}

// ---- host launchers (instantiated per big prime in qs_xform_*.cu) ------------------
struct XLaunch {
  int threads;
  size_t smem;
  int64_t rows;
  int warm = 0;  // input kernels: dry pass allowed (XRowArgs::warm; few rows, one CTA per row)
  XPeerGather pg = {};  // output kernels: y1 shards pushed by the ranks (flags == null: none)
};

template <int BIG, bool CL>
int run_xrfft_rows(const XLaunch &L, cudaStream_t s, int inverse, const void *x, int64_t ld_x, void *y,
                   int64_t ld_y, int dtype, const XPlan &p, const float2 *phase, float scale);
template <int BIG, bool CL>
int run_xinput_rfft(const XLaunch &L, cudaStream_t s, const void *x, int dtype, const XPlan &p, const float2 *phase,
                    float scale, __half *x2h, float *rowscale, int n_pad, float *y1, int64_t m_local);
template <int BIG, bool CL>
int run_xoutput_rfft(const XLaunch &L, cudaStream_t s, const float *y1, int64_t ld_y1, int64_t shards,
                     int64_t batch, const XPlan &p, const float2 *phase, const float *bias, float scale, void *y,
                     int dtype);
template <bool CL>
int run_xfwht_rows(const XLaunch &L, cudaStream_t s, const void *x, int64_t ld_x, void *y, int64_t ld_y, int dtype,
                   const XPlan &p, const float *pre, const float *post, float scale);
template <bool CL>
int run_xinput_rht(const XLaunch &L, cudaStream_t s, const void *x, int dtype, const XPlan &p, const float *sv,
                   float scale, __half *x2h, float *rowscale, int n_pad, float *y1, int64_t m_local);
template <bool CL>
int run_xoutput_rht(const XLaunch &L, cudaStream_t s, const float *y1, int64_t ld_y1, int64_t shards,
                    int64_t batch, const XPlan &p, const float *su, const float *bias, float scale, void *y,
                    int dtype);

inline int xlaunch_sms() {
  static int cached[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && cached[dev]) return cached[dev];
  int n = 148;
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  if (dev < 64) cached[dev] = n;
  return n;
}

template <typename... KArgs, typename... Args>
cudaError_t xlaunch_ex(const cudaLaunchConfig_t &cfg, void (*kern)(KArgs...), Args... args) {
  return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

// Launches `kern` over L.rows rows (grid chunks of at most 65535 rows along y
// for clusters) with programmatic stream serialization, and a (C, 1, 1)
// cluster when CL.
template <bool CL, typename... KArgs, typename... Args>
int xlaunch(const char *what, void (*kern)(KArgs...), const XLaunch &L, int C, cudaStream_t s, Args... args) {
  QS_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(L.smem)));
  if (CL && C > 8) QS_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
  const int64_t chunk = CL ? 65535 : (int64_t(1) << 31) - 1;
  for (int64_t r0 = 0; r0 < L.rows; r0 += chunk) {
    const int64_t nr = L.rows - r0 < chunk ? L.rows - r0 : chunk;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = CL ? dim3(C, static_cast<unsigned>(nr)) : dim3(static_cast<unsigned>(nr));
    cfg.blockDim = dim3(L.threads);
    cfg.dynamicSmemBytes = L.smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    int na = 1;
    if (CL) {
      attr[1].id = cudaLaunchAttributeClusterDimension;
      attr[1].val.clusterDim.x = C;
      attr[1].val.clusterDim.y = 1;
      attr[1].val.clusterDim.z = 1;
      na = 2;
    }
    cfg.attrs = attr;
    cfg.numAttrs = na;
    // Few rows leave most SMs free: the dependent kernel may start its
    // prologue at once.  Many rows: its CTAs would take SMs this grid still
    // needs, so it is released only at exit.
    const int early = L.rows * 2 <= xlaunch_sms() ? 1 : 0;
    XRowArgs ra{r0, C, early, early && L.warm && !CL ? 1 : 0, xbusy_flag(), L.pg};
    const cudaError_t e = xlaunch_ex(cfg, kern, args..., ra);
    if (e != cudaSuccess) return fail(QS_ERR_CUDA, "%s launch failed: %s", what, cudaGetErrorString(e));
  }
  return QS_OK;
}

#define QS_DEFINE_XFFT_RUNNERS(BIG, CL)                                                                        \
  template <>                                                                                                  \
  int run_xrfft_rows<BIG, CL>(const XLaunch &L, cudaStream_t s, int inverse, const void *x, int64_t ld_x,     \
                              void *y, int64_t ld_y, int dtype, const XPlan &p, const float2 *phase,           \
                              float scale) {                                                                   \
    return xlaunch<CL>("rfft", xrfft_rows_kernel<BIG, CL>, L, p.C, s, inverse, x, ld_x, y, ld_y, dtype, p,    \
                       phase, scale);                                                                          \
  }                                                                                                            \
  template <>                                                                                                  \
  int run_xinput_rfft<BIG, CL>(const XLaunch &L, cudaStream_t s, const void *x, int dtype, const XPlan &p,     \
                               const float2 *phase, float scale, __half *x2h, float *rowscale, int n_pad,      \
                               float *y1, int64_t m_local) {                                                   \
    return xlaunch<CL>("linear_input_rfft", xinput_rfft_kernel<BIG, CL>, L, p.C, s, x, dtype, p, phase,       \
                       scale, x2h, rowscale, n_pad, y1, m_local);                                              \
  }                                                                                                            \
  template <>                                                                                                  \
  int run_xoutput_rfft<BIG, CL>(const XLaunch &L, cudaStream_t s, const float *y1, int64_t ld_y1,             \
                                int64_t shards, int64_t batch, const XPlan &p, const float2 *phase,            \
                                const float *bias, float scale, void *y, int dtype) {                          \
    return xlaunch<CL>("linear_output_rfft", xoutput_rfft_kernel<BIG, CL>, L, p.C, s, y1, ld_y1, shards,      \
                       batch, p, phase, bias, scale, y, dtype);                                                \
  }

#define QS_DEFINE_XFWHT_RUNNERS(CL)                                                                            \
  template <>                                                                                                  \
  int run_xfwht_rows<CL>(const XLaunch &L, cudaStream_t s, const void *x, int64_t ld_x, void *y,              \
                         int64_t ld_y, int dtype, const XPlan &p, const float *pre, const float *post,         \
                         float scale) {                                                                        \
    return xlaunch<CL>("fwht", xfwht_rows_kernel<CL>, L, p.C, s, x, ld_x, y, ld_y, dtype, p, pre, post,       \
                       scale);                                                                                 \
  }                                                                                                            \
  template <>                                                                                                  \
  int run_xinput_rht<CL>(const XLaunch &L, cudaStream_t s, const void *x, int dtype, const XPlan &p,           \
                         const float *sv, float scale, __half *x2h, float *rowscale, int n_pad, float *y1,     \
                         int64_t m_local) {                                                                    \
    return xlaunch<CL>("linear_input_rht", xinput_rht_kernel<CL>, L, p.C, s, x, dtype, p, sv, scale, x2h,     \
                       rowscale, n_pad, y1, m_local);                                                          \
  }                                                                                                            \
  template <>                                                                                                  \
  int run_xoutput_rht<CL>(const XLaunch &L, cudaStream_t s, const float *y1, int64_t ld_y1, int64_t shards,   \
                          int64_t batch, const XPlan &p, const float *su, const float *bias, float scale,      \
                          void *y, int dtype) {                                                                \
    return xlaunch<CL>("linear_output_rht", xoutput_rht_kernel<CL>, L, p.C, s, y1, ld_y1, shards, batch, p,   \
                       su, bias, scale, y, dtype);                                                             \
  }

#define QS_FOR_EACH_XBIG(X) X(0) X(11) X(13) X(17) X(19) X(23) X(29) X(31) X(37) X(41) X(43)

}  // namespace qs
