// Codebook construction for RVQ checkpoints: the stage-scale sweeps of
// quipsharp/rvq.py:28-66 (fit_stage_scale, fit_residual_stage_scale), which
// quipsharp/checkpoint.py:60-77 (build_codebook) runs at load time to rebuild a
// 3/4-bit codebook from (bits, seed).  For every candidate scale s and every
// Gaussian sample x (8 floats), the kernel quantizes x / s with the swept
// codebook and accumulates ||x - s q||^2; the candidate with the smallest mean
// wins (the first one on ties, as the reference's strict `<` keeps).
//
// Nearest-point rules restated (per 8-vector y):
//  * E8P (quipsharp/codebooks/e8p.py:104-160): for z = y + 1/4 and z = y - 1/4,
//    each of the 256 base rows a takes the signs that agree with z coordinate
//    by coordinate (flip where z_i a_i < 0), repaired to an even number of flips
//    by toggling the coordinate with the smallest |z_i a_i| (the first on ties);
//    the row with the smallest ||z - v||^2 wins (the first on ties) and the +
//    side wins ties between the sides; the value is v - 1/4 (+ side) or
//    v + 1/4 (- side).
//  * E8 1-bit (quipsharp/codebooks/e8_1bit.py:81-84): the table row with the
//    smallest ||y - t||^2 (the first on ties).
//  * RVQ (quipsharp/rvq.py:69-80): r = y; per stage: q = Q(r / s_i),
//    total += q s_i, r -= q s_i.
// The values that reach the error follow the reference's float32 operation
// order, each operation rounded on its own (IEEE division, no contraction into
// fused multiply-adds); the error of each candidate is summed in double.
#include "qs_common.cuh"
#include "qs_launch.h"

namespace qs {

namespace {

constexpr int kFitThreads = 128;

struct FitArgs {
  const float *x;  // (samples, 8)
  int64_t samples;
  int nprev;       // stages quantized away first (fit_residual_stage_scale)
  int prev_kind[kFitMaxStages];
  float prev_scale[kFitMaxStages];
  int rvq;         // the swept codebook is an RVQ of `nst` stages (else one plain codebook)
  int nst;
  int kind[kFitMaxStages];
  float scale[kFitMaxStages];
  float cand[kFitMaxCandidates];
  double *partial;  // (ncand, gridDim.x)
};

struct FitTables {
  const float *e8p;  // 256 x 8 base rows
  const float *one;  // 256 x 8 1-bit table
};

__device__ __forceinline__ void e8p_side(const float (&z)[8], const float *a, int k, float &best, int &bk,
                                         uint32_t &bf) {
  uint32_t f = 0;
  float mn = __int_as_float(0x7f800000);
  int mc = 0;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float p = __fmul_rn(z[j], a[j]);
    if (p < 0.f) f |= 1u << j;
    const float ap = fabsf(p);
    if (ap < mn) {
      mn = ap;
      mc = j;
    }
  }
  if (__popc(f) & 1) f ^= 1u << mc;
  float d = 0.f;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float v = (f >> j) & 1u ? -a[j] : a[j];
    const float e = __fsub_rn(z[j], v);
    d = __fadd_rn(d, __fmul_rn(e, e));
  }
  if (d < best) {
    best = d;
    bk = k;
    bf = f;
  }
}

__device__ void e8p_nearest(const float (&y)[8], const float *tab, float (&out)[8]) {
  float zp[8], zm[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    zp[j] = __fadd_rn(y[j], 0.25f);
    zm[j] = __fsub_rn(y[j], 0.25f);
  }
  float bp = __int_as_float(0x7f800000), bm = bp;
  int kp = 0, km = 0;
  uint32_t fp = 0, fm = 0;
#pragma unroll 2
  for (int k = 0; k < 256; ++k) {
    const float *a = tab + 8 * k;
    e8p_side(zp, a, k, bp, kp, fp);
    e8p_side(zm, a, k, bm, km, fm);
  }
  const bool plus = bp <= bm;
  const float *a = tab + 8 * (plus ? kp : km);
  const uint32_t f = plus ? fp : fm;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float v = (f >> j) & 1u ? -a[j] : a[j];
    out[j] = plus ? __fsub_rn(v, 0.25f) : __fadd_rn(v, 0.25f);
  }
}

__device__ void onebit_nearest(const float (&y)[8], const float *tab, float (&out)[8]) {
  float best = __int_as_float(0x7f800000);
  int bk = 0;
#pragma unroll 2
  for (int k = 0; k < 256; ++k) {
    const float *t = tab + 8 * k;
    float d = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float e = __fsub_rn(y[j], t[j]);
      d = __fadd_rn(d, __fmul_rn(e, e));
    }
    if (d < best) {
      best = d;
      bk = k;
    }
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) out[j] = tab[8 * bk + j];
}

__device__ __forceinline__ void stage_nearest(int kind, const float (&y)[8], const FitTables &t, float (&out)[8]) {
  if (kind == QS_CB_E8P) e8p_nearest(y, t.e8p, out);
  else onebit_nearest(y, t.one, out);
}

__device__ void rvq_quantize8(int n, const int *kind, const float *scale, const float (&x)[8], const FitTables &t,
                              float (&total)[8]) {
  float r[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    r[j] = x[j];
    total[j] = 0.f;
  }
  for (int i = 0; i < n; ++i) {
    float y[8], q[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) y[j] = __fdiv_rn(r[j], scale[i]);
    stage_nearest(kind[i], y, t, q);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float qs = __fmul_rn(q[j], scale[i]);
      total[j] = __fadd_rn(total[j], qs);
      r[j] = __fsub_rn(r[j], qs);
    }
  }
}

__global__ void __launch_bounds__(kFitThreads) fit_sweep_kernel(FitArgs a) {
  __shared__ float tab_e8p[256 * 8], tab_one[256 * 8];
  __shared__ double red[kFitThreads / 32];
  for (int i = threadIdx.x; i < 256 * 8; i += blockDim.x) {
    tab_e8p[i] = kE8pAbsF32[i];
    tab_one[i] = kE81BitF32[i];
  }
  __syncthreads();
  const FitTables t{tab_e8p, tab_one};
  const float s = a.cand[blockIdx.y];
  const int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  double err = 0.0;
  if (i < a.samples) {
    float x[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) x[j] = a.x[8 * i + j];
    if (a.nprev) {  // fit_residual_stage_scale: sweep on x - rvq_quantize(x, prev)
      float v[8];
      rvq_quantize8(a.nprev, a.prev_kind, a.prev_scale, x, t, v);
#pragma unroll
      for (int j = 0; j < 8; ++j) x[j] = __fsub_rn(x[j], v[j]);
    }
    float y[8], q[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) y[j] = __fdiv_rn(x[j], s);
    if (a.rvq) rvq_quantize8(a.nst, a.kind, a.scale, y, t, q);
    else stage_nearest(a.kind[0], y, t, q);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float e = __fsub_rn(x[j], __fmul_rn(q[j], s));
      err += static_cast<double>(__fmul_rn(e, e));
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) err += __shfl_down_sync(0xffffffffu, err, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = err;
  __syncthreads();
  if (threadIdx.x == 0) {
    double sum = 0.0;
    for (int w = 0; w < kFitThreads / 32; ++w) sum += red[w];
    a.partial[static_cast<int64_t>(blockIdx.y) * gridDim.x + blockIdx.x] = sum;
  }
}

// Mean error per candidate (partials summed in a fixed order) and the first
// candidate with the smallest mean.
__global__ void __launch_bounds__(kFitMaxCandidates) fit_finish_kernel(const double *partial, int nblk, int ncand,
                                                                       double count, double *mse, int *best) {
  __shared__ double s_mse[kFitMaxCandidates];
  const int c = threadIdx.x;
  if (c < ncand) {
    double sum = 0.0;
    for (int b = 0; b < nblk; ++b) sum += partial[static_cast<int64_t>(c) * nblk + b];
    s_mse[c] = sum / count;
    mse[c] = s_mse[c];
  }
  __syncthreads();
  if (c == 0) {
    int bi = 0;
    for (int k = 1; k < ncand; ++k)
      if (s_mse[k] < s_mse[bi]) bi = k;
    *best = bi;
  }
}

int fit_blocks(int64_t samples) { return static_cast<int>((samples + kFitThreads - 1) / kFitThreads); }

}  // namespace

int64_t fit_workspace_bytes(int64_t samples, int ncand) {
  return round_up(static_cast<int64_t>(fit_blocks(samples)) * ncand * 8, 256);
}

int launch_fit_sweep(const float *x, int64_t samples, int nprev, const int *prev_kinds, const float *prev_scales,
                     int rvq, int nst, const int *kinds, const float *stage_scales, const float *candidates,
                     int ncand, void *workspace, double *mse, int *best, cudaStream_t s) {
  FitArgs a{};
  a.x = x;
  a.samples = samples;
  a.nprev = nprev;
  for (int i = 0; i < nprev; ++i) {
    a.prev_kind[i] = prev_kinds[i];
    a.prev_scale[i] = prev_scales[i];
  }
  a.rvq = rvq;
  a.nst = nst;
  for (int i = 0; i < nst; ++i) {
    a.kind[i] = kinds[i];
    a.scale[i] = rvq ? stage_scales[i] : 1.f;
  }
  for (int c = 0; c < ncand; ++c) a.cand[c] = candidates[c];
  a.partial = static_cast<double *>(workspace);
  const int nblk = fit_blocks(samples);
  fit_sweep_kernel<<<dim3(nblk, ncand), kFitThreads, 0, s>>>(a);
  int st = check_launch("fit_sweep");
  if (st) return st;
  fit_finish_kernel<<<1, kFitMaxCandidates, 0, s>>>(a.partial, nblk, ncand, static_cast<double>(samples) * 8.0,
                                                     mse, best);
  return check_launch("fit_finish");
}

}  // namespace qs
