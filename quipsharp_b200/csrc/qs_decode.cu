// Bit-exact codebook decode: E8PCodebook.dequantize, E8OneBitCodebook.dequantize,
// rvq_dequantize and dequantize_linear, writing float32.
//
// Every decoded value of both codebooks is a multiple of 1/4 below 3 in
// magnitude, so the sign flips and the +-1/4 shift are exact in float32; the
// only roundings are the float32 multiplies by the stage and layer scales,
// done here with __fmul_rn / __fadd_rn in the reference's order so the result
// matches torch bit for bit.
#include "qs_common.cuh"
#include "qs_launch.h"

namespace qs {

// Set when a 1-bit index falls outside [-256, 256).  Read back (with a stream
// synchronisation) by the launchers; concurrent calls on one device share it.
static __device__ int g_decode_error;

// E8P: code = [abs:8][sign7:7][shift:1]; coordinate i < 7 flips with bit (7-i),
// coordinate 7 with the parity of bits 1..7; shift bit 1 -> +1/4, 0 -> -1/4
// (quipsharp/codebooks/e8p.py:92-101, 174-180).
__device__ __forceinline__ void decode_e8p(int64_t code, float (&v)[8]) {
  const uint32_t c = static_cast<uint32_t>(code) & 0xFFFFu;
  const uint32_t abs_idx = c >> 8;
  const uint32_t parity = __popc(c & 0xFEu) & 1u;
  const float shift = (c & 1u) ? 0.25f : -0.25f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const uint32_t flip = i < 7 ? (c >> (7 - i)) & 1u : parity;
    const float base = kE8pAbsF32[abs_idx * 8 + i];
    v[i] = __fadd_rn(flip ? -base : base, shift);
  }
}

// 1-bit E8: table gather with torch's negative-index wrap; returns false if
// the index is out of range (quipsharp/codebooks/e8_1bit.py:86-87).
__device__ __forceinline__ bool decode_1bit(int64_t idx, float (&v)[8]) {
  if (idx < -256 || idx >= 256) {
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = 0.f;
    return false;
  }
  const int r = static_cast<int>(idx < 0 ? idx + 256 : idx);
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = kE81BitF32[r * 8 + i];
  return true;
}

__device__ __forceinline__ int64_t load_code(const void *p, int64_t i, int dt) {
  switch (dt) {
    case QS_I16: return static_cast<const int16_t *>(p)[i];
    case QS_I32: return static_cast<const int32_t *>(p)[i];
    default: return static_cast<const int64_t *>(p)[i];
  }
}

__device__ __forceinline__ bool decode_kind(int kind, int64_t code, float (&v)[8]) {
  if (kind == QS_CB_E8P) {
    decode_e8p(code, v);
    return true;
  }
  return decode_1bit(code, v);
}

__device__ __forceinline__ void store8(float *out, const float (&v)[8]) {
  float4 *o = reinterpret_cast<float4 *>(out);
  o[0] = make_float4(v[0], v[1], v[2], v[3]);
  o[1] = make_float4(v[4], v[5], v[6], v[7]);
}

__global__ void decode_kernel(int kind, const void *codes, int code_dtype, int64_t count,
                              float *out) {
  const int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (i >= count) return;
  float v[8];
  if (!decode_kind(kind, load_code(codes, i, code_dtype), v)) atomicExch(&g_decode_error, 1);
  store8(out + i * 8, v);
}

struct StageArgs {
  const void *codes[2];
  int kinds[2];
  float scales[2];
};

// sum_s fl32(decode_s(code) * s_s), stage order (quipsharp/rvq.py:83-88).
__global__ void rvq_decode_kernel(int stages, StageArgs a, int code_dtype, int64_t count,
                                  float *out) {
  const int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (i >= count) return;
  float tot[8];
  bool ok = true;
  for (int s = 0; s < stages; ++s) {
    float v[8];
    ok &= decode_kind(a.kinds[s], load_code(a.codes[s], i, code_dtype), v);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float p = __fmul_rn(v[j], a.scales[s]);
      tot[j] = s == 0 ? p : __fadd_rn(tot[j], p);
    }
  }
  if (!ok) atomicExch(&g_decode_error, 1);
  store8(out + i * 8, tot);
}

// dequantize_linear (quipsharp/quantize.py:107-113) over the int16 buffer of
// QuantizedLinear (quipsharp/checkpoint.py:136: codes & 0xFFFF).  One thread
// per (row, block): W[row, 8*blk : 8*blk+8].
__global__ void dequantize_linear_kernel(const int16_t *codes, int stages, StageArgs a,
                                         int has_stage_scales, const float *layer_scale,
                                         int64_t m, int64_t T, float *out) {
  const int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (i >= m * T) return;
  const float ls = *layer_scale;
  float tot[8];
  bool ok = true;
  for (int s = 0; s < stages; ++s) {
    const int64_t code = static_cast<uint16_t>(codes[s * m * T + i]);
    float v[8];
    ok &= decode_kind(a.kinds[s], code, v);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float p = has_stage_scales ? __fmul_rn(v[j], a.scales[s]) : v[j];
      tot[j] = s == 0 ? p : __fadd_rn(tot[j], p);
    }
  }
  if (!ok) atomicExch(&g_decode_error, 1);
#pragma unroll
  for (int j = 0; j < 8; ++j) tot[j] = __fmul_rn(tot[j], ls);
  store8(out + i * 8, tot);
}

static int reset_flag(cudaStream_t s) {
  static const int zero = 0;
  QS_CUDA_TRY(cudaMemcpyToSymbolAsync(g_decode_error, &zero, sizeof(int), 0,
                                      cudaMemcpyHostToDevice, s));
  return QS_OK;
}

static int read_flag(cudaStream_t s) {
  int flag = 0;
  QS_CUDA_TRY(cudaMemcpyFromSymbolAsync(&flag, g_decode_error, sizeof(int), 0,
                                        cudaMemcpyDeviceToHost, s));
  QS_CUDA_TRY(cudaStreamSynchronize(s));
  if (flag) return fail(QS_ERR_INDEX, "index out of range for the 1-bit codebook (size 256)");
  return QS_OK;
}

static bool any_1bit(int stages, const int *kinds) {
  for (int i = 0; i < stages; ++i)
    if (kinds[i] == QS_CB_E8_1BIT) return true;
  return false;
}

int launch_decode(int kind, const void *codes, int code_dtype, int64_t count, float *out,
                  cudaStream_t s) {
  const bool check = kind == QS_CB_E8_1BIT;
  if (check) {
    int st = reset_flag(s);
    if (st) return st;
  }
  const int threads = 256;
  decode_kernel<<<ceil_div(count, threads), threads, 0, s>>>(kind, codes, code_dtype, count, out);
  int st = check_launch("decode");
  if (st || !check) return st;
  return read_flag(s);
}

int launch_rvq_decode(int stages, const int *kinds, const void *const *codes, int code_dtype,
                      const float *stage_scales, int64_t count, float *out, cudaStream_t s) {
  StageArgs a{};
  for (int i = 0; i < stages; ++i) {
    a.codes[i] = codes[i];
    a.kinds[i] = kinds[i];
    a.scales[i] = stage_scales[i];
  }
  const bool check = any_1bit(stages, kinds);
  if (check) {
    int st = reset_flag(s);
    if (st) return st;
  }
  rvq_decode_kernel<<<ceil_div(count, 256), 256, 0, s>>>(stages, a, code_dtype, count, out);
  int st = check_launch("rvq_decode");
  if (st || !check) return st;
  return read_flag(s);
}

int launch_dequantize_linear(const int16_t *codes, int stages, const int *kinds,
                             const float *stage_scales, const float *layer_scale, int64_t m,
                             int64_t n, float *out, cudaStream_t s) {
  StageArgs a{};
  for (int i = 0; i < stages; ++i) {
    a.kinds[i] = kinds[i];
    a.scales[i] = stage_scales ? stage_scales[i] : 1.f;
  }
  const bool check = any_1bit(stages, kinds);
  if (check) {
    int st = reset_flag(s);
    if (st) return st;
  }
  const int64_t T = n / 8;
  dequantize_linear_kernel<<<ceil_div(m * T, 256), 256, 0, s>>>(
      codes, stages, a, stage_scales != nullptr, layer_scale, m, T, out);
  int st = check_launch("dequantize_linear");
  if (st || !check) return st;
  return read_flag(s);
}

}  // namespace qs
