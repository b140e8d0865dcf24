// Shared helpers for the quipsharp_b200 kernels (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/quipsharp_b200.h"

namespace qs {

// ---- error reporting -------------------------------------------------------
void set_error(const char *fmt, ...);
int fail(int status, const char *fmt, ...);
int check_launch(const char *what);

#define QS_CUDA_TRY(expr)                                                           \
  do {                                                                              \
    cudaError_t _e = (expr);                                                        \
    if (_e != cudaSuccess)                                                          \
      return ::qs::fail(QS_ERR_CUDA, "%s: %s", #expr, cudaGetErrorString(_e));    \
  } while (0)

// ---- programmatic dependent launch ----------------------------------------
// The forward's kernels are launched with programmatic stream serialization:
// a kernel may start while its predecessor on the stream is still running,
// runs its prologue (tables, weight prefetch), and calls pdl_wait() before it
// touches anything the predecessor writes or reads (pdl_wait returns once the
// predecessor has completed and its writes are visible).  pdl_launch_dependents()
// lets the successor start its own prologue early.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <typename... KArgs, typename... Args>
inline int launch_pdl(const char *what, void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                      cudaStream_t s, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
  if (e != cudaSuccess) return fail(QS_ERR_CUDA, "%s launch failed: %s", what, cudaGetErrorString(e));
  return QS_OK;
}

// ---- element load / store --------------------------------------------------
__device__ __forceinline__ float load_as_float(const void *p, int64_t i, int dtype) {
  switch (dtype) {
    case QS_F16: return __half2float(static_cast<const __half *>(p)[i]);
    case QS_BF16: return __bfloat162float(static_cast<const __nv_bfloat16 *>(p)[i]);
    default: return static_cast<const float *>(p)[i];
  }
}

__device__ __forceinline__ void store_from_float(void *p, int64_t i, int dtype, float v) {
  switch (dtype) {
    case QS_F16: static_cast<__half *>(p)[i] = __float2half_rn(v); break;
    case QS_BF16: static_cast<__nv_bfloat16 *>(p)[i] = __float2bfloat16_rn(v); break;
    default: static_cast<float *>(p)[i] = v; break;
  }
}

__host__ __device__ __forceinline__ int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }
__host__ __device__ __forceinline__ int64_t round_up(int64_t a, int64_t b) { return ceil_div(a, b) * b; }

// ---- bit helpers -----------------------------------------------------------
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}

__device__ __forceinline__ uint32_t shf_l_wrap(uint32_t lo, uint32_t hi, uint32_t n) {
  // (hi:lo) << n, upper 32 bits
  uint32_t d;
  asm("shf.l.wrap.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(lo), "r"(hi), "r"(n));
  return d;
}

// x * 2^k as an integer multiply-add (runs on the FMA pipe, not the ALU pipe).
__device__ __forceinline__ uint32_t imul(uint32_t x, uint32_t k) {
  uint32_t d;
  asm("mul.lo.u32 %0, %1, %2;" : "=r"(d) : "r"(x), "r"(k));
  return d;
}

__device__ __forceinline__ uint32_t imad(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("mad.lo.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

__device__ __forceinline__ uint32_t hadd2_u32(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("add.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// Read-only streaming load (weights read once per launch).  Not volatile:
// ordering follows data dependencies so loads can overlap with compute.
__device__ __forceinline__ uint4 ldg_nc_v4(const void *p) {
  uint4 v;
  asm("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
      : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
      : "l"(p));
  return v;
}

// D (16x8 f32) += A (16x16 f16, row) * B (16x8 f16, col).  Not volatile: the
// accumulator operands order dependent mma; independent ones may interleave
// with the decode of the next code.
__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                          uint32_t a3, uint32_t b0, uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// d = A * B (zero accumulator input: no registers to clear first).
__device__ __forceinline__ void mma_16816_zc(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                             uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%10,%10,%10,%10};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(0.f));
}

// ---- constant tables ---------------------------------------------------------
// Generated at build time from quipsharp_b200/codebooks/tables.py (internal
// linkage, one copy per translation unit):
//   kE8pAbsF32 / kE81BitF32   : the 256x8 float32 codebook tables;
//   kE8pHiBytes / kE81BitHiBytes : fp16 high bytes of the signed entries,
//       .x = coordinates 0..3 (byte i = coordinate i), .y = coordinates 4..7.
//       Every E8P entry is +-{0.5,1.5,2.5} and every 1-bit entry is in
//       {0, +-0.5, +-1, +-2}, so each has a zero fp16 low byte;
//   kDftCos / kDftSin          : cos/sin(2*pi*k/p) for the odd-prime FFT radices.
constexpr int kNumPrimes = 13;
__host__ __device__ constexpr int prime_at(int i) {
  return i == 0 ? 3 : i == 1 ? 5 : i == 2 ? 7 : i == 3 ? 11 : i == 4 ? 13 : i == 5 ? 17
       : i == 6 ? 19 : i == 7 ? 23 : i == 8 ? 29 : i == 9 ? 31 : i == 10 ? 37 : i == 11 ? 41 : 43;
}
__host__ __device__ constexpr int prime_offset(int p) {
  int off = 0;
  for (int i = 0; i < kNumPrimes && prime_at(i) != p; ++i) off += prime_at(i);
  return off;
}
constexpr int kPrimeTableLen = 3 + 5 + 7 + 11 + 13 + 17 + 19 + 23 + 29 + 31 + 37 + 41 + 43;
#include "qs_tables_gen.inc"

// ---- packed weight-stream geometry ----------------------------------------
// Item = 16 weight rows x 32 codes (256 input features).  E8P items are 1024 B,
// 1-bit items 512 B.  Items are stored code-chunk-major: item = kc * RT + rt
// (RT = padded rows / 16), so a warp walking consecutive items streams one
// contiguous byte range.  Rows are padded to 16 and the input features to 256
// with code 0 (padded rows are never stored back; padded features meet zero
// activations).
constexpr int kRowsPerTile = 16;
constexpr int kCodesPerChunk = 32;
__host__ __device__ inline int64_t padded_m(int64_t m) { return round_up(m, kRowsPerTile); }
__host__ __device__ inline int64_t padded_T(int64_t n) { return round_up(n / 8, kCodesPerChunk); }
__host__ __device__ inline int64_t item_bytes(int kind) { return kind == QS_CB_E8P ? 1024 : 512; }
__host__ __device__ inline int64_t stage_bytes(int kind, int64_t m, int64_t n) {
  return (padded_m(m) / kRowsPerTile) * (padded_T(n) / kCodesPerChunk) * item_bytes(kind);
}

}  // namespace qs
