// Re-lays QuantizedLinear codes (int16, (stages, m, n/8), quipsharp/checkpoint.py:99-103)
// into the weight stream the fused matmuls read.
//
// Geometry (qs_common.cuh): an "item" is 16 weight rows x 32 codes; items are
// stored code-chunk-major.  Inside an item, lane l = 4*g + t of the consuming
// warp owns rows g and g+8 and codes [8t, 8t+8) of each; its bytes are
// contiguous:
//   E8P item (1024 B): [half h (row g+8h)][lane l] -> 16 B quad of 8 codes;
//   1-bit item (512 B): [lane l] -> 8 index bytes of row g, then 8 of row g+8.
//
//   E8P quad (16 B) of 8 codes of one row:
//     w0 = abs index bytes of codes 0..3, w1 = abs index bytes of codes 4..7,
//     w2 bit (8j + 7 - c) = P_j of code c (j = 0..3),
//     w3 bit (8j + 7 - c) = P_{4+j} of code c (j = 0..2), bit (31 - c) = NOT shift_c,
//   where P_0..P_7 are the prefix parities of the code's eight sign flips taken in
//   the coordinate order (2, 0, 3, 1, 6, 4, 7, 5).  The flips f_0..f_6 are code
//   bits 7..1 (e8p.py:174-180) and the 8th flip is their parity (e8p.py:97), so
//   the last prefix parity is always 0 and is not stored.  The decoders recover
//   every flip with one shift and one XOR per word (flip = P_j ^ P_{j-1}), which
//   leaves the flips of coordinates (0, 1) and (4, 5) on byte sign bits 1 and 3
//   and those of (2, 3) and (6, 7) on byte sign bits 0 and 2: after one more
//   shift by the code's slot c (and by 8 for the second pair), the two flips of
//   a natural coordinate pair sit on bits 15 and 31, the sign bits of an f16x2
//   word.
//   1-bit (8 B) of 8 codes of one row: the 8 index bytes (1 bit/weight; the
//   reference stores them as int16).
#include "qs_common.cuh"
#include "qs_launch.h"

namespace qs {

static __device__ int g_pack_error;

// Coordinate order of the prefix parities (byte j of w2, then of w3).
__device__ __forceinline__ int sign_slice_coord(int j) {
  constexpr int order = 0x57461302;  // nibbles: 2, 0, 3, 1, 6, 4, 7, 5
  return (order >> (4 * j)) & 7;
}

__global__ void pack_e8p_kernel(const int16_t *codes, int64_t m, int64_t T, int64_t RT, int64_t Tq,
                                uint8_t *out) {
  const int64_t tid = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  const int64_t mp = RT * kRowsPerTile;
  if (tid >= mp * Tq) return;
  const int64_t r = tid / Tq, q = tid % Tq;  // row, quad of 8 codes
  uint32_t w0 = 0, w1 = 0, w2 = 0, w3 = 0;
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    const int64_t col = q * 8 + c;
    const uint32_t code = (r < m && col < T) ? static_cast<uint16_t>(codes[r * T + col]) : 0u;
    const uint32_t idx = code >> 8;
    if (c < 4) w0 |= idx << (8 * c);
    else w1 |= idx << (8 * (c - 4));
    uint32_t f[8], par = 0;
#pragma unroll
    for (int i = 0; i < 7; ++i) {
      f[i] = (code >> (7 - i)) & 1u;
      par ^= f[i];
    }
    f[7] = par;
    uint32_t P = 0;
#pragma unroll
    for (int j = 0; j < 7; ++j) {
      P ^= f[sign_slice_coord(j)];
      if (j < 4) w2 |= P << (8 * j + 7 - c);
      else w3 |= P << (8 * (j - 4) + 7 - c);
    }
    w3 |= ((code & 1u) ^ 1u) << (31 - c);
  }
  const int64_t rt = r / kRowsPerTile, rr = r % kRowsPerTile;
  const int64_t kc = q / 4, t = q % 4;
  const int64_t h = rr / 8, lane = (rr % 8) * 4 + t;
  uint4 *dst = reinterpret_cast<uint4 *>(out + (kc * RT + rt) * 1024 + h * 512 + lane * 16);
  *dst = make_uint4(w0, w1, w2, w3);
}

__global__ void pack_1bit_kernel(const int16_t *codes, int64_t m, int64_t T, int64_t RT, int64_t Tq,
                                 uint8_t *out) {
  const int64_t tid = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  const int64_t mp = RT * kRowsPerTile;
  if (tid >= mp * Tq) return;
  const int64_t r = tid / Tq, q = tid % Tq;
  uint32_t lo = 0, hi = 0;
  bool bad = false;
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    const int64_t col = q * 8 + c;
    const uint32_t code = (r < m && col < T) ? static_cast<uint16_t>(codes[r * T + col]) : 0u;
    bad |= code >= 256u;
    if (c < 4) lo |= (code & 0xFFu) << (8 * c);
    else hi |= (code & 0xFFu) << (8 * (c - 4));
  }
  if (bad) atomicExch(&g_pack_error, 1);
  const int64_t rt = r / kRowsPerTile, rr = r % kRowsPerTile;
  const int64_t kc = q / 4, t = q % 4;
  const int64_t h = rr / 8, lane = (rr % 8) * 4 + t;
  uint2 *dst = reinterpret_cast<uint2 *>(out + (kc * RT + rt) * 512 + lane * 16 + h * 8);
  *dst = make_uint2(lo, hi);
}

int launch_pack(const int16_t *codes, int stages, const int *kinds, int64_t m, int64_t n,
                void *packed, cudaStream_t s) {
  const int64_t T = n / 8, RT = padded_m(m) / kRowsPerTile, Tq = padded_T(n) / 8;
  const int64_t threads = padded_m(m) * Tq;
  static const int zero = 0;
  QS_CUDA_TRY(cudaMemcpyToSymbolAsync(g_pack_error, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, s));
  uint8_t *dst = static_cast<uint8_t *>(packed);
  bool check = false;
  for (int st = 0; st < stages; ++st) {
    const int16_t *src = codes + st * m * T;
    if (kinds[st] == QS_CB_E8P) {
      pack_e8p_kernel<<<ceil_div(threads, 256), 256, 0, s>>>(src, m, T, RT, Tq, dst);
    } else {
      pack_1bit_kernel<<<ceil_div(threads, 256), 256, 0, s>>>(src, m, T, RT, Tq, dst);
      check = true;
    }
    int e = check_launch("pack");
    if (e) return e;
    dst += round_up(stage_bytes(kinds[st], m, n), 256);
  }
  if (!check) return QS_OK;
  int flag = 0;
  QS_CUDA_TRY(cudaMemcpyFromSymbolAsync(&flag, g_pack_error, sizeof(int), 0, cudaMemcpyDeviceToHost, s));
  QS_CUDA_TRY(cudaStreamSynchronize(s));
  if (flag) return fail(QS_ERR_INDEX, "index out of range for the 1-bit codebook (size 256)");
  return QS_OK;
}

}  // namespace qs
