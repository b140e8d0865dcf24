// Re-lays QuantizedLinear codes (int16, (stages, m, n/8), quipsharp/checkpoint.py:99-103)
// into the weight stream the fused matmul reads.
//
// Geometry: an "item" is 16 weight rows x 32 codes (256 input features).  Items
// are stored code-chunk-major (item = kc * RT + rt, RT = ceil(m/16)) so a warp
// walking consecutive items reuses its activation fragments and streams a
// contiguous range.  Inside an item, lane l = 4*g + t of the consuming warp owns
// rows g and g+8 and codes [8t, 8t+8) of each; its bytes are contiguous:
//
//   E8P item (1024 B): [half h (row g+8h)][lane l] -> 16 B "quad" of 8 codes:
//     w0 = abs index bytes of codes 0..3, w1 = abs index bytes of codes 4..7,
//     w2 bit (8j + 7 - c) = g_j of code c (j = 0..3),
//     w3 bit (8j + 7 - c) = g_{4+j} of code c (j = 0..2), bit (31 - c) = NOT shift_c,
//   where the sign flips f_0..f_6 of the code (f_i = bit 7-i, e8p.py:174-180) are
//   stored as prefix parities g_i = f_0 ^ ... ^ f_i.  Then f_i = g_{i-1} ^ g_i and
//   the inferred 8th flip (parity of f_0..f_6, e8p.py:97) is simply g_6, so the
//   decoder recovers all eight flips with one shift and one XOR.
//   1-bit item (512 B): [lane l] -> 8 index bytes of row g, then 8 of row g+8.
//
// Padding rows / codes are filled with code 0 (rows are never stored back; the
// padded input features meet zero activations).
#include "qs_common.cuh"
#include "qs_launch.h"

namespace qs {

static __device__ int g_pack_error;

__global__ void pack_e8p_kernel(const int16_t *codes, int64_t m, int64_t T, int64_t RT,
                                int64_t Tq, uint8_t *out) {
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
    uint32_t g = 0;
#pragma unroll
    for (int i = 0; i < 7; ++i) {
      g ^= (code >> (7 - i)) & 1u;  // prefix parity of f_0..f_i
      if (i < 4) w2 |= g << (8 * i + 7 - c);
      else w3 |= g << (8 * (i - 4) + 7 - c);
    }
    w3 |= ((code & 1u) ^ 1u) << (31 - c);
  }
  const int64_t rt = r / kRowsPerTile, rr = r % kRowsPerTile;
  const int64_t kc = q / 4, t = q % 4;
  const int64_t h = rr / 8, lane = (rr % 8) * 4 + t;
  uint4 *dst = reinterpret_cast<uint4 *>(out + (kc * RT + rt) * 1024 + h * 512 + lane * 16);
  *dst = make_uint4(w0, w1, w2, w3);
}

__global__ void pack_1bit_kernel(const int16_t *codes, int64_t m, int64_t T, int64_t RT,
                                 int64_t Tq, uint8_t *out) {
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
