// Fused codebook decode + matmul for the decode regime (1 to 32 tokens):
//   y1[tok, row] += layer_scale * rowscale[tok] * sum_s s_s * sum_k x2h[tok, k] * What_s[row, k]
//
// Weights stream from HBM once in the packed layout of qs_pack.cu and are
// decoded in registers into fp16 mma.sync A fragments; the tokens form the
// N=8 side of m16n8k16 (swap-AB GEMV).  Each warp works on its own: no
// cross-warp pipeline, so no synchronisation cost per unit of work.  (A
// tcgen05 variant -- decoded weights stored to TMEM as the A operand of
// kind::f16 / kind::f8f6f4 MMAs with N = 16 -- was measured slower here: a
// tcgen05.mma holds its issuing thread for ~155 cycles whatever N is, so skinny
// MMAs are issue-bound, and the hand-offs between decode and issuing warps cost
// more than the whole per-warp decode of this kernel.)
// Decode of one code (8 weights):
//   * one 16-byte shared-memory load of the table row, laid out as the four
//     f16x2 words of the natural coordinate pairs (0,1), (2,3), (4,5), (6,7) (all
//     table values have a zero low byte; the table is replicated 8x so the 8
//     lanes of a quarter-warp hit distinct banks),
//   * E8P: the eight sign flips are XORed into the words' sign bits.  The packed
//     quad stores prefix parities of the flips in the coordinate order
//     (2, 0, 3, 1, 6, 4, 7, 5), so one shift and one XOR recover all flips of a
//     quad's 8 codes; after a further shift by the code's slot c (and by 8 more
//     for the second pair of a word's coordinates) the two flips of a pair sit
//     on bits 15 and 31, so each word takes one AND-XOR; the +-1/4 shift is
//     added by the tensor core (see shift_words).  1-bit: the words are used as
//     loaded.  All decoded values are exact in fp16.
//   * The activations need no reordering: word w of a code's 16 bytes is the
//     pair (2w, 2w+1), the order of the decoded weight words.
// RVQ stages accumulate separately (exact weights) and are combined with their
// float32 stage scales in the epilogue.  Each warp walks a contiguous range of
// (code-chunk, row-tile) items (16 rows x 32 codes, one contiguous 1 KB / 512 B
// per stage in the packed stream); partial sums of a row tile are added to the
// float32 y1 with atomics (y1 is zeroed by the input-transform kernel).
#include "qs_common.cuh"
#include "qs_launch.h"
#include "qs_tp.cuh"

namespace qs {

constexpr int kGemvThreads = 256;
constexpr int kTblBytes = 256 * 256;  // 256 rows x (8 E8P replicas + 8 1-bit replicas) x 16 B

struct GemvArgs {
  const __half *x2h;       // (batch, n_pad)
  const float *rowscale;   // (batch)
  const uint8_t *stage[2];
  float sscale[2];
  const float *layer_scale;
  float *y1;               // (batch, m)
  int64_t m, RT, KC, n_pad, items;  // RT: 16-row tiles, KC: 32-code chunks
  int tok0, ntok;
};

// Tensor parallelism: the push of the finished y1 shard to every rank by all
// CTAs after a grid barrier (a separate kernel instance: the one-GPU kernel
// carries neither the arguments nor the tail, which measurably slowed it).
struct GemvPush {
  TpPush push;
  uint64_t wait_ns;  // bound of the barrier
  int *error;        // set when it ran out
};

// f16x2 words of the natural coordinate pairs (0,1), (2,3), (4,5), (6,7) from
// the fp16 high bytes of coordinates 0..3 (hb.x) and 4..7 (hb.y).
__device__ __forceinline__ uint4 pair_words(uint2 hb) {
  return make_uint4(prmt(hb.x, 0u, 0x1404u), prmt(hb.x, 0u, 0x3424u), prmt(hb.y, 0u, 0x1404u),
                    prmt(hb.y, 0u, 0x3424u));
}

// Fill the replicated table: thread i < 256 owns table row i (256 bytes: 8
// replicas of its E8P entry, then 8 of its 1-bit entry, 16 bytes each).
__device__ __forceinline__ void load_table(uint8_t *tbl) {
  for (int row = threadIdx.x; row < 256; row += blockDim.x) {
    const uint4 e = pair_words(kE8pHiBytes[row]), o = pair_words(kE81BitHiBytes[row]);
    uint4 *dst = reinterpret_cast<uint4 *>(tbl + row * 256);
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      dst[(r + row) & 7] = e;  // rotate the write order to spread banks
      dst[8 + ((r + row) & 7)] = o;
    }
  }
}

// Table row of the code whose index is byte csel of idxsrc.  lane_off: this
// lane's replica offset within a row.  A plain shared-memory load (not asm) so
// the compiler can hoist it ahead of the previous code's work while keeping it
// after the table fill barrier.
__device__ __forceinline__ uint4 table_row(const uint8_t *tbl, uint32_t lane_off, uint32_t idxsrc, int csel) {
  const uint32_t idx = prmt(idxsrc, 0u, 0x4440u | static_cast<uint32_t>(csel));
  return *reinterpret_cast<const uint4 *>(tbl + imad(idx, 256u, lane_off));
}

// Decoded f16x2 words of one E8P code: W = pairs (0,1), (2,3), (4,5), (6,7)
// holding sign*|t| exactly.  fa / fb: flips of coordinates (2,0,3,1) / (6,4,7,5)
// on the byte sign bits, shifted by the code's slot; fa8 / fb8: the same
// shifted by 8 more.
__device__ __forceinline__ void e8p_words(const uint8_t *tbl, uint32_t lane_off, uint32_t idxsrc, int csel,
                                          uint32_t fa, uint32_t fa8, uint32_t fb, uint32_t fb8, uint32_t (&W)[4]) {
  const uint4 T = table_row(tbl, lane_off, idxsrc, csel);
  W[0] = T.x ^ (fa & 0x80008000u);
  W[1] = T.y ^ (fa8 & 0x80008000u);
  W[2] = T.z ^ (fb & 0x80008000u);
  W[3] = T.w ^ (fb8 & 0x80008000u);
}

__device__ __forceinline__ void onebit_words(const uint8_t *tbl, uint32_t lane_off, uint32_t idxsrc, int csel,
                                             uint32_t (&W)[4]) {
  const uint4 T = table_row(tbl, lane_off, idxsrc, csel);
  W[0] = T.x;
  W[1] = T.y;
  W[2] = T.z;
  W[3] = T.w;
}

// The +-1/4 shifts of the 8 codes of a quad as four f16x2 words of +-0.25:
// sw[p] holds (code 2p, code 2p+1) in (low, high) halves.  w3 carries the
// negated shift bit of code c at bit 31-c (qs_pack.cu).
__device__ __forceinline__ void shift_words(uint32_t w3, uint32_t (&sw)[4]) {
  const uint32_t u = prmt(w3, imul(w3, 2u), 0x7030u);  // byte1 <- w3.b3, byte3 <- (w3<<1).b3
#pragma unroll
  for (int p = 0; p < 4; ++p) sw[p] = 0x34003400u ^ (imul(u, 1u << (2 * p)) & 0x80008000u);
}

// One stage of one item: 8 codes for each of the lane's two rows (16 mma per
// token group), plus 2 mma per token group for the E8P shifts against the
// per-code activation sums sf.  Each decoded fragment feeds all NTG groups.
// acc / acc2 are outputs (the first mma starts them from zero).
template <int KIND, int NTG>
__device__ __forceinline__ void stage_item(const uint8_t *tbl, uint32_t off_e8p, uint32_t off_1b, const uint4 &qa,
                                           const uint4 &qb, const uint32_t (&bf)[NTG][32],
                                           const uint32_t (&sf)[NTG][4], float (&acc)[NTG][4],
                                           float (&acc2)[NTG][4]) {
  if constexpr (KIND == QS_CB_E8P) {
    const uint32_t faa = qa.z ^ imul(qa.z, 256u), fab = qb.z ^ imul(qb.z, 256u);
    const uint32_t fba = (qa.w & 0x00FFFFFFu) ^ shf_l_wrap(qa.z, qa.w, 8);
    const uint32_t fbb = (qb.w & 0x00FFFFFFu) ^ shf_l_wrap(qb.z, qb.w, 8);
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      uint32_t Wa[4], Wb[4];
      e8p_words(tbl, off_e8p, c < 4 ? qa.x : qa.y, c & 3, imul(faa, 1u << c), imul(faa, 256u << c),
                imul(fba, 1u << c), imul(fba, 256u << c), Wa);
      e8p_words(tbl, off_e8p, c < 4 ? qb.x : qb.y, c & 3, imul(fab, 1u << c), imul(fab, 256u << c),
                imul(fbb, 1u << c), imul(fbb, 256u << c), Wb);
#pragma unroll
      for (int tg = 0; tg < NTG; ++tg) {
        if (c == 0) {  // the first products start the accumulators
          mma_16816_zc(acc[tg], Wa[0], Wb[0], Wa[1], Wb[1], bf[tg][4 * c + 0], bf[tg][4 * c + 1]);
          mma_16816_zc(acc2[tg], Wa[2], Wb[2], Wa[3], Wb[3], bf[tg][4 * c + 2], bf[tg][4 * c + 3]);
        } else {
          mma_16816(acc[tg], Wa[0], Wb[0], Wa[1], Wb[1], bf[tg][4 * c + 0], bf[tg][4 * c + 1]);
          mma_16816(acc2[tg], Wa[2], Wb[2], Wa[3], Wb[3], bf[tg][4 * c + 2], bf[tg][4 * c + 3]);
        }
      }
    }
    uint32_t swa[4], swb[4];
    shift_words(qa.w, swa);
    shift_words(qb.w, swb);
#pragma unroll
    for (int tg = 0; tg < NTG; ++tg) {
      mma_16816(acc[tg], swa[0], swb[0], swa[1], swb[1], sf[tg][0], sf[tg][1]);
      mma_16816(acc2[tg], swa[2], swb[2], swa[3], swb[3], sf[tg][2], sf[tg][3]);
    }
  } else {
    // 1-bit quad: qa = 16 bytes: row g codes 0..7 in (x, y), row g+8 in (z, w)
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      uint32_t Wa[4], Wb[4];
      onebit_words(tbl, off_1b, c < 4 ? qa.x : qa.y, c & 3, Wa);
      onebit_words(tbl, off_1b, c < 4 ? qa.z : qa.w, c & 3, Wb);
#pragma unroll
      for (int tg = 0; tg < NTG; ++tg) {
        if (c == 0) {  // the first products start the accumulators
          mma_16816_zc(acc[tg], Wa[0], Wb[0], Wa[1], Wb[1], bf[tg][4 * c + 0], bf[tg][4 * c + 1]);
          mma_16816_zc(acc2[tg], Wa[2], Wb[2], Wa[3], Wb[3], bf[tg][4 * c + 2], bf[tg][4 * c + 3]);
        } else {
          mma_16816(acc[tg], Wa[0], Wb[0], Wa[1], Wb[1], bf[tg][4 * c + 0], bf[tg][4 * c + 1]);
          mma_16816(acc2[tg], Wa[2], Wb[2], Wa[3], Wb[3], bf[tg][4 * c + 2], bf[tg][4 * c + 3]);
        }
      }
    }
  }
}

// Quad registers of one item: stage 0 in q[0..n0), stage 1 in q[n0..n0+n1),
// with n = 2 for E8P (rows g and g+8) and 1 for 1-bit (both rows in 16 B).
template <int K>
constexpr int nquads() { return K == QS_CB_E8P ? 2 : 1; }

// 32-bit index arithmetic throughout (items < 2^31 / 1024, batch * m < 2^31:
// checked by the launcher), which keeps the per-item integer work small.
template <int K0, int K1, int NST>
__device__ __forceinline__ void load_item(const GemvArgs &a, uint32_t it, int lane, uint4 (&q)[4]) {
  constexpr uint32_t b0 = K0 == QS_CB_E8P ? 1024u : 512u, b1 = K1 == QS_CB_E8P ? 1024u : 512u;
  const uint8_t *p0 = a.stage[0] + (it * b0 + static_cast<uint32_t>(lane) * 16u);
  q[0] = ldg_nc_v4(p0);
  if constexpr (K0 == QS_CB_E8P) q[1] = ldg_nc_v4(p0 + 512);
  if constexpr (NST == 2) {
    constexpr int o = nquads<K0>();
    const uint8_t *p1 = a.stage[1] + (it * b1 + static_cast<uint32_t>(lane) * 16u);
    q[o] = ldg_nc_v4(p1);
    if constexpr (K1 == QS_CB_E8P) q[o + 1] = ldg_nc_v4(p1 + 512);
  }
}

// Activation fragments of one code chunk for token g (or zeros): bf holds
// the 64 fp16 inputs of codes 8t..8t+7 (B operands of the 16 mma) as the
// coordinate pairs (0,1), (2,3), (4,5), (6,7) of each code (the order of the
// decoded weight words), sf the per-code sums as (code 2p, code 2p+1) f16x2
// pairs (B operands of the shift mma).
__device__ __forceinline__ void load_activations(const GemvArgs &a, uint32_t kc, int g, int t,
                                                 uint32_t (&bf)[32], uint32_t (&sf)[4]) {
  if (g < a.ntok) {
    const uint4 *src = reinterpret_cast<const uint4 *>(
        a.x2h + (static_cast<uint32_t>(a.tok0 + g) * static_cast<uint32_t>(a.n_pad) + kc * 256u + t * 64u));
    float sum[8];
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      const uint4 v = __ldg(src + c);
      bf[4 * c + 0] = v.x;  // (x0, x1)
      bf[4 * c + 1] = v.y;  // (x2, x3)
      bf[4 * c + 2] = v.z;  // (x4, x5)
      bf[4 * c + 3] = v.w;  // (x6, x7)
      const float2 f0 = __half22float2(*reinterpret_cast<const __half2 *>(&v.x));
      const float2 f1 = __half22float2(*reinterpret_cast<const __half2 *>(&v.y));
      const float2 f2 = __half22float2(*reinterpret_cast<const __half2 *>(&v.z));
      const float2 f3 = __half22float2(*reinterpret_cast<const __half2 *>(&v.w));
      sum[c] = ((f0.x + f0.y) + (f1.x + f1.y)) + ((f2.x + f2.y) + (f3.x + f3.y));
    }
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      const __half2 h = __floats2half2_rn(sum[2 * p], sum[2 * p + 1]);
      sf[p] = *reinterpret_cast<const uint32_t *>(&h);
    }
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i) bf[i] = 0u;
#pragma unroll
    for (int p = 0; p < 4; ++p) sf[p] = 0u;
  }
}

// NTG token groups of 8 per pass (1: batches <= 8, two CTAs per SM; 2: batches
// 9 and more in passes of 16 tokens over the weights, one CTA per SM for the
// registers; the tcgen05 GEMM takes over at kTcMinBatch).
template <int K0, int K1, int NST, int NTG>
__device__ __forceinline__ void gemv_items(const GemvArgs &a, const uint8_t *tbl, uint32_t start, uint32_t end,
                                           uint4 (&q)[4], uint4 (&nq)[4]) {
  const int lane = threadIdx.x & 31;
  const uint32_t m = static_cast<uint32_t>(a.m), RT = static_cast<uint32_t>(a.RT);
  pdl_wait();  // x2h, rowscale and the zeroed y1 come from the input-transform kernel

  const uint32_t off_e8p = (lane & 7) * 16;        // E8P replicas: bytes [0, 128) of a row
  const uint32_t off_1b = 128 + (lane & 7) * 16;   // 1-bit replicas: bytes [128, 256)
  const int g = lane >> 2, t = lane & 3;
  const float ls = *a.layer_scale;
  float tokscale[NTG][2];  // layer scale x per-token x2 scale of this lane's output tokens
#pragma unroll
  for (int tg = 0; tg < NTG; ++tg)
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int tok = 8 * tg + 2 * t + j;
      tokscale[tg][j] = tok < a.ntok ? ls * a.rowscale[a.tok0 + tok] : 0.f;
    }

  uint32_t bf[NTG][32], sf[NTG][4];
  uint32_t kc = start / RT, rt = start % RT;
#pragma unroll
  for (int tg = 0; tg < NTG; ++tg) load_activations(a, kc, 8 * tg + g, t, bf[tg], sf[tg]);
  // One item: decode + mma of both stages from the quads in qq, atomics into y1,
  // then advance the row tile (and the activations at a code-chunk boundary).
  auto process = [&](uint32_t it, const uint4 (&qq)[4]) {
    float acc0[NTG][4], acc0b[NTG][4], acc1[NTG][4], acc1b[NTG][4];
    stage_item<K0, NTG>(tbl, off_e8p, off_1b, qq[0], qq[nquads<K0>() - 1], bf, sf, acc0, acc0b);
    if constexpr (NST == 2) {
      constexpr int o = nquads<K0>();
      stage_item<K1, NTG>(tbl, off_e8p, off_1b, qq[o], qq[o + nquads<K1>() - 1], bf, sf, acc1, acc1b);
    }
    // epilogue: c0 (row g, tok 2t), c1 (row g, tok 2t+1), c2/c3 rows g+8
    const uint32_t row0 = rt * kRowsPerTile + g, row1 = row0 + 8;
#pragma unroll
    for (int tg = 0; tg < NTG; ++tg) {
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int tok = 8 * tg + 2 * t + j;
        if (tok < a.ntok) {
          const uint32_t gt = static_cast<uint32_t>(a.tok0 + tok);
          const float f = tokscale[tg][j];
          float v0 = a.sscale[0] * (acc0[tg][j] + acc0b[tg][j]);
          float v1 = a.sscale[0] * (acc0[tg][2 + j] + acc0b[tg][2 + j]);
          if constexpr (NST == 2) {
            v0 = fmaf(a.sscale[1], acc1[tg][j] + acc1b[tg][j], v0);
            v1 = fmaf(a.sscale[1], acc1[tg][2 + j] + acc1b[tg][2 + j], v1);
          }
          if (row0 < m) atomicAdd(a.y1 + (gt * m + row0), v0 * f);
          if (row1 < m) atomicAdd(a.y1 + (gt * m + row1), v1 * f);
        }
      }
    }
    if (++rt == RT) {
      rt = 0;
      ++kc;
      if (it + 1 < end) {
#pragma unroll
        for (int tg = 0; tg < NTG; ++tg) load_activations(a, kc, 8 * tg + g, t, bf[tg], sf[tg]);
      }
    }
  };
  // two items per trip with ping-pong quad registers (no copies between items)
  for (uint32_t it = start; it < end; it += 2) {
    if (it + 1 < end) load_item<K0, K1, NST>(a, it + 1, lane, nq);
    process(it, q);
    if (it + 1 >= end) break;
    if (it + 2 < end) load_item<K0, K1, NST>(a, it + 2, lane, q);
    process(it + 1, nq);
  }
}

template <int K0, int K1, int NST, int NTG>
__device__ __forceinline__ void gemv_body(const GemvArgs &a, uint8_t *gsm) {
  pdl_launch_dependents();
  // 256-byte aligned table rows: the row index is multiplied by 256 and the
  // lane replica offset (< 256) added in one integer multiply-add
  uint8_t *tbl = gsm + ((256u - (smem_u32(gsm) & 255u)) & 255u);
  const int lane = threadIdx.x & 31;
  const int64_t warp = blockIdx.x * (kGemvThreads / 32) + (threadIdx.x >> 5);
  const int64_t nwarps = static_cast<int64_t>(gridDim.x) * (kGemvThreads / 32);
  const uint32_t start = static_cast<uint32_t>(warp * a.items / nwarps);
  const uint32_t end = static_cast<uint32_t>((warp + 1) * a.items / nwarps);
  // prologue, independent of the previous kernel: first weights in flight, table fill
  uint4 q[4], nq[4];
  if (start < end) load_item<K0, K1, NST>(a, start, lane, q);
  load_table(tbl);
  __syncthreads();
  if (start < end) gemv_items<K0, K1, NST, NTG>(a, tbl, start, end, q, nq);
}

template <int K0, int K1, int NST, int NTG>
__global__ void __launch_bounds__(kGemvThreads, NTG == 1 ? 2 : 1) gemv_kernel(GemvArgs a) {
  extern __shared__ __align__(256) uint8_t gsm[];
  gemv_body<K0, K1, NST, NTG>(a, gsm);
}

template <int K0, int K1, int NST, int NTG>
__global__ void __launch_bounds__(kGemvThreads, NTG == 1 ? 2 : 1) gemv_push_kernel(GemvArgs a, GemvPush p) {
  extern __shared__ __align__(256) uint8_t gsm[];
  gemv_body<K0, K1, NST, NTG>(a, gsm);
  // every thread of every CTA arrives; the broadcast word sits past the table
  tp_push_grid(p.push, p.wait_ns, p.error, reinterpret_cast<unsigned *>(gsm + kTblBytes + 256));
}

static int num_sms() {
  static int cached[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && cached[dev]) return cached[dev];
  int n = 148;
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  if (dev < 64) cached[dev] = n;
  return n;
}

template <int K0, int K1, int NST>
static int run_gemv(GemvArgs &a, int64_t batch, cudaStream_t s, const TpPush *push) {
  // batches above 8: passes of 16 tokens (two token groups); else one pass of 8
  const bool two = batch > 8;
  auto kern = two ? gemv_kernel<K0, K1, NST, 2> : gemv_kernel<K0, K1, NST, 1>;
  auto kpush = two ? gemv_push_kernel<K0, K1, NST, 2> : gemv_push_kernel<K0, K1, NST, 1>;
  QS_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kTblBytes + 256));
  if (push) QS_CUDA_TRY(cudaFuncSetAttribute(kpush, cudaFuncAttributeMaxDynamicSharedMemorySize, kTblBytes + 512));
  const int per_pass = two ? 16 : 8;
  const int64_t warps_needed = a.items;
  int grid = (two ? 1 : 2) * num_sms();
  if (warps_needed < static_cast<int64_t>(grid) * (kGemvThreads / 32))
    grid = static_cast<int>(ceil_div(warps_needed, kGemvThreads / 32));
  for (int64_t tok0 = 0; tok0 < batch; tok0 += per_pass) {
    a.tok0 = static_cast<int>(tok0);
    a.ntok = static_cast<int>(batch - tok0 < per_pass ? batch - tok0 : per_pass);
    int st;
    if (push && tok0 + per_pass >= batch) {  // the last pass pushes every token's rows
      GemvPush p{*push, pipeline_wait_ns(), device_error_flag()};
      if (!p.error) return fail(QS_ERR_CUDA, "device error flag unavailable");
      // table (256-byte aligned inside the first 256 + kTblBytes bytes), then the push's word
      st = launch_pdl("gemv_push", kpush, dim3(grid), dim3(kGemvThreads), kTblBytes + 512, s, a, p);
    } else {
      st = launch_pdl("gemv", kern, dim3(grid), dim3(kGemvThreads), kTblBytes + 256, s, a);
    }
    if (st) return st;
  }
  return QS_OK;
}

int launch_matmul(const void *x2ws, int64_t batch, int64_t n, int64_t m, const void *packed,
                  int stages, const int *kinds, const float *stage_scales,
                  const float *layer_scale, float *y1, cudaStream_t s, const TpPush *push) {
  if (batch >= kTcMinBatch) {
    if (push) return fail(QS_ERR_INVALID_ARG, "the prefill matmul does not push");
    return launch_matmul_tc(x2ws, batch, n, m, packed, stages, kinds, stage_scales, layer_scale, y1, s);
  }
  // the decode kernel indexes with 32 bits
  if (batch * m >= (int64_t(1) << 31) || stage_bytes(QS_CB_E8P, m, n) >= (int64_t(1) << 31) ||
      batch * padded_T(n) * 8 >= (int64_t(1) << 31))
    return fail(QS_ERR_UNSUPPORTED, "decode matmul of %lld x %lld at batch %lld exceeds 32-bit indexing",
                (long long)m, (long long)n, (long long)batch);
  GemvArgs a{};
  a.n_pad = padded_T(n) * 8;
  a.x2h = static_cast<const __half *>(x2ws);
  a.rowscale = reinterpret_cast<const float *>(static_cast<const char *>(x2ws) +
                                               round_up(batch * a.n_pad * 2, 256));
  a.m = m;
  a.RT = padded_m(m) / kRowsPerTile;
  a.KC = padded_T(n) / kCodesPerChunk;
  a.items = a.RT * a.KC;
  a.layer_scale = layer_scale;
  a.y1 = y1;
  const uint8_t *p = static_cast<const uint8_t *>(packed);
  for (int st = 0; st < stages; ++st) {
    a.stage[st] = p;
    a.sscale[st] = stage_scales ? stage_scales[st] : 1.f;
    p += round_up(stage_bytes(kinds[st], m, n), 256);
  }
  const int k0 = kinds[0], k1 = stages == 2 ? kinds[1] : 0;
  if (stages == 1) {
    return k0 == QS_CB_E8P ? run_gemv<QS_CB_E8P, 0, 1>(a, batch, s, push)
                           : run_gemv<QS_CB_E8_1BIT, 0, 1>(a, batch, s, push);
  }
  if (k0 == QS_CB_E8P && k1 == QS_CB_E8_1BIT) return run_gemv<QS_CB_E8P, QS_CB_E8_1BIT, 2>(a, batch, s, push);
  if (k0 == QS_CB_E8P && k1 == QS_CB_E8P) return run_gemv<QS_CB_E8P, QS_CB_E8P, 2>(a, batch, s, push);
  if (k0 == QS_CB_E8_1BIT && k1 == QS_CB_E8P) return run_gemv<QS_CB_E8_1BIT, QS_CB_E8P, 2>(a, batch, s, push);
  return run_gemv<QS_CB_E8_1BIT, QS_CB_E8_1BIT, 2>(a, batch, s, push);
}

}  // namespace qs
