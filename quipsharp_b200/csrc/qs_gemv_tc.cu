// Fused codebook decode + tcgen05 matmul for the decode regime (1 to 32 tokens):
//   y1[tok, row] += layer_scale * rowscale[tok] * sum_s s_s * sum_k x2h[tok, k] * What_s[row, k]
//
// The weights stream from HBM once (packed layout of qs_pack.cu).  Each CTA
// (one per SM) takes a contiguous range of "chunks" -- a chunk is one 128-row
// tile x 128 input features (16 codes per row per stage) -- in row-tile-major
// order, and accumulates each row tile it touches in TMEM; partial sums of a
// tile leave through float32 atomics into y1 (zeroed by the input step).
//
// Warp roles:
//   warp 0      producer: per chunk, one bulk copy of each stage's codes (the
//               chunk's codes are contiguous in the packed stream) and two TMA
//               loads of the activations (64 features x ntok tokens each, 128-byte
//               swizzle, rows ntok.. of the tile stay zero) into a ring stage.
//               The codes of the first stages are requested before waiting for
//               the previous kernel (they do not depend on it);
//   warp 1      allocates TMEM; lane 0 issues tcgen05.mma with A = the decoded
//               weights in TMEM (M = 128 rows, K = 16), B = the activation tile
//               (N = 16 or 32 tokens), D = float32 per stage in TMEM;
//   decode      G groups of four warps taking alternate chunks: thread r of a
//               group owns weight row r (= its TMEM lane), decodes its 16 codes
//               per stage into f16x2 words and writes them to its TMEM lane with
//               tcgen05.st (no shared-memory round trip for the weights).  The
//               +-1/4 E8P shifts are not added per weight: they form a second A
//               operand (one +-0.25 per code) multiplied by the per-code sums of
//               the 8 activations each code covers (computed per chunk by the
//               group, B' tile), i.e. one more K=16 MMA per chunk;
//   epilogue    four warps: per finished row tile, TMEM -> registers -> stage,
//               layer and per-token scales -> atomics into y1, while the MMA
//               fills the other of two TMEM accumulators.
// Decode of one E8P code: one 16-byte shared load of the table row (the four
// f16x2 words of the natural coordinate pairs; the table is replicated 8x so
// the 8 lanes of a quarter warp read distinct banks), then per word one shift
// and one AND-XOR applying the two sign flips (bit layout in qs_pack.cu).
// 1-bit codes: the table words as loaded.  Every decoded value is exact in fp16;
// RVQ stages accumulate separately and meet their float32 stage scales in the
// epilogue.  Every mbarrier wait is bounded (pipeline_wait_ns()); on timeout the
// kernel records an error (qs_device_status) and winds down after draining its
// own copies and MMAs.
#include <cuda.h>

#include <mutex>

#include "qs_common.cuh"
#include "qs_launch.h"
#include "qs_sm100.cuh"

namespace qs {

static __device__ int g_gemv_error;  // set by a bounded wait that ran out

namespace {

constexpr int kChunkCodes = 16;  // codes per row per stage in one chunk (128 input features)
constexpr uint64_t kDrainLimitNs = 4000000000ull;
constexpr int kTableBytes = 256 * 8 * 16;  // 256 rows x 8 replicas x four f16x2 words

__host__ __device__ constexpr int code_bytes(int kind) { return kind == QS_CB_E8P ? 4096 : 2048; }

template <int K0, int K1, int NST, int NT>
struct GCfg {
  static constexpr int groups = NST == 1 ? 4 : (NT == 16 ? 3 : 2);
  static constexpr int stages = NT == 16 ? 8 : 6;
  static constexpr int threads = 32 * (2 + 4 * groups + 4);
  static constexpr int epi_warp0 = 2 + 4 * groups;
  // TMEM: D[2 accumulators][NST stages][NT tokens], then per group and stage the
  // 64 columns of decoded weights (128 fp16 per row) and 8 columns of shifts.
  static constexpr int d_cols = 2 * NST * NT;
  static constexpr int a_cols = 72 * NST;
  static constexpr int tmem_used = d_cols + groups * a_cols;
  static constexpr uint32_t tmem_cols = tmem_used <= 256 ? 256 : 512;
  static_assert(tmem_used <= 512, "TMEM budget");
  // ring stage: B (2 K-blocks x NT rows x 128 B, 128-byte swizzle), B' (NT rows x
  // 128 B, codes 0..15 in the first 32 bytes of each row), then the codes
  static constexpr int b_off = 0;
  static constexpr int bp_off = 2 * NT * 128;
  static constexpr int c0_off = bp_off + NT * 128;
  static constexpr int c1_off = c0_off + code_bytes(K0);
  static constexpr int stage_bytes = ((c1_off + (NST == 2 ? code_bytes(K1) : 0) + 1023) / 1024) * 1024;
  static constexpr int ring_bytes = stages * stage_bytes;
  static constexpr int bar_bytes = 256;
  // at least 118 KB so two CTAs of the tcgen05 kernels never share an SM (each
  // allocates TMEM up front and holds it until exit)
  static constexpr int needed = 1024 + ring_bytes + NST * kTableBytes + bar_bytes;
  static constexpr int smem_bytes = needed < 118 * 1024 ? 118 * 1024 : needed;
  static_assert(smem_bytes <= 227 * 1024, "shared memory budget");
};

struct GvArgs {
  const uint8_t *stage[2];
  float sscale[2];
  const float *layer_scale;
  const float *rowscale;  // (batch)
  float *y1;              // (batch, m)
  int64_t m;
  int64_t Tq;  // code groups (of 8) per row in the packed stream
  int kch;     // chunks per row tile
  int total;   // row tiles x chunks
  int ntok;
  uint64_t wait_ns;
};

__device__ __forceinline__ void set_error() { atomicExch(&g_gemv_error, 1); }

// Four f16x2 words of the natural coordinate pairs of a table row (every entry
// of both codebooks has a zero fp16 low byte).
__device__ __forceinline__ uint4 pair_words(uint2 hb) {
  return make_uint4(prmt(hb.x, 0u, 0x1404u), prmt(hb.x, 0u, 0x3424u), prmt(hb.y, 0u, 0x1404u),
                    prmt(hb.y, 0u, 0x3424u));
}

__device__ __forceinline__ void fill_table(uint8_t *tbl, int kind) {
  for (int i = threadIdx.x; i < 256 * 8; i += blockDim.x) {
    const int row = i >> 3;
    reinterpret_cast<uint4 *>(tbl)[i] = pair_words(kind == QS_CB_E8P ? kE8pHiBytes[row] : kE81BitHiBytes[row]);
  }
}

// Table row of the code whose index is byte csel of idxsrc (tbl already offset
// to this lane's replica).
__device__ __forceinline__ uint4 table_row(const uint8_t *tbl, uint32_t idxsrc, int csel) {
  const uint32_t idx = prmt(idxsrc, 0u, 0x4440u | static_cast<uint32_t>(csel));
  return *reinterpret_cast<const uint4 *>(tbl + idx * 128u);
}

// One stage of one chunk for this thread's row: 16 codes -> 64 TMEM columns of
// f16x2 words at a_addr (+ 8 columns of shift words for E8P).
template <int K>
__device__ __forceinline__ void decode_chunk_row(const uint8_t *codes, int r, const uint8_t *tbl, uint32_t a_addr) {
  if constexpr (K == QS_CB_E8P) {
    uint32_t sw[8];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint4 q = *reinterpret_cast<const uint4 *>(codes + h * 2048 + r * 16);
      const uint32_t fa = q.z ^ imul(q.z, 256u);
      const uint32_t fb = (q.w & 0x00FFFFFFu) ^ shf_l_wrap(q.z, q.w, 8);
      const uint32_t fa8 = imul(fa, 256u), fb8 = imul(fb, 256u);
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        uint32_t w[16];
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) {
          const int c = 4 * half + cc;
          const uint4 T = table_row(tbl, c < 4 ? q.x : q.y, c & 3);
          w[4 * cc + 0] = T.x ^ (imul(fa, 1u << c) & 0x80008000u);
          w[4 * cc + 1] = T.y ^ (imul(fa8, 1u << c) & 0x80008000u);
          w[4 * cc + 2] = T.z ^ (imul(fb, 1u << c) & 0x80008000u);
          w[4 * cc + 3] = T.w ^ (imul(fb8, 1u << c) & 0x80008000u);
        }
        sm100::tmem_st_16(a_addr + 32 * h + 16 * half, w);
      }
      // +-1/4 of codes (2p, 2p+1) in the (low, high) halves; w3 bit 31 - c = NOT shift_c
      const uint32_t u = prmt(q.w, imul(q.w, 2u), 0x7030u);
#pragma unroll
      for (int p = 0; p < 4; ++p) sw[4 * h + p] = 0x34003400u ^ (imul(u, 1u << (2 * p)) & 0x80008000u);
    }
    sm100::tmem_st_8(a_addr + 64, sw);
  } else {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint2 q = *reinterpret_cast<const uint2 *>(codes + h * 1024 + r * 8);
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        uint32_t w[16];
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) {
          const uint4 T = table_row(tbl, half == 0 ? q.x : q.y, cc);
          w[4 * cc + 0] = T.x;
          w[4 * cc + 1] = T.y;
          w[4 * cc + 2] = T.z;
          w[4 * cc + 3] = T.w;
        }
        sm100::tmem_st_16(a_addr + 32 * h + 16 * half, w);
      }
    }
  }
}

template <int K0, int K1, int NST, int NT>
__global__ void __launch_bounds__(GCfg<K0, K1, NST, NT>::threads, 1)
    gemv_tc_kernel(const __grid_constant__ CUtensorMap tmap_x, GvArgs a) {
  using C = GCfg<K0, K1, NST, NT>;
  constexpr int S = C::stages, G = C::groups;
  extern __shared__ __align__(1024) uint8_t dsm[];
  pdl_launch_dependents();
  uint8_t *ring = dsm + ((1024u - (smem_u32(dsm) & 1023u)) & 1023u);
  uint8_t *tbl0 = ring + C::ring_bytes;
  uint8_t *tbl1 = tbl0 + kTableBytes;
  uint64_t *bars = reinterpret_cast<uint64_t *>(tbl0 + NST * kTableBytes);
  // bars: full[S], empty[S], a_full[G], a_empty[G], acc_full[2], acc_empty[2], drain, TMEM holder
  const uint32_t bar0 = smem_u32(bars);
  auto full = [&](int s) { return bar0 + 8u * s; };
  auto empty = [&](int s) { return bar0 + 8u * (S + s); };
  auto a_full = [&](int g) { return bar0 + 8u * (2 * S + g); };
  auto a_empty = [&](int g) { return bar0 + 8u * (2 * S + G + g); };
  auto acc_full = [&](int b) { return bar0 + 8u * (2 * S + 2 * G + b); };
  auto acc_empty = [&](int b) { return bar0 + 8u * (2 * S + 2 * G + 2 + b); };
  const uint32_t drain = bar0 + 8u * (2 * S + 2 * G + 4);
  uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(bars + 2 * S + 2 * G + 5);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  const int start = static_cast<int>(static_cast<int64_t>(blockIdx.x) * a.total / gridDim.x);
  const int end = static_cast<int>(static_cast<int64_t>(blockIdx.x + 1) * a.total / gridDim.x);
  const int nq = end - start;

  // ---- setup (independent of the previous kernel)
  fill_table(tbl0, K0);
  if constexpr (NST == 2) fill_table(tbl1, K1);
  // B / B' tiles start at zero: the token rows the loads never write stay zero
  for (int i = threadIdx.x; i < S * (C::c0_off / 16); i += blockDim.x) {
    const int s = i / (C::c0_off / 16), o = i % (C::c0_off / 16);
    reinterpret_cast<uint4 *>(ring + s * C::stage_bytes)[o] = make_uint4(0u, 0u, 0u, 0u);
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      sm100::mbar_init(full(s), 1);
      sm100::mbar_init(empty(s), 1);
    }
    for (int g = 0; g < G; ++g) {
      sm100::mbar_init(a_full(g), 128);
      sm100::mbar_init(a_empty(g), 1);
    }
    for (int b = 0; b < 2; ++b) {
      sm100::mbar_init(acc_full(b), 1);
      sm100::mbar_init(acc_empty(b), 128);
    }
    sm100::mbar_init(drain, 1);
    sm100::fence_barrier_init();
    sm100::prefetch_tmap(&tmap_x);
  }
  if (warp == 1) sm100::tmem_alloc(smem_u32(tmem_holder), C::tmem_cols);
  sm100::fence_proxy_async_smem();  // the zero fill before any TMA write / MMA read of it
  sm100::tc_fence_before_sync();
  __syncthreads();
  sm100::tc_fence_after_sync();
  const uint32_t tmem = *tmem_holder;

  if (warp == 0) {
    // ---- producer
    if (lane == 0 && nq > 0) {
      const uint32_t tx = code_bytes(K0) + (NST == 2 ? code_bytes(K1) : 0) + 2u * a.ntok * 128u;
      auto load_codes = [&](int q) {
        const int u = start + q, rt = u / a.kch, c = u % a.kch;
        uint8_t *st = ring + (q % S) * C::stage_bytes;
        const int64_t grp = rt * a.Tq + 2 * c;  // first code group of the chunk
        sm100::bulk_g2s(smem_u32(st + C::c0_off), a.stage[0] + grp * (code_bytes(K0) / 2), code_bytes(K0),
                        full(q % S));
        if constexpr (NST == 2)
          sm100::bulk_g2s(smem_u32(st + C::c1_off), a.stage[1] + grp * (code_bytes(K1) / 2), code_bytes(K1),
                          full(q % S));
      };
      auto load_x = [&](int q) {
        const int c = (start + q) % a.kch;
        uint8_t *st = ring + (q % S) * C::stage_bytes;
        sm100::tma_load_2d(smem_u32(st + C::b_off), &tmap_x, c * 128, 0, full(q % S));
        sm100::tma_load_2d(smem_u32(st + C::b_off + NT * 128), &tmap_x, c * 128 + 64, 0, full(q % S));
      };
      const int npre = nq < S ? nq : S;
      for (int q = 0; q < npre; ++q) {
        sm100::mbar_arrive_expect_tx(full(q), tx);
        load_codes(q);
      }
      pdl_wait();  // x2h comes from the input-transform kernel
      for (int q = 0; q < npre; ++q) load_x(q);
      int issued = npre;
      for (int q = npre; q < nq; ++q) {
        const int s = q % S;
        if (!sm100::mbar_wait_bounded(empty(s), static_cast<uint32_t>(((q / S) - 1) & 1), a.wait_ns)) {
          set_error();
          break;
        }
        sm100::mbar_arrive_expect_tx(full(s), tx);
        load_codes(q);
        load_x(q);
        issued = q + 1;
      }
      // wind down: every copy this thread issued must have landed before the CTA exits
      for (int q = issued > S ? issued - S : 0; q < issued; ++q)
        if (!sm100::mbar_wait_bounded(full(q % S), static_cast<uint32_t>((q / S) & 1), kDrainLimitNs)) set_error();
    }
  } else if (warp == 1) {
    // ---- MMA issuer
    if (lane == 0 && nq > 0) {
      constexpr uint32_t idesc = sm100::idesc_f16_f32(kRowTile, NT);
      const int rt0 = start / a.kch;
      for (int q = 0; q < nq; ++q) {
        const int u = start + q, rt = u / a.kch, tile = rt - rt0, b = tile & 1;
        const bool first = q == 0 || u % a.kch == 0;
        const bool last = q == nq - 1 || (u + 1) % a.kch == 0;
        if (first && tile >= 2 &&
            !sm100::mbar_wait_bounded(acc_empty(b), static_cast<uint32_t>(((tile >> 1) - 1) & 1), a.wait_ns)) {
          set_error();
          break;
        }
        const int g = q % G, s = q % S;
        if (!sm100::mbar_wait_bounded(a_full(g), static_cast<uint32_t>((q / G) & 1), a.wait_ns)) {
          set_error();
          break;
        }
        sm100::tc_fence_after_sync();
        const uint32_t st = smem_u32(ring + s * C::stage_bytes);
        const uint64_t bd[2] = {sm100::sw128_kmajor_desc(st + C::b_off),
                                sm100::sw128_kmajor_desc(st + C::b_off + NT * 128)};
        const uint64_t bpd = sm100::sw128_kmajor_desc(st + C::bp_off);
        const uint32_t ag = tmem + C::d_cols + g * C::a_cols;
#pragma unroll
        for (int j = 0; j < NST; ++j) {
          const uint32_t d = tmem + (b * NST + j) * NT, aj = ag + 72 * j;
#pragma unroll
          for (int k = 0; k < 8; ++k)  // K = 16 per MMA: +32 bytes in the swizzled 128-byte row
            sm100::umma_f16_ts(d, aj + 8 * k, bd[k >> 2] + 2 * (k & 3), idesc, !(first && k == 0));
          if ((j == 0 ? K0 : K1) == QS_CB_E8P) sm100::umma_f16_ts(d, aj + 64, bpd, idesc, 1u);
        }
        sm100::umma_commit(a_empty(g));
        sm100::umma_commit(empty(s));
        if (last) sm100::umma_commit(acc_full(b));
      }
      // wind down: every MMA issued must be complete before TMEM and the ring are freed
      sm100::umma_commit(drain);
      if (!sm100::mbar_wait_bounded(drain, 0, kDrainLimitNs)) set_error();
    }
  } else if (warp < C::epi_warp0) {
    // ---- decode groups: thread <-> weight row r of the tile (its TMEM lane)
    const int g = (warp - 2) >> 2;
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const int gt = ((warp - 2) & 3) * 32 + lane;  // thread index within the group
    const uint32_t a0 = tmem + (static_cast<uint32_t>(quarter * 32) << 16) + C::d_cols + g * C::a_cols;
    const uint8_t *t0 = tbl0 + (lane & 7) * 16, *t1 = tbl1 + (lane & 7) * 16;
    for (int j = 0;; ++j) {
      const int q = g + G * j;
      if (q >= nq) break;
      const int s = q % S;
      if (!sm100::mbar_wait_warp(full(s), static_cast<uint32_t>((q / S) & 1), a.wait_ns)) {
        set_error();
        break;
      }
      if (j > 0 && !sm100::mbar_wait_warp(a_empty(g), static_cast<uint32_t>((j - 1) & 1), a.wait_ns)) {
        set_error();
        break;
      }
      sm100::tc_fence_after_sync();
      uint8_t *st = ring + s * C::stage_bytes;
      if (K0 == QS_CB_E8P || (NST == 2 && K1 == QS_CB_E8P)) {
        // B': sum of the 8 activations of each code of the chunk, per token (fp16)
        for (int i = gt; i < a.ntok * kChunkCodes; i += 128) {
          const int t = i >> 4, c = i & 15;
          const uint8_t *row = st + C::b_off + (c >> 3) * (NT * 128) + (t >> 3) * 1024 + (t & 7) * 128;
          const uint4 v = *reinterpret_cast<const uint4 *>(row + (((c & 7) ^ (t & 7)) << 4));
          const float2 f0 = __half22float2(*reinterpret_cast<const __half2 *>(&v.x));
          const float2 f1 = __half22float2(*reinterpret_cast<const __half2 *>(&v.y));
          const float2 f2 = __half22float2(*reinterpret_cast<const __half2 *>(&v.z));
          const float2 f3 = __half22float2(*reinterpret_cast<const __half2 *>(&v.w));
          const float sum = ((f0.x + f0.y) + (f1.x + f1.y)) + ((f2.x + f2.y) + (f3.x + f3.y));
          __half *bp = reinterpret_cast<__half *>(st + C::bp_off + (t >> 3) * 1024 + (t & 7) * 128 +
                                                  (((c >> 3) ^ (t & 7)) << 4)) +
                       (c & 7);
          *bp = __float2half_rn(sum);
        }
        sm100::fence_proxy_async_smem();  // B' before the MMA reads it
        __syncwarp();                     // converged again for the warp-collective TMEM stores
      }
      decode_chunk_row<K0>(st + C::c0_off, r, t0, a0);
      if constexpr (NST == 2) decode_chunk_row<K1>(st + C::c1_off, r, t1, a0 + 72);
      sm100::tmem_st_wait();
      sm100::tc_fence_before_sync();
      sm100::mbar_arrive(a_full(g));
    }
  } else {
    // ---- epilogue: TMEM lane quarter warp & 3
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
    pdl_wait();  // rowscale and the zeroed y1 come from the input-transform kernel
    if (nq > 0) {
      const float ls = *a.layer_scale;
      const int rt0 = start / a.kch, rt1 = (end - 1) / a.kch;
      for (int rt = rt0; rt <= rt1; ++rt) {
        const int tile = rt - rt0, b = tile & 1;
        if (!sm100::mbar_wait_warp(acc_full(b), static_cast<uint32_t>((tile >> 1) & 1), a.wait_ns)) {
          set_error();
          break;
        }
        sm100::tc_fence_after_sync();
        float v0[NT], v1[NT];
        {
          uint32_t u0[NT], u1[NT];
          if constexpr (NT == 16) {
            sm100::tmem_ld_16(lane_base + (b * NST) * NT, u0);
            if constexpr (NST == 2) sm100::tmem_ld_16(lane_base + (b * NST + 1) * NT, u1);
          } else {
            sm100::tmem_ld_32(lane_base + (b * NST) * NT, u0);
            if constexpr (NST == 2) sm100::tmem_ld_32(lane_base + (b * NST + 1) * NT, u1);
          }
          sm100::tmem_ld_wait();
#pragma unroll
          for (int t = 0; t < NT; ++t) {
            v0[t] = __uint_as_float(u0[t]);
            v1[t] = NST == 2 ? __uint_as_float(u1[t]) : 0.f;
          }
        }
        sm100::tc_fence_before_sync();
        sm100::mbar_arrive(acc_empty(b));
        const int64_t row = static_cast<int64_t>(rt) * kRowTile + r;
        if (row < a.m) {
#pragma unroll
          for (int t = 0; t < NT; ++t) {
            if (t < a.ntok) {
              float v = a.sscale[0] * v0[t];
              if constexpr (NST == 2) v = fmaf(a.sscale[1], v1[t], v);
              atomicAdd(a.y1 + (static_cast<int64_t>(t) * a.m + row), v * (ls * a.rowscale[t]));
            }
          }
        }
      }
    }
  }
  // ---- teardown
  sm100::tc_fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    sm100::tc_fence_after_sync();
    sm100::tmem_dealloc(tmem, C::tmem_cols);
  }
}

int gemv_num_sms() {
  static int cached[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && cached[dev]) return cached[dev];
  int n = 148;
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  if (dev < 64) cached[dev] = n;
  return n;
}

template <int K0, int K1, int NST, int NT>
int run_gemv_tc(const CUtensorMap &map, const GvArgs &a, cudaStream_t s) {
  using C = GCfg<K0, K1, NST, NT>;
  auto kern = gemv_tc_kernel<K0, K1, NST, NT>;
  QS_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::smem_bytes));
  const int grid = a.total < gemv_num_sms() ? a.total : gemv_num_sms();
  return launch_pdl("gemv_tc", kern, dim3(grid), dim3(C::threads), C::smem_bytes, s, map, a);
}

template <int K0, int K1, int NST>
int run_gemv_nt(const CUtensorMap &map, const GvArgs &a, cudaStream_t s) {
  return a.ntok <= 16 ? run_gemv_tc<K0, K1, NST, 16>(map, a, s) : run_gemv_tc<K0, K1, NST, 32>(map, a, s);
}

}  // namespace

int take_gemv_error(cudaStream_t s, int *flag) {
  static const int zero = 0;
  *flag = 0;
  QS_CUDA_TRY(cudaMemcpyFromSymbolAsync(flag, g_gemv_error, sizeof(int), 0, cudaMemcpyDeviceToHost, s));
  QS_CUDA_TRY(cudaStreamSynchronize(s));
  if (*flag) {
    QS_CUDA_TRY(cudaMemcpyToSymbolAsync(g_gemv_error, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, s));
    QS_CUDA_TRY(cudaStreamSynchronize(s));
  }
  return QS_OK;
}

int launch_matmul(const void *x2ws, int64_t batch, int64_t n, int64_t m, const void *packed,
                  int stages, const int *kinds, const float *stage_scales,
                  const float *layer_scale, float *y1, cudaStream_t s) {
  if (batch >= kTcMinBatch)
    return launch_matmul_tc(x2ws, batch, n, m, packed, stages, kinds, stage_scales, layer_scale, y1, s);
  const int64_t n_pad = padded_T(n) * 8;
  const int64_t tiles = padded_m(m) / kRowTile, kch = n_pad / (8 * kChunkCodes);
  if (tiles * kch >= (int64_t(1) << 31))
    return fail(QS_ERR_UNSUPPORTED, "decode matmul of %lld x %lld exceeds the chunk index range", (long long)m,
                (long long)n);
  GvArgs a{};
  a.rowscale = reinterpret_cast<const float *>(static_cast<const char *>(x2ws) + round_up(batch * n_pad * 2, 256));
  a.layer_scale = layer_scale;
  a.y1 = y1;
  a.m = m;
  a.Tq = n_pad / 8 / 8;
  a.kch = static_cast<int>(kch);
  a.total = static_cast<int>(tiles * kch);
  a.ntok = static_cast<int>(batch);
  a.wait_ns = pipeline_wait_ns();
  const uint8_t *p = static_cast<const uint8_t *>(packed);
  for (int st = 0; st < stages; ++st) {
    a.stage[st] = p;
    a.sscale[st] = stage_scales ? stage_scales[st] : 1.f;
    p += round_up(stage_bytes(kinds[st], m, n), 256);
  }
  CUtensorMap map;
  int st = encode_fp16_rows_map(&map, x2ws, n_pad, batch, 64, static_cast<int>(batch), true);
  if (st) return st;
  const int k0 = kinds[0], k1 = stages == 2 ? kinds[1] : 0;
  if (stages == 1)
    return k0 == QS_CB_E8P ? run_gemv_nt<QS_CB_E8P, 0, 1>(map, a, s) : run_gemv_nt<QS_CB_E8_1BIT, 0, 1>(map, a, s);
  if (k0 == QS_CB_E8P && k1 == QS_CB_E8_1BIT) return run_gemv_nt<QS_CB_E8P, QS_CB_E8_1BIT, 2>(map, a, s);
  if (k0 == QS_CB_E8P && k1 == QS_CB_E8P) return run_gemv_nt<QS_CB_E8P, QS_CB_E8P, 2>(map, a, s);
  if (k0 == QS_CB_E8_1BIT && k1 == QS_CB_E8P) return run_gemv_nt<QS_CB_E8_1BIT, QS_CB_E8P, 2>(map, a, s);
  return run_gemv_nt<QS_CB_E8_1BIT, QS_CB_E8_1BIT, 2>(map, a, s);
}

}  // namespace qs
