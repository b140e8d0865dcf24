// Fused codebook decode + tcgen05 GEMM for prefill-sized batches:
//   y1[tok, row] = layer_scale * rowscale[tok] * sum_s s_s * sum_k x2h[tok, k] * What_s[row, k]
//
// CTA tile: 128 weight rows (M, TMEM lanes) x 256 tokens (N, TMEM columns),
// K in steps of 64 input features (one 128-byte swizzled row per operand row).
// Warp roles (64 + 128 G threads, G decode groups: 4 for one-stage codebooks,
// 2 for two-stage RVQ):
//   warp 0      TMA producer: the activation tile (256 tokens x 64 fp16) of each
//               K step into a 4- (3-) stage ring, 128-byte swizzle;
//   warp 1      allocates TMEM; lane 0 issues tcgen05.mma (M=128, N=256, K=16,
//               fp16 x fp16 -> fp32) and tcgen05.commit to free ring stages;
//   warps 2..   decode, in G groups of four warps taking alternate K steps:
//               thread r of a group decodes weight row r of the tile (8 codes,
//               read from the same packed stream as the decode-regime kernel)
//               into the A tile of the ring stage, in the UMMA K-major
//               128-byte-swizzle layout; then the epilogue, each group over
//               1/G of the token columns: TMEM -> registers -> scales -> y1
//               (float32, coalesced per token).
// Decoded weights are exact in fp16 (the E8P shift is added with an f16x2 add),
// RVQ stages accumulate in separate TMEM accumulators and meet their float32
// stage scales in the epilogue.  Every mbarrier wait is bounded: on timeout the
// kernel records an error (read by qs_device_status) and winds down.
#include <cuda.h>

#include <atomic>
#include <mutex>

#include "qs_common.cuh"
#include "qs_launch.h"
#include "qs_sm100.cuh"

namespace qs {

static __device__ int g_tc_error;  // set by a bounded wait that ran out

namespace {

constexpr int kBM = 128;
constexpr int kBN = 256;
constexpr int kBK = 64;
constexpr int kATile = kBM * kBK * 2;  // 16 KB
constexpr int kBTile = kBN * kBK * 2;  // 32 KB
// Drains (waiting for this CTA's own TMA loads and tensor-core ops before it
// frees shared memory and TMEM) always use this long limit: those operations
// complete by themselves, so only a broken GPU could exhaust it.  Pipeline waits
// (on other warps of the CTA) use the run-time limit passed in TcArgs::wait_ns.
constexpr uint64_t kDrainLimitNs = 4000000000ull;

// Ring stages and decode groups.  A decode group waiting for the MMA to free
// stage s for its K step ks relies on the MMA having consumed ks - 2S already
// (otherwise the parity wait could pass one phase early); its own previous
// wait, at ks - G, guarantees consumption of ks - G - S, so G <= S is required.
template <int NST>
struct Cfg {
  static constexpr int stages = NST == 1 ? 4 : 3;
  static constexpr int groups = NST == 1 ? 4 : 2;  // <= stages, divides the 4 K steps of a code chunk
  static constexpr int threads = 64 + 128 * groups;
  static_assert(groups <= stages && 4 % groups == 0, "decode groups vs ring stages");
  static constexpr int stage_bytes = NST * kATile + kBTile;
  static constexpr int ring_bytes = stages * stage_bytes;
  // codebook tables of the stages' kinds, each row replicated `reps` times so the
  // lanes of a warp read their own copies (bank-conflict free for 16 replicas:
  // a 128-byte row holds one 8-byte replica per bank pair)
  static constexpr int reps = NST == 1 ? 16 : 8;
  static constexpr int table_entries = 256 * reps;
  static constexpr int tables_bytes = NST * table_entries * 8;
  static constexpr int bar_bytes = 256;
  static constexpr int smem_bytes = 1024 /*align slack*/ + ring_bytes + tables_bytes + bar_bytes;
  static constexpr uint32_t tmem_cols = NST * kBN;
};

struct TcArgs {
  const uint8_t *stage[2];
  float sscale[2];
  const float *layer_scale;
  const float *rowscale;
  float *y1;
  int64_t m, m_pad, RT, batch;  // RT: 16-row tiles of the packed stream
  int ksteps;
  uint64_t wait_ns;  // limit of every pipeline wait (pipeline_wait_ns())
};

__device__ __forceinline__ void set_error() { atomicExch(&g_tc_error, 1); }

// E8P: 8 codes of one row (a packed quad) -> 8 x 16-byte chunks of fp16
// weights (shift included), written to the row's swizzled positions.  The
// table holds each entry's fp16 high bytes in the sign bit-slice order of the
// quad (coordinates 2, 0, 3, 1 and 6, 4, 7, 5, qs_pack.cu), so one AND-XOR applies
// four flips; byte permutes then give the natural f16x2 pairs.
__device__ __forceinline__ void decode_e8p_row(const uint4 &q, const uint2 *tbl, int reps, uint8_t *arow, int rsw) {
  const uint32_t fa = q.z ^ (q.z << 8);
  const uint32_t fb = (q.w & 0x00FFFFFFu) ^ shf_l_wrap(q.z, q.w, 8);
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    const uint32_t src = c < 4 ? q.x : q.y;
    const uint32_t idx = (src >> (8 * (c & 3))) & 0xFFu;
    const uint2 T = tbl[idx * reps];
    const uint32_t tl = T.x ^ ((fa << c) & 0x80808080u);
    const uint32_t th = T.y ^ ((fb << c) & 0x80808080u);
    const uint32_t sw = 0x34003400u ^ (prmt(q.w << c, 0u, 0xB4B4u) & 0x80008000u);
    uint4 w;
    w.x = hadd2_u32(prmt(tl, 0u, 0x3414u), sw);  // (0, 1)
    w.y = hadd2_u32(prmt(tl, 0u, 0x2404u), sw);  // (2, 3)
    w.z = hadd2_u32(prmt(th, 0u, 0x3414u), sw);  // (4, 5)
    w.w = hadd2_u32(prmt(th, 0u, 0x2404u), sw);  // (6, 7)
    *reinterpret_cast<uint4 *>(arow + ((c ^ rsw) << 4)) = w;
  }
}

// Table row of the prefill decode: E8P high bytes reordered to the quad's
// sign bit-slice order; 1-bit high bytes in natural order.
__device__ __forceinline__ uint2 gemm_table_entry(int kind, int row) {
  if (kind == QS_CB_E8P) {
    const uint2 h = kE8pHiBytes[row];
    return make_uint2(prmt(h.x, 0u, 0x1302u), prmt(h.y, 0u, 0x1302u));
  }
  return kE81BitHiBytes[row];
}

// 1-bit: 8 index bytes of one row -> 8 chunks.
__device__ __forceinline__ void decode_1bit_row(const uint2 &q, const uint2 *tbl, int reps, uint8_t *arow, int rsw) {
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    const uint32_t src = c < 4 ? q.x : q.y;
    const uint2 T = tbl[((src >> (8 * (c & 3))) & 0xFFu) * reps];
    uint4 w;
    w.x = prmt(T.x, 0u, 0x1404u);
    w.y = prmt(T.x, 0u, 0x3424u);
    w.z = prmt(T.y, 0u, 0x1404u);
    w.w = prmt(T.y, 0u, 0x3424u);
    *reinterpret_cast<uint4 *>(arow + ((c ^ rsw) << 4)) = w;
  }
}

// Per-row codes of one decode group's K steps within a 32-code chunk (4 K
// steps; group dg of G takes steps dg, dg + G, ...): a 16-byte quad per K step
// for E8P, 8 index bytes per K step for 1-bit.
template <int K, int SPG>
struct RowChunk;
template <int SPG>
struct RowChunk<QS_CB_E8P, SPG> {
  uint4 q[SPG];
};
template <int SPG>
struct RowChunk<QS_CB_E8_1BIT, SPG> {
  uint2 q[SPG];
};

template <int K, int G>
__device__ __forceinline__ void load_row_chunk(const uint8_t *stage, int64_t RT, int64_t kc, int64_t R, int dg,
                                               bool valid, RowChunk<K, 4 / G> &rc) {
  // item (kc, R / 16) of the packed stream; this row's quads in it (qs_pack.cu)
  const int64_t rtg = R >> 4, rr = R & 15, half = rr >> 3, g = rr & 7;
  if constexpr (K == QS_CB_E8P) {
    const uint8_t *p = stage + (kc * RT + rtg) * 1024 + half * 512 + g * 64;
#pragma unroll
    for (int u = 0; u < 4 / G; ++u) rc.q[u] = valid ? ldg_nc_v4(p + 16 * (dg + G * u)) : make_uint4(0u, 0u, 0u, 0u);
  } else {
    const uint8_t *p = stage + (kc * RT + rtg) * 512 + g * 64 + half * 8;
#pragma unroll
    for (int u = 0; u < 4 / G; ++u)
      rc.q[u] = valid ? __ldg(reinterpret_cast<const uint2 *>(p + 16 * (dg + G * u))) : make_uint2(0u, 0u);
  }
}

template <int K, int SPG>
__device__ __forceinline__ void decode_row(const RowChunk<K, SPG> &rc, int t, const uint2 *tbl, int reps,
                                           uint8_t *arow, int rsw) {
  // tbl: this stage's table already offset to the thread's replica
  if constexpr (K == QS_CB_E8P) decode_e8p_row(rc.q[t], tbl, reps, arow, rsw);
  else decode_1bit_row(rc.q[t], tbl, reps, arow, rsw);
}

template <int K0, int K1, int NST>
__global__ void __launch_bounds__(Cfg<NST>::threads, 1) gemm_tc_kernel(const __grid_constant__ CUtensorMap tmap_x,
                                                               TcArgs a) {
  using C = Cfg<NST>;
  constexpr int S = C::stages, G = C::groups, SPG = 4 / G;
  extern __shared__ __align__(1024) uint8_t dsm[];
  pdl_launch_dependents();
  // 1024-byte aligned ring (the swizzle atom); tables and barriers after it.
  uint8_t *base = dsm + ((1024u - (smem_u32(dsm) & 1023u)) & 1023u);
  uint8_t *ring = base;
  uint2 *tbl0 = reinterpret_cast<uint2 *>(base + C::ring_bytes);  // stage 0's codebook
  uint2 *tbl1 = tbl0 + C::table_entries;                            // stage 1's (RVQ)
  uint64_t *bars = reinterpret_cast<uint64_t *>(base + C::ring_bytes + C::tables_bytes);
  // bars: full_a[S], full_b[S], empty[S], acc_full, drain, then the TMEM address holder
  const uint32_t bar0 = smem_u32(bars);
  auto full_a = [&](int s) { return bar0 + 8u * s; };
  auto full_b = [&](int s) { return bar0 + 8u * (S + s); };
  auto empty = [&](int s) { return bar0 + 8u * (2 * S + s); };
  const uint32_t acc_full = bar0 + 8u * (3 * S);
  const uint32_t drain = bar0 + 8u * (3 * S + 1);
  uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(bars + 3 * S + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t m0 = static_cast<int64_t>(blockIdx.x) * kBM;
  const int n0 = blockIdx.y * kBN;

  // ---- setup (independent of the previous kernel)
  for (int i = threadIdx.x; i < C::table_entries; i += blockDim.x) {
    const int row = i / C::reps;
    tbl0[i] = gemm_table_entry(K0, row);
    if constexpr (NST == 2) tbl1[i] = gemm_table_entry(K1, row);
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      sm100::mbar_init(full_a(s), 128);
      sm100::mbar_init(full_b(s), 1);
      sm100::mbar_init(empty(s), 1);
    }
    sm100::mbar_init(acc_full, 1);
    sm100::mbar_init(drain, 1);
    sm100::fence_barrier_init();
    sm100::prefetch_tmap(&tmap_x);
  }
  if (warp == 1) sm100::tmem_alloc(smem_u32(tmem_holder), C::tmem_cols);
  sm100::tc_fence_before_sync();
  __syncthreads();
  sm100::tc_fence_after_sync();
  const uint32_t tmem = *tmem_holder;
  pdl_wait();  // x2h / rowscale come from the input-transform kernel

  const int K = a.ksteps;
  if (warp == 0) {
    // ---- TMA producer
    if (lane == 0) {
      int issued = 0;
      for (int ks = 0; ks < K; ++ks) {
        const int s = ks % S, use = ks / S;
        if (use > 0 && !sm100::mbar_wait_bounded(empty(s), (use - 1) & 1, a.wait_ns)) {
          set_error();
          break;
        }
        uint8_t *bt = ring + s * C::stage_bytes + NST * kATile;
        sm100::mbar_arrive_expect_tx(full_b(s), kBTile);
        sm100::tma_load_2d(smem_u32(bt), &tmap_x, ks * kBK, n0, full_b(s));
        issued = ks + 1;
      }
      // wind down: every load this thread issued must have landed before the CTA exits
      for (int ks = issued > S ? issued - S : 0; ks < issued; ++ks)
        if (!sm100::mbar_wait_bounded(full_b(ks % S), (ks / S) & 1, kDrainLimitNs)) set_error();
    }
  } else if (warp == 1) {
    // ---- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = sm100::idesc_f16_f32(kBM, kBN);
      bool ok = true;
      for (int ks = 0; ks < K && ok; ++ks) {
        const int s = ks % S, use = ks / S;
        ok = sm100::mbar_wait_bounded(full_a(s), use & 1, a.wait_ns) &&
             sm100::mbar_wait_bounded(full_b(s), use & 1, a.wait_ns);
        if (!ok) {
          set_error();
          break;
        }
        sm100::tc_fence_after_sync();
        uint8_t *st = ring + s * C::stage_bytes;
        const uint64_t bdesc = sm100::sw128_kmajor_desc(smem_u32(st + NST * kATile));
#pragma unroll
        for (int j = 0; j < NST; ++j) {
          const uint64_t adesc = sm100::sw128_kmajor_desc(smem_u32(st + j * kATile));
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k)  // +32 bytes per K=16 slice inside the swizzled row
            sm100::umma_f16(tmem + j * kBN, adesc + 2 * k, bdesc + 2 * k, idesc, (ks | k) != 0);
        }
        sm100::umma_commit(empty(s));
      }
      sm100::umma_commit(acc_full);
      // wind down: every MMA issued must be complete before TMEM and the ring are freed
      // (on the error path nobody else waits for them)
      sm100::umma_commit(drain);
      if (!sm100::mbar_wait_bounded(drain, 0, kDrainLimitNs)) set_error();
    }
  } else {
    // ---- decode producers (group dg of 128 threads, thread r <-> tile row r)
    const int dg = (warp - 2) >> 2;
    const int r = (threadIdx.x - 64) & 127;
    const int64_t R = m0 + r;
    const bool valid = R < a.m_pad;
    const int rsw = r & 7;
    // codes two chunks ahead of the decode (a chunk is ~1 us of MMA work)
    RowChunk<K0, SPG> c0, n0c, nn0c;
    RowChunk<K1, SPG> c1, n1c, nn1c;
    load_row_chunk<K0, G>(a.stage[0], a.RT, 0, R, dg, valid, c0);
    if constexpr (NST == 2) load_row_chunk<K1, G>(a.stage[1], a.RT, 0, R, dg, valid, c1);
    if (K / 4 > 1) {
      load_row_chunk<K0, G>(a.stage[0], a.RT, 1, R, dg, valid, n0c);
      if constexpr (NST == 2) load_row_chunk<K1, G>(a.stage[1], a.RT, 1, R, dg, valid, n1c);
    }
    const int rowoff = (r >> 3) * 1024 + (r & 7) * 128;
    const int rep = lane % C::reps;  // this thread's table replica
    bool ok = true;
    for (int kc = 0; kc < K / 4 && ok; ++kc) {  // one 32-code chunk = 4 K steps
      if (kc + 2 < K / 4) {
        load_row_chunk<K0, G>(a.stage[0], a.RT, kc + 2, R, dg, valid, nn0c);
        if constexpr (NST == 2) load_row_chunk<K1, G>(a.stage[1], a.RT, kc + 2, R, dg, valid, nn1c);
      }
#pragma unroll
      for (int t = 0; t < SPG; ++t) {
        const int ks = kc * 4 + dg + G * t, s = ks % S, use = ks / S;
        if (use > 0 && !sm100::mbar_wait_bounded(empty(s), (use - 1) & 1, a.wait_ns)) {
          set_error();
          ok = false;
          break;
        }
        uint8_t *st = ring + s * C::stage_bytes;
        decode_row<K0>(c0, t, tbl0 + rep, C::reps, st + rowoff, rsw);
        if constexpr (NST == 2) decode_row<K1>(c1, t, tbl1 + rep, C::reps, st + kATile + rowoff, rsw);
        sm100::fence_proxy_async_smem();
        sm100::mbar_arrive(full_a(s));
      }
      c0 = n0c;
      n0c = nn0c;
      if constexpr (NST == 2) {
        c1 = n1c;
        n1c = nn1c;
      }
    }
    // ---- epilogue
    // one outcome per warp: the TMEM loads below are warp-collective
    const bool ok_warp = __all_sync(0xffffffffu, ok);
    if (ok_warp && sm100::mbar_wait_warp(acc_full, 0, a.wait_ns)) {
      sm100::tc_fence_after_sync();
      const int quarter = warp & 3;  // TMEM lanes this warp may read
      const int64_t row = m0 + quarter * 32 + lane;
      const uint32_t lane_addr = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
      const float ls = *a.layer_scale;
      constexpr int cols = kBN / G;
      for (int c = dg * cols; c < (dg + 1) * cols; c += 16) {
        uint32_t v0[16], v1[16];
        sm100::tmem_ld_16(lane_addr + c, v0);
        if constexpr (NST == 2) sm100::tmem_ld_16(lane_addr + kBN + c, v1);
        sm100::tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int64_t tok = n0 + c + j;
          if (tok < a.batch && row < a.m) {
            float v = a.sscale[0] * __uint_as_float(v0[j]);
            if constexpr (NST == 2) v = fmaf(a.sscale[1], __uint_as_float(v1[j]), v);
            a.y1[tok * a.m + row] = v * ls * a.rowscale[tok];
          }
        }
      }
    } else if (ok_warp) {
      set_error();
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

// ---- persistent variant (one-stage codebooks) -----------------------------------
// One CTA per SM loops over output tiles (tile t = blockIdx.x + i * gridDim.x,
// weight-row tile fastest).  TMEM holds two 256-column accumulators: the MMA
// issuer fills accumulator i & 1 for the CTA's i-th tile while four dedicated
// epilogue warps drain the other one, so a tile's epilogue and the next tile's
// pipeline fill overlap its successor's mainloop.  The ring's K-step sequence
// runs on across tiles (global step gs = tile_index * K + ks), and the decode
// groups prefetch weight codes two 32-code chunks ahead across tile boundaries.
// Barriers: full_a / full_b / empty per ring stage as above; acc_full[b]
// (tcgen05.commit after a tile's last MMA) and acc_empty[b] (128 epilogue
// arrivals) per accumulator.  Each waiter's own previous wait on a barrier
// proves the phase two back complete, so every parity wait is exact.
// The dependent kernel is released only when a CTA reaches its last tile, so
// its CTAs cannot take SMs while this grid still has work queued.
struct PCfg {
  static constexpr int stages = 4;
  static constexpr int groups = 4;
  static constexpr int decode_warps = 4 * groups;
  static constexpr int epi_warp0 = 2 + decode_warps;  // warps 18..21: TMEM lane quarters 2, 3, 0, 1
  static constexpr int threads = 32 * (epi_warp0 + 4);
  static constexpr uint32_t tmem_cols = 2 * Cfg<1>::tmem_cols;  // two accumulators
  static_assert(threads > Cfg<1>::threads, "persistent kernel adds epilogue warps");
};

template <int K0>
__global__ void __launch_bounds__(PCfg::threads, 1) gemm_tc_persistent_kernel(
    const __grid_constant__ CUtensorMap tmap_x, TcArgs a, int tiles_m, int tiles_total) {
  using C = Cfg<1>;  // ring and table geometry
  constexpr int S = PCfg::stages, G = PCfg::groups;
  static_assert(S == C::stages && G == C::groups, "persistent ring geometry");
  extern __shared__ __align__(1024) uint8_t dsm[];
  uint8_t *base = dsm + ((1024u - (smem_u32(dsm) & 1023u)) & 1023u);
  uint8_t *ring = base;
  uint2 *tbl0 = reinterpret_cast<uint2 *>(base + C::ring_bytes);
  uint64_t *bars = reinterpret_cast<uint64_t *>(base + C::ring_bytes + C::tables_bytes);
  // bars: full_a[S], full_b[S], empty[S], acc_full[2], acc_empty[2], drain, then the TMEM address holder
  const uint32_t bar0 = smem_u32(bars);
  auto full_a = [&](int s) { return bar0 + 8u * s; };
  auto full_b = [&](int s) { return bar0 + 8u * (S + s); };
  auto empty = [&](int s) { return bar0 + 8u * (2 * S + s); };
  auto acc_full = [&](int b) { return bar0 + 8u * (3 * S + b); };
  auto acc_empty = [&](int b) { return bar0 + 8u * (3 * S + 2 + b); };
  const uint32_t drain = bar0 + 8u * (3 * S + 4);
  uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(bars + 3 * S + 5);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  for (int i = threadIdx.x; i < C::table_entries; i += blockDim.x) tbl0[i] = gemm_table_entry(K0, i / C::reps);
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      sm100::mbar_init(full_a(s), 128);
      sm100::mbar_init(full_b(s), 1);
      sm100::mbar_init(empty(s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      sm100::mbar_init(acc_full(b), 1);
      sm100::mbar_init(acc_empty(b), 128);
    }
    sm100::mbar_init(drain, 1);
    sm100::fence_barrier_init();
    sm100::prefetch_tmap(&tmap_x);
  }
  if (warp == 1) sm100::tmem_alloc(smem_u32(tmem_holder), PCfg::tmem_cols);
  sm100::tc_fence_before_sync();
  __syncthreads();
  sm100::tc_fence_after_sync();
  const uint32_t tmem = *tmem_holder;
  pdl_wait();  // x2h / rowscale come from the input-transform kernel

  const int K = a.ksteps;
  const int my_tiles = tiles_total > static_cast<int>(blockIdx.x)
                           ? (tiles_total - 1 - static_cast<int>(blockIdx.x)) / static_cast<int>(gridDim.x) + 1
                           : 0;
  if (my_tiles == 0 && threadIdx.x == 0) pdl_launch_dependents();
  auto tile_of = [&](int i) { return static_cast<int>(blockIdx.x) + i * static_cast<int>(gridDim.x); };

  if (warp == 0) {
    // ---- TMA producer
    if (lane == 0) {
      int64_t gs = 0, issued = 0;
      bool ok = true;
      for (int i = 0; i < my_tiles && ok; ++i) {
        const int n0 = (tile_of(i) / tiles_m) * kBN;
        for (int ks = 0; ks < K; ++ks, ++gs) {
          const int s = static_cast<int>(gs % S);
          const int64_t use = gs / S;
          if (use > 0 && !sm100::mbar_wait_bounded(empty(s), static_cast<uint32_t>((use - 1) & 1), a.wait_ns)) {
            set_error();
            ok = false;
            break;
          }
          sm100::mbar_arrive_expect_tx(full_b(s), kBTile);
          sm100::tma_load_2d(smem_u32(ring + s * C::stage_bytes + kATile), &tmap_x, ks * kBK, n0, full_b(s));
          issued = gs + 1;
        }
      }
      for (int64_t g = issued > S ? issued - S : 0; g < issued; ++g)
        if (!sm100::mbar_wait_bounded(full_b(static_cast<int>(g % S)), static_cast<uint32_t>((g / S) & 1), kDrainLimitNs))
          set_error();
    }
  } else if (warp == 1) {
    // ---- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = sm100::idesc_f16_f32(kBM, kBN);
      int64_t gs = 0;
      bool ok = true;
      for (int i = 0; i < my_tiles && ok; ++i) {
        const int b = i & 1, u = i >> 1;
        if (u > 0 && !sm100::mbar_wait_bounded(acc_empty(b), static_cast<uint32_t>((u - 1) & 1), a.wait_ns)) {
          set_error();
          break;
        }
        sm100::tc_fence_after_sync();
        for (int ks = 0; ks < K; ++ks, ++gs) {
          const int s = static_cast<int>(gs % S);
          const uint32_t par = static_cast<uint32_t>((gs / S) & 1);
          ok = sm100::mbar_wait_bounded(full_a(s), par, a.wait_ns) &&
               sm100::mbar_wait_bounded(full_b(s), par, a.wait_ns);
          if (!ok) {
            set_error();
            break;
          }
          sm100::tc_fence_after_sync();
          uint8_t *st = ring + s * C::stage_bytes;
          const uint64_t adesc = sm100::sw128_kmajor_desc(smem_u32(st));
          const uint64_t bdesc = sm100::sw128_kmajor_desc(smem_u32(st + kATile));
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k)
            sm100::umma_f16(tmem + b * kBN, adesc + 2 * k, bdesc + 2 * k, idesc, (ks | k) != 0);
          sm100::umma_commit(empty(s));
        }
        sm100::umma_commit(acc_full(b));
      }
      // wind down: every MMA issued must be complete before TMEM and the ring are freed
      sm100::umma_commit(drain);
      if (!sm100::mbar_wait_bounded(drain, 0, kDrainLimitNs)) set_error();
    }
  } else if (warp < PCfg::epi_warp0) {
    // ---- decode producers (group dg of 128 threads, thread r <-> tile row r)
    const int dg = (warp - 2) >> 2;
    const int r = (threadIdx.x - 64) & 127;
    const int rsw = r & 7;
    const int rowoff = (r >> 3) * 1024 + (r & 7) * 128;
    const int rep = lane % C::reps;
    const int KC = K / 4;
    const int nchunks = my_tiles * KC;
    auto chunk_load = [&](int q, RowChunk<K0, 1> &rc) {
      const int mt = tile_of(q / KC) % tiles_m;
      const int64_t R = static_cast<int64_t>(mt) * kBM + r;
      load_row_chunk<K0, G>(a.stage[0], a.RT, q % KC, R, dg, R < a.m_pad, rc);
    };
    RowChunk<K0, 1> c0, n0c, nn0c;
    if (nchunks > 0) chunk_load(0, c0);
    if (nchunks > 1) chunk_load(1, n0c);
    bool ok = true;
    for (int q = 0; q < nchunks && ok; ++q) {
      if (q + 2 < nchunks) chunk_load(q + 2, nn0c);
      const int64_t gs = static_cast<int64_t>(q) * 4 + dg;  // this group's K step of the chunk
      const int s = static_cast<int>(gs % S);
      const int64_t use = gs / S;
      if (use > 0 && !sm100::mbar_wait_bounded(empty(s), static_cast<uint32_t>((use - 1) & 1), a.wait_ns)) {
        set_error();
        ok = false;
        break;
      }
      decode_row<K0>(c0, 0, tbl0 + rep, C::reps, ring + s * C::stage_bytes + rowoff, rsw);
      sm100::fence_proxy_async_smem();
      sm100::mbar_arrive(full_a(s));
      c0 = n0c;
      n0c = nn0c;
    }
  } else {
    // ---- epilogue warps: TMEM lane quarter warp & 3, all 256 token columns
    const int quarter = warp & 3;
    const float ls = *a.layer_scale;
    for (int i = 0; i < my_tiles; ++i) {
      const int b = i & 1, u = i >> 1;
      if (!sm100::mbar_wait_warp(acc_full(b), static_cast<uint32_t>(u & 1), a.wait_ns)) {
        set_error();
        break;
      }
      if (i == my_tiles - 1 && threadIdx.x == 32 * PCfg::epi_warp0) pdl_launch_dependents();
      sm100::tc_fence_after_sync();
      const int t = tile_of(i);
      const int64_t row = static_cast<int64_t>(t % tiles_m) * kBM + quarter * 32 + lane;
      const int n0 = (t / tiles_m) * kBN;
      const uint32_t lane_addr = tmem + b * kBN + (static_cast<uint32_t>(quarter * 32) << 16);
      for (int c = 0; c < kBN; c += 16) {
        uint32_t v[16];
        sm100::tmem_ld_16(lane_addr + c, v);
        sm100::tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int64_t tok = n0 + c + j;
          if (tok < a.batch && row < a.m)
            a.y1[tok * a.m + row] = a.sscale[0] * __uint_as_float(v[j]) * ls * a.rowscale[tok];
        }
      }
      sm100::tc_fence_before_sync();
      sm100::mbar_arrive(acc_empty(b));
    }
  }
  // ---- teardown
  sm100::tc_fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    sm100::tc_fence_after_sync();
    sm100::tmem_dealloc(tmem, PCfg::tmem_cols);
  }
}

}  // namespace

// ---- tensor maps over the fp16 activation rows (x2h: rows x n_pad) ----------
using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                   const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

int encode_fp16_rows_map(CUtensorMap *map, const void *x2h, int64_t n_pad, int64_t rows, int box_x, int box_y,
                         bool swizzle128) {
  static EncodeTiledFn fn = nullptr;
  static std::mutex mu;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (!fn) {
      void *p = nullptr;
      cudaDriverEntryPointQueryResult q;
      QS_CUDA_TRY(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q));
      if (!p || q != cudaDriverEntryPointSuccess) return fail(QS_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
      fn = reinterpret_cast<EncodeTiledFn>(p);
    }
  }
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(n_pad), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(n_pad * 2)};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(box_x), static_cast<cuuint32_t>(box_y)};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void *>(x2h), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(QS_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
  return QS_OK;
}

namespace {

static int tc_num_sms() {
  static int cached[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && cached[dev]) return cached[dev];
  int n = 148;
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  if (dev < 64) cached[dev] = n;
  return n;
}

template <int K0>
int run_gemm_persistent(const CUtensorMap &map, const TcArgs &a, cudaStream_t s) {
  using C = Cfg<1>;
  auto kern = gemm_tc_persistent_kernel<K0>;
  QS_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::smem_bytes));
  const int tiles_m = static_cast<int>(ceil_div(a.m, kBM));
  const int tiles_total = tiles_m * static_cast<int>(ceil_div(a.batch, kBN));
  const int grid = tiles_total < tc_num_sms() ? tiles_total : tc_num_sms();
  return launch_pdl("gemm_tc", kern, dim3(grid), dim3(PCfg::threads), C::smem_bytes, s, map, a, tiles_m,
                    tiles_total);
}

template <int K0, int K1, int NST>
int run_gemm(const CUtensorMap &map, const TcArgs &a, cudaStream_t s) {
  using C = Cfg<NST>;
  auto kern = gemm_tc_kernel<K0, K1, NST>;
  QS_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::smem_bytes));
  const dim3 grid(static_cast<unsigned>(ceil_div(a.m, kBM)), static_cast<unsigned>(ceil_div(a.batch, kBN)));
  return launch_pdl("gemm_tc", kern, grid, dim3(C::threads), C::smem_bytes, s, map, a);
}

}  // namespace

int launch_matmul_tc(const void *x2ws, int64_t batch, int64_t n, int64_t m, const void *packed, int stages,
                     const int *kinds, const float *stage_scales, const float *layer_scale, float *y1,
                     cudaStream_t s) {
  const int64_t n_pad = padded_T(n) * 8;
  TcArgs a{};
  a.rowscale = reinterpret_cast<const float *>(static_cast<const char *>(x2ws) + round_up(batch * n_pad * 2, 256));
  a.layer_scale = layer_scale;
  a.y1 = y1;
  a.m = m;
  a.m_pad = padded_m(m);
  a.RT = padded_m(m) / kRowsPerTile;
  a.batch = batch;
  a.ksteps = static_cast<int>(n_pad / kBK);
  a.wait_ns = pipeline_wait_ns();
  const uint8_t *p = static_cast<const uint8_t *>(packed);
  for (int st = 0; st < stages; ++st) {
    a.stage[st] = p;
    a.sscale[st] = stage_scales ? stage_scales[st] : 1.f;
    p += round_up(stage_bytes(kinds[st], m, n), 256);
  }
  CUtensorMap map;
  int st = encode_fp16_rows_map(&map, x2ws, n_pad, batch, kBK, kBN, true);
  if (st) return st;
  const int k0 = kinds[0], k1 = stages == 2 ? kinds[1] : 0;
  if (stages == 1)
    return k0 == QS_CB_E8P ? run_gemm_persistent<QS_CB_E8P>(map, a, s) : run_gemm_persistent<QS_CB_E8_1BIT>(map, a, s);
  if (k0 == QS_CB_E8P && k1 == QS_CB_E8_1BIT) return run_gemm<QS_CB_E8P, QS_CB_E8_1BIT, 2>(map, a, s);
  if (k0 == QS_CB_E8P && k1 == QS_CB_E8P) return run_gemm<QS_CB_E8P, QS_CB_E8P, 2>(map, a, s);
  if (k0 == QS_CB_E8_1BIT && k1 == QS_CB_E8P) return run_gemm<QS_CB_E8_1BIT, QS_CB_E8P, 2>(map, a, s);
  return run_gemm<QS_CB_E8_1BIT, QS_CB_E8_1BIT, 2>(map, a, s);
}

// Limit of the kernels' pipeline waits, read by every launcher (process-wide).
static std::atomic<uint64_t> g_wait_ns{kDefaultWaitNs};

uint64_t pipeline_wait_ns() { return g_wait_ns.load(std::memory_order_relaxed); }

void set_pipeline_wait_ns(uint64_t ns) { g_wait_ns.store(ns ? ns : kDefaultWaitNs, std::memory_order_relaxed); }

int *device_error_flag() {
  static int *cached[64] = {nullptr};
  static std::mutex mu;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  if (!cached[dev]) {
    void *p = nullptr;
    if (cudaGetSymbolAddress(&p, g_tc_error) != cudaSuccess) return nullptr;
    cached[dev] = static_cast<int *>(p);
  }
  return cached[dev];
}

int device_status(cudaStream_t s) {
  int flag = 0;
  static const int zero = 0;
  QS_CUDA_TRY(cudaMemcpyFromSymbolAsync(&flag, g_tc_error, sizeof(int), 0, cudaMemcpyDeviceToHost, s));
  QS_CUDA_TRY(cudaStreamSynchronize(s));
  if (flag) {
    QS_CUDA_TRY(cudaMemcpyToSymbolAsync(g_tc_error, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, s));
    QS_CUDA_TRY(cudaStreamSynchronize(s));
    return fail(QS_ERR_TIMEOUT, "a bounded wait timed out (prefill matmul pipeline or tensor-parallel shard arrival); "
                "the results of that launch are invalid");
  }
  return QS_OK;
}

}  // namespace qs
