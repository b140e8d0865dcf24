// Push of a column-sharded layer's y1 shard to every rank (tensor parallelism
// over peer memory; see qs_tp.cu): the descriptor and the device routines that
// the push kernel and the decode matmul's push tail share.
//
// Two receive formats:
//  * flagged (prefill batches): plain floats, then after a system-scope fence
//    the call's sequence number stored into flag [seq & 1][this rank] of every
//    rank (release); the reader waits for all flags, then reads the floats;
//  * self-validating words (decode batches): each float travels as one 8-byte
//    word {value bits, seq} written by a single aligned 64-bit store, so a
//    reader that sees seq in a word also sees its value: no fences and no
//    flags, the reader waits per word (twice the bytes, which are few here).
#pragma once

#include "qs_common.cuh"

namespace qs {

constexpr int kTpMaxRanks = 8;

struct TpPush {
  const float *y1;           // this rank's private shard (count floats)
  float *dst[kTpMaxRanks];   // every rank's receive buffer (region 0) + this shard's gathered offset
  int *flag[kTpMaxRanks];    // every rank's flags (region 0) + this rank
  unsigned *ctl;             // this rank's [call sequence number, finished CTAs]
  int64_t count;
  int64_t stride;            // floats between the parity regions of a receive buffer
  int nflag_stride;          // ints between the parity regions of a flag array (world)
  int world;                 // 0: no push
  int words;                 // 1: self-validating 8-byte words (stride and dst in floats, 2 per word)
};

// Copies floats [i0, count) step `step` of the shard into every rank's region
// `off` (remote stores over the interconnect; the own copy is local).  Loads go
// through L2 (the shard was written by device-scope atomics of other CTAs).
__device__ __forceinline__ void tp_push_copy(const TpPush &a, int64_t off, int64_t i0, int64_t step, unsigned seq) {
  if (a.words) {  // float i -> word i of the region: {bits, seq}
    for (int64_t i = i0; i < a.count; i += step) {
      const uint32_t bits = __float_as_uint(__ldcg(a.y1 + i));
      for (int r = 0; r < a.world; ++r) {
        uint32_t *w = reinterpret_cast<uint32_t *>(a.dst[r] + off) + 2 * i;
        asm volatile("st.global.v2.u32 [%0], {%1, %2};" ::"l"(w), "r"(bits), "r"(seq) : "memory");
      }
    }
    return;
  }
  bool vec = (a.count & 3) == 0 && (reinterpret_cast<uintptr_t>(a.y1) & 15) == 0;
  for (int r = 0; r < a.world; ++r) vec = vec && (reinterpret_cast<uintptr_t>(a.dst[r] + off) & 15) == 0;
  if (vec) {
    const float4 *src = reinterpret_cast<const float4 *>(a.y1);
    for (int64_t i = i0; i < a.count / 4; i += step) {
      const float4 v = __ldcg(src + i);
      for (int r = 0; r < a.world; ++r) reinterpret_cast<float4 *>(a.dst[r] + off)[i] = v;
    }
  } else {
    for (int64_t i = i0; i < a.count; i += step) {
      const float v = __ldcg(a.y1 + i);
      for (int r = 0; r < a.world; ++r) a.dst[r][off + i] = v;
    }
  }
}

// Announces call `seq` to every rank (thread 0, after the CTA's pushed data):
// records the sequence number, resets the arrival count, and after a
// system-scope fence stores seq into flag [seq & 1][this rank] of every rank.
__device__ __forceinline__ void tp_announce(const TpPush &a, unsigned seq) {
  a.ctl[1] = 0;
  a.ctl[0] = seq;
  __threadfence_system();
  for (int r = 0; r < a.world; ++r)
    asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(a.flag[r] + (seq & 1u) * a.nflag_stride), "r"(seq)
                 : "memory");
}

// End of the decode matmul that produced the shard (word format; every thread
// of every CTA calls it).  A grid barrier (arrival count ctl[1], bounded wait;
// every CTA of the grid is resident, since the next kernel is released only
// once all of them have started) makes the shard complete, then every CTA
// pushes its 1/grid slice of it, so the copy runs on all SMs at once; the last
// CTA to finish (count ctl[2]) records the call's sequence number and resets
// the counts.  Every CTA read the old sequence number before arriving.
// s_seq: a shared-memory word of the caller's (its own allocation, so the
// caller's shared-memory layout stays as it is without a push).
__device__ __forceinline__ void tp_push_grid(const TpPush &a, uint64_t wait_ns, int *error, unsigned *s_seq_slot) {
  unsigned &s_seq = *s_seq_slot;
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned seq = *reinterpret_cast<volatile unsigned *>(a.ctl) + 1u;
    __threadfence();  // this CTA's shard writes before its arrival
    atomicAdd(a.ctl + 1, 1u);
    uint64_t t0 = 0;
    while (*reinterpret_cast<volatile unsigned *>(a.ctl + 1) < gridDim.x) {
      uint64_t t;
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
      if (!t0) t0 = t;
      if (t - t0 > wait_ns) {  // cannot happen with a resident grid; leave rather than hang
        atomicExch(error, 1);
        break;
      }
    }
    __threadfence();
    s_seq = seq;
  }
  __syncthreads();
  const unsigned seq = s_seq;
  const int64_t per = (a.count + gridDim.x - 1) / gridDim.x;
  const int64_t lo = blockIdx.x * per, hi = lo + per < a.count ? lo + per : a.count;
  const int64_t off = (seq & 1u) * a.stride;
  for (int64_t i = lo + threadIdx.x; i < hi; i += blockDim.x) {
    const uint32_t bits = __float_as_uint(__ldcg(a.y1 + i));
    for (int r = 0; r < a.world; ++r) {
      uint32_t *w = reinterpret_cast<uint32_t *>(a.dst[r] + off) + 2 * i;
      asm volatile("st.global.v2.u32 [%0], {%1, %2};" ::"l"(w), "r"(bits), "r"(seq) : "memory");
    }
  }
  __syncthreads();
  if (threadIdx.x == 0 && atomicAdd(a.ctl + 2, 1u) == gridDim.x - 1) {  // every CTA is past the barrier
    a.ctl[1] = 0;
    a.ctl[2] = 0;
    a.ctl[0] = seq;
  }
}

}  // namespace qs
