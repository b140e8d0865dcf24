// Column-sharded tensor parallelism over peer memory (NVLink / NVSwitch).
//
// Rank r of P holds weight rows [r m/P, (r+1) m/P).  Per layer call:
//   1. input step: x -> x2 (local workspace); zero the private y1 shard
//      (decode batches: the matmul accumulates into it);
//   2. fused decode + matmul of the local rows into the private y1 (batch, m/P);
//   3. push of y1 into every rank's receive buffer (remote stores over the
//      interconnect; this rank's own copy is a local store) at the rank-major
//      gathered position of this rank's shard, in the region of the call's
//      sequence number s (s & 1):
//      * decode batches: by the matmul itself (gemv_push_kernel): after a grid
//        barrier every CTA stores its slice as 8-byte words {value, s} (qs_tp.cuh);
//      * prefill batches: tp_push_kernel stores plain floats, then after a
//        system-scope fence stores s into flag [s & 1][this rank] of every rank;
//   4. output step: reads the gathered y1 once it has arrived (words: each word
//      holds s; flags: every flag [s & 1][0..P) holds s; bounded waits) and
//      applies the full-width output transform, signs / phases, bias and cast.
// The sequence number lives in device memory (recorded by the last CTA of each
// push), so CUDA graphs holding any number of calls replay in any order with
// eager calls.  Two regions suffice: a rank pushes call s + 2 only after its own
// output step of call s + 1, which saw every rank's call-s+1 data, which each
// rank pushes after its output step of call s (stream order) -- so nobody
// still reads region s & 1.
#include <cuda.h>

#include <cstring>
#include <mutex>

#include "qs_common.cuh"
#include "qs_launch.h"
#include "qs_tp.cuh"
#include "qs_xform.cuh"

namespace qs {

namespace {

constexpr int kPushThreads = 256;

// Separate push (prefill batches, or a shard computed by the caller): every CTA
// copies its part, then arrives; the last CTA announces the call.
__global__ void __launch_bounds__(kPushThreads) tp_push_kernel(TpPush a) {
  __shared__ unsigned s_seq;
  pdl_wait();  // the matmul's y1 writes are complete
  if (threadIdx.x == 0) s_seq = *reinterpret_cast<volatile unsigned *>(a.ctl) + 1u;
  __syncthreads();
  const unsigned seq = s_seq;
  const int64_t tid = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  tp_push_copy(a, (seq & 1u) * a.stride, tid, static_cast<int64_t>(gridDim.x) * blockDim.x, seq);
  __syncthreads();
  if (threadIdx.x == 0) {
    if (a.words) {
      __threadfence();  // the sequence number is read by every CTA before the last one records it
      if (atomicAdd(a.ctl + 1, 1u) == gridDim.x - 1) {
        a.ctl[1] = 0;
        a.ctl[0] = seq;
      }
    } else {
      __threadfence_system();  // this CTA's pushed data before its arrival count
      // every CTA read the old sequence number before its arrival count
      if (atomicAdd(a.ctl + 1, 1u) == gridDim.x - 1) tp_announce(a, seq);
    }
  }
  pdl_launch_dependents();
}

using GetAddressRangeFn = CUresult (*)(CUdeviceptr *, size_t *, CUdeviceptr);

int allocation_base(const void *ptr, char **base) {
  static GetAddressRangeFn fn = nullptr;
  static std::mutex mu;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (!fn) {
      void *p = nullptr;
      cudaDriverEntryPointQueryResult q;
      QS_CUDA_TRY(cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q));
      if (!p || q != cudaDriverEntryPointSuccess) return fail(QS_ERR_CUDA, "cuMemGetAddressRange unavailable");
      fn = reinterpret_cast<GetAddressRangeFn>(p);
    }
  }
  CUdeviceptr b = 0;
  size_t sz = 0;
  const CUresult r = fn(&b, &sz, reinterpret_cast<CUdeviceptr>(ptr));
  if (r != CUDA_SUCCESS) return fail(QS_ERR_INVALID_ARG, "pointer is not device memory (%d)", static_cast<int>(r));
  *base = reinterpret_cast<char *>(b);
  return QS_OK;
}

int check_peers(const qs_tp_peers *pe) {
  if (!pe) return fail(QS_ERR_INVALID_ARG, "null peers");
  if (pe->world < 1 || pe->world > kMaxPeers || pe->rank < 0 || pe->rank >= pe->world)
    return fail(QS_ERR_INVALID_ARG, "bad world %d / rank %d (at most %d ranks)", pe->world, pe->rank, kMaxPeers);
  if (!pe->ctl || (reinterpret_cast<uintptr_t>(pe->ctl) & 15)) return fail(QS_ERR_INVALID_ARG, "bad ctl words");
  for (int r = 0; r < pe->world; ++r)
    if (!pe->recv[r] || !pe->flags[r]) return fail(QS_ERR_INVALID_ARG, "missing buffer of rank %d", r);
  return QS_OK;
}

}  // namespace

int ipc_export(const void *ptr, void *handle, int64_t *offset) {
  char *base = nullptr;
  int st = allocation_base(ptr, &base);
  if (st) return st;
  cudaIpcMemHandle_t h;
  QS_CUDA_TRY(cudaIpcGetMemHandle(&h, base));
  std::memcpy(handle, &h, sizeof(h));
  *offset = static_cast<const char *>(ptr) - base;
  return QS_OK;
}

int ipc_import(const void *handle, int64_t offset, void **ptr) {
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void *base = nullptr;
  QS_CUDA_TRY(cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess));
  *ptr = static_cast<char *>(base) + offset;
  return QS_OK;
}

int ipc_close(void *ptr, int64_t offset) {
  QS_CUDA_TRY(cudaIpcCloseMemHandle(static_cast<char *>(ptr) - offset));
  return QS_OK;
}

int64_t tp_workspace_bytes(int64_t batch, int64_t n, int64_t m_local) {
  return round_up(linear_input_bytes(batch, n), 256) + round_up(batch * m_local * 4, 256);
}

// Decode batches exchange self-validating words (qs_tp.cuh), prefill batches
// flagged floats; push and output step pick the same format from the batch.
static bool word_format(int64_t batch) { return batch < kTcMinBatch; }

static int make_push(const qs_tp_peers *pe, const float *y1, int64_t batch, int64_t m_local, TpPush &a) {
  int st = check_peers(pe);
  if (st) return st;
  const int64_t per = word_format(batch) ? 2 : 1;  // floats of receive region per value
  if (batch * m_local * pe->world * per > pe->recv_floats) return fail(QS_ERR_WORKSPACE, "receive buffers too small");
  a = TpPush{};
  a.words = word_format(batch) ? 1 : 0;
  a.y1 = y1;
  a.count = batch * m_local;
  a.stride = pe->recv_floats;
  a.nflag_stride = pe->world;
  a.world = pe->world;
  a.ctl = pe->ctl;
  for (int r = 0; r < pe->world; ++r) {
    a.dst[r] = pe->recv[r] + per * pe->rank * a.count;
    a.flag[r] = pe->flags[r] + pe->rank;
  }
  return QS_OK;
}

int launch_tp_push(const qs_tp_peers *pe, const float *y1, int64_t batch, int64_t m_local, cudaStream_t s) {
  TpPush a;
  int st = make_push(pe, y1, batch, m_local, a);
  if (st) return st;
  // ~16 KB of shard per CTA, at most one wave of 4 CTAs per SM
  const int64_t want = (a.count + 4095) / 4096;
  const int64_t most = 4 * static_cast<int64_t>(xlaunch_sms());
  const int grid = static_cast<int>(want < 1 ? 1 : want > most ? most : want);
  return launch_pdl("tp_push", tp_push_kernel, dim3(grid), dim3(kPushThreads), 0, s, a);
}

int launch_matmul_tp(const void *x2ws, int64_t batch, int64_t n, int64_t m_local, const void *packed, int stages,
                     const int *kinds, const float *stage_scales, const float *layer_scale, float *y1,
                     const qs_tp_peers *pe, cudaStream_t s) {
  if (batch >= kTcMinBatch) {  // the tcgen05 GEMM, then the push kernel
    int st = launch_matmul(x2ws, batch, n, m_local, packed, stages, kinds, stage_scales, layer_scale, y1, s);
    return st ? st : launch_tp_push(pe, y1, batch, m_local, s);
  }
  TpPush push;  // the decode matmul's CTAs push the shard after a grid barrier
  int st = make_push(pe, y1, batch, m_local, push);
  return st ? st : launch_matmul(x2ws, batch, n, m_local, packed, stages, kinds, stage_scales, layer_scale, y1, s, &push);
}

int launch_output_peers(const qs_tp_peers *pe, int64_t batch, int64_t m, int transform, const float *su,
                        const void *phase_u, const float *bias, void *y, int y_dtype, cudaStream_t s) {
  int st = check_peers(pe);
  if (st) return st;
  if (m % pe->world) return fail(QS_ERR_INVALID_ARG, "m=%lld not divisible by %d ranks", (long long)m, pe->world);
  if (transform == QS_RFFT && (m / pe->world) % 2)
    return fail(QS_ERR_INVALID_ARG, "RFFT shards must hold an even number of columns");
  if (batch * m * (word_format(batch) ? 2 : 1) > pe->recv_floats)
    return fail(QS_ERR_WORKSPACE, "receive buffers too small");
  XPeerGather pg{};
  pg.words = word_format(batch) ? 1 : 0;
  pg.base = pe->recv[pe->rank];
  pg.stride = pe->recv_floats;
  pg.flags = pe->flags[pe->rank];
  pg.seq = pe->ctl;
  pg.nflags = pe->world;
  pg.wait_ns = pipeline_wait_ns();
  pg.error = device_error_flag();
  if (!pg.error) return fail(QS_ERR_CUDA, "device error flag unavailable");
  return launch_linear_output(nullptr, m, pe->world, batch, m, transform, su, phase_u, bias, y, y_dtype, s, &pg);
}

int launch_linear_fwd_tp(const void *x, int x_dtype, int64_t batch, int64_t n, int64_t m, const void *packed,
                         int stages, const int *kinds, const float *stage_scales, const float *layer_scale,
                         int transform, const float *su, const float *sv, const void *phase_u, const void *phase_v,
                         const float *bias, void *y, void *workspace, const qs_tp_peers *pe, cudaStream_t s) {
  const int64_t m_local = m / pe->world;
  float *y1 = reinterpret_cast<float *>(static_cast<char *>(workspace) + round_up(linear_input_bytes(batch, n), 256));
  const bool tc = batch >= kTcMinBatch;  // the prefill GEMM writes every y1 element
  int st = launch_linear_input(x, x_dtype, batch, n, transform, sv, phase_v, workspace, tc ? nullptr : y1, m_local, s);
  if (st) return st;
  st = launch_matmul_tp(workspace, batch, n, m_local, packed, stages, kinds, stage_scales, layer_scale, y1, pe, s);
  if (st) return st;
  return launch_output_peers(pe, batch, m, transform, su, phase_u, bias, y, x_dtype, s);
}

}  // namespace qs
