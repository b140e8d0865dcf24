// Measurement probe (not part of the library): time per tcgen05.mma seen by the
// issuing thread, for M = 128 and N from 16 to 256, kind::f16 (K = 16) and
// kind::f8f6f4 (K = 32), A in TMEM, B in shared memory, one or several
// accumulator chains, one or several issuing warps per CTA.  Operand values are
// zeros (only timing is read); every address stays inside the CTA's 512 TMEM
// columns and 120 KB of shared memory, and every wait is bounded.
// Build and run on a B200:
//   nvcc -gencode arch=compute_100a,code=sm_100a -O3 -std=c++17 --expt-relaxed-constexpr \
//     -I quipsharp_b200/csrc -I quipsharp_b200/_build -I include \
//     quipsharp_b200/probe/tcgen05_mma_issue.cu -o tcgen05_mma_issue && ./tcgen05_mma_issue
#include <cstdio>
#include <cstdint>
#include <cuda_runtime.h>
#include "qs_common.cuh"
#include "qs_sm100.cuh"
using namespace qs;

__device__ unsigned long long g_t[4096][4];

template <int KIND, int N>
__global__ void __launch_bounds__(128, 1) bench(int nmma, int nchain, int avary, int acc_mode, int issuers) {
  extern __shared__ __align__(1024) uint8_t dsm[];
  uint8_t *base = dsm + ((1024u - (smem_u32(dsm) & 1023u)) & 1023u);
  uint64_t *bars = reinterpret_cast<uint64_t *>(base + 64 * 1024);
  uint32_t *holder = reinterpret_cast<uint32_t *>(bars + 8);
  for (int i = threadIdx.x; i < 64 * 1024 / 16; i += blockDim.x) reinterpret_cast<uint4 *>(base)[i] = make_uint4(0, 0, 0, 0);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < 4; ++i) sm100::mbar_init(smem_u32(bars + i), 1);
    sm100::fence_barrier_init();
  }
  if (warp == 0) sm100::tmem_alloc(smem_u32(holder), 512);
  sm100::fence_proxy_async_smem();
  sm100::tc_fence_before_sync();
  __syncthreads();
  sm100::tc_fence_after_sync();
  const uint32_t tmem = *holder;
  if (lane == 0 && warp < issuers) {
    constexpr uint32_t idesc = sm100::idesc_f16_f32(128, N);
    const uint64_t bd = sm100::sw128_kmajor_desc(smem_u32(base + warp * 16384));
    const unsigned long long t0 = sm100::globaltimer_ns();
    for (int i = 0; i < nmma; ++i) {
      const uint32_t d = tmem + 256 * (warp & 1) + N * (i % nchain);   // chains: distinct D columns (<= 256/N)
      const uint32_t a = tmem + 256 * (warp & 1) + 192 + (avary ? 8 * (i % 8) : 0);
      const uint32_t acc = acc_mode ? 1u : 0u;
      if (KIND == 0) sm100::umma_f16_ts(d, a, bd + 2 * (i & 3), idesc, acc);
      else sm100::umma_f8_ts(d, a, bd + 2 * (i & 3), idesc, acc);
    }
    const unsigned long long t1 = sm100::globaltimer_ns();
    sm100::umma_commit(smem_u32(bars + warp));
    sm100::mbar_wait_bounded(smem_u32(bars + warp), 0, 2000000000ull);
    const unsigned long long t2 = sm100::globaltimer_ns();
    if (blockIdx.x < 4096 && warp == 0) { g_t[blockIdx.x][0] = t0; g_t[blockIdx.x][1] = t1; g_t[blockIdx.x][2] = t2; }
  }
  sm100::tc_fence_before_sync();
  __syncthreads();
  if (warp == 0) {
    sm100::tc_fence_after_sync();
    sm100::tmem_dealloc(tmem, 512);
  }
}

template <int KIND, int N>
void run(const char *name, int nmma, int nchain, int avary, int acc, int issuers, int grid) {
  auto k = bench<KIND, N>;
  cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, 120 * 1024);
  k<<<grid, 128, 120 * 1024>>>(nmma, nchain, avary, acc, issuers);  // warm
  cudaEvent_t e0, e1; cudaEventCreate(&e0); cudaEventCreate(&e1);
  cudaEventRecord(e0);
  k<<<grid, 128, 120 * 1024>>>(nmma, nchain, avary, acc, issuers);
  cudaEventRecord(e1);
  cudaError_t err = cudaDeviceSynchronize();
  float ms = 0; cudaEventElapsedTime(&ms, e0, e1);
  static unsigned long long h[4096][4];
  cudaMemcpyFromSymbol(h, g_t, sizeof(h));
  double issue = (double)(h[0][1] - h[0][0]) / nmma, total = (double)(h[0][2] - h[0][0]) / nmma;
  printf("%-34s N=%3d mma=%5d chains=%d avary=%d acc=%d issuers=%d grid=%3d : issue %6.1f ns/mma, complete %6.1f ns/mma (per issuer), kernel %.1f us %s\n",
         name, N, nmma, nchain, avary, acc, issuers, grid, issue, total, ms * 1e3, err ? cudaGetErrorString(err) : "");
}

int main() {
  int sms = 148;
  run<1, 16>("f8 chain", 2000, 1, 1, 1, 1, 1);
  run<1, 16>("f8 4 chains", 2000, 4, 1, 1, 1, 1);
  run<1, 16>("f8 noacc same a", 2000, 1, 0, 0, 1, 1);
  run<1, 16>("f8 chain 2 issuers", 2000, 1, 1, 1, 2, 1);
  run<1, 16>("f8 chain 4 issuers", 2000, 1, 1, 1, 4, 1);
  run<1, 32>("f8 chain", 2000, 1, 1, 1, 1, 1);
  run<1, 64>("f8 chain", 2000, 1, 1, 1, 1, 1);
  run<1, 128>("f8 chain", 2000, 1, 1, 1, 1, 1);
  run<1, 256>("f8 chain", 1000, 1, 1, 1, 1, 1);
  run<0, 16>("f16 chain", 2000, 1, 1, 1, 1, 1);
  run<0, 16>("f16 4 chains", 2000, 4, 1, 1, 1, 1);
  run<0, 256>("f16 chain", 1000, 1, 1, 1, 1, 1);
  run<1, 16>("f8 chain all SMs", 2000, 1, 1, 1, 1, sms);
  run<1, 16>("f8 4 chains 4 issuers all SMs", 2000, 4, 1, 1, 4, sms);
  return 0;
}
