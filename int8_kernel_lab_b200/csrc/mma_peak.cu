// mma_peak.cu - the int8 tensor-core ceiling of this GPU, as the conv kernels
// can use it.
//
// Every CTA (or CTA pair) issues back-to-back tcgen05.mma kind::i8
// instructions (M = 128 per CTA, N = 256, K = 32 bytes) on operands resident
// in its shared memory, with the conv kernels' pattern of one commit per
// 128-byte k-block and two k-blocks in flight.  There is no global-memory
// traffic, so the rate is the tensor pipe's alone.  Operands are either
// pseudo-random full-range bytes (the switching activity of a real int8
// convolution, which is what the 1 kW power cap responds to) or zeros
// (--zeros: the clock-limited ceiling).
//
//   mma_peak [--ms N] [--launches N] [--zeros] [--single]
//
// prints the TOPS of each launch and a JSON summary line with the median.
// Sample the SM clock alongside (nvidia-smi) to see what the cap allows.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <vector>

#include "sm100.cuh"

namespace {

using namespace i8c;

constexpr int kThreadsPeak = 128;
constexpr int kOperandBytes = 65536;  // A (32 KB) + B (32 KB), SW128 atoms
constexpr int kSmemPeak = kOperandBytes + 2048;

template <bool PAIR>
__global__ void __launch_bounds__(kThreadsPeak, 1)
    mma_peak_kernel(long long kblocks, int zeros, uint32_t *status) {
  extern __shared__ uint8_t raw[];
  uint8_t *sm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(raw) + 1023) &
                                            ~static_cast<uintptr_t>(1023));
  uint64_t *done = reinterpret_cast<uint64_t *>(sm + kOperandBytes);
  uint64_t *ring = done + 1;  // two commit barriers: k-blocks in flight
  uint32_t *slot = reinterpret_cast<uint32_t *>(ring + 2);
  const int warp = threadIdx.x >> 5;
  for (int i = threadIdx.x; i < kOperandBytes / 4; i += blockDim.x) {
    uint32_t h = (static_cast<uint32_t>(i) + 1u) * 2654435761u ^ (blockIdx.x * 40503u);
    h ^= h >> 13;
    h *= 0x5bd1e995u;
    h ^= h >> 15;
    reinterpret_cast<uint32_t *>(sm)[i] = zeros ? 0u : h;
  }
  fence_proxy_async_smem();
  if (threadIdx.x == 0) {
    mbar_init(done, 1);
    mbar_init(&ring[0], 1);
    mbar_init(&ring[1], 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    if constexpr (PAIR) {
      tmem_alloc_pair(slot, 256);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(slot, 256);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (PAIR) cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem = *slot;
  const bool leader = !PAIR || cluster_ctarank() == 0;
  const WaitCtx wctx{4000000000ull, status};
  if (threadIdx.x == 0 && leader) {
    const uint32_t idesc = idesc_s8(PAIR ? 256 : 128, 256);
    const uint32_t a = smem_u32(sm), b = smem_u32(sm + kOperandBytes / 2);
    for (long long kb = 0; kb < kblocks; ++kb) {
      const int r = static_cast<int>(kb & 1);
      // The k-block issued two blocks ago (same barrier) must be complete.
      if (!mbar_wait(&ring[r], static_cast<uint32_t>(((kb >> 1) & 1) ^ 1), wctx, 1u)) break;
      tc_fence_after();
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const uint64_t ad = smem_desc(a + 32 * k, 16, 1024, Layout::kSw128);
        const uint64_t bd = smem_desc(b + 32 * k, 16, 1024, Layout::kSw128);
        if constexpr (PAIR)
          umma_i8_pair(tmem, ad, bd, idesc, 1u);
        else
          umma_i8(tmem, ad, bd, idesc, 1u);
      }
      if constexpr (PAIR)
        umma_commit_pair(&ring[r], 0x3);
      else
        umma_commit(&ring[r]);
    }
    // Arrives when every MMA issued above is complete (in both CTAs).
    if constexpr (PAIR)
      umma_commit_pair(done, 0x3);
    else
      umma_commit(done);
  }
  if (threadIdx.x == 0) mbar_wait(done, 0, wctx, 2u);
  tc_fence_before();
  __syncthreads();
  if constexpr (PAIR) cluster_sync_all();
  if (warp == 0) {
    __syncwarp();
    tc_fence_after();
    if constexpr (PAIR)
      tmem_dealloc_pair(tmem, 256);
    else
      tmem_dealloc(tmem, 256);
  }
}

bool ok(cudaError_t e, const char *what) {
  if (e == cudaSuccess) return true;
  std::fprintf(stderr, "%s: %s\n", what, cudaGetErrorString(e));
  return false;
}

}  // namespace

int main(int argc, char **argv) {
  double ms_target = 200.0;
  int launches = 6;
  bool zeros = false, pair = true;
  for (int i = 1; i < argc; ++i) {
    if (!std::strcmp(argv[i], "--ms") && i + 1 < argc) ms_target = std::atof(argv[++i]);
    else if (!std::strcmp(argv[i], "--launches") && i + 1 < argc) launches = std::atoi(argv[++i]);
    else if (!std::strcmp(argv[i], "--zeros")) zeros = true;
    else if (!std::strcmp(argv[i], "--single")) pair = false;
    else {
      std::fprintf(stderr, "usage: mma_peak [--ms N] [--launches N] [--zeros] [--single]\n");
      return 2;
    }
  }
  if (ms_target <= 0 || ms_target > 2000 || launches < 1) {
    std::fprintf(stderr, "mma_peak: --ms must be in (0, 2000], --launches >= 1\n");
    return 2;
  }
  int sms = 0;
  if (!ok(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, 0), "device")) return 1;
  uint32_t *status = nullptr;
  if (!ok(cudaMalloc(&status, sizeof(uint32_t)), "cudaMalloc") ||
      !ok(cudaMemset(status, 0, sizeof(uint32_t)), "cudaMemset"))
    return 1;
  auto kernel = pair ? mma_peak_kernel<true> : mma_peak_kernel<false>;
  if (!ok(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemPeak),
          "smem attribute"))
    return 1;
  const int ctas = pair ? sms / 2 * 2 : sms;
  // One 128-byte k-block: 4 MMAs of 128 x 256 x 32 per CTA.
  const double ops_per_kblock = 2.0 * 128 * 256 * 128 * ctas;
  long long kblocks = 1000;
  cudaEvent_t start, stop;
  cudaEventCreate(&start);
  cudaEventCreate(&stop);
  std::vector<double> tops;
  for (int l = -1; l < launches; ++l) {  // launch -1 calibrates the length
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(ctas, 1, 1);
    cfg.blockDim = dim3(kThreadsPeak, 1, 1);
    cfg.dynamicSmemBytes = kSmemPeak;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = pair ? 2 : 1;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaEventRecord(start);
    if (!ok(cudaLaunchKernelEx(&cfg, kernel, kblocks, zeros ? 1 : 0, status), "launch")) return 1;
    cudaEventRecord(stop);
    if (!ok(cudaEventSynchronize(stop), "kernel")) return 1;
    float ms = 0;
    cudaEventElapsedTime(&ms, start, stop);
    const double t = ops_per_kblock * kblocks / (ms * 1e-3) / 1e12;
    if (l < 0) {
      kblocks = std::max(1000LL, static_cast<long long>(kblocks * ms_target / ms));
      continue;
    }
    tops.push_back(t);
    std::printf("launch %d: %.3f ms, %.1f TOPS\n", l, ms, t);
  }
  uint32_t word = 0;
  cudaMemcpy(&word, status, sizeof(word), cudaMemcpyDeviceToHost);
  if (word != 0) {
    std::fprintf(stderr, "mma_peak: a bounded wait gave up (status %u)\n", word);
    return 1;
  }
  std::sort(tops.begin(), tops.end());
  std::printf(
      "{\"metric\": \"int8_tensor_tops\", \"median\": %.1f, \"max\": %.1f, \"operands\": \"%s\", "
      "\"cta_group\": %d, \"ctas\": %d, \"ms_per_launch\": %.0f}\n",
      tops[tops.size() / 2], tops.back(), zeros ? "zero" : "random", pair ? 2 : 1, ctas,
      ms_target);
  return 0;
}
