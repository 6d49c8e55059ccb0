// mma_ceiling.cu - the int8 tensor-pipe ceiling of this GPU, measured.
//
// One CTA per SM issues back-to-back tcgen05.mma kind::i8 (M=128, N=256,
// K=32, operands K-major SW128 in shared memory, s32 accumulators in TMEM)
// with no memory traffic at all.  Four operand pairs are used in turn, so
// consecutive MMAs read different bytes; they are filled with hashed random
// bytes, zeros or ones.  Per fill the tool prints the median throughput over
// the repetitions, the SM clock the kernel actually ran at (clock64 against
// the global timer, per CTA, median over CTAs) and operations per clock per
// SM, the figure that does not depend on the clock.  Every barrier wait is
// bounded (2 s) and reports through a status word.
//
//   mma_ceiling [--iters N] [--reps R]
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <vector>

#include "sm100.cuh"

namespace {

using namespace i8c;

constexpr int kThreads = 128;
constexpr int kPairs = 4;                  // operand pairs used in turn
constexpr int kABytes = 128 * 128;         // 128 rows x 128 bytes
constexpr int kBBytes = 256 * 128;         // 256 rows x 128 bytes
constexpr int kOperandBytes = kPairs * (kABytes + kBBytes);
constexpr int kSmem = kOperandBytes + 1024 + 64;
constexpr int kMaxCtas = 1024;

__device__ uint32_t g_status;
__device__ long long g_cycles[kMaxCtas * 2];
__device__ unsigned long long g_ns[kMaxCtas * 2];

__global__ void __launch_bounds__(kThreads, 1) mma_loop(int iters, int fill, uint64_t limit_ns) {
  extern __shared__ uint8_t raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(raw) + 1023) &
                                              ~static_cast<uintptr_t>(1023));
  uint8_t *a = smem;
  uint8_t *b = smem + kPairs * kABytes;
  uint64_t *done = reinterpret_cast<uint64_t *>(smem + kOperandBytes);
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(done + 1);
  const bool timer = threadIdx.x == 0 && blockIdx.x < kMaxCtas;
  if (timer) {
    g_cycles[2 * blockIdx.x] = clock64();
    g_ns[2 * blockIdx.x] = global_timer_ns();
  }
  for (int i = threadIdx.x; i < kOperandBytes / 4; i += kThreads) {
    uint32_t h = (static_cast<uint32_t>(i) + 1u) * 2654435761u ^ (blockIdx.x * 40503u);
    h ^= h >> 15;
    h *= 2246822519u;
    h ^= h >> 13;
    reinterpret_cast<uint32_t *>(smem)[i] = fill == 0 ? h : fill == 1 ? 0u : 0x01010101u;
  }
  if (threadIdx.x == 0) {
    mbar_init(done, 1);
    fence_mbar_init();
  }
  if (threadIdx.x < 32) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  fence_proxy_async_smem();  // the operand bytes are read by the tensor core
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (threadIdx.x == 0) {
    const uint32_t idesc = idesc_s8(128, 256);
    const uint64_t a0 = smem_desc(smem_u32(a), 16, 1024, Layout::kSw128);
    const uint64_t b0 = smem_desc(smem_u32(b), 16, 1024, Layout::kSw128);
    for (int it = 0; it < iters; ++it) {
      const uint32_t d = tmem + static_cast<uint32_t>(it & 1) * 256;  // two accumulators
      const uint32_t pair = static_cast<uint32_t>(it) % kPairs;
#pragma unroll
      for (int k = 0; k < 4; ++k)
        umma_i8(d, a0 + pair * (kABytes >> 4) + 2 * k, b0 + pair * (kBBytes >> 4) + 2 * k, idesc,
                it > 1 || k > 0 ? 1u : 0u);
    }
    umma_commit(done);
    const WaitCtx ctx{limit_ns, &g_status};
    mbar_wait(done, 0, ctx, 1u);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (timer) {
    g_cycles[2 * blockIdx.x + 1] = clock64();
    g_ns[2 * blockIdx.x + 1] = global_timer_ns();
  }
  if (threadIdx.x < 32) tmem_dealloc(tmem, 512);
}

bool ok(cudaError_t e, const char *what) {
  if (e == cudaSuccess) return true;
  fprintf(stderr, "%s: %s\n", what, cudaGetErrorString(e));
  return false;
}

}  // namespace

int main(int argc, char **argv) {
  int iters = 20000, reps = 5;
  for (int i = 1; i < argc; ++i) {
    if (!strcmp(argv[i], "--iters") && i + 1 < argc) iters = atoi(argv[++i]);
    else if (!strcmp(argv[i], "--reps") && i + 1 < argc) reps = atoi(argv[++i]);
    else {
      fprintf(stderr, "usage: mma_ceiling [--iters N] [--reps R]\n");
      return 2;
    }
  }
  if (iters < 2 || reps < 1) {
    fprintf(stderr, "usage: mma_ceiling [--iters N >= 2] [--reps R >= 1]\n");
    return 2;
  }
  int sms = 0, major = 0;
  if (!ok(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, 0), "device") ||
      !ok(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, 0), "device"))
    return 1;
  if (major != 10) {
    fprintf(stderr, "needs an sm_100 device\n");
    return 1;
  }
  const int ctas = sms < kMaxCtas ? sms : kMaxCtas;
  if (!ok(cudaFuncSetAttribute(mma_loop, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem),
          "smem attribute"))
    return 1;
  cudaEvent_t e0, e1;
  if (!ok(cudaEventCreate(&e0), "event") || !ok(cudaEventCreate(&e1), "event")) return 1;
  const char *names[] = {"random", "zero", "ones"};
  const double ops_per_cta = 2.0 * 128 * 256 * 32 * 4.0 * iters;
  for (int fill = 0; fill < 3; ++fill) {
    mma_loop<<<ctas, kThreads, kSmem>>>(100, fill, 2000000000ull);
    if (!ok(cudaDeviceSynchronize(), "warm-up")) return 1;
    std::vector<double> tops, mhz;
    for (int r = 0; r < reps; ++r) {
      cudaEventRecord(e0);
      mma_loop<<<ctas, kThreads, kSmem>>>(iters, fill, 2000000000ull);
      cudaEventRecord(e1);
      if (!ok(cudaEventSynchronize(e1), "run")) return 1;
      float ms = 0;
      cudaEventElapsedTime(&ms, e0, e1);
      tops.push_back(ops_per_cta * ctas / (ms * 1e-3) / 1e12);
      std::vector<long long> cyc(2 * kMaxCtas);
      std::vector<unsigned long long> ns(2 * kMaxCtas);
      if (!ok(cudaMemcpyFromSymbol(cyc.data(), g_cycles, sizeof(long long) * cyc.size()), "read") ||
          !ok(cudaMemcpyFromSymbol(ns.data(), g_ns, sizeof(unsigned long long) * ns.size()), "read"))
        return 1;
      std::vector<double> per_cta;
      for (int c = 0; c < ctas; ++c)
        if (ns[2 * c + 1] > ns[2 * c])
          per_cta.push_back((cyc[2 * c + 1] - cyc[2 * c]) * 1e3 / (ns[2 * c + 1] - ns[2 * c]));
      std::sort(per_cta.begin(), per_cta.end());
      mhz.push_back(per_cta.empty() ? 0.0 : per_cta[per_cta.size() / 2]);
    }
    std::sort(tops.begin(), tops.end());
    std::sort(mhz.begin(), mhz.end());
    uint32_t status = 0;
    cudaMemcpyFromSymbol(&status, g_status, sizeof(status));
    const double t = tops[reps / 2], f = mhz[reps / 2];
    printf("operands %-6s %7.0f TOPS  SM clock %4.0f MHz  %5.0f ops/clk/SM  (%d CTAs, %d iterations, "
           "median of %d)%s\n",
           names[fill], t, f, f > 0 ? t * 1e12 / (f * 1e6) / ctas : 0.0, ctas, iters, reps,
           status ? "  WAIT TIMED OUT" : "");
    if (status) return 1;
  }
  return 0;
}
