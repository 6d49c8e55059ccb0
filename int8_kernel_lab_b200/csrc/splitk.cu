// splitk.cu - SPLITK family: the R*S*C reduction of one output tile split
// across the CTAs of a thread-block cluster, reduced through distributed
// shared memory.  No reference counterpart.
//
// For small-M, deep-reduction layers (e.g. 7x7 feature maps with 512-2048
// input channels) the generic kernel has only a handful of 128-row tiles for
// 148 SMs.  Here a cluster of `splits` CTAs (<= 8) computes one tile:
//   1. CTA r runs k-blocks [r*KB/splits, (r+1)*KB/splits) of the tap x
//      channel-block reduction: TMA im2col / tiled loads, tcgen05 kind::i8
//      into its own TMEM accumulator (M = 128, N = BN).
//   2. Its epilogue warps copy the int32 partial into its own shared memory
//      (the operand ring is idle by then).
//   3. Cluster barrier; CTA r then sums rows [r*128/splits, (r+1)*128/splits)
//      of all `splits` partials with ld.shared::cluster, adds the bias and
//      writes those output rows with 16-byte stores.
//   4. Cluster barrier before exit, so no partial disappears while read.
// Integer addition is exact and associative, so the result is bit-identical
// to the unsplit kernels.
#include <cuda.h>
#include <cuda_runtime.h>

#include <atomic>
#include <mutex>

#include "conv_common.h"
#include "int8conv_rules.h"
#include "launch.h"
#include "sm100.cuh"

namespace i8c {

constexpr int kMaxSplits = 8;

struct SplitGeom {
  ConvGeom g;       // M, K, P, Q, ... and bn, stages, tmem_cols, n_tiles, num_tiles
  int32_t splits;   // CTAs per cluster
  int32_t part_pitch;  // bytes per row of the shared-memory partial (4*BN + 16)
  int32_t ring_bytes;  // bytes of the operand ring (>= 128 * part_pitch)
};

__device__ __forceinline__ int4 ld_cluster_v4(uint32_t addr) {
  int4 v;
  asm volatile("ld.shared::cluster.v4.s32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}

template <int CBLK>
struct SplitSwizzle;
template <>
struct SplitSwizzle<128> {
  static constexpr Layout kLayout = Layout::kSw128;
};
template <>
struct SplitSwizzle<64> {
  static constexpr Layout kLayout = Layout::kSw64;
};
template <>
struct SplitSwizzle<32> {
  static constexpr Layout kLayout = Layout::kSw32;
};

template <int CBLK, bool REQ>
__global__ void __launch_bounds__(kSplitThreads, 1)
    splitk_kernel(const __grid_constant__ CUtensorMap tmap_x,
                  const __grid_constant__ CUtensorMap tmap_w, const SplitGeom sg,
                  const int32_t *__restrict__ bias, int32_t *__restrict__ out,
                  const RunCtl ctl, const Requant rq) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const ConvGeom &g = sg.g;
  const uint32_t a_bytes = kBlockM * CBLK;
  const uint32_t b_bytes = g.bn * CBLK;
  uint8_t *a_ring = smem;
  uint8_t *b_ring = smem + g.stages * a_bytes;
  uint8_t *partial = smem;  // reuses the ring once every MMA is done
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + sg.ring_bytes);
  uint64_t *empty = full + g.stages;
  uint64_t *tfull = empty + g.stages;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(tfull + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const WaitCtx wctx{ctl.wait_ns, ctl.status};
  const int split = static_cast<int>(cluster_ctarank());
  const int tile = static_cast<int>(blockIdx.x) / sg.splits;
  const int m_tile = tile / g.n_tiles;
  const int n_tile = tile - m_tile * g.n_tiles;
  const int m0 = m_tile * kBlockM;
  const int n0 = n_tile * g.bn;
  const int kb_begin = static_cast<int>((static_cast<int64_t>(g.kblocks) * split) / sg.splits);
  const int kb_end = static_cast<int>((static_cast<int64_t>(g.kblocks) * (split + 1)) / sg.splits);

  if (threadIdx.x == 0) {
    for (int i = 0; i < g.stages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    mbar_init(tfull, 1);
    fence_mbar_init();
    tma_prefetch_desc(&tmap_x);
    tma_prefetch_desc(&tmap_w);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, g.tmem_cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  bool epi_ok = true;
  // Programmatic stream serialisation: nothing touches global memory before
  // the previous kernel in the stream is complete.
  griddep_wait();
  griddep_launch_dependents();

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      const int img = m0 / g.PQ;
      const int rem = m0 - img * g.PQ;
      const int p = rem / g.Q;
      const int q = rem - p * g.Q;
      const int x_w = q * g.stride_w - g.pad_w;
      const int x_h = p * g.stride_h - g.pad_h;
      int stage = 0;
      uint32_t phase = 0;
      long armed = 0;
      for (int kb = kb_begin; kb < kb_end; ++kb) {
        if (!mbar_wait(&empty[stage], phase ^ 1u, wctx, kStatusTimeoutEmpty)) break;
        if (!ctl.starve) {
          const int tap = kb / g.cblocks;
          const int cb = kb - tap * g.cblocks;
          const int r = tap / g.S;
          const int s = tap - r * g.S;
          mbar_arrive_expect_tx(&full[stage], a_bytes + b_bytes);
          ++armed;
          tma_load_im2col_4d(a_ring + stage * a_bytes, &tmap_x, &full[stage], cb * CBLK, x_w, x_h,
                             img, static_cast<uint16_t>(s * g.dil_w),
                             static_cast<uint16_t>(r * g.dil_h));
          tma_load_3d(b_ring + stage * b_bytes, &tmap_w, &full[stage], cb * CBLK, tap, n0);
        }
        if (++stage == g.stages) {
          stage = 0;
          phase ^= 1u;
        }
      }
      for (long i = 0, n = armed < g.stages ? armed : g.stages; i < n; ++i) {
        if (--stage < 0) {
          stage = g.stages - 1;
          phase ^= 1u;
        }
        mbar_wait(&full[stage], phase, wctx, kStatusTimeoutTeardown);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      const uint32_t idesc = idesc_s8(kBlockM, g.bn);
      constexpr Layout kLayout = SplitSwizzle<CBLK>::kLayout;
      constexpr uint32_t kAtom = 8 * CBLK;
      // Descriptors built once; a byte offset d adds d >> 4 (see conv_kernel).
      const uint64_t a_desc0 = smem_desc(smem_u32(a_ring), 16, kAtom, kLayout);
      const uint64_t b_desc0 = smem_desc(smem_u32(b_ring), 16, kAtom, kLayout);
      int stage = 0;
      uint32_t phase = 0;
      uint32_t accumulate = 0;
      bool ok = true;
      for (int kb = kb_begin; kb < kb_end; ++kb) {
        if (!mbar_wait(&full[stage], phase, wctx, kStatusTimeoutFull)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint64_t ad = a_desc0 + ((stage * a_bytes) >> 4);
        const uint64_t bd = b_desc0 + ((stage * b_bytes) >> 4);
#pragma unroll
        for (int k = 0; k < CBLK / 32; ++k) {
          umma_i8(tmem_base, ad + 2 * k, bd + 2 * k, idesc, accumulate);  // +32 bytes per MMA
          accumulate = 1;
        }
        umma_commit(&empty[stage]);
        if (++stage == g.stages) {
          stage = 0;
          phase ^= 1u;
        }
      }
      (void)ok;
      // Arrives once every MMA issued above is complete (also when the
      // k-range was empty or a wait ran out: nothing is left in flight).
      umma_commit(tfull);
    }
  } else {
    // ---------------- partial -> shared memory (warps 2..5) ----------------
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    epi_ok = __all_sync(0xffffffffu, mbar_wait(tfull, 0, wctx, kStatusTimeoutAccum));
    tc_fence_after();
    const bool have = kb_end > kb_begin && epi_ok;
    const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16);
    int4 *dst = reinterpret_cast<int4 *>(partial + row * sg.part_pitch);
    for (int c0 = 0; c0 < g.bn; c0 += 32) {
      uint32_t v[32];
      if (have) {
        tmem_ld_32x32b_x32(taddr + c0, v);
        tmem_ld_wait();
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = 0;
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        if (c0 + 4 * j < g.bn)
          dst[c0 / 4 + j] = make_int4(static_cast<int32_t>(v[4 * j]), static_cast<int32_t>(v[4 * j + 1]),
                                      static_cast<int32_t>(v[4 * j + 2]),
                                      static_cast<int32_t>(v[4 * j + 3]));
      }
    }
  }

  // Every partial of the cluster is in shared memory after this barrier.
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, g.tmem_cols);
  }

  // ---------------- cluster reduction: this CTA's row slice ----------------
  const int rows_per = (kBlockM + sg.splits - 1) / sg.splits;
  const int r_begin = split * rows_per;
  const int r_end = r_begin + rows_per < kBlockM ? r_begin + rows_per : kBlockM;
  const int groups = g.bn / 4;  // 16-byte column groups per row
  const uint32_t part_base = smem_u32(partial);
  const bool vec_k = (g.K & 3) == 0;
  for (int item = threadIdx.x; item < (r_end - r_begin) * groups; item += kSplitThreads) {
    const int rr = r_begin + item / groups;
    const int cg = item - (item / groups) * groups;
    const int m = m0 + rr;
    const int col = n0 + 4 * cg;
    if (m >= g.M || col >= g.K) continue;
    const uint32_t off = part_base + rr * sg.part_pitch + cg * 16;
    // Every split's load is issued before any is summed, so the remote
    // latencies overlap instead of adding up.
    int4 part[kMaxSplits];
#pragma unroll
    for (int p = 0; p < kMaxSplits; ++p)
      if (p < sg.splits) part[p] = ld_cluster_v4(mapa_shared(off, static_cast<uint32_t>(p)));
    int4 acc = make_int4(0, 0, 0, 0);
#pragma unroll
    for (int p = 0; p < kMaxSplits; ++p) {
      if (p < sg.splits) {
        acc.x += part[p].x;
        acc.y += part[p].y;
        acc.z += part[p].z;
        acc.w += part[p].w;
      }
    }
    if constexpr (REQ) {
      // Four int8 outputs of one row: NHWC bytes m*K + col.., or one quarter
      // of a 32-channel vector in NCHW_VECT_C (K % 32 == 0).
      const int32_t a4[4] = {acc.x, acc.y, acc.z, acc.w};
      const int32_t lo = rq.relu ? rq.zero_point : -128;
      int32_t y4[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const bool in = col + j < g.K;
        y4[j] = in ? rq_apply_dev(static_cast<int32_t>(static_cast<uint32_t>(a4[j]) +
                                                       static_cast<uint32_t>(__ldg(bias + col + j))),
                                  rq_channel(__ldg(rq.multiplier + col + j),
                                             __ldg(rq.exponent + col + j)),
                                  rq.zero_point, lo)
                   : 0;
      }
      int8_t *out8 = reinterpret_cast<int8_t *>(out);
      if (rq.layout == 1) {
        const int img = m / g.PQ;
        const int pq = m - img * g.PQ;
        *reinterpret_cast<uint32_t *>(
            out8 + ((static_cast<int64_t>(img) * (g.K >> 5) + (col >> 5)) * g.PQ + pq) * 32 +
            (col & 31)) = rq_pack4(y4[0], y4[1], y4[2], y4[3]);
      } else if (vec_k) {
        *reinterpret_cast<uint32_t *>(out8 + static_cast<int64_t>(m) * g.K + col) =
            rq_pack4(y4[0], y4[1], y4[2], y4[3]);
      } else {
        for (int j = 0; j < 4 && col + j < g.K; ++j)
          out8[static_cast<int64_t>(m) * g.K + col + j] = static_cast<int8_t>(y4[j]);
      }
      continue;
    }
    int32_t *o = out + static_cast<int64_t>(m) * g.K + col;
    if (vec_k) {
      const int4 bb = __ldg(reinterpret_cast<const int4 *>(bias + col));
      acc.x += bb.x;
      acc.y += bb.y;
      acc.z += bb.z;
      acc.w += bb.w;
      *reinterpret_cast<int4 *>(o) = acc;
    } else {
      const int32_t a4[4] = {acc.x, acc.y, acc.z, acc.w};
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (col + j < g.K) o[j] = a4[j] + __ldg(bias + col + j);
    }
  }
  // Peers may still be reading this CTA's partial.
  cluster_sync_all();
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------

static int split_cblk(int c) { return i8c_channel_block(c); }

// Plans a split-K launch; false if the shape has too little reduction to
// split.  `clusters[c]` = clusters of size c that can be resident at once.
static bool plan_split(const int8conv_shape &s, const int32_t *clusters, SplitGeom &sg,
                       int &cblk) {
  const int32_t out_h = (s.h + 2 * s.pad_h - s.dilation_h * (s.r - 1) - 1) / s.stride_h + 1;
  const int32_t out_w = (s.w + 2 * s.pad_w - s.dilation_w * (s.s - 1) - 1) / s.stride_w + 1;
  cblk = split_cblk(s.c);
  ConvGeom &g = sg.g;
  g = ConvGeom{};
  g.M = s.n * out_h * out_w;
  g.K = s.k;
  g.P = out_h;
  g.Q = out_w;
  g.PQ = out_h * out_w;
  g.R = s.r;
  g.S = s.s;
  g.pad_h = s.pad_h;
  g.pad_w = s.pad_w;
  g.stride_h = s.stride_h;
  g.stride_w = s.stride_w;
  g.dil_h = s.dilation_h;
  g.dil_w = s.dilation_w;
  g.cblocks = (s.c + cblk - 1) / cblk;
  g.kblocks = s.r * s.s * g.cblocks;
  if (g.kblocks < 2) return false;
  g.bn = s.k <= 128 ? (s.k + 15) / 16 * 16 : 128;
  g.acc_stride = (g.bn + 31) / 32 * 32;
  int cols = 32;
  while (cols < g.acc_stride) cols <<= 1;
  g.tmem_cols = cols;
  g.m_tiles = (g.M + kBlockM - 1) / kBlockM;
  g.n_tiles = (s.k + g.bn - 1) / g.bn;
  g.num_tiles = g.m_tiles * g.n_tiles;
  // The largest split whose clusters all run in one wave; with too many
  // tiles for that, pairs of CTAs in several waves.
  int splits = i8c_split_count(g.num_tiles, g.kblocks, clusters);
  if (splits < 2) splits = 2;
  sg.splits = splits;
  sg.part_pitch = 4 * g.bn + 16;
  const int per_stage = kBlockM * cblk + g.bn * cblk;
  const int budget = kMaxSmem - 1024 - 512;
  int stages = budget / per_stage;
  if (stages > 8) stages = 8;
  const int k_per_split = (g.kblocks + splits - 1) / splits;
  if (stages > k_per_split && k_per_split >= 2) stages = k_per_split;
  if (stages < 2) stages = 2;
  g.stages = stages;
  int ring = stages * per_stage;
  const int need = kBlockM * sg.part_pitch;
  if (ring < need) ring = need;
  sg.ring_bytes = (ring + 1023) & ~1023;
  const int total = 1024 + sg.ring_bytes + (2 * stages + 1) * 8 + 16;
  return total <= kMaxSmem;
}

bool splitk_eligible_runtime(const int8conv_shape &s) {
  SplitGeom sg;
  int cblk = 0;
  const int32_t b200[9] = I8C_B200_CLUSTERS;
  return plan_split(s, b200, sg, cblk);
}

template <int CBLK, bool REQ>
static int8conv_status launch_split_t(const int8conv_shape &s, const SplitGeom &sg,
                                      const int8_t *x, const int8_t *w, const int32_t *b,
                                      void *y, const Requant &rq, cudaStream_t stream) {
  CUtensorMap maps[2];
  int8conv_status st = activation_map_im2col(s, x, CBLK, kBlockM, sg.g.Q, sg.g.P, &maps[0]);
  if (st != INT8CONV_OK) return st;
  st = filter_map_tiled(s, w, CBLK, sg.g.bn, &maps[1]);
  if (st != INT8CONV_OK) return st;
  const uint32_t total = 1024 + sg.ring_bytes + (2 * sg.g.stages + 1) * 8 + 16;
  const uint32_t smem = total > kMaxSmem / 2 + 1024 ? total : kMaxSmem / 2 + 1024;
  auto kernel = splitk_kernel<CBLK, REQ>;
  static std::atomic<uint32_t> smem_set[64];
  std::atomic<uint32_t> &slot = smem_set[device_info().device & 63];
  if (slot.load(std::memory_order_relaxed) < smem) {
    if (!ensure_smem_attr(reinterpret_cast<const void *>(kernel), kMaxSmem))
      return INT8CONV_CUDA_ERROR;
    slot.store(kMaxSmem, std::memory_order_relaxed);
  }
  LaunchPlan plan;
  plan.func = reinterpret_cast<const void *>(kernel);
  plan.grid = dim3(sg.g.num_tiles * sg.splits, 1, 1);
  plan.block = dim3(kSplitThreads, 1, 1);
  plan.smem = smem;
  plan.cluster = sg.splits;
  plan_args(plan, maps[0], maps[1], sg, b, static_cast<int32_t *>(y), run_ctl(), rq);
  return launch_plan(plan, stream);
}

// Resident clusters per cluster size on the current device, queried once
// per device (cudaOccupancyMaxActiveClusters; one CTA per SM, like every
// split-K launch).  Falls back to the B200 table if the query fails.
static const int32_t *cluster_table() {
  static int32_t table[64][9];
  static std::atomic<int> ready[64];
  static std::mutex fill;
  DeviceInfo &dev = device_info();
  const int d = dev.device & 63;
  if (ready[d].load(std::memory_order_acquire)) return table[d];
  // One thread fills a device's row; the others wait here and then read it.
  std::lock_guard<std::mutex> lock(fill);
  if (ready[d].load(std::memory_order_relaxed)) return table[d];
  const int32_t b200[9] = I8C_B200_CLUSTERS;
  int32_t t[9];
  auto kernel = splitk_kernel<128, false>;
  const bool attr_ok = ensure_smem_attr(reinterpret_cast<const void *>(kernel), kMaxSmem);
  for (int c = 0; c < 9; ++c) {
    t[c] = b200[c];
    if (c < 2 || !attr_ok) continue;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(c * 16, 1, 1);
    cfg.blockDim = dim3(kSplitThreads, 1, 1);
    cfg.dynamicSmemBytes = kMaxSmem / 2 + 1024;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = c;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kernel, &cfg) == cudaSuccess && n > 0)
      t[c] = n;
    else
      cudaGetLastError();
  }
  t[1] = dev.sm_count;
  for (int c = 0; c < 9; ++c) table[d][c] = t[c];
  ready[d].store(1, std::memory_order_release);
  return table[d];
}

template <bool REQ>
static int8conv_status launch_split(const int8conv_shape &s, const int8_t *x, const int8_t *w,
                                    const int32_t *b, void *y, const Requant &rq,
                                    cudaStream_t stream) {
  SplitGeom sg;
  int cblk = 0;
  if (!plan_split(s, cluster_table(), sg, cblk)) return INT8CONV_NOT_ELIGIBLE;
  switch (cblk) {
    case 128:
      return launch_split_t<128, REQ>(s, sg, x, w, b, y, rq, stream);
    case 64:
      return launch_split_t<64, REQ>(s, sg, x, w, b, y, rq, stream);
    default:
      return launch_split_t<32, REQ>(s, sg, x, w, b, y, rq, stream);
  }
}

int8conv_status launch_splitk_impl(const int8conv_shape &s, const int8_t *x, const int8_t *w,
                                   const int32_t *b, int32_t *y, cudaStream_t stream) {
  return launch_split<false>(s, x, w, b, y, Requant{}, stream);
}

int8conv_status launch_splitk_requant(const int8conv_shape &s, const int8_t *x, const int8_t *w,
                                      const int32_t *b, const Requant &rq, int8_t *y,
                                      cudaStream_t stream) {
  return launch_split<true>(s, x, w, b, y, rq, stream);
}

}  // namespace i8c
