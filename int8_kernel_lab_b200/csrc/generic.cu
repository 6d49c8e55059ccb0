// generic.cu - GENERIC family: INT8 implicit-GEMM convolution on tcgen05.
//
// Replaces generic_implicit_gemm_kernel / _sm80_kernel of the reference
// (include/generic_implicit_gemm.cuh:90-153, :170-227).  Same contract:
//   out[m*K + k] = bias[k] + sum_{r,s,c} X[n, oy*sh + r*dh - ph, ox*sw + s*dw - pw, c] * W[k,r,s,c]
// with padding taps skipped (here: zero-filled by TMA, which adds nothing).
//
// B200 design (one persistent CTA per SM, 6 warps):
//   warp 0     TMA producer.  Per k-block (tap r,s x channel block) it loads
//              A = 128 output pixels x CBLK channels with an im2col tensor map
//              (padding/stride/dilation handled by the TMA unit: bounding-box
//              corners, traversal strides, per-tap offsets) and
//              B = BN filters x CBLK channels with a tiled tensor map over the
//              filter viewed as [K][R*S][C].  Both land swizzled (SW128/64/32)
//              in a multi-stage ring guarded by mbarriers.
//   warp 1     MMA issuer: tcgen05.mma.cta_group::1.kind::i8, M=128, N=BN,
//              K=32 per instruction, int32 accumulators in TMEM.  Two TMEM
//              accumulator buffers let the epilogue of tile i overlap the
//              mainloop of tile i+1.
//   warps 2-5  epilogue: tcgen05.ld (one output pixel row per thread),
//              + bias, 16-byte int32 stores of the NHWK output.
// The reference's odd-K epilogue bug (:218-225) has no counterpart: every
// column < K is stored.
#include <cuda.h>
#include <cuda_runtime.h>

#include "conv_common.h"
#include "launch.h"
#include "sm100.cuh"

namespace i8c {

template <int CBLK>
struct SwizzleOf;
template <>
struct SwizzleOf<128> {
  static constexpr Layout kLayout = Layout::kSw128;
};
template <>
struct SwizzleOf<64> {
  static constexpr Layout kLayout = Layout::kSw64;
};
template <>
struct SwizzleOf<32> {
  static constexpr Layout kLayout = Layout::kSw32;
};

// Shared-memory plan, identical on host and device.
struct GenericSmem {
  uint32_t a_bytes, b_bytes;     // one stage of A / B
  uint32_t a_off, b_off, bar_off;
  uint32_t total;                // bytes requested at launch (incl. alignment slack)
};

__host__ __device__ inline GenericSmem generic_smem_plan(int cblk, int bn, int stages) {
  GenericSmem p;
  p.a_bytes = kBlockM * cblk;
  p.b_bytes = bn * cblk;
  p.a_off = 0;
  p.b_off = p.a_off + stages * p.a_bytes;
  p.bar_off = p.b_off + stages * p.b_bytes;
  // full[stages], empty[stages], tfull[2], tempty[2], drain, tmem slot
  const uint32_t bar_bytes = (2 * stages + 5) * 8 + 8;
  p.total = 1024 + p.bar_off + bar_bytes;
  return p;
}

template <int CBLK>
__global__ void __launch_bounds__(kThreads, 1)
    generic_conv_kernel(const __grid_constant__ CUtensorMap tmap_x,
                        const __grid_constant__ CUtensorMap tmap_w, const ConvGeom g,
                        const int32_t *__restrict__ bias, int32_t *__restrict__ out,
                        const RunCtl ctl) {
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte alignment: the SW128 atom (8 rows x 128 B) must start on it.
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const GenericSmem plan = generic_smem_plan(CBLK, g.bn, g.stages);
  uint8_t *a_ring = smem + plan.a_off;
  uint8_t *b_ring = smem + plan.b_off;
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + plan.bar_off);
  uint64_t *empty = full + g.stages;
  uint64_t *tfull = empty + g.stages;
  uint64_t *tempty = tfull + 2;
  uint64_t *drain = tempty + 2;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const WaitCtx wctx{ctl.wait_ns, ctl.status};

  if (threadIdx.x == 0) {
    for (int i = 0; i < g.stages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], 4 * 32);
    }
    mbar_init(drain, 1);
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

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      int stage = 0;
      uint32_t phase = 0;
      long issued = 0;
      const uint32_t stage_tx = plan.a_bytes + plan.b_bytes;
      bool ok = true;
      for (int tile = blockIdx.x; tile < g.num_tiles && ok; tile += gridDim.x) {
        const int m_tile = tile / g.n_tiles;
        const int n_tile = tile - m_tile * g.n_tiles;
        const int m0 = m_tile * kBlockM;
        const int n0 = n_tile * g.bn;
        const int img = m0 / g.PQ;
        const int rem = m0 - img * g.PQ;
        const int p = rem / g.Q;
        const int q = rem - p * g.Q;
        const int x_w = q * g.stride_w - g.pad_w;
        const int x_h = p * g.stride_h - g.pad_h;
        int tap = 0, cb = 0, r = 0, s = 0;
        for (int kb = 0; kb < g.kblocks; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, wctx, kStatusTimeoutEmpty)) {
            ok = false;
            break;
          }
          if (!ctl.starve) {
            mbar_arrive_expect_tx(&full[stage], stage_tx);
            tma_load_im2col_4d(a_ring + stage * plan.a_bytes, &tmap_x, &full[stage], cb * CBLK,
                               x_w, x_h, img, static_cast<uint16_t>(s * g.dil_w),
                               static_cast<uint16_t>(r * g.dil_h));
            tma_load_3d(b_ring + stage * plan.b_bytes, &tmap_w, &full[stage], cb * CBLK, tap,
                        n0);
            ++issued;
          }
          if (++stage == g.stages) {
            stage = 0;
            phase ^= 1u;
          }
          if (++cb == g.cblocks) {
            cb = 0;
            ++tap;
            if (++s == g.S) {
              s = 0;
              ++r;
            }
          }
        }
      }
      // Copies still in flight must land before the CTA exits: wait for the
      // phases this thread armed most recently (immediate on the normal path).
      const long pending = issued < g.stages ? issued : g.stages;
      for (long i = 0; i < pending; ++i) {
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
      constexpr Layout kLayout = SwizzleOf<CBLK>::kLayout;
      constexpr uint32_t kAtom = 8 * CBLK;  // 8 rows x CBLK bytes
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < g.num_tiles && ok; tile += gridDim.x) {
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, wctx, kStatusTimeoutDrain)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * g.acc_stride);
        for (int kb = 0; kb < g.kblocks; ++kb) {
          if (!mbar_wait(&full[stage], phase, wctx, kStatusTimeoutFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(a_ring + stage * plan.a_bytes);
          const uint32_t b_addr = smem_u32(b_ring + stage * plan.b_bytes);
#pragma unroll
          for (int k = 0; k < CBLK / 32; ++k) {
            const uint64_t a_desc = smem_desc(a_addr + 32 * k, 16, kAtom, kLayout);
            const uint64_t b_desc = smem_desc(b_addr + 32 * k, 16, kAtom, kLayout);
            umma_i8(d_tmem, a_desc, b_desc, idesc, (kb | k) != 0 ? 1u : 0u);
          }
          umma_commit(&empty[stage]);
          if (++stage == g.stages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(&tfull[acc]);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      // Every MMA issued must finish before TMEM is released.
      umma_commit(drain);
      mbar_wait(drain, 0, wctx, kStatusTimeoutTeardown);
    }
  } else {
    // ---------------- epilogue (warps 2..5) ----------------
    const int quarter = warp & 3;  // TMEM lane quarter this warp may access
    const int row = quarter * 32 + lane;
    const bool vec_k = (g.K & 3) == 0;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = blockIdx.x; tile < g.num_tiles; tile += gridDim.x) {
      const int m_tile = tile / g.n_tiles;
      const int n_tile = tile - m_tile * g.n_tiles;
      const int m = m_tile * kBlockM + row;
      const int n0 = n_tile * g.bn;
      // All lanes wait; the vote keeps the warp converged for tcgen05.ld even
      // if the wait runs out on some lanes only.
      if (!__all_sync(0xffffffffu, mbar_wait(&tfull[acc], acc_phase, wctx, kStatusTimeoutAccum)))
        break;
      tc_fence_after();
      const uint32_t taddr =
          tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + acc * g.acc_stride;
      int32_t *dst_row = out + static_cast<int64_t>(m) * g.K + n0;
      for (int c0 = 0; c0 < g.bn; c0 += 32) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(taddr + c0, v);
        tmem_ld_wait();
        if (m < g.M) {
          const int col0 = n0 + c0;
          if (vec_k && c0 + 32 <= g.bn && col0 + 32 <= g.K) {
            const int4 *b4 = reinterpret_cast<const int4 *>(bias + col0);
            int4 *d4 = reinterpret_cast<int4 *>(dst_row + c0);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const int4 bb = __ldg(b4 + j);
              int4 o;
              o.x = static_cast<int32_t>(v[4 * j + 0]) + bb.x;
              o.y = static_cast<int32_t>(v[4 * j + 1]) + bb.y;
              o.z = static_cast<int32_t>(v[4 * j + 2]) + bb.z;
              o.w = static_cast<int32_t>(v[4 * j + 3]) + bb.w;
              d4[j] = o;
            }
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              if (c0 + j < g.bn && col0 + j < g.K)
                dst_row[c0 + j] = static_cast<int32_t>(v[j]) + __ldg(bias + col0 + j);
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&tempty[acc]);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, g.tmem_cols);
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------

static int pick_cblk(int c) {
  if (c % 128 == 0) return 128;
  if (c % 64 == 0) return 64;
  return 32;
}

static int pick_bn(int k) {
  if (k <= 256) return (k + 15) / 16 * 16;
  // Balance the N tiles: the smallest multiple of 16 giving ceil(k/256) tiles.
  const int tiles = (k + 255) / 256;
  const int per = (k + tiles - 1) / tiles;
  return (per + 15) / 16 * 16;
}

static int next_pow2(int v) {
  int p = 32;
  while (p < v) p <<= 1;
  return p;
}

bool generic_plan(const int8conv_shape &s, ConvGeom &g, int &cblk) {
  const int32_t out_h = (s.h + 2 * s.pad_h - s.dilation_h * (s.r - 1) - 1) / s.stride_h + 1;
  const int32_t out_w = (s.w + 2 * s.pad_w - s.dilation_w * (s.s - 1) - 1) / s.stride_w + 1;
  cblk = pick_cblk(s.c);
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
  g.bn = pick_bn(s.k);
  g.acc_stride = (g.bn + 31) / 32 * 32;
  g.tmem_cols = next_pow2(2 * g.acc_stride);
  const GenericSmem one = generic_smem_plan(cblk, g.bn, 1);
  const int per_stage = one.a_bytes + one.b_bytes;
  int stages = (kMaxSmem - 1024 - 256) / per_stage;
  if (stages > 8) stages = 8;
  if (stages < 2) return false;
  g.stages = stages;
  g.m_tiles = (g.M + kBlockM - 1) / kBlockM;
  g.n_tiles = (s.k + g.bn - 1) / g.bn;
  g.num_tiles = g.m_tiles * g.n_tiles;
  return g.tmem_cols <= 512;
}

template <int CBLK>
static int8conv_status launch_generic_t(const int8conv_shape &s, const ConvGeom &g,
                                        const int8_t *x, const int8_t *w, const int32_t *b,
                                        int32_t *y, cudaStream_t stream) {
  DeviceInfo &dev = device_info();
  CUtensorMap maps[2];
  int8conv_status st = activation_map_im2col(s, x, CBLK, kBlockM, g.Q, &maps[0]);
  if (st != INT8CONV_OK) return st;
  st = filter_map_tiled(s, w, CBLK, g.bn, &maps[1]);
  if (st != INT8CONV_OK) return st;
  const GenericSmem plan = generic_smem_plan(CBLK, g.bn, g.stages);
  auto kernel = generic_conv_kernel<CBLK>;
  if (!ensure_smem_attr(reinterpret_cast<const void *>(kernel), plan.total))
    return INT8CONV_CUDA_ERROR;
  const int grid = g.num_tiles < dev.sm_count ? g.num_tiles : dev.sm_count;
  kernel<<<grid, kThreads, plan.total, stream>>>(maps[0], maps[1], g, b, y, run_ctl());
  note_launch();
  return cudaGetLastError() == cudaSuccess ? INT8CONV_OK : INT8CONV_CUDA_ERROR;
}

int8conv_status launch_generic_impl(const int8conv_shape &s, const int8_t *x, const int8_t *w,
                                    const int32_t *b, int32_t *y, cudaStream_t stream) {
  ConvGeom g;
  int cblk = 0;
  if (!generic_plan(s, g, cblk)) return INT8CONV_NOT_ELIGIBLE;
  switch (cblk) {
    case 128:
      return launch_generic_t<128>(s, g, x, w, b, y, stream);
    case 64:
      return launch_generic_t<64>(s, g, x, w, b, y, stream);
    default:
      return launch_generic_t<32>(s, g, x, w, b, y, stream);
  }
}

}  // namespace i8c
