// conv_kernel.cu - GENERIC, STRIP and HALO families: INT8 implicit-GEMM
// convolution on tcgen05 tensor cores.
//
// Contract of the reference kernels it replaces (generic_implicit_gemm_kernel,
// include/generic_implicit_gemm.cuh:90-153 / :170-227, and spatial_strip_kernel,
// include/spatial_strip.cuh:118-196 / :214-286):
//   out[m*K + k] = bias[k] + sum_{r,s,c} X[n, oy*sh + r*dh - ph, ox*sw + s*dw - pw, c] * W[k,r,s,c]
// with padding taps contributing nothing (here: zero-filled by TMA).
//
// B200 design (persistent CTAs, 6 warps each; 18 with the int8 epilogue;
// 3 more with the gather staging):
//   warp 0     TMA producer.  Activations come through an im2col tensor map
//              (padding, stride and dilation are done by the TMA unit:
//              bounding-box corners, traversal strides, per-tap offsets),
//              filters through a tiled map over W viewed as [K][R*S][C].
//              Tiles land swizzled (SW128/64/32 for 128/64/32-byte channel
//              blocks) in mbarrier-guarded rings.
//   warp 1     MMA issuer: tcgen05.mma kind::i8, K=32 bytes per instruction,
//              int32 accumulators in TMEM.  Two accumulator buffers let the
//              epilogue of tile i overlap the mainloop of tile i+1.
//   warps 2-5  epilogue: tcgen05.ld (one output pixel row per thread),
//              + bias, a 32 x 32 int32 block staged in 128-byte-swizzled
//              shared memory and written by one TMA tensor store (rows >= M
//              and columns >= K clipped).  STRIP stages only a block's
//              valid rows (consecutive output pixels), compacted, and stores
//              them through the map whose box has that many rows.  Where a
//              TMA store does not apply (HALO padded rows, K % 4 != 0, a
//              block crossing into the next N tile) the staged block is
//              transposed and leaves as 16-byte stores that write whole
//              128-byte row segments.
//   warps 2-17 with the requantised int8 epilogue (REQ): four warps per TMEM
//              lane quarter, each owning every fourth 32-column block;
//              per-N-tile channel tables in shared memory; 32 x 32-byte TMA
//              stores (NHWC) or 32-byte vector stores (NCHW_VECT_C).
//
// Single CTA (PAIR = false): cta_group::1, M = 128 rows per tile.
// CTA pair (PAIR = true, cluster of 2): cta_group::2, M = 256 rows per tile.
//   Each CTA loads its own 128 rows of A and half of the BN filter rows of B;
//   the leader (rank 0) arms its barriers for both CTAs' bytes and issues the
//   MMAs, which read A and B from both CTAs' shared memory, so every filter
//   tile crosses L2 -> SM once per 256 output rows instead of once per 128.
//   Commits arrive on both CTAs' barriers; each epilogue drains its own TMEM
//   and releases the accumulator on the leader.
//
// GENERIC: per k-block (tap r,s x channel block) one A tile of output pixels
//   and one B tile.
// STRIP (stride_w = dilation_w = 1): the M dimension runs over padded-row
//   positions (n, oy, j), j < Wp = out_w + S - 1.  Per (r, channel block) ONE
//   im2col load of 128 + S - 1 consecutive positions feeds all S filter
//   columns: the A descriptor of column s starts s rows later in the same
//   swizzled strip (the swizzle follows absolute shared-memory address bits,
//   so a whole-row shift needs no re-layout).  Positions j >= out_w are
//   computed and dropped by the epilogue.  The reference reused a 130-pixel
//   strip across the 3 filter columns the same way (spatial_strip.cuh:17-29,
//   :98-116), for out_w % 128 == 0 only.
// HALO (unit strides): the M dimension runs over the zero-padded image
//   (Hp x Wp positions per image); one staged tile of 128 + (R-1)*dh*Wp +
//   (S-1)*dw positions per channel block feeds all R*S taps, tap (r, s)
//   reading it r*dh*Wp + s*dw rows further on.
// GATHER (GENERIC on shapes the im2col tensor map cannot encode: stride > 8,
//   pad > 127, tap span > 127): four gather warps (warp 0 and three after
//   the epilogue's) stage the same 128-row tiles, 32 rows each, with
//   asynchronous 16-byte copies into the same swizzled layout
//   (gather_producer); the filter, the MMA issuer and the epilogue are
//   GENERIC's.  Single CTAs only.
// The reference's odd-K epilogue bug (generic_implicit_gemm.cuh:218-225) has
// no counterpart: every column < K is stored.
#include <cuda.h>
#include <cuda_runtime.h>

#include <atomic>

#include "conv_common.h"
#include "int8conv_rules.h"
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

// Epilogue staging: 4 warps x 2 buffers x (32 rows x 128 B) (int32 output),
// or 16 warps x (32 x 32 B block + channel tables) (int8 output).
constexpr uint32_t kEpilogueStaging = 4 * 2 * 32 * 128;
constexpr uint32_t kOneCtaPerSm = kMaxSmem / 2 + 1024;

// Kernel variants: how the A operand (output pixels x channels) is staged.
constexpr int kModeGeneric = 0;  // one im2col tile per tap and channel block
constexpr int kModeStrip = 1;    // one row strip per (filter row, channel block)
constexpr int kModeHalo = 2;     // one halo tile per channel block
constexpr int kModeGather = 3;   // GENERIC's tiles staged by a gather warp (any shape)
// Row table of the gather warp: one int4 per row of a 128-row tile.
constexpr uint32_t kGatherRowTable = kBlockM * 16;
// Largest staged tile (rows of CBLK bytes): im2col loads move at most 1024
// pixels, and a few stages must fit in shared memory.
constexpr int kMaxStagedRows = 512;

// Shared-memory plan, identical on host and device.
struct SmemPlan {
  uint32_t a_bytes, b_bytes;  // one stage of A / B (this CTA's share)
  uint32_t a_off, b_off, stage_off, bar_off;
  uint32_t rows_off;          // gather row table (GATHER only)
  uint32_t total;             // bytes requested at launch (incl. alignment slack)
};

__host__ __device__ inline SmemPlan smem_plan(int cblk, int b_rows, int a_rows, int a_stages,
                                              int b_stages, bool gather = false) {
  SmemPlan p;
  p.a_bytes = a_rows * cblk;
  p.b_bytes = b_rows * cblk;
  p.a_off = 0;
  p.b_off = p.a_off + a_stages * p.a_bytes;
  // Epilogue staging starts on a 1024-byte boundary: it doubles as the
  // 128-byte-swizzled source of the TMA output stores.
  p.stage_off = (p.b_off + b_stages * p.b_bytes + 1023) & ~1023u;
  p.bar_off = p.stage_off + kEpilogueStaging;
  // a_full/a_empty[a_stages], b_full/b_empty[b_stages], tfull[2], tempty[2], drain, slot
  const uint32_t bar_bytes = (2 * a_stages + 2 * b_stages + 5) * 8 + 8;
  p.rows_off = (p.bar_off + bar_bytes + 15) & ~15u;
  p.total = 1024 + (gather ? p.rows_off + kGatherRowTable : p.bar_off + bar_bytes);
  return p;
}

// Ring position: stage index and the parity of its current fill.
struct Ring {
  int stage = 0;
  uint32_t phase = 0;
  __device__ __forceinline__ void next(int stages) {
    if (++stage == stages) {
      stage = 0;
      phase ^= 1u;
    }
  }
  __device__ __forceinline__ void prev(int stages) {
    if (--stage < 0) {
      stage = stages - 1;
      phase ^= 1u;
    }
  }
};

// One work unit of the persistent schedule: a whole tile, or one column part
// of a tile of the last wave (see ConvGeom::split_f).
struct Unit {
  int m_tile;  // 128- or 256-row tile index
  int n0;      // first output channel of the unit
  int bn;      // output channels of the unit
};

__device__ __forceinline__ Unit unit_at(const ConvGeom &g, int u) {
  int tile = u, part = 0, bn = g.bn;
  if (u >= g.split_from) {
    const int idx = u - g.split_from;
    tile = g.split_from + idx / g.split_f;
    part = idx - (idx / g.split_f) * g.split_f;
    bn = g.bn / g.split_f;
  }
  Unit t;
  t.m_tile = tile / g.n_tiles;
  t.n0 = (tile - t.m_tile * g.n_tiles) * g.bn + part * bn;
  t.bn = bn;
  return t;
}

template <bool PAIR>
__device__ __forceinline__ void commit_to(uint64_t *bar) {
  if constexpr (PAIR)
    umma_commit_pair(bar, 0x3);
  else
    umma_commit(bar);
}

// GATHER producer: GENERIC's A tiles for shapes the im2col tensor map cannot
// encode (stride > 8, pad > 127, tap span > 127, or a bounding-box corner out
// of range), in the same swizzled layout TMA would write, so the MMA issuer
// and the epilogue are GENERIC's.  This is the reference's gather
// (generic_implicit_gemm.cuh:46-69: 16-byte vectors at (n, iy, ix, c), zero
// for padding taps and rows past M) done by kGatherWarps warps with
// asynchronous 16-byte copies, each warp owning 32 rows of the 128-row tile
// and keeping `g.gather_lag` k-blocks in flight.
//
// Per tile a warp tabulates, in shared memory, each of its rows' input
// origin (oy*sh - ph, ox*sw - pw) and that origin's byte offset in X; per
// k-block (tap r,s x channel block) the tap's offset (r*dh*W + s*dw)*C is the
// same for every row, so a 16-byte chunk costs a bounds check and an add.
// Lane (row sub-index, 16-byte chunk) copies its chunk of every
// (32 / chunks)-th row of the warp's 32.  A k-block is published once every
// lane's copies have landed: each lane fences its generic-proxy writes for
// the tensor cores' async-proxy reads and arrives on the stage's barrier,
// which also counts the filter tile's TMA bytes (warp 0's lane 0 arms and
// issues it): 1 + 32 * kGatherWarps arrivals per phase.
constexpr int kGatherWarps = 4;

template <int CBLK>
__device__ __forceinline__ void gather_producer(const ConvGeom &g, const int8_t *__restrict__ x,
                                                const CUtensorMap *tmap_w, uint8_t *a_ring,
                                                uint8_t *b_ring, const SmemPlan &plan,
                                                int4 *rowtab, uint64_t *b_full,
                                                uint64_t *b_empty, const RunCtl &ctl,
                                                const WaitCtx &wctx, int tile_first,
                                                int tile_step, int gw, int lane) {
  constexpr int kChunks = CBLK / 16;          // 16-byte chunks per row
  constexpr int kRowsPerPass = 32 / kChunks;  // rows one warp-wide pass covers
  constexpr int kPasses = 32 / kRowsPerPass;  // passes over the warp's 32 rows
  constexpr uint32_t kSwMask = kChunks - 1;   // 128/64/32-byte swizzle: chunk ^= row bits
  const int chunk = lane % kChunks;
  const int rsub = lane / kChunks;
  const int row_base = 32 * gw;               // this warp's rows of the tile
  const int lag = g.gather_lag;
  const bool loads_filter = gw == 0 && lane == 0;
  const bool row_blocks = g.row_blocks != 0;
  int4 *mytab = rowtab + row_base;
  Ring rb;           // next stage to fill
  Ring rp;           // oldest stage filled but not yet published
  int pending = 0;   // k-blocks issued and not yet published
  long armed_b = 0;  // filter loads issued (warp 0, lane 0)
  auto publish = [&]() {
    // This lane's copies of the k-block are complete (cp_async_wait);
    // make them visible to the async proxy, then arrive.
    fence_proxy_async_smem();
    mbar_arrive(&b_full[rp.stage]);
    rp.next(g.stages);
    --pending;
  };
  bool ok = true;
  for (int tile = tile_first; tile < g.num_units && ok; tile += tile_step) {
    const Unit t = unit_at(g, tile);
    // Row table of this warp's 32 rows (every lane has issued the previous
    // tile's copies, whose source addresses are already in registers):
    // input origin and its byte offset.  Rows past M get an origin no tap
    // can bring inside the image.
    __syncwarp();
    {
      const int m = t.m_tile * kBlockM + row_base + lane;
      int4 e = make_int4(-(1 << 30), -(1 << 30), 0, 0);
      if (m < g.M) {
        const int img = m / g.PQ;
        const int rem = m - img * g.PQ;
        const int oy = rem / g.Q;
        const int ox = rem - oy * g.Q;
        const int iy0 = oy * g.stride_h - g.pad_h;
        const int ix0 = ox * g.stride_w - g.pad_w;
        const int64_t off = ((static_cast<int64_t>(img) * g.H + iy0) * g.W + ix0) * g.C;
        e = make_int4(iy0, ix0, static_cast<int>(off & 0xffffffffll), static_cast<int>(off >> 32));
      }
      mytab[lane] = e;
    }
    __syncwarp();
    int cb = 0, r = 0, s = 0, tap = 0;
    for (int kb = 0; kb < g.kblocks; ++kb) {
      if (!__all_sync(0xffffffffu,
                      mbar_wait(&b_empty[rb.stage], rb.phase ^ 1u, wctx, kStatusTimeoutEmpty))) {
        ok = false;
        break;
      }
      if (!ctl.starve) {
        if (loads_filter) {
          // Row k-blocks read the filter viewed as [K][R][S*C] (coordinate r),
          // tap k-blocks as [K][R*S][C] (coordinate tap).
          mbar_arrive_expect_tx(&b_full[rb.stage], plan.b_bytes);
          tma_load_3d(b_ring + rb.stage * plan.b_bytes, tmap_w, &b_full[rb.stage], cb * CBLK,
                      row_blocks ? r : tap, t.n0);
          ++armed_b;
        }
        const uint32_t a_base = smem_u32(a_ring + rb.stage * plan.a_bytes);
        const int dy = r * g.dil_h;
        int dx;
        bool c_ok;
        int64_t tap_off;
        if (row_blocks) {
          // Byte o of the filter row's S*C span: tap o / C, channel o % C (a
          // 16-byte chunk never straddles two taps: C % 16 == 0).
          const int o = cb * CBLK + chunk * 16;
          c_ok = o < g.S * g.C;
          dx = o / g.C;
          tap_off = static_cast<int64_t>(dy) * g.W * g.C + o;
        } else {
          dx = s * g.dil_w;
          const int c_off = cb * CBLK + chunk * 16;
          c_ok = c_off < g.C;
          tap_off = (static_cast<int64_t>(dy) * g.W + dx) * g.C + c_off;
        }
#pragma unroll
        for (int i = 0; i < kPasses; ++i) {
          const int row = row_base + rsub + i * kRowsPerPass;
          const int4 e = rowtab[row];
          const bool in = c_ok && static_cast<unsigned>(e.x + dy) < static_cast<unsigned>(g.H) &&
                          static_cast<unsigned>(e.y + dx) < static_cast<unsigned>(g.W);
          const int64_t off =
              (static_cast<int64_t>(e.w) << 32 | static_cast<uint32_t>(e.z)) + tap_off;
          const int8_t *src = in ? x + off : x;
          const uint32_t so = static_cast<uint32_t>(row * CBLK + chunk * 16);
          cp_async_16(a_base + (so ^ (((so >> 7) & kSwMask) << 4)), src, in ? 16u : 0u);
        }
        cp_async_commit();
        ++pending;
        if (pending > lag) {
          if (lag >= 3)
            cp_async_wait<3>();
          else if (lag == 2)
            cp_async_wait<2>();
          else
            cp_async_wait<1>();
          publish();
        }
      }
      rb.next(g.stages);
      if (++cb == g.cblocks) {
        cb = 0;
        if (row_blocks) {
          ++r;
        } else {
          ++tap;
          if (++s == g.S) {
            s = 0;
            ++r;
          }
        }
      }
    }
  }
  // Publish what is still in flight (also on the error path: the shared
  // memory must not be released under a pending copy).
  cp_async_wait<0>();
  while (pending > 0) publish();
  // The filter loads armed most recently land before the CTA exits.
  if (loads_filter) {
    for (long i = 0, n = armed_b < g.stages ? armed_b : g.stages; i < n; ++i) {
      rb.prev(g.stages);
      mbar_wait(&b_full[rb.stage], rb.phase, wctx, kStatusTimeoutTeardown);
    }
  }
}

// Requantisation of one thread's 32 accumulators (this warp's row, a
// 32-column block): four channels per word.  `table` holds the block's 32
// channel entries (rq_entry, bias included); every lane reads each entry with
// one broadcast load.  `lo` is the lower clamp (the zero point with ReLU,
// else -128).
// `slow`: some channel of the block needs the general path (decided once per
// block, so the common case is straight-line code).
__device__ __forceinline__ void requant_block(const uint32_t (&v)[32], const int4 *table,
                                              int32_t zero_point, int32_t lo, bool slow,
                                              uint32_t (&w8)[8]) {
  if (!slow) {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      int32_t y[4];
#pragma unroll
      for (int t = 0; t < 4; ++t)
        y[t] = rq_apply_fast(v[4 * j + t], table[4 * j + t], zero_point, lo);
      w8[j] = rq_pack4(y[0], y[1], y[2], y[3]);
    }
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      int32_t y[4];
#pragma unroll
      for (int t = 0; t < 4; ++t)
        y[t] = rq_apply_entry(v[4 * j + t], table[4 * j + t], zero_point, lo);
      w8[j] = rq_pack4(y[0], y[1], y[2], y[3]);
    }
  }
}

// Epilogue warps: 4 for int32 output (one per TMEM lane quarter); 16 for the
// requantised int8 output, whose per-element fixed-point arithmetic needs the
// issue slots (four warps per lane quarter, each owning every fourth
// 32-column block).  Eight int32 warps (two per quarter, one staging buffer
// each) were measured on B200 and dropped: 5a and 5c unchanged within 2 %,
// 3b 15.8 -> 17.7 us and the launch-bound shapes 0.4-0.7 us slower.
template <bool REQ>
constexpr int epilogue_warps() {
  return REQ ? 16 : 4;
}
// Threads of a launch: producer and MMA warps, the epilogue warps, and for
// the gather staging its three more gather warps (after the epilogue's).
template <int MODE, bool REQ>
constexpr int kernel_threads() {
  return 64 + 32 * epilogue_warps<REQ>() + (MODE == kModeGather ? 32 * (kGatherWarps - 1) : 0);
}

// Output tensor maps of a launch.  GENERIC and the gather staging: one map
// over NHWK viewed as [M][K], box 32 x 32.  STRIP with the int32 epilogue:
// maps of the same view with boxes of 32, 31, ... rows (ConvGeom::store_maps
// of them), one store per epilogue block of its valid rows, staged compactly.
constexpr int kMaxStoreMaps = 8;
struct alignas(64) StripOutMaps {
  CUtensorMap rows[kMaxStoreMaps];
};
template <int MODE, bool REQ>
struct OutMaps {
  using type = CUtensorMap;
};
template <>
struct OutMaps<kModeStrip, false> {
  using type = StripOutMaps;
};

template <int CBLK, int MODE, bool PAIR, bool REQ>
__global__ void __launch_bounds__(kernel_threads<MODE, REQ>(), 1)
    conv_kernel(const __grid_constant__ CUtensorMap tmap_x,
                const __grid_constant__ CUtensorMap tmap_w,
                const __grid_constant__ typename OutMaps<MODE, REQ>::type tmap_y,
                const ConvGeom g,
                const int8_t *__restrict__ x, const int32_t *__restrict__ bias,
                int32_t *__restrict__ out, const RunCtl ctl, const Requant rq) {
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte alignment: the SW128 atom (8 rows x 128 B) starts on it.  The
  // offset is the same in both CTAs of a pair (same kernel, same smem size).
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  constexpr int kTileRows = PAIR ? 2 * kBlockM : kBlockM;
  constexpr bool STRIP = MODE == kModeStrip;
  constexpr bool HALO = MODE == kModeHalo;
  constexpr bool SHIFT = STRIP || HALO;  // A operand = shifted views of one staged tile
  constexpr bool GATHER = MODE == kModeGather;
  static_assert(!(GATHER && PAIR), "the gather staging runs single CTAs");
  const int a_stages = SHIFT ? g.a_stages : g.stages;
  const int a_rows = SHIFT ? g.a_rows : kBlockM;
  const int b_rows = PAIR ? g.bn / 2 : g.bn;
  const SmemPlan plan = smem_plan(CBLK, b_rows, a_rows, a_stages, g.stages, GATHER);
  uint8_t *a_ring = smem + plan.a_off;
  uint8_t *b_ring = smem + plan.b_off;
  int4 *staging = reinterpret_cast<int4 *>(smem + plan.stage_off);
  uint64_t *a_full = reinterpret_cast<uint64_t *>(smem + plan.bar_off);
  uint64_t *a_empty = a_full + a_stages;
  uint64_t *b_full = a_empty + a_stages;
  uint64_t *b_empty = b_full + g.stages;
  uint64_t *tfull = b_empty + g.stages;
  uint64_t *tempty = tfull + 2;
  uint64_t *drain = tempty + 2;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const WaitCtx wctx{ctl.wait_ns, ctl.status};
  const int m_span = SHIFT ? g.PWp : g.PQ;     // positions per image
  const int m_row = SHIFT ? g.Wp : g.Q;        // positions per output row
  const uint32_t rank = PAIR ? cluster_ctarank() : 0u;
  const bool leader = rank == 0;
  const int tile_first = PAIR ? static_cast<int>(blockIdx.x >> 1) : static_cast<int>(blockIdx.x);
  const int tile_step = PAIR ? static_cast<int>(gridDim.x >> 1) : static_cast<int>(gridDim.x);

  if (warp == 0) {
    // The barriers are contiguous (a_full, a_empty, b_full, b_empty, tfull,
    // tempty, drain); lane i initialises barriers i, i + 32, ...  One thread
    // initialising all of them in sequence held up the first loads of the
    // small layers by about 0.3 us on B200.
    const int n_ab = 2 * a_stages + 2 * g.stages;
    for (int i = lane; i < n_ab + 5; i += 32) {
      uint32_t count = 1;
      // GATHER: the filter load's arrival plus one per gather lane.
      if (GATHER && i >= 2 * a_stages && i < 2 * a_stages + g.stages) count = 1 + 32 * kGatherWarps;
      // tempty: one arrival per epilogue warp (of both CTAs for a pair).
      if (i >= n_ab + 2 && i < n_ab + 4) count = (PAIR ? 2 : 1) * epilogue_warps<REQ>();
      mbar_init(&a_full[i], count);
    }
    fence_mbar_init();
    if (lane == 0) {
      if constexpr (!GATHER) tma_prefetch_desc(&tmap_x);
      tma_prefetch_desc(&tmap_w);
    }
  }
  if (warp == 1) {
    if constexpr (PAIR) {
      tmem_alloc_pair(tmem_slot, g.tmem_cols);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_slot, g.tmem_cols);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  __syncthreads();
  // A pair signals each other's barriers: both must be initialised first.
  if constexpr (PAIR) cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // Launched with programmatic stream serialisation: the set-up above may run
  // while the previous kernel in the stream finishes.  Each role that reads
  // or writes global memory (the producers, the epilogue warps) waits for
  // that kernel to complete before its first access (griddep_wait); the MMA
  // issuer touches only shared memory and TMEM.  The first epilogue warp lets
  // the next kernel's set-up start.

  constexpr int kFirstExtraGather = 2 + epilogue_warps<REQ>();
  if (GATHER && (warp == 0 || warp >= kFirstExtraGather)) {
    griddep_wait();
    gather_producer<CBLK>(g, x, &tmap_w, a_ring, b_ring, plan,
                          reinterpret_cast<int4 *>(smem + plan.rows_off), b_full, b_empty, ctl,
                          wctx, tile_first, tile_step,
                          warp == 0 ? 0 : warp - kFirstExtraGather + 1, lane);
  } else if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      griddep_wait();
      Ring ra, rb;
      long armed_a = 0, armed_b = 0;
      const uint32_t a_tx = (SHIFT ? g.strip_px : kBlockM) * CBLK;
      const uint32_t b_tx = plan.b_bytes;
      // A pair credits all bytes to the leader's barriers, armed for both CTAs.
      const uint32_t tx_mult = PAIR ? 2u : 1u;
      auto full_addr = [&](uint64_t *bar) -> uint32_t {
        return PAIR ? mapa_shared(smem_u32(bar), 0) : smem_u32(bar);
      };
      bool ok = true;
      for (int tile = tile_first; tile < g.num_units && ok; tile += tile_step) {
        const Unit t = unit_at(g, tile);
        const int m_tile = t.m_tile;
        const int m0 = m_tile * kTileRows + static_cast<int>(rank) * kBlockM;
        // Each CTA of a pair loads its half of the unit's filter rows (a box
        // of b_rows; a split unit uses the first bn/2 of them).
        const int n0 = t.n0 + static_cast<int>(rank) * (PAIR ? t.bn / 2 : 0);
        const int img = m0 / m_span;
        const int rem = m0 - img * m_span;
        const int p = rem / m_row;
        const int q = rem - p * m_row;
        const int x_w = q * g.stride_w - g.pad_w;
        const int x_h = p * g.stride_h - g.pad_h;
        if constexpr (SHIFT) {
          // STRIP: one staged row strip per (filter row r, channel block),
          //   shared by the S filter columns.
          // HALO: one staged halo tile per channel block, shared by all R*S taps.
          const int groups = STRIP ? g.R * g.cblocks : g.cblocks;
          const int taps = STRIP ? g.S : g.R * g.S;
          for (int grp = 0; grp < groups && ok; ++grp) {
            const int ra_row = STRIP ? grp / g.cblocks : 0;
            const int cb = STRIP ? grp - ra_row * g.cblocks : grp;
            if (!mbar_wait(&a_empty[ra.stage], ra.phase ^ 1u, wctx, kStatusTimeoutEmpty)) {
              ok = false;
              break;
            }
            if (!ctl.starve) {
              if (leader) {
                mbar_arrive_expect_tx(&a_full[ra.stage], tx_mult * a_tx);
                ++armed_a;
              }
              void *dst = a_ring + ra.stage * plan.a_bytes;
              const uint16_t oh = static_cast<uint16_t>(ra_row * g.dil_h);
              if constexpr (PAIR)
                tma_load_im2col_4d_pair(dst, &tmap_x, full_addr(&a_full[ra.stage]), cb * CBLK,
                                        x_w, x_h, img, 0, oh);
              else
                tma_load_im2col_4d(dst, &tmap_x, &a_full[ra.stage], cb * CBLK, x_w, x_h, img, 0,
                                   oh);
            }
            ra.next(a_stages);
            for (int t = 0; t < taps; ++t) {
              const int tap = STRIP ? ra_row * g.S + t : t;
              if (!mbar_wait(&b_empty[rb.stage], rb.phase ^ 1u, wctx, kStatusTimeoutEmpty)) {
                ok = false;
                break;
              }
              if (!ctl.starve) {
                if (leader) {
                  mbar_arrive_expect_tx(&b_full[rb.stage], tx_mult * b_tx);
                  ++armed_b;
                }
                void *dst = b_ring + rb.stage * plan.b_bytes;
                if constexpr (PAIR)
                  tma_load_3d_pair(dst, &tmap_w, full_addr(&b_full[rb.stage]), cb * CBLK, tap, n0);
                else
                  tma_load_3d(dst, &tmap_w, &b_full[rb.stage], cb * CBLK, tap, n0);
              }
              rb.next(g.stages);
            }
          }
        } else {
          int tap = 0, cb = 0, r = 0, s = 0;
          for (int kb = 0; kb < g.kblocks; ++kb) {
            if (!mbar_wait(&b_empty[rb.stage], rb.phase ^ 1u, wctx, kStatusTimeoutEmpty)) {
              ok = false;
              break;
            }
            if (!ctl.starve) {
              // A and B of one k-block share a stage index and one barrier.
              if (leader) {
                mbar_arrive_expect_tx(&b_full[rb.stage], tx_mult * (a_tx + b_tx));
                ++armed_b;
              }
              void *adst = a_ring + rb.stage * plan.a_bytes;
              void *bdst = b_ring + rb.stage * plan.b_bytes;
              const uint16_t ow = static_cast<uint16_t>(s * g.dil_w);
              const uint16_t oh = static_cast<uint16_t>(r * g.dil_h);
              if constexpr (PAIR) {
                const uint32_t bar = full_addr(&b_full[rb.stage]);
                tma_load_im2col_4d_pair(adst, &tmap_x, bar, cb * CBLK, x_w, x_h, img, ow, oh);
                tma_load_3d_pair(bdst, &tmap_w, bar, cb * CBLK, tap, n0);
              } else {
                tma_load_im2col_4d(adst, &tmap_x, &b_full[rb.stage], cb * CBLK, x_w, x_h, img,
                                   ow, oh);
                tma_load_3d(bdst, &tmap_w, &b_full[rb.stage], cb * CBLK, tap, n0);
              }
            }
            rb.next(g.stages);
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
      }
      // Copies still in flight must land before the CTA exits: wait for the
      // fills armed most recently (immediate on the normal path).  For a pair
      // the leader's barriers count both CTAs' copies.
      for (long i = 0, n = armed_b < g.stages ? armed_b : g.stages; i < n; ++i) {
        rb.prev(g.stages);
        mbar_wait(&b_full[rb.stage], rb.phase, wctx, kStatusTimeoutTeardown);
      }
      for (long i = 0, n = armed_a < a_stages ? armed_a : a_stages; i < n; ++i) {
        ra.prev(a_stages);
        mbar_wait(&a_full[ra.stage], ra.phase, wctx, kStatusTimeoutTeardown);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      // ---------------- MMA issuer (the leader of a pair) ----------------
      const uint32_t idesc_full = idesc_s8(kTileRows, g.bn);
      const uint32_t idesc_part = idesc_s8(kTileRows, g.bn / g.split_f);
      constexpr Layout kLayout = SwizzleOf<CBLK>::kLayout;
      constexpr uint32_t kAtom = 8 * CBLK;  // 8 rows x CBLK bytes
      // Shared-memory descriptors are built once: moving the operand start by
      // d bytes adds d >> 4 to the descriptor's 14-bit start-address field
      // (operand addresses stay below 256 KB, so nothing carries out of it).
      // One add per MMA instead of a full rebuild keeps the issuing thread
      // ahead of the tensor pipe (a rebuilt pair of descriptors cost the
      // thread about 70 cycles per 128-cycle MMA on B200).
      const uint64_t a_desc0 = smem_desc(smem_u32(a_ring), 16, kAtom, kLayout);
      const uint64_t b_desc0 = smem_desc(smem_u32(b_ring), 16, kAtom, kLayout);
      const uint32_t a_step = plan.a_bytes >> 4;
      const uint32_t b_step = plan.b_bytes >> 4;
      Ring ra, rb;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      uint32_t idesc = idesc_full;
      // A CTA with a single tile whose k-blocks (and staged A tiles) fit the
      // rings never refills a stage, so its MMAs release none (a commit costs
      // the issuing thread about as much as an MMA).
      const int a_used = STRIP ? g.R * g.cblocks : g.cblocks;
      const bool refill = tile_first + tile_step < g.num_units || g.kblocks > g.stages ||
                          (SHIFT && a_used > a_stages);
      auto mma = [&](uint32_t d, uint64_t a, uint64_t b, uint32_t accumulate) {
        if constexpr (PAIR)
          umma_i8_pair(d, a, b, idesc, accumulate);
        else
          umma_i8(d, a, b, idesc, accumulate);
      };
      for (int tile = tile_first; tile < g.num_units && ok; tile += tile_step) {
        idesc = tile >= g.split_from ? idesc_part : idesc_full;
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, wctx, kStatusTimeoutDrain)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * g.acc_stride);
        uint32_t accumulate = 0;
        if constexpr (SHIFT) {
          // One flat loop over the k-blocks in the producer's order: groups
          // (a staged tile each: filter row x channel block for a strip, a
          // channel block for a halo tile), then the taps that share it.  Tap
          // t reads the staged tile `shift` rows further on: filter column s
          // for a strip; r*dh*Wp + s*dw for a halo tile, kept incrementally.
          const int taps = STRIP ? g.S : g.R * g.S;
          const int row_step = g.dil_h * g.Wp;
          int t = 0, shift = 0, col = 0;
          uint64_t a_desc = a_desc0;
          for (int kb = 0; kb < g.kblocks; ++kb) {
            if (t == 0) {
              if (!mbar_wait(&a_full[ra.stage], ra.phase, wctx, kStatusTimeoutFull)) {
                ok = false;
                break;
              }
              a_desc = a_desc0 + ra.stage * a_step;
            }
            if (!mbar_wait(&b_full[rb.stage], rb.phase, wctx, kStatusTimeoutFull)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint64_t ad = a_desc + ((shift * CBLK) >> 4);
            const uint64_t bd = b_desc0 + rb.stage * b_step;
#pragma unroll
            for (int k = 0; k < CBLK / 32; ++k) {
              mma(d_tmem, ad + 2 * k, bd + 2 * k, accumulate);  // +32 bytes per MMA
              accumulate = 1;
            }
            if (refill) commit_to<PAIR>(&b_empty[rb.stage]);
            rb.next(g.stages);
            if (++t == taps) {
              t = shift = col = 0;
              if (refill) commit_to<PAIR>(&a_empty[ra.stage]);
              ra.next(a_stages);
            } else if (STRIP) {
              shift = t;
            } else if (++col == g.S) {
              col = 0;
              shift += row_step - (g.S - 1) * g.dil_w;
            } else {
              shift += g.dil_w;
            }
          }
        } else {
          for (int kb = 0; kb < g.kblocks; ++kb) {
            if (!mbar_wait(&b_full[rb.stage], rb.phase, wctx, kStatusTimeoutFull)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint64_t ad = a_desc0 + rb.stage * a_step;
            const uint64_t bd = b_desc0 + rb.stage * b_step;
#pragma unroll
            for (int k = 0; k < CBLK / 32; ++k) {
              mma(d_tmem, ad + 2 * k, bd + 2 * k, accumulate);  // +32 bytes per MMA
              accumulate = 1;
            }
            if (refill) commit_to<PAIR>(&b_empty[rb.stage]);
            rb.next(g.stages);
          }
        }
        if (!ok) break;
        commit_to<PAIR>(&tfull[acc]);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      // Every MMA issued must finish before TMEM is released (in both CTAs).
      commit_to<PAIR>(drain);
      mbar_wait(drain, 0, wctx, kStatusTimeoutTeardown);
    } else if (lane == 0 && PAIR) {
      // The peer's TMEM and shared memory stay in use until the leader's MMAs
      // are done; the leader's final commit arrives here too.
      mbar_wait(drain, 0, wctx, kStatusTimeoutTeardown);
    }
  } else if constexpr (REQ) {
    // ---------------- int8 epilogue (warps 2..17) ----------------
    griddep_wait();
    if (warp == 2) griddep_launch_dependents();
    constexpr int kGroups = epilogue_warps<REQ>() / 4;
    const int quarter = warp & 3;          // TMEM lane quarter this warp may access
    const int cgroup = (warp - 2) >> 2;    // 32-column blocks cgroup, cgroup + 4, ...
    const int row = quarter * 32 + lane;
    const int m_limit = SHIFT ? g.Mp : g.M;
    const uint32_t tempty_leader0 =
        PAIR ? mapa_shared(smem_u32(&tempty[0]), 0) : smem_u32(&tempty[0]);
    const uint32_t tempty_leader1 =
        PAIR ? mapa_shared(smem_u32(&tempty[1]), 0) : smem_u32(&tempty[1]);
    const int32_t lo = rq.relu ? rq.zero_point : -128;
    int8_t *out8 = reinterpret_cast<int8_t *>(out);
    // Per warp: one 32-row x 32-byte staging buffer (TMA store source) and
    // the channel tables of its (at most two: BN <= 256) 32-column blocks,
    // rebuilt only when the tile's N offset changes.
    uint8_t *stg_w = reinterpret_cast<uint8_t *>(staging) + (warp - 2) * 2048;
    int4 *tables = reinterpret_cast<int4 *>(stg_w + 1024);
    int table_n0 = -1, table_bn = 0;
    uint32_t slow_blocks = 0;  // bit b: block b has a slow-path channel
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = tile_first; tile < g.num_units; tile += tile_step) {
      const Unit t = unit_at(g, tile);
      const int m_tile = t.m_tile;
      const int pos = m_tile * kTileRows + static_cast<int>(rank) * kBlockM + row;
      const int n0 = t.n0;
      const int bn = t.bn;
      bool valid = pos < m_limit;
      int m = pos;
      if constexpr (SHIFT) {
        const int img = pos / g.PWp;
        const int rem = pos - img * g.PWp;
        const int i = rem / g.Wp;
        const int j = rem - i * g.Wp;
        valid = valid && j < g.Q && i < g.P;
        m = (img * g.P + i) * g.Q + j;
      }
      // Every warp, with or without a block of this tile, waits for the
      // accumulator, so all of them arrive on tempty once per tile.
      if (!__all_sync(0xffffffffu, mbar_wait(&tfull[acc], acc_phase, wctx, kStatusTimeoutAccum)))
        break;
      tc_fence_after();
      const uint32_t taddr =
          tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + acc * g.acc_stride;
      const int row0 = m_tile * kTileRows + static_cast<int>(rank) * kBlockM + quarter * 32;
      if (n0 != table_n0 || bn != table_bn) {
        // Lane l fills entry l of each block's table (zero past BN or K).
        __syncwarp();
        slow_blocks = 0;
        for (int b = 0, c0 = 32 * cgroup; c0 < bn; ++b, c0 += 32 * kGroups) {
          const int c = n0 + c0 + lane;
          const bool in = c0 + lane < bn && c < g.K;
          const int4 e =
              in ? rq_entry(__ldg(bias + c), __ldg(rq.multiplier + c), __ldg(rq.exponent + c))
                 : make_int4(0, 0, 0, 0);
          tables[b * 32 + lane] = e;
          if (__any_sync(0xffffffffu, (e.w >> 16) != 0)) slow_blocks |= 1u << b;
        }
        __syncwarp();
        table_n0 = n0;
        table_bn = bn;
      }
      bool released = false;
      auto release = [&] {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if constexpr (PAIR)
            mbar_arrive_cluster(acc ? tempty_leader1 : tempty_leader0);
          else
            mbar_arrive(&tempty[acc]);
        }
        released = true;
      };
      for (int b = 0, c0 = 32 * cgroup; c0 < bn; ++b, c0 += 32 * kGroups) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(taddr + c0, v);
        tmem_ld_wait();
        if (c0 + 32 * kGroups >= bn) release();  // this warp's last read of the tile
        const int col0 = n0 + c0;
        uint32_t w8[8];
        requant_block(v, tables + b * 32, rq.zero_point, lo, ((slow_blocks >> b) & 1u) != 0, w8);
        const int4 lo16 = make_int4(static_cast<int32_t>(w8[0]), static_cast<int32_t>(w8[1]),
                                    static_cast<int32_t>(w8[2]), static_cast<int32_t>(w8[3]));
        const int4 hi16 = make_int4(static_cast<int32_t>(w8[4]), static_cast<int32_t>(w8[5]),
                                    static_cast<int32_t>(w8[6]), static_cast<int32_t>(w8[7]));
        if (g.tma_store) {
          // 32 rows x 32 bytes leave as one TMA store (columns >= K, rows >= M
          // clipped); the previous block's store has read the buffer by now
          // (a whole block of arithmetic ago), the wait makes sure.
          int4 *stg = reinterpret_cast<int4 *>(stg_w);
          if (lane == 0) bulk_wait_group_read<0>();
          __syncwarp();
          stg[2 * lane] = lo16;
          stg[2 * lane + 1] = hi16;
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&tmap_y, stg, col0, row0);
            bulk_commit_group();
          }
        } else if (valid && col0 < g.K) {
          if (rq.layout == 1) {
            // NCHW_VECT_C: the block is one 32-channel vector of this pixel
            // (bn, K and col0 are multiples of 32); a warp writes 1 KB.
            const int img = m / g.PQ;
            const int pq = m - img * g.PQ;
            int4 *dst = reinterpret_cast<int4 *>(
                out8 + ((static_cast<int64_t>(img) * (g.K >> 5) + (col0 >> 5)) * g.PQ + pq) * 32);
            __stcs(dst, lo16);
            __stcs(dst + 1, hi16);
          } else {
            int8_t *dst = out8 + static_cast<int64_t>(m) * g.K + col0;
            const int span = bn - c0 < g.K - col0 ? bn - c0 : g.K - col0;
            if (span >= 32 && (g.K & 15) == 0) {
              __stcs(reinterpret_cast<int4 *>(dst), lo16);
              __stcs(reinterpret_cast<int4 *>(dst) + 1, hi16);
            } else {
#pragma unroll
              for (int t = 0; t < 32; ++t)
                if (t < span) dst[t] = static_cast<int8_t>((w8[t >> 2] >> (8 * (t & 3))) & 0xffu);
            }
          }
        }
      }
      if (!released) release();  // no block of this tile for this warp
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
    // Stores still reading shared memory finish before the CTA exits.
    if (g.tma_store && lane == 0) bulk_wait_group_read_all();
  } else {
    // ---------------- epilogue (warps 2..5) ----------------
    griddep_wait();
    if (warp == 2) griddep_launch_dependents();
    const int quarter = warp & 3;  // TMEM lane quarter this warp may access
    const int row = quarter * 32 + lane;
    const bool vec_k = (g.K & 3) == 0;
    const int m_limit = SHIFT ? g.Mp : g.M;
    const uint32_t tempty_leader0 =
        PAIR ? mapa_shared(smem_u32(&tempty[0]), 0) : smem_u32(&tempty[0]);
    const uint32_t tempty_leader1 =
        PAIR ? mapa_shared(smem_u32(&tempty[1]), 0) : smem_u32(&tempty[1]);
    int acc = 0;
    uint32_t acc_phase = 0;
    // The first tile's bias lines come into L1 while the mainloop runs.
    if (tile_first < g.num_units && lane < 8 && quarter == 0) {
      const Unit t = unit_at(g, tile_first);
      const int c = t.n0 + 32 * lane;
      if (32 * lane < t.bn && c < g.K) prefetch_l1(bias + c);
    }
    // Staging buffers alternate by a block counter that runs across tiles, so
    // consecutive stores never share a buffer even when BN/32 is odd.
    int ci = 0;
    for (int tile = tile_first; tile < g.num_units; tile += tile_step) {
      const Unit t = unit_at(g, tile);
      const int m_tile = t.m_tile;
      const int pos = m_tile * kTileRows + static_cast<int>(rank) * kBlockM + row;
      const int n0 = t.n0;
      const int bn = t.bn;
      bool valid = pos < m_limit;
      int m = pos;
      if constexpr (SHIFT) {
        // Padded-grid position (img, i, j): an output only for i < P, j < Q.
        const int img = pos / g.PWp;
        const int rem = pos - img * g.PWp;
        const int i = rem / g.Wp;
        const int j = rem - i * g.Wp;
        valid = valid && j < g.Q && i < g.P;
        m = (img * g.P + i) * g.Q + j;
      }
      // STRIP: this warp's 32 positions hold `strip_v` valid ones, which are
      // consecutive output pixels from `strip_m0` on (rows and images follow
      // each other in NHWK); lane l stages its row at `strip_d`, its rank
      // among the valid lanes, and the block leaves through map 32 - strip_v.
      int strip_v = 0, strip_d = 0, strip_m0 = 0;
      if constexpr (STRIP) {
        const uint32_t vmask = __ballot_sync(0xffffffffu, valid);
        strip_v = __popc(vmask);
        strip_d = __popc(vmask & ((1u << lane) - 1u));
        strip_m0 = __shfl_sync(0xffffffffu, m, vmask ? __ffs(static_cast<int>(vmask)) - 1 : 0);
      }
      const bool strip_tma = STRIP && g.tma_store && strip_v > 0 && 32 - strip_v < g.store_maps;
      // All lanes wait; the vote keeps the warp converged for tcgen05.ld even
      // if the wait runs out on some lanes only.
      if (!__all_sync(0xffffffffu, mbar_wait(&tfull[acc], acc_phase, wctx, kStatusTimeoutAccum)))
        break;
      tc_fence_after();
      const uint32_t taddr =
          tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + acc * g.acc_stride;
      // Each 32x32 int32 block (this warp's 32 rows x 32 columns) goes through
      // shared memory, swizzled by 16-byte chunk ^ (row & 7): the 128-byte TMA
      // swizzle.  Thread-per-row global stores would issue one L2 request per
      // 16 B; instead the block leaves as one TMA tensor store (rows >= M and
      // columns >= K clipped by the TMA unit), or, where that does not apply,
      // as 16-byte stores that write whole 128-byte row segments.
      int4 *stg_w = staging + (warp - 2) * 2 * 256;
      const int q = lane & 7;    // 16-byte column group this lane stores
      const int rsub = lane >> 3;
      const int row0 = m_tile * kTileRows + static_cast<int>(rank) * kBlockM + quarter * 32;
      for (int c0 = 0; c0 < bn; c0 += 32) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(taddr + c0, v);
        tmem_ld_wait();
        if (c0 + 32 >= bn) {
          // Last read of this accumulator: hand it back to the MMA issuer now.
          tc_fence_before();
          __syncwarp();
          if (lane == 0) {
            if constexpr (PAIR)
              mbar_arrive_cluster(acc ? tempty_leader1 : tempty_leader0);
            else
              mbar_arrive(&tempty[acc]);
          }
        }
        const int col0 = n0 + c0;
        if constexpr (STRIP) {
          if (strip_tma) {
            int4 *stg = stg_w + (ci & 1) * 256;
            // The store issued two blocks ago read this buffer: let it finish.
            if (lane == 0) bulk_wait_group_read<1>();
            __syncwarp();
            if (valid) {
#pragma unroll
              for (int j = 0; j < 8; ++j) {
                const bool in = c0 + 4 * j < bn && col0 + 4 * j < g.K;
                const int4 bb = in ? __ldg(reinterpret_cast<const int4 *>(bias + col0) + j)
                                   : make_int4(0, 0, 0, 0);
                stg[strip_d * 8 + (j ^ (strip_d & 7))] = make_int4(
                    static_cast<int32_t>(v[4 * j]) + bb.x, static_cast<int32_t>(v[4 * j + 1]) + bb.y,
                    static_cast<int32_t>(v[4 * j + 2]) + bb.z,
                    static_cast<int32_t>(v[4 * j + 3]) + bb.w);
              }
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              tma_store_2d(&tmap_y.rows[32 - strip_v], stg, col0, strip_m0);
              bulk_commit_group();
            }
            ++ci;
            continue;
          }
          // 16-byte stores through buffer 0: earlier TMA stores must have
          // read it.
          if (g.tma_store) {
            if (lane == 0) bulk_wait_group_read<0>();
            __syncwarp();
          }
        } else {
          if (g.tma_store) {
            int4 *stg = stg_w + (ci & 1) * 256;
            // The store issued two blocks ago read this buffer: let it finish.
            if (lane == 0) bulk_wait_group_read<1>();
            __syncwarp();
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const bool in = c0 + 4 * j < bn && col0 + 4 * j < g.K;
              const int4 bb = in ? __ldg(reinterpret_cast<const int4 *>(bias + col0) + j)
                                 : make_int4(0, 0, 0, 0);
              stg[lane * 8 + (j ^ (lane & 7))] = make_int4(
                  static_cast<int32_t>(v[4 * j]) + bb.x, static_cast<int32_t>(v[4 * j + 1]) + bb.y,
                  static_cast<int32_t>(v[4 * j + 2]) + bb.z,
                  static_cast<int32_t>(v[4 * j + 3]) + bb.w);
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              tma_store_2d(&tmap_y, stg, col0, row0);
              bulk_commit_group();
            }
            ++ci;
            continue;
          }
        }
        int4 *stg = stg_w;
#pragma unroll
        for (int j = 0; j < 8; ++j)
          stg[lane * 8 + (j ^ (lane & 7))] =
              make_int4(static_cast<int32_t>(v[4 * j]), static_cast<int32_t>(v[4 * j + 1]),
                        static_cast<int32_t>(v[4 * j + 2]), static_cast<int32_t>(v[4 * j + 3]));
        __syncwarp();
        if (vec_k) {
          // K % 4 == 0: 16-byte groups are wholly inside or outside [0, K).
          const bool col_ok = c0 + 4 * q < bn && col0 + 4 * q < g.K;
          const int4 bb = col_ok ? __ldg(reinterpret_cast<const int4 *>(bias + col0) + q)
                                 : make_int4(0, 0, 0, 0);
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int r = 4 * i + rsub;
            const int mr = __shfl_sync(0xffffffffu, m, r);
            const bool vr = __shfl_sync(0xffffffffu, valid ? 1 : 0, r) != 0;
            if (vr && col_ok) {
              int4 o = stg[r * 8 + (q ^ (r & 7))];
              o.x += bb.x;
              o.y += bb.y;
              o.z += bb.z;
              o.w += bb.w;
              __stcs(reinterpret_cast<int4 *>(out + static_cast<int64_t>(mr) * g.K + col0) + q, o);
            }
          }
        } else {
          const bool col_ok = c0 + lane < bn && col0 + lane < g.K;
          const int32_t bl = col_ok ? __ldg(bias + col0 + lane) : 0;
          const int32_t *stg32 = reinterpret_cast<const int32_t *>(stg);
          for (int r = 0; r < 32; ++r) {
            const int mr = __shfl_sync(0xffffffffu, m, r);
            const bool vr = __shfl_sync(0xffffffffu, valid ? 1 : 0, r) != 0;
            if (vr && col_ok)
              out[static_cast<int64_t>(mr) * g.K + col0 + lane] =
                  stg32[(r * 8 + ((lane >> 2) ^ (r & 7))) * 4 + (lane & 3)] + bl;
          }
        }
        __syncwarp();
      }
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
    // Stores still reading shared memory finish before the CTA exits.
    if (g.tma_store && lane == 0) bulk_wait_group_read_all();
  }

  tc_fence_before();
  __syncthreads();
  // Neither CTA of a pair leaves while the other may still touch its shared
  // memory (remote barrier arrivals, MMA operand reads).
  if constexpr (PAIR) cluster_sync_all();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    if constexpr (PAIR)
      tmem_dealloc_pair(tmem_base, g.tmem_cols);
    else
      tmem_dealloc(tmem_base, g.tmem_cols);
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------

static int pick_cblk(int c) { return i8c_channel_block(c); }

// `align` = 16, or 32 when every 32-column block must hold whole
// 32-channel vectors (NCHW_VECT_C output).

// Output of a launch: the int32 contract or one of the int8 layouts.
constexpr int kOutInt32 = 0;
constexpr int kOutInt8Nhwc = 1;
constexpr int kOutInt8VectC = 2;

static int next_pow2(int v) {
  int p = 32;
  while (p < v) p <<= 1;
  return p;
}

// Fills the launch geometry; false if the shape does not fit the kernel.
// `slots` = tiles the grid runs at once (CTA pairs or single CTAs).
static bool plan_geometry(const int8conv_shape &s, int mode, bool pair, int out_kind, int slots,
                          ConvGeom &g, int &cblk) {
  const int32_t out_h = (s.h + 2 * s.pad_h - s.dilation_h * (s.r - 1) - 1) / s.stride_h + 1;
  const int32_t out_w = (s.w + 2 * s.pad_w - s.dilation_w * (s.s - 1) - 1) / s.stride_w + 1;
  cblk = pick_cblk(s.c);
  g = ConvGeom{};
  const bool gemm_rows = mode == kModeGeneric || mode == kModeGather;  // A rows = output pixels
  g.M = s.n * out_h * out_w;
  g.K = s.k;
  g.H = s.h;
  g.W = s.w;
  g.C = s.c;
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
  // The gather with unit horizontal dilation may take 128-byte k-blocks of a
  // filter row's S*C contiguous bytes: a small C no longer pays one k-block
  // (and its zero padding) per tap.  Taken where it stages no more bytes than
  // per-tap blocks do.  ViT-B/16 with C = 16: 32 k-blocks of 128 bytes per
  // tile instead of 256 of 32 (half of them zero).
  g.row_blocks = 0;
  const int64_t row_padded = static_cast<int64_t>(s.r) * ((s.s * s.c + 127) / 128) * 128;
  const int64_t tap_padded = static_cast<int64_t>(g.kblocks) * cblk;
  if (mode == kModeGather && s.dilation_w == 1 && row_padded <= tap_padded) {
    cblk = 128;
    g.row_blocks = 1;
    g.cblocks = (s.s * s.c + 127) / 128;
    g.kblocks = s.r * g.cblocks;
  }
  // Single CTAs may run narrower N tiles (i8c_narrow_bn) over their row
  // tiles: output pixels (GENERIC), or positions of the padded grid (STRIP:
  // out_h x Wp per image; HALO: Hp x Wp).
  const int bn_align = out_kind == kOutInt8VectC ? 32 : 16;
  if (pair) {
    g.bn = i8c_pick_bn(s.k, bn_align);
  } else if (gemm_rows) {
    g.bn = i8c_generic_bn(&s, bn_align, slots);
  } else {
    const int64_t wp = out_w + static_cast<int64_t>(s.s - 1) * s.dilation_w;
    const int64_t hp = mode == kModeHalo ? out_h + static_cast<int64_t>(s.r - 1) * s.dilation_h
                                         : out_h;
    g.bn = i8c_narrow_bn(s.k, bn_align, (s.n * hp * wp + kBlockM - 1) / kBlockM, slots);
  }
  g.pair = pair ? 1 : 0;
  g.acc_stride = (g.bn + 31) / 32 * 32;
  g.tmem_cols = next_pow2(2 * g.acc_stride);
  if (g.tmem_cols > 512) return false;
  const int tile_rows = pair ? 2 * kBlockM : kBlockM;
  const int b_bytes = (pair ? g.bn / 2 : g.bn) * cblk;
  // Shared memory left for the rings: minus the base alignment slack (1 KB),
  // the staging buffer and its 1 KB alignment, and the barriers.
  const int budget = kMaxSmem - 2048 - 512 - static_cast<int>(kEpilogueStaging) -
                     (mode == kModeGather ? static_cast<int>(kGatherRowTable) + 16 : 0);
  int64_t positions = g.M;
  if (!gemm_rows) {
    // Padded grid: STRIP pads the row only (Wp = Q + S - 1, out_h rows);
    // HALO pads both (Hp x Wp, every tap is a shift of one staged tile).
    const bool halo = mode == kModeHalo;
    g.Wp = out_w + (s.s - 1) * s.dilation_w;
    g.rows = halo ? out_h + (s.r - 1) * s.dilation_h : out_h;
    g.PWp = g.rows * g.Wp;
    positions = static_cast<int64_t>(s.n) * g.PWp;
    if (positions >= (int64_t(1) << 31) - 512) return false;  // int32 row index + one tile
    g.Mp = static_cast<int32_t>(positions);
    const int64_t shift = halo ? static_cast<int64_t>(s.r - 1) * s.dilation_h * g.Wp +
                                     static_cast<int64_t>(s.s - 1) * s.dilation_w
                               : s.s - 1;
    if (kBlockM + shift > kMaxStagedRows) return false;
    g.strip_px = static_cast<int32_t>(kBlockM + shift);
    g.a_rows = (g.strip_px + 7) / 8 * 8;
    const int a_bytes = g.a_rows * cblk;
    // Ring of staged tiles: enough to keep the taps that share one flowing.
    g.a_stages = 3;
    int b_stages = (budget - g.a_stages * a_bytes) / b_bytes;
    if (b_stages > 12) b_stages = 12;
    if (b_stages < 2) {
      g.a_stages = 2;
      b_stages = (budget - g.a_stages * a_bytes) / b_bytes;
      if (b_stages > 12) b_stages = 12;
    }
    if (b_stages < 2) return false;
    g.stages = b_stages;
  } else {
    const int per_stage = kBlockM * cblk + b_bytes;
    int stages = budget / per_stage;
    if (stages > 12) stages = 12;
    if (stages < 2) return false;
    g.stages = stages;
    g.a_stages = stages;
    g.a_rows = kBlockM;
    g.gather_lag = stages - 1 < 3 ? stages - 1 : 3;
  }
  g.m_tiles = static_cast<int32_t>((positions + tile_rows - 1) / tile_rows);
  g.n_tiles = (s.k + g.bn - 1) / g.bn;
  g.num_tiles = g.m_tiles * g.n_tiles;
  // Tail balancing (i8c_pick_split): the last partial wave's tiles become f
  // column parts each.
  g.split_from = g.num_tiles;
  g.split_f = 1;
  g.num_units = g.num_tiles;
  const int best_f = i8c_pick_split(g.num_tiles, slots, g.bn);
  if (best_f > 1) {
    const int rem = g.num_tiles % slots;
    g.split_f = best_f;
    g.split_from = g.num_tiles - rem;
    g.num_units = g.split_from + best_f * rem;
  }
  // TMA output stores: GENERIC rows are contiguous in NHWK; the row pitch
  // 4*K must be a multiple of 16 bytes; a 32-column block must not reach into
  // the next N tile (columns >= K are clipped, columns of a neighbour are not).
  // int8 NHWC: rows of K bytes (K % 16 == 0), 32-column blocks.
  if (out_kind == kOutInt32)
    g.tma_store = gemm_rows && s.k % 4 == 0 && (g.bn % 32 == 0 || g.n_tiles == 1);
  else if (out_kind == kOutInt8Nhwc)
    g.tma_store = gemm_rows && s.k % 16 == 0 && (g.bn % 32 == 0 || g.n_tiles == 1);
  else
    g.tma_store = 0;
  // STRIP, int32: every epilogue block (32 positions from a multiple of 32)
  // drops the padded positions j >= out_w it holds; its valid ones are
  // consecutive output pixels.  One map per possible count of dropped
  // positions, if there are at most kMaxStoreMaps of them.
  g.store_maps = 0;
  if (mode == kModeStrip && out_kind == kOutInt32 && s.k % 4 == 0 &&
      (g.bn % 32 == 0 || g.n_tiles == 1)) {
    // Every padded row ends in a run of Wp - Q dropped positions.  With at
    // least 32 valid positions between runs a block meets one run at most;
    // otherwise (short rows) count over the Wp block starts, which repeat.
    const int run = g.Wp - g.Q;
    int most = 0;
    if (g.Q >= 32) {
      most = run < 32 ? run : 32;
    } else {
      for (int t = 0; t < g.Wp; ++t) {
        int dropped = 0;
        for (int r = 0; r < 32; ++r) dropped += (32 * t + r) % g.Wp >= g.Q ? 1 : 0;
        if (dropped > most) most = dropped;
      }
    }
    if (most + 1 <= kMaxStoreMaps) {
      g.store_maps = most + 1;
      g.tma_store = 1;
    }
  }
  return true;
}

template <int CBLK, int MODE, bool PAIR, bool REQ>
static int8conv_status launch_t(const int8conv_shape &s, const ConvGeom &g, const int8_t *x,
                                const int8_t *w, const int32_t *b, void *y, const Requant &rq,
                                cudaStream_t stream) {
  DeviceInfo &dev = device_info();
  CUtensorMap maps[3];
  constexpr bool SHIFT = MODE == kModeStrip || MODE == kModeHalo;
  constexpr bool GATHER = MODE == kModeGather;
  const int pixels = SHIFT ? g.strip_px : kBlockM;
  const int count_w = SHIFT ? g.Wp : g.Q;
  const int count_h = MODE == kModeHalo ? g.rows : g.P;
  const int b_rows = PAIR ? g.bn / 2 : g.bn;
  int8conv_status st = INT8CONV_OK;
  maps[0] = CUtensorMap{};  // GATHER reads the activations through `x`
  if (!GATHER) {
    st = activation_map_im2col(s, x, CBLK, pixels, count_w, count_h, &maps[0]);
    if (st != INT8CONV_OK) return st;
  }
  st = g.row_blocks ? filter_map_rows(s, w, CBLK, b_rows, &maps[1])
                    : filter_map_tiled(s, w, CBLK, b_rows, &maps[1]);
  if (st != INT8CONV_OK) return st;
  maps[2] = CUtensorMap{};
  typename OutMaps<MODE, REQ>::type out_maps{};
  if constexpr (MODE == kModeStrip && !REQ) {
    for (int i = 0; i < g.store_maps; ++i) {
      st = output_map_rows(static_cast<int32_t *>(y), g.M, g.K, 32 - i, &out_maps.rows[i]);
      if (st != INT8CONV_OK) return st;
    }
  } else {
    if (g.tma_store) {
      st = REQ ? output_map_i8(static_cast<int8_t *>(y), g.M, g.K, &maps[2])
               : output_map_tiled(static_cast<int32_t *>(y), g.M, g.K, &maps[2]);
      if (st != INT8CONV_OK) return st;
    }
    out_maps = maps[2];
  }
  const SmemPlan plan =
      smem_plan(CBLK, b_rows, SHIFT ? g.a_rows : kBlockM, g.a_stages, g.stages, GATHER);
  auto kernel = conv_kernel<CBLK, MODE, PAIR, REQ>;
  // At least half an SM's shared memory: one CTA per SM, so a CTA never waits
  // for another's TMEM columns.
  const uint32_t smem_bytes = plan.total > kOneCtaPerSm ? plan.total : kOneCtaPerSm;
  // The opt-in shared-memory limit is set once per device and instantiation.
  static std::atomic<uint32_t> smem_set[64];
  std::atomic<uint32_t> &slot = smem_set[dev.device & 63];
  if (slot.load(std::memory_order_relaxed) < smem_bytes) {
    if (!ensure_smem_attr(reinterpret_cast<const void *>(kernel), kMaxSmem))
      return INT8CONV_CUDA_ERROR;
    slot.store(kMaxSmem, std::memory_order_relaxed);
  }
  const int ctas = PAIR ? 2 * (g.num_units < dev.sm_count / 2 ? g.num_units : dev.sm_count / 2)
                        : (g.num_units < dev.sm_count ? g.num_units : dev.sm_count);
  LaunchPlan lp;
  lp.func = reinterpret_cast<const void *>(kernel);
  lp.grid = dim3(ctas, 1, 1);
  lp.block = dim3(kernel_threads<MODE, REQ>(), 1, 1);
  lp.smem = smem_bytes;
  lp.cluster = PAIR ? 2 : 1;
  plan_args(lp, maps[0], maps[1], out_maps, g, x, b, static_cast<int32_t *>(y), run_ctl(), rq);
  return launch_plan(lp, stream);
}

template <int MODE, bool PAIR, bool REQ>
static int8conv_status launch_cblk(const int8conv_shape &s, const ConvGeom &g, int cblk,
                                   const int8_t *x, const int8_t *w, const int32_t *b, void *y,
                                   const Requant &rq, cudaStream_t stream) {
  switch (cblk) {
    case 128:
      return launch_t<128, MODE, PAIR, REQ>(s, g, x, w, b, y, rq, stream);
    case 64:
      return launch_t<64, MODE, PAIR, REQ>(s, g, x, w, b, y, rq, stream);
    default:
      return launch_t<32, MODE, PAIR, REQ>(s, g, x, w, b, y, rq, stream);
  }
}

// CTA pairs halve the filter bytes per output row.  Measured on B200 they pay
// off when the filter tile is at least 192 columns, there is at least one wave
// of 256-row tiles, and either the reduction is deep (R*S*C >= 1024: 5a 354 vs
// 401 us, 5b 92 vs 102 us, 5c with 192 columns 35.2 vs 36.6 us) or there are
// many waves (big_1x1_s1, 4096 tiles: 262 vs 266 us).  Narrower, shallower or
// smaller layers run faster as single CTAs (3b: 17 vs 23 us,
// nonmultiple8_k255: 61 vs 65 us, batch16 bottleneck expand: 24 vs 27 us).
static bool use_pair(const int8conv_shape &s, int mode, int out_kind) {
  const int pairing = pairing_mode();
  if (pairing == 1 || mode == kModeGather) return false;  // the gather warp feeds one CTA
  ConvGeom g;
  int cblk = 0;
  if (!plan_geometry(s, mode, true, out_kind, device_info().sm_count / 2, g, cblk)) return false;
  if (pairing == 2) return true;
  const int64_t reduction = static_cast<int64_t>(s.r) * s.s * s.c;
  return g.bn >= 192 && g.num_tiles >= device_info().sm_count &&
         (reduction >= 1024 || g.num_tiles >= 1024);
}

template <int MODE, bool REQ>
static int8conv_status launch_mode(const int8conv_shape &s, const int8_t *x, const int8_t *w,
                                   const int32_t *b, void *y, const Requant &rq, int out_kind,
                                   cudaStream_t stream) {
  ConvGeom g;
  int cblk = 0;
  const int sms = device_info().sm_count;
  if constexpr (MODE != kModeGather) {
    if (use_pair(s, MODE, out_kind)) {
      if (!plan_geometry(s, MODE, true, out_kind, sms / 2, g, cblk)) return INT8CONV_NOT_ELIGIBLE;
      return launch_cblk<MODE, true, REQ>(s, g, cblk, x, w, b, y, rq, stream);
    }
  }
  if (!plan_geometry(s, MODE, false, out_kind, sms, g, cblk)) return INT8CONV_NOT_ELIGIBLE;
  return launch_cblk<MODE, false, REQ>(s, g, cblk, x, w, b, y, rq, stream);
}

// GENERIC stages the activations through the im2col tensor map where it can
// be encoded, else with the gather warp (same tiles, same MMA and epilogue).
int8conv_status launch_generic_impl(const int8conv_shape &s, const int8_t *x, const int8_t *w,
                                    const int32_t *b, int32_t *y, cudaStream_t stream) {
  if (!i8c_im2col_ok(&s) || staging_mode() == 1)
    return launch_mode<kModeGather, false>(s, x, w, b, y, Requant{}, kOutInt32, stream);
  return launch_mode<kModeGeneric, false>(s, x, w, b, y, Requant{}, kOutInt32, stream);
}

int8conv_status launch_strip_impl(const int8conv_shape &s, const int8_t *x, const int8_t *w,
                                  const int32_t *b, int32_t *y, cudaStream_t stream) {
  return launch_mode<kModeStrip, false>(s, x, w, b, y, Requant{}, kOutInt32, stream);
}

int8conv_status launch_halo_impl(const int8conv_shape &s, const int8_t *x, const int8_t *w,
                                 const int32_t *b, int32_t *y, cudaStream_t stream) {
  return launch_mode<kModeHalo, false>(s, x, w, b, y, Requant{}, kOutInt32, stream);
}

int8conv_status launch_conv_requant(int strategy, const int8conv_shape &s, const int8_t *x,
                                    const int8_t *w, const int32_t *b, const Requant &rq,
                                    int8_t *y, cudaStream_t stream) {
  const int out_kind = rq.layout == 1 ? kOutInt8VectC : kOutInt8Nhwc;
  switch (strategy) {
    case INT8CONV_GENERIC:
      if (!i8c_im2col_ok(&s) || staging_mode() == 1)
        return launch_mode<kModeGather, true>(s, x, w, b, y, rq, out_kind, stream);
      return launch_mode<kModeGeneric, true>(s, x, w, b, y, rq, out_kind, stream);
    case INT8CONV_STRIP:
      return launch_mode<kModeStrip, true>(s, x, w, b, y, rq, out_kind, stream);
    case INT8CONV_HALO:
      return launch_mode<kModeHalo, true>(s, x, w, b, y, rq, out_kind, stream);
    default:
      return INT8CONV_NOT_ELIGIBLE;
  }
}

}  // namespace i8c
