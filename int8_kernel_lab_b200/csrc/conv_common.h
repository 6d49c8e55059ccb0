// conv_common.h - host/device types shared by the kernel families.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "int8conv.h"

namespace i8c {

// Geometry of one launch, in GEMM terms (M = output pixels, N = output
// channels, reduction = R*S taps x channel blocks).  Derived on the host from
// int8conv_shape with the formulas of the reference's conv_shape.cuh:22-28.
struct ConvGeom {
  int32_t M;         // n * out_h * out_w
  int32_t K;         // output channels (GEMM N)
  int32_t H, W, C;   // input height, width, channels (gather staging)
  int32_t P, Q;      // out_h, out_w
  int32_t PQ;        // out_h * out_w
  int32_t R, S;
  int32_t pad_h, pad_w;
  int32_t stride_h, stride_w;
  int32_t dil_h, dil_w;
  int32_t cblocks;   // channel blocks per tap
  int32_t kblocks;   // R * S * cblocks
  int32_t bn;        // CTA tile width in output channels (multiple of 16, <= 256)
  int32_t acc_stride;// TMEM columns between the two accumulator buffers
  int32_t tmem_cols; // TMEM columns allocated (power of two)
  int32_t pair;      // 1: cta_group::2 CTA pairs, 256-row tiles
  int32_t tma_store; // 1: epilogue writes 32x32 blocks with TMA tensor stores
  int32_t stages;    // shared-memory ring depth (B ring; also A for GENERIC)
  int32_t m_tiles, n_tiles, num_tiles;
  // Tail balancing: tiles [split_from, num_tiles) (the last, partial wave)
  // are each cut into split_f column parts of bn / split_f, so that wave
  // finishes sooner; work units are the whole tiles before split_from, then
  // the parts.  split_f = 1 and num_units = num_tiles when nothing is cut.
  int32_t split_from, split_f, num_units;
  // STRIP / HALO: the M dimension runs over padded-grid positions
  // (n, i, j), j in [0, Wp), i in [0, rows); positions with j >= out_w or
  // i >= out_h are computed and discarded.
  int32_t Wp;        // padded row width
  int32_t rows;      // padded-grid rows per image (out_h for STRIP, Hp for HALO)
  int32_t PWp;       // rows * Wp
  int32_t Mp;        // n * out_h * Wp
  int32_t strip_px;  // pixels per staged load (128 + largest tap shift)
  int32_t a_rows;    // rows reserved per staged tile (strip_px rounded up to 8)
  int32_t a_stages;  // staged-tile ring depth
  // GATHER: k-blocks whose copies may still be in flight when the next one
  // is issued (1..3, fewer than `stages`).
  int32_t gather_lag;
  // GATHER with unit horizontal dilation: a k-block is 128 contiguous bytes
  // of one filter row's S*C span (several taps of a small C at once) instead
  // of one tap's channel block; `cblocks` = ceil(S*C / 128) per filter row.
  int32_t row_blocks;
  // STRIP with TMA output stores: the number of output tensor maps, map i
  // with a box of 32 - i rows.  An epilogue block of 32 padded positions
  // holds 32 - i valid ones (consecutive output pixels); staged compactly,
  // they leave as one store through map i.  Blocks with fewer valid
  // positions (the grid's tail) use 16-byte stores.
  int32_t store_maps;
};

// Failure-detection controls passed to every kernel.
struct RunCtl {
  uint32_t *status;     // device status word (bit set on a wait timeout)
  uint64_t wait_ns;     // per-wait limit
  uint32_t starve;      // test hook: producer issues no copies
};

constexpr int kBlockM = 128;         // MMA M (rows = output pixels)
constexpr int kSplitThreads = 192;   // 6 warps (SPLITK kernel)
constexpr int kMaxSmem = 232448;     // 227 KB opt-in limit per block on sm_100

}  // namespace i8c
