/*
 * int8conv_rules.h - shape algebra and per-family capability predicates.
 *
 * Header-only and dependency-free so the same rules are evaluated by the C ABI
 * (runtime), the C++ drop-in header (compile time, constexpr) and the tests.
 *
 * Shape formulas follow include/conv_shape.cuh:22-35 of the reference exactly,
 * including C++ integer division (truncation toward zero) in out_h/out_w.
 */
#ifndef INT8CONV_RULES_H_
#define INT8CONV_RULES_H_

#include <stdint.h>

#include "int8conv.h"

#ifdef __cplusplus
#define I8C_RULE constexpr inline
#else
#define I8C_RULE static inline
#endif

/* TMA limits of the activation im2col tensor map.  They bound the im2col
 * bounding-box corners ([-128,127] for a 4-D tensor map), the im2col tap
 * offsets and the traversal strides (1..8).  Shapes beyond them run GENERIC's
 * gather staging instead (i8c_im2col_ok). */
#define I8C_MAX_PAD 127
#define I8C_MAX_TAP_SPAN 127
#define I8C_MAX_STRIDE 8
#define I8C_MAX_DIM (1 << 24)

/* conv_shape.cuh:22-23 */
I8C_RULE int32_t i8c_out_h(const int8conv_shape *s) {
  return (s->h + 2 * s->pad_h - s->dilation_h * (s->r - 1) - 1) / s->stride_h + 1;
}
/* conv_shape.cuh:24-25 */
I8C_RULE int32_t i8c_out_w(const int8conv_shape *s) {
  return (s->w + 2 * s->pad_w - s->dilation_w * (s->s - 1) - 1) / s->stride_w + 1;
}

/* conv_shape.cuh:34-35 plus range checks the template got for free. */
I8C_RULE int i8c_shape_valid(const int8conv_shape *s) {
  return s != 0 && s->n > 0 && s->h > 0 && s->w > 0 && s->c > 0 && s->k > 0 &&
         s->r > 0 && s->s > 0 && s->pad_h >= 0 && s->pad_w >= 0 &&
         s->stride_h > 0 && s->stride_w > 0 && s->dilation_h > 0 &&
         s->dilation_w > 0 && s->n <= I8C_MAX_DIM && s->h <= I8C_MAX_DIM &&
         s->w <= I8C_MAX_DIM && s->c <= I8C_MAX_DIM && s->k <= I8C_MAX_DIM &&
         s->r <= 4096 && s->s <= 4096 && s->pad_h <= I8C_MAX_DIM &&
         s->pad_w <= I8C_MAX_DIM && s->stride_h <= I8C_MAX_DIM &&
         s->stride_w <= I8C_MAX_DIM && s->dilation_h <= 4096 &&
         s->dilation_w <= 4096 &&
         /* conv_shape.cuh:34 */ s->c % 16 == 0 &&
         /* conv_shape.cuh:35 */ i8c_out_h(s) > 0 && i8c_out_w(s) > 0 &&
         /* The kernels' int32 row index runs up to one 256-row tile past the
          * last output row, and the NHWC pixel index stays inside int32. */
         (int64_t)s->n * i8c_out_h(s) * i8c_out_w(s) < ((int64_t)1 << 31) - 512 &&
         (int64_t)s->n * s->h * s->w < ((int64_t)1 << 31);
}

/* Upper corner of the im2col bounding box along one spatial dimension such
 * that the box holds exactly `count` traversal positions starting at -pad. */
I8C_RULE int32_t i8c_upper_corner(int32_t extent, int32_t pad, int32_t stride,
                                  int32_t count) {
  return -pad + (count - 1) * stride + 1 - extent;
}

I8C_RULE int i8c_corner_ok(int32_t v) { return v >= -128 && v <= 127; }

/* 1 if the activations of the shape can be staged through a TMA im2col tensor
 * map (GENERIC's fast staging; required by STRIP, HALO and SPLITK). */
I8C_RULE int i8c_im2col_ok(const int8conv_shape *s) {
  return i8c_shape_valid(s) && s->pad_h <= I8C_MAX_PAD && s->pad_w <= I8C_MAX_PAD &&
         s->stride_h <= I8C_MAX_STRIDE && s->stride_w <= I8C_MAX_STRIDE &&
         (int64_t)(s->r - 1) * s->dilation_h <= I8C_MAX_TAP_SPAN &&
         (int64_t)(s->s - 1) * s->dilation_w <= I8C_MAX_TAP_SPAN &&
         i8c_corner_ok(i8c_upper_corner(s->w, s->pad_w, s->stride_w, i8c_out_w(s))) &&
         i8c_corner_ok(i8c_upper_corner(s->h, s->pad_h, s->stride_h, i8c_out_h(s)));
}

/* GENERIC: every valid shape, like the reference's generic family
 * (generic_implicit_gemm.cuh, whose gather at :46-69 handles any stride, pad
 * and dilation; conv_shape.cuh:34-35 are its only conditions).  Shapes the
 * im2col map cannot encode are staged by a gather warp instead of TMA. */
I8C_RULE int i8c_generic_eligible(const int8conv_shape *s) { return i8c_shape_valid(s); }

/* STRIP: one TMA-loaded row strip of (128 + S - 1) padded-row pixels is
 * reused across the S filter columns.  Needs unit horizontal stride and
 * dilation (the reference's own conditions, spatial_strip.cuh:11-15) and
 * 2 <= S <= 16.  Every shape the reference's predicate accepts is accepted
 * here; out_w % 128 and the r == 3 restriction are dropped because the B200
 * kernel tiles the padded row instead of whole 128-pixel output rows. */
I8C_RULE int i8c_strip_eligible(const int8conv_shape *s) {
  return i8c_im2col_ok(s) && s->stride_w == 1 && s->dilation_w == 1 &&
         s->s >= 2 && s->s <= 16 &&
         i8c_corner_ok(i8c_upper_corner(s->w, s->pad_w, 1, i8c_out_w(s) + s->s - 1));
}

/* Channel block (bytes of C per k-block, one swizzle width: 128, 64 or 32)
 * the kernels use for a shape.  Each k-block costs its CBLK bytes of MMA work
 * plus a fixed cost worth about 128 bytes (a pipeline round trip and one
 * im2col request per pixel); channels past C in the last block are
 * zero-filled by TMA.  The cheapest block wins, ties going to the one with
 * less zero padding (C = 48 -> 64, C = 96 -> 128, C = 160 or 192 -> 128,
 * C % 128 == 0 -> 128).  Measured on B200 for C = 192 (BASELINE 5c): two
 * 128-byte blocks, one of them half padding, beat three 64-byte blocks
 * (36.4 vs 38.8 us per launch). */
I8C_RULE int32_t i8c_channel_block(int32_t c) {
  int32_t best = 32;
  int64_t best_cost = -1, best_pad = 0;
  for (int32_t cb = 128; cb >= 32; cb /= 2) {
    const int64_t blocks = (c + cb - 1) / cb;
    const int64_t cost = blocks * (cb + 128);
    const int64_t pad = blocks * cb - c;
    if (best_cost < 0 || cost < best_cost || (cost == best_cost && pad < best_pad)) {
      best = cb;
      best_cost = cost;
      best_pad = pad;
    }
  }
  return best;
}

/* SPLITK: the R*S*C reduction of each output tile is split across the CTAs
 * of a cluster, so there must be at least two k-blocks (tap x channel block)
 * to split.  Activations come through the im2col map. */
I8C_RULE int i8c_splitk_eligible(const int8conv_shape *s) {
  return i8c_im2col_ok(s) &&
         (int64_t)s->r * s->s * ((s->c + i8c_channel_block(s->c) - 1) / i8c_channel_block(s->c)) >= 2;
}

/* Thread-block clusters that can be resident at once on a B200 (148 SMs), by
 * cluster size 0..8, with one CTA per SM (every kernel here asks for at least
 * half an SM's shared memory).  Measured with cudaOccupancyMaxActiveClusters;
 * GPC boundaries make the larger sizes lose SMs (8 x 15 = 120 of 148). */
#define I8C_B200_CLUSTERS {0, 148, 74, 45, 33, 26, 22, 15, 15}

/* SPLITK cluster size for `tiles` output tiles and `kblocks` k-blocks: the
 * largest split in [2, min(8, kblocks)] whose clusters all fit in one wave
 * (tiles <= clusters[split]); 0 if none does.  `clusters` is indexed by
 * cluster size, like I8C_B200_CLUSTERS. */
I8C_RULE int32_t i8c_split_count(int64_t tiles, int64_t kblocks, const int32_t *clusters) {
  for (int32_t split = kblocks < 8 ? (int32_t)kblocks : 8; split >= 2; --split)
    if (tiles <= clusters[split]) return split;
  return 0;
}

/* Output tiles of the SPLITK kernel: 128 rows x BN columns, BN <= 128. */
I8C_RULE int64_t i8c_split_tiles(const int8conv_shape *s) {
  const int64_t m = (int64_t)s->n * i8c_out_h(s) * i8c_out_w(s);
  return (m + 127) / 128 * ((s->k + 127) / 128);
}

/* GENERIC's N-tile width: K itself up to 256 (rounded up to `align`), else
 * the narrowest multiple of `align` that cuts K into ceil(K/256) equal tiles. */
I8C_RULE int32_t i8c_pick_bn(int32_t k, int32_t align) {
  if (k <= 256) return (k + align - 1) / align * align;
  const int32_t tiles = (k + 255) / 256;
  const int32_t per = (k + tiles - 1) / tiles;
  return (per + align - 1) / align * align;
}

/* Tail balancing of the persistent GENERIC/STRIP/HALO grid: with `slots`
 * tiles running at once, the last wave is partial when num_tiles % slots !=
 * 0.  Cutting each tile of that wave into f column parts (N = bn/f, 32-column
 * aligned for the stores) spreads it over more slots.  A part still loads its
 * tile's whole activation block and filter box, so it costs about 1/f + 0.2
 * of a tile (B200 sweep of all 51 workloads: parts in several waves, e.g. 98
 * tiles on 148 CTAs as 392 quarters, were slower).  Spans are in 1/20 tile.
 * Returns the f in {1, 2, 4} with the shortest span; bn = 0 skips the rule
 * that bn be a multiple of 32 f. */
I8C_RULE int32_t i8c_pick_split(int64_t num_tiles, int32_t slots, int32_t bn) {
  if (slots <= 0) return 1;
  const int64_t waves = num_tiles / slots;
  const int64_t rem = num_tiles - waves * slots;
  int32_t best_f = 1;
  int64_t best_span = 20 * waves + (rem > 0 ? 20 : 0);
  for (int32_t f = 2; f <= 4 && rem > 0; f *= 2) {
    if (bn != 0 && bn % (32 * f) != 0) continue;
    const int64_t span = 20 * waves + ((f * rem + slots - 1) / slots) * (20 / f + 4);
    if (span < best_span) {
      best_span = span;
      best_f = f;
    }
  }
  return best_f;
}

/* N-tile width for single CTAs with `slots` of them resident, over `m_tiles`
 * 128-row tiles.  A layer whose tiles fill less than one wave, and whose
 * width is not a multiple of 64 (so tail balancing cannot cut it into column
 * parts), runs narrower N tiles instead, as many as the span model asks for.
 * A narrow tile loads only its own filter rows, while each column part of a
 * wide tile would load the whole filter box (B200, K = 100 on 25 row tiles:
 * four 32-column tiles 13.4-14.1 us per launch against 16.2 us for one
 * 112-column tile and 16.2 us for four parts of a 128-column tile). */
I8C_RULE int32_t i8c_narrow_bn(int32_t k, int32_t align, int64_t m_tiles, int32_t slots) {
  int32_t bn = i8c_pick_bn(k, align);
  const int64_t tiles = m_tiles * ((k + bn - 1) / bn);
  if (slots > 0 && tiles < slots && i8c_pick_split(tiles, slots, bn) == 1) {
    const int32_t f = i8c_pick_split(tiles, slots, 0);
    if (f > 1) {
      int32_t narrow = ((bn + f - 1) / f + 31) / 32 * 32;
      if (narrow < 32) narrow = 32;
      if (narrow < bn) bn = narrow;
    }
  }
  return bn;
}

/* GENERIC's N-tile width for single CTAs: its rows are the output pixels. */
I8C_RULE int32_t i8c_generic_bn(const int8conv_shape *s, int32_t align, int32_t slots) {
  const int64_t m_tiles = ((int64_t)s->n * i8c_out_h(s) * i8c_out_w(s) + 127) / 128;
  return i8c_narrow_bn(s->k, align, m_tiles, slots);
}

/* HALO: positions run over the zero-padded image (Hp x Wp, Hp = out_h +
 * (R-1)*dh, Wp = out_w + (S-1)*dw); one staged halo tile of
 * 128 + (R-1)*dh*Wp + (S-1)*dw pixels per channel block feeds all R*S taps.
 * Needs unit strides and a staged tile of at most 512 pixels (small spatial
 * layers). */
I8C_RULE int i8c_halo_eligible(const int8conv_shape *s) {
  return i8c_im2col_ok(s) && s->stride_h == 1 && s->stride_w == 1 &&
         128 + (int64_t)(s->r - 1) * s->dilation_h *
                   (i8c_out_w(s) + (int64_t)(s->s - 1) * s->dilation_w) +
                 (int64_t)(s->s - 1) * s->dilation_w <= 512 &&
         i8c_corner_ok(i8c_upper_corner(s->w, s->pad_w, 1,
                                        i8c_out_w(s) + (s->s - 1) * s->dilation_w)) &&
         i8c_corner_ok(i8c_upper_corner(s->h, s->pad_h, 1,
                                        i8c_out_h(s) + (s->r - 1) * s->dilation_h));
}

I8C_RULE int i8c_eligible(const int8conv_shape *s, int strategy) {
  return strategy == INT8CONV_GENERIC   ? i8c_generic_eligible(s)
         : strategy == INT8CONV_STRIP   ? i8c_strip_eligible(s)
         : strategy == INT8CONV_HALO    ? i8c_halo_eligible(s)
         : strategy == INT8CONV_SPLITK  ? i8c_splitk_eligible(s)
                                        : 0;
}

#undef I8C_RULE
#endif /* INT8CONV_RULES_H_ */
