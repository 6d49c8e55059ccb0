// requant.cuh - int32 accumulator -> int8 output (requantised epilogue).
//
// The int32 result of a launch (accumulator + bias, the reference's output
// contract) is scaled to int8 per output channel k with integer-only fixed
// point, the scheme of gemmlowp / TensorFlow Lite ("quantized multiplier":
// a Q31 multiplier and a power-of-two exponent, SaturatingRoundingDoublingHighMul
// followed by RoundingDivideByPOT):
//
//   t = acc + bias[k]                      two's-complement wrap (as the int32 output)
//   e = clamp(exponent[k], -31, 31)
//   t = e > 0 ? saturate_int32(t * 2^e) : t
//   u = srdhm(t, multiplier[k])            (t * multiplier + nudge) / 2^31, truncating
//                                          division, nudge = +2^30 or 1 - 2^30 by sign;
//                                          INT32_MIN * INT32_MIN saturates to INT32_MAX
//   v = e < 0 ? rdbpot(u, -e) : u          u / 2^-e rounded half away from zero
//   y = clamp(v + zero_point, relu ? zero_point : -128, 127)
//
// multiplier 2^30 with exponent 1 is the plain saturating cast
// y = clamp(acc + bias, -128, 127): cuDNN's INT8x32 output with alpha = 1,
// beta = 0 (the reference's cuDNN comparison, include/cudnn_legacy.cuh:51-55).
#pragma once

#include <stdint.h>

namespace i8c {

// Requantised-output parameters of one launch (device pointers, K entries).
struct Requant {
  const int32_t *multiplier;
  const int32_t *exponent;
  int32_t zero_point;
  int32_t relu;     // 1: clamp below at zero_point
  int32_t layout;   // 0: NHWC int8 [M][K]; 1: NCHW_VECT_C int8x32 [N][K/32][P][Q][32]
};

__host__ __device__ __forceinline__ int32_t rq_srdhm(int32_t a, int32_t b) {
  if (a == INT32_MIN && b == INT32_MIN) return INT32_MAX;
  const int64_t ab = static_cast<int64_t>(a) * static_cast<int64_t>(b);
  const int64_t t = ab + (ab >= 0 ? (int64_t(1) << 30) : (int64_t(1) - (int64_t(1) << 30)));
  // Division by 2^31 truncating toward zero (|t| < 2^63, so -t is exact).
  const int64_t q = t >= 0 ? (t >> 31) : -((-t) >> 31);
  return static_cast<int32_t>(q);
}

__host__ __device__ __forceinline__ int32_t rq_rdbpot(int32_t x, int e) {
  const int32_t mask = static_cast<int32_t>((uint32_t(1) << e) - 1u);
  const int32_t rem = x & mask;
  const int32_t threshold = (mask >> 1) + (x < 0 ? 1 : 0);
  return (x >> e) + (rem > threshold ? 1 : 0);
}

// One output value; `t` is the int32 accumulator plus bias.
__host__ __device__ __forceinline__ int32_t rq_apply(int32_t t, int32_t multiplier,
                                                     int32_t exponent, int32_t zero_point,
                                                     bool relu) {
  const int e = exponent < -31 ? -31 : (exponent > 31 ? 31 : exponent);
  if (e > 0) {
    const int64_t s = static_cast<int64_t>(t) * (int64_t(1) << e);
    t = s > INT32_MAX ? INT32_MAX : (s < INT32_MIN ? INT32_MIN : static_cast<int32_t>(s));
  }
  int32_t v = rq_srdhm(t, multiplier);
  if (e < 0) v = rq_rdbpot(v, -e);
  int64_t y = static_cast<int64_t>(v) + zero_point;
  const int64_t lo = relu ? zero_point : -128;
  if (y < lo) y = lo;
  if (y > 127) y = 127;
  return static_cast<int32_t>(y);
}

#ifdef __CUDACC__
// Device form of rq_apply for one output channel's parameters, which are the
// same for every lane of a warp (lanes are pixels, the loop runs over
// channels), so the rare cases (left shift, INT32_MIN multiplier, no right
// shift) are uniform branches.  Same results as rq_apply for every input.
struct RqChannel {
  int32_t multiplier;
  int32_t left;       // exponent > 0: left shift
  int32_t right;      // exponent < 0: right shift
  int32_t mask;       // 2^right - 1
};

__device__ __forceinline__ RqChannel rq_channel(int32_t multiplier, int32_t exponent) {
  const int e = exponent < -31 ? -31 : (exponent > 31 ? 31 : exponent);
  RqChannel c;
  c.multiplier = multiplier;
  c.left = e > 0 ? e : 0;
  c.right = e < 0 ? -e : 0;
  c.mask = static_cast<int32_t>((uint32_t(1) << c.right) - 1u);
  return c;
}

// `lo` = the lower clamp: zero_point with ReLU, else -128.
__device__ __forceinline__ int32_t rq_apply_dev(int32_t t, const RqChannel &c, int32_t zero_point,
                                                int32_t lo) {
  if (c.left > 0) {
    const int64_t s = static_cast<int64_t>(t) * (int64_t(1) << c.left);
    t = s > INT32_MAX ? INT32_MAX : (s < INT32_MIN ? INT32_MIN : static_cast<int32_t>(s));
  }
  // The doubling high multiply.  For ab = t * multiplier, the nudge-then-
  // truncate form equals floor((ab + 2^30) / 2^31) for every ab (ab < 0,
  // ab = -(k*2^31 + r): both give -k - [r > 2^30]), so one 64-bit add and an
  // arithmetic shift suffice; only INT32_MIN * INT32_MIN saturates.
  int32_t v;
  if (c.multiplier == INT32_MIN && t == INT32_MIN)
    v = INT32_MAX;
  else
    v = static_cast<int32_t>((static_cast<int64_t>(t) * c.multiplier + (int64_t(1) << 30)) >> 31);
  if (c.right > 0) {
    const int32_t rem = v & c.mask;
    const int32_t threshold = (c.mask >> 1) + (v < 0 ? 1 : 0);
    v = (v >> c.right) + (rem > threshold ? 1 : 0);
  }
  // |v| is clamped first so that adding the zero point cannot overflow; the
  // final clamp makes the result the same.
  v = v < -4096 ? -4096 : (v > 4096 ? 4096 : v);
  v += zero_point;
  v = v < lo ? lo : v;
  return v > 127 ? 127 : v;
}
#endif

#ifdef __CUDACC__
// One channel's parameters as the int8 epilogue keeps them in shared memory:
// {bias, multiplier, mask = 2^right - 1, right | left << 8 | slow << 16};
// slow marks the rare channels that need rq_apply_dev's general path (a left
// shift, or the INT32_MIN multiplier).
__device__ __forceinline__ int4 rq_entry(int32_t bias, int32_t multiplier, int32_t exponent) {
  const RqChannel c = rq_channel(multiplier, exponent);
  const int32_t slow = (c.left > 0 || multiplier == INT32_MIN) ? 1 : 0;
  return make_int4(bias, multiplier, c.mask, c.right | (c.left << 8) | (slow << 16));
}

__device__ __forceinline__ int32_t rq_sat_add(int32_t a, int32_t b) {
  int32_t r;
  asm("add.sat.s32 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

// rq_apply_dev on an accumulator and its channel's entry (bias not yet
// added), for entries without the slow flag: straight-line code, so a block
// of them interleaves freely.
__device__ __forceinline__ int32_t rq_apply_fast(uint32_t acc, const int4 &e, int32_t zero_point,
                                                 int32_t lo) {
  const int32_t t = static_cast<int32_t>(acc + static_cast<uint32_t>(e.x));
  int32_t v = static_cast<int32_t>((static_cast<int64_t>(t) * e.y + (int64_t(1) << 30)) >> 31);
  // Rounding divide by 2^right (right = 0: mask 0, v unchanged).
  const int32_t rem = v & e.z;
  const int32_t threshold = (e.z >> 1) + (v < 0 ? 1 : 0);
  v = (v >> (e.w & 0xff)) + (rem > threshold ? 1 : 0);
  v = rq_sat_add(v, zero_point);
  v = v < lo ? lo : v;
  return v > 127 ? 127 : v;
}

// Any entry: the general path for slow-flagged channels.
__device__ __forceinline__ int32_t rq_apply_entry(uint32_t acc, const int4 &e, int32_t zero_point,
                                                  int32_t lo) {
  if (e.w >> 16) {
    RqChannel c;
    c.multiplier = e.y;
    c.right = e.w & 0xff;
    c.left = (e.w >> 8) & 0xff;
    c.mask = e.z;
    return rq_apply_dev(static_cast<int32_t>(acc + static_cast<uint32_t>(e.x)), c, zero_point, lo);
  }
  return rq_apply_fast(acc, e, zero_point, lo);
}
#endif

// Four consecutive channels packed little-endian into one word.
__host__ __device__ __forceinline__ uint32_t rq_pack4(int32_t a, int32_t b, int32_t c, int32_t d) {
  return (static_cast<uint32_t>(a) & 0xffu) | ((static_cast<uint32_t>(b) & 0xffu) << 8) |
         ((static_cast<uint32_t>(c) & 0xffu) << 16) | ((static_cast<uint32_t>(d) & 0xffu) << 24);
}

}  // namespace i8c
