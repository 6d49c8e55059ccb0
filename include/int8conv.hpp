// int8conv.hpp - C++ drop-in for the reference's header-only launchers.
//
// A caller of pthodima/int8_kernel_lab includes this header instead of
// include/conv_shape.cuh, include/generic_implicit_gemm.cuh and
// include/spatial_strip.cuh, links libint8conv.so, and keeps its call sites:
//
//   using Shape = ConvShape<N, H, W, C, K, R, S, PH, PW, SH, SW, DH, DW>;   // conv_shape.cuh:5-36
//   launch_generic<Shape>(input, filter, bias, output, stream);            // generic_implicit_gemm.cuh:155-165
//   launch_generic_sm80<Shape>(input, filter, bias, output, stream);       // generic_implicit_gemm.cuh:229-238
//   if constexpr (kSpatialStripEligible<Shape>)                            // spatial_strip.cuh:11-15
//     launch_spatial_strip<Shape>(input, filter, bias, output, stream);   // spatial_strip.cuh:289-301
//
// Differences, all documented in the C header:
//   * the launchers return int8conv_status (void call sites still compile);
//     kernel launch errors also surface through cudaGetLastError() as before;
//   * kSpatialStripEligible is the B200 strip kernel's predicate, a superset
//     of the reference's (every shape the reference accepted stays eligible);
//   * launch_spatial_strip keeps the compile-time static_assert on
//     eligibility, like the reference.
#ifndef INT8CONV_HPP_
#define INT8CONV_HPP_

#include <cuda_runtime.h>

#include <cstddef>

#include "int8conv.h"
#include "int8conv_rules.h"

template <int Batch, int Height, int Width, int Channels, int Filters, int FilterH, int FilterW,
          int PadH, int PadW, int StrideH, int StrideW, int DilationH, int DilationW>
struct ConvShape {
  static constexpr int n = Batch;
  static constexpr int h = Height;
  static constexpr int w = Width;
  static constexpr int c = Channels;
  static constexpr int k = Filters;
  static constexpr int r = FilterH;
  static constexpr int s = FilterW;
  static constexpr int pad_h = PadH;
  static constexpr int pad_w = PadW;
  static constexpr int stride_h = StrideH;
  static constexpr int stride_w = StrideW;
  static constexpr int dilation_h = DilationH;
  static constexpr int dilation_w = DilationW;
  static constexpr int out_h = (h + 2 * pad_h - dilation_h * (r - 1) - 1) / stride_h + 1;
  static constexpr int out_w = (w + 2 * pad_w - dilation_w * (s - 1) - 1) / stride_w + 1;
  static constexpr int gemm_m = n * out_h * out_w;
  static constexpr int gemm_n = k;
  static constexpr int gemm_k = r * s * c;
  static constexpr size_t input_elements = static_cast<size_t>(n) * h * w * c;
  static constexpr size_t filter_elements = static_cast<size_t>(k) * r * s * c;
  static constexpr size_t output_elements = static_cast<size_t>(gemm_m) * gemm_n;

  static constexpr int8conv_shape runtime() {
    return int8conv_shape{n, h, w, c, k, r, s, pad_h, pad_w, stride_h, stride_w,
                          dilation_h, dilation_w};
  }

  static_assert(c % 16 == 0, "input channels must be divisible by 16");
  static_assert(out_h > 0 && out_w > 0, "output must be nonempty");
};

namespace int8conv_detail {
template <class Shape>
constexpr bool strip_eligible() {
  constexpr int8conv_shape shape = Shape::runtime();
  return i8c_strip_eligible(&shape) != 0;
}
template <class Shape>
constexpr bool generic_eligible() {
  constexpr int8conv_shape shape = Shape::runtime();
  return i8c_generic_eligible(&shape) != 0;
}
}  // namespace int8conv_detail

template <class Shape>
inline constexpr bool kSpatialStripEligible = int8conv_detail::strip_eligible<Shape>();

template <class Shape>
inline int8conv_status launch_generic(const int8_t *input, const int8_t *filter,
                                      const int32_t *bias, int32_t *output,
                                      cudaStream_t stream = 0) {
  // Every shape ConvShape accepts (c % 16 == 0, non-empty output) with its
  // fields in the engine's ranges; stride, pad and dilation are unbounded
  // within them, as in the reference's generic launcher.
  static_assert(int8conv_detail::generic_eligible<Shape>(),
                "shape fields out of the generic kernel's range");
  constexpr int8conv_shape shape = Shape::runtime();
  return int8conv_launch_generic(&shape, input, filter, bias, output, stream);
}

// The reference's SM80 (m16n8k32) generic launcher; one B200 kernel serves both.
template <class Shape>
inline int8conv_status launch_generic_sm80(const int8_t *input, const int8_t *filter,
                                           const int32_t *bias, int32_t *output,
                                           cudaStream_t stream = 0) {
  return launch_generic<Shape>(input, filter, bias, output, stream);
}

template <class Shape>
inline int8conv_status launch_spatial_strip(const int8_t *input, const int8_t *filter,
                                            const int32_t *bias, int32_t *output,
                                            cudaStream_t stream = 0) {
  static_assert(kSpatialStripEligible<Shape>, "shape is not eligible for spatial strip");
  constexpr int8conv_shape shape = Shape::runtime();
  return int8conv_launch_spatial_strip(&shape, input, filter, bias, output, stream);
}

#endif  // INT8CONV_HPP_
