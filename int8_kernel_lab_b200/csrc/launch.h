// launch.h - host-side services shared by the kernel families: per-device
// properties, TMA tensor-map encoding (with a small cache), the device status
// word and the failure-detection controls.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include <type_traits>

#include "conv_common.h"
#include "int8conv.h"
#include "requant.cuh"

namespace i8c {

struct DeviceInfo {
  int device = -1;
  int sm_count = 0;
  int cc_major = 0, cc_minor = 0;
  uint32_t *status = nullptr;   // address of the module's __device__ status word
};

// Properties of the calling thread's current device (cached per device).
DeviceInfo &device_info();

// INT8CONV_OK when the current device is an sm_100 part.
int8conv_status check_device();

// Run controls for the next launch: status word, wait limit, starve hook.
RunCtl run_ctl();

void note_launch();

// CTA pairing policy: 0 auto, 1 single CTAs only, 2 pairs whenever possible.
int pairing_mode();

// GENERIC activation staging: 0 auto (im2col map where encodable), 1 gather.
int staging_mode();

// Sets the dynamic shared-memory limit of `kernel` once per device.
bool ensure_smem_attr(const void *kernel, int bytes);

// im2col tensor map over the NHWC activations: `channels` bytes per pixel
// (swizzle = channels bytes), `pixels` traversal positions per load, and a
// bounding box per image holding `count_w` positions per row (out_w for
// GENERIC, the padded width for STRIP/HALO) and `count_h` rows (out_h, or the
// padded height for HALO), starting at (-pad_w, -pad_h).
int8conv_status activation_map_im2col(const int8conv_shape &s, const int8_t *x, int channels,
                                      int pixels, int count_w, int count_h, CUtensorMap *map);

// Tiled tensor map over the KRSC filter viewed as [K][R*S][C], box
// (channels, 1, rows).
int8conv_status filter_map_tiled(const int8conv_shape &s, const int8_t *w, int channels,
                                 int rows, CUtensorMap *map);

// Tiled tensor map over the KRSC filter viewed as [K][R][S*C] (each filter
// row's S*C bytes contiguous), box (channels, 1, rows): the gather staging's
// row k-blocks.
int8conv_status filter_map_rows(const int8conv_shape &s, const int8_t *w, int channels, int rows,
                                CUtensorMap *map);

// Tiled tensor map over the NHWK int32 output viewed as [M][K], box 32 x 32,
// 128-byte swizzle (the epilogue's staging layout).
int8conv_status output_map_tiled(int32_t *y, int64_t m, int k, CUtensorMap *map);

// The same view with a box of 32 columns x `rows` rows (1..32), 128-byte
// swizzle: STRIP's stores of a block's valid rows, staged compactly.
int8conv_status output_map_rows(int32_t *y, int64_t m, int k, int rows, CUtensorMap *map);

// Tiled tensor map over the NHWC int8 requantised output viewed as [M][K]
// (K % 16 == 0), box 32 x 32, no swizzle: one epilogue warp's 32 rows x 32
// columns per store.
int8conv_status output_map_i8(int8_t *y, int64_t m, int k, CUtensorMap *map);

// Requantised-output variants of the family launchers (`rq` non-null; `y`
// int8 in rq->layout).
int8conv_status launch_conv_requant(int strategy, const int8conv_shape &s, const int8_t *x,
                                    const int8_t *w, const int32_t *b, const Requant &rq,
                                    int8_t *y, cudaStream_t stream);
int8conv_status launch_splitk_requant(const int8conv_shape &s, const int8_t *x, const int8_t *w,
                                      const int32_t *b, const Requant &rq, int8_t *y,
                                      cudaStream_t stream);

// A fully planned launch: kernel, grid, shared memory, cluster size and the
// kernel's argument block (tensor maps, geometry, pointers), so a repeated
// launch of the same shape on the same buffers skips planning and descriptor
// encoding.  The run controls (status word, wait limit, starve hook) are
// refreshed from the current settings at every launch.
struct LaunchPlan {
  const void *func = nullptr;
  dim3 grid, block;
  uint32_t smem = 0;
  uint32_t cluster = 1;                 // thread-block cluster size (x)
  int nargs = 0;
  uint16_t offset[12] = {};             // argument k lives at blob + offset[k]
  int ctl_arg = -1;                     // index of the RunCtl argument
  alignas(64) unsigned char blob[2048];  // argument values, kernel-parameter aligned
};

// Bytes the kernel arguments take when packed with their alignments.
template <class... Args>
constexpr size_t packed_args_size() {
  size_t at = 0;
  ((at = (at + alignof(Args) - 1) / alignof(Args) * alignof(Args) + sizeof(Args)), ...);
  return at;
}

// Packs typed kernel arguments into plan->blob (their types must be the
// kernel's parameter types, in order).
template <class... Args>
void plan_args(LaunchPlan &plan, const Args &...args) {
  static_assert(packed_args_size<std::decay_t<Args>...>() <= sizeof(LaunchPlan::blob),
                "kernel arguments exceed the plan's argument block");
  size_t at = 0;
  plan.nargs = 0;
  auto put = [&](const auto &a) {
    using T = std::decay_t<decltype(a)>;
    at = (at + alignof(T) - 1) / alignof(T) * alignof(T);
    memcpy(plan.blob + at, &a, sizeof(T));
    if (std::is_same<T, RunCtl>::value) plan.ctl_arg = plan.nargs;
    plan.offset[plan.nargs++] = static_cast<uint16_t>(at);
    at += sizeof(T);
  };
  (put(args), ...);
}

// Launches a plan on `stream` with programmatic stream serialisation (and the
// plan's cluster size); records it for the calling thread's plan cache when a
// capture is active.
int8conv_status launch_plan(LaunchPlan &plan, cudaStream_t stream);

// Plan capture around one family launch: the family launcher hands its plan
// to launch_plan, which copies it to `*out` when capture is on for this thread.
void plan_capture_begin(LaunchPlan *out);
void plan_capture_end();

// Family launchers (valid, eligible shape; pointers already checked).
int8conv_status launch_generic_impl(const int8conv_shape &s, const int8_t *x, const int8_t *w,
                                    const int32_t *b, int32_t *y, cudaStream_t stream);
int8conv_status launch_strip_impl(const int8conv_shape &s, const int8_t *x, const int8_t *w,
                                  const int32_t *b, int32_t *y, cudaStream_t stream);
int8conv_status launch_host_pipeline(int strategy, const int8conv_shape &s, const int8_t *hx,
                                     const int8_t *hw, const int32_t *hb, int32_t *hy,
                                     int8_t *dx, int8_t *dw, int32_t *db, int32_t *dy,
                                     int chunks, cudaStream_t stream);
int8conv_status launch_halo_impl(const int8conv_shape &s, const int8_t *x, const int8_t *w,
                                 const int32_t *b, int32_t *y, cudaStream_t stream);
int8conv_status launch_splitk_impl(const int8conv_shape &s, const int8_t *x, const int8_t *w,
                                   const int32_t *b, int32_t *y, cudaStream_t stream);

}  // namespace i8c
