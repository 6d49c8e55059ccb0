// abi.cu - the extern "C" boundary declared in include/int8conv.h.
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include <atomic>

#include "int8conv.h"
#include "int8conv_rules.h"
#include "launch.h"

namespace i8c {
extern std::atomic<uint64_t> g_wait_limit_ns;
extern std::atomic<uint32_t> g_starve;
extern std::atomic<uint64_t> g_launches;
extern std::atomic<int> g_pairing;
extern std::atomic<int> g_staging;
}  // namespace i8c

namespace {

bool aligned16(const void *p) { return p != nullptr && (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// Per-thread cache of launch plans.  A launch whose device, family, shape,
// buffers, CTA pairing and epilogue match an earlier launch on this thread
// replays that plan (kernel, grid, tensor maps, geometry) instead of planning
// and encoding descriptors again.  Thread-local, so no locking; a plan only
// depends on the key's fields (the tensor maps hold the buffer addresses).
struct PlanKey {
  int32_t device, strategy, pairing, staging, out_kind;
  int8conv_shape shape;
  int32_t zero_point, relu;
  const void *x, *w, *b, *y, *multiplier, *exponent;
};
struct PlanSlot {
  PlanKey key;
  i8c::LaunchPlan plan;
  bool used = false;
};
constexpr int kPlanSlots = 32;
thread_local PlanSlot t_plans[kPlanSlots];

PlanKey plan_key(int strategy, const int8conv_shape &s, const void *x, const void *w,
                 const void *b, const void *y, int out_kind, const int8conv_requant *rq) {
  PlanKey k;
  memset(&k, 0, sizeof(k));
  k.device = i8c::device_info().device;
  k.strategy = strategy;
  k.pairing = i8c::pairing_mode();
  k.staging = i8c::staging_mode();
  k.out_kind = out_kind;
  k.shape = s;
  k.x = x;
  k.w = w;
  k.b = b;
  k.y = y;
  if (rq != nullptr) {
    k.zero_point = rq->zero_point;
    k.relu = rq->relu;
    k.multiplier = rq->multiplier;
    k.exponent = rq->exponent;
  }
  return k;
}

PlanSlot &plan_slot(const PlanKey &key) {
  const uint64_t *p = reinterpret_cast<const uint64_t *>(&key);
  uint64_t h = 0x9e3779b97f4a7c15ull;
  for (size_t i = 0; i < sizeof(PlanKey) / 8; ++i) h = (h ^ p[i]) * 0x100000001b3ull;
  return t_plans[(h >> 32) % kPlanSlots];
}

// The cached plan of an earlier successful launch with exactly this key, or
// nullptr.  Every argument check of a launch depends on the key's fields
// alone (device, family as requested, shape, buffers, pairing, staging,
// epilogue), so a launch that finds its plan skips them.
i8c::LaunchPlan *cached_plan(const PlanKey &key) {
  PlanSlot &slot = plan_slot(key);
  return slot.used && memcmp(&slot.key, &key, sizeof(PlanKey)) == 0 ? &slot.plan : nullptr;
}

// Runs `launch` (the family launcher) with plan capture on and caches what it
// launched under `key`.
template <class Launch>
int8conv_status launch_cached(const PlanKey &key, Launch launch) {
  PlanSlot &slot = plan_slot(key);
  i8c::LaunchPlan plan;
  i8c::plan_capture_begin(&plan);
  const int8conv_status st = launch();
  i8c::plan_capture_end();
  if (st == INT8CONV_OK && plan.func != nullptr) {
    slot.key = key;
    slot.plan = plan;
    slot.used = true;
  }
  return st;
}

// The kernel families implemented in this build.  A family whose kernel is
// not built reports every shape as ineligible.
bool family_built(int strategy) {
  return strategy >= INT8CONV_GENERIC && strategy < INT8CONV_NUM_STRATEGIES;
}

int8conv_status launch_family(int strategy, const int8conv_shape *shape, const int8_t *input,
                              const int8_t *filter, const int32_t *bias, int32_t *output,
                              void *workspace, size_t workspace_bytes, void *stream) {
  if (shape == nullptr) return INT8CONV_BAD_SHAPE;
  (void)workspace;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const PlanKey key = plan_key(strategy, *shape, input, filter, bias, output, 0, nullptr);
  if (i8c::LaunchPlan *plan = cached_plan(key)) {
    if (workspace_bytes < int8conv_workspace_bytes(shape, strategy))
      return INT8CONV_WORKSPACE_TOO_SMALL;
    return i8c::launch_plan(*plan, st);
  }
  if (!i8c_shape_valid(shape)) return INT8CONV_BAD_SHAPE;
  if (strategy == INT8CONV_AUTO) strategy = int8conv_select(shape);
  if (strategy < 0 || strategy >= INT8CONV_NUM_STRATEGIES) return INT8CONV_BAD_ARGUMENT;
  if (!int8conv_eligible(shape, strategy)) return INT8CONV_NOT_ELIGIBLE;
  if (!aligned16(input) || !aligned16(filter) || !aligned16(bias) || !aligned16(output))
    return INT8CONV_BAD_POINTER;
  if (workspace_bytes < int8conv_workspace_bytes(shape, strategy))
    return INT8CONV_WORKSPACE_TOO_SMALL;
  const int8conv_status dev = i8c::check_device();
  if (dev != INT8CONV_OK) return dev;
  return launch_cached(key, [&]() -> int8conv_status {
    switch (strategy) {
      case INT8CONV_GENERIC:
        return i8c::launch_generic_impl(*shape, input, filter, bias, output, st);
      case INT8CONV_STRIP:
        return i8c::launch_strip_impl(*shape, input, filter, bias, output, st);
      case INT8CONV_HALO:
        return i8c::launch_halo_impl(*shape, input, filter, bias, output, st);
      case INT8CONV_SPLITK:
        return i8c::launch_splitk_impl(*shape, input, filter, bias, output, st);
      default:
        return INT8CONV_NOT_ELIGIBLE;
    }
  });
}

}  // namespace

extern "C" {

int int8conv_abi_version(void) { return INT8CONV_ABI_VERSION; }

int int8conv_shape_valid(const int8conv_shape *shape) { return i8c_shape_valid(shape); }

int8conv_status int8conv_shape_dims(const int8conv_shape *s, int8conv_dims *d) {
  if (!i8c_shape_valid(s) || d == nullptr) return INT8CONV_BAD_SHAPE;
  d->out_h = i8c_out_h(s);
  d->out_w = i8c_out_w(s);
  d->gemm_m = static_cast<int64_t>(s->n) * d->out_h * d->out_w;
  d->gemm_n = s->k;
  d->gemm_k = static_cast<int64_t>(s->r) * s->s * s->c;
  d->input_elements = static_cast<int64_t>(s->n) * s->h * s->w * s->c;
  d->filter_elements = static_cast<int64_t>(s->k) * s->r * s->s * s->c;
  d->output_elements = d->gemm_m * d->gemm_n;
  return INT8CONV_OK;
}

int int8conv_eligible(const int8conv_shape *shape, int strategy) {
  if (!family_built(strategy)) return 0;
  return i8c_eligible(shape, strategy);
}

int int8conv_select(const int8conv_shape *shape) {
  // B200 dispatch policy, from conv_lab sweeps on B200:
  //  * GENERIC (with CTA pairs where they pay off) wins every large layer;
  //    STRIP's strip reuse no longer pays once the epilogue uses TMA stores
  //    (5a 357 vs 396 us, 5c 39 vs 51 us).
  //  * SPLITK when the layer has too few 128-row output tiles to occupy half
  //    the GPU but a reduction deep enough to split (7x7 and 14x14 layers):
  //    at least 10 k-blocks.  With 8 or 9 (a 1x1 over C = 1024, a 3x3 over
  //    C <= 128) GENERIC's tail-balanced column parts are as fast or faster
  //    (51-workload sweep on one B200: darknet_res_13_reduce 13.6 vs 15.0 us,
  //    dilated_3x3 13.6 vs 15.0, cfg1_smoke 13.5 vs 13.7).
  //    The split must fit in one wave of resident clusters (B200 table):
  //    two waves lost to GENERIC in the sweep (batch8_3x3, darknet_down_52).
  //  * Except where GENERIC runs narrow N tiles (i8c_generic_bn): those fill
  //    the GPU without a reduction (4c, K = 100: 13.4-13.8 us per launch
  //    against 15.1-15.2 us for SPLITK, three interleaved runs on one box).
  //    There each narrow tile stages all nine taps of its 128 rows again;
  //    HALO stages one halo tile per row tile and channel block, so where it
  //    is eligible it runs instead (4c: 6.11-6.16 against 6.97-7.02 us per
  //    launch in graph replay, 13.63-13.76 against 13.66-13.79 us per
  //    launch back to back, three interleaved runs on one box).
  if (!i8c_shape_valid(shape)) return INT8CONV_GENERIC;
  const int32_t clusters[9] = I8C_B200_CLUSTERS;
  // GENERIC's narrow-tile rule runs with the current device's SM count (the
  // kernel's planner uses it); the B200 count where no sm_100 device is
  // current (host-only use).  The split-K table below is B200's.
  int slots = clusters[1];
  if (i8c::check_device() == INT8CONV_OK) slots = i8c::device_info().sm_count;
  if (i8c_generic_bn(shape, 16, slots) < i8c_pick_bn(shape->k, 16) &&
      int8conv_eligible(shape, INT8CONV_GENERIC))
    return int8conv_eligible(shape, INT8CONV_HALO) ? INT8CONV_HALO : INT8CONV_GENERIC;
  const int64_t m = static_cast<int64_t>(shape->n) * i8c_out_h(shape) * i8c_out_w(shape);
  const int64_t n_tiles = (shape->k + 255) / 256;
  const int64_t tiles = (m + 127) / 128 * n_tiles;
  const int32_t cblk = i8c_channel_block(shape->c);
  const int64_t kblocks =
      static_cast<int64_t>(shape->r) * shape->s * ((shape->c + cblk - 1) / cblk);
  if (int8conv_eligible(shape, INT8CONV_SPLITK) && tiles < 74 && kblocks >= 10 &&
      i8c_split_count(i8c_split_tiles(shape), kblocks, clusters) >= 2)
    return INT8CONV_SPLITK;
  return INT8CONV_GENERIC;
}

size_t int8conv_workspace_bytes(const int8conv_shape *shape, int strategy) {
  (void)shape;
  (void)strategy;
  return 0;
}

const char *int8conv_strategy_name(int strategy) {
  switch (strategy) {
    case INT8CONV_GENERIC:
      return "generic";
    case INT8CONV_STRIP:
      return "strip";
    case INT8CONV_HALO:
      return "halo";
    case INT8CONV_SPLITK:
      return "splitk";
    case INT8CONV_AUTO:
      return "auto";
    default:
      return "unknown";
  }
}

const char *int8conv_status_string(int status) {
  switch (status) {
    case INT8CONV_OK:
      return "ok";
    case INT8CONV_NOT_ELIGIBLE:
      return "shape not eligible for this strategy";
    case INT8CONV_BAD_SHAPE:
      return "invalid convolution shape";
    case INT8CONV_BAD_POINTER:
      return "null or misaligned (16-byte) buffer";
    case INT8CONV_CUDA_ERROR:
      return "CUDA error";
    case INT8CONV_DEVICE_TIMEOUT:
      return "device wait timed out";
    case INT8CONV_WORKSPACE_TOO_SMALL:
      return "workspace too small";
    case INT8CONV_UNSUPPORTED_DEVICE:
      return "device is not sm_100";
    case INT8CONV_BAD_ARGUMENT:
      return "bad argument";
    default:
      return "unknown status";
  }
}

int8conv_status int8conv_launch(int strategy, const int8conv_shape *shape, const int8_t *input,
                                const int8_t *filter, const int32_t *bias, int32_t *output,
                                void *workspace, size_t workspace_bytes, void *stream) {
  return launch_family(strategy, shape, input, filter, bias, output, workspace,
                       workspace_bytes, stream);
}

int8conv_status int8conv_launch_generic(const int8conv_shape *shape, const int8_t *input,
                                        const int8_t *filter, const int32_t *bias,
                                        int32_t *output, void *stream) {
  return launch_family(INT8CONV_GENERIC, shape, input, filter, bias, output, nullptr, 0, stream);
}

int8conv_status int8conv_launch_spatial_strip(const int8conv_shape *shape, const int8_t *input,
                                              const int8_t *filter, const int32_t *bias,
                                              int32_t *output, void *stream) {
  return launch_family(INT8CONV_STRIP, shape, input, filter, bias, output, nullptr, 0, stream);
}

int8conv_status int8conv_launch_halo(const int8conv_shape *shape, const int8_t *input,
                                     const int8_t *filter, const int32_t *bias, int32_t *output,
                                     void *stream) {
  return launch_family(INT8CONV_HALO, shape, input, filter, bias, output, nullptr, 0, stream);
}

int8conv_status int8conv_launch_splitk(const int8conv_shape *shape, const int8_t *input,
                                       const int8_t *filter, const int32_t *bias,
                                       int32_t *output, void *workspace, size_t workspace_bytes,
                                       void *stream) {
  return launch_family(INT8CONV_SPLITK, shape, input, filter, bias, output, workspace,
                       workspace_bytes, stream);
}

int8conv_status int8conv_launch_requant(int strategy, const int8conv_shape *shape,
                                        const int8_t *input, const int8_t *filter,
                                        const int32_t *bias, const int8conv_requant *requant,
                                        int8_t *output, void *workspace, size_t workspace_bytes,
                                        void *stream) {
  if (shape == nullptr) return INT8CONV_BAD_SHAPE;
  if (requant == nullptr) return INT8CONV_BAD_ARGUMENT;
  (void)workspace;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const PlanKey key = plan_key(strategy, *shape, input, filter, bias, output,
                               1 + requant->layout, requant);
  if (i8c::LaunchPlan *plan = cached_plan(key)) {
    if (workspace_bytes < int8conv_workspace_bytes(shape, strategy))
      return INT8CONV_WORKSPACE_TOO_SMALL;
    return i8c::launch_plan(*plan, st);
  }
  if (!i8c_shape_valid(shape)) return INT8CONV_BAD_SHAPE;
  if (requant->layout != INT8CONV_LAYOUT_NHWC && requant->layout != INT8CONV_LAYOUT_NCHW_VECT_C)
    return INT8CONV_BAD_ARGUMENT;
  if (requant->zero_point < -128 || requant->zero_point > 127) return INT8CONV_BAD_ARGUMENT;
  if (requant->relu != 0 && requant->relu != 1) return INT8CONV_BAD_ARGUMENT;
  if (strategy == INT8CONV_AUTO) strategy = int8conv_select(shape);
  if (strategy < 0 || strategy >= INT8CONV_NUM_STRATEGIES) return INT8CONV_BAD_ARGUMENT;
  if (!int8conv_eligible(shape, strategy)) return INT8CONV_NOT_ELIGIBLE;
  if (requant->layout == INT8CONV_LAYOUT_NCHW_VECT_C && shape->k % 32 != 0)
    return INT8CONV_NOT_ELIGIBLE;
  if (!aligned16(input) || !aligned16(filter) || !aligned16(bias) || !aligned16(output) ||
      !aligned16(requant->multiplier) || !aligned16(requant->exponent))
    return INT8CONV_BAD_POINTER;
  if (workspace_bytes < int8conv_workspace_bytes(shape, strategy))
    return INT8CONV_WORKSPACE_TOO_SMALL;
  const int8conv_status dev = i8c::check_device();
  if (dev != INT8CONV_OK) return dev;
  const i8c::Requant rq{requant->multiplier, requant->exponent, requant->zero_point,
                        requant->relu, requant->layout};
  return launch_cached(key, [&]() -> int8conv_status {
    if (strategy == INT8CONV_SPLITK)
      return i8c::launch_splitk_requant(*shape, input, filter, bias, rq, output, st);
    return i8c::launch_conv_requant(strategy, *shape, input, filter, bias, rq, output, st);
  });
}

int8conv_status int8conv_launch_host(int strategy, const int8conv_shape *shape,
                                     const int8_t *host_input, const int8_t *host_filter,
                                     const int32_t *host_bias, int32_t *host_output,
                                     int8_t *dev_input, int8_t *dev_filter, int32_t *dev_bias,
                                     int32_t *dev_output, int chunks, void *stream) {
  if (!i8c_shape_valid(shape)) return INT8CONV_BAD_SHAPE;
  if (strategy != INT8CONV_AUTO && (strategy < 0 || strategy >= INT8CONV_NUM_STRATEGIES))
    return INT8CONV_BAD_ARGUMENT;
  if (chunks < 1) return INT8CONV_BAD_ARGUMENT;
  if (strategy != INT8CONV_AUTO && !int8conv_eligible(shape, strategy))
    return INT8CONV_NOT_ELIGIBLE;
  if (!host_input || !host_filter || !host_bias || !host_output || !aligned16(dev_input) ||
      !aligned16(dev_filter) || !aligned16(dev_bias) || !aligned16(dev_output))
    return INT8CONV_BAD_POINTER;
  const int8conv_status dev = i8c::check_device();
  if (dev != INT8CONV_OK) return dev;
  return i8c::launch_host_pipeline(strategy, *shape, host_input, host_filter, host_bias,
                                   host_output, dev_input, dev_filter, dev_bias, dev_output,
                                   chunks, static_cast<cudaStream_t>(stream));
}

int8conv_status int8conv_device_status(void) {
  if (cudaDeviceSynchronize() != cudaSuccess) return INT8CONV_CUDA_ERROR;
  i8c::DeviceInfo &d = i8c::device_info();
  if (d.status == nullptr) return INT8CONV_CUDA_ERROR;
  uint32_t word = 0;
  if (cudaMemcpy(&word, d.status, sizeof(word), cudaMemcpyDeviceToHost) != cudaSuccess)
    return INT8CONV_CUDA_ERROR;
  if (word != 0) {
    const uint32_t zero = 0;
    if (cudaMemcpy(d.status, &zero, sizeof(zero), cudaMemcpyHostToDevice) != cudaSuccess)
      return INT8CONV_CUDA_ERROR;
    return INT8CONV_DEVICE_TIMEOUT;
  }
  return INT8CONV_OK;
}

void int8conv_set_wait_limit_ns(uint64_t ns) {
  i8c::g_wait_limit_ns.store(ns == 0 ? 2000000000ull : ns);
}

void int8conv_debug_starve_producer(int on) { i8c::g_starve.store(on ? 1u : 0u); }

uint64_t int8conv_launch_count(void) { return i8c::g_launches.load(); }

int8conv_status int8conv_set_cta_pairing(int mode) {
  if (mode < 0 || mode > 2) return INT8CONV_BAD_ARGUMENT;
  i8c::g_pairing.store(mode);
  return INT8CONV_OK;
}

int8conv_status int8conv_set_generic_staging(int mode) {
  if (mode < 0 || mode > 1) return INT8CONV_BAD_ARGUMENT;
  i8c::g_staging.store(mode);
  return INT8CONV_OK;
}

}  // extern "C"
