// host.cu - per-device state, tensor-map encoding and run controls.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <stdint.h>
#include <string.h>

#include <atomic>
#include <mutex>

#include "launch.h"

namespace i8c {

// Module-scope status word: kernels OR timeout bits into it, the host reads
// and clears it in int8conv_device_status().  One copy per device.
__device__ uint32_t g_device_status;

std::atomic<uint64_t> g_wait_limit_ns{2000000000ull};
std::atomic<uint32_t> g_starve{0};
std::atomic<uint64_t> g_launches{0};
std::atomic<int> g_pairing{0};
std::atomic<int> g_staging{0};

namespace {

constexpr int kMaxDevices = 64;
DeviceInfo g_devices[kMaxDevices];
// 1 once g_devices[i] is filled in; the release store publishes the fields
// to threads that read the flag with acquire (static storage: starts at 0).
std::atomic<int> g_device_ready[kMaxDevices];
std::mutex g_device_mutex;

PFN_cuTensorMapEncodeTiled_v12000 g_encode_tiled = nullptr;
PFN_cuTensorMapEncodeIm2col_v12000 g_encode_im2col = nullptr;
int g_driver_version = 0;
std::once_flag g_driver_once;

void load_driver_entry_points() {
  cudaDriverEntryPointQueryResult q;
  void *fn = nullptr;
  if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) ==
          cudaSuccess &&
      q == cudaDriverEntryPointSuccess)
    g_encode_tiled = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  fn = nullptr;
  if (cudaGetDriverEntryPoint("cuTensorMapEncodeIm2col", &fn, cudaEnableDefault, &q) ==
          cudaSuccess &&
      q == cudaDriverEntryPointSuccess)
    g_encode_im2col = reinterpret_cast<PFN_cuTensorMapEncodeIm2col_v12000>(fn);
  cudaDriverGetVersion(&g_driver_version);
}

// Small cache of encoded maps: a launch with the same buffers and shape reuses
// the 128-byte descriptor instead of re-encoding it on every call.
struct MapKey {
  int32_t device, kind, channels, rows, count_w, pad;
  int8conv_shape shape;
  const void *ptr;
};
struct MapEntry {
  MapKey key;
  CUtensorMap map;
  bool used;
};
// Direct-mapped by an FNV-1a hash of the key: a hit costs one comparison.
constexpr int kMapCache = 512;
MapEntry g_maps[kMapCache];
std::mutex g_map_mutex;

uint32_t key_slot(const MapKey &key) {
  const unsigned char *p = reinterpret_cast<const unsigned char *>(&key);
  uint32_t h = 2166136261u;
  for (size_t i = 0; i < sizeof(MapKey); ++i) h = (h ^ p[i]) * 16777619u;
  return h % kMapCache;
}

bool map_lookup(const MapKey &key, CUtensorMap *map) {
  const uint32_t slot = key_slot(key);
  std::lock_guard<std::mutex> lock(g_map_mutex);
  const MapEntry &e = g_maps[slot];
  if (e.used && memcmp(&e.key, &key, sizeof(MapKey)) == 0) {
    *map = e.map;
    return true;
  }
  return false;
}

void map_store(const MapKey &key, const CUtensorMap &map) {
  const uint32_t slot = key_slot(key);
  std::lock_guard<std::mutex> lock(g_map_mutex);
  MapEntry &e = g_maps[slot];
  e.key = key;
  e.map = map;
  e.used = true;
}

MapKey make_key(int kind, const int8conv_shape &s, const void *ptr, int channels, int rows,
                int count_w) {
  MapKey k;
  memset(&k, 0, sizeof(k));
  k.device = device_info().device;
  k.kind = kind;
  k.channels = channels;
  k.rows = rows;
  k.count_w = count_w;
  k.shape = s;
  k.ptr = ptr;
  return k;
}

CUtensorMapSwizzle swizzle_for(int bytes) {
  switch (bytes) {
    case 128:
      return CU_TENSOR_MAP_SWIZZLE_128B;
    case 64:
      return CU_TENSOR_MAP_SWIZZLE_64B;
    case 32:
      return CU_TENSOR_MAP_SWIZZLE_32B;
    default:
      return CU_TENSOR_MAP_SWIZZLE_NONE;
  }
}

}  // namespace

DeviceInfo &device_info() {
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= kMaxDevices) dev = 0;
  DeviceInfo &d = g_devices[dev];
  if (g_device_ready[dev].load(std::memory_order_acquire) == 0) {
    std::lock_guard<std::mutex> lock(g_device_mutex);
    if (g_device_ready[dev].load(std::memory_order_relaxed) == 0) {
      cudaDeviceProp prop;
      if (cudaGetDeviceProperties(&prop, dev) == cudaSuccess) {
        d.sm_count = prop.multiProcessorCount;
        d.cc_major = prop.major;
        d.cc_minor = prop.minor;
      }
      void *addr = nullptr;
      if (cudaGetSymbolAddress(&addr, g_device_status) == cudaSuccess)
        d.status = static_cast<uint32_t *>(addr);
      d.device = dev;
      g_device_ready[dev].store(1, std::memory_order_release);
    }
  }
  return d;
}

int8conv_status check_device() {
  DeviceInfo &d = device_info();
  if (d.sm_count == 0) return INT8CONV_CUDA_ERROR;
  if (d.cc_major != 10) return INT8CONV_UNSUPPORTED_DEVICE;
  return INT8CONV_OK;
}

RunCtl run_ctl() {
  RunCtl c;
  c.status = device_info().status;
  c.wait_ns = g_wait_limit_ns.load(std::memory_order_relaxed);
  c.starve = g_starve.load(std::memory_order_relaxed);
  return c;
}

void note_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

namespace {
thread_local LaunchPlan *t_capture = nullptr;
}  // namespace

void plan_capture_begin(LaunchPlan *out) { t_capture = out; }
void plan_capture_end() { t_capture = nullptr; }

int8conv_status launch_plan(LaunchPlan &plan, cudaStream_t stream) {
  if (plan.ctl_arg >= 0) {
    // The status word's address is the plan device's (fixed per device); the
    // wait limit and the starve hook are re-read at every launch.
    RunCtl ctl;
    unsigned char *at = plan.blob + plan.offset[plan.ctl_arg];
    memcpy(&ctl, at, sizeof(ctl));
    if (ctl.status == nullptr) ctl.status = device_info().status;
    ctl.wait_ns = g_wait_limit_ns.load(std::memory_order_relaxed);
    ctl.starve = g_starve.load(std::memory_order_relaxed);
    memcpy(at, &ctl, sizeof(ctl));
  }
  if (t_capture != nullptr) *t_capture = plan;
  void *args[12];
  for (int i = 0; i < plan.nargs; ++i) args[i] = plan.blob + plan.offset[i];
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = plan.grid;
  cfg.blockDim = plan.block;
  cfg.dynamicSmemBytes = plan.smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = plan.cluster;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = plan.cluster > 1 ? 2 : 1;
  const cudaError_t err = cudaLaunchKernelExC(&cfg, plan.func, args);
  note_launch();
  return err == cudaSuccess ? INT8CONV_OK : INT8CONV_CUDA_ERROR;
}

int pairing_mode() { return g_pairing.load(std::memory_order_relaxed); }

int staging_mode() { return g_staging.load(std::memory_order_relaxed); }

bool ensure_smem_attr(const void *kernel, int bytes) {
  // Remember the largest limit already set per (device, kernel).
  struct Entry {
    int device;
    const void *kernel;
    int bytes;
  };
  static Entry table[256];
  static int used = 0;
  static std::mutex mutex;
  const int dev = device_info().device;
  std::lock_guard<std::mutex> lock(mutex);
  for (int i = 0; i < used; ++i) {
    if (table[i].device == dev && table[i].kernel == kernel) {
      if (table[i].bytes >= bytes) return true;
      if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) !=
          cudaSuccess)
        return false;
      table[i].bytes = bytes;
      return true;
    }
  }
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) !=
      cudaSuccess)
    return false;
  if (used < 256) table[used++] = Entry{dev, kernel, bytes};
  return true;
}

int8conv_status activation_map_im2col(const int8conv_shape &s, const int8_t *x, int channels,
                                      int pixels, int count_w, int count_h, CUtensorMap *map) {
  MapKey key = make_key(1, s, x, channels, pixels, count_w);
  key.pad = count_h;
  if (map_lookup(key, map)) return INT8CONV_OK;
  std::call_once(g_driver_once, load_driver_entry_points);
  if (!g_encode_im2col) return INT8CONV_CUDA_ERROR;
  cuuint64_t dims[4] = {(cuuint64_t)s.c, (cuuint64_t)s.w, (cuuint64_t)s.h, (cuuint64_t)s.n};
  cuuint64_t strides[3] = {(cuuint64_t)s.c, (cuuint64_t)s.w * s.c, (cuuint64_t)s.h * s.w * s.c};
  // Bounding box per image: traversal starts at -pad and holds exactly
  // count_w x count_h positions (stride apart); the upper corner is chosen so.
  int lower[2] = {-s.pad_w, -s.pad_h};
  int upper[2] = {-s.pad_w + (count_w - 1) * s.stride_w + 1 - s.w,
                  -s.pad_h + (count_h - 1) * s.stride_h + 1 - s.h};
  cuuint32_t estr[4] = {1, (cuuint32_t)s.stride_w, (cuuint32_t)s.stride_h, 1};
  CUresult rc = g_encode_im2col(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, const_cast<int8_t *>(x),
                                dims, strides, lower, upper, (cuuint32_t)channels,
                                (cuuint32_t)pixels, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                swizzle_for(channels), CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (rc != CUDA_SUCCESS) return INT8CONV_CUDA_ERROR;
  // Driver <= 13.1 mis-handles im2col maps over tensors smaller than 128 KB
  // unless bit 21 of the descriptor's second word is cleared (the same
  // workaround CUTLASS applies in cute/atom/copy_traits_sm90_im2col.hpp).
  const uint64_t bytes = (uint64_t)s.n * s.h * s.w * s.c;
  if (g_driver_version <= 13010 && bytes < 131072)
    reinterpret_cast<uint64_t *>(map)[1] &= ~(1ull << 21);
  map_store(key, *map);
  return INT8CONV_OK;
}

int8conv_status filter_map_tiled(const int8conv_shape &s, const int8_t *w, int channels,
                                 int rows, CUtensorMap *map) {
  const MapKey key = make_key(2, s, w, channels, rows, 0);
  if (map_lookup(key, map)) return INT8CONV_OK;
  std::call_once(g_driver_once, load_driver_entry_points);
  if (!g_encode_tiled) return INT8CONV_CUDA_ERROR;
  cuuint64_t dims[3] = {(cuuint64_t)s.c, (cuuint64_t)s.r * s.s, (cuuint64_t)s.k};
  cuuint64_t strides[2] = {(cuuint64_t)s.c, (cuuint64_t)s.r * s.s * s.c};
  cuuint32_t box[3] = {(cuuint32_t)channels, 1, (cuuint32_t)rows};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult rc = g_encode_tiled(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<int8_t *>(w),
                               dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                               swizzle_for(channels), CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (rc != CUDA_SUCCESS) return INT8CONV_CUDA_ERROR;
  map_store(key, *map);
  return INT8CONV_OK;
}

int8conv_status filter_map_rows(const int8conv_shape &s, const int8_t *w, int channels, int rows,
                                CUtensorMap *map) {
  const MapKey key = make_key(5, s, w, channels, rows, 0);
  if (map_lookup(key, map)) return INT8CONV_OK;
  std::call_once(g_driver_once, load_driver_entry_points);
  if (!g_encode_tiled) return INT8CONV_CUDA_ERROR;
  const uint64_t row_bytes = static_cast<uint64_t>(s.s) * s.c;
  cuuint64_t dims[3] = {(cuuint64_t)row_bytes, (cuuint64_t)s.r, (cuuint64_t)s.k};
  cuuint64_t strides[2] = {(cuuint64_t)row_bytes, (cuuint64_t)row_bytes * s.r};
  cuuint32_t box[3] = {(cuuint32_t)channels, 1, (cuuint32_t)rows};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult rc = g_encode_tiled(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<int8_t *>(w),
                               dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                               swizzle_for(channels), CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (rc != CUDA_SUCCESS) return INT8CONV_CUDA_ERROR;
  map_store(key, *map);
  return INT8CONV_OK;
}

int8conv_status output_map_tiled(int32_t *y, int64_t m, int k, CUtensorMap *map) {
  int8conv_shape key_shape{};
  key_shape.n = static_cast<int32_t>(m);
  key_shape.k = k;
  const MapKey key = make_key(3, key_shape, y, 32, 32, 0);
  if (map_lookup(key, map)) return INT8CONV_OK;
  std::call_once(g_driver_once, load_driver_entry_points);
  if (!g_encode_tiled) return INT8CONV_CUDA_ERROR;
  cuuint64_t dims[2] = {(cuuint64_t)k, (cuuint64_t)m};
  cuuint64_t strides[1] = {(cuuint64_t)k * 4};
  cuuint32_t box[2] = {32, 32};
  cuuint32_t estr[2] = {1, 1};
  CUresult rc = g_encode_tiled(map, CU_TENSOR_MAP_DATA_TYPE_INT32, 2, y, dims, strides, box, estr,
                               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                               CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (rc != CUDA_SUCCESS) return INT8CONV_CUDA_ERROR;
  map_store(key, *map);
  return INT8CONV_OK;
}

int8conv_status output_map_rows(int32_t *y, int64_t m, int k, int rows, CUtensorMap *map) {
  int8conv_shape key_shape{};
  key_shape.n = static_cast<int32_t>(m);
  key_shape.k = k;
  const MapKey key = make_key(6, key_shape, y, 32, rows, 0);
  if (map_lookup(key, map)) return INT8CONV_OK;
  std::call_once(g_driver_once, load_driver_entry_points);
  if (!g_encode_tiled) return INT8CONV_CUDA_ERROR;
  cuuint64_t dims[2] = {(cuuint64_t)k, (cuuint64_t)m};
  cuuint64_t strides[1] = {(cuuint64_t)k * 4};
  cuuint32_t box[2] = {32, (cuuint32_t)rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult rc = g_encode_tiled(map, CU_TENSOR_MAP_DATA_TYPE_INT32, 2, y, dims, strides, box, estr,
                               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                               CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (rc != CUDA_SUCCESS) return INT8CONV_CUDA_ERROR;
  map_store(key, *map);
  return INT8CONV_OK;
}

int8conv_status output_map_i8(int8_t *y, int64_t m, int k, CUtensorMap *map) {
  int8conv_shape key_shape{};
  key_shape.n = static_cast<int32_t>(m);
  key_shape.k = k;
  const MapKey key = make_key(4, key_shape, y, 32, 32, 0);
  if (map_lookup(key, map)) return INT8CONV_OK;
  std::call_once(g_driver_once, load_driver_entry_points);
  if (!g_encode_tiled) return INT8CONV_CUDA_ERROR;
  cuuint64_t dims[2] = {(cuuint64_t)k, (cuuint64_t)m};
  cuuint64_t strides[1] = {(cuuint64_t)k};
  cuuint32_t box[2] = {32, 32};
  cuuint32_t estr[2] = {1, 1};
  CUresult rc = g_encode_tiled(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, y, dims, strides, box, estr,
                               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                               CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (rc != CUDA_SUCCESS) return INT8CONV_CUDA_ERROR;
  map_store(key, *map);
  return INT8CONV_OK;
}

}  // namespace i8c
