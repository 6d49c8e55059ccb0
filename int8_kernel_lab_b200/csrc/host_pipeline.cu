// host_pipeline.cu - int8conv_launch_host: host-buffer convolution with the
// PCIe copies overlapped with compute.
//
// The batch is split into `chunks` groups of whole images (every image is an
// independent convolution).  Group boundaries fall on image counts whose
// output offset is a multiple of 16 bytes (the kernels' alignment rule): with
// out_h*out_w*K odd, every fourth image; input offsets are always aligned
// (C % 16 == 0).  Per group i, on three streams:
//   h2d stream:  copy input images of group i          -> event in[i]
//   compute:     wait in[i]; launch on group i's shape  -> event done[i]
//   d2h stream:  wait done[i]; copy output rows of group i
// so the copy of group i+1, the kernel of group i and the read-back of group
// i-1 proceed together (B200 has separate copy engines per direction).  The
// caller's stream finally waits for the last read-back.  Streams and events
// are created once per device and reused; no device memory is allocated.
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>

#include "int8conv.h"
#include "int8conv_rules.h"
#include "launch.h"

namespace i8c {
namespace {

constexpr int kMaxChunks = 64;

struct PipelineState {
  bool ready = false;
  cudaStream_t h2d = nullptr, compute = nullptr, d2h = nullptr;
  cudaEvent_t start = nullptr;
  cudaEvent_t in[kMaxChunks] = {};
  cudaEvent_t done[kMaxChunks] = {};
  cudaEvent_t out = nullptr;
  std::mutex mutex;  // one pipeline in flight per device at a time
};

PipelineState g_pipes[64];

bool init_pipe(PipelineState &p) {
  if (p.ready) return true;
  auto ok = [](cudaError_t e) { return e == cudaSuccess; };
  if (!ok(cudaStreamCreateWithFlags(&p.h2d, cudaStreamNonBlocking)) ||
      !ok(cudaStreamCreateWithFlags(&p.compute, cudaStreamNonBlocking)) ||
      !ok(cudaStreamCreateWithFlags(&p.d2h, cudaStreamNonBlocking)) ||
      !ok(cudaEventCreateWithFlags(&p.start, cudaEventDisableTiming)) ||
      !ok(cudaEventCreateWithFlags(&p.out, cudaEventDisableTiming)))
    return false;
  for (int i = 0; i < kMaxChunks; ++i) {
    if (!ok(cudaEventCreateWithFlags(&p.in[i], cudaEventDisableTiming)) ||
        !ok(cudaEventCreateWithFlags(&p.done[i], cudaEventDisableTiming)))
      return false;
  }
  p.ready = true;
  return true;
}

}  // namespace

int8conv_status launch_host_pipeline(int strategy, const int8conv_shape &s, const int8_t *hx,
                                     const int8_t *hw, const int32_t *hb, int32_t *hy,
                                     int8_t *dx, int8_t *dw, int32_t *db, int32_t *dy,
                                     int chunks, cudaStream_t stream) {
  DeviceInfo &dev = device_info();
  PipelineState &p = g_pipes[dev.device & 63];
  std::lock_guard<std::mutex> lock(p.mutex);
  if (!init_pipe(p)) return INT8CONV_CUDA_ERROR;
  const int32_t out_h = i8c_out_h(&s), out_w = i8c_out_w(&s);
  const size_t in_image = static_cast<size_t>(s.h) * s.w * s.c;
  const size_t out_image = static_cast<size_t>(out_h) * out_w * s.k;
  // Images per boundary unit: the output offset of `step` images is a
  // multiple of four int32 values.
  const int step = out_image % 4 == 0 ? 1 : out_image % 2 == 0 ? 2 : 4;
  const int units = (s.n + step - 1) / step;
  if (chunks < 1) chunks = 1;
  if (chunks > units) chunks = units;
  if (chunks > kMaxChunks) chunks = kMaxChunks;
  auto ok = [](cudaError_t e) { return e == cudaSuccess; };
  // On an error part-way through, copies already queued may still be reading
  // or writing the caller's host buffers: wait for them before returning, so
  // the caller may free those buffers as soon as the call fails.
  auto fail = [&](int8conv_status st) {
    cudaStreamSynchronize(p.h2d);
    cudaStreamSynchronize(p.compute);
    cudaStreamSynchronize(p.d2h);
    return st;
  };
  // Everything the caller queued on `stream` before this call happens first.
  if (!ok(cudaEventRecord(p.start, stream)) || !ok(cudaStreamWaitEvent(p.h2d, p.start, 0)))
    return INT8CONV_CUDA_ERROR;
  const size_t filter_bytes = static_cast<size_t>(s.k) * s.r * s.s * s.c;
  if (!ok(cudaMemcpyAsync(dw, hw, filter_bytes, cudaMemcpyHostToDevice, p.h2d)) ||
      !ok(cudaMemcpyAsync(db, hb, sizeof(int32_t) * s.k, cudaMemcpyHostToDevice, p.h2d)))
    return fail(INT8CONV_CUDA_ERROR);
  int first = 0;
  for (int c = 0; c < chunks; ++c) {
    const int64_t unit_end = static_cast<int64_t>(units) * (c + 1) / chunks;
    const int last = unit_end * step < s.n ? static_cast<int>(unit_end * step) : s.n;
    const int images = last - first;
    int8conv_shape part = s;
    part.n = images;
    const size_t x_off = first * in_image;
    const size_t y_off = first * out_image;
    if (!ok(cudaMemcpyAsync(dx + x_off, hx + x_off, images * in_image, cudaMemcpyHostToDevice,
                            p.h2d)) ||
        !ok(cudaEventRecord(p.in[c], p.h2d)) || !ok(cudaStreamWaitEvent(p.compute, p.in[c], 0)))
      return fail(INT8CONV_CUDA_ERROR);
    const int fam = strategy == INT8CONV_AUTO ? int8conv_select(&part) : strategy;
    const int8conv_status st = int8conv_launch(fam, &part, dx + x_off, dw, db, dy + y_off, nullptr,
                                               0, p.compute);
    if (st != INT8CONV_OK) return fail(st);
    if (!ok(cudaEventRecord(p.done[c], p.compute)) ||
        !ok(cudaStreamWaitEvent(p.d2h, p.done[c], 0)) ||
        !ok(cudaMemcpyAsync(hy + y_off, dy + y_off, images * out_image * sizeof(int32_t),
                            cudaMemcpyDeviceToHost, p.d2h)))
      return fail(INT8CONV_CUDA_ERROR);
    first = last;
  }
  if (!ok(cudaEventRecord(p.out, p.d2h)) || !ok(cudaStreamWaitEvent(stream, p.out, 0)))
    return fail(INT8CONV_CUDA_ERROR);
  return INT8CONV_OK;
}

}  // namespace i8c
