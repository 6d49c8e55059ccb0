// conv_lab.cpp - the lab's command-line harness, over the C ABI.
//
// Mirrors src/conv_lab.cu of pthodima/int8_kernel_lab:
//   * same flags: --strategy, --csv, --warmup N (20), --iterations N (101)
//     (conv_lab.cu:112-145), plus --case/--config to pick a workloads.csv row
//     at run time (the reference compiles one binary per case), --values,
//     --seed, --batch, --peak-tops, --no-graph, --pairing;
//   * same flow: seeded inputs, device buffers, launch, validate before
//     timing, per-launch event median (conv_lab.cu:88-110), winner, CSV or
//     human line, exit code 0 only if every run was correct and one ran
//     (conv_lab.cu:241);
//   * same first 16 CSV columns in the same order (conv_lab.cu:223-230), then
//     the appended ones: eligible_halo, eligible_splitk, halo_ms, splitk_ms,
//     halo_correct, splitk_correct, gpus, tops, roofline_frac, oracle_ms,
//     oracle_threads, graph_ms, selected (the family int8conv_select picks),
//     epilogue, l2 ("warm", or "rotated:<sets>" with --rotate-l2).
// --staging gather runs GENERIC with its gather warp on every shape
// (int8conv_set_generic_staging), to time it against the im2col staging.
// --rotate-l2 times every launch on the next of enough input/output sets
// that together span twice the L2, so memory-bound shapes are timed L2-cold
// (the reference times one buffer set, L2-warm for small shapes).
// --epilogue int8 | int8x32 times int8conv_launch_requant (NHWC or cuDNN's
// NCHW_VECT_C int8 output) with seeded per-channel multipliers and exponents.
// Validation compares EVERY output element (the reference checks 2048
// strided samples above 65536 outputs, conv_lab.cu:72-77) against a direct
// host convolution with the loop nest of conv_lab.cu:39-66;
// --validate-samples N checks the first and last output rows plus N random
// outputs instead (for multi-Top stress shapes).
// --strategy both = generic + strip (as in the reference); all = the four
// families; auto = the dispatch policy's pick; or one family name.
#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <fstream>
#include <functional>
#include <iomanip>
#include <iostream>
#include <memory>
#include <random>
#include <sstream>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

#include "int8conv.h"
#include "requant.cuh"

namespace {

// A failed CUDA runtime call ends the run (exit code 1, the call named).
struct CudaFailure : std::runtime_error {
  using std::runtime_error::runtime_error;
};

void check(cudaError_t status, const char *what) {
  if (status == cudaSuccess) return;
  throw CudaFailure(std::string(what) + ": " + cudaGetErrorString(status));
}

// Device array of `count` T (at least one element, so an empty tensor still
// has a valid, aligned address), freed with its owner.
struct CudaFree {
  void operator()(void *p) const { cudaFree(p); }
};
template <class T>
using DeviceArray = std::unique_ptr<T, CudaFree>;

template <class T>
DeviceArray<T> device_array(size_t count) {
  void *p = nullptr;
  check(cudaMalloc(&p, (count == 0 ? 1 : count) * sizeof(T)), "cudaMalloc");
  return DeviceArray<T>(static_cast<T *>(p));
}

struct Options {
  std::string strategy = "both";
  bool csv = false;
  int warmup = 20;
  int iterations = 101;
  std::string case_name = "smoke";
  std::string config;
  std::string values = "full";
  uint32_t seed = 20260925;
  int batch = 0;
  double peak_tops = 4500.0;
  bool graph = true;
  int pairing = 0;
  long long validate_samples = 0;  // 0: every output
  std::string epilogue = "int32";  // int32 | int8 (NHWC) | int8x32 (NCHW_VECT_C)
  bool rotate_l2 = false;          // time over rotating buffer sets (L2-cold)
  int staging = 0;                 // GENERIC staging: 0 auto, 1 gather
};

[[noreturn]] void usage() {
  std::cerr << "usage: conv_lab [--strategy generic|strip|halo|splitk|both|all|auto] [--csv] "
               "[--warmup N] [--iterations N] [--case NAME] [--config CSV] "
               "[--values full|reference|ones] [--seed S] [--batch N] [--peak-tops T] "
               "[--no-graph] [--pairing auto|single|pair] [--validate-samples N] "
               "[--epilogue int32|int8|int8x32] [--rotate-l2] [--staging auto|gather]\n";
  std::exit(EXIT_FAILURE);
}

Options parse_options(int argc, char **argv) {
  Options o;
  for (int i = 1; i < argc; ++i) {
    const std::string arg = argv[i];
    auto value = [&]() -> std::string {
      if (i + 1 >= argc) usage();
      return argv[++i];
    };
    if (arg == "--csv") o.csv = true;
    else if (arg == "--no-graph") o.graph = false;
    else if (arg == "--rotate-l2") o.rotate_l2 = true;
    else if (arg == "--staging") {
      const std::string v = value();
      o.staging = v == "auto" ? 0 : v == "gather" ? 1 : -1;
      if (o.staging < 0) usage();
    }
    else if (arg == "--strategy") o.strategy = value();
    else if (arg == "--warmup") o.warmup = std::stoi(value());
    else if (arg == "--iterations") o.iterations = std::stoi(value());
    else if (arg == "--case") o.case_name = value();
    else if (arg == "--config") o.config = value();
    else if (arg == "--values") o.values = value();
    else if (arg == "--seed") o.seed = static_cast<uint32_t>(std::stoul(value()));
    else if (arg == "--batch") o.batch = std::stoi(value());
    else if (arg == "--peak-tops") o.peak_tops = std::stod(value());
    else if (arg == "--validate-samples") o.validate_samples = std::stoll(value());
    else if (arg == "--epilogue") o.epilogue = value();
    else if (arg == "--pairing") {
      const std::string v = value();
      o.pairing = v == "auto" ? 0 : v == "single" ? 1 : v == "pair" ? 2 : -1;
      if (o.pairing < 0) usage();
    } else usage();
  }
  const std::vector<std::string> ok = {"generic", "strip", "halo", "splitk", "both", "all", "auto"};
  if (std::find(ok.begin(), ok.end(), o.strategy) == ok.end() || o.warmup < 0 ||
      o.iterations <= 0 || (o.values != "full" && o.values != "reference" && o.values != "ones") || o.batch < 0 ||
      (o.epilogue != "int32" && o.epilogue != "int8" && o.epilogue != "int8x32")) {
    std::cerr << "invalid benchmark options\n";
    std::exit(EXIT_FAILURE);
  }
  return o;
}

std::string default_config(const char *argv0) {
  // lib/conv_lab -> ../workloads.csv
  std::string self = argv0;
  const size_t slash = self.find_last_of('/');
  const std::string dir = slash == std::string::npos ? "." : self.substr(0, slash);
  return dir + "/../workloads.csv";
}

bool load_case(const std::string &path, const std::string &name, int8conv_shape &shape) {
  std::ifstream file(path);
  if (!file) return false;
  std::string line;
  std::getline(file, line);  // header: name,n,h,w,c,k,r,s,pad_h,pad_w,stride_h,stride_w,dilation_h,dilation_w
  while (std::getline(file, line)) {
    std::stringstream ss(line);
    std::string cell;
    std::getline(ss, cell, ',');
    if (cell != name) continue;
    int32_t v[13];
    for (int i = 0; i < 13; ++i) {
      if (!std::getline(ss, cell, ',')) return false;
      v[i] = std::stoi(cell);
    }
    shape = int8conv_shape{v[0], v[1], v[2], v[3], v[4], v[5], v[6],
                           v[7], v[8], v[9], v[10], v[11], v[12]};
    return true;
  }
  return false;
}

// Dot product of one tap over C channels, compiled for several x86 levels
// (the loader picks the best one the host supports).
__attribute__((target_clones("default", "arch=x86-64-v3", "arch=x86-64-v4"))) int32_t
tap_dot(const int8_t *xp, const int8_t *wp, int c) {
  int32_t sum = 0;
  for (int i = 0; i < c; ++i) sum += int32_t(xp[i]) * int32_t(wp[i]);
  return sum;
}

// One output element by direct convolution: the loop nest of the reference's
// reference_value (conv_lab.cu:39-66).
int32_t direct_value(const int8conv_shape &s, const int8conv_dims &d, const std::vector<int8_t> &x,
                     const std::vector<int8_t> &w, const std::vector<int32_t> &b, int64_t m,
                     int k) {
  const int ox = static_cast<int>(m % d.out_w);
  const int oy = static_cast<int>((m / d.out_w) % d.out_h);
  const int64_t n = m / (static_cast<int64_t>(d.out_w) * d.out_h);
  int32_t sum = b[k];
  for (int fy = 0; fy < s.r; ++fy) {
    const int iy = oy * s.stride_h + fy * s.dilation_h - s.pad_h;
    if (iy < 0 || iy >= s.h) continue;
    for (int fx = 0; fx < s.s; ++fx) {
      const int ix = ox * s.stride_w + fx * s.dilation_w - s.pad_w;
      if (ix < 0 || ix >= s.w) continue;
      sum += tap_dot(&x[((n * s.h + iy) * s.w + ix) * s.c],
                     &w[((static_cast<int64_t>(k) * s.r + fy) * s.s + fx) * s.c], s.c);
    }
  }
  return sum;
}

// Compares the GPU output with direct convolution: every output when
// `samples` is 0 (the default; the reference checks only 2048 strided samples
// above 65536 outputs, conv_lab.cu:72-77), else the first and last output
// rows plus `samples` seeded random outputs.
// `expect` maps the int32 value and its channel to the value the epilogue
// writes (the identity for int32 output, the requantisation for int8).
bool validate_all(const int8conv_shape &s, const int8conv_dims &d,
                  const std::vector<int8_t> &x, const std::vector<int8_t> &w,
                  const std::vector<int32_t> &b, const std::vector<int32_t> &y,
                  const char *label, int threads, double &ms, long long samples,
                  const std::function<int32_t(int32_t, int)> &expect) {
  const auto t0 = std::chrono::steady_clock::now();
  std::vector<long long> first_bad(threads, -1);
  std::vector<std::thread> pool;
  std::vector<int64_t> picks;
  if (samples > 0) {
    std::mt19937_64 rng(12345);
    std::uniform_int_distribution<int64_t> pick(0, d.output_elements - 1);
    for (int k = 0; k < s.k; ++k) {
      picks.push_back(k);
      picks.push_back((d.gemm_m - 1) * s.k + k);
    }
    for (long long i = 0; i < samples; ++i) picks.push_back(pick(rng));
  }
  for (int t = 0; t < threads; ++t) {
    pool.emplace_back([&, t] {
      if (samples > 0) {
        for (size_t i = t; i < picks.size(); i += threads) {
          const int64_t idx = picks[i];
          const int k = static_cast<int>(idx % s.k);
          if (y[idx] != expect(direct_value(s, d, x, w, b, idx / s.k, k), k)) {
            first_bad[t] = idx;
            return;
          }
        }
        return;
      }
      for (int64_t m = t; m < d.gemm_m; m += threads) {
        for (int k = 0; k < s.k; ++k) {
          if (y[m * s.k + k] != expect(direct_value(s, d, x, w, b, m, k), k)) {
            first_bad[t] = m * s.k + k;
            return;
          }
        }
      }
    });
  }
  for (auto &th : pool) th.join();
  ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
  for (long long idx : first_bad) {
    if (idx >= 0) {
      std::cerr << label << " mismatch at output " << idx << ": got " << y[idx] << '\n';
      return false;
    }
  }
  return true;
}

// Per-launch device time, the reference's method (src/conv_lab.cu:88-110):
// `warmup` untimed launches, then `iterations` launches each bracketed by its
// own pair of events and completed before the next starts; the median.
// `launch(i)` runs the i-th timed launch (the buffer set it uses may rotate).
template <class Function>
float median_launch_ms(Function launch, int warmup, int iterations) {
  for (int i = 0; i < warmup; ++i) launch(i);
  check(cudaDeviceSynchronize(), "warm-up launches");
  std::vector<cudaEvent_t> marks(2 * static_cast<size_t>(iterations));
  for (auto &e : marks) check(cudaEventCreate(&e), "cudaEventCreate");
  for (int i = 0; i < iterations; ++i) {
    check(cudaEventRecord(marks[2 * i]), "cudaEventRecord");
    launch(warmup + i);
    check(cudaEventRecord(marks[2 * i + 1]), "cudaEventRecord");
    check(cudaEventSynchronize(marks[2 * i + 1]), "cudaEventSynchronize");
  }
  std::vector<float> times(iterations);
  for (int i = 0; i < iterations; ++i)
    check(cudaEventElapsedTime(&times[i], marks[2 * i], marks[2 * i + 1]), "elapsed time");
  for (auto e : marks) cudaEventDestroy(e);
  std::nth_element(times.begin(), times.begin() + iterations / 2, times.end());
  return times[iterations / 2];
}

// Launch time amortised over a CUDA graph of `count` back-to-back launches
// (launch(stream, i): the i-th, whose buffer set may rotate).
template <class Function>
float measure_graph(Function launch, int count, int replays) {
  cudaStream_t stream;
  check(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking), "stream");
  cudaGraph_t graph;
  cudaGraphExec_t exec;
  check(cudaStreamBeginCapture(stream, cudaStreamCaptureModeThreadLocal), "capture");
  for (int i = 0; i < count; ++i) launch(stream, i);
  check(cudaStreamEndCapture(stream, &graph), "end capture");
  check(cudaGraphInstantiate(&exec, graph, 0), "instantiate");
  check(cudaGraphLaunch(exec, stream), "graph warmup");
  check(cudaStreamSynchronize(stream), "graph sync");
  cudaEvent_t start, stop;
  check(cudaEventCreate(&start), "event");
  check(cudaEventCreate(&stop), "event");
  std::vector<float> samples;
  for (int r = 0; r < replays; ++r) {
    check(cudaEventRecord(start, stream), "record");
    check(cudaGraphLaunch(exec, stream), "graph launch");
    check(cudaEventRecord(stop, stream), "record");
    check(cudaEventSynchronize(stop), "sync");
    float ms = 0;
    check(cudaEventElapsedTime(&ms, start, stop), "elapsed");
    samples.push_back(ms / count);
  }
  std::sort(samples.begin(), samples.end());
  cudaEventDestroy(start);
  cudaEventDestroy(stop);
  cudaGraphExecDestroy(exec);
  cudaGraphDestroy(graph);
  cudaStreamDestroy(stream);
  return samples[samples.size() / 2];
}

std::string fmt(double v) {
  std::ostringstream os;
  os << v;
  return os.str();
}

int run_lab(int argc, char **argv) {
  Options parsed;
  try {
    parsed = parse_options(argc, argv);
  } catch (const std::exception &) {  // a non-numeric value for a numeric flag
    usage();
  }
  const Options options = parsed;
  int8conv_set_cta_pairing(options.pairing);
  int8conv_set_generic_staging(options.staging);
  const std::string config = options.config.empty() ? default_config(argv[0]) : options.config;
  int8conv_shape shape;
  if (!load_case(config, options.case_name, shape)) {
    std::cerr << "unknown case " << options.case_name << " in " << config << '\n';
    return EXIT_FAILURE;
  }
  if (options.batch > 0) shape.n = options.batch;
  int8conv_dims d;
  if (int8conv_shape_dims(&shape, &d) != INT8CONV_OK) {
    std::cerr << "invalid shape for case " << options.case_name << '\n';
    return EXIT_FAILURE;
  }

  // Seeded host inputs (conv_lab.cu:149-157); --values full uses the whole
  // int8 range and a bias in [-65536, 65536].  --values ones sets every input
  // and filter byte to 1: the same work with operands that barely toggle, to
  // show how much of a layer's time the power-managed SM clock costs on
  // random operands.
  std::mt19937 rng(options.seed);
  const bool ref_values = options.values == "reference";
  const bool ones = options.values == "ones";
  std::uniform_int_distribution<int> values(ones ? 1 : ref_values ? -4 : -128,
                                            ones ? 1 : ref_values ? 4 : 127);
  std::uniform_int_distribution<int> bias_values(ref_values ? -31 : -65536,
                                                 ref_values ? 31 : 65536);
  std::vector<int8_t> input(d.input_elements), filter(d.filter_elements);
  std::vector<int32_t> bias(shape.k);
  for (auto &v : input) v = static_cast<int8_t>(values(rng));
  for (auto &v : filter) v = static_cast<int8_t>(values(rng));
  for (auto &v : bias) v = bias_values(rng);
  // int8 epilogues: per-channel Q31 multipliers in [2^30, 2^31) and
  // exponents in [-13, -8], which spread the accumulators over int8.
  const bool int8_out = options.epilogue != "int32";
  const int layout = options.epilogue == "int8x32" ? INT8CONV_LAYOUT_NCHW_VECT_C
                                                    : INT8CONV_LAYOUT_NHWC;
  std::vector<int32_t> multiplier(shape.k), exponent(shape.k);
  std::uniform_int_distribution<int32_t> mult_values(1 << 30, 0x7fffffff);
  std::uniform_int_distribution<int32_t> exp_values(-13, -8);
  for (auto &v : multiplier) v = mult_values(rng);
  for (auto &v : exponent) v = exp_values(rng);

  // Input/output sets: one, or with --rotate-l2 enough that consecutive timed
  // launches never find their operands in L2 (the sets together span at
  // least twice the L2 size); every set holds the same input.
  const size_t out_bytes = static_cast<size_t>(d.output_elements) * (int8_out ? 1 : 4);
  const size_t set_bytes = input.size() + out_bytes;
  int l2_bytes = 0;
  {
    int dev = 0;
    check(cudaGetDevice(&dev), "cudaGetDevice");
    check(cudaDeviceGetAttribute(&l2_bytes, cudaDevAttrL2CacheSize, dev), "L2 size");
  }
  const int sets = options.rotate_l2 && set_bytes < 2 * static_cast<size_t>(l2_bytes)
                       ? static_cast<int>((2 * static_cast<size_t>(l2_bytes) + set_bytes - 1) /
                                          set_bytes)
                       : 1;
  std::vector<DeviceArray<int8_t>> d_inputs;
  std::vector<DeviceArray<int32_t>> d_outputs;
  std::vector<DeviceArray<int8_t>> d_outputs8;
  for (int i = 0; i < sets; ++i) {
    d_inputs.push_back(device_array<int8_t>(input.size()));
    d_outputs.push_back(device_array<int32_t>(int8_out ? 1 : d.output_elements));
    d_outputs8.push_back(device_array<int8_t>(int8_out ? d.output_elements : 1));
  }
  auto d_filter = device_array<int8_t>(filter.size());
  auto d_bias = device_array<int32_t>(bias.size());
  auto d_multiplier = device_array<int32_t>(shape.k);
  auto d_exponent = device_array<int32_t>(shape.k);
  check(cudaMemcpy(d_multiplier.get(), multiplier.data(), shape.k * sizeof(int32_t),
                   cudaMemcpyHostToDevice),
        "copy multipliers");
  check(cudaMemcpy(d_exponent.get(), exponent.data(), shape.k * sizeof(int32_t),
                   cudaMemcpyHostToDevice),
        "copy exponents");
  const int8conv_requant requant{d_multiplier.get(), d_exponent.get(), 0, 0, layout};
  auto expect = [&](int32_t v, int k) -> int32_t {
    return int8_out ? i8c::rq_apply(v, multiplier[k], exponent[k], 0, false) : v;
  };
  for (auto &d_input : d_inputs)
    check(cudaMemcpy(d_input.get(), input.data(), input.size(), cudaMemcpyHostToDevice),
          "copy input");
  check(cudaMemcpy(d_filter.get(), filter.data(), filter.size(), cudaMemcpyHostToDevice),
        "copy filter");
  check(cudaMemcpy(d_bias.get(), bias.data(), bias.size() * sizeof(int32_t),
                   cudaMemcpyHostToDevice),
        "copy bias");

  // Families to run.
  bool run[INT8CONV_NUM_STRATEGIES] = {false, false, false, false};
  if (options.strategy == "both") run[INT8CONV_GENERIC] = run[INT8CONV_STRIP] = true;
  else if (options.strategy == "all") std::fill(run, run + INT8CONV_NUM_STRATEGIES, true);
  else if (options.strategy == "auto") run[int8conv_select(&shape)] = true;
  else {
    for (int f = 0; f < INT8CONV_NUM_STRATEGIES; ++f)
      if (options.strategy == int8conv_strategy_name(f)) run[f] = true;
  }
  bool eligible[INT8CONV_NUM_STRATEGIES];
  float ms[INT8CONV_NUM_STRATEGIES], graph_ms[INT8CONV_NUM_STRATEGIES];
  bool correct[INT8CONV_NUM_STRATEGIES];
  double oracle_ms = 0;
  const int threads = std::max(1u, std::thread::hardware_concurrency());
  std::vector<int32_t> output(d.output_elements);
  for (int f = 0; f < INT8CONV_NUM_STRATEGIES; ++f) {
    eligible[f] = int8conv_eligible(&shape, f) != 0 &&
                  (layout != INT8CONV_LAYOUT_NCHW_VECT_C || !int8_out || shape.k % 32 == 0);
    ms[f] = -1.0f;
    graph_ms[f] = -1.0f;
    correct[f] = true;
    if (!run[f] || !eligible[f]) continue;
    const size_t ws_bytes = int8conv_workspace_bytes(&shape, f);
    auto workspace = device_array<uint8_t>(ws_bytes);
    // Launch number i uses buffer set i % sets.
    auto launch_on = [&](cudaStream_t stream, int i) {
      const int set = i % sets;
      const int8conv_status st =
          int8_out ? int8conv_launch_requant(f, &shape, d_inputs[set].get(), d_filter.get(),
                                             d_bias.get(), &requant, d_outputs8[set].get(),
                                             workspace.get(), ws_bytes, stream)
                   : int8conv_launch(f, &shape, d_inputs[set].get(), d_filter.get(),
                                     d_bias.get(), d_outputs[set].get(), workspace.get(),
                                     ws_bytes, stream);
      if (st != INT8CONV_OK) {
        std::cerr << int8conv_strategy_name(f) << " launch: " << int8conv_status_string(st)
                  << '\n';
        std::exit(EXIT_FAILURE);
      }
    };
    auto launch = [&](int i) { launch_on(nullptr, i); };
    if (int8_out)
      check(cudaMemset(d_outputs8[0].get(), 0xA5, d.output_elements), "poison");
    else
      check(cudaMemset(d_outputs[0].get(), 0xA5, d.output_elements * sizeof(int32_t)), "poison");
    launch(0);
    check(cudaGetLastError(), "launch");
    check(cudaDeviceSynchronize(), "synchronize");
    if (int8conv_device_status() != INT8CONV_OK) {
      std::cerr << int8conv_strategy_name(f) << ": device wait timed out\n";
      correct[f] = false;
      continue;
    }
    if (int8_out) {
      // Back to NHWK order, widened, so one validator serves every epilogue.
      std::vector<int8_t> out8(d.output_elements);
      check(cudaMemcpy(out8.data(), d_outputs8[0].get(), out8.size(), cudaMemcpyDeviceToHost),
            "copy output");
      const int64_t pq = static_cast<int64_t>(d.out_h) * d.out_w;
      for (int64_t i = 0; i < d.output_elements; ++i) {
        const int64_t m = i / shape.k;
        const int k = static_cast<int>(i % shape.k);
        const int64_t src =
            layout == INT8CONV_LAYOUT_NHWC
                ? i
                : ((m / pq * (shape.k / 32) + k / 32) * pq + m % pq) * 32 + k % 32;
        output[i] = out8[src];
      }
    } else {
      check(cudaMemcpy(output.data(), d_outputs[0].get(), output.size() * sizeof(int32_t),
                       cudaMemcpyDeviceToHost),
            "copy output");
    }
    double vms = 0;
    correct[f] = validate_all(shape, d, input, filter, bias, output,
                              int8conv_strategy_name(f), threads, vms, options.validate_samples,
                              expect);
    oracle_ms = std::max(oracle_ms, vms);
    if (!correct[f]) continue;
    ms[f] = median_launch_ms(launch, options.warmup, options.iterations);
    if (options.graph) graph_ms[f] = measure_graph(launch_on, 20, 11);
  }

  int winner = -1;
  for (int f = 0; f < INT8CONV_NUM_STRATEGIES; ++f)
    if (ms[f] >= 0 && (winner < 0 || ms[f] < ms[winner])) winner = f;
  const char *winner_name = winner < 0 ? "none" : int8conv_strategy_name(winner);
  const double ops = 2.0 * double(d.gemm_m) * double(d.gemm_n) * double(d.gemm_k);
  const double tops = winner < 0 ? -1.0 : ops / (ms[winner] * 1e-3) / 1e12;
  bool all_correct = true;
  for (int f = 0; f < INT8CONV_NUM_STRATEGIES; ++f) all_correct = all_correct && correct[f];

  if (options.csv) {
    std::cout << "case,n,h,w,c,k,r,s,out_h,out_w,eligible_strip,generic_ms,strip_ms,winner,"
                 "generic_correct,strip_correct,eligible_halo,eligible_splitk,halo_ms,splitk_ms,"
                 "halo_correct,splitk_correct,gpus,tops,roofline_frac,oracle_ms,oracle_threads,"
                 "graph_ms,selected,epilogue,l2\n";
    std::cout << options.case_name << ',' << shape.n << ',' << shape.h << ',' << shape.w << ','
              << shape.c << ',' << shape.k << ',' << shape.r << ',' << shape.s << ',' << d.out_h
              << ',' << d.out_w << ',' << (eligible[INT8CONV_STRIP] ? 1 : 0) << ','
              << ms[INT8CONV_GENERIC] << ',' << ms[INT8CONV_STRIP] << ',' << winner_name << ','
              << (correct[INT8CONV_GENERIC] ? 1 : 0) << ',' << (correct[INT8CONV_STRIP] ? 1 : 0)
              << ',' << (eligible[INT8CONV_HALO] ? 1 : 0) << ','
              << (eligible[INT8CONV_SPLITK] ? 1 : 0) << ',' << ms[INT8CONV_HALO] << ','
              << ms[INT8CONV_SPLITK] << ',' << (correct[INT8CONV_HALO] ? 1 : 0) << ','
              << (correct[INT8CONV_SPLITK] ? 1 : 0) << ",1," << fmt(tops) << ','
              << fmt(tops < 0 ? -1.0 : tops / options.peak_tops) << ',' << fmt(oracle_ms) << ','
              << threads << ',' << (winner < 0 ? -1.0f : graph_ms[winner]) << ','
              << int8conv_strategy_name(int8conv_select(&shape)) << ',' << options.epilogue
              << ',' << (options.rotate_l2 ? "rotated:" + std::to_string(sets) : std::string("warm"))
              << '\n';
  } else {
    std::cout << options.case_name << ":";
    for (int f = 0; f < INT8CONV_NUM_STRATEGIES; ++f) {
      std::cout << ' ' << int8conv_strategy_name(f) << ' ';
      if (!eligible[f]) std::cout << "ineligible";
      else if (!run[f]) std::cout << "not run";
      else if (ms[f] >= 0)
        std::cout << std::fixed << std::setprecision(4) << ms[f] << " ms";
      else std::cout << "failed";
      std::cout << (f + 1 < INT8CONV_NUM_STRATEGIES ? "," : "");
    }
    std::cout << ", winner " << winner_name;
    if (winner >= 0) std::cout << " (" << std::setprecision(1) << tops << " TOPS)";
    std::cout << '\n';
  }
  return all_correct && winner >= 0 ? 0 : 1;
}

}  // namespace

int main(int argc, char **argv) {
  try {
    return run_lab(argc, argv);
  } catch (const CudaFailure &e) {
    std::cerr << e.what() << '\n';
    return EXIT_FAILURE;
  }
}
