// ref_driver.cu - TEST INFRASTRUCTURE ONLY: wraps the reference's own code.
//
// Built by oracle/Makefile, only where the reference sources are present, into
// oracle/_ref/ref_<case> (git-ignored).  It compiles src/conv_lab.cu of
// pthodima/int8_kernel_lab unchanged, where it lies, with the case header that
// the reference's own scripts/gen_case.py writes, and renames its main() so
// this file can add two modes:
//
//   ref_<case> cpu IN.bin FILTER.bin BIAS.bin OUT.bin [m_begin m_end [threads [steps]]]
//       Computes output rows [m_begin, m_end) with the reference's CPU oracle
//       reference_value<TestShape> (src/conv_lab.cu:39-66), called once per
//       output element exactly as validate<Shape> does (conv_lab.cu:78), over
//       `threads` OpenMP threads, `steps` times (default 1).  Prints one JSON
//       line with the wall time of every repetition.
//   ref_<case> lab [conv_lab flags...]
//       Runs the reference's own conv_lab main (src/conv_lab.cu:246-248):
//       its mma.sync kernels built for this GPU, its validation and timing.
//
// The product never links or runs this.
#define main int8_lab_reference_conv_lab_main
#include "conv_lab.cu"
#undef main

#include <omp.h>

#include <chrono>
#include <cstdio>
#include <cstring>
#include <fstream>

namespace {

template <class T>
bool read_file(const char *path, std::vector<T> &data, size_t elements) {
  data.resize(elements);
  std::ifstream file(path, std::ios::binary);
  if (!file) return false;
  file.read(reinterpret_cast<char *>(data.data()),
            static_cast<std::streamsize>(elements * sizeof(T)));
  return static_cast<size_t>(file.gcount()) == elements * sizeof(T);
}

int cpu_mode(int argc, char **argv) {
  using Shape = TestShape;
  if (argc < 6) {
    std::fprintf(stderr, "usage: %s cpu IN FILTER BIAS OUT [m_begin m_end [threads [steps]]]\n",
                 argv[0]);
    return 2;
  }
  std::vector<int8_t> input, filter;
  std::vector<int32_t> bias;
  if (!read_file(argv[2], input, Shape::input_elements) ||
      !read_file(argv[3], filter, Shape::filter_elements) ||
      !read_file(argv[4], bias, static_cast<size_t>(Shape::k))) {
    std::fprintf(stderr, "short or missing input file\n");
    return 2;
  }
  long long m_begin = 0, m_end = Shape::gemm_m;
  int threads = omp_get_max_threads();
  if (argc >= 8) {
    m_begin = std::atoll(argv[6]);
    m_end = std::atoll(argv[7]);
  }
  if (argc >= 9) threads = std::atoi(argv[8]);
  int steps = 1;
  if (argc >= 10) steps = std::atoi(argv[9]);
  if (m_begin < 0 || m_end > Shape::gemm_m || m_begin > m_end || threads <= 0 || steps <= 0) {
    std::fprintf(stderr, "bad row range or thread count\n");
    return 2;
  }
  const size_t rows = static_cast<size_t>(m_end - m_begin);
  std::vector<int32_t> output(rows * Shape::k);
  std::vector<double> seconds;
  for (int step = 0; step < steps; ++step) {
    const auto start = std::chrono::steady_clock::now();
#pragma omp parallel for schedule(dynamic, 16) num_threads(threads)
    for (long long m = m_begin; m < m_end; ++m) {
      for (int k = 0; k < Shape::k; ++k) {
        const size_t index = static_cast<size_t>(m) * Shape::k + k;
        output[static_cast<size_t>(m - m_begin) * Shape::k + k] =
            reference_value<Shape>(input, filter, bias, index);
      }
    }
    seconds.push_back(
        std::chrono::duration<double>(std::chrono::steady_clock::now() - start).count());
  }
  std::ofstream out(argv[5], std::ios::binary);
  out.write(reinterpret_cast<const char *>(output.data()),
            static_cast<std::streamsize>(output.size() * sizeof(int32_t)));
  if (!out) {
    std::fprintf(stderr, "cannot write %s\n", argv[5]);
    return 2;
  }
  double total = 0;
  for (double t : seconds) total += t;
  const double ops = 2.0 * static_cast<double>(rows) * Shape::k * Shape::r * Shape::s * Shape::c;
  std::printf("{\"case\": \"%s\", \"rows\": %lld, \"threads\": %d, \"steps\": %d, "
              "\"seconds\": %.6f, \"gops\": %.3f, \"step_seconds\": [",
              kCaseName, static_cast<long long>(rows), threads, steps, total / steps,
              ops * steps / total / 1e9);
  for (size_t i = 0; i < seconds.size(); ++i)
    std::printf("%s%.6f", i ? ", " : "", seconds[i]);
  std::printf("]}\n");
  return 0;
}

}  // namespace

int main(int argc, char **argv) {
  if (argc >= 2 && std::strcmp(argv[1], "cpu") == 0) return cpu_mode(argc, argv);
  if (argc >= 2 && std::strcmp(argv[1], "lab") == 0) {
    argv[1] = argv[0];
    return int8_lab_reference_conv_lab_main(argc - 1, argv + 1);
  }
  std::fprintf(stderr, "usage: %s cpu ... | lab [conv_lab flags]\n", argv[0]);
  return 2;
}
