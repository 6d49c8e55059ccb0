/*
 * conv_oracle.c - CPU INT32 convolution oracle.  TEST INFRASTRUCTURE ONLY.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg may load
 * this file's library, and only as the checker or the timed CPU baseline.  The
 * product path (int8_kernel_lab_b200, libint8conv.so) never calls it.
 *
 * Restates reference_value<Shape> of src/conv_lab.cu:39-66 of
 * pthodima/int8_kernel_lab with a runtime shape:
 *   - output index -> (batch, oy, ox, channel) as in conv_lab.cu:43-47;
 *   - sum starts at bias[channel] (conv_lab.cu:48);
 *   - for fy, for fx, for c, int32 accumulate (conv_lab.cu:49-64);
 *   - iy = oy*stride_h + fy*dilation_h - pad_h, skipped when outside [0, h)
 *     (conv_lab.cu:50-51), and the same for ix (conv_lab.cu:53-55);
 *   - X index ((batch*h + iy)*w + ix)*c + ci, W index ((k*r + fy)*s + fx)*c + ci
 *     (conv_lab.cu:57-60).
 * Unlike validate<Shape> (conv_lab.cu:68-86), which checks 2048 strided
 * samples of large outputs, callers here compute and compare every output.
 *
 * Parity is pinned by oracle/_ref (the reference's own reference_value built
 * from its sources by oracle/Makefile) and by tests/golden fixtures.
 */
#include <stddef.h>
#include <stdint.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

typedef struct oracle_shape {
  int32_t n, h, w, c, k, r, s;
  int32_t pad_h, pad_w;
  int32_t stride_h, stride_w;
  int32_t dilation_h, dilation_w;
} oracle_shape;

/* conv_shape.cuh:22-25 (C integer division, like the template). */
int32_t oracle_out_h(const oracle_shape *s) {
  return (s->h + 2 * s->pad_h - s->dilation_h * (s->r - 1) - 1) / s->stride_h + 1;
}
int32_t oracle_out_w(const oracle_shape *s) {
  return (s->w + 2 * s->pad_w - s->dilation_w * (s->s - 1) - 1) / s->stride_w + 1;
}

/* Dot product of one (fy, fx) tap: the innermost loop of conv_lab.cu:56-62.
 * Compiled for several x86 levels; the loader picks the best one the host has,
 * so the same build runs on any x86-64 host. */
__attribute__((target_clones("default", "arch=x86-64-v3", "arch=x86-64-v4")))
static int32_t tap_dot(const int8_t *x, const int8_t *w, int32_t c) {
  int32_t sum = 0;
  for (int32_t ci = 0; ci < c; ++ci) sum += (int32_t)x[ci] * (int32_t)w[ci];
  return sum;
}

/* One output element; the loop nest of conv_lab.cu:39-66. */
int32_t oracle_value(const oracle_shape *s, const int8_t *input,
                     const int8_t *filter, const int32_t *bias,
                     int64_t output_index) {
  const int32_t out_h = oracle_out_h(s), out_w = oracle_out_w(s);
  const int32_t channel = (int32_t)(output_index % s->k);
  const int64_t m = output_index / s->k;
  const int32_t ox = (int32_t)(m % out_w);
  const int32_t oy = (int32_t)((m / out_w) % out_h);
  const int64_t batch = m / ((int64_t)out_h * out_w);
  int32_t sum = bias[channel];
  for (int32_t fy = 0; fy < s->r; ++fy) {
    const int32_t iy = oy * s->stride_h + fy * s->dilation_h - s->pad_h;
    if (iy < 0 || iy >= s->h) continue;
    for (int32_t fx = 0; fx < s->s; ++fx) {
      const int32_t ix = ox * s->stride_w + fx * s->dilation_w - s->pad_w;
      if (ix < 0 || ix >= s->w) continue;
      const int8_t *x = input + (((batch * s->h + iy) * s->w + ix) * (int64_t)s->c);
      const int8_t *w = filter + ((((int64_t)channel * s->r + fy) * s->s + fx) * s->c);
      sum += tap_dot(x, w, s->c);
    }
  }
  return sum;
}

/* Output rows [m_begin, m_end) (all K channels each) into out_rows, which holds
 * (m_end - m_begin) * k int32.  `threads` <= 0 means all OpenMP threads. */
void oracle_conv_rows(const oracle_shape *s, const int8_t *input,
                      const int8_t *filter, const int32_t *bias, int64_t m_begin,
                      int64_t m_end, int32_t *out_rows, int threads) {
#ifdef _OPENMP
  if (threads <= 0) threads = omp_get_max_threads();
#pragma omp parallel for schedule(dynamic, 16) num_threads(threads)
#endif
  for (int64_t m = m_begin; m < m_end; ++m) {
    for (int32_t k = 0; k < s->k; ++k) {
      out_rows[(m - m_begin) * s->k + k] =
          oracle_value(s, input, filter, bias, m * (int64_t)s->k + k);
    }
  }
  (void)threads;
}

/* The full NHWK output. */
void oracle_conv(const oracle_shape *s, const int8_t *input, const int8_t *filter,
                 const int32_t *bias, int32_t *output, int threads) {
  const int64_t m = (int64_t)s->n * oracle_out_h(s) * oracle_out_w(s);
  oracle_conv_rows(s, input, filter, bias, 0, m, output, threads);
}

/* Selected outputs: out[i] = value at indices[i]. */
void oracle_values(const oracle_shape *s, const int8_t *input, const int8_t *filter,
                   const int32_t *bias, const int64_t *indices, int64_t count,
                   int32_t *out, int threads) {
#ifdef _OPENMP
  if (threads <= 0) threads = omp_get_max_threads();
#pragma omp parallel for schedule(static) num_threads(threads)
#endif
  for (int64_t i = 0; i < count; ++i)
    out[i] = oracle_value(s, input, filter, bias, indices[i]);
  (void)threads;
}

int oracle_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

/* ---- requantised int8 output (no reference counterpart) -------------------
 * Restates the published gemmlowp / TensorFlow Lite fixed-point requantisation
 * (SaturatingRoundingDoublingHighMul, then RoundingDivideByPOT) with plain C
 * integer division, independently of the engine's shift-based kernel code:
 *   e = clamp(exponent, -31, 31); t = e > 0 ? saturate(t * 2^e) : t
 *   u = (t*mult + (t*mult >= 0 ? 2^30 : 1 - 2^30)) / 2^31   (C division truncates)
 *       INT32_MIN * INT32_MIN -> INT32_MAX
 *   v = e < 0 ? u / 2^-e rounded half away from zero : u
 *   y = clamp(v + zero_point, relu ? zero_point : -128, 127)             */
static int32_t oracle_srdhm(int32_t a, int32_t b) {
  if (a == INT32_MIN && b == INT32_MIN) return INT32_MAX;
  const int64_t ab = (int64_t)a * (int64_t)b;
  const int64_t nudge = ab >= 0 ? ((int64_t)1 << 30) : (1 - ((int64_t)1 << 30));
  return (int32_t)((ab + nudge) / ((int64_t)1 << 31));
}

static int32_t oracle_div_pot_round(int32_t x, int e) {
  const int64_t d = (int64_t)1 << e;
  int64_t q = (int64_t)x / d;
  const int64_t r = (int64_t)x % d;
  const int64_t twice = r < 0 ? -2 * r : 2 * r;
  if (twice >= d) q += x < 0 ? -1 : 1;
  return (int32_t)q;
}

int32_t oracle_requant_value(int32_t t, int32_t multiplier, int32_t exponent,
                             int32_t zero_point, int32_t relu) {
  int e = exponent;
  if (e < -31) e = -31;
  if (e > 31) e = 31;
  if (e > 0) {
    int64_t v = (int64_t)t;
    for (int i = 0; i < e; ++i) v *= 2;
    if (v > INT32_MAX) v = INT32_MAX;
    if (v < INT32_MIN) v = INT32_MIN;
    t = (int32_t)v;
  }
  int32_t u = oracle_srdhm(t, multiplier);
  if (e < 0) u = oracle_div_pot_round(u, -e);
  int64_t y = (int64_t)u + zero_point;
  const int64_t lo = relu ? zero_point : -128;
  if (y < lo) y = lo;
  if (y > 127) y = 127;
  return (int32_t)y;
}

/* NHWK int32 (accumulator + bias, as oracle_conv returns) -> NHWK int8. */
void oracle_requant(const int32_t *acc, int64_t rows, int32_t k, const int32_t *multiplier,
                    const int32_t *exponent, int32_t zero_point, int32_t relu, int8_t *out,
                    int threads) {
#ifdef _OPENMP
  if (threads <= 0) threads = omp_get_max_threads();
#pragma omp parallel for schedule(static) num_threads(threads)
#endif
  for (int64_t m = 0; m < rows; ++m)
    for (int32_t c = 0; c < k; ++c)
      out[m * k + c] = (int8_t)oracle_requant_value(acc[m * k + c], multiplier[c], exponent[c],
                                                    zero_point, relu);
  (void)threads;
}
