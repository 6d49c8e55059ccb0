/*
 * int8conv.h - C ABI of the B200 (sm_100a) INT8 implicit-GEMM convolution engine.
 *
 * Contract (same as the lab this replaces, README.md:6-11 of pthodima/int8_kernel_lab):
 *   input  : NHWC int8
 *   filter : KRSC int8
 *   bias   : K    int32
 *   output : NHWK int32,  output[m*K + k] = bias[k] + sum_{r,s,c} x * w
 * where m = (n*out_h + oy)*out_w + ox, and padding taps contribute nothing.
 *
 * Every entry point is plain C: plain pointers, sizes and a `void *stream` that
 * is a cudaStream_t (NULL = legacy default stream).  The caller owns all device
 * buffers; launches are asynchronous on the stream and never allocate.
 *
 * Status codes are returned instead of the reference's compile-time
 * static_asserts, so an ineligible strategy is a runtime answer
 * (INT8CONV_NOT_ELIGIBLE), not a build error.
 */
#ifndef INT8CONV_H_
#define INT8CONV_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define INT8CONV_ABI_VERSION 1

/* The 13 shape fields, in the column order of workloads.csv:1
 * (name,n,h,w,c,k,r,s,pad_h,pad_w,stride_h,stride_w,dilation_h,dilation_w).
 * Replaces the compile-time ConvShape<...> template of include/conv_shape.cuh:5-36. */
typedef struct int8conv_shape {
  int32_t n, h, w, c, k, r, s;
  int32_t pad_h, pad_w;
  int32_t stride_h, stride_w;
  int32_t dilation_h, dilation_w;
} int8conv_shape;

/* Derived quantities; formulas of include/conv_shape.cuh:22-32. */
typedef struct int8conv_dims {
  int32_t out_h, out_w;
  int64_t gemm_m; /* n * out_h * out_w */
  int64_t gemm_n; /* k */
  int64_t gemm_k; /* r * s * c */
  int64_t input_elements, filter_elements, output_elements;
} int8conv_dims;

typedef enum int8conv_status {
  INT8CONV_OK = 0,
  INT8CONV_NOT_ELIGIBLE = 1,     /* strategy's predicate rejects the shape */
  INT8CONV_BAD_SHAPE = 2,        /* conv_shape.cuh:34-35 checks, or a non-positive field */
  INT8CONV_BAD_POINTER = 3,      /* NULL, or not 16-byte aligned */
  INT8CONV_CUDA_ERROR = 4,       /* a CUDA runtime/driver call failed */
  INT8CONV_DEVICE_TIMEOUT = 5,   /* a bounded device wait gave up (see int8conv_device_status) */
  INT8CONV_WORKSPACE_TOO_SMALL = 6,
  INT8CONV_UNSUPPORTED_DEVICE = 7, /* not an sm_100 device */
  INT8CONV_BAD_ARGUMENT = 8
} int8conv_status;

/* Kernel families.  GENERIC and STRIP mirror launch_generic / launch_spatial_strip
 * (include/generic_implicit_gemm.cuh:155-165, include/spatial_strip.cuh:289-301);
 * HALO and SPLITK have no counterpart in the reference. */
typedef enum int8conv_strategy {
  INT8CONV_GENERIC = 0,
  INT8CONV_STRIP = 1,
  INT8CONV_HALO = 2,
  INT8CONV_SPLITK = 3,
  INT8CONV_AUTO = 100 /* dispatch policy: int8conv_select() */
} int8conv_strategy;

#define INT8CONV_NUM_STRATEGIES 4

/* ---- shape algebra (host only, no GPU needed) ---------------------------- */

/* 1 if the shape passes conv_shape.cuh:34-35 (c % 16 == 0, non-empty output)
 * and every field is in range; 0 otherwise. */
int int8conv_shape_valid(const int8conv_shape *shape);

/* Fills *dims (conv_shape.cuh:22-32).  INT8CONV_BAD_SHAPE if invalid. */
int8conv_status int8conv_shape_dims(const int8conv_shape *shape, int8conv_dims *dims);

/* Capability predicate of one family (spatial_strip.cuh:11-15 is the
 * reference's only one).  1 = the family's kernel computes this shape. */
int int8conv_eligible(const int8conv_shape *shape, int strategy);

/* Family chosen by the B200 dispatch policy (always an eligible one). */
int int8conv_select(const int8conv_shape *shape);

/* Device scratch a launch of `strategy` needs, in bytes (0 for most). */
size_t int8conv_workspace_bytes(const int8conv_shape *shape, int strategy);

const char *int8conv_strategy_name(int strategy);
const char *int8conv_status_string(int status);
int int8conv_abi_version(void);

/* ---- launches --------------------------------------------------------------*/

/* Launch one family (or INT8CONV_AUTO) on `stream`.  `workspace` may be NULL
 * when int8conv_workspace_bytes() is 0.  Asynchronous: errors inside the
 * kernel surface on the next synchronisation, and device wait timeouts via
 * int8conv_device_status(). */
int8conv_status int8conv_launch(int strategy, const int8conv_shape *shape,
                                const int8_t *input, const int8_t *filter,
                                const int32_t *bias, int32_t *output,
                                void *workspace, size_t workspace_bytes,
                                void *stream);

/* launch_generic<Shape>(input, filter, bias, output, stream)
 * (include/generic_implicit_gemm.cuh:155-165; also stands in for
 * launch_generic_sm80, :229-238). */
int8conv_status int8conv_launch_generic(const int8conv_shape *shape,
                                        const int8_t *input, const int8_t *filter,
                                        const int32_t *bias, int32_t *output,
                                        void *stream);

/* launch_spatial_strip<Shape>(...) (include/spatial_strip.cuh:289-301). */
int8conv_status int8conv_launch_spatial_strip(const int8conv_shape *shape,
                                              const int8_t *input, const int8_t *filter,
                                              const int32_t *bias, int32_t *output,
                                              void *stream);

/* No reference counterpart: small-spatial layers. */
int8conv_status int8conv_launch_halo(const int8conv_shape *shape,
                                     const int8_t *input, const int8_t *filter,
                                     const int32_t *bias, int32_t *output,
                                     void *stream);

/* No reference counterpart: the R*S*C reduction split across a CTA cluster. */
int8conv_status int8conv_launch_splitk(const int8conv_shape *shape,
                                       const int8_t *input, const int8_t *filter,
                                       const int32_t *bias, int32_t *output,
                                       void *workspace, size_t workspace_bytes,
                                       void *stream);

/* ---- requantised int8 output ---------------------------------------------------*/

/* Output layouts of the requantised launch. */
typedef enum int8conv_layout {
  INT8CONV_LAYOUT_NHWC = 0,        /* int8 [N][out_h][out_w][K]: the next layer's input layout */
  INT8CONV_LAYOUT_NCHW_VECT_C = 1  /* cuDNN INT8x32: int8 [N][K/32][out_h][out_w][32], K % 32 == 0 */
} int8conv_layout;

/* Per-output-channel fixed-point scaling (gemmlowp / TensorFlow Lite
 * "quantized multiplier").  With t = output[m*K + k] of the int32 contract
 * (accumulator + bias, two's-complement):
 *   e = clamp(exponent[k], -31, 31)
 *   t = e > 0 ? saturate_int32(t * 2^e) : t
 *   u = (t * multiplier[k] + nudge) / 2^31    truncating division; nudge = 2^30 for
 *                                             t * multiplier >= 0, else 1 - 2^30;
 *                                             INT32_MIN * INT32_MIN gives INT32_MAX
 *   v = e < 0 ? u / 2^-e rounded half away from zero : u
 *   y = clamp(v + zero_point, relu ? zero_point : -128, 127)
 * multiplier = 2^30, exponent = 1 gives y = clamp(t, -128, 127), the int8
 * output of cuDNN's INT8x32 convolution with alpha = 1, beta = 0 (the
 * reference's cuDNN comparison, include/cudnn_legacy.cuh:51-55). */
typedef struct int8conv_requant {
  const int32_t *multiplier; /* K entries, device memory, 16-byte aligned */
  const int32_t *exponent;   /* K entries, device memory, 16-byte aligned */
  int32_t zero_point;        /* in [-128, 127] */
  int32_t relu;              /* 0 or 1: fused ReLU (clamp below at zero_point) */
  int32_t layout;            /* int8conv_layout */
} int8conv_requant;

/* Launch one family (or INT8CONV_AUTO) with the int8 epilogue above instead
 * of the int32 output: `output` receives N*out_h*out_w*K int8 values in
 * `requant->layout`.  No reference counterpart (the reference writes int32
 * only; its cuDNN baseline writes INT8x32).  NOT_ELIGIBLE for
 * INT8CONV_LAYOUT_NCHW_VECT_C when K % 32 != 0; BAD_ARGUMENT for a zero point,
 * relu flag or layout out of range; BAD_POINTER for a NULL or misaligned
 * multiplier / exponent array. */
int8conv_status int8conv_launch_requant(int strategy, const int8conv_shape *shape,
                                        const int8_t *input, const int8_t *filter,
                                        const int32_t *bias, const int8conv_requant *requant,
                                        int8_t *output, void *workspace,
                                        size_t workspace_bytes, void *stream);

/* ---- host buffers ------------------------------------------------------------*/

/* End-to-end convolution of HOST buffers (no reference counterpart; the
 * reference copies synchronously around each launch, src/conv_lab.cu:163-168,
 * :190-192).  Copies the filter and bias, then streams the batch through the
 * GPU in `chunks` groups of whole images: the host->device copy of group i+1,
 * the convolution of group i and the device->host copy of group i-1 overlap
 * on separate streams.  The device buffers are the caller's and hold the full
 * tensors; pinned host memory is needed for the copies to overlap.  Returns
 * after enqueueing: `stream` waits for every copy and launch, so synchronising
 * it (or any later work on it) sees the finished host output.  The chunk
 * launches run strategy `strategy` (or the dispatch policy for INT8CONV_AUTO)
 * on each group's shape.  On an error after the first copy was queued, the
 * call first waits for the copies and launches it already queued, so the
 * host buffers are no longer in use when it returns. */
int8conv_status int8conv_launch_host(int strategy, const int8conv_shape *shape,
                                     const int8_t *host_input, const int8_t *host_filter,
                                     const int32_t *host_bias, int32_t *host_output,
                                     int8_t *dev_input, int8_t *dev_filter,
                                     int32_t *dev_bias, int32_t *dev_output,
                                     int chunks, void *stream);

/* ---- device status ---------------------------------------------------------*/

/* Synchronises the current device and returns INT8CONV_DEVICE_TIMEOUT if any
 * kernel of this library gave up a bounded wait since the last call (then
 * clears the flag), INT8CONV_CUDA_ERROR on a sticky CUDA error, else OK. */
int8conv_status int8conv_device_status(void);

/* Device wait limit in nanoseconds for launches on the calling thread's
 * current device (default 2e9).  Tests shorten it. */
void int8conv_set_wait_limit_ns(uint64_t ns);

/* Test hook for failure detection: when `on` is nonzero the next launches skip
 * issuing their global->shared copies, so the consumer waits run out and the
 * kernel returns with INT8CONV_DEVICE_TIMEOUT recorded.  Nothing is left in
 * flight and the context stays usable. */
void int8conv_debug_starve_producer(int on);

/* CTA pairing of the GENERIC and STRIP kernels (process-wide):
 * 0 = automatic (pairs of CTAs sharing one 256-row tensor-core tile through
 * tcgen05 cta_group::2 when the problem has enough tiles to fill the GPU),
 * 1 = single CTAs only, 2 = pairs whenever the shape allows.  Every mode
 * computes identical results; the choice only moves performance. */
int8conv_status int8conv_set_cta_pairing(int mode);

/* Activation staging of GENERIC (process-wide): 0 = automatic (the TMA
 * im2col tensor map wherever it can encode the shape, else the gather warp),
 * 1 = the gather warp for every shape.  Both compute identical results; the
 * gather exists for shapes beyond the im2col limits (stride > 8, pad > 127,
 * (R-1)*dilation > 127), and forcing it lets tests compare the two stagings
 * on any shape. */
int8conv_status int8conv_set_generic_staging(int mode);

/* Number of kernels this library has launched in this process. */
uint64_t int8conv_launch_count(void);

#ifdef __cplusplus
}
#endif

#endif /* INT8CONV_H_ */
