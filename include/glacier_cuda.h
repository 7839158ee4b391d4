/*
 * glacier_cuda.h -- C ABI of the B200 (sm_100a) INT4 decode library.
 *
 * This is the drop-in boundary for Glacier Engine's native kernel seam.  The
 * reference's Zig host declares its native kernels with `extern fn` and links
 * them statically (src/backends/cpu/int4_matmul.zig:29-204,
 * src/int4_executor.zig:33-61, src/decode_lane4.zig:221-264,
 * src/sampling.zig:17) and drives its GPU backend through a persistent-weight
 * handle API (src/backends/metal/backend.zig:571-595).  Every entry point
 * below names the reference interface it replaces.
 *
 * Conventions (kept from the reference seam):
 *  - plain pointers and sizes; no framework types cross the boundary;
 *  - functions return int status: 0 = ok, negative = error; on a validation
 *    error nothing is written (validation happens before any launch, as in
 *    PreparedQ8MatvecPlan.init, int4_matmul.zig:580-635);
 *  - "device" pointers live in GPU memory of the current device; `stream` is a
 *    cudaStream_t passed as void* (NULL = legacy default stream); work is
 *    enqueued asynchronously unless the function says it synchronises;
 *  - kernels keep no global state, so concurrent calls on different streams
 *    with disjoint outputs are safe (the reference executor calls its kernels
 *    concurrently on disjoint row ranges, int4_matmul.zig:693-726).
 */
#ifndef GLACIER_CUDA_H
#define GLACIER_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GLACIER_CUDA_OK 0
#define GLACIER_CUDA_EINVAL (-1)       /* arguments rejected before any write */
#define GLACIER_CUDA_ECUDA (-2)        /* CUDA runtime / driver error */
#define GLACIER_CUDA_ENOMEM (-3)       /* device allocation failed */
#define GLACIER_CUDA_EMASK (-4)        /* sampling.zig:40 InvalidEligibleMask */
#define GLACIER_CUDA_ENAN (-5)         /* sampling.zig:41 EligibleLogitNaN */
#define GLACIER_CUDA_EUNSUPPORTED (-6) /* shape outside the kernels' contract */

/* Greedy reduction result; same 24-byte layout as glacier_argmax_result
 * (src/backends/cpu/int4_neon.c:8-19). */
typedef struct glacier_argmax_result {
  float value;
  size_t index;
  int valid;
  int saw_nan;
} glacier_argmax_result;

/* Thread-local message for the last failing call on this host thread. */
const char *glacier_cuda_last_error(void);

/* Library ABI version (major << 16 | minor). */
int glacier_cuda_version(void);

/* Device-side status word of the current device: 0 = ok, 1 = a kernel gave up
 * a bounded wait (its outputs are invalid).  Synchronises the device.  clear != 0
 * resets the word.  No reference counterpart: the reference's CPU kernels
 * cannot stall; its Metal backend reports device loss through its lifecycle
 * contract (src/core/device_loss_*.zig). */
int glacier_cuda_device_status(int clear);

/* ------------------------------------------------------------------------
 * (a) INT4 group-dequant matvec, FP32 activations, on caller device buffers.
 * packed: row-major codes, two per byte, low nibble first, zero point 7
 * (src/core/quant.zig:164-177); scales: one per group along the flat element
 * index (src/model/qio.zig:15), i.e. [out_f, in_f/group] when rows hold whole
 * groups.  bias may be NULL.  y = x * dequant(W)^T + bias.
 * ---------------------------------------------------------------------- */

/* Replaces glacier_int4_matvec_neon_f32 (src/backends/cpu/int4_matmul.zig:29-38). */
int glacier_cuda_int4_matvec_f32(const float *x, const uint8_t *packed, const float *scales,
                                 const float *bias, float *y, size_t out_features,
                                 size_t in_features, size_t group_size, void *stream);

/* Replaces glacier_int4_matvec_neon_f16scale (src/backends/cpu/int4_matmul.zig:40-49);
 * scales are IEEE binary16 bit patterns. */
int glacier_cuda_int4_matvec_f16scale(const float *x, const uint8_t *packed,
                                      const uint16_t *scales, const float *bias, float *y,
                                      size_t out_features, size_t in_features,
                                      size_t group_size, void *stream);

/* Batched form of linearInt4OnTheFly (src/backends/cpu/int4_matmul.zig:215-305):
 * x [batch, in_f] and y [batch, out_f], row-major. scale_is_f16 selects the
 * scale element type. */
int glacier_cuda_int4_linear(const float *x, size_t batch, const uint8_t *packed,
                             const void *scales, int scale_is_f16, const float *bias, float *y,
                             size_t out_features, size_t in_features, size_t group_size,
                             void *stream);

#ifdef __cplusplus
}
#endif

#endif /* GLACIER_CUDA_H */
