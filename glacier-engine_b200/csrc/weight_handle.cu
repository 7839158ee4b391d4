// Persistent INT4 weight handles: the reference's Metal persistent-weight API
// (src/backends/metal/backend.zig:571-595, shim.m:4005-4111 and 5502-5624) on
// the B200 kernels, plus device-pointer matvec / matmul, a fused LM-head
// greedy selection, and the finite-value check the executor gates on
// (glacier_all_finite_f32_neon, int4_neon.c:67-80).
//
// A context binds a device and one stream.  A weight handle owns the
// device copy of the codes, f32 scales in 16-byte aligned rows (so the
// tensor-core GEMV takes group-32 matrices), and reusable input/output
// buffers for the host-pointer dispatch, which is synchronous like the Metal
// command buffer's waitUntilCompleted.
#include <algorithm>
#include <cstring>
#include <vector>

#include "common.cuh"

namespace glacier {

size_t argmax_workspace_bytes(size_t batch, size_t n);
size_t matmul_workspace_bytes(size_t batch, size_t in_features, size_t out_features);
int int4_matmul(const Int4Weight& w, const float* x, size_t batch, const float* bias, float* y, void* workspace,
                size_t workspace_bytes, cudaStream_t st);
int argmax_rows(const float* logits, size_t ld, size_t batch, size_t n, const uint64_t* words, size_t word_count,
                glacier_argmax_result* out, int32_t* tokens, int32_t* status, void* workspace, size_t ws_bytes,
                cudaStream_t stream);

namespace {

__global__ void set_one_kernel(int32_t* r) { *r = 1; }

__global__ void all_finite_kernel(const float* __restrict__ v, size_t n, int32_t* __restrict__ r) {
  bool bad = false;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    bad |= !isfinite(v[i]);
  if (__syncthreads_or(bad) && threadIdx.x == 0) *r = 0;
}

struct DeviceBuffer {
  void* p = nullptr;
  size_t bytes = 0;
  ~DeviceBuffer() {
    if (p) cudaFree(p);
  }
  int ensure(size_t n) {
    if (bytes >= n) return GLACIER_CUDA_OK;
    if (p) cudaFree(p);
    p = nullptr;
    bytes = 0;
    if (cudaMalloc(&p, n) != cudaSuccess) {
      cudaGetLastError();
      return set_error(GLACIER_CUDA_ENOMEM, "cudaMalloc(%zu) failed", n);
    }
    bytes = n;
    return GLACIER_CUDA_OK;
  }
};

}  // namespace
}  // namespace glacier

using namespace glacier;

struct glacier_cuda_context {
  int device = 0;
  cudaStream_t stream = nullptr;
};

struct glacier_cuda_int4_weight {
  int device = 0;
  uint32_t in_f = 0, out_f = 0, group = 0;
  DeviceBuffer packed, scales, input, output, logits, argmax_ws, argmax_out, matmul_ws;
  DeviceBuffer lm_arg;  // LM-head argmax in the GEMV epilogue: winner records per 32 rows
  Int4Weight w;
};

namespace {

int bind(int device) {
  GLC_CHECK_CUDA(cudaSetDevice(device));
  return GLACIER_CUDA_OK;
}

}  // namespace

extern "C" {

glacier_cuda_context* glacier_cuda_context_create(int device_ordinal) {
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess || device_ordinal < 0 || device_ordinal >= count) {
    cudaGetLastError();
    set_error(GLACIER_CUDA_EINVAL, "context_create: device %d of %d", device_ordinal, count);
    return nullptr;
  }
  auto* ctx = new glacier_cuda_context;
  ctx->device = device_ordinal;
  if (bind(device_ordinal) || cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking) != cudaSuccess) {
    cudaGetLastError();
    set_error(GLACIER_CUDA_ECUDA, "context_create: stream creation failed");
    delete ctx;
    return nullptr;
  }
  return ctx;
}

void glacier_cuda_context_destroy(glacier_cuda_context* ctx) {
  if (!ctx) return;
  cudaSetDevice(ctx->device);
  if (ctx->stream) {
    cudaStreamSynchronize(ctx->stream);
    cudaStreamDestroy(ctx->stream);
  }
  delete ctx;
}

void* glacier_cuda_context_stream(glacier_cuda_context* ctx) { return ctx ? (void*)ctx->stream : nullptr; }

// glacier_metal_int4_weight_create_admitted (shim.m:4005-4061): the same
// admission (power-of-two group, non-empty shape, at most 2^32 elements, enough
// packed bytes and scales) and NULL on any failure.  scale_dtype 0 keeps f32
// scales (the portable numerics); 1 takes IEEE fp16 bit patterns, the
// reference's fp16 scale cache (int4_weights.zig:348-358), which also lets
// batches of 5 to 128 rows run on the tcgen05 GEMM.
glacier_cuda_int4_weight* glacier_cuda_int4_weight_create_ex(glacier_cuda_context* ctx, const uint8_t* packed,
                                                            uint64_t packed_bytes, const void* scales,
                                                            uint64_t scale_count, uint32_t scale_dtype,
                                                            uint32_t group_size, uint32_t in_features,
                                                            uint32_t out_features) {
  if (!ctx || !packed || !scales || group_size == 0 || (group_size & (group_size - 1)) || !in_features ||
      !out_features || scale_dtype > 1) {
    set_error(GLACIER_CUDA_EINVAL,
              "int4_weight_create: null argument, empty shape, non-power-of-two group or unknown scale type");
    return nullptr;
  }
  const uint64_t elements = (uint64_t)in_features * out_features;
  const uint64_t need_packed = (elements + 1) / 2, need_scales = (elements + group_size - 1) / group_size;
  if (elements > UINT32_MAX || packed_bytes < need_packed || scale_count < need_scales) {
    set_error(GLACIER_CUDA_EINVAL, "int4_weight_create: %llu packed bytes / %llu scales for %u x %u (group %u)",
              (unsigned long long)packed_bytes, (unsigned long long)scale_count, out_features, in_features,
              group_size);
    return nullptr;
  }
  if (bind(ctx->device)) return nullptr;
  auto* h = new glacier_cuda_int4_weight;
  h->device = ctx->device;
  h->in_f = in_features;
  h->out_f = out_features;
  h->group = group_size;
  Int4Weight& w = h->w;
  const size_t esz = scale_dtype ? 2 : 4;
  w.f16 = scale_dtype == 1;
  w.M = out_features;
  w.K = in_features;
  w.group = group_size;
  // Rows that hold whole groups keep one 16-byte aligned scale row per output
  // row; otherwise groups straddle rows and the scales stay one flat array.
  const bool rows = in_features % group_size == 0;
  const size_t per_row = in_features / group_size;
  const size_t stride = rows ? ceil_div(per_row * esz, (size_t)16) * 16 / esz : 0;
  const size_t scale_bytes = rows ? (size_t)out_features * stride * esz : need_scales * esz;
  bool ok = !h->packed.ensure(need_packed) && !h->scales.ensure(scale_bytes) &&
            !h->input.ensure((size_t)in_features * 4) && !h->output.ensure((size_t)out_features * 4);
  if (ok) {
    ok = cudaMemcpy(h->packed.p, packed, need_packed, cudaMemcpyHostToDevice) == cudaSuccess;
    if (scale_dtype == 1) {
      const uint16_t* hs = static_cast<const uint16_t*>(scales);
      for (uint64_t i = 0; i < need_scales && !w.nonfinite; ++i) w.nonfinite = half_bits_nonfinite(hs[i]);
    }
    if (ok && rows) {
      std::vector<uint8_t> staged((size_t)out_features * stride * esz, 0);
      const uint8_t* src = static_cast<const uint8_t*>(scales);
      for (size_t r = 0; r < out_features; ++r)
        memcpy(&staged[r * stride * esz], src + r * per_row * esz, per_row * esz);
      ok = cudaMemcpy(h->scales.p, staged.data(), scale_bytes, cudaMemcpyHostToDevice) == cudaSuccess;
    } else if (ok) {
      ok = cudaMemcpy(h->scales.p, scales, scale_bytes, cudaMemcpyHostToDevice) == cudaSuccess;
    }
    if (!ok) {
      cudaGetLastError();
      set_error(GLACIER_CUDA_ECUDA, "int4_weight_create: upload failed");
    }
  }
  if (ok) {
    w.packed = (const uint8_t*)h->packed.p;
    w.scales = h->scales.p;
    w.scale_stride = stride;
    ok = int4_weight_prepare(w) == GLACIER_CUDA_OK;
  }
  if (!ok) {
    delete h;
    return nullptr;
  }
  return h;
}

glacier_cuda_int4_weight* glacier_cuda_int4_weight_create(glacier_cuda_context* ctx, const uint8_t* packed,
                                                         uint64_t packed_bytes, const float* scales,
                                                         uint64_t scale_count, uint32_t group_size,
                                                         uint32_t in_features, uint32_t out_features) {
  return glacier_cuda_int4_weight_create_ex(ctx, packed, packed_bytes, scales, scale_count, 0, group_size,
                                            in_features, out_features);
}

void glacier_cuda_int4_weight_destroy(glacier_cuda_int4_weight* weight) {
  if (!weight) return;
  cudaSetDevice(weight->device);
  delete weight;
}

// glacier_metal_int4_matvec_dispatch (shim.m:5502-5624): host input in, the
// step runs to completion, and the result stays in the handle until
// glacier_cuda_int4_weight_read_output copies it out.  input_count and
// output_count must cover the matrix; nothing runs otherwise.
int glacier_cuda_int4_matvec_dispatch(glacier_cuda_context* ctx, glacier_cuda_int4_weight* weight,
                                      const float* input, uint64_t input_count, float* output,
                                      uint64_t output_count) {
  GLC_REQUIRE(ctx && weight && input && output, "int4_matvec_dispatch: null argument");
  GLC_REQUIRE(input_count >= weight->in_f && output_count >= weight->out_f,
              "int4_matvec_dispatch: %llu inputs / %llu outputs for %u x %u", (unsigned long long)input_count,
              (unsigned long long)output_count, weight->out_f, weight->in_f);
  GLC_REQUIRE(ctx->device == weight->device, "int4_matvec_dispatch: weight and context on different devices");
  int rc = bind(ctx->device);
  if (rc) return rc;
  GLC_CHECK_CUDA(
      cudaMemcpyAsync(weight->input.p, input, (size_t)weight->in_f * 4, cudaMemcpyHostToDevice, ctx->stream));
  if ((rc = int4_linear(weight->w, (const float*)weight->input.p, weight->in_f, 1, nullptr,
                        (float*)weight->output.p, weight->out_f, ctx->stream)))
    return rc;
  GLC_CHECK_CUDA(cudaStreamSynchronize(ctx->stream));
  return GLACIER_CUDA_OK;
}

// glacier_metal_int4_weight_read_output (shim.m:4101-4111).
int glacier_cuda_int4_weight_read_output(glacier_cuda_int4_weight* weight, float* output, uint64_t output_count) {
  GLC_REQUIRE(weight && output && output_count >= weight->out_f, "int4_weight_read_output: bad output");
  int rc = bind(weight->device);
  if (rc) return rc;
  GLC_CHECK_CUDA(cudaMemcpy(output, weight->output.p, (size_t)weight->out_f * 4, cudaMemcpyDeviceToHost));
  return GLACIER_CUDA_OK;
}

// Device-pointer forms on the caller's stream (NULL: the context-free default
// stream).  matvec is one row; matmul is `batch` rows of x (row stride ldx) into
// y (row stride ldy).
int glacier_cuda_int4_weight_matvec(glacier_cuda_int4_weight* weight, const float* x, float* y, const float* bias,
                                    void* stream) {
  GLC_REQUIRE(weight, "int4_weight_matvec: null weight");
  return int4_linear(weight->w, x, weight->in_f, 1, bias, y, weight->out_f, (cudaStream_t)stream);
}

int glacier_cuda_int4_weight_matmul(glacier_cuda_int4_weight* weight, const float* x, size_t ldx, float* y,
                                    size_t ldy, size_t batch, const float* bias, void* stream) {
  GLC_REQUIRE(weight && ldx >= weight->in_f && ldy >= weight->out_f, "int4_weight_matmul: bad strides");
  const cudaStream_t s = (cudaStream_t)stream;
  // Dense rows of more than four activations go to the tcgen05 GEMM when the
  // weight qualifies (fp16 scales, groups 8/16/32); its workspace is the handle's.
  if (batch > 4 && batch <= 128 && ldx == weight->in_f && ldy == weight->out_f && weight->w.tcg && weight->w.f16) {
    int rc = bind(weight->device);
    if (rc) return rc;
    const size_t ws = matmul_workspace_bytes(batch, weight->in_f, weight->out_f);
    if ((rc = weight->matmul_ws.ensure(ws))) return rc;
    return int4_matmul(weight->w, x, batch, bias, y, weight->matmul_ws.p, ws, s);
  }
  return int4_linear(weight->w, x, ldx, batch, bias, y, ldy, s);
}

// The LM head and its greedy selection in one call: logits = x * W^T for each
// of `batch` rows, then argmaxEligible (sampling.zig:55-107) per row with the
// optional eligibility bitsets.  logits_out may be NULL (the handle keeps a
// scratch row block).  Scratch grows on first use for a batch size and is
// reused after.
int glacier_cuda_int4_weight_lmhead_argmax(glacier_cuda_int4_weight* weight, const float* x, size_t batch,
                                           const uint64_t* eligible_words, size_t word_count, int32_t* tokens_out,
                                           int32_t* status_out, glacier_argmax_result* results_out,
                                           float* logits_out, void* stream) {
  GLC_REQUIRE(weight && x && tokens_out && batch > 0, "int4_weight_lmhead_argmax: null argument");
  int rc = bind(weight->device);
  if (rc) return rc;
  const size_t n = weight->out_f;
  const cudaStream_t s = (cudaStream_t)stream;
  if (!status_out) {
    if ((rc = weight->argmax_out.ensure(batch * 4))) return rc;
    status_out = (int32_t*)weight->argmax_out.p;
  }
  // Up to four rows on the tensor-core GEMV: the argmax runs in its epilogue and
  // no logits are written unless logits_out is given.
  if (batch <= 4 && weight->w.tc) {
    if ((rc = weight->lm_arg.ensure(argmax_records_bytes(batch, n)))) return rc;
    ArgmaxEpi ae;
    ae.words = eligible_words;
    ae.word_count = (int)word_count;
    ae.tokens = tokens_out;
    ae.status = status_out;
    ae.results = results_out;
    ae.partials = static_cast<int4*>(weight->lm_arg.p);
    if (eligible_words)
      GLC_REQUIRE(word_count == ceil_div(n, 64), "argmax: eligible mask needs %zu words per row, got %zu",
                  ceil_div(n, 64), word_count);
    rc = int4_linear_argmax(weight->w, x, weight->in_f, batch, logits_out, n, ae, s);
    if (rc != GLACIER_CUDA_EUNSUPPORTED) return rc;
  }
  float* logits = logits_out;
  if (!logits) {
    if ((rc = weight->logits.ensure(batch * n * 4))) return rc;
    logits = (float*)weight->logits.p;
  }
  const size_t ws = argmax_workspace_bytes(batch, n);
  if ((rc = weight->argmax_ws.ensure(ws))) return rc;
  if ((rc = int4_linear(weight->w, x, weight->in_f, batch, nullptr, logits, n, s))) return rc;
  return argmax_rows(logits, n, batch, n, eligible_words, word_count, results_out, tokens_out, status_out,
                     weight->argmax_ws.p, ws, s);
}

// glacier_all_finite_f32_neon (int4_neon.c:67-80) on device: *result = 1 when
// every value is finite, else 0.
int glacier_cuda_all_finite_f32(const float* values, size_t count, int32_t* result, void* stream) {
  GLC_REQUIRE(result && (values || count == 0), "all_finite: null argument");
  const cudaStream_t s = (cudaStream_t)stream;
  set_one_kernel<<<1, 1, 0, s>>>(result);
  GLC_CHECK_LAUNCH();
  if (count == 0) return GLACIER_CUDA_OK;
  const unsigned blocks = (unsigned)std::min<size_t>(ceil_div(count, (size_t)256), (size_t)4 * sm_count());
  all_finite_kernel<<<blocks, 256, 0, s>>>(values, count, result);
  GLC_CHECK_LAUNCH();
  return GLACIER_CUDA_OK;
}

}  // extern "C"
