/*
 * glacier_oracle.c -- CPU restatement of Glacier Engine's INT4 decode path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the CUDA
 * library and the timed CPU baseline ("port") in bench.py.  Only tests/,
 * __graft_entry__.smoke() and bench.py's cpu_baseline / --impl reference legs
 * load it.  The product path (libglacier_cuda.so) never links or calls it.
 *
 * The reference (mienetic/glacier-engine) is Zig 0.15 plus AArch64 NEON C and
 * cannot be built on this x86_64 host, so each function below restates the
 * reference's *portable* Zig path, keeping its loop structure, accumulation
 * order and operation order (separate multiply and add: compile with
 * -ffp-contract=off).  Every function cites the reference file:line it follows.
 *
 * Known, documented deviations from the reference binary:
 *   - expf/powf/cosf/sinf come from the C library instead of Zig's std.math
 *     ports; both are faithfully rounded single-precision functions.
 *   - the attention context cap of 4096 (src/forward.zig:386) is lifted so the
 *     BASELINE 7B configuration (contexts up to 4096+256) can be checked.
 */
#include <math.h>
#include <pthread.h>
#include <stddef.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define GOR_EXPORT __attribute__((visibility("default")))

/* ------------------------------------------------------------------------ */
/* quant.zig / qio.zig                                                        */
/* ------------------------------------------------------------------------ */

static size_t ceil_div(size_t n, size_t d) { return n / d + (n % d != 0); }

/* src/core/quant.zig:164-177 writeNibbleOrByte: low nibble first. */
static void write_code(uint8_t *buf, size_t idx, uint8_t val, int int4)
{
    if (!int4) { buf[idx] = val; return; }
    size_t b = idx / 2;
    if (idx % 2 == 0) buf[b] = (uint8_t)((buf[b] & 0xF0) | (val & 0x0F));
    else buf[b] = (uint8_t)((buf[b] & 0x0F) | ((val & 0x0F) << 4));
}

/* src/core/quant.zig:179-190 readNibbleOrByte. */
static uint8_t read_code(const uint8_t *buf, size_t idx, int int4)
{
    if (!int4) return buf[idx];
    uint8_t byte = buf[idx / 2];
    return (idx % 2 == 0) ? (uint8_t)(byte & 0x0F) : (uint8_t)((byte >> 4) & 0x0F);
}

/* src/core/quant.zig:36-111 quantize (f32 source).  precision: 1 = INT4, 0 = INT8.
 * packed must hold ceil(n*bits/8) bytes, scales ceil(n/group) floats.
 * Returns 0, or -1 for group 0 (error.BadGroupSize). */
GOR_EXPORT int gor_quantize(const float *src, size_t n, uint32_t group, int precision,
                            uint8_t *packed, float *scales)
{
    if (n == 0) return 0;
    if (group == 0) return -1;
    const int int4 = precision == 1;
    const int bits = int4 ? 4 : 8;
    const int32_t qzero = (1 << (bits - 1)) - 1;            /* 127 or 7 */
    const int32_t qmin = -qzero;
    const int32_t qmax = (int4 && group >= 16) ? qzero + 1 : qzero; /* quant.zig:54 */
    memset(packed, 0, ceil_div(n * (size_t)bits, 8));
    size_t elem = 0, g = 0;
    while (elem < n) {
        size_t end = elem + ((size_t)group < n - elem ? (size_t)group : n - elem);
        float min_value = 0.0f, max_value = 0.0f;
        for (size_t i = elem; i < end; ++i) {
            float fv = src[i];
            min_value = fminf(min_value, fv);
            max_value = fmaxf(max_value, fv);
        }
        const float negative_scale = -min_value / (float)(-qmin);
        const float positive_scale = max_value / (float)qmax;
        const float scale = fmaxf(negative_scale, positive_scale);
        scales[g] = scale;
        const float inv_scale = scale == 0.0f ? 0.0f : 1.0f / scale;
        for (size_t i = elem; i < end; ++i) {
            /* @round rounds half away from zero, like roundf. */
            int32_t q = (int32_t)roundf(src[i] * inv_scale);
            if (q < qmin) q = qmin;
            if (q > qmax) q = qmax;
            write_code(packed, i, (uint8_t)(q + qzero), int4);
        }
        elem = end;
        ++g;
    }
    return 0;
}

/* src/core/quant.zig:114-162 dequantize to f32.  Returns 0 or -1 (group 0). */
GOR_EXPORT int gor_dequantize(const uint8_t *packed, const float *scales, uint32_t group,
                              int precision, size_t n, float *out)
{
    if (n == 0) return 0;
    if (group == 0) return -1;
    const int int4 = precision == 1;
    const int32_t qmax = int4 ? 7 : 127; /* (1 << (bits-1)) - 1, quant.zig:129 */
    size_t i = 0, g = 0;
    while (i < n) {
        size_t end = i + ((size_t)group < n - i ? (size_t)group : n - i);
        const float scale = scales[g];
        for (size_t j = i; j < end; ++j) {
            int32_t q = (int32_t)read_code(packed, j, int4) - qmax;
            out[j] = (float)q * scale;
        }
        i = end;
        ++g;
    }
    return 0;
}

#define GOR_QIO_MAGIC 0x514F4954u /* src/model/qio.zig:27 */
#define GOR_QIO_HEADER 16u        /* src/model/qio.zig:28 */

static void put_u32(uint8_t *p, uint32_t v)
{
    p[0] = (uint8_t)v; p[1] = (uint8_t)(v >> 8); p[2] = (uint8_t)(v >> 16); p[3] = (uint8_t)(v >> 24);
}
static uint32_t get_u32(const uint8_t *p)
{
    return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}

/* Bytes encodePage would return for n elements. */
GOR_EXPORT size_t gor_qio_payload_size(size_t n, uint32_t group, int precision)
{
    if (group == 0) return 0;
    size_t bits = precision == 1 ? 4 : 8;
    return GOR_QIO_HEADER + ceil_div(n, group) * 4 + ceil_div(n * bits, 8);
}

/* src/model/qio.zig:73-113 encodePage (f32 source). Returns bytes written or 0. */
GOR_EXPORT size_t gor_qio_encode(const float *src, size_t n, uint32_t group, int precision,
                                 uint8_t *out, size_t out_cap)
{
    size_t total = gor_qio_payload_size(n, group, precision);
    if (total == 0 || out_cap < total || n > 0xFFFFFFFFu) return 0;
    size_t ngroups = ceil_div(n, group);
    put_u32(out, GOR_QIO_MAGIC);
    put_u32(out + 4, (uint32_t)n);
    put_u32(out + 8, group);
    out[12] = (uint8_t)(precision == 1 ? 1 : 0);
    out[13] = out[14] = out[15] = 0;
    float *scales = (float *)malloc(ngroups * sizeof(float) + 1);
    if (!scales) return 0;
    if (gor_quantize(src, n, group, precision, out + GOR_QIO_HEADER + ngroups * 4, scales) != 0) {
        free(scales);
        return 0;
    }
    for (size_t i = 0; i < ngroups; ++i) {
        uint32_t bitsv;
        memcpy(&bitsv, &scales[i], 4);
        put_u32(out + GOR_QIO_HEADER + i * 4, bitsv);
    }
    free(scales);
    return total;
}

/* src/model/qio.zig:49-70 readQuantHeader and :116-160 decodePage.
 * Status: 0 ok, 1 TruncatedHeader, 2 BadMagic, 3 BadGroupSize, 4 BadPrecision,
 * 5 TruncatedScales, 6 TruncatedPacked.  Header fields are written on success
 * of the header stage; out (may be NULL) receives the dequantized elements. */
GOR_EXPORT int gor_qio_decode(const uint8_t *payload, size_t len, uint32_t *num_elements,
                              uint32_t *group_size, int *precision, float *out)
{
    if (len < GOR_QIO_HEADER) return 1;
    if (get_u32(payload) != GOR_QIO_MAGIC) return 2;
    uint32_t n = get_u32(payload + 4), g = get_u32(payload + 8);
    if (g == 0) return 3;
    if (payload[12] > 1) return 4;
    int prec = payload[12];
    *num_elements = n;
    *group_size = g;
    *precision = prec;
    size_t ngroups = ceil_div(n, g);
    size_t packed_off = GOR_QIO_HEADER + ngroups * 4;
    if (len < packed_off) return 5;
    size_t packed_len = ceil_div((size_t)n * (prec == 1 ? 4 : 8), 8);
    if (len - packed_off < packed_len) return 6;
    if (!out) return 0;
    float *scales = (float *)malloc(ngroups * sizeof(float) + 1);
    if (!scales) return 7;
    for (size_t i = 0; i < ngroups; ++i) {
        uint32_t b = get_u32(payload + GOR_QIO_HEADER + i * 4);
        memcpy(&scales[i], &b, 4);
    }
    gor_dequantize(payload + packed_off, scales, g, prec, n, out);
    free(scales);
    return 0;
}

/* ------------------------------------------------------------------------ */
/* int4_matmul.zig: linearInt4OnTheFly (FP32 activations)                    */
/* ------------------------------------------------------------------------ */

/* src/backends/cpu/int4_matmul.zig:22-26 NIBBLE_TO_OFFSET */
static const float k_nibble_to_offset[16] = {-7, -6, -5, -4, -3, -2, -1, 0, 1, 2, 3, 4, 5, 6, 7, 8};

static float dequant_element(const uint8_t *packed, const float *scales, size_t idx, size_t group)
{
    /* int4_matmul.zig:3198-3207 dequantElement */
    uint8_t byte = packed[idx / 2];
    uint8_t nib = (idx & 1) == 0 ? (byte & 0x0F) : ((byte >> 4) & 0x0F);
    return k_nibble_to_offset[nib] * scales[idx / group];
}

static void load_int4x8(const uint8_t *packed, size_t off, float q[8])
{
    /* int4_matmul.zig:3220-3236 loadInt4x8 (off is even) */
    const uint8_t *b = packed + off / 2;
    for (int i = 0; i < 4; ++i) {
        q[2 * i] = k_nibble_to_offset[b[i] & 0xF];
        q[2 * i + 1] = k_nibble_to_offset[(b[i] >> 4) & 0xF];
    }
}

static float reduce8(const float v[8])
{
    /* @reduce(.Add, Vec8) restated as an ordered reduction. */
    float s = v[0];
    for (int i = 1; i < 8; ++i) s += v[i];
    return s;
}

/* One output row of linearInt4OnTheFly, int4_matmul.zig:262-301. */
static float linear_row(const float *x_row, const uint8_t *packed, const float *scales,
                        const float *bias, size_t o, size_t in_f, size_t group)
{
    float acc = bias ? bias[o] : 0.0f;
    const size_t w_row_start = o * in_f;
    if (group % 8 == 0 && w_row_start % group == 0 && in_f % group == 0) {
        /* Group-by-group Vec8 path (int4_matmul.zig:271-282). */
        float vacc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        size_t elem = 0;
        size_t group_idx = w_row_start / group;
        while (elem < in_f) {
            const size_t group_end = elem + group;
            const float scale = scales[group_idx];
            while (elem < group_end) {
                float q[8];
                load_int4x8(packed, w_row_start + elem, q);
                for (int l = 0; l < 8; ++l) {
                    float t = q[l] * x_row[elem + l];
                    t = t * scale;
                    vacc[l] = vacc[l] + t;
                }
                elem += 8;
            }
            ++group_idx;
        }
        acc += reduce8(vacc);
    } else {
        /* Generic path (int4_matmul.zig:283-300). */
        size_t elem = 0;
        while (elem + 8 <= in_f) {
            const size_t gidx = w_row_start + elem;
            const size_t gi0 = gidx / group, gi1 = (gidx + 7) / group;
            if (gidx % 2 != 0 || gi0 != gi1) {
                acc += x_row[elem] * dequant_element(packed, scales, gidx, group);
                elem += 1;
                continue;
            }
            float q[8], prod[8];
            load_int4x8(packed, gidx, q);
            for (int l = 0; l < 8; ++l) prod[l] = q[l] * x_row[elem + l];
            acc += reduce8(prod) * scales[gi0];
            elem += 8;
        }
        while (elem < in_f) {
            acc += x_row[elem] * dequant_element(packed, scales, w_row_start + elem, group);
            elem += 1;
        }
    }
    return acc;
}

static void linear_rows(const float *x, size_t batch, const uint8_t *packed, const float *scales,
                        const float *bias, float *out, size_t out_f, size_t in_f, size_t group,
                        size_t row_start, size_t row_end)
{
    for (size_t i = 0; i < batch; ++i)
        for (size_t o = row_start; o < row_end; ++o)
            out[i * out_f + o] = linear_row(x + i * in_f, packed, scales, bias, o, in_f, group);
}

/* int4_matmul.zig:215-305 linearInt4OnTheFly.  y[batch,out_f] = x[batch,in_f] W^T + bias.
 * bias may be NULL.  Returns 0, or -1 on a shape error (group 0). */
GOR_EXPORT int gor_linear_int4_f32(const float *x, size_t batch, const uint8_t *packed,
                                   const float *scales, const float *bias, float *out,
                                   size_t out_f, size_t in_f, size_t group)
{
    if (group == 0) return -1;
    linear_rows(x, batch, packed, scales, bias, out, out_f, in_f, group, 0, out_f);
    return 0;
}

typedef struct {
    const float *x; size_t batch; const uint8_t *packed; const float *scales; const float *bias;
    float *out; size_t out_f, in_f, group, start, end;
} linear_job;

static void *linear_job_run(void *p)
{
    linear_job *j = (linear_job *)p;
    linear_rows(j->x, j->batch, j->packed, j->scales, j->bias, j->out, j->out_f, j->in_f,
                j->group, j->start, j->end);
    return NULL;
}

/* int4_matmul.zig:3046-3162 linearInt4WeightParallelMode: at most 16 disjoint
 * row tasks split as out_f*t/T, bit-identical to the serial kernel.  The
 * reference uses a single-row activation (batch 1); batches > 1 split the same
 * rows across tasks here so the CPU baseline can use every host core. */
GOR_EXPORT int gor_linear_int4_f32_mt(const float *x, size_t batch, const uint8_t *packed,
                                      const float *scales, const float *bias, float *out,
                                      size_t out_f, size_t in_f, size_t group, size_t max_tasks)
{
    if (group == 0) return -1;
    size_t tasks = max_tasks < out_f ? max_tasks : out_f;
    if (tasks > 16) tasks = 16;
    if (tasks < 2) return gor_linear_int4_f32(x, batch, packed, scales, bias, out, out_f, in_f, group);
    linear_job jobs[16];
    pthread_t th[16];
    for (size_t t = 0; t < tasks; ++t) {
        size_t s = out_f * t / tasks, e = out_f * (t + 1) / tasks;
        if ((s * in_f) % 2 != 0 || (e * in_f) % 2 != 0 || (s * in_f) % group != 0 || (e * in_f) % group != 0)
            return gor_linear_int4_f32(x, batch, packed, scales, bias, out, out_f, in_f, group);
        jobs[t] = (linear_job){x, batch, packed, scales, bias, out, out_f, in_f, group, s, e};
    }
    for (size_t t = 1; t < tasks; ++t) pthread_create(&th[t], NULL, linear_job_run, &jobs[t]);
    linear_job_run(&jobs[0]);
    for (size_t t = 1; t < tasks; ++t) pthread_join(th[t], NULL);
    return 0;
}

/* ------------------------------------------------------------------------ */
/* int4_matmul.zig: Q8 activations (the reference's default decode numerics) */
/* ------------------------------------------------------------------------ */

/* Activation block of the Q8 path: 32 for group 8, else the weight group
 * (int4_matmul.zig:361, :535-538 q8ActivationScaleCount). */
GOR_EXPORT size_t gor_q8_activation_group(size_t group) { return group == 8 ? 32 : group; }

/* One row of the Q8 activation quantizer of linearInt4Q8OnTheFly
 * (int4_matmul.zig:365-394): per activation block, scale = max|x| / 127 and
 * q = clamp(round(x * (1/scale)), -127, 127), rounding half away from zero
 * (Zig @round); an all-zero block has scale 0 and q = 0. */
GOR_EXPORT void gor_q8_quantize_row(const float *x, size_t in_f, size_t group, int8_t *q, float *a_scales)
{
    const size_t ag = gor_q8_activation_group(group);
    const size_t ngroups = ceil_div(in_f, ag);
    for (size_t g = 0; g < ngroups; ++g) {
        const size_t start = g * ag, end = start + ag < in_f ? start + ag : in_f;
        float max_abs = 0.0f;
        for (size_t i = start; i < end; ++i) max_abs = fmaxf(max_abs, fabsf(x[i]));
        const float scale = max_abs / 127.0f;
        a_scales[g] = scale;
        if (scale == 0.0f) {
            memset(q + start, 0, end - start);
            continue;
        }
        const float inv = 1.0f / scale;
        for (size_t i = start; i < end; ++i) {
            long qi = (long)roundf(x[i] * inv);
            if (qi < -127) qi = -127;
            if (qi > 127) qi = 127;
            q[i] = (int8_t)qi;
        }
    }
}

/* int4_matmul.zig:335-418 linearInt4Q8OnTheFly.  Each batch row is quantized
 * independently; per output row acc starts at the bias and adds, group by
 * group in order, (float)(sum (u - 7) * q) * w_scale * a_scale.  Inputs longer
 * than 16384 or with more than 2048 activation blocks take the FP32 path
 * (:369-371).  Returns 0, or -1 on a shape error. */
GOR_EXPORT int gor_linear_int4_q8(const float *x, size_t batch, const uint8_t *packed, const float *scales,
                                  const float *bias, float *out, size_t out_f, size_t in_f, size_t group)
{
    if (group == 0 || in_f % group != 0) return -1;
    const size_t ag = gor_q8_activation_group(group);
    if (in_f > 16384 || ceil_div(in_f, ag) > 2048)
        return gor_linear_int4_f32(x, batch, packed, scales, bias, out, out_f, in_f, group);
    int8_t *q = (int8_t *)malloc(in_f);
    float *as = (float *)malloc(ceil_div(in_f, ag) * sizeof(float));
    if (!q || !as) {
        free(q);
        free(as);
        return -1;
    }
    const size_t groups = in_f / group;
    for (size_t b = 0; b < batch; ++b) {
        gor_q8_quantize_row(x + b * in_f, in_f, group, q, as);
        for (size_t row = 0; row < out_f; ++row) {
            float acc = bias ? bias[row] : 0.0f;
            const size_t row_start = row * in_f;
            for (size_t og = 0; og < groups; ++og) {
                const size_t start = og * group, end = start + group;
                int32_t dot = 0;
                for (size_t col = start; col < end; ++col) {
                    const size_t idx = row_start + col;
                    const uint8_t byte = packed[idx / 2];
                    const int32_t nib = (idx & 1) == 0 ? (byte & 0x0F) : (byte >> 4);
                    dot += (nib - 7) * (int32_t)q[col];
                }
                float t = (float)dot * scales[(row_start + start) / group];
                t = t * as[start / ag];
                acc = acc + t;
            }
            out[b * out_f + row] = acc;
        }
    }
    free(q);
    free(as);
    return 0;
}

/* int4_matmul.zig:422-532 linearInt4WeightQ8 as it dispatches on a non-AArch64
 * host: an LM-head-sized output (out_f > 65536) takes the FP32 path
 * (linearInt4Weight, :460-462), everything else linearInt4Q8OnTheFly. */
GOR_EXPORT int gor_linear_int4_weight_q8(const float *x, size_t batch, const uint8_t *packed, const float *scales,
                                         const float *bias, float *out, size_t out_f, size_t in_f, size_t group)
{
    if (out_f > 65536) return gor_linear_int4_f32(x, batch, packed, scales, bias, out, out_f, in_f, group);
    return gor_linear_int4_q8(x, batch, packed, scales, bias, out, out_f, in_f, group);
}

/* ------------------------------------------------------------------------ */
/* kernels.zig: RMSNorm, fused residual RMSNorm, SwiGLU                      */
/* ------------------------------------------------------------------------ */

static float reduce16(const float v[16])
{
    float s = v[0];
    for (int i = 1; i < 16; ++i) s += v[i];
    return s;
}

/* src/backends/cpu/kernels.zig:141-220 rmsNormF32 */
GOR_EXPORT void gor_rmsnorm_f32(const float *x, size_t batch, size_t dim, const float *weight,
                                float eps, float *out)
{
    const size_t vec_end = dim - (dim % 16);
    for (size_t i = 0; i < batch; ++i) {
        const float *row = x + i * dim;
        float sum_vec[16] = {0};
        size_t k = 0;
        for (; k < vec_end; k += 16)
            for (int l = 0; l < 16; ++l) sum_vec[l] = sum_vec[l] + row[k + l] * row[k + l];
        float sum_sq = reduce16(sum_vec);
        for (; k < dim; ++k) sum_sq += row[k] * row[k];
        const float rms = sqrtf(sum_sq / (float)dim + eps);
        const float inv = 1.0f / rms;
        for (k = 0; k < dim; ++k) out[i * dim + k] = row[k] * inv * weight[k];
    }
}

/* src/backends/cpu/kernels.zig:322-401 addRmsNormF32: residual = a + b, out = rmsnorm(residual). */
GOR_EXPORT void gor_add_rmsnorm_f32(const float *a, const float *b, float *residual, size_t batch,
                                    size_t dim, const float *weight, float eps, float *out)
{
    const size_t vec_end = dim - (dim % 16);
    for (size_t i = 0; i < batch; ++i) {
        const size_t r0 = i * dim;
        float sum_vec[16] = {0};
        size_t k = 0;
        for (; k < vec_end; k += 16)
            for (int l = 0; l < 16; ++l) {
                float v = a[r0 + k + l] + b[r0 + k + l];
                residual[r0 + k + l] = v;
                sum_vec[l] = sum_vec[l] + v * v;
            }
        float sum_sq = reduce16(sum_vec);
        for (; k < dim; ++k) {
            float v = a[r0 + k] + b[r0 + k];
            residual[r0 + k] = v;
            sum_sq += v * v;
        }
        const float rms = sqrtf(sum_sq / (float)dim + eps);
        const float inv = 1.0f / rms;
        for (k = 0; k < dim; ++k) out[r0 + k] = residual[r0 + k] * inv * weight[k];
    }
}

/* src/backends/cpu/kernels.zig:465-507 siluMulF32: out = g * (1/(1+exp(-g))) * u. */
GOR_EXPORT void gor_silu_mul_f32(const float *gate, const float *up, float *out, size_t n)
{
    for (size_t k = 0; k < n; ++k) {
        const float g = gate[k];
        const float sig = 1.0f / (1.0f + expf(-g));
        out[k] = g * sig * up[k];
    }
}

/* src/generate.zig:3642-3645 addInto */
static void add_into(float *dst, const float *a, const float *b, size_t n)
{
    for (size_t i = 0; i < n; ++i) dst[i] = a[i] + b[i];
}

/* ------------------------------------------------------------------------ */
/* generate.zig RopeTable (NeoX half-split rotary)                            */
/* ------------------------------------------------------------------------ */

/* src/generate.zig:791-808 RopeTable.init: cos/sin[positions][head_dim/2]. */
GOR_EXPORT void gor_rope_table_init(float *cos_t, float *sin_t, size_t positions, size_t head_dim,
                                    float theta)
{
    const size_t half = head_dim / 2;
    for (size_t pos = 0; pos < positions; ++pos)
        for (size_t pair = 0; pair < half; ++pair) {
            const float exponent = (float)(2 * pair) / (float)head_dim;
            const float freq = 1.0f / powf(theta, exponent);
            const float angle = (float)pos * freq;
            cos_t[pos * half + pair] = cosf(angle);
            sin_t[pos * half + pair] = sinf(angle);
        }
}

/* src/generate.zig:816-831 RopeTable.apply on one row of num_heads heads. */
GOR_EXPORT void gor_rope_apply(const float *cos_t, const float *sin_t, size_t positions, float *row,
                               size_t pos, size_t num_heads, size_t head_dim)
{
    const size_t half = head_dim / 2;
    if (pos >= positions) return;
    const size_t f = pos * half;
    for (size_t h = 0; h < num_heads; ++h) {
        const size_t off = h * head_dim;
        for (size_t p = 0; p < half; ++p) {
            const float x0 = row[off + p], x1 = row[off + p + half];
            const float c = cos_t[f + p], s = sin_t[f + p];
            row[off + p] = x0 * c - x1 * s;
            row[off + p + half] = x0 * s + x1 * c;
        }
    }
}

/* ------------------------------------------------------------------------ */
/* paged_kv_cache.zig page geometry and paged_attention.zig                   */
/* ------------------------------------------------------------------------ */

#define GOR_PAGE_POSITIONS 16 /* src/paged_kv_cache.zig:16 */

/* src/paged_kv_cache.zig:1421-1442 payloadOffset: ((layer*2 + value)*16 + row)*dim floats. */
GOR_EXPORT size_t gor_page_payload_offset(size_t layer, int value, size_t row_in_page, size_t kv_dim)
{
    return ((layer * 2 + (value ? 1 : 0)) * GOR_PAGE_POSITIONS + row_in_page) * kv_dim;
}

static float *kv_row(float *pool, size_t page_floats, const int32_t *block_table, size_t pos,
                     size_t layer, int value, size_t kv_dim)
{
    size_t page = (size_t)block_table[pos / GOR_PAGE_POSITIONS];
    return pool + page * page_floats +
           gor_page_payload_offset(layer, value, pos % GOR_PAGE_POSITIONS, kv_dim);
}

/* src/paged_kv_cache.zig:1074-1103 appendRowTxn: write k and v rows at position pos. */
GOR_EXPORT void gor_kv_append(float *pool, size_t page_floats, const int32_t *block_table, size_t pos,
                              size_t layer, size_t kv_dim, const float *k, const float *v)
{
    memcpy(kv_row(pool, page_floats, block_table, pos, layer, 0, kv_dim), k, kv_dim * sizeof(float));
    memcpy(kv_row(pool, page_floats, block_table, pos, layer, 1, kv_dim), v, kv_dim * sizeof(float));
}

/* src/paged_attention.zig:108-216 attentionMultiHead for one decode query row
 * (q_seq = 1, so attend_up_to = kv_seq - 1).  Pages hold every layer; the
 * block table maps logical page -> physical page in `pool`. */
GOR_EXPORT int gor_paged_attention(const float *q, const float *pool, size_t page_floats,
                                   const int32_t *block_table, size_t kv_seq, size_t layer,
                                   size_t num_heads, size_t num_kv_heads, size_t head_dim, float *out)
{
    const size_t eff_kv = num_kv_heads == 0 ? num_heads : num_kv_heads;
    if (kv_seq == 0 || head_dim == 0 || eff_kv == 0 || num_heads % eff_kv != 0) return -1;
    const size_t group = num_heads / eff_kv;
    const size_t kv_dim = eff_kv * head_dim;
    const float scale = 1.0f / sqrtf((float)head_dim);
    float *scores = (float *)malloc(kv_seq * sizeof(float));
    if (!scores) return -2;
    const size_t vec_end = head_dim - (head_dim % 8);
    for (size_t h = 0; h < num_heads; ++h) {
        const float *qh = q + h * head_dim;
        const size_t kv_off = (h / group) * head_dim;
        float max_score = -INFINITY;
        for (size_t j = 0; j < kv_seq; ++j) {
            const float *kh = kv_row((float *)pool, page_floats, block_table, j, layer, 0, kv_dim) + kv_off;
            float dv[8] = {0};
            size_t d = 0;
            for (; d < vec_end; d += 8)
                for (int l = 0; l < 8; ++l) dv[l] = dv[l] + qh[d + l] * kh[d + l];
            float dot = reduce8(dv);
            for (; d < head_dim; ++d) dot += qh[d] * kh[d];
            scores[j] = dot * scale;
            if (scores[j] > max_score) max_score = scores[j];
        }
        float sum_exp = 0.0f;
        for (size_t j = 0; j < kv_seq; ++j) {
            scores[j] = expf(scores[j] - max_score);
            sum_exp += scores[j];
        }
        const float inv = 1.0f / sum_exp;
        float *oh = out + h * head_dim;
        for (size_t d = 0; d < head_dim; ++d) oh[d] = 0.0f;
        for (size_t j = 0; j < kv_seq; ++j) {
            const float w = scores[j] * inv;
            const float *vh = kv_row((float *)pool, page_floats, block_table, j, layer, 1, kv_dim) + kv_off;
            for (size_t d = 0; d < head_dim; ++d) oh[d] += w * vh[d];
        }
    }
    free(scores);
    return 0;
}

/* ------------------------------------------------------------------------ */
/* sampling.zig: argmax and eligible-vocabulary argmax                        */
/* ------------------------------------------------------------------------ */

/* src/sampling.zig:194-207 argmax: strict '>' so the first maximum wins. */
GOR_EXPORT size_t gor_argmax(const float *v, size_t n)
{
    size_t best_i = 0;
    float best_v = v[0];
    for (size_t i = 1; i < n; ++i)
        if (v[i] > best_v) { best_v = v[i]; best_i = i; }
    return best_i;
}

/* src/sampling.zig:55-107 argmaxEligible.
 * Returns 0 ok, 1 InvalidEligibleMask, 2 EligibleLogitNaN. */
GOR_EXPORT int gor_argmax_eligible(const float *logits, size_t n, const uint64_t *words,
                                   size_t word_count, size_t *token_index, size_t *eligible_rows)
{
    const size_t expect = n / 64 + (n % 64 != 0);
    if (expect == 0 || word_count != expect) return 1;
    if (n % 64 != 0) {
        const uint64_t valid_tail = (((uint64_t)1) << (n % 64)) - 1;
        if (words[expect - 1] & ~valid_tail) return 1;
    }
    size_t rows = 0;
    for (size_t w = 0; w < word_count; ++w) rows += (size_t)__builtin_popcountll(words[w]);
    if (rows == 0 || rows > n) return 1;
    size_t best_index = 0;
    float best_value = 0.0f;
    int have = 0;
    for (size_t w = 0; w < word_count; ++w) {
        uint64_t rem = words[w];
        while (rem) {
            const size_t tok = w * 64 + (size_t)__builtin_ctzll(rem);
            const float v = logits[tok];
            if (isnan(v)) return 2;
            if (!have || v > best_value) { best_index = tok; best_value = v; have = 1; }
            rem &= rem - 1;
        }
    }
    *token_index = best_index;
    *eligible_rows = rows;
    return 0;
}

/* ------------------------------------------------------------------------ */
/* generate.zig: one cached decode step (forwardLayerCached + decode loop)   */
/* ------------------------------------------------------------------------ */

typedef struct {
    const uint8_t *packed; /* row-major codes, low nibble first */
    const float *scales;   /* one f32 scale per group along the flat index */
    size_t out_f, in_f, group;
} gor_int4;

typedef struct {
    gor_int4 wq, wk, wv, wo, wg, wu, wd;
    const float *bq, *bk, *bv, *bo; /* nullable */
    const float *input_norm, *post_attn_norm;
} gor_layer;

typedef struct {
    size_t num_layers, dim, hidden, num_heads, num_kv_heads, head_dim, vocab;
    float eps;
    const uint16_t *embedding_f16; /* [vocab][dim] IEEE half bits */
    const float *final_norm;
    gor_int4 lm_head;
    const gor_layer *layers;
    const float *rope_cos, *rope_sin;
    size_t rope_positions;
    size_t threads; /* row tasks per projection (1 = serial) */
} gor_model;

static float half_to_float(uint16_t h)
{
    const uint32_t sign = (uint32_t)(h & 0x8000) << 16;
    uint32_t exp = (h >> 10) & 0x1F, man = h & 0x3FF, bits;
    if (exp == 0) {
        if (man == 0) bits = sign;
        else {
            int e = -1;
            do { ++e; man <<= 1; } while ((man & 0x400) == 0);
            bits = sign | ((uint32_t)(127 - 15 - e) << 23) | ((man & 0x3FF) << 13);
        }
    } else if (exp == 31) bits = sign | 0x7F800000u | (man << 13);
    else bits = sign | ((exp + 127 - 15) << 23) | (man << 13);
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

GOR_EXPORT float gor_half_to_float(uint16_t h) { return half_to_float(h); }

static void project(const gor_model *m, const gor_int4 *w, const float *bias, const float *x, float *y)
{
    gor_linear_int4_f32_mt(x, 1, w->packed, w->scales, bias, y, w->out_f, w->in_f, w->group,
                           m->threads ? m->threads : 1);
}

/* One token through every layer, generate.zig:1511-1967 (separate MLP layout,
 * FP32 activations) with the decode-loop wrapper at generate.zig:5366-5450.
 * Writes the token's K/V rows at `pos` into the paged pool, then (if logits is
 * non-NULL) the final-norm LM-head logits.  Returns 0 or a negative error. */
GOR_EXPORT int gor_decode_token(const gor_model *m, float *pool, size_t page_floats,
                                const int32_t *block_table, size_t pos, uint32_t token, float *logits,
                                float *final_hidden)
{
    if (token >= m->vocab) return -1;
    const size_t dim = m->dim, hid = m->hidden, kv_dim = m->num_kv_heads * m->head_dim;
    const size_t q_dim = m->num_heads * m->head_dim;
    float *buf = (float *)malloc(sizeof(float) * (4 * dim + 2 * q_dim + 2 * kv_dim + 3 * hid + 8));
    if (!buf) return -2;
    float *x = buf, *h_norm = x + dim, *h = h_norm + dim, *tmp = h + dim;
    float *q = tmp + dim, *attn = q + q_dim, *k = attn + q_dim, *v = k + kv_dim;
    float *gate = v + kv_dim, *up = gate + hid, *act = up + hid;
    /* loadEmbeddingRow, generate.zig:3653-3663 (fp16 table -> f32 row). */
    for (size_t i = 0; i < dim; ++i) x[i] = half_to_float(m->embedding_f16[(size_t)token * dim + i]);
    for (size_t l = 0; l < m->num_layers; ++l) {
        const gor_layer *L = &m->layers[l];
        gor_rmsnorm_f32(x, 1, dim, L->input_norm, m->eps, h_norm);
        project(m, &L->wq, L->bq, h_norm, q);
        project(m, &L->wk, L->bk, h_norm, k);
        project(m, &L->wv, L->bv, h_norm, v);
        gor_rope_apply(m->rope_cos, m->rope_sin, m->rope_positions, k, pos, m->num_kv_heads, m->head_dim);
        gor_kv_append(pool, page_floats, block_table, pos, l, kv_dim, k, v);
        gor_rope_apply(m->rope_cos, m->rope_sin, m->rope_positions, q, pos, m->num_heads, m->head_dim);
        if (gor_paged_attention(q, pool, page_floats, block_table, pos + 1, l, m->num_heads,
                                m->num_kv_heads, m->head_dim, attn) != 0) {
            free(buf);
            return -3;
        }
        project(m, &L->wo, L->bo, attn, tmp);
        add_into(h, x, tmp, dim);
        gor_rmsnorm_f32(h, 1, dim, L->post_attn_norm, m->eps, h_norm);
        project(m, &L->wg, NULL, h_norm, gate);
        project(m, &L->wu, NULL, h_norm, up);
        gor_silu_mul_f32(gate, up, act, hid);
        project(m, &L->wd, NULL, act, tmp);
        add_into(x, h, tmp, dim);
    }
    /* Final norm + LM head, generate.zig:5452-5460 and projectLmHead :3665. */
    gor_rmsnorm_f32(x, 1, dim, m->final_norm, m->eps, h_norm);
    if (final_hidden) memcpy(final_hidden, h_norm, dim * sizeof(float));
    if (logits) project(m, &m->lm_head, NULL, h_norm, logits);
    free(buf);
    return 0;
}

/* ------------------------------------------------------------------------ */
/* progressive_int4.zig: the Prism 1 + 1 + 2-bit decomposition (research     */
/* track in the reference; scalar oracle only)                               */
/* ------------------------------------------------------------------------ */

/* progressive_int4.zig:1-12, :874-880 decomposeValidNibble: coarse 8*b3 - 4,
 * middle 4*b2 - 2, fine (u & 3) - 1; their sum is u - 7.  tier 1, 2 or 4. */
GOR_EXPORT int gor_prism_value(uint8_t nibble, int tier)
{
    const int coarse = (nibble & 8) ? 4 : -4;
    const int middle = (nibble & 4) ? 2 : -2;
    const int fine = (int)(nibble & 3) - 1;
    return tier == 1 ? coarse : tier == 2 ? coarse + middle : coarse + middle + fine;
}

/* PackedPlanes.init (progressive_int4.zig:149-184): bit i % 8 of byte i / 8 in
 * the coarse and middle planes, two-bit lane i % 4 of byte i / 4 in the fine
 * plane; padding bits zero.  Planes are sized ceil(n/8), ceil(n/8), ceil(n/4). */
GOR_EXPORT void gor_prism_split(const uint8_t *packed, size_t n, uint8_t *coarse1, uint8_t *middle1,
                                uint8_t *fine2)
{
    memset(coarse1, 0, ceil_div(n, 8));
    memset(middle1, 0, ceil_div(n, 8));
    memset(fine2, 0, ceil_div(n, 4));
    for (size_t i = 0; i < n; ++i) {
        const uint8_t u = (packed[i / 2] >> ((i & 1) * 4)) & 15;
        coarse1[i / 8] |= (uint8_t)(((u >> 3) & 1) << (i & 7));
        middle1[i / 8] |= (uint8_t)(((u >> 2) & 1) << (i & 7));
        fine2[i / 4] |= (uint8_t)((u & 3) << ((i & 3) * 2));
    }
}

/* dotAll (progressive_int4.zig:730-755): one sequential pass, per element
 * result += x * (tier_value * scale), multiply and add rounded separately. */
GOR_EXPORT void gor_prism_dot_all(const float *x, const uint8_t *packed, const float *scales, size_t n,
                                  size_t group, float out[3])
{
    float r1 = 0.f, r2 = 0.f, r4 = 0.f;
    for (size_t i = 0; i < n; ++i) {
        const uint8_t u = (packed[i / 2] >> ((i & 1) * 4)) & 15;
        const float s = scales[i / group];
        r1 += x[i] * ((float)gor_prism_value(u, 1) * s);
        r2 += x[i] * ((float)gor_prism_value(u, 2) * s);
        r4 += x[i] * ((float)gor_prism_value(u, 4) * s);
    }
    out[0] = r1;
    out[1] = r2;
    out[2] = r4;
}

/* dotP1/P2/P4PlanesUnchecked (progressive_int4.zig:1000-1041): the same
 * order over the split planes; a tier reads only the planes it needs
 * (middle1 may be NULL for tier 1, fine2 NULL below tier 4). */
GOR_EXPORT float gor_prism_dot_planes(const float *x, int tier, const uint8_t *coarse1, const uint8_t *middle1,
                                      const uint8_t *fine2, const float *scales, size_t n, size_t group)
{
    float r = 0.f;
    for (size_t i = 0; i < n; ++i) {
        const int c = (coarse1[i / 8] >> (i & 7)) & 1 ? 4 : -4;
        int v = c;
        if (tier >= 2) v += (middle1[i / 8] >> (i & 7)) & 1 ? 2 : -2;
        if (tier == 4) {
            const uint8_t u = (uint8_t)((((coarse1[i / 8] >> (i & 7)) & 1) << 3) |
                                        (((middle1[i / 8] >> (i & 7)) & 1) << 2) | ((fine2[i / 4] >> ((i & 3) * 2)) & 3));
            v = (int)u - 7; /* the integer is rebuilt before scaling (:1032-1035) */
        }
        r += x[i] * ((float)v * scales[i / group]);
    }
    return r;
}
