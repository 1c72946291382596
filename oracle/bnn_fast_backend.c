/*
 * bnn_fast_backend.c - a multi-threaded CPU backend of the BNN_* API v2.
 *
 * TEST INFRASTRUCTURE ONLY. Linked with the reference engine's own sources
 * (oracle/Makefile target _ref/libbnn_engine_fast.so) it gives a reference
 * engine fast enough to check the device engine at the benchmark's full
 * Qwen3-1.7B shape (1.72 G weights per token), where the single-threaded
 * soft backend needs ~15 s per token. Never linked into the product.
 *
 * Arithmetic is that of the soft backend (bnn-accelerator/soft-bnn-accelerator.c),
 * so results are bit-identical to it:
 *   - each input row is quantised by oracle_quantize_row (QuantizeRow, soft :175-211);
 *   - the group dot pos = sum of x[k] over the set bits is exact integer
 *     arithmetic, so any summation order gives the same integer. Here it is
 *     read from a per-row table: for every weight byte position b and byte
 *     value v, T[b][v] = sum of x[8b + j] over the set bits j of v; a group
 *     of 128 weights is then 16 table reads. D = 2 pos - total (soft :251-258);
 *   - the FP32 scale-accumulate acc = fl(acc + fl(F32(scale_g) * D_g)) runs in
 *     increasing g, then Y = fl(acc * s) (soft :260-274), compiled with
 *     -ffp-contract=off like the reference;
 *   - output channels are independent, so they are split across OpenMP
 *     threads without changing any rounding.
 * Argument checks follow BNN_Execute (soft :513-603) in the same order for
 * the statuses the engine can observe. Group size 128 only (the engine's
 * Q1_0 group); other group sizes are reported as unsupported by MatrixCreate.
 * tests/test_fast_backend.py checks it against the soft backend.
 */
#include <fenv.h>
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "bnn-accelerator.h"

#ifdef __FAST_MATH__
#error "the oracle must be compiled without fast-math"
#endif

#define FAST_GROUP 128u
#define FAST_MAX_FEATURES 8192u

float oracle_half_to_float(uint16_t h);
float oracle_quantize_row(const float* x, uint32_t count, int8_t* q);

struct bnn_accel_device {
    size_t matrix_count, buffer_count;
};

struct bnn_accel_matrix {
    BNN_Device owner;
    uint32_t in_features, out_features, groups;
    uint8_t* bits;     /* [out][in/8] */
    float* scales;     /* [out][groups], binary16 already widened (exact) */
};

struct bnn_accel_buffer {
    BNN_Device owner;
    size_t bytes;
    unsigned char* data;
};

static int mul_fits(size_t a, size_t b, size_t* out) {
    if (a != 0 && b > SIZE_MAX / a)
        return 0;
    *out = a * b;
    return 1;
}

static int range_fits(size_t size, size_t offset, size_t bytes) {
    return offset <= size && bytes <= size - offset;
}

/* rows rows of row_bytes bytes, stride apart, from offset inside size bytes */
static int rows_fit(size_t size, size_t offset, size_t stride, size_t row_bytes, uint32_t rows) {
    size_t span;
    if (!mul_fits(stride, (size_t)rows - 1u, &span) || span > SIZE_MAX - row_bytes)
        return 0;
    return range_fits(size, offset, span + row_bytes);
}

BNN_Status BNN_DeviceOpen(uint32_t device_index, BNN_Device* out_device) {
    if (out_device == NULL)
        return BNN_EINVAL;
    *out_device = NULL;
    if (device_index != 0)
        return BNN_ENOTSUP;
    *out_device = calloc(1, sizeof **out_device);
    return *out_device ? BNN_OK : BNN_ENOMEM;
}

BNN_Status BNN_DeviceClose(BNN_Device device) {
    if (device == NULL)
        return BNN_EINVAL;
    if (device->matrix_count != 0 || device->buffer_count != 0)
        return BNN_EBUSY;
    free(device);
    return BNN_OK;
}

BNN_Status BNN_DeviceGetCaps(BNN_Device device, BNN_Caps* caps) {
    if (device == NULL || caps == NULL)
        return BNN_EINVAL;
    memset(caps, 0, sizeof *caps);
    caps->api_version = BNN_API_VERSION;
    caps->max_in_features = FAST_MAX_FEATURES;
    caps->max_out_features = FAST_MAX_FEATURES;
    caps->max_rows = UINT32_MAX;
    caps->group_size = FAST_GROUP;
    caps->supported_ops = BNN_CAP_GEMV | BNN_CAP_GEMM | BNN_CAP_DOT_GROUPS | BNN_CAP_GEMV_F32 | BNN_CAP_GEMM_F32;
    return BNN_OK;
}

BNN_Status BNN_MatrixCreate(BNN_Device device, const BNN_MatrixDesc* desc, BNN_Matrix* out_matrix) {
    if (out_matrix == NULL)
        return BNN_EINVAL;
    *out_matrix = NULL;
    if (device == NULL || desc == NULL || desc->weight_bits == NULL || desc->scale_fp16 == NULL)
        return BNN_EINVAL;
    if (desc->group_size != FAST_GROUP)
        return BNN_ENOTSUP;
    if (desc->in_features == 0 || desc->out_features == 0 || desc->in_features % FAST_GROUP != 0)
        return BNN_EINVAL;
    if (desc->in_features > FAST_MAX_FEATURES || desc->out_features > FAST_MAX_FEATURES)
        return BNN_ENOTSUP;
    const uint32_t groups = desc->in_features / FAST_GROUP;
    const size_t nbits = (size_t)desc->out_features * (desc->in_features / 8u);
    const size_t nscales = (size_t)desc->out_features * groups;
    if (desc->weight_bytes != nbits || desc->scale_count != nscales)
        return BNN_EINVAL;
    for (size_t i = 0; i < nscales; ++i)
        if ((desc->scale_fp16[i] & 0x7c00u) == 0x7c00u)
            return BNN_EINVAL; /* NaN / Inf scale */
    BNN_Matrix m = calloc(1, sizeof *m);
    if (m == NULL)
        return BNN_ENOMEM;
    m->bits = malloc(nbits);
    m->scales = malloc(nscales * sizeof(float));
    if (m->bits == NULL || m->scales == NULL) {
        free(m->bits);
        free(m->scales);
        free(m);
        return BNN_ENOMEM;
    }
    memcpy(m->bits, desc->weight_bits, nbits);
    for (size_t i = 0; i < nscales; ++i)
        m->scales[i] = oracle_half_to_float(desc->scale_fp16[i]);
    m->owner = device;
    m->in_features = desc->in_features;
    m->out_features = desc->out_features;
    m->groups = groups;
    ++device->matrix_count;
    *out_matrix = m;
    return BNN_OK;
}

void BNN_MatrixDestroy(BNN_Matrix m) {
    if (m == NULL)
        return;
    --m->owner->matrix_count;
    free(m->bits);
    free(m->scales);
    free(m);
}

BNN_Status BNN_BufferAlloc(BNN_Device device, size_t bytes, BNN_Buffer* out_buffer) {
    if (out_buffer == NULL)
        return BNN_EINVAL;
    *out_buffer = NULL;
    if (device == NULL || bytes == 0)
        return BNN_EINVAL;
    BNN_Buffer b = calloc(1, sizeof *b);
    if (b == NULL)
        return BNN_ENOMEM;
    b->data = malloc(bytes);
    if (b->data == NULL) {
        free(b);
        return BNN_ENOMEM;
    }
    b->owner = device;
    b->bytes = bytes;
    ++device->buffer_count;
    *out_buffer = b;
    return BNN_OK;
}

void BNN_BufferFree(BNN_Buffer b) {
    if (b == NULL)
        return;
    --b->owner->buffer_count;
    free(b->data);
    free(b);
}

BNN_Status BNN_BufferWrite(BNN_Buffer b, size_t offset, const void* src, size_t bytes) {
    if (b == NULL || (bytes != 0 && src == NULL))
        return BNN_EINVAL;
    if (!range_fits(b->bytes, offset, bytes))
        return BNN_ERANGE;
    if (bytes)
        memcpy(b->data + offset, src, bytes);
    return BNN_OK;
}

BNN_Status BNN_BufferRead(BNN_Buffer b, size_t offset, void* dst, size_t bytes) {
    if (b == NULL || (bytes != 0 && dst == NULL))
        return BNN_EINVAL;
    if (!range_fits(b->bytes, offset, bytes))
        return BNN_ERANGE;
    if (bytes)
        memcpy(dst, b->data + offset, bytes);
    return BNN_OK;
}

/* T[b][v] for the byte positions of one quantised row (see the header). */
static void build_table(const int8_t* q, uint32_t k, int16_t* table) {
    for (uint32_t b = 0; b < k / 8u; ++b) {
        int16_t* t = table + (size_t)b * 256u;
        t[0] = 0;
        for (uint32_t v = 1; v < 256; ++v)
            t[v] = (int16_t)(t[v & (v - 1u)] + q[8u * b + (uint32_t)__builtin_ctz(v)]);
    }
}

/* One quantised row against every output channel. mode 0: int16 D per
 * (n, g); 1: FP32 Z (I8 ops); 2: FP32 Z * s (F32 ops). */
static void compute_row(const struct bnn_accel_matrix* m, const int8_t* q, float s, int mode, unsigned char* out,
                        int16_t* table) {
    const uint32_t G = m->groups, k = m->in_features;
    int32_t totals[FAST_MAX_FEATURES / FAST_GROUP];
    for (uint32_t g = 0; g < G; ++g) {
        int32_t t = 0;
        for (uint32_t i = 0; i < FAST_GROUP; ++i)
            t += q[g * FAST_GROUP + i];
        totals[g] = t;
    }
    build_table(q, k, table);
    const size_t row_bytes = k / 8u;
#pragma omp parallel for schedule(static)
    for (int64_t nn = 0; nn < (int64_t)m->out_features; ++nn) {
        const uint8_t* w = m->bits + (size_t)nn * row_bytes;
        const float* sc = m->scales + (size_t)nn * G;
        float acc = 0.0f;
        for (uint32_t g = 0; g < G; ++g) {
            const int16_t* t = table + (size_t)g * 16u * 256u;
            const uint8_t* wg = w + g * 16u;
            int32_t pos = 0;
            for (uint32_t b = 0; b < 16; ++b)
                pos += t[b * 256u + wg[b]];
            const int32_t d = 2 * pos - totals[g];
            if (mode == 0) {
                const int16_t v = (int16_t)d;
                memcpy(out + ((size_t)nn * G + g) * sizeof(int16_t), &v, sizeof v);
            } else {
                const float term = sc[g] * (float)d;
                acc = acc + term;
            }
        }
        if (mode != 0) {
            const float y = mode == 2 ? acc * s : acc;
            memcpy(out + (size_t)nn * sizeof(float), &y, sizeof y);
        }
    }
}

BNN_Status BNN_Execute(BNN_Device device, const BNN_Job* job) {
    if (device == NULL || job == NULL || job->matrix == NULL || job->input.buffer == NULL ||
        job->output.buffer == NULL || job->rows == 0)
        return BNN_EINVAL;
    BNN_Type in_t, out_t;
    switch (job->operation) {
        case BNN_OP_GEMV:
        case BNN_OP_GEMM: in_t = BNN_TYPE_I8; out_t = BNN_TYPE_F32; break;
        case BNN_OP_DOT_GROUPS: in_t = BNN_TYPE_I8; out_t = BNN_TYPE_I16; break;
        case BNN_OP_GEMV_F32:
        case BNN_OP_GEMM_F32: in_t = BNN_TYPE_F32; out_t = BNN_TYPE_F32; break;
        default: return BNN_ENOTSUP;
    }
    if ((job->operation == BNN_OP_GEMV || job->operation == BNN_OP_GEMV_F32) && job->rows != 1)
        return BNN_EINVAL;
    if (job->input.type != in_t || job->output.type != out_t)
        return BNN_EINVAL;
    const struct bnn_accel_matrix* m = job->matrix;
    if (m->owner != device || job->input.buffer->owner != device || job->output.buffer->owner != device ||
        job->input.buffer == job->output.buffer)
        return BNN_EINVAL;
    const size_t in_el = in_t == BNN_TYPE_F32 ? sizeof(float) : 1u;
    const size_t in_row = (size_t)m->in_features * in_el;
    const size_t out_row = job->operation == BNN_OP_DOT_GROUPS ? (size_t)m->out_features * m->groups * 2u
                                                                : (size_t)m->out_features * 4u;
    const size_t in_stride = job->input.row_stride ? job->input.row_stride : in_row;
    const size_t out_stride = job->output.row_stride ? job->output.row_stride : out_row;
    if (in_stride < in_row || out_stride < out_row)
        return BNN_EINVAL;
    if (!rows_fit(job->input.buffer->bytes, job->input.offset, in_stride, in_row, job->rows) ||
        !rows_fit(job->output.buffer->bytes, job->output.offset, out_stride, out_row, job->rows))
        return BNN_ERANGE;
    if (job->operation != BNN_OP_DOT_GROUPS && fegetround() != FE_TONEAREST)
        return BNN_ENOTSUP;
    const unsigned char* in = job->input.buffer->data + job->input.offset;
    unsigned char* out = job->output.buffer->data + job->output.offset;
    const uint32_t K = m->in_features;
    /* every row is checked before any output is written (soft :586-592) */
    for (uint32_t r = 0; r < job->rows; ++r)
        for (uint32_t i = 0; i < K; ++i) {
            if (in_t == BNN_TYPE_F32) {
                float v;
                memcpy(&v, in + (size_t)r * in_stride + (size_t)i * 4u, 4);
                if (!isfinite(v))
                    return BNN_ERANGE;
            } else if ((int8_t)in[(size_t)r * in_stride + i] == INT8_MIN) {
                return BNN_ERANGE;
            }
        }
    int16_t* table = malloc((size_t)(K / 8u) * 256u * sizeof(int16_t));
    int8_t* q = malloc(K);
    float* xrow = malloc((size_t)K * sizeof(float));
    if (table == NULL || q == NULL || xrow == NULL) {
        free(table);
        free(q);
        free(xrow);
        return BNN_ENOMEM;
    }
    for (uint32_t r = 0; r < job->rows; ++r) {
        const unsigned char* src = in + (size_t)r * in_stride;
        unsigned char* dst = out + (size_t)r * out_stride;
        if (in_t == BNN_TYPE_F32) {
            memcpy(xrow, src, (size_t)K * 4u);
            const float s = oracle_quantize_row(xrow, K, q);
            compute_row(m, q, s, 2, dst, table);
        } else {
            memcpy(q, src, K);
            compute_row(m, q, 0.0f, job->operation == BNN_OP_DOT_GROUPS ? 0 : 1, dst, table);
        }
    }
    free(table);
    free(q);
    free(xrow);
    return BNN_OK;
}

const char* BNN_StatusString(BNN_Status status) {
    switch (status) {
        case BNN_OK: return "ok";
        case BNN_EINVAL: return "invalid argument";
        case BNN_ENOMEM: return "out of memory";
        case BNN_ENOTSUP: return "not supported";
        case BNN_ERANGE: return "out of range";
        case BNN_EBUSY: return "busy";
        case BNN_EIO: return "I/O error";
        case BNN_ETIMEOUT: return "timeout";
    }
    return "unknown status";
}
