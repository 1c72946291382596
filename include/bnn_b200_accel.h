/*
 * bnn_b200_accel.h - the BNN_* accelerator API v2, as exported by libbnn_b200.so.
 *
 * This is the drop-in boundary. The B200 backend exports exactly the eleven
 * C functions that the reference's accelerator interface declares, with the
 * same argument meaning, status codes and ownership rules, so the reference
 * engine (bnn-sw-v2/linear.c, qwen3/, bnn-mlp/) and its CLI link against
 * this library in place of bnn-accelerator/soft-bnn-accelerator.c with no
 * source change. Types, enum values and struct layouts are kept identical
 * to bnn-accelerator/bnn-accelerator.h (an ABI requirement, checked by
 * tests/test_abi.py); the text here is this project's own.
 *
 * Numeric contract (reference bnn-accelerator/bnn-accelerator.h:121-204):
 *   weights W[n][k] in {-1,+1}, bit k of row n at byte k>>3, bit k&7, 1 = +1;
 *   one binary16 scale per (n, group of G=128 consecutive k);
 *   D[m][n][g] = sum_{k in g} Q[m][k] * W[n][k]  (exact integer);
 *   Z[m][n]    = fl(...fl(fl(F32(scale[n][0])*D0) + fl(F32(scale[n][1])*D1))...)
 *                accumulated in increasing g, each product rounded, no FMA;
 *   *_F32 ops quantize each full logical input row: a = max|x|,
 *   s = (a == 0) ? 1 : fl(a/127) (FLT_TRUE_MIN if that rounds to 0),
 *   Q = clamp(roundf(fl(x/s)), -127, 127), and return Y = fl(Z * s).
 */
#ifndef BNN_B200_ACCEL_H
#define BNN_B200_ACCEL_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Same value as the reference (bnn-accelerator.h:12): callers compiled
 * against API v2 link against this library unchanged. */
#define BNN_API_VERSION 2u

/* Opaque handles; the structs are private to the backend (bnn-accelerator.h:14-16). */
typedef struct bnn_accel_device* BNN_Device;
typedef struct bnn_accel_matrix* BNN_Matrix;
typedef struct bnn_accel_buffer* BNN_Buffer;

/* Status codes (bnn-accelerator.h:18-27). */
typedef enum {
    BNN_OK = 0,
    BNN_EINVAL = -1,   /* bad argument, handle, type or shape */
    BNN_ENOMEM = -2,   /* device or host allocation failed */
    BNN_ENOTSUP = -3,  /* unknown op, unsupported size, FP environment */
    BNN_ERANGE = -4,   /* view outside its buffer, or input value out of range */
    BNN_EBUSY = -5,    /* device still owns matrices or buffers */
    BNN_EIO = -6,      /* CUDA runtime failure (output may be partial) */
    BNN_ETIMEOUT = -7  /* device-side bounded wait expired */
} BNN_Status;

/* Operations (bnn-accelerator.h:35-41). */
typedef enum {
    BNN_OP_GEMV = 1,       /* [1][K] I8  -> [1][N] F32, Z            */
    BNN_OP_GEMM = 2,       /* [M][K] I8  -> [M][N] F32, Z            */
    BNN_OP_DOT_GROUPS = 3, /* [M][K] I8  -> [M][N][K/G] I16, D       */
    BNN_OP_GEMV_F32 = 4,   /* [1][K] F32 -> [1][N] F32, Y = Z * s    */
    BNN_OP_GEMM_F32 = 5    /* [M][K] F32 -> [M][N] F32, Y = Z * s    */
} BNN_Operation;

/* Element types of a buffer view (bnn-accelerator.h:43). */
typedef enum { BNN_TYPE_I8 = 1, BNN_TYPE_F32 = 2, BNN_TYPE_I16 = 3 } BNN_Type;

/* Capability bits; deliberately different from the operation enum
 * (bnn-accelerator.h:46-52). */
typedef enum {
    BNN_CAP_GEMV = 1u << 0,
    BNN_CAP_GEMM = 1u << 1,
    BNN_CAP_DOT_GROUPS = 1u << 2,
    BNN_CAP_GEMV_F32 = 1u << 3,
    BNN_CAP_GEMM_F32 = 1u << 4
} BNN_OperationCaps;

/* Logical limits reported by BNN_DeviceGetCaps (bnn-accelerator.h:62-69).
 * The B200 backend reports the same limits as the soft backend
 * (max_in = max_out = 8192, max_rows = UINT32_MAX, group 128, all ops):
 * callers such as linear.c chunk larger out_features themselves. */
typedef struct {
    uint32_t api_version;
    uint32_t max_in_features;
    uint32_t max_out_features;
    uint32_t max_rows;
    uint32_t group_size;
    uint32_t supported_ops;
} BNN_Caps;

/* Host description of a W1 matrix (bnn-accelerator.h:71-102).
 * weight_bits: row-major [out][in/8]; scale_fp16: row-major [out][in/G]
 * binary16 bit patterns as host uint16_t values; both arrays required and
 * sized exactly. BNN_MatrixCreate copies both to device memory (repacked
 * into the kernel's layout) before it returns. */
typedef struct {
    uint32_t in_features;
    uint32_t out_features;
    uint32_t group_size;

    const uint8_t* weight_bits;
    size_t weight_bytes;

    const uint16_t* scale_fp16;
    size_t scale_count;
} BNN_MatrixDesc;

/* Borrowed, stateless view into an untyped buffer (bnn-accelerator.h:104-119).
 * offset and row_stride are in bytes and may be unaligned; row_stride 0
 * means packed rows. */
typedef struct {
    BNN_Buffer buffer;
    BNN_Type type;
    size_t offset;
    size_t row_stride;
} BNN_BufferView;

/* One contraction job (bnn-accelerator.h:121-161). rows must be non-zero;
 * both GEMV ops require rows == 1; input and output must be different
 * buffer handles. */
typedef struct {
    BNN_Operation operation;
    BNN_Matrix matrix;
    BNN_BufferView input;
    BNN_BufferView output;
    uint32_t rows;
} BNN_Job;

/* Replaces BNN_DeviceOpen (bnn-accelerator.h:171; soft-bnn-accelerator.c:310-328).
 * device_index selects a CUDA device (remapped by the BNN_B200_DEVICE
 * environment variable, a comma-separated list of CUDA ordinals). Each
 * open returns an independent handle with its own stream and scratch. */
BNN_Status BNN_DeviceOpen(uint32_t device_index, BNN_Device* out_device);
/* Replaces BNN_DeviceClose (bnn-accelerator.h:173; soft :330-339):
 * BNN_EBUSY while matrices or buffers are alive. */
BNN_Status BNN_DeviceClose(BNN_Device device);
/* Replaces BNN_DeviceGetCaps (bnn-accelerator.h:174; soft :341-356). */
BNN_Status BNN_DeviceGetCaps(BNN_Device device, BNN_Caps* out_caps);

/* Replaces BNN_MatrixCreate (bnn-accelerator.h:176; soft :358-429). */
BNN_Status BNN_MatrixCreate(BNN_Device device, const BNN_MatrixDesc* desc, BNN_Matrix* out_matrix);
/* Replaces BNN_MatrixDestroy (bnn-accelerator.h:177; soft :431-440). NULL is a no-op. */
void BNN_MatrixDestroy(BNN_Matrix matrix);

/* Replaces BNN_BufferAlloc (bnn-accelerator.h:180; soft :442-475): device memory. */
BNN_Status BNN_BufferAlloc(BNN_Device device, size_t bytes, BNN_Buffer* out_buffer);
/* Replaces BNN_BufferFree (bnn-accelerator.h:181; soft :477-485). NULL is a no-op. */
void BNN_BufferFree(BNN_Buffer buffer);
/* Replace BNN_BufferWrite/Read (bnn-accelerator.h:188-189; soft :487-511):
 * synchronous, bounds-checked host<->device byte copies. */
BNN_Status BNN_BufferWrite(BNN_Buffer buffer, size_t offset, const void* src, size_t bytes);
BNN_Status BNN_BufferRead(BNN_Buffer buffer, size_t offset, void* dst, size_t bytes);

/* Replaces BNN_Execute (bnn-accelerator.h:205; soft :513-603). Synchronous.
 * Argument, input-value and allocation failures leave the output untouched;
 * on success only logical output elements are written. */
BNN_Status BNN_Execute(BNN_Device device, const BNN_Job* job);

/* Replaces BNN_StatusString (bnn-accelerator.h:207; soft :605-626). */
const char* BNN_StatusString(BNN_Status status);

#ifdef __cplusplus
}
#endif

#endif
