/*
 * bnn_b200_ext.h - extensions of libbnn_b200.so beyond the BNN_* API v2.
 *
 * None of these has a counterpart in the reference: they expose what a
 * device-resident caller (the engine in this repository, benchmarks, CUDA
 * graph capture) needs that the synchronous host API cannot give. They take
 * the same handles and follow the same validation rules as BNN_Execute.
 */
#ifndef BNN_B200_EXT_H
#define BNN_B200_EXT_H

#include "bnn_b200_accel.h"

#ifdef __cplusplus
extern "C" {
#endif

/* BNN_MatrixCreate without the 8192 in/out feature limit (the engine's
 * loader uploads lm_head's 151669 rows as one matrix). All other checks and
 * status codes are those of BNN_MatrixCreate. */
BNN_Status bnn_b200_matrix_create_unbounded(BNN_Device device, const BNN_MatrixDesc* desc,
                                            BNN_Matrix* out_matrix);

/* Validates and enqueues a job on the device's stream and returns without
 * waiting. The input check's verdict is read by bnn_b200_sync. Jobs enqueued
 * back to back share the device's scratch and run in order. */
BNN_Status bnn_b200_execute_async(BNN_Device device, const BNN_Job* job);

/* Waits for the device's stream; returns BNN_ERANGE if the last enqueued
 * job rejected its input, BNN_EIO on a CUDA failure, else BNN_OK. */
BNN_Status bnn_b200_sync(BNN_Device device);

/* The cudaStream_t every call of this handle runs on (for CUDA events). A
 * one-row job whose input no job of this handle still in flight writes may
 * read that input as soon as the previous kernel on the stream lets it start
 * (programmatic dependent launch): a kernel of the caller's own on this
 * stream that calls griddepcontrol.launch_dependents before it has finished
 * writing a job's input must not come right before that job. */
void* bnn_b200_device_stream(BNN_Device device);

/* CUDA ordinal behind the handle. */
int bnn_b200_device_ordinal(BNN_Device device);

/* Device address of a buffer's first byte (for callers that hand device
 * pointers to their own kernels). */
void* bnn_b200_buffer_device_ptr(BNN_Buffer buffer);

/* Test hook for the bounded device waits (BNN_ETIMEOUT, bnn-accelerator.h:25-26,
 * 202). No counterpart in the reference. Sets the limit after which a wait
 * inside BNN_Execute's kernels gives up (limit_ns; 0 restores the default of
 * one second) and, when starve_producer is non-zero, makes the contraction's
 * copy warps issue nothing, so the next GEMV/GEMV_F32/small-GEMM job's waits
 * for weight tiles run out and it returns BNN_ETIMEOUT without touching its
 * output. Affects every device in the process; waits for this handle's
 * stream first. Call with (0, 0) to return to normal operation. */
BNN_Status bnn_b200_test_wait_limit(BNN_Device device, uint64_t limit_ns, int starve_producer);

/* GEMM_F32 that allocates nothing. No counterpart in the reference.
 *
 * For callers that cannot let a library allocate device memory while they
 * run: programs whose framework allocator already holds the GPU's free
 * memory, or hot loops that cannot absorb cudaMalloc's implicit device-wide
 * synchronisation. BNN_Execute may cudaMalloc its per-job scratch; this call
 * uses a fixed scratch array compiled into the library instead (136 KiB on
 * every GPU that loads it, held until the process exits).
 *
 * x: device pointer to rows x in_features packed FP32 inputs; y: device
 * pointer to rows x out_features packed FP32 outputs. Same quantisation and
 * arithmetic as BNN_OP_GEMM_F32 (bit-identical results), synchronous on the
 * matrix's device. Limits: rows <= 16 and in_features <= 8192; larger jobs
 * return BNN_ERANGE without running (use BNN_Execute). Other statuses as
 * BNN_Execute: BNN_EINVAL for NULL arguments or rows == 0, BNN_ERANGE for a
 * NaN/Inf input (y untouched), BNN_ENOTSUP when the FP rounding mode is not
 * to-nearest, BNN_EIO on a CUDA failure.
 *
 * The first call on a device (after each BNN_DeviceOpen there) looks up the
 * scratch's device address (cudaGetSymbolAddress) and sets the prep kernel's
 * shared-memory limit. Every call is synchronous: it waits for its own
 * kernels on the device's stream before it returns, so no call can be
 * recorded into a CUDA graph (stream capture). After cudaDeviceReset every handle of that device is
 * dead; open a new device handle (which also renews this set-up) before the
 * next call. All calls share the one scratch array and it keeps the last
 * call's contents: calls that overlap on the GPU race and must be
 * serialised. */
BNN_Status bnn_b200_gemm_f32_noalloc(BNN_Matrix matrix, const float* x, uint32_t rows, float* y);

#ifdef __cplusplus
}
#endif

#endif
