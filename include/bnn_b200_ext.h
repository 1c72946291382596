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

/* The cudaStream_t every call of this handle runs on (for CUDA events). */
void* bnn_b200_device_stream(BNN_Device device);

/* CUDA ordinal behind the handle. */
int bnn_b200_device_ordinal(BNN_Device device);

/* Device address of a buffer's first byte (for callers that hand device
 * pointers to their own kernels). */
void* bnn_b200_buffer_device_ptr(BNN_Buffer buffer);

#ifdef __cplusplus
}
#endif

#endif
