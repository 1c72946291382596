// bnn_internal.h - private handle layouts shared by the C-ABI translation units.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

#include "bnn_b200_accel.h"

struct bnn_accel_device {
    int ordinal;              // CUDA device ordinal
    int sm_count;             // streaming multiprocessors of that device
    cudaStream_t stream;      // every call of this handle runs on it, then syncs
    size_t matrix_count;
    size_t buffer_count;
    // Per-job scratch: sliced int8 activations, group totals, row scales.
    void* scratch;
    size_t scratch_bytes;
    int* d_status;            // [0] verdict of prep + contraction jobs (reset per job);
                              // [1], [2] verdicts of single-kernel jobs, used in turn:
                              // each such job clears the other slot for the next one,
                              // so no reset sits between two of them and the next
                              // job's launch overlaps this one's tail (PDL)
    int* h_status;            // pinned host mirror
    int* last_status;         // the verdict word of the last enqueued job
    uint32_t single_jobs;     // single-kernel jobs enqueued (picks the slot)
    // Output byte ranges [begin, end) of the jobs enqueued since the stream
    // was last drained: a single-kernel job whose input meets none of them
    // reads it before its grid-dependency wait (GemvArgs::early_input).
    static constexpr uint32_t kMaxInflightOutputs = 256;
    uintptr_t inflight_out[kMaxInflightOutputs][2];
    uint32_t inflight_count;
    bool inflight_overflow;   // more outputs than the table holds: no early reads until drained
};

struct bnn_accel_matrix {
    BNN_Device owner;
    uint32_t in_features;
    uint32_t out_features;
    uint32_t groups;
    unsigned char* wblocks;   // packed 8-row blocks: sign bits + scales (w1a8_gemv.cuh)
};

struct bnn_accel_buffer {
    BNN_Device owner;
    size_t bytes;
    unsigned char* data;      // device memory
};

// A matrix of in x out features whose packed blocks are zero (every bit -1,
// every scale +0); the caller fills them on the device (the engine's Q1_0
// loader). Counts towards the device's matrices like BNN_MatrixCreate.
extern "C" BNN_Status bnn_b200_matrix_alloc(BNN_Device device, uint32_t in_features, uint32_t out_features,
                                            BNN_Matrix* out_matrix);

// Drops the allocation-free GEMM's cached per-device set-up (bnn_noalloc.cu);
// BNN_DeviceOpen calls it so a re-created device context is set up afresh.
void bnn_noalloc_forget(int ordinal);

namespace bnn {

// Makes `ordinal` current for the lifetime of the guard, restoring the
// caller's device afterwards.
class DeviceGuard {
  public:
    explicit DeviceGuard(int ordinal) {
        ok_ = cudaGetDevice(&prev_) == cudaSuccess && cudaSetDevice(ordinal) == cudaSuccess;
    }
    ~DeviceGuard() {
        if (prev_ >= 0)
            cudaSetDevice(prev_);
    }
    bool ok() const { return ok_; }

  private:
    int prev_ = -1;
    bool ok_ = false;
};

// The kernels' test hooks (the wait limit and the starved copy producer,
// bnn_sync.cuh and w1a8_gemv.cuh) are device globals, one copy per
// translation unit. The contraction templates are instantiated in several
// units and the host link keeps one launch stub of each, so a launch may run
// another unit's instance: bnn_b200_test_wait_limit sets every unit's copy.
cudaError_t set_test_hooks_engine(unsigned long long limit_ns, int starve);
cudaError_t set_test_hooks_noalloc(unsigned long long limit_ns, int starve);

}  // namespace bnn
