// bnn_noalloc.cu - GEMM_F32 for callers that cannot allocate device memory.
//
// BNN_Execute keeps its per-job scratch (the quantised, re-sliced input rows,
// their group totals and scales, and a status word) in memory that the
// device handle cudaMalloc's and grows on demand. Some callers cannot let a
// library allocate while they run: a host framework whose caching allocator
// already owns the free device memory (a fresh cudaMalloc can then fail even
// though the framework has room), or a latency-critical loop that cannot take
// cudaMalloc's implicit device-wide synchronisation. bnn_b200_gemm_f32_noalloc
// serves them: the same prep + contraction kernels, with the scratch in the
// fixed array below, which is part of the library image and exists on every
// GPU that loads libbnn_b200.so until the process exits.
//
// Limits: rows <= kNoAllocMaxRows (16) and in_features <= kNoAllocMaxK (8192),
// i.e. 16 * 8192 B of sliced int8 activations + 16 * 64 * 4 B of totals +
// 16 row scales + the status word: 136 KiB of device memory per GPU.
// Every call uses the same array, so calls that overlap on the GPU (from two
// host threads, or two devices' handles of the same GPU used concurrently)
// race on it; like all BNN_* calls on a device, callers must serialise them.
// Each call is synchronous: it waits for its own kernels before returning.
#include <cfenv>
#include <cstring>
#include <mutex>

#include "bnn_b200_ext.h"
#include "bnn_internal.h"
#include "w1a8_prep.cuh"

namespace {

constexpr uint32_t kNoAllocMaxRows = 16;
constexpr uint32_t kNoAllocMaxK = 8192;
constexpr size_t kActBytes = (size_t)kNoAllocMaxRows * kNoAllocMaxK;                 // sliced int8 rows
constexpr size_t kTotBytes = (size_t)kNoAllocMaxRows * (kNoAllocMaxK / 128) * 4;     // group totals
constexpr size_t kScaleOffset = kActBytes + kTotBytes;                               // row scales
constexpr size_t kStatusOffset = kScaleOffset + 256;                                 // status word
constexpr size_t kScratchBytes = kStatusOffset + 256;

// The scratch itself. In host code this name is only a stand-in for the
// symbol; the device address is obtained per device with cudaGetSymbolAddress.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_setup_mutex;
void* g_scratch_addr[kMaxDevices] = {};

// Per-device set-up, run by the first call on `ordinal` (the current device):
// the scratch's device address (cudaGetSymbolAddress) and the prep kernel's
// shared-memory limit, both checked. BNN_DeviceOpen forgets the entry
// (bnn_noalloc_forget), so a process that reset the device and opened a new
// handle looks the address up again instead of using a stale one.
BNN_Status scratch_setup(int ordinal, unsigned char** out) {
    if (ordinal < 0 || ordinal >= kMaxDevices)
        return BNN_ENOTSUP;
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    if (!g_scratch_addr[ordinal]) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr ||
            cudaFuncSetAttribute(bnn::w1a8_prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)bnn::prep_smem_bytes(kNoAllocMaxK)) != cudaSuccess) {
            cudaGetLastError();
            return BNN_EIO;
        }
        g_scratch_addr[ordinal] = p;
    }
    *out = static_cast<unsigned char*>(g_scratch_addr[ordinal]);
    return BNN_OK;
}

}  // namespace

void bnn_noalloc_forget(int ordinal) {
    if (ordinal < 0 || ordinal >= kMaxDevices)
        return;
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    g_scratch_addr[ordinal] = nullptr;
}

extern "C" BNN_Status bnn_b200_gemm_f32_noalloc(BNN_Matrix matrix, const float* x, uint32_t rows, float* y) {
    if (matrix == nullptr || x == nullptr || y == nullptr || rows == 0)
        return BNN_EINVAL;
    if (rows > kNoAllocMaxRows || matrix->in_features > kNoAllocMaxK)
        return BNN_ERANGE;  // beyond the fixed scratch: use BNN_Execute instead
    if (std::fegetround() != FE_TONEAREST)
        return BNN_ENOTSUP;
    BNN_Device device = matrix->owner;
    bnn::DeviceGuard guard(device->ordinal);
    if (!guard.ok())
        return BNN_EIO;
    unsigned char* scratch = nullptr;
    BNN_Status st = scratch_setup(device->ordinal, &scratch);
    if (st != BNN_OK)
        return st;

    const uint32_t K = matrix->in_features, G = matrix->groups;
    uint32_t* act = reinterpret_cast<uint32_t*>(scratch);
    int32_t* totals = reinterpret_cast<int32_t*>(scratch + kActBytes);
    float* rscale = reinterpret_cast<float*>(scratch + kScaleOffset);
    int* status = reinterpret_cast<int*>(scratch + kStatusOffset);
    cudaStream_t s = device->stream;

    // The status word keeps the previous call's verdict: clear it first.
    if (cudaMemsetAsync(status, 0, sizeof(int), s) != cudaSuccess)
        return BNN_EIO;
    bnn::PrepArgs pa = {};
    pa.in = reinterpret_cast<const unsigned char*>(x);
    pa.in_stride = (size_t)K * 4u;
    pa.kind = bnn::kInputF32;
    pa.k = K;
    pa.m = rows;
    pa.act = act;
    pa.totals = totals;
    pa.row_scale = rscale;
    pa.status = status;
    bnn::w1a8_prep_kernel<<<rows, bnn::kPrepThreads, bnn::prep_smem_bytes(K), s>>>(pa);
    // A prep that did not launch would leave the previous call's rows in the
    // shared scratch: stop before the contraction reads them.
    if (cudaGetLastError() != cudaSuccess)
        return BNN_EIO;

    const bnn::GemvLaunch cl =
        bnn::plan_gemv(device->sm_count, matrix->out_features, G, rows, bnn::kProSliced, bnn::kEpiView);
    bnn::GemvArgs ga = {};
    ga.wblocks = matrix->wblocks;
    ga.n = matrix->out_features;
    ga.groups = G;
    ga.m = rows;
    ga.tiles = cl.tiles;
    ga.stages = cl.stages;
    ga.blocks_per_tile = cl.blocks_per_tile;
    ga.act = act;
    ga.totals = totals;
    ga.row_scale = rscale;
    ga.out = reinterpret_cast<unsigned char*>(y);
    ga.out_stride = (size_t)matrix->out_features * 4u;
    ga.status = status;
    if (bnn::launch_gemv(cl, rows, ga, s, false) != cudaSuccess) {
        cudaGetLastError();
        cudaStreamSynchronize(s);  // the prep may still run: leave nothing in flight
        return BNN_EIO;
    }
    int verdict = 0;
    if (cudaMemcpyAsync(&verdict, status, sizeof(int), cudaMemcpyDeviceToHost, s) != cudaSuccess ||
        cudaStreamSynchronize(s) != cudaSuccess) {
        cudaGetLastError();
        return BNN_EIO;
    }
    if (verdict & bnn::kStatusTimeout)
        return BNN_ETIMEOUT;
    return verdict ? BNN_ERANGE : BNN_OK;
}

namespace bnn {
cudaError_t set_test_hooks_noalloc(unsigned long long limit_ns, int starve) {
    cudaError_t e = cudaMemcpyToSymbol(g_wait_ns_limit, &limit_ns, sizeof limit_ns);
    if (e == cudaSuccess)
        e = cudaMemcpyToSymbol(g_test_starve_producer, &starve, sizeof starve);
    return e;
}
}  // namespace bnn
