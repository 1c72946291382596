// bnn_accel.cu - the BNN_* accelerator API v2 on a B200 (libbnn_b200.so).
//
// Host side of the drop-in boundary declared in include/bnn_b200_accel.h.
// Argument checks follow the reference soft backend's order exactly so every
// misuse returns the same status code (soft-bnn-accelerator.c:310-603); the
// work itself runs on the device:
//   BNN_MatrixCreate -> device copy of bits and scales, packed by w1a8_pack_kernel
//   BNN_Execute      -> w1a8_prep_kernel (validate + quantise every row), then
//                       w1a8_gemv_kernel, then one synchronous status read.
// A rejected input is detected by the prep kernel before the contraction
// kernel writes anything, so the output stays untouched (bnn-accelerator.h:201).
#include <cfenv>
#include <climits>
#include <cstdlib>
#include <cstring>
#include <new>
#include <string>
#include <vector>

#include "bnn_b200_ext.h"
#include "bnn_internal.h"
#include "w1a8_prep.cuh"

namespace {

constexpr uint32_t kMaxFeatures = 8192u;  // same logical limits as the soft backend
constexpr uint32_t kGroupSize = 128u;

bool size_mul(size_t a, size_t b, size_t* r) {
    if (a != 0 && b > SIZE_MAX / a)
        return false;
    *r = a * b;
    return true;
}

bool range_fits(size_t capacity, size_t offset, size_t bytes) {
    return offset <= capacity && bytes <= capacity - offset;
}

// Last row inside the buffer, without computing (rows-1)*stride (soft :65-77).
bool rows_fit(size_t capacity, size_t offset, size_t stride, size_t row_bytes, uint32_t rows) {
    if (rows == 0 || row_bytes == 0 || stride < row_bytes || offset > capacity)
        return false;
    size_t available = capacity - offset;
    if (row_bytes > available)
        return false;
    return (uintmax_t)(rows - 1u) <= (uintmax_t)((available - row_bytes) / stride);
}

BNN_Status op_types(BNN_Operation op, BNN_Type* in, BNN_Type* out) {
    switch (op) {
    case BNN_OP_GEMV:
    case BNN_OP_GEMM:
        *in = BNN_TYPE_I8;
        *out = BNN_TYPE_F32;
        return BNN_OK;
    case BNN_OP_DOT_GROUPS:
        *in = BNN_TYPE_I8;
        *out = BNN_TYPE_I16;
        return BNN_OK;
    case BNN_OP_GEMV_F32:
    case BNN_OP_GEMM_F32:
        *in = BNN_TYPE_F32;
        *out = BNN_TYPE_F32;
        return BNN_OK;
    default:
        return BNN_ENOTSUP;
    }
}

// Maps a caller's device_index to a CUDA ordinal. BNN_B200_DEVICE, if set,
// is a comma-separated list: index i selects the i-th listed ordinal.
bool resolve_ordinal(uint32_t index, int* ordinal) {
    int count = 0;
    if (cudaGetDeviceCount(&count) != cudaSuccess || count <= 0)
        return false;
    const char* env = std::getenv("BNN_B200_DEVICE");
    if (env && *env) {
        std::vector<int> list;
        std::string s(env);
        size_t start = 0;
        while (start <= s.size()) {
            size_t comma = s.find(',', start);
            std::string item = s.substr(start, comma == std::string::npos ? std::string::npos : comma - start);
            if (!item.empty())
                list.push_back(std::atoi(item.c_str()));
            if (comma == std::string::npos)
                break;
            start = comma + 1;
        }
        if (index >= list.size() || list[index] < 0 || list[index] >= count)
            return false;
        *ordinal = list[index];
        return true;
    }
    if (index >= (uint32_t)count)
        return false;
    *ordinal = (int)index;
    return true;
}

// Grows the per-device scratch to at least `bytes` (256-byte aligned parts).
BNN_Status ensure_scratch(BNN_Device d, size_t bytes) {
    if (d->scratch_bytes >= bytes)
        return BNN_OK;
    if (d->scratch) {
        cudaStreamSynchronize(d->stream);
        cudaFree(d->scratch);
        d->scratch = nullptr;
        d->scratch_bytes = 0;
    }
    void* p = nullptr;
    if (cudaMalloc(&p, bytes) != cudaSuccess) {
        cudaGetLastError();
        return BNN_ENOMEM;
    }
    d->scratch = p;
    d->scratch_bytes = bytes;
    return BNN_OK;
}

size_t align256(size_t x) { return (x + 255u) & ~(size_t)255u; }

}  // namespace

extern "C" {

BNN_Status BNN_DeviceOpen(uint32_t device_index, BNN_Device* out_device) {
    if (out_device == nullptr)
        return BNN_EINVAL;
    *out_device = nullptr;
    int ordinal = -1;
    if (!resolve_ordinal(device_index, &ordinal)) {
        cudaGetLastError();
        return BNN_ENOTSUP;
    }
    bnn::DeviceGuard guard(ordinal);
    if (!guard.ok())
        return BNN_EIO;
    auto* d = new (std::nothrow) bnn_accel_device();
    if (!d)
        return BNN_ENOMEM;
    d->ordinal = ordinal;
    bnn_noalloc_forget(ordinal);
    if (cudaDeviceGetAttribute(&d->sm_count, cudaDevAttrMultiProcessorCount, ordinal) != cudaSuccess) {
        delete d;
        return BNN_EIO;
    }
    if (cudaStreamCreateWithFlags(&d->stream, cudaStreamNonBlocking) != cudaSuccess) {
        delete d;
        return BNN_EIO;
    }
    if (cudaMalloc(&d->d_status, 3 * sizeof(int)) != cudaSuccess ||
        cudaMemset(d->d_status, 0, 3 * sizeof(int)) != cudaSuccess ||
        cudaMallocHost(&d->h_status, sizeof(int)) != cudaSuccess) {
        cudaGetLastError();
        if (d->d_status)
            cudaFree(d->d_status);
        cudaStreamDestroy(d->stream);
        delete d;
        return BNN_ENOMEM;
    }
    d->last_status = d->d_status;
    d->single_jobs = 0;
    d->inflight_count = 0;
    d->inflight_overflow = false;
    *out_device = d;
    return BNN_OK;
}

BNN_Status BNN_DeviceClose(BNN_Device device) {
    if (device == nullptr)
        return BNN_EINVAL;
    if (device->matrix_count != 0 || device->buffer_count != 0)
        return BNN_EBUSY;
    bnn::DeviceGuard guard(device->ordinal);
    cudaStreamSynchronize(device->stream);
    if (device->scratch)
        cudaFree(device->scratch);
    cudaFree(device->d_status);
    cudaFreeHost(device->h_status);
    cudaStreamDestroy(device->stream);
    delete device;
    return BNN_OK;
}

BNN_Status BNN_DeviceGetCaps(BNN_Device device, BNN_Caps* out_caps) {
    if (device == nullptr || out_caps == nullptr)
        return BNN_EINVAL;
    std::memset(out_caps, 0, sizeof *out_caps);
    out_caps->api_version = BNN_API_VERSION;
    out_caps->max_in_features = kMaxFeatures;
    out_caps->max_out_features = kMaxFeatures;
    out_caps->max_rows = UINT32_MAX;
    out_caps->group_size = kGroupSize;
    out_caps->supported_ops =
        BNN_CAP_GEMV | BNN_CAP_GEMM | BNN_CAP_DOT_GROUPS | BNN_CAP_GEMV_F32 | BNN_CAP_GEMM_F32;
    return BNN_OK;
}

// Shared by BNN_MatrixCreate and the engine's unbounded loader: validates the
// description (limit == 0 disables the 8192 feature cap) and uploads it.
static BNN_Status bnn_b200_matrix_create_limited(BNN_Device device, const BNN_MatrixDesc* desc,
                                                 BNN_Matrix* out_matrix, uint32_t limit) {
    if (out_matrix == nullptr)
        return BNN_EINVAL;
    *out_matrix = nullptr;
    if (device == nullptr || desc == nullptr)
        return BNN_EINVAL;
    if (desc->in_features == 0 || desc->out_features == 0 || desc->group_size == 0 ||
        desc->group_size > 256u || desc->group_size % 8u != 0)
        return BNN_EINVAL;
    if ((limit && (desc->in_features > limit || desc->out_features > limit)) ||
        desc->group_size != kGroupSize)
        return BNN_ENOTSUP;
    if (desc->in_features % kGroupSize != 0)
        return BNN_EINVAL;
    size_t weight_bytes, scale_count, scale_bytes;
    if (!size_mul(desc->out_features, desc->in_features / 8u, &weight_bytes) ||
        !size_mul(desc->out_features, desc->in_features / kGroupSize, &scale_count) ||
        !size_mul(scale_count, sizeof(uint16_t), &scale_bytes))
        return BNN_ERANGE;
    if (desc->weight_bits == nullptr || desc->scale_fp16 == nullptr ||
        desc->weight_bytes != weight_bytes || desc->scale_count != scale_count)
        return BNN_EINVAL;
    for (size_t i = 0; i < scale_count; ++i)
        if ((desc->scale_fp16[i] & 0x7c00u) == 0x7c00u)
            return BNN_EINVAL;  // NaN or Inf scale
    if (device->matrix_count == SIZE_MAX)
        return BNN_ERANGE;

    bnn::DeviceGuard guard(device->ordinal);
    if (!guard.ok())
        return BNN_EIO;
    auto* m = new (std::nothrow) bnn_accel_matrix();
    if (!m)
        return BNN_ENOMEM;
    const uint32_t groups = desc->in_features / kGroupSize;
    size_t nblocks = (desc->out_features + bnn::kRowBlock - 1) / bnn::kRowBlock;
    nblocks = (nblocks + bnn::kBlockPad - 1) / bnn::kBlockPad * bnn::kBlockPad;
    const size_t packed_bytes = nblocks * bnn::block_bytes(groups);
    uint8_t* raw = nullptr;
    uint16_t* raw_scales = nullptr;
    if (cudaMalloc(&m->wblocks, packed_bytes) != cudaSuccess || cudaMalloc(&raw, weight_bytes) != cudaSuccess ||
        cudaMalloc(&raw_scales, scale_bytes) != cudaSuccess) {
        cudaGetLastError();
        if (m->wblocks) cudaFree(m->wblocks);
        if (raw) cudaFree(raw);
        if (raw_scales) cudaFree(raw_scales);
        delete m;
        return BNN_ENOMEM;
    }
    cudaStream_t s = device->stream;
    bool ok = cudaMemcpyAsync(raw, desc->weight_bits, weight_bytes, cudaMemcpyHostToDevice, s) == cudaSuccess &&
              cudaMemcpyAsync(raw_scales, desc->scale_fp16, scale_bytes, cudaMemcpyHostToDevice, s) == cudaSuccess;
    if (ok) {
        const size_t chunks = nblocks * groups * bnn::kRowBlock;
        const unsigned grid = (unsigned)std::min<size_t>((chunks + 255) / 256, 148u * 16u);
        bnn::w1a8_pack_kernel<<<grid, 256, 0, s>>>(raw, raw_scales, desc->out_features, groups, nblocks,
                                                   m->wblocks);
        ok = cudaGetLastError() == cudaSuccess && cudaStreamSynchronize(s) == cudaSuccess;
    }
    cudaFree(raw);
    cudaFree(raw_scales);
    if (!ok) {
        cudaFree(m->wblocks);
        delete m;
        return BNN_EIO;
    }
    m->owner = device;
    m->in_features = desc->in_features;
    m->out_features = desc->out_features;
    m->groups = groups;
    ++device->matrix_count;
    *out_matrix = m;
    return BNN_OK;
}

BNN_Status bnn_b200_matrix_alloc(BNN_Device device, uint32_t in_features, uint32_t out_features,
                                 BNN_Matrix* out_matrix) {
    if (out_matrix == nullptr)
        return BNN_EINVAL;
    *out_matrix = nullptr;
    if (device == nullptr || in_features == 0 || in_features % kGroupSize != 0 || out_features == 0)
        return BNN_EINVAL;
    bnn::DeviceGuard guard(device->ordinal);
    if (!guard.ok())
        return BNN_EIO;
    auto* m = new (std::nothrow) bnn_accel_matrix();
    if (!m)
        return BNN_ENOMEM;
    const uint32_t groups = in_features / kGroupSize;
    size_t nblocks = (out_features + bnn::kRowBlock - 1) / bnn::kRowBlock;
    nblocks = (nblocks + bnn::kBlockPad - 1) / bnn::kBlockPad * bnn::kBlockPad;
    const size_t packed_bytes = nblocks * bnn::block_bytes(groups);
    if (cudaMalloc(&m->wblocks, packed_bytes) != cudaSuccess) {
        cudaGetLastError();
        delete m;
        return BNN_ENOMEM;
    }
    if (cudaMemsetAsync(m->wblocks, 0, packed_bytes, device->stream) != cudaSuccess ||
        cudaStreamSynchronize(device->stream) != cudaSuccess) {
        cudaFree(m->wblocks);
        delete m;
        return BNN_EIO;
    }
    m->owner = device;
    m->in_features = in_features;
    m->out_features = out_features;
    m->groups = groups;
    ++device->matrix_count;
    *out_matrix = m;
    return BNN_OK;
}

BNN_Status BNN_MatrixCreate(BNN_Device device, const BNN_MatrixDesc* desc, BNN_Matrix* out_matrix) {
    return bnn_b200_matrix_create_limited(device, desc, out_matrix, kMaxFeatures);
}

void BNN_MatrixDestroy(BNN_Matrix matrix) {
    if (matrix == nullptr)
        return;
    bnn::DeviceGuard guard(matrix->owner->ordinal);
    cudaStreamSynchronize(matrix->owner->stream);
    --matrix->owner->matrix_count;
    cudaFree(matrix->wblocks);
    delete matrix;
}

BNN_Status BNN_BufferAlloc(BNN_Device device, size_t bytes, BNN_Buffer* out_buffer) {
    if (out_buffer == nullptr)
        return BNN_EINVAL;
    *out_buffer = nullptr;
    if (device == nullptr || bytes == 0)
        return BNN_EINVAL;
    if (device->buffer_count == SIZE_MAX)
        return BNN_ERANGE;
    bnn::DeviceGuard guard(device->ordinal);
    if (!guard.ok())
        return BNN_EIO;
    auto* b = new (std::nothrow) bnn_accel_buffer();
    if (!b)
        return BNN_ENOMEM;
    if (cudaMalloc(&b->data, bytes) != cudaSuccess) {
        cudaGetLastError();
        delete b;
        return BNN_ENOMEM;
    }
    b->owner = device;
    b->bytes = bytes;
    ++device->buffer_count;
    *out_buffer = b;
    return BNN_OK;
}

void BNN_BufferFree(BNN_Buffer buffer) {
    if (buffer == nullptr)
        return;
    bnn::DeviceGuard guard(buffer->owner->ordinal);
    cudaStreamSynchronize(buffer->owner->stream);
    --buffer->owner->buffer_count;
    cudaFree(buffer->data);
    delete buffer;
}

BNN_Status BNN_BufferWrite(BNN_Buffer buffer, size_t offset, const void* src, size_t bytes) {
    if (buffer == nullptr || (bytes != 0 && src == nullptr))
        return BNN_EINVAL;
    if (!range_fits(buffer->bytes, offset, bytes))
        return BNN_ERANGE;
    if (bytes == 0)
        return BNN_OK;
    bnn::DeviceGuard guard(buffer->owner->ordinal);
    cudaStream_t s = buffer->owner->stream;
    if (cudaMemcpyAsync(buffer->data + offset, src, bytes, cudaMemcpyHostToDevice, s) != cudaSuccess ||
        cudaStreamSynchronize(s) != cudaSuccess) {
        cudaGetLastError();
        return BNN_EIO;
    }
    return BNN_OK;
}

BNN_Status BNN_BufferRead(BNN_Buffer buffer, size_t offset, void* dst, size_t bytes) {
    if (buffer == nullptr || (bytes != 0 && dst == nullptr))
        return BNN_EINVAL;
    if (!range_fits(buffer->bytes, offset, bytes))
        return BNN_ERANGE;
    if (bytes == 0)
        return BNN_OK;
    bnn::DeviceGuard guard(buffer->owner->ordinal);
    cudaStream_t s = buffer->owner->stream;
    if (cudaMemcpyAsync(dst, buffer->data + offset, bytes, cudaMemcpyDeviceToHost, s) != cudaSuccess ||
        cudaStreamSynchronize(s) != cudaSuccess) {
        cudaGetLastError();
        return BNN_EIO;
    }
    return BNN_OK;
}

// Validates a job exactly as the reference does (soft :527-573) and fills in
// the resolved strides. Returns BNN_OK when the job may run.
static BNN_Status check_job(BNN_Device device, const BNN_Job* job, BNN_Type* in_type,
                            size_t* in_stride, size_t* out_stride) {
    if (device == nullptr || job == nullptr || job->matrix == nullptr ||
        job->input.buffer == nullptr || job->output.buffer == nullptr || job->rows == 0)
        return BNN_EINVAL;
    BNN_Type out_type;
    BNN_Status st = op_types(job->operation, in_type, &out_type);
    if (st != BNN_OK)
        return st;
    if ((job->operation == BNN_OP_GEMV || job->operation == BNN_OP_GEMV_F32) && job->rows != 1)
        return BNN_EINVAL;
    if (job->input.type != *in_type || job->output.type != out_type)
        return BNN_EINVAL;
    const BNN_Matrix m = job->matrix;
    if (m->owner != device || job->input.buffer->owner != device ||
        job->output.buffer->owner != device || job->input.buffer == job->output.buffer)
        return BNN_EINVAL;
    size_t in_row_bytes, out_row_bytes, out_elems;
    if (!size_mul(m->in_features, *in_type == BNN_TYPE_F32 ? 4u : 1u, &in_row_bytes))
        return BNN_ERANGE;
    if (job->operation == BNN_OP_DOT_GROUPS) {
        if (!size_mul(m->out_features, m->groups, &out_elems) ||
            !size_mul(out_elems, sizeof(int16_t), &out_row_bytes))
            return BNN_ERANGE;
    } else if (!size_mul(m->out_features, sizeof(float), &out_row_bytes)) {
        return BNN_ERANGE;
    }
    *in_stride = job->input.row_stride ? job->input.row_stride : in_row_bytes;
    *out_stride = job->output.row_stride ? job->output.row_stride : out_row_bytes;
    if (*in_stride < in_row_bytes || *out_stride < out_row_bytes)
        return BNN_EINVAL;
    if (!rows_fit(job->input.buffer->bytes, job->input.offset, *in_stride, in_row_bytes, job->rows) ||
        !rows_fit(job->output.buffer->bytes, job->output.offset, *out_stride, out_row_bytes, job->rows))
        return BNN_ERANGE;
    if (job->operation != BNN_OP_DOT_GROUPS && std::fegetround() != FE_TONEAREST)
        return BNN_ENOTSUP;
    return BNN_OK;
}

// Outputs of the jobs in flight (see bnn_accel_device::inflight_out).
static bool inflight_meets(const bnn_accel_device* d, uintptr_t begin, uintptr_t end) {
    if (d->inflight_overflow)
        return true;
    for (uint32_t i = 0; i < d->inflight_count; ++i)
        if (begin < d->inflight_out[i][1] && d->inflight_out[i][0] < end)
            return true;
    return false;
}

static void inflight_add(bnn_accel_device* d, uintptr_t begin, uintptr_t end) {
    if (d->inflight_count == bnn_accel_device::kMaxInflightOutputs) {
        d->inflight_overflow = true;
        return;
    }
    d->inflight_out[d->inflight_count][0] = begin;
    d->inflight_out[d->inflight_count][1] = end;
    d->inflight_count++;
}

static void inflight_clear(bnn_accel_device* d) {
    d->inflight_count = 0;
    d->inflight_overflow = false;
}

// Enqueues prep + contraction for a validated job on the device stream,
// without synchronising. Rows are processed in chunks so the grid's y
// dimension stays within limits; the prep pass over ALL rows runs before
// any contraction so a bad last row still leaves the output untouched.
static BNN_Status enqueue_job(BNN_Device device, const BNN_Job* job, BNN_Type in_type,
                              size_t in_stride, size_t out_stride) {
    const BNN_Matrix m = job->matrix;
    const uint32_t K = m->in_features, G = m->groups, M = job->rows;
    cudaStream_t s = device->stream;
    // every job's output joins the in-flight set (whatever path runs it)
    {
        const uintptr_t ob = reinterpret_cast<uintptr_t>(job->output.buffer->data + job->output.offset);
        inflight_add(device, ob, ob + (size_t)(M - 1) * out_stride +
                                     (size_t)m->out_features * (job->operation == BNN_OP_DOT_GROUPS ? 2u * G : 4u));
    }
    // Jobs of at most kRowsPerCta rows (F32 rows 16-byte aligned, int8 rows
    // 4-byte aligned): every contraction CTA loads, validates and quantises
    // (kProQuant) or slices (kProI8) all of them in its prologue before it
    // writes anything, so a rejected row still leaves the output untouched
    // and no separate prep pass is needed. The job is one kernel: launched
    // with programmatic dependent launch, its weight stream starts while the
    // previous kernel of the stream drains (weights are immutable;
    // activations and outputs are touched only after the kernel's
    // grid-dependency wait, or activations before it when no job in flight
    // writes them), and its verdict goes to the slot that the previous
    // single-kernel job cleared.
    const unsigned char* in_ptr = job->input.buffer->data + job->input.offset;
    const bool f32 = in_type == BNN_TYPE_F32;
    const uint32_t in_align = f32 ? 16u : 4u;
    if (M <= (uint32_t)bnn::kRowsPerCta && K <= bnn::kMaxPrologueK &&
        (reinterpret_cast<uintptr_t>(in_ptr) & (in_align - 1u)) == 0 && (M == 1 || in_stride % in_align == 0)) {
        const uint32_t slot = 1u + (device->single_jobs & 1u);
        const int pro = f32 ? bnn::kProQuant : bnn::kProI8;
        const int epi = job->operation == BNN_OP_DOT_GROUPS ? bnn::kEpiDotGroups : bnn::kEpiView;
        const bnn::GemvLaunch cl = bnn::plan_gemv(device->sm_count, m->out_features, G, M, pro, epi);
        bnn::GemvArgs ga = {};
        ga.wblocks = m->wblocks;
        ga.n = m->out_features;
        ga.groups = G;
        ga.m = M;
        ga.tiles = cl.tiles;
        ga.stages = cl.stages;
        ga.blocks_per_tile = cl.blocks_per_tile;
        const size_t elem = f32 ? 4u : 1u;
        if (f32)
            ga.x = reinterpret_cast<const float*>(in_ptr);
        else
            ga.xq = reinterpret_cast<const int8_t*>(in_ptr);
        ga.x_stride = M == 1 ? K : in_stride / elem;
        {
            // the input may be read early when no job in flight writes it
            // (this job's own output is in the set already: in place never is)
            const uintptr_t ib = reinterpret_cast<uintptr_t>(in_ptr);
            ga.early_input =
                inflight_meets(device, ib, ib + (size_t)(M - 1) * ga.x_stride * elem + (size_t)K * elem) ? 0 : 1;
        }
        ga.out = job->output.buffer->data + job->output.offset;
        ga.out_stride = out_stride;
        ga.status = device->d_status + slot;
        ga.status_next = device->d_status + (3u - slot);
        if (bnn::launch_gemv(cl, M, ga, s, true) != cudaSuccess)
            return BNN_EIO;
        device->single_jobs++;
        device->last_status = device->d_status + slot;
        return BNN_OK;
    }
    device->last_status = device->d_status;
    // From kMmaMinRows rows the group dots run on the tensor cores
    // (w1a8_mma.cuh); below, and for K beyond the tensor-core kernel's
    // shared memory, on the dp4a contraction (w1a8_gemv.cuh).
    const bool mma = M >= bnn::kMmaMinRows && bnn::mma_fits(G);
    const size_t act_bytes = align256(mma ? bnn::mma_a_bytes(M, G) : (size_t)M * K);
    const size_t tot_bytes = mma ? 0 : align256((size_t)M * G * 4u);
    const size_t scl_bytes = align256((size_t)M * 4u);
    BNN_Status st = ensure_scratch(device, act_bytes + tot_bytes + scl_bytes);
    if (st != BNN_OK)
        return st;
    auto* base = static_cast<unsigned char*>(device->scratch);
    uint32_t* act = reinterpret_cast<uint32_t*>(base);
    int32_t* totals = reinterpret_cast<int32_t*>(base + act_bytes);
    float* rscale = reinterpret_cast<float*>(base + act_bytes + tot_bytes);

    if (cudaMemsetAsync(device->d_status, 0, sizeof(int), s) != cudaSuccess)
        return BNN_EIO;
    bnn::PrepArgs pa = {};
    pa.in = job->input.buffer->data + job->input.offset;
    pa.in_stride = in_stride;
    pa.kind = in_type == BNN_TYPE_F32 ? bnn::kInputF32 : bnn::kInputI8;
    pa.k = K;
    pa.m = M;
    pa.act = act;
    pa.a_sw = mma ? base : nullptr;
    pa.totals = totals;
    pa.row_scale = rscale;
    pa.status = device->d_status;
    const size_t prep_smem = bnn::prep_smem_bytes(K);
    cudaFuncSetAttribute(bnn::w1a8_prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)bnn::prep_smem_bytes(kMaxFeatures));
    for (uint32_t r0 = 0; r0 < M; r0 += 65535u * 1024u) {
        const uint32_t rows = std::min<uint32_t>(M - r0, 65535u * 1024u);
        bnn::PrepArgs chunk = pa;
        chunk.in = pa.in + (size_t)r0 * in_stride;
        chunk.act = act + (size_t)r0 * G * bnn::kWordsPerGroup;
        chunk.row0 = r0;
        chunk.totals = totals + (size_t)r0 * G;
        chunk.row_scale = rscale + r0;
        chunk.m = rows;
        bnn::w1a8_prep_kernel<<<rows, bnn::kPrepThreads, prep_smem, s>>>(chunk);
    }

    const int epi = job->operation == BNN_OP_DOT_GROUPS ? bnn::kEpiDotGroups : bnn::kEpiView;
    unsigned char* out = job->output.buffer->data + job->output.offset;
    if (mma) {
        const uint32_t rows_per_launch = 65535u * bnn::kMmaM;
        for (uint32_t r0 = 0; r0 < M; r0 += rows_per_launch) {
            bnn::MmaArgs ma = {};
            ma.wblocks = m->wblocks;
            ma.n = m->out_features;
            ma.groups = G;
            ma.m = std::min<uint32_t>(M - r0, rows_per_launch);
            ma.a_sw = base + (size_t)(r0 / bnn::kMmaM) * G * bnn::kMmaATile;
            ma.row_scale = in_type == BNN_TYPE_F32 ? rscale + r0 : nullptr;
            ma.out = out + (size_t)r0 * out_stride;
            ma.out_stride = out_stride;
            ma.epi = epi;
            ma.status = device->d_status;
            if (bnn::launch_mma(ma, device->sm_count, s) != cudaSuccess)
                return BNN_EIO;
        }
        return BNN_OK;
    }
    const bnn::GemvLaunch cl = bnn::plan_gemv(device->sm_count, m->out_features, G, M, bnn::kProSliced, epi);
    const uint32_t rows_per_launch = 65535u * bnn::kRowsPerCta;
    for (uint32_t r0 = 0; r0 < M; r0 += rows_per_launch) {
        const uint32_t rows = std::min<uint32_t>(M - r0, rows_per_launch);
        bnn::GemvArgs ga = {};
        ga.wblocks = m->wblocks;
        ga.n = m->out_features;
        ga.groups = G;
        ga.m = rows;
        ga.tiles = cl.tiles;
        ga.stages = cl.stages;
        ga.blocks_per_tile = cl.blocks_per_tile;
        ga.act = act + (size_t)r0 * G * bnn::kWordsPerGroup;
        ga.totals = totals + (size_t)r0 * G;
        ga.row_scale = in_type == BNN_TYPE_F32 ? rscale + r0 : nullptr;
        ga.out = out + (size_t)r0 * out_stride;
        ga.out_stride = out_stride;
        ga.status = device->d_status;
        if (bnn::launch_gemv(cl, rows, ga, s, false) != cudaSuccess)
            return BNN_EIO;
    }
    if (cudaGetLastError() != cudaSuccess)
        return BNN_EIO;
    return BNN_OK;
}

BNN_Status BNN_Execute(BNN_Device device, const BNN_Job* job) {
    BNN_Type in_type;
    size_t in_stride = 0, out_stride = 0;
    BNN_Status st = check_job(device, job, &in_type, &in_stride, &out_stride);
    if (st != BNN_OK)
        return st;
    bnn::DeviceGuard guard(device->ordinal);
    if (!guard.ok())
        return BNN_EIO;
    st = enqueue_job(device, job, in_type, in_stride, out_stride);
    if (st != BNN_OK)
        return st;
    return bnn_b200_sync(device);
}

BNN_Status bnn_b200_matrix_create_unbounded(BNN_Device device, const BNN_MatrixDesc* desc,
                                            BNN_Matrix* out_matrix) {
    return bnn_b200_matrix_create_limited(device, desc, out_matrix, 0);
}

BNN_Status bnn_b200_execute_async(BNN_Device device, const BNN_Job* job) {
    BNN_Type in_type;
    size_t in_stride = 0, out_stride = 0;
    BNN_Status st = check_job(device, job, &in_type, &in_stride, &out_stride);
    if (st != BNN_OK)
        return st;
    bnn::DeviceGuard guard(device->ordinal);
    if (!guard.ok())
        return BNN_EIO;
    return enqueue_job(device, job, in_type, in_stride, out_stride);
}

BNN_Status bnn_b200_sync(BNN_Device device) {
    if (device == nullptr)
        return BNN_EINVAL;
    bnn::DeviceGuard guard(device->ordinal);
    cudaStream_t s = device->stream;
    if (cudaMemcpyAsync(device->h_status, device->last_status, sizeof(int), cudaMemcpyDeviceToHost, s) != cudaSuccess ||
        cudaStreamSynchronize(s) != cudaSuccess) {
        cudaGetLastError();
        return BNN_EIO;
    }
    inflight_clear(device);
    const int st = *device->h_status;
    if (st & bnn::kStatusTimeout)
        return BNN_ETIMEOUT;
    return st ? BNN_ERANGE : BNN_OK;
}

BNN_Status bnn_b200_test_wait_limit(BNN_Device device, uint64_t limit_ns, int starve_producer) {
    if (device == nullptr)
        return BNN_EINVAL;
    bnn::DeviceGuard guard(device->ordinal);
    if (!guard.ok())
        return BNN_EIO;
    const unsigned long long limit = limit_ns ? (unsigned long long)limit_ns : bnn::kWaitNsLimit;
    const int starve = starve_producer ? 1 : 0;
    // no job of this handle may run while the limits change
    if (cudaStreamSynchronize(device->stream) != cudaSuccess ||
        cudaMemcpyToSymbol(bnn::g_wait_ns_limit, &limit, sizeof limit) != cudaSuccess ||
        cudaMemcpyToSymbol(bnn::g_test_starve_producer, &starve, sizeof starve) != cudaSuccess ||
        bnn::set_test_hooks_engine(limit, starve) != cudaSuccess ||
        bnn::set_test_hooks_noalloc(limit, starve) != cudaSuccess) {
        cudaGetLastError();
        return BNN_EIO;
    }
    return BNN_OK;
}

void* bnn_b200_device_stream(BNN_Device device) {
    return device ? static_cast<void*>(device->stream) : nullptr;
}

int bnn_b200_device_ordinal(BNN_Device device) { return device ? device->ordinal : -1; }

void* bnn_b200_buffer_device_ptr(BNN_Buffer buffer) {
    return buffer ? static_cast<void*>(buffer->data) : nullptr;
}

const char* BNN_StatusString(BNN_Status status) {
    switch (status) {
    case BNN_OK: return "success";
    case BNN_EINVAL: return "invalid argument";
    case BNN_ENOMEM: return "out of memory";
    case BNN_ENOTSUP: return "unsupported operation or configuration";
    case BNN_ERANGE: return "buffer or input range error";
    case BNN_EBUSY: return "device still owns resources";
    case BNN_EIO: return "device I/O error";
    case BNN_ETIMEOUT: return "device timeout";
    default: return "unknown status";
    }
}

}  // extern "C"
