// A projection that allocates nothing.
//
// jl_project stages its input through the model's pinned host buffer and
// device scratch.  Some callers cannot allocate device memory at the time they
// need a projection: a host that runs with a fixed memory reservation (another
// allocator already owns the rest of the device), or code inside a latency
// budget that cannot afford cudaMalloc's implicit device synchronisation.
// project_noalloc serves them: device-resident input and output owned by the
// caller, and every byte of scratch (pass header, error flag, split-K
// tickets, activation pieces and split-K partials) taken from one file-scope
// device array of fixed size.  The array lives as long as the module, so the
// call runs no cudaMalloc, cudaFree or allocating library routine.
//
// Every call on a device shares that device's array, which keeps the
// previous call's contents: the setup kernel clears the split-K tickets and
// the error flag (the only parts read before they are written) at the start
// of every call.  Calls whose work overlaps on the GPU (different streams,
// different host threads) race on the array.
//
// CUDA loads a module, with its __device__ arrays, and each kernel lazily,
// at first use (CUDA_MODULE_LOADING=LAZY, the default since 12.2).  So the
// array's address, this file's kernels and the pinned host word the error
// flag is read into are all set up by noalloc_prepare, which model creation
// runs once per device: a call itself loads and allocates nothing.
#include <cuda_runtime.h>

#include <mutex>

#include "jl_internal.h"

namespace jl {

namespace {

// 4 MiB: the largest split-K workspace of the shipped presets (Qwen3-8B
// gate/up at 8 rows) needs 1.5 MiB, pieces and tickets well under 1 MiB.
constexpr size_t NOALLOC_SCRATCH_BYTES = (size_t)4 << 20;
constexpr size_t NOALLOC_HEADER_BYTES = 256;  // PassHdr at 0, error flag at 64
constexpr int NOALLOC_MAX_ROWS = 8;
constexpr int MAX_DEVICES = 64;

static __device__ __align__(256) uint8_t g_noalloc_scratch[NOALLOC_SCRATCH_BYTES];

struct DeviceScratch {
    std::once_flag once;
    uint8_t* ptr = nullptr;
    int* host_flag = nullptr;  // pinned word the error flag is copied into
    cudaError_t err = cudaSuccess;
};
DeviceScratch g_devices[MAX_DEVICES];

// Writes the pass header and clears the error flag and split-K tickets.
__global__ void k_noalloc_begin(PassHdr* hdr, int rows, int* err, int* tickets, int n_tickets) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i == 0) {
        hdr->rows = rows;
        hdr->head_rows = rows;
        *err = 0;
    }
    if (i < n_tickets) tickets[i] = 0;
}

// The device address of g_noalloc_scratch on `device` (which is current)
// and the pinned word its error flag is read into, set up once per device:
// the address lookup loads this file's module (and with it the array), and
// the attribute query loads the setup kernel.
jl_status scratch_for(int device, uint8_t** out, int** host_flag) {
    if (device < 0 || device >= MAX_DEVICES) {
        set_error("project_noalloc: device %d out of range", device);
        return JL_ERR_INVALID_ARG;
    }
    DeviceScratch& d = g_devices[device];
    std::call_once(d.once, [&d]() {
        void* p = nullptr;
        d.err = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        d.ptr = (uint8_t*)p;
        cudaFuncAttributes fa;
        if (d.err == cudaSuccess) d.err = cudaFuncGetAttributes(&fa, k_noalloc_begin);
        if (d.err == cudaSuccess) d.err = cudaMallocHost(&d.host_flag, sizeof(int));
        if (d.err != cudaSuccess) cudaGetLastError();
    });
    if (d.err != cudaSuccess || !d.ptr || !d.host_flag) {
        set_error("project_noalloc: set-up failed on device %d: %s", device, cudaGetErrorString(d.err));
        return JL_ERR_CUDA;
    }
    *out = d.ptr;
    if (host_flag) *host_flag = d.host_flag;
    return JL_OK;
}

struct DeviceRestore {
    int prev = -1;
    ~DeviceRestore() {
        if (prev >= 0) cudaSetDevice(prev);
    }
};

}  // namespace

jl_status noalloc_prepare(int device) {
    uint8_t* p = nullptr;
    return scratch_for(device, &p, nullptr);
}

jl_status project_noalloc(jl_model* m, int layer, int which, const float* x, size_t rows, float* y,
                          cudaStream_t stream) {
    if (rows < 1 || rows > (size_t)NOALLOC_MAX_ROWS) {
        set_error("project_noalloc: rows must be 1..%d, got %zu", NOALLOC_MAX_ROWS, rows);
        return JL_ERR_INVALID_ARG;
    }
    if (which < 0 || which > 4 || (which != 4 && (layer < 0 || layer >= m->layers))) {
        set_error("project_noalloc: bad layer %d or projection %d", layer, which);
        return JL_ERR_INVALID_ARG;
    }
    const MxProj* p = nullptr;
    int epi = MXE_STORE, win = m->hidden, wout = m->hidden;
    const int QW = m->q_heads * HEAD, KVW = m->kv_heads * HEAD;
    switch (which) {
        case 0: p = &m->lw[layer].mx_qkv; wout = QW + 2 * KVW; break;
        case 1: p = &m->lw[layer].mx_o; win = QW; break;
        case 2: p = &m->lw[layer].mx_gateup; epi = MXE_SWIGLU; wout = m->inter; break;
        case 3: p = &m->lw[layer].mx_down; win = m->inter; break;
        default: p = &m->mx_head; wout = m->vocab; break;
    }
    if (!p->a) {
        set_error("project_noalloc: projection %d of this model is not MXFP4 on the tensor-core path",
                  which);
        return JL_ERR_INVALID_ARG;
    }
    const MxScratchPlan plan = mx_scratch_plan(*p, (int)rows);
    if (NOALLOC_HEADER_BYTES + plan.total > NOALLOC_SCRATCH_BYTES) {
        set_error("project_noalloc: this projection at %zu rows needs %zu bytes of scratch, more than "
                  "the fixed %zu",
                  rows, NOALLOC_HEADER_BYTES + plan.total, NOALLOC_SCRATCH_BYTES);
        return JL_ERR_INVALID_ARG;
    }
    DeviceRestore restore;
    JL_CUDA(cudaGetDevice(&restore.prev));
    JL_CUDA(cudaSetDevice(m->device));
    uint8_t* base = nullptr;
    int* host_flag = nullptr;
    JL_TRY(scratch_for(m->device, &base, &host_flag));
    PassHdr* hdr = (PassHdr*)base;
    int* err = (int*)(base + 64);
    uint8_t* scratch = base + NOALLOC_HEADER_BYTES;
    cudaStream_t st = stream ? stream : m->stream;
    k_noalloc_begin<<<(p->T + 255) / 256, 256, 0, st>>>(hdr, (int)rows, err, (int*)scratch, p->T);
    JL_CUDA(cudaGetLastError());
    JL_TRY(mx_project_with(*p, epi, hdr, (int)rows, x, win, y, wout, scratch, err, m->sms, st));
    // the flag comes back on the caller's stream into the pinned word: no
    // copy on the legacy default stream, which would wait for other streams
    JL_CUDA(cudaMemcpyAsync(host_flag, err, sizeof(int), cudaMemcpyDeviceToHost, st));
    JL_CUDA(cudaStreamSynchronize(st));
    const int flag = *host_flag;
    if (flag) {
        set_error("project_noalloc: a device-side wait timed out (flag %d)", flag);
        return JL_ERR_TIMEOUT;
    }
    return JL_OK;
}

}  // namespace jl
