// sq_step_async_noalloc: the asynchronous decode step (sq_readout followed by
// sq_writeback) with its per-request scratch held in a file-scope device array
// instead of caller-allocated memory.
//
// Some callers of this library cannot allocate device memory when they run a
// decode step: a serving process that reserves its whole device budget at
// start-up and forbids allocations afterwards, or a host-language binding that
// has no device allocator of its own and can only hand over the pointers of
// buffers it was given.  This entry point needs nothing from them beyond the
// inputs and outputs (pages, slots, step arguments, out).
//
// Limits and sharing:
//  * the array holds kNoAllocScratchBytes (16 MiB); every GPU that loads the
//    library keeps it until the process exits;
//  * a call needs round_up(batch * 8, 256) + batch * sq_scratch_floats(plan) * 4
//    bytes of it (48 KiB per request for 32 heads of K = V = 128, so up to 341
//    such requests); larger calls return SQ_ERR_CAPACITY before any work;
//  * every call shares the array and it keeps the last call's contents.  Nothing
//    in it needs to start at zero: the writeback half reads only values the
//    readout half of the same call wrote.  Calls whose work overlaps on the GPU
//    (different streams, or different host threads, without ordering between
//    them) race on the array;
//  * the first call on a device looks up the array's device address
//    (cudaGetSymbolAddress) with that device current and caches it; make that
//    first call before any stream capture on the device.
// No cudaMalloc, cudaFree or allocating library routine is called.
#include <cuda_runtime.h>

#include <mutex>

#include "../../include/stepquant_b200.h"

namespace sq {
int32_t validate_plan(const sq_plan *p);  // sq_abi.cu
}  // namespace sq

namespace {

constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_setup_mutex;
void *g_scratch_address[kMaxDevices] = {};

// Device address of g_noalloc_scratch on the current device (looked up once per device).
int32_t scratch_address(void **out) {
    int device = 0;
    if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= kMaxDevices) return SQ_ERR_CUDA;
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    if (!g_scratch_address[device]) {
        void *ptr = nullptr;
        if (cudaGetSymbolAddress(&ptr, g_noalloc_scratch) != cudaSuccess || !ptr) return SQ_ERR_CUDA;
        g_scratch_address[device] = ptr;
    }
    *out = g_scratch_address[device];
    return SQ_OK;
}

}  // namespace

extern "C" {

int64_t sq_noalloc_scratch_bytes(void) { return int64_t(kNoAllocScratchBytes); }

int32_t sq_step_async_noalloc(const sq_plan *plan, uint8_t *pages, int64_t num_slots, const int64_t *slots,
                              int32_t batch, const sq_step_args *args, int32_t *status, sq_stream_t stream) {
    if (batch < 0) return SQ_ERR_ARGUMENT;
    if (batch == 0) return SQ_OK;
    // The plan's own error code (argument, shape or unsupported), as sq_readout returns it.
    if (int32_t e = sq::validate_plan(plan)) return e;
    const int64_t floats = sq_scratch_floats(plan);
    const int64_t slot_bytes = (int64_t(batch) * 8 + 255) / 256 * 256;
    const int64_t need = slot_bytes + int64_t(batch) * floats * 4;
    if (need > int64_t(kNoAllocScratchBytes)) return SQ_ERR_CAPACITY;
    void *base = nullptr;
    if (int32_t e = scratch_address(&base)) return e;
    int64_t *stable = static_cast<int64_t *>(base);
    float *scratch = reinterpret_cast<float *>(static_cast<unsigned char *>(base) + slot_bytes);
    if (int32_t e = sq_readout(plan, pages, num_slots, slots, batch, args, scratch, stable, status, stream)) return e;
    return sq_writeback(plan, pages, num_slots, stable, batch, scratch, nullptr, status, stream);
}

}  // extern "C"
