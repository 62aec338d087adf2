// Writeback streams confined to an SM budget (green contexts).
//
// The background requantization can be kept off most of the GPU by running it
// on a stream of a green context that owns `sm_budget` SMs; the foreground
// readout keeps the whole device.  The driver entry points are looked up at
// run time (cudaGetDriverEntryPoint), so the library links against the
// runtime only.  Each (device, budget) pair gets one context and one
// non-blocking stream, created on first use and kept until the process exits:
// captured CUDA graphs hold the stream.  The persistent kernels size their
// grids from the SMs of the stream they are launched on (sq_fast.cu,
// stream_sms), so a budgeted stream gets a grid of its own size.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <map>
#include <mutex>
#include <utility>

#include "../../include/stepquant_b200.h"

namespace {

struct BudgetStream {
    CUstream stream;
    int actual_sms;
};

struct DriverCalls {
    PFN_cuDeviceGet_v2000 device_get = nullptr;
    PFN_cuDeviceGetDevResource_v12040 get_resource = nullptr;
    PFN_cuDevSmResourceSplitByCount_v12040 split = nullptr;
    PFN_cuDevResourceGenerateDesc_v12040 describe = nullptr;
    PFN_cuGreenCtxCreate_v12040 create_context = nullptr;
    PFN_cuGreenCtxStreamCreate_v12050 create_stream = nullptr;
    bool ok = false;
};

template <class F>
bool lookup(const char *name, F &fn) {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint(name, &p, cudaEnableDefault, &q) != cudaSuccess || q != cudaDriverEntryPointSuccess ||
        !p) {
        (void)cudaGetLastError();
        return false;
    }
    fn = reinterpret_cast<F>(p);
    return true;
}

const DriverCalls &driver() {
    static DriverCalls calls;
    static std::once_flag once;
    std::call_once(once, [] {
        calls.ok = lookup("cuDeviceGet", calls.device_get) && lookup("cuDeviceGetDevResource", calls.get_resource) &&
                   lookup("cuDevSmResourceSplitByCount", calls.split) &&
                   lookup("cuDevResourceGenerateDesc", calls.describe) &&
                   lookup("cuGreenCtxCreate", calls.create_context) &&
                   lookup("cuGreenCtxStreamCreate", calls.create_stream);
    });
    return calls;
}

std::mutex g_mutex;
std::map<std::pair<int, int>, BudgetStream> g_streams;  // (device, budget) -> stream, never released

// One green context holding at least `budget` SMs of `device`, and a stream in it.
int32_t create(int device, int budget, BudgetStream *out) {
    const DriverCalls &d = driver();
    if (!d.ok) return SQ_ERR_UNSUPPORTED;
    CUdevice dev;
    if (d.device_get(&dev, device) != CUDA_SUCCESS) return SQ_ERR_CUDA;
    CUdevResource whole;
    if (d.get_resource(dev, &whole, CU_DEV_RESOURCE_TYPE_SM) != CUDA_SUCCESS) return SQ_ERR_CUDA;
    CUdevResource part;
    unsigned int groups = 1;
    if (d.split(&part, &groups, &whole, nullptr, 0, static_cast<unsigned int>(budget)) != CUDA_SUCCESS || groups != 1)
        return SQ_ERR_CUDA;
    CUdevResourceDesc desc;
    if (d.describe(&desc, &part, 1) != CUDA_SUCCESS) return SQ_ERR_CUDA;
    CUgreenCtx context;
    if (d.create_context(&context, desc, dev, CU_GREEN_CTX_DEFAULT_STREAM) != CUDA_SUCCESS) return SQ_ERR_CUDA;
    CUstream stream;
    if (d.create_stream(&stream, context, CU_STREAM_NON_BLOCKING, 0) != CUDA_SUCCESS) return SQ_ERR_CUDA;
    out->stream = stream;
    out->actual_sms = static_cast<int>(part.sm.smCount);
    return SQ_OK;
}

}  // namespace

extern "C" {

int32_t sq_budget_stream(int32_t device, int32_t sm_budget, sq_stream_t *stream, int32_t *actual_sms,
                         int32_t *total_sms) {
    if (!stream || !actual_sms || !total_sms) return SQ_ERR_ARGUMENT;
    int count = 0;
    if (cudaGetDeviceCount(&count) != cudaSuccess) return SQ_ERR_CUDA;
    if (device < 0 || device >= count) return SQ_ERR_ARGUMENT;
    int sms = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) return SQ_ERR_CUDA;
    *total_sms = sms;
    if (sm_budget < 1 || sm_budget > sms) return SQ_ERR_ARGUMENT;
    std::lock_guard<std::mutex> lock(g_mutex);
    auto key = std::make_pair(int(device), int(sm_budget));
    auto it = g_streams.find(key);
    if (it == g_streams.end()) {
        BudgetStream made;
        if (int32_t e = create(device, sm_budget, &made)) return e;
        it = g_streams.emplace(key, made).first;
    }
    *stream = reinterpret_cast<sq_stream_t>(it->second.stream);
    *actual_sms = it->second.actual_sms;
    return SQ_OK;
}

}  // extern "C"
