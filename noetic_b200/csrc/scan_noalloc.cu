// scan_noalloc.cu -- the time-chunked scan for callers that cannot allocate.
//
// nk_scan_device(..., chunked = 1) obtains its per-call scratch (the decay
// product, partial state and carry of every time block) with cudaMalloc.
// Some callers cannot do that in the middle of their work: a host that has
// handed the whole device memory budget to its own pool allocator, so a
// stray cudaMalloc can fail or fragment that pool; and a latency-critical
// loop for which cudaMalloc / cudaFree are unacceptable because they may
// synchronise the whole device.  nk_scan_chunked_noalloc_device runs the
// same three kernels on a fixed scratch array that lives in this library's
// device image instead, and allocates nothing.
//
// The array is a file-scope __device__ symbol of NK_SCAN_NOALLOC_SCRATCH_FLOATS
// floats (12 MiB).  Every GPU that loads this library holds it until the
// process exits.  In host code the symbol's name is only a host-side
// stand-in, so its device address is looked up with cudaGetSymbolAddress
// once per device, with that device current, on the first call made on
// that device; make that first call before any stream capture.  The address
// is cached together with the unique id of the CUDA context it belongs to:
// after a cudaDeviceReset (or any teardown of the primary context) the
// module is loaded again and the array may move, so the next call sees a new
// context id and looks the address up again instead of writing through a
// stale pointer.  That call is then a first call again (before any capture).
//
// All calls share the one array.  Nothing in it has to start at zero: each
// call writes every scratch entry it reads before reading it.  Two calls
// whose work overlaps on the GPU (different streams, or different host
// threads, without ordering between them) race on the array and may produce
// wrong results; order them on one stream or synchronise between them.

#include <cuda.h>

#include <exception>
#include <new>
#include <mutex>
#include <string>

#include "../../include/noetic_gpu.h"
#include "nk_kernels.h"

namespace {

static __device__ __align__(256) float g_scan_scratch[NK_SCAN_NOALLOC_SCRATCH_FLOATS];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
struct ScratchAddr {
    float *ptr = nullptr;
    unsigned long long ctx_id = 0;  // context the address was looked up in
};
ScratchAddr g_scratch[kMaxDevices];

nk_status noalloc_fail(nk_status st, const std::string &msg) {
    nk::set_last_error("nk_scan_chunked_noalloc_device: " + msg);
    return st;
}

// Unique id of the calling thread's current context (0 when there is none
// yet, or when the driver does not offer the calls).  The driver entry points
// are looked up through the runtime, so the library keeps loading on hosts
// without a GPU driver.
unsigned long long current_ctx_id() {
    using GetCurrent = CUresult (*)(CUcontext *);
    using GetId = CUresult (*)(CUcontext, unsigned long long *);
    static GetCurrent get_current = nullptr;
    static GetId get_id = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_current = (GetCurrent)p;
        p = nullptr;
        if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_id = (GetId)p;
    });
    if (!get_current || !get_id) return 0;
    CUcontext ctx = nullptr;
    if (get_current(&ctx) != CUDA_SUCCESS || !ctx) return 0;
    unsigned long long id = 0;
    if (get_id(ctx, &id) != CUDA_SUCCESS) return 0;
    return id;
}

nk_status scan_noalloc(const float *a, const float *b, float *h, uint64_t batch, uint64_t t, uint64_t d,
                       void *stream) {
    nk::set_last_error("");
    uint64_t n = 0;
    if (!nk::scan_elements(batch, t, d, n))
        return noalloc_fail(NK_ERR_INVALID, "scan shape too large: batch * t * d exceeds 2^37 elements");
    if (n == 0) return NK_OK;
    if (!a || !b || !h) return noalloc_fail(NK_ERR_INVALID, "null argument");
    // n <= 2^37 here, so every factor and the block count fit comfortably.
    const uint64_t blocks = (t + NK_SCAN_TIME_BLOCK - 1) / NK_SCAN_TIME_BLOCK;
    const uint64_t need = nk::scan_chunked_scratch_floats((int64_t)batch, (int64_t)t, (int64_t)d);
    if (need > NK_SCAN_NOALLOC_SCRATCH_FLOATS)
        return noalloc_fail(NK_ERR_INVALID, "batch * ceil(t / " + std::to_string(NK_SCAN_TIME_BLOCK) + ") * d = " +
                                                std::to_string(batch * blocks * d) +
                                                " exceeds the fixed scratch limit of " +
                                                std::to_string(NK_SCAN_NOALLOC_SCRATCH_FLOATS / 3) +
                                                "; use nk_scan_device for larger scans");
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices)
        return noalloc_fail(NK_ERR_CUDA, std::string("no usable current device: ") + cudaGetErrorString(e));
    float *scratch = nullptr;
    {
        std::lock_guard<std::mutex> lock(g_mu);
        ScratchAddr &slot = g_scratch[dev];
        const unsigned long long id = current_ctx_id();
        if (!slot.ptr || id == 0 || id != slot.ctx_id) {
            void *p = nullptr;
            e = cudaGetSymbolAddress(&p, g_scan_scratch);
            if (e != cudaSuccess) {
                cudaGetLastError();
                slot = ScratchAddr{};
                return noalloc_fail(NK_ERR_CUDA, std::string("cudaGetSymbolAddress failed: ") + cudaGetErrorString(e));
            }
            // The lookup makes the device's primary context current if it was not.
            slot.ptr = (float *)p;
            slot.ctx_id = current_ctx_id();
        }
        scratch = slot.ptr;
    }
    e = nk::scan_chunked(a, b, h, (int64_t)batch, (int64_t)t, (int64_t)d, scratch, (cudaStream_t)stream);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return noalloc_fail(NK_ERR_CUDA, std::string("launch failed: ") + cudaGetErrorString(e));
    }
    return NK_OK;
}

}  // namespace

extern "C" nk_status nk_scan_chunked_noalloc_device(const float *a, const float *b, float *h, uint64_t batch,
                                                    uint64_t t, uint64_t d, void *stream) {
    // Nothing may unwind across the C ABI: a failed string allocation in a
    // message becomes a status.
    try {
        return scan_noalloc(a, b, h, batch, t, d, stream);
    } catch (const std::bad_alloc &) {
        try {
            nk::set_last_error("nk_scan_chunked_noalloc_device: host allocation failed");
        } catch (...) {
        }
        return NK_ERR_OOM;
    } catch (const std::exception &ex) {
        try {
            nk::set_last_error(std::string("nk_scan_chunked_noalloc_device: ") + ex.what());
        } catch (...) {
        }
        return NK_ERR_INVALID;
    } catch (...) {
        return NK_ERR_INVALID;
    }
}
