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
// that device; make that first call before any stream capture.
//
// All calls share the one array.  Nothing in it has to start at zero: each
// call writes every scratch entry it reads before reading it.  Two calls
// whose work overlaps on the GPU (different streams, or different host
// threads, without ordering between them) race on the array and may produce
// wrong results; order them on one stream or synchronise between them.

#include <mutex>
#include <string>

#include "../../include/noetic_gpu.h"
#include "nk_kernels.h"

namespace {

static __device__ __align__(256) float g_scan_scratch[NK_SCAN_NOALLOC_SCRATCH_FLOATS];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
float *g_scratch_ptr[kMaxDevices] = {};

}  // namespace

extern "C" nk_status nk_scan_chunked_noalloc_device(const float *a, const float *b, float *h, uint64_t batch,
                                                    uint64_t t, uint64_t d, void *stream) {
    nk::set_last_error("");
    uint64_t n = 0;
    if (!nk::scan_elements(batch, t, d, n)) {
        nk::set_last_error("nk_scan_chunked_noalloc_device: batch * t * d overflows the scan size limit; the "
                           "scratch limit is batch * ceil(t / " + std::to_string(NK_SCAN_TIME_BLOCK) + ") * d <= " +
                           std::to_string(NK_SCAN_NOALLOC_SCRATCH_FLOATS / 3));
        return NK_ERR_INVALID;
    }
    if (n == 0) return NK_OK;
    if (!a || !b || !h) {
        nk::set_last_error("nk_scan_chunked_noalloc_device: null argument");
        return NK_ERR_INVALID;
    }
    const uint64_t blocks = (t + NK_SCAN_TIME_BLOCK - 1) / NK_SCAN_TIME_BLOCK;
    const bool huge = batch > (1ull << 32) || t > (1ull << 40) || d > (1ull << 32);
    const uint64_t need = huge ? ~0ull : nk::scan_chunked_scratch_floats((int64_t)batch, (int64_t)t, (int64_t)d);
    if (huge || need > NK_SCAN_NOALLOC_SCRATCH_FLOATS) {
        nk::set_last_error("nk_scan_chunked_noalloc_device: batch * ceil(t / " +
                           std::to_string(NK_SCAN_TIME_BLOCK) + ") * d = " +
                           (huge ? std::string("(overflow)") : std::to_string(batch * blocks * d)) +
                           " exceeds the fixed scratch limit of " +
                           std::to_string(NK_SCAN_NOALLOC_SCRATCH_FLOATS / 3) +
                           "; use nk_scan_device for larger scans");
        return NK_ERR_INVALID;
    }
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
        nk::set_last_error(std::string("nk_scan_chunked_noalloc_device: no usable current device: ") +
                           cudaGetErrorString(e));
        return NK_ERR_CUDA;
    }
    float *scratch = nullptr;
    {
        std::lock_guard<std::mutex> lock(g_mu);
        if (!g_scratch_ptr[dev]) {
            void *p = nullptr;
            e = cudaGetSymbolAddress(&p, g_scan_scratch);
            if (e != cudaSuccess) {
                cudaGetLastError();
                nk::set_last_error(std::string("nk_scan_chunked_noalloc_device: cudaGetSymbolAddress failed: ") +
                                   cudaGetErrorString(e));
                return NK_ERR_CUDA;
            }
            g_scratch_ptr[dev] = (float *)p;
        }
        scratch = g_scratch_ptr[dev];
    }
    e = nk::scan_chunked((const float *)a, (const float *)b, h, (int64_t)batch, (int64_t)t, (int64_t)d, scratch,
                         (cudaStream_t)stream);
    if (e != cudaSuccess) {
        cudaGetLastError();
        nk::set_last_error(std::string("nk_scan_chunked_noalloc_device: launch failed: ") + cudaGetErrorString(e));
        return NK_ERR_CUDA;
    }
    return NK_OK;
}
