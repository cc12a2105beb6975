// tc_gemm.cu -- tcgen05 3xTF32 projection engine (sm_100a).
//
// Not yet enabled: every projection runs on the f32 CUDA-core kernels.

#include "nk_tc.h"

namespace nk {

bool tc_eligible(int, int, int) { return false; }

cudaError_t tc_weights_build(TcWeights &w, const std::vector<TcSource> &) {
    w.ready = false;
    return cudaSuccess;
}

void tc_weights_free(TcWeights &w) {
    if (w.arena) cudaFree(w.arena);
    w.arena = nullptr;
    w.ops.clear();
    w.ready = false;
}

void tc_scratch_free(TcScratch &s) {
    if (s.a_hi) cudaFree(s.a_hi);
    if (s.a_lo) cudaFree(s.a_lo);
    s = TcScratch{};
}

cudaError_t tc_gemm(const GemmArgs &, const TcOperand &, TcScratch &, cudaStream_t, int *launches) {
    if (launches) *launches = 0;
    return cudaErrorNotSupported;
}

}  // namespace nk
