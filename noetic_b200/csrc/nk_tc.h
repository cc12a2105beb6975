// nk_tc.h -- tensor-core (tcgen05, 3xTF32) projection engine.
#pragma once

#include <cstddef>
#include <cstdint>
#include <vector>
#include <cuda_runtime.h>

#include "nk_kernels.h"

namespace nk {

// One weight matrix [N, K] in 3xTF32 operand form: hi = tf32(w), lo =
// tf32(w - hi), both K-major and zero-padded to the tile grid, plus the
// TMA descriptors that load them.
struct TcOperand {
    const float *hi = nullptr, *lo = nullptr;
    int N = 0, K = 0, N_pad = 0, K_pad = 0;
    alignas(64) unsigned char map_hi[128];
    alignas(64) unsigned char map_lo[128];
};

struct TcWeights {
    bool ready = false;
    std::vector<TcOperand> ops;
    float *arena = nullptr;
    int device = -1;
};

struct TcSource {
    const float *w;
    int N, K;
};

// Activation operand staging (hi/lo split of A) reused across calls.
struct TcScratch {
    float *a_hi = nullptr, *a_lo = nullptr;
    size_t cap = 0;  // floats per buffer
};

// Whether the tcgen05 engine takes a projection of this shape.
bool tc_eligible(int M, int N, int K);

cudaError_t tc_weights_build(TcWeights &w, const std::vector<TcSource> &srcs);
void tc_weights_free(TcWeights &w);
void tc_scratch_free(TcScratch &s);

// C = epilogue(A . W^T) with the same epilogue as gemm_nt_simt.  A kernel
// whose bounded waits expire writes a nonzero code to *err (device int).
cudaError_t tc_gemm(const GemmArgs &p, const TcOperand &W, TcScratch &s, cudaStream_t st, int *err,
                    int *launches);

}  // namespace nk
