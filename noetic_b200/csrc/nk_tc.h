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
    // > 0: rows [0, H) and [H, 2H) (gate and value of a SwiGLU) are stored
    // interleaved in blocks of 32: gate rows 32b..32b+31, then value rows
    // 32b..32b+31, so a tile holds both halves of its channels.
    int pair_half = 0;
    alignas(64) unsigned char map_hi[128];     // 256-row boxes
    alignas(64) unsigned char map_lo[128];
    alignas(64) unsigned char map_hi128[128];  // 128-row boxes
    alignas(64) unsigned char map_lo128[128];
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
    int pair_half = 0;  // H: interleave gate / value rows (needs N == 2H, H % 32 == 0)
};

// Epilogue of one projection: either store C = acc (+ bias) (R + ...), or
// (best_val != nullptr) write each row's first maximum over every column
// half tile into best_val / best_idx [M, tc_argmax_parts(N, bn)] without storing C.
struct TcEpilogue {
    float *C = nullptr;
    int ldc = 0;
    const float *bias = nullptr;
    const float *R = nullptr;
    int ldr = 0;
    float *best_val = nullptr;
    uint32_t *best_idx = nullptr;
    // SwiGLU mode (operand with pair_half = H): instead of C, write
    // s[m, j] = SiLU(acc_gate + bias[j]) * (acc_value + bias[H + j]) for
    // j < H, row stride ldc, as f32 into C (C_lo == nullptr) or as the 3xTF32
    // operand pair hi = tf32(s) into C, lo = tf32(s - hi) into C_lo.
    bool swiglu = false;
    float *C_lo = nullptr;
    // Stream-K workspace (store and SwiGLU modes with 256-wide tiles): one
    // partial tile per SM and one counter per SM, zero between launches.
    float *ws = nullptr;
    size_t ws_floats = 0;
    int *flags = nullptr;
    int n_flags = 0;
    // L2 policies: weights evict-last, staged outputs evict-first.
    bool l2hints = true;
    // Sampling preparation (temperature > 0; store mode without bias or
    // residual, 128- or 256-wide single-SM tiles): C = pen(acc) / temperature
    // (infer.rs:239-256), the repetition penalty applied where bit (row, col)
    // of pen_bits [M][pen_words] is set (nullable: none), and per row and
    // half tile the maximum of the finite outputs and the count of +inf ones
    // into prep_max / prep_pinf [M, tc_argmax_parts(N, bn)].
    float temperature = 0.0f;
    float rep_penalty = 1.0f;
    const uint32_t *pen_bits = nullptr;
    int pen_words = 0;
    float *prep_max = nullptr;
    uint32_t *prep_pinf = nullptr;
    // Stream-K hand-off wait bound in ns (0: 1 s).  Test control: with
    // withhold_publish no partial tile is published, so the finishers' waits
    // run out and the kernel reports code 121 instead of completing.
    uint64_t handoff_wait_ns = 0;
    bool withhold_publish = false;
    // Incremented by the number of kernels tc_gemm launched (nullable): one,
    // or two when a single row of tiles is split along K and reduced.
    uint64_t *launches = nullptr;
    // Set (nullable) to the number of argmax / sampling partials per row the
    // launch wrote: tc_argmax_parts(N, bn), or ceil(N / 1024) when a small
    // projection was split along K.
    int *parts_out = nullptr;
    // RMSNorm folded into the projections (tensor.rs:298-312).  Consumer:
    // with rs_parts ([M, rs_nparts] partial sums of squares of the
    // un-normalised rows x), the A operand is the split of x * gain and each
    // accumulator row is multiplied by 1 / sqrt(sum / rs_d + rs_eps) before
    // the bias.  Producer (store mode): nx_hi / nx_lo [M, N] receive the
    // split of x * nx_gain of the stored rows x, and nx_ss [M, ceil(N / 32)]
    // each row's sum of squares per 32-column chunk.
    const float *rs_parts = nullptr;
    int rs_nparts = 0;
    int rs_d = 0;
    float rs_eps = 0.0f;
    float *nx_hi = nullptr, *nx_lo = nullptr;
    const float *nx_gain = nullptr;
    float *nx_ss = nullptr;
    // 256-wide store / SwiGLU / sampling epilogues write through bulk tensor
    // stores (C 16-byte aligned, ldc a multiple of 4) unless this is set.
    bool no_tma_store = false;
    // Tiles in the plain row-major order instead of groups of column blocks
    // whose weights fit in 24 MB of L2.
    bool no_tile_group = false;
    // Work taken over by the split-K reduction when the projection is split
    // along K (128-wide tiles in one wave, M <= 2048); *post_done (nullable) is set to 1
    // when it was, else 0 and the caller runs the separate kernel.
    //  - post_norm (store mode with N = d): after the row x is stored, its
    //    RMSNorm x * r * gain, r = 1 / sqrt(mean(x^2) + eps) (tensor.rs:298-312,
    //    the same operations as rmsnorm_rows), goes to post_norm_hi / _lo as
    //    the 3xTF32 operand pair, or as f32 to post_norm_f32.
    //  - post_ssm (store mode, N = 3E, no residual): instead of storing u, the
    //    decode step's recurrent branch (infer.rs:155-176, as ssm_decode) runs
    //    on the reduced (v, z, o) of each channel: conv ring, h update of
    //    post_state [M][k+1][E] at post_heads, and the gated output to
    //    post_g_hi / _lo (pair) or post_g_f32.
    const float *post_norm_gain = nullptr;
    float post_norm_eps = 0.0f;
    float *post_norm_hi = nullptr, *post_norm_lo = nullptr, *post_norm_f32 = nullptr;
    float *post_state = nullptr;
    const uint32_t *post_heads = nullptr;
    const float *post_conv_w = nullptr, *post_conv_b = nullptr;
    int post_k = 0;
    float *post_g_hi = nullptr, *post_g_lo = nullptr, *post_g_f32 = nullptr;
    int *post_done = nullptr;
};

// Whether the tcgen05 engine takes a projection of this shape.
bool tc_eligible(int M, int N, int K);

// Tile choice for an M x N projection: TC_PAIR (the CTA-pair kernel, 256 x
// 256 tiles on two SMs) when allow_pair and it fills every SM pair twice;
// else 128 x 256 tiles (spread over the SMs by stream-K when stream_k, the
// store and SwiGLU epilogues) or 128 x 128 tiles, whichever keeps more SM
// time busy; and the number of column tiles of that choice.
constexpr int TC_PAIR = 2;
int tc_pick_bn(int M, int N, bool allow_pair = false, bool stream_k = true);
int tc_tiles_n(int N, int bn);
// Stream-K workspace (one 128 x 256 partial tile per SM) a caller provides.
size_t tc_stream_k_ws_floats();
// Argmax partials per row: one per half tile (each epilogue warpgroup owns half the columns).
int tc_argmax_parts(int N, int bn);

cudaError_t tc_weights_build(TcWeights &w, const std::vector<TcSource> &srcs);
// hi / lo [cols, ld_out] = the operand pair of the transpose of src [rows,
// cols], output columns rows .. ld_out - 1 zero; *nonfinite (nullable) = 1
// when src holds inf or NaN.  ld_out < 2^21 * 32 rows of tiles.
cudaError_t tc_split_transposed(const float *src, int rows, int cols, int ld_out, float *hi, float *lo,
                                int *nonfinite, cudaStream_t st);
// A TcOperand over an already split [N, K] pair (K % 4 == 0); false if the
// tensor maps cannot be encoded.
bool tc_operand_from(const float *hi, const float *lo, int N, int K, TcOperand &op);
void tc_weights_free(TcWeights &w);

// epilogue(A . W^T) with A given as its hi/lo operand pair [M, K] (dense).
// A kernel whose bounded waits expire writes a nonzero code to *err.
cudaError_t tc_gemm(const float *A_hi, const float *A_lo, int M, int K, const TcOperand &W, const TcEpilogue &ep,
                    int bn, cudaStream_t st, int *err);

}  // namespace nk
