// scan.cu -- the first-order linear recurrence h_t = a_t h_{t-1} + b_t over
// [batch, T, D] (layout (b*T + t)*D + j), scan.rs:35-225, and its adjoint
// c_t = g_t + a_{t+1} c_{t+1} (scan.rs:227-260) in the same two forms.
//
// scan_sequential: one thread per (b, j) walks time; loads are coalesced
//   along j.  Optimal when batch * D fills the GPU.
// scan_chunked: the work-efficient three-pass associative scan of
//   scan_chunked (scan.rs:79-97) with time blocks mapped to threads:
//     1. local scan of each time block from zero plus its decay product;
//     2. composition of block maps, (A_L, B_L) then (A_R, B_R) ==
//        (A_R A_L, A_R B_L + B_R), giving the carry entering each block;
//     3. fold h_t += (prod_{r<=t} a_r) * carry_in, stopping once the product
//        reaches zero.
//   The reference flushes decay products below 1e-30 to zero to dodge slow
//   x86 denormals; GPU denormal arithmetic is full speed, so products decay
//   naturally (values below 1e-30 times an O(1) carry cannot move an f32 h
//   of the same row beyond rounding).

#include "../../include/noetic_gpu.h"
#include "nk_common.cuh"
#include "nk_kernels.h"

namespace nk {

namespace {

constexpr int SCAN_TB = 256;  // time steps per block in the chunked scan
// The public header states the time block in the no-allocation scan's limit.
static_assert(SCAN_TB == (int)NK_SCAN_TIME_BLOCK, "NK_SCAN_TIME_BLOCK must equal the chunked scan's time block");
constexpr int SCAN_PB = 8;    // steps whose operands the chunked passes load ahead of use

inline unsigned blocks_for(int64_t n, int threads) { return (unsigned)((n + threads - 1) / threads); }

__global__ void scan_seq_k(const float *__restrict__ a, const float *__restrict__ b,
                           float *__restrict__ h, int64_t batch, int64_t t, int64_t d) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= batch * d) return;
    const int64_t bi = i / d, j = i - bi * d;
    const size_t base = (size_t)bi * t * d + j;
    float carry = 0.0f;
    int64_t ti = 0;
    // Unrolled by 4 so the independent loads of a and b issue ahead of the
    // dependent multiply-add chain.
    for (; ti + 4 <= t; ti += 4) {
        const size_t o = base + (size_t)ti * d;
        const float a0 = a[o], a1 = a[o + d], a2 = a[o + 2 * d], a3 = a[o + 3 * d];
        const float b0 = b[o], b1 = b[o + d], b2 = b[o + 2 * d], b3 = b[o + 3 * d];
        carry = a0 * carry + b0;
        h[o] = carry;
        carry = a1 * carry + b1;
        h[o + d] = carry;
        carry = a2 * carry + b2;
        h[o + 2 * d] = carry;
        carry = a3 * carry + b3;
        h[o + 3 * d] = carry;
    }
    for (; ti < t; ++ti) {
        const size_t o = base + (size_t)ti * d;
        carry = a[o] * carry + b[o];
        h[o] = carry;
    }
}

__global__ void scan_local_k(const float *__restrict__ a, const float *__restrict__ b,
                             float *__restrict__ h, float *__restrict__ blkA, float *__restrict__ blkB,
                             int64_t batch, int64_t t, int64_t d, int64_t nblk) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= batch * nblk * d) return;
    const int64_t j = i % d, bc = i / d;
    const int64_t c = bc % nblk, bi = bc / nblk;
    const int64_t t0 = c * SCAN_TB, t1 = min(t, t0 + SCAN_TB);
    float A = 1.0f, carry = 0.0f;
    for (int64_t tb = t0; tb < t1; tb += SCAN_PB) {
        float av[SCAN_PB], bv[SCAN_PB];
#pragma unroll
        for (int e = 0; e < SCAN_PB; ++e) {
            const size_t o = ((size_t)bi * t + tb + e) * d + j;
            av[e] = tb + e < t1 ? a[o] : 1.0f;
            bv[e] = tb + e < t1 ? b[o] : 0.0f;
        }
#pragma unroll
        for (int e = 0; e < SCAN_PB; ++e) {
            if (tb + e >= t1) break;
            carry = av[e] * carry + bv[e];
            h[((size_t)bi * t + tb + e) * d + j] = carry;
            A = A * av[e];
        }
    }
    blkA[i] = A;
    blkB[i] = carry;
}

__global__ void scan_carry_k(const float *__restrict__ blkA, const float *__restrict__ blkB,
                             float *__restrict__ carry, int64_t batch, int64_t d, int64_t nblk) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= batch * d) return;
    const int64_t bi = i / d, j = i - bi * d;
    float c = 0.0f;
    for (int64_t k = 0; k < nblk; ++k) {
        const size_t o = ((size_t)bi * nblk + k) * d + j;
        carry[o] = c;
        c = blkA[o] * c + blkB[o];
    }
}

__global__ void scan_fix_k(const float *__restrict__ a, float *__restrict__ h,
                           const float *__restrict__ carry, int64_t batch, int64_t t, int64_t d,
                           int64_t nblk) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= batch * nblk * d) return;
    const int64_t j = i % d, bc = i / d;
    const int64_t c = bc % nblk, bi = bc / nblk;
    if (c == 0) return;
    const float cin = carry[i];
    if (cin == 0.0f) return;
    const int64_t t0 = c * SCAN_TB, t1 = min(t, t0 + SCAN_TB);
    float P = 1.0f;
    for (int64_t tb = t0; tb < t1; tb += SCAN_PB) {
        float av[SCAN_PB], hv[SCAN_PB];
#pragma unroll
        for (int e = 0; e < SCAN_PB; ++e) {
            const size_t o = ((size_t)bi * t + tb + e) * d + j;
            av[e] = tb + e < t1 ? a[o] : 1.0f;
            hv[e] = tb + e < t1 ? h[o] : 0.0f;
        }
        bool done = false;
#pragma unroll
        for (int e = 0; e < SCAN_PB; ++e) {
            if (tb + e >= t1) break;
            P = P * av[e];
            if (P == 0.0f) {
                done = true;
                break;
            }
            h[((size_t)bi * t + tb + e) * d + j] = hv[e] + P * cin;
        }
        if (done) break;
    }
}

// ---- the adjoint (scan.rs:227-260): c_t = g_t + a_{t+1} c_{t+1}, c_T = 0,
// a reverse-time scan with the multiplier one step ahead.

__global__ void adj_seq_k(const float *__restrict__ a, const float *__restrict__ g, float *__restrict__ c,
                          int64_t batch, int64_t t, int64_t d) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= batch * d) return;
    const int64_t bi = i / d, j = i - bi * d;
    const size_t base = (size_t)bi * t * d + j;
    float carry = 0.0f;
    int64_t ti = t;
    for (; ti >= 4; ti -= 4) {
        const size_t o = base + (size_t)(ti - 1) * d;
        const float g0 = g[o], g1 = g[o - d], g2 = g[o - 2 * d], g3 = g[o - 3 * d];
        const float a0 = a[o], a1 = a[o - d], a2 = a[o - 2 * d], a3 = a[o - 3 * d];
        float cv = g0 + carry;
        c[o] = cv;
        carry = a0 * cv;
        cv = g1 + carry;
        c[o - d] = cv;
        carry = a1 * cv;
        cv = g2 + carry;
        c[o - 2 * d] = cv;
        carry = a2 * cv;
        cv = g3 + carry;
        c[o - 3 * d] = cv;
        carry = a3 * cv;
    }
    for (; ti > 0; --ti) {
        const size_t o = base + (size_t)(ti - 1) * d;
        const float cv = g[o] + carry;
        c[o] = cv;
        carry = a[o] * cv;
    }
}

// Pass 1: each time block from a zero carry, walking down; the block's map
// from the carry entering at its top to the carry leaving below its bottom
// is X_out = A X_in + B with A the product of the block's a and B the local
// carry leaving it.
__global__ void adj_local_k(const float *__restrict__ a, const float *__restrict__ g, float *__restrict__ c,
                            float *__restrict__ blkA, float *__restrict__ blkB, int64_t batch, int64_t t, int64_t d,
                            int64_t nblk) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= batch * nblk * d) return;
    const int64_t j = i % d, bc = i / d;
    const int64_t k = bc % nblk, bi = bc / nblk;
    const int64_t t0 = k * SCAN_TB, t1 = min(t, t0 + SCAN_TB);
    float A = 1.0f, carry = 0.0f;
    for (int64_t tb = t1 - 1; tb >= t0; tb -= SCAN_PB) {  // steps tb, tb - 1, ... walking down
        float av[SCAN_PB], gv[SCAN_PB];
#pragma unroll
        for (int e = 0; e < SCAN_PB; ++e) {
            const size_t o = ((size_t)bi * t + tb - e) * d + j;
            av[e] = tb - e >= t0 ? a[o] : 1.0f;
            gv[e] = tb - e >= t0 ? g[o] : 0.0f;
        }
#pragma unroll
        for (int e = 0; e < SCAN_PB; ++e) {
            if (tb - e < t0) break;
            const float cv = gv[e] + carry;
            c[((size_t)bi * t + tb - e) * d + j] = cv;
            carry = av[e] * cv;
            A = A * av[e];
        }
    }
    blkA[i] = A;
    blkB[i] = carry;
}

// Pass 2: compose the block maps from the last block down; carry[k] is the
// carry entering block k at its top.
__global__ void adj_carry_k(const float *__restrict__ blkA, const float *__restrict__ blkB, float *__restrict__ carry,
                            int64_t batch, int64_t d, int64_t nblk) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= batch * d) return;
    const int64_t bi = i / d, j = i - bi * d;
    float x = 0.0f;
    for (int64_t k = nblk - 1; k >= 0; --k) {
        const size_t o = ((size_t)bi * nblk + k) * d + j;
        carry[o] = x;
        x = blkA[o] * x + blkB[o];
    }
}

// Pass 3: c_t += (prod of a strictly between t and the block top) * carry_in,
// walking down, stopping once the product reaches zero.
__global__ void adj_fix_k(const float *__restrict__ a, float *__restrict__ c, const float *__restrict__ carry,
                          int64_t batch, int64_t t, int64_t d, int64_t nblk) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= batch * nblk * d) return;
    const int64_t j = i % d, bc = i / d;
    const int64_t k = bc % nblk, bi = bc / nblk;
    if (k == nblk - 1) return;
    const float cin = carry[i];
    if (cin == 0.0f) return;
    const int64_t t0 = k * SCAN_TB, t1 = min(t, t0 + SCAN_TB);
    float P = 1.0f;
    for (int64_t tb = t1 - 1; tb >= t0; tb -= SCAN_PB) {
        float av[SCAN_PB], cv[SCAN_PB];
#pragma unroll
        for (int e = 0; e < SCAN_PB; ++e) {
            const size_t o = ((size_t)bi * t + tb - e) * d + j;
            av[e] = tb - e >= t0 ? a[o] : 1.0f;
            cv[e] = tb - e >= t0 ? c[o] : 0.0f;
        }
        bool done = false;
#pragma unroll
        for (int e = 0; e < SCAN_PB; ++e) {
            if (tb - e < t0) break;
            c[((size_t)bi * t + tb - e) * d + j] = cv[e] + P * cin;
            P = P * av[e];
            if (P == 0.0f) {
                done = true;
                break;
            }
        }
        if (done) break;
    }
}

}  // namespace

size_t scan_chunked_scratch_floats(int64_t batch, int64_t t, int64_t d) {
    const int64_t nblk = (t + SCAN_TB - 1) / SCAN_TB;
    return (size_t)3 * batch * nblk * d;
}

cudaError_t scan_sequential(const float *a, const float *b, float *h, int64_t batch, int64_t t,
                            int64_t d, cudaStream_t st) {
    if (batch * t * d == 0) return cudaSuccess;
    scan_seq_k<<<blocks_for(batch * d, 128), 128, 0, st>>>(a, b, h, batch, t, d);
    return cudaGetLastError();
}

cudaError_t scan_chunked(const float *a, const float *b, float *h, int64_t batch, int64_t t,
                         int64_t d, float *scratch, cudaStream_t st) {
    if (batch * t * d == 0) return cudaSuccess;
    const int64_t nblk = (t + SCAN_TB - 1) / SCAN_TB;
    const int64_t per = batch * nblk * d;
    float *blkA = scratch, *blkB = scratch + per, *carry = scratch + 2 * per;
    scan_local_k<<<blocks_for(per, 128), 128, 0, st>>>(a, b, h, blkA, blkB, batch, t, d, nblk);
    scan_carry_k<<<blocks_for(batch * d, 128), 128, 0, st>>>(blkA, blkB, carry, batch, d, nblk);
    scan_fix_k<<<blocks_for(per, 128), 128, 0, st>>>(a, h, carry, batch, t, d, nblk);
    return cudaGetLastError();
}

cudaError_t scan_adjoint_sequential(const float *a, const float *g, float *c, int64_t batch, int64_t t, int64_t d,
                                    cudaStream_t st) {
    if (batch * t * d == 0) return cudaSuccess;
    adj_seq_k<<<blocks_for(batch * d, 128), 128, 0, st>>>(a, g, c, batch, t, d);
    return cudaGetLastError();
}

cudaError_t scan_adjoint_chunked(const float *a, const float *g, float *c, int64_t batch, int64_t t, int64_t d,
                                 float *scratch, cudaStream_t st) {
    if (batch * t * d == 0) return cudaSuccess;
    const int64_t nblk = (t + SCAN_TB - 1) / SCAN_TB;
    const int64_t per = batch * nblk * d;
    float *blkA = scratch, *blkB = scratch + per, *carry = scratch + 2 * per;
    adj_local_k<<<blocks_for(per, 128), 128, 0, st>>>(a, g, c, blkA, blkB, batch, t, d, nblk);
    adj_carry_k<<<blocks_for(batch * d, 128), 128, 0, st>>>(blkA, blkB, carry, batch, d, nblk);
    adj_fix_k<<<blocks_for(per, 128), 128, 0, st>>>(a, c, carry, batch, t, d, nblk);
    return cudaGetLastError();
}

}  // namespace nk
