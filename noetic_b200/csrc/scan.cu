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
// scan_onepass: the same block decomposition with the carries passed between
//   consecutive time blocks by decoupled look-back inside one kernel, so
//   every element is read and written once (12 bytes of HBM traffic).
//   The reference flushes decay products below 1e-30 to zero to dodge slow
//   x86 denormals; GPU denormal arithmetic is full speed, so products decay
//   naturally (values below 1e-30 times an O(1) carry cannot move an f32 h
//   of the same row beyond rounding).

#include <algorithm>

#include "../../include/noetic_gpu.h"
#include "nk_chain.cuh"
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

// ---- one-pass form: every element is read once and written once.
//
// A block is OP_TB consecutive steps of one chain (one batch entry, 32
// channels: lane = channel, so every row access is one 128-byte segment);
// warp w of a CTA holds steps [w OP_TW, (w+1) OP_TW) of it in registers.
// Each warp scans its steps from a zero state, the warps' maps compose in
// shared memory into the block's map, the block's entering state comes from
// its predecessors by decoupled look-back (nk_chain.cuh), and every step is
// finished as local + (product of the multipliers up to it) * entering
// state, the same fold as the three-pass form, before its single store.
// ADJ = the adjoint, walking down in time: step t takes the carry x, writes
// c_t = g_t + x and passes a_t c_t on.
constexpr int OP_WARPS = 8, OP_TW = 16, OP_TB = OP_WARPS * OP_TW;
constexpr int OP_ERR = 131;  // look-back wait expired

struct OpShape {
    const float *a, *b;
    float *h;
    int64_t t, d, ngrp, n_chains, slots;
};

// Element offset of step 0 of the warp's part of block tk, and its count of
// existing steps (step i sits at o0 + i * (ADJ ? -d : d)).
template <bool ADJ>
__device__ __forceinline__ int op_locate(const OpShape &sh, int64_t tk, int64_t &o0) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t blk = tk / sh.n_chains, chain = tk - blk * sh.n_chains;
    const int64_t bi = chain / sh.ngrp, j = (chain - bi * sh.ngrp) * 32 + lane;
    const int64_t q0 = blk * OP_TB + (int64_t)warp * OP_TW;
    const int64_t left = sh.t - q0;
    o0 = (bi * sh.t + (ADJ ? sh.t - 1 - q0 : q0)) * sh.d + j;
    return j >= sh.d || left <= 0 ? 0 : left >= OP_TW ? OP_TW : (int)left;
}

template <bool ADJ>
__device__ __forceinline__ void op_load(const OpShape &sh, int64_t tk, float (&m)[OP_TW], float (&v)[OP_TW]) {
    int64_t o0 = 0;
    const int nv = tk < sh.slots ? op_locate<ADJ>(sh, tk, o0) : 0;
    const int64_t sd = ADJ ? -sh.d : sh.d;
#pragma unroll
    for (int i = 0; i < OP_TW; ++i) {
        const bool ok = i < nv;
        m[i] = ok ? __ldcs(sh.a + o0 + i * sd) : 1.0f;
        v[i] = ok ? __ldcs(sh.b + o0 + i * sd) : 0.0f;
    }
}

struct OpShared {
    float sA[OP_WARPS][32], sB[OP_WARPS][32], cin[32];
    int next;
};

template <bool ADJ>
__device__ __forceinline__ void op_finish(const OpShape &sh, const ChainWs &ws, OpShared &sm, int64_t tk,
                                          float (&m)[OP_TW], float (&v)[OP_TW]) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // Local scan; m[i] becomes the factor of the entering state in step i's
    // output: the inclusive product (forward) or the exclusive one (adjoint).
    float s = 0.0f, P = 1.0f;
#pragma unroll
    for (int i = 0; i < OP_TW; ++i) {
        if (ADJ) {
            const float out = v[i] + s;
            v[i] = out;
            s = m[i] * out;
            const float pe = P;
            P = P * m[i];
            m[i] = pe;
        } else {
            s = m[i] * s + v[i];
            v[i] = s;
            P = P * m[i];
            m[i] = P;
        }
    }
    sm.sA[warp][lane] = P;
    sm.sB[warp][lane] = s;
    __syncthreads();
    if (warp == 0) {
        // Warp maps in order: (sA, sB)[w] becomes the map from the block's
        // entering state to warp w's; (eA, eB) ends as the block's map.
        float eA = 1.0f, eB = 0.0f;
#pragma unroll
        for (int w = 0; w < OP_WARPS; ++w) {
            const float wA = sm.sA[w][lane], wB = sm.sB[w][lane];
            sm.sA[w][lane] = eA;
            sm.sB[w][lane] = eB;
            eB = fmaf(wA, eB, wB);
            eA = wA * eA;
        }
        sm.cin[lane] = chain_carry(ws, tk, sh.n_chains, eA, eB, 0.0f, OP_ERR, nullptr);
    }
    __syncthreads();
    const float e = fmaf(sm.sA[warp][lane], sm.cin[lane], sm.sB[warp][lane]);
    int64_t o0 = 0;
    const int nv = op_locate<ADJ>(sh, tk, o0);
    const int64_t sd = ADJ ? -sh.d : sh.d;
#pragma unroll
    for (int i = 0; i < OP_TW; ++i)
        if (i < nv) __stcs(sh.h + o0 + i * sd, fmaf(m[i], e, v[i]));
}

template <bool ADJ>
__global__ void __launch_bounds__(OP_WARPS * 32) scan_onepass_k(const OpShape sh, ChainWs ws) {
    __shared__ OpShared sm;
    float m[OP_TW], v[OP_TW];
    if (threadIdx.x == 0) sm.next = atomicAdd(ws.ticket, 1);
    __syncthreads();
    const int64_t tk = sm.next;
    op_load<ADJ>(sh, tk, m, v);
    op_finish<ADJ>(sh, ws, sm, tk, m, v);
}

// The same scan with each block staged in shared memory: a CTA of SM_WARPS
// warps takes SM_TB = SM_WARPS * SM_TW steps of one chain, copies the block's
// a and b rows (128 bytes each) into shared memory with 16-byte cp.async,
// scans there in place (b becomes the local state, a the factor of the
// entering state), and stores each finished row once.  No block data sits in
// registers, so a CTA's whole block is in flight at once and the occupancy is
// set by shared memory.  Needs d % 4 == 0 and 16-byte aligned a, b.
constexpr int SM_WARPS = 8, SM_TW = 16, SM_TB = SM_WARPS * SM_TW;
static_assert(SM_TB == OP_TB, "both one-pass kernels take the same blocks");

__device__ __forceinline__ void cp_async16(void *smem_dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(smem_dst)),
                 "l"(src)
                 : "memory");
}

template <bool ADJ>
__global__ void __launch_bounds__(SM_WARPS * 32) scan_onepass_smem_k(const OpShape sh, ChainWs ws) {
    __shared__ __align__(16) float ta[SM_TB][32], tb[SM_TB][32];
    __shared__ float sA[SM_WARPS][32], sB[SM_WARPS][32], s_cin[32];
    __shared__ int s_tk;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) s_tk = atomicAdd(ws.ticket, 1);
    __syncthreads();
    const int64_t tk = s_tk;
    const int64_t blk = tk / sh.n_chains, chain = tk - blk * sh.n_chains;
    const int64_t bi = chain / sh.ngrp, j0 = (chain - bi * sh.ngrp) * 32;
    const int64_t q0 = blk * SM_TB;
    // Row r of the block is step q0 + r: time q0 + r (forward) or t - 1 - q0 - r.
    for (int idx = threadIdx.x; idx < SM_TB * 8; idx += SM_WARPS * 32) {
        const int r = idx >> 3, seg = idx & 7;
        const int64_t q = q0 + r, j = j0 + 4 * seg;
        if (q < sh.t && j < sh.d) {
            const size_t o = ((size_t)bi * sh.t + (size_t)(ADJ ? sh.t - 1 - q : q)) * sh.d + j;
            cp_async16(&ta[r][4 * seg], sh.a + o);
            cp_async16(&tb[r][4 * seg], sh.b + o);
        } else {
            *reinterpret_cast<float4 *>(&ta[r][4 * seg]) = make_float4(1.f, 1.f, 1.f, 1.f);
            *reinterpret_cast<float4 *>(&tb[r][4 * seg]) = make_float4(0.f, 0.f, 0.f, 0.f);
        }
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
    __syncthreads();
    // Local scan of the warp's rows from a zero state, in place.
    float st = 0.0f, P = 1.0f;
    const int r0 = warp * SM_TW;
#pragma unroll 4
    for (int i = 0; i < SM_TW; ++i) {
        const float av = ta[r0 + i][lane], bv = tb[r0 + i][lane];
        if (ADJ) {
            const float out = bv + st;
            tb[r0 + i][lane] = out;
            ta[r0 + i][lane] = P;
            st = av * out;
            P = P * av;
        } else {
            st = av * st + bv;
            P = P * av;
            tb[r0 + i][lane] = st;
            ta[r0 + i][lane] = P;
        }
    }
    sA[warp][lane] = P;
    sB[warp][lane] = st;
    __syncthreads();
    if (warp == 0) {
        float eA = 1.0f, eB = 0.0f;
#pragma unroll
        for (int w = 0; w < SM_WARPS; ++w) {
            const float wA = sA[w][lane], wB = sB[w][lane];
            sA[w][lane] = eA;
            sB[w][lane] = eB;
            eB = fmaf(wA, eB, wB);
            eA = wA * eA;
        }
        s_cin[lane] = chain_carry(ws, tk, sh.n_chains, eA, eB, 0.0f, OP_ERR, nullptr);
    }
    __syncthreads();
    const float e = fmaf(sA[warp][lane], s_cin[lane], sB[warp][lane]);
    const int64_t j = j0 + lane;
    if (j < sh.d) {
#pragma unroll 4
        for (int i = 0; i < SM_TW; ++i) {
            const int64_t q = q0 + r0 + i;
            if (q >= sh.t) break;
            __stcs(sh.h + ((size_t)bi * sh.t + (size_t)(ADJ ? sh.t - 1 - q : q)) * sh.d + j,
                   fmaf(ta[r0 + i][lane], e, tb[r0 + i][lane]));
        }
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

size_t scan_onepass_slots(int64_t batch, int64_t t, int64_t d) {
    return (size_t)batch * (size_t)((d + 31) / 32) * (size_t)((t + OP_TB - 1) / OP_TB);
}

bool scan_onepass_suits(int64_t batch, int64_t t, int64_t d) {
    // At least half of every warp's lanes carry a channel, and the chain
    // scratch stays a few percent of the data.
    return batch * t * d > 0 && d >= 16;
}

size_t scan_onepass_scratch_bytes(int64_t batch, int64_t t, int64_t d) {
    return chain_ws_bytes(scan_onepass_slots(batch, t, d));
}

cudaError_t scan_onepass(const float *a, const float *b, float *h, int64_t batch, int64_t t, int64_t d, bool adjoint,
                         void *scratch, cudaStream_t st) {
    if (batch * t * d == 0) return cudaSuccess;
    const size_t slots = scan_onepass_slots(batch, t, d);
    const int64_t ngrp = (d + 31) / 32;
    cudaError_t e = cudaMemsetAsync(scratch, 0, chain_ws_bytes(slots), st);
    if (e != cudaSuccess) return e;
    const ChainWs ws = chain_ws(scratch, slots);
    const OpShape sh{a, b, h, t, d, ngrp, batch * ngrp, (int64_t)slots};
    const bool staged = d % 4 == 0 && ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b)) & 15) == 0;
    if (staged) {
        if (adjoint)
            scan_onepass_smem_k<true><<<(unsigned)slots, SM_WARPS * 32, 0, st>>>(sh, ws);
        else
            scan_onepass_smem_k<false><<<(unsigned)slots, SM_WARPS * 32, 0, st>>>(sh, ws);
    } else if (adjoint) {
        scan_onepass_k<true><<<(unsigned)slots, OP_WARPS * 32, 0, st>>>(sh, ws);
    } else {
        scan_onepass_k<false><<<(unsigned)slots, OP_WARPS * 32, 0, st>>>(sh, ws);
    }
    return cudaGetLastError();
}

int scan_onepass_status(const void *scratch) {
    int v = 0;
    if (cudaMemcpy(&v, reinterpret_cast<const int *>(scratch) + 1, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess)
        return -1;
    return v;
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
