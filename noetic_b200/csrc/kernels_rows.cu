// kernels_rows.cu -- per-row and per-channel kernels of the token loop.
//
// Decoder state layout in HBM, per layer: [S][k+1][E] f32 -- rows 0..k-1 are
// the circular conv ring (infer.rs:12-19, [conv_k, inner]) and row k is the
// recurrent state h.  One conv_head per stream, shared by every layer (all
// layers advance their head once per token, infer.rs:157).

#include <algorithm>

#include "nk_chain.cuh"
#include "nk_common.cuh"
#include "nk_kernels.h"

namespace nk {

namespace {

constexpr int KMAX = 64;

inline unsigned blocks_for(int64_t n, int threads) { return (unsigned)((n + threads - 1) / threads); }

__global__ void embed_rows_k(const uint32_t *__restrict__ tokens, const float *__restrict__ emb,
                             float *__restrict__ x, int M, int d, int vocab, int *err) {
    pdl_wait();
    pdl_trigger();
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (int64_t)M * d) return;
    const int m = (int)(i / d), j = (int)(i - (int64_t)m * d);
    uint32_t t = tokens[m];
    if (t >= (uint32_t)vocab) {
        if (j == 0) atomicExch(err, 1);
        t = 0;
    }
    x[i] = emb[(size_t)t * d + j];
}

__global__ void embed_prompt_k(const uint32_t *__restrict__ ids, const uint32_t *__restrict__ lens,
                               int max_t, int t0, int tc, const float *__restrict__ emb,
                               float *__restrict__ x, int S, int d, int vocab, int *err) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (int64_t)S * tc * d) return;
    const int64_t row = i / d;
    const int j = (int)(i - row * d);
    const int s = (int)(row / tc), t = (int)(row - (int64_t)s * tc);
    uint32_t tok = 0;
    if (t0 + t < (int)lens[s]) {
        tok = ids[(size_t)s * max_t + t0 + t];
        if (tok >= (uint32_t)vocab) {
            if (j == 0) atomicExch(err, 1);
            tok = 0;
        }
    }
    x[i] = emb[(size_t)tok * d + j];
}

// Stores one produced activation either as f32 or as the 3xTF32 operand pair
// (hi = tf32(v), lo = tf32(v - hi)) that the tensor-core projection reads.
__device__ __forceinline__ void put(const RowOut &o, size_t i, float v) {
    if (o.hi) {
        const float h = tf32_round(v);
        o.hi[i] = h;
        o.lo[i] = tf32_round(v - h);
    } else {
        o.f32[i] = v;
    }
}

__device__ __forceinline__ void put4(const RowOut &o, size_t i, float4 v) {
    if (o.hi) {
        float4 h, l;
        h.x = tf32_round(v.x); l.x = tf32_round(v.x - h.x);
        h.y = tf32_round(v.y); l.y = tf32_round(v.y - h.y);
        h.z = tf32_round(v.z); l.z = tf32_round(v.z - h.z);
        h.w = tf32_round(v.w); l.w = tf32_round(v.w - h.w);
        *reinterpret_cast<float4 *>(o.hi + i) = h;
        *reinterpret_cast<float4 *>(o.lo + i) = l;
    } else {
        *reinterpret_cast<float4 *>(o.f32 + i) = v;
    }
}

// One warp per row.
__global__ void rmsnorm_k(const float *__restrict__ x, const float *__restrict__ gain, float eps, RowOut out,
                          int M, int d) {
    pdl_wait();
    pdl_trigger();
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (warp >= M) return;
    const float *xr = x + (size_t)warp * d;
    float ms = 0.0f;
    for (int j = lane; j < d; j += 32) ms = fmaf(xr[j], xr[j], ms);
    ms = warp_sum(ms);
    const float r = 1.0f / sqrtf(ms / (float)d + eps);
    const size_t base = (size_t)warp * d;
    for (int j = lane; j < d; j += 32) put(out, base + j, xr[j] * r * gain[j]);
}

__global__ void advance_heads_k(uint32_t *heads, const uint32_t *adv, int S, int k) {
    pdl_wait();
    pdl_trigger();
    const int s = blockIdx.x * blockDim.x + threadIdx.x;
    if (s >= S) return;
    const uint32_t a = adv ? adv[s] : 1u;
    heads[s] = (uint32_t)((heads[s] + (uint64_t)a) % (uint32_t)k);
}

// After a prompt chunk [t0, t0+tc): each stream advanced by its valid count.
__global__ void advance_heads_prompt_k(uint32_t *heads, const uint32_t *lens, int t0, int tc, int S,
                                       int k) {
    const int s = blockIdx.x * blockDim.x + threadIdx.x;
    if (s >= S) return;
    int nv = (int)lens[s] - t0;
    nv = nv < 0 ? 0 : (nv > tc ? tc : nv);
    heads[s] = (uint32_t)((heads[s] + (uint64_t)nv) % (uint32_t)k);
}

// infer.rs:155-176 for VW consecutive channels of one stream (VW = 4 uses
// 16-byte loads; rows of u, the ring, h and g are 16-byte aligned when E % 4 == 0).
template <int K, int VW>
__global__ void ssm_decode_k(const float *__restrict__ u, float *__restrict__ state,
                             const uint32_t *__restrict__ heads, const float *__restrict__ conv_w,
                             const float *__restrict__ conv_b, RowOut g, int S, int E, int k_dyn) {
    pdl_wait();
    pdl_trigger();
    const int k = K > 0 ? K : k_dyn;
    const int j0 = (blockIdx.x * blockDim.x + threadIdx.x) * VW;
    if (j0 >= E) return;
    for (int s = blockIdx.y; s < S; s += gridDim.y) {
        const float *ur = u + (size_t)s * 3 * E;
        float *ring = state + (size_t)s * (k + 1) * E;
        const uint32_t head = heads[s];
        float v[VW], sum[VW], z[VW], o[VW], h[VW];
        if (VW == 4) {
            const float4 a = *reinterpret_cast<const float4 *>(ur + j0);
            const float4 b = *reinterpret_cast<const float4 *>(ur + E + j0);
            const float4 c = *reinterpret_cast<const float4 *>(ur + 2 * E + j0);
            const float4 hh = *reinterpret_cast<const float4 *>(ring + (size_t)k * E + j0);
            const float4 cb = *reinterpret_cast<const float4 *>(conv_b + j0);
            const float4 w0 = *reinterpret_cast<const float4 *>(conv_w + j0);
            v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
            z[0] = b.x; z[1] = b.y; z[2] = b.z; z[3] = b.w;
            o[0] = c.x; o[1] = c.y; o[2] = c.z; o[3] = c.w;
            h[0] = hh.x; h[1] = hh.y; h[2] = hh.z; h[3] = hh.w;
            sum[0] = cb.x + w0.x * v[0]; sum[1] = cb.y + w0.y * v[1];
            sum[2] = cb.z + w0.z * v[2]; sum[3] = cb.w + w0.w * v[3];
            *reinterpret_cast<float4 *>(ring + (size_t)head * E + j0) = a;
        } else {
#pragma unroll
            for (int c = 0; c < VW; ++c) {
                const int j = j0 + c;
                v[c] = ur[j];
                z[c] = ur[E + j];
                o[c] = ur[2 * E + j];
                h[c] = ring[(size_t)k * E + j];
                sum[c] = conv_b[j] + conv_w[j] * v[c];
                ring[(size_t)head * E + j] = v[c];
            }
        }
        // Older taps q = 1..k-1 (q = 0 is the value just written), q ascending
        // as in the reference's sum.
        for (int q = 1; q < k; ++q) {
            const uint32_t slot = (head + (uint32_t)k - (uint32_t)q) % (uint32_t)k;
            if (VW == 4) {
                const float4 r = *reinterpret_cast<const float4 *>(ring + (size_t)slot * E + j0);
                const float4 w = *reinterpret_cast<const float4 *>(conv_w + (size_t)q * E + j0);
                sum[0] = sum[0] + w.x * r.x; sum[1] = sum[1] + w.y * r.y;
                sum[2] = sum[2] + w.z * r.z; sum[3] = sum[3] + w.w * r.w;
            } else {
#pragma unroll
                for (int c = 0; c < VW; ++c)
                    sum[c] = sum[c] + conv_w[(size_t)q * E + j0 + c] * ring[(size_t)slot * E + j0 + c];
            }
        }
        float gv[VW];
#pragma unroll
        for (int c = 0; c < VW; ++c) {
            const float value = silu(sum[c]);
            const float decay = sigmoid(z[c]);
            h[c] = decay * h[c] + (1.0f - decay) * value;
            gv[c] = h[c] * silu(o[c]);
        }
        const size_t gi = (size_t)s * E + j0;
        if (VW == 4) {
            float4 hh, gg;
            hh.x = h[0]; hh.y = h[1]; hh.z = h[2]; hh.w = h[3];
            gg.x = gv[0]; gg.y = gv[1]; gg.z = gv[2]; gg.w = gv[3];
            *reinterpret_cast<float4 *>(ring + (size_t)k * E + j0) = hh;
            put4(g, gi, gg);
        } else {
#pragma unroll
            for (int c = 0; c < VW; ++c) {
                ring[(size_t)k * E + j0 + c] = h[c];
                put(g, gi + c, gv[c]);
            }
        }
    }
}

// Sequential-in-time prefill of one prompt chunk for one (stream, channel):
// dwconv (autograd.rs:550-575) continuing from the ring, SiLU, decay, the
// scan h_t = a_t h_{t-1} + (1 - a_t) v_t (model.rs:156-163), output gate.
template <int K>
__global__ void ssm_prefill_seq_k(const float *__restrict__ u, float *__restrict__ state,
                                  const uint32_t *__restrict__ heads, const uint32_t *__restrict__ lens,
                                  int t0, int tc, const float *__restrict__ conv_w,
                                  const float *__restrict__ conv_b, RowOut y, int S,
                                  int E, int k_dyn) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (int64_t)S * E) return;
    const int s = (int)(i / E), j = (int)(i - (int64_t)s * E);
    const int k = K > 0 ? K : k_dyn;
    constexpr int W = K > 0 ? K : KMAX;
    const int len = (int)lens[s];
    int nv = len - t0;
    nv = nv < 0 ? 0 : (nv > tc ? tc : nv);
    float *ring = state + (size_t)s * (k + 1) * E;
    const uint32_t head0 = heads[s];
    float win[W];
    float w[W];
    // win[q] = raw v at position (current - q); before the chunk the ring
    // holds position -1 at head0, -2 at head0-1, ...
#pragma unroll
    for (int q = 0; q < W; ++q) {
        if (q < k) {
            const uint32_t slot = (head0 + (uint32_t)k - (uint32_t)q) % (uint32_t)k;
            win[q] = ring[(size_t)slot * E + j];
            w[q] = conv_w[(size_t)q * E + j];
        } else {
            win[q] = 0.0f;
            w[q] = 0.0f;
        }
    }
    const float bias = conv_b[j];
    float h = ring[(size_t)k * E + j];
    const float *ur = u + (size_t)s * tc * 3 * E;
    const size_t ybase = (size_t)s * tc * E + j;
    for (int t = 0; t < nv; ++t) {
        const float *row = ur + (size_t)t * 3 * E;
        const float v = row[j];
#pragma unroll
        for (int q = W - 1; q > 0; --q) win[q] = win[q - 1];
        win[0] = v;
        float sum = bias;
#pragma unroll
        for (int q = 0; q < W; ++q)
            if (q < k) sum = sum + w[q] * win[q];
        const float value = silu(sum);
        const float decay = sigmoid(row[E + j]);
        h = decay * h + (1.0f - decay) * value;
        put(y, ybase + (size_t)t * E, h * silu(row[2 * E + j]));
    }
    for (int t = nv; t < tc; ++t) put(y, ybase + (size_t)t * E, 0.0f);
    if (nv > 0) {
        const uint32_t head1 = (uint32_t)((head0 + (uint64_t)nv) % (uint32_t)k);
#pragma unroll
        for (int q = 0; q < W; ++q)
            if (q < k) {
                const uint32_t slot = (head1 + (uint32_t)k - (uint32_t)q) % (uint32_t)k;
                ring[(size_t)slot * E + j] = win[q];
            }
        ring[(size_t)k * E + j] = h;
    }
}

// ---- time-parallel prefill: blocks of TB positions per (stream, channel)
constexpr int TB = 64;
constexpr int PB = 8;  // positions whose operands are loaded ahead of use

__device__ __forceinline__ float raw_v(const float *ur, const float *ring, uint32_t head0, int k,
                                       int p, int E, int j) {
    // p >= 0: a position inside the chunk; p < 0: one of the k-1 positions
    // before it, held in the ring (p = -1 at head0).
    if (p >= 0) return ur[(size_t)p * 3 * E + j];
    const uint32_t slot = (uint32_t)(((int)head0 + 1 + p + 2 * k) % k);
    return ring[(size_t)slot * E + j];
}

// Pass 1: local scan of one time block from h = 0; writes h_local into y and
// the block's (decay product, final local h).  KW > 0: conv widths k <= KW,
// the window of raw v in registers; KW == 0: any width, every tap loaded.
template <int KW>
__global__ void ssm_chunk_local_k(const float *__restrict__ u, const float *__restrict__ state,
                                  const uint32_t *__restrict__ heads, const uint32_t *__restrict__ lens,
                                  int t0, int tc, const float *__restrict__ conv_w,
                                  const float *__restrict__ conv_b, float *__restrict__ y,
                                  float *__restrict__ blkA, float *__restrict__ blkH, int S, int E,
                                  int k, int nblk) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (int64_t)S * nblk * E) return;
    const int j = (int)(i % E);
    const int64_t sc = i / E;
    const int c = (int)(sc % nblk), s = (int)(sc / nblk);
    int nv = (int)lens[s] - t0;
    nv = nv < 0 ? 0 : (nv > tc ? tc : nv);
    const int p0 = c * TB, p1 = min(nv, p0 + TB);
    float A = 1.0f, h = 0.0f;
    if (p0 < p1) {
        const float *ur = u + (size_t)s * tc * 3 * E;
        const float *ring = state + (size_t)s * (k + 1) * E;
        const uint32_t head0 = heads[s];
        const float bias = conv_b[j];
        float *yr = y + (size_t)s * tc * E;
        // Conv taps and the window of raw v in registers: before position p
        // is shifted in, win[q] = v at p - 1 - q (so after the shift win[q] =
        // v at p - q).  The operands of PB positions are loaded ahead of
        // their use, so the loads overlap instead of waiting one round trip
        // per position.
        constexpr int W = KW > 0 ? KW : 1;
        float cw[W], win[W];
#pragma unroll
        for (int q = 0; q < W; ++q) {
            cw[q] = q < k ? conv_w[(size_t)q * E + j] : 0.0f;
            win[q] = (KW > 0 && q + 1 < k) ? raw_v(ur, ring, head0, k, p0 - 1 - q, E, j) : 0.0f;
        }
        for (int pb = p0; pb < p1; pb += PB) {
            float vv[PB], zz[PB];
#pragma unroll
            for (int e = 0; e < PB; ++e) {
                const int p = pb + e;
                vv[e] = p < p1 ? ur[(size_t)p * 3 * E + j] : 0.0f;
                zz[e] = p < p1 ? ur[(size_t)p * 3 * E + E + j] : 0.0f;
            }
#pragma unroll
            for (int e = 0; e < PB; ++e) {
                const int p = pb + e;
                if (p >= p1) break;
                float sum = bias;
                if constexpr (KW > 0) {
#pragma unroll
                    for (int q = W - 1; q > 0; --q) win[q] = win[q - 1];
                    win[0] = vv[e];
#pragma unroll
                    for (int q = 0; q < W; ++q)
                        if (q < k) sum = sum + cw[q] * win[q];
                } else {
                    for (int q = 0; q < k; ++q)
                        sum = sum + conv_w[(size_t)q * E + j] * (q == 0 ? vv[e] : raw_v(ur, ring, head0, k, p - q, E, j));
                }
                const float value = silu(sum);
                const float decay = sigmoid(zz[e]);
                h = decay * h + (1.0f - decay) * value;
                A = A * decay;
                yr[(size_t)p * E + j] = h;
            }
        }
    }
    blkA[i] = A;
    blkH[i] = h;
}

// Pass 2: compose block maps in order, (A_L, H_L) then (A_R, H_R) ==
// (A_R A_L, A_R H_L + H_R) (scan.rs:5-8); carry[c] = state entering block c.
__global__ void ssm_chunk_carry_k(const float *__restrict__ state, const uint32_t *__restrict__ lens,
                                  int t0, int tc, const float *__restrict__ blkA,
                                  const float *__restrict__ blkH, float *__restrict__ carry, int S,
                                  int E, int k, int nblk) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (int64_t)S * E) return;
    const int s = (int)(i / E), j = (int)(i - (int64_t)s * E);
    float c = state[(size_t)s * (k + 1) * E + (size_t)k * E + j];
    for (int b = 0; b < nblk; ++b) {
        const size_t o = ((size_t)s * nblk + b) * E + j;
        carry[o] = c;
        c = blkA[o] * c + blkH[o];
    }
}

// Pass 3: h_t = h_local_t + (prod a) * carry_in, y = h * SiLU(o); the last
// block of each stream also writes h and the conv ring back to the state.
__global__ void ssm_chunk_fix_k(const float *__restrict__ u, float *__restrict__ state,
                                const uint32_t *__restrict__ heads, const uint32_t *__restrict__ lens,
                                int t0, int tc, const float *y, RowOut yout,
                                const float *__restrict__ carry, int S, int E, int k, int nblk) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (int64_t)S * nblk * E) return;
    const int j = (int)(i % E);
    const int64_t sc = i / E;
    const int c = (int)(sc % nblk), s = (int)(sc / nblk);
    int nv = (int)lens[s] - t0;
    nv = nv < 0 ? 0 : (nv > tc ? tc : nv);
    const int p0 = c * TB, p1 = min(nv, p0 + TB);
    const float *yr = y + (size_t)s * tc * E;
    const size_t ybase = (size_t)s * tc * E + j;
    if (p0 >= p1) {
        for (int p = max(p0, nv); p < min(tc, p0 + TB); ++p) put(yout, ybase + (size_t)p * E, 0.0f);
        return;
    }
    const float *ur = u + (size_t)s * tc * 3 * E;
    const float cin = carry[i];
    float P = 1.0f, h = 0.0f;
    for (int pb = p0; pb < p1; pb += PB) {
        float zz[PB], oo[PB], yl[PB];  // loaded PB positions ahead
#pragma unroll
        for (int e = 0; e < PB; ++e) {
            const int p = pb + e;
            zz[e] = p < p1 ? ur[(size_t)p * 3 * E + E + j] : 0.0f;
            oo[e] = p < p1 ? ur[(size_t)p * 3 * E + 2 * E + j] : 0.0f;
            yl[e] = p < p1 ? yr[(size_t)p * E + j] : 0.0f;
        }
#pragma unroll
        for (int e = 0; e < PB; ++e) {
            const int p = pb + e;
            if (p >= p1) break;
            const float decay = sigmoid(zz[e]);
            P = P * decay;
            h = yl[e] + P * cin;
            put(yout, ybase + (size_t)p * E, h * silu(oo[e]));
        }
    }
    for (int p = p1; p < min(tc, p0 + TB); ++p) put(yout, ybase + (size_t)p * E, 0.0f);
    if (p1 == nv) {
        // Last block holding valid positions: write the state back.
        float *ring = state + (size_t)s * (k + 1) * E;
        const uint32_t head0 = heads[s];
        const uint32_t head1 = (uint32_t)((head0 + (uint64_t)nv) % (uint32_t)k);
        float win[KMAX];
        for (int q = 0; q < k; ++q) win[q] = raw_v(ur, ring, head0, k, nv - 1 - q, E, j);
        for (int q = 0; q < k; ++q) {
            const uint32_t slot = (head1 + (uint32_t)k - (uint32_t)q) % (uint32_t)k;
            ring[(size_t)slot * E + j] = win[q];
        }
        ring[(size_t)k * E + j] = h;
    }
}

// ---- one-pass time-parallel prefill: the scan of the chunk's positions in
// one kernel, carries between time blocks by decoupled look-back
// (nk_chain.cuh).  A CTA of OP_WARPS warps takes OP_TB positions of one chain
// (a stream and 32 consecutive channels, lane = channel); warp w holds
// positions [w OP_TW, (w+1) OP_TW) of the block in registers.  Each position's
// v, z and o are read once and its gated output written once.
constexpr int OP_WARPS = 8, OP_TW = 16, OP_TB = OP_WARPS * OP_TW;
constexpr int OP_ERR = 131;  // look-back wait expired

template <int KW>
__global__ void __launch_bounds__(OP_WARPS * 32) ssm_onepass_k(
    const float *__restrict__ u, float *__restrict__ state, const uint32_t *__restrict__ heads,
    const uint32_t *__restrict__ lens, int t0, int tc, const float *__restrict__ conv_w,
    const float *__restrict__ conv_b, RowOut yout, int E, int k, int ngrp, int n_chains, ChainWs ws, int *err) {
    __shared__ int s_tk;
    __shared__ float sA[OP_WARPS][32], sB[OP_WARPS][32], s_cin[32];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) s_tk = atomicAdd(ws.ticket, 1);
    __syncthreads();
    const int tk = s_tk;
    const int blk = tk / n_chains, chain = tk - blk * n_chains;
    const int s = chain / ngrp, j = (chain - s * ngrp) * 32 + lane;
    const bool col = j < E;
    int nv = (int)lens[s] - t0;
    nv = nv < 0 ? 0 : (nv > tc ? tc : nv);
    const int p0 = blk * OP_TB + warp * OP_TW;
    const int left = col ? nv - p0 : 0;
    const int nw = left <= 0 ? 0 : left >= OP_TW ? OP_TW : left;  // valid positions of the warp
    const float *ur = u + (size_t)s * tc * 3 * E;
    float *ring = state + (size_t)s * (k + 1) * E;
    const uint32_t head0 = heads[s];
    const size_t ybase = (size_t)s * tc * E + j;

    // Decay and input of the warp's positions; m becomes the inclusive decay
    // product, v the local state (from zero).
    float m[OP_TW], v[OP_TW], o[OP_TW];
    if (nw > 0) {
        const float bias = conv_b[j];
        constexpr int W = KW > 0 ? KW : 1;
        float cw[W], win[W];
#pragma unroll
        for (int q = 0; q < W; ++q) {
            cw[q] = q < k ? conv_w[(size_t)q * E + j] : 0.0f;
            win[q] = (KW > 0 && q + 1 < k) ? raw_v(ur, ring, head0, k, p0 - 1 - q, E, j) : 0.0f;
        }
#pragma unroll
        for (int i = 0; i < OP_TW; ++i) {
            const bool ok = i < nw;
            const float *row = ur + (size_t)(p0 + i) * 3 * E;
            v[i] = ok ? __ldcs(row + j) : 0.0f;
            m[i] = ok ? __ldcs(row + E + j) : 0.0f;
            o[i] = ok ? __ldcs(row + 2 * E + j) : 0.0f;
        }
#pragma unroll
        for (int i = 0; i < OP_TW; ++i) {
            if (i >= nw) {
                m[i] = 1.0f;
                v[i] = 0.0f;
                continue;
            }
            float sum = bias;
            if constexpr (KW > 0) {
#pragma unroll
                for (int q = W - 1; q > 0; --q) win[q] = win[q - 1];
                win[0] = v[i];
#pragma unroll
                for (int q = 0; q < W; ++q)
                    if (q < k) sum = sum + cw[q] * win[q];
            } else {
                for (int q = 0; q < k; ++q)
                    sum = sum + conv_w[(size_t)q * E + j] *
                                    (q == 0 ? v[i] : raw_v(ur, ring, head0, k, p0 + i - q, E, j));
            }
            const float value = silu(sum);
            const float decay = sigmoid(m[i]);
            m[i] = decay;
            v[i] = (1.0f - decay) * value;
        }
    } else {
#pragma unroll
        for (int i = 0; i < OP_TW; ++i) {
            m[i] = 1.0f;
            v[i] = 0.0f;
            o[i] = 0.0f;
        }
    }
    // h = decay h + (1 - decay) value (model.rs:156-163) from h = 0.
    float h = 0.0f, P = 1.0f;
#pragma unroll
    for (int i = 0; i < OP_TW; ++i) {
        h = m[i] * h + v[i];
        v[i] = h;
        P = P * m[i];
        m[i] = P;
    }
    sA[warp][lane] = P;
    sB[warp][lane] = h;
    __syncthreads();
    if (warp == 0) {
        float eA = 1.0f, eB = 0.0f;
#pragma unroll
        for (int w = 0; w < OP_WARPS; ++w) {
            const float wA = sA[w][lane], wB = sB[w][lane];
            sA[w][lane] = eA;
            sB[w][lane] = eB;
            eB = fmaf(wA, eB, wB);
            eA = wA * eA;
        }
        // A chain starts from the layer's recurrent state.
        const float first = (tk < n_chains && col) ? ring[(size_t)k * E + j] : 0.0f;
        s_cin[lane] = chain_carry(ws, tk, n_chains, eA, eB, first, OP_ERR, err);
    }
    __syncthreads();
    if (!col) return;
    const float e = fmaf(sA[warp][lane], s_cin[lane], sB[warp][lane]);
    float hlast = 0.0f;
#pragma unroll
    for (int i = 0; i < OP_TW; ++i) {
        const int p = p0 + i;
        if (p >= tc) break;
        if (i < nw) {
            const float hv = fmaf(m[i], e, v[i]);
            if (p == nv - 1) hlast = hv;
            put(yout, ybase + (size_t)p * E, hv * silu(o[i]));
        } else {
            put(yout, ybase + (size_t)p * E, 0.0f);
        }
    }
    if (nw > 0 && p0 + nw == nv) {
        // The warp holding the last valid position writes h and the conv ring
        // back to the state (raw v of positions nv-1 .. nv-k, gathered first).
        const uint32_t head1 = (uint32_t)((head0 + (uint64_t)nv) % (uint32_t)k);
        float wv[KMAX];
        for (int q = 0; q < k; ++q) wv[q] = raw_v(ur, ring, head0, k, nv - 1 - q, E, j);
        for (int q = 0; q < k; ++q) {
            const uint32_t slot = (head1 + (uint32_t)k - (uint32_t)q) % (uint32_t)k;
            ring[(size_t)slot * E + j] = wv[q];
        }
        ring[(size_t)k * E + j] = hlast;
    }
}

// The same prefill with each block staged in shared memory: the v rows of
// the block and of the OP_HALO positions before it, and its z and o rows,
// arrive by 16-byte cp.async (every row segment is 128 bytes of one
// position); each warp scans its positions there in place (v becomes the
// local state, z the decay product) and writes each gated output once.
// Needs E % 4 == 0, a 16-byte aligned u and conv widths k <= OP_HALO.
constexpr int OP_HALO = 8;
constexpr size_t OP_SMEM_BYTES = (size_t)(OP_HALO + 3 * OP_TB) * 32 * sizeof(float);

__device__ __forceinline__ void cp_async16(void *smem_dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(smem_dst)),
                 "l"(src)
                 : "memory");
}

template <int KW>
__global__ void __launch_bounds__(OP_WARPS * 32) ssm_onepass_smem_k(
    const float *__restrict__ u, float *__restrict__ state, const uint32_t *__restrict__ heads,
    const uint32_t *__restrict__ lens, int t0, int tc, const float *__restrict__ conv_w,
    const float *__restrict__ conv_b, RowOut yout, int E, int k, int ngrp, int n_chains, ChainWs ws, int *err) {
    extern __shared__ __align__(16) float op_smem[];
    float(*tv)[32] = reinterpret_cast<float(*)[32]>(op_smem);                       // [OP_HALO + OP_TB]
    float(*tz)[32] = reinterpret_cast<float(*)[32]>(op_smem + (OP_HALO + OP_TB) * 32);  // [OP_TB]
    float(*to)[32] = reinterpret_cast<float(*)[32]>(op_smem + (OP_HALO + 2 * OP_TB) * 32);
    __shared__ int s_tk;
    __shared__ float sA[OP_WARPS][32], sB[OP_WARPS][32], s_cin[32];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) s_tk = atomicAdd(ws.ticket, 1);
    __syncthreads();
    const int tk = s_tk;
    const int blk = tk / n_chains, chain = tk - blk * n_chains;
    const int s = chain / ngrp, j0 = (chain - s * ngrp) * 32, j = j0 + lane;
    int nv = (int)lens[s] - t0;
    nv = nv < 0 ? 0 : (nv > tc ? tc : nv);
    const int pb = blk * OP_TB;  // the block's first position
    const float *ur = u + (size_t)s * tc * 3 * E;
    float *ring = state + (size_t)s * (k + 1) * E;
    const uint32_t head0 = heads[s];
    // Rows: v of positions pb - OP_HALO .. pb + OP_TB - 1, z and o of the
    // block's positions; positions before the chunk come from the ring.
    for (int idx = threadIdx.x; idx < (OP_HALO + 3 * OP_TB) * 8; idx += OP_WARPS * 32) {
        const int row = idx >> 3, seg = idx & 7, jj = j0 + 4 * seg;
        float *dst;
        int p, f;
        if (row < OP_HALO + OP_TB) {
            dst = &tv[row][4 * seg];
            p = pb - OP_HALO + row;
            f = 0;
        } else if (row < OP_HALO + 2 * OP_TB) {
            dst = &tz[row - OP_HALO - OP_TB][4 * seg];
            p = pb + row - OP_HALO - OP_TB;
            f = 1;
        } else {
            dst = &to[row - OP_HALO - 2 * OP_TB][4 * seg];
            p = pb + row - OP_HALO - 2 * OP_TB;
            f = 2;
        }
        if (jj < E && p >= 0 && p < nv) {
            cp_async16(dst, ur + (size_t)p * 3 * E + (size_t)f * E + jj);
        } else {
            float4 val = make_float4(0.f, 0.f, 0.f, 0.f);
            if (jj < E && p < 0 && p >= -(k - 1) && f == 0) {
                const uint32_t slot = (uint32_t)(((int)head0 + 1 + p + 2 * k) % k);
                val = *reinterpret_cast<const float4 *>(ring + (size_t)slot * E + jj);
            }
            *reinterpret_cast<float4 *>(dst) = val;
        }
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
    __syncthreads();
    const int r0 = warp * OP_TW;  // the warp's first row in the block
    const int left = j < E ? nv - (pb + r0) : 0;
    const int nw = left <= 0 ? 0 : left >= OP_TW ? OP_TW : left;  // valid positions of the warp
    constexpr int W = KW > 0 ? KW : OP_HALO;
    float cw[W], win[W];
    const float bias = j < E ? conv_b[j] : 0.0f;
#pragma unroll
    for (int q = 0; q < W; ++q) {
        cw[q] = (q < k && j < E) ? conv_w[(size_t)q * E + j] : 0.0f;
        // before position r0 is shifted in, win[q] = v at r0 - 1 - q
        win[q] = q + 1 < k ? tv[OP_HALO + r0 - 1 - q][lane] : 0.0f;
    }
    __syncthreads();  // every warp holds its window before rows turn into states
    float h = 0.0f, P = 1.0f;
#pragma unroll 4
    for (int i = 0; i < OP_TW; ++i) {
        const int r = r0 + i;
        float m = 1.0f, add = 0.0f;
        if (i < nw) {
#pragma unroll
            for (int q = W - 1; q > 0; --q) win[q] = win[q - 1];
            win[0] = tv[OP_HALO + r][lane];
            float sum = bias;
#pragma unroll
            for (int q = 0; q < W; ++q)
                if (q < k) sum = sum + cw[q] * win[q];
            const float value = silu(sum);
            m = sigmoid(tz[r][lane]);
            add = (1.0f - m) * value;
        }
        // h = decay h + (1 - decay) value (model.rs:156-163) from h = 0.
        h = m * h + add;
        P = P * m;
        tv[OP_HALO + r][lane] = h;
        tz[r][lane] = P;
    }
    sA[warp][lane] = P;
    sB[warp][lane] = h;
    __syncthreads();
    if (warp == 0) {
        float eA = 1.0f, eB = 0.0f;
#pragma unroll
        for (int w = 0; w < OP_WARPS; ++w) {
            const float wA = sA[w][lane], wB = sB[w][lane];
            sA[w][lane] = eA;
            sB[w][lane] = eB;
            eB = fmaf(wA, eB, wB);
            eA = wA * eA;
        }
        // A chain starts from the layer's recurrent state.
        const float first = (tk < n_chains && j < E) ? ring[(size_t)k * E + j] : 0.0f;
        s_cin[lane] = chain_carry(ws, tk, n_chains, eA, eB, first, OP_ERR, err);
    }
    __syncthreads();
    if (j >= E) return;
    const float e = fmaf(sA[warp][lane], s_cin[lane], sB[warp][lane]);
    const size_t ybase = (size_t)s * tc * E + j;
    float hlast = 0.0f;
#pragma unroll 4
    for (int i = 0; i < OP_TW; ++i) {
        const int r = r0 + i, p = pb + r;
        if (p >= tc) break;
        if (i < nw) {
            const float hv = fmaf(tz[r][lane], e, tv[OP_HALO + r][lane]);
            if (p == nv - 1) hlast = hv;
            put(yout, ybase + (size_t)p * E, hv * silu(to[r][lane]));
        } else {
            put(yout, ybase + (size_t)p * E, 0.0f);
        }
    }
    if (nw > 0 && pb + r0 + nw == nv) {
        // The warp holding the last valid position writes h and the conv ring
        // back to the state (raw v of positions nv-1 .. nv-k, gathered first).
        const uint32_t head1 = (uint32_t)((head0 + (uint64_t)nv) % (uint32_t)k);
        float wv[OP_HALO];
        for (int q = 0; q < k; ++q) wv[q] = raw_v(ur, ring, head0, k, nv - 1 - q, E, j);
        for (int q = 0; q < k; ++q) {
            const uint32_t slot = (head1 + (uint32_t)k - (uint32_t)q) % (uint32_t)k;
            ring[(size_t)slot * E + j] = wv[q];
        }
        ring[(size_t)k * E + j] = hlast;
    }
}

template <int VW>
__global__ void swiglu_k(const float *__restrict__ up, RowOut out, int M, int H) {
    const int j = (blockIdx.x * blockDim.x + threadIdx.x) * VW;
    if (j >= H) return;
    for (int m = blockIdx.y; m < M; m += gridDim.y) {
        const float *r = up + (size_t)m * 2 * H;
        const size_t o = (size_t)m * H + j;
        if (VW == 4) {
            const float4 a = *reinterpret_cast<const float4 *>(r + j);
            const float4 b = *reinterpret_cast<const float4 *>(r + H + j);
            float4 v;
            v.x = silu(a.x) * b.x; v.y = silu(a.y) * b.y; v.z = silu(a.z) * b.z; v.w = silu(a.w) * b.w;
            put4(out, o, v);
        } else {
            put(out, o, silu(r[j]) * r[H + j]);
        }
    }
}

// Per row: the best (value, index) over the column tiles' partial maxima,
// earliest tile first on ties (argmax, tensor.rs:354-365).
// One CTA per row; (value, tile) pairs reduce with "larger value, then
// earlier tile" so ties resolve to the earliest tile as in a serial scan.
__global__ void argmax_partials_k(const float *__restrict__ val, const uint32_t *__restrict__ idx, int n_tiles,
                                  int M, uint32_t *__restrict__ out) {
    pdl_wait();
    pdl_trigger();
    const int m = blockIdx.x;
    float bv = -INFINITY;
    int bt = n_tiles;
    for (int t = threadIdx.x; t < n_tiles; t += blockDim.x) {
        const float v = val[(size_t)m * n_tiles + t];
        if (v > bv) {  // strided by thread: the first t with a larger value wins
            bv = v;
            bt = t;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int ot = __shfl_xor_sync(0xffffffffu, bt, o);
        if (ov > bv || (ov == bv && ot < bt)) {
            bv = ov;
            bt = ot;
        }
    }
    __shared__ float sv[32];
    __shared__ int st[32];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) {
        sv[warp] = bv;
        st[warp] = bt;
    }
    __syncthreads();
    if (warp == 0) {
        const int nw = blockDim.x >> 5;
        bv = lane < nw ? sv[lane] : -INFINITY;
        bt = lane < nw ? st[lane] : n_tiles;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int ot = __shfl_xor_sync(0xffffffffu, bt, o);
            if (ov > bv || (ov == bv && ot < bt)) {
                bv = ov;
                bt = ot;
            }
        }
        if (lane == 0) out[m] = (bv == -INFINITY || bt >= n_tiles) ? 0u : idx[(size_t)m * n_tiles + bt];
    }
}

// Graph::softmax_ce forward per row (autograd.rs:579-624): the row maximum,
// the f32 sum of exp(v - max), p = max(exp(v_t - max) / max(sum, 1e-30),
// 1e-20), nll = -ln(p) in f64.  Row r of the block is logits row r of a
// prompt chunk (stream-major, tcc positions per stream); its position in the
// [batch, T] sequence layout is s * T + t0 + (r0 + r) % tcc with s = (r0 + r) / tcc.
// A non-finite logit sets *err = 3 (the reference rejects it).
__global__ void softmax_ce_rows_k(const float *__restrict__ logits, int V, int r0, int tcc, int T, int t0,
                                  const uint32_t *__restrict__ targets, double *__restrict__ nll,
                                  uint32_t *__restrict__ counted, int *err) {
    const int r = blockIdx.x;
    const float *row = logits + (size_t)r * V;
    const int g = r0 + r, s = g / tcc;
    const size_t pos = (size_t)s * T + t0 + (g - s * tcc);
    __shared__ float red[32];
    __shared__ int bad;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    if (threadIdx.x == 0) bad = 0;
    __syncthreads();
    float mx = -INFINITY;
    for (int j = threadIdx.x; j < V; j += blockDim.x) {
        const float v = row[j];
        if (!isfinite(v)) bad = 1;
        mx = fmaxf(mx, v);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (lane == 0) red[warp] = mx;
    __syncthreads();
    mx = lane < nw ? red[lane] : -INFINITY;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    __syncthreads();
    float sum = 0.0f;
    for (int j = threadIdx.x; j < V; j += blockDim.x) sum += expf(row[j] - mx);
    sum = warp_sum(sum);
    if (lane == 0) red[warp] = sum;
    __syncthreads();
    if (threadIdx.x == 0) {
        float tot = 0.0f;
        for (int w = 0; w < nw; ++w) tot += red[w];
        const uint32_t t = targets[pos];
        if (bad) atomicExch(err, 3);
        if (t != 0xFFFFFFFFu && t < (uint32_t)V) {
            const float inv = 1.0f / fmaxf(tot, 1e-30f);
            const float pr = fmaxf(expf(row[t] - mx) * inv, 1e-20f);
            nll[pos] = -log((double)pr);
            counted[pos] = 1u;
        } else {
            nll[pos] = 0.0;
            counted[pos] = 0u;
        }
    }
}

// Mean of nll over counted rows (1 when none), in a fixed order: thread i
// sums rows i, i + blockDim, ... ascending, then a fixed tree.
__global__ void ce_mean_k(const double *__restrict__ nll, const uint32_t *__restrict__ counted, size_t n,
                          float *out) {
    __shared__ double ssum[1024];
    __shared__ unsigned long long scnt[1024];
    double a = 0.0;
    unsigned long long c = 0;
    for (size_t i = threadIdx.x; i < n; i += blockDim.x) {
        a += nll[i];
        c += counted[i];
    }
    ssum[threadIdx.x] = a;
    scnt[threadIdx.x] = c;
    __syncthreads();
    for (int w = blockDim.x >> 1; w > 0; w >>= 1) {
        if ((int)threadIdx.x < w) {
            ssum[threadIdx.x] += ssum[threadIdx.x + w];
            scnt[threadIdx.x] += scnt[threadIdx.x + w];
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) *out = (float)(ssum[0] / (scnt[0] ? (double)scnt[0] : 1.0));
}

// Block per row: first index of the maximum over non-NaN entries; 0 when
// the maximum is -inf or every entry is NaN (tensor.rs:354-365).
__global__ void argmax_rows_k(const float *__restrict__ x, uint32_t *__restrict__ out, int V) {
    const float *row = x + (size_t)blockIdx.x * V;
    float bv = -INFINITY;
    int bi = V;
    for (int i = threadIdx.x; i < V; i += blockDim.x) {
        const float v = row[i];
        if (!isnan(v) && (v > bv || (v == bv && i < bi))) {
            bv = v;
            bi = i;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) {
            bv = ov;
            bi = oi;
        }
    }
    __shared__ float sv[32];
    __shared__ int si[32];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) {
        sv[warp] = bv;
        si[warp] = bi;
    }
    __syncthreads();
    if (warp == 0) {
        const int nw = blockDim.x >> 5;
        bv = lane < nw ? sv[lane] : -INFINITY;
        bi = lane < nw ? si[lane] : V;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ov > bv || (ov == bv && oi < bi)) {
                bv = ov;
                bi = oi;
            }
        }
        if (lane == 0) out[blockIdx.x] = (bv == -INFINITY || bi >= V) ? 0u : (uint32_t)bi;
    }
}

__global__ void gather_last_k(const float *__restrict__ x, const uint32_t *__restrict__ lens, int t0,
                              int tc, float *__restrict__ last, int S, int d) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (int64_t)S * d) return;
    const int s = (int)(i / d), j = (int)(i - (int64_t)s * d);
    const int p = (int)lens[s] - 1 - t0;
    if (p >= 0 && p < tc) last[i] = x[((size_t)s * tc + p) * d + j];
}

__global__ void gather_rows_k(const float *__restrict__ src, const uint32_t *__restrict__ idx,
                              float *__restrict__ dst, int n, int d) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (int64_t)n * d) return;
    const int r = (int)(i / d), j = (int)(i - (int64_t)r * d);
    dst[i] = src[(size_t)idx[r] * d + j];
}

__global__ void scatter_rows_k(const float *__restrict__ src, const uint32_t *__restrict__ idx,
                               float *__restrict__ dst, int n, int d) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (int64_t)n * d) return;
    const int r = (int)(i / d), j = (int)(i - (int64_t)r * d);
    dst[(size_t)idx[r] * d + j] = src[i];
}

__global__ void history_push_k(uint32_t *history, uint32_t *history_len, const uint32_t *tok, int S,
                               int window) {
    const int s = blockIdx.x * blockDim.x + threadIdx.x;
    if (s >= S || window <= 0) return;
    uint32_t *h = history + (size_t)s * window;
    uint32_t n = history_len[s];
    if (n < (uint32_t)window) {
        h[n] = tok[s];
        history_len[s] = n + 1;
    } else {
        for (int i = 0; i + 1 < window; ++i) h[i] = h[i + 1];
        h[window - 1] = tok[s];
    }
}

}  // namespace

cudaError_t embed_rows(const uint32_t *tokens, const float *emb, float *x, int M, int d, int vocab,
                       int *err, cudaStream_t st) {
    const int64_t n = (int64_t)M * d;
    if (n == 0) return cudaSuccess;
    return pdl_launch(embed_rows_k, dim3(blocks_for(n, 256)), dim3(256), 0, st, tokens, emb, x, M, d, vocab, err);
}

cudaError_t embed_prompt_chunk(const uint32_t *ids, const uint32_t *lens, int max_t, int t0, int tc,
                               const float *emb, float *x, int S, int d, int vocab, int *err,
                               cudaStream_t st) {
    const int64_t n = (int64_t)S * tc * d;
    if (n == 0) return cudaSuccess;
    embed_prompt_k<<<blocks_for(n, 256), 256, 0, st>>>(ids, lens, max_t, t0, tc, emb, x, S, d, vocab,
                                                       err);
    return cudaGetLastError();
}

cudaError_t rmsnorm_rows(const float *x, const float *gain, float eps, RowOut out, int M, int d,
                         cudaStream_t st) {
    if (M == 0) return cudaSuccess;
    return pdl_launch(rmsnorm_k, dim3(blocks_for((int64_t)M * 32, 256)), dim3(256), 0, st, x, gain, eps, out, M, d);
}

cudaError_t advance_heads(uint32_t *heads, const uint32_t *adv, int S, int k, cudaStream_t st) {
    if (S == 0) return cudaSuccess;
    return pdl_launch(advance_heads_k, dim3(blocks_for(S, 256)), dim3(256), 0, st, heads, adv, S, k);
}

cudaError_t advance_heads_prompt(uint32_t *heads, const uint32_t *lens, int t0, int tc, int S, int k,
                                 cudaStream_t st) {
    if (S == 0) return cudaSuccess;
    advance_heads_prompt_k<<<blocks_for(S, 256), 256, 0, st>>>(heads, lens, t0, tc, S, k);
    return cudaGetLastError();
}

cudaError_t ssm_decode(const float *u, float *state, const uint32_t *heads, const float *conv_w,
                       const float *conv_b, RowOut g, int S, int E, int k, cudaStream_t st) {
    if ((int64_t)S * E == 0) return cudaSuccess;
    const bool vec = (E % 4 == 0);
    const int per = vec ? 4 : 1;
    dim3 grid((unsigned)((E / per + 127) / 128), (unsigned)std::min(S, 65535));
    switch (vec ? k : -k) {
#define NK_CASE(KK)                                                                                        \
    case KK: return pdl_launch(ssm_decode_k<KK, 4>, grid, dim3(128), 0, st, u, state, heads, conv_w, conv_b, g, \
                               S, E, k);                                                                    \
    case -KK: return pdl_launch(ssm_decode_k<KK, 1>, grid, dim3(128), 0, st, u, state, heads, conv_w, conv_b, \
                                g, S, E, k);
        NK_CASE(1) NK_CASE(2) NK_CASE(3) NK_CASE(4) NK_CASE(5) NK_CASE(6) NK_CASE(7) NK_CASE(8)
#undef NK_CASE
        default:
            if (vec) return pdl_launch(ssm_decode_k<0, 4>, grid, dim3(128), 0, st, u, state, heads, conv_w, conv_b, g, S, E, k);
            return pdl_launch(ssm_decode_k<0, 1>, grid, dim3(128), 0, st, u, state, heads, conv_w, conv_b, g, S, E, k);
    }
}

cudaError_t ssm_prefill_seq(const float *u, float *state, const uint32_t *heads,
                            const uint32_t *lens, int t0, int tc, const float *conv_w,
                            const float *conv_b, RowOut y, int S, int E, int k, cudaStream_t st) {
    const int64_t n = (int64_t)S * E;
    if (n == 0) return cudaSuccess;
    if (k > KMAX) return cudaErrorInvalidValue;
    const unsigned grid = blocks_for(n, 128);
    switch (k) {
#define NK_CASE(KK)                                                                                 \
    case KK:                                                                                        \
        ssm_prefill_seq_k<KK><<<grid, 128, 0, st>>>(u, state, heads, lens, t0, tc, conv_w, conv_b, \
                                                    y, S, E, k);                                    \
        break;
        NK_CASE(1) NK_CASE(2) NK_CASE(3) NK_CASE(4) NK_CASE(5) NK_CASE(6) NK_CASE(7) NK_CASE(8)
#undef NK_CASE
        default:
            ssm_prefill_seq_k<0><<<grid, 128, 0, st>>>(u, state, heads, lens, t0, tc, conv_w, conv_b,
                                                        y, S, E, k);
    }
    return cudaGetLastError();
}

size_t ssm_prefill_chunked_scratch_floats(int S, int E, int tc) {
    const int nblk = (tc + TB - 1) / TB;
    return (size_t)3 * S * nblk * E;
}

cudaError_t ssm_prefill_chunked(const float *u, float *state, const uint32_t *heads,
                                const uint32_t *lens, int t0, int tc, const float *conv_w,
                                const float *conv_b, float *y, RowOut yout, float *scratch, int S, int E,
                                int k, cudaStream_t st) {
    if ((int64_t)S * E == 0 || tc == 0) return cudaSuccess;
    if (k > KMAX) return cudaErrorInvalidValue;
    const int nblk = (tc + TB - 1) / TB;
    const size_t per = (size_t)S * nblk * E;
    float *blkA = scratch, *blkH = scratch + per, *carry = scratch + 2 * per;
    const int64_t n = (int64_t)per;
    if (k <= 4)
        ssm_chunk_local_k<4><<<blocks_for(n, 128), 128, 0, st>>>(u, state, heads, lens, t0, tc, conv_w, conv_b, y,
                                                                 blkA, blkH, S, E, k, nblk);
    else if (k <= 8)
        ssm_chunk_local_k<8><<<blocks_for(n, 128), 128, 0, st>>>(u, state, heads, lens, t0, tc, conv_w, conv_b, y,
                                                                 blkA, blkH, S, E, k, nblk);
    else
        ssm_chunk_local_k<0><<<blocks_for(n, 128), 128, 0, st>>>(u, state, heads, lens, t0, tc, conv_w, conv_b, y,
                                                                 blkA, blkH, S, E, k, nblk);
    ssm_chunk_carry_k<<<blocks_for((int64_t)S * E, 128), 128, 0, st>>>(state, lens, t0, tc, blkA,
                                                                       blkH, carry, S, E, k, nblk);
    ssm_chunk_fix_k<<<blocks_for(n, 128), 128, 0, st>>>(u, state, heads, lens, t0, tc, y, yout, carry,
                                                        S, E, k, nblk);
    return cudaGetLastError();
}

static size_t onepass_slots(int S, int E, int tc) {
    return (size_t)S * (size_t)((E + 31) / 32) * (size_t)((tc + OP_TB - 1) / OP_TB);
}

size_t ssm_prefill_onepass_scratch_bytes(int S, int E, int tc) { return chain_ws_bytes(onepass_slots(S, E, tc)); }

cudaError_t ssm_prefill_onepass(const float *u, float *state, const uint32_t *heads, const uint32_t *lens, int t0,
                                int tc, const float *conv_w, const float *conv_b, RowOut yout, void *scratch, int S,
                                int E, int k, int *err, cudaStream_t st) {
    if ((int64_t)S * E == 0 || tc == 0) return cudaSuccess;
    if (k > KMAX) return cudaErrorInvalidValue;
    const size_t slots = onepass_slots(S, E, tc);
    if (slots > (size_t)INT32_MAX) return cudaErrorInvalidValue;
    cudaError_t e = cudaMemsetAsync(scratch, 0, chain_ws_bytes(slots), st);
    if (e != cudaSuccess) return e;
    const ChainWs ws = chain_ws(scratch, slots);
    const int ngrp = (E + 31) / 32, nc = S * ngrp;
    const dim3 grid((unsigned)slots), block(OP_WARPS * 32);
    if (E % 4 == 0 && k <= OP_HALO && (reinterpret_cast<uintptr_t>(u) & 15) == 0 &&
        (reinterpret_cast<uintptr_t>(state) & 15) == 0) {
        static bool attr_set[2] = {false, false};
        auto kern = k <= 4 ? ssm_onepass_smem_k<4> : ssm_onepass_smem_k<8>;
        bool &set = attr_set[k <= 4 ? 0 : 1];
        if (!set) {
            e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)OP_SMEM_BYTES);
            if (e != cudaSuccess) return e;
            set = true;
        }
        kern<<<grid, block, OP_SMEM_BYTES, st>>>(u, state, heads, lens, t0, tc, conv_w, conv_b, yout, E, k, ngrp, nc,
                                                 ws, err);
        return cudaGetLastError();
    }
    if (k <= 4)
        ssm_onepass_k<4><<<grid, block, 0, st>>>(u, state, heads, lens, t0, tc, conv_w, conv_b, yout, E, k, ngrp, nc,
                                                 ws, err);
    else if (k <= 8)
        ssm_onepass_k<8><<<grid, block, 0, st>>>(u, state, heads, lens, t0, tc, conv_w, conv_b, yout, E, k, ngrp, nc,
                                                 ws, err);
    else
        ssm_onepass_k<0><<<grid, block, 0, st>>>(u, state, heads, lens, t0, tc, conv_w, conv_b, yout, E, k, ngrp, nc,
                                                 ws, err);
    return cudaGetLastError();
}

cudaError_t swiglu_rows(const float *up, RowOut s, int M, int H, cudaStream_t st) {
    if ((int64_t)M * H == 0) return cudaSuccess;
    const bool vec = (H % 4 == 0);
    const int per = vec ? 4 : 1;
    dim3 grid((unsigned)((H / per + 127) / 128), (unsigned)std::min(M, 65535));
    if (vec) swiglu_k<4><<<grid, 128, 0, st>>>(up, s, M, H);
    else swiglu_k<1><<<grid, 128, 0, st>>>(up, s, M, H);
    return cudaGetLastError();
}

cudaError_t argmax_partials(const float *val, const uint32_t *idx, int n_tiles, int M, uint32_t *out,
                            cudaStream_t st) {
    if (M == 0) return cudaSuccess;
    return pdl_launch(argmax_partials_k, dim3(M), dim3(256), 0, st, val, idx, n_tiles, M, out);
}

cudaError_t softmax_ce_rows(const float *logits, int rows, int V, int r0, int tcc, int T, int t0,
                            const uint32_t *targets, double *nll, uint32_t *counted, int *err, cudaStream_t st) {
    if (rows == 0) return cudaSuccess;
    softmax_ce_rows_k<<<rows, 256, 0, st>>>(logits, V, r0, tcc, T, t0, targets, nll, counted, err);
    return cudaGetLastError();
}

cudaError_t ce_mean(const double *nll, const uint32_t *counted, size_t n, float *out, cudaStream_t st) {
    ce_mean_k<<<1, 1024, 0, st>>>(nll, counted, n, out);
    return cudaGetLastError();
}

cudaError_t argmax_rows(const float *x, uint32_t *out, int M, int V, cudaStream_t st) {
    if (M == 0) return cudaSuccess;
    argmax_rows_k<<<M, 256, 0, st>>>(x, out, V);
    return cudaGetLastError();
}

cudaError_t gather_last_rows(const float *x, const uint32_t *lens, int t0, int tc, float *last,
                             int S, int d, cudaStream_t st) {
    const int64_t n = (int64_t)S * d;
    if (n == 0) return cudaSuccess;
    gather_last_k<<<blocks_for(n, 256), 256, 0, st>>>(x, lens, t0, tc, last, S, d);
    return cudaGetLastError();
}

cudaError_t gather_rows(const float *src, const uint32_t *idx, float *dst, int n, int d,
                        cudaStream_t st) {
    const int64_t t = (int64_t)n * d;
    if (t == 0) return cudaSuccess;
    gather_rows_k<<<blocks_for(t, 256), 256, 0, st>>>(src, idx, dst, n, d);
    return cudaGetLastError();
}

cudaError_t scatter_rows(const float *src, const uint32_t *idx, float *dst, int n, int d,
                         cudaStream_t st) {
    const int64_t t = (int64_t)n * d;
    if (t == 0) return cudaSuccess;
    scatter_rows_k<<<blocks_for(t, 256), 256, 0, st>>>(src, idx, dst, n, d);
    return cudaGetLastError();
}

cudaError_t history_push(uint32_t *history, uint32_t *history_len, const uint32_t *tok, int S,
                         int window, cudaStream_t st) {
    if (S == 0 || window <= 0) return cudaSuccess;
    history_push_k<<<blocks_for(S, 128), 128, 0, st>>>(history, history_len, tok, S, window);
    return cudaGetLastError();
}

// *flag = 1 if any of x[0, n) is inf or NaN (checkpoint validation).
__global__ void any_nonfinite_k(const float *__restrict__ x, size_t n, int *flag) {
    bool bad = false;
    const size_t n4 = n / 4;
    const float4 *x4 = reinterpret_cast<const float4 *>(x);
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (size_t)gridDim.x * blockDim.x) {
        const float4 v = x4[i];
        bad |= !isfinite(v.x) || !isfinite(v.y) || !isfinite(v.z) || !isfinite(v.w);
    }
    for (size_t i = 4 * n4 + (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        bad |= !isfinite(x[i]);
    if (__syncthreads_or(bad) && threadIdx.x == 0) atomicExch(flag, 1);
}

cudaError_t any_nonfinite(const float *x, size_t n, int *flag, cudaStream_t st) {
    if (n == 0) return cudaSuccess;
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const size_t blocks = std::min<size_t>((n / 4 + 255) / 256 + 1, (size_t)sms * 8);
    any_nonfinite_k<<<(unsigned)blocks, 256, 0, st>>>(x, n, flag);
    return cudaGetLastError();
}

}  // namespace nk
