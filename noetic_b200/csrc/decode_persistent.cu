// decode_persistent.cu -- the whole decode step for 1..4 streams as ONE
// persistent kernel (Decoder::step, infer.rs:106-200, for every stream).
//
// With a handful of streams every projection is a matrix-vector product and
// the step is bound by reading the weights once (1.445 GB per token for the
// d=1024 / 24-layer / vocab-32768 model).  One CTA per SM runs the step:
//
//   producer warp   streams the weight rows this CTA owns, for every layer
//                   and phase, into a ring of shared-memory stages with
//                   cp.async.bulk (mbarrier completion, a few copies in
//                   flight).  Weights do not depend on activations, so the
//                   stream runs ahead across phases and layers, limited only
//                   by free stages, while the consumers wait at grid barriers.
//   15 consumer     per phase: fetch the residual stream x from L2, take
//   warps           the streamed rows, apply the epilogue, publish, meet at
//                   a grid barrier.  (16 warps in all: 128 registers each.)
//
// Every streamed row is d floats long.  A layer is two phases, each ending
// in one grid barrier (release-add, bounded acquire spin):
//
//   P1  RMSNorm(x) -> W_in rows (v_j, z_j, o_j) of the CTA's channels j; the
//       conv ring, SiLU, decay, h update and output gate give g_j locally
//       (infer.rs:143-176); then rows j of W_out^T (the out projection
//       stored transposed) scaled by g_j give the CTA's share of W_out . g
//       for all d outputs (infer.rs:178-182).
//   P2  RMSNorm(x) -> W_up rows (a_j, b_j) of the CTA's hidden channels;
//       s_j = SiLU(a_j) * b_j locally (infer.rs:185-190); then rows j of
//       W_down^T scaled by s_j give the CTA's share of W_down . s
//       (infer.rs:191-195).
//
// The shares meet in a 64-bit fixed-point accumulator (value * 2^32, integer
// atomic adds): integer addition is associative, so the sum is the same
// whatever order the CTAs arrive in and the step is deterministic.  The
// owner of each output element adds the residual and the bias once.  Three
// accumulators rotate: phase q reads buffer q % 3, adds into (q + 1) % 3 and
// clears its slice of (q + 2) % 3 (read one phase earlier, written one phase
// later).  The fixed-point form covers |x| < 2^31 at 2^-32 resolution; a
// non-finite activation is not representable (the multi-kernel engines
// carry NaN and infinity through as the reference does).
//
// After the last layer the tied logits over the CTA's vocabulary rows give a
// first-maximum partial per CTA, and the last CTA to finish reduces them to
// the greedy token (infer.rs:198-199, tensor.rs:354-365).
//
// The grid is one CTA per SM, launched cooperatively so every CTA is
// resident.  Every wait is bounded (~1 s of %globaltimer): an expired grid
// barrier sets the error flag and the CTA stops computing but keeps the copy
// pipeline consistent; an expired mbarrier wait stops the pipeline and the
// producer waits (bounded) for its copies in flight.  No multicast copy.

#include <algorithm>

#include "nk_common.cuh"
#include "nk_kernels.h"

#ifndef ACC_REPLICAS
#define ACC_REPLICAS 4
#endif

namespace nk {

namespace {

constexpr int CWARPS = 15;                   // consumer warps (16 warps in all: 128 registers each)
constexpr int CTHREADS = CWARPS * 32;        // consumer threads (named barrier 1)
constexpr int PTHREADS = CTHREADS + 32;      // + one producer warp
constexpr int STAGE_BYTES = 48 * 1024;      // 12 rows of 1024 floats
constexpr int SMEM_LIMIT = 227 * 1024;
constexpr uint64_t WAIT_NS = 1000000000ull;  // bound of every wait
constexpr int KCONV = 8;                     // largest conv width this kernel takes
constexpr int NPT = 5;                       // outputs per consumer thread: d <= NPT * CTHREADS
constexpr int MAXR = 4;                      // streams
constexpr int MAXD = 2048;                   // model width
constexpr double FX_ONE = 4294967296.0;      // fixed-point scale 2^32
constexpr int PACE_CHUNKS = 2;               // weight copies in flight per CTA
constexpr int NREP = ACC_REPLICAS;           // accumulator replicas (CTA c adds into replica c % NREP)

struct PersistParams {
    const uint32_t *tokens;
    uint32_t *tokens_out;
    const float *emb, *norm_f;
    float eps;
    float *state;
    uint32_t *heads;
    float *logits;
    float *best_val;
    uint32_t *best_idx;
    int *err;
    long long *acc;                // [3][MAXR][d] residual stream, fixed point
    uint32_t *sync;                // [0] grid-barrier arrivals, [1] logits CTAs done
    const PersistLayer *layers;    // device array [n_layer]
    int M, d, E, H, k, V, n_layer;
    int nstage;                    // ring stages
    int res_cap, gval_cap;         // floats of per-row results, of local g / s values
    int ob_cap, unit_cap, ops_cap; // operand block: owner bias, per-unit and whole-block floats
    uint64_t barrier_wait_ns;      // bound of the grid-barrier wait
    int withhold_arrival;          // test control: CTA 0 skips its first grid-barrier arrival
};

__device__ __forceinline__ uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ uint64_t gtimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// try_wait suspends the thread until the phase completes or the time hint
// (ns) runs out, so a waiting warp does not spin on the issue slots.
__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3; selp.u32 %0, 1, 0, p; }"
        : "=r"(done) : "r"(bar), "r"(parity), "r"(20000u) : "memory");
    return done != 0;
}

__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity) {
    if (mbar_try(bar, parity)) return true;
    const uint64_t t0 = gtimer();
    while (!mbar_try(bar, parity))
        if (gtimer() - t0 > WAIT_NS) return false;
    return true;
}

__device__ __forceinline__ void cp_async4(float *dst, const float *src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async16(float *dst, const float *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

__device__ __forceinline__ void consumer_sync() { asm volatile("bar.sync 1, %0;" ::"n"(CTHREADS) : "memory"); }

__device__ __forceinline__ unsigned long long to_fx(float v) {
    return (unsigned long long)__double2ll_rn((double)v * FX_ONE);
}
__device__ __forceinline__ float from_fx(long long v) { return (float)((double)v * (1.0 / FX_ONE)); }

// Fire-and-forget reduction (no value returned to the thread).
__device__ __forceinline__ void fx_add(long long *dst, float v) {
    asm volatile("red.relaxed.gpu.global.add.u64 [%0], %1;" ::"l"(dst), "l"(to_fx(v)) : "memory");
}

// The weight rows of one phase owned by this CTA: `nreg` regions of n
// contiguous d-float rows; in a layer phase the last region is the
// transposed projection (scaled rows, summed), the others are dot products.
struct Phase {
    const float *src[4];
    int nreg, n, u0;
};

// kind: 0 = P1, 1 = P2, 2 = logits.  Units (channels, hidden channels,
// vocabulary rows) are split evenly over the CTAs.
__device__ __forceinline__ Phase make_phase(const PersistParams &p, const PersistLayer *L, int kind) {
    const int G = gridDim.x, c = blockIdx.x;
    const int U = kind == 0 ? p.E : kind == 1 ? p.H : p.V;
    const int u0 = (int)((int64_t)U * c / G), u1 = (int)((int64_t)U * (c + 1) / G);
    const size_t d = (size_t)p.d;
    Phase ph;
    ph.n = u1 - u0;
    ph.u0 = u0;
    if (kind == 0) {
        ph.nreg = 4;
        ph.src[0] = L->in_w + (size_t)u0 * d;
        ph.src[1] = L->in_w + (size_t)(p.E + u0) * d;
        ph.src[2] = L->in_w + (size_t)(2 * p.E + u0) * d;
        ph.src[3] = L->out_wT + (size_t)u0 * d;
    } else if (kind == 1) {
        ph.nreg = 3;
        ph.src[0] = L->up_w + (size_t)u0 * d;
        ph.src[1] = L->up_w + (size_t)(p.H + u0) * d;
        ph.src[2] = L->down_wT + (size_t)u0 * d;
        ph.src[3] = nullptr;
    } else {
        ph.nreg = 1;
        ph.src[0] = p.emb + (size_t)u0 * d;
        ph.src[1] = ph.src[2] = ph.src[3] = nullptr;
    }
    return ph;
}

// Walks the chunks (up to R rows of one region) of every phase in stream
// order, skipping phases in which the CTA owns no rows.
struct Cursor {
    int q, rg, r0;
    Phase ph;
};

__device__ __forceinline__ void cursor_load(const PersistParams &p, const PersistLayer *layers, int n_phases, Cursor &c) {
    for (; c.q < n_phases; ++c.q) {
        const int kind = c.q == n_phases - 1 ? 2 : (c.q & 1);
        c.ph = make_phase(p, kind < 2 ? &layers[c.q >> 1] : nullptr, kind);
        c.rg = 0;
        c.r0 = 0;
        if (c.ph.n > 0) return;
    }
}

__device__ __forceinline__ void cursor_next(const PersistParams &p, const PersistLayer *layers, int n_phases, int R,
                                            Cursor &c) {
    c.r0 += R;
    if (c.r0 < c.ph.n) return;
    c.r0 = 0;
    if (++c.rg < c.ph.nreg) return;
    ++c.q;
    cursor_load(p, layers, n_phases, c);
}

// acc[r] = w . act[r] over d (act rows d floats apart), warp-wide: every
// lane gets the sums.
// Each lane keeps one partial sum per float4 component (four independent
// multiply-add chains instead of one), added as (x + y) + (z + w) at the end.
template <int MR>
__device__ __forceinline__ void dot_row(const float *w, const float *act, int d, float (&acc)[MR]) {
    const int lane = threadIdx.x & 31;
    float4 part[MR];
#pragma unroll
    for (int r = 0; r < MR; ++r) part[r] = make_float4(0.f, 0.f, 0.f, 0.f);
    const int d4 = d >> 2;
#pragma unroll 4
    for (int k4 = lane; k4 < d4; k4 += 32) {
        const float4 wv = *reinterpret_cast<const float4 *>(w + 4 * k4);
#pragma unroll
        for (int r = 0; r < MR; ++r) {
            const float4 a = *reinterpret_cast<const float4 *>(act + r * d + 4 * k4);
            part[r].x = fmaf(wv.x, a.x, part[r].x);
            part[r].y = fmaf(wv.y, a.y, part[r].y);
            part[r].z = fmaf(wv.z, a.z, part[r].z);
            part[r].w = fmaf(wv.w, a.w, part[r].w);
        }
    }
#pragma unroll
    for (int r = 0; r < MR; ++r) acc[r] = warp_sum((part[r].x + part[r].y) + (part[r].z + part[r].w));
}

// The same sum with act held in registers: a[r * (AREGS / MR) + i] is
// act[r][4 (lane + 32 i) ..], for d / 4 <= 32 * AREGS / MR.  The products
// are added in the same order as dot_row, so both give identical sums.
constexpr int AREGS = 8;  // float4 registers per lane for act

template <int MR>
__device__ __forceinline__ void dot_row_reg(const float *w, const float4 (&a)[AREGS], int d4, float (&acc)[MR]) {
    constexpr int A = AREGS / MR;
    const int lane = threadIdx.x & 31;
    float4 wv[A];
#pragma unroll
    for (int i = 0; i < A; ++i) {
        const int k4 = lane + 32 * i;
        wv[i] = k4 < d4 ? *reinterpret_cast<const float4 *>(w + 4 * k4) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int r = 0; r < MR; ++r) {
        float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int i = 0; i < A; ++i) {
            const float4 x = a[r * A + i];
            s.x = fmaf(wv[i].x, x.x, s.x);
            s.y = fmaf(wv[i].y, x.y, s.y);
            s.z = fmaf(wv[i].z, x.z, s.z);
            s.w = fmaf(wv[i].w, x.w, s.w);
        }
        acc[r] = (s.x + s.y) + (s.z + s.w);
    }
#pragma unroll
    for (int r = 0; r < MR; ++r) acc[r] = warp_sum(acc[r]);
}

template <int MR>
__global__ void __launch_bounds__(PTHREADS, 1) decode_step_persistent_k(const __grid_constant__ PersistParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int NS = p.nstage, d = p.d;
    uint8_t *ring = smem;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + (size_t)NS * STAGE_BYTES);  // full[NS], empty[NS]
    float *act = reinterpret_cast<float *>(bars + 2 * NS);  // [MR][d] normalised input
    float *res = act + MR * d;                              // [res_cap] dot products
    float *gval = res + p.res_cap;                          // [gval_cap] local g or s
    PersistLayer *layers = reinterpret_cast<PersistLayer *>(gval + p.gval_cap);  // [n_layer]
    // Operand blocks of two consecutive phases (buffer q & 1): gain [d],
    // owner bias [ob_cap], per-unit operands [unit_cap], per-(unit, stream)
    // state operands.
    float *opsb = reinterpret_cast<float *>(layers + p.n_layer);
    __shared__ float red[MR][CWARPS];
    __shared__ float wbest[CWARPS][MR];
    __shared__ uint32_t widx[CWARPS][MR];
    __shared__ uint32_t s_tok[MR], s_head[MR];
    __shared__ int s_abort, s_dead, s_last;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int M = p.M, G = gridDim.x;
    const uint32_t full0 = smem_u32(&bars[0]), empty0 = smem_u32(&bars[NS]);
    const size_t accsz = (size_t)MAXR * d;
    const int R = STAGE_BYTES / (d * 4);  // rows per stage
    const int n_phases = 2 * p.n_layer + 1;

    if (tid == 0) {
        s_abort = 0;
        s_dead = 0;
        s_last = 0;
        for (int s = 0; s < NS; ++s) {
            asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(full0 + 8 * s), "r"(1) : "memory");
            asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(empty0 + 8 * s), "r"(CWARPS) : "memory");
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    {
        const uint64_t *src = reinterpret_cast<const uint64_t *>(p.layers);
        uint64_t *dst = reinterpret_cast<uint64_t *>(layers);
        const int words = p.n_layer * (int)(sizeof(PersistLayer) / 8);
        for (int i = tid; i < words; i += PTHREADS) dst[i] = src[i];
    }
    if (tid < MR) {
        uint32_t t = 0, h = 0;
        if (tid < M) {
            t = p.tokens[tid];
            if (t >= (uint32_t)p.V) {
                atomicExch(p.err, 1);
                t = 0;
            }
            h = (p.heads[tid] + 1u) % (uint32_t)p.k;
        }
        s_tok[tid] = t;
        s_head[tid] = h;
    }
    __syncthreads();

    if (warp == CWARPS) {
        // ---------------- producer: every phase's regions, in order
        if (lane == 0) {
            int stage = 0, issued = 0;
            uint32_t parity = 0;
            const uint32_t row_bytes = (uint32_t)d * 4u;
            // Paced: at most PACE_CHUNKS copies in flight.  That is enough to
            // keep HBM busy (bandwidth x unloaded latency over the SMs),
            // while a deeper queue of weight requests would sit in front of
            // the latency-bound synchronisation traffic (accumulator atomics,
            // barrier, input loads) in the memory system.  Filled stages
            // wait in the ring until the consumers take them.
            Cursor ld{0, 0, 0, {}};
            cursor_load(p, layers, n_phases, ld);
            while (ld.q < n_phases) {
                if (!mbar_wait_bounded(empty0 + 8 * stage, parity ^ 1u)) {
                    atomicExch(p.err, 111);
                    *(volatile int *)&s_dead = 1;
                }
                if (issued >= PACE_CHUNKS) {
                    const int j = issued - PACE_CHUNKS;
                    if (!mbar_wait_bounded(full0 + 8 * (j % NS), (uint32_t)(j / NS) & 1u)) {
                        atomicExch(p.err, 111);
                        *(volatile int *)&s_dead = 1;
                    }
                }
                if (*(volatile int *)&s_dead) break;
                const uint32_t bytes = (uint32_t)min(R, ld.ph.n - ld.r0) * row_bytes;
                const uint32_t fb = full0 + 8 * stage;
                asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(fb), "r"(bytes) : "memory");
                asm volatile(
                    "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                    ::"r"(smem_u32(ring + (size_t)stage * STAGE_BYTES)),
                    "l"((uint64_t)(ld.ph.src[ld.rg] + (size_t)ld.r0 * d)), "r"(bytes), "r"(fb)
                    : "memory");
                ++issued;
                if (++stage == NS) {
                    stage = 0;
                    parity ^= 1u;
                }
                cursor_next(p, layers, n_phases, R, ld);
            }
            // After a stopped pipeline, wait (bounded) for the copies that may
            // still be in flight -- the last NS issued -- so that none lands
            // after the CTA exits.
            if (*(volatile int *)&s_dead) {
                int st2 = 0;
                uint32_t ph2 = 0;
                for (int i = 0; i < issued; ++i) {
                    if (i >= issued - NS) mbar_wait_bounded(full0 + 8 * st2, ph2);
                    if (++st2 == NS) {
                        st2 = 0;
                        ph2 ^= 1u;
                    }
                }
            }
        }
    } else {
        // ---------------- consumers
        int stage = 0;
        uint32_t parity = 0;
        uint32_t barrier_target = 0;
        // The output elements [dN0, dN1) whose residual and bias this CTA adds.
        const int dN0 = (int)((int64_t)d * blockIdx.x / G), dN1 = (int)((int64_t)d * (blockIdx.x + 1) / G);
        float wb[MR];
        uint32_t wi[MR];
#pragma unroll
        for (int r = 0; r < MR; ++r) {
            wb[r] = -INFINITY;
            wi[r] = 0xFFFFFFFFu;
        }
        auto chunk_wait = [&]() {
            if (!*(volatile int *)&s_dead && !mbar_wait_bounded(full0 + 8 * stage, parity)) {
                if (lane == 0) atomicExch(p.err, 112);
                *(volatile int *)&s_dead = 1;
            }
        };
        auto chunk_release = [&]() {
            __syncwarp();
            if (lane == 0)
                asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(empty0 + 8 * stage) : "memory");
            if (++stage == NS) {
                stage = 0;
                parity ^= 1u;
            }
        };
        auto live = [&]() { return !*(volatile int *)&s_dead && !*(volatile int *)&s_abort; };

        // The small operands of phase q2 (norm gain, the owner's bias slice,
        // biases / conv taps of the CTA's units, the conv ring and h of its
        // channels) are copied into operand block q2 & 1 a phase ahead of
        // use: the weight stream evicts them from L2 every step, and an HBM
        // round trip at the start of a phase would sit on the critical path.
        // Each thread waits for its copies before the CTA barrier that ends
        // the phase before q2.
        const int kk = p.k, E = p.E, H = p.H;
        auto issue_ops = [&](int q2) {
            if (q2 < n_phases) {
                const int kind2 = q2 == n_phases - 1 ? 2 : (q2 & 1);
                const PersistLayer *L2 = kind2 < 2 ? &layers[q2 >> 1] : nullptr;
                const Phase ph2 = make_phase(p, L2, kind2);
                float *b = opsb + (size_t)(q2 & 1) * p.ops_cap;
                const float *gain = kind2 == 0 ? L2->n1 : kind2 == 1 ? L2->n2 : p.norm_f;
                for (int t = tid; t < (d >> 2); t += CTHREADS) cp_async16(b + 4 * t, gain + 4 * t);
                if (kind2 < 2) {
                    const float *bias = kind2 == 0 ? L2->out_b : L2->down_b;
                    for (int t = tid; t < dN1 - dN0; t += CTHREADS) cp_async4(b + d + t, bias + dN0 + t);
                    float *bu = b + d + p.ob_cap;
                    const int u0 = ph2.u0;
                    if (kind2 == 0) {
                        const int per = 4 + kk;
                        for (int t = tid; t < ph2.n * per; t += CTHREADS) {
                            const int i = t / per, f = t - i * per, u = u0 + i;
                            const float *src = f < 3 ? L2->in_b + (size_t)f * E + u
                                               : f == 3 ? L2->conv_b + u
                                                        : L2->conv_w + (size_t)(f - 4) * E + u;
                            cp_async4(bu + i * (4 + KCONV) + f, src);
                        }
                        float *bs = bu + p.unit_cap;
                        const float *st = p.state + (size_t)(q2 >> 1) * M * (kk + 1) * E;
                        for (int t = tid; t < ph2.n * M * kk; t += CTHREADS) {
                            const int i = t / (M * kk), rem = t - i * (M * kk), r = rem / kk, qq = rem - r * kk;
                            // qq == 0: h; qq >= 1: the ring value qq steps back.
                            const uint32_t slot =
                                qq == 0 ? (uint32_t)kk : (s_head[r] + (uint32_t)kk - (uint32_t)qq) % (uint32_t)kk;
                            cp_async4(bs + (i * MR + r) * KCONV + qq,
                                      st + (size_t)r * (kk + 1) * E + (size_t)slot * E + u0 + i);
                        }
                    } else {
                        for (int t = tid; t < ph2.n * 2; t += CTHREADS) {
                            const int i = t >> 1, f = t & 1;
                            cp_async4(bu + 2 * i + f, L2->up_b + (size_t)f * H + u0 + i);
                        }
                    }
                }
            }
            cp_async_commit();
        };
        issue_ops(0);
        cp_async_wait_all();
        consumer_sync();

        for (int q = 0; q < n_phases; ++q) {
            const int kind = q == n_phases - 1 ? 2 : (q & 1);
            const int layer = q >> 1;
            const PersistLayer *L = kind < 2 ? &layers[layer] : nullptr;
            const Phase ph = make_phase(p, L, kind);
            const long long *acc_in = p.acc + (size_t)(q % 3) * NREP * accsz;
            long long *acc_out = p.acc + ((size_t)((q + 1) % 3) * NREP + blockIdx.x % NREP) * accsz;
            long long *acc_clear = p.acc + (size_t)((q + 2) % 3) * NREP * accsz;
            float *state = kind == 0 ? p.state + (size_t)layer * M * (kk + 1) * E : nullptr;
            const float *ops = opsb + (size_t)(q & 1) * p.ops_cap;
            issue_ops(q + 1);
            // thread t < n * MR owns the epilogue of unit i = t / MR, stream r = t % MR
            const int ei = tid / MR, er = tid % MR, ej = ph.u0 + ei;
            const bool mine = kind < 2 && tid < ph.n * MR && er < M;

            // ---- input x of every stream: the embedding rows in the first
            // phase, else the accumulator.  The CTA adds x + bias of its
            // output elements into the next accumulator and clears its slice
            // of the one two phases ahead.  act = x * gain; the RMSNorm scale
            // rs (tensor.rs:298-312) multiplies the dot products instead:
            // W . (x rs gain) = rs (W . (x gain)).
            float rs[MR];
            {
                const int d4 = d >> 2;
                const float *obias = kind < 2 ? ops + d : nullptr;  // [n - dN0]
                const float *gain = ops;
                constexpr int IPT = (MR * MAXD / 4 + CTHREADS - 1) / CTHREADS;  // items per thread
                float4 xv[IPT], gg[IPT];
#pragma unroll
                for (int i = 0; i < IPT; ++i) {
                    const int t = tid + i * CTHREADS;
                    xv[i] = gg[i] = make_float4(0.f, 0.f, 0.f, 0.f);
                    if (t < MR * d4) {
                        const int r = t / d4, c4 = t - r * d4;
                        gg[i] = *reinterpret_cast<const float4 *>(gain + 4 * c4);
                        if (r < M) {
                            if (q == 0) {
                                xv[i] = __ldg(reinterpret_cast<const float4 *>(p.emb + (size_t)s_tok[r] * d + 4 * c4));
                            } else {
                                const long long *src = acc_in + (size_t)r * d + 4 * c4;
                                longlong2 a0 = __ldcg(reinterpret_cast<const longlong2 *>(src));
                                longlong2 a1 = __ldcg(reinterpret_cast<const longlong2 *>(src + 2));
#pragma unroll
                                for (int rp = 1; rp < NREP; ++rp) {
                                    const longlong2 b0 = __ldcg(reinterpret_cast<const longlong2 *>(src + rp * accsz));
                                    const longlong2 b1 =
                                        __ldcg(reinterpret_cast<const longlong2 *>(src + rp * accsz + 2));
                                    a0.x += b0.x;
                                    a0.y += b0.y;
                                    a1.x += b1.x;
                                    a1.y += b1.y;
                                }
                                xv[i] = make_float4(from_fx(a0.x), from_fx(a0.y), from_fx(a1.x), from_fx(a1.y));
                            }
                        }
                    }
                }
                float ss[MR];
#pragma unroll
                for (int r = 0; r < MR; ++r) ss[r] = 0.0f;
#pragma unroll
                for (int i = 0; i < IPT; ++i) {
                    const int t = tid + i * CTHREADS;
                    if (t < MR * d4) {
                        const int r = t / d4, c4 = t - r * d4;
                        const float4 v = xv[i];
                        if (obias && r < M && 4 * c4 + 3 >= dN0 && 4 * c4 < dN1) {
                            const float vv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                            for (int e = 0; e < 4; ++e) {
                                const int n = 4 * c4 + e;
                                if (n >= dN0 && n < dN1) {
                                    fx_add(acc_out + (size_t)r * d + n, vv[e] + obias[n - dN0]);
#pragma unroll
                                    for (int rp = 0; rp < NREP; ++rp) acc_clear[rp * accsz + (size_t)r * d + n] = 0;
                                }
                            }
                        }
                        *reinterpret_cast<float4 *>(act + r * d + 4 * c4) =
                            make_float4(v.x * gg[i].x, v.y * gg[i].y, v.z * gg[i].z, v.w * gg[i].w);
                        float sq = v.x * v.x;
                        sq = fmaf(v.y, v.y, sq);
                        sq = fmaf(v.z, v.z, sq);
                        sq = fmaf(v.w, v.w, sq);
#pragma unroll
                        for (int rr = 0; rr < MR; ++rr)
                            if (rr == r) ss[rr] += sq;
                    }
                }
#pragma unroll
                for (int r = 0; r < MR; ++r) {
                    const float sum = warp_sum(ss[r]);
                    if (lane == 0) red[r][warp] = sum;
                }
                if (kind == 2 && blockIdx.x == 0 && tid < M) p.heads[tid] = s_head[tid];
                consumer_sync();
#pragma unroll
                for (int r = 0; r < MR; ++r) {
                    float tot = 0.0f;
#pragma unroll
                    for (int w = 0; w < CWARPS; ++w) tot += red[r][w];
                    rs[r] = r < M ? 1.0f / sqrtf(tot / (float)d + p.eps) : 0.0f;
                }
            }

            // ---- dot-product regions: one warp per row, round-robin; act in
            // registers when it fits (half the shared-memory reads per row)
            const int ndot = kind == 0 ? 3 : kind == 1 ? 2 : 1;
            const int d4 = d >> 2;
            const bool areg = d4 <= 32 * (AREGS / MR);
            float4 a[AREGS];
#pragma unroll
            for (int i = 0; i < AREGS; ++i) {
                const int r = i / (AREGS / MR), k4 = lane + 32 * (i % (AREGS / MR));
                a[i] = areg && k4 < d4 ? *reinterpret_cast<const float4 *>(act + r * d + 4 * k4)
                                       : make_float4(0.f, 0.f, 0.f, 0.f);
            }
            int row = 0;
            for (int rg = 0; rg < ndot; ++rg) {
                for (int r0 = 0; r0 < ph.n; r0 += R) {
                    const int rows = min(R, ph.n - r0);
                    chunk_wait();
                    const bool go = live();
                    const float *chunk = reinterpret_cast<const float *>(ring + (size_t)stage * STAGE_BYTES);
                    for (int j = (warp - row % CWARPS + CWARPS) % CWARPS; go && j < rows; j += CWARPS) {
                        float acc[MR];
                        if (areg)
                            dot_row_reg<MR>(chunk + (size_t)j * d, a, d4, acc);
                        else
                            dot_row<MR>(chunk + (size_t)j * d, act, d, acc);
#pragma unroll
                        for (int r = 0; r < MR; ++r) acc[r] *= rs[r];
                        const int i = r0 + j;
                        if (kind < 2) {
                            if (lane < MR) {
                                float v = acc[0];
#pragma unroll
                                for (int r = 1; r < MR; ++r)
                                    if (lane == r) v = acc[r];
                                res[(rg * ph.n + i) * MR + lane] = v;
                            }
                        } else {
                            const int u = ph.u0 + i;
#pragma unroll
                            for (int r = 0; r < MR; ++r) {
                                if (r >= M) continue;
                                if (p.logits && lane == r) p.logits[(size_t)r * p.V + u] = acc[r];
                                if (!isnan(acc[r]) && acc[r] > wb[r]) {
                                    wb[r] = acc[r];
                                    wi[r] = (uint32_t)u;
                                }
                            }
                        }
                    }
                    chunk_release();
                    row += rows;
                }
            }
            if (kind == 2) break;

            // ---- local epilogue: g_j (conv ring, recurrence, gate) or s_j
            consumer_sync();
            if (live() && tid < ph.n * MR) {
                float gv = 0.0f;
                const float *bu = ops + d + p.ob_cap;
                if (mine && kind == 0) {
                    const float *uo = bu + ei * (4 + KCONV);                      // in_b x3, conv_b, taps
                    const float *so = bu + p.unit_cap + (ei * MR + er) * KCONV;  // h, ring values
                    const float v = res[(0 * ph.n + ei) * MR + er] + uo[0];
                    const float zz = res[(1 * ph.n + ei) * MR + er] + uo[1];
                    const float oo = res[(2 * ph.n + ei) * MR + er] + uo[2];
                    float *ring_s = state + (size_t)er * (kk + 1) * E;
                    ring_s[(size_t)s_head[er] * E + ej] = v;
                    float sum = uo[3];
#pragma unroll
                    for (int qq = 0; qq < KCONV; ++qq)
                        if (qq < kk) sum = sum + uo[4 + qq] * (qq == 0 ? v : so[qq]);
                    const float value = silu(sum);
                    const float decay = sigmoid(zz);
                    const float h = decay * so[0] + (1.0f - decay) * value;
                    ring_s[(size_t)kk * E + ej] = h;
                    gv = h * silu(oo);
                } else if (mine) {
                    const float a = res[(0 * ph.n + ei) * MR + er];
                    const float b = res[(1 * ph.n + ei) * MR + er];
                    gv = silu(a + bu[2 * ei]) * (b + bu[2 * ei + 1]);
                }
                gval[ei * MR + er] = gv;  // zero for streams >= M
            }
            consumer_sync();

            // ---- the transposed projection: the CTA's share of W . g over
            // every output (rows scaled by the local values), then one
            // fixed-point add per output and stream.
            {
                float part[MR][NPT];
#pragma unroll
                for (int r = 0; r < MR; ++r)
#pragma unroll
                    for (int i = 0; i < NPT; ++i) part[r][i] = 0.0f;
                for (int r0 = 0; r0 < ph.n; r0 += R) {
                    const int rows = min(R, ph.n - r0);
                    chunk_wait();
                    const bool go = live();
                    const float *chunk = reinterpret_cast<const float *>(ring + (size_t)stage * STAGE_BYTES);
                    for (int j = 0; go && j < rows; ++j) {
                        float gj[MR];
#pragma unroll
                        for (int r = 0; r < MR; ++r) gj[r] = gval[(r0 + j) * MR + r];
                        const float *w = chunk + (size_t)j * d;
#pragma unroll
                        for (int i = 0; i < NPT; ++i) {
                            const int n = tid + i * CTHREADS;
                            if (n < d) {
                                const float wv = w[n];
#pragma unroll
                                for (int r = 0; r < MR; ++r) part[r][i] = fmaf(wv, gj[r], part[r][i]);
                            }
                        }
                    }
                    chunk_release();
                }
                if (live() && ph.n > 0) {
#pragma unroll
                    for (int i = 0; i < NPT; ++i) {
                        const int n = tid + i * CTHREADS;
#pragma unroll
                        for (int r = 0; r < MR; ++r)
                            if (n < d && r < M) fx_add(acc_out + (size_t)r * d + n, part[r][i]);
                    }
                }
            }

            // ---- grid barrier: every CTA's share of this phase is in the
            // accumulator after it
            barrier_target += (uint32_t)G;
            cp_async_wait_all();  // the next phase's operand block
            consumer_sync();
            if (tid == 0) {
                // The CTA barrier above orders the consumers' writes before
                // this release; the acquire orders the other CTAs' writes
                // before the CTA barrier below.
                if (!(p.withhold_arrival && blockIdx.x == 0 && barrier_target == (uint32_t)G))
                    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p.sync), "r"(1u) : "memory");
                if (!*(volatile int *)&s_abort) {
                    const uint64_t t0 = gtimer();
                    for (;;) {
                        uint32_t v;
                        asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p.sync) : "memory");
                        if (v >= barrier_target) break;
                        if (gtimer() - t0 > p.barrier_wait_ns) {
                            atomicExch(p.err, 113);
                            *(volatile int *)&s_abort = 1;
                            break;
                        }
                    }
                }
            }
            consumer_sync();
        }

        // ---- first maximum of the CTA's vocabulary rows; the last CTA to
        // finish reduces every CTA's partial (earlier CTAs own earlier rows)
        // and returns the accumulators and barrier words to zero for the
        // next launch (every other CTA has read its last accumulator).
        if (p.tokens_out) {
            if (lane == 0) {
#pragma unroll
                for (int r = 0; r < MR; ++r) {
                    wbest[warp][r] = wb[r];
                    widx[warp][r] = wi[r];
                }
            }
            consumer_sync();
            if (tid < M) {
                float b = -INFINITY;
                uint32_t bi = 0xFFFFFFFFu;
                for (int w = 0; w < CWARPS; ++w) {
                    const float v = wbest[w][tid];
                    const uint32_t ix = widx[w][tid];
                    if (v > b || (v == b && ix < bi)) {
                        b = v;
                        bi = ix;
                    }
                }
                p.best_val[(size_t)tid * G + blockIdx.x] = b;
                p.best_idx[(size_t)tid * G + blockIdx.x] = bi;
            }
        }
        consumer_sync();
        if (tid == 0) {
            __threadfence();
            const uint32_t done = atomicAdd(p.sync + 1, 1u);
            s_last = done == (uint32_t)G - 1;
            __threadfence();
        }
        consumer_sync();
        if (s_last) {
            if (p.tokens_out && tid < M) {
                float b = -INFINITY;
                uint32_t bi = 0xFFFFFFFFu;
                for (int c = 0; c < G; ++c) {
                    const float v = __ldcg(p.best_val + (size_t)tid * G + c);
                    const uint32_t ix = __ldcg(p.best_idx + (size_t)tid * G + c);
                    if (v > b || (v == b && ix < bi)) {
                        b = v;
                        bi = ix;
                    }
                }
                p.tokens_out[tid] = (b == -INFINITY || bi == 0xFFFFFFFFu) ? 0u : bi;
            }
            for (int b = 0; b < 3 * NREP; ++b)
                for (int t = tid; t < (M * d) / 2; t += CTHREADS)
                    __stcg(reinterpret_cast<longlong2 *>(p.acc + (size_t)b * accsz) + t, make_longlong2(0, 0));
            if (tid == 0) {
                p.sync[0] = 0u;
                p.sync[1] = 0u;
            }
        }
    }
    __syncthreads();
}

int sm_count() {
    static int n = 0;
    if (!n) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        if (n <= 0) n = 1;
    }
    return n;
}

// Shared-memory plan from the largest per-CTA unit counts of the two layer
// phases.  Every region is a multiple of 4 floats, so each stays 16-byte
// aligned.
struct Plan {
    int res_cap, gval_cap, ob_cap, unit_cap, ops_cap, nstage;
    size_t smem;
};

constexpr int round4(int v) { return (v + 3) & ~3; }

// Ring, mbarriers, act, res, gval, layer table, two operand blocks.
size_t plan_bytes(const Plan &pl, int mr, int d, int n_layer, int nstage) {
    return (size_t)nstage * STAGE_BYTES + 16 * (size_t)nstage +
           4 * ((size_t)mr * d + pl.res_cap + pl.gval_cap + 2 * (size_t)pl.ops_cap) +
           (size_t)n_layer * sizeof(PersistLayer);
}

Plan make_plan(int mr, int d, int E, int H, int n_layer, int G) {
    const int ce = (E + G - 1) / G, ch = (H + G - 1) / G;
    Plan pl{};
    pl.res_cap = round4(std::max(3 * ce, 2 * ch) * mr);
    pl.gval_cap = round4(std::max(ce, ch) * mr);
    pl.ob_cap = round4((d + G - 1) / G);
    pl.unit_cap = round4(std::max(ce * (4 + KCONV), 2 * ch));
    pl.ops_cap = d + pl.ob_cap + pl.unit_cap + round4(ce * mr * KCONV);
    pl.nstage = 12;
    while (pl.nstage > 2 && plan_bytes(pl, mr, d, n_layer, pl.nstage) + 2048 > (size_t)SMEM_LIMIT) --pl.nstage;
    pl.smem = plan_bytes(pl, mr, d, n_layer, pl.nstage);
    return pl;
}

template <int MR>
cudaError_t launch_mr(const PersistStepArgs &a, cudaStream_t st) {
    const int G = sm_count();
    PersistParams p{};
    p.tokens = a.tokens;
    p.tokens_out = a.tokens_out;
    p.emb = a.emb;
    p.norm_f = a.norm_f;
    p.eps = a.eps;
    p.state = a.state;
    p.heads = a.heads;
    p.logits = a.logits;
    p.best_val = a.best_val;
    p.best_idx = a.best_idx;
    p.err = a.err;
    p.acc = reinterpret_cast<long long *>(a.ws);
    p.sync = reinterpret_cast<uint32_t *>(p.acc + (size_t)3 * NREP * MAXR * a.d);
    p.layers = a.layers;
    p.M = a.M;
    p.d = a.d;
    p.E = a.E;
    p.H = a.H;
    p.k = a.k;
    p.V = a.V;
    p.n_layer = a.n_layer;
    const Plan pl = make_plan(MR, a.d, a.E, a.H, a.n_layer, G);
    p.res_cap = pl.res_cap;
    p.gval_cap = pl.gval_cap;
    p.ob_cap = pl.ob_cap;
    p.unit_cap = pl.unit_cap;
    p.ops_cap = pl.ops_cap;
    p.nstage = pl.nstage;
    p.barrier_wait_ns = a.barrier_wait_ns ? a.barrier_wait_ns : WAIT_NS;
    p.withhold_arrival = a.withhold_arrival ? 1 : 0;
    const size_t smem = pl.smem;
    static size_t smem_set[MAXR + 1] = {};
    cudaError_t e;
    if (smem > smem_set[MR]) {
        e = cudaFuncSetAttribute(decode_step_persistent_k<MR>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        smem_set[MR] = smem;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)G);
    cfg.blockDim = dim3(PTHREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, decode_step_persistent_k<MR>, p);
}

// out[c][r] = in[r][c] for in [rows, cols] row-major, through 32 x 32 tiles.
__global__ void transpose_k(const float *__restrict__ in, float *__restrict__ out, int rows, int cols) {
    __shared__ float tile[32][33];
    const int c0 = blockIdx.x * 32, r0 = blockIdx.y * 32;
    for (int i = threadIdx.y; i < 32; i += blockDim.y) {
        const int r = r0 + i, c = c0 + threadIdx.x;
        if (r < rows && c < cols) tile[i][threadIdx.x] = in[(size_t)r * cols + c];
    }
    __syncthreads();
    for (int i = threadIdx.y; i < 32; i += blockDim.y) {
        const int c = c0 + i, r = r0 + threadIdx.x;
        if (r < rows && c < cols) out[(size_t)c * rows + r] = tile[threadIdx.x][i];
    }
}

}  // namespace

int persistent_partials() { return sm_count(); }

size_t persistent_ws_bytes(int d) { return (size_t)3 * NREP * MAXR * d * sizeof(long long) + 2 * sizeof(uint32_t); }

bool persistent_step_supported(int M, int d, int E, int H, int k, int V, int n_layer) {
    if (M < 1 || M > MAXR || n_layer < 1 || k < 1 || k > KCONV || V < 1 || E < 1 || H < 1) return false;
    if (d < 4 || d % 4 || d > MAXD) return false;
    if ((size_t)d * 4 > (size_t)STAGE_BYTES) return false;  // a row fits one stage
    const int G = sm_count();
    // One epilogue thread per (owned unit, stream).
    const int ce = (E + G - 1) / G, ch = (H + G - 1) / G;
    if (std::max(ce, ch) * MAXR > CTHREADS) return false;
    const Plan pl = make_plan(MAXR, d, E, H, n_layer, G);
    return plan_bytes(pl, MAXR, d, n_layer, 2) + 2048 <= (size_t)SMEM_LIMIT;
}

cudaError_t persistent_step(const PersistStepArgs &a, cudaStream_t st) {
    if (a.M <= 1) return launch_mr<1>(a, st);
    if (a.M <= 2) return launch_mr<2>(a, st);
    return launch_mr<4>(a, st);
}

cudaError_t transpose(const float *in, float *out, int rows, int cols, cudaStream_t st) {
    if ((int64_t)rows * cols == 0) return cudaSuccess;
    const dim3 grid((unsigned)((cols + 31) / 32), (unsigned)((rows + 31) / 32));
    transpose_k<<<grid, dim3(32, 8), 0, st>>>(in, out, rows, cols);
    return cudaGetLastError();
}

}  // namespace nk
