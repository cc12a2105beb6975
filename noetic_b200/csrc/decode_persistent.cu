// decode_persistent.cu -- the whole decode step for 1..4 streams as ONE
// persistent kernel (Decoder::step, infer.rs:106-200, for every stream).
//
// With a handful of streams every projection is a matrix-vector product and
// the step is bound by reading the weights once (1.445 GB per token for the
// d=1024 / 24-layer / vocab-32768 model).  Launching a kernel per projection
// leaves HBM idle at every kernel boundary (ramp-down, launch, ramp-up), which
// at ~100 launches per token costs more than half the step.  Here one CTA per
// SM runs the whole step:
//
//   producer warp   walks the fixed sequence of weight rows this CTA owns,
//                   for every layer and phase, and streams them into a ring
//                   of shared-memory stages with cp.async.bulk (global ->
//                   shared, mbarrier completion).  Weights do not depend on
//                   activations, so the stream runs ahead across phases and
//                   layers, limited only by free stages; HBM stays busy
//                   while the consumers wait at grid barriers.
//   16 consumer     per phase: read the phase's input vector (RMSNorm of x,
//   warps           g, or SwiGLU output) from L2 into shared memory, take
//                   the streamed rows round-robin (one warp per row, f32
//                   FMA dot products), apply the phase's epilogue, then a
//                   grid-wide barrier publishes the outputs.
//
// Phases per layer (rows owned by CTA c: an even split of the phase's units):
//   A  in_proj rows (v_j, z_j, o_j) of owned channels j; conv ring, SiLU,
//      decay, h update, output gate                 (infer.rs:143-176)
//   B  out_proj rows n: x[n] += W_out[n] . g + b    (infer.rs:178-182)
//   C  up_proj rows (a_j, b_j) of owned hidden channels: SiLU(a) * b
//                                                   (infer.rs:185-190)
//   D  down_proj rows n: x[n] += W_down[n] . s + b  (infer.rs:191-195)
// then the tied logits over owned vocabulary rows with a first-maximum
// partial per CTA, and the last CTA to finish reduces the partials to the
// greedy token (infer.rs:198-199, tensor.rs:354-365).
//
// The grid is one CTA per SM, launched cooperatively so every CTA is
// resident.  Every wait is bounded (~1 s of %globaltimer): an expired grid
// barrier sets the error flag and the CTA stops computing but keeps the
// copy pipeline consistent; an expired mbarrier wait stops the pipeline.
// No multicast copy is used.

#include <algorithm>

#include "nk_common.cuh"
#include "nk_kernels.h"

namespace nk {

namespace {

constexpr int CWARPS = 16;                   // consumer warps
constexpr int CTHREADS = CWARPS * 32;        // consumer threads (named barrier 1)
constexpr int PTHREADS = CTHREADS + 32;      // + one producer warp
constexpr int STAGE_BYTES = 24 * 1024;       // 6 rows of 1024 f32, 2 rows of 3072
constexpr int SMEM_LIMIT = 227 * 1024;
constexpr uint64_t WAIT_NS = 1000000000ull;  // bound of every wait
constexpr int KCONV = 8;                     // largest conv width this kernel takes

struct PersistParams {
    const uint32_t *tokens;
    uint32_t *tokens_out;
    const float *emb, *norm_f;
    float eps;
    float *x, *g, *state;
    uint32_t *heads;
    float *logits;
    float *best_val;
    uint32_t *best_idx;
    int *err;
    uint32_t *sync;  // [0] grid-barrier arrivals, [1] logits CTAs done; zero at launch
    const SmallLayer *layers;  // device array [n_layer]
    int M, d, E, H, k, V, n_layer;
    int nstage;   // ring stages
    int res_cap;  // floats of per-row results (phases A and C)
};

__device__ __forceinline__ uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ uint64_t gtimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
        : "=r"(done) : "r"(bar), "r"(parity) : "memory");
    return done != 0;
}

__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity) {
    if (mbar_try(bar, parity)) return true;
    const uint64_t t0 = gtimer();
    while (!mbar_try(bar, parity))
        if (gtimer() - t0 > WAIT_NS) return false;
    return true;
}

__device__ __forceinline__ void consumer_sync() { asm volatile("bar.sync 1, %0;" ::"n"(CTHREADS) : "memory"); }

__device__ __forceinline__ float4 ld_cg4(const float *p) { return __ldcg(reinterpret_cast<const float4 *>(p)); }

// One phase of the sequence: up to three regions of contiguous weight rows
// (each `n` rows of K floats) owned by this CTA, streamed in chunks of R rows.
struct Phase {
    const float *src[3];
    int nreg, n, K, R, u0;
};

// kind: 0 A (in_ssm), 1 B (out), 2 C (up), 3 D (down), 4 logits.
__device__ __forceinline__ Phase make_phase(const PersistParams &p, int layer, int kind) {
    const int G = gridDim.x, c = blockIdx.x;
    int U;
    switch (kind) {
        case 0: U = p.E; break;
        case 1: U = p.d; break;
        case 2: U = p.H; break;
        case 3: U = p.d; break;
        default: U = p.V; break;
    }
    const int u0 = (int)((int64_t)U * c / G), u1 = (int)((int64_t)U * (c + 1) / G);
    Phase ph;
    ph.n = u1 - u0;
    ph.u0 = u0;
    if (kind == 4) {
        ph.K = p.d;
        ph.nreg = 1;
        ph.src[0] = p.emb + (size_t)u0 * p.d;
    } else {
        const SmallLayer &L = p.layers[layer];
        switch (kind) {
            case 0:
                ph.K = p.d;
                ph.nreg = 3;
                ph.src[0] = L.in_w + (size_t)u0 * p.d;
                ph.src[1] = L.in_w + (size_t)(p.E + u0) * p.d;
                ph.src[2] = L.in_w + (size_t)(2 * p.E + u0) * p.d;
                break;
            case 1:
                ph.K = p.E;
                ph.nreg = 1;
                ph.src[0] = L.out_w + (size_t)u0 * p.E;
                break;
            case 2:
                ph.K = p.d;
                ph.nreg = 2;
                ph.src[0] = L.up_w + (size_t)u0 * p.d;
                ph.src[1] = L.up_w + (size_t)(p.H + u0) * p.d;
                break;
            default:
                ph.K = p.H;
                ph.nreg = 1;
                ph.src[0] = L.down_w + (size_t)u0 * p.H;
                break;
        }
    }
    ph.R = min(STAGE_BYTES / (ph.K * 4), 64);
    return ph;
}

// dst[r][:] = RMSNorm(src[r][:]) * gain for r < M (tensor.rs:298-312); the
// rows are read from L2 (other CTAs wrote them).  Rows r >= M are zero.
template <int MR>
__device__ __forceinline__ void norm_to_smem(const float *const (&src)[MR], const float *gain, float eps, int M, int d,
                                             float *dst, float (*red)[CWARPS]) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int d4 = d >> 2;
    float ss[MR];
#pragma unroll
    for (int r = 0; r < MR; ++r) ss[r] = 0.0f;
#pragma unroll
    for (int r = 0; r < MR; ++r) {
        for (int c = tid; c < d4; c += CTHREADS) {
            const float4 v = r < M ? ld_cg4(src[r] + 4 * c) : make_float4(0.f, 0.f, 0.f, 0.f);
            *reinterpret_cast<float4 *>(dst + r * d + 4 * c) = v;
            ss[r] = fmaf(v.x, v.x, ss[r]);
            ss[r] = fmaf(v.y, v.y, ss[r]);
            ss[r] = fmaf(v.z, v.z, ss[r]);
            ss[r] = fmaf(v.w, v.w, ss[r]);
        }
    }
#pragma unroll
    for (int r = 0; r < MR; ++r) {
        const float s = warp_sum(ss[r]);
        if (lane == 0) red[r][warp] = s;
    }
    consumer_sync();
#pragma unroll
    for (int r = 0; r < MR; ++r) {
        float tot = 0.0f;
#pragma unroll
        for (int w = 0; w < CWARPS; ++w) tot += red[r][w];
        const float rs = r < M ? 1.0f / sqrtf(tot / (float)d + eps) : 0.0f;
        for (int c = tid; c < d4; c += CTHREADS) {
            float4 v = *reinterpret_cast<float4 *>(dst + r * d + 4 * c);
            const float4 gg = *reinterpret_cast<const float4 *>(gain + 4 * c);
            v.x = v.x * rs * gg.x;
            v.y = v.y * rs * gg.y;
            v.z = v.z * rs * gg.z;
            v.w = v.w * rs * gg.w;
            *reinterpret_cast<float4 *>(dst + r * d + 4 * c) = v;
        }
    }
    consumer_sync();
}

template <int MR>
__device__ __forceinline__ void copy_to_smem(const float *src, int M, int K, float *dst) {
    const int K4 = K >> 2;
    for (int i = threadIdx.x; i < MR * K4; i += CTHREADS) {
        const int r = i / K4;
        const float4 v = r < M ? ld_cg4(src + (size_t)r * K + 4 * (i - r * K4)) : make_float4(0.f, 0.f, 0.f, 0.f);
        *reinterpret_cast<float4 *>(dst + 4 * i) = v;
    }
    consumer_sync();
}

// acc[r] = w . act[r] over K, warp-wide (every lane gets the sums).
template <int MR>
__device__ __forceinline__ void dot_row(const float *w, const float *act, int K, float (&acc)[MR]) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int r = 0; r < MR; ++r) acc[r] = 0.0f;
    const int K4 = K >> 2;
#pragma unroll 4
    for (int k4 = lane; k4 < K4; k4 += 32) {
        const float4 wv = *reinterpret_cast<const float4 *>(w + 4 * k4);
#pragma unroll
        for (int r = 0; r < MR; ++r) {
            const float4 a = *reinterpret_cast<const float4 *>(act + r * K + 4 * k4);
            float s = acc[r];
            s = fmaf(wv.x, a.x, s);
            s = fmaf(wv.y, a.y, s);
            s = fmaf(wv.z, a.z, s);
            s = fmaf(wv.w, a.w, s);
            acc[r] = s;
        }
    }
#pragma unroll
    for (int r = 0; r < MR; ++r) acc[r] = warp_sum(acc[r]);
}

template <int MR>
__global__ void __launch_bounds__(PTHREADS, 1) decode_step_persistent_k(const __grid_constant__ PersistParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int NS = p.nstage;
    uint8_t *ring = smem;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + (size_t)NS * STAGE_BYTES);  // full[NS], empty[NS]
    const int KMAX = max(p.d, max(p.E, p.H));
    float *act = reinterpret_cast<float *>(bars + 2 * NS);  // [MR][KMAX]
    float *res = act + MR * KMAX;                           // [res_cap]
    __shared__ float red[MR][CWARPS];
    __shared__ float wbest[CWARPS][MR];
    __shared__ uint32_t widx[CWARPS][MR];
    __shared__ uint32_t s_tok[MR], s_head[MR];
    __shared__ int s_abort, s_dead, s_last;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int M = p.M;
    const uint32_t full0 = smem_u32(&bars[0]), empty0 = smem_u32(&bars[NS]);

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

    const int n_phases = 4 * p.n_layer + 1;

    if (warp == CWARPS) {
        // ---------------- producer
        if (lane == 0) {
            int stage = 0;
            uint32_t parity = 0;
            int issued = 0;
            for (int q = 0; q < n_phases && !*(volatile int *)&s_dead; ++q) {
                const Phase ph = make_phase(p, q >> 2, q == n_phases - 1 ? 4 : (q & 3));
                const uint32_t row_bytes = (uint32_t)ph.K * 4u;
                for (int rg = 0; rg < ph.nreg; ++rg) {
                    for (int r0 = 0; r0 < ph.n; r0 += ph.R) {
                        if (!mbar_wait_bounded(empty0 + 8 * stage, parity ^ 1u)) {
                            atomicExch(p.err, 111);
                            *(volatile int *)&s_dead = 1;
                            break;
                        }
                        if (*(volatile int *)&s_dead) break;
                        const uint32_t bytes = (uint32_t)min(ph.R, ph.n - r0) * row_bytes;
                        const uint32_t fb = full0 + 8 * stage;
                        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(fb), "r"(bytes)
                                     : "memory");
                        asm volatile(
                            "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                            ::"r"(smem_u32(ring + (size_t)stage * STAGE_BYTES)),
                            "l"((uint64_t)(ph.src[rg] + (size_t)r0 * ph.K)), "r"(bytes), "r"(fb)
                            : "memory");
                        ++issued;
                        if (++stage == NS) {
                            stage = 0;
                            parity ^= 1u;
                        }
                    }
                    if (*(volatile int *)&s_dead) break;
                }
            }
            // The consumers wait for every chunk they use; after a stopped
            // pipeline, wait (bounded) for the last copies still in flight so
            // none lands after the CTA exits.
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
        const unsigned G = gridDim.x;
        float wb[MR];
        uint32_t wi[MR];
#pragma unroll
        for (int r = 0; r < MR; ++r) {
            wb[r] = -INFINITY;
            wi[r] = 0xFFFFFFFFu;
        }
        for (int q = 0; q < n_phases; ++q) {
            const int layer = q >> 2;
            const int kind = q == n_phases - 1 ? 4 : (q & 3);
            const Phase ph = make_phase(p, layer, kind);
            const SmallLayer *L = kind < 4 ? &p.layers[layer] : nullptr;
            const int K = ph.K;
            float *state = kind == 0 ? p.state + (size_t)layer * M * (p.k + 1) * p.E : nullptr;

            // ---- operands of the phase epilogue, fetched before anything
            // waits: thread t < n * MR owns row i = t / MR for stream r = t % MR.
            const bool mine = kind != 4 && tid < ph.n * MR && (tid % MR) < M;
            const int ei = tid / MR, er = tid % MR, ej = ph.u0 + ei;
            float pb0 = 0.f, pb1 = 0.f, pb2 = 0.f, pcb = 0.f, ph_old = 0.f, pbase = 0.f;
            float pcw[KCONV], prv[KCONV];
#pragma unroll
            for (int qq = 0; qq < KCONV; ++qq) pcw[qq] = prv[qq] = 0.f;
            if (mine) {
                if (kind == 0) {
                    const int E = p.E, kk = p.k;
                    pb0 = L->in_b[ej];
                    pb1 = L->in_b[E + ej];
                    pb2 = L->in_b[2 * E + ej];
                    pcb = L->conv_b[ej];
                    const float *ring_s = state + (size_t)er * (kk + 1) * E;
                    const uint32_t head = s_head[er];
#pragma unroll
                    for (int qq = 0; qq < KCONV; ++qq)
                        if (qq < kk) {
                            pcw[qq] = L->conv_w[(size_t)qq * E + ej];
                            if (qq > 0) prv[qq] = ring_s[(size_t)((head + (uint32_t)kk - (uint32_t)qq) % (uint32_t)kk) * E + ej];
                        }
                    ph_old = ring_s[(size_t)kk * E + ej];
                } else if (kind == 2) {
                    pb0 = L->up_b[ej];
                    pb1 = L->up_b[p.H + ej];
                } else {
                    pb0 = kind == 1 ? L->out_b[ej] : L->down_b[ej];
                    pbase = (kind == 1 && layer == 0) ? __ldg(p.emb + (size_t)s_tok[er] * p.d + ej)
                                                      : p.x[(size_t)er * p.d + ej];
                }
            }

            // ---- input vector of the phase
            if (kind == 0 || kind == 2 || kind == 4) {
                // Layer 0 normalises the tokens' embedding rows directly.
                const bool from_emb = kind == 0 && layer == 0;
                const float *gain = kind == 0 ? L->n1 : kind == 2 ? L->n2 : p.norm_f;
                const float *rows[MR];
#pragma unroll
                for (int r = 0; r < MR; ++r)
                    rows[r] = from_emb ? p.emb + (size_t)s_tok[r] * p.d : p.x + (size_t)r * p.d;
                norm_to_smem<MR>(rows, gain, p.eps, M, p.d, act, red);
            } else {
                copy_to_smem<MR>(p.g, M, K, act);
            }
            if (kind == 4 && blockIdx.x == 0 && tid < M) p.heads[tid] = s_head[tid];

            // ---- the streamed rows, round-robin over the consumer warps
            int row = 0;  // phase row counter across regions
            for (int rg = 0; rg < ph.nreg; ++rg) {
                for (int r0 = 0; r0 < ph.n; r0 += ph.R) {
                    const int rows = min(ph.R, ph.n - r0);
                    if (!*(volatile int *)&s_dead && !mbar_wait_bounded(full0 + 8 * stage, parity)) {
                        if (lane == 0) atomicExch(p.err, 112);
                        *(volatile int *)&s_dead = 1;
                    }
                    const bool live = !*(volatile int *)&s_dead && !*(volatile int *)&s_abort;
                    const float *chunk = reinterpret_cast<const float *>(ring + (size_t)stage * STAGE_BYTES);
                    // Rows row .. row+rows-1 of the phase; warp w takes those == w (mod CWARPS).
                    for (int j = (warp - row % CWARPS + CWARPS) % CWARPS; j < rows; j += CWARPS) {
                        if (!live) break;
                        float acc[MR];
                        dot_row<MR>(chunk + (size_t)j * K, act, K, acc);
                        const int i = r0 + j;  // row within the region
                        const int u = ph.u0 + i;
                        if (kind != 4) {
                            if (lane < MR) {
                                float v = acc[0];
#pragma unroll
                                for (int r = 1; r < MR; ++r)
                                    if (lane == r) v = acc[r];
                                res[(rg * ph.n + i) * MR + lane] = v;
                            }
                        } else {
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
                    __syncwarp();
                    if (lane == 0)
                        asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(empty0 + 8 * stage) : "memory");
                    if (++stage == NS) {
                        stage = 0;
                        parity ^= 1u;
                    }
                    row += rows;
                }
            }

            // ---- phase epilogue: thread t < n * MR owns (row i, stream r)
            // and applies it with the operands it fetched at phase start.
            if (kind != 4) {
                consumer_sync();
                const bool live = !*(volatile int *)&s_dead && !*(volatile int *)&s_abort;
                if (live && mine) {
                    if (kind == 0) {
                        const int E = p.E, kk = p.k;
                        const float v = res[(0 * ph.n + ei) * MR + er] + pb0;
                        const float zz = res[(1 * ph.n + ei) * MR + er] + pb1;
                        const float oo = res[(2 * ph.n + ei) * MR + er] + pb2;
                        float *ring_s = state + (size_t)er * (kk + 1) * E;
                        const uint32_t head = s_head[er];
                        ring_s[(size_t)head * E + ej] = v;
                        float sum = pcb;
#pragma unroll
                        for (int qq = 0; qq < KCONV; ++qq)
                            if (qq < kk) sum = sum + pcw[qq] * (qq == 0 ? v : prv[qq]);
                        const float value = silu(sum);
                        const float decay = sigmoid(zz);
                        const float h = decay * ph_old + (1.0f - decay) * value;
                        ring_s[(size_t)kk * E + ej] = h;
                        p.g[(size_t)er * E + ej] = h * silu(oo);
                    } else if (kind == 2) {
                        const float a = res[(0 * ph.n + ei) * MR + er];
                        const float b = res[(1 * ph.n + ei) * MR + er];
                        p.g[(size_t)er * p.H + ej] = silu(a + pb0) * (b + pb1);
                    } else {
                        p.x[(size_t)er * p.d + ej] = pbase + (res[ei * MR + er] + pb0);
                    }
                }
            }
            if (kind != 4) {
                // ---- grid barrier: every CTA's outputs of this phase are visible after it
                barrier_target += G;
                consumer_sync();
                if (tid == 0) {
                    // The CTA barrier above orders every consumer's writes
                    // before this release; the acquire below orders the
                    // other CTAs' writes before the barrier after it.
                    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p.sync), "r"(1u) : "memory");
                    if (!*(volatile int *)&s_abort) {
                        const uint64_t t0 = gtimer();
                        for (;;) {
                            uint32_t v;
                            asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p.sync) : "memory");
                            if (v >= barrier_target) break;
                            if (gtimer() - t0 > WAIT_NS) {
                                atomicExch(p.err, 113);
                                *(volatile int *)&s_abort = 1;
                                break;
                            }
                        }
                    }
                }
                consumer_sync();
            }
        }

        // ---- first maximum of the CTA's vocabulary rows, then the last CTA
        // reduces every CTA's partial (earlier CTAs own earlier rows).
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
            consumer_sync();
            if (tid == 0) {
                __threadfence();
                const uint32_t done = atomicAdd(p.sync + 1, 1u);
                s_last = done == G - 1;
                __threadfence();
            }
            consumer_sync();
            if (s_last && tid < M) {
                float b = -INFINITY;
                uint32_t bi = 0xFFFFFFFFu;
                for (unsigned c = 0; c < G; ++c) {
                    const float v = __ldcg(p.best_val + (size_t)tid * G + c);
                    const uint32_t ix = __ldcg(p.best_idx + (size_t)tid * G + c);
                    if (v > b || (v == b && ix < bi)) {
                        b = v;
                        bi = ix;
                    }
                }
                p.tokens_out[tid] = (b == -INFINITY || bi == 0xFFFFFFFFu) ? 0u : bi;
            }
        }
    }
    __syncthreads();
}

template <int MR>
size_t smem_bytes(int d, int E, int H, int res_cap, int nstage) {
    const int kmax = std::max(d, std::max(E, H));
    return (size_t)nstage * STAGE_BYTES + 16 * (size_t)nstage + 4 * ((size_t)MR * kmax + res_cap);
}

template <int MR>
int stages_for(int d, int E, int H, int res_cap) {
    int ns = 12;
    while (ns > 2 && smem_bytes<MR>(d, E, H, res_cap, ns) + 2048 > (size_t)SMEM_LIMIT) --ns;
    return ns;
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

int res_cap_for(int d, int E, int H, int G) {
    const int cd = (d + G - 1) / G, ce = (E + G - 1) / G, ch = (H + G - 1) / G;
    return std::max(cd, std::max(3 * ce, 2 * ch));
}

template <int MR>
cudaError_t launch_mr(const SmallStepArgs &a, const SmallLayer *layers_dev, uint32_t *sync, cudaStream_t st) {
    const int G = sm_count();
    PersistParams p{};
    p.tokens = a.tokens;
    p.tokens_out = a.tokens_out;
    p.emb = a.emb;
    p.norm_f = a.norm_f;
    p.eps = a.eps;
    p.x = a.x;
    p.g = a.g;
    p.state = a.state;
    p.heads = a.heads;
    p.logits = a.logits;
    p.best_val = a.best_val;
    p.best_idx = a.best_idx;
    p.err = a.err;
    p.sync = sync;
    p.layers = layers_dev;
    p.M = a.M;
    p.d = a.d;
    p.E = a.E;
    p.H = a.H;
    p.k = a.k;
    p.V = a.V;
    p.n_layer = a.n_layer;
    p.res_cap = res_cap_for(a.d, a.E, a.H, G) * MR;
    p.nstage = stages_for<MR>(a.d, a.E, a.H, p.res_cap);
    const size_t smem = smem_bytes<MR>(a.d, a.E, a.H, p.res_cap, p.nstage);
    static size_t smem_set = 0;
    cudaError_t e;
    if (smem > smem_set) {
        e = cudaFuncSetAttribute(decode_step_persistent_k<MR>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        smem_set = smem;
    }
    e = cudaMemsetAsync(sync, 0, 2 * sizeof(uint32_t), st);
    if (e != cudaSuccess) return e;
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

}  // namespace

int persistent_partials() { return sm_count(); }

bool persistent_step_supported(int M, int d, int E, int H, int k, int V, int n_layer) {
    if (M < 1 || M > 4 || n_layer < 1 || k < 1 || k > KCONV) return false;
    if (d % 4 || E % 4 || H % 4) return false;
    // Every row fits one stage; the staging of the widest activation and two
    // ring stages fit in shared memory.
    if ((size_t)std::max(d, std::max(E, H)) * 4 > (size_t)STAGE_BYTES) return false;
    const int G = sm_count();
    // One epilogue thread per (owned row, stream) of every phase.
    const int most = std::max(std::max((d + G - 1) / G, (E + G - 1) / G), (H + G - 1) / G);
    if (most * 4 > CTHREADS) return false;
    const int rc = res_cap_for(d, E, H, G) * 4;
    return smem_bytes<4>(d, E, H, rc, 2) + 2048 <= (size_t)SMEM_LIMIT;
}

cudaError_t persistent_step(const SmallStepArgs &a, const SmallLayer *layers_dev, uint32_t *sync,
                            cudaStream_t st) {
    if (a.M <= 1) return launch_mr<1>(a, layers_dev, sync, st);
    if (a.M <= 2) return launch_mr<2>(a, layers_dev, sync, st);
    return launch_mr<4>(a, layers_dev, sync, st);
}

}  // namespace nk
