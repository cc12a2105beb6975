// small_batch.cu -- the decode step for a handful of streams (M <= 8).
//
// With few streams every projection is a matrix-vector product: each weight
// is read once per token, so the step is bound by HBM bandwidth (1.445 GB per
// token for the d=1024 / 24-layer / vocab-32768 model).  The step is four
// fused kernels per layer plus the logits:
//
//   in_ssm      RMSNorm(x) -> W_in rows (v_j, z_j, o_j) -> conv ring, SiLU,
//               decay, h update, output gate            (infer.rs:143-176)
//   proj_res    x += W . act + b  (out_proj and down)    (infer.rs:178-182, 191-195)
//   up_swiglu   RMSNorm(x) -> W_up rows (a_j, b_j) -> SiLU(a) * b (infer.rs:185-190)
//   logits      RMSNorm(x) -> emb rows, first-maximum partials (infer.rs:198-199)
//
// One warp owns one output feature (or channel), so the recurrent update and
// SwiGLU happen in the warp that produced their inputs.  Each CTA first issues
// an L2 bulk prefetch of its weight rows, then waits on the previous kernel
// (griddepcontrol.wait), then lets the next kernel launch
// (griddepcontrol.launch_dependents).  Launched with programmatic dependent
// launch, each kernel's weights stream from HBM into L2 while the previous
// kernel computes; launched normally the two griddepcontrol instructions are
// no-ops.  Activations are f32; products accumulate in f32 FMA.

#include <algorithm>

#include "nk_common.cuh"
#include "nk_kernels.h"

namespace nk {

namespace {

constexpr int WARPS = 4;
constexpr int THREADS = WARPS * 32;


// Bulk prefetch into L2 of the 16-byte aligned part of [p, p + bytes): the
// start rounds up and the end rounds down, so no byte outside the range is
// touched.
__device__ __forceinline__ void prefetch_l2(const float *p, uint32_t bytes) {
    const uint64_t a0 = (uint64_t)p, a1 = a0 + bytes;
    const uint64_t s = (a0 + 15) & ~15ull, e = a1 & ~15ull;
    if (e > s)
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(s), "r"((uint32_t)(e - s)) : "memory");
}

// Prefetch rows [r0, r0 + n) of a row-major [rows, cols] f32 matrix.
__device__ __forceinline__ void prefetch_rows(const float *w, int rows, int cols, int r0, int n) {
    if (r0 >= rows) return;
    n = min(n, rows - r0);
    const uint64_t bytes = (uint64_t)n * cols * 4;
    const float *p = w + (size_t)r0 * cols;
    // Split into chunks of at most 2^30 bytes (a single chunk in practice).
    for (uint64_t off = 0; off < bytes; off += (1ull << 30)) {
        const uint64_t left = bytes - off;
        prefetch_l2(p + off / 4, (uint32_t)(left < (1ull << 30) ? left : (1ull << 30)));
    }
}

// xs[r][:] = x[r][:] * rsqrt(mean(x^2) + eps) * gain for r < M (tensor.rs:298-312),
// rows r >= M zero.  Every thread issues all of its 16-byte loads before
// using any, and the sum of squares reduces across the whole CTA, so the
// prologue costs one L2 round trip.
template <int MR>
__device__ __forceinline__ void norm_rows_to_smem(const float *__restrict__ x, const float *__restrict__ gain,
                                                  float eps, int M, int d, float *xs) {
    __shared__ float red[MR][WARPS];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float ss[MR];
    if ((d & 3) == 0) {
        constexpr int PT = 4;  // float4 chunks per thread per row covers d <= 2048
        const int d4 = d >> 2;
        float4 v[MR][PT];
#pragma unroll
        for (int r = 0; r < MR; ++r)
#pragma unroll
            for (int i = 0; i < PT; ++i) {
                const int c = threadIdx.x + i * THREADS;
                v[r][i] = (r < M && c < d4) ? *reinterpret_cast<const float4 *>(x + (size_t)r * d + 4 * c)
                                            : make_float4(0.f, 0.f, 0.f, 0.f);
            }
        for (int c = threadIdx.x + PT * THREADS; c < d4; c += THREADS)  // d > 2048: remaining chunks
            for (int r = 0; r < M; ++r) {
                const float4 t = *reinterpret_cast<const float4 *>(x + (size_t)r * d + 4 * c);
                *reinterpret_cast<float4 *>(xs + r * d + 4 * c) = t;
            }
#pragma unroll
        for (int r = 0; r < MR; ++r) {
            float a = 0.0f;
#pragma unroll
            for (int i = 0; i < PT; ++i) {
                a = fmaf(v[r][i].x, v[r][i].x, a);
                a = fmaf(v[r][i].y, v[r][i].y, a);
                a = fmaf(v[r][i].z, v[r][i].z, a);
                a = fmaf(v[r][i].w, v[r][i].w, a);
            }
            for (int c = threadIdx.x + PT * THREADS; c < d4; c += THREADS)
                if (r < M) {
                    const float4 t = *reinterpret_cast<const float4 *>(xs + r * d + 4 * c);
                    a = fmaf(t.x, t.x, a); a = fmaf(t.y, t.y, a); a = fmaf(t.z, t.z, a); a = fmaf(t.w, t.w, a);
                }
            ss[r] = warp_sum(a);
        }
        if (lane == 0)
#pragma unroll
            for (int r = 0; r < MR; ++r) red[r][warp] = ss[r];
        __syncthreads();
#pragma unroll
        for (int r = 0; r < MR; ++r) {
            float tot = 0.0f;
#pragma unroll
            for (int w = 0; w < WARPS; ++w) tot += red[r][w];
            const float rs = (r < M) ? 1.0f / sqrtf(tot / (float)d + eps) : 0.0f;
#pragma unroll
            for (int i = 0; i < PT; ++i) {
                const int c = threadIdx.x + i * THREADS;
                if (c < d4) {
                    const float4 gg = *reinterpret_cast<const float4 *>(gain + 4 * c);
                    float4 o;
                    o.x = v[r][i].x * rs * gg.x; o.y = v[r][i].y * rs * gg.y;
                    o.z = v[r][i].z * rs * gg.z; o.w = v[r][i].w * rs * gg.w;
                    *reinterpret_cast<float4 *>(xs + r * d + 4 * c) = o;
                }
            }
            for (int c = threadIdx.x + PT * THREADS; c < d4; c += THREADS) {
                const float4 gg = *reinterpret_cast<const float4 *>(gain + 4 * c);
                float4 t = *reinterpret_cast<const float4 *>(xs + r * d + 4 * c);
                t.x = t.x * rs * gg.x; t.y = t.y * rs * gg.y; t.z = t.z * rs * gg.z; t.w = t.w * rs * gg.w;
                *reinterpret_cast<float4 *>(xs + r * d + 4 * c) = t;
            }
        }
    } else {
        for (int i = M * d + threadIdx.x; i < MR * d; i += THREADS) xs[i] = 0.0f;
        for (int r = warp; r < M; r += WARPS) {
            const float *xr = x + (size_t)r * d;
            float ms = 0.0f;
            for (int j = lane; j < d; j += 32) ms = fmaf(xr[j], xr[j], ms);
            ms = warp_sum(ms);
            const float rs = 1.0f / sqrtf(ms / (float)d + eps);
            for (int j = lane; j < d; j += 32) xs[r * d + j] = xr[j] * rs * gain[j];
        }
    }
    __syncthreads();
}

// as[r][:] = a[r][:] for r < M, zero for M <= r < MR; all loads issued first.
template <int MR>
__device__ __forceinline__ void copy_rows_to_smem(const float *__restrict__ a, int M, int K, float *as) {
    if ((K & 3) == 0) {
        constexpr int PT = 8;  // covers MR * K <= 4096 floats per... per thread batch
        const int n4 = (M * K) >> 2;
        float4 v[PT];
        for (int base = 0; base < n4; base += PT * THREADS) {
#pragma unroll
            for (int i = 0; i < PT; ++i) {
                const int c = base + threadIdx.x + i * THREADS;
                v[i] = c < n4 ? *reinterpret_cast<const float4 *>(a + 4 * c) : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int i = 0; i < PT; ++i) {
                const int c = base + threadIdx.x + i * THREADS;
                if (c < n4) *reinterpret_cast<float4 *>(as + 4 * c) = v[i];
            }
        }
    } else {
        for (int i = threadIdx.x; i < M * K; i += THREADS) as[i] = a[i];
    }
    for (int i = M * K + threadIdx.x; i < MR * K; i += THREADS) as[i] = 0.0f;
    __syncthreads();
}

// acc[r] += w_row . xs[r] over K (lane-strided; 16-byte loads when K % 4 == 0).
template <int MR, bool VEC>
__device__ __forceinline__ void dot_rows(const float *__restrict__ wrow, const float *xs, int K, float (&acc)[MR]) {
    const int lane = threadIdx.x & 31;
    if (VEC) {
        const float4 *w4 = reinterpret_cast<const float4 *>(wrow);
#pragma unroll 4
        for (int k4 = lane; k4 < (K >> 2); k4 += 32) {
            const float4 w = w4[k4];
#pragma unroll
            for (int r = 0; r < MR; ++r) {
                const float4 x = *reinterpret_cast<const float4 *>(xs + r * K + 4 * k4);
                float s = acc[r];
                s = fmaf(w.x, x.x, s);
                s = fmaf(w.y, x.y, s);
                s = fmaf(w.z, x.z, s);
                s = fmaf(w.w, x.w, s);
                acc[r] = s;
            }
        }
    } else {
        for (int k = lane; k < K; k += 32) {
            const float w = wrow[k];
#pragma unroll
            for (int r = 0; r < MR; ++r) acc[r] = fmaf(w, xs[r * K + k], acc[r]);
        }
    }
}

// A warp's weight row held in registers: lane l holds the float4 chunks
// l, l + 32, ... (NW of them); chunks past the row end read as zero.
template <int NW>
struct RowRegs {
    float4 v[NW > 0 ? NW : 1];
};

template <int NW>
__device__ __forceinline__ void load_row(const float *__restrict__ wrow, int K, RowRegs<NW> &r) {
    const int lane = threadIdx.x & 31;
    const float4 *w4 = reinterpret_cast<const float4 *>(wrow);
#pragma unroll
    for (int i = 0; i < NW; ++i) {
        const int k4 = lane + 32 * i;
        r.v[i] = (k4 < (K >> 2)) ? __ldg(w4 + k4) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
}

template <int MR, int NW>
__device__ __forceinline__ void dot_regs(const RowRegs<NW> &w, const float *xs, int K, float (&acc)[MR]) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int i = 0; i < NW; ++i) {
        const int k4 = lane + 32 * i;
        if (k4 < (K >> 2)) {
#pragma unroll
            for (int r = 0; r < MR; ++r) {
                const float4 x = *reinterpret_cast<const float4 *>(xs + r * K + 4 * k4);
                float s = acc[r];
                s = fmaf(w.v[i].x, x.x, s);
                s = fmaf(w.v[i].y, x.y, s);
                s = fmaf(w.v[i].z, x.z, s);
                s = fmaf(w.v[i].w, x.w, s);
                acc[r] = s;
            }
        }
    }
}

template <int MR>
__device__ __forceinline__ void reduce_all(float (&acc)[MR]) {
#pragma unroll
    for (int r = 0; r < MR; ++r) acc[r] = warp_sum(acc[r]);
}

// ---- in_proj + recurrent step: warp = channel j
template <int MR, bool VEC, int NW>
__global__ void __launch_bounds__(THREADS) in_ssm_k(const float *__restrict__ x, const float *__restrict__ gain,
                                                    float eps, const float *__restrict__ w_in,
                                                    const float *__restrict__ b_in, const float *__restrict__ conv_w,
                                                    const float *__restrict__ conv_b, float *__restrict__ state,
                                                    const uint32_t *__restrict__ heads, float *__restrict__ g,
                                                    int M, int d, int E, int k) {
    extern __shared__ __align__(16) float xs[];  // [MR][d]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int j0 = blockIdx.x * WARPS;
    const int j = j0 + warp;
    const int jc = j < E ? j : E - 1;
    // The weights do not depend on the previous kernel: read them first.
    RowRegs<NW> wv, wz, wo;
    if (NW > 0) {
        load_row<NW>(w_in + (size_t)jc * d, d, wv);
        load_row<NW>(w_in + (size_t)(E + jc) * d, d, wz);
        load_row<NW>(w_in + (size_t)(2 * E + jc) * d, d, wo);
    } else if (threadIdx.x == 0) {
        prefetch_rows(w_in, 3 * E, d, j0, WARPS);
        prefetch_rows(w_in, 3 * E, d, E + j0, min(WARPS, E - j0));
        prefetch_rows(w_in, 3 * E, d, 2 * E + j0, min(WARPS, E - j0));
    }
    pdl_wait();
    pdl_trigger();
    norm_rows_to_smem<MR>(x, gain, eps, M, d, xs);
    if (j >= E) return;
    float av[MR] = {}, az[MR] = {}, ao[MR] = {};
    if (NW > 0) {
        dot_regs<MR, NW>(wv, xs, d, av);
        dot_regs<MR, NW>(wz, xs, d, az);
        dot_regs<MR, NW>(wo, xs, d, ao);
    } else {
        dot_rows<MR, VEC>(w_in + (size_t)j * d, xs, d, av);
        dot_rows<MR, VEC>(w_in + (size_t)(E + j) * d, xs, d, az);
        dot_rows<MR, VEC>(w_in + (size_t)(2 * E + j) * d, xs, d, ao);
    }
    reduce_all<MR>(av);
    reduce_all<MR>(az);
    reduce_all<MR>(ao);
#pragma unroll
    for (int r = 0; r < MR; ++r) {
        if (lane != r || r >= M) continue;
        const float v = av[r] + b_in[j];
        const float zz = az[r] + b_in[E + j];
        const float oo = ao[r] + b_in[2 * E + j];
        float *ring = state + (size_t)r * (k + 1) * E;
        const uint32_t head = heads[r];
        ring[(size_t)head * E + j] = v;
        float sum = conv_b[j];
        for (int q = 0; q < k; ++q) {
            const uint32_t slot = (head + (uint32_t)k - (uint32_t)q) % (uint32_t)k;
            sum = sum + conv_w[(size_t)q * E + j] * (q == 0 ? v : ring[(size_t)slot * E + j]);
        }
        const float value = silu(sum);
        const float decay = sigmoid(zz);
        float *hp = ring + (size_t)k * E + j;
        const float h = decay * (*hp) + (1.0f - decay) * value;
        *hp = h;
        g[(size_t)r * E + j] = h * silu(oo);
    }
}

// ---- x[r, n] += W[n] . act[r] + b[n]: warp = output feature n
template <int MR, bool VEC, int NW>
__global__ void __launch_bounds__(THREADS) proj_res_k(const float *__restrict__ act, const float *__restrict__ w,
                                                      const float *__restrict__ b, float *__restrict__ x, int M,
                                                      int N, int K) {
    extern __shared__ __align__(16) float as[];  // [MR][K]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n0 = blockIdx.x * WARPS;
    const int n = n0 + warp;
    RowRegs<NW> wr;
    if (NW > 0) load_row<NW>(w + (size_t)(n < N ? n : N - 1) * K, K, wr);
    else if (threadIdx.x == 0) prefetch_rows(w, N, K, n0, WARPS);
    pdl_wait();
    pdl_trigger();
    copy_rows_to_smem<MR>(act, M, K, as);
    if (n >= N) return;
    float acc[MR] = {};
    if (NW > 0) dot_regs<MR, NW>(wr, as, K, acc);
    else dot_rows<MR, VEC>(w + (size_t)n * K, as, K, acc);
    reduce_all<MR>(acc);
#pragma unroll
    for (int r = 0; r < MR; ++r)
        if (lane == r && r < M) {
            float *xp = x + (size_t)r * N + n;
            *xp = *xp + (acc[r] + b[n]);
        }
}

// ---- up_proj + SwiGLU: warp = hidden channel j (rows j and H + j)
template <int MR, bool VEC, int NW>
__global__ void __launch_bounds__(THREADS) up_swiglu_k(const float *__restrict__ x, const float *__restrict__ gain,
                                                       float eps, const float *__restrict__ w_up,
                                                       const float *__restrict__ b_up, float *__restrict__ s, int M,
                                                       int d, int H) {
    extern __shared__ __align__(16) float xs[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int j0 = blockIdx.x * WARPS;
    const int j = j0 + warp;
    const int jc = j < H ? j : H - 1;
    RowRegs<NW> wa, wb;
    if (NW > 0) {
        load_row<NW>(w_up + (size_t)jc * d, d, wa);
        load_row<NW>(w_up + (size_t)(H + jc) * d, d, wb);
    } else if (threadIdx.x == 0) {
        prefetch_rows(w_up, 2 * H, d, j0, min(WARPS, H - j0));
        prefetch_rows(w_up, 2 * H, d, H + j0, min(WARPS, H - j0));
    }
    pdl_wait();
    pdl_trigger();
    norm_rows_to_smem<MR>(x, gain, eps, M, d, xs);
    if (j >= H) return;
    float aa[MR] = {}, ab[MR] = {};
    if (NW > 0) {
        dot_regs<MR, NW>(wa, xs, d, aa);
        dot_regs<MR, NW>(wb, xs, d, ab);
    } else {
        dot_rows<MR, VEC>(w_up + (size_t)j * d, xs, d, aa);
        dot_rows<MR, VEC>(w_up + (size_t)(H + j) * d, xs, d, ab);
    }
    reduce_all<MR>(aa);
    reduce_all<MR>(ab);
#pragma unroll
    for (int r = 0; r < MR; ++r)
        if (lane == r && r < M) s[(size_t)r * H + j] = silu(aa[r] + b_up[j]) * (ab[r] + b_up[H + j]);
}

// ---- tied logits: each warp owns LROWS vocabulary rows; optional logits
// store; per-CTA first maximum per stream -> partials [M, gridDim.x].
constexpr int LROWS = 2;

template <int MR, bool VEC, int NW>
__global__ void __launch_bounds__(THREADS) logits_k(const float *__restrict__ x, const float *__restrict__ gain,
                                                    float eps, const float *__restrict__ emb, float *__restrict__ logits,
                                                    float *__restrict__ best_val, uint32_t *__restrict__ best_idx,
                                                    int M, int d, int V) {
    extern __shared__ __align__(16) float xs[];
    __shared__ float sbv[WARPS][MR];
    __shared__ uint32_t sbi[WARPS][MR];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int v0 = blockIdx.x * WARPS * LROWS;
    RowRegs<NW> wrow[LROWS];
    if (NW > 0) {
#pragma unroll
        for (int i = 0; i < LROWS; ++i) {
            const int v = v0 + warp * LROWS + i;
            load_row<NW>(emb + (size_t)(v < V ? v : V - 1) * d, d, wrow[i]);
        }
    } else if (threadIdx.x == 0) {
        prefetch_rows(emb, V, d, v0, WARPS * LROWS);
    }
    pdl_wait();
    pdl_trigger();
    norm_rows_to_smem<MR>(x, gain, eps, M, d, xs);
    float bv[MR];
    uint32_t bi[MR];
#pragma unroll
    for (int r = 0; r < MR; ++r) {
        bv[r] = -INFINITY;
        bi[r] = 0xFFFFFFFFu;
    }
#pragma unroll
    for (int i = 0; i < LROWS; ++i) {
        const int v = v0 + warp * LROWS + i;
        if (v >= V) break;
        float acc[MR] = {};
        if (NW > 0) dot_regs<MR, NW>(wrow[i], xs, d, acc);
        else dot_rows<MR, VEC>(emb + (size_t)v * d, xs, d, acc);
        reduce_all<MR>(acc);
#pragma unroll
        for (int r = 0; r < MR; ++r) {
            if (r >= M) continue;
            if (logits && lane == r) logits[(size_t)r * V + v] = acc[r];
            if (!isnan(acc[r]) && acc[r] > bv[r]) {
                bv[r] = acc[r];
                bi[r] = (uint32_t)v;
            }
        }
    }
    if (lane == 0) {
#pragma unroll
        for (int r = 0; r < MR; ++r) {
            sbv[warp][r] = bv[r];
            sbi[warp][r] = bi[r];
        }
    }
    __syncthreads();
    if (threadIdx.x < M) {
        const int r = threadIdx.x;
        float b = -INFINITY;
        uint32_t idx = 0xFFFFFFFFu;
        for (int w = 0; w < WARPS; ++w)  // warps own increasing row ranges
            if (sbv[w][r] > b) {
                b = sbv[w][r];
                idx = sbi[w][r];
            }
        best_val[(size_t)r * gridDim.x + blockIdx.x] = b;
        best_idx[(size_t)r * gridDim.x + blockIdx.x] = idx;
    }
}

__global__ void embed_step_k(const uint32_t *__restrict__ tokens, const float *__restrict__ emb,
                             float *__restrict__ x, uint32_t *__restrict__ heads, int M, int d, int vocab, int k,
                             int *err) {
    pdl_wait();
    pdl_trigger();
    for (int r = 0; r < M; ++r) {
        uint32_t t = tokens[r];
        if (t >= (uint32_t)vocab) {
            if (threadIdx.x == 0 && blockIdx.x == 0) atomicExch(err, 1);
            t = 0;
        }
        for (int j = blockIdx.x * blockDim.x + threadIdx.x; j < d; j += gridDim.x * blockDim.x)
            x[(size_t)r * d + j] = emb[(size_t)t * d + j];
    }
    if (blockIdx.x == 0 && threadIdx.x < M) heads[threadIdx.x] = (heads[threadIdx.x] + 1u) % (uint32_t)k;
}

// Launch with programmatic dependent launch allowed.
template <class Kern, class... Args>
cudaError_t launch_pdl(Kern kern, unsigned grid, size_t smem, cudaStream_t st, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    return cudaLaunchKernelEx(&cfg, kern, args...);
}

// float4 chunks per lane holding a whole row of width K in registers (0: the
// row is streamed instead).  Register rows need 16-byte aligned rows.
constexpr int nw_for(int K, bool vec) {
    return !vec ? 0 : K <= 128 ? 1 : K <= 256 ? 2 : K <= 512 ? 4 : K <= 1024 ? 8 : K <= 2048 ? 16 : K <= 3072 ? 24 : 0;
}

template <int MR, bool VEC, int NWD, int NWE, int NWH>
cudaError_t step_impl(const SmallStepArgs &a, cudaStream_t st, int *launches) {
    const int M = a.M, d = a.d, E = a.E, H = a.H, k = a.k, V = a.V;
    cudaError_t e = launch_pdl(embed_step_k, (unsigned)std::min(8, (d + THREADS - 1) / THREADS), 0, st, a.tokens,
                               a.emb, a.x, a.heads, M, d, V, k, a.err);
    if (e != cudaSuccess) return e;
    int n = 1;
    const size_t smem_d = (size_t)MR * d * 4, smem_e = (size_t)MR * E * 4, smem_h = (size_t)MR * H * 4;
    for (int l = 0; l < a.n_layer; ++l) {
        const SmallLayer &L = a.layers[l];
        float *state = a.state + (size_t)l * M * (k + 1) * E;
        e = launch_pdl(in_ssm_k<MR, VEC, NWD>, (unsigned)((E + WARPS - 1) / WARPS), smem_d, st, (const float *)a.x, L.n1,
                       a.eps, L.in_w, L.in_b, L.conv_w, L.conv_b, state, (const uint32_t *)a.heads, a.g, M, d, E, k);
        if (e != cudaSuccess) return e;
        e = launch_pdl(proj_res_k<MR, VEC, NWE>, (unsigned)((d + WARPS - 1) / WARPS), smem_e, st, (const float *)a.g,
                       L.out_w, L.out_b, a.x, M, d, E);
        if (e != cudaSuccess) return e;
        e = launch_pdl(up_swiglu_k<MR, VEC, NWD>, (unsigned)((H + WARPS - 1) / WARPS), smem_d, st, (const float *)a.x, L.n2,
                       a.eps, L.up_w, L.up_b, a.g, M, d, H);
        if (e != cudaSuccess) return e;
        e = launch_pdl(proj_res_k<MR, VEC, NWH>, (unsigned)((d + WARPS - 1) / WARPS), smem_h, st, (const float *)a.g,
                       L.down_w, L.down_b, a.x, M, d, H);
        if (e != cudaSuccess) return e;
        n += 4;
    }
    const int n_tiles = small_logit_tiles(V);
    e = launch_pdl(logits_k<MR, VEC, NWD>, (unsigned)n_tiles, smem_d, st, (const float *)a.x, a.norm_f, a.eps, a.emb,
                   a.logits, a.best_val, a.best_idx, M, d, V);
    if (e != cudaSuccess) return e;
    n += 1;
    if (a.tokens_out) {
        e = argmax_partials(a.best_val, a.best_idx, n_tiles, M, a.tokens_out, st);
        if (e != cudaSuccess) return e;
        n += 1;
    }
    if (launches) *launches = n;
    return cudaSuccess;
}

}  // namespace

int small_logit_tiles(int V) { return (V + WARPS * LROWS - 1) / (WARPS * LROWS); }

bool small_step_supported(int M, int d, int E, int H, int k) {
    // Dynamic smem holds MR rows of the widest activation.
    const int widest = std::max(d, std::max(E, H));
    return M >= 1 && M <= GEMV_MAX_ROWS && (size_t)GEMV_MAX_ROWS * widest * 4 <= 200 * 1024 && k <= 64;
}

template <int MR>
cudaError_t step_mr(const SmallStepArgs &a, cudaStream_t st, int *launches) {
    const bool vec = (a.d % 4 == 0) && (a.E % 4 == 0) && (a.H % 4 == 0);
    // Register-resident rows for the shapes of the benchmark models (d = E =
    // 1024, H = 3072; d = E = 192 / 512 / 768); every other shape streams.
    if (vec && a.d == 1024 && a.E == 1024 && a.H == 3072) return step_impl<MR, true, 8, 8, 24>(a, st, launches);
    if (vec && a.d <= 256 && a.E <= 256 && a.H <= 768) return step_impl<MR, true, 2, 2, 8>(a, st, launches);
    if (vec && a.d <= 512 && a.E <= 512 && a.H <= 1536) return step_impl<MR, true, 4, 4, 16>(a, st, launches);
    if (vec && a.d <= 768 && a.E <= 768 && a.H <= 2304) return step_impl<MR, true, 8, 8, 24>(a, st, launches);
    if (vec) return step_impl<MR, true, 0, 0, 0>(a, st, launches);
    return step_impl<MR, false, 0, 0, 0>(a, st, launches);
}

cudaError_t small_step(const SmallStepArgs &a, cudaStream_t st, int *launches) {
    if (a.M <= 1) return step_mr<1>(a, st, launches);
    if (a.M <= 2) return step_mr<2>(a, st, launches);
    if (a.M <= 4) return step_mr<4>(a, st, launches);
    return step_mr<8>(a, st, launches);
}

}  // namespace nk
