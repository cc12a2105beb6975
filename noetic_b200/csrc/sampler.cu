// sampler.cu -- sample_token (infer.rs:228-305) for every stream on the device.
//
// One CTA per stream.  Steps follow the reference in order:
//   1. repetition penalty once per distinct token of the last rep_window
//      history entries (divide positive logits, multiply the rest);
//   2. greedy -> argmax (first strict maximum, NaN skipped);
//   3. divide by max(temperature, 1e-4);
//   4. softmax_inplace with its +inf / all-invalid / bad-sum rules
//      (tensor.rs:314-352);
//   5. order by (probability desc under f32::total_cmp, index asc) -- a
//      bitonic sort of 64-bit keys in shared memory -- and keep top_k;
//   6. nucleus: the shortest prefix whose f32 cumulative sum reaches
//      clamp(top_p, 0, 1), at least one entry;
//   7. f64 total; non-finite or <= 0 -> candidates[rng.below(n)], else
//      draw = f32_unit * total and walk the f64 CDF.
// The per-stream xoshiro256++ state (4 x u64) is read and written back, so
// it advances exactly as the reference's Rng does (one f32_unit or below per
// token).  Sums are block reductions instead of sequential loops and expf is
// CUDA's, so probabilities agree with the reference to f32 rounding and the
// sampled token agrees except at CDF / nucleus boundaries.

#include "nk_common.cuh"
#include "nk_kernels.h"

namespace nk {

namespace {

constexpr int SAMPLE_THREADS = 1024;
constexpr int SAMPLE_MAX_V = 16384;

__device__ __forceinline__ uint64_t sort_key(float p, uint32_t idx) {
    const uint32_t ordered = (uint32_t)total_key(p) ^ 0x80000000u;  // increasing with p
    return ((uint64_t)(~ordered) << 32) | idx;                        // ascending == p desc, idx asc
}

__device__ __forceinline__ float key_prob(uint64_t key) {
    const uint32_t ordered = ~(uint32_t)(key >> 32);
    const int32_t tk = (int32_t)(ordered ^ 0x80000000u);
    // total_key is an involution on the bit pattern.
    const int32_t bits = tk ^ (int32_t)((uint32_t)(tk >> 31) >> 1);
    return __int_as_float(bits);
}

template <class T, class Op>
__device__ T block_reduce(T v, Op op, T *red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = op(v, __shfl_xor_sync(0xffffffffu, v, o));
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    const int nw = blockDim.x >> 5;
    T r = red[0];
    for (int w = 1; w < nw; ++w) r = op(r, red[w]);
    return r;
}

// Exclusive block scan of one value per thread (thread order).
template <class T>
__device__ T block_exclusive_scan(T v, T *red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    T incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const T n = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl = incl + n;
    }
    __syncthreads();
    if (lane == 31) red[warp] = incl;
    __syncthreads();
    T base = T(0);
    for (int w = 0; w < warp; ++w) base = base + red[w];
    return base + incl - v;
}

__global__ void __launch_bounds__(SAMPLE_THREADS)
sample_rows_k(float *__restrict__ logits_all, int V, SampleParams cfg,
              const uint32_t *__restrict__ history, const uint32_t *__restrict__ history_len,
              int history_stride, uint64_t *__restrict__ rng_all, uint32_t *__restrict__ out,
              int *err) {
    extern __shared__ __align__(16) uint64_t keys[];
    __shared__ float redf[32];
    __shared__ double redd[32];
    __shared__ int redi[32];
    const int s = blockIdx.x;
    const int tid = threadIdx.x;
    float *logits = logits_all + (size_t)s * V;

    // 1. repetition penalty (sequential: the window is short and order matters
    //    only through "first occurrence").
    if (tid == 0 && isfinite(cfg.rep_penalty) && cfg.rep_penalty > 1.0f && cfg.rep_window > 0 &&
        history != nullptr) {
        const uint32_t *h = history + (size_t)s * history_stride;
        const uint64_t n = history_len[s];
        const uint64_t start = n > cfg.rep_window ? n - cfg.rep_window : 0;
        for (uint64_t i = start; i < n; ++i) {
            const uint32_t tok = h[i];
            if (tok >= (uint32_t)V) continue;
            bool seen = false;
            for (uint64_t q = start; q < i; ++q)
                if (h[q] == tok) {
                    seen = true;
                    break;
                }
            if (seen) continue;
            if (logits[tok] > 0.0f)
                logits[tok] = logits[tok] / cfg.rep_penalty;
            else
                logits[tok] = logits[tok] * cfg.rep_penalty;
        }
    }
    __syncthreads();

    // 2. greedy
    if (cfg.greedy) {
        float bv = -INFINITY;
        int bi = V;
        for (int i = tid; i < V; i += blockDim.x) {
            const float v = logits[i];
            if (!isnan(v) && (v > bv || (v == bv && i < bi))) {
                bv = v;
                bi = i;
            }
        }
        const float mx = block_reduce(bv, [](float a, float b) { return fmaxf(a, b); }, redf);
        const int cand = (bv == mx) ? bi : V;
        const int first = block_reduce(cand, [](int a, int b) { return a < b ? a : b; }, redi);
        if (tid == 0) out[s] = (mx == -INFINITY || first >= V) ? 0u : (uint32_t)first;
        return;
    }

    // 3. temperature
    const float temperature =
        (isfinite(cfg.temperature) && cfg.temperature > 1e-4f) ? cfg.temperature : 1e-4f;
    int pinf = 0;
    float mx = -INFINITY;
    for (int i = tid; i < V; i += blockDim.x) {
        const float v = logits[i] / temperature;
        logits[i] = v;
        if (v == INFINITY) ++pinf;
        if (isfinite(v) && v > mx) mx = v;
    }
    // 4. softmax_inplace
    const int n_pinf = block_reduce(pinf, [](int a, int b) { return a + b; }, redi);
    if (n_pinf > 0) {
        const float p = 1.0f / (float)n_pinf;
        for (int i = tid; i < V; i += blockDim.x) logits[i] = (logits[i] == INFINITY) ? p : 0.0f;
    } else {
        mx = block_reduce(mx, [](float a, float b) { return fmaxf(a, b); }, redf);
        if (mx == -INFINITY) {
            for (int i = tid; i < V; i += blockDim.x) logits[i] = 1.0f / (float)V;
        } else {
            float part = 0.0f;
            for (int i = tid; i < V; i += blockDim.x) {
                const float v = logits[i];
                const float e = isfinite(v) ? expf(v - mx) : 0.0f;
                logits[i] = e;
                part += e;
            }
            const float sum = block_reduce(part, [](float a, float b) { return a + b; }, redf);
            if (!isfinite(sum) || sum <= 0.0f) {
                for (int i = tid; i < V; i += blockDim.x) logits[i] = 1.0f / (float)V;
            } else {
                const float inv = 1.0f / sum;
                for (int i = tid; i < V; i += blockDim.x) logits[i] = logits[i] * inv;
            }
        }
    }
    __syncthreads();

    // 5. sort keys (bitonic, power-of-two padded with the largest key)
    int n = 1;
    while (n < V) n <<= 1;
    for (int i = tid; i < n; i += blockDim.x) keys[i] = i < V ? sort_key(logits[i], (uint32_t)i) : ~0ull;
    __syncthreads();
    for (int size = 2; size <= n; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int i = tid; i < (n >> 1); i += blockDim.x) {
                const int lo = 2 * i - (i & (stride - 1));
                const int hi = lo + stride;
                const bool up = ((lo & size) == 0);
                const uint64_t a = keys[lo], b = keys[hi];
                if ((a > b) == up) {
                    keys[lo] = b;
                    keys[hi] = a;
                }
            }
            __syncthreads();
        }
    }
    const int keep = (cfg.top_k == 0 || cfg.top_k > (uint64_t)V) ? V : (int)cfg.top_k;

    // 6. nucleus cut over contiguous per-thread segments of the sorted list.
    const float top_p = isfinite(cfg.top_p) ? fminf(fmaxf(cfg.top_p, 0.0f), 1.0f) : 1.0f;
    const int seg = (keep + blockDim.x - 1) / blockDim.x;
    const int b0 = min(tid * seg, keep), b1 = min(b0 + seg, keep);
    float local = 0.0f;
    for (int i = b0; i < b1; ++i) local += key_prob(keys[i]);
    const float before = block_exclusive_scan(local, redf);
    int cut = keep;  // number kept if the threshold is never reached
    {
        float c = before;
        for (int i = b0; i < b1; ++i) {
            c += key_prob(keys[i]);
            if (c >= top_p) {
                cut = i + 1;
                break;
            }
        }
    }
    int kept = block_reduce(cut, [](int a, int b) { return a < b ? a : b; }, redi);
    if (kept < 1) kept = 1;

    // 7. f64 total and categorical draw
    const int seg2 = (kept + blockDim.x - 1) / blockDim.x;
    const int c0 = min(tid * seg2, kept), c1 = min(c0 + seg2, kept);
    double dl = 0.0;
    for (int i = c0; i < c1; ++i) dl += (double)key_prob(keys[i]);
    const double total = block_reduce(dl, [](double a, double b) { return a + b; }, redd);
    __shared__ double s_draw;
    __shared__ int s_mode;
    if (tid == 0) {
        uint64_t st[4];
        for (int q = 0; q < 4; ++q) st[q] = rng_all[(size_t)s * 4 + q];
        if (!isfinite(total) || total <= 0.0) {
            int e = 0;
            const uint64_t pick = xoshiro_below(st, (uint64_t)kept, &e);
            if (e) atomicExch(err, 2);
            out[s] = (uint32_t)(keys[pick] & 0xffffffffu);
            s_mode = 1;
        } else {
            s_draw = (double)xoshiro_f32_unit(st) * total;
            s_mode = 0;
        }
        for (int q = 0; q < 4; ++q) rng_all[(size_t)s * 4 + q] = st[q];
    }
    __syncthreads();
    if (s_mode != 0) return;
    const double draw = s_draw;
    const double dbefore = block_exclusive_scan(dl, redd);
    int pick = kept - 1;
    {
        double c = dbefore;
        for (int i = c0; i < c1; ++i) {
            c += (double)key_prob(keys[i]);
            if (draw - c <= 0.0) {
                pick = i;
                break;
            }
        }
        // The CDF is non-decreasing, so threads past the crossing report a
        // later index; the minimum is the reference's first index with
        // draw <= 0, and kept - 1 is its fall-back (infer.rs:304).
    }
    const int chosen = block_reduce(pick, [](int a, int b) { return a < b ? a : b; }, redi);
    if (tid == 0) out[s] = (uint32_t)(keys[chosen] & 0xffffffffu);
}

}  // namespace

int sample_max_vocab() { return SAMPLE_MAX_V; }

cudaError_t sample_rows(float *logits, int S, int V, SampleParams cfg, const uint32_t *history,
                        const uint32_t *history_len, int history_stride, uint64_t *rng,
                        uint32_t *out, int *err, cudaStream_t st) {
    if (S == 0) return cudaSuccess;
    int n = 1;
    while (n < V) n <<= 1;
    const size_t smem = cfg.greedy ? 0 : (size_t)n * sizeof(uint64_t);
    if (!cfg.greedy && V > SAMPLE_MAX_V) return cudaErrorInvalidValue;
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(sample_rows_k, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)smem);
        if (e != cudaSuccess) return e;
    }
    sample_rows_k<<<S, SAMPLE_THREADS, smem, st>>>(logits, V, cfg, history, history_len,
                                                   history_stride, rng, out, err);
    return cudaGetLastError();
}

}  // namespace nk
