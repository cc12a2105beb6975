// sampler.cu -- sample_token (infer.rs:228-305) for every stream on the device,
// at any vocabulary size.
//
// One CTA of 256 threads per stream (grid-stride over streams).  Steps follow
// the reference in order:
//   1. repetition penalty once per distinct token of the last rep_window
//      history entries (divide positive logits, multiply the rest);
//   2. greedy -> argmax (first strict maximum, NaN skipped);
//   3. divide by max(temperature, 1e-4);
//   4. softmax_inplace with its +inf / all-invalid / bad-sum rules
//      (tensor.rs:314-352);
//   5. order by (probability desc under f32::total_cmp, index asc), keep
//      top_k;
//   6. nucleus: the shortest prefix whose f32 cumulative sum reaches
//      clamp(top_p, 0, 1), at least one entry;
//   7. f64 total; non-finite or <= 0 -> candidates[rng.below(n)], else
//      draw = f32_unit * total and walk the f64 CDF.
//
// Reproducing the reference's decisions needs its f32 rounding, not just its
// mathematics: at V = 32768 the f32 running sums of step 4 and step 6 carry
// rounding errors (~1e-6..1e-5) far larger than the gap between neighbouring
// cumulative values, so any other summation order moves the nucleus cut.
// Both sums are therefore computed bit-exactly in the reference's sequential
// order, in parallel (seq_add_tile): while the running sum s stays inside one
// binade [2^E, 2^(E+1)) every sum is a multiple of u = 2^(E-23), so adding x
// rounds x to that grid (ties to even, which depends only on the parity of
// s / u) and the run is an integer prefix sum of per-element increments
// (a block scan over parity-indexed increment pairs); the one element at
// which s leaves the binade is added with an ordinary f32 addition and the
// scan restarts on the next binade's grid.  exp is evaluated in double and
// rounded once to f32, the correctly rounded value, which glibc's expf (the
// reference's libm) returns for all but ~1e-3 of arguments; divisions and
// products are the IEEE f32 operations the reference performs.
//
// Ordering without sorting the whole vocabulary: probabilities are
// non-negative, so their f32 bit patterns K order them.  When top_k <= 4096
// a radix select on K (8-bit digits from the exponent down, each refinement
// one filtered histogram pass) finds the smallest key range holding the
// top_k entries and at most 4096, which are collected into shared memory and
// bitonic-sorted on (~K << 32 | index).  For larger top_k (top_k = 0 keeps
// the whole vocabulary) a lazy MSD radix sort runs in per-CTA global scratch:
// stable scatters by 8-bit digit (so equal keys stay in index order), a stack
// of segments processed from the highest keys down, each segment of at most
// 4096 keys (or a run of adjacent ones) sorted in shared memory and walked by
// the nucleus sum, larger ones split by the next digit; everything past the
// nucleus cut or past top_k is never sorted.
//
// The per-stream xoshiro256++ state (4 x u64) is read and written back, so it
// advances exactly as the reference's Rng does (one f32_unit or below per
// token).  The f64 total and CDF walk use tree-ordered f64 sums, which differ
// from the sequential ones by ~1e-16 of the total.

#include <algorithm>
#include <climits>

#include "nk_common.cuh"
#include "nk_kernels.h"

namespace nk {

namespace {

constexpr int ST = 256;          // threads per sampler CTA
constexpr int NW = ST / 32;      // warps
constexpr int IPT = 4;           // elements per thread in a tile
constexpr int TILE = ST * IPT;   // elements per tile
constexpr int CH = 4096;         // keys sorted in shared memory at once
constexpr int STACK = 4 * 256 + 16;
constexpr int SEQ_CHUNK = 64;    // terms one warp adds one by one where crossings cluster
constexpr uint32_t FULL = 0xffffffffu;
constexpr uint32_t GRID_TOP = 1u << 24;  // s / u reaches 2^24 when s leaves its binade
constexpr int SAT = 1 << 25;             // saturation of grid increments ("leaves the binade")
static_assert(ST == 256, "one thread per radix digit in stable_scatter");

// ---------------------------------------------------------------- keys
__device__ __forceinline__ uint64_t make_key(uint32_t K, uint32_t idx) { return ((uint64_t)(~K) << 32) | idx; }
__device__ __forceinline__ uint32_t key_K(uint64_t key) { return ~(uint32_t)(key >> 32); }
__device__ __forceinline__ float key_p(uint64_t key) { return __uint_as_float(key_K(key)); }
__device__ __forceinline__ uint32_t key_idx(uint64_t key) { return (uint32_t)key; }

// Radix digits of a probability's bit pattern K (K < 2^31), most significant
// first: the exponent, then three mantissa pieces.
__device__ __forceinline__ uint32_t digit_of(uint32_t K, int level) {
    switch (level) {
        case 0: return (K >> 23) & 0xffu;
        case 1: return (K >> 15) & 0xffu;
        case 2: return (K >> 7) & 0xffu;
        default: return K & 0x7fu;
    }
}
__device__ __forceinline__ int digit_shift(int level) { return level == 0 ? 23 : level == 1 ? 15 : level == 2 ? 7 : 0; }
__device__ __forceinline__ uint32_t digit_mask(int level) { return level == 3 ? 0x7fu : 0xffu; }

// ---------------------------------------------------------------- shared memory
struct Map2 {
    int a0, a1;  // grid increment for an incoming running sum of even / odd grid count
};

struct SampSmem {
    uint64_t keys[CH];
    uint32_t hist[256];
    uint32_t sbase[256];
    uint32_t wcnt[NW][256];
    uint32_t stk_start[STACK];
    uint32_t stk_cnt[STACK];
    uint8_t stk_lvl[STACK];
    uint8_t stk_buf[STACK];
    Map2 wmap[NW];
    float redf[NW];
    double redd[NW];
    int redi[NW];
    unsigned long long redu[NW];
    float sval;
    float s_before;
    int ev;
    uint32_t counter;
    int sp;
    int scalar_i[4];
    uint32_t scalar_u[4];
    double draw;
};

// ---------------------------------------------------------------- block helpers
template <class T, class Op>
__device__ T block_reduce(T v, Op op, T *red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = op(v, __shfl_xor_sync(FULL, v, o));
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    T r = red[0];
#pragma unroll
    for (int w = 1; w < NW; ++w) r = op(r, red[w]);
    return r;
}

// Exclusive prefix sum over threads in thread order; *total = block sum.
template <class T>
__device__ T block_excl_scan(T v, T *red, T *total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    T incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const T n = __shfl_up_sync(FULL, incl, o);
        if (lane >= o) incl = incl + n;
    }
    __syncthreads();
    if (lane == 31) red[warp] = incl;
    __syncthreads();
    T base = T(0), all = T(0);
#pragma unroll
    for (int w = 0; w < NW; ++w) {
        if (w < warp) base = base + red[w];
        all = all + red[w];
    }
    *total = all;
    return base + incl - v;
}

// Warp-aggregated shared-memory histogram increment.
__device__ __forceinline__ void hist_add(uint32_t *hist, uint32_t d, bool valid) {
    const uint32_t key = valid ? d : 0xffffu;
    const uint32_t peers = __match_any_sync(FULL, key);
    const int leader = __ffs(peers) - 1;
    if (valid && (int)(threadIdx.x & 31) == leader) atomicAdd(&hist[d], (uint32_t)__popc(peers));
}

// ---------------------------------------------------------------- exact sequential f32 sums
__device__ __forceinline__ Map2 map_id() { return Map2{0, 0}; }

// A then B.
__device__ __forceinline__ Map2 map_then(Map2 A, Map2 B) {
    Map2 r;
    r.a0 = min(SAT, A.a0 + ((A.a0 & 1) ? B.a1 : B.a0));
    r.a1 = min(SAT, A.a1 + (((A.a1 + 1) & 1) ? B.a1 : B.a0));
    return r;
}

// The binade of s >= 0: s = N * 2^(E - 23), N < 2^24.  Zero, subnormals and the
// first normal binade share the grid 2^-149 (E = -126, N = the bit pattern).
struct Grid {
    int E;
    uint32_t N0;
};
__device__ __forceinline__ Grid grid_of(float s) {
    const uint32_t b = __float_as_uint(s);
    const uint32_t be = b >> 23;
    if (be <= 1) return Grid{-126, b};
    return Grid{(int)be - 127, (1u << 23) | (b & 0x7fffffu)};
}
__device__ __forceinline__ float grid_value(int E, uint32_t N) {
    if (E == -126) return __uint_as_float(N);
    return __uint_as_float(((uint32_t)(E + 127) << 23) | (N & 0x7fffffu));
}

// Increment of the grid count when x >= 0 is added on the grid of binade E:
// x / u rounded to an integer, ties to the even total (parity-dependent);
// SAT when x alone leaves the binade.
__device__ __forceinline__ Map2 elem_map(float x, int E) {
    const uint32_t b = __float_as_uint(x);
    const uint32_t be = b >> 23;
    const int ex = be ? (int)be - 127 : -126;
    const uint32_t mx = be ? ((b & 0x7fffffu) | (1u << 23)) : (b & 0x7fffffu);
    const int sh = E - ex;  // x / u = mx * 2^-sh
    if (sh < 0) return Map2{SAT, SAT};
    if (sh == 0) return Map2{(int)mx, (int)mx};
    if (sh >= 25) return Map2{0, 0};
    const uint32_t F = mx >> sh, rem = mx & ((1u << sh) - 1u), half = 1u << (sh - 1);
    if (rem < half) return Map2{(int)F, (int)F};
    if (rem > half) return Map2{(int)F + 1, (int)F + 1};
    return (F & 1u) ? Map2{(int)F + 1, (int)F} : Map2{(int)F, (int)F + 1};
}

// Smallest grid count N with N * 2^(E-23) >= thr; UINT_MAX when no count
// below 2^24 reaches it (or thr is +inf / NaN).
__device__ __forceinline__ uint32_t grid_threshold(float thr, int E) {
    if (!(thr < INFINITY)) return 0xffffffffu;
    if (thr <= 0.0f) return 0u;
    const double q = ldexp((double)thr, 23 - E);
    if (q >= (double)GRID_TOP) return 0xffffffffu;
    return (uint32_t)ceil(q);
}

// s <- fl(...fl(fl(s + x_0) + x_1)...) over x_j = get(j), j in [0, n),
// n <= TILE, every x_j finite and >= 0; sm.sval holds s.  Stops at the first
// j with s_{j+1} >= thr and returns j (sm.sval = s_{j+1}); else returns -1.
// Bit-identical to the sequential loop (see the file comment).
template <class Get>
__device__ int seq_add_tile(const Get &get, int n, float thr, SampSmem &sm, bool first_tile = true) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    int pos = 0;
    // The running sum's binade crossings cluster where it is still small
    // compared with the terms (the first few dozen terms of a sum); there one
    // warp adds the terms one by one, every lane holding the same running sum
    // (cheaper than a block scan per crossing), and the block scan takes over
    // once crossings are far apart.
    bool one_by_one = first_tile;
    for (;;) {
        __syncthreads();
        const float s = sm.sval;
        if (pos >= n) return -1;
        if (one_by_one) {
            const int m = min(SEQ_CHUNK, n - pos);
            if (warp == 0) {
                float acc = s;
                int found = INT_MAX;
                for (int b = 0; b < m && found == INT_MAX; b += 32) {
                    const float x = b + lane < m ? get(pos + b + lane) : 0.0f;
                    for (int k = 0; k < 32 && b + k < m; ++k) {
                        acc = __fadd_rn(acc, __shfl_sync(FULL, x, k));
                        if (acc >= thr) {
                            found = pos + b + k;
                            break;
                        }
                    }
                }
                if (lane == 0) {
                    sm.sval = acc;
                    sm.ev = found;
                }
            }
            __syncthreads();
            const int f = sm.ev;
            if (f != INT_MAX) {
                __syncthreads();
                return f;
            }
            pos += m;
            one_by_one = false;
            continue;
        }
        const Grid g = grid_of(s);
        const uint32_t nthr = grid_threshold(thr, g.E);
        Map2 m[IPT];
        Map2 acc = map_id();
        const int j0 = pos + tid * IPT;
#pragma unroll
        for (int q = 0; q < IPT; ++q) {
            const int j = j0 + q;
            m[q] = j < n ? elem_map(get(j), g.E) : map_id();
            acc = map_then(acc, m[q]);
        }
        Map2 inc = acc;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            Map2 up;
            up.a0 = __shfl_up_sync(FULL, inc.a0, o);
            up.a1 = __shfl_up_sync(FULL, inc.a1, o);
            if (lane >= o) inc = map_then(up, inc);
        }
        Map2 ex;
        ex.a0 = __shfl_up_sync(FULL, inc.a0, 1);
        ex.a1 = __shfl_up_sync(FULL, inc.a1, 1);
        if (lane == 0) ex = map_id();
        if (lane == 31) sm.wmap[warp] = inc;
        if (tid == 0) sm.ev = INT_MAX;
        __syncthreads();
        Map2 wp = map_id();
        for (int w = 0; w < warp; ++w) wp = map_then(wp, sm.wmap[w]);
        const Map2 pre = map_then(wp, ex);
        const int par0 = (int)(g.N0 & 1u);
        uint32_t N = g.N0 + (uint32_t)(par0 ? pre.a1 : pre.a0);
        int my_ev = INT_MAX;
        uint32_t n_ev = 0;
#pragma unroll
        for (int q = 0; q < IPT; ++q) {
            const int j = j0 + q;
            if (j < n && my_ev == INT_MAX) {
                const uint32_t na = N + (uint32_t)((N & 1u) ? m[q].a1 : m[q].a0);
                if (na >= GRID_TOP || na >= nthr) {
                    my_ev = j;
                    n_ev = N;
                }
                N = na;
            }
        }
        if (my_ev != INT_MAX) atomicMin(&sm.ev, my_ev);
        __syncthreads();
        const int ev = sm.ev;
        if (ev == INT_MAX) {
            if (tid == ST - 1) {
                const Map2 tot = map_then(pre, acc);
                sm.sval = grid_value(g.E, g.N0 + (uint32_t)(par0 ? tot.a1 : tot.a0));
            }
            pos = n;
            continue;
        }
        if (my_ev == ev) sm.s_before = grid_value(g.E, n_ev);
        __syncthreads();
        if (tid == 0) sm.sval = __fadd_rn(sm.s_before, get(ev));
        __syncthreads();
        if (sm.sval >= thr) {
            __syncthreads();
            return ev;
        }
        one_by_one = ev - pos < SEQ_CHUNK;  // crossings close together
        pos = ev + 1;
    }
}

// ---------------------------------------------------------------- sorting
// Ascending bitonic sort of keys[0, n), n <= CH, padded with ~0.
__device__ void smem_sort(uint64_t *keys, int n) {
    int np = 1;
    while (np < n) np <<= 1;
    for (int i = n + threadIdx.x; i < np; i += ST) keys[i] = ~0ull;
    __syncthreads();
    for (int size = 2; size <= np; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int i = threadIdx.x; i < (np >> 1); i += ST) {
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
}

// Stable scatter of elements [0, n) (key = get(i), digit d = dig(key)) whose
// digit is kept (d >= d_min) to dst[sm.sbase[d] + rank], rank counting
// earlier elements of the same digit; sm.sbase must hold each digit's first
// position and advances.  Elements are handled in index order by tiles of
// TILE: warp w owns 128 consecutive ones, lane order within each step of 32.
template <class GetKey, class Dig>
__device__ void stable_scatter(const GetKey &get, int n, const Dig &dig, uint32_t d_min, uint64_t *dst,
                               SampSmem &sm) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t lt = (1u << lane) - 1u;
    for (int i = tid; i < NW * 256; i += ST) (&sm.wcnt[0][0])[i] = 0;
    __syncthreads();
    for (int base = 0; base < n; base += TILE) {
        uint64_t key[IPT];
        uint32_t dg[IPT], rk[IPT];
#pragma unroll
        for (int q = 0; q < IPT; ++q) {
            const int i = base + warp * (32 * IPT) + q * 32 + lane;
            const bool valid = i < n;
            key[q] = valid ? get(i) : 0ull;
            const uint32_t d = valid ? dig(key[q]) : 0u;
            const bool take = valid && d >= d_min;
            dg[q] = take ? d : 0xffffu;
            const uint32_t peers = __match_any_sync(FULL, dg[q]);
            const uint32_t before = take ? sm.wcnt[warp][d] : 0u;
            rk[q] = before + (uint32_t)__popc(peers & lt);
            __syncwarp();
            if (take && (int)lane == __ffs(peers) - 1) sm.wcnt[warp][d] = before + (uint32_t)__popc(peers);
            __syncwarp();
        }
        __syncthreads();
        // digit t: per-warp starting offsets within this tile, then the
        // running base advances by the tile's count.
        {
            const int d = tid;
            uint32_t run = sm.sbase[d];
            for (int w = 0; w < NW; ++w) {
                const uint32_t c = sm.wcnt[w][d];
                sm.wcnt[w][d] = run;
                run += c;
            }
            sm.sbase[d] = run;
        }
        __syncthreads();
#pragma unroll
        for (int q = 0; q < IPT; ++q)
            if (dg[q] != 0xffffu) dst[sm.wcnt[warp][dg[q]] + rk[q]] = key[q];
        __syncthreads();
        for (int i = tid; i < NW * 256; i += ST) (&sm.wcnt[0][0])[i] = 0;
        __syncthreads();
    }
}

// ---------------------------------------------------------------- the kernel
struct SampleArgs {
    float *logits;
    int S, V;
    SampleParams cfg;
    const uint32_t *history, *history_len;
    int history_stride;
    uint64_t *rng;
    uint32_t *out;
    int *err;
    uint64_t *ws;     // per-CTA scratch for the lazy sort: 2 * ws_keys keys per CTA
    size_t ws_keys;
    // Rows already penalised and divided by the temperature by the logits
    // projection's epilogue, with per-part maxima / +inf counts (nullable).
    const float *prep_max;
    const uint32_t *prep_pinf;
    int prep_parts;
};

// Walk sorted keys get(0..n) through the nucleus sum; returns the number
// kept once the running f32 sum reaches top_p, or -1 when it did not.
template <class Get>
__device__ int nucleus_walk(const Get &get, int n, float top_p, SampSmem &sm) {
    for (int b = 0; b < n; b += TILE) {
        const int m = min(TILE, n - b);
        const int j = seq_add_tile([&](int i) { return get(b + i); }, m, top_p, sm, b == 0);
        if (j >= 0) return b + j + 1;
    }
    return -1;
}

// f64 total of sorted keys get(0..kept), the draw, and the CDF walk; returns
// the chosen position in the sorted order (thread-uniform).
template <class Get>
__device__ int draw_position(const Get &get, int kept, uint64_t *rng, int *err, SampSmem &sm) {
    const int tid = threadIdx.x;
    double part = 0.0;
    for (int i = tid; i < kept; i += ST) part += (double)key_p(get(i));
    const double total = block_reduce(part, [](double a, double b) { return a + b; }, sm.redd);
    if (tid == 0) {
        uint64_t st[4];
        for (int q = 0; q < 4; ++q) st[q] = rng[q];
        if (!isfinite(total) || total <= 0.0) {
            int e = 0;
            sm.scalar_i[0] = (int)xoshiro_below(st, (uint64_t)kept, &e);
            if (e) atomicExch(err, 2);
            sm.scalar_i[1] = 1;
        } else {
            sm.draw = (double)xoshiro_f32_unit(st) * total;
            sm.scalar_i[1] = 0;
        }
        for (int q = 0; q < 4; ++q) rng[q] = st[q];
    }
    __syncthreads();
    if (sm.scalar_i[1]) return sm.scalar_i[0];
    const double draw = sm.draw;
    double carry = 0.0;
    for (int b = 0; b < kept; b += TILE) {
        double v[IPT];
        double mine = 0.0;
#pragma unroll
        for (int q = 0; q < IPT; ++q) {
            const int i = b + tid * IPT + q;
            v[q] = i < kept ? (double)key_p(get(i)) : 0.0;
            mine += v[q];
        }
        double tile_total;
        double c = carry + block_excl_scan(mine, sm.redd, &tile_total);
        int pick = INT_MAX;
#pragma unroll
        for (int q = 0; q < IPT; ++q) {
            const int i = b + tid * IPT + q;
            c += v[q];
            if (i < kept && pick == INT_MAX && draw - c <= 0.0) pick = i;
        }
        const int first = block_reduce(pick, [](int a, int b2) { return a < b2 ? a : b2; }, sm.redi);
        if (first != INT_MAX) return first;
        carry += tile_total;
    }
    return kept - 1;  // infer.rs:304: fall back to the last candidate
}

__device__ void sample_one(const SampleArgs &a, int s, SampSmem &sm) {
    const int tid = threadIdx.x;
    const int V = a.V;
    const SampleParams &cfg = a.cfg;
    float *logits = a.logits + (size_t)s * V;

    const bool prepped = a.prep_max != nullptr && !cfg.greedy;
    // 1. repetition penalty (sequential: the window is short and order
    //    matters only through "first occurrence").
    if (!prepped && tid == 0 && isfinite(cfg.rep_penalty) && cfg.rep_penalty > 1.0f && cfg.rep_window > 0 &&
        a.history != nullptr) {
        const uint32_t *h = a.history + (size_t)s * a.history_stride;
        const uint64_t n = a.history_len[s];
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
            const float v = logits[tok];
            logits[tok] = v > 0.0f ? __fdiv_rn(v, cfg.rep_penalty) : __fmul_rn(v, cfg.rep_penalty);
        }
    }
    __syncthreads();

    // 2. greedy
    if (cfg.greedy) {
        float bv = -INFINITY;
        int bi = V;
        for (int i = tid; i < V; i += ST) {
            const float v = logits[i];
            if (!isnan(v) && (v > bv || (v == bv && i < bi))) {
                bv = v;
                bi = i;
            }
        }
        const float mx = block_reduce(bv, [](float x, float y) { return fmaxf(x, y); }, sm.redf);
        const int cand = (bv == mx) ? bi : V;
        const int first = block_reduce(cand, [](int x, int y) { return x < y ? x : y; }, sm.redi);
        if (tid == 0) a.out[s] = (mx == -INFINITY || first >= V) ? 0u : (uint32_t)first;
        __syncthreads();
        return;
    }

    // 3. temperature
    const float temperature =
        (isfinite(cfg.temperature) && cfg.temperature > 1e-4f) ? cfg.temperature : 1e-4f;
    int pinf = 0;
    float mx = -INFINITY;
    if (prepped) {
        // Steps 1 and 3 ran in the projection epilogue: combine its parts.
        for (int i = tid; i < a.prep_parts; i += ST) {
            const size_t slot = (size_t)s * a.prep_parts + i;
            pinf += (int)a.prep_pinf[slot];
            mx = fmaxf(mx, a.prep_max[slot]);
        }
    } else {
        for (int i = tid; i < V; i += ST) {
            const float v = __fdiv_rn(logits[i], temperature);
            logits[i] = v;
            if (v == INFINITY) ++pinf;
            if (isfinite(v) && v > mx) mx = v;
        }
    }
    // 4. softmax_inplace
    const int n_pinf = block_reduce(pinf, [](int x, int y) { return x + y; }, sm.redi);
    mx = block_reduce(mx, [](float x, float y) { return fmaxf(x, y); }, sm.redf);
    bool uniform = false;
    if (n_pinf > 0) {
        const float p = __fdiv_rn(1.0f, (float)n_pinf);
        for (int i = tid; i < V; i += ST) logits[i] = (logits[i] == INFINITY) ? p : 0.0f;
    } else if (mx == -INFINITY) {
        uniform = true;
    } else {
        // e = exp(v - max) into the row and a shared tile, then the exact
        // sequential f32 sum of the tile.
        float *tilebuf = reinterpret_cast<float *>(sm.keys);
        if (tid == 0) sm.sval = 0.0f;
        for (int b = 0; b < V; b += TILE) {
            const int n = min(TILE, V - b);
            __syncthreads();
            for (int j = tid; j < n; j += ST) {
                const float v = logits[b + j];
                const float e = isfinite(v) ? (float)exp((double)__fsub_rn(v, mx)) : 0.0f;
                logits[b + j] = e;
                tilebuf[j] = e;
            }
            seq_add_tile([&](int j) { return tilebuf[j]; }, n, INFINITY, sm, b == 0);
        }
        __syncthreads();
        const float sum = sm.sval;
        if (!isfinite(sum) || sum <= 0.0f) {
            uniform = true;
        } else {
            // Probabilities, with the level-0 histogram of their exponents.
            const float inv = __fdiv_rn(1.0f, sum);
            for (int i = tid; i < 256; i += ST) sm.hist[i] = 0;
            __syncthreads();
            for (int b = 0; b < V; b += ST) {
                const int i = b + tid;
                const bool valid = i < V;
                uint32_t K = 0;
                if (valid) {
                    const float p = __fmul_rn(logits[i], inv);
                    logits[i] = p;
                    K = __float_as_uint(p);
                }
                hist_add(sm.hist, digit_of(K, 0), valid);
            }
            __syncthreads();
        }
    }
    if (uniform) {
        const float p = __fdiv_rn(1.0f, (float)V);
        for (int i = tid; i < V; i += ST) logits[i] = p;
    }
    if (n_pinf > 0 || uniform) {
        // Level-0 histogram of the probabilities' exponents.
        __syncthreads();
        for (int i = tid; i < 256; i += ST) sm.hist[i] = 0;
        __syncthreads();
        for (int b = 0; b < V; b += ST) {
            const int i = b + tid;
            const bool valid = i < V;
            hist_add(sm.hist, valid ? digit_of(__float_as_uint(logits[i]), 0) : 0u, valid);
        }
        __syncthreads();
    }

    const int keep = (cfg.top_k == 0 || cfg.top_k > (uint64_t)V) ? V : (int)cfg.top_k;
    const float top_p = isfinite(cfg.top_p) ? fminf(fmaxf(cfg.top_p, 0.0f), 1.0f) : 1.0f;
    uint64_t *rng = a.rng + (size_t)s * 4;

    if (keep <= CH) {
        // 5a. radix select of the smallest key range holding the top `keep`
        //     entries and at most CH, collected and sorted in shared memory.
        uint32_t prefix = 0, pmask = 0, above = 0;
        uint32_t klo = 0;
        int ties = 0;  // 1: the boundary key is exact and its ties are taken in index order
        for (int level = 0; level < 4; ++level) {
            if (level > 0) {
                for (int i = tid; i < 256; i += ST) sm.hist[i] = 0;
                __syncthreads();
                for (int b = 0; b < V; b += ST) {
                    const int i = b + tid;
                    const uint32_t K = i < V ? __float_as_uint(logits[i]) : 0u;
                    const bool in = i < V && (K & pmask) == prefix;
                    hist_add(sm.hist, in ? digit_of(K, level) : 0u, in);
                }
                __syncthreads();
            }
            if (tid == 0) {
                uint32_t cum = above;
                int d = (int)digit_mask(level);
                for (; d > 0; --d) {
                    if (cum + sm.hist[d] >= (uint32_t)keep) break;
                    cum += sm.hist[d];
                }
                sm.scalar_u[0] = (uint32_t)d;
                sm.scalar_u[1] = cum;               // entries above digit d
                sm.scalar_u[2] = sm.hist[d];
            }
            __syncthreads();
            const uint32_t d = sm.scalar_u[0], ab = sm.scalar_u[1], ceq = sm.scalar_u[2];
            const int sh = digit_shift(level);
            if (ab + ceq <= (uint32_t)CH) {
                klo = prefix | (d << sh);
                break;
            }
            prefix |= d << sh;
            pmask |= digit_mask(level) << sh;
            above = ab;
            if (level == 3) {
                klo = prefix;
                ties = 1;
            }
        }
        int n_c;
        if (!ties) {
            if (tid == 0) sm.counter = 0;
            __syncthreads();
            for (int i = tid; i < V; i += ST) {
                const uint32_t K = __float_as_uint(logits[i]);
                if (K >= klo) sm.keys[atomicAdd(&sm.counter, 1u)] = make_key(K, (uint32_t)i);
            }
            __syncthreads();
            n_c = (int)sm.counter;
        } else {
            // Entries above the exact boundary key, then its ties in index
            // order until `keep` are held.
            if (tid == 0) sm.counter = 0;
            __syncthreads();
            for (int i = tid; i < V; i += ST) {
                const uint32_t K = __float_as_uint(logits[i]);
                if (K > klo) sm.keys[atomicAdd(&sm.counter, 1u)] = make_key(K, (uint32_t)i);
            }
            __syncthreads();
            const int n_above = (int)sm.counter;
            const int want = keep - n_above;
            int taken = 0;
            for (int b = 0; b < V && taken < want; b += ST) {
                const int i = b + tid;
                const bool f = i < V && __float_as_uint(logits[i]) == klo;
                int tot;
                const int r = block_excl_scan(f ? 1 : 0, sm.redi, &tot);
                if (f && taken + r < want) sm.keys[n_above + taken + r] = make_key(klo, (uint32_t)i);
                taken += tot;
            }
            __syncthreads();
            n_c = n_above + min(taken, want);
        }
        smem_sort(sm.keys, n_c);
        const int lim = min(keep, n_c);
        // 6. nucleus
        if (tid == 0) sm.sval = 0.0f;
        int kept = nucleus_walk([&](int i) { return key_p(sm.keys[i]); }, lim, top_p, sm);
        if (kept < 0) kept = lim;
        kept = max(kept, 1);
        // 7. draw
        const int pos = draw_position([&](int i) { return sm.keys[i]; }, kept, rng, a.err, sm);
        if (tid == 0) a.out[s] = key_idx(sm.keys[pos]);
        __syncthreads();
        return;
    }

    // 5b. lazy MSD radix sort in this CTA's scratch (A holds the final order).
    uint64_t *A = a.ws + (size_t)blockIdx.x * 2 * a.ws_keys;
    uint64_t *B = A + a.ws_keys;
    if (tid == 0) {
        uint32_t cum = 0;
        int d = 255;
        for (; d > 0; --d) {
            if (cum + sm.hist[d] >= (uint32_t)keep) break;
            cum += sm.hist[d];
        }
        sm.scalar_u[0] = (uint32_t)d;
        uint32_t pos = 0;
        for (int e = 255; e >= d; --e) {
            sm.sbase[e] = pos;
            pos += sm.hist[e];
        }
        sm.sp = 0;
        for (int e = d; e <= 255; ++e)
            if (sm.hist[e]) {
                sm.stk_start[sm.sp] = sm.sbase[e];
                sm.stk_cnt[sm.sp] = sm.hist[e];
                sm.stk_lvl[sm.sp] = 1;
                sm.stk_buf[sm.sp] = 0;
                ++sm.sp;
            }
    }
    __syncthreads();
    {
        const uint32_t d_min = sm.scalar_u[0];
        stable_scatter([&](int i) { return make_key(__float_as_uint(logits[i]), (uint32_t)i); }, V,
                       [](uint64_t k) { return digit_of(key_K(k), 0); }, d_min, A, sm);
    }
    int taken = 0, kept = -1;
    if (tid == 0) sm.sval = 0.0f;
    __syncthreads();
    while (sm.sp > 0 && kept < 0 && taken < keep) {
        const int top = sm.sp - 1;
        const uint32_t start = sm.stk_start[top], cnt = sm.stk_cnt[top];
        const int lvl = sm.stk_lvl[top], buf = sm.stk_buf[top];
        __syncthreads();
        if (cnt > (uint32_t)CH && lvl <= 3) {
            // Split by the next digit; drop sub-bins past `keep`.
            uint64_t *src = (buf ? B : A) + start;
            uint64_t *dst = (buf ? A : B);
            for (int i = tid; i < 256; i += ST) sm.hist[i] = 0;
            __syncthreads();
            for (uint32_t b = 0; b < cnt; b += ST) {
                const uint32_t i = b + tid;
                const bool valid = i < cnt;
                hist_add(sm.hist, valid ? digit_of(key_K(src[i]), lvl) : 0u, valid);
            }
            __syncthreads();
            if (tid == 0) {
                const uint32_t need = (uint32_t)keep - start;
                uint32_t cum = 0;
                int d = (int)digit_mask(lvl);
                for (; d > 0; --d) {
                    if (cum + sm.hist[d] >= need) break;
                    cum += sm.hist[d];
                }
                sm.scalar_u[0] = (uint32_t)d;
                uint32_t pos = start;
                for (int e = 255; e >= d; --e) {
                    sm.sbase[e] = pos;
                    pos += sm.hist[e];
                }
                int sp = top;  // pop the split segment
                for (int e = d; e <= 255; ++e)
                    if (sm.hist[e] && sp < STACK) {
                        sm.stk_start[sp] = sm.sbase[e];
                        sm.stk_cnt[sp] = sm.hist[e];
                        sm.stk_lvl[sp] = (uint8_t)(lvl + 1);
                        sm.stk_buf[sp] = (uint8_t)(buf ^ 1);
                        ++sp;
                    }
                sm.sp = sp;
            }
            __syncthreads();
            const uint32_t d_min = sm.scalar_u[0];
            stable_scatter([&](int i) { return src[i]; }, (int)cnt,
                           [lvl](uint64_t k) { return digit_of(key_K(k), lvl); }, d_min, dst, sm);
            continue;
        }
        if (cnt > (uint32_t)CH) {
            // Every key of the segment is equal and the stable scatters kept
            // index order: already sorted.
            if (buf)
                for (uint32_t i = tid; i < cnt; i += ST) A[start + i] = B[start + i];
            if (tid == 0) sm.sp = top;
            __syncthreads();
            const int lim = min((int)cnt, keep - taken);
            const int k = nucleus_walk([&](int i) { return key_p(A[start + i]); }, lim, top_p, sm);
            if (k >= 0) kept = taken + k;
            taken += lim;
            continue;
        }
        // A run of adjacent small segments, sorted together in shared memory.
        if (tid == 0) {
            uint32_t total = 0;
            int r = top;
            while (r >= 0 && sm.stk_cnt[r] <= (uint32_t)CH && total + sm.stk_cnt[r] <= (uint32_t)CH) {
                total += sm.stk_cnt[r];
                --r;
            }
            sm.scalar_u[0] = total;
            sm.scalar_i[0] = r + 1;  // first stack entry of the run
        }
        __syncthreads();
        const uint32_t total = sm.scalar_u[0];
        const int r0 = sm.scalar_i[0];
        for (int e = top; e >= r0; --e) {
            const uint64_t *src = (sm.stk_buf[e] ? B : A) + sm.stk_start[e];
            const uint32_t off = sm.stk_start[e] - start;
            for (uint32_t i = tid; i < sm.stk_cnt[e]; i += ST) sm.keys[off + i] = src[i];
        }
        __syncthreads();
        if (tid == 0) sm.sp = r0;
        smem_sort(sm.keys, (int)total);
        for (uint32_t i = tid; i < total; i += ST) A[start + i] = sm.keys[i];
        const int lim = min((int)total, keep - taken);
        const int k = nucleus_walk([&](int i) { return key_p(sm.keys[i]); }, lim, top_p, sm);
        if (k >= 0) kept = taken + k;
        taken += lim;
        __syncthreads();
    }
    if (kept < 0) kept = taken;
    kept = max(kept, 1);
    __syncthreads();
    const int pos = draw_position([&](int i) { return A[i]; }, kept, rng, a.err, sm);
    if (tid == 0) a.out[s] = key_idx(A[pos]);
    __syncthreads();
}

// Bit (s, t) of bits [S][words] set for every token t < V among the last
// `window` history entries of stream s (the tokens infer.rs:236-248
// penalises, each once).
__global__ void pen_bitmap_k(const uint32_t *__restrict__ history, const uint32_t *__restrict__ history_len,
                             int stride, uint64_t window, int V, uint32_t *__restrict__ bits, int words) {
    const int s = blockIdx.x;
    uint32_t *row = bits + (size_t)s * words;
    for (int i = threadIdx.x; i < words; i += blockDim.x) row[i] = 0u;
    __syncthreads();
    const uint32_t *h = history + (size_t)s * stride;
    const uint64_t n = history_len[s];
    const uint64_t start = n > window ? n - window : 0;
    for (uint64_t i = start + threadIdx.x; i < n; i += blockDim.x) {
        const uint32_t t = h[i];
        if (t < (uint32_t)V) atomicOr(&row[t >> 5], 1u << (t & 31u));
    }
}

// out[s * n_new + *column] = tok[s]; the column counter advances in a
// separate launch (collect_next_k) so that every thread reads the same one.
__global__ void collect_tokens_k(const uint32_t *__restrict__ tok, uint32_t *__restrict__ out, int S, int n_new,
                                 const int *__restrict__ column) {
    const int s = blockIdx.x * blockDim.x + threadIdx.x;
    const int c = *column;
    if (s < S && c >= 0 && c < n_new) out[(size_t)s * n_new + c] = tok[s];
}
__global__ void collect_next_k(int *column) { *column += 1; }

__global__ void __launch_bounds__(ST) sample_rows_k(SampleArgs a) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    SampSmem &sm = *reinterpret_cast<SampSmem *>(smem_raw);
    for (int s = blockIdx.x; s < a.S; s += gridDim.x) sample_one(a, s, sm);
}

int resident_ctas() {
    static int cached = 0;
    if (cached) return cached;
    int dev = 0, sms = 0, per = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 148;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (cudaFuncSetAttribute(sample_rows_k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(SampSmem)) !=
        cudaSuccess)
        return 148;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, sample_rows_k, ST, sizeof(SampSmem));
    cached = std::max(1, sms) * std::max(1, per);
    return cached;
}

bool needs_lazy_sort(int V, const SampleParams &cfg) {
    if (cfg.greedy) return false;
    const uint64_t keep = (cfg.top_k == 0 || cfg.top_k > (uint64_t)V) ? (uint64_t)V : cfg.top_k;
    return keep > (uint64_t)CH;
}

}  // namespace

size_t sample_ws_bytes(int S, int V, SampleParams cfg, size_t budget) {
    if (S <= 0 || V <= 0 || !needs_lazy_sort(V, cfg)) return 0;
    const size_t per = (size_t)2 * V * sizeof(uint64_t);
    size_t ctas = std::min<size_t>((size_t)S, (size_t)resident_ctas());
    if (budget) ctas = std::max<size_t>(1, std::min(ctas, budget / per));
    return ctas * per;
}

cudaError_t collect_tokens(const uint32_t *tok, uint32_t *out, int S, int n_new, int *column, cudaStream_t st) {
    if (S <= 0) return cudaSuccess;
    collect_tokens_k<<<(S + 255) / 256, 256, 0, st>>>(tok, out, S, n_new, column);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    collect_next_k<<<1, 1, 0, st>>>(column);
    return cudaGetLastError();
}

cudaError_t sample_pen_bitmap(const uint32_t *history, const uint32_t *history_len, int history_stride,
                              SampleParams cfg, int S, int V, uint32_t *bits, int words, cudaStream_t st) {
    if (S <= 0 || words <= 0) return cudaSuccess;
    const uint64_t window = (history && isfinite(cfg.rep_penalty) && cfg.rep_penalty > 1.0f) ? cfg.rep_window : 0;
    if (!history || !history_len || window == 0) return cudaMemsetAsync(bits, 0, (size_t)S * words * 4, st);
    pen_bitmap_k<<<S, 128, 0, st>>>(history, history_len, history_stride, window, V, bits, words);
    return cudaGetLastError();
}

cudaError_t sample_rows(float *logits, int S, int V, SampleParams cfg, const uint32_t *history,
                        const uint32_t *history_len, int history_stride, uint64_t *rng, uint32_t *out, int *err,
                        void *ws, size_t ws_bytes, cudaStream_t st, const SamplePrepared *prep) {
    if (S <= 0 || V <= 0) return cudaSuccess;
    static bool attr_set = false;
    if (!attr_set) {
        cudaError_t e = cudaFuncSetAttribute(sample_rows_k, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)sizeof(SampSmem));
        if (e != cudaSuccess) return e;
        attr_set = true;
    }
    int grid = std::min(S, resident_ctas());
    SampleArgs a{logits, S, V, cfg, history, history_len, history_stride, rng, out, err, nullptr, 0,
                 prep ? prep->max : nullptr, prep ? prep->pinf : nullptr, prep ? prep->parts : 0};
    if (needs_lazy_sort(V, cfg)) {
        const size_t per = (size_t)2 * V * sizeof(uint64_t);
        const size_t fit = ws ? ws_bytes / per : 0;
        if (fit == 0) return cudaErrorInvalidValue;
        grid = (int)std::min<size_t>((size_t)grid, fit);
        a.ws = (uint64_t *)ws;
        a.ws_keys = (size_t)V;
    }
    sample_rows_k<<<grid, ST, sizeof(SampSmem), st>>>(a);
    return cudaGetLastError();
}

}  // namespace nk
