// tc_gemm.cu -- tensor-core projections for sm_100a: C = epilogue(A . W^T)
// in f32 accuracy with 3xTF32 on tcgen05.
//
// Split: a = a_hi + a_lo with a_hi = tf32(a), a_lo = tf32(a - a_hi) (the
// error-corrected TF32 product of Ootomo & Yokota 2022, "3xTF32" in
// CUTLASS); A.W^T = A_hi.W_hi^T + A_hi.W_lo^T + A_lo.W_hi^T, dropping the
// A_lo.W_lo^T term (~2^-22 relative).  Weights are split once at load; the
// activation operand pair is written by the kernel that produces the
// activation (RMSNorm, the SSM update, the SwiGLU epilogue, the prefill
// passes), and gemm_tn splits both operands with one transposing pass.
//
// Kernel structure: persistent, at most one CTA per SM slot (BN = 256: one
// per SM; BN = 128: two), each walking 128 x BN output tiles in steps of the
// grid size, n fastest; 384 threads:
//   warp 0      TMA producer: K-blocks of 16 f32 (one 64-byte swizzle row)
//               for A_hi, A_lo, W_hi, W_lo into a 4-stage (BN 256) or
//               3-stage (BN 128) smem ring (cp.async.bulk.tensor, 64B
//               swizzle, zero fill out of bounds).  It runs on into the next
//               tile's K-blocks while the epilogue drains the current one;
//   warp 1      TMEM allocator and MMA issuer: per K-block, 2 k-steps x 3
//               tcgen05.mma.cta_group::1.kind::tf32 (M=128, N=BN, K=8):
//               hi*hi into one f32 TMEM accumulator, hi*lo and lo*hi into a
//               second one; tcgen05.commit frees the stage, and after the
//               last K-block signals the epilogue.  The tensor core
//               truncates when it adds into an accumulator, so the error of a
//               chain grows with its length; keeping the small correction
//               products out of the main chain makes it three times shorter,
//               and the epilogue adds the two chains in round-to-nearest f32;
//   warps 4-11  epilogue, two warpgroups each draining half of the tile's
//               columns: tcgen05.ld 32 columns at a time (lane = row), bias,
//               residual add, store (or the first maximum of its columns);
//               then they hand the accumulators back to the MMA warp.
// Every mbarrier wait is bounded (~1 s of %globaltimer); on expiry the kernel
// records an error code, every role leaves its loop, TMEM is freed and the
// CTA exits -- the host reports the code instead of the GPU hanging.
// No TMA multicast is used anywhere.

#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdio>
#include <mutex>

#include "nk_common.cuh"
#include "nk_tc.h"

namespace nk {

namespace {

// BK = 16 f32 = one 64-byte swizzle row.  Tile width BN is 256 (one CTA per
// SM, 4 stages of 48 KiB, 512 TMEM columns) or 128 (two CTAs per SM, 3
// stages of 32 KiB, 256 TMEM columns each, so one CTA's epilogue overlaps the
// other's main loop and small grids still cover every SM).
constexpr int BM = 128, BK = 16;
// Rows up to which projections whose 128-wide tiles fit one wave are split
// along K (decode of up to 2048 streams; measured at the headline widths, ms
// per step against stream-K 256-wide tiles: 6.2 vs 7.7 at 1024 streams,
// 9.73 vs 10.0-10.2 at 2048).
constexpr int SPLIT_MAX_M = 2048;
constexpr int ROWRED_COLS = 1024; // columns per partial of the split-K argmax / sampling reduction
constexpr int SWIZZLE_BYTES = BK * 4;                       // 64
constexpr int ATOM_BYTES = 8 * SWIZZLE_BYTES;               // 8 rows: 512
constexpr int A_BYTES = BM * BK * 4;                       // 8 KiB
// Warp roles: 0 TMA producer, 1 TMEM allocator + MMA issuer, 2-3 idle,
// 4..11 epilogue (two warpgroups, each draining half the tile's columns).
constexpr int EPI_WARPS = 8;
constexpr int THREADS = (4 + EPI_WARPS) * 32;
constexpr uint64_t WAIT_NS = 1000000000ull;  // bound of every mbarrier wait

template <int BN>
struct Tile {
    static constexpr int B_BYTES = BN * BK * 4;
    static constexpr int STAGE_BYTES = 2 * A_BYTES + 2 * B_BYTES;
    static constexpr int STAGES = BN == 256 ? 4 : 3;
    // BN = 256: a 32 x 32 f32 transpose buffer per epilogue warp, so the
    // epilogue reads and writes whole 128-byte row segments.
    static constexpr int EPI_BYTES = BN == 256 ? EPI_WARPS * 32 * 32 * 4 : 0;
    static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + EPI_BYTES + 1024 + 256;
    static constexpr int CTAS_PER_SM = BN == 256 ? 1 : 2;
    // Two f32 accumulators of BN columns: the hi*hi products and the two
    // small correction products are summed in separate TMEM chains.
    static constexpr uint32_t TMEM_COLS = 2 * BN;
    // Instruction descriptor: D f32, A/B tf32, both K-major, M=128, N=BN.
    static constexpr uint32_t IDESC = (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(BN >> 3) << 17) |
                                      ((uint32_t)(BM >> 4) << 24);
};

struct TcArgs {
    float *C;
    int ldc;
    int M, N, K;
    const float *bias;
    const float *R;
    int ldr;
    float *best_val;     // argmax mode when non-null: per-row best of this tile
    uint32_t *best_idx;
    int n_tiles;
    int *err;
    int swiglu_H;        // SwiGLU mode when > 0 (interleaved operand)
    float *C_lo;         // SwiGLU mode: lo half of the operand pair, or null for f32
    // Tiles [0, sk_t0) run whole, tile c + w gridDim.x on CTA c.  With
    // skb > 0 (256-wide store and SwiGLU modes) the remaining tiles -- the
    // partial last wave -- are spread by K-block (stream-K): CTA c then owns
    // K-blocks [c skb, (c+1) skb) of their tile-major K-block sequence.  A
    // tile cut at a range boundary is finished by the CTA that holds its
    // first K-blocks: the CTAs holding the rest write their partial tile to
    // ws slot c and set flags[c]; the finisher adds the slots in order.  A
    // finishing piece is the last piece of its CTA and a partial piece the
    // first of its CTA's stream-K range, so no CTA waits on work queued
    // behind a wait.  Whole waves stay data-parallel so that concurrently
    // running CTAs share A rows in L2.
    int skb;
    int sk_t0;
    float *ws;
    int *flags;
    int l2hints;  // 1: weights loaded evict-last, staged outputs stored evict-first
    // Sampling preparation of a logits projection (temperature > 0; store
    // mode, no bias / residual, whole tiles): C = pen(acc) / temperature,
    // pen = the repetition penalty where bit (row, column) of pen_bits
    // ([M][pen_words] u32) is set; per row and half tile the maximum of the
    // finite outputs and the number of +inf ones go to prep_max / prep_pinf
    // (slot layout of the argmax partials).
    float temperature;
    float rep_penalty;
    const uint32_t *pen_bits;
    int pen_words;
    float *prep_max;
    uint32_t *prep_pinf;
    // Bound of the stream-K hand-off waits (ns), and a test control: when
    // set, no CTA publishes its partial tiles, so every finisher's wait runs
    // out and reports code 121 (the failure path, exercised without a fault).
    uint64_t handoff_wait_ns;
    int withhold_publish;
    // Split-K (splits > 0; 128-wide tiles, store and SwiGLU modes, one row
    // of tiles): piece g is K-blocks [s * kps, (s + 1) * kps) of tile
    // g / splits, s = g % splits, and its raw sum goes to
    // split_part[(s * M + row) * N + col]; splitk_reduce_k then adds the
    // pieces in split order and applies the epilogue.
    int splits;
    int kps;
    float *split_part;
    // RMSNorm folded into the neighbouring projections (tensor.rs:298-312):
    // a consumer (rs_parts != null) multiplies each accumulator row by
    // 1 / sqrt(ms / rs_d + rs_eps), ms = the sum of rs_parts[row][0 ..
    // rs_nparts) in order; its A operand is the split of x * gain.  A
    // producer (store mode, nx_hi != null) also writes that operand for the
    // next projection, nx = split(x * nx_gain) ([M, N]), and per row and
    // 32-column chunk the sum of x^2 into nx_ss[row * nx_nparts + chunk].
    const float *rs_parts;
    int rs_nparts;
    int rs_d;
    float rs_eps;
    float *nx_hi, *nx_lo;
    const float *nx_gain;
    float *nx_ss;
    int nx_nparts;
    // 1: the 256-wide store and SwiGLU epilogues write each 32 x 32 chunk
    // with a TMA bulk store from the warp's staging buffer (mapC / mapClo),
    // so the stores drain while the next tile's MMAs run.
    int tma_store;
    // Tile order: tiles go in groups of group_n column blocks (0: one group),
    // column blocks fastest within a group, so the CTAs running at once read
    // one group's weight columns, which stay in L2 from wave to wave.
    int group_n;
};

// Tile t -> (row block tm, column block tn) in the grouped order.
__device__ __forceinline__ void tile_coords(int t, int n_tiles_n, int m_tiles, int group_n, int &tm, int &tn) {
    if (group_n <= 0 || group_n >= n_tiles_n) {
        tm = t / n_tiles_n;
        tn = t - tm * n_tiles_n;
        return;
    }
    const int per_group = group_n * m_tiles;
    const int g = t / per_group, r = t - g * per_group;
    const int width = min(group_n, n_tiles_n - g * group_n);
    tm = r / width;
    tn = g * group_n + (r - tm * width);
}

// 1 / sqrt(ms / d + eps) of a row from its partial sums of squares (1 when
// the projection's input was normalised already).
__device__ __forceinline__ float folded_row_scale(const TcArgs &p, int row) {
    if (!p.rs_parts || row >= p.M) return 1.0f;
    const float *pp = p.rs_parts + (size_t)row * p.rs_nparts;
    float ms = 0.0f;
    for (int i = 0; i < p.rs_nparts; ++i) ms = ms + pp[i];
    return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ms, (float)p.rs_d), p.rs_eps)));
}

// infer.rs:239-247 then 253-256 for one logit: the repetition penalty when
// the token is in the history window, then the temperature division.
__device__ __forceinline__ float sample_prep(float x, bool penalised, const TcArgs &p) {
    if (penalised) x = x > 0.0f ? __fdiv_rn(x, p.rep_penalty) : __fmul_rn(x, p.rep_penalty);
    return __fdiv_rn(x, p.temperature);
}

// One piece of a CTA's work: tile t, K-blocks [kb0, kb1).  np < 0: a partial
// piece (written to ws slot blockIdx.x); np == 0: the whole tile; np > 0:
// the tile's first K-blocks, finished after adding slots blockIdx.x + 1 ..
// blockIdx.x + np.
struct Piece {
    int t, kb0, kb1, np, split;
};

__device__ __forceinline__ bool next_piece(const TcArgs &p, int n_tiles, int kblocks, int &cursor, Piece &pc) {
    const int G = gridDim.x, c = blockIdx.x;
    if (p.splits > 0) {
        const long g = (long)c + (long)cursor * G;
        if (g >= (long)n_tiles * p.splits) return false;
        ++cursor;
        pc.t = (int)(g / p.splits);
        pc.split = (int)(g % p.splits);
        pc.kb0 = pc.split * p.kps;
        pc.kb1 = min(kblocks, pc.kb0 + p.kps);
        pc.np = 0;
        return true;
    }
    pc.split = -1;
    const int dp_tiles = p.skb > 0 ? p.sk_t0 : n_tiles;
    const int n_dp = c < dp_tiles ? (dp_tiles - c + G - 1) / G : 0;
    if (cursor < n_dp) {
        pc.t = c + cursor * G;
        ++cursor;
        pc.kb0 = 0;
        pc.kb1 = kblocks;
        pc.np = 0;
        return true;
    }
    if (p.skb <= 0) return false;
    const long total = (long)(n_tiles - p.sk_t0) * kblocks;
    const long begin = (long)c * p.skb;
    const long end = begin + p.skb < total ? begin + p.skb : total;
    const long pos = begin + (cursor - n_dp);
    if (pos >= end) return false;
    const int tl = (int)(pos / kblocks);
    pc.t = p.sk_t0 + tl;
    pc.kb0 = (int)(pos - (long)tl * kblocks);
    pc.kb1 = (int)((long)pc.kb0 + (end - pos) < kblocks ? (long)pc.kb0 + (end - pos) : kblocks);
    cursor += pc.kb1 - pc.kb0;
    if (pc.kb0 == 0 && pc.kb1 == kblocks) pc.np = 0;
    else if (pc.kb0 > 0) pc.np = -1;
    else pc.np = (kblocks - pc.kb1 + p.skb - 1) / p.skb;
    return true;
}

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ uint64_t globaltimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

// Bounded wait for the phase of parity `parity` to complete.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
    uint32_t done = 0;
    asm volatile(
        "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
        : "=r"(done) : "r"(bar), "r"(parity) : "memory");
    if (done) return true;
    const uint64_t t0 = globaltimer();
    for (;;) {
        asm volatile(
            "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
            : "=r"(done) : "r"(bar), "r"(parity) : "memory");
        if (done) return true;
        if (globaltimer() - t0 > WAIT_NS) return false;
    }
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap *map, uint32_t bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
        ::"r"(dst), "l"((uint64_t)map), "r"(bar), "r"(x), "r"(y)
        : "memory");
}

// The same load with an L2 cache policy (createpolicy) attached.
__device__ __forceinline__ void tma_load_2d_hint(uint32_t dst, const CUtensorMap *map, uint32_t bar, int x, int y,
                                                 uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, {%3, %4}], [%2], %5;"
        ::"r"(dst), "l"((uint64_t)map), "r"(bar), "r"(x), "r"(y), "l"(policy)
        : "memory");
}

// L2 policies: weights are re-read by every row tile and should stay; the
// epilogue's outputs stream out and should leave first.
__device__ __forceinline__ uint64_t policy_evict_last() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}
__device__ __forceinline__ uint64_t policy_evict_first() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}
__device__ __forceinline__ void st_stream(float *p, float v, uint64_t pol) {
    asm volatile("st.global.L2::cache_hint.f32 [%0], %1, %2;" ::"l"(p), "f"(v), "l"(pol) : "memory");
}

// Bulk tensor store of a 32 x 32 f32 box (128-byte swizzle, the staging
// buffer's layout) at column x (a multiple of 32: 16-byte aligned) and row y
// (>= 0); rows and columns past the tensor are not written.
__device__ __forceinline__ void tma_store_box(const CUtensorMap *map, uint32_t src, int x, int y, uint64_t pol) {
    asm volatile(
        "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group.L2::cache_hint [%0, {%2, %3}], [%1], %4;"
        ::"l"((uint64_t)map), "r"(src), "r"(x), "r"(y), "l"(pol)
        : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Wait until this thread's bulk stores have read their shared-memory source.
__device__ __forceinline__ void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// Wait until this thread's bulk stores are complete.
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// K-major operand with the 64-byte swizzle (layout type 4): rows of 64 bytes,
// 8-row groups ATOM_BYTES apart.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr) {
    return (uint64_t)((addr >> 4) & 0x3FFFu) | (1ull << 16) | ((uint64_t)(ATOM_BYTES >> 4) << 32) | (1ull << 46) |
           (4ull << 61);
}

__device__ __forceinline__ void mma_tf32(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc,
                                         uint32_t accumulate) {
    asm volatile(
        "{ .reg .pred p; setp.ne.b32 p, %4, 0; tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p; }"
        ::"r"(d_tmem), "l"(a), "l"(b), "r"(idesc), "r"(accumulate));
}

__device__ __forceinline__ void mma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
          "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
          "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
          "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
          "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// One epilogue warp's share of a tile: TMEM lanes q*32 .. q*32+31 (output
// rows m0 + q*32 + lane), TMEM columns [c_begin, c_end) (output columns
// n0 + c).  Store mode writes C (+bias, +residual); SwiGLU mode writes the
// gated product; argmax mode folds the columns into (best, best_n).
// Stream-K (stg only): part_out != null writes this piece's partial tile
// ([BM][BN] raw sums, no bias / residual / SwiGLU) instead of C; parts !=
// null adds the nparts partial tiles at parts, parts + BM*BN, ... in order
// before the bias and residual (or SwiGLU).
// Kernel variants: the general projection (store / SwiGLU / argmax
// epilogues, stream-K), the logits projection with the sampling epilogue,
// and split-K pieces; separate instantiations keep each one's registers.
constexpr int MODE_GENERAL = 0, MODE_PREP = 1, MODE_SPLIT = 2, MODE_FOLD = 3, MODE_TMA = 4;
// MODE_TMA: the general projection whose 256-wide store and SwiGLU
// epilogues write through bulk tensor stores (stream-K partial tiles still
// take the staged transposed writes).
// Variants that carry the folded RMSNorm (its row scale, and the next
// projection's operand and sums of squares).
constexpr bool mode_folds(int mode) { return mode == MODE_PREP || mode == MODE_FOLD; }

template <int BN, int MODE = MODE_GENERAL>
__device__ __forceinline__ void epilogue_cols(const TcArgs &p, uint32_t tmem, int q, int lane, int m0, int n0,
                                              int c_begin, int c_end, bool argmax_mode, bool vec, float &best,
                                              uint32_t &best_n, float *stg, const float *parts = nullptr,
                                              int nparts = 0, float *part_out = nullptr, int split = -1,
                                              const CUtensorMap *mapC = nullptr, const CUtensorMap *mapClo = nullptr) {
    const int row = m0 + q * 32 + lane;
    if constexpr (MODE == MODE_SPLIT) {
        // Split-K piece: the raw sum of both accumulator chains, rows < M.
        for (int c0 = c_begin; c0 < c_end; c0 += 32) {
            if (n0 + c0 >= p.N) break;  // warp-uniform
            float v[32], corr[32];
            tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)c0, v);
            tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(BN + c0), corr);
            if (row < p.M) {
                float *dst = p.split_part + ((size_t)split * p.M + row) * p.N + n0 + c0;
                const bool full = n0 + c0 + 32 <= p.N && (p.N & 3) == 0;
#pragma unroll
                for (int j = 0; j < 32; j += 4) {
                    if (full) {
                        *reinterpret_cast<float4 *>(dst + j) =
                            make_float4(v[j] + corr[j], v[j + 1] + corr[j + 1], v[j + 2] + corr[j + 2],
                                        v[j + 3] + corr[j + 3]);
                    } else {
#pragma unroll
                        for (int jj = 0; jj < 4; ++jj)
                            if (n0 + c0 + j + jj < p.N) dst[j + jj] = v[j + jj] + corr[j + jj];
                    }
                }
            }
        }
        return;
    }
    constexpr bool FOLD = mode_folds(MODE);
    float rscale = 1.0f;  // this lane's row: the folded RMSNorm scale
    if constexpr (FOLD) rscale = folded_row_scale(p, row);
    if ((MODE == MODE_TMA || MODE == MODE_PREP) && stg && !argmax_mode && p.tma_store && !part_out) {
        // Each 32 x 32 chunk is finished in registers (lane = row: both
        // accumulator chains, then the stream-K partials in order, the bias,
        // the residual, or the SwiGLU) and written by one bulk tensor store
        // from this warp's staging buffer, whose float4 slots are XOR-swizzled
        // by row exactly as the 128-byte TMA swizzle lays out a 32-float box.
        // The warp waits only until the previous store has read the buffer.
        const uint64_t pol_out = policy_evict_first();
        const int rbase = m0 + q * 32;
        const uint32_t stg_s = smem_u32(stg);
        auto stage_row = [&](const float (&o)[32]) {
            if (lane == 0) bulk_wait_read();
            __syncwarp();
#pragma unroll
            for (int c4 = 0; c4 < 8; ++c4)
                *reinterpret_cast<float4 *>(stg + lane * 32 + 4 * (c4 ^ (lane & 7))) =
                    make_float4(o[4 * c4], o[4 * c4 + 1], o[4 * c4 + 2], o[4 * c4 + 3]);
            fence_async_smem();
            __syncwarp();
        };
        if (p.swiglu_H) {
            for (int c0 = c_begin; c0 < c_end; c0 += 64) {
                if (n0 + c0 >= p.N) break;  // warp-uniform
                const int j0 = (n0 + c0) >> 1;
                const uint32_t ta = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)c0;
                float sv[32];
#pragma unroll
                for (int sub = 0; sub < 32; sub += 16) {
                    float a[16], b[16], t[16];
                    tmem_ld16(ta + sub, a);
                    tmem_ld16(ta + BN + sub, t);
#pragma unroll
                    for (int jj = 0; jj < 16; ++jj) a[jj] = a[jj] + t[jj];
                    tmem_ld16(ta + 32 + sub, b);
                    tmem_ld16(ta + BN + 32 + sub, t);
#pragma unroll
                    for (int jj = 0; jj < 16; ++jj) b[jj] = b[jj] + t[jj];
                    for (int ks = 0; ks < nparts; ++ks) {
                        const float *pt = parts + (size_t)ks * BM * BN + (size_t)(q * 32 + lane) * BN + c0 + sub;
#pragma unroll
                        for (int jj = 0; jj < 16; jj += 4) {
                            const float4 pa = *reinterpret_cast<const float4 *>(pt + jj);
                            const float4 pb = *reinterpret_cast<const float4 *>(pt + 32 + jj);
                            a[jj] = a[jj] + pa.x; a[jj + 1] = a[jj + 1] + pa.y;
                            a[jj + 2] = a[jj + 2] + pa.z; a[jj + 3] = a[jj + 3] + pa.w;
                            b[jj] = b[jj] + pb.x; b[jj + 1] = b[jj + 1] + pb.y;
                            b[jj + 2] = b[jj + 2] + pb.z; b[jj + 3] = b[jj + 3] + pb.w;
                        }
                    }
                    if constexpr (FOLD) {
#pragma unroll
                        for (int jj = 0; jj < 16; ++jj) {
                            a[jj] = a[jj] * rscale;
                            b[jj] = b[jj] * rscale;
                        }
                    }
                    const int j = j0 + sub;
#pragma unroll
                    for (int jj = 0; jj < 16; ++jj)
                        sv[sub + jj] = silu(a[jj] + p.bias[j + jj]) * (b[jj] + p.bias[p.swiglu_H + j + jj]);
                }
                if (p.C_lo) {
                    float hv[32];
#pragma unroll
                    for (int jj = 0; jj < 32; ++jj) {
                        hv[jj] = tf32_round(sv[jj]);
                        sv[jj] = tf32_round(sv[jj] - hv[jj]);
                    }
                    stage_row(hv);
                    if (lane == 0) {
                        tma_store_box(mapC, stg_s, j0, rbase, pol_out);
                        bulk_commit();
                    }
                    stage_row(sv);
                    if (lane == 0) {
                        tma_store_box(mapClo, stg_s, j0, rbase, pol_out);
                        bulk_commit();
                    }
                } else {
                    stage_row(sv);
                    if (lane == 0) {
                        tma_store_box(mapC, stg_s, j0, rbase, pol_out);
                        bulk_commit();
                    }
                }
            }
            return;
        }
        for (int c0 = c_begin; c0 < c_end; c0 += 32) {
            if (n0 + c0 >= p.N) break;  // warp-uniform
            const int nb = n0 + c0;
            float v[32], corr[32];
            tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)c0, v);
            tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(BN + c0), corr);
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = v[j] + corr[j];
            if constexpr (MODE == MODE_PREP) {
                const uint32_t pw =
                    (p.pen_bits && row < p.M) ? p.pen_bits[(size_t)row * p.pen_words + (nb >> 5)] : 0u;
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    const float y = sample_prep(v[j] * rscale, (pw >> j) & 1u, p);
                    v[j] = y;
                    if (nb + j < p.N) {
                        if (y == INFINITY) ++best_n;
                        if (isfinite(y) && y > best) best = y;
                    }
                }
            } else {
                for (int ks = 0; ks < nparts; ++ks) {
                    const float *pt = parts + (size_t)ks * BM * BN + (size_t)(q * 32 + lane) * BN + c0;
#pragma unroll
                    for (int j = 0; j < 32; j += 4) {
                        const float4 pv = *reinterpret_cast<const float4 *>(pt + j);
                        v[j] = v[j] + pv.x;
                        v[j + 1] = v[j + 1] + pv.y;
                        v[j + 2] = v[j + 2] + pv.z;
                        v[j + 3] = v[j + 3] + pv.w;
                    }
                }
                if constexpr (FOLD) {
#pragma unroll
                    for (int j = 0; j < 32; ++j) v[j] = v[j] * rscale;
                }
                if (p.bias) {
#pragma unroll
                    for (int j = 0; j < 32; ++j)
                        if (nb + j < p.N) v[j] = v[j] + p.bias[nb + j];
                }
                if (p.R && row < p.M) {
                    const float *rr = p.R + (size_t)row * p.ldr + nb;
                    if (vec && nb + 32 <= p.N) {
#pragma unroll
                        for (int j = 0; j < 32; j += 4) {
                            const float4 r4 = *reinterpret_cast<const float4 *>(rr + j);
                            v[j] = r4.x + v[j];
                            v[j + 1] = r4.y + v[j + 1];
                            v[j + 2] = r4.z + v[j + 2];
                            v[j + 3] = r4.w + v[j + 3];
                        }
                    } else {
#pragma unroll
                        for (int j = 0; j < 32; ++j)
                            if (nb + j < p.N) v[j] = rr[j] + v[j];
                    }
                }
            }
            stage_row(v);
            if (lane == 0) {
                tma_store_box(mapC, stg_s, nb, rbase, pol_out);
                bulk_commit();
            }
        }
        return;
    }
    if (stg && !argmax_mode) {
        const uint64_t pol_out = policy_evict_first();
        // Transpose each 32 x 32 chunk through this warp's shared buffer
        // (float4 slots XOR-swizzled by row: conflict-free both ways), then
        // lane = column, so every load and store is one 128-byte row segment.
        const int rbase = m0 + q * 32;
        if (MODE != MODE_TMA && p.swiglu_H && !part_out) {
            // 64-column blocks: 32 gate columns, then the 32 value columns of
            // the same channels; both accumulator chains summed first.
            for (int c0 = c_begin; c0 < c_end; c0 += 64) {
                if (n0 + c0 >= p.N) break;  // warp-uniform
                const int j0 = (n0 + c0) >> 1;
                const uint32_t ta = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)c0;
#pragma unroll
                for (int sub = 0; sub < 32; sub += 16) {
                    float a[16], b[16], t[16];
                    tmem_ld16(ta + sub, a);
                    tmem_ld16(ta + BN + sub, t);
#pragma unroll
                    for (int jj = 0; jj < 16; ++jj) a[jj] = a[jj] + t[jj];
                    tmem_ld16(ta + 32 + sub, b);
                    tmem_ld16(ta + BN + 32 + sub, t);
#pragma unroll
                    for (int jj = 0; jj < 16; ++jj) b[jj] = b[jj] + t[jj];
                    for (int ks = 0; ks < nparts; ++ks) {
                        const float *pt = parts + (size_t)ks * BM * BN + (size_t)(q * 32 + lane) * BN + c0 + sub;
#pragma unroll
                        for (int jj = 0; jj < 16; jj += 4) {
                            const float4 pa = *reinterpret_cast<const float4 *>(pt + jj);
                            const float4 pb = *reinterpret_cast<const float4 *>(pt + 32 + jj);
                            a[jj] = a[jj] + pa.x; a[jj + 1] = a[jj + 1] + pa.y;
                            a[jj + 2] = a[jj + 2] + pa.z; a[jj + 3] = a[jj + 3] + pa.w;
                            b[jj] = b[jj] + pb.x; b[jj + 1] = b[jj + 1] + pb.y;
                            b[jj + 2] = b[jj + 2] + pb.z; b[jj + 3] = b[jj + 3] + pb.w;
                        }
                    }
                    if constexpr (FOLD) {
#pragma unroll
                        for (int jj = 0; jj < 16; ++jj) {
                            a[jj] = a[jj] * rscale;
                            b[jj] = b[jj] * rscale;
                        }
                    }
                    const int j = j0 + sub;
#pragma unroll
                    for (int jj = 0; jj < 16; jj += 4) {
                        float4 sv;
                        sv.x = silu(a[jj + 0] + p.bias[j + jj + 0]) * (b[jj + 0] + p.bias[p.swiglu_H + j + jj + 0]);
                        sv.y = silu(a[jj + 1] + p.bias[j + jj + 1]) * (b[jj + 1] + p.bias[p.swiglu_H + j + jj + 1]);
                        sv.z = silu(a[jj + 2] + p.bias[j + jj + 2]) * (b[jj + 2] + p.bias[p.swiglu_H + j + jj + 2]);
                        sv.w = silu(a[jj + 3] + p.bias[j + jj + 3]) * (b[jj + 3] + p.bias[p.swiglu_H + j + jj + 3]);
                        const int c4 = (sub + jj) >> 2;
                        *reinterpret_cast<float4 *>(stg + lane * 32 + 4 * (c4 ^ (lane & 7))) = sv;
                    }
                }
                __syncwarp();
                const int jc = j0 + lane;
#pragma unroll 8
                for (int r = 0; r < 32; ++r) {
                    const int grow = rbase + r;
                    const float sv = stg[r * 32 + 4 * ((lane >> 2) ^ (r & 7)) + (lane & 3)];
                    if (grow < p.M) {
                        if (p.C_lo) {
                            const float h = tf32_round(sv);
                            if (p.l2hints) {
                                st_stream(p.C + (size_t)grow * p.ldc + jc, h, pol_out);
                                st_stream(p.C_lo + (size_t)grow * p.ldc + jc, tf32_round(sv - h), pol_out);
                            } else {
                                p.C[(size_t)grow * p.ldc + jc] = h;
                                p.C_lo[(size_t)grow * p.ldc + jc] = tf32_round(sv - h);
                            }
                        } else {
                            if (p.l2hints) st_stream(p.C + (size_t)grow * p.ldc + jc, sv, pol_out);
                            else p.C[(size_t)grow * p.ldc + jc] = sv;
                        }
                    }
                }
                __syncwarp();
            }
            return;
        }
        for (int c0 = c_begin; c0 < c_end; c0 += 32) {
            if (n0 + c0 >= p.N) break;  // warp-uniform
            float v[32], corr[32];
            tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)c0, v);
            tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(BN + c0), corr);
            if constexpr (MODE == MODE_PREP) {
                // lane = row here: penalty bits of 32 columns in one word,
                // the row's running maximum and +inf count in registers.
                const int nb = n0 + c0;
                const uint32_t pw =
                    (p.pen_bits && row < p.M) ? p.pen_bits[(size_t)row * p.pen_words + (nb >> 5)] : 0u;
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    const float y = sample_prep((v[j] + corr[j]) * rscale, (pw >> j) & 1u, p);
                    v[j] = y;
                    corr[j] = 0.0f;
                    if (nb + j < p.N) {
                        if (y == INFINITY) ++best_n;
                        if (isfinite(y) && y > best) best = y;
                    }
                }
            }
#pragma unroll
            for (int c4 = 0; c4 < 8; ++c4) {
                float4 o;
                o.x = v[4 * c4 + 0] + corr[4 * c4 + 0];
                o.y = v[4 * c4 + 1] + corr[4 * c4 + 1];
                o.z = v[4 * c4 + 2] + corr[4 * c4 + 2];
                o.w = v[4 * c4 + 3] + corr[4 * c4 + 3];
                *reinterpret_cast<float4 *>(stg + lane * 32 + 4 * (c4 ^ (lane & 7))) = o;
            }
            __syncwarp();
            const int col = n0 + c0 + lane;
            const bool cok = col < p.N;
            if (MODE == MODE_TMA || part_out) {  // (MODE_TMA reaches here only for partial tiles)
#pragma unroll 8
                for (int r = 0; r < 32; ++r)
                    part_out[(size_t)(q * 32 + r) * BN + c0 + lane] = stg[r * 32 + 4 * ((lane >> 2) ^ (r & 7)) + (lane & 3)];
                __syncwarp();
                continue;
            }
            if (parts) {
                for (int ks = 0; ks < nparts; ++ks) {
                    const float *pt = parts + (size_t)ks * BM * BN + (size_t)(q * 32) * BN + c0 + lane;
                    float pv[32];
#pragma unroll
                    for (int r = 0; r < 32; ++r) pv[r] = pt[(size_t)r * BN];
#pragma unroll
                    for (int r = 0; r < 32; ++r) {
                        float *sp = stg + r * 32 + 4 * ((lane >> 2) ^ (r & 7)) + (lane & 3);
                        *sp = *sp + pv[r];
                    }
                }
            }
            const float bcol = (p.bias && cok) ? p.bias[col] : 0.0f;
            // All 32 residual rows are requested before any is used.
            float rv[32];
            if (p.R) {
#pragma unroll
                for (int r = 0; r < 32; ++r)
                    rv[r] = (rbase + r < p.M && cok) ? p.R[(size_t)(rbase + r) * p.ldr + col] : 0.0f;
            }
            const float gcol = (FOLD && p.nx_hi && cok) ? p.nx_gain[col] : 0.0f;
#pragma unroll
            for (int r = 0; r < 32; ++r) {
                const int grow = rbase + r;
                float o = stg[r * 32 + 4 * ((lane >> 2) ^ (r & 7)) + (lane & 3)];
                if constexpr (MODE == MODE_FOLD) {  // (the sampling epilogue scaled in the first stage)
                    if (p.rs_parts) o = o * __shfl_sync(0xffffffffu, rscale, r);
                }
                if (grow < p.M && cok) {
                    if (p.bias) o = o + bcol;
                    if (p.R) o = rv[r] + o;
                    if (p.l2hints) st_stream(p.C + (size_t)grow * p.ldc + col, o, pol_out);
                    else p.C[(size_t)grow * p.ldc + col] = o;
                }
                if constexpr (FOLD) {
                    if (p.nx_hi) {
                        // The next projection's operand x * gain, and the
                        // row's sum of squares over these 32 columns.
                        const bool ok = grow < p.M && cok;
                        if (ok) {
                            const float y = o * gcol, h = tf32_round(y);
                            st_stream(p.nx_hi + (size_t)grow * p.N + col, h, pol_out);
                            st_stream(p.nx_lo + (size_t)grow * p.N + col, tf32_round(y - h), pol_out);
                        }
                        const float sq = warp_sum(ok ? o * o : 0.0f);
                        if (lane == 0 && grow < p.M) p.nx_ss[(size_t)grow * p.nx_nparts + ((n0 + c0) >> 5)] = sq;
                    }
                }
            }
            __syncwarp();
        }
        return;
    }
    // SwiGLU: 64-column blocks of (32 gate, 32 value) columns of the
    // same 32 channels; both accumulator chains summed first.
    for (int c0 = c_begin; p.swiglu_H && c0 < c_end; c0 += 64) {
        if (n0 + c0 >= p.N) break;  // warp-uniform
        const int j0 = (n0 + c0) >> 1;
        const uint32_t ta = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)c0;
#pragma unroll
        for (int sub = 0; sub < 32; sub += 16) {
            float a[16], b[16], t[16];
            tmem_ld16(ta + sub, a);
            tmem_ld16(ta + BN + sub, t);
#pragma unroll
            for (int jj = 0; jj < 16; ++jj) a[jj] = a[jj] + t[jj];
            tmem_ld16(ta + 32 + sub, b);
            tmem_ld16(ta + BN + 32 + sub, t);
#pragma unroll
            for (int jj = 0; jj < 16; ++jj) b[jj] = b[jj] + t[jj];
            if constexpr (FOLD) {
#pragma unroll
                for (int jj = 0; jj < 16; ++jj) {
                    a[jj] = a[jj] * rscale;
                    b[jj] = b[jj] * rscale;
                }
            }
            if (row < p.M) {
                const int j = j0 + sub;
                float *out = p.C + (size_t)row * p.ldc + j;
#pragma unroll
                for (int jj = 0; jj < 16; jj += 4) {
                    float4 sv;
                    sv.x = silu(a[jj + 0] + p.bias[j + jj + 0]) * (b[jj + 0] + p.bias[p.swiglu_H + j + jj + 0]);
                    sv.y = silu(a[jj + 1] + p.bias[j + jj + 1]) * (b[jj + 1] + p.bias[p.swiglu_H + j + jj + 1]);
                    sv.z = silu(a[jj + 2] + p.bias[j + jj + 2]) * (b[jj + 2] + p.bias[p.swiglu_H + j + jj + 2]);
                    sv.w = silu(a[jj + 3] + p.bias[j + jj + 3]) * (b[jj + 3] + p.bias[p.swiglu_H + j + jj + 3]);
                    if (p.C_lo) {
                        float4 h, l;
                        h.x = tf32_round(sv.x); l.x = tf32_round(sv.x - h.x);
                        h.y = tf32_round(sv.y); l.y = tf32_round(sv.y - h.y);
                        h.z = tf32_round(sv.z); l.z = tf32_round(sv.z - h.z);
                        h.w = tf32_round(sv.w); l.w = tf32_round(sv.w - h.w);
                        *reinterpret_cast<float4 *>(out + jj) = h;
                        *reinterpret_cast<float4 *>(p.C_lo + (size_t)row * p.ldc + j + jj) = l;
                    } else {
                        *reinterpret_cast<float4 *>(out + jj) = sv;
                    }
                }
            }
        }
    }
    for (int c0 = c_begin; !p.swiglu_H && c0 < c_end; c0 += 32) {
        if (n0 + c0 >= p.N) break;  // warp-uniform
        float v[32], corr[32];
        tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)c0, v);
        tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(BN + c0), corr);
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = v[j] + corr[j];
        if constexpr (FOLD) {
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = v[j] * rscale;
        }
        const int nb = n0 + c0;
        if constexpr (MODE == MODE_PREP) {
            const uint32_t pw = (p.pen_bits && row < p.M) ? p.pen_bits[(size_t)row * p.pen_words + (nb >> 5)] : 0u;
#pragma unroll
            for (int j = 0; j < 32; ++j) {
                v[j] = sample_prep(v[j], (pw >> j) & 1u, p);
                if (nb + j < p.N) {
                    if (v[j] == INFINITY) ++best_n;
                    if (isfinite(v[j]) && v[j] > best) best = v[j];
                }
            }
        }
        if (argmax_mode) {
            // First strict maximum over this tile's columns, NaN skipped.
#pragma unroll
            for (int j = 0; j < 32; ++j) {
                float o = v[j];
                if (p.bias && nb + j < p.N) o = o + p.bias[nb + j];
                if (nb + j < p.N && !isnan(o) && o > best) {
                    best = o;
                    best_n = (uint32_t)(nb + j);
                }
            }
            continue;
        }
        if (FOLD && p.nx_hi) {
            // The stored x, the next projection's operand x * gain and the
            // row's sum of squares over these 32 columns (in column order).
            if (row < p.M) {
                float sq = 0.0f;
                for (int j = 0; j < 32; ++j) {
                    const int n = nb + j;
                    if (n < p.N) {
                        float o = v[j];
                        if (p.bias) o = o + p.bias[n];
                        if (p.R) o = p.R[(size_t)row * p.ldr + n] + o;
                        p.C[(size_t)row * p.ldc + n] = o;
                        const float y = o * p.nx_gain[n], h = tf32_round(y);
                        p.nx_hi[(size_t)row * p.N + n] = h;
                        p.nx_lo[(size_t)row * p.N + n] = tf32_round(y - h);
                        sq = sq + o * o;
                    }
                }
                p.nx_ss[(size_t)row * p.nx_nparts + (nb >> 5)] = sq;
            }
            continue;
        }
        if (row < p.M) {
            float *crow = p.C + (size_t)row * p.ldc;
            const float *rrow = p.R ? p.R + (size_t)row * p.ldr : nullptr;
            if (vec && nb + 32 <= p.N) {
#pragma unroll
                for (int j = 0; j < 32; j += 4) {
                    float4 o;
                    o.x = v[j + 0]; o.y = v[j + 1]; o.z = v[j + 2]; o.w = v[j + 3];
                    if (p.bias) {
                        const float4 b = *reinterpret_cast<const float4 *>(p.bias + nb + j);
                        o.x = o.x + b.x; o.y = o.y + b.y; o.z = o.z + b.z; o.w = o.w + b.w;
                    }
                    if (rrow) {
                        const float4 r = *reinterpret_cast<const float4 *>(rrow + nb + j);
                        o.x = r.x + o.x; o.y = r.y + o.y; o.z = r.z + o.z; o.w = r.w + o.w;
                    }
                    *reinterpret_cast<float4 *>(crow + nb + j) = o;
                }
            } else {
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    const int n = nb + j;
                    if (n < p.N) {
                        float o = v[j];
                        if (p.bias) o = o + p.bias[n];
                        if (rrow) o = rrow[n] + o;
                        crow[n] = o;
                    }
                }
            }
        }
    }
}

template <int BN, int MODE>
__global__ void __launch_bounds__(THREADS, Tile<BN>::CTAS_PER_SM)
tc_gemm_kernel(const __grid_constant__ CUtensorMap mapAh, const __grid_constant__ CUtensorMap mapAl,
               const __grid_constant__ CUtensorMap mapBh, const __grid_constant__ CUtensorMap mapBl,
               const __grid_constant__ CUtensorMap mapC, const __grid_constant__ CUtensorMap mapClo, TcArgs p) {
    using T = Tile<BN>;
    constexpr int STAGES = T::STAGES, STAGE_BYTES = T::STAGE_BYTES, B_BYTES = T::B_BYTES;
    constexpr uint32_t TMEM_COLS = T::TMEM_COLS, IDESC = T::IDESC;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    // 1024-byte aligned tile area (swizzle atoms must not straddle their period).
    uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    // full[S], empty[S], acc_full, acc_empty after the stages and transpose buffers
    uint64_t *bars = (uint64_t *)(smem + STAGES * STAGE_BYTES + T::EPI_BYTES);
    uint32_t *tmem_slot = (uint32_t *)(bars + 2 * STAGES + 2);
    __shared__ int s_abort;
    __shared__ int s_epi_cnt, s_go;  // stream-K hand-offs among the epilogue warps

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n_tiles_n = (p.N + BN - 1) / BN;
    const int m_tiles = (p.M + BM - 1) / BM;
    const int n_tiles = n_tiles_n * m_tiles;
    const int kblocks = (p.K + BK - 1) / BK;

    const uint32_t bar_full0 = smem_u32(&bars[0]);
    const uint32_t bar_empty0 = smem_u32(&bars[STAGES]);
    const uint32_t bar_acc_full = smem_u32(&bars[2 * STAGES]);
    const uint32_t bar_acc_empty = smem_u32(&bars[2 * STAGES + 1]);

    if (threadIdx.x == 0) {
        s_abort = 0;
        s_epi_cnt = 0;
        s_go = 0;
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(bar_full0 + 8 * s, 1);
            mbar_init(bar_empty0 + 8 * s, 1);
        }
        mbar_init(bar_acc_full, 1);
        mbar_init(bar_acc_empty, EPI_WARPS);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&mapAh) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&mapAl) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&mapBh) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&mapBl) : "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *tmem_slot;
    // Prologue done: let the next kernel in the stream start its own.  The
    // weights do not depend on the previous kernel, so the producer issues
    // the weight tiles of its first STAGES K-blocks before it waits for that
    // kernel to finish writing this one's activations.
    pdl_trigger();
    const uint64_t pol_w = policy_evict_last();
    auto load_b = [&](uint8_t *st, uint32_t full, int kx, int n0) {
        if (p.l2hints) {
            tma_load_2d_hint(smem_u32(st + 2 * A_BYTES), &mapBh, full, kx, n0, pol_w);
            tma_load_2d_hint(smem_u32(st + 2 * A_BYTES + B_BYTES), &mapBl, full, kx, n0, pol_w);
        } else {
            tma_load_2d(smem_u32(st + 2 * A_BYTES), &mapBh, full, kx, n0);
            tma_load_2d(smem_u32(st + 2 * A_BYTES + B_BYTES), &mapBl, full, kx, n0);
        }
    };
    int pre = 0, cursor0 = 0;
    Piece pc0;
    bool have0 = false;
    if (warp == 0 && lane == 0) {
        have0 = next_piece(p, n_tiles, kblocks, cursor0, pc0);
        if (have0) {
            int tm0, tn0;
            tile_coords(pc0.t, n_tiles_n, m_tiles, p.group_n, tm0, tn0);
            const int n0 = tn0 * BN;
            for (int kb = pc0.kb0; kb < pc0.kb1 && pre < STAGES; ++kb, ++pre) {
                const uint32_t full = bar_full0 + 8 * pre;
                mbar_expect_tx(full, STAGE_BYTES);
                load_b(smem + pre * STAGE_BYTES, full, kb * BK, n0);
            }
        }
    }
    pdl_wait();

    if (warp == 0 && lane == 0) {
        // ---- TMA producer: runs ahead into the next piece's K-blocks while
        // the epilogue drains the current one.  The first `pre` stages have
        // their weight tiles and byte counts in place already.
        int stage = 0;
        uint32_t phase = 0;
        int issued = 0, cursor = cursor0;
        Piece pc = pc0;
        bool have = have0;
        while (!*(volatile int *)&s_abort && have) {
            int tm, tn;
            tile_coords(pc.t, n_tiles_n, m_tiles, p.group_n, tm, tn);
            const int m0 = tm * BM, n0 = tn * BN;
            if (p.R && p.splits <= 0 && pc.np >= 0 && p.ldr % 4 == 0) {
                // The residual rows this piece's epilogue will add go to L2
                // while its K-blocks stream, so the epilogue finds them there.
                const int cols = min(BN, p.N - n0), rows = min(BM, p.M - m0);
                const uint32_t bytes = (uint32_t)((cols * 4) & ~15);
                for (int r = 0; bytes && r < rows; ++r)
                    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(
                                     (uint64_t)(p.R + (size_t)(m0 + r) * p.ldr + n0)),
                                 "r"(bytes)
                                 : "memory");
            }
            for (int kb = pc.kb0; kb < pc.kb1; ++kb) {
                const bool fresh = issued >= pre;
                if (fresh && !mbar_wait(bar_empty0 + 8 * stage, phase ^ 1)) {
                    atomicExch(p.err, 101);
                    s_abort = 1;
                    break;
                }
                if (*(volatile int *)&s_abort) break;
                uint8_t *st = smem + stage * STAGE_BYTES;
                const uint32_t full = bar_full0 + 8 * stage;
                if (fresh) mbar_expect_tx(full, STAGE_BYTES);
                const int kx = kb * BK;
                tma_load_2d(smem_u32(st), &mapAh, full, kx, m0);
                tma_load_2d(smem_u32(st + A_BYTES), &mapAl, full, kx, m0);
                if (fresh) load_b(st, full, kx, n0);
                ++issued;
                if (++stage == STAGES) {
                    stage = 0;
                    phase ^= 1;
                }
            }
            have = next_piece(p, n_tiles, kblocks, cursor, pc);
        }
        // Drain: wait (bounded) until the last issued stages have landed, so
        // no copy is still writing this CTA's shared memory when it exits
        // (stages whose weight tiles went out before the wait included).
        {
            int s2 = 0;
            uint32_t ph2 = 0;
            const int n_drain = issued > pre ? issued : pre;
            for (int i = 0; i < n_drain; ++i) {
                if (i >= n_drain - STAGES) mbar_wait(bar_full0 + 8 * s2, ph2);
                if (++s2 == STAGES) {
                    s2 = 0;
                    ph2 ^= 1;
                }
            }
        }
    } else if (warp == 1 && lane == 0) {
        // ---- MMA issuer
        int stage = 0;
        uint32_t phase = 0;
        int i = 0, cursor = 0;
        Piece pc;
        for (; next_piece(p, n_tiles, kblocks, cursor, pc); ++i) {
            // The accumulators are free once the epilogue drained piece i - 1.
            if (!mbar_wait(bar_acc_empty, (uint32_t)((i & 1) ^ 1)) || *(volatile int *)&s_abort) {
                atomicExch(p.err, 104);
                s_abort = 1;
                break;
            }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            bool ok = true;
            for (int kb = pc.kb0; kb < pc.kb1; ++kb) {
                if (!mbar_wait(bar_full0 + 8 * stage, phase) || *(volatile int *)&s_abort) {
                    atomicExch(p.err, 102);
                    s_abort = 1;
                    ok = false;
                    break;
                }
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint32_t base = smem_u32(smem + stage * STAGE_BYTES);
                const uint64_t dAh = smem_desc(base), dAl = smem_desc(base + A_BYTES);
                const uint64_t dBh = smem_desc(base + 2 * A_BYTES), dBl = smem_desc(base + 2 * A_BYTES + B_BYTES);
#pragma unroll
                for (int kk = 0; kk < BK / 8; ++kk) {
                    const uint64_t off = (uint64_t)((kk * 32) >> 4);  // 8 tf32 = 32 bytes along the swizzled row
                    const uint32_t acc = (kb != pc.kb0 || kk) ? 1u : 0u;
                    mma_tf32(tmem, dAh + off, dBh + off, IDESC, acc);
                    mma_tf32(tmem + BN, dAh + off, dBl + off, IDESC, acc);
                    mma_tf32(tmem + BN, dAl + off, dBh + off, IDESC, 1u);
                }
                mma_commit(bar_empty0 + 8 * stage);
                if (++stage == STAGES) {
                    stage = 0;
                    phase ^= 1;
                }
            }
            // Arrives once every MMA issued above has completed (also on the
            // abort path, so TMEM is never freed under a running MMA).
            mma_commit(bar_acc_full);
            if (!ok) break;
        }
    } else if (warp >= 4) {
        // ---- epilogue: warps 4..3+EPI_WARPS; warp w reads TMEM lanes
        // 32*(w%4) .. +31 and half of the columns (warpgroup (w-4)/4).
        const int q = warp & 3;
        const int half = (warp - 4) >> 2;
        constexpr int COLS = BN / 2;
        const bool vec = (p.ldc % 4 == 0) && (!p.R || p.ldr % 4 == 0);
        const bool argmax_mode = p.best_val != nullptr;
        const size_t tile_floats = (size_t)BM * BN;
        int i = 0, cursor = 0, n_part = 0, n_fin = 0;
        Piece pc;
        for (; next_piece(p, n_tiles, kblocks, cursor, pc); ++i) {
            int tm, tn;
            tile_coords(pc.t, n_tiles_n, m_tiles, p.group_n, tm, tn);
            const int m0 = tm * BM, n0 = tn * BN;
            const bool ok = mbar_wait(bar_acc_full, (uint32_t)(i & 1)) && !*(volatile int *)&s_abort;
            __syncwarp();
            if (!ok) {
                if (lane == 0) atomicExch(p.err, 103);
                break;
            }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const float *parts = nullptr;
            float *part_out = nullptr;
            if (pc.np < 0) {
                part_out = p.ws + (size_t)blockIdx.x * tile_floats;
            } else if (pc.np > 0) {
                // Wait (bounded) until the next np CTAs published their
                // partials of this tile, then every epilogue warp reads them.
                parts = p.ws + (size_t)(blockIdx.x + 1) * tile_floats;
                ++n_fin;
                if (warp == 4 && lane == 0) {
                    for (int c = 1; c <= pc.np; ++c) {
                        const uint64_t t0 = globaltimer();
                        for (;;) {
                            int v;
                            asm volatile("ld.acquire.gpu.global.s32 %0, [%1];"
                                         : "=r"(v)
                                         : "l"(p.flags + blockIdx.x + c)
                                         : "memory");
                            if (v) break;
                            if (globaltimer() - t0 > p.handoff_wait_ns) {
                                atomicExch(p.err, 121);
                                break;
                            }
                        }
                        p.flags[blockIdx.x + c] = 0;  // ready for the next launch
                    }
                    __threadfence_block();
                    *(volatile int *)&s_go = n_fin;
                }
                if (lane == 0) {
                    const uint64_t t0 = globaltimer();
                    while (*(volatile int *)&s_go < n_fin)
                        if (globaltimer() - t0 > WAIT_NS) {
                            atomicExch(p.err, 122);
                            break;
                        }
                    __threadfence();
                }
                __syncwarp();
            }
            const int row = m0 + q * 32 + lane;
            constexpr bool prep_mode = MODE == MODE_PREP;
            float best = -INFINITY;
            uint32_t best_n = prep_mode ? 0u : 0xFFFFFFFFu;
            float *stg =
                BN == 256 ? reinterpret_cast<float *>(smem + STAGES * STAGE_BYTES) + (warp - 4) * 1024 : nullptr;
            epilogue_cols<BN, MODE>(p, tmem, q, lane, m0, n0, half * COLS, (half + 1) * COLS, argmax_mode, vec, best, best_n,
                              stg, parts, pc.np > 0 ? pc.np : 0, part_out, pc.split, &mapC, &mapClo);
            // TMEM of this piece fully read: hand the accumulators back.
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            __syncwarp();
            if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar_acc_empty) : "memory");
            if (part_out) {
                // Publish the partial once all eight epilogue warps wrote theirs.
                ++n_part;
                if (lane == 0) {
                    __threadfence();
                    atomicAdd(&s_epi_cnt, 1);
                }
                if (warp == 4 && lane == 0) {
                    const uint64_t t0 = globaltimer();
                    while (*(volatile int *)&s_epi_cnt < EPI_WARPS * n_part)
                        if (globaltimer() - t0 > WAIT_NS) {
                            atomicExch(p.err, 123);
                            break;
                        }
                    __threadfence();
                    if (!p.withhold_publish)
                        asm volatile("st.release.gpu.global.s32 [%0], %1;" ::"l"(p.flags + blockIdx.x), "r"(1)
                                     : "memory");
                }
                __syncwarp();
            }
            if (argmax_mode && row < p.M) {
                // Each warpgroup holds the first maximum of its half of the
                // tile's columns: partial 2*tile_n + half, so partial order is
                // column order and the reduction's earliest-partial tie rule
                // keeps the first maximum.
                const size_t slot = (size_t)row * p.n_tiles + 2 * tn + half;
                p.best_val[slot] = best;
                p.best_idx[slot] = best_n;
            }
            if (prep_mode && row < p.M) {  // MODE_PREP only
                const size_t slot = (size_t)row * p.n_tiles + 2 * tn + half;
                p.prep_max[slot] = best;
                p.prep_pinf[slot] = best_n;
            }
        }
        // Every bulk store this warp issued has completed before the CTA
        // exits (its staging buffer stays valid, and the next kernel's reads
        // see the outputs).
        if (BN == 256 && p.tma_store && lane == 0) bulk_wait_all();
        __syncwarp();
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
    }
}

// ---------------------------------------------------------------------------
// CTA-pair kernel (tcgen05 cta_group::2): a cluster of two CTAs on two SMs
// computes a 256 x 256 tile.  CTA r (rank in the pair) loads A rows
// [128 r, 128 r + 128) and W rows [128 r, 128 r + 128) of the tile, so each
// SM stages 32 KiB per K-block instead of 48 KiB and its tensor core reads
// half of W from its own shared memory; the leader (rank 0) issues
// tcgen05.mma.cta_group::2 (M = 256, N = 256) and each CTA's TMEM receives
// its own 128 rows x 256 columns.  Both CTAs' tensor copies (each into its
// own shared memory, from this GPU's memory only) complete on the leader's
// full barrier; the leader's tcgen05.commit arrives on both CTAs' empty and
// acc_full barriers; both CTAs' epilogue warps arrive on the leader's
// acc_empty barrier.
constexpr int P_STAGES = 6;
constexpr int P_HALF_BYTES = 128 * BK * 4;              // 8 KiB: 128 rows x one K-block
constexpr int P_STAGE_BYTES = 4 * P_HALF_BYTES;         // A_hi, A_lo, W_hi, W_lo halves
constexpr int P_SMEM_BYTES = P_STAGES * P_STAGE_BYTES + 1024 + 256;
constexpr uint32_t P_TMEM_COLS = 512;
// D f32, A/B tf32, both K-major, M = 256 (the pair), N = 256.
constexpr uint32_t P_IDESC = (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(256 >> 3) << 17) |
                             ((uint32_t)(256 >> 4) << 24);

__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

// Address of the same shared-memory offset in the pair's rank-0 CTA.
__device__ __forceinline__ uint32_t at_rank0(uint32_t addr) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, 0;" : "=r"(r) : "r"(addr));
    return r;
}

__device__ __forceinline__ void pair_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap *map, uint32_t bar_rank0, int x,
                                                 int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
        ::"r"(dst), "l"((uint64_t)map), "r"(bar_rank0), "r"(x), "r"(y)
        : "memory");
}

__device__ __forceinline__ void mma_tf32_pair(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc,
                                              uint32_t accumulate) {
    asm volatile(
        "{ .reg .pred p; setp.ne.b32 p, %4, 0; tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, p; }"
        ::"r"(d_tmem), "l"(a), "l"(b), "r"(idesc), "r"(accumulate));
}

// Arrive on the barrier at this offset in both CTAs of the pair once every
// MMA issued so far has completed.
__device__ __forceinline__ void mma_commit_pair(uint32_t bar) {
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;"
        ::"r"(bar), "h"((unsigned short)3)
        : "memory");
}

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(THREADS, 1)
tc_pair_kernel(const __grid_constant__ CUtensorMap mapAh, const __grid_constant__ CUtensorMap mapAl,
               const __grid_constant__ CUtensorMap mapBh, const __grid_constant__ CUtensorMap mapBl, TcArgs p) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint64_t *bars = (uint64_t *)(smem + P_STAGES * P_STAGE_BYTES);  // full[S], empty[S], acc_full, acc_empty
    uint32_t *tmem_slot = (uint32_t *)(bars + 2 * P_STAGES + 2);
    __shared__ int s_abort;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_rank();
    const int pair = blockIdx.x >> 1, n_pairs = gridDim.x >> 1;
    const int n_tiles_n = (p.N + 255) / 256;
    const int n_tiles = n_tiles_n * ((p.M + 255) / 256);
    const int kblocks = (p.K + BK - 1) / BK;

    const uint32_t bar_full0 = smem_u32(&bars[0]);
    const uint32_t bar_empty0 = smem_u32(&bars[P_STAGES]);
    const uint32_t bar_acc_full = smem_u32(&bars[2 * P_STAGES]);
    const uint32_t bar_acc_empty = smem_u32(&bars[2 * P_STAGES + 1]);

    if (threadIdx.x == 0) {
        s_abort = 0;
        for (int s = 0; s < P_STAGES; ++s) {
            mbar_init(bar_full0 + 8 * s, 1);
            mbar_init(bar_empty0 + 8 * s, 1);
        }
        mbar_init(bar_acc_full, 1);
        mbar_init(bar_acc_empty, 2 * EPI_WARPS);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&mapAh) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&mapAl) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&mapBh) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&mapBl) : "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(P_TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    pair_sync();  // both CTAs' barriers initialised before any cross-CTA signal
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *tmem_slot;
    // Prologue done: let the next kernel in the stream start its own, then
    // wait until the previous one has finished writing this one's inputs.
    pdl_trigger();
    pdl_wait();

    if (warp == 0 && lane == 0) {
        // ---- TMA producer (both CTAs): this CTA's halves, completing on the
        // leader's full barrier; the leader also arms it with both halves' bytes.
        int stage = 0;
        uint32_t phase = 0;
        int issued = 0;
        const uint32_t full0_r0 = at_rank0(bar_full0);
        for (int t = pair; t < n_tiles && !*(volatile int *)&s_abort; t += n_pairs) {
            const int m0 = (t / n_tiles_n) * 256 + (int)rank * 128;
            const int nb = (t % n_tiles_n) * 256 + (int)rank * 128;
            for (int kb = 0; kb < kblocks; ++kb) {
                if (!mbar_wait(bar_empty0 + 8 * stage, phase ^ 1)) {
                    atomicExch(p.err, 105);
                    s_abort = 1;
                    break;
                }
                if (*(volatile int *)&s_abort) break;
                uint8_t *st = smem + stage * P_STAGE_BYTES;
                if (rank == 0) mbar_expect_tx(bar_full0 + 8 * stage, 2 * P_STAGE_BYTES);
                const uint32_t full = full0_r0 + 8 * stage;
                const int kx = kb * BK;
                tma_load_2d_pair(smem_u32(st), &mapAh, full, kx, m0);
                tma_load_2d_pair(smem_u32(st + P_HALF_BYTES), &mapAl, full, kx, m0);
                tma_load_2d_pair(smem_u32(st + 2 * P_HALF_BYTES), &mapBh, full, kx, nb);
                tma_load_2d_pair(smem_u32(st + 3 * P_HALF_BYTES), &mapBl, full, kx, nb);
                ++issued;
                if (++stage == P_STAGES) {
                    stage = 0;
                    phase ^= 1;
                }
            }
        }
        // Drain: a stage's copies have landed once the leader's MMAs have
        // consumed it, which its empty barrier records; wait (bounded) for the
        // last issued stages so no copy still writes this CTA's shared memory
        // when it exits.
        {
            int s2 = 0;
            uint32_t ph2 = 0;
            for (int i = 0; i < issued; ++i) {
                if (i >= issued - P_STAGES) mbar_wait(bar_empty0 + 8 * s2, ph2);
                if (++s2 == P_STAGES) {
                    s2 = 0;
                    ph2 ^= 1;
                }
            }
        }
    } else if (warp == 1 && lane == 0 && rank == 0) {
        // ---- MMA issuer (leader only)
        int stage = 0;
        uint32_t phase = 0;
        int i = 0;
        for (int t = pair; t < n_tiles; t += n_pairs, ++i) {
            if (!mbar_wait(bar_acc_empty, (uint32_t)((i & 1) ^ 1)) || *(volatile int *)&s_abort) {
                atomicExch(p.err, 108);
                s_abort = 1;
                break;
            }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            bool ok = true;
            for (int kb = 0; kb < kblocks; ++kb) {
                if (!mbar_wait(bar_full0 + 8 * stage, phase) || *(volatile int *)&s_abort) {
                    atomicExch(p.err, 106);
                    s_abort = 1;
                    ok = false;
                    break;
                }
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint32_t base = smem_u32(smem + stage * P_STAGE_BYTES);
                const uint64_t dAh = smem_desc(base), dAl = smem_desc(base + P_HALF_BYTES);
                const uint64_t dBh = smem_desc(base + 2 * P_HALF_BYTES), dBl = smem_desc(base + 3 * P_HALF_BYTES);
#pragma unroll
                for (int kk = 0; kk < BK / 8; ++kk) {
                    const uint64_t off = (uint64_t)((kk * 32) >> 4);
                    const uint32_t acc = (kb | kk) ? 1u : 0u;
                    mma_tf32_pair(tmem, dAh + off, dBh + off, P_IDESC, acc);
                    mma_tf32_pair(tmem + 256, dAh + off, dBl + off, P_IDESC, acc);
                    mma_tf32_pair(tmem + 256, dAl + off, dBh + off, P_IDESC, 1u);
                }
                mma_commit_pair(bar_empty0 + 8 * stage);
                if (++stage == P_STAGES) {
                    stage = 0;
                    phase ^= 1;
                }
            }
            mma_commit_pair(bar_acc_full);
            if (!ok) break;
        }
    } else if (warp >= 4) {
        // ---- epilogue (both CTAs): this CTA's 128 rows x 256 columns
        const int q = warp & 3;
        const int half = (warp - 4) >> 2;
        const bool vec = (p.ldc % 4 == 0) && (!p.R || p.ldr % 4 == 0);
        const bool argmax_mode = p.best_val != nullptr;
        const uint32_t acc_empty_r0 = at_rank0(bar_acc_empty);
        int i = 0;
        for (int t = pair; t < n_tiles; t += n_pairs, ++i) {
            const int m0 = (t / n_tiles_n) * 256 + (int)rank * 128;
            const int tn = t % n_tiles_n;
            const int n0 = tn * 256;
            const bool ok = mbar_wait(bar_acc_full, (uint32_t)(i & 1)) && !*(volatile int *)&s_abort;
            __syncwarp();
            if (!ok) {
                if (lane == 0) atomicExch(p.err, 107);
                break;
            }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const int row = m0 + q * 32 + lane;
            float best = -INFINITY;
            uint32_t best_n = 0xFFFFFFFFu;
            epilogue_cols<256>(p, tmem, q, lane, m0, n0, half * 128, half * 128 + 128, argmax_mode, vec, best,
                               best_n, nullptr);
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            __syncwarp();
            if (lane == 0)
                asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(acc_empty_r0)
                             : "memory");
            if (argmax_mode && row < p.M) {
                const size_t slot = (size_t)row * p.n_tiles + 2 * tn + half;
                p.best_val[slot] = best;
                p.best_idx[slot] = best_n;
            }
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    pair_sync();  // the peer is done with this CTA's barriers and TMEM
    if (warp == 1) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(P_TMEM_COLS) : "memory");
    }
}

// hi = tf32(x), lo = tf32(x - hi), over rows x cols with a row stride.
// pair_half = H > 0: source row r lands at the interleaved position (gate
// rows r < H and value rows H + r in alternating blocks of 32).
__global__ void split_tf32_k(const float *__restrict__ src, int ld, float *__restrict__ hi,
                             float *__restrict__ lo, int rows, int cols, int pair_half) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (int64_t)rows * cols) return;
    const int64_t r = i / cols;
    const int c = (int)(i - r * cols);
    int64_t rd = r;
    if (pair_half > 0) {
        const int64_t v = r < pair_half ? r : r - pair_half;
        rd = (v >> 5) * 64 + (r < pair_half ? 0 : 32) + (v & 31);
    }
    const float x = src[(size_t)r * ld + c];
    const float h = tf32_round(x);
    hi[(size_t)rd * cols + c] = h;
    lo[(size_t)rd * cols + c] = tf32_round(x - h);
}

// hi / lo [cols, ld_out] = the split of the transpose of src [rows, cols]
// (row stride cols), columns rows .. ld_out - 1 of the output zero (K
// padding to a multiple of 4).  32 x 32 tiles through shared memory keep
// both the reads and the writes coalesced.  *nonfinite = 1 if any element
// is inf or NaN.
__global__ void split_tf32_t_k(const float *__restrict__ src, int rows, int cols, int ld_out,
                               float *__restrict__ hi, float *__restrict__ lo, int *nonfinite) {
    __shared__ float tile[32][33];
    const int c0 = blockIdx.x * 32;
    const int64_t r0 = (int64_t)blockIdx.y * 32;
    bool bad = false;
    for (int i = threadIdx.y; i < 32; i += blockDim.y) {
        const int64_t r = r0 + i;
        const int c = c0 + threadIdx.x;
        float x = 0.0f;
        if (r < rows && c < cols) {
            x = src[(size_t)r * cols + c];
            bad |= !isfinite(x);
        }
        tile[i][threadIdx.x] = x;
    }
    if (bad && nonfinite) atomicExch(nonfinite, 1);
    __syncthreads();
    for (int i = threadIdx.y; i < 32; i += blockDim.y) {
        const int c = c0 + i;
        const int64_t r = r0 + threadIdx.x;
        if (c < cols && r < ld_out) {
            const float x = tile[threadIdx.x][i];
            const float h = tf32_round(x);
            hi[(size_t)c * ld_out + r] = h;
            lo[(size_t)c * ld_out + r] = tf32_round(x - h);
        }
    }
}

// Split-K reduction: out = sum over splits (in split order) of the pieces'
// raw sums, then the store epilogue (bias, residual) or the SwiGLU epilogue
// of the interleaved operand (output channel j: gate column 64 (j / 32) +
// j % 32, value column 32 later), with the same f32 operations as the
// single-piece epilogues.
// part[0] + part[plane] + ... + part[(splits - 1) plane], added in that
// order; the loads of eight pieces are issued before their adds, so a
// reduction waits one memory round trip per eight pieces, not per piece.
__device__ __forceinline__ float split_sum(const float *pp, int splits, size_t plane) {
    float o = pp[0];
    for (int s0 = 1; s0 < splits; s0 += 8) {
        float v[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) v[e] = s0 + e < splits ? pp[(size_t)(s0 + e) * plane] : 0.0f;
#pragma unroll
        for (int e = 0; e < 8; ++e)
            if (s0 + e < splits) o = o + v[e];
    }
    return o;
}

__global__ void splitk_reduce_k(const float *__restrict__ part, int splits, TcArgs p) {
    pdl_trigger();
    pdl_wait();
    const int M = p.M, N = p.N, swiglu_H = p.swiglu_H;
    const int cols = swiglu_H ? swiglu_H : N;
    const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
    const bool valid = i < (long)M * cols;
    const int m = valid ? (int)(i / cols) : 0, c = valid ? (int)(i - (long)m * cols) : 0;
    const size_t plane = (size_t)M * N;
    const float rscale = valid ? folded_row_scale(p, m) : 1.0f;
    if (swiglu_H) {
        if (!valid) return;
        const int cg = 64 * (c >> 5) + (c & 31), cv = cg + 32;
        float g = split_sum(part + (size_t)m * N + cg, splits, plane);
        float v = split_sum(part + (size_t)m * N + cv, splits, plane);
        if (p.rs_parts) {
            g = g * rscale;
            v = v * rscale;
        }
        const float sv = silu(g + p.bias[c]) * (v + p.bias[swiglu_H + c]);
        if (p.C_lo) {
            const float h = tf32_round(sv);
            p.C[(size_t)m * p.ldc + c] = h;
            p.C_lo[(size_t)m * p.ldc + c] = tf32_round(sv - h);
        } else {
            p.C[(size_t)m * p.ldc + c] = sv;
        }
        return;
    }
    float o = 0.0f;
    if (valid) {
        o = split_sum(part + (size_t)m * N + c, splits, plane);
        if (p.rs_parts) o = o * rscale;
        if (p.bias) o = o + p.bias[c];
        if (p.R) o = p.R[(size_t)m * p.ldr + c] + o;
        p.C[(size_t)m * p.ldc + c] = o;
    }
    if (p.nx_hi) {
        // Folded RMSNorm producer (N % 32 == 0: a warp holds 32 consecutive
        // columns of one row): the next operand and the chunk's sum of squares.
        if (valid) {
            const float y = o * p.nx_gain[c], h = tf32_round(y);
            p.nx_hi[(size_t)m * N + c] = h;
            p.nx_lo[(size_t)m * N + c] = tf32_round(y - h);
        }
        const float sq = warp_sum(valid ? o * o : 0.0f);
        if ((threadIdx.x & 31) == 0 && valid) p.nx_ss[(size_t)m * p.nx_nparts + (c >> 5)] = sq;
    }
}

// Split-K reduction of a residual projection that also applies the next
// RMSNorm: one CTA per row sums the pieces of all N columns as
// splitk_reduce_k does, stores the row x, then computes r = 1 / sqrt(mean(x^2)
// + eps) with the lane-strided sum of rmsnorm_k and writes x * r * gain.
struct PostNorm {
    const float *gain;
    float eps;
    float *hi, *lo, *f32;
};

__global__ void __launch_bounds__(256) splitk_reduce_norm_k(const float *__restrict__ part, int splits, TcArgs p,
                                                             PostNorm pn) {
    pdl_trigger();
    pdl_wait();
    extern __shared__ float xrow[];
    __shared__ float s_r;
    const int m = blockIdx.x, N = p.N;
    const size_t plane = (size_t)p.M * N;
    const float rscale = folded_row_scale(p, m);
    for (int c = threadIdx.x; c < N; c += blockDim.x) {
        float o = split_sum(part + (size_t)m * N + c, splits, plane);
        if (p.rs_parts) o = o * rscale;
        if (p.bias) o = o + p.bias[c];
        if (p.R) o = p.R[(size_t)m * p.ldr + c] + o;
        p.C[(size_t)m * p.ldc + c] = o;
        xrow[c] = o;
    }
    __syncthreads();
    if (threadIdx.x < 32) {
        float ms = 0.0f;
        for (int j = threadIdx.x; j < N; j += 32) ms = fmaf(xrow[j], xrow[j], ms);
        ms = warp_sum(ms);
        if (threadIdx.x == 0) s_r = 1.0f / sqrtf(ms / (float)N + pn.eps);
    }
    __syncthreads();
    const float r = s_r;
    for (int c = threadIdx.x; c < N; c += blockDim.x) {
        const float y = xrow[c] * r * pn.gain[c];
        const size_t o = (size_t)m * N + c;
        if (pn.hi) {
            const float h = tf32_round(y);
            pn.hi[o] = h;
            pn.lo[o] = tf32_round(y - h);
        } else {
            pn.f32[o] = y;
        }
    }
}

// Split-K reduction of the input projection (N = 3E) that runs the decode
// step's recurrent branch on each channel's reduced (v, z, o) instead of
// storing u.
struct PostSsm {
    float *state;
    const uint32_t *heads;
    const float *conv_w, *conv_b;
    int k, E;
    float *hi, *lo, *f32;
};

template <int K>
__global__ void __launch_bounds__(256) splitk_reduce_ssm_k(const float *__restrict__ part, int splits, TcArgs p,
                                                            PostSsm ps) {
    pdl_trigger();
    pdl_wait();
    const int E = ps.E, k = ps.k;
    const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long)p.M * E) return;
    const int m = (int)(i / E), j = (int)(i - (long)m * E);
    const size_t plane = (size_t)p.M * p.N;
    const float *row = part + (size_t)m * p.N + j;
    const float rscale = folded_row_scale(p, m);
    // The three columns (v, z, o) of the channel, each summed over the pieces
    // in split order; the loads of eight pieces of all three go out together.
    float u[3] = {row[0], row[E], row[2 * E]};
    for (int s0 = 1; s0 < splits; s0 += 8) {
        float t[3][8];
#pragma unroll
        for (int e = 0; e < 8; ++e)
#pragma unroll
            for (int f = 0; f < 3; ++f) t[f][e] = s0 + e < splits ? row[(size_t)(s0 + e) * plane + f * E] : 0.0f;
#pragma unroll
        for (int e = 0; e < 8; ++e)
#pragma unroll
            for (int f = 0; f < 3; ++f)
                if (s0 + e < splits) u[f] = u[f] + t[f][e];
    }
#pragma unroll
    for (int f = 0; f < 3; ++f) {
        if (p.rs_parts) u[f] = u[f] * rscale;
        if (p.bias) u[f] = u[f] + p.bias[f * E + j];
    }
    float *ring = ps.state + (size_t)m * (k + 1) * E;
    const float gv = ssm_step_channel<K>(u[0], u[1], u[2], ring, ps.heads[m], k, E, j, ps.conv_w, ps.conv_b);
    const size_t o = (size_t)m * E + j;
    if (ps.hi) {
        const float h = tf32_round(gv);
        ps.hi[o] = h;
        ps.lo[o] = tf32_round(gv - h);
    } else {
        ps.f32[o] = gv;
    }
}

// Split-K reduction of the argmax and sampling epilogues: block (chunk,
// row) sums the pieces of ROWRED_COLS columns of one row in split order,
// then either (argmax) records the first maximum of the chunk (NaN skipped)
// or (PREP) writes pen(sum) / temperature and records the maximum of the
// finite values and the +inf count; partial (row, chunk) goes to slot
// row * parts + chunk, the layout the tile epilogues use.
template <bool PREP>
__global__ void __launch_bounds__(256) splitk_rowred_k(const float *__restrict__ part, int splits, int M, int N,
                                                        TcArgs p, int parts) {
    pdl_trigger();
    pdl_wait();
    const int row = blockIdx.y, chunk = blockIdx.x;
    const int c0 = chunk * ROWRED_COLS, c1 = min(N, c0 + ROWRED_COLS);
    const size_t plane = (size_t)M * N;
    const float rscale = folded_row_scale(p, row);
    float best = -INFINITY;
    uint32_t tag = PREP ? 0u : 0xFFFFFFFFu;  // +inf count, or the first maximum's column
    for (int c = c0 + (int)threadIdx.x; c < c1; c += blockDim.x) {
        float o = split_sum(part + (size_t)row * N + c, splits, plane);
        if (p.rs_parts) o = o * rscale;
        if constexpr (PREP) {
            const bool pen = p.pen_bits && ((p.pen_bits[(size_t)row * p.pen_words + (c >> 5)] >> (c & 31)) & 1u);
            const float y = sample_prep(o, pen, p);
            p.C[(size_t)row * p.ldc + c] = y;
            if (y == INFINITY) ++tag;
            if (isfinite(y) && y > best) best = y;
        } else {
            if (!isnan(o) && o > best) {  // columns ascend per thread: the first maximum stays
                best = o;
                tag = (uint32_t)c;
            }
        }
    }
    __shared__ float sb[8];
    __shared__ uint32_t st[8];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ob = __shfl_xor_sync(0xffffffffu, best, o);
        const uint32_t ot = __shfl_xor_sync(0xffffffffu, tag, o);
        if constexpr (PREP) {
            best = fmaxf(best, ob);
            tag += ot;
        } else if (ob > best || (ob == best && ot < tag)) {
            best = ob;
            tag = ot;
        }
    }
    if (lane == 0) {
        sb[warp] = best;
        st[warp] = tag;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < (int)(blockDim.x >> 5); ++w) {
            if constexpr (PREP) {
                best = fmaxf(best, sb[w]);
                tag += st[w];
            } else if (sb[w] > best || (sb[w] == best && st[w] < tag)) {
                best = sb[w];
                tag = st[w];
            }
        }
        const size_t slot = (size_t)row * parts + chunk;
        if constexpr (PREP) {
            p.prep_max[slot] = best;
            p.prep_pinf[slot] = tag;
        } else {
            p.best_val[slot] = best;
            p.best_idx[slot] = tag;
        }
    }
}

// ---- host side
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = (PFN_cuTensorMapEncodeTiled_v12000)p;
    });
    return fn;
}

// 2-D f32 map over [rows, cols] (cols contiguous), box {BK, box_rows}, 64B
// swizzle, zero fill outside the tensor.
// 2-D f32 map over [rows, cols] with row stride ld floats, box {32, 32},
// 128-byte swizzle: the epilogue's bulk stores.
bool make_store_map(CUtensorMap *map, const float *base, int rows, int cols, int ld) {
    auto fn = encode_fn();
    if (!fn || ld % 4 != 0 || ((uintptr_t)base & 15) != 0) return false;
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)ld * sizeof(float)};
    cuuint32_t box[2] = {32, 32};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, (void *)base, dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

bool make_map(CUtensorMap *map, const float *base, int rows, int cols, int box_rows) {
    auto fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)cols * sizeof(float)};
    cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, (void *)base, dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

cudaError_t split(const float *src, int ld, float *hi, float *lo, int rows, int cols, cudaStream_t st,
                  int pair_half = 0) {
    const int64_t n = (int64_t)rows * cols;
    if (n == 0) return cudaSuccess;
    split_tf32_k<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(src, ld, hi, lo, rows, cols, pair_half);
    return cudaGetLastError();
}

}  // namespace

// Any M: a tile past the last row reads zeros (the A map's rows beyond M
// are filled, never read) and the epilogues mask rows >= M, so 9..127
// streams take one 128-row tile instead of the CUDA-core GEMM.
bool tc_eligible(int M, int N, int K) {
    return M >= 1 && N >= 128 && K >= 8 && K % 4 == 0 && encode_fn() != nullptr;
}

int sm_count_cached() {
    static int num_sms = 0;
    if (!num_sms) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&num_sms, cudaDevAttrMultiProcessorCount, dev);
        if (num_sms <= 0) num_sms = 148;
    }
    return num_sms;
}

// The CTA-pair kernel when allowed and it fills every SM pair at least
// twice.  128 x 128 tiles for a single row of tiles.  Otherwise 128 x 256
// tiles, spread by stream-K (so any tile count keeps every SM busy) when
// the epilogue allows it; for the argmax epilogue
// whole tiles, compared with 128 x 128 tiles by the fraction of SM time each
// keeps busy (a 128-wide tile moves 4/3 the operand bytes per flop, and the
// main loop is bound by operand bandwidth into shared memory).
int tc_pick_bn(int M, int N, bool allow_pair, bool stream_k) {
    const int num_sms = sm_count_cached();
    const long tiles256 = (long)((N + 255) / 256) * ((M + BM - 1) / BM);
    const long pair_tiles = (long)((N + 255) / 256) * ((M + 255) / 256);
    if (allow_pair && N >= 256 && pair_tiles >= 2L * (num_sms / 2)) return TC_PAIR;
    // One row of tiles (M <= 128, e.g. decode of 9-128 streams), or a small
    // projection of at most SPLIT_MAX_M rows whose 128-wide tiles fill under
    // half of the CTA slots: 128-wide tiles, split along K over the SMs by
    // tc_gemm (every epilogue mode).
    if (N < 256 || M <= BM) return 128;
    if (M <= SPLIT_MAX_M && (long)((N + 127) / 128) * ((M + BM - 1) / BM) <= num_sms) return 128;
    if (stream_k) return 256;
    const double e256 =
        (double)tiles256 / ((double)((tiles256 + num_sms - 1) / num_sms) * num_sms);
    const long tiles128 = (long)((N + 127) / 128) * ((M + BM - 1) / BM);
    const long slots128 = 2L * num_sms;
    const double e128 = 0.75 * (double)tiles128 / ((double)((tiles128 + slots128 - 1) / slots128) * slots128);
    return e256 >= e128 ? 256 : 128;
}

size_t tc_stream_k_ws_floats() { return (size_t)sm_count_cached() * BM * 256; }

int tc_tiles_n(int N, int bn) {
    const int w = bn == TC_PAIR ? 256 : bn;
    return (N + w - 1) / w;
}
int tc_argmax_parts(int N, int bn) { return 2 * tc_tiles_n(N, bn); }

cudaError_t tc_split_transposed(const float *src, int rows, int cols, int ld_out, float *hi, float *lo,
                                int *nonfinite, cudaStream_t st) {
    if (ld_out < rows || cols <= 0 || ld_out <= 0) return cols <= 0 ? cudaSuccess : cudaErrorInvalidValue;
    const dim3 grid((unsigned)((cols + 31) / 32), (unsigned)((ld_out + 31) / 32));
    if (grid.y > 65535u) return cudaErrorInvalidValue;
    split_tf32_t_k<<<grid, dim3(32, 8), 0, st>>>(src, rows, cols, ld_out, hi, lo, nonfinite);
    return cudaGetLastError();
}

bool tc_operand_from(const float *hi, const float *lo, int N, int K, TcOperand &op) {
    if (K % 4 != 0 || N <= 0 || K <= 0) return false;
    op.hi = hi;
    op.lo = lo;
    op.N = op.N_pad = N;
    op.K = op.K_pad = K;
    op.pair_half = 0;
    return make_map((CUtensorMap *)op.map_hi, hi, N, K, 256) && make_map((CUtensorMap *)op.map_lo, lo, N, K, 256) &&
           make_map((CUtensorMap *)op.map_hi128, hi, N, K, 128) && make_map((CUtensorMap *)op.map_lo128, lo, N, K, 128);
}

cudaError_t tc_weights_build(TcWeights &w, const std::vector<TcSource> &srcs) {
    tc_weights_free(w);
    size_t total = 0;
    for (const TcSource &s : srcs) total += 2 * (((size_t)s.N * s.K + 63) & ~size_t(63));
    cudaError_t e = cudaMalloc(&w.arena, total * sizeof(float));
    if (e != cudaSuccess) return e;
    size_t off = 0;
    w.ops.resize(srcs.size());
    for (size_t i = 0; i < srcs.size(); ++i) {
        const TcSource &s = srcs[i];
        TcOperand &op = w.ops[i];
        const size_t n = ((size_t)s.N * s.K + 63) & ~size_t(63);
        float *hi = w.arena + off, *lo = w.arena + off + n;
        off += 2 * n;
        const bool pair = s.pair_half > 0 && s.pair_half % 32 == 0 && s.N == 2 * s.pair_half;
        e = split(s.w, s.K, hi, lo, s.N, s.K, nullptr, pair ? s.pair_half : 0);
        if (e != cudaSuccess) return e;
        op.pair_half = pair ? s.pair_half : 0;
        op.hi = hi;
        op.lo = lo;
        op.N = s.N;
        op.K = s.K;
        op.N_pad = s.N;
        op.K_pad = s.K;
        if (s.K % 4 == 0) {
            if (!make_map((CUtensorMap *)op.map_hi, hi, s.N, s.K, 256) ||
                !make_map((CUtensorMap *)op.map_lo, lo, s.N, s.K, 256) ||
                !make_map((CUtensorMap *)op.map_hi128, hi, s.N, s.K, 128) ||
                !make_map((CUtensorMap *)op.map_lo128, lo, s.N, s.K, 128))
                return cudaErrorInvalidValue;
        }
    }
    e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return e;
    w.ready = true;
    return cudaSuccess;
}

void tc_weights_free(TcWeights &w) {
    if (w.arena) cudaFree(w.arena);
    w.arena = nullptr;
    w.ops.clear();
    w.ready = false;
}

template <int BN, int MODE>
cudaError_t launch_tc(const CUtensorMap &mAh, const CUtensorMap &mAl, const TcOperand &W, TcArgs a, int M,
                      cudaStream_t st, const CUtensorMap *mC = nullptr, const CUtensorMap *mClo = nullptr) {
    static thread_local int attr_dev = -1;
    int dev = 0;
    cudaGetDevice(&dev);
    if (attr_dev != dev) {
        cudaError_t e = cudaFuncSetAttribute(tc_gemm_kernel<BN, MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             Tile<BN>::SMEM_BYTES);
        if (e != cudaSuccess) return e;
        attr_dev = dev;
    }
    const unsigned char *mh = BN == 256 ? W.map_hi : W.map_hi128;
    const unsigned char *ml = BN == 256 ? W.map_lo : W.map_lo128;
    // Persistent: at most one CTA per SM slot, each walking tiles in steps
    // of the grid size (n fastest, so neighbouring CTAs share the A rows).
    static int num_sms = 0;
    if (!num_sms) {
        cudaDeviceGetAttribute(&num_sms, cudaDevAttrMultiProcessorCount, dev);
        if (num_sms <= 0) num_sms = 148;
    }
    const long tiles = (long)tc_tiles_n(W.N, BN) * ((M + BM - 1) / BM);
    const long slots = (long)num_sms * Tile<BN>::CTAS_PER_SM;
    unsigned grid = (unsigned)std::min<long>(a.splits > 0 ? tiles * a.splits : tiles, slots);
    a.skb = 0;
    a.sk_t0 = (int)tiles;
    // The A operand pair (hi + lo) of this projection; when it fits well
    // inside L2, CTAs far apart in the tile order lose nothing by reading
    // different rows of it, and every tile is spread by K.
    const bool a_in_l2 = (size_t)M * W.K * 8 <= ((size_t)48 << 20);
    if (BN == 256 && !a.best_val && !(a.temperature > 0.0f) && a.ws && a.flags && (tiles % slots != 0 || a_in_l2)) {
        // Whole waves stay whole tiles (unless A fits in L2); the rest is
        // spread over every CTA in equal K-block ranges of at least 8 K-blocks.
        const long dp = a_in_l2 ? 0 : (tiles / slots) * slots;
        const long kblocks = (W.K + BK - 1) / BK;
        const long total = (tiles - dp) * kblocks;
        long ctas = std::min<long>(slots, std::max<long>(1, total / 8));
        const long per = (total + ctas - 1) / ctas;
        ctas = (total + per - 1) / per;
        a.skb = (int)per;
        a.sk_t0 = (int)dp;
        grid = (unsigned)(dp > 0 ? slots : ctas);
    }
    // Unused maps are passed as copies of an operand map (never read).
    if (BN != 256 || !mC) a.tma_store = 0;
    const CUtensorMap &oc = a.tma_store ? *mC : mAh;
    const CUtensorMap &ocl = a.tma_store && mClo ? *mClo : oc;
    return pdl_launch(tc_gemm_kernel<BN, MODE>, dim3(grid), dim3(THREADS), Tile<BN>::SMEM_BYTES, st, mAh, mAl,
                      *(const CUtensorMap *)mh, *(const CUtensorMap *)ml, oc, ocl, a);
}

cudaError_t launch_pair(const CUtensorMap &mAh, const CUtensorMap &mAl, const TcOperand &W, TcArgs a, int M,
                        cudaStream_t st) {
    static thread_local int attr_dev = -1;
    int dev = 0;
    cudaGetDevice(&dev);
    if (attr_dev != dev) {
        cudaError_t e = cudaFuncSetAttribute(tc_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, P_SMEM_BYTES);
        if (e != cudaSuccess) return e;
        attr_dev = dev;
    }
    static int num_sms = 0;
    if (!num_sms) {
        cudaDeviceGetAttribute(&num_sms, cudaDevAttrMultiProcessorCount, dev);
        if (num_sms <= 0) num_sms = 148;
    }
    // Persistent pairs: each cluster of two CTAs walks 256 x 256 tiles.
    const long tiles = (long)((W.N + 255) / 256) * ((M + 255) / 256);
    const unsigned pairs = (unsigned)std::max<long>(1, std::min<long>(tiles, num_sms / 2));
    tc_pair_kernel<<<2 * pairs, THREADS, P_SMEM_BYTES, st>>>(mAh, mAl, *(const CUtensorMap *)W.map_hi128,
                                                             *(const CUtensorMap *)W.map_lo128, a);
    return cudaGetLastError();
}

cudaError_t tc_gemm(const float *A_hi, const float *A_lo, int M, int K, const TcOperand &W, const TcEpilogue &ep,
                    int bn, cudaStream_t st, int *err) {
    if (ep.post_done) *ep.post_done = 0;
    if (W.K != K || M <= 0 || (bn != 128 && bn != 256 && bn != TC_PAIR)) return cudaErrorInvalidValue;
    // SwiGLU mode and the interleaved operand go together; argmax never with it.
    if (ep.swiglu != (W.pair_half > 0) || (ep.swiglu && (ep.best_val || !ep.bias))) return cudaErrorInvalidValue;
    // Tiles read A rows while other tiles' epilogues write: no output may
    // overlap the A operand.
    {
        auto overlap = [](const float *a, size_t na, const float *b, size_t nb) {
            return a && b && a < b + nb && b < a + na;
        };
        const size_t na = (size_t)M * K, nc = (size_t)M * (size_t)std::max(ep.ldc, 1);
        for (const float *o : {(const float *)ep.C, (const float *)ep.C_lo})
            if (overlap(o, nc, A_hi, na) || overlap(o, nc, A_lo, na)) return cudaErrorInvalidValue;
    }
    alignas(64) CUtensorMap mAh, mAl;
    if (!make_map(&mAh, A_hi, M, K, BM) || !make_map(&mAl, A_lo, M, K, BM)) return cudaErrorInvalidValue;
    const bool prep = ep.temperature > 0.0f;
    if (prep && (bn == TC_PAIR || ep.swiglu || ep.best_val || ep.bias || ep.R || !ep.C || !ep.prep_max ||
                 !ep.prep_pinf || !(ep.temperature < INFINITY) || (ep.pen_bits && ep.pen_words < (W.N + 31) / 32)))
        return cudaErrorInvalidValue;
    TcArgs a{ep.C, ep.ldc, M, W.N, K, ep.bias, ep.R, ep.ldr, ep.best_val, ep.best_idx, tc_argmax_parts(W.N, bn), err,
              ep.swiglu ? W.pair_half : 0, ep.C_lo, 0, 0, ep.ws, ep.flags, ep.l2hints ? 1 : 0,
              prep ? ep.temperature : 0.0f, ep.rep_penalty, ep.pen_bits, ep.pen_words, ep.prep_max, ep.prep_pinf,
              ep.handoff_wait_ns ? ep.handoff_wait_ns : WAIT_NS, ep.withhold_publish ? 1 : 0, 0, 0, nullptr,
              ep.rs_parts, ep.rs_nparts, ep.rs_d, ep.rs_eps, ep.nx_hi, ep.nx_lo, ep.nx_gain, ep.nx_ss,
              (W.N + 31) / 32, 0};
    const bool fold = ep.rs_parts || ep.nx_hi;
    if (fold && (bn == TC_PAIR || (ep.rs_parts && (ep.rs_nparts <= 0 || ep.rs_d <= 0)) ||
                 (ep.nx_hi && (!ep.nx_lo || !ep.nx_gain || !ep.nx_ss || ep.swiglu || ep.best_val || prep ||
                               W.N % 32 != 0))))
        return cudaErrorInvalidValue;
    // Grouped tile order: the column blocks whose weight pair (W_hi + W_lo,
    // 8 bytes per element) fits in 24 MB form a group, so a wave reads one
    // group's weights, which L2 keeps for the next wave, while the A rows
    // stream once per group.
    if (bn != TC_PAIR && !ep.no_tile_group) {
        const int w = bn == 256 ? 256 : 128;
        const size_t col_bytes = (size_t)w * K * 8;
        const int gn = (int)std::max<size_t>(1, ((size_t)24 << 20) / col_bytes);
        a.group_n = gn < tc_tiles_n(W.N, bn) ? gn : 0;
    }
    if (a.ws) {
        // Stream-K needs one partial slot and one counter per SM.
        const int sms = sm_count_cached();
        if (ep.n_flags < sms || ep.ws_floats < (size_t)sms * BM * 256) {
            a.ws = nullptr;
            a.flags = nullptr;
        }
    }
    // One row of tiles that fills under half of the CTA slots: split K so
    // that every SM streams its share of the weights (the regime of 9-128
    // streams, where the projection is bound by the weight stream).
    int splits = 0, kps = 0;
    if (bn == 128 && ep.ws && M <= SPLIT_MAX_M) {
        const long slots = 2L * sm_count_cached();
        const long tiles = (long)tc_tiles_n(W.N, 128) * ((M + BM - 1) / BM);
        const int kblocks = (K + BK - 1) / BK;
        if (tiles * 2 <= slots && kblocks >= 4) {
            // Pieces: one per CTA slot, or one per SM up to 128 rows, where a
            // piece's fixed cost (pipeline fill, partial tile written and
            // re-read) outweighs its share of the weight stream (measured
            // at the d768 widths: 0.80 vs 0.89 ms per step at 16 streams,
            // 0.96 vs 1.02 at 64, but 1.40 vs 1.37 at 256).
            const long pieces = M <= 128 ? slots / 2 : slots;
            splits = (int)std::min<long>(kblocks / 2, std::max<long>(2, pieces / tiles));
            kps = (kblocks + splits - 1) / splits;
            splits = (kblocks + kps - 1) / kps;
            while (splits > 1 && (size_t)splits * M * W.N > ep.ws_floats) {
                kps *= 2;
                splits = (kblocks + kps - 1) / kps;
            }
            if (splits < 2) splits = 0;
        }
    }
    if (ep.launches) *ep.launches += splits ? 2 : 1;
    if (ep.parts_out) *ep.parts_out = splits ? (W.N + ROWRED_COLS - 1) / ROWRED_COLS : tc_argmax_parts(W.N, bn);
    if (bn == TC_PAIR) return launch_pair(mAh, mAl, W, a, M, st);
    if (splits) {
        a.splits = splits;
        a.kps = kps;
        a.split_part = ep.ws;
        a.best_val = nullptr;  // the pieces write raw sums; the reduction applies the epilogue
        a.temperature = 0.0f;
        cudaError_t e = launch_tc<128, MODE_SPLIT>(mAh, mAl, W, a, M, st);
        if (e != cudaSuccess) return e;
        if (ep.best_val || prep) {
            TcArgs r = a;
            r.best_val = ep.best_val;
            r.best_idx = ep.best_idx;
            r.temperature = prep ? ep.temperature : 0.0f;
            const int parts = (W.N + ROWRED_COLS - 1) / ROWRED_COLS;
            const dim3 grid((unsigned)parts, (unsigned)M);
            return prep ? pdl_launch(splitk_rowred_k<true>, grid, dim3(256), 0, st, (const float *)ep.ws, splits, M,
                                     W.N, r, parts)
                        : pdl_launch(splitk_rowred_k<false>, grid, dim3(256), 0, st, (const float *)ep.ws, splits, M,
                                     W.N, r, parts);
        }
        if (!ep.swiglu && !ep.nx_hi && ep.post_norm_gain && (ep.post_norm_hi ? ep.post_norm_lo != nullptr
                                                                              : ep.post_norm_f32 != nullptr)) {
            const PostNorm pn{ep.post_norm_gain, ep.post_norm_eps, ep.post_norm_hi, ep.post_norm_lo,
                              ep.post_norm_f32};
            if (ep.post_done) *ep.post_done = 1;
            return pdl_launch(splitk_reduce_norm_k, dim3((unsigned)M), dim3(256), (size_t)W.N * sizeof(float), st,
                              (const float *)ep.ws, splits, a, pn);
        }
        if (!ep.swiglu && !ep.nx_hi && !ep.R && ep.post_state && W.N % 3 == 0 && ep.post_heads && ep.post_conv_w &&
            ep.post_conv_b && ep.post_k >= 1 && (ep.post_g_hi ? ep.post_g_lo != nullptr : ep.post_g_f32 != nullptr)) {
            const int E = W.N / 3;
            const PostSsm ps{ep.post_state, ep.post_heads, ep.post_conv_w, ep.post_conv_b, ep.post_k, E,
                             ep.post_g_hi, ep.post_g_lo, ep.post_g_f32};
            if (ep.post_done) *ep.post_done = 1;
            const long outs = (long)M * E;
            const dim3 grid((unsigned)((outs + 255) / 256));
            const float *part = ep.ws;
            switch (ps.k) {
                case 2: return pdl_launch(splitk_reduce_ssm_k<2>, grid, dim3(256), 0, st, part, splits, a, ps);
                case 3: return pdl_launch(splitk_reduce_ssm_k<3>, grid, dim3(256), 0, st, part, splits, a, ps);
                case 4: return pdl_launch(splitk_reduce_ssm_k<4>, grid, dim3(256), 0, st, part, splits, a, ps);
                default: return pdl_launch(splitk_reduce_ssm_k<0>, grid, dim3(256), 0, st, part, splits, a, ps);
            }
        }
        const long outs = (long)M * (ep.swiglu ? W.pair_half : W.N);
        return pdl_launch(splitk_reduce_k, dim3((unsigned)((outs + 255) / 256)), dim3(256), 0, st,
                          (const float *)ep.ws, splits, a);
    }
    // Bulk-store epilogue for 256-wide tiles (store, SwiGLU and sampling
    // modes): the output as a tensor of [M, cols] with row stride ldc.
    alignas(64) CUtensorMap mC, mClo;
    const CUtensorMap *pC = nullptr, *pClo = nullptr;
    if (bn == 256 && !ep.no_tma_store && ep.C && !ep.best_val && !(ep.nx_hi)) {
        const int cols = ep.swiglu ? W.pair_half : W.N;
        if (make_store_map(&mC, ep.C, M, cols, ep.ldc) &&
            (!ep.C_lo || make_store_map(&mClo, ep.C_lo, M, cols, ep.ldc))) {
            pC = &mC;
            pClo = ep.C_lo ? &mClo : nullptr;
            a.tma_store = 1;
        }
    }
    if (prep)
        return bn == 256 ? launch_tc<256, MODE_PREP>(mAh, mAl, W, a, M, st, pC, pClo)
                         : launch_tc<128, MODE_PREP>(mAh, mAl, W, a, M, st);
    if (fold) {
        a.tma_store = 0;
        return bn == 256 ? launch_tc<256, MODE_FOLD>(mAh, mAl, W, a, M, st)
                         : launch_tc<128, MODE_FOLD>(mAh, mAl, W, a, M, st);
    }
    if (bn == 256 && a.tma_store) return launch_tc<256, MODE_TMA>(mAh, mAl, W, a, M, st, pC, pClo);
    return bn == 256 ? launch_tc<256, MODE_GENERAL>(mAh, mAl, W, a, M, st)
                     : launch_tc<128, MODE_GENERAL>(mAh, mAl, W, a, M, st);
}

}  // namespace nk
