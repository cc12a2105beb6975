// train.cu -- the training-side ops around the scan: gemm_tn (the weight-
// gradient product, tensor.rs:156-198), the depthwise-conv backward
// (Op::DwConv, autograd.rs:1050-1097) and the fused AdamW step
// (optim.rs:33-72).  All three are HBM- or FMA-bound elementwise / GEMM
// work in f32.

#include <algorithm>

#include "nk_common.cuh"
#include "nk_kernels.h"
#include "nk_tc.h"

namespace nk {

namespace {

// ---------------------------------------------------------------- gemm_tn
// C[m, n] = sum_q A[q, m] B[q, n].  A 64 x 64 tile of C per 256-thread
// block, 4 x 4 outputs per thread, 16 rows of A and B staged in shared
// memory per step.  Both operands are contiguous along m / n, so the tile
// loads coalesce without a transpose.  A zero element of A skips its
// product, as kern_tn does (a zero times a non-finite B adds nothing).
constexpr int TN_BM = 64, TN_BN = 64, TN_BK = 16;

// only_if != nullptr: do nothing unless *only_if is set (the exact
// recomputation behind the tensor-core path, see gemm_tn_tc).
__global__ void __launch_bounds__(256) gemm_tn_k(const float *__restrict__ A, const float *__restrict__ B,
                                                 float *__restrict__ C, int64_t p, int m, int n,
                                                 const int *only_if) {
    if (only_if && *only_if == 0) return;
    __shared__ __align__(16) float As[TN_BK][TN_BM];
    __shared__ __align__(16) float Bs[TN_BK][TN_BN];
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    const int m0 = blockIdx.y * TN_BM, n0 = blockIdx.x * TN_BN;
    float acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = 0.0f;
    for (int64_t q0 = 0; q0 < p; q0 += TN_BK) {
#pragma unroll
        for (int l = 0; l < (TN_BK * TN_BM) / 256; ++l) {
            const int i = threadIdx.x + l * 256, r = i / TN_BM, c = i % TN_BM;
            const int64_t q = q0 + r;
            As[r][c] = (q < p && m0 + c < m) ? A[q * m + m0 + c] : 0.0f;
            Bs[r][c] = (q < p && n0 + c < n) ? B[q * n + n0 + c] : 0.0f;
        }
        __syncthreads();
#pragma unroll
        for (int r = 0; r < TN_BK; ++r) {
            const float4 a4 = *reinterpret_cast<const float4 *>(&As[r][ty * 4]);
            const float4 b4 = *reinterpret_cast<const float4 *>(&Bs[r][tx * 4]);
            const float a[4] = {a4.x, a4.y, a4.z, a4.w}, b[4] = {b4.x, b4.y, b4.z, b4.w};
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = a[i] == 0.0f ? acc[i][j] : fmaf(a[i], b[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int mm = m0 + ty * 4 + i;
        if (mm >= m) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int nn = n0 + tx * 4 + j;
            if (nn < n) C[(size_t)mm * n + nn] = acc[i][j];
        }
    }
}

// ---------------------------------------------------------------- dwconv backward
// gx[b, s, j] += sum_{q < k, s + q < t} go[b, s + q, j] w[q, j]: one thread
// per element, q ascending, a rounded product then a rounded add -- the
// order in which the reference's loop (ti ascending, src = ti - q) adds
// into each gx element, so the result is bit-identical.
__global__ void dwconv_gx_k(const float *__restrict__ w, const float *__restrict__ go, float *__restrict__ gx,
                            int64_t rows, int64_t t, int d, int k) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= rows * d) return;
    const int64_t row = i / d;
    const int j = (int)(i - row * d);
    const int64_t s = row % t;
    float acc = gx[i];
    for (int q = 0; q < k && s + q < t; ++q)
        acc = __fadd_rn(acc, __fmul_rn(go[i + (int64_t)q * d], w[(size_t)q * d + j]));
    gx[i] = acc;
}

// The same with four channels per thread (d % 4 == 0): threadIdx.x walks
// channel quads, threadIdx.y and the grid's y walk rows.
__global__ void __launch_bounds__(256) dwconv_gx4_k(const float4 *__restrict__ w, const float4 *__restrict__ go,
                                                    float4 *__restrict__ gx, int64_t rows, int64_t t, int d4, int k) {
    const int j4 = blockIdx.x * 64 + threadIdx.x;
    if (j4 >= d4) return;
    const int64_t step = (int64_t)gridDim.y * 4;
    for (int64_t row = (int64_t)blockIdx.y * 4 + threadIdx.y; row < rows; row += step) {
        const int64_t s = row % t;
        const size_t i = (size_t)row * d4 + j4;
        float4 acc = gx[i];
        for (int q = 0; q < k && s + q < t; ++q) {
            const float4 g = go[i + (size_t)q * d4], wq = w[(size_t)q * d4 + j4];
            acc.x = __fadd_rn(acc.x, __fmul_rn(g.x, wq.x));
            acc.y = __fadd_rn(acc.y, __fmul_rn(g.y, wq.y));
            acc.z = __fadd_rn(acc.z, __fmul_rn(g.z, wq.z));
            acc.w = __fadd_rn(acc.w, __fmul_rn(g.w, wq.w));
        }
        gx[i] = acc;
    }
}

constexpr int DW_ROWS = 1024;  // rows per partial-sum chunk
constexpr int DW_KMAX = 16;    // conv widths the weight-gradient kernel takes

// Partial sums of gw[q, j] = sum go[b, ti, j] x[b, ti - q, j] (ti >= q) and
// gb[j] = sum go[., j] over one chunk of DW_ROWS rows and 32 channels: lane
// = channel, the 8 warps split the rows, then a fixed-order sum over the
// warps.  part [chunk][k + 1][d] (row k is the bias).
__global__ void __launch_bounds__(256) dwconv_wgrad_part_k(const float *__restrict__ x, const float *__restrict__ go,
                                                           float *__restrict__ part, int64_t rows, int64_t t, int d,
                                                           int k) {
    __shared__ float red[8][DW_KMAX + 1][32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int j = blockIdx.y * 32 + lane;
    const int64_t r0 = (int64_t)blockIdx.x * DW_ROWS, r1 = min(rows, r0 + DW_ROWS);
    float acc[DW_KMAX + 1];
#pragma unroll
    for (int q = 0; q <= DW_KMAX; ++q) acc[q] = 0.0f;
    if (j < d) {
        int64_t ti = (r0 + warp) % t;  // time index of the row, advanced without a division
        for (int64_t row = r0 + warp; row < r1; row += 8) {
            const float g = go[row * d + j];
            acc[DW_KMAX] += g;
#pragma unroll
            for (int q = 0; q < DW_KMAX; ++q)
                if (q < k && ti >= q) acc[q] = fmaf(g, x[(row - q) * d + j], acc[q]);
            ti += 8;
            while (ti >= t) ti -= t;
        }
    }
#pragma unroll
    for (int q = 0; q <= DW_KMAX; ++q) red[warp][q][lane] = acc[q];
    __syncthreads();
    for (int e = threadIdx.x; e < (k + 1) * 32; e += blockDim.x) {
        const int q = e / 32, l = e % 32, jj = blockIdx.y * 32 + l;
        const int slot = q == k ? DW_KMAX : q;
        float s = 0.0f;
        for (int w8 = 0; w8 < 8; ++w8) s += red[w8][slot][l];
        if (jj < d) part[((size_t)blockIdx.x * (k + 1) + q) * d + jj] = s;
    }
}

// The same partial sums with four channels per lane (d % 4 == 0; 128
// channels per block), for conv widths k <= KT.
template <int KT>
__global__ void __launch_bounds__(256) dwconv_wgrad_part4_k(const float4 *__restrict__ x, const float4 *__restrict__ go,
                                                            float *__restrict__ part, int64_t rows, int64_t t, int d4,
                                                            int k) {
    __shared__ float4 red[8][32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int j4 = blockIdx.y * 32 + lane;
    const int64_t r0 = (int64_t)blockIdx.x * DW_ROWS, r1 = min(rows, r0 + DW_ROWS);
    float4 acc[KT + 1];
#pragma unroll
    for (int q = 0; q <= KT; ++q) acc[q] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (j4 < d4) {
        int64_t ti = (r0 + warp) % t;
        for (int64_t row = r0 + warp; row < r1; row += 8) {
            const float4 g = go[(size_t)row * d4 + j4];
            acc[KT].x += g.x;
            acc[KT].y += g.y;
            acc[KT].z += g.z;
            acc[KT].w += g.w;
#pragma unroll
            for (int q = 0; q < KT; ++q)
                if (q < k && ti >= q) {
                    const float4 xv = x[(size_t)(row - q) * d4 + j4];
                    acc[q].x = fmaf(g.x, xv.x, acc[q].x);
                    acc[q].y = fmaf(g.y, xv.y, acc[q].y);
                    acc[q].z = fmaf(g.z, xv.z, acc[q].z);
                    acc[q].w = fmaf(g.w, xv.w, acc[q].w);
                }
            ti += 8;
            while (ti >= t) ti -= t;
        }
    }
    // Fixed-order sum over the 8 warps, one gradient row at a time.
#pragma unroll
    for (int q = 0; q <= KT; ++q) {
        if (q < k || q == KT) {
            red[warp][lane] = acc[q];
            __syncthreads();
            if (warp == 0 && j4 < d4) {
                float4 sum = red[0][lane];
                for (int w8 = 1; w8 < 8; ++w8) {
                    const float4 o = red[w8][lane];
                    sum.x += o.x;
                    sum.y += o.y;
                    sum.z += o.z;
                    sum.w += o.w;
                }
                const int qo = q == KT ? k : q;
                reinterpret_cast<float4 *>(part + ((size_t)blockIdx.x * (k + 1) + qo) * (size_t)d4 * 4)[j4] = sum;
            }
            __syncthreads();
        }
    }
}

// gw[q, j] += sum over chunks in order; gb[j] likewise (row k).
__global__ void dwconv_wgrad_sum_k(const float *__restrict__ part, int chunks, float *__restrict__ gw,
                                   float *__restrict__ gb, int d, int k) {
    const int e = blockIdx.x * blockDim.x + threadIdx.x;
    if (e >= (k + 1) * d) return;
    const int q = e / d, j = e - q * d;
    float *dst = q < k ? (gw ? gw + (size_t)q * d + j : nullptr) : (gb ? gb + j : nullptr);
    if (!dst) return;
    float s = *dst;
    for (int c = 0; c < chunks; ++c) s += part[((size_t)c * (k + 1) + q) * d + j];
    *dst = s;
}

// ---------------------------------------------------------------- AdamW
// One element per thread, every operation a correctly rounded f32 product,
// sum, quotient or square root in the reference's order, so the update is
// bit-identical to it.  A non-finite gradient or parameter leaves that
// element untouched and sets *err = 4.
__global__ void adamw_k(float *__restrict__ val, const float *__restrict__ grad, float *__restrict__ m,
                        float *__restrict__ v, int64_t n, AdamwParams a, int *err) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const float gr = grad[i], pv = val[i];
        if (!isfinite(gr) || !isfinite(pv)) {
            atomicExch(err, 4);
            continue;
        }
        const float mi = __fadd_rn(__fmul_rn(a.b1, m[i]), __fmul_rn(__fsub_rn(1.0f, a.b1), gr));
        const float vi = __fadd_rn(__fmul_rn(a.b2, v[i]), __fmul_rn(__fmul_rn(__fsub_rn(1.0f, a.b2), gr), gr));
        m[i] = mi;
        v[i] = vi;
        const float mh = __fmul_rn(mi, a.inv_bc1), vh = __fmul_rn(vi, a.inv_bc2);
        float upd = __fdiv_rn(mh, __fadd_rn(__fsqrt_rn(vh), a.eps));
        if (a.decay && a.wd != 0.0f) upd = __fadd_rn(upd, __fmul_rn(a.wd, pv));
        val[i] = __fsub_rn(pv, __fmul_rn(a.lr, upd));
    }
}

__device__ __forceinline__ bool adamw_one(float &pv, float gr, float &mv, float &vv, const AdamwParams &a) {
    if (!isfinite(gr) || !isfinite(pv)) return false;
    const float mi = __fadd_rn(__fmul_rn(a.b1, mv), __fmul_rn(__fsub_rn(1.0f, a.b1), gr));
    const float vi = __fadd_rn(__fmul_rn(a.b2, vv), __fmul_rn(__fmul_rn(__fsub_rn(1.0f, a.b2), gr), gr));
    mv = mi;
    vv = vi;
    const float mh = __fmul_rn(mi, a.inv_bc1), vh = __fmul_rn(vi, a.inv_bc2);
    float upd = __fdiv_rn(mh, __fadd_rn(__fsqrt_rn(vh), a.eps));
    if (a.decay && a.wd != 0.0f) upd = __fadd_rn(upd, __fmul_rn(a.wd, pv));
    pv = __fsub_rn(pv, __fmul_rn(a.lr, upd));
    return true;
}

// Four elements per thread and iteration (16-byte accesses); the same
// per-element arithmetic as adamw_k.  An element with a non-finite gradient
// or parameter keeps its old value and moments.
__global__ void adamw4_k(float4 *__restrict__ val, const float4 *__restrict__ grad, float4 *__restrict__ m,
                         float4 *__restrict__ v, int64_t n4, AdamwParams a, int *err) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
        const float4 g = grad[i];
        float4 p = val[i], mm = m[i], vv = v[i];
        bool ok = adamw_one(p.x, g.x, mm.x, vv.x, a);  // false: left as it was
        ok &= adamw_one(p.y, g.y, mm.y, vv.y, a);
        ok &= adamw_one(p.z, g.z, mm.z, vv.z, a);
        ok &= adamw_one(p.w, g.w, mm.w, vv.w, a);
        if (!ok) atomicExch(err, 4);
        val[i] = p;
        m[i] = mm;
        v[i] = vv;
    }
}

int sm_count_train() {
    static int n = 0;
    if (!n) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        if (n <= 0) n = 1;
    }
    return n;
}

}  // namespace

cudaError_t gemm_tn(const float *a, const float *b, float *c, int64_t p, int m, int n, cudaStream_t st) {
    if (m <= 0 || n <= 0) return cudaSuccess;
    const dim3 grid((unsigned)((n + TN_BN - 1) / TN_BN), (unsigned)((m + TN_BM - 1) / TN_BM));
    gemm_tn_k<<<grid, 256, 0, st>>>(a, b, c, p, m, n, nullptr);
    return cudaGetLastError();
}

// The tensor-core form: C = (A^T)(B^T)^T on the tcgen05 3xTF32 projection
// engine.  Both operands are split (tf32 hi + tf32 remainder) straight into
// K-major form by a transposing split, K = p padded to a multiple of 4 with
// zeros; stream-K spreads the long K over the SMs.  A zero element of A
// times inf / NaN in B is not a skipped product on the tensor core, so when
// either operand holds a non-finite value (flagged by the splits) the exact
// kernel recomputes C on the device.
static int64_t round4(int64_t v) { return (v + 3) & ~int64_t(3); }

bool gemm_tn_tc_eligible(int64_t p, int m, int n) {
    const int64_t p4 = round4(p);
    return p >= 8 && p4 < (int64_t)65535 * 32 && tc_eligible(m, n, (int)p4);
}

size_t gemm_tn_tc_scratch_floats(int64_t p, int m, int n) {
    return (size_t)2 * (size_t)(m + n) * (size_t)round4(p) + tc_stream_k_ws_floats();
}

int gemm_tn_tc_flag_ints() { return 2 + sm_count_train(); }

cudaError_t gemm_tn_tc(const float *a, const float *b, float *c, int64_t p, int m, int n, float *scratch, int *flags,
                       cudaStream_t st) {
    const int p4 = (int)round4(p);
    float *Ahi = scratch, *Alo = Ahi + (size_t)m * p4, *Bhi = Alo + (size_t)m * p4, *Blo = Bhi + (size_t)n * p4;
    float *ws = Blo + (size_t)n * p4;
    cudaError_t e = tc_split_transposed(a, (int)p, m, p4, Ahi, Alo, flags, st);
    if (e != cudaSuccess) return e;
    e = tc_split_transposed(b, (int)p, n, p4, Bhi, Blo, flags, st);
    if (e != cudaSuccess) return e;
    TcOperand W;
    if (!tc_operand_from(Bhi, Blo, n, p4, W)) return cudaErrorInvalidValue;
    TcEpilogue ep;
    ep.C = c;
    ep.ldc = n;
    ep.ws = ws;
    ep.ws_floats = tc_stream_k_ws_floats();
    ep.flags = flags + 2;
    ep.n_flags = sm_count_train();
    e = tc_gemm(Ahi, Alo, m, p4, W, ep, tc_pick_bn(m, n, false, true), st, flags + 1);
    if (e != cudaSuccess) return e;
    const dim3 grid((unsigned)((n + TN_BN - 1) / TN_BN), (unsigned)((m + TN_BM - 1) / TN_BM));
    gemm_tn_k<<<grid, 256, 0, st>>>(a, b, c, p, m, n, flags);
    return cudaGetLastError();
}

size_t dwconv_backward_scratch_floats(int64_t rows, int d, int k) {
    return (size_t)((rows + DW_ROWS - 1) / DW_ROWS) * (size_t)(k + 1) * (size_t)d;
}

int dwconv_max_k() { return DW_KMAX; }

cudaError_t dwconv_backward(const float *x, const float *w, const float *go, float *gx, float *gw, float *gb,
                            int64_t batch, int64_t t, int d, int k, float *scratch, cudaStream_t st) {
    const int64_t rows = batch * t;
    if (rows == 0 || d == 0) return cudaSuccess;
    if (gx) {
        const bool vec = d % 4 == 0 && ((uintptr_t)w | (uintptr_t)go | (uintptr_t)gx) % 16 == 0;
        if (vec) {
            const int d4 = d / 4;
            const dim3 grid((unsigned)((d4 + 63) / 64), (unsigned)std::min<int64_t>((rows + 3) / 4, 16384));
            dwconv_gx4_k<<<grid, dim3(64, 4), 0, st>>>(reinterpret_cast<const float4 *>(w),
                                                       reinterpret_cast<const float4 *>(go),
                                                       reinterpret_cast<float4 *>(gx), rows, t, d4, k);
        } else {
            const int64_t n = rows * d;
            dwconv_gx_k<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(w, go, gx, rows, t, d, k);
        }
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    if (gw || gb) {
        const int chunks = (int)((rows + DW_ROWS - 1) / DW_ROWS);
        const bool vec = d % 4 == 0 && ((uintptr_t)x | (uintptr_t)go | (uintptr_t)scratch) % 16 == 0;
        if (vec) {
            const int d4 = d / 4;
            const dim3 grid((unsigned)chunks, (unsigned)((d4 + 31) / 32));
            const float4 *x4 = reinterpret_cast<const float4 *>(x), *g4 = reinterpret_cast<const float4 *>(go);
            if (k <= 4)
                dwconv_wgrad_part4_k<4><<<grid, 256, 0, st>>>(x4, g4, scratch, rows, t, d4, k);
            else if (k <= 8)
                dwconv_wgrad_part4_k<8><<<grid, 256, 0, st>>>(x4, g4, scratch, rows, t, d4, k);
            else
                dwconv_wgrad_part4_k<16><<<grid, 256, 0, st>>>(x4, g4, scratch, rows, t, d4, k);
        } else {
            dwconv_wgrad_part_k<<<dim3((unsigned)chunks, (unsigned)((d + 31) / 32)), 256, 0, st>>>(x, go, scratch, rows,
                                                                                                     t, d, k);
        }
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return e;
        const int e_n = (k + 1) * d;
        dwconv_wgrad_sum_k<<<(unsigned)((e_n + 255) / 256), 256, 0, st>>>(scratch, chunks, gw, gb, d, k);
        return cudaGetLastError();
    }
    return cudaSuccess;
}

cudaError_t adamw_step(float *val, const float *grad, float *m, float *v, int64_t n, const AdamwParams &a, int *err,
                       cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    const bool vec = ((uintptr_t)val | (uintptr_t)grad | (uintptr_t)m | (uintptr_t)v) % 16 == 0;
    const int64_t n4 = vec ? n / 4 : 0;
    if (n4 > 0) {
        const int64_t blocks = std::min<int64_t>((n4 + 255) / 256, (int64_t)sm_count_train() * 16);
        adamw4_k<<<(unsigned)blocks, 256, 0, st>>>(reinterpret_cast<float4 *>(val), reinterpret_cast<const float4 *>(grad),
                                                    reinterpret_cast<float4 *>(m), reinterpret_cast<float4 *>(v), n4, a,
                                                    err);
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    const int64_t rest = n - 4 * n4;
    if (rest > 0) {
        const int64_t o = 4 * n4;
        const int64_t blocks = std::min<int64_t>((rest + 255) / 256, (int64_t)sm_count_train() * 16);
        adamw_k<<<(unsigned)blocks, 256, 0, st>>>(val + o, grad + o, m + o, v + o, rest, a, err);
    }
    return cudaGetLastError();
}

}  // namespace nk
