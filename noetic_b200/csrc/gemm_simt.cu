// gemm_simt.cu -- f32 CUDA-core projections: C = epilogue(A . B^T).
//
// A is [M, K] row-major (activations, K contiguous), B is [N, K] row-major
// (a weight stored [out, in] like every Linear in the reference, nn.rs:22).
// This is the exact-f32 engine: it serves small stream batches (GEMV-shaped,
// HBM-bound), shapes the tensor-core path does not take, and the f32 check of
// that path.  Reference arithmetic: tensor.rs:101-151 (gemm_nt) and
// tensor.rs:221-273 (matvec_nt); accumulation order differs (tree / tiled
// sums instead of four strided accumulators), so results agree to f32
// rounding, not bit-for-bit.
//
// Epilogue: v = acc (+ bias[n]); out = v, or out = R[m, n] + v when a
// residual is given (the residual add of infer.rs:180-182 / 193-195, which
// adds the bias-complete projection to x).  C may alias R.

#include "nk_kernels.h"
#include "nk_common.cuh"

namespace nk {

namespace {

constexpr int BM = 128, BN = 128, BK = 8, PAD = 4;

template <bool VEC>
__device__ __forceinline__ void load_tile(const float *__restrict__ P, int ld, int rows, int K,
                                          int r0, int k0, int tid, float4 &v) {
    const int r = tid >> 1, kq = (tid & 1) * 4;
    const int gr = r0 + r, gk = k0 + kq;
    if (VEC) {
        if (gr < rows && gk + 3 < K) {
            v = *reinterpret_cast<const float4 *>(P + (size_t)gr * ld + gk);
        } else {
            v.x = (gr < rows && gk + 0 < K) ? P[(size_t)gr * ld + gk + 0] : 0.0f;
            v.y = (gr < rows && gk + 1 < K) ? P[(size_t)gr * ld + gk + 1] : 0.0f;
            v.z = (gr < rows && gk + 2 < K) ? P[(size_t)gr * ld + gk + 2] : 0.0f;
            v.w = (gr < rows && gk + 3 < K) ? P[(size_t)gr * ld + gk + 3] : 0.0f;
        }
    } else {
        v.x = (gr < rows && gk + 0 < K) ? P[(size_t)gr * ld + gk + 0] : 0.0f;
        v.y = (gr < rows && gk + 1 < K) ? P[(size_t)gr * ld + gk + 1] : 0.0f;
        v.z = (gr < rows && gk + 2 < K) ? P[(size_t)gr * ld + gk + 2] : 0.0f;
        v.w = (gr < rows && gk + 3 < K) ? P[(size_t)gr * ld + gk + 3] : 0.0f;
    }
}

__device__ __forceinline__ void store_tile(float (*S)[BM + PAD], int tid, const float4 &v) {
    const int r = tid >> 1, kq = (tid & 1) * 4;
    S[kq + 0][r] = v.x;
    S[kq + 1][r] = v.y;
    S[kq + 2][r] = v.z;
    S[kq + 3][r] = v.w;
}

// 128x128 tile, 256 threads, 8x8 outputs per thread (two 4x4 quadrants per
// axis so shared-memory reads are conflict-free float4s), register-staged
// double buffering over K in steps of 8.
template <bool VEC>
__global__ void __launch_bounds__(256) gemm_nt_tiled(GemmArgs p) {
    __shared__ __align__(16) float As[2][BK][BM + PAD];
    __shared__ __align__(16) float Bs[2][BK][BN + PAD];
    const int tid = threadIdx.x;
    const int tx = tid & 15, ty = tid >> 4;
    const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
    const int K = p.K;

    float acc[8][8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = 0.0f;

    float4 ra, rb;
    load_tile<VEC>(p.A, p.lda, p.M, K, m0, 0, tid, ra);
    load_tile<VEC>(p.B, p.ldb, p.N, K, n0, 0, tid, rb);
    store_tile(As[0], tid, ra);
    store_tile(Bs[0], tid, rb);
    __syncthreads();

    const int ktiles = (K + BK - 1) / BK;
    for (int kt = 0; kt < ktiles; ++kt) {
        const int cur = kt & 1;
        const bool more = kt + 1 < ktiles;
        if (more) {
            load_tile<VEC>(p.A, p.lda, p.M, K, m0, (kt + 1) * BK, tid, ra);
            load_tile<VEC>(p.B, p.ldb, p.N, K, n0, (kt + 1) * BK, tid, rb);
        }
#pragma unroll
        for (int kk = 0; kk < BK; ++kk) {
            float a[8], b[8];
            float4 t;
            t = *reinterpret_cast<const float4 *>(&As[cur][kk][ty * 4]);
            a[0] = t.x; a[1] = t.y; a[2] = t.z; a[3] = t.w;
            t = *reinterpret_cast<const float4 *>(&As[cur][kk][64 + ty * 4]);
            a[4] = t.x; a[5] = t.y; a[6] = t.z; a[7] = t.w;
            t = *reinterpret_cast<const float4 *>(&Bs[cur][kk][tx * 4]);
            b[0] = t.x; b[1] = t.y; b[2] = t.z; b[3] = t.w;
            t = *reinterpret_cast<const float4 *>(&Bs[cur][kk][64 + tx * 4]);
            b[4] = t.x; b[5] = t.y; b[6] = t.z; b[7] = t.w;
#pragma unroll
            for (int i = 0; i < 8; ++i)
#pragma unroll
                for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
        }
        if (more) {
            store_tile(As[cur ^ 1], tid, ra);
            store_tile(Bs[cur ^ 1], tid, rb);
        }
        __syncthreads();
    }

#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int m = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + (i - 4));
        if (m >= p.M) continue;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int n = n0 + (j < 4 ? tx * 4 + j : 64 + tx * 4 + (j - 4));
            if (n >= p.N) continue;
            float v = acc[i][j];
            if (p.bias) v = v + p.bias[n];
            if (p.R) v = p.R[(size_t)m * p.ldr + n] + v;
            p.C[(size_t)m * p.ldc + n] = v;
        }
    }
}

// Skinny GEMM (M <= GEMV_MAX_ROWS): each warp produces WARP_ROWS output
// features for every row of A.  The weight rows stream once from HBM with
// 16-byte loads; A sits in shared memory.  This is the batch-1 decode
// projection (matvec_nt, tensor.rs:221-245).
constexpr int WARP_ROWS = 2;

template <int MR, bool VEC>
__global__ void __launch_bounds__(256) gemv_nt(GemmArgs p) {
    extern __shared__ __align__(16) float xs[];  // [MR][K]
    const int K = p.K;
    for (int i = threadIdx.x; i < MR * K; i += blockDim.x) {
        const int r = i / K, k = i - r * K;
        xs[i] = (r < p.M) ? p.A[(size_t)r * p.lda + k] : 0.0f;
    }
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n_base = (blockIdx.x * (blockDim.x >> 5) + warp) * WARP_ROWS;
    float acc[WARP_ROWS][MR];
#pragma unroll
    for (int w = 0; w < WARP_ROWS; ++w)
#pragma unroll
        for (int r = 0; r < MR; ++r) acc[w][r] = 0.0f;

    if (VEC) {
        const int K4 = K >> 2;
#pragma unroll
        for (int w = 0; w < WARP_ROWS; ++w) {
            const int n = n_base + w;
            if (n >= p.N) break;
            const float4 *wr = reinterpret_cast<const float4 *>(p.B + (size_t)n * p.ldb);
#pragma unroll 4
            for (int k4 = lane; k4 < K4; k4 += 32) {
                const float4 wv = __ldg(wr + k4);
#pragma unroll
                for (int r = 0; r < MR; ++r) {
                    const float4 xv = *reinterpret_cast<const float4 *>(xs + r * K + 4 * k4);
                    float a = acc[w][r];
                    a = fmaf(wv.x, xv.x, a);
                    a = fmaf(wv.y, xv.y, a);
                    a = fmaf(wv.z, xv.z, a);
                    a = fmaf(wv.w, xv.w, a);
                    acc[w][r] = a;
                }
            }
        }
    } else {
#pragma unroll
        for (int w = 0; w < WARP_ROWS; ++w) {
            const int n = n_base + w;
            if (n >= p.N) break;
            const float *wr = p.B + (size_t)n * p.ldb;
            for (int k = lane; k < K; k += 32) {
                const float wv = __ldg(wr + k);
#pragma unroll
                for (int r = 0; r < MR; ++r) acc[w][r] = fmaf(wv, xs[r * K + k], acc[w][r]);
            }
        }
    }
#pragma unroll
    for (int w = 0; w < WARP_ROWS; ++w) {
        const int n = n_base + w;
#pragma unroll
        for (int r = 0; r < MR; ++r) {
            const float s = warp_sum(acc[w][r]);
            if (lane == 0 && n < p.N && r < p.M) {
                float v = s;
                if (p.bias) v = v + p.bias[n];
                if (p.R) v = p.R[(size_t)r * p.ldr + n] + v;
                p.C[(size_t)r * p.ldc + n] = v;
            }
        }
    }
}

template <int MR>
cudaError_t launch_gemv(const GemmArgs &p, cudaStream_t st) {
    const int warps = 8;
    const int per_cta = warps * WARP_ROWS;
    dim3 grid((p.N + per_cta - 1) / per_cta);
    const size_t smem = (size_t)MR * p.K * sizeof(float);
    const bool vec = (p.K % 4 == 0) && (p.ldb % 4 == 0) && ((uintptr_t)p.B % 16 == 0);
    if (vec) {
        if (smem > 48 * 1024)
            cudaFuncSetAttribute(gemv_nt<MR, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        gemv_nt<MR, true><<<grid, warps * 32, smem, st>>>(p);
    } else {
        if (smem > 48 * 1024)
            cudaFuncSetAttribute(gemv_nt<MR, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        gemv_nt<MR, false><<<grid, warps * 32, smem, st>>>(p);
    }
    return cudaGetLastError();
}

}  // namespace

size_t gemv_smem_bytes(int m, int k) { return (size_t)(m <= 1 ? 1 : m <= 2 ? 2 : m <= 4 ? 4 : 8) * k * 4; }

cudaError_t gemm_nt_simt(const GemmArgs &p, cudaStream_t st) {
    if (p.M <= 0 || p.N <= 0) return cudaSuccess;
    if (p.M <= GEMV_MAX_ROWS && gemv_smem_bytes(p.M, p.K) <= 200 * 1024) {
        if (p.M <= 1) return launch_gemv<1>(p, st);
        if (p.M <= 2) return launch_gemv<2>(p, st);
        if (p.M <= 4) return launch_gemv<4>(p, st);
        return launch_gemv<8>(p, st);
    }
    dim3 grid((p.N + BN - 1) / BN, (p.M + BM - 1) / BM);
    const bool vec = (p.K % 4 == 0) && (p.lda % 4 == 0) && (p.ldb % 4 == 0) &&
                     ((uintptr_t)p.A % 16 == 0) && ((uintptr_t)p.B % 16 == 0);
    if (vec)
        gemm_nt_tiled<true><<<grid, 256, 0, st>>>(p);
    else
        gemm_nt_tiled<false><<<grid, 256, 0, st>>>(p);
    return cudaGetLastError();
}

}  // namespace nk
