// nk_common.cuh -- device helpers shared by the token-loop kernels.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace nk {

// tensor.rs:276-283: the branchy stable sigmoid, 1 / (1 + e^-x) for x >= 0
// and e^x / (1 + e^x) below, written without a branch: e = exp(-|x|) is the
// exponential either branch takes, and the numerator is 1 or e, so each
// lane performs exactly its branch's operations while a warp with inputs of
// both signs runs one exp and one division instead of both paths.  CUDA's
// expf is used (the reference calls the platform libm expf); results agree
// within expf's error bound, not bit-for-bit.  NaN propagates as in the
// reference's second branch.
__device__ __forceinline__ float sigmoid(float x) {
    const bool pos = x >= 0.0f;
    const float e = expf(pos ? -x : x);
    return (pos ? 1.0f : e) / (1.0f + e);
}

__device__ __forceinline__ float silu(float x) { return x * sigmoid(x); }

// The recurrent branch of one decode step for one (stream, channel),
// infer.rs:155-176: write v into the conv ring at `head` (the already
// advanced slot), causal conv over the ring (taps q = 0..k-1, q ascending),
// SiLU, sigmoid decay, h = decay h + (1 - decay) value, output gate.  ring is
// the stream's layer state [k+1][E] (row k = h).  Returns the gated output.
// The same operations, in the same order, as ssm_decode_k.  K > 0 fixes
// the conv width at compile time (k_dyn must equal it); K = 0 takes k_dyn.
template <int K>
__device__ __forceinline__ float ssm_step_channel(float v, float z, float o, float *ring, uint32_t head, int k_dyn,
                                                  int E, int j, const float *conv_w, const float *conv_b) {
    const int k = K > 0 ? K : k_dyn;
    float sum = conv_b[j] + conv_w[j] * v;
    ring[(size_t)head * E + j] = v;
#pragma unroll
    for (int q = 1; q < (K > 0 ? K : 64); ++q) {
        if (q >= k) break;
        const uint32_t slot = (head + (uint32_t)k - (uint32_t)q) % (uint32_t)k;
        sum = sum + conv_w[(size_t)q * E + j] * ring[(size_t)slot * E + j];
    }
    const float value = silu(sum);
    const float decay = sigmoid(z);
    const float h = decay * ring[(size_t)k * E + j] + (1.0f - decay) * value;
    ring[(size_t)k * E + j] = h;
    return h * silu(o);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// ---- xoshiro256++ (rng.rs:46-56), f32_unit (rng.rs:65-67), below (rng.rs:75-90)
__device__ __forceinline__ uint64_t rotl64(uint64_t x, int k) { return (x << k) | (x >> (64 - k)); }

__device__ __forceinline__ uint64_t xoshiro_next(uint64_t s[4]) {
    const uint64_t result = rotl64(s[0] + s[3], 23) + s[0];
    const uint64_t t = s[1] << 17;
    s[2] ^= s[0];
    s[3] ^= s[1];
    s[1] ^= s[2];
    s[0] ^= s[3];
    s[2] ^= t;
    s[3] = rotl64(s[3], 45);
    return result;
}

__device__ __forceinline__ float xoshiro_f32_unit(uint64_t s[4]) {
    return (float)(xoshiro_next(s) >> 40) * (1.0f / 16777216.0f);
}

// Lemire threshold rejection then modulo.  The expected number of draws is
// below 2 for every n; the loop is capped (a cap that can only be reached
// with probability < 2^-64) so that a corrupted state cannot spin forever.
__device__ __forceinline__ uint64_t xoshiro_below(uint64_t s[4], uint64_t n, int *err) {
    if (n <= 1) return 0;
    const uint64_t threshold = (0ull - n) % n;
    for (int it = 0; it < 64; ++it) {
        uint64_t r = xoshiro_next(s);
        if (r >= threshold) return r % n;
    }
    if (err) *err = 1;
    return 0;
}

// f32::total_cmp as an order-preserving signed integer.
__device__ __forceinline__ int32_t total_key(float f) {
    int32_t b = __float_as_int(f);
    return b ^ (int32_t)((uint32_t)(b >> 31) >> 1);
}

// 3xTF32 operand split: hi keeps the tf32-representable leading bits
// (round to nearest, ties away), lo is the exact remainder rounded to tf32.
__device__ __forceinline__ float tf32_round(float x) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
    return __uint_as_float(r);
}

// Programmatic dependent launch.  A kernel launched with programmatic stream
// serialization (pdl_launch) may start while its predecessor in the stream
// is still running: pdl_wait() blocks until the predecessor grid has
// completed and its writes are visible, pdl_trigger() lets the successor
// start its own prologue.  Launched normally, both are no-ops.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <class... KArgs, class... Args>
inline cudaError_t pdl_launch(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args &&...args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

}  // namespace nk
