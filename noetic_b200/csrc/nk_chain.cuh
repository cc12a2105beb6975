// nk_chain.cuh -- carries between the time blocks of a one-pass scan.
//
// A one-pass scan gives every CTA one time block of one chain (a row of the
// scan: one stream or batch entry and a group of 32 channels, lane = channel)
// and passes the state between consecutive blocks of a chain through global
// memory, by decoupled look-back: a block publishes its map h_out = A h_in + B
// (status 1), walks back over the published maps of its predecessors until it
// meets one that has published its inclusive value (status 2), composes them
// ((A_L, B_L) then (A_R, B_R) = (A_R A_L, A_R B_L + B_R), scan.rs:5-8), and
// publishes its own inclusive value.
//
// Every published value travels in one 64-bit word together with its status
// (status in the high half, the f32 bits in the low half), written and read
// with single relaxed 64-bit accesses at GPU scope: a reader sees either the
// cleared word or the complete one, so no fence orders a value against a
// separate flag.  Each lane (channel) walks back on its own words.
//
// CTAs take their blocks from a ticket counter, ticket = block * n_chains +
// chain, so every predecessor of a block holds a smaller ticket and was taken
// by a running CTA before it; a block publishes its map before it waits for
// anything, so every wait ends.  The wait is still bounded: on expiry it
// writes an error code, takes a zero carry and returns, and the host reports
// the code.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace nk {

// Scratch of a one-pass scan with `slots` blocks: a 16-byte header (ticket
// counter, error word), then per block three words per lane: A and B of the
// block's map and its inclusive value.  All of it must be zero at launch
// (chain_ws_bytes from the start).
struct ChainWs {
    int *ticket;
    int *err;
    unsigned long long *words;  // [slots][3][32]
};

inline size_t chain_ws_bytes(size_t slots) { return 16 + 8 * 96 * slots; }
inline ChainWs chain_ws(void *base, size_t) {
    int *w = reinterpret_cast<int *>(base);
    ChainWs ws;
    ws.ticket = w;
    ws.err = w + 1;
    ws.words = reinterpret_cast<unsigned long long *>(w + 4);
    return ws;
}

constexpr uint64_t CHAIN_WAIT_NS = 1000000000ull;

__device__ __forceinline__ uint64_t chain_gtimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void chain_put(unsigned long long *p, uint32_t status, float v) {
    const unsigned long long w = ((unsigned long long)status << 32) | __float_as_uint(v);
    asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}

__device__ __forceinline__ unsigned long long chain_get(const unsigned long long *p) {
    unsigned long long w;
    asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
    return w;
}

__device__ __forceinline__ uint32_t chain_status(unsigned long long w) { return (uint32_t)(w >> 32); }
__device__ __forceinline__ float chain_value(unsigned long long w) { return __uint_as_float((uint32_t)w); }

// Called by one full warp (lane = channel) with the CTA's block map (eA, eB);
// returns the lane's state entering the block.  tk is the CTA's ticket;
// blocks with tk < n_chains start their chain and enter with `first` (the
// chain's initial state).  err_code is written to *ws.err (and *err_extra
// when given) if a wait expires.
__device__ __forceinline__ float chain_carry(const ChainWs &ws, int64_t tk, int64_t n_chains, float eA, float eB,
                                             float first, int err_code, int *err_extra) {
    const int lane = threadIdx.x & 31;
    unsigned long long *mine = ws.words + (size_t)tk * 96 + lane;
    if (tk < n_chains) {
        chain_put(mine + 64, 2u, fmaf(eA, first, eB));
        return first;
    }
    chain_put(mine, 1u, eA);
    chain_put(mine + 32, 1u, eB);
    float accA = 1.0f, accB = 0.0f, cin = 0.0f;
    int64_t jb = tk - n_chains;
    uint64_t t0 = 0;
    bool timed = false;
    for (;;) {
        const unsigned long long *pw = ws.words + (size_t)jb * 96 + lane;
        const unsigned long long wi = chain_get(pw + 64), wa = chain_get(pw), wb = chain_get(pw + 32);
        if (chain_status(wi) == 2u) {
            cin = fmaf(accA, chain_value(wi), accB);
            break;
        }
        if (chain_status(wa) == 1u && chain_status(wb) == 1u) {
            accB = fmaf(accA, chain_value(wb), accB);
            accA = accA * chain_value(wa);
            jb -= n_chains;  // a chain's first block publishes its inclusive value, so jb stays >= 0
            continue;
        }
        __nanosleep(32);
        if (!timed) {
            t0 = chain_gtimer();
            timed = true;
        } else if (chain_gtimer() - t0 > CHAIN_WAIT_NS) {
            atomicExch(ws.err, err_code);
            if (err_extra) atomicExch(err_extra, err_code);
            cin = 0.0f;
            break;
        }
    }
    chain_put(mine + 64, 2u, fmaf(eA, cin, eB));
    return cin;
}

}  // namespace nk
