// nk_kernels.h -- host-side launchers of the token-loop kernels.
#pragma once

#include <cstddef>
#include <cstdint>
#include <string>
#include <cuda_runtime.h>

namespace nk {

// C[M,N] = (A[M,K] . B[N,K]^T) (+ bias[N]) (R[M,N] + ...).
struct GemmArgs {
    const float *A;
    int lda;
    const float *B;
    int ldb;
    float *C;
    int ldc;
    int M, N, K;
    const float *bias;  // nullable
    const float *R;     // nullable residual, may alias C
    int ldr;
};

constexpr int GEMV_MAX_ROWS = 8;

// Where a producer kernel writes its activations: f32 (f32 != nullptr), or
// the 3xTF32 operand pair hi = tf32(v), lo = tf32(v - hi) (hi, lo != nullptr)
// that the tensor-core projection consumes directly.
struct RowOut {
    float *f32;
    float *hi;
    float *lo;
};
inline RowOut f32_out(float *p) { return RowOut{p, nullptr, nullptr}; }

cudaError_t gemm_nt_simt(const GemmArgs &p, cudaStream_t st);

// ---- elementwise / row kernels (kernels_rows.cu)

// x[m,:] = emb[tokens[m],:]; tokens >= vocab set *err and read row 0.
cudaError_t embed_rows(const uint32_t *tokens, const float *emb, float *x, int M, int d, int vocab,
                       int *err, cudaStream_t st);

// Prompt-chunk gather: row (s, t) of x = emb[ids[s*max_t + t0 + t]] for
// t < tc (rows past a stream's length read token 0 and are ignored).
cudaError_t embed_prompt_chunk(const uint32_t *ids, const uint32_t *lens, int max_t, int t0, int tc,
                               const float *emb, float *x, int S, int d, int vocab, int *err,
                               cudaStream_t st);

// out = x * (1 / sqrt(mean(x^2) + eps)) * gain, per row (tensor.rs:298-312).
cudaError_t rmsnorm_rows(const float *x, const float *gain, float eps, RowOut out, int M, int d,
                         cudaStream_t st);

// heads[s] = (heads[s] + adv[s]) % k, adv == nullptr means +1.
cudaError_t advance_heads(uint32_t *heads, const uint32_t *adv, int S, int k, cudaStream_t st);
// heads[s] += clamp(lens[s] - t0, 0, tc) (mod k): a prompt chunk's advance.
cudaError_t advance_heads_prompt(uint32_t *heads, const uint32_t *lens, int t0, int tc, int S, int k,
                                 cudaStream_t st);

// One decode step of the recurrent branch for layer state [S][k+1][E]:
// ring write, causal conv, SiLU, sigmoid decay, h update, output gate
// (infer.rs:155-176).  heads[] are the already-advanced slots.
cudaError_t ssm_decode(const float *u, float *state, const uint32_t *heads, const float *conv_w,
                       const float *conv_b, RowOut g, int S, int E, int k, cudaStream_t st);

// Prefill of one prompt chunk for layer state [S][k+1][E] (sequential in time
// per (stream, channel)); y[S*tc, E]; heads[] are the slots at chunk start.
cudaError_t ssm_prefill_seq(const float *u, float *state, const uint32_t *heads,
                            const uint32_t *lens, int t0, int tc, const float *conv_w,
                            const float *conv_b, RowOut y, int S, int E, int k, cudaStream_t st);

// Same result, time-parallel: local scans over time blocks, carry composition,
// fix-up (the chunked associative scan of scan.rs:98-225 fused with the conv).
// y [S*tc, E] f32 holds the local scans; the gated output goes to yout.
cudaError_t ssm_prefill_chunked(const float *u, float *state, const uint32_t *heads,
                                const uint32_t *lens, int t0, int tc, const float *conv_w,
                                const float *conv_b, float *y, RowOut yout, float *scratch, int S, int E,
                                int k, cudaStream_t st);
size_t ssm_prefill_chunked_scratch_floats(int S, int E, int tc);
// Same result in one kernel: time blocks of 128 positions of 32 channels
// with carries by decoupled look-back; v, z and o read once, the gated output
// written once.  scratch of ssm_prefill_onepass_scratch_bytes (cleared by the
// call); an expired look-back wait writes 131 to *err.
cudaError_t ssm_prefill_onepass(const float *u, float *state, const uint32_t *heads, const uint32_t *lens, int t0,
                                int tc, const float *conv_w, const float *conv_b, RowOut yout, void *scratch, int S,
                                int E, int k, int *err, cudaStream_t st);
size_t ssm_prefill_onepass_scratch_bytes(int S, int E, int tc);

// s[m,j] = SiLU(up[m,j]) * up[m,H+j] (infer.rs:188-190).
cudaError_t swiglu_rows(const float *up, RowOut s, int M, int H, cudaStream_t st);

// out[m] = argmax over per-tile partial maxima (val/idx [M, n_tiles]).
cudaError_t argmax_partials(const float *val, const uint32_t *idx, int n_tiles, int M, uint32_t *out,
                            cudaStream_t st);

// out[m] = argmax(x[m,:]) (tensor.rs:354-365), first strict maximum, NaN skipped.
cudaError_t argmax_rows(const float *x, uint32_t *out, int M, int V, cudaStream_t st);

// Cross-entropy of one block of logits rows against targets (softmax_ce,
// autograd.rs:579-624): rows r of the block sit at sequence position
// s * T + t0 + (r0 + r) % tcc, s = (r0 + r) / tcc; nll / counted per position.
cudaError_t softmax_ce_rows(const float *logits, int rows, int V, int r0, int tcc, int T, int t0,
                            const uint32_t *targets, double *nll, uint32_t *counted, int *err, cudaStream_t st);
// Mean nll over counted positions (1 when none) into *out, fixed order.
cudaError_t ce_mean(const double *nll, const uint32_t *counted, size_t n, float *out, cudaStream_t st);

// Gather rows x[s*tc + (lens[s]-1-t0)] for streams whose last prompt token lies
// in [t0, t0+tc) into last[s].
cudaError_t gather_last_rows(const float *x, const uint32_t *lens, int t0, int tc, float *last,
                             int S, int d, cudaStream_t st);

// Row gather / scatter by index list.
cudaError_t gather_rows(const float *src, const uint32_t *idx, float *dst, int n, int d,
                        cudaStream_t st);
cudaError_t scatter_rows(const float *src, const uint32_t *idx, float *dst, int n, int d,
                         cudaStream_t st);

// ---- small-batch decode step (small_batch.cu): M <= GEMV_MAX_ROWS streams,
// four fused kernels per layer with L2 weight prefetch ahead of the
// programmatic-dependent-launch wait.
struct SmallLayer {
    const float *n1, *in_w, *in_b, *conv_w, *conv_b, *out_w, *out_b, *n2, *up_w, *up_b, *down_w, *down_b;
};
struct SmallStepArgs {
    const uint32_t *tokens;  // device [M]
    uint32_t *tokens_out;    // device [M] greedy choice, nullable
    const float *emb, *norm_f;
    float eps;
    float *x, *g, *state;    // x [M,d], g [M,max(E,H)], state [L][M][k+1][E]
    uint32_t *heads;
    float *logits;           // [M,V] nullable
    float *best_val;         // [M, small_logit_tiles(V)]
    uint32_t *best_idx;
    int *err;
    int M, d, E, H, k, V, n_layer;
    const SmallLayer *layers;  // host array [n_layer]
};
bool small_step_supported(int M, int d, int E, int H, int k);
int small_logit_tiles(int V);
cudaError_t small_step(const SmallStepArgs &a, cudaStream_t st, int *launches);

// ---- the whole decode step for 1..4 streams as one persistent cooperative
// kernel (decode_persistent.cu): two grid barriers per layer, the out and
// down projections read transposed (out_wT [E][d], down_wT [H][d]).
struct PersistLayer {
    const float *n1, *in_w, *in_b, *conv_w, *conv_b, *out_wT, *out_b, *n2, *up_w, *up_b, *down_wT, *down_b;
};
struct PersistStepArgs {
    const uint32_t *tokens;  // device [M]
    uint32_t *tokens_out;    // device [M] greedy choice, nullable
    const float *emb, *norm_f;
    float eps;
    float *state;            // [L][M][k+1][E]
    uint32_t *heads;
    float *logits;           // [M,V] nullable
    float *best_val;         // [M, persistent_partials()]
    uint32_t *best_idx;
    int *err;
    void *ws;                // persistent_ws_bytes(d): zero before the first launch and after an
                             // error; every completed launch leaves it zero
    const PersistLayer *layers;  // device array [n_layer]
    int M, d, E, H, k, V, n_layer;
    // Grid-barrier wait bound in ns (0: 1 s).  Test control: with
    // withhold_arrival CTA 0 skips its first barrier arrival, so every CTA's
    // wait runs out and the kernel reports code 113 instead of completing.
    uint64_t barrier_wait_ns = 0;
    int withhold_arrival = 0;
};
bool persistent_step_supported(int M, int d, int E, int H, int k, int V, int n_layer);
int persistent_partials();
size_t persistent_ws_bytes(int d);
cudaError_t persistent_step(const PersistStepArgs &a, cudaStream_t st);
// out[c][r] = in[r][c] for in [rows, cols] row-major.
cudaError_t transpose(const float *in, float *out, int rows, int cols, cudaStream_t st);

// ---- sampler (sampler.cu): sample_token for every row.
struct SampleParams {
    float temperature;
    uint64_t top_k;
    float top_p;
    float rep_penalty;
    uint64_t rep_window;
    uint32_t greedy;
};
// Any V.  Configurations that keep more than 4096 candidates (top_k == 0 or
// top_k > 4096) sort in per-CTA global scratch `ws` (sample_ws_bytes; fewer
// CTAs run when ws holds fewer slots); others need none (ws may be null).
// prep (nullable): the rows already hold pen(logit) / temperature, written by
// the logits projection's sampling epilogue, whose per-part maxima of the
// finite values and +inf counts ([S, parts]) replace steps 1 and 3.
struct SamplePrepared {
    const float *max;
    const uint32_t *pinf;
    int parts;
};
cudaError_t sample_rows(float *logits, int S, int V, SampleParams cfg, const uint32_t *history,
                        const uint32_t *history_len, int history_stride, uint64_t *rng,
                        uint32_t *out, int *err, void *ws, size_t ws_bytes, cudaStream_t st,
                        const SamplePrepared *prep = nullptr);
// Token collection of generate: out[s * n_new + *column] = tok[s], then
// *column += 1 (two launches; graph-capturable, the column lives on the device).
cudaError_t collect_tokens(const uint32_t *tok, uint32_t *out, int S, int n_new, int *column, cudaStream_t st);
// bits [S][words] = the distinct tokens < V of each stream's last rep_window
// history entries (all zero when the penalty is off), for the sampling
// epilogue of the logits projection.
cudaError_t sample_pen_bitmap(const uint32_t *history, const uint32_t *history_len, int history_stride,
                              SampleParams cfg, int S, int V, uint32_t *bits, int words, cudaStream_t st);
// Scratch sample_rows wants for S rows (0 when none); with budget > 0 at most
// that many bytes, but always at least one CTA's slot.
size_t sample_ws_bytes(int S, int V, SampleParams cfg, size_t budget = 0);

// History ring maintenance for generate (cli.rs:495-503).
cudaError_t history_push(uint32_t *history, uint32_t *history_len, const uint32_t *tok, int S,
                         int window, cudaStream_t st);

// ---- scans (scan.cu)
// scan_adjoint (scan.rs:227-260): c_t = g_t + a_{t+1} c_{t+1}, c_T = 0; the
// chunked form uses the same scratch as scan_chunked.
cudaError_t scan_adjoint_sequential(const float *a, const float *g, float *c, int64_t batch, int64_t t, int64_t d,
                                    cudaStream_t st);
cudaError_t scan_adjoint_chunked(const float *a, const float *g, float *c, int64_t batch, int64_t t, int64_t d,
                                 float *scratch, cudaStream_t st);
cudaError_t scan_sequential(const float *a, const float *b, float *h, int64_t batch, int64_t t,
                            int64_t d, cudaStream_t st);
cudaError_t scan_chunked(const float *a, const float *b, float *h, int64_t batch, int64_t t,
                         int64_t d, float *scratch, cudaStream_t st);
size_t scan_chunked_scratch_floats(int64_t batch, int64_t t, int64_t d);
// One-pass chunked scan (forward, or the adjoint when `adjoint`): one kernel
// with decoupled look-back between time blocks; scratch of
// scan_onepass_scratch_bytes, cleared by the call itself.  After the stream
// has synchronised, scan_onepass_status reads the scratch's error word (0, or
// 131 when a look-back wait expired).  Suited to d >= 16.
bool scan_onepass_suits(int64_t batch, int64_t t, int64_t d);
size_t scan_onepass_scratch_bytes(int64_t batch, int64_t t, int64_t d);
cudaError_t scan_onepass(const float *a, const float *b, float *h, int64_t batch, int64_t t, int64_t d, bool adjoint,
                         void *scratch, cudaStream_t st);
int scan_onepass_status(const void *scratch);

// Largest array the stand-alone ops take: 2^37 floats (512 GB, more than a
// device holds), so element counts, byte counts and every grid derived from
// them stay far from overflow (scan grids within 2^30 blocks).
constexpr uint64_t MAX_ELEMENTS = 1ull << 37;
// out = a * b; false when the product exceeds MAX_ELEMENTS (no wrap-around).
inline bool checked_mul(uint64_t a, uint64_t b, uint64_t &out) {
    out = 0;
    if (a != 0 && b > MAX_ELEMENTS / a) return false;
    out = a * b;
    return true;
}
// n = batch * t * d within MAX_ELEMENTS; any zero size gives n = 0 (an empty scan).
inline bool scan_elements(uint64_t batch, uint64_t t, uint64_t d, uint64_t &n) {
    uint64_t bt = 0;
    return checked_mul(batch, t, bt) && checked_mul(bt, d, n);
}

// ---- training-side ops (train.cu)
// gemm_tn (tensor.rs:156-198): C[m, n] = A[p, m]^T B[p, n].
cudaError_t gemm_tn(const float *a, const float *b, float *c, int64_t p, int m, int n, cudaStream_t st);
// The same product on the tcgen05 3xTF32 engine: scratch holds
// gemm_tn_tc_scratch_floats() floats, flags gemm_tn_tc_flag_ints() ints, zero
// before the call ([0] non-finite operand -> exact recompute, [1] kernel
// error code, the rest stream-K counters, left zero).
bool gemm_tn_tc_eligible(int64_t p, int m, int n);
size_t gemm_tn_tc_scratch_floats(int64_t p, int m, int n);
int gemm_tn_tc_flag_ints();
cudaError_t gemm_tn_tc(const float *a, const float *b, float *c, int64_t p, int m, int n, float *scratch, int *flags,
                       cudaStream_t st);
// Op::DwConv backward (autograd.rs:1050-1097): accumulates into gx [batch*t, d],
// gw [k, d], gb [d] (each nullable); scratch holds
// dwconv_backward_scratch_floats() floats when gw or gb is given; k <= dwconv_max_k().
cudaError_t dwconv_backward(const float *x, const float *w, const float *go, float *gx, float *gw, float *gb,
                            int64_t batch, int64_t t, int d, int k, float *scratch, cudaStream_t st);
size_t dwconv_backward_scratch_floats(int64_t rows, int d, int k);
int dwconv_max_k();
// AdamW::step (optim.rs:33-72) for one parameter tensor; the bias corrections
// 1 / (1 - b^t) come from the host.  A non-finite gradient or parameter sets *err = 4.
struct AdamwParams {
    float lr, b1, b2, eps, wd, inv_bc1, inv_bc2;
    int decay;
};
cudaError_t adamw_step(float *val, const float *grad, float *m, float *v, int64_t n, const AdamwParams &a, int *err,
                       cudaStream_t st);

// *flag = 1 if x[0, n) (16-byte aligned) holds inf or NaN; *flag is not cleared.
cudaError_t any_nonfinite(const float *x, size_t n, int *flag, cudaStream_t st);

// Sets the thread-local message that nk_last_error() returns.
void set_last_error(const std::string &msg);

}  // namespace nk
