/*
 * noetic_gpu.h -- C ABI of the B200 token loop of the noetic language model.
 *
 * The reference (noetic, Rust, std-only) has no FFI layer; its boundary is the
 * crate API listed beside each entry point below.  Each declaration cites the
 * reference interface it replaces (file:line inside the noetic crate).
 *
 * Conventions
 *   - Every call returns nk_status (0 == NK_OK).  Nothing aborts or throws
 *     across the ABI; nk_last_error() returns a thread-local message for the
 *     last failing call on the calling thread.
 *   - Handles are opaque.  A model lives on one CUDA device; a decoder belongs
 *     to one model and owns its device state, scratch and CUDA stream.
 *   - Host pointers are borrowed for the duration of the call only.  Entry
 *     points whose name ends in _device take device pointers instead and do
 *     not synchronise; everything else synchronises the decoder's stream
 *     before returning.
 *   - A handle is not thread-safe; use one decoder per host thread.
 *   - All arithmetic is f32 with f32 state (f64 where the reference's sampler
 *     uses f64).  Token ids are u32; invalid ids and shapes are rejected on
 *     the host before any launch.
 */
#ifndef NOETIC_GPU_H
#define NOETIC_GPU_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

typedef enum nk_status {
    NK_OK = 0,
    NK_ERR_INVALID = 1,     /* bad argument, shape or token id            */
    NK_ERR_CUDA = 2,        /* a CUDA runtime/driver call failed          */
    NK_ERR_OOM = 3,         /* device allocation failed                   */
    NK_ERR_IO = 4,          /* checkpoint file error (ckpt.rs InvalidData) */
    NK_ERR_UNSUPPORTED = 5, /* valid for the reference, not supported here */
    NK_ERR_DEVICE = 6       /* a kernel reported an error status          */
} nk_status;

/* model.rs:20-30 LmConfig (usize fields widened to u64). */
typedef struct nk_config {
    uint64_t vocab, d_model, n_layer, expand, conv_k, mlp_mult;
    float eps, tau_max;
} nk_config;

/* infer.rs:211-219 SampleCfg. */
typedef struct nk_sample_cfg {
    float temperature;
    uint64_t top_k;
    float top_p;
    float rep_penalty;
    uint64_t rep_window;
    uint32_t greedy;
} nk_sample_cfg;

typedef struct nk_model nk_model;
typedef struct nk_decoder nk_decoder;

/* Thread-local description of the last error on this thread. */
const char *nk_last_error(void);

/* Number of CUDA devices visible to this process. */
nk_status nk_device_count(int *count);

/* model.rs:37-76 LmConfig::check. */
nk_status nk_config_check(const nk_config *cfg);

/* ---------------------------------------------------------------- model */

/* Graph + Lm parameter storage (autograd.rs:92-112, model.rs:175-180) on
 * `device`.  Tensors start zeroed; fill them with nk_model_init_random,
 * nk_model_set_tensor or nk_model_load_ckpt.  device == -1 creates a
 * host-only model (initialisation and checkpoint I/O, no decoder). */
nk_status nk_model_create(const nk_config *cfg, int device, nk_model **out);
nk_status nk_model_destroy(nk_model *model);
nk_status nk_model_config(const nk_model *model, nk_config *out);

/* Lm::new(g, &mut Rng::new(seed), cfg) (model.rs:183-206): the reference's
 * seeded initialiser, bit-for-bit (SplitMix64 / xoshiro256++ / Marsaglia
 * polar draws in creation order).  rng_after[4] (nullable) receives the
 * generator state after initialisation, which is the sampler state that
 * `noetic gen` continues with (cli.rs:898-947). */
nk_status nk_model_init_random(nk_model *model, uint64_t seed, uint64_t rng_after[4]);

/* Number of named tensors and their names / shapes in creation order
 * (the checkpoint order, ckpt.rs:161-173). */
nk_status nk_model_tensor_count(const nk_model *model, uint64_t *count);
nk_status nk_model_tensor_info(const nk_model *model, uint64_t index, const char **name,
                               uint32_t *rank, uint64_t shape[4]);

/* Copy one named parameter (ckpt tensor name, e.g. "blk0.ssm.in_proj.w")
 * from host memory.  The shape must match exactly (ckpt.rs:424). */
nk_status nk_model_set_tensor(nk_model *model, const char *name, const float *data,
                              const uint64_t *shape, uint32_t rank);
nk_status nk_model_get_tensor(const nk_model *model, const char *name, float *out,
                              uint64_t numel);

/* ckpt::crc32 (ckpt.rs:35-54): the checkpoint format's CRC-32 (IEEE,
 * reflected 0xEDB88320), computed the way the loader does it: 16 MiB pieces
 * CRC'd separately and combined. */
nk_status nk_crc32(const uint8_t *data, uint64_t n, uint32_t *out);

/* ckpt::load (ckpt.rs:299-383) + the config rules of cmd_gen
 * (cli.rs:909-920) + apply_exact (ckpt.rs:410-436), into a new model on
 * `device`.  Rejects corrupt, truncated, inconsistent or mismatched files
 * with NK_ERR_IO; nothing of a rejected file is returned.  For a device
 * model the file goes straight to device memory: headers are scanned first,
 * then the payload is streamed in 16 MiB chunks through pinned buffers by
 * several host threads (CRC on the host, copies async), the CRC checked at
 * the end and every value checked finite on the device.  device == -1 reads
 * the file into a host-only model. */
nk_status nk_model_load_ckpt(const char *path, int device, nk_model **out);

/* ckpt::save (ckpt.rs:125-200) of the model tensors with the metadata keys
 * cmd_gen needs.  Used to hand models between implementations. */
nk_status nk_model_save_ckpt(const nk_model *model, const char *path);

/* Lm::loss (model.rs:228-234): the batched forward Lm::logits (model.rs:209-226)
 * of `batch` sequences of `t` tokens from the zero state, then the mean
 * cross-entropy Graph::softmax_ce (autograd.rs:579-624) in nats over the
 * positions whose target is not 0xFFFFFFFF (1 when there are none).  ids and
 * targets: host [batch * t], sequence-major.  logits_out (host [batch * t,
 * vocab]) is optional.  Tokens or targets out of range: NK_ERR_INVALID; a
 * non-finite logit: NK_ERR_DEVICE.  Runs on a scratch decoder of `batch`
 * streams; no other decoder's state is touched. */
nk_status nk_model_loss(nk_model *model, const uint32_t *ids, const uint32_t *targets, uint32_t batch,
                        uint32_t t, float *loss_out, float *logits_out);

/* ---------------------------------------------------------------- decoder */

/* Decoder::new (infer.rs:86-88) for n_streams independent streams, each
 * with its own LmState (infer.rs:21-35). */
nk_status nk_decoder_create(nk_model *model, uint32_t n_streams, nk_decoder **out);
nk_status nk_decoder_destroy(nk_decoder *dec);
nk_status nk_decoder_streams(const nk_decoder *dec, uint32_t *n_streams);

/* LmState::reset / Decoder::reset (infer.rs:37-44, 90-92) for streams
 * [first, first+count). */
nk_status nk_decoder_reset(nk_decoder *dec, uint32_t first, uint32_t count);

/* Decoder::step (infer.rs:100-103, 106-200) for every stream: tokens[S]
 * host; logits_out[S*vocab] host (nullable).  The logits also stay on the
 * device as the input of nk_decoder_sample (Decoder::logits_mut). */
nk_status nk_decoder_step(nk_decoder *dec, const uint32_t *tokens, float *logits_out);

/* The prompt loop of cli.rs:generate (cli.rs:478-480: one Decoder::step per
 * prompt token) computed with the chunked parallel scan instead
 * (model.rs:148-165 semantics).  ids is [S, max_t] row-major; lens[S] are
 * the prompt lengths (0 <= len <= max_t; a stream with len 0 is left as it
 * is).  Continues from each stream's current state.  last_logits[S*vocab]
 * (nullable) receives the logits after each stream's last prompt token. */
nk_status nk_decoder_prefill(nk_decoder *dec, const uint32_t *ids, const uint32_t *lens,
                             uint32_t max_t, float *last_logits);

/* sample_token (infer.rs:228-305) applied to the logits of the last step /
 * prefill for every stream.  history is [S, history_stride] with per-stream
 * lengths history_len[S] (each <= history_stride; nullable when
 * rep_window == 0 or rep_penalty <= 1); rng_state[S][4] (host, in/out) is the
 * per-stream xoshiro256++ state (rng.rs:17-22).  out_tokens[S] host.  Any
 * vocabulary size; the softmax and nucleus sums are the reference's
 * sequential f32 sums, bit for bit.  Configurations keeping more than 4096
 * candidates (top_k == 0 or > 4096) sort in decoder-owned scratch (2 * vocab
 * * 8 bytes per concurrently sampled stream, at most 256 MiB), allocated on
 * first use. */
nk_status nk_decoder_sample(nk_decoder *dec, const nk_sample_cfg *cfg, const uint32_t *history,
                            const uint32_t *history_len, uint32_t history_stride,
                            uint64_t *rng_state, uint32_t *out_tokens);

/* cli.rs:generate (cli.rs:470-518) on token ids for every stream: prefill
 * each prompt (an empty prompt becomes [10]), then n_new sampled tokens with
 * a rep_window history, stepping after every token but the last.
 * rng_state[S][4] in/out; out_tokens[S*n_new] host.  When the tensor cores
 * run the logits projection, its epilogue applies the repetition penalty
 * and temperature and emits per-row maxima for the sampler (sampled
 * configurations), or the argmax itself (greedy without a penalty), so the
 * step and the draw share one pass over the logits. */
nk_status nk_decoder_generate(nk_decoder *dec, const uint32_t *ids, const uint32_t *lens,
                              uint32_t max_t, uint32_t n_new, const nk_sample_cfg *cfg,
                              uint64_t *rng_state, uint32_t *out_tokens);

/* LmState access for streams [first, first+count): state is
 * [count, n_layer, (conv_k+1)*E] (per layer the conv ring [conv_k, E] then
 * h [E], infer.rs:12-19), heads[count] the shared conv_head. */
nk_status nk_decoder_get_state(nk_decoder *dec, uint32_t first, uint32_t count, float *state,
                               uint32_t *heads);
nk_status nk_decoder_set_state(nk_decoder *dec, uint32_t first, uint32_t count,
                               const float *state, const uint32_t *heads);

/* Device-resident greedy step: tokens_in / tokens_out are device u32[S].
 * One Decoder::step plus sample_token with greedy = true and no repetition
 * penalty (infer.rs:248-250, tensor.rs:354-365).  Asynchronous on the
 * decoder's stream. */
nk_status nk_decoder_step_greedy_device(nk_decoder *dec, const uint32_t *tokens_in,
                                        uint32_t *tokens_out);

/* Host-buffer greedy step: copies tokens in, steps, copies the argmax
 * tokens out (synchronous). */
nk_status nk_decoder_step_greedy(nk_decoder *dec, const uint32_t *tokens_in,
                                 uint32_t *tokens_out);

/* The decoder's CUDA stream (cudaStream_t) and a wait for it. */
nk_status nk_decoder_cuda_stream(nk_decoder *dec, void **stream);
nk_status nk_decoder_sync(nk_decoder *dec);

/* Engine flags: 0 = automatic (tensor-core 3xTF32 projections where the
 * shape allows it; for 1-4 streams of a model with 96 MiB of weights or
 * more the whole step as one persistent cooperative kernel, otherwise for
 * <= 8 streams the fused small-batch step).  Bit 0: f32
 * CUDA-core projections only.  Bit 1 / bit 2: force the time-chunked /
 * sequential prefill scan.  Bit 3: no fused small-batch step.  Bits 4 / 5:
 * tensor-core tiles 128 / 256 columns wide (default: 128 when N < 256 or
 * the streams fit one row of tiles (<= 128), else 256 with stream-K for the
 * store and SwiGLU epilogues; for the argmax epilogue the width with the
 * higher modelled SM occupancy).  Bit 6: the persistent step kernel for
 * 1-4 streams (the default when the weights take 96 MiB or more; smaller,
 * L2-resident models take the fused small-batch kernels unless bit 6 is set).  Bit 7: the CTA-pair projection kernel (256 x 256 tiles on two
 * SMs) wherever N >= 256.  Bit 8: whole tiles per CTA instead of stream-K
 * (equal K-block ranges per SM, partial tiles summed in a fixed order).
 * Bit 9: no L2 cache policies on projection loads and stores.  Bit 10: no
 * persistent step kernel (1-4 streams take the fused small-batch kernels).
 * Bit 11: generate stores the logits and runs the stand-alone sampler
 * instead of the logits projection's sampling / argmax epilogues.
 * Bits 12 / 13 are test controls of the failure path: the tensor-core
 * projections publish no stream-K partial tile (their finishers' bounded
 * waits run out: error code 121), or the persistent step's first CTA skips
 * its first grid-barrier arrival (every CTA's bounded wait runs out: code
 * 113); those waits are bounded at 2 ms instead of 1 s.  The call returns
 * NK_ERR_DEVICE; the decoder stays usable (restore its state with
 * nk_decoder_set_state: the failed step's results are not valid).
 * Bit 14: RMSNorm folded into the tensor-core decode step's projections
 * (each residual projection's epilogue writes the next projection's
 * gain-scaled operand and the rows' sums of squares, and the consumer scales
 * its rows by the RMSNorm factor) instead of the stand-alone kernels, at
 * every batch; 47 fewer launches per step.  The default folds below 384
 * streams at model widths of 512 and more (where the projections are split
 * along K and the rows are wide enough), not otherwise: above, the longer
 * epilogue, not overlapped with the main loop, measured slower.
 * Bit 15: the 256-wide projection epilogues store from the threads through
 * a transposing buffer instead of the default bulk tensor stores.
 * Bits 16 / 17: with projections split along K (up to 2048 streams), the
 * reductions do not apply the next RMSNorm (taken over from 384 streams) /
 * do not run the recurrent branch; the separate kernels run instead, with
 * the same results.
 * Bit 18: no RMSNorm folding below 384 streams (stand-alone norm kernels).
 * Bit 19: projection tiles in plain row-major order instead of groups of
 * column blocks whose weights fit in L2. */
nk_status nk_decoder_set_engine(nk_decoder *dec, int engine);

/* Number of kernels this decoder has launched so far. */
nk_status nk_decoder_launch_count(const nk_decoder *dec, uint64_t *count);

/* Device-time profile of the projections (the dominant kernels) and of the
 * sampler, measured with CUDA events recorded on the decoder's stream around
 * every projection and sampler launch between nk_decoder_profile_begin and
 * nk_decoder_profile_end. */
typedef struct nk_profile {
    double proj_ms;          /* summed device time of projection launches   */
    uint64_t proj_launches;  /* projection launches                          */
    double proj_flops;       /* useful f32 flops, 2*M*N*K summed             */
    double proj_bytes;       /* algorithmic bytes: A, W, bias, R read + C    */
    uint64_t launches;       /* every kernel launched while profiling        */
    int tensor_core;         /* 1 if any projection ran on tcgen05           */
    double sample_ms;        /* summed device time of sampler launches      */
    uint64_t sample_launches;
} nk_profile;
nk_status nk_decoder_profile_begin(nk_decoder *dec);
nk_status nk_decoder_profile_end(nk_decoder *dec, nk_profile *out);

/* ---------------------------------------------------------------- ops */

/* scan_adjoint (scan.rs:227-260), the reverse-mode gradient of the
 * recurrence: c_t = g_t + a_{t+1} c_{t+1} with c_T = 0, over [batch, t, d]
 * host arrays (layout (b*t + i)*d + j); chunked = 1 uses the time-parallel
 * form of nk_scan_device (equal to the sequential one within f32 rounding).
 * The _device form takes device pointers and a CUDA stream.
 * batch * t * d <= 2^37, else NK_ERR_INVALID. */
nk_status nk_scan_adjoint(const float *a, const float *g, float *c, uint64_t batch, uint64_t t, uint64_t d,
                          int chunked, int device);
nk_status nk_scan_adjoint_device(const float *a, const float *g, float *c, uint64_t batch, uint64_t t, uint64_t d,
                                 int chunked, void *stream);

/* ---------------------------------------------------------------- BPE text I/O
 * Byte-level BPE (bpe.rs), host only: tokens 0..255 are bytes, merge i makes
 * token 256 + i.  Prompts are encoded to ids before prefill, generated ids
 * decoded to bytes after. */
typedef struct nk_bpe nk_bpe;
/* Bpe::bytes_only (bpe.rs:47-53): 256 byte tokens, no merges. */
nk_status nk_bpe_create_bytes_only(nk_bpe **out);
/* Bpe::load (bpe.rs:309-380): the "noetic-bpe 1" merges file, with the
 * reference's limits (64 MiB file, 1,000,000 merges, 1 MiB per token, 128
 * MiB of token bytes) and checks; a bad file is NK_ERR_IO. */
nk_status nk_bpe_load(const char *path, nk_bpe **out);
/* Bpe::save (bpe.rs:288-307): temporary file, then rename. */
nk_status nk_bpe_save(const nk_bpe *bpe, const char *path);
nk_status nk_bpe_destroy(nk_bpe *bpe);
nk_status nk_bpe_vocab_size(const nk_bpe *bpe, uint64_t *out);
/* The pair that merge i joins. */
nk_status nk_bpe_merge(const nk_bpe *bpe, uint64_t i, uint32_t *a, uint32_t *b);
/* Bpe::encode (bpe.rs:252-258): UTF-8 text (len bytes; invalid UTF-8 is
 * NK_ERR_INVALID) split by Bpe::pretokenize (bpe.rs:77-115, char::is_alphabetic
 * = the Unicode 15.0 Alphabetic property), each chunk merged lowest rank
 * first.  *n_out = the id count; NK_ERR_INVALID when it exceeds cap. */
nk_status nk_bpe_encode(const nk_bpe *bpe, const char *text, uint64_t len, uint32_t *ids, uint64_t cap,
                        uint64_t *n_out);
/* Bpe::encode_bytes (bpe.rs:262-266): any bytes, no pre-token boundaries. */
nk_status nk_bpe_encode_bytes(const nk_bpe *bpe, const uint8_t *bytes, uint64_t len, uint32_t *ids, uint64_t cap,
                              uint64_t *n_out);
/* Bpe::decode_bytes (bpe.rs:268-279): an out-of-range id is NK_ERR_INVALID
 * (the reference returns None).  *n_out = the byte count. */
nk_status nk_bpe_decode_bytes(const nk_bpe *bpe, const uint32_t *ids, uint64_t n, uint8_t *out, uint64_t cap,
                              uint64_t *n_out);

/* gemm_tn (tensor.rs:156-198): C[m, n] = A[p, m]^T B[p, n], the weight-
 * gradient product; a zero element of A skips its product as kern_tn does.
 * Host arrays, run on `device`; the _device form takes device pointers and a
 * CUDA stream.  m < 2^22, n < 2^31, and p*m, p*n, m*n <= 2^37, else
 * NK_ERR_INVALID. */
nk_status nk_gemm_tn(const float *a, const float *b, float *c, uint64_t p, uint64_t m, uint64_t n, int device);
nk_status nk_gemm_tn_device(const float *a, const float *b, float *c, uint64_t p, uint64_t m, uint64_t n,
                            void *stream);

/* Op::DwConv backward (autograd.rs:1050-1097) of y[b,t,j] = bias[j] +
 * sum_{q < min(t+1, k)} w[q,j] x[b,t-q,j]: the gradients ADD into gx
 * [batch*t*d], gw [k*d] and gb [d] (each nullable, as Graph::backward
 * accumulates).  gx follows the reference's order bit for bit; gw and gb are
 * sums over batch*t rows in a fixed blocked order (deterministic, equal to
 * the sequential sums within f32 rounding).  k <= 16, d < 2^21,
 * batch * t * d <= 2^37.  Host arrays on `device`; the _device form takes
 * device pointers and a CUDA stream. */
nk_status nk_dwconv_backward(const float *x, const float *w, const float *go, float *gx, float *gw, float *gb,
                             uint64_t batch, uint64_t t, uint64_t d, uint64_t k, int device);
nk_status nk_dwconv_backward_device(const float *x, const float *w, const float *go, float *gx, float *gw,
                                    float *gb, uint64_t batch, uint64_t t, uint64_t d, uint64_t k, void *stream);

/* AdamW::step (optim.rs:33-72) for one parameter tensor and its moments: t
 * is the step counter after its increment (>= 1), decay the parameter's
 * Param::decay.  Bit-identical to the reference's f32 arithmetic.  Invalid
 * hyper-parameters are refused before any work; a non-finite gradient or
 * parameter returns NK_ERR_INVALID (the reference asserts), with that
 * element untouched and the others updated.  Host arrays on `device`; the
 * _device form takes device pointers and a CUDA stream (synchronous: it
 * reads the error flag).  n <= 2^37. */
typedef struct nk_adamw_cfg {
    float lr, b1, b2, eps, wd; /* AdamW::new defaults: b1 0.9, b2 0.95, eps 1e-8 */
    uint64_t t;
    int decay;
} nk_adamw_cfg;
nk_status nk_adamw_step(float *val, const float *grad, float *m, float *v, uint64_t n, const nk_adamw_cfg *cfg,
                        int device);
nk_status nk_adamw_step_device(float *val, const float *grad, float *m, float *v, uint64_t n,
                               const nk_adamw_cfg *cfg, void *stream);

/* scan_sequential / scan_chunked (scan.rs:35-57, 98-225):
 * h[b,t,j] = a[b,t,j] * h[b,t-1,j] + b[b,t,j], h[b,-1,j] = 0, layout
 * (b*T + t)*D + j.  Host pointers; runs on `device`.  chunked != 0 selects
 * the time-chunked associative scan: for d >= 16 one kernel that passes the
 * state between time blocks of 128 steps by decoupled look-back (each
 * element read and written once), else the three-pass form.  batch * t * d
 * <= 2^37 (checked without wrap-around), else NK_ERR_INVALID. */
nk_status nk_scan(const float *a, const float *b, float *h, uint64_t batch, uint64_t t,
                  uint64_t d, int chunked, int device);

/* Same on device pointers, on `stream` (cudaStream_t, may be NULL for the
 * legacy default stream): asynchronous for chunked = 0; chunked != 0 waits
 * for the stream, and returns NK_ERR_DEVICE (code 131) if a time block's
 * look-back wait expired (bounded at 1 s). */
nk_status nk_scan_device(const float *a, const float *b, float *h, uint64_t batch, uint64_t t,
                         uint64_t d, int chunked, void *stream);

/* Time-chunked scan that allocates nothing.  No counterpart in the
 * reference; it exists for callers that cannot allocate device memory in the
 * middle of their work: a host whose own pool allocator owns the whole
 * device memory budget (a stray cudaMalloc there can fail or fragment the
 * pool), or a latency-critical loop that cannot afford the device-wide
 * synchronisation cudaMalloc / cudaFree may cause.  It computes the
 * three-pass time-chunked scan (equal to nk_scan_device(..., chunked = 1,
 * ...) within f32 rounding), on device pointers, asynchronously on
 * `stream`, but its scratch is a fixed array of
 * NK_SCAN_NOALLOC_SCRATCH_FLOATS floats (12 MiB) inside the library's device
 * image, which every GPU that loads the library holds until the process
 * exits.  Limit: batch * ceil(t / NK_SCAN_TIME_BLOCK) * d <= 1048576
 * (three scratch floats per stream, time block and channel); larger scans
 * return NK_ERR_INVALID with a message.  It calls no allocator at all.  The
 * first call on each device looks up the array's device address (with that
 * device current), so make that first call before any stream capture.  After
 * a cudaDeviceReset the array may sit at a new address: the next call sees
 * the new context and looks it up again, so it too is a first call.  All
 * calls share the array: calls whose GPU work overlaps (other streams or
 * threads without ordering) race and may return wrong results; order them. */
#define NK_SCAN_TIME_BLOCK 256u
#define NK_SCAN_NOALLOC_SCRATCH_FLOATS (3u * 1048576u)
nk_status nk_scan_chunked_noalloc_device(const float *a, const float *b, float *h, uint64_t batch,
                                         uint64_t t, uint64_t d, void *stream);

/* sample_token (infer.rs:228-305) on one host logit row, computed on the
 * device.  logits[vocab] is mutated like the reference (penalised, then
 * tempered and normalised when not greedy); rng_state[4] in/out. */
nk_status nk_sample_token(float *logits, uint64_t vocab, const nk_sample_cfg *cfg,
                          const uint32_t *history, uint64_t n_history, uint64_t *rng_state,
                          uint32_t *out_token, int device);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif

#ifdef __cplusplus
}
#endif
#endif /* NOETIC_GPU_H */
